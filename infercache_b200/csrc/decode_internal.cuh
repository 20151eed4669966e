// Internal entry points shared between the decode translation units.
#pragma once

#include <cuda_runtime.h>

#include "../../include/infercache.h"

namespace ic {

// Tensor-core kernel A, one cluster per (session, KV head) (fp16 / bf16).
int launch_decode_mma(const ic_decode_args& a, cudaStream_t stream);
// Tensor-core kernel A, one CTA streams a whole (session, KV head) group.
int launch_decode_stream(const ic_decode_args& a, cudaStream_t stream);
// Tensor-core kernel A, one CTA per group with four independent warp pipelines.
int launch_decode_lean(const ic_decode_args& a, cudaStream_t stream);
// Tensor-core kernel A, CTAs over slot chunks, merged by the last CTA (workspace).
int launch_decode_split(const ic_decode_args& a, cudaStream_t stream);
int64_t decode_split_workspace_bytes(const ic_decode_args& a);

}  // namespace ic
