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
// Tensor-core kernel A, a cluster of CTAs over slot chunks, merged through DSMEM.
int launch_decode_split(const ic_decode_args& a, cudaStream_t stream);

}  // namespace ic
