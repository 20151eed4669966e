// Internal entry points shared between the decode translation units.
#pragma once

#include <cuda_runtime.h>

#include "../../include/infercache.h"

namespace ic {

// Tensor-core variant of kernel A (fp16 / bf16 pools, head_dim 128).
int launch_decode_mma(const ic_decode_args& a, cudaStream_t stream);

}  // namespace ic
