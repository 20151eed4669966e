// Tensor-core helpers shared by the fp16 / bf16 decode kernels: mma.sync
// m16n8k16 with fp32 accumulation, ldmatrix loads, and the conversions used to
// split P into a high and a low half-precision part.
#pragma once

#include "common.cuh"

namespace ic {

// P is multiplied by 2^12 before the split so that small probabilities stay
// in the normal half-precision range; the product is scaled back exactly.
constexpr float P_SCALE = 4096.0f;
constexpr float P_UNSCALE = 1.0f / 4096.0f;

template <typename T> struct Mma;
template <> struct Mma<__half> {
  __device__ static void run(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ static uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  __device__ static float back(uint16_t b) { return __half2float(__ushort_as_half(b)); }
};
template <> struct Mma<__nv_bfloat16> {
  __device__ static void run(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ static uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  __device__ static float back(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
};

__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}


}  // namespace ic
