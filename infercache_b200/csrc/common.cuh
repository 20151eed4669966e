// Shared device helpers for the sm_100a kernels: dtype conversion, mbarrier
// and bulk-copy (TMA engine) wrappers, cluster / DSMEM access, bounded waits,
// and the status plumbing of the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cooperative_groups.h>
#include <stdint.h>

#include <atomic>

#include "../../include/infercache.h"

namespace ic {

namespace cg = cooperative_groups;

constexpr unsigned FULL_MASK = 0xffffffffu;

// ---- dtype helpers ---------------------------------------------------------
template <typename T> struct DT;
template <> struct DT<float> {
  static constexpr int code = IC_F32;
  __device__ static float to_f(float x) { return x; }
  __device__ static float from_f(float x) { return x; }
};
template <> struct DT<__half> {
  static constexpr int code = IC_F16;
  __device__ static float to_f(__half x) { return __half2float(x); }
  __device__ static __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct DT<__nv_bfloat16> {
  static constexpr int code = IC_BF16;
  __device__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

inline int dtype_size(int dt) { return dt == IC_F32 ? 4 : 2; }

// Load 4 consecutive elements as floats (p must be aligned to 4 elements).
__device__ __forceinline__ void load4(const float* p, float* o) {
  float4 v = *reinterpret_cast<const float4*>(p);
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
__device__ __forceinline__ void load4(const __half* p, float* o) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __half2 a = *reinterpret_cast<__half2*>(&u.x), b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float* o) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x), b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
}

// ---- shared-memory addressing ---------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for an mbarrier phase with a time limit (default 2 s).  On timeout the
// IC_DEVFLAG_TIMEOUT bit is OR-ed into *status and false is returned; the
// caller keeps its control flow uniform (cluster barriers must still be
// reached) and its results are then undefined, which the host reports as
// IC_ERR_DEVICE_TIMEOUT.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int32_t* status,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) {
      if (status) atomicOr(status, IC_DEVFLAG_TIMEOUT);
      return false;
    }
  }
}

// ---- bulk copy global -> shared through the TMA engine ---------------------
// Untiled cp.async.bulk into this CTA only: both addresses 16-byte aligned, size a
// multiple of 16.  Completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---- 16-byte asynchronous global -> shared copies (LDGSTS), L1 bypassed ------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's committed groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- programmatic dependent launch ------------------------------------------------
// Wait until the grids this one depends on have completed and their writes
// are visible (returns at once when launched without the PDL attribute).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next grid in the stream to begin launching.
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---- cluster helpers ---------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Split cluster barrier: every thread of every CTA arrives, then waits.
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Asynchronous stores into a (possibly remote) CTA's shared memory, completing
// as transaction bytes on that CTA's mbarrier.
__device__ __forceinline__ void st_async_v2(uint32_t addr, uint32_t x, uint32_t y, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "r"(x), "r"(y), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void st_async_v4(uint32_t addr, uint32_t x, uint32_t y, uint32_t z, uint32_t w,
                                            uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   addr),
               "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
               : "memory");
}

// ---- warp reductions ---------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(FULL_MASK, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}

// Argmin ordering used by every eviction decision: NaN sorts first (as
// torch.argmin / numpy.argmin return the first NaN), then smaller value, then
// lower slot index (the first index of the minimum).
__device__ __forceinline__ bool argmin_less(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na || nb) return na && (!nb || ia < ib);
  return a < b || (a == b && ia < ib);
}
__device__ __forceinline__ void warp_argmin(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(FULL_MASK, v, o);
    int oi = __shfl_xor_sync(FULL_MASK, i, o);
    if (argmin_less(ov, oi, v, i)) { v = ov; i = oi; }
  }
}
// The argmin (v, i) as above together with r, the fminf of every other value
// (the runner-up; NaN values are skipped as fminf skips them).  Every lane
// ends with the same triple.
__device__ __forceinline__ void argmin2_take(float& v, int& i, float& r, float ov, int oi, float orr) {
  if (argmin_less(ov, oi, v, i)) {
    r = fminf(fminf(r, orr), v);
    v = ov;
    i = oi;
  } else {
    r = fminf(fminf(r, orr), ov);
  }
}
__device__ __forceinline__ void warp_argmin2(float& v, int& i, float& r) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL_MASK, v, o);
    const int oi = __shfl_xor_sync(FULL_MASK, i, o);
    const float orr = __shfl_xor_sync(FULL_MASK, r, o);
    argmin2_take(v, i, r, ov, oi, orr);
  }
}

// ---- host-side status plumbing ----------------------------------------------
void set_last_error(const char* msg);
int launch_status(const char* what);

// Kernel attributes set with cudaFuncSetAttribute apply to the current
// device's copy of the kernel, so the record of what has been applied is kept
// per device: a process that drives several GPUs sets each one.  Entries are
// atomics, so host threads may launch concurrently.
constexpr int IC_MAX_DEVICES = 64;

inline int current_device_index() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return d;
}

struct PerDeviceLimit {
  std::atomic<int> v[IC_MAX_DEVICES];
};

struct PerDeviceOnce {
  std::atomic<int> done[IC_MAX_DEVICES];
};

// Run `fn` once per device (every time on a device index beyond the table).
template <typename Fn>
inline void once_per_device(PerDeviceOnce* once, Fn fn) {
  const int dev = current_device_index();
  if (dev >= 0 && dev < IC_MAX_DEVICES) {
    if (once->done[dev].load(std::memory_order_acquire)) return;
    fn();
    once->done[dev].store(1, std::memory_order_release);
    return;
  }
  fn();
}

// Raise a kernel's dynamic shared-memory limit on the current device to
// `bytes` if it is below it.  Returns IC_OK or IC_ERR_UNSUPPORTED.
template <typename F>
inline int ensure_dynamic_smem(F* kernel, int bytes, PerDeviceLimit* limit) {
  if (bytes <= 48 * 1024) return IC_OK;
  const int dev = current_device_index();
  const bool tracked = dev >= 0 && dev < IC_MAX_DEVICES;
  if (tracked && bytes <= limit->v[dev].load(std::memory_order_acquire)) return IC_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_last_error("kernel needs more shared memory than the device allows");
    return IC_ERR_UNSUPPORTED;
  }
  if (tracked) {
    int cur = limit->v[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !limit->v[dev].compare_exchange_weak(cur, bytes, std::memory_order_acq_rel)) {
    }
  }
  return IC_OK;
}

}  // namespace ic
