// Tensor-level cache operations with the reference's triton_ops names and
// semantics, for callers that hold plain K / V buffers and an importance
// vector rather than a SessionBatch:
//
//  * index_rows      gather_cache_kv   (triton_ops.py:107-135): rows of
//                    [H, N, D] at given indices -> [H, F, D]
//  * scatter_mass    scatter_importance (:148-175): importance[slot_f] +=
//                    mean over (L, H, Q) of the attention weights of column f
//  * argmin_range    topk_min_slot      (:207-235): first index of the minimum
//                    of x[start, start + n) (NaN counts as smallest, as torch)
//  * compact_attention compact_sdp_attention (:251-287): softmax(q k^T *
//                    scale) v over the given slots, one query row per batch
//
// The fused decode path does not use these (kernels A and B cover them); they
// exist so a user of the reference's GPU helpers finds them here.
#include <math.h>

#include "common.cuh"

namespace ic {
namespace {

__global__ void index_rows_kernel(const ic_index_rows_args a, int vecs, int esz) {
  const int h = blockIdx.y;
  const size_t row_bytes = static_cast<size_t>(a.D) * esz;
  const char* src = static_cast<const char*>(a.src) + static_cast<size_t>(h) * a.stride_h * esz;
  char* dst = static_cast<char*>(a.out) + static_cast<size_t>(h) * a.F * row_bytes;
  const int per_block = blockDim.x / vecs;
  const int vi = threadIdx.x % vecs, ri = threadIdx.x / vecs;
  if (ri >= per_block) return;
  for (int f = blockIdx.x * per_block + ri; f < a.F; f += gridDim.x * per_block) {
    const int64_t r = a.idx[f];
    int4 val = make_int4(0, 0, 0, 0);
    if (r >= 0 && r < a.N) val = reinterpret_cast<const int4*>(src + r * a.stride_n * esz)[vi];
    reinterpret_cast<int4*>(dst + f * row_bytes)[vi] = val;
  }
}

// one thread per column: the mean over rows in row order, then one add
__global__ void scatter_mass_kernel(const ic_scatter_mass_args a, int n) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= n) return;
  float s = 0.f;
  for (int r = 0; r < a.rows; ++r) s += a.weights[static_cast<size_t>(r) * a.width + f];
  const int64_t slot = a.slots[f];
  if (slot >= 0 && slot < a.budget) atomicAdd(a.importance + slot, s / static_cast<float>(a.rows));
}

__global__ void argmin_range_kernel(const ic_argmin_args a) {
  __shared__ float sv[32];
  __shared__ int si[32];
  float v = INFINITY;
  int i = INT_MAX;
  for (int j = threadIdx.x; j < a.n; j += blockDim.x) {
    const float x = a.x[a.start + j];
    if (argmin_less(x, j, v, i)) { v = x; i = j; }
  }
  warp_argmin(v, i);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[w] = v; si[w] = i; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    v = lane < nw ? sv[lane] : INFINITY;
    i = lane < nw ? si[lane] : INT_MAX;
    warp_argmin(v, i);
    if (lane == 0) {
      *a.out_idx = static_cast<int64_t>(a.start) + (i == INT_MAX ? 0 : i);
      if (a.out_val) *a.out_val = v;
    }
  }
}

template <typename T>
__device__ __forceinline__ float ld(const T* p) { return DT<T>::to_f(*p); }

// grid (H, B), 4 warps; each warp runs an online softmax over every 4th slot,
// then the warps merge.  D <= 256, a multiple of 32.
template <typename T>
__global__ void compact_attention_kernel(const ic_compact_attn_args a) {
  constexpr int NW = 4, MAXE = 8;
  __shared__ float wm[NW], wl[NW];
  __shared__ float wacc[NW][256];
  const int h = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.D / 32;
  const T* q = static_cast<const T*>(a.q) + (static_cast<size_t>(b) * a.H + h) * a.D;
  const T* kb = static_cast<const T*>(a.k_buf) + static_cast<size_t>(h) * a.k_stride_h;
  const T* vb = static_cast<const T*>(a.v_buf) + static_cast<size_t>(h) * a.v_stride_h;
  float qr[MAXE], acc[MAXE];
#pragma unroll
  for (int e = 0; e < MAXE; ++e) {
    qr[e] = e < E ? ld(q + lane + 32 * e) : 0.f;
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int f = warp; f < a.F; f += NW) {
    const int64_t slot = a.slots[f];
    if (slot < 0 || slot >= a.budget) continue;
    const T* kr = kb + slot * a.k_stride_n;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < MAXE; ++e)
      if (e < E) s = fmaf(qr[e], ld(kr + lane + 32 * e), s);
    s = warp_sum(s) * a.scale;
    const float mn = fmaxf(m, s);
    const float c = expf(m - mn), p = expf(s - mn);
    const T* vr = vb + slot * a.v_stride_n;
#pragma unroll
    for (int e = 0; e < MAXE; ++e)
      if (e < E) acc[e] = fmaf(acc[e], c, p * ld(vr + lane + 32 * e));
    l = fmaf(l, c, p);
    m = mn;
  }
  if (lane == 0) { wm[warp] = m; wl[warp] = l; }
#pragma unroll
  for (int e = 0; e < MAXE; ++e)
    if (e < E) wacc[warp][lane + 32 * e] = acc[e];
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w]);
    float L = 0.f, sc[NW];
    for (int w = 0; w < NW; ++w) {
      sc[w] = wm[w] == -INFINITY ? 0.f : expf(wm[w] - M);
      L = fmaf(wl[w], sc[w], L);
    }
    T* o = static_cast<T*>(a.out) + (static_cast<size_t>(b) * a.H + h) * a.D;
    for (int e = 0; e < E; ++e) {
      float x = 0.f;
      for (int w = 0; w < NW; ++w) x = fmaf(wacc[w][lane + 32 * e], sc[w], x);
      o[lane + 32 * e] = DT<T>::from_f(L > 0.f ? x / L : 0.f);
    }
  }
}

int esize(int dt) { return dt == IC_F32 ? 4 : 2; }

}  // namespace
}  // namespace ic

extern "C" int ic_index_rows(const ic_index_rows_args* a, void* stream) {
  if (!a || !a->src || !a->out || (!a->idx && a->F > 0) || a->H < 1 || a->N < 0 || a->F < 0 || a->D < 1 ||
      (a->dtype != IC_F32 && a->dtype != IC_F16 && a->dtype != IC_BF16)) {
    ic::set_last_error("index_rows: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  const int esz = ic::esize(a->dtype);
  if ((a->D * esz) % 16 || (a->stride_n * esz) % 16 || (a->stride_h * esz) % 16 ||
      (reinterpret_cast<uintptr_t>(a->src) & 15) || (reinterpret_cast<uintptr_t>(a->out) & 15)) {
    ic::set_last_error("index_rows: rows must be 16-byte aligned multiples of 16 bytes");
    return IC_ERR_UNSUPPORTED;
  }
  if (a->F == 0) return IC_OK;
  const int vecs = a->D * esz / 16;
  if (vecs > 256) {
    ic::set_last_error("index_rows: row too long");
    return IC_ERR_UNSUPPORTED;
  }
  const int threads = vecs >= 256 ? 256 : (256 / vecs) * vecs;
  const int per = threads / vecs;
  int gx = (a->F + per - 1) / per;
  if (gx > 4096) gx = 4096;
  ic::index_rows_kernel<<<dim3(gx, a->H), threads, 0, static_cast<cudaStream_t>(stream)>>>(*a, vecs, esz);
  return ic::launch_status("index_rows");
}

extern "C" int ic_scatter_mass(const ic_scatter_mass_args* a, void* stream) {
  if (!a || !a->weights || !a->slots || !a->importance || a->rows < 1 || a->width < 0 || a->n_slots < 0 ||
      a->budget < 1) {
    ic::set_last_error("scatter_mass: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  const int n = a->width < a->n_slots ? a->width : a->n_slots;
  if (n == 0) return IC_OK;
  ic::scatter_mass_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(*a, n);
  return ic::launch_status("scatter_mass");
}

extern "C" int ic_argmin_range(const ic_argmin_args* a, void* stream) {
  if (!a || !a->x || !a->out_idx || a->start < 0 || a->n < 1) {
    ic::set_last_error("argmin_range: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  ic::argmin_range_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return ic::launch_status("argmin_range");
}

extern "C" int ic_compact_attention(const ic_compact_attn_args* a, void* stream) {
  if (!a || !a->q || !a->k_buf || !a->v_buf || !a->out || (!a->slots && a->F > 0) || a->B < 1 || a->H < 1 ||
      a->F < 0 || a->budget < 1 || a->B > 65535) {
    ic::set_last_error("compact_attention: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  if (a->D < 32 || a->D > 256 || a->D % 32) {
    ic::set_last_error("compact_attention: head_dim must be a multiple of 32 up to 256");
    return IC_ERR_UNSUPPORTED;
  }
  const dim3 grid(a->H, a->B);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case IC_F32: ic::compact_attention_kernel<float><<<grid, 128, 0, st>>>(*a); break;
    case IC_F16: ic::compact_attention_kernel<__half><<<grid, 128, 0, st>>>(*a); break;
    case IC_BF16: ic::compact_attention_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(*a); break;
    default:
      ic::set_last_error("compact_attention: bad dtype");
      return IC_ERR_INVALID_ARG;
  }
  return ic::launch_status("compact_attention");
}
