// Kernel A: fused decode step for one layer over all sessions.
//
// One thread-block cluster of CL CTAs per (session, KV head).  The budget+1
// logical slots (the last one is the staging row that receives the token
// being decoded) are split into CL contiguous chunks.  Each CTA:
//   1. issues one TMA-engine bulk copy per K row and per V row of its chunk,
//      addressed through the session's slot table (a per-slot page table),
//      into padded shared-memory rows; the CTA owning the staging row writes
//      the new K/V into the pool and into shared memory instead;
//   2. computes the scores of the G query heads of the group (CUDA cores,
//      lanes split head_dim, one transpose-reduction for all G heads);
//   3. exchanges per-head maxima and then exp-sums with the other CTAs of its
//      cluster through distributed shared memory, so every probability is
//      exp(s - m) / l with the exact global m and l;
//   4. adds the received mass of each slot summed over the group's query
//      heads to the slot's running sum over layers (layer 0 stores it);
//   5. computes its partial P.V and reduces the partials across the cluster
//      through DSMEM in a fixed CTA order.
// No global scratch, no atomics: results are deterministic run to run.
#include <math.h>

#include "common.cuh"
#include "decode_internal.cuh"

namespace ic {

constexpr int DEC_THREADS = 256;
constexpr int DEC_D = 128;

struct DecodeSmem {
  int chunk, chunk_pad, rowb;
  int k_off, v_off, sc_off, ob_off, red_off, occ_off, bar_off, total;
};

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ inline DecodeSmem decode_smem(int chunk, int dsize, int GP) {
  DecodeSmem L;
  L.chunk = chunk;
  L.chunk_pad = align_up(chunk > 0 ? chunk : 1, 4);
  L.rowb = DEC_D * dsize + 16;  // +16 B: rows start on different bank groups
  int o = 0;
  L.k_off = o; o = align_up(o + chunk * L.rowb, 128);
  L.v_off = o; o = align_up(o + chunk * L.rowb, 128);
  L.sc_off = o; o = align_up(o + GP * L.chunk_pad * 4, 128);
  L.ob_off = o; o = align_up(o + GP * DEC_D * 4, 128);
  L.red_off = o; o = align_up(o + 2 * GP * 4, 16);
  L.occ_off = o; o = align_up(o + chunk, 16);
  L.bar_off = o; o += 16;
  L.total = o;
  return L;
}

// Sum COUNT per-head partials across the 32 lanes of a warp with one
// transpose-reduction: each step halves the heads a lane carries and pairs
// lanes across bit MASK.  On return the lane holds the full dot product of
// head `head` (lanes that differ only in the low bits hold the same value).
template <int COUNT, int MASK>
struct HeadReduce {
  __device__ __forceinline__ static float run(float* part, int lane, int& head) {
    constexpr int HALF = COUNT / 2;
    const bool up = (lane & MASK) != 0;
#pragma unroll
    for (int i = 0; i < HALF; ++i) {
      const float send = up ? part[i] : part[i + HALF];
      const float keep = up ? part[i + HALF] : part[i];
      part[i] = keep + __shfl_xor_sync(FULL_MASK, send, MASK);
    }
    if (up) head += HALF;
    return HeadReduce<HALF, MASK / 2>::run(part, lane, head);
  }
};
template <int MASK>
struct HeadReduce<1, MASK> {
  __device__ __forceinline__ static float run(float* part, int, int&) {
    float v = part[0];
#pragma unroll
    for (int m = MASK; m >= 1; m >>= 1) v += __shfl_xor_sync(FULL_MASK, v, m);
    return v;
  }
};

template <typename T, int CL, int GP>
__global__ void __launch_bounds__(DEC_THREADS, 1) decode_kernel(const ic_decode_args a, int chunk) {
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int budget = a.tiers.budget, ntot = budget + 1;
  const int Hkv = a.pool.num_kv_heads, Hq = a.num_q_heads, G = Hq / Hkv;
  const int t0 = c * chunk;
  const int n = max(0, min(chunk, ntot - t0));
  const int stage_t = budget - t0;
  const bool has_stage = stage_t >= 0 && stage_t < n;

  const DecodeSmem L = decode_smem(chunk, sizeof(T), GP);
  unsigned char* Ks = smem + L.k_off;
  unsigned char* Vs = smem + L.v_off;
  float* sc = reinterpret_cast<float*>(smem + L.sc_off);
  float* ob = reinterpret_cast<float*>(smem + L.ob_off);
  float* red_m = reinterpret_cast<float*>(smem + L.red_off);
  float* red_l = red_m + GP;
  uint8_t* occ_s = smem + L.occ_off;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  const int cp = L.chunk_pad;
  const int rowb = L.rowb;

  const size_t plane = static_cast<size_t>(a.pool.pool_tokens) * DEC_D;
  const size_t lh = static_cast<size_t>(a.layer) * Hkv + h;
  const T* pk = static_cast<const T*>(a.pool.k) + lh * plane;
  const T* pv = static_cast<const T*>(a.pool.v) + lh * plane;
  const int32_t* st = a.sess.slot_table + static_cast<size_t>(s) * ntot;
  const uint8_t* occ_g = a.sess.occupied + static_cast<size_t>(s) * budget;
  constexpr uint32_t ROW_BYTES = DEC_D * sizeof(T);

  // -- 1. loads --------------------------------------------------------------
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    const uint32_t rows = static_cast<uint32_t>(n - (has_stage ? 1 : 0));
    mbar_arrive_expect_tx(&bar[0], rows * ROW_BYTES);
    mbar_arrive_expect_tx(&bar[1], rows * ROW_BYTES);
  }
  __syncthreads();
  for (int t = tid; t < n; t += DEC_THREADS) {
    const int slot = t0 + t;
    if (slot == budget) continue;
    int row = st[slot];
    if (static_cast<unsigned long long>(row) >= static_cast<unsigned long long>(a.pool.pool_tokens)) {
      if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
      row = 0;
    }
    bulk_g2s(Ks + t * rowb, pk + static_cast<size_t>(row) * DEC_D, ROW_BYTES, &bar[0]);
    bulk_g2s(Vs + t * rowb, pv + static_cast<size_t>(row) * DEC_D, ROW_BYTES, &bar[1]);
    occ_s[t] = occ_g[slot];
  }
  if (has_stage) {
    int row = st[budget];
    const bool row_ok =
        static_cast<unsigned long long>(row) < static_cast<unsigned long long>(a.pool.pool_tokens);
    if (!row_ok && tid == 0 && a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
    const T* kn = static_cast<const T*>(a.k_new) + (static_cast<size_t>(s) * Hkv + h) * DEC_D;
    const T* vn = static_cast<const T*>(a.v_new) + (static_cast<size_t>(s) * Hkv + h) * DEC_D;
    T* dk = static_cast<T*>(a.pool.k) + lh * plane + static_cast<size_t>(row) * DEC_D;
    T* dv = static_cast<T*>(a.pool.v) + lh * plane + static_cast<size_t>(row) * DEC_D;
    T* sk = reinterpret_cast<T*>(Ks + stage_t * rowb);
    T* sv = reinterpret_cast<T*>(Vs + stage_t * rowb);
    for (int d = tid; d < DEC_D; d += DEC_THREADS) {
      const T kv = kn[d], vv = vn[d];
      sk[d] = kv;
      sv[d] = vv;
      if (row_ok) { dk[d] = kv; dv[d] = vv; }
    }
    if (tid == 0) occ_s[stage_t] = 1;
  }

  // q of the group's heads, 4 consecutive elements of head_dim per lane
  float qr[GP][4];
  {
    const T* qb = static_cast<const T*>(a.q) + (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * DEC_D;
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      if (g < G) {
        load4(qb + static_cast<size_t>(g) * DEC_D + 4 * lane, qr[g]);
      } else {
        qr[g][0] = qr[g][1] = qr[g][2] = qr[g][3] = 0.f;
      }
    }
  }

  // -- 2. scores --------------------------------------------------------------
  mbar_wait_bounded(&bar[0], 0, a.sess.dev_status);
  __syncthreads();  // staging row and occupancy flags written by threads
  const float scale = a.scale;
  for (int t = warp; t < n; t += DEC_THREADS / 32) {
    float kf[4];
    load4(reinterpret_cast<const T*>(Ks + t * rowb) + 4 * lane, kf);
    float part[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g)
      part[g] = fmaf(qr[g][3], kf[3], fmaf(qr[g][2], kf[2], fmaf(qr[g][1], kf[1], qr[g][0] * kf[0])));
    int head = 0;
    const float dot = HeadReduce<GP, 16>::run(part, lane, head);
    if ((lane & (32 / GP - 1)) == 0 && head < G) sc[head * cp + t] = occ_s[t] ? dot * scale : -INFINITY;
  }
  __syncthreads();

  // -- 3. softmax across the cluster -----------------------------------------
  for (int g = warp; g < G; g += DEC_THREADS / 32) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[g * cp + t]);
    m = warp_max(m);
    if (lane == 0) red_m[g] = m;
  }
  cluster.sync();
  for (int g = warp; g < G; g += DEC_THREADS / 32) {
    float m = -INFINITY;
    if (lane < CL) m = *cluster.map_shared_rank(&red_m[g], lane);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float e = expf(sc[g * cp + t] - m);
      sc[g * cp + t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) red_l[g] = l;
  }
  cluster.sync();
  for (int g = warp; g < G; g += DEC_THREADS / 32) {
    float tot = 0.f;
    if (lane == 0) {
#pragma unroll 1
      for (int r = 0; r < CL; ++r) tot += *cluster.map_shared_rank(&red_l[g], r);
    }
    tot = __shfl_sync(FULL_MASK, tot, 0);
    for (int t = lane; t < n; t += 32) sc[g * cp + t] = sc[g * cp + t] / tot;
  }
  __syncthreads();

  // -- 4. received mass per slot, summed over the group's heads in order -----
  {
    // launches of this kernel are serialised, so the previous layer's sum is final
    float* mrow = a.mass + (static_cast<size_t>(s) * Hkv + h) * ntot + t0;
    for (int t = tid; t < n; t += DEC_THREADS) {
      float m = 0.f;
      for (int g = 0; g < G; ++g) m += sc[g * cp + t];
      mrow[t] = a.layer == 0 ? m : __fadd_rn(mrow[t], m);
    }
  }

  // -- 5. P.V and the cluster reduction -----------------------------------------
  mbar_wait_bounded(&bar[1], 0, a.sess.dev_status);
  {
    constexpr int HPT = GP / (DEC_THREADS / DEC_D);  // heads per thread
    const int d = tid % DEC_D;
    const int hb = (tid / DEC_D) * HPT;
    float acc[HPT];
#pragma unroll
    for (int i = 0; i < HPT; ++i) acc[i] = 0.f;
    for (int t = 0; t < n; ++t) {
      const float vf = DT<T>::to_f(reinterpret_cast<const T*>(Vs + t * rowb)[d]);
#pragma unroll
      for (int i = 0; i < HPT; ++i) acc[i] = fmaf(sc[(hb + i) * cp + t], vf, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < HPT; ++i) ob[(hb + i) * DEC_D + d] = acc[i];
  }
  cluster.sync();
  {
    const int total = G * DEC_D;
    const int per = (total + CL - 1) / CL;
    const int e0 = c * per, e1 = min(total, e0 + per);
    for (int e = e0 + tid; e < e1; e += DEC_THREADS) {
      float v = 0.f;
#pragma unroll 1
      for (int r = 0; r < CL; ++r) v += *cluster.map_shared_rank(&ob[e], r);
      const size_t o = (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * DEC_D + e;
      if (a.out_dtype == IC_F32)
        static_cast<float*>(a.out)[o] = v;
      else
        static_cast<T*>(a.out)[o] = DT<T>::from_f(v);
    }
  }
  cluster.sync();  // keep this CTA's shared memory alive until peers are done
}

template <typename T, int CL, int GP>
static int launch_decode(const ic_decode_args& a, cudaStream_t stream) {
  const int ntot = a.tiers.budget + 1;
  const int chunk = (ntot + CL - 1) / CL;
  const DecodeSmem L = decode_smem(chunk, sizeof(T), GP);
  if (L.total > 227 * 1024) {
    set_last_error("decode: budget too large for one cluster's shared memory");
    return IC_ERR_UNSUPPORTED;
  }
  auto kern = decode_kernel<T, CL, GP>;
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(kern, L.total, &smem_limit)) return rc;
  static PerDeviceOnce configured;
  once_per_device(&configured, [&] {
    if (CL > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaGetLastError();
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, a.pool.num_kv_heads, a.sess.num_sessions);
  cfg.blockDim = dim3(DEC_THREADS, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, a, chunk);
  return launch_status("decode_layer");
}

template <typename T, int GP>
static int dispatch_cl(const ic_decode_args& a, cudaStream_t stream) {
  int cl = a.cluster_size;
  if (cl == 0) {
    // 16-CTA clusters when the per-CTA chunk would not fit or when there are
    // few (session, head) groups to spread over 148 SMs.
    const int ntot = a.tiers.budget + 1;
    const int groups = a.sess.num_sessions * a.pool.num_kv_heads;
    const bool fits8 = decode_smem((ntot + 7) / 8, sizeof(T), GP).total <= 227 * 1024;
    cl = (!fits8 || groups * 8 < 148) ? 16 : 8;
  }
  if (cl == 8) return launch_decode<T, 8, GP>(a, stream);
  if (cl == 16) return launch_decode<T, 16, GP>(a, stream);
  set_last_error("decode: cluster_size must be 0, 8 or 16");
  return IC_ERR_INVALID_ARG;
}

template <typename T>
static int dispatch_gp(const ic_decode_args& a, cudaStream_t stream) {
  const int G = a.num_q_heads / a.pool.num_kv_heads;
  if (G <= 8) return dispatch_cl<T, 8>(a, stream);
  return dispatch_cl<T, 16>(a, stream);
}

}  // namespace ic

extern "C" int ic_decode_layer(const ic_decode_args* a, void* stream) {
  using namespace ic;
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->sess.num_sessions == 0) return IC_OK;
  if (!a->pool.k || !a->pool.v || !a->q || !a->k_new || !a->v_new || !a->out || !a->mass ||
      !a->sess.slot_table || !a->sess.occupied) {
    set_last_error("decode: null pointer");
    return IC_ERR_INVALID_ARG;
  }
  if (a->pool.head_dim != DEC_D) {
    set_last_error("decode: head_dim must be 128");
    return IC_ERR_UNSUPPORTED;
  }
  const int Hkv = a->pool.num_kv_heads;
  if (Hkv <= 0 || a->num_q_heads <= 0 || a->num_q_heads % Hkv != 0 || a->num_q_heads / Hkv > 16) {
    set_last_error("decode: num_q_heads must be a multiple of num_kv_heads with group <= 16");
    return IC_ERR_UNSUPPORTED;
  }
  if (a->tiers.budget <= 0 || a->tiers.budget != a->tiers.sink_size + a->tiers.recent_size +
                                                     a->tiers.important_size ||
      a->layer < 0 || a->layer >= a->pool.num_layers || a->sess.num_sessions < 0 ||
      a->pool.pool_tokens <= 0 || a->sess.num_sessions > 65535 || Hkv > 65535) {
    set_last_error("decode: bad sizes");
    return IC_ERR_INVALID_ARG;
  }
  if (a->out_dtype != a->pool.dtype && a->out_dtype != IC_F32) {
    set_last_error("decode: out_dtype must be the pool dtype or float32");
    return IC_ERR_INVALID_ARG;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int variant = a->kernel_variant;
  if (variant < IC_DECODE_AUTO || variant > IC_DECODE_TENSOR_SPLIT) {
    set_last_error("decode: bad kernel_variant");
    return IC_ERR_INVALID_ARG;
  }
  // AUTO on fp16 / bf16: when the step's inputs are all ready (consecutive
  // layers then overlap) the lean kernel (up to 16 query heads per KV head,
  // else the streaming kernel); one layer at a time, the slot-split kernel.
  const int G = a->num_q_heads / a->pool.num_kv_heads;
  if (a->pool.dtype != IC_F32 && variant == IC_DECODE_TENSOR_SPLIT) return launch_decode_split(*a, st);
  if (a->pool.dtype != IC_F32 && variant == IC_DECODE_AUTO && !(a->inputs_ready && a->pdl) && G <= 16) {
    // shapes the slot-split kernel does not cover (budgets beyond 16 CTAs of
    // 256 slots) fall through to the cluster kernel
    const int rc = launch_decode_split(*a, st);
    if (rc != IC_ERR_UNSUPPORTED) return rc;
  }
  if (a->pool.dtype != IC_F32 &&
      (variant == IC_DECODE_TENSOR_LEAN || (variant == IC_DECODE_AUTO && a->inputs_ready && a->pdl && G <= 16)))
    return launch_decode_lean(*a, st);
  if (a->pool.dtype != IC_F32 &&
      (variant == IC_DECODE_TENSOR_STREAM || (variant == IC_DECODE_AUTO && a->inputs_ready && a->pdl)))
    return launch_decode_stream(*a, st);
  if (a->pool.dtype != IC_F32 && variant != IC_DECODE_CUDA_CORES) return launch_decode_mma(*a, st);
  if (a->pool.dtype == IC_F32 && variant >= IC_DECODE_TENSOR_CORES) {
    set_last_error("decode: the tensor-core variant needs an fp16 or bf16 pool");
    return IC_ERR_UNSUPPORTED;
  }
  switch (a->pool.dtype) {
    case IC_F32: return dispatch_gp<float>(*a, st);
    case IC_F16: return dispatch_gp<__half>(*a, st);
    case IC_BF16: return dispatch_gp<__nv_bfloat16>(*a, st);
    default: set_last_error("decode: bad dtype"); return IC_ERR_INVALID_ARG;
  }
}

extern "C" int ic_decode_step(const ic_step_args* a, void* stream) {
  using namespace ic;
  if (!a) return IC_ERR_INVALID_ARG;
  ic_decode_args d = a->layer0;
  const int esz = dtype_size(d.pool.dtype);
  const int osz = dtype_size(d.out_dtype);
  d.inputs_ready = 1;
  for (int l = 0; l < d.pool.num_layers; ++l) {
    d.layer = l;
    d.q = static_cast<const char*>(a->layer0.q) + static_cast<int64_t>(l) * a->q_layer_stride * esz;
    d.k_new = static_cast<const char*>(a->layer0.k_new) + static_cast<int64_t>(l) * a->kv_layer_stride * esz;
    d.v_new = static_cast<const char*>(a->layer0.v_new) + static_cast<int64_t>(l) * a->kv_layer_stride * esz;
    d.out = static_cast<char*>(a->layer0.out) + static_cast<int64_t>(l) * a->out_layer_stride * osz;
    const int rc = ic_decode_layer(&d, stream);
    if (rc != IC_OK) return rc;
  }
  // the eviction follows a kernel-A layer, which writes none of the session
  // state it stages: that staging need not wait for the layer
  ic_evict_args e = a->evict;
  if (e.pdl == 1) e.pdl = 2;
  return ic_evict_update(&e, stream);
}
