// Kernel A, fp16 / bf16: the fused decode step with tensor-core contractions.
//
// Same cluster decomposition as the fp32 kernel (one cluster of CL CTAs per
// (session, KV head), contiguous chunks of the budget+1 logical slots, K/V
// rows staged in shared memory by TMA-engine bulk copies through the slot
// table, cluster-wide softmax through DSMEM, fixed-order cluster reduction of
// P.V).  The two contractions run on the tensor cores with mma.sync m16n8k16
// (fp32 accumulate):
//   * scores  S[16 x n] = Q[16 x 128] . K^T   -- rows are the G <= 16 query
//     heads of the group (unused rows zero), B fragments from ldmatrix on the
//     padded K rows (272-byte stride: conflict-free);
//   * output  O[16 x 128] = P[16 x n] . V      -- P is split into a high and a
//     low half-precision part (P * 2^12 = hi + lo, each rounded), so the
//     product keeps ~22 bits of P; B fragments from ldmatrix.trans on V.
// Softmax, the received mass and every reduction stay in fp32.
#include <math.h>

#include "common.cuh"
#include "decode_internal.cuh"

namespace ic {

constexpr int MMA_THREADS = 256;
constexpr int MMA_D = 128;
constexpr float P_SCALE = 4096.0f;           // 2^12
constexpr float P_UNSCALE = 1.0f / 4096.0f;  // exact

struct MmaSmem {
  int chunk, npad, cp, ppad, rowb;
  int k_off, v_off, sc_off, p_off, ob_off, red_off, occ_off, bar_off, total;
};

__host__ __device__ inline int mma_align(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ inline MmaSmem mma_smem(int chunk, int GP) {
  MmaSmem L;
  L.chunk = chunk;
  L.npad = mma_align(chunk > 0 ? chunk : 1, 16);
  L.cp = L.npad;
  L.ppad = L.npad + 8;  // half-precision P row stride: conflict-free A fragments
  L.rowb = MMA_D * 2 + 16;
  int o = 0;
  L.k_off = o; o = mma_align(o + L.npad * L.rowb, 128);
  L.v_off = o; o = mma_align(o + L.npad * L.rowb, 128);
  L.sc_off = o; o = mma_align(o + GP * L.cp * 4, 128);
  L.p_off = o; o = mma_align(o + 2 * GP * L.ppad * 2, 128);
  L.ob_off = o; o = mma_align(o + GP * MMA_D * 4, 128);
  L.red_off = o; o = mma_align(o + 2 * GP * 4, 16);
  L.occ_off = o; o = mma_align(o + L.npad, 16);
  L.bar_off = o; o += 16;
  L.total = o;
  return L;
}

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

template <typename T, int CL, int GP>
__global__ void __launch_bounds__(MMA_THREADS, 1) decode_mma_kernel(const ic_decode_args a, int chunk) {
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;  // mma fragment row / column-pair
  const int budget = a.tiers.budget, ntot = budget + 1;
  const int Hkv = a.pool.num_kv_heads, Hq = a.num_q_heads, G = Hq / Hkv;
  const int t0 = c * chunk;
  const int n = max(0, min(chunk, ntot - t0));
  const int stage_t = budget - t0;
  const bool has_stage = stage_t >= 0 && stage_t < n;

  const MmaSmem L = mma_smem(chunk, GP);
  unsigned char* Ks = smem + L.k_off;
  unsigned char* Vs = smem + L.v_off;
  float* sc = reinterpret_cast<float*>(smem + L.sc_off);
  uint16_t* Ph = reinterpret_cast<uint16_t*>(smem + L.p_off);
  uint16_t* Pl = Ph + GP * L.ppad;
  float* ob = reinterpret_cast<float*>(smem + L.ob_off);
  float* red_m = reinterpret_cast<float*>(smem + L.red_off);
  float* red_l = red_m + GP;
  uint8_t* occ_s = smem + L.occ_off;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  const int cp = L.cp, ppad = L.ppad, rowb = L.rowb, npad = L.npad;

  const size_t plane = static_cast<size_t>(a.pool.pool_tokens) * MMA_D;
  const size_t lh = static_cast<size_t>(a.layer) * Hkv + h;
  const T* pk = static_cast<const T*>(a.pool.k) + lh * plane;
  const T* pv = static_cast<const T*>(a.pool.v) + lh * plane;
  const int32_t* st = a.sess.slot_table + static_cast<size_t>(s) * ntot;
  const uint8_t* occ_g = a.sess.occupied + static_cast<size_t>(s) * budget;
  constexpr uint32_t ROW_BYTES = MMA_D * sizeof(T);

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
  for (int t = tid; t < n; t += MMA_THREADS) {
    const int slot = t0 + t;
    if (slot == budget) continue;
    int row = st[slot];
    if (static_cast<unsigned long long>(row) >= static_cast<unsigned long long>(a.pool.pool_tokens)) {
      if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
      row = 0;
    }
    bulk_g2s(Ks + t * rowb, pk + static_cast<size_t>(row) * MMA_D, ROW_BYTES, &bar[0]);
    bulk_g2s(Vs + t * rowb, pv + static_cast<size_t>(row) * MMA_D, ROW_BYTES, &bar[1]);
    occ_s[t] = occ_g[slot];
  }
  // zero the padding rows so the last k-steps multiply finite values
  for (int i = tid; i < (npad - n) * (MMA_D / 8); i += MMA_THREADS) {
    const int t = n + i / (MMA_D / 8), v = i % (MMA_D / 8);
    reinterpret_cast<int4*>(Ks + t * rowb)[v] = make_int4(0, 0, 0, 0);
    reinterpret_cast<int4*>(Vs + t * rowb)[v] = make_int4(0, 0, 0, 0);
  }
  if (has_stage) {
    int row = st[budget];
    const bool row_ok =
        static_cast<unsigned long long>(row) < static_cast<unsigned long long>(a.pool.pool_tokens);
    if (!row_ok && tid == 0 && a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
    const T* kn = static_cast<const T*>(a.k_new) + (static_cast<size_t>(s) * Hkv + h) * MMA_D;
    const T* vn = static_cast<const T*>(a.v_new) + (static_cast<size_t>(s) * Hkv + h) * MMA_D;
    T* dk = static_cast<T*>(a.pool.k) + lh * plane + static_cast<size_t>(row) * MMA_D;
    T* dv = static_cast<T*>(a.pool.v) + lh * plane + static_cast<size_t>(row) * MMA_D;
    if (tid < MMA_D / 8) {
      const int4 kv = reinterpret_cast<const int4*>(kn)[tid];
      const int4 vv = reinterpret_cast<const int4*>(vn)[tid];
      reinterpret_cast<int4*>(Ks + stage_t * rowb)[tid] = kv;
      reinterpret_cast<int4*>(Vs + stage_t * rowb)[tid] = vv;
      if (row_ok) {
        reinterpret_cast<int4*>(dk)[tid] = kv;
        reinterpret_cast<int4*>(dv)[tid] = vv;
      }
    }
    if (tid == 0) occ_s[stage_t] = 1;
  }

  // Q A-fragments: rows g (and g + 8 when GP == 16) of the group's heads
  uint32_t qa[8][4];
  {
    const T* qb = static_cast<const T*>(a.q) + (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * MMA_D;
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(qb + static_cast<size_t>(g) * MMA_D);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(qb + static_cast<size_t>(g + 8) * MMA_D);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int w = kk * 8 + tq;  // 32-bit word of d = 16 kk + 2 tq
      qa[kk][0] = g < G ? q0[w] : 0u;
      qa[kk][2] = g < G ? q0[w + 4] : 0u;
      qa[kk][1] = (GP > 8 && g + 8 < G) ? q1[w] : 0u;
      qa[kk][3] = (GP > 8 && g + 8 < G) ? q1[w + 4] : 0u;
    }
  }

  // -- 2. scores on the tensor cores -------------------------------------------
  mbar_wait_bounded(&bar[0], 0, a.sess.dev_status);
  __syncthreads();
  const float scale = a.scale;
  const uint32_t ks_base = smem_addr(Ks);
  const int nb8 = (n + 7) / 8;
  for (int blk = warp; blk < nb8; blk += MMA_THREADS / 32) {
    const int n0 = blk * 8;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t row_addr = ks_base + (n0 + (lane & 7)) * rowb + (lane >> 3) * 16;
#pragma unroll
    for (int kk2 = 0; kk2 < 4; ++kk2) {
      uint32_t b[4];
      ldsm_x4(b, row_addr + kk2 * 64);
      Mma<T>::run(acc, qa[2 * kk2][0], qa[2 * kk2][1], qa[2 * kk2][2], qa[2 * kk2][3], b[0], b[1]);
      Mma<T>::run(acc, qa[2 * kk2 + 1][0], qa[2 * kk2 + 1][1], qa[2 * kk2 + 1][2], qa[2 * kk2 + 1][3], b[2], b[3]);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = n0 + 2 * tq + j;
      if (t < n) {
        const bool o = occ_s[t] != 0;
        if (g < G) sc[g * cp + t] = o ? acc[j] * scale : -INFINITY;
        if (GP > 8 && g + 8 < G) sc[(g + 8) * cp + t] = o ? acc[2 + j] * scale : -INFINITY;
      }
    }
  }
  __syncthreads();

  // -- 3. softmax across the cluster -----------------------------------------
  for (int gg = warp; gg < G; gg += MMA_THREADS / 32) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[gg * cp + t]);
    m = warp_max(m);
    if (lane == 0) red_m[gg] = m;
  }
  cluster.sync();
  for (int gg = warp; gg < G; gg += MMA_THREADS / 32) {
    float m = -INFINITY;
    if (lane < CL) m = *cluster.map_shared_rank(&red_m[gg], lane);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float e = expf(sc[gg * cp + t] - m);
      sc[gg * cp + t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) red_l[gg] = l;
  }
  cluster.sync();
  for (int gg = warp; gg < GP; gg += MMA_THREADS / 32) {
    if (gg < G) {
      float tot = 0.f;
      if (lane == 0) {
#pragma unroll 1
        for (int r = 0; r < CL; ++r) tot += *cluster.map_shared_rank(&red_l[gg], r);
      }
      tot = __shfl_sync(FULL_MASK, tot, 0);
      for (int t = lane; t < npad; t += 32) {
        float p = 0.f;
        if (t < n) {
          p = sc[gg * cp + t] / tot;
          sc[gg * cp + t] = p;
        }
        const float ps = p * P_SCALE;
        const uint16_t hb = Mma<T>::bits(ps);
        Ph[gg * ppad + t] = hb;
        Pl[gg * ppad + t] = Mma<T>::bits(ps - Mma<T>::back(hb));
      }
    } else {
      for (int t = lane; t < npad; t += 32) {
        Ph[gg * ppad + t] = 0;
        Pl[gg * ppad + t] = 0;
      }
    }
  }
  __syncthreads();

  // -- 4. received mass per slot, summed over the group's heads in order -----
  {
    float* mrow = a.mass + (static_cast<size_t>(s) * Hkv + h) * ntot + t0;
    for (int t = tid; t < n; t += MMA_THREADS) {
      float m = 0.f;
      for (int gg = 0; gg < G; ++gg) m += sc[gg * cp + t];
      mrow[t] = a.accumulate ? mrow[t] + m : m;
    }
  }

  // -- 5. P.V on the tensor cores: warp w owns head_dim columns [16w, 16w+16) --
  mbar_wait_bounded(&bar[1], 0, a.sess.dev_status);
  {
    float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const uint32_t vs_base = smem_addr(Vs);
    const int n0 = warp * 16;
    const uint32_t vaddr = vs_base + (((lane >> 3) & 1) * 8 + (lane & 7)) * rowb + (n0 + (lane >> 4) * 8) * 2;
    const uint32_t* ph0 = reinterpret_cast<const uint32_t*>(Ph + g * ppad);
    const uint32_t* pl0 = reinterpret_cast<const uint32_t*>(Pl + g * ppad);
    const uint32_t* ph1 = reinterpret_cast<const uint32_t*>(Ph + (g + 8) * ppad);
    const uint32_t* pl1 = reinterpret_cast<const uint32_t*>(Pl + (g + 8) * ppad);
    for (int k0 = 0; k0 < npad; k0 += 16) {
      const int w = k0 / 2 + tq;  // 32-bit word of column k0 + 2 tq
      const uint32_t h0 = ph0[w], h2 = ph0[w + 4], l0 = pl0[w], l2 = pl0[w + 4];
      const uint32_t h1 = GP > 8 ? ph1[w] : 0u, h3 = GP > 8 ? ph1[w + 4] : 0u;
      const uint32_t l1 = GP > 8 ? pl1[w] : 0u, l3 = GP > 8 ? pl1[w + 4] : 0u;
      uint32_t b[4];
      ldsm_x4_t(b, vaddr + k0 * rowb);
      Mma<T>::run(o[0], h0, h1, h2, h3, b[0], b[1]);
      Mma<T>::run(o[0], l0, l1, l2, l3, b[0], b[1]);
      Mma<T>::run(o[1], h0, h1, h2, h3, b[2], b[3]);
      Mma<T>::run(o[1], l0, l1, l2, l3, b[2], b[3]);
    }
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int d = n0 + nb * 8 + 2 * tq + j;
        if (g < G) ob[g * MMA_D + d] = o[nb][j] * P_UNSCALE;
        if (GP > 8 && g + 8 < G) ob[(g + 8) * MMA_D + d] = o[nb][2 + j] * P_UNSCALE;
      }
  }
  cluster.sync();
  {
    const int total = G * MMA_D;
    const int per = (total + CL - 1) / CL;
    const int e0 = c * per, e1 = min(total, e0 + per);
    for (int e = e0 + tid; e < e1; e += MMA_THREADS) {
      float v = 0.f;
#pragma unroll 1
      for (int r = 0; r < CL; ++r) v += *cluster.map_shared_rank(&ob[e], r);
      const size_t oi = (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * MMA_D + e;
      if (a.out_dtype == IC_F32)
        static_cast<float*>(a.out)[oi] = v;
      else
        static_cast<T*>(a.out)[oi] = DT<T>::from_f(v);
    }
  }
  cluster.sync();
}

template <typename T, int CL, int GP>
static int launch_mma(const ic_decode_args& a, cudaStream_t stream) {
  const int ntot = a.tiers.budget + 1;
  const int chunk = (ntot + CL - 1) / CL;
  const MmaSmem L = mma_smem(chunk, GP);
  if (L.total > 227 * 1024) {
    set_last_error("decode: budget too large for one cluster's shared memory");
    return IC_ERR_UNSUPPORTED;
  }
  auto kern = decode_mma_kernel<T, CL, GP>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (CL > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, a.pool.num_kv_heads, a.sess.num_sessions);
  cfg.blockDim = dim3(MMA_THREADS, 1, 1);
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
static int mma_cl(const ic_decode_args& a, cudaStream_t stream) {
  int cl = a.cluster_size;
  if (cl == 0) {
    const int ntot = a.tiers.budget + 1;
    const int groups = a.sess.num_sessions * a.pool.num_kv_heads;
    const bool fits8 = mma_smem((ntot + 7) / 8, GP).total <= 227 * 1024;
    cl = (!fits8 || groups * 8 < 148) ? 16 : 8;
  }
  if (cl == 8) return launch_mma<T, 8, GP>(a, stream);
  if (cl == 16) return launch_mma<T, 16, GP>(a, stream);
  set_last_error("decode: cluster_size must be 0, 8 or 16");
  return IC_ERR_INVALID_ARG;
}

int launch_decode_mma(const ic_decode_args& a, cudaStream_t stream) {
  const int G = a.num_q_heads / a.pool.num_kv_heads;
  if (a.pool.dtype == IC_F16) return G <= 8 ? mma_cl<__half, 8>(a, stream) : mma_cl<__half, 16>(a, stream);
  if (a.pool.dtype == IC_BF16)
    return G <= 8 ? mma_cl<__nv_bfloat16, 8>(a, stream) : mma_cl<__nv_bfloat16, 16>(a, stream);
  set_last_error("decode_mma: dtype must be fp16 or bf16");
  return IC_ERR_INVALID_ARG;
}

}  // namespace ic
