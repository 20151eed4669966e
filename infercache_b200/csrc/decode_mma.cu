// Kernel A, fp16 / bf16: the fused decode step with tensor-core
// contractions, partials combined through distributed shared memory.
//
// One thread-block cluster of CL CTAs per (session, KV head); CTA c owns a
// contiguous chunk of the budget+1 logical slots (the last slot is the staging
// row that receives the token being decoded).  Per CTA:
//   1. the chunk's pool rows are looked up in the session's slot table and
//      gathered into padded shared-memory rows with 16-byte asynchronous copies
//      spread over all threads (K rows in one group, V rows in a second), so the
//      whole chunk is requested within a few hundred cycles; the CTA owning the
//      staging row writes the new K/V into the pool and into shared memory;
//   2. scores S[16 x n] = Q[16 x 128] . K^T on the tensor cores (mma.sync
//      m16n8k16, fp32 accumulate; rows are the G <= 16 query heads of the
//      group), two 8-slot blocks in flight per warp;
//   3. softmax in one cluster exchange: each CTA publishes its per-head
//      (max, sum of exp(s - max)); after one cluster barrier every CTA reads
//      the CL pairs in parallel and combines them in a fixed order, so all CTAs
//      hold the same global max and sum;
//   4. the received mass of each slot, summed over the group's heads in order,
//      is written (first layer of a step) or added to the value fetched at the
//      start (later layers);
//   5. O = P . V on the tensor cores with P split into high and low
//      half-precision parts (P * 2^12 = hi + lo, ~22 bits of P), four
//      independent accumulator chains per warp;
//   6. the CL partial outputs are reduced through distributed shared memory:
//      CTA c owns a slice of the output and loads the CL partials of it in
//      parallel, summing them in CTA order.
// No global scratch, no atomics, deterministic.
#include <math.h>

#include "common.cuh"
#include "decode_internal.cuh"
#include "mma_helpers.cuh"

namespace ic {

constexpr int MMA_THREADS = 256;
constexpr int MMA_WARPS = MMA_THREADS / 32;
constexpr int MMA_D = 128;
constexpr int MAXT = 2;                      // chunk <= MAXT * MMA_THREADS

struct MmaSmem {
  int npad, cp, ppad, rowb;
  int k_off, v_off, sc_off, p_off, ob_off, red_off, row_off, occ_off, total;
};

__host__ __device__ inline int mma_align(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ inline MmaSmem mma_smem(int chunk, int GP) {
  MmaSmem L;
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
  L.row_off = o; o = mma_align(o + L.npad * 4, 16);
  L.occ_off = o; o = mma_align(o + L.npad, 16);
  L.total = o;
  return L;
}

template <typename T, int CL, int GP>
__global__ void __launch_bounds__(MMA_THREADS, 1) decode_mma_kernel(const ic_decode_args a, int chunk) {
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;  // mma fragment row / column pair
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
  float* red = reinterpret_cast<float*>(smem + L.red_off);  // [GP][2] local (max, sum)
  int32_t* rowidx = reinterpret_cast<int32_t*>(smem + L.row_off);
  uint8_t* occ_s = smem + L.occ_off;
  const int cp = L.cp, ppad = L.ppad, rowb = L.rowb, npad = L.npad;

  // With programmatic dependent launch, layers after the first gather their
  // K/V rows before waiting on the previous kernel (only the eviction kernel
  // rewrites the slot table, and it completed before layer 0 let its
  // dependents launch); q and the new K/V come after the wait unless the
  // caller marked them ready for the whole step.
  const bool early = a.pdl && a.layer > 0;
  if (a.pdl && !early) grid_dependency_wait();

  const size_t plane = static_cast<size_t>(a.pool.pool_tokens) * MMA_D;
  const size_t lh = static_cast<size_t>(a.layer) * Hkv + h;
  const T* pk = static_cast<const T*>(a.pool.k) + lh * plane;
  const T* pv = static_cast<const T*>(a.pool.v) + lh * plane;
  const int32_t* st = a.sess.slot_table + static_cast<size_t>(s) * ntot;
  const uint8_t* occ_g = a.sess.occupied + static_cast<size_t>(s) * budget;

  // q A-fragments (rows g, and g + 8 when GP == 16): loaded before the K/V
  // traffic when possible so they do not queue behind it
  uint32_t qa[8][4];
  auto load_inputs = [&]() {
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
  };
  if (!early || a.inputs_ready) load_inputs();

  // -- 1. gather the chunk's rows ------------------------------------------------
  for (int t = tid; t < n; t += MMA_THREADS) {
    const int slot = t0 + t;
    int row = -1;
    uint8_t o = 1;
    if (slot != budget) {
      row = st[slot];
      o = occ_g[slot];
      if (static_cast<unsigned long long>(row) >= static_cast<unsigned long long>(a.pool.pool_tokens)) {
        if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
        row = 0;
      }
    }
    rowidx[t] = row;
    occ_s[t] = o;
  }
  __syncthreads();
  constexpr int VPR = MMA_D * 2 / 16;  // 16-byte vectors per row
  for (int pass = 0; pass < 2; ++pass) {
    unsigned char* dst = pass == 0 ? Ks : Vs;
    const T* src = pass == 0 ? pk : pv;
    for (int i = tid; i < n * VPR; i += MMA_THREADS) {
      const int t = i / VPR, v = i % VPR;
      const int row = rowidx[t];
      if (row >= 0) cp_async16(dst + t * rowb + v * 16, src + static_cast<size_t>(row) * MMA_D + v * 8);
    }
    cp_async_commit();
  }
  if (early) {
    grid_dependency_wait();
    if (!a.inputs_ready) load_inputs();
  }
  if (a.pdl) grid_launch_dependents();
  // the previous layers' mass sum of this CTA's slots, final once the grid
  // dependency wait has returned: fetched now so its latency overlaps the scores
  float* mrow = a.mass + (static_cast<size_t>(s) * Hkv + h) * ntot + t0;
  float mprev[MAXT];
#pragma unroll
  for (int i = 0; i < MAXT; ++i) {
    const int t = tid + i * MMA_THREADS;
    mprev[i] = (a.layer != 0 && t < n) ? mrow[t] : 0.f;
  }
  for (int i = tid; i < (npad - n) * VPR; i += MMA_THREADS) {
    const int t = n + i / VPR, v = i % VPR;
    reinterpret_cast<int4*>(Ks + t * rowb)[v] = make_int4(0, 0, 0, 0);
    reinterpret_cast<int4*>(Vs + t * rowb)[v] = make_int4(0, 0, 0, 0);
  }
  if (has_stage && tid < VPR) {
    const int row = st[budget];
    const bool row_ok =
        static_cast<unsigned long long>(row) < static_cast<unsigned long long>(a.pool.pool_tokens);
    if (!row_ok && tid == 0 && a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
    const int4 kv = reinterpret_cast<const int4*>(static_cast<const T*>(a.k_new) +
                                                  (static_cast<size_t>(s) * Hkv + h) * MMA_D)[tid];
    const int4 vv = reinterpret_cast<const int4*>(static_cast<const T*>(a.v_new) +
                                                  (static_cast<size_t>(s) * Hkv + h) * MMA_D)[tid];
    reinterpret_cast<int4*>(Ks + stage_t * rowb)[tid] = kv;
    reinterpret_cast<int4*>(Vs + stage_t * rowb)[tid] = vv;
    if (row_ok) {
      reinterpret_cast<int4*>(static_cast<T*>(a.pool.k) + lh * plane + static_cast<size_t>(row) * MMA_D)[tid] = kv;
      reinterpret_cast<int4*>(static_cast<T*>(a.pool.v) + lh * plane + static_cast<size_t>(row) * MMA_D)[tid] = vv;
    }
  }

  // -- 2. scores on the tensor cores, two 8-slot blocks per warp in flight -------
  cp_async_wait<1>();
  __syncthreads();
  const float scale = a.scale;
  {
    const uint32_t ks_base = smem_addr(Ks);
    const int nb8 = (n + 7) / 8;
    for (int blk = warp; blk < nb8; blk += 2 * MMA_WARPS) {
      const int blk2 = blk + MMA_WARPS < nb8 ? blk + MMA_WARPS : blk;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const uint32_t ra = ks_base + (blk * 8 + (lane & 7)) * rowb + (lane >> 3) * 16;
      const uint32_t rb = ks_base + (blk2 * 8 + (lane & 7)) * rowb + (lane >> 3) * 16;
#pragma unroll
      for (int kk2 = 0; kk2 < 4; ++kk2) {
        uint32_t b[4], b2[4];
        ldsm_x4(b, ra + kk2 * 64);
        ldsm_x4(b2, rb + kk2 * 64);
        const uint32_t* x = qa[2 * kk2];
        const uint32_t* y = qa[2 * kk2 + 1];
        Mma<T>::run(acc[0], x[0], x[1], x[2], x[3], b[0], b[1]);
        Mma<T>::run(acc[1], x[0], x[1], x[2], x[3], b2[0], b2[1]);
        Mma<T>::run(acc[0], y[0], y[1], y[2], y[3], b[2], b[3]);
        Mma<T>::run(acc[1], y[0], y[1], y[2], y[3], b2[2], b2[3]);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && blk2 == blk) break;
        const int n0 = (u == 0 ? blk : blk2) * 8;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int t = n0 + 2 * tq + j;
          if (t < n) {
            const bool o = occ_s[t] != 0;
            if (g < G) sc[g * cp + t] = o ? acc[u][j] * scale : -INFINITY;
            if (GP > 8 && g + 8 < G) sc[(g + 8) * cp + t] = o ? acc[u][2 + j] * scale : -INFINITY;
          }
        }
      }
    }
  }
  __syncthreads();

  // -- 3. local (max, sum of exp) per head, one cluster exchange ----------------
  for (int gg = warp; gg < G; gg += MMA_WARPS) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[gg * cp + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float e = m == -INFINITY ? 0.f : expf(sc[gg * cp + t] - m);
      sc[gg * cp + t] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      red[2 * gg] = m;
      red[2 * gg + 1] = l;
    }
  }
  cluster.sync();
  for (int gg = warp; gg < GP; gg += MMA_WARPS) {
    if (gg >= G) {
      for (int t = lane; t < npad; t += 32) { Ph[gg * ppad + t] = 0; Pl[gg * ppad + t] = 0; }
      continue;
    }
    float mr = -INFINITY, lr = 0.f;
    if (lane < CL) {
      const float* rp = cluster.map_shared_rank(&red[2 * gg], lane);
      mr = rp[0];
      lr = rp[1];
    }
    const float M = warp_max(mr);
    const float Lsum = warp_sum(mr == -INFINITY ? 0.f : lr * expf(mr - M));
    const float mc = red[2 * gg];
    const float f = mc == -INFINITY ? 0.f : expf(mc - M) / Lsum;
    for (int t = lane; t < npad; t += 32) {
      float p = 0.f;
      if (t < n) {
        p = sc[gg * cp + t] * f;
        sc[gg * cp + t] = p;
      }
      const float ps = p * P_SCALE;
      const uint16_t hb = Mma<T>::bits(ps);
      Ph[gg * ppad + t] = hb;
      Pl[gg * ppad + t] = Mma<T>::bits(ps - Mma<T>::back(hb));
    }
  }
  __syncthreads();

  // -- 4. received mass per slot, summed over the group's heads in order -------
#pragma unroll
  for (int i = 0; i < MAXT; ++i) {
    const int t = tid + i * MMA_THREADS;
    if (t < n) {
      float m = 0.f;
      for (int gg = 0; gg < G; ++gg) m += sc[gg * cp + t];
      mrow[t] = a.layer == 0 ? m : __fadd_rn(mprev[i], m);
    }
  }

  // -- 5. P.V on the tensor cores: warp w owns head_dim columns [16w, 16w+16) ---
  cp_async_wait<0>();
  __syncthreads();
  {
    float oh[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    float ol[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int n0 = warp * 16;
    const uint32_t vaddr = smem_addr(Vs) + (((lane >> 3) & 1) * 8 + (lane & 7)) * rowb + (n0 + (lane >> 4) * 8) * 2;
    const uint32_t* ph0 = reinterpret_cast<const uint32_t*>(Ph + g * ppad);
    const uint32_t* pl0 = reinterpret_cast<const uint32_t*>(Pl + g * ppad);
    const uint32_t* ph1 = reinterpret_cast<const uint32_t*>(Ph + (g + 8) * ppad);
    const uint32_t* pl1 = reinterpret_cast<const uint32_t*>(Pl + (g + 8) * ppad);
#pragma unroll 2
    for (int k0 = 0; k0 < npad; k0 += 16) {
      const int w = k0 / 2 + tq;  // 32-bit word of column k0 + 2 tq
      const uint32_t h0 = ph0[w], h2 = ph0[w + 4], l0 = pl0[w], l2 = pl0[w + 4];
      const uint32_t h1 = GP > 8 ? ph1[w] : 0u, h3 = GP > 8 ? ph1[w + 4] : 0u;
      const uint32_t l1 = GP > 8 ? pl1[w] : 0u, l3 = GP > 8 ? pl1[w + 4] : 0u;
      uint32_t b[4];
      ldsm_x4_t(b, vaddr + k0 * rowb);
      Mma<T>::run(oh[0], h0, h1, h2, h3, b[0], b[1]);
      Mma<T>::run(ol[0], l0, l1, l2, l3, b[0], b[1]);
      Mma<T>::run(oh[1], h0, h1, h2, h3, b[2], b[3]);
      Mma<T>::run(ol[1], l0, l1, l2, l3, b[2], b[3]);
    }
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int d = n0 + nb * 8 + 2 * tq + j;
        if (g < G) ob[g * MMA_D + d] = (oh[nb][j] + ol[nb][j]) * P_UNSCALE;
        if (GP > 8 && g + 8 < G) ob[(g + 8) * MMA_D + d] = (oh[nb][2 + j] + ol[nb][2 + j]) * P_UNSCALE;
      }
  }
  cluster.sync();

  // -- 6. CTA c reduces its slice of the output over the CL partials -----------
  {
    const int per = G * MMA_D / CL;
    for (int e = c * per + tid; e < (c + 1) * per; e += MMA_THREADS) {
      float part[CL];
#pragma unroll
      for (int r = 0; r < CL; ++r) part[r] = *cluster.map_shared_rank(&ob[e], r);
      float v = part[0];
#pragma unroll
      for (int r = 1; r < CL; ++r) v += part[r];
      const size_t oi = (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * MMA_D + e;
      if (a.out_dtype == IC_F32)
        static_cast<float*>(a.out)[oi] = v;
      else
        static_cast<T*>(a.out)[oi] = DT<T>::from_f(v);
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still read its shared memory
}

template <typename T, int CL, int GP>
static int launch_mma(const ic_decode_args& a, cudaStream_t stream) {
  const int ntot = a.tiers.budget + 1;
  const int chunk = (ntot + CL - 1) / CL;
  const MmaSmem L = mma_smem(chunk, GP);
  if (L.total > 227 * 1024 || chunk > MAXT * MMA_THREADS) {
    set_last_error("decode: budget too large for one cluster's shared memory");
    return IC_ERR_UNSUPPORTED;
  }
  auto kern = decode_mma_kernel<T, CL, GP>;
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(kern, L.total, &smem_limit)) return rc;
  static PerDeviceOnce configured;
  once_per_device(&configured, [&] {
    if (CL > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaGetLastError();
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL, a.pool.num_kv_heads, a.sess.num_sessions);
  cfg.blockDim = dim3(MMA_THREADS, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, kern, a, chunk);
  return launch_status("decode_layer");
}

template <typename T, int GP>
static int mma_cl(const ic_decode_args& a, cudaStream_t stream) {
  int cl = a.cluster_size;
  const int ntot = a.tiers.budget + 1;
  if (cl == 0) {
    // 8-CTA clusters pack onto the GPCs best; 16 when the chunk would not fit
    const int c8 = (ntot + 7) / 8;
    cl = (mma_smem(c8, GP).total <= 227 * 1024 && c8 <= MAXT * MMA_THREADS) ? 8 : 16;
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
