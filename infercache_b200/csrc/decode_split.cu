// Kernel A, fp16 / bf16, slot-split form: one layer at a time over all
// sessions, for a decoder that computes each layer's q from the previous
// layer's output (the layers cannot overlap the way ic_decode_step lets them).
//
// The launch fills the machine on its own: the budget + 1 logical slots of a
// (session, KV head) group are cut into CL chunks of 16-slot blocks, one CTA
// per chunk, the group's CTAs one thread-block cluster.  At 16 sessions x 2 KV
// heads x 1041 slots CL = 3: 96 CTAs of eleven warps, 352 slots each (two
// 16-slot blocks per warp), one CTA per SM (by default the fewest CTAs per
// group that fit, with at least 64 CTAs in the launch).
// Per CTA:
//   1. every warp looks up its one or two 16-slot blocks in the session's slot
//      table and copies their K rows, then their V rows, into padded shared-
//      memory rows with 16-byte asynchronous copies (two commit groups, so the
//      scores start as soon as K has landed); slots past the last are zero
//      rows; the staging slot (the token being decoded) takes k_new / v_new,
//      which the CTA also writes to the pool.  With programmatic dependent
//      launch, layers after the first issue these copies before waiting for the
//      previous kernel: it does not write this layer's pool rows;
//   2. S^T = K . Q^T on the tensor cores (mma.sync m16n8k16, the warp's K rows
//      as A through ldmatrix, the group's query heads as B in registers), the
//      warp's exact per-head maximum, P = 2^(s - max);
//   3. O^T = V^T . P^T (V rows transposed by ldmatrix.trans, the S^T fragment
//      turned into the P^T operand by movmatrix.trans);
//   4. the warps merge into the CTA's per-head (max, sum, O);
//   5. the cluster merges without a cluster-wide barrier on the way: every CTA
//      pushes its (max, sum) pairs into every peer's shared memory with
//      st.async, completing on the peer's mbarrier; once all CL pairs have
//      arrived each CTA knows the group's softmax, scales its O and pushes
//      slice j of it to CTA j, then, while the slices travel, adds the received
//      mass of its own slots (summed over the group's heads in head order) to
//      the running sum over layers; CTA j sums the CL slices it receives in CTA
//      order (deterministic) and writes its part of `out`.
// No global scratch and no atomics.
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "decode_internal.cuh"
#include "mma_helpers.cuh"

namespace ic {
namespace {

constexpr int SP_D = 128;
constexpr int SP_MAXW = 12;                 // warps per CTA at most
constexpr int SP_MAXCL = 16;                // CTAs per cluster at most
constexpr int SP_PITCH = SP_D * 2 + 16;     // padded row: conflict-free ldmatrix
constexpr float SP_LOG2E = 1.4426950408889634f;

__host__ __device__ inline int sp_align(int x, int a) { return (x + a - 1) / a * a; }

// The geometry of one launch: CL CTAs per group, `chunk` slots per CTA
// (16-slot blocks), W warps of RB blocks each.
struct SplitGeom {
  int cl, chunk, blocks, rb, w, slice;
};

__host__ __device__ inline SplitGeom split_geometry(int ntot, int hs, int cl_req) {
  SplitGeom g;
  // cl_req CTAs per group; 0: 8 (portable cluster size) while they hold at most
  // 16 blocks of 16 slots each, else as many as 16-block CTAs need
  const int cl0 = cl_req > 0 ? cl_req : (ntot <= 8 * 256 ? 8 : (ntot + 255) / 256);
  g.blocks = (ntot + 16 * cl0 - 1) / (16 * cl0);
  g.chunk = 16 * g.blocks;
  g.cl = (ntot + g.chunk - 1) / g.chunk;
  // two 16-slot blocks per warp once a CTA holds more than four: fewer warps
  // to merge measured faster at every cluster size tried
  g.rb = g.blocks > 4 ? 2 : 1;
  g.w = (g.blocks + g.rb - 1) / g.rb;
  g.slice = sp_align((hs * SP_D + g.cl - 1) / g.cl, 4);  // O floats reduced by each CTA
  return g;
}

struct SplitSmem {
  int k_off, v_off, sc_off, row_off, occ_off, stin_off, red_off, ocs_off, cst_off, bar_off, total, pitch, rows;
};

__host__ __device__ inline SplitSmem split_smem(const SplitGeom& g, int hs) {
  SplitSmem L;
  L.rows = 16 * g.rb * g.w;  // rows the warps cover (>= chunk)
  int o = 0;
  L.k_off = o;    o += L.rows * SP_PITCH;
  L.v_off = o;    o += L.rows * SP_PITCH;
  L.pitch = L.rows + 4;
  L.sc_off = o;   o += hs * L.pitch * 4;
  L.row_off = o;  o += L.rows * 4;
  L.occ_off = o;  o = sp_align(o + L.rows, 16);
  L.stin_off = o; o += SP_MAXCL * hs * 2 * 4;        // [CL][hs] (max, sum) from every CTA
  L.red_off = o;  o += g.cl * g.slice * 4;           // [CL][slice] O slices from every CTA
  L.ocs_off = o;  o += hs * SP_D * 4;                // this CTA's merged O [hs][128]
  L.cst_off = o;  o += 4 * hs * 4;                   // m_cta, l_cta, M, 1 / L per head
  L.bar_off = o;  o += 16;                           // mbarriers: stats, O slices
  L.total = o;
  return L;
}

__device__ __forceinline__ uint32_t sp_movtrans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t sp_pack(float lo, float hi) {
  return static_cast<uint32_t>(Mma<T>::bits(lo)) | (static_cast<uint32_t>(Mma<T>::bits(hi)) << 16);
}

__device__ __forceinline__ float sp_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Wait for an mbarrier phase completed by other CTAs' st.async (cluster-scope
// acquire), bounded like mbar_wait_bounded.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, int32_t* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (global_timer_ns() - t0 > 2000000000ull) {
      if (status) atomicOr(status, IC_DEVFLAG_TIMEOUT);
      return false;
    }
  }
}

template <typename T, int NG, int RB>
__global__ void __launch_bounds__(SP_MAXW * 32, 1) decode_split_kernel(const ic_decode_args a, SplitGeom geo) {
  constexpr int HS = NG * 8;        // query heads per group, padded to the mma's n = 8
  constexpr int R = 16 * RB;        // slots per warp
  constexpr bool SPLITP = std::is_same<T, __nv_bfloat16>::value;  // P as high + low bf16
  extern __shared__ __align__(128) unsigned char smem[];
  const int c = static_cast<int>(cluster_ctarank());
  const int h = blockIdx.y, s = blockIdx.z;
  const int nthr = blockDim.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int budget = a.tiers.budget, ntot = budget + 1;
  const int Hkv = a.pool.num_kv_heads, Hq = a.num_q_heads, G = Hq / Hkv;
  const int CL = geo.cl, chunk = geo.chunk, W = geo.w, SL = geo.slice;
  const SplitSmem L = split_smem(geo, HS);
  unsigned char* Ks = smem + L.k_off;
  unsigned char* Vs = smem + L.v_off;
  float* sc = reinterpret_cast<float*>(smem + L.sc_off);  // [HS][pitch] log2-scaled scores
  int32_t* rows = reinterpret_cast<int32_t*>(smem + L.row_off);
  uint8_t* occ_s = smem + L.occ_off;
  float* stin = reinterpret_cast<float*>(smem + L.stin_off);   // [CL][HS][2]
  float* red = reinterpret_cast<float*>(smem + L.red_off);     // [CL][SL]
  float* ocs = reinterpret_cast<float*>(smem + L.ocs_off);     // [HS][SP_D]
  float* cst = reinterpret_cast<float*>(smem + L.cst_off);     // [4][HS]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  const int pitch = L.pitch;
  const int own0 = c * chunk;                      // first slot of this CTA
  const int nown = max(0, min(chunk, ntot - own0));  // slots it owns
  const int red_len = max(0, min(SL, HS * SP_D - c * SL));  // O floats it reduces

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&bar[0], static_cast<uint32_t>(CL * HS * 2 * 4));
    mbar_arrive_expect_tx(&bar[1], static_cast<uint32_t>(CL * red_len * 4));
  }
  // peers may push into this CTA's shared memory once every CTA has passed here
  cluster_arrive_release();

  // Layer 0 may follow the eviction kernel, which rewrites the slot table and
  // occupancy: wait first.  Later layers read nothing the previous kernel
  // writes until the grid-dependency wait below.
  const bool early = a.pdl && a.layer > 0;
  if (a.pdl && !early) grid_dependency_wait();

  const size_t plane = static_cast<size_t>(a.pool.pool_tokens) * SP_D;
  const size_t lh = static_cast<size_t>(a.layer) * Hkv + h;
  const T* pk = static_cast<const T*>(a.pool.k) + lh * plane;
  const T* pv = static_cast<const T*>(a.pool.v) + lh * plane;
  const int32_t* st = a.sess.slot_table + static_cast<size_t>(s) * ntot;
  const uint8_t* occ_g = a.sess.occupied + static_cast<size_t>(s) * budget;

  // ---- 1. this warp's rows: slot table, then 16-byte asynchronous copies -------
  const int wbase = warp * R;              // first row of this warp in the CTA
  if (lane < R) {
    const int r = wbase + lane;
    const int t = own0 + r;
    int row = -1;                          // pool row; -2 staging slot; -1 no slot
    uint8_t o = 0;
    if (r < nown) {
      if (t < budget) {
        row = st[t];
        o = occ_g[t];
        if (static_cast<unsigned long long>(row) >= static_cast<unsigned long long>(a.pool.pool_tokens)) {
          if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
          row = 0;
          o = 0;
        }
      } else {
        row = -2;
        o = 1;
      }
    }
    rows[r] = row;
    occ_s[r] = o;
  }
  __syncwarp();
  // K rows in one commit group, V rows in a second; half-warps take a row per
  // pass (256 contiguous bytes); rows without a slot are zero (their scores are
  // masked; V must be finite)
  constexpr int VPR = SP_D * 2 / 16;  // 16-byte vectors per row
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    unsigned char* dst = pass == 0 ? Ks : Vs;
    const T* src = pass == 0 ? pk : pv;
#pragma unroll 4
    for (int i = lane; i < R * VPR; i += 32) {
      const int r = wbase + i / VPR, v = i % VPR;
      const int row = rows[r];
      unsigned char* d = dst + r * SP_PITCH + v * 16;
      if (row >= 0)
        cp_async16(d, src + static_cast<size_t>(row) * SP_D + v * 8);
      else if (row == -1)
        *reinterpret_cast<int4*>(d) = make_int4(0, 0, 0, 0);
    }
    cp_async_commit();
  }

  if (early) grid_dependency_wait();
  if (a.pdl) grid_launch_dependents();

  // ---- q of the group as the B operand (Q^T), after the wait: it may come from
  // the previous kernel; heads past G are zero
  uint32_t qb[NG][8][2];
  {
    const T* qg = static_cast<const T*>(a.q) + (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * SP_D;
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) {
      const int head = nt * 8 + g;
      const uint32_t* qr = reinterpret_cast<const uint32_t*>(qg + static_cast<size_t>(head) * SP_D);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[nt][kk][0] = head < G ? qr[kk * 8 + tq] : 0u;
        qb[nt][kk][1] = head < G ? qr[kk * 8 + 4 + tq] : 0u;
      }
    }
  }
  // the staging slot: the new token's K/V into shared memory and the pool
  if (own0 + wbase <= budget && budget < own0 + wbase + R && budget - own0 < nown) {
    const int r = budget - own0;
    const T* kn = static_cast<const T*>(a.k_new) + (static_cast<size_t>(s) * Hkv + h) * SP_D;
    const T* vn = static_cast<const T*>(a.v_new) + (static_cast<size_t>(s) * Hkv + h) * SP_D;
    if (lane < VPR) {
      const int4 kv = reinterpret_cast<const int4*>(kn)[lane];
      const int4 vv = reinterpret_cast<const int4*>(vn)[lane];
      reinterpret_cast<int4*>(Ks + r * SP_PITCH)[lane] = kv;
      reinterpret_cast<int4*>(Vs + r * SP_PITCH)[lane] = vv;
      const int row = st[budget];
      if (static_cast<unsigned long long>(row) < static_cast<unsigned long long>(a.pool.pool_tokens)) {
        reinterpret_cast<int4*>(static_cast<T*>(a.pool.k) + lh * plane + static_cast<size_t>(row) * SP_D)[lane] = kv;
        reinterpret_cast<int4*>(static_cast<T*>(a.pool.v) + lh * plane + static_cast<size_t>(row) * SP_D)[lane] = vv;
      } else if (lane == 0 && a.sess.dev_status) {
        atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
      }
    }
  }
  // the previous layers' mass sum of this CTA's slots (final once the grid
  // dependency wait has returned), fetched now so its latency overlaps the scores
  float* macc = a.mass + (static_cast<size_t>(s) * Hkv + h) * ntot + own0;
  float mprev[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = tid + i * nthr;
    if (a.layer > 0 && r < nown) mprev[i] = macc[r];
  }

  // ---- 2. S^T = K Q^T, the warp's per-head max, P ---------------------------------
  const float sl2 = a.scale * SP_LOG2E;
  cp_async_wait<1>();
  __syncwarp();
  float acc[RB][NG][4];
#pragma unroll
  for (int rb = 0; rb < RB; ++rb) {
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) acc[rb][nt][0] = acc[rb][nt][1] = acc[rb][nt][2] = acc[rb][nt][3] = 0.f;
    const uint32_t ka = smem_addr(Ks) + (wbase + rb * 16 + (lane & 15)) * SP_PITCH + (lane >> 4) * 16;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t ar[4];
      ldsm_x4(ar, ka + kk * 32);
#pragma unroll
      for (int nt = 0; nt < NG; ++nt)
        Mma<T>::run(acc[rb][nt], ar[0], ar[1], ar[2], ar[3], qb[nt][kk][0], qb[nt][kk][1]);
    }
  }
  float mw[NG][2];
#pragma unroll
  for (int nt = 0; nt < NG; ++nt) mw[nt][0] = mw[nt][1] = -INFINITY;
#pragma unroll
  for (int rb = 0; rb < RB; ++rb) {
    const int r0 = wbase + rb * 16;
    const bool ok0 = occ_s[r0 + g] != 0, ok1 = occ_s[r0 + g + 8] != 0;
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) {
      // [0], [1]: row g, heads 2tq, 2tq+1; [2], [3]: row g + 8
      const float x0 = ok0 ? acc[rb][nt][0] * sl2 : -INFINITY, x1 = ok0 ? acc[rb][nt][1] * sl2 : -INFINITY;
      const float x2 = ok1 ? acc[rb][nt][2] * sl2 : -INFINITY, x3 = ok1 ? acc[rb][nt][3] * sl2 : -INFINITY;
      acc[rb][nt][0] = x0; acc[rb][nt][1] = x1; acc[rb][nt][2] = x2; acc[rb][nt][3] = x3;
      float* sc0 = sc + (nt * 8 + 2 * tq) * pitch + r0;
      sc0[g] = x0;
      sc0[pitch + g] = x1;
      sc0[g + 8] = x2;
      sc0[pitch + g + 8] = x3;
      mw[nt][0] = fmaxf(mw[nt][0], fmaxf(x0, x2));
      mw[nt][1] = fmaxf(mw[nt][1], fmaxf(x1, x3));
    }
  }
#pragma unroll
  for (int nt = 0; nt < NG; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) mw[nt][j] = fmaxf(mw[nt][j], __shfl_xor_sync(FULL_MASK, mw[nt][j], off));

  float lw[NG][2];
  uint32_t bh[RB][NG][2], bl[RB][NG][2];
#pragma unroll
  for (int nt = 0; nt < NG; ++nt) lw[nt][0] = lw[nt][1] = 0.f;
#pragma unroll
  for (int rb = 0; rb < RB; ++rb) {
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) {
      float p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float m = mw[nt][i & 1];
        p[i] = m == -INFINITY ? 0.f : sp_ex2(acc[rb][nt][i] - m);
      }
      lw[nt][0] += p[0] + p[2];
      lw[nt][1] += p[1] + p[3];
      const uint32_t h01 = sp_pack<T>(p[0], p[1]), h23 = sp_pack<T>(p[2], p[3]);
      bh[rb][nt][0] = sp_movtrans(h01);
      bh[rb][nt][1] = sp_movtrans(h23);
      if (SPLITP) {
        const float r0f = p[0] - Mma<T>::back(static_cast<uint16_t>(h01 & 0xffffu));
        const float r1f = p[1] - Mma<T>::back(static_cast<uint16_t>(h01 >> 16));
        const float r2f = p[2] - Mma<T>::back(static_cast<uint16_t>(h23 & 0xffffu));
        const float r3f = p[3] - Mma<T>::back(static_cast<uint16_t>(h23 >> 16));
        bl[rb][nt][0] = sp_movtrans(sp_pack<T>(r0f, r1f));
        bl[rb][nt][1] = sp_movtrans(sp_pack<T>(r2f, r3f));
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < NG; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) lw[nt][j] += __shfl_xor_sync(FULL_MASK, lw[nt][j], off);

  // ---- 3. O^T = V^T P^T -------------------------------------------------------------
  cp_async_wait<0>();
  __syncwarp();
  float o[NG][8][4];
#pragma unroll
  for (int nt = 0; nt < NG; ++nt)
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
#pragma unroll
  for (int rb = 0; rb < RB; ++rb) {
    const uint32_t va =
        smem_addr(Vs) + (wbase + rb * 16 + (lane & 7) + ((lane >> 4) << 3)) * SP_PITCH + ((lane >> 3) & 1) * 16;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      uint32_t ar[4];
      ldsm_x4_t(ar, va + mt * 32);
#pragma unroll
      for (int nt = 0; nt < NG; ++nt) {
        Mma<T>::run(o[nt][mt], ar[0], ar[1], ar[2], ar[3], bh[rb][nt][0], bh[rb][nt][1]);
        if (SPLITP) Mma<T>::run(o[nt][mt], ar[0], ar[1], ar[2], ar[3], bl[rb][nt][0], bl[rb][nt][1]);
      }
    }
  }

  // ---- 4. merge the warps into the CTA's (max, sum, O) ------------------------------
  __syncthreads();  // K / V rows are free: the warp buffers alias them
  float* wo = reinterpret_cast<float*>(smem);  // [W][HS][SP_D]
  float* wm = wo + W * HS * SP_D;              // [W][HS]
  float* wl = wm + W * HS;                     // [W][HS]
#pragma unroll
  for (int nt = 0; nt < NG; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int head = nt * 8 + 2 * tq + j;
      float* dst = wo + (warp * HS + head) * SP_D;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        dst[mt * 16 + g] = o[nt][mt][j];
        dst[mt * 16 + g + 8] = o[nt][mt][2 + j];
      }
      if (g == 0) {
        wm[warp * HS + head] = mw[nt][j];
        wl[warp * HS + head] = lw[nt][j];
      }
    }
  }
  __syncthreads();
  float* m_cta = cst;
  float* l_cta = cst + HS;
  float* gM = cst + 2 * HS;
  float* gI = cst + 3 * HS;
  for (int e = tid; e < HS * (SP_D / 4); e += nthr) {
    const int head = e / (SP_D / 4), d0 = (e % (SP_D / 4)) * 4;
    float M = -INFINITY;
    for (int w = 0; w < W; ++w) M = fmaxf(M, wm[w * HS + head]);
    float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f, lsum = 0.f;
    for (int w = 0; w < W; ++w) {
      const float m = wm[w * HS + head];
      const float f = m == -INFINITY ? 0.f : sp_ex2(m - M);
      lsum = fmaf(wl[w * HS + head], f, lsum);
      const float4 u = *reinterpret_cast<const float4*>(wo + (w * HS + head) * SP_D + d0);
      x0 = fmaf(u.x, f, x0); x1 = fmaf(u.y, f, x1); x2 = fmaf(u.z, f, x2); x3 = fmaf(u.w, f, x3);
    }
    *reinterpret_cast<float4*>(ocs + head * SP_D + d0) = make_float4(x0, x1, x2, x3);
    if (d0 == 0) {
      m_cta[head] = M;
      l_cta[head] = lsum;
    }
  }
  __syncthreads();

  // ---- 5. cluster merge --------------------------------------------------------------
  cluster_wait_acquire();  // every peer has initialised its mbarriers
  if (tid < HS) {
    const uint32_t src = smem_addr(stin + (c * HS + tid) * 2);
    const uint32_t b0 = smem_addr(&bar[0]);
    const uint32_t mx = __float_as_uint(m_cta[tid]), ls = __float_as_uint(l_cta[tid]);
    for (int j = 0; j < CL; ++j) st_async_v2(map_shared(src, j), mx, ls, map_shared(b0, j));
  }
  mbar_wait_cluster_bounded(&bar[0], 0, a.sess.dev_status);
  if (tid < HS) {
    float M = -INFINITY;
    for (int j = 0; j < CL; ++j) M = fmaxf(M, stin[(j * HS + tid) * 2]);
    float lsum = 0.f;
    for (int j = 0; j < CL; ++j) {
      const float m = stin[(j * HS + tid) * 2];
      lsum = fmaf(stin[(j * HS + tid) * 2 + 1], m == -INFINITY ? 0.f : sp_ex2(m - M), lsum);
    }
    gM[tid] = M;
    gI[tid] = lsum > 0.f ? 1.f / lsum : 0.f;
  }
  __syncthreads();
  // this CTA's O scaled to the group's softmax, slice j pushed to CTA j
  {
    const uint32_t b1 = smem_addr(&bar[1]);
    for (int e4 = tid; e4 < HS * SP_D / 4; e4 += nthr) {
      const int e = 4 * e4, head = e / SP_D;
      const float m = m_cta[head];
      const float f = m == -INFINITY ? 0.f : sp_ex2(m - gM[head]) * gI[head];
      const float4 u = *reinterpret_cast<const float4*>(ocs + e);
      const int j = e / SL, off = e - j * SL;
      const uint32_t dst = map_shared(smem_addr(red + c * SL + off), j);
      st_async_v4(dst, __float_as_uint(u.x * f), __float_as_uint(u.y * f), __float_as_uint(u.z * f),
                  __float_as_uint(u.w * f), map_shared(b1, j));
    }
  }
  // received mass of this CTA's slots (exact softmax, heads in order), folded into
  // the running sum over layers after the previous layer's kernel has completed
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = tid + i * nthr;
    if (r < nown) {
      float m = 0.f;
      for (int head = 0; head < G; ++head) {
        const float x = sc[head * pitch + r];
        if (x != -INFINITY) m += sp_ex2(x - gM[head]) * gI[head];
      }
      macc[r] = a.layer == 0 ? m : __fadd_rn(mprev[i], m);
    }
  }
  for (int r = tid + 2 * nthr; r < nown; r += nthr) {  // chunks longer than two rows per thread
    float m = 0.f;
    for (int head = 0; head < G; ++head) {
      const float x = sc[head * pitch + r];
      if (x != -INFINITY) m += sp_ex2(x - gM[head]) * gI[head];
    }
    macc[r] = a.layer == 0 ? m : __fadd_rn(macc[r], m);
  }
  mbar_wait_cluster_bounded(&bar[1], 0, a.sess.dev_status);
  // sum the CL slices of this CTA's part of O in CTA order; heads past G are padding
  {
    const size_t ob = (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * SP_D;
    for (int e4 = tid; e4 < red_len / 4; e4 += nthr) {
      const int e = c * SL + 4 * e4, head = e / SP_D;
      if (head >= G) continue;
      float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
      for (int j = 0; j < CL; ++j) {
        const float4 u = *reinterpret_cast<const float4*>(red + j * SL + 4 * e4);
        x0 += u.x; x1 += u.y; x2 += u.z; x3 += u.w;
      }
      const size_t o0 = ob + e;
      if (a.out_dtype == IC_F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(a.out) + o0) = make_float4(x0, x1, x2, x3);
      } else {
        *reinterpret_cast<uint2*>(static_cast<T*>(a.out) + o0) = make_uint2(sp_pack<T>(x0, x1), sp_pack<T>(x2, x3));
      }
    }
  }
}

template <typename T, int NG, int RB>
int launch_split(const ic_decode_args& a, cudaStream_t stream, const SplitGeom& geo) {
  const SplitSmem L = split_smem(geo, NG * 8);
  auto kern = decode_split_kernel<T, NG, RB>;
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(kern, L.total, &smem_limit)) return rc;
  if (geo.cl > 8) {
    static PerDeviceOnce nonportable;
    once_per_device(&nonportable, [&] {
      cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      cudaGetLastError();
    });
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(geo.cl, a.pool.num_kv_heads, a.sess.num_sessions);
  cfg.blockDim = dim3(32 * geo.w, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = geo.cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, kern, a, geo);
  return launch_status("decode_layer (split)");
}

template <typename T>
int split_dispatch(const ic_decode_args& a, cudaStream_t stream, const SplitGeom& g, int hs) {
  if (hs == 8) return g.rb == 1 ? launch_split<T, 1, 1>(a, stream, g) : launch_split<T, 1, 2>(a, stream, g);
  return g.rb == 1 ? launch_split<T, 2, 1>(a, stream, g) : launch_split<T, 2, 2>(a, stream, g);
}

}  // namespace

int launch_decode_split(const ic_decode_args& a, cudaStream_t stream) {
  const int G = a.num_q_heads / a.pool.num_kv_heads;
  if (G > 16) {
    set_last_error("decode (split): at most 16 query heads per KV head");
    return IC_ERR_UNSUPPORTED;
  }
  if (a.cluster_size < 0 || a.cluster_size > SP_MAXCL) {
    set_last_error("decode (split): cluster_size must be 0 (choose) or 1..16");
    return IC_ERR_INVALID_ARG;
  }
  const int hs = G <= 8 ? 8 : 16;
  const int ntot = a.tiers.budget + 1, groups = a.sess.num_sessions * a.pool.num_kv_heads;
  auto fits = [&](const SplitGeom& x) {
    return x.blocks <= 2 * SP_MAXW && x.cl <= SP_MAXCL && split_smem(x, hs).total <= 227 * 1024;
  };
  // Default CTAs per group, from timings of chained one-layer launches (16
  // query / 2 KV heads, budgets 1040 and 2048, 4 to 32 sessions): fewer,
  // larger CTAs win as long as the launch still has 64 CTAs or more -- the
  // fewest per group (up to 8) that fit and reach 64; else the rule of
  // split_geometry.
  SplitGeom g = split_geometry(ntot, hs, a.cluster_size);
  if (a.cluster_size == 0) {
    for (int c = 1; c <= 8; ++c) {
      if (groups * c < 64) continue;
      const SplitGeom x = split_geometry(ntot, hs, c);
      if (x.cl == c && fits(x)) {
        g = x;
        break;
      }
    }
  }
  if (g.blocks > 2 * SP_MAXW || g.cl > SP_MAXCL) {
    set_last_error("decode (split): budget too large for 16 CTAs of 384 slots");
    return IC_ERR_UNSUPPORTED;
  }
  const SplitSmem L = split_smem(g, hs);
  if (L.total > 227 * 1024) {
    set_last_error("decode (split): chunk too large for one CTA's shared memory");
    return IC_ERR_UNSUPPORTED;
  }
  if (a.pool.dtype == IC_F16) return split_dispatch<__half>(a, stream, g, hs);
  if (a.pool.dtype == IC_BF16) return split_dispatch<__nv_bfloat16>(a, stream, g, hs);
  set_last_error("decode (split): dtype must be fp16 or bf16");
  return IC_ERR_INVALID_ARG;
}

}  // namespace ic
