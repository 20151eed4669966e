// Kernel A, fp16 / bf16, slot-split form: one layer at a time over all
// sessions, for a decoder that computes each layer's q from the previous
// layer's output (the layers cannot overlap the way ic_decode_step lets them).
//
// The launch fills the machine on its own: the budget + 1 logical slots of
// every (session, KV head) group are cut into chunks of 64 or 128 slots, one
// CTA per (chunk, KV head, session) -- at 16 sessions x 2 KV heads x 1041
// slots, 544 CTAs of four warps.  Per CTA:
//   1. each warp looks up its 16 or 32 slots in the session's slot table and
//      issues one 256-byte cp.async.bulk per K row and per V row into padded
//      shared-memory rows, completing on the warp's own two mbarriers (K, V);
//      slots past the last are zero rows, the staging slot (the token being
//      decoded) takes k_new / v_new, which the CTA also writes to the pool.
//      With programmatic dependent launch, layers after the first issue these
//      copies before waiting for the previous kernel: the pool rows of this
//      layer are not written by it;
//   2. S^T = K . Q^T on the tensor cores (mma.sync m16n8k16, the warp's K rows
//      as A through ldmatrix, the group's query heads as B in registers), the
//      warp's exact per-head maximum, P = 2^(s - max);
//   3. O^T = V^T . P^T (V rows transposed by ldmatrix.trans, the S^T fragment
//      turned into the P^T operand by movmatrix.trans);
//   4. the four warps merge into the CTA's (max, sum, O), which go to the
//      caller's workspace together with the chunk's log2-scaled scores;
//   5. the CTA that arrives last for its group (an atomic counter in the
//      workspace, no waiting) merges the chunks in chunk order -- so the
//      result does not depend on arrival order -- writes `out`, computes every
//      slot's received mass from the stored scores with the exact softmax
//      (summed over the group's heads in head order) and folds it into the
//      running sum over layers, then resets the counter for the next launch.
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "decode_internal.cuh"
#include "mma_helpers.cuh"

namespace ic {
namespace {

constexpr int SP_D = 128;
constexpr int SP_W = 4;                     // warps per CTA
constexpr int SP_THREADS = SP_W * 32;
constexpr int SP_PITCH = SP_D * 2 + 16;     // padded row: conflict-free ldmatrix
constexpr uint32_t SP_ROW_BYTES = SP_D * 2;
constexpr int SP_MAX_SPLITS = 64;
constexpr float SP_LOG2E = 1.4426950408889634f;

__host__ __device__ inline int sp_align(int x, int a) { return (x + a - 1) / a * a; }

struct SplitSmem {
  int k_off, v_off, sc_off, row_off, occ_off, bar_off, flag_off, total, pitch;
};

__host__ __device__ inline SplitSmem split_smem(int chunk, int hs) {
  SplitSmem L;
  int o = 0;
  L.k_off = o;   o += chunk * SP_PITCH;
  L.v_off = o;   o += chunk * SP_PITCH;
  L.pitch = chunk + 4;
  L.sc_off = o;  o += hs * L.pitch * 4;
  L.row_off = o; o += chunk * 4;
  L.occ_off = o; o = sp_align(o + chunk, 16);
  L.bar_off = o; o += 2 * SP_W * 8;
  L.flag_off = o; o += 16;
  L.total = o;
  return L;
}

// Floats of one (session, KV head) group's workspace: per chunk the CTA's
// per-head max and sum, its unnormalised O [hs][128] and the chunk's
// log2-scaled scores [chunk][hs].
__host__ __device__ inline size_t split_group_floats(int splits, int chunk, int hs) {
  return static_cast<size_t>(splits) * hs * (2 + SP_D + chunk);
}
__host__ __device__ inline size_t split_counter_bytes(size_t groups) { return (groups * 4 + 255) / 256 * 256; }

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

template <typename T, int NG, int RB>
__global__ void __launch_bounds__(SP_THREADS, 4) decode_split_kernel(const ic_decode_args a, int splits) {
  constexpr int HS = NG * 8;        // query heads per group, padded to the mma's n = 8
  constexpr int R = 16 * RB;        // slots per warp
  constexpr int CHUNK = SP_W * R;   // slots per CTA
  constexpr bool SPLITP = std::is_same<T, __nv_bfloat16>::value;  // P as high + low bf16
  extern __shared__ __align__(128) unsigned char smem[];
  const int c = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int budget = a.tiers.budget, ntot = budget + 1;
  const int Hkv = a.pool.num_kv_heads, Hq = a.num_q_heads, G = Hq / Hkv;
  const SplitSmem L = split_smem(CHUNK, HS);
  unsigned char* Ks = smem + L.k_off;
  unsigned char* Vs = smem + L.v_off;
  float* sc = reinterpret_cast<float*>(smem + L.sc_off);  // [HS][pitch] log2-scaled scores
  int32_t* rows = reinterpret_cast<int32_t*>(smem + L.row_off);
  uint8_t* occ_s = smem + L.occ_off;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);  // [warp][K, V]
  int* flag = reinterpret_cast<int*>(smem + L.flag_off);
  const int pitch = L.pitch;

  if (tid == 0) {
    for (int i = 0; i < 2 * SP_W; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
  }
  __syncthreads();

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

  // ---- 1. this warp's rows: slot table, then one bulk copy per K and V row ------
  const int wbase = warp * R;              // first row of this warp in the CTA
  const int t0 = c * CHUNK + wbase;        // its first logical slot
  uint64_t* kbar = &bar[2 * warp];
  uint64_t* vbar = &bar[2 * warp + 1];
  int my_row = -1;                         // pool row; -2 staging slot; -1 past the last slot
  bool my_copy = false;
  if (lane < R) {
    const int t = t0 + lane;
    uint8_t o = 0;
    if (t < budget) {
      my_row = st[t];
      o = occ_g[t];
      if (static_cast<unsigned long long>(my_row) >= static_cast<unsigned long long>(a.pool.pool_tokens)) {
        if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
        my_row = 0;
        o = 0;
      }
      my_copy = true;
    } else if (t == budget) {
      my_row = -2;
      o = 1;
    }
    rows[wbase + lane] = my_row;
    occ_s[wbase + lane] = o;
  }
  const uint32_t ncopy = __popc(__ballot_sync(FULL_MASK, my_copy));
  if (lane == 0) {
    mbar_arrive_expect_tx(kbar, ncopy * SP_ROW_BYTES);
    mbar_arrive_expect_tx(vbar, ncopy * SP_ROW_BYTES);
  }
  __syncwarp();
  if (my_copy) {
    bulk_g2s(Ks + (wbase + lane) * SP_PITCH, pk + static_cast<size_t>(my_row) * SP_D, SP_ROW_BYTES, kbar);
    bulk_g2s(Vs + (wbase + lane) * SP_PITCH, pv + static_cast<size_t>(my_row) * SP_D, SP_ROW_BYTES, vbar);
  }
  // rows past the last slot are zero (their scores are masked; V must be finite)
  constexpr int VPR = SP_D * 2 / 16;  // 16-byte vectors per row
  for (int i = lane; i < R * VPR; i += 32) {
    const int r = i / VPR, v = i % VPR;
    if (rows[wbase + r] == -1) {
      reinterpret_cast<int4*>(Ks + (wbase + r) * SP_PITCH)[v] = make_int4(0, 0, 0, 0);
      reinterpret_cast<int4*>(Vs + (wbase + r) * SP_PITCH)[v] = make_int4(0, 0, 0, 0);
    }
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
  if (t0 <= budget && budget < t0 + R) {
    const int r = budget - t0;
    const T* kn = static_cast<const T*>(a.k_new) + (static_cast<size_t>(s) * Hkv + h) * SP_D;
    const T* vn = static_cast<const T*>(a.v_new) + (static_cast<size_t>(s) * Hkv + h) * SP_D;
    if (lane < VPR) {
      const int4 kv = reinterpret_cast<const int4*>(kn)[lane];
      const int4 vv = reinterpret_cast<const int4*>(vn)[lane];
      reinterpret_cast<int4*>(Ks + (wbase + r) * SP_PITCH)[lane] = kv;
      reinterpret_cast<int4*>(Vs + (wbase + r) * SP_PITCH)[lane] = vv;
      const int row = st[budget];
      if (static_cast<unsigned long long>(row) < static_cast<unsigned long long>(a.pool.pool_tokens)) {
        reinterpret_cast<int4*>(static_cast<T*>(a.pool.k) + lh * plane + static_cast<size_t>(row) * SP_D)[lane] = kv;
        reinterpret_cast<int4*>(static_cast<T*>(a.pool.v) + lh * plane + static_cast<size_t>(row) * SP_D)[lane] = vv;
      } else if (lane == 0 && a.sess.dev_status) {
        atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
      }
    }
  }
  __syncwarp();

  // ---- 2. S^T = K Q^T, the warp's per-head max, P ---------------------------------
  const float sl2 = a.scale * SP_LOG2E;
  const bool k_ok = mbar_wait_bounded(kbar, 0, a.sess.dev_status);
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
  const bool v_ok = mbar_wait_bounded(vbar, 0, a.sess.dev_status);
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
  // a copy that outlived its bounded wait must land before the CTA leaves
  if (!k_ok) mbar_wait_bounded(kbar, 0, a.sess.dev_status);
  if (!v_ok) mbar_wait_bounded(vbar, 0, a.sess.dev_status);

  // ---- 4. merge the warps; the CTA's partial to the workspace -----------------------
  __syncthreads();  // K / V rows are free: the merge buffers alias them
  float* wo = reinterpret_cast<float*>(smem);  // [warp][HS][SP_D]
  float* wm = wo + SP_W * HS * SP_D;           // [warp][HS]
  float* wl = wm + SP_W * HS;                  // [warp][HS]
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
  const size_t groups = static_cast<size_t>(a.sess.num_sessions) * Hkv;
  const size_t grp = static_cast<size_t>(s) * Hkv + h;
  int* counter = static_cast<int*>(a.workspace) + grp;
  float* ws = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + split_counter_bytes(groups)) +
              grp * split_group_floats(splits, CHUNK, HS);
  float* ws_m = ws;                                     // [splits][HS]
  float* ws_l = ws_m + splits * HS;                     // [splits][HS]
  float* ws_o = ws_l + splits * HS;                     // [splits][HS][SP_D]
  float* ws_x = ws_o + static_cast<size_t>(splits) * HS * SP_D;  // [splits * CHUNK][HS]
  for (int e = tid; e < HS * (SP_D / 8); e += SP_THREADS) {
    const int head = e / (SP_D / 8), d0 = (e % (SP_D / 8)) * 8;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < SP_W; ++w) M = fmaxf(M, wm[w * HS + head]);
    float f[SP_W], lsum = 0.f;
#pragma unroll
    for (int w = 0; w < SP_W; ++w) {
      const float m = wm[w * HS + head];
      f[w] = m == -INFINITY ? 0.f : sp_ex2(m - M);
      lsum = fmaf(wl[w * HS + head], f[w], lsum);
    }
    float x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = 0.f;
#pragma unroll
      for (int w = 0; w < SP_W; ++w) x[i] = fmaf(wo[(w * HS + head) * SP_D + d0 + i], f[w], x[i]);
    }
    float4* dst = reinterpret_cast<float4*>(ws_o + (static_cast<size_t>(c) * HS + head) * SP_D + d0);
    __stcg(dst, make_float4(x[0], x[1], x[2], x[3]));
    __stcg(dst + 1, make_float4(x[4], x[5], x[6], x[7]));
    if (d0 == 0) {
      __stcg(ws_m + c * HS + head, M);
      __stcg(ws_l + c * HS + head, lsum);
    }
  }
  for (int t = tid; t < CHUNK; t += SP_THREADS) {
    float4* dst = reinterpret_cast<float4*>(ws_x + (static_cast<size_t>(c) * CHUNK + t) * HS);
#pragma unroll
    for (int q4 = 0; q4 < HS / 4; ++q4)
      __stcg(dst + q4, make_float4(sc[(4 * q4) * pitch + t], sc[(4 * q4 + 1) * pitch + t],
                                   sc[(4 * q4 + 2) * pitch + t], sc[(4 * q4 + 3) * pitch + t]));
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) flag[0] = atomicAdd(counter, 1) == splits - 1;
  __syncthreads();
  if (!flag[0]) return;

  // ---- 5. the last CTA of the group: merge the chunks in order ------------------------
  __threadfence();
  float* fcs = reinterpret_cast<float*>(smem);   // [splits][HS] chunk weights, then / L
  float* fls = fcs + SP_MAX_SPLITS * HS;         // [splits][HS] chunk sums
  float* gM = fls + SP_MAX_SPLITS * HS;          // [HS] global max
  float* gI = gM + HS;                           // [HS] 1 / global sum
  for (int i = tid; i < splits * HS; i += SP_THREADS) {
    fcs[i] = __ldcg(ws_m + i);
    fls[i] = __ldcg(ws_l + i);
  }
  __syncthreads();
  if (tid < HS) {
    float M = -INFINITY;
    for (int k = 0; k < splits; ++k) M = fmaxf(M, fcs[k * HS + tid]);
    float lsum = 0.f;
    for (int k = 0; k < splits; ++k) {
      const float m = fcs[k * HS + tid];
      const float f = m == -INFINITY ? 0.f : sp_ex2(m - M);
      fcs[k * HS + tid] = f;
      lsum = fmaf(fls[k * HS + tid], f, lsum);
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    gM[tid] = M;
    gI[tid] = inv;
    for (int k = 0; k < splits; ++k) fcs[k * HS + tid] *= inv;
  }
  __syncthreads();
  {
    const size_t ob = (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * SP_D;
    for (int e = tid; e < G * (SP_D / 8); e += SP_THREADS) {
      const int head = e / (SP_D / 8), d0 = (e % (SP_D / 8)) * 8;
      float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const float4* src = reinterpret_cast<const float4*>(ws_o + static_cast<size_t>(head) * SP_D + d0);
      constexpr size_t CSTRIDE = static_cast<size_t>(HS) * SP_D / 4;  // float4s per chunk
      int k = 0;
      for (; k + 4 <= splits; k += 4) {  // four chunks' loads in flight
        float4 u[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          u[i][0] = __ldcg(src + (k + i) * CSTRIDE);
          u[i][1] = __ldcg(src + (k + i) * CSTRIDE + 1);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float f = fcs[(k + i) * HS + head];
          x[0] = fmaf(u[i][0].x, f, x[0]); x[1] = fmaf(u[i][0].y, f, x[1]);
          x[2] = fmaf(u[i][0].z, f, x[2]); x[3] = fmaf(u[i][0].w, f, x[3]);
          x[4] = fmaf(u[i][1].x, f, x[4]); x[5] = fmaf(u[i][1].y, f, x[5]);
          x[6] = fmaf(u[i][1].z, f, x[6]); x[7] = fmaf(u[i][1].w, f, x[7]);
        }
      }
      for (; k < splits; ++k) {
        const float4 u0 = __ldcg(src + k * CSTRIDE), u1 = __ldcg(src + k * CSTRIDE + 1);
        const float f = fcs[k * HS + head];
        x[0] = fmaf(u0.x, f, x[0]); x[1] = fmaf(u0.y, f, x[1]);
        x[2] = fmaf(u0.z, f, x[2]); x[3] = fmaf(u0.w, f, x[3]);
        x[4] = fmaf(u1.x, f, x[4]); x[5] = fmaf(u1.y, f, x[5]);
        x[6] = fmaf(u1.z, f, x[6]); x[7] = fmaf(u1.w, f, x[7]);
      }
      const size_t o0 = ob + static_cast<size_t>(head) * SP_D + d0;
      if (a.out_dtype == IC_F32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + o0);
        dst[0] = make_float4(x[0], x[1], x[2], x[3]);
        dst[1] = make_float4(x[4], x[5], x[6], x[7]);
      } else {
        *reinterpret_cast<uint4*>(static_cast<T*>(a.out) + o0) =
            make_uint4(sp_pack<T>(x[0], x[1]), sp_pack<T>(x[2], x[3]), sp_pack<T>(x[4], x[5]),
                       sp_pack<T>(x[6], x[7]));
      }
    }
  }
  // received mass of every slot (exact softmax, heads in order), folded into
  // the running sum over layers: the previous layer completed before the
  // grid-dependency wait returned
  float* macc = a.mass + grp * ntot;
  for (int tb = 0; tb < ntot; tb += 4 * SP_THREADS) {
    float xs[4][HS];
    float prev[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = tb + i * SP_THREADS + tid;
      const bool in = t < ntot;
      const float4* src = reinterpret_cast<const float4*>(ws_x + static_cast<size_t>(in ? t : 0) * HS);
#pragma unroll
      for (int q4 = 0; q4 < HS / 4; ++q4) {
        const float4 u = __ldcg(src + q4);
        xs[i][4 * q4] = u.x; xs[i][4 * q4 + 1] = u.y; xs[i][4 * q4 + 2] = u.z; xs[i][4 * q4 + 3] = u.w;
      }
      prev[i] = (a.layer > 0 && in) ? macc[t] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = tb + i * SP_THREADS + tid;
      if (t >= ntot) continue;
      float m = 0.f;
#pragma unroll
      for (int head = 0; head < HS; ++head) {
        const float xv = xs[i][head];
        if (head < G && xv != -INFINITY) m += sp_ex2(xv - gM[head]) * gI[head];
      }
      macc[t] = a.layer == 0 ? m : __fadd_rn(prev[i], m);
    }
  }
  if (tid == 0) *counter = 0;  // ready for the next launch
}

struct SplitGeom {
  int rb, chunk, splits, hs;
};

inline SplitGeom split_geometry(int ntot, int G, int split_rows) {
  SplitGeom g;
  g.hs = G <= 8 ? 8 : 16;
  if (split_rows == 64 || split_rows == 128) {
    g.chunk = split_rows;
  } else {
    g.chunk = (ntot + 63) / 64 <= SP_MAX_SPLITS ? 64 : 128;
  }
  g.rb = g.chunk / (16 * SP_W);
  g.splits = (ntot + g.chunk - 1) / g.chunk;
  return g;
}

inline size_t split_workspace_bytes(int num_sessions, int Hkv, const SplitGeom& g) {
  const size_t groups = static_cast<size_t>(num_sessions) * Hkv;
  return split_counter_bytes(groups) + groups * split_group_floats(g.splits, g.chunk, g.hs) * 4;
}

template <typename T, int NG, int RB>
int launch_split(const ic_decode_args& a, cudaStream_t stream, int splits) {
  constexpr int CHUNK = SP_W * 16 * RB;
  const SplitSmem L = split_smem(CHUNK, NG * 8);
  auto kern = decode_split_kernel<T, NG, RB>;
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(kern, L.total, &smem_limit)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, a.pool.num_kv_heads, a.sess.num_sessions);
  cfg.blockDim = dim3(SP_THREADS, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, a, splits);
  return launch_status("decode_layer (split)");
}

template <typename T>
int split_dispatch(const ic_decode_args& a, cudaStream_t stream, const SplitGeom& g) {
  if (g.hs == 8)
    return g.rb == 1 ? launch_split<T, 1, 1>(a, stream, g.splits) : launch_split<T, 1, 2>(a, stream, g.splits);
  return g.rb == 1 ? launch_split<T, 2, 1>(a, stream, g.splits) : launch_split<T, 2, 2>(a, stream, g.splits);
}

}  // namespace

int64_t decode_split_workspace_bytes(const ic_decode_args& a) {
  const int ntot = a.tiers.budget + 1;
  const int Hkv = a.pool.num_kv_heads;
  const int G = Hkv > 0 ? a.num_q_heads / Hkv : 0;
  // the larger of the two chunk shapes, so any split_rows setting fits
  size_t need = 0;
  for (int rows : {64, 128}) {
    const SplitGeom g = split_geometry(ntot, G, rows);
    if (g.splits > SP_MAX_SPLITS) continue;
    const size_t b = split_workspace_bytes(a.sess.num_sessions, Hkv, g);
    if (b > need) need = b;
  }
  return static_cast<int64_t>(need);
}

int launch_decode_split(const ic_decode_args& a, cudaStream_t stream) {
  const int G = a.num_q_heads / a.pool.num_kv_heads;
  if (G > 16) {
    set_last_error("decode (split): at most 16 query heads per KV head");
    return IC_ERR_UNSUPPORTED;
  }
  if (a.split_rows != 0 && a.split_rows != 64 && a.split_rows != 128) {
    set_last_error("decode (split): split_rows must be 0, 64 or 128");
    return IC_ERR_INVALID_ARG;
  }
  const int ntot = a.tiers.budget + 1;
  const SplitGeom g = split_geometry(ntot, G, a.split_rows);
  if (g.splits > SP_MAX_SPLITS) {
    set_last_error("decode (split): budget too large (at most 64 chunks of 128 slots)");
    return IC_ERR_UNSUPPORTED;
  }
  if (!a.workspace || (reinterpret_cast<uintptr_t>(a.workspace) & 255) != 0) {
    set_last_error("decode (split): workspace must be a 256-byte aligned device buffer");
    return IC_ERR_INVALID_ARG;
  }
  if (a.workspace_bytes < static_cast<int64_t>(split_workspace_bytes(a.sess.num_sessions, a.pool.num_kv_heads, g))) {
    set_last_error("decode (split): workspace smaller than ic_decode_workspace_bytes()");
    return IC_ERR_INVALID_ARG;
  }
  if (a.pool.dtype == IC_F16) return split_dispatch<__half>(a, stream, g);
  if (a.pool.dtype == IC_BF16) return split_dispatch<__nv_bfloat16>(a, stream, g);
  set_last_error("decode (split): dtype must be fp16 or bf16");
  return IC_ERR_INVALID_ARG;
}

}  // namespace ic

extern "C" int64_t ic_decode_workspace_bytes(const ic_decode_args* a) {
  if (!a || a->pool.num_kv_heads <= 0 || a->num_q_heads <= 0 || a->tiers.budget <= 0 || a->sess.num_sessions < 0) {
    ic::set_last_error("decode_workspace_bytes: bad sizes");
    return IC_ERR_INVALID_ARG;
  }
  return ic::decode_split_workspace_bytes(*a);
}
