// Kernel C: summary-pass scorer on the 5th-generation tensor cores.
//
// The reference scores a prompt's tokens by the attention mass each key
// receives, sum over heads and query rows of softmax(QK^T) (_attention_mass,
// two_pass.py:104-137), after materialising P [H, T, T].  Here two kernels
// stream the causal triangle in 128 x 128 tiles and never store P:
//
//  1. summary_fwd_kernel, one CTA per (sequence, query head, pair of 128-row
//     query tiles): S = Q K^T into TMEM (tcgen05.mma, operands staged by
//     TMA), the row softmax in registers (one warpgroup per query tile, one
//     thread per row, online max kept unless it grows by more than 2^8, so O
//     is rescaled only then), P written back to TMEM as 16-bit, O += P V
//     into TMEM (P read from TMEM); epilogue O / l and the row log-sum-exp.
//  2. summary_colsum_kernel, one CTA per (sequence, query head, 128-key
//     tile): S^T = K Q^T into TMEM for every query tile at or below the
//     diagonal, then p = exp2(s * scale * log2 e - lse2) with one thread per
//     key summing its column in fp32 registers — a fixed order, so the result
//     is deterministic.  Part of the exponentials run on the FP32 pipe
//     (exp2_poly.cuh), the rest on the multi-function unit.
//  3. summary_head_sum_kernel: colsum = sum over heads in head order; then
//     summary_normalise_kernel: the normalised importance with a fixed-shape
//     block reduction.
//
// Roles inside a CTA: warp 0 issues TMA loads, warp 1 owns TMEM and issues
// the MMAs (one thread; the forward kernel hands P V to a second issuing
// warp), the remaining warps move data between TMEM and registers.  Every mbarrier wait is bounded; on timeout the CTA sets
// IC_DEVFLAG_TIMEOUT, stops issuing work, waits (bounded) for its own
// in-flight MMAs, frees TMEM and exits.
#include <cuda.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "exp2_poly.cuh"
#include "tc05.cuh"

namespace ic {
namespace {

constexpr int SB = 128;           // tile rows / columns
constexpr int SD = 128;           // head dim
constexpr int SUB = SB * 64 * 2;  // one 64-column swizzled sub-tile: 16 KB
constexpr int TILE = 2 * SUB;     // a 128 x 128 16-bit tile: 32 KB
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr float RESCALE_LOG2 = 8.0f;  // keep a stale max while P <= 2^8

template <typename T> struct AbFormat;
template <> struct AbFormat<__half> { static constexpr int v = 0; };
template <> struct AbFormat<__nv_bfloat16> { static constexpr int v = 1; };

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// K-major descriptor for K step kk (16 elements) of a 128-row tile.
__device__ __forceinline__ uint64_t kdesc(uint32_t tile_saddr, int kk) {
  return tc::sw128_desc(tile_saddr + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
}
// MN-major descriptor for K step kk (16 rows) of a [128 rows(K) x 128 cols(N)]
// tile: the N halves are the two sub-tiles (LBO = SUB), 8-row atoms 1024 B.
__device__ __forceinline__ uint64_t mndesc(uint32_t tile_saddr, int kk) {
  return tc::sw128_desc(tile_saddr + kk * 2048, SUB, 1024);
}

// Warp-uniform bounded wait by every lane.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int32_t* status, volatile int* abort) {
  int ok = *abort ? 0 : (mbar_wait_bounded(bar, parity, status) ? 1 : 0);
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) *abort = 1;
  return ok != 0;
}
// Single-thread bounded wait.
__device__ __forceinline__ bool one_wait(uint64_t* bar, uint32_t parity, int32_t* status, volatile int* abort) {
  if (*abort) return false;
  if (mbar_wait_bounded(bar, parity, status)) return true;
  *abort = 1;
  return false;
}

struct SumParams {
  int T, n_t, Hq, Hkv, G;
  float sl2;  // scale * log2(e)
  void* out;
  float* lse;
  float* head_mass;
  int32_t* status;
};

// ------------------------------------------------------------------------------
// 1. forward: O and the row log-sum-exp
// ------------------------------------------------------------------------------
// One CTA per (sequence, query head, pair of 128-row query tiles qa = 2i,
// qb = 2i + 1).  Both tiles share every K / V tile they read; one softmax
// warpgroup per query tile.  The score tiles take turns in one TMEM buffer
// (S_a(0), S_b(0), S_a(1), ...): each softmax copies its S tile to registers
// at once, so the next Q K^T starts while it exponentiates.  P goes back to
// TMEM as 16-bit pairs and P V reads it there (tcgen05.mma with A in TMEM),
// so P never touches shared memory, whose bandwidth the tensor-core operand
// reads and the TMA writes already use.  Q K^T and P V are issued by two
// threads in different warps, so a blocked issue or wait on one side never
// holds back the other.
// TMEM columns: S 0, P_a 128, P_b 192, O_a 256, O_b 384.
// K and V tiles stream through one ring in consumption order K0 K1 V0 K2 V1
// ... V(n-1) (K one tile ahead); a K slot is released once both tiles'
// Q K^T are done, a V slot once both P V are done.
constexpr int FWD_THREADS = 352;  // producer, Q K^T issuer, two softmax warpgroups, P V issuer
constexpr int FWD_RS = 5;         // K / V ring slots
constexpr int F_Q = 0;            // Q_a, Q_b
constexpr int F_R = 2 * TILE;
constexpr int F_BAR = F_R + FWD_RS * TILE;
constexpr int F_NBAR = 20;
constexpr int F_BYTES = F_BAR + F_NBAR * 8 + 16 + 1024;  // + alignment slack
// Of every 8 column pairs, how many are exponentiated on the FP32 pipe.  0:
// measured on B200, 2 or 3 slowed this kernel (its softmax threads already
// sit at the 168-register cap of a 352-thread CTA).
constexpr int FWD_POLY_PAIRS = 0;

template <typename T, bool WITH_O>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    summary_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const SumParams p) {
  constexpr int LPS = WITH_O ? 2 : 1;  // ring loads per key step
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* r_full = bars + 1;    // [FWD_RS]
  uint64_t* r_empty = bars + 6;   // [FWD_RS]
  uint64_t* s_full = bars + 11;   // [2]: tile a, tile b
  uint64_t* s_free = bars + 13;   // the S buffer has been copied out
  uint64_t* p_full = bars + 14;   // [2]
  uint64_t* pv_done = bars + 16;  // [2]
  uint64_t* mma_done = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + F_BAR + F_NBAR * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + F_BAR + F_NBAR * 8 + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_pair = (p.n_t + 1) >> 1;
  const int n_bh = (int)gridDim.x / n_pair;
  const int bh = (int)blockIdx.x % n_bh;
  const int qa = 2 * (n_pair - 1 - (int)blockIdx.x / n_bh);  // longest rows first, over all heads
  const bool has_b = qa + 1 < p.n_t;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int kvz = b * p.Hkv + h / p.G;
  const int na = qa + 1;              // key tiles of tile a: 0 .. qa
  const int nb = has_b ? qa + 2 : 0;  // key tiles of tile b: 0 .. qa + 1
  const int n = has_b ? nb : na;
  constexpr uint32_t IDESC = tc::idesc_f16(AbFormat<T>::v, 128, 128, 0, 0);
  constexpr uint32_t IDESC_PV = tc::idesc_f16(AbFormat<T>::v, 128, 128, 0, 1);
  // ring position of key tile j and of value tile j
  auto u_k = [&](int j) { return WITH_O ? (j == 0 ? 0 : 2 * j - 1) : j; };
  auto u_v = [&](int j) { return j == n - 1 ? 2 * n - 1 : 2 * j + 2; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < FWD_RS; ++i) {
      mbar_init(r_full + i, 1);
      mbar_init(r_empty + i, 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(s_full + x, 1);
      mbar_init(p_full + x, 128);
      mbar_init(pv_done + x, 1);
    }
    mbar_init(s_free, 128);
    mbar_init(mma_done, WITH_O ? 2 : 1);  // one commit per issuing thread
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer: Q_a, Q_b, then K0 K1 V0 K2 V1 ... through the ring ---
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, has_b ? 2 * TILE : TILE);
      for (int x = 0; x < (has_b ? 2 : 1); ++x) {
        tc::tma_load_3d(smem + F_Q + x * TILE, &tq, 0, (qa + x) * SB, bh, q_full);
        tc::tma_load_3d(smem + F_Q + x * TILE + SUB, &tq, 64, (qa + x) * SB, bh, q_full);
      }
      const int n_loads = n * LPS;
      int issued = 0;
      for (int u = 0; u < n_loads; ++u) {
        const int st = u % FWD_RS;
        if (u >= FWD_RS && !one_wait(r_empty + st, ((u / FWD_RS) - 1) & 1, p.status, abort)) break;
        // inverse of u_k / u_v
        const bool is_v = WITH_O && u > 0 && (u == n_loads - 1 || (u & 1) == 0);
        const int j = !WITH_O ? u : is_v ? (u == n_loads - 1 ? n - 1 : u / 2 - 1) : (u + 1) / 2;
        const CUtensorMap* m = is_v ? &tv : &tk;
        mbar_arrive_expect_tx(r_full + st, TILE);
        tc::tma_load_3d(smem + F_R + st * TILE, m, 0, j * SB, kvz, r_full + st);
        tc::tma_load_3d(smem + F_R + st * TILE + SUB, m, 64, j * SB, kvz, r_full + st);
        issued = u + 1;
      }
      // drain: every issued load has landed before the CTA may exit
      mbar_wait_bounded(q_full, 0, p.status, 200000000ull);
      for (int u = issued - FWD_RS < 0 ? 0 : issued - FWD_RS; u < issued; ++u)
        mbar_wait_bounded(r_full + u % FWD_RS, (u / FWD_RS) & 1, p.status, 200000000ull);
    }
  } else if (warp == 1) {
    // ---- Q K^T issuer: S_a(j), S_b(j) in turn through the one S buffer --------
    if (lane == 0) {
      const uint32_t sq = sbase + F_Q;
      int n_s = 0;  // score tiles issued into the S buffer so far
      auto issue_s = [&](int x, int j) -> bool {
        if (n_s >= 1 && !one_wait(s_free, (n_s - 1) & 1, p.status, abort)) return false;
        tc::fence_after();
        const uint32_t sk = sbase + F_R + (u_k(j) % FWD_RS) * TILE;
#pragma unroll
        for (int kk = 0; kk < SD / 16; ++kk)
          tc::mma_ss(tmem, kdesc(sq + x * TILE, kk), kdesc(sk, kk), IDESC, kk > 0 ? 1u : 0u);
        tc::commit(s_full + x);
        ++n_s;
        return true;
      };
      bool ok = one_wait(q_full, 0, p.status, abort);
      for (int j = 0; ok && j < n; ++j) {
        const int u = u_k(j);
        if (!(ok = one_wait(r_full + u % FWD_RS, (u / FWD_RS) & 1, p.status, abort))) break;
        if (j < na && !(ok = issue_s(0, j))) break;
        if (j < nb && !(ok = issue_s(1, j))) break;
        tc::commit(r_empty + u % FWD_RS);
      }
      tc::commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status);
    }
  } else if (warp == FWD_THREADS / 32 - 1) {
    // ---- P V issuer: O_a += P_a V(j), O_b += P_b V(j), P read from TMEM -------
    if (lane == 0 && WITH_O) {
      bool ok = true;
      for (int j = 0; ok && j < n; ++j) {
        const int u = u_v(j);
        if (!(ok = one_wait(r_full + u % FWD_RS, (u / FWD_RS) & 1, p.status, abort))) break;
        const uint32_t sv = sbase + F_R + (u % FWD_RS) * TILE;
        for (int x = 0; x < 2; ++x) {
          if (j >= (x ? nb : na)) continue;
          if (!(ok = one_wait(p_full + x, j & 1, p.status, abort))) break;
          tc::fence_after();
#pragma unroll
          for (int kk = 0; kk < SB / 16; ++kk)
            tc::mma_ts(tmem + 256 + x * 128, tmem + 128 + x * 64 + kk * 8, mndesc(sv, kk), IDESC_PV,
                       (j > 0 || kk > 0) ? 1u : 0u);
          tc::commit(pv_done + x);
        }
        if (ok) tc::commit(r_empty + u % FWD_RS);
      }
      tc::commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status);
    }
  } else {
    // ---- softmax warpgroups: x = 0 (warps 2-5) tile a, x = 1 (warps 6-9) tile b;
    //      thread = query row --------------------------------------------------
    const int x = warp >= 6 ? 1 : 0;
    const int nx = x ? nb : na;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t ts = tmem + lane_off, tp = tmem + lane_off + 128 + x * 64;
    const uint32_t to = tmem + lane_off + 256 + x * 128;
    float m_used = -INFINITY, l = 0.f;
    float s[SB];
    bool ok = true;
    for (int j = 0; j < nx; ++j) {
      if (!(ok = warp_wait(s_full + x, j & 1, p.status, abort))) break;
      tc::fence_after();
#pragma unroll
      for (int c = 0; c < SB; c += 32) tc::tmem_ld32(ts + c, s + c);
      tc::tmem_wait_ld();
      tc::fence_before();
      tc::mbar_arrive(s_free);

      if (j == nx - 1) {  // diagonal tile: key c is visible to row r iff c <= r
#pragma unroll
        for (int c = 0; c < SB; ++c) s[c] = c <= r ? s[c] : -INFINITY;
      }
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = s[i];
#pragma unroll
      for (int c = 8; c < SB; ++c) m8[c & 7] = fmaxf(m8[c & 7], s[c]);
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * p.sl2;
      const float m_new = mx > m_used + RESCALE_LOG2 ? mx : m_used;
      const float alpha = m_new == m_used ? 1.f : tc::ex2(m_used - m_new);
      // row sum in four chains (column c into chain c mod 4), two per f32x2 register
      poly::f2 r2[2] = {poly::splat(0.f), poly::splat(0.f)};
      const poly::f2 sl2 = poly::splat(p.sl2), neg_m = poly::splat(-m_new);
#pragma unroll
      for (int c0 = 0; c0 < SB; c0 += 16) {
        float pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // columns c0 + 2i, c0 + 2i + 1
          const poly::f2 x = poly::fma2(poly::pack(s[c0 + 2 * i], s[c0 + 2 * i + 1]), sl2, neg_m);
          float e0, e1;
          if (i < FWD_POLY_PAIRS) {
            poly::unpack(poly::exp2x2(x), e0, e1);
          } else {
            poly::unpack(x, e0, e1);
            e0 = tc::ex2(e0);
            e1 = tc::ex2(e1);
          }
          r2[i & 1] = poly::add2(r2[i & 1], poly::pack(e0, e1));
          if (WITH_O) pk[i] = __uint_as_float(pack2(e0, e1, (T*)nullptr));
        }
        if (WITH_O) {
          if (c0 == 0 && j >= 1) {
            if (!(ok = warp_wait(pv_done + x, (j - 1) & 1, p.status, abort))) break;
            tc::fence_after();
          }
          tc::tmem_st8(tp + c0 / 2, pk);
        }
      }
      if (!ok) break;
      float r4[4];
      poly::unpack(r2[0], r4[0], r4[1]);
      poly::unpack(r2[1], r4[2], r4[3]);
      l = l * alpha + ((r4[0] + r4[1]) + (r4[2] + r4[3]));
      if (WITH_O) {
        if (j >= 1 && __any_sync(0xffffffffu, m_new != m_used)) {
          const float a = m_new != m_used ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < SD; c += 16) {
            float o[16];
            tc::tmem_ld16(to + c, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= a;
            tc::tmem_st16(to + c, o);
          }
        }
        tc::tmem_wait_st();
        tc::fence_before();
        tc::mbar_arrive(p_full + x);
      }
      m_used = m_new;
    }
    const int row = (qa + x) * SB + r;
    if (nx > 0 && ok && WITH_O) ok = warp_wait(pv_done + x, (nx - 1) & 1, p.status, abort);
    if (nx > 0 && ok) {
      tc::fence_after();
      if (row < p.T) p.lse[(size_t)bh * p.T + row] = (m_used + log2f(l)) * LN2;
      if (WITH_O) {
        const float inv = 1.f / l;
        T* orow = reinterpret_cast<T*>(p.out) + ((size_t)bh * p.T + row) * SD;
#pragma unroll 1
        for (int c = 0; c < SD; c += 32) {
          float o[32];
          tc::tmem_ld32(to + c, o);
          tc::tmem_wait_ld();
          if (row < p.T) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              w.x = pack2(o[8 * q + 0] * inv, o[8 * q + 1] * inv, (T*)nullptr);
              w.y = pack2(o[8 * q + 2] * inv, o[8 * q + 3] * inv, (T*)nullptr);
              w.z = pack2(o[8 * q + 4] * inv, o[8 * q + 5] * inv, (T*)nullptr);
              w.w = pack2(o[8 * q + 6] * inv, o[8 * q + 7] * inv, (T*)nullptr);
              *reinterpret_cast<uint4*>(orow + c + 8 * q) = w;
            }
          }
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}
// ------------------------------------------------------------------------------
// 2. column sums: received mass per key, per query head
// ------------------------------------------------------------------------------
constexpr int COL_THREADS = 320;  // producer, MMA, two groups of 4 warps
constexpr int COL_NS = 4;
constexpr int C_K = 0;
constexpr int C_Q = TILE;
constexpr int C_LSE = C_Q + COL_NS * TILE;
constexpr int C_RED = C_LSE + COL_NS * SB * 4;
constexpr int C_BAR = C_RED + SB * 4;
constexpr int C_NBAR = 20;
constexpr int C_BYTES = C_BAR + C_NBAR * 8 + 16 + 1024;
// Of every 8 query pairs, how many are exponentiated on the FP32 pipe: 2
// (measured on B200 against 0 and 3: 3.6% and 4.2% less kernel time).
constexpr int COL_POLY_PAIRS = 2;

template <typename T>
__global__ void __launch_bounds__(COL_THREADS, 1)
    summary_colsum_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const SumParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C_BAR);
  uint64_t* k_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [4]
  uint64_t* q_empty = bars + 5;   // [4]
  uint64_t* s_full = bars + 9;    // [4]
  uint64_t* s_free = bars + 13;   // [4]
  uint64_t* mma_done = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C_BAR + C_NBAR * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + C_BAR + C_NBAR * 8 + 4);
  float* lse_s = reinterpret_cast<float*>(smem + C_LSE);  // [4][128], -lse in log2 units
  float* red = reinterpret_cast<float*>(smem + C_RED);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = p.n_t;
  // (sequence, head)-major, so the CTAs running at once share one head's Q
  // tiles in L2; longest columns first within a head
  const int bh = blockIdx.x / n_t;
  const int kt = (int)(blockIdx.x % n_t);
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int kvz = b * p.Hkv + h / p.G;
  const int n = n_t - kt;  // query tiles at or below the diagonal: kt .. n_t-1
  constexpr uint32_t IDESC = tc::idesc_f16(AbFormat<T>::v, 128, 128, 0, 0);

  if (threadIdx.x == 0) {
    mbar_init(k_full, 1);
    for (int i = 0; i < COL_NS; ++i) {
      mbar_init(q_full + i, 32);
      mbar_init(q_empty + i, 1 + 128);
      mbar_init(s_full + i, 1);
      mbar_init(s_free + i, 128);
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;  // S^T buffers at +0, +128, +256, +384

  if (warp == 0) {
    // ---- producer: K tile once, then Q tiles + their lse rows ---------------
    if (lane == 0) {
      mbar_arrive_expect_tx(k_full, TILE);
      tc::tma_load_3d(smem + C_K, &tk, 0, kt * SB, kvz, k_full);
      tc::tma_load_3d(smem + C_K + SUB, &tk, 64, kt * SB, kvz, k_full);
    }
    int issued = 0;
    for (int t = 0; t < n; ++t) {
      const int st = t % COL_NS, i = kt + t;
      if (t >= COL_NS && !warp_wait(q_empty + st, ((t / COL_NS) - 1) & 1, p.status, abort)) break;
      const float* lrow = p.lse + (size_t)bh * p.T + (size_t)i * SB;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = lane * 4 + u;
        lse_s[st * SB + c] = i * SB + c < p.T ? -lrow[c] * LOG2E : -INFINITY;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full + st, TILE);
        tc::tma_load_3d(smem + C_Q + st * TILE, &tq, 0, i * SB, bh, q_full + st);
        tc::tma_load_3d(smem + C_Q + st * TILE + SUB, &tq, 64, i * SB, bh, q_full + st);
      } else {
        tc::mbar_arrive(q_full + st);
      }
      issued = t + 1;
    }
    if (lane == 0) {
      mbar_wait_bounded(k_full, 0, p.status, 200000000ull);
      for (int t = issued - COL_NS < 0 ? 0 : issued - COL_NS; t < issued; ++t)
        mbar_wait_bounded(q_full + t % COL_NS, (t / COL_NS) & 1, p.status, 200000000ull);
    }
  } else if (warp == 1) {
    // ---- MMA issuer: S^T = K . Q^T per query tile ---------------------------------
    if (lane == 0) {
      const uint32_t sk = sbase + C_K;
      bool ok = one_wait(k_full, 0, p.status, abort);
      for (int t = 0; ok && t < n; ++t) {
        const int st = t % COL_NS;
        if (!one_wait(q_full + st, (t / COL_NS) & 1, p.status, abort)) break;
        if (t >= COL_NS && !one_wait(s_free + st, ((t / COL_NS) - 1) & 1, p.status, abort)) break;
        tc::fence_after();
        const uint32_t sq = sbase + C_Q + st * TILE;
#pragma unroll
        for (int kk = 0; kk < SD / 16; ++kk)
          tc::mma_ss(tmem + st * 128, kdesc(sk, kk), kdesc(sq, kk), IDESC, kk > 0 ? 1u : 0u);
        tc::commit(s_full + st);
        tc::commit(q_empty + st);
      }
      tc::commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status);
    }
  } else {
    // ---- column sums: thread = key row of the tile; group g takes tiles g, g+2, ...
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float acc = 0.f;
    float s[SB];
    for (int t = g; t < n; t += 2) {
      const int st = t % COL_NS;
      if (!warp_wait(s_full + st, (t / COL_NS) & 1, p.status, abort)) break;
      if (!warp_wait(q_full + st, (t / COL_NS) & 1, p.status, abort)) break;
      tc::fence_after();
#pragma unroll
      for (int c = 0; c < SB; c += 32) tc::tmem_ld32(tmem + lane_off + st * 128 + c, s + c);
      tc::tmem_wait_ld();
      tc::fence_before();
      tc::mbar_arrive(s_free + st);
      const float* ls = lse_s + st * SB;  // -lse2 per query
      float a4[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains, summed in a fixed order
      if (t == 0) {  // diagonal tile: query c sees key r iff c >= r
#pragma unroll
        for (int c = 0; c < SB; ++c) {
          const float e = tc::ex2(fmaf(s[c], p.sl2, ls[c]));
          a4[c & 3] += c >= r ? e : 0.f;
        }
      } else {
        // pairs of queries; COL_POLY_PAIRS of every 8 pairs take 2^x on the
        // FP32 pipe, the rest on the multi-function unit
        const poly::f2 sl2 = poly::splat(p.sl2);
        poly::f2 acc2[2] = {poly::splat(0.f), poly::splat(0.f)};
#pragma unroll
        for (int c = 0; c < SB; c += 2) {
          const poly::f2 x =
              poly::fma2(poly::pack(s[c], s[c + 1]), sl2, *reinterpret_cast<const poly::f2*>(ls + c));
          poly::f2 e;
          if (((c >> 1) & 7) < COL_POLY_PAIRS) {
            e = poly::exp2x2(x);
          } else {
            float x0, x1;
            poly::unpack(x, x0, x1);
            e = poly::pack(tc::ex2(x0), tc::ex2(x1));
          }
          acc2[(c >> 1) & 1] = poly::add2(acc2[(c >> 1) & 1], e);
        }
        poly::unpack(acc2[0], a4[0], a4[1]);
        poly::unpack(acc2[1], a4[2], a4[3]);
      }
      acc += (a4[0] + a4[1]) + (a4[2] + a4[3]);
      tc::mbar_arrive(q_empty + st);
    }
    // group 1 hands its partial to group 0, which adds it in a fixed order
    if (g == 1) red[r] = acc;
    tc::named_sync(1, 256);
    if (g == 0) {
      const int key = kt * SB + r;
      if (key < p.T && !*abort) p.head_mass[(size_t)bh * p.T + key] = acc + red[r];
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------
// 3. colsum over heads and the normalised importance (one CTA per sequence)
// ------------------------------------------------------------------------------
constexpr int RED_THREADS = 1024;
constexpr int RED_COLS = 1024;  // columns per CTA of the head sum

// colsum[b, j] (+)= sum over heads in head order of head_mass[b, h, j]; one
// CTA per (sequence, 1024 columns).
__global__ void __launch_bounds__(RED_COLS)
    summary_head_sum_kernel(const float* __restrict__ head_mass, float* colsum, int Hq, int T, int accumulate) {
  const int b = blockIdx.y, j = blockIdx.x * RED_COLS + threadIdx.x;
  if (j >= T) return;
  const float* hm = head_mass + (size_t)b * Hq * T + j;
  float* cs = colsum + (size_t)b * T + j;
  float v = accumulate ? *cs : 0.f;
  for (int hh = 0; hh < Hq; ++hh) v += hm[(size_t)hh * T];
  *cs = v;
}

// importance[b, :] = colsum[b, :] / sum(colsum[b, :]), the sum taken by a
// fixed-shape block reduction (one CTA per sequence).
__global__ void __launch_bounds__(RED_THREADS)
    summary_normalise_kernel(const float* __restrict__ colsum, float* importance, int T) {
  __shared__ float part[RED_THREADS / 32];
  __shared__ float total_s;
  const int b = blockIdx.x;
  const float* cs = colsum + (size_t)b * T;
  float tot = 0.f;
  for (int j = threadIdx.x; j < T; j += RED_THREADS) tot += cs[j];
  tot = warp_sum(tot);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = tot;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = part[threadIdx.x];
    v = warp_sum(v);
    if (threadIdx.x == 0) total_s = v;
  }
  __syncthreads();
  const float total = total_s;
  float* im = importance + (size_t)b * T;
  for (int j = threadIdx.x; j < T; j += RED_THREADS) im[j] = total > 1e-9f ? cs[j] / total : cs[j];
}

// ------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// [rows_outer][T][128] 16-bit tensor, boxes of 64 columns x 128 rows, 128-B swizzle.
int make_map(CUtensorMap* m, const void* base, int dt, int T, int outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_last_error("summary_score: cuTensorMapEncodeTiled unavailable");
    return IC_ERR_CUDA;
  }
  const cuuint64_t dims[3] = {(cuuint64_t)SD, (cuuint64_t)T, (cuuint64_t)outer};
  const cuuint64_t strides[2] = {(cuuint64_t)SD * 2, (cuuint64_t)T * SD * 2};
  const cuuint32_t box[3] = {64, SB, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, dt == IC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("summary_score: tensor map encoding failed");
    return IC_ERR_INVALID_ARG;
  }
  return IC_OK;
}

template <typename T>
int launch_summary(const ic_summary_args* a, cudaStream_t st) {
  const int T_ = a->seq_len, n_t = (T_ + SB - 1) / SB;
  const int BHq = a->batch * a->num_q_heads, BHkv = a->batch * a->num_kv_heads;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, a->q, a->dtype, T_, BHq)) != IC_OK) return rc;
  if ((rc = make_map(&mk, a->k, a->dtype, T_, BHkv)) != IC_OK) return rc;
  if (a->out && (rc = make_map(&mv, a->v, a->dtype, T_, BHkv)) != IC_OK) return rc;
  if (!a->out) mv = mk;
  SumParams p;
  p.T = T_;
  p.n_t = n_t;
  p.Hq = a->num_q_heads;
  p.Hkv = a->num_kv_heads;
  p.G = a->num_q_heads / a->num_kv_heads;
  p.sl2 = a->scale * LOG2E;
  p.out = a->out;
  p.lse = a->lse;
  p.head_mass = a->head_mass;
  p.status = a->dev_status;

  static PerDeviceLimit lim_fwd_o, lim_fwd, lim_col;
  const unsigned grid = (unsigned)(BHq * n_t);
  const unsigned grid_fwd = (unsigned)(BHq * ((n_t + 1) / 2));
  if (a->out) {
    if ((rc = ensure_dynamic_smem(summary_fwd_kernel<T, true>, F_BYTES, &lim_fwd_o)) != IC_OK) return rc;
    summary_fwd_kernel<T, true><<<grid_fwd, FWD_THREADS, F_BYTES, st>>>(mq, mk, mv, p);
  } else {
    if ((rc = ensure_dynamic_smem(summary_fwd_kernel<T, false>, F_BYTES, &lim_fwd)) != IC_OK) return rc;
    summary_fwd_kernel<T, false><<<grid_fwd, FWD_THREADS, F_BYTES, st>>>(mq, mk, mv, p);
  }
  if ((rc = launch_status("summary_fwd_kernel")) != IC_OK) return rc;
  if (!a->head_mass) return IC_OK;
  if ((rc = ensure_dynamic_smem(summary_colsum_kernel<T>, C_BYTES, &lim_col)) != IC_OK) return rc;
  summary_colsum_kernel<T><<<grid, COL_THREADS, C_BYTES, st>>>(mq, mk, p);
  if ((rc = launch_status("summary_colsum_kernel")) != IC_OK) return rc;
  summary_head_sum_kernel<<<dim3((unsigned)((T_ + RED_COLS - 1) / RED_COLS), (unsigned)a->batch), RED_COLS, 0, st>>>(
      a->head_mass, a->colsum, a->num_q_heads, T_, a->accumulate);
  if ((rc = launch_status("summary_head_sum_kernel")) != IC_OK) return rc;
  if (!a->importance) return IC_OK;
  summary_normalise_kernel<<<a->batch, RED_THREADS, 0, st>>>(a->colsum, a->importance, T_);
  return launch_status("summary_normalise_kernel");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace ic

extern "C" int ic_summary_score(const ic_summary_args* a, void* stream) {
  if (!a || !a->q || !a->k || !a->lse || !a->dev_status || (a->head_mass && !a->colsum) ||
      (!a->head_mass && !a->out)) {
    ic::set_last_error("summary_score: null argument");
    return IC_ERR_INVALID_ARG;
  }
  if (a->out && !a->v) {
    ic::set_last_error("summary_score: out requires v");
    return IC_ERR_INVALID_ARG;
  }
  if (a->batch < 1 || a->num_q_heads < 1 || a->num_kv_heads < 1 || a->seq_len < 1 ||
      a->num_q_heads % a->num_kv_heads != 0 || a->batch > 65535 || a->seq_len > (1 << 24)) {
    ic::set_last_error("summary_score: bad shape");
    return IC_ERR_INVALID_ARG;
  }
  if (a->head_dim != 128 || (a->dtype != IC_F16 && a->dtype != IC_BF16)) {
    ic::set_last_error("summary_score: needs head_dim 128 and fp16 / bf16");
    return IC_ERR_UNSUPPORTED;
  }
  if (!ic::aligned16(a->q) || !ic::aligned16(a->k) || (a->v && !ic::aligned16(a->v)) ||
      (a->out && !ic::aligned16(a->out))) {
    ic::set_last_error("summary_score: q / k / v / out must be 16-byte aligned");
    return IC_ERR_INVALID_ARG;
  }
  const long long ntiles = (long long)a->batch * a->num_q_heads * ((a->seq_len + 127) / 128);
  if (ntiles > 0x7fffffffLL) {
    ic::set_last_error("summary_score: too many tiles");
    return IC_ERR_INVALID_ARG;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return a->dtype == IC_BF16 ? ic::launch_summary<__nv_bfloat16>(a, st) : ic::launch_summary<__half>(a, st);
}

// ------------------------------------------------------------------------------
// 4. ic_summary_score_static: the scorer with its per-head mass in a library-owned
//    static device array, for callers that cannot allocate device memory
// ------------------------------------------------------------------------------
// The array's address is looked up once per device and kept: after a
// cudaDeviceReset (or any teardown of the primary context) the module is
// loaded again and the cached address is stale, so calls after a device reset
// are not supported.
//
// Some callers cannot hand this library a scratch buffer: code that runs
// while another allocator owns all of the GPU's free memory (a serving
// process that reserved it up front), or a binding from a language with no
// CUDA allocator at hand.  They still pass q / k / v and every output; the
// per-head received mass [B, Hq, T], which ic_summary_score takes from the
// caller, lives here instead.  The array is IC_SUMMARY_STATIC_MASS_MAX floats
// (16 MiB) and is held by every GPU that loads the library until the process
// exits.
namespace {

static __device__ __align__(256) float ic_summary_mass_scratch[IC_SUMMARY_STATIC_MASS_MAX];

constexpr int kScratchMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_addr[kScratchMaxDevices];  // device address of the array, per device

// The array's device address on the current device.  Host code cannot use
// the array's name as an address (it names a host-side stand-in), so the
// first call on each device asks the runtime for it, with that device current.
int scratch_address(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    ic::set_last_error("summary_score_static: cudaGetDevice failed");
    return IC_ERR_CUDA;
  }
  if (dev < 0 || dev >= kScratchMaxDevices) {
    ic::set_last_error("summary_score_static: device index beyond 63");
    return IC_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, ic_summary_mass_scratch);
    if (e != cudaSuccess || !p) {
      ic::set_last_error("summary_score_static: cudaGetSymbolAddress of the static scratch failed");
      return IC_ERR_CUDA;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return IC_OK;
}

}  // namespace

extern "C" int ic_summary_score_static(const ic_summary_args* a, void* stream) {
  if (!a || !a->q || !a->k || !a->lse || !a->colsum || !a->dev_status) {
    ic::set_last_error("summary_score_static: null argument (q, k, lse, colsum and dev_status are required)");
    return IC_ERR_INVALID_ARG;
  }
  if (a->head_mass) {
    ic::set_last_error("summary_score_static: head_mass must be NULL (the per-head mass lives in the static scratch)");
    return IC_ERR_INVALID_ARG;
  }
  if (a->batch < 1 || a->num_q_heads < 1 || a->seq_len < 1) {
    ic::set_last_error("summary_score_static: bad shape");
    return IC_ERR_INVALID_ARG;
  }
  const long long need = (long long)a->batch * a->num_q_heads * a->seq_len;
  if (need > (long long)IC_SUMMARY_STATIC_MASS_MAX) {
    ic::set_last_error("summary_score_static: batch * num_q_heads * seq_len exceeds the static scratch "
                       "(IC_SUMMARY_STATIC_MASS_MAX floats); use ic_summary_score with a caller buffer");
    return IC_ERR_INVALID_ARG;
  }
  float* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != IC_OK) return rc;
  // every element of the mass that the column sum reads is written earlier in
  // the same call, so the array needs no clearing between calls -- except after
  // a bounded wait gave up (dev_status reports IC_DEVFLAG_TIMEOUT): the forward
  // kernel then skips its stores and the outputs are undefined
  ic_summary_args b = *a;
  b.head_mass = scratch;
  return ic_summary_score(&b, stream);
}
