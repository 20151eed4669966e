// Kernel C: summary-pass scorer on the 5th-generation tensor cores.
//
// The reference scores a prompt's tokens by the attention mass each key
// receives, sum over heads and query rows of softmax(QK^T) (_attention_mass,
// two_pass.py:104-137), after materialising P [H, T, T].  Here two kernels
// stream the causal triangle in 128 x 128 tiles and never store P:
//
//  1. summary_fwd_kernel, one CTA per (sequence, query head, 128-row query
//     tile): S = Q K^T into TMEM (tcgen05.mma, operands staged by TMA), the
//     row softmax in registers (one thread per row, online max kept unless it
//     grows by more than 2^8, so O is rescaled only then), P written as
//     16-bit to shared memory, O += P V into TMEM; epilogue O / l and the row
//     log-sum-exp.
//  2. summary_colsum_kernel, one CTA per (sequence, query head, 128-key
//     tile): S^T = K Q^T into TMEM for every query tile at or below the
//     diagonal, then p = exp2(s * scale * log2 e - lse2) with one thread per
//     key summing its column in fp32 registers — a fixed order, so the result
//     is deterministic.
//  3. summary_reduce_kernel: colsum = sum over heads in head order, and the
//     normalised importance with a fixed-shape block reduction.
//
// Roles inside a CTA: warp 0 issues TMA loads, warp 1 owns TMEM and issues
// the MMAs (one thread), the remaining warps move data between TMEM and
// registers.  Every mbarrier wait is bounded; on timeout the CTA sets
// IC_DEVFLAG_TIMEOUT, stops issuing work, waits (bounded) for its own
// in-flight MMAs, frees TMEM and exits.
#include <cuda.h>
#include <math.h>

#include "common.cuh"
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

// Byte offset of 16-byte chunk `q` (columns 8q .. 8q+7) of row `r` in a
// 128-column K-major tile stored as two 128-byte-swizzled sub-tiles.
__device__ __forceinline__ uint32_t sw_chunk(int r, int q) {
  return (uint32_t)((q >> 3) * SUB + r * 128 + (((q & 7) ^ (r & 7)) << 4));
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
constexpr int FWD_THREADS = 192;
constexpr int FWD_KS = 3;  // K ring: a K tile is free once its Q K^T is done
constexpr int FWD_VS = 2;  // V ring: a V tile is free once its P V is done
constexpr int F_Q = 0;
constexpr int F_K = TILE;
constexpr int F_V = F_K + FWD_KS * TILE;
constexpr int F_P = F_V + FWD_VS * TILE;
constexpr int F_BAR = F_P + TILE;
constexpr int F_NBAR = 20;
constexpr int F_BYTES = F_BAR + F_NBAR * 8 + 16 + 1024;  // + alignment slack

template <typename T, bool WITH_O>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    summary_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const SumParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [3]
  uint64_t* k_empty = bars + 4;   // [3]
  uint64_t* v_full = bars + 7;    // [2]
  uint64_t* v_empty = bars + 9;   // [2]
  uint64_t* s_full = bars + 11;   // [2]
  uint64_t* s_free = bars + 13;   // [2]
  uint64_t* p_full = bars + 15;
  uint64_t* pv_done = bars + 16;
  uint64_t* mma_done = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + F_BAR + F_NBAR * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + F_BAR + F_NBAR * 8 + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = p.n_t;
  const int bh = blockIdx.x / n_t;
  const int qt = n_t - 1 - (int)(blockIdx.x % n_t);  // longest rows first
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int kvz = b * p.Hkv + h / p.G;
  const int n = qt + 1;  // key tiles at or below the diagonal
  constexpr uint32_t IDESC = tc::idesc_f16(AbFormat<T>::v, 128, 128, 0, 0);
  constexpr uint32_t IDESC_PV = tc::idesc_f16(AbFormat<T>::v, 128, 128, 0, 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < FWD_KS; ++i) {
      mbar_init(k_full + i, 1);
      mbar_init(k_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(v_full + i, 1);
      mbar_init(v_empty + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(s_free + i, 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(mma_done, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 512);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;  // S0: +0, S1: +128, O: +256

  if (warp == 0) {
    // ---- TMA producers: lane 0 streams Q and the K tiles, lane 1 the V tiles ----
    if (lane == 0) {
      int issued = 0;
      mbar_arrive_expect_tx(q_full, TILE);
      tc::tma_load_3d(smem + F_Q, &tq, 0, qt * SB, bh, q_full);
      tc::tma_load_3d(smem + F_Q + SUB, &tq, 64, qt * SB, bh, q_full);
      for (int j = 0; j < n; ++j) {
        const int st = j % FWD_KS;
        if (j >= FWD_KS && !one_wait(k_empty + st, ((j / FWD_KS) - 1) & 1, p.status, abort)) break;
        mbar_arrive_expect_tx(k_full + st, TILE);
        tc::tma_load_3d(smem + F_K + st * TILE, &tk, 0, j * SB, kvz, k_full + st);
        tc::tma_load_3d(smem + F_K + st * TILE + SUB, &tk, 64, j * SB, kvz, k_full + st);
        issued = j + 1;
      }
      // drain: every issued load has landed before the CTA may exit
      mbar_wait_bounded(q_full, 0, p.status, 200000000ull);
      for (int j = issued - FWD_KS < 0 ? 0 : issued - FWD_KS; j < issued; ++j)
        mbar_wait_bounded(k_full + j % FWD_KS, (j / FWD_KS) & 1, p.status, 200000000ull);
    } else if (lane == 1 && WITH_O) {
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % FWD_VS;
        if (j >= FWD_VS && !one_wait(v_empty + st, ((j / FWD_VS) - 1) & 1, p.status, abort)) break;
        mbar_arrive_expect_tx(v_full + st, TILE);
        tc::tma_load_3d(smem + F_V + st * TILE, &tv, 0, j * SB, kvz, v_full + st);
        tc::tma_load_3d(smem + F_V + st * TILE + SUB, &tv, 64, j * SB, kvz, v_full + st);
        issued = j + 1;
      }
      for (int j = issued - FWD_VS < 0 ? 0 : issued - FWD_VS; j < issued; ++j)
        mbar_wait_bounded(v_full + j % FWD_VS, (j / FWD_VS) & 1, p.status, 200000000ull);
    }
  } else if (warp == 1) {
    // ---- MMA issuer -----------------------------------------------------------
    if (lane == 0) {
      const uint32_t sq = sbase + F_Q, sp = sbase + F_P;
      auto issue_pv = [&](int t) -> bool {
        if (!one_wait(p_full, t & 1, p.status, abort)) return false;
        if (!one_wait(v_full + t % FWD_VS, (t / FWD_VS) & 1, p.status, abort)) return false;
        tc::fence_after();
        const uint32_t sv = sbase + F_V + (t % FWD_VS) * TILE;
#pragma unroll
        for (int kk = 0; kk < SB / 16; ++kk)
          tc::mma_ss(tmem + 256, kdesc(sp, kk), mndesc(sv, kk), IDESC_PV, (t > 0 || kk > 0) ? 1u : 0u);
        tc::commit(pv_done);
        tc::commit(v_empty + t % FWD_VS);
        return true;
      };
      bool ok = one_wait(q_full, 0, p.status, abort);
      for (int j = 0; ok && j < n; ++j) {
        const int st = j % FWD_KS, sb = j & 1;
        if (!one_wait(k_full + st, (j / FWD_KS) & 1, p.status, abort)) break;
        if (j >= 2 && !one_wait(s_free + sb, ((j - 2) >> 1) & 1, p.status, abort)) break;
        tc::fence_after();
        const uint32_t sk = sbase + F_K + st * TILE;
#pragma unroll
        for (int kk = 0; kk < SD / 16; ++kk)
          tc::mma_ss(tmem + sb * 128, kdesc(sq, kk), kdesc(sk, kk), IDESC, kk > 0 ? 1u : 0u);
        tc::commit(s_full + sb);
        tc::commit(k_empty + st);
        if (WITH_O && j >= 1) ok = issue_pv(j - 1);
      }
      if (WITH_O && ok && !*abort) issue_pv(n - 1);
      tc::commit(mma_done);
      mbar_wait_bounded(mma_done, 0, p.status);
    }
  } else {
    // ---- softmax warps: thread = query row ------------------------------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    unsigned char* ps = smem + F_P;
    float m_used = -INFINITY, l = 0.f;
    float s[SB];
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      if (!(ok = warp_wait(s_full + sb, (j >> 1) & 1, p.status, abort))) break;
      tc::fence_after();
#pragma unroll
      for (int c = 0; c < SB; c += 32) tc::tmem_ld32(tmem + lane_off + sb * 128 + c, s + c);
      tc::tmem_wait_ld();
      tc::fence_before();
      tc::mbar_arrive(s_free + sb);

      // raw row maximum with eight independent chains (the scale is positive,
      // so scaling the maximum equals the maximum of the scaled scores)
      if (j == n - 1) {  // diagonal tile: key c is visible to row r iff c <= r
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
      float r4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < SB; ++c) {
        s[c] = tc::ex2(fmaf(s[c], p.sl2, -m_new));
        r4[c & 3] += s[c];
      }
      l = l * alpha + ((r4[0] + r4[1]) + (r4[2] + r4[3]));
      if (WITH_O) {
        // P buffer and O are free once the previous P . V has completed
        if (j >= 1) {
          if (!(ok = warp_wait(pv_done, (j - 1) & 1, p.status, abort))) break;
          tc::fence_after();
          if (__any_sync(0xffffffffu, m_new != m_used)) {
            const float a = m_new != m_used ? alpha : 1.f;
#pragma unroll 1
            for (int c = 0; c < SD; c += 32) {
              float o[32];
              tc::tmem_ld32(tmem + lane_off + 256 + c, o);
              tc::tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= a;
              tc::tmem_st32(tmem + lane_off + 256 + c, o);
            }
            tc::tmem_wait_st();
          }
        }
#pragma unroll
        for (int q = 0; q < SB / 8; ++q) {
          uint4 w;
          w.x = pack2(s[8 * q + 0], s[8 * q + 1], (T*)nullptr);
          w.y = pack2(s[8 * q + 2], s[8 * q + 3], (T*)nullptr);
          w.z = pack2(s[8 * q + 4], s[8 * q + 5], (T*)nullptr);
          w.w = pack2(s[8 * q + 6], s[8 * q + 7], (T*)nullptr);
          *reinterpret_cast<uint4*>(ps + sw_chunk(r, q)) = w;
        }
        fence_proxy_async_smem();
        tc::fence_before();
        tc::mbar_arrive(p_full);
      }
      m_used = m_new;
    }
    const int row = qt * SB + r;
    if (ok && WITH_O) ok = warp_wait(pv_done, (n - 1) & 1, p.status, abort);
    if (ok) {
      tc::fence_after();
      if (row < p.T) p.lse[(size_t)bh * p.T + row] = (m_used + log2f(l)) * LN2;
      if (WITH_O) {
        const float inv = 1.f / l;
        T* orow = reinterpret_cast<T*>(p.out) + ((size_t)bh * p.T + row) * SD;
#pragma unroll 1
        for (int c = 0; c < SD; c += 32) {
          float o[32];
          tc::tmem_ld32(tmem + lane_off + 256 + c, o);
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
  float* lse_s = reinterpret_cast<float*>(smem + C_LSE);  // [4][128], log2 units
  float* red = reinterpret_cast<float*>(smem + C_RED);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = p.n_t;
  const int bh = blockIdx.x / n_t;
  const int kt = (int)(blockIdx.x % n_t);  // longest columns first
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
        lse_s[st * SB + c] = i * SB + c < p.T ? lrow[c] * LOG2E : INFINITY;
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
      const float* ls = lse_s + st * SB;
      float a4[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains, summed in a fixed order
      if (t == 0) {  // diagonal tile: query c sees key r iff c >= r
#pragma unroll
        for (int c = 0; c < SB; ++c) {
          const float e = tc::ex2(fmaf(s[c], p.sl2, -ls[c]));
          a4[c & 3] += c >= r ? e : 0.f;
        }
      } else {
#pragma unroll
        for (int c = 0; c < SB; ++c) a4[c & 3] += tc::ex2(fmaf(s[c], p.sl2, -ls[c]));
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

__global__ void __launch_bounds__(RED_THREADS)
    summary_reduce_kernel(const float* __restrict__ head_mass, float* colsum, float* importance, int Hq, int T,
                          int accumulate) {
  __shared__ float part[RED_THREADS / 32];
  __shared__ float total_s;
  const int b = blockIdx.x;
  const float* hm = head_mass + (size_t)b * Hq * T;
  float* cs = colsum + (size_t)b * T;
  float tot = 0.f;
  for (int j = threadIdx.x; j < T; j += RED_THREADS) {
    float v = accumulate ? cs[j] : 0.f;
    for (int hh = 0; hh < Hq; ++hh) v += hm[(size_t)hh * T + j];
    cs[j] = v;
    tot += v;
  }
  if (!importance) return;
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

  static int lim_fwd_o = 0, lim_fwd = 0, lim_col = 0;
  const unsigned grid = (unsigned)(BHq * n_t);
  if (a->out) {
    if ((rc = ensure_dynamic_smem(summary_fwd_kernel<T, true>, F_BYTES, &lim_fwd_o)) != IC_OK) return rc;
    summary_fwd_kernel<T, true><<<grid, FWD_THREADS, F_BYTES, st>>>(mq, mk, mv, p);
  } else {
    if ((rc = ensure_dynamic_smem(summary_fwd_kernel<T, false>, F_BYTES, &lim_fwd)) != IC_OK) return rc;
    summary_fwd_kernel<T, false><<<grid, FWD_THREADS, F_BYTES, st>>>(mq, mk, mv, p);
  }
  if ((rc = launch_status("summary_fwd_kernel")) != IC_OK) return rc;
  if (!a->head_mass) return IC_OK;
  if ((rc = ensure_dynamic_smem(summary_colsum_kernel<T>, C_BYTES, &lim_col)) != IC_OK) return rc;
  summary_colsum_kernel<T><<<grid, COL_THREADS, C_BYTES, st>>>(mq, mk, p);
  if ((rc = launch_status("summary_colsum_kernel")) != IC_OK) return rc;
  summary_reduce_kernel<<<a->batch, RED_THREADS, 0, st>>>(a->head_mass, a->colsum, a->importance,
                                                          a->num_q_heads, T_, a->accumulate);
  return launch_status("summary_reduce_kernel");
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
