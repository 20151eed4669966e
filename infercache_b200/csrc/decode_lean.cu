// Kernel A, fp16 / bf16, lean form: one CTA per (session, KV head), four
// independent warp pipelines, no block-wide barrier while K/V stream.
//
// Each warp owns a contiguous run of 16-slot chunks of the session's slot
// table and streams, per chunk, the 16 K rows and 16 V rows (16-byte
// asynchronous copies through the slot table, double-buffered per warp):
//   S^T = K . Q^T   mma.sync m16n8k16 with the chunk's K rows as A (ldmatrix)
//                   and the group's query heads as B: eight heads fill n = 8
//                   exactly, and Q^T stays in registers for the whole pass.
//   online softmax  per head (a column of S^T): the running max is replaced
//                   only when a chunk raises it by more than 2^8, so the
//                   accumulator is rarely rescaled and P stays <= 2^8.
//   O^T += V^T P^T  V rows transposed by ldmatrix.trans as A, P^T as B: the
//                   S^T accumulator fragment becomes the B fragment with one
//                   movmatrix.trans per 8 x 8 block.  P enters as fp16 for an
//                   fp16 cache (2^-11 relative) and as a bf16 high + low pair
//                   for a bf16 cache.
// Each chunk's scaled scores go to shared memory; after the four warps'
// (max, sum, O) are merged, the exact softmax gives every slot's received
// mass (summed over the group's heads), which the CTA adds to the slot's
// running sum over layers once the previous layer has completed.
//
// The last logical slot is the staging row: its K/V come from k_new / v_new,
// which the CTA also writes to the pool.  Programmatic dependent launch
// follows the streaming kernel's protocol: with inputs_ready, layers after
// the first read nothing another running kernel writes and let the next
// layer launch at once; the grid-dependency wait before the mass fold keeps
// the sum and completion in layer order for the eviction kernel.
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "decode_internal.cuh"
#include "mma_helpers.cuh"

namespace ic {
namespace {

constexpr int LN_D = 128;
constexpr int LN_R = 16;                       // rows per chunk
constexpr int LN_PITCH = LN_D * 2 + 16;        // padded row: conflict-free ldmatrix
constexpr int LN_STAGE = 2 * LN_R * LN_PITCH;  // K chunk + V chunk
constexpr float LN_LOG2E = 1.4426950408889634f;
constexpr float LN_RESCALE = 8.0f;

__host__ __device__ inline int ln_align(int x, int a) { return (x + a - 1) / a * a; }

struct LeanSmem {
  int nch, ntp, pitch;  // chunks, padded slots, score row pitch (words)
  int sc_off, row_off, occ_off, stat_off, total;
};

__host__ __device__ inline LeanSmem lean_smem(int ntot, int NG, int W) {
  LeanSmem L;
  L.nch = (ntot + LN_R - 1) / LN_R;
  L.ntp = L.nch * LN_R;
  L.pitch = ln_align(L.ntp, 32) + 4;  // pitch % 32 == 4: conflict-free score stores
  int o = W * 2 * LN_STAGE;          // the merge buffers and mass alias the ring afterwards
  const int merge = W * NG * 8 * (LN_D + 2) * 4 + L.ntp * 4;
  if (merge > o) o = merge;
  o = ln_align(o, 128);
  L.sc_off = o;   o = ln_align(o + NG * 8 * L.pitch * 4, 16);
  L.row_off = o;  o = ln_align(o + L.ntp * 4, 16);
  L.occ_off = o;  o = ln_align(o + L.ntp, 16);
  L.stat_off = o; o = ln_align(o + 2 * NG * 8 * 4, 16);
  L.total = o;
  return L;
}

__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  return static_cast<uint32_t>(Mma<T>::bits(lo)) | (static_cast<uint32_t>(Mma<T>::bits(hi)) << 16);
}

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T, int NG, int W>
__global__ void __launch_bounds__(W * 32, 8 / W) decode_lean_kernel(const ic_decode_args a) {
  constexpr int NT = W * 32;
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr bool SPLIT = std::is_same<T, __nv_bfloat16>::value;  // P as high + low bf16
  const int h = blockIdx.x, s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int budget = a.tiers.budget, ntot = budget + 1;
  const int Hkv = a.pool.num_kv_heads, Hq = a.num_q_heads, G = Hq / Hkv;
  const LeanSmem L = lean_smem(ntot, NG, W);
  const int nch = L.nch, ntp = L.ntp, pitch = L.pitch;
  float* sc = reinterpret_cast<float*>(smem + L.sc_off);  // [NG*8][pitch] log2-scaled scores
  int32_t* rows = reinterpret_cast<int32_t*>(smem + L.row_off);
  uint8_t* occ_s = smem + L.occ_off;
  float* stat = reinterpret_cast<float*>(smem + L.stat_off);  // [NG*8] max, [NG*8] 1 / sum

  const bool early = a.pdl && a.inputs_ready && a.layer > 0;
  if (a.pdl && !early) grid_dependency_wait();
  if (a.pdl) grid_launch_dependents();

  const size_t plane = static_cast<size_t>(a.pool.pool_tokens) * LN_D;
  const size_t lh = static_cast<size_t>(a.layer) * Hkv + h;
  const T* pk = static_cast<const T*>(a.pool.k) + lh * plane;
  const T* pv = static_cast<const T*>(a.pool.v) + lh * plane;
  const int32_t* st = a.sess.slot_table + static_cast<size_t>(s) * ntot;
  const uint8_t* occ_g = a.sess.occupied + static_cast<size_t>(s) * budget;
  const T* kn = static_cast<const T*>(a.k_new) + (static_cast<size_t>(s) * Hkv + h) * LN_D;
  const T* vn = static_cast<const T*>(a.v_new) + (static_cast<size_t>(s) * Hkv + h) * LN_D;
  const float sl2 = a.scale * LN_LOG2E;

  // Q^T as the B operand: b[kk][0] = q[head 8 nt + g][16 kk + 2 tq, +1],
  // b[kk][1] = the same at + 8 (heads past G are zero)
  uint32_t qb[NG][8][2];
  {
    const T* qg = static_cast<const T*>(a.q) + (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * LN_D;
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) {
      const int head = nt * 8 + g;
      const uint32_t* qr = reinterpret_cast<const uint32_t*>(qg + static_cast<size_t>(head) * LN_D);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[nt][kk][0] = head < G ? qr[kk * 8 + tq] : 0u;
        qb[nt][kk][1] = head < G ? qr[kk * 8 + 4 + tq] : 0u;
      }
    }
  }

  // slot table: pool row per logical slot; -2 = staging row, -1 = padding
  for (int t = tid; t < ntp; t += NT) {
    int row = -1;
    uint8_t o = 0;
    if (t < budget) {
      row = st[t];
      o = occ_g[t];
      if (static_cast<unsigned long long>(row) >= static_cast<unsigned long long>(a.pool.pool_tokens)) {
        if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
        row = 0;
        o = 0;
      }
    } else if (t == budget) {
      row = -2;
      o = 1;
    }
    rows[t] = row;
    occ_s[t] = o;
  }
  constexpr int VPR = LN_D * 2 / 16;  // 16-byte vectors per row
  if (tid < VPR) {  // the new token's K/V into the staging row of this layer
    const int row = st[budget];
    if (static_cast<unsigned long long>(row) < static_cast<unsigned long long>(a.pool.pool_tokens)) {
      reinterpret_cast<int4*>(static_cast<T*>(a.pool.k) + lh * plane + static_cast<size_t>(row) * LN_D)[tid] =
          reinterpret_cast<const int4*>(kn)[tid];
      reinterpret_cast<int4*>(static_cast<T*>(a.pool.v) + lh * plane + static_cast<size_t>(row) * LN_D)[tid] =
          reinterpret_cast<const int4*>(vn)[tid];
    } else if (tid == 0 && a.sess.dev_status) {
      atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
    }
  }
  __syncthreads();

  // this warp's chunks
  const int per = (nch + W - 1) / W;
  const int c0 = warp * per;
  const int c1 = min(nch, c0 + per);
  constexpr int NSTG = 2;
  unsigned char* wring = smem + warp * NSTG * LN_STAGE;

  auto issue = [&](int c) {
    if (c < c1) {
      unsigned char* dk = wring + ((c - c0) % NSTG) * LN_STAGE;
      unsigned char* dv = dk + LN_R * LN_PITCH;
      const int v = lane & 15;
#pragma unroll
      for (int i = 0; i < LN_R / 2; ++i) {
        const int r = (lane >> 4) + 2 * i;
        const int row = rows[c * LN_R + r];
        unsigned char* d0 = dk + r * LN_PITCH + v * 16;
        unsigned char* d1 = dv + r * LN_PITCH + v * 16;
        if (row >= 0) {
          cp_async16(d0, pk + static_cast<size_t>(row) * LN_D + v * 8);
          cp_async16(d1, pv + static_cast<size_t>(row) * LN_D + v * 8);
        } else if (row == -2) {
          *reinterpret_cast<int4*>(d0) = reinterpret_cast<const int4*>(kn)[v];
          *reinterpret_cast<int4*>(d1) = reinterpret_cast<const int4*>(vn)[v];
        } else {
          *reinterpret_cast<int4*>(d0) = make_int4(0, 0, 0, 0);
          *reinterpret_cast<int4*>(d1) = make_int4(0, 0, 0, 0);
        }
      }
    }
    cp_async_commit();
  };

  float m_run[NG][2], l_run[NG][2];
  float o[NG][8][4];
#pragma unroll
  for (int nt = 0; nt < NG; ++nt) {
    m_run[nt][0] = m_run[nt][1] = -INFINITY;
    l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
  }

#pragma unroll
  for (int i = 0; i < NSTG - 1; ++i) issue(c0 + i);
  for (int c = c0; c < c1; ++c) {
    issue(c + NSTG - 1);
    cp_async_wait<NSTG - 1>();
    __syncwarp();
    const unsigned char* bk = wring + ((c - c0) % NSTG) * LN_STAGE;
    const unsigned char* bv = bk + LN_R * LN_PITCH;
    const int r0 = c * LN_R;

    // ---- S^T = K Q^T for the chunk's 16 rows ------------------------------------
    float acc[NG][4];
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    const uint32_t ka = smem_addr(bk) + (lane & 15) * LN_PITCH + (lane >> 4) * 16;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t ar[4];
      ldsm_x4(ar, ka + kk * 32);
#pragma unroll
      for (int nt = 0; nt < NG; ++nt) Mma<T>::run(acc[nt], ar[0], ar[1], ar[2], ar[3], qb[nt][kk][0], qb[nt][kk][1]);
    }
    const bool ok0 = occ_s[r0 + g] != 0, ok1 = occ_s[r0 + g + 8] != 0;
    bool any_rescale = false;
    float alpha[NG][2];
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) {
      // x[0], x[1]: row g, heads 2tq, 2tq+1; x[2], x[3]: row g + 8
      float x0 = ok0 ? acc[nt][0] * sl2 : -INFINITY, x1 = ok0 ? acc[nt][1] * sl2 : -INFINITY;
      float x2 = ok1 ? acc[nt][2] * sl2 : -INFINITY, x3 = ok1 ? acc[nt][3] * sl2 : -INFINITY;
      acc[nt][0] = x0; acc[nt][1] = x1; acc[nt][2] = x2; acc[nt][3] = x3;
      float* sc0 = sc + (nt * 8 + 2 * tq) * pitch + r0;
      sc0[g] = x0;
      sc0[pitch + g] = x1;
      sc0[g + 8] = x2;
      sc0[pitch + g + 8] = x3;
      float ma = fmaxf(x0, x2), mb = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, off));
        mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      }
      const float mc[2] = {ma, mb};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        alpha[nt][j] = 1.f;
        if (mc[j] > m_run[nt][j] + LN_RESCALE) {
          alpha[nt][j] = m_run[nt][j] == -INFINITY ? 0.f : fast_ex2(m_run[nt][j] - mc[j]);
          m_run[nt][j] = mc[j];
          any_rescale = true;
        }
      }
    }
    if (__any_sync(0xffffffffu, any_rescale)) {
#pragma unroll
      for (int nt = 0; nt < NG; ++nt) {
        l_run[nt][0] *= alpha[nt][0];
        l_run[nt][1] *= alpha[nt][1];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[nt][mt][0] *= alpha[nt][0];
          o[nt][mt][1] *= alpha[nt][1];
          o[nt][mt][2] *= alpha[nt][0];
          o[nt][mt][3] *= alpha[nt][1];
        }
      }
    }
    // ---- P^T fragments ----------------------------------------------------------
    uint32_t bh[NG][2], bl[NG][2];
#pragma unroll
    for (int nt = 0; nt < NG; ++nt) {
      float p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float m = m_run[nt][i & 1];
        p[i] = m == -INFINITY ? 0.f : fast_ex2(acc[nt][i] - m);
      }
      l_run[nt][0] += p[0] + p[2];
      l_run[nt][1] += p[1] + p[3];
      const uint32_t h01 = pack_pair<T>(p[0], p[1]), h23 = pack_pair<T>(p[2], p[3]);
      bh[nt][0] = movtrans(h01);
      bh[nt][1] = movtrans(h23);
      if (SPLIT) {
        const float r0f = p[0] - Mma<T>::back(static_cast<uint16_t>(h01 & 0xffffu));
        const float r1f = p[1] - Mma<T>::back(static_cast<uint16_t>(h01 >> 16));
        const float r2f = p[2] - Mma<T>::back(static_cast<uint16_t>(h23 & 0xffffu));
        const float r3f = p[3] - Mma<T>::back(static_cast<uint16_t>(h23 >> 16));
        bl[nt][0] = movtrans(pack_pair<T>(r0f, r1f));
        bl[nt][1] = movtrans(pack_pair<T>(r2f, r3f));
      }
    }
    // ---- O^T += V^T P^T ---------------------------------------------------------
    const uint32_t va = smem_addr(bv) + ((lane & 7) + ((lane >> 4) << 3)) * LN_PITCH + ((lane >> 3) & 1) * 16;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      uint32_t ar[4];
      ldsm_x4_t(ar, va + mt * 32);
#pragma unroll
      for (int nt = 0; nt < NG; ++nt) {
        Mma<T>::run(o[nt][mt], ar[0], ar[1], ar[2], ar[3], bh[nt][0], bh[nt][1]);
        if (SPLIT) Mma<T>::run(o[nt][mt], ar[0], ar[1], ar[2], ar[3], bl[nt][0], bl[nt][1]);
      }
    }
    __syncwarp();  // every lane is done with this buffer before it is refilled
  }
  cp_async_wait<0>();

  // ---- merge the four warps --------------------------------------------------------
#pragma unroll
  for (int nt = 0; nt < NG; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) l_run[nt][j] += __shfl_xor_sync(0xffffffffu, l_run[nt][j], off);
  __syncthreads();  // the ring is free: merge buffers alias it
  constexpr int HS = NG * 8;
  float* wo = reinterpret_cast<float*>(smem);          // [warp][head][LN_D]
  float* wm = wo + W * HS * LN_D;                // [warp][head]
  float* wl = wm + W * HS;                       // [warp][head]
  float* ms = wl + W * HS;                       // [ntp] this layer's mass per slot
#pragma unroll
  for (int nt = 0; nt < NG; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int head = nt * 8 + 2 * tq + j;
      float* dst = wo + (warp * HS + head) * LN_D;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        dst[mt * 16 + g] = o[nt][mt][j];
        dst[mt * 16 + g + 8] = o[nt][mt][2 + j];
      }
      if (g == 0) {
        wm[warp * HS + head] = m_run[nt][j];
        wl[warp * HS + head] = l_run[nt][j];
      }
    }
  }
  __syncthreads();
  {
    const size_t ob = (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * LN_D;
    for (int e = tid; e < HS * (LN_D / 8); e += NT) {
      const int head = e / (LN_D / 8), d0 = (e % (LN_D / 8)) * 8;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < W; ++w) M = fmaxf(M, wm[w * HS + head]);
      float f[W], Lsum = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float mw = wm[w * HS + head];
        f[w] = mw == -INFINITY ? 0.f : fast_ex2(mw - M);
        Lsum = fmaf(wl[w * HS + head], f[w], Lsum);
      }
      const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
      if (d0 == 0) {
        stat[head] = M;
        stat[HS + head] = inv;
      }
      if (head < G) {
        // eight consecutive outputs leave as one 16-byte store (two for fp32),
        // which also keeps the writes whole when `out` is mapped host memory
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          x[i] = 0.f;
#pragma unroll
          for (int w = 0; w < W; ++w) x[i] = fmaf(wo[(w * HS + head) * LN_D + d0 + i], f[w], x[i]);
          x[i] *= inv;
        }
        const size_t o0 = ob + static_cast<size_t>(head) * LN_D + d0;
        if (a.out_dtype == IC_F32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + o0);
          dst[0] = make_float4(x[0], x[1], x[2], x[3]);
          dst[1] = make_float4(x[4], x[5], x[6], x[7]);
        } else {
          *reinterpret_cast<uint4*>(static_cast<T*>(a.out) + o0) =
              make_uint4(pack_pair<T>(x[0], x[1]), pack_pair<T>(x[2], x[3]), pack_pair<T>(x[4], x[5]),
                         pack_pair<T>(x[6], x[7]));
        }
      }
    }
  }
  __syncthreads();
  // ---- received mass of every slot, exact softmax, heads in order -------------------
  for (int t = tid; t < ntot; t += NT) {
    float m = 0.f;
    for (int head = 0; head < G; ++head) {
      const float x = sc[head * pitch + t];
      if (x != -INFINITY) m += fast_ex2(x - stat[head]) * stat[HS + head];
    }
    ms[t] = m;
  }
  // Fold into the running sum in layer order: after the previous layer has
  // completed (which also keeps completion in layer order for kernel B).
  if (a.pdl) grid_dependency_wait();
  float* macc = a.mass + (static_cast<size_t>(s) * Hkv + h) * ntot;
  for (int t0 = 0; t0 < ntot; t0 += 8 * NT) {  // all loads of a batch before its stores
    float x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int t = t0 + i * NT + tid;
      x[i] = (a.layer > 0 && t < ntot) ? macc[t] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int t = t0 + i * NT + tid;
      if (t < ntot) macc[t] = a.layer == 0 ? ms[t] : __fadd_rn(x[i], ms[t]);
    }
  }
}

template <typename T, int NG, int W>
int launch_one(const ic_decode_args& a, cudaStream_t stream, const LeanSmem& L) {
  auto kern = decode_lean_kernel<T, NG, W>;
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(kern, L.total, &smem_limit)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.pool.num_kv_heads, a.sess.num_sessions, 1);
  cfg.blockDim = dim3(W * 32, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, a);
  return launch_status("decode_layer (lean)");
}

// Four warp pipelines per CTA when two CTAs fit an SM (the best shape at the
// 1040-slot budget); eight, one CTA per SM, when the budget's score buffer
// leaves room for only one.
template <typename T, int NG>
int launch_lean(const ic_decode_args& a, cudaStream_t stream) {
  constexpr int SM_BYTES = 228 * 1024, CTA_RESERVED = 1024;
  const int ntot = a.tiers.budget + 1;
  const LeanSmem L4 = lean_smem(ntot, NG, 4);
  if (2 * (L4.total + CTA_RESERVED) <= SM_BYTES) return launch_one<T, NG, 4>(a, stream, L4);
  const LeanSmem L8 = lean_smem(ntot, NG, 8);
  if (L8.total <= 227 * 1024) return launch_one<T, NG, 8>(a, stream, L8);
  if (L4.total <= 227 * 1024) return launch_one<T, NG, 4>(a, stream, L4);
  set_last_error("decode (lean): budget too large for one CTA's shared memory");
  return IC_ERR_UNSUPPORTED;
}

}  // namespace

int launch_decode_lean(const ic_decode_args& a, cudaStream_t stream) {
  const int G = a.num_q_heads / a.pool.num_kv_heads;
  if (G > 16) {
    set_last_error("decode (lean): at most 16 query heads per KV head");
    return IC_ERR_UNSUPPORTED;
  }
  if (a.pool.dtype == IC_F16)
    return G <= 8 ? launch_lean<__half, 1>(a, stream) : launch_lean<__half, 2>(a, stream);
  if (a.pool.dtype == IC_BF16)
    return G <= 8 ? launch_lean<__nv_bfloat16, 1>(a, stream) : launch_lean<__nv_bfloat16, 2>(a, stream);
  set_last_error("decode (lean): dtype must be fp16 or bf16");
  return IC_ERR_INVALID_ARG;
}

}  // namespace ic

