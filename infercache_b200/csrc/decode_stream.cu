// Kernel A, fp16 / bf16, streaming form: one CTA streams one whole
// (session, KV head) group with no inter-CTA communication.
//
// Grid (Hkv, S).  The CTA copies the session's slot table into shared memory
// and streams the group's rows through a ring of NS stages of RB rows each,
// filled with 16-byte asynchronous copies (LDGSTS) addressed through the slot
// table: first all K rows, then all V rows.  The last logical slot is the
// staging row: its K/V come from k_new / v_new (also written to the pool).
//   K stages: S = Q . K^T on the tensor cores (mma.sync m16n8k16, fp32
//     accumulate; rows are the G <= 16 query heads), scores kept in shared
//     memory; while a stage's MMAs run, the warp that owns a head folds the
//     previous stage into that head's running (max, sum of exp), so after the
//     K pass every head's softmax max and sum are exact without any exchange.
//   Between the passes every thread turns its slots' scores into
//     p = exp(s - max) / sum, writes each slot's received mass summed over
//     the heads in order to its running sum over layers, and replaces each score
//     by a 32-bit word packing p as high and low half-precision parts
//     (~22 bits of P); the V-pass fragments re-pair the halves by byte permutes.
//   V stages: O += P . V on the tensor cores.
// One __syncthreads per stage guards the ring.
//
// Launch overlap: with programmatic dependent launch and inputs_ready (every
// layer's q / k_new / v_new exist before the step starts) the kernel lets the
// next layer launch at once and reads nothing another running kernel writes:
// the slot table and occupancy change only in the eviction kernel, which
// finished before layer 0 (which waits for it first) let later layers launch.
// Between the K and V passes the kernel waits for the previous layer before
// it adds its mass to the running sum, which keeps the sum in layer order and
// completion in layer order, so the eviction kernel that waits on the last
// layer sees every layer's mass.
#include <math.h>

#include "common.cuh"
#include "decode_internal.cuh"
#include "mma_helpers.cuh"

namespace ic {

constexpr int ST_THREADS = 256;
constexpr int ST_WARPS = ST_THREADS / 32;
constexpr int ST_D = 128;
constexpr int ST_RB = 64;  // rows per stage: one 8-row score block per warp
constexpr int ST_NS = 4;   // ring stages

__host__ __device__ inline int st_align(int x, int a) { return (x + a - 1) / a * a; }

struct StreamSmem {
  int ntp, nst, rowb, ppad;
  int sc_off, ring_off, row_off, occ_off, misc_off, total;
};

__host__ __device__ inline StreamSmem stream_smem(int ntot, int GP) {
  StreamSmem L;
  L.ntp = st_align(ntot, ST_RB);
  L.nst = L.ntp / ST_RB;
  L.rowb = ST_D * 2 + 16;  // padded rows: conflict-free ldmatrix
  L.ppad = L.ntp + 8;      // row stride of sc in words: conflict-free fragments
  int o = 0;
  // [GP][ppad] words: fp32 scores, then packed (hi, lo) halves of P in place
  L.sc_off = o;   o = st_align(o + GP * L.ppad * 4, 128);
  L.ring_off = o; o = st_align(o + ST_NS * ST_RB * L.rowb, 128);
  L.row_off = o;  o = st_align(o + L.ntp * 4, 16);
  L.occ_off = o;  o = st_align(o + L.ntp, 16);
  L.misc_off = o; o = st_align(o + 2 * GP * 4, 16);
  L.total = o;
  return L;
}

template <typename T, int GP>
__global__ void __launch_bounds__(ST_THREADS, 1) decode_stream_kernel(const ic_decode_args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int h = blockIdx.x, s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;  // mma fragment row / column pair
  const int budget = a.tiers.budget, ntot = budget + 1;
  const int Hkv = a.pool.num_kv_heads, Hq = a.num_q_heads, G = Hq / Hkv;

  const StreamSmem L = stream_smem(ntot, GP);
  const int ntp = L.ntp, nst = L.nst, rowb = L.rowb, ppad = L.ppad;
  float* sc = reinterpret_cast<float*>(smem + L.sc_off);  // [GP][ppad] scores, then packed P
  unsigned char* ring = smem + L.ring_off;
  int32_t* rows = reinterpret_cast<int32_t*>(smem + L.row_off);
  uint8_t* occ_s = smem + L.occ_off;
  float* stat = reinterpret_cast<float*>(smem + L.misc_off);  // [GP] max, [GP] 1/sum
  uint32_t* pw = reinterpret_cast<uint32_t*>(smem + L.sc_off);  // packed P after the K pass

  const bool early = a.pdl && a.inputs_ready && a.layer > 0;
  if (a.pdl && !early) grid_dependency_wait();
  if (a.pdl) grid_launch_dependents();

  const size_t plane = static_cast<size_t>(a.pool.pool_tokens) * ST_D;
  const size_t lh = static_cast<size_t>(a.layer) * Hkv + h;
  const T* pk = static_cast<const T*>(a.pool.k) + lh * plane;
  const T* pv = static_cast<const T*>(a.pool.v) + lh * plane;
  const int32_t* st = a.sess.slot_table + static_cast<size_t>(s) * ntot;
  const uint8_t* occ_g = a.sess.occupied + static_cast<size_t>(s) * budget;
  const T* kn = static_cast<const T*>(a.k_new) + (static_cast<size_t>(s) * Hkv + h) * ST_D;
  const T* vn = static_cast<const T*>(a.v_new) + (static_cast<size_t>(s) * Hkv + h) * ST_D;

  // q A-fragments: rows g (and g + 8 when GP == 16) of the group's heads
  uint32_t qa[8][4];
  {
    const T* qb = static_cast<const T*>(a.q) + (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * ST_D;
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(qb + static_cast<size_t>(g) * ST_D);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(qb + static_cast<size_t>(g + 8) * ST_D);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int w = kk * 8 + tq;  // 32-bit word of d = 16 kk + 2 tq
      qa[kk][0] = g < G ? q0[w] : 0u;
      qa[kk][2] = g < G ? q0[w + 4] : 0u;
      qa[kk][1] = (GP > 8 && g + 8 < G) ? q1[w] : 0u;
      qa[kk][3] = (GP > 8 && g + 8 < G) ? q1[w + 4] : 0u;
    }
  }

  // slot table of the session: pool row per logical slot; -2 marks the
  // staging row (fed from k_new / v_new), -1 the padding past the budget
  for (int t = tid; t < ntp; t += ST_THREADS) {
    int row = -1;
    uint8_t o = 0;
    if (t < budget) {
      row = st[t];
      o = occ_g[t];
      if (static_cast<unsigned long long>(row) >= static_cast<unsigned long long>(a.pool.pool_tokens)) {
        if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
        row = 0;
      }
    } else if (t == budget) {
      row = -2;
      o = 1;
    }
    rows[t] = row;
    occ_s[t] = o;
  }
  constexpr int VPR = ST_D * 2 / 16;  // 16-byte vectors per row
  if (tid < VPR) {  // the new token's K/V into the staging row of this layer
    const int row = st[budget];
    if (static_cast<unsigned long long>(row) < static_cast<unsigned long long>(a.pool.pool_tokens)) {
      reinterpret_cast<int4*>(static_cast<T*>(a.pool.k) + lh * plane + static_cast<size_t>(row) * ST_D)[tid] =
          reinterpret_cast<const int4*>(kn)[tid];
      reinterpret_cast<int4*>(static_cast<T*>(a.pool.v) + lh * plane + static_cast<size_t>(row) * ST_D)[tid] =
          reinterpret_cast<const int4*>(vn)[tid];
    } else if (tid == 0 && a.sess.dev_status) {
      atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
    }
  }
  __syncthreads();

  const int total_st = 2 * nst;
  auto issue = [&](int k) {
    if (k < total_st) {
      const bool is_k = k < nst;
      const int base = (is_k ? k : k - nst) * ST_RB;
      unsigned char* dst = ring + (k % ST_NS) * ST_RB * rowb;
      const T* src = is_k ? pk : pv;
      const int4* nrow = reinterpret_cast<const int4*>(is_k ? kn : vn);
      for (int i = tid; i < ST_RB * VPR; i += ST_THREADS) {
        const int t = i / VPR, v = i % VPR;
        const int row = rows[base + t];
        unsigned char* d = dst + t * rowb + v * 16;
        if (row >= 0)
          cp_async16(d, src + static_cast<size_t>(row) * ST_D + v * 8);
        else
          *reinterpret_cast<int4*>(d) = row == -2 ? nrow[v] : make_int4(0, 0, 0, 0);
      }
    }
    cp_async_commit();  // one group per stage, empty past the end
  };
#pragma unroll
  for (int k = 0; k < ST_NS - 1; ++k) issue(k);

  constexpr int HPW = GP / ST_WARPS > 0 ? GP / ST_WARPS : 1;  // heads owned per warp
  float run_m[HPW], run_l[HPW];
#pragma unroll
  for (int i = 0; i < HPW; ++i) { run_m[i] = -INFINITY; run_l[i] = 0.f; }
  // fold K stage `kst` (its 64 scores per head) into the owned heads' running
  // (max, sum of exp)
  auto fold = [&](int kst) {
    const int base = kst * ST_RB;
#pragma unroll
    for (int i = 0; i < HPW; ++i) {
      const int gg = warp + i * ST_WARPS;
      if (gg < G) {
        const float x0 = sc[gg * ppad + base + lane], x1 = sc[gg * ppad + base + lane + 32];
        const float mn = fmaxf(run_m[i], warp_max(fmaxf(x0, x1)));
        if (mn != -INFINITY) {
          float e = (x0 == -INFINITY ? 0.f : expf(x0 - mn)) + (x1 == -INFINITY ? 0.f : expf(x1 - mn));
          e = warp_sum(e);
          run_l[i] = (run_m[i] == -INFINITY ? 0.f : run_l[i] * expf(run_m[i] - mn)) + e;
          run_m[i] = mn;
        }
      }
    }
  };
  float oh[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  float ol[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const float scale = a.scale;

  for (int k = 0; k < total_st; ++k) {
    cp_async_wait<ST_NS - 2>();
    __syncthreads();  // stage k visible to all; every warp is past stage k-1
    if (k == nst) {
      // ---- between the passes: exact softmax, mass, packed P ------------------
      fold(nst - 1);
#pragma unroll
      for (int i = 0; i < HPW; ++i) {
        const int gg = warp + i * ST_WARPS;
        if (gg < G && lane == 0) {
          stat[gg] = run_m[i];
          stat[GP + gg] = 1.f / run_l[i];
        }
      }
      __syncthreads();
      // the running mass sum is folded in layer order: wait for the previous
      // layer here (this also keeps completion in layer order)
      if (a.pdl) grid_dependency_wait();
      float* mcol = a.mass + (static_cast<size_t>(s) * Hkv + h) * ntot;
      for (int t = tid; t < ntp; t += ST_THREADS) {
        float m = 0.f;
#pragma unroll
        for (int gg = 0; gg < GP; ++gg) {
          float p = 0.f;
          if (gg < G) {
            const float sv = sc[gg * ppad + t];
            p = sv == -INFINITY ? 0.f : expf(sv - stat[gg]) * stat[GP + gg];
            m += p;
          }
          const float ps = p * P_SCALE;
          const uint32_t hb = Mma<T>::bits(ps);
          pw[gg * ppad + t] = hb | (static_cast<uint32_t>(Mma<T>::bits(ps - Mma<T>::back(hb))) << 16);
        }
        if (t < ntot) mcol[t] = a.layer == 0 ? m : __fadd_rn(mcol[t], m);
      }
      __syncthreads();
    }
    issue(k + ST_NS - 1);
    const unsigned char* buf = ring + (k % ST_NS) * ST_RB * rowb;
    if (k < nst) {
      // ---- scores of rows [8w, 8w + 8) of this stage; fold the previous stage --
      const int base = k * ST_RB;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const uint32_t ra = smem_addr(buf) + (warp * 8 + (lane & 7)) * rowb + (lane >> 3) * 16;
#pragma unroll
      for (int kk2 = 0; kk2 < 4; ++kk2) {
        uint32_t b[4];
        ldsm_x4(b, ra + kk2 * 64);
        const uint32_t* x = qa[2 * kk2];
        const uint32_t* y = qa[2 * kk2 + 1];
        Mma<T>::run(acc[0], x[0], x[1], x[2], x[3], b[0], b[1]);
        Mma<T>::run(acc[1], y[0], y[1], y[2], y[3], b[2], b[3]);
      }
      if (k > 0) fold(k - 1);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int t = base + warp * 8 + 2 * tq + j;
        const bool o = occ_s[t] != 0;
        if (g < G) sc[g * ppad + t] = o ? (acc[0][j] + acc[1][j]) * scale : -INFINITY;
        if (GP > 8 && g + 8 < G) sc[(g + 8) * ppad + t] = o ? (acc[0][2 + j] + acc[1][2 + j]) * scale : -INFINITY;
      }
    } else {
      // ---- O += P . V: warp w owns head_dim columns [16w, 16w + 16) --------------
      const int base = (k - nst) * ST_RB;
      const int n0 = warp * 16;
      const uint32_t vaddr = smem_addr(buf) + (((lane >> 3) & 1) * 8 + (lane & 7)) * rowb + (n0 + (lane >> 4) * 8) * 2;
      // packed words of columns (c, c + 1) re-paired into (hi, hi) and (lo, lo)
      const uint2* r0 = reinterpret_cast<const uint2*>(pw + g * ppad);
      const uint2* r1 = reinterpret_cast<const uint2*>(pw + (g + 8) * ppad);
#pragma unroll
      for (int k0 = 0; k0 < ST_RB; k0 += 16) {
        const int w = (base + k0) / 2 + tq;  // pair index of column base + k0 + 2 tq
        const uint2 x0 = r0[w], x2 = r0[w + 4];
        const uint32_t h0 = __byte_perm(x0.x, x0.y, 0x5410), l0 = __byte_perm(x0.x, x0.y, 0x7632);
        const uint32_t h2 = __byte_perm(x2.x, x2.y, 0x5410), l2 = __byte_perm(x2.x, x2.y, 0x7632);
        uint32_t h1 = 0u, h3 = 0u, l1 = 0u, l3 = 0u;
        if (GP > 8) {
          const uint2 x1 = r1[w], x3 = r1[w + 4];
          h1 = __byte_perm(x1.x, x1.y, 0x5410);
          l1 = __byte_perm(x1.x, x1.y, 0x7632);
          h3 = __byte_perm(x3.x, x3.y, 0x5410);
          l3 = __byte_perm(x3.x, x3.y, 0x7632);
        }
        uint32_t b[4];
        ldsm_x4_t(b, vaddr + k0 * rowb);
        Mma<T>::run(oh[0], h0, h1, h2, h3, b[0], b[1]);
        Mma<T>::run(ol[0], l0, l1, l2, l3, b[0], b[1]);
        Mma<T>::run(oh[1], h0, h1, h2, h3, b[2], b[3]);
        Mma<T>::run(ol[1], l0, l1, l2, l3, b[2], b[3]);
      }
    }
  }
  cp_async_wait<0>();

  // ---- the group's output rows ----------------------------------------------------
  {
    const size_t ob = (static_cast<size_t>(s) * Hq + static_cast<size_t>(h) * G) * ST_D;
    const int n0 = warp * 16;
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int d = n0 + nb * 8 + 2 * tq + j;
        const float v0 = (oh[nb][j] + ol[nb][j]) * P_UNSCALE;
        const float v1 = (oh[nb][2 + j] + ol[nb][2 + j]) * P_UNSCALE;
        if (a.out_dtype == IC_F32) {
          if (g < G) static_cast<float*>(a.out)[ob + g * ST_D + d] = v0;
          if (GP > 8 && g + 8 < G) static_cast<float*>(a.out)[ob + (g + 8) * ST_D + d] = v1;
        } else {
          if (g < G) static_cast<T*>(a.out)[ob + g * ST_D + d] = DT<T>::from_f(v0);
          if (GP > 8 && g + 8 < G) static_cast<T*>(a.out)[ob + (g + 8) * ST_D + d] = DT<T>::from_f(v1);
        }
      }
  }
}

template <typename T, int GP>
static int launch_stream(const ic_decode_args& a, cudaStream_t stream) {
  const StreamSmem L = stream_smem(a.tiers.budget + 1, GP);
  if (L.total > 227 * 1024) {
    set_last_error("decode (stream): budget too large for one CTA's shared memory");
    return IC_ERR_UNSUPPORTED;
  }
  auto kern = decode_stream_kernel<T, GP>;
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(kern, L.total, &smem_limit)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.pool.num_kv_heads, a.sess.num_sessions, 1);
  cfg.blockDim = dim3(ST_THREADS, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, a);
  return launch_status("decode_layer (stream)");
}

int launch_decode_stream(const ic_decode_args& a, cudaStream_t stream) {
  const int G = a.num_q_heads / a.pool.num_kv_heads;
  if (a.pool.dtype == IC_F16)
    return G <= 8 ? launch_stream<__half, 8>(a, stream) : launch_stream<__half, 16>(a, stream);
  if (a.pool.dtype == IC_BF16)
    return G <= 8 ? launch_stream<__nv_bfloat16, 8>(a, stream) : launch_stream<__nv_bfloat16, 16>(a, stream);
  set_last_error("decode (stream): dtype must be fp16 or bf16");
  return IC_ERR_INVALID_ARG;
}

}  // namespace ic
