// Graph (cluster-routed) cache: sinks, a recent ring and n_clusters clusters
// of cluster_capacity slots, each cluster with an online mean of its tokens'
// layer-0 / head-0 keys as centroid (graph_cache.py:218-495).
//
// Storage is one slot store K/V [L, H, NS, D] (NS = sink + recent + C * cap;
// slot order: sinks, ring, cluster 0, cluster 1, ...) with per-slot
// positions, per-cluster-slot scores, centroids [C, D] float32, cluster fill
// and centroid counts, and ctrl = {sink fill, ring pointer, ring fill}.
//
// A push of T tokens (or a bulk load after a reset) is two phases.  The
// routing kernel (one CTA) replays the reference's per-token decisions on the
// layer-0 / head-0 keys only -- where each token goes, which cluster a
// displaced ring token joins (cosine similarity to the centroids, threshold,
// first empty or least-filled cluster), which slot a full cluster evicts
// (first index of the minimum score), the centroid updates -- and records for
// every slot where its content now comes from: unchanged, an old slot, or a
// new token.  The copy kernels then move the K/V rows of every layer and head
// in parallel: first the rows that come from old slots (only ring slots move,
// into cluster slots), then the rows that come from the new tokens.
//
// Centroid arithmetic is float32 with each operation rounded on its own, in
// the reference's order ((c * n + k) / (n + 1), (c * n - k) / (n - 1)), so
// centroids are bit-identical; cosine similarities are float32 warp sums.
#include <math.h>

#include "common.cuh"

namespace ic {
namespace {

constexpr int GR_THREADS = 256;
constexpr int GR_D = 128;  // head_dim the routing kernel handles

__device__ __forceinline__ float load_as_float(const void* p, size_t i, int dt) {
  if (dt == IC_F32) return static_cast<const float*>(p)[i];
  if (dt == IC_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

struct GraphView {
  ic_graph_state g;
  int NS, ring0, cl0;
  __device__ int cslot(int c, int i) const { return cl0 + c * g.cluster_capacity + i; }
};

// source codes in slot_src: -1 unchanged, t >= 0 new token t, -2 - s old slot
// s, SRC_CLEAR zeroed (an empty slot after a reset)
constexpr int SRC_CLEAR = -0x40000000;
__device__ __forceinline__ int old_code(int s) { return -2 - s; }

// cos(q, centroid[c]) for every cluster (-1 when empty) into sims[], by the
// whole CTA: warp w takes clusters w, w + 8, ...; lane l holds q[4l .. 4l+3].
__device__ void cluster_sims(const float* q, const float* cent, const int* cnt, int C, float* sims) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float qq = 0.f;
  float qv[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    qv[u] = q[4 * lane + u];
    qq = fmaf(qv[u], qv[u], qq);
  }
  qq = warp_sum(qq);
  const float qn = fmaxf(sqrtf(qq), 1e-6f);
  for (int c = warp; c < C; c += GR_THREADS / 32) {
    float cc = 0.f, qc = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float x = cent[c * GR_D + 4 * lane + u];
      cc = fmaf(x, x, cc);
      qc = fmaf(qv[u], x, qc);
    }
    cc = warp_sum(cc);
    qc = warp_sum(qc);
    if (lane == 0) sims[c] = cnt[c] == 0 ? -1.f : qc / (qn * fmaxf(sqrtf(cc), 1e-6f));
  }
}

__global__ void __launch_bounds__(GR_THREADS) graph_route_kernel(const ic_graph_push_args a) {
  extern __shared__ __align__(16) unsigned char gsm[];
  const ic_graph_state& g = a.g;
  const int C = g.n_clusters, cap = g.cluster_capacity, R = g.recent_size, SK = g.sink_size;
  GraphView V{g, SK + R + C * cap, SK, SK + R};
  const int NS = V.NS, tid = threadIdx.x;
  int64_t* pos = reinterpret_cast<int64_t*>(gsm);               // [NS]
  float* cent = reinterpret_cast<float*>(pos + NS);             // [C][D]
  float* score = cent + C * GR_D;                               // [C * cap]
  int* src = reinterpret_cast<int*>(score + C * cap);           // [NS] content source
  int* fill = src + NS;                                         // [C]
  int* cnt = fill + C;                                          // [C]
  float* sims = reinterpret_cast<float*>(cnt + C);              // [C]
  float* key = sims + C;                                        // [D] routing key
  __shared__ int ctrl_s[3];
  __shared__ int dec_c, dec_slot, dec_evict, disp;

  // ---- load (or clear) the state ---------------------------------------------------
  for (int i = tid; i < C * GR_D; i += GR_THREADS) cent[i] = a.reset ? 0.f : g.centroid[i];
  for (int i = tid; i < C * cap; i += GR_THREADS) score[i] = a.reset ? 0.f : g.scores[i];
  for (int i = tid; i < NS; i += GR_THREADS) {
    pos[i] = a.reset ? -1 : g.positions[i];
    src[i] = a.reset ? -1 : old_code(i);
  }
  for (int i = tid; i < C; i += GR_THREADS) {
    fill[i] = a.reset ? 0 : g.cl_fill[i];
    cnt[i] = a.reset ? 0 : g.c_count[i];
  }
  if (tid < 3) ctrl_s[tid] = a.reset ? 0 : g.ctrl[tid];
  __syncthreads();

  for (int t = 0; t < a.T; ++t) {
    const int64_t position = a.positions[t];
    const float sc = a.scores ? a.scores[t] : 0.f;
    // sinks fill by absolute position (graph_cache.py:303-309)
    if (position < SK && ctrl_s[0] < SK) {
      __syncthreads();
      if (tid == 0) {
        const int s = ctrl_s[0];
        src[s] = t;
        pos[s] = position;
        ctrl_s[0] = s + 1;
      }
      __syncthreads();
      continue;
    }
    const int ptr = ctrl_s[1];
    const int rs = V.ring0 + ptr;
    if (tid == 0) disp = pos[rs] >= 0;
    __syncthreads();
    if (disp) {
      // the displaced token's layer-0 / head-0 key, from where its content is now
      const int s0 = src[rs];
      for (int d = tid; d < GR_D; d += GR_THREADS) {
        key[d] = s0 >= 0 ? load_as_float(a.k_src, static_cast<size_t>(s0) * a.stride_t + d, g.dtype)
                         : load_as_float(g.k, static_cast<size_t>(-2 - s0) * GR_D + d, g.dtype);
      }
      __syncthreads();
      cluster_sims(key, cent, cnt, C, sims);
      __syncthreads();
      if (tid == 0) {
        // best cluster (first maximum); below threshold: first empty, else least filled
        int bi = -1;
        float bs = -2.f;
        for (int c = 0; c < C; ++c)
          if (sims[c] > bs) { bs = sims[c]; bi = c; }
        if (bs < g.sim_threshold) {
          int e = -1;
          for (int c = 0; c < C && e < 0; ++c)
            if (fill[c] == 0) e = c;
          if (e < 0) {
            e = 0;
            for (int c = 1; c < C; ++c)
              if (fill[c] < fill[e]) e = c;
          }
          bi = e;
        }
        dec_c = bi;
        if (fill[bi] >= cap) {
          int ei = 0;
          for (int i = 1; i < fill[bi]; ++i)
            if (score[bi * cap + i] < score[bi * cap + ei]) ei = i;
          dec_evict = ei;
          dec_slot = ei;
        } else {
          dec_evict = -1;
          dec_slot = fill[bi];
        }
      }
      __syncthreads();
      const int c = dec_c, slot = dec_slot, cs = V.cslot(c, slot);
      if (dec_evict >= 0) {
        // remove the evicted token from the centroid (graph_cache.py:160-169)
        const int se = src[cs];
        const int n = cnt[c];
        for (int d = tid; d < GR_D; d += GR_THREADS) {
          if (n > 1) {
            const float old = se >= 0 ? load_as_float(a.k_src, static_cast<size_t>(se) * a.stride_t + d, g.dtype)
                                      : load_as_float(g.k, static_cast<size_t>(-2 - se) * GR_D + d, g.dtype);
            cent[c * GR_D + d] = __fdiv_rn(__fsub_rn(__fmul_rn(cent[c * GR_D + d], static_cast<float>(n)), old),
                                           static_cast<float>(n - 1));
          } else {
            cent[c * GR_D + d] = 0.f;
          }
        }
      }
      __syncthreads();
      if (tid == 0) {
        if (dec_evict >= 0) cnt[c] = cnt[c] > 1 ? cnt[c] - 1 : 0;
        else fill[c] += 1;
        src[cs] = src[rs];
        pos[cs] = pos[rs];
        score[c * cap + slot] = sc;  // the current token's score (graph_cache.py:314)
      }
      __syncthreads();
      // add the new member (graph_cache.py:181-184)
      const float n = static_cast<float>(cnt[c]);
      for (int d = tid; d < GR_D; d += GR_THREADS)
        cent[c * GR_D + d] = __fdiv_rn(__fadd_rn(__fmul_rn(cent[c * GR_D + d], n), key[d]), n + 1.f);
      __syncthreads();
      if (tid == 0) cnt[c] += 1;
    }
    if (tid == 0) {
      src[rs] = t;
      pos[rs] = position;
      ctrl_s[2] = ctrl_s[2] + 1 < R ? ctrl_s[2] + 1 : R;
      ctrl_s[1] = (ptr + 1) % R;
    }
    __syncthreads();
  }

  // ---- write the state back; slot sources for the copy kernels ---------------------
  for (int i = tid; i < C * GR_D; i += GR_THREADS) g.centroid[i] = cent[i];
  for (int i = tid; i < C * cap; i += GR_THREADS) g.scores[i] = score[i];
  for (int i = tid; i < NS; i += GR_THREADS) {
    g.positions[i] = pos[i];
    const int s = src[i];
    a.slot_src[i] = s == old_code(i) ? -1 : (a.reset && s < 0 ? SRC_CLEAR : s);
  }
  for (int i = tid; i < C; i += GR_THREADS) {
    g.cl_fill[i] = fill[i];
    g.c_count[i] = cnt[i];
  }
  if (tid < 3) g.ctrl[tid] = ctrl_s[tid];
}

// Copy phase: one thread per 16-byte vector of a (layer, head, slot) row.
// phase 0: rows whose source is an old slot; phase 1: rows from new tokens
// (and rows cleared by a reset).
template <typename T>
__global__ void graph_copy_kernel(const ic_graph_push_args a, int phase) {
  const ic_graph_state& g = a.g;
  const int NS = g.sink_size + g.recent_size + g.n_clusters * g.cluster_capacity;
  constexpr int VPR = GR_D * static_cast<int>(sizeof(T)) / 16;
  const int64_t total = static_cast<int64_t>(g.num_layers) * g.num_kv_heads * NS * VPR;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int vec = static_cast<int>(e % VPR);
    const int64_t row = e / VPR;  // (l * H + h) * NS + slot
    const int slot = static_cast<int>(row % NS);
    const int64_t lh = row / NS;
    const int s = a.slot_src[slot];
    if (s == -1) continue;
    const bool from_old = s <= -2 && s != SRC_CLEAR;
    if ((phase == 0) != from_old) continue;
    int4 kv, vv;
    if (s == SRC_CLEAR) {
      kv = vv = make_int4(0, 0, 0, 0);
    } else if (from_old) {
      const int64_t o = (lh * NS + (-2 - s)) * VPR + vec;
      kv = reinterpret_cast<const int4*>(g.k)[o];
      vv = reinterpret_cast<const int4*>(g.v)[o];
    } else {
      const int l = static_cast<int>(lh / g.num_kv_heads), h = static_cast<int>(lh % g.num_kv_heads);
      const int64_t o = l * a.stride_l + h * a.stride_h + static_cast<int64_t>(s) * a.stride_t;
      kv = reinterpret_cast<const int4*>(static_cast<const T*>(a.k_src) + o)[vec];
      vv = reinterpret_cast<const int4*>(static_cast<const T*>(a.v_src) + o)[vec];
    }
    reinterpret_cast<int4*>(g.k)[row * VPR + vec] = kv;
    reinterpret_cast<int4*>(g.v)[row * VPR + vec] = vv;
  }
}

// Cluster selection for a query and the retrieve order of the slots
// (graph_cache.py:363-440): sinks in slot order, the first ring-fill ring
// slots by position, then each selected non-empty cluster by position.
__global__ void __launch_bounds__(GR_THREADS) graph_select_kernel(const ic_graph_select_args a) {
  const ic_graph_state& g = a.g;
  const int C = g.n_clusters, cap = g.cluster_capacity, R = g.recent_size, SK = g.sink_size;
  const int ring0 = SK, cl0 = SK + R;
  const int tid = threadIdx.x;
  __shared__ float qm[GR_D];
  __shared__ float sims[1024];
  __shared__ unsigned char sel[1024];
  __shared__ int base_s;
  const int H = g.num_kv_heads;
  for (int d = tid; d < GR_D; d += GR_THREADS) {
    float s = 0.f;
    for (int h = 0; h < H; ++h) s += a.query[h * GR_D + d];
    qm[d] = s / static_cast<float>(H);
  }
  __syncthreads();
  cluster_sims(qm, g.centroid, g.c_count, C, sims);
  __syncthreads();
  if (tid == 0) {
    for (int c = 0; c < C; ++c) sel[c] = 0;
    if (a.top_n > 0) {
      // the top_n largest similarities (ties: lower index first)
      const int k = a.top_n < C ? a.top_n : C;
      for (int r = 0; r < k; ++r) {
        int bi = -1;
        for (int c = 0; c < C; ++c)
          if (!sel[c] && (bi < 0 || sims[c] > sims[bi])) bi = c;
        sel[bi] = 1;
      }
    } else {
      bool any = false;
      for (int c = 0; c < C; ++c) {
        sel[c] = sims[c] >= a.threshold;
        any = any || sel[c];
      }
      if (!any) {
        int bi = 0;
        for (int c = 1; c < C; ++c)
          if (sims[c] > sims[bi]) bi = c;
        sel[bi] = 1;
      }
    }
    for (int c = 0; c < C; ++c) a.selected[c] = sel[c];
  }
  __syncthreads();
  const int sink_fill = g.ctrl[0], ring_fill = g.ctrl[2];
  // sinks
  for (int i = tid; i < sink_fill; i += GR_THREADS) a.slots[i] = i;
  // ring by position (positions are distinct: rank = number of smaller ones)
  for (int i = tid; i < ring_fill; i += GR_THREADS) {
    const int64_t p = g.positions[ring0 + i];
    int rank = 0;
    for (int j = 0; j < ring_fill; ++j) rank += g.positions[ring0 + j] < p;
    a.slots[sink_fill + rank] = ring0 + i;
  }
  if (tid == 0) base_s = sink_fill + ring_fill;
  __syncthreads();
  for (int c = 0; c < C; ++c) {
    const int f = g.cl_fill[c];
    if (!sel[c] || f == 0) continue;
    const int base = base_s;
    for (int i = tid; i < f; i += GR_THREADS) {
      const int64_t p = g.positions[cl0 + c * cap + i];
      int rank = 0;
      for (int j = 0; j < f; ++j) rank += g.positions[cl0 + c * cap + j] < p;
      a.slots[base + rank] = cl0 + c * cap + i;
    }
    __syncthreads();
    if (tid == 0) base_s = base + f;
    __syncthreads();
  }
  if (tid == 0) *a.count = base_s;
}

bool graph_state_ok(const ic_graph_state& g) {
  return g.k && g.v && g.positions && g.scores && g.centroid && g.cl_fill && g.c_count && g.ctrl &&
         g.num_layers > 0 && g.num_kv_heads > 0 && g.head_dim == GR_D && g.sink_size >= 0 &&
         g.recent_size >= 1 && g.n_clusters >= 1 && g.n_clusters <= 1024 && g.cluster_capacity >= 1 &&
         (g.dtype == IC_F16 || g.dtype == IC_BF16 || g.dtype == IC_F32);
}

size_t route_smem(const ic_graph_state& g) {
  const size_t C = g.n_clusters, cap = g.cluster_capacity;
  const size_t NS = g.sink_size + g.recent_size + C * cap;
  return C * GR_D * 4 + C * cap * 4 + NS * 8 + NS * 4 + 2 * C * 4 + C * 4 + GR_D * 4;
}

}  // namespace
}  // namespace ic

using namespace ic;

extern "C" int ic_graph_push(const ic_graph_push_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->T < 0 || !graph_state_ok(a->g) || !a->slot_src || (a->T > 0 && (!a->k_src || !a->v_src || !a->positions))) {
    set_last_error("graph_push: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  if (a->T == 0 && !a->reset) return IC_OK;
  const size_t smem = route_smem(a->g);
  if (smem > 200 * 1024) {
    set_last_error("graph_push: cache too large for the routing kernel's shared memory");
    return IC_ERR_UNSUPPORTED;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static PerDeviceLimit lim;
  if (const int rc = ensure_dynamic_smem(graph_route_kernel, static_cast<int>(smem), &lim)) return rc;
  graph_route_kernel<<<1, GR_THREADS, smem, st>>>(*a);
  if (const int rc = launch_status("graph_push (route)")) return rc;
  for (int phase = 0; phase < 2; ++phase) {
    if (a->g.dtype == IC_F32) graph_copy_kernel<float><<<296, 256, 0, st>>>(*a, phase);
    else if (a->g.dtype == IC_F16) graph_copy_kernel<__half><<<296, 256, 0, st>>>(*a, phase);
    else graph_copy_kernel<__nv_bfloat16><<<296, 256, 0, st>>>(*a, phase);
    if (const int rc = launch_status("graph_push (copy)")) return rc;
  }
  return IC_OK;
}

extern "C" int ic_graph_select(const ic_graph_select_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (!graph_state_ok(a->g) || !a->query || !a->selected || !a->slots || !a->count) {
    set_last_error("graph_select: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  graph_select_kernel<<<1, GR_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return launch_status("graph_select");
}
