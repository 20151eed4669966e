// Kernel D: tier fill of a prompt (load_from_hf_output) and the K/V copy of
// the chosen tokens into the pool.
//
// The reference walks the prompt token by token (hierarchical_cache.py:209-235):
// the first sink_size tokens whose position is < sink_size become sinks; the
// last recent_size tokens (minus those) fill the ring in order; every other
// token fills L2 in order and, once L2 is full, replaces the first-index
// minimum of L2 iff its score is strictly greater.  The final slot of a token
// depends on that whole replacement history, so it is replayed exactly.
//
// One warp per session walks the prompt 32 tokens at a time: ballots give the
// sink / ring ranks in one step, and L2 candidates that cannot beat the
// current minimum are rejected by one ballot.  Each lane owns the L2 slots
// j = lane (mod 32) and caches their minimum; a replacement rescans only the
// owner's slots and re-reduces the 32 lane minima.
#include "common.cuh"

namespace ic {

__global__ void __launch_bounds__(32) tier_fill_kernel(const ic_tier_fill_args a) {
  extern __shared__ unsigned char sm[];
  const int cap = a.tiers.important_size;
  float* vals = reinterpret_cast<float*>(sm);               // [cap]
  int32_t* toks = reinterpret_cast<int32_t*>(sm + static_cast<size_t>(cap) * 4);  // [cap]

  const int i = blockIdx.x;                 // prompt index
  const int s = a.session0 + i;             // session row
  const int lane = threadIdx.x;
  const int B = a.tiers.budget, T = a.T;
  const int sink = a.tiers.sink_size, recent = a.tiers.recent_size;
  const int l2s = sink + recent;
  const float* sc = a.scores + static_cast<size_t>(i) * T;
  const int64_t* pp = a.positions ? a.positions + static_cast<size_t>(i) * T : nullptr;
  int32_t* stok = a.slot_token + static_cast<size_t>(i) * B;
  int64_t* pos = a.sess.positions + static_cast<size_t>(s) * B;
  float* imp = a.sess.importance + static_cast<size_t>(s) * B;
  uint8_t* occ = a.sess.occupied + static_cast<size_t>(s) * B;

  for (int j = lane; j < B; j += 32) {
    stok[j] = -1;
    pos[j] = -1;
    imp[j] = 0.f;
    occ[j] = 0;
  }
  __syncwarp();

  int sink_seen = 0;   // tokens with position < sink seen so far
  int recent_fill = 0;
  int l2fill = 0;
  long long evictions = 0;
  float lmin = __int_as_float(0x7f800000);  // this lane's minimum over its L2 slots
  int lidx = 0x7fffffff;
  float gmin = lmin;
  int gidx = lidx;
  const unsigned lt_mask = (1u << lane) - 1u;

  for (int base = 0; base < T; base += 32) {
    const int tok = base + lane;
    const bool valid = tok < T;
    const long long p = valid ? (pp ? pp[tok] : tok) : 0;
    const float x = valid ? sc[tok] : 0.f;

    // sinks: the first `sink` tokens with position < sink
    const bool sc_c = valid && p < sink;
    const unsigned bs = __ballot_sync(FULL_MASK, sc_c);
    const int srank = sink_seen + __popc(bs & lt_mask);
    const bool is_sink = sc_c && srank < sink;
    if (is_sink) {
      stok[srank] = tok; pos[srank] = p; imp[srank] = x; occ[srank] = 1;
    }
    sink_seen += __popc(bs);

    // recent tail: the last `recent` tokens that are not sinks
    const bool tail = valid && !is_sink && (T - tok) <= recent;
    const unsigned bt = __ballot_sync(FULL_MASK, tail);
    if (tail) {
      const int rr = recent_fill + __popc(bt & lt_mask);
      if (rr < recent) {
        const int slot = sink + rr;
        stok[slot] = tok; pos[slot] = p; imp[slot] = x; occ[slot] = 1;
      }
    }
    recent_fill = min(recent, recent_fill + __popc(bt));

    // L2 candidates, in token order
    const bool cand = valid && !is_sink && (T - tok) > recent;
    unsigned bc = __ballot_sync(FULL_MASK, cand);
    if (bc == 0u || cap == 0) continue;
    // fill phase: candidates take the free L2 slots in order
    const int room = cap - l2fill;
    if (room > 0) {
      const int crank = __popc(bc & lt_mask);
      if (cand && crank < room) {
        vals[l2fill + crank] = x;
        toks[l2fill + crank] = tok;
      }
      const int placed = min(room, __popc(bc));
      // drop the placed candidates (the lowest `placed` set bits)
      for (int k = 0; k < placed; ++k) bc &= bc - 1u;
      l2fill += placed;
      __syncwarp();
      if (l2fill == cap) {
        // L2 just became full: per-lane minima, then the warp minimum
        for (int j = lane; j < cap; j += 32)
          if (argmin_less(vals[j], j, lmin, lidx)) { lmin = vals[j]; lidx = j; }
        gmin = lmin; gidx = lidx;
        warp_argmin(gmin, gidx);
      }
      if (l2fill < cap) continue;
    }
    // replacement phase: candidates strictly greater than the current minimum
    unsigned live = bc & __ballot_sync(FULL_MASK, cand && x > gmin);
    while (live) {
      const int src = __ffs(live) - 1;
      const float xs = __shfl_sync(FULL_MASK, x, src);
      const int ts = __shfl_sync(FULL_MASK, tok, src);
      const int e = gidx;  // L2-local index of the first-index minimum
      if (lane == (e & 31)) {
        vals[e] = xs;
        toks[e] = ts;
        lmin = __int_as_float(0x7f800000);
        lidx = 0x7fffffff;
        for (int j = lane; j < cap; j += 32)
          if (argmin_less(vals[j], j, lmin, lidx)) { lmin = vals[j]; lidx = j; }
      }
      ++evictions;
      __syncwarp();
      gmin = lmin; gidx = lidx;
      warp_argmin(gmin, gidx);
      // the minimum only grows, so candidates that failed stay failed
      const unsigned later = src >= 31 ? 0u : (~0u << (src + 1));
      live = later & bc & __ballot_sync(FULL_MASK, cand && x > gmin);
    }
  }
  __syncwarp();
  for (int j = lane; j < l2fill; j += 32) {
    const int slot = l2s + j;
    const int tk = toks[j];
    stok[slot] = tk;
    pos[slot] = pp ? pp[tk] : tk;
    imp[slot] = vals[j];
    occ[slot] = 1;
  }
  if (lane == 0) {
    int32_t* ctrl = a.sess.ctrl + static_cast<size_t>(s) * IC_CTRL_WORDS;
    for (int w = 0; w < IC_CTRL_WORDS; ++w) ctrl[w] = 0;
    ctrl[IC_CTRL_SINK_FILL] = min(sink_seen, sink);
    ctrl[IC_CTRL_RECENT_FILL] = recent_fill;
    ctrl[IC_CTRL_RECENT_PTR] = sink;
    ctrl[IC_CTRL_IMPORTANT_FILL] = l2fill;
    int64_t* cnt = a.sess.counters + static_cast<size_t>(s) * IC_COUNTER_WORDS;
    for (int w = 0; w < IC_COUNTER_WORDS; ++w) cnt[w] = 0;
    cnt[IC_CNT_TOKENS_SEEN] = T;
    cnt[IC_CNT_EVICTIONS] = evictions;
  }
}

template <typename TD, typename TS>
__global__ void load_layer_kernel(const ic_load_layer_args a) {
  const int B = a.tiers.budget, ntot = B + 1, D = a.pool.head_dim;
  const int h = blockIdx.y;
  const int32_t* stt = a.sess.slot_table + static_cast<size_t>(a.session) * ntot;
  const size_t plane = static_cast<size_t>(a.pool.pool_tokens) * D;
  const size_t lh = static_cast<size_t>(a.layer) * a.pool.num_kv_heads + h;
  TD* dk = static_cast<TD*>(a.pool.k) + lh * plane;
  TD* dv = static_cast<TD*>(a.pool.v) + lh * plane;
  const TS* sk = static_cast<const TS*>(a.k_src) + h * a.stride_h;
  const TS* sv = static_cast<const TS*>(a.v_src) + h * a.stride_h;
  for (int j = blockIdx.x; j < B; j += gridDim.x) {
    const int tok = a.slot_token[j];
    if (tok < 0 || tok >= a.T) continue;
    const int row = stt[j];
    if (row < 0 || row >= a.pool.pool_tokens) continue;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      dk[static_cast<size_t>(row) * D + d] = DT<TD>::from_f(DT<TS>::to_f(sk[tok * a.stride_t + d]));
      dv[static_cast<size_t>(row) * D + d] = DT<TD>::from_f(DT<TS>::to_f(sv[tok * a.stride_t + d]));
    }
  }
}

template <typename TD>
static int launch_load(const ic_load_layer_args& a, cudaStream_t st) {
  dim3 grid(min(a.tiers.budget, 1024), a.pool.num_kv_heads);
  switch (a.src_dtype) {
    case IC_F32: load_layer_kernel<TD, float><<<grid, 128, 0, st>>>(a); break;
    case IC_F16: load_layer_kernel<TD, __half><<<grid, 128, 0, st>>>(a); break;
    case IC_BF16: load_layer_kernel<TD, __nv_bfloat16><<<grid, 128, 0, st>>>(a); break;
    default: set_last_error("load_layer: bad src dtype"); return IC_ERR_INVALID_ARG;
  }
  return launch_status("load_layer");
}

}  // namespace ic

using namespace ic;

extern "C" int ic_tier_fill(const ic_tier_fill_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->n == 0) return IC_OK;
  const ic_tiers& t = a->tiers;
  if (t.budget != t.sink_size + t.recent_size + t.important_size || t.recent_size < 1 || t.sink_size < 0 ||
      t.important_size < 0 || a->T < 0 || a->n < 0 || a->session0 < 0 ||
      a->session0 + a->n > a->sess.num_sessions || !a->scores || !a->slot_token || !a->sess.positions ||
      !a->sess.importance || !a->sess.occupied || !a->sess.ctrl || !a->sess.counters) {
    set_last_error("tier_fill: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  const size_t smem = static_cast<size_t>(t.important_size) * 8;
  if (smem > 200 * 1024) { set_last_error("tier_fill: important_size too large"); return IC_ERR_UNSUPPORTED; }
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(tier_fill_kernel, static_cast<int>(smem), &smem_limit)) return rc;
  tier_fill_kernel<<<a->n, 32, smem, static_cast<cudaStream_t>(stream)>>>(*a);
  return launch_status("tier_fill");
}

extern "C" int ic_load_layer(const ic_load_layer_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (!a->pool.k || !a->pool.v || !a->k_src || !a->v_src || !a->slot_token || !a->sess.slot_table ||
      a->layer < 0 || a->layer >= a->pool.num_layers || a->session < 0 ||
      a->session >= a->sess.num_sessions || a->T < 0) {
    set_last_error("load_layer: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  if (a->T == 0) return IC_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->pool.dtype) {
    case IC_F32: return launch_load<float>(*a, st);
    case IC_F16: return launch_load<__half>(*a, st);
    case IC_BF16: return launch_load<__nv_bfloat16>(*a, st);
    default: set_last_error("load_layer: bad pool dtype"); return IC_ERR_INVALID_ARG;
  }
}
