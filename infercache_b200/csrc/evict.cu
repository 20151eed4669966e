// Kernel B and the per-session metadata kernels.
//
//  * evict_update  -- once per session-step: decayed importance + received
//    mass, promotion / eviction of the token leaving the recent ring with an
//    exact first-index argmin over L2, slot-table rotation so the staging row
//    (already holding the new token's K/V in every layer) becomes the ring
//    slot, ring advance, counters and an event record.
//  * sort_slots    -- occupied slots in (position, slot) order.
//  * boost_sorted  -- the reference push's mean attention weight, mapped from
//    position rank to slot.
//  * append_staging / reset_sessions.
//
// One CTA per session; importance arithmetic is float32 with every multiply
// and add rounded separately (no contraction), so the update is
// importance * decay, rounded, plus mass / div, rounded.
#include "common.cuh"

namespace ic {

constexpr int EV_THREADS = 512;

// Importance of slot j after this step's decay and received mass: the slot's
// mass is MH contiguous columns of ML layers; each column is summed in layer
// order, then the columns in head order (all loads of a batch issued before
// its adds), and importance = fl(fl(importance * decay) + fl(sum / div)).
__device__ __forceinline__ float updated_importance(const ic_evict_args& a, int s, int j, float v) {
  const int ntot = a.tiers.budget + 1;
  float add = 0.f;
  if (a.mass) {
    const int MH = a.mass_heads, ML = a.mass_layers;
    const float* base = a.mass + (static_cast<size_t>(s) * MH * ntot + j) * ML;
    const size_t hstride = static_cast<size_t>(ntot) * ML;
    float tot = 0.f, acc = 0.f;
    if ((ML & 3) == 0) {
      constexpr int NV = 20;  // float4 loads per batch
      const int per_h = ML / 4, nvec = MH * per_h;
      for (int v0 = 0; v0 < nvec; v0 += NV) {
        float4 x[NV];
#pragma unroll
        for (int u = 0; u < NV; ++u) {
          const int vi = v0 + u;
          x[u] = vi < nvec ? *reinterpret_cast<const float4*>(base + (vi / per_h) * hstride + (vi % per_h) * 4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < NV; ++u) {
          const int vi = v0 + u;
          if (vi >= nvec) break;
          const int hh = vi / per_h, l4 = vi % per_h;
          const float xs[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) acc = (l4 == 0 && q == 0) ? xs[q] : __fadd_rn(acc, xs[q]);
          if (l4 == per_h - 1) tot = hh == 0 ? acc : __fadd_rn(tot, acc);
        }
      }
    } else {
      for (int hh = 0; hh < MH; ++hh) {
        const float* m = base + hh * hstride;
        for (int l0 = 0; l0 < ML; l0 += 8) {
          float x[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) x[u] = l0 + u < ML ? m[l0 + u] : 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (l0 + u < ML) acc = (l0 + u == 0) ? x[u] : __fadd_rn(acc, x[u]);
        }
        tot = hh == 0 ? acc : __fadd_rn(tot, acc);
      }
    }
    add = __fdiv_rn(tot, a.mass_div);
  }
  return __fadd_rn(__fmul_rn(v, a.decay), add);
}

// Step one of kernel B spread over the grid: one thread per slot updates the
// importance of every occupied slot of every session.
constexpr int IU_THREADS = 128;

__global__ void __launch_bounds__(IU_THREADS) importance_update_kernel(const ic_evict_args a) {
  const int s = blockIdx.y, j = blockIdx.x * IU_THREADS + threadIdx.x;
  const int B = a.tiers.budget;
  grid_dependency_wait();  // the last layer's mass is complete
  grid_launch_dependents();
  if (j >= B) return;
  const size_t o = static_cast<size_t>(s) * B + j;
  if (a.sess.occupied[o]) a.sess.importance[o] = updated_importance(a, s, j, a.sess.importance[o]);
}

template <bool REDUCED>
__global__ void __launch_bounds__(EV_THREADS) evict_kernel(const ic_evict_args a) {
  // shared: positions [budget], importance [budget], slot table [budget + 1],
  // occupancy [budget]
  extern __shared__ __align__(16) unsigned char ev_smem[];
  __shared__ float red_v[EV_THREADS / 32];
  __shared__ int red_i[EV_THREADS / 32];
  __shared__ float red_r[EV_THREADS / 32];
  __shared__ int amin_slot;
  __shared__ float runner_up;

  const int s = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = a.tiers.budget, ntot = B + 1;
  int64_t* pos_s = reinterpret_cast<int64_t*>(ev_smem);
  float* imp_s = reinterpret_cast<float*>(pos_s + B);
  int32_t* stt_s = reinterpret_cast<int32_t*>(imp_s + B);
  const int sink = a.tiers.sink_size, recent = a.tiers.recent_size, cap = a.tiers.important_size;
  const int l2s = sink + recent;

  int32_t* ctrl = a.sess.ctrl + static_cast<size_t>(s) * IC_CTRL_WORDS;
  int64_t* cnt = a.sess.counters + static_cast<size_t>(s) * IC_COUNTER_WORDS;
  float* imp = a.sess.importance + static_cast<size_t>(s) * B;
  uint8_t* occ = a.sess.occupied + static_cast<size_t>(s) * B;
  int64_t* pos = a.sess.positions + static_cast<size_t>(s) * B;
  int32_t* stt = a.sess.slot_table + static_cast<size_t>(s) * ntot;

  uint8_t* occ_s = reinterpret_cast<uint8_t*>(stt_s + ntot);

  // Launched with programmatic dependent launch: the mass must be complete
  // before it is read, and the next step's first layer waits for us.  With
  // pdl == 2 the kernel before this one writes none of the session state read
  // here (kernel A writes only the mass, `out` and the staging rows), so that
  // state is staged first and only the mass waits.
  const bool stage_early = !REDUCED && a.pdl == 2;
  if (!stage_early) {
    grid_dependency_wait();
    grid_launch_dependents();
  }

  // 1. stage the slot table, positions, importance and occupancy, so the
  // decision below reads shared memory only
  for (int j = tid; j < ntot; j += EV_THREADS) stt_s[j] = stt[j];
  for (int j = tid; j < B; j += EV_THREADS) {
    pos_s[j] = pos[j];
    imp_s[j] = imp[j];
    occ_s[j] = occ[j];
  }
  // Snapshot the decision inputs: every thread must branch identically, and
  // thread 0 rewrites ctrl / occupied below.
  __shared__ int snap_r, snap_fill, snap_disp, snap_rf;
  __shared__ int64_t snap_cnt[IC_COUNTER_WORDS], snap_newpos;
  if (tid == 0) {
    snap_r = ctrl[IC_CTRL_RECENT_PTR];
    snap_fill = ctrl[IC_CTRL_IMPORTANT_FILL];
    snap_rf = ctrl[IC_CTRL_RECENT_FILL];
    snap_newpos = a.new_pos[s];
    for (int i = 0; i < IC_COUNTER_WORDS; ++i) snap_cnt[i] = cnt[i];
    const bool ok = snap_r >= sink && snap_r < l2s && snap_fill >= 0 && snap_fill <= cap;
    if (!ok) {
      if (a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
      snap_r = -1;
    } else {
      snap_disp = occ[snap_r] != 0;
    }
  }
  if (stage_early) {
    grid_dependency_wait();
    grid_launch_dependents();
  }
  // decay + boost of every occupied slot (already applied when REDUCED); each
  // thread updates the slots it staged
  if (!REDUCED) {
    constexpr int EV_MH = 8, EV_PER = 3;  // heads and slots per thread on the fast path
    if (a.mass && a.mass_layers == 1 && a.mass_heads <= EV_MH && B <= EV_PER * EV_THREADS) {
      // one mass column per head: every load of the thread's slots is issued
      // before any is used, then the same sums in head order as below
      const int MH = a.mass_heads;
      const float* base = a.mass + static_cast<size_t>(s) * MH * ntot;
      float mv[EV_PER][EV_MH];
#pragma unroll
      for (int i = 0; i < EV_PER; ++i) {
        const int j = tid + i * EV_THREADS;
        const bool on = j < B && occ_s[j];
#pragma unroll
        for (int hh = 0; hh < EV_MH; ++hh)
          mv[i][hh] = on && hh < MH ? base[static_cast<size_t>(hh) * ntot + j] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < EV_PER; ++i) {
        const int j = tid + i * EV_THREADS;
        if (j >= B || !occ_s[j]) continue;
        float tot = mv[i][0];
#pragma unroll
        for (int hh = 1; hh < EV_MH; ++hh)
          if (hh < MH) tot = __fadd_rn(tot, mv[i][hh]);
        const float v = __fadd_rn(__fmul_rn(imp_s[j], a.decay), __fdiv_rn(tot, a.mass_div));
        imp[j] = v;
        imp_s[j] = v;
      }
    } else {
      for (int j = tid; j < B; j += EV_THREADS) {
        if (!occ_s[j]) continue;
        const float v = updated_importance(a, s, j, imp_s[j]);
        imp[j] = v;
        imp_s[j] = v;
      }
    }
  }
  if (tid == 0 && a.advance_pos) a.new_pos[s] = snap_newpos + 1;  // the next step's position
  __syncthreads();
  if (snap_r < 0) return;  // corrupted ring state: reported, nothing written

  const int r = snap_r;
  const int l2fill = snap_fill;
  const bool displaced = snap_disp != 0;
  const float score = imp_s[r];
  const bool need_argmin = displaced && !(score <= 0.f) && l2fill >= cap && cap > 0;

  // 2. first-index argmin over the filled L2 slice, and the smallest other
  // score (the runner-up, to count decisions that rest on a near-tie), in one
  // pass and one block reduction
  if (need_argmin) {
    float bv = __int_as_float(0x7f800000);  // +inf
    int bi = 0x7fffffff;
    float sv = __int_as_float(0x7f800000);
    for (int j = l2s + tid; j < l2s + l2fill; j += EV_THREADS)
      argmin2_take(bv, bi, sv, imp_s[j], j, __int_as_float(0x7f800000));
    warp_argmin2(bv, bi, sv);
    if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; red_r[warp] = sv; }
    __syncthreads();
    if (warp == 0) {
      const bool has = lane < EV_THREADS / 32;
      bv = has ? red_v[lane] : __int_as_float(0x7f800000);
      bi = has ? red_i[lane] : 0x7fffffff;
      sv = has ? red_r[lane] : __int_as_float(0x7f800000);
      warp_argmin2(bv, bi, sv);
      if (lane == 0) {
        amin_slot = bi;
        runner_up = sv;
      }
    }
    __syncthreads();
  }

  // 3. apply the decision (one thread, from the staged copies)
  if (tid == 0) {
    int64_t kind = IC_EV_NONE, dpos = -1, target = -1, epos = -1;
    const int32_t row_r = stt_s[r], row_s = stt_s[B];
    int32_t new_stage = row_r;
    int64_t evictions = snap_cnt[IC_CNT_EVICTIONS], promotions = snap_cnt[IC_CNT_PROMOTIONS];
    int64_t near_ties = snap_cnt[IC_CNT_NEAR_TIES];
    if (displaced) {
      dpos = pos_s[r];
      int tgt = -1;
      if (score <= 0.f) {
        kind = IC_EV_DROP;
      } else if (l2fill < cap) {
        tgt = l2s + l2fill;
        ctrl[IC_CTRL_IMPORTANT_FILL] = l2fill + 1;
        kind = IC_EV_FILL;
      } else if (cap > 0) {
        target = amin_slot;
        const float lo = imp_s[amin_slot];
        if (l2fill > 1 && runner_up - lo <= 1e-6f * fabsf(lo)) near_ties += 1;
        if (score > imp_s[amin_slot]) {
          tgt = amin_slot;
          kind = IC_EV_EVICT;
          epos = pos_s[tgt];
          evictions += 1;
        } else {
          kind = IC_EV_REJECT;
        }
      } else {
        kind = IC_EV_REJECT;
      }
      if (tgt >= 0) {
        target = tgt;
        new_stage = stt_s[tgt];
        stt[tgt] = row_r;
        pos[tgt] = dpos;
        imp[tgt] = score;
        occ[tgt] = 1;
        promotions += 1;
      }
    }
    stt[r] = row_s;
    stt[B] = new_stage;
    pos[r] = snap_newpos;
    imp[r] = 0.f;
    occ[r] = 1;
    const int rf = snap_rf;
    ctrl[IC_CTRL_RECENT_FILL] = rf + 1 < recent ? rf + 1 : recent;
    ctrl[IC_CTRL_RECENT_PTR] = sink + (r - sink + 1) % recent;
    cnt[IC_CNT_TOKENS_SEEN] = snap_cnt[IC_CNT_TOKENS_SEEN] + 1;
    cnt[IC_CNT_STEPS] = snap_cnt[IC_CNT_STEPS] + 1;
    cnt[IC_CNT_EVICTIONS] = evictions;
    cnt[IC_CNT_PROMOTIONS] = promotions;
    cnt[IC_CNT_NEAR_TIES] = near_ties;
    if (a.events) {
      int64_t* e = a.events + static_cast<size_t>(s) * 4;
      e[0] = kind; e[1] = dpos; e[2] = target; e[3] = epos;
    }
  }
}

// ---------------------------------------------------------------------------
constexpr int SORT_THREADS = 1024;

__global__ void __launch_bounds__(SORT_THREADS) sort_slots_kernel(const ic_sort_args a) {
  extern __shared__ unsigned char sm[];
  const int s = blockIdx.x, B = a.tiers.budget;
  int64_t* ps = reinterpret_cast<int64_t*>(sm);
  uint8_t* os = sm + static_cast<size_t>(B) * 8;
  __shared__ int fill_s;
  const int64_t* pos = a.sess.positions + static_cast<size_t>(s) * B;
  const uint8_t* occ = a.sess.occupied + static_cast<size_t>(s) * B;
  int32_t* out = a.sorted_slots + static_cast<size_t>(s) * B;
  if (threadIdx.x == 0) fill_s = 0;
  for (int j = threadIdx.x; j < B; j += SORT_THREADS) {
    ps[j] = pos[j];
    os[j] = occ[j];
    out[j] = -1;
  }
  __syncthreads();
  int local = 0;
  for (int j = threadIdx.x; j < B; j += SORT_THREADS) {
    if (!os[j]) continue;
    ++local;
    const int64_t pj = ps[j];
    int rank = 0;
    for (int i = 0; i < B; ++i) rank += os[i] && (ps[i] < pj || (ps[i] == pj && i < j));
    out[rank] = j;
  }
  atomicAdd(&fill_s, local);  // integer count: order-independent
  __syncthreads();
  if (threadIdx.x == 0) a.fill[s] = fill_s;
}

__global__ void boost_sorted_kernel(const ic_boost_args a) {
  const int s = blockIdx.x, B = a.tiers.budget, ntot = B + 1;
  float* mo = a.mass_out + static_cast<size_t>(s) * ntot;
  for (int j = threadIdx.x; j < ntot; j += blockDim.x) mo[j] = 0.f;
  __syncthreads();
  const int fill = a.fill[s];
  const int n = a.width < fill ? a.width : fill;
  const size_t per_sess = static_cast<size_t>(a.L) * a.H * a.Q * a.width;
  const float* w = a.weights + s * per_sess;
  const float cnt = static_cast<float>(a.L * a.H * a.Q);
  for (int rk = threadIdx.x; rk < n; rk += blockDim.x) {
    float total = 0.f;
    for (int hh = 0; hh < a.H; ++hh) {
      float acc = 0.f;
      bool first = true;
      for (int l = 0; l < a.L; ++l)
        for (int q = 0; q < a.Q; ++q) {
          const float x = w[((static_cast<size_t>(l) * a.H + hh) * a.Q + q) * a.width + rk];
          acc = first ? x : __fadd_rn(acc, x);
          first = false;
        }
      total = hh == 0 ? acc : __fadd_rn(total, acc);
    }
    const int slot = a.sorted_slots[static_cast<size_t>(s) * B + rk];
    if (slot >= 0) mo[slot] = __fdiv_rn(total, cnt);
  }
}

template <typename T>
__global__ void append_staging_kernel(const ic_append_args a) {
  const int l = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int D = a.pool.head_dim, B = a.tiers.budget;
  const int row = a.sess.slot_table[static_cast<size_t>(s) * (B + 1) + B];
  if (row < 0 || row >= a.pool.pool_tokens) {
    if (threadIdx.x == 0 && a.sess.dev_status) atomicOr(a.sess.dev_status, IC_DEVFLAG_BAD_ROW);
    return;
  }
  const size_t dst = ((static_cast<size_t>(l) * a.pool.num_kv_heads + h) * a.pool.pool_tokens + row) * D;
  const size_t src = s * a.stride_s + l * a.stride_l + h * a.stride_h;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    static_cast<T*>(a.pool.k)[dst + d] = static_cast<const T*>(a.k)[src + d];
    static_cast<T*>(a.pool.v)[dst + d] = static_cast<const T*>(a.v)[src + d];
  }
}

__global__ void reset_meta_kernel(const ic_reset_args a) {
  const int s = a.session0 + blockIdx.x, B = a.tiers.budget;
  for (int j = threadIdx.x; j < B; j += blockDim.x) {
    a.sess.positions[static_cast<size_t>(s) * B + j] = -1;
    a.sess.importance[static_cast<size_t>(s) * B + j] = 0.f;
    a.sess.occupied[static_cast<size_t>(s) * B + j] = 0;
  }
  if (threadIdx.x < IC_CTRL_WORDS)
    a.sess.ctrl[static_cast<size_t>(s) * IC_CTRL_WORDS + threadIdx.x] =
        threadIdx.x == IC_CTRL_RECENT_PTR ? a.tiers.sink_size : 0;
  if (threadIdx.x < IC_COUNTER_WORDS) a.sess.counters[static_cast<size_t>(s) * IC_COUNTER_WORDS + threadIdx.x] = 0;
}

template <typename T>
__global__ void reset_kv_kernel(const ic_reset_args a) {
  const int s = a.session0 + blockIdx.z;
  const int lh = blockIdx.y;  // layer * Hkv + head
  const int ntot = a.tiers.budget + 1, D = a.pool.head_dim;
  const int32_t* stt = a.sess.slot_table + static_cast<size_t>(s) * ntot;
  for (int j = blockIdx.x; j < ntot; j += gridDim.x) {
    const int row = stt[j];
    if (row < 0 || row >= a.pool.pool_tokens) continue;
    const size_t base = (static_cast<size_t>(lh) * a.pool.pool_tokens + row) * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      static_cast<T*>(a.pool.k)[base + d] = T(0.f);
      static_cast<T*>(a.pool.v)[base + d] = T(0.f);
    }
  }
}

static bool tiers_ok(const ic_tiers& t) {
  return t.sink_size >= 0 && t.recent_size >= 1 && t.important_size >= 0 &&
         t.budget == t.sink_size + t.recent_size + t.important_size && t.budget > 0;
}

}  // namespace ic

using namespace ic;

extern "C" int ic_evict_update(const ic_evict_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->sess.num_sessions == 0) return IC_OK;
  if (!tiers_ok(a->tiers) || a->sess.num_sessions < 0 || !a->new_pos || !a->sess.slot_table ||
      !a->sess.positions || !a->sess.importance || !a->sess.occupied || !a->sess.ctrl ||
      !a->sess.counters || (a->mass && (a->mass_heads < 1 || a->mass_layers < 1 || !(a->mass_div > 0.f))) ||
      a->pdl < 0 || a->pdl > 2) {
    set_last_error("evict_update: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  const size_t smem = static_cast<size_t>(a->tiers.budget) * (sizeof(int64_t) + sizeof(float) + 1) +
                     static_cast<size_t>(a->tiers.budget + 1) * sizeof(int32_t);
  if (smem > 200 * 1024) { set_last_error("evict_update: budget too large"); return IC_ERR_UNSUPPORTED; }
  // With many mass columns to sum, the per-slot update runs as its own wide
  // kernel first (the columns are then the bulk of kernel B's reads); the
  // per-session decision kernel starts from the updated importance.
  const bool split = a->mass != nullptr && a->mass_layers >= 8;
  static PerDeviceLimit smem_limit_r, smem_limit_f;
  int rc = split ? ensure_dynamic_smem(evict_kernel<true>, static_cast<int>(smem), &smem_limit_r)
                 : ensure_dynamic_smem(evict_kernel<false>, static_cast<int>(smem), &smem_limit_f);
  if (rc) return rc;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a->pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (split) {
    cfg.gridDim = dim3((a->tiers.budget + IU_THREADS - 1) / IU_THREADS, a->sess.num_sessions, 1);
    cfg.blockDim = dim3(IU_THREADS, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cudaLaunchKernelEx(&cfg, importance_update_kernel, *a);
    if ((rc = launch_status("evict_update (importance)")) != IC_OK) return rc;
  }
  cfg.gridDim = dim3(a->sess.num_sessions, 1, 1);
  cfg.blockDim = dim3(EV_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  if (split)
    cudaLaunchKernelEx(&cfg, evict_kernel<true>, *a);
  else
    cudaLaunchKernelEx(&cfg, evict_kernel<false>, *a);
  return launch_status("evict_update");
}

extern "C" int ic_sort_slots(const ic_sort_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->sess.num_sessions == 0) return IC_OK;
  if (!tiers_ok(a->tiers) || !a->sorted_slots || !a->fill || !a->sess.positions || !a->sess.occupied) {
    set_last_error("sort_slots: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  const size_t smem = static_cast<size_t>(a->tiers.budget) * 9;
  if (smem > 200 * 1024) { set_last_error("sort_slots: budget too large"); return IC_ERR_UNSUPPORTED; }
  static PerDeviceLimit smem_limit;
  if (const int rc = ensure_dynamic_smem(sort_slots_kernel, static_cast<int>(smem), &smem_limit)) return rc;
  sort_slots_kernel<<<a->sess.num_sessions, SORT_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(*a);
  return launch_status("sort_slots");
}

extern "C" int ic_boost_sorted(const ic_boost_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->num_sessions == 0) return IC_OK;
  if (!tiers_ok(a->tiers) || !a->weights || !a->sorted_slots || !a->fill || !a->mass_out || a->L < 1 ||
      a->H < 1 || a->Q < 1 || a->width < 0) {
    set_last_error("boost_sorted: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  boost_sorted_kernel<<<a->num_sessions, 256, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return launch_status("boost_sorted");
}

extern "C" int ic_append_staging(const ic_append_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->sess.num_sessions == 0) return IC_OK;
  if (!tiers_ok(a->tiers) || !a->k || !a->v || !a->pool.k || !a->pool.v || !a->sess.slot_table ||
      a->pool.head_dim <= 0) {
    set_last_error("append_staging: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  dim3 grid(a->pool.num_layers, a->pool.num_kv_heads, a->sess.num_sessions);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->pool.dtype) {
    case IC_F32: append_staging_kernel<float><<<grid, 128, 0, st>>>(*a); break;
    case IC_F16: append_staging_kernel<__half><<<grid, 128, 0, st>>>(*a); break;
    case IC_BF16: append_staging_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(*a); break;
    default: set_last_error("append_staging: bad dtype"); return IC_ERR_INVALID_ARG;
  }
  return launch_status("append_staging");
}

extern "C" int ic_reset_sessions(const ic_reset_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->n == 0) return IC_OK;
  if (!tiers_ok(a->tiers) || a->n < 0 || a->session0 < 0 || a->session0 + a->n > a->sess.num_sessions ||
      !a->sess.positions || !a->sess.importance || !a->sess.occupied || !a->sess.ctrl || !a->sess.counters) {
    set_last_error("reset_sessions: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  reset_meta_kernel<<<a->n, 256, 0, st>>>(*a);
  int rc = launch_status("reset_sessions");
  if (rc != IC_OK || !a->zero_kv) return rc;
  if (!a->pool.k || !a->pool.v || !a->sess.slot_table) return IC_ERR_INVALID_ARG;
  dim3 grid(64, a->pool.num_layers * a->pool.num_kv_heads, a->n);
  switch (a->pool.dtype) {
    case IC_F32: reset_kv_kernel<float><<<grid, 128, 0, st>>>(*a); break;
    case IC_F16: reset_kv_kernel<__half><<<grid, 128, 0, st>>>(*a); break;
    case IC_BF16: reset_kv_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(*a); break;
    default: return IC_ERR_INVALID_ARG;
  }
  return launch_status("reset_sessions");
}
