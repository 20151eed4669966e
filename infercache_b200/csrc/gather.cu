// Row gathers and writes over the page pool.
//
//  * gather_slots: pool rows of chosen logical slots of one session (through
//    the slot table) into a dense [L', Hkv, n, D] tensor -- the position-ordered
//    export of to_hf_past_key_values and the gather_cache_kv op.
//  * page_gather / page_write: PagedSessionView rows addressed by a page list
//    (token t lives in row page_ids[t / 16] * 16 + t % 16).
//
// These are HBM-bound copies: one CTA moves whole 16-byte vectors of full rows
// (head_dim * dtype bytes, a multiple of 16 for the supported shapes), rows
// spread over the grid's x dimension.
#include "common.cuh"

namespace ic {

constexpr int PAGE = 16;

__device__ __forceinline__ int64_t page_row(const int32_t* page_ids, int64_t t) {
  return static_cast<int64_t>(page_ids[t / PAGE]) * PAGE + t % PAGE;
}

// Copies `vecs` 16-byte vectors per row.
__global__ void gather_slots_kernel(const ic_gather_args a, int vecs) {
  const int h = blockIdx.y;
  const int l = a.layer_begin + blockIdx.z;
  const int B = a.tiers.budget, ntot = B + 1, Hkv = a.pool.num_kv_heads;
  const int esz = a.pool.dtype == IC_F32 ? 4 : 2;
  const size_t row_bytes = static_cast<size_t>(a.pool.head_dim) * esz;
  const int32_t* stt = a.sess.slot_table + static_cast<size_t>(a.session) * ntot;
  const size_t plane_rows = static_cast<size_t>(a.pool.pool_tokens);
  const char* srck = static_cast<const char*>(a.pool.k) + (static_cast<size_t>(l) * Hkv + h) * plane_rows * row_bytes;
  const char* srcv = static_cast<const char*>(a.pool.v) + (static_cast<size_t>(l) * Hkv + h) * plane_rows * row_bytes;
  char* dk = static_cast<char*>(a.k_out) + (static_cast<size_t>(blockIdx.z) * Hkv + h) * a.n * row_bytes;
  char* dv = static_cast<char*>(a.v_out) + (static_cast<size_t>(blockIdx.z) * Hkv + h) * a.n * row_bytes;
  const int per_block = blockDim.x / vecs;  // rows handled per block iteration
  const int vi = threadIdx.x % vecs, ri = threadIdx.x / vecs;
  if (ri >= per_block) return;
  for (int r = blockIdx.x * per_block + ri; r < a.n; r += gridDim.x * per_block) {
    const int slot = a.slots[r];
    int4 kv = make_int4(0, 0, 0, 0), vv = make_int4(0, 0, 0, 0);
    if (slot >= 0 && slot < ntot) {
      const int row = stt[slot];
      if (row >= 0 && row < a.pool.pool_tokens) {
        kv = reinterpret_cast<const int4*>(srck + row * row_bytes)[vi];
        vv = reinterpret_cast<const int4*>(srcv + row * row_bytes)[vi];
      }
    }
    reinterpret_cast<int4*>(dk + r * row_bytes)[vi] = kv;
    reinterpret_cast<int4*>(dv + r * row_bytes)[vi] = vv;
  }
}

template <bool WRITE>
__global__ void page_rows_kernel(const ic_page_rows_args a, int vecs) {
  const int h = blockIdx.y;
  const int lz = blockIdx.z;
  const int l = a.layer_begin + lz;
  const int H = a.pool.num_kv_heads;
  const int esz = a.pool.dtype == IC_F32 ? 4 : 2;
  const size_t row_bytes = static_cast<size_t>(a.pool.head_dim) * esz;
  char* poolk = static_cast<char*>(a.pool.k) + (static_cast<size_t>(l) * H + h) * a.pool.pool_tokens * row_bytes;
  char* poolv = static_cast<char*>(a.pool.v) + (static_cast<size_t>(l) * H + h) * a.pool.pool_tokens * row_bytes;
  const int per_block = blockDim.x / vecs;
  const int vi = threadIdx.x % vecs, ri = threadIdx.x / vecs;
  if (ri >= per_block) return;
  const int64_t lim = static_cast<int64_t>(a.n_page_ids) * PAGE;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * per_block + ri; t < a.n_tokens;
       t += static_cast<int64_t>(gridDim.x) * per_block) {
    const int64_t lt = a.start_token + t;  // token index within the session
    if (lt >= lim) continue;
    const int64_t row = page_row(a.page_ids, lt);
    if (row < 0 || row >= a.pool.pool_tokens) continue;
    // buffer element offset of (lz, h, t)
    const int64_t bo = (lz * a.stride_l + h * a.stride_h + t * a.stride_t) * esz;
    int4* pk = reinterpret_cast<int4*>(poolk + row * row_bytes) + vi;
    int4* pv = reinterpret_cast<int4*>(poolv + row * row_bytes) + vi;
    int4* bk = reinterpret_cast<int4*>(static_cast<char*>(a.k_buf) + bo) + vi;
    int4* bv = reinterpret_cast<int4*>(static_cast<char*>(a.v_buf) + bo) + vi;
    if (WRITE) { *pk = *bk; *pv = *bv; } else { *bk = *pk; *bv = *pv; }
  }
}

// Many page lists in one launch: the descriptors travel as the kernel's
// parameter block (read in place through __grid_constant__); block x of the
// grid belongs to descriptor i when blk_off[i] <= x < blk_off[i + 1].
struct PageDesc {
  const int32_t* page_ids;
  char* k_buf;
  char* v_buf;
  int64_t n_page_ids, start_token, n_tokens;
  int64_t stride_l, stride_h, stride_t;
};

struct PageBatch {
  ic_pool pool;
  int32_t layer_begin, count;
  int32_t blk_off[IC_PAGE_BATCH_MAX + 1];
  PageDesc d[IC_PAGE_BATCH_MAX];
};

template <bool WRITE>
__global__ void page_rows_batch_kernel(const __grid_constant__ PageBatch b, int vecs) {
  const int bx = blockIdx.x;
  int i = 0;
  while (i + 1 < b.count && b.blk_off[i + 1] <= bx) ++i;
  const PageDesc& d = b.d[i];
  const int h = blockIdx.y;
  const int lz = blockIdx.z;
  const int l = b.layer_begin + lz;
  const int H = b.pool.num_kv_heads;
  const int esz = b.pool.dtype == IC_F32 ? 4 : 2;
  const size_t row_bytes = static_cast<size_t>(b.pool.head_dim) * esz;
  char* poolk = static_cast<char*>(b.pool.k) + (static_cast<size_t>(l) * H + h) * b.pool.pool_tokens * row_bytes;
  char* poolv = static_cast<char*>(b.pool.v) + (static_cast<size_t>(l) * H + h) * b.pool.pool_tokens * row_bytes;
  const int per_block = blockDim.x / vecs;
  const int vi = threadIdx.x % vecs, ri = threadIdx.x / vecs;
  if (ri >= per_block) return;
  const int64_t t = static_cast<int64_t>(bx - b.blk_off[i]) * per_block + ri;
  if (t >= d.n_tokens) return;
  const int64_t lt = d.start_token + t;
  if (lt >= d.n_page_ids * PAGE) return;
  const int64_t row = page_row(d.page_ids, lt);
  if (row < 0 || row >= b.pool.pool_tokens) return;
  const int64_t bo = (lz * d.stride_l + h * d.stride_h + t * d.stride_t) * esz;
  int4* pk = reinterpret_cast<int4*>(poolk + row * row_bytes) + vi;
  int4* pv = reinterpret_cast<int4*>(poolv + row * row_bytes) + vi;
  int4* bk = reinterpret_cast<int4*>(d.k_buf + bo) + vi;
  int4* bv = reinterpret_cast<int4*>(d.v_buf + bo) + vi;
  if (WRITE) { *pk = *bk; *pv = *bv; } else { *bk = *pk; *bv = *pv; }
}

static bool same_pool(const ic_pool& x, const ic_pool& y) {
  return x.k == y.k && x.v == y.v && x.pool_tokens == y.pool_tokens && x.num_layers == y.num_layers &&
         x.num_kv_heads == y.num_kv_heads && x.head_dim == y.head_dim && x.dtype == y.dtype;
}

static int row_vecs(const ic_pool& p) {
  const int esz = p.dtype == IC_F32 ? 4 : 2;
  const int bytes = p.head_dim * esz;
  if (bytes % 16 != 0 || bytes > 16 * 256) return -1;
  return bytes / 16;
}

}  // namespace ic

using namespace ic;

extern "C" int ic_gather_slots(const ic_gather_args* a, void* stream) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->n == 0 || a->layer_end == a->layer_begin) return IC_OK;
  const int vecs = row_vecs(a->pool);
  if (vecs < 0) { set_last_error("gather_slots: row size must be a multiple of 16 bytes"); return IC_ERR_UNSUPPORTED; }
  if (a->n < 0 || !a->slots || !a->k_out || !a->v_out || !a->pool.k || !a->pool.v || !a->sess.slot_table ||
      a->session < 0 || a->session >= a->sess.num_sessions || a->layer_begin < 0 ||
      a->layer_end > a->pool.num_layers || a->layer_begin > a->layer_end) {
    set_last_error("gather_slots: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  const int threads = 256;
  const int per_block = threads / vecs;
  dim3 grid(min((a->n + per_block - 1) / per_block, 4096), a->pool.num_kv_heads, a->layer_end - a->layer_begin);
  gather_slots_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(*a, vecs);
  return launch_status("gather_slots");
}

// Argument checks shared by the single and batched forms (a non-empty token
// range and layer range).
static bool page_rows_ok(const ic_page_rows_args* a) {
  const int esz = a->pool.dtype == IC_F32 ? 4 : 2;
  const bool aligned = ((a->stride_l * esz) % 16 == 0) && ((a->stride_h * esz) % 16 == 0) &&
                       ((a->stride_t * esz) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a->k_buf) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(a->v_buf) % 16 == 0);
  return !(a->n_tokens < 0 || !a->page_ids || !a->k_buf || !a->v_buf || !a->pool.k || !a->pool.v || !aligned ||
           a->layer_begin < 0 || a->layer_end > a->pool.num_layers || a->layer_begin > a->layer_end ||
           a->start_token < 0 || a->start_token + a->n_tokens > static_cast<int64_t>(a->n_page_ids) * PAGE);
}

static int page_rows(const ic_page_rows_args* a, void* stream, bool write) {
  if (!a) return IC_ERR_INVALID_ARG;
  if (a->n_tokens == 0 || a->layer_end == a->layer_begin) return IC_OK;
  const int vecs = row_vecs(a->pool);
  if (vecs < 0) { set_last_error("page rows: row size must be a multiple of 16 bytes"); return IC_ERR_UNSUPPORTED; }
  if (!page_rows_ok(a)) {
    set_last_error("page rows: bad arguments");
    return IC_ERR_INVALID_ARG;
  }
  const int threads = 256;
  const int per_block = threads / vecs;
  const int64_t blocks = (a->n_tokens + per_block - 1) / per_block;
  dim3 grid(static_cast<unsigned>(blocks < 4096 ? blocks : 4096), a->pool.num_kv_heads, a->layer_end - a->layer_begin);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (write)
    page_rows_kernel<true><<<grid, threads, 0, st>>>(*a, vecs);
  else
    page_rows_kernel<false><<<grid, threads, 0, st>>>(*a, vecs);
  return launch_status(write ? "page_write" : "page_gather");
}

static int page_rows_batch(const ic_page_rows_args* a, int32_t count, void* stream, bool write) {
  if (!a || count < 1 || count > IC_PAGE_BATCH_MAX) {
    set_last_error("page rows (batch): 1 <= count <= IC_PAGE_BATCH_MAX descriptors");
    return IC_ERR_INVALID_ARG;
  }
  const int vecs = row_vecs(a[0].pool);
  if (vecs < 0) { set_last_error("page rows: row size must be a multiple of 16 bytes"); return IC_ERR_UNSUPPORTED; }
  PageBatch b = {};
  b.pool = a[0].pool;
  b.layer_begin = a[0].layer_begin;
  b.count = count;
  const int per_block = 256 / vecs;
  int64_t blocks = 0;
  for (int i = 0; i < count; ++i) {
    const ic_page_rows_args& x = a[i];
    if (!same_pool(x.pool, a[0].pool) || x.layer_begin != a[0].layer_begin || x.layer_end != a[0].layer_end ||
        (x.n_tokens != 0 && !page_rows_ok(&x)) || x.n_tokens < 0) {
      set_last_error("page rows (batch): bad arguments, or descriptors on different pools or layer ranges");
      return IC_ERR_INVALID_ARG;
    }
    b.blk_off[i] = static_cast<int32_t>(blocks);
    b.d[i] = PageDesc{x.page_ids, static_cast<char*>(x.k_buf), static_cast<char*>(x.v_buf), x.n_page_ids,
                      x.start_token, x.n_tokens, x.stride_l, x.stride_h, x.stride_t};
    blocks += (x.n_tokens + per_block - 1) / per_block;
    if (blocks > 0x7fffffff) {
      set_last_error("page rows (batch): too many tokens for one launch");
      return IC_ERR_UNSUPPORTED;
    }
  }
  b.blk_off[count] = static_cast<int32_t>(blocks);
  const int layers = a[0].layer_end - a[0].layer_begin;
  if (blocks == 0 || layers == 0) return IC_OK;
  if (a[0].layer_begin < 0 || a[0].layer_end > a[0].pool.num_layers || layers < 0) {
    set_last_error("page rows (batch): bad layer range");
    return IC_ERR_INVALID_ARG;
  }
  dim3 grid(static_cast<unsigned>(blocks), a[0].pool.num_kv_heads, layers);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (write)
    page_rows_batch_kernel<true><<<grid, 256, 0, st>>>(b, vecs);
  else
    page_rows_batch_kernel<false><<<grid, 256, 0, st>>>(b, vecs);
  return launch_status(write ? "page_write (batch)" : "page_gather (batch)");
}

extern "C" int ic_page_gather(const ic_page_rows_args* a, void* stream) { return page_rows(a, stream, false); }
extern "C" int ic_page_write(const ic_page_rows_args* a, void* stream) { return page_rows(a, stream, true); }
extern "C" int ic_page_gather_batch(const ic_page_rows_args* a, int32_t count, void* stream) {
  return page_rows_batch(a, count, stream, false);
}
extern "C" int ic_page_write_batch(const ic_page_rows_args* a, int32_t count, void* stream) {
  return page_rows_batch(a, count, stream, true);
}
