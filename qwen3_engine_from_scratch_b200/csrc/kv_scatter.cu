// KV-cache slot scatter: copy new K/V rows (head_dim bf16 = 256 bytes each)
// into the paged pool.  HBM-bound byte movement; eight threads share a row,
// each moving chunks c and c + 8 (16 bytes each) of K and of V, so every
// access of the eight is one fully used 128-byte line and a warp writes four
// 256-byte rows of each tensor with 16-byte vector stores.
//
//   rows  mode: position = seq_lens[row_ids[b]] + s, page from the 2-D block
//               table (update_kv_batch_kernel, qwen3/kernels/paged_attention.py:
//               292-350, and PagedKVCache.update, qwen3/PagedKVcache.py:187-214)
//   span  mode: one request, position = start_pos + s with start_pos from the
//               host (PagedKVCache.update exactly: its write position is the
//               handle's host seq_len, qwen3/PagedKVcache.py:189-203), page from
//               one block-table row of num_pages allocated entries
//   slots mode: slot = slot_mapping[t] = phys * block_size + offset
//
// Every index is range-checked; an out-of-range index sets a dev_status bit
// and the row is skipped (never written out of bounds).
#include "common.cuh"

namespace {

constexpr int kChunksPerRow = 16;  // 128 bf16 = 256 bytes = 16 x 16 B
constexpr int kThreadsPerRow = kChunksPerRow / 2;  // two 16-byte pieces per thread
constexpr int kThreads = 256;

B200_DEVICE uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

struct RowsArgs {
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  int64_t kn_b, kn_h, kn_s, vn_b, vn_h, vn_s;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  int64_t kp_blk, kp_layer, kp_h, kp_slot, vp_blk, vp_layer, vp_h, vp_slot;
  const int32_t* seq_lens;
  const int32_t* block_table;
  int64_t bt_row;
  const int32_t* row_ids;  // nullptr: span mode (row 0 of block_table, position start_pos + s)
  int64_t start_pos;
  int batch, n_tokens, num_kv_heads, block_size, num_blocks, max_pages, max_requests, layer;
  int32_t* dev_status;
};

// Quotient and remainder of a non-negative position by the page size, in 32
// bits whenever the position fits (64-bit division costs several times more).
B200_DEVICE int64_t page_of(int64_t pos, int block_size, int64_t* off) {
  if (pos <= 0x7fffffff) {
    const int p = static_cast<int>(pos);
    const int page = p / block_size;
    *off = p - page * block_size;
    return page;
  }
  const int64_t page = pos / block_size;
  *off = pos - page * block_size;
  return page;
}

// Each thread moves two 16-byte pieces of a row of K and of V (chunks c and
// c + 8, so 8 consecutive threads cover a 128-byte line per access): half as
// many threads pay the row's index arithmetic.  IdxT: int when the thread
// count fits, else int64_t.
template <typename IdxT>
__global__ void __launch_bounds__(kThreads) kv_scatter_rows_kernel(const RowsArgs a) {
  // launched with b200host::launch_pdl: nothing read or written before this
  b200::pdl_begin();
  const IdxT idx = static_cast<IdxT>(blockIdx.x) * kThreads + threadIdx.x;
  const int chunk = static_cast<int>(idx & (kThreadsPerRow - 1));
  IdxT r = idx / kThreadsPerRow;  // (b, s, h) row index
  const IdxT total = static_cast<IdxT>(a.batch) * a.n_tokens * a.num_kv_heads;
  if (r >= total) return;
  const int h = static_cast<int>(r % a.num_kv_heads);
  r /= a.num_kv_heads;
  const int s = static_cast<int>(r % a.n_tokens);
  const int b = static_cast<int>(r / a.n_tokens);

  int row = 0;
  int64_t pos;
  if (a.row_ids != nullptr) {
    row = a.row_ids[b];
    if (row < 0 || row >= a.max_requests) {
      if (chunk == 0) b200::flag_error(a.dev_status, B200_DEV_BAD_ROW);
      return;
    }
    pos = static_cast<int64_t>(a.seq_lens[row]) + s;
  } else {
    pos = a.start_pos + s;
  }
  int64_t off = 0;
  const int64_t page = pos < 0 ? -1 : page_of(pos, a.block_size, &off);
  if (pos < 0 || page >= a.max_pages) {
    if (chunk == 0) b200::flag_error(a.dev_status, B200_DEV_SEQ_OVERFLOW);
    return;
  }
  const int phys = a.block_table[row * a.bt_row + page];
  if (phys < 0 || phys >= a.num_blocks) {
    if (chunk == 0) b200::flag_error(a.dev_status, B200_DEV_BAD_PAGE);
    return;
  }
  const int64_t e = static_cast<int64_t>(chunk) * 8;
  const __nv_bfloat16* ks = a.k_new + b * a.kn_b + h * a.kn_h + s * a.kn_s + e;
  const __nv_bfloat16* vs = a.v_new + b * a.vn_b + h * a.vn_h + s * a.vn_s + e;
  const uint4 k0 = ld_stream(ks), k1 = ld_stream(ks + 64);
  const uint4 v0 = ld_stream(vs), v1 = ld_stream(vs + 64);
  __nv_bfloat16* kd = a.k_pool + phys * a.kp_blk + a.layer * a.kp_layer + h * a.kp_h +
                      off * a.kp_slot + e;
  __nv_bfloat16* vd = a.v_pool + phys * a.vp_blk + a.layer * a.vp_layer + h * a.vp_h +
                      off * a.vp_slot + e;
  *reinterpret_cast<uint4*>(kd) = k0;
  *reinterpret_cast<uint4*>(kd + 64) = k1;
  *reinterpret_cast<uint4*>(vd) = v0;
  *reinterpret_cast<uint4*>(vd + 64) = v1;
}

struct SlotsArgs {
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t k_t, k_h, v_t, v_h;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  int64_t kp_blk, kp_layer, kp_h, kp_slot, vp_blk, vp_layer, vp_h, vp_slot;
  const void* slots;
  int slot_is_int64;
  int n_tokens, num_kv_heads, block_size, num_blocks, layer;
  int32_t* dev_status;
};

template <typename IdxT>
__global__ void __launch_bounds__(kThreads) kv_scatter_slots_kernel(const SlotsArgs a) {
  // launched with b200host::launch_pdl: nothing read or written before this
  b200::pdl_begin();
  const IdxT idx = static_cast<IdxT>(blockIdx.x) * kThreads + threadIdx.x;
  const int chunk = static_cast<int>(idx & (kThreadsPerRow - 1));
  const IdxT r = idx / kThreadsPerRow;  // (t, h) row index
  if (r >= static_cast<IdxT>(a.n_tokens) * a.num_kv_heads) return;
  const int h = static_cast<int>(r % a.num_kv_heads);
  const IdxT t = r / a.num_kv_heads;
  const int64_t slot = a.slot_is_int64 ? static_cast<const int64_t*>(a.slots)[t]
                                       : static_cast<int64_t>(static_cast<const int32_t*>(a.slots)[t]);
  if (slot < 0) return;  // padding token
  int64_t off = 0;
  const int64_t phys = page_of(slot, a.block_size, &off);
  if (phys >= a.num_blocks) {
    if (chunk == 0) b200::flag_error(a.dev_status, B200_DEV_BAD_SLOT);
    return;
  }
  const int64_t e = static_cast<int64_t>(chunk) * 8;
  const __nv_bfloat16* ks = a.k + t * a.k_t + h * a.k_h + e;
  const __nv_bfloat16* vs = a.v + t * a.v_t + h * a.v_h + e;
  const uint4 k0 = ld_stream(ks), k1 = ld_stream(ks + 64);
  const uint4 v0 = ld_stream(vs), v1 = ld_stream(vs + 64);
  __nv_bfloat16* kd = a.k_pool + phys * a.kp_blk + a.layer * a.kp_layer + h * a.kp_h +
                      off * a.kp_slot + e;
  __nv_bfloat16* vd = a.v_pool + phys * a.vp_blk + a.layer * a.vp_layer + h * a.vp_h +
                      off * a.vp_slot + e;
  *reinterpret_cast<uint4*>(kd) = k0;
  *reinterpret_cast<uint4*>(kd + 64) = k1;
  *reinterpret_cast<uint4*>(vd) = v0;
  *reinterpret_cast<uint4*>(vd + 64) = v1;
}

bool mult8(int64_t s) { return (s & 7) == 0; }

// rows / span mode over `rows` (token, kv head) rows
int launch_rows(const RowsArgs& a, int64_t rows, void* stream) {
  const int64_t threads = rows * kThreadsPerRow;
  const int64_t blocks = (threads + kThreads - 1) / kThreads;
  if (blocks > 0x7fffffff) return B200_ERR_INVALID_ARGUMENT;
  const dim3 grid(static_cast<unsigned>(blocks));
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  return b200host::status_from_cuda(
      blocks * kThreads <= 0x7fffffff
          ? b200host::launch_pdl(kv_scatter_rows_kernel<int>, grid, dim3(kThreads), 0, s, a)
          : b200host::launch_pdl(kv_scatter_rows_kernel<int64_t>, grid, dim3(kThreads), 0, s, a));
}

}  // namespace

extern "C" int b200_kv_scatter_rows(
    const void* k_new, const void* v_new, int64_t kn_stride_b, int64_t kn_stride_h,
    int64_t kn_stride_s, int64_t vn_stride_b, int64_t vn_stride_h, int64_t vn_stride_s,
    void* k_pool, void* v_pool, int64_t kp_stride_blk, int64_t kp_stride_layer,
    int64_t kp_stride_h, int64_t kp_stride_slot, int64_t vp_stride_blk, int64_t vp_stride_layer,
    int64_t vp_stride_h, int64_t vp_stride_slot, const int32_t* seq_lens,
    const int32_t* block_table, int64_t bt_stride_row, const int32_t* row_ids, int batch,
    int n_tokens, int num_kv_heads, int head_dim, int block_size, int num_blocks, int max_pages,
    int max_requests, int layer, int32_t* dev_status, void* stream) {
  if (batch < 0 || n_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0 ||
      max_pages <= 0 || max_requests <= 0 || layer < 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (batch == 0 || n_tokens == 0) return B200_OK;
  if (!k_new || !v_new || !k_pool || !v_pool || !seq_lens || !block_table || !row_ids)
    return B200_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return B200_ERR_UNSUPPORTED;
  if (!b200host::aligned16(k_new) || !b200host::aligned16(v_new) ||
      !b200host::aligned16(k_pool) || !b200host::aligned16(v_pool))
    return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {kn_stride_b, kn_stride_h, kn_stride_s, vn_stride_b,
                             vn_stride_h, vn_stride_s, kp_stride_blk, kp_stride_layer,
                             kp_stride_h, kp_stride_slot, vp_stride_blk, vp_stride_layer,
                             vp_stride_h, vp_stride_slot};
  for (int64_t s : strides)
    if (!mult8(s)) return B200_ERR_ALIGNMENT;

  RowsArgs a;
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.kn_b = kn_stride_b; a.kn_h = kn_stride_h; a.kn_s = kn_stride_s;
  a.vn_b = vn_stride_b; a.vn_h = vn_stride_h; a.vn_s = vn_stride_s;
  a.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  a.kp_blk = kp_stride_blk; a.kp_layer = kp_stride_layer; a.kp_h = kp_stride_h;
  a.kp_slot = kp_stride_slot;
  a.vp_blk = vp_stride_blk; a.vp_layer = vp_stride_layer; a.vp_h = vp_stride_h;
  a.vp_slot = vp_stride_slot;
  a.seq_lens = seq_lens; a.block_table = block_table; a.bt_row = bt_stride_row;
  a.row_ids = row_ids;
  a.start_pos = 0;
  a.batch = batch; a.n_tokens = n_tokens; a.num_kv_heads = num_kv_heads;
  a.block_size = block_size; a.num_blocks = num_blocks; a.max_pages = max_pages;
  a.max_requests = max_requests; a.layer = layer; a.dev_status = dev_status;

  return launch_rows(a, static_cast<int64_t>(batch) * n_tokens * num_kv_heads, stream);
}

extern "C" int b200_kv_scatter_slots(
    const void* k, const void* v, int64_t k_stride_t, int64_t k_stride_h, int64_t v_stride_t,
    int64_t v_stride_h, void* k_pool, void* v_pool, int64_t kp_stride_blk,
    int64_t kp_stride_layer, int64_t kp_stride_h, int64_t kp_stride_slot, int64_t vp_stride_blk,
    int64_t vp_stride_layer, int64_t vp_stride_h, int64_t vp_stride_slot,
    const void* slot_mapping, int slot_is_int64, int n_tokens, int num_kv_heads, int head_dim,
    int block_size, int num_blocks, int layer, int32_t* dev_status, void* stream) {
  if (n_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0 || layer < 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (n_tokens == 0) return B200_OK;
  if (!k || !v || !k_pool || !v_pool || !slot_mapping) return B200_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return B200_ERR_UNSUPPORTED;
  if (!b200host::aligned16(k) || !b200host::aligned16(v) || !b200host::aligned16(k_pool) ||
      !b200host::aligned16(v_pool))
    return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {k_stride_t, k_stride_h, v_stride_t, v_stride_h,
                             kp_stride_blk, kp_stride_layer, kp_stride_h, kp_stride_slot,
                             vp_stride_blk, vp_stride_layer, vp_stride_h, vp_stride_slot};
  for (int64_t s : strides)
    if (!mult8(s)) return B200_ERR_ALIGNMENT;

  SlotsArgs a;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.k_t = k_stride_t; a.k_h = k_stride_h; a.v_t = v_stride_t; a.v_h = v_stride_h;
  a.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  a.kp_blk = kp_stride_blk; a.kp_layer = kp_stride_layer; a.kp_h = kp_stride_h;
  a.kp_slot = kp_stride_slot;
  a.vp_blk = vp_stride_blk; a.vp_layer = vp_stride_layer; a.vp_h = vp_stride_h;
  a.vp_slot = vp_stride_slot;
  a.slots = slot_mapping; a.slot_is_int64 = slot_is_int64;
  a.n_tokens = n_tokens; a.num_kv_heads = num_kv_heads; a.block_size = block_size;
  a.num_blocks = num_blocks; a.layer = layer; a.dev_status = dev_status;

  const int64_t threads = static_cast<int64_t>(n_tokens) * num_kv_heads * kThreadsPerRow;
  const int64_t blocks = (threads + kThreads - 1) / kThreads;
  if (blocks > 0x7fffffff) return B200_ERR_INVALID_ARGUMENT;
  const dim3 grid(static_cast<unsigned>(blocks));
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  return b200host::status_from_cuda(
      blocks * kThreads <= 0x7fffffff
          ? b200host::launch_pdl(kv_scatter_slots_kernel<int>, grid, dim3(kThreads), 0, s, a)
          : b200host::launch_pdl(kv_scatter_slots_kernel<int64_t>, grid, dim3(kThreads), 0, s, a));
}

extern "C" int b200_kv_scatter_span(
    const void* k_new, const void* v_new, int64_t kn_stride_h, int64_t kn_stride_s,
    int64_t vn_stride_h, int64_t vn_stride_s, void* k_pool, void* v_pool, int64_t kp_stride_blk,
    int64_t kp_stride_layer, int64_t kp_stride_h, int64_t kp_stride_slot, int64_t vp_stride_blk,
    int64_t vp_stride_layer, int64_t vp_stride_h, int64_t vp_stride_slot,
    const int32_t* block_table_row, int num_pages, int start_pos, int n_tokens, int num_kv_heads,
    int head_dim, int block_size, int num_blocks, int layer, int32_t* dev_status, void* stream) {
  if (n_tokens < 0 || num_pages < 0 || start_pos < 0 || num_kv_heads <= 0 || block_size <= 0 ||
      num_blocks <= 0 || layer < 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (n_tokens == 0) return B200_OK;
  if (!k_new || !v_new || !k_pool || !v_pool || !block_table_row || num_pages == 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return B200_ERR_UNSUPPORTED;
  if (!b200host::aligned16(k_new) || !b200host::aligned16(v_new) ||
      !b200host::aligned16(k_pool) || !b200host::aligned16(v_pool))
    return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {kn_stride_h, kn_stride_s, vn_stride_h, vn_stride_s,
                             kp_stride_blk, kp_stride_layer, kp_stride_h, kp_stride_slot,
                             vp_stride_blk, vp_stride_layer, vp_stride_h, vp_stride_slot};
  for (int64_t s : strides)
    if (!mult8(s)) return B200_ERR_ALIGNMENT;

  RowsArgs a;
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.kn_b = 0; a.kn_h = kn_stride_h; a.kn_s = kn_stride_s;
  a.vn_b = 0; a.vn_h = vn_stride_h; a.vn_s = vn_stride_s;
  a.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  a.kp_blk = kp_stride_blk; a.kp_layer = kp_stride_layer; a.kp_h = kp_stride_h;
  a.kp_slot = kp_stride_slot;
  a.vp_blk = vp_stride_blk; a.vp_layer = vp_stride_layer; a.vp_h = vp_stride_h;
  a.vp_slot = vp_stride_slot;
  a.seq_lens = nullptr; a.block_table = block_table_row; a.bt_row = 0;
  a.row_ids = nullptr;
  a.start_pos = start_pos;
  a.batch = 1; a.n_tokens = n_tokens; a.num_kv_heads = num_kv_heads;
  a.block_size = block_size; a.num_blocks = num_blocks; a.max_pages = num_pages;
  a.max_requests = 1; a.layer = layer; a.dev_status = dev_status;

  return launch_rows(a, static_cast<int64_t>(n_tokens) * num_kv_heads, stream);
}
