// Allocation-free variant of the split-K paged decode entry point.
//
// Who needs it: callers that cannot allocate device memory at the moment they
// launch decode.  Examples are serving engines that hand (almost) all of HBM
// to the KV-cache pool up front and run their own fixed arena, plugins and
// foreign-language bindings (Go / Java / Rust FFI) that get raw device
// pointers but no device allocator to call, and latency-critical loops that
// must not take cudaMalloc's cost or its implicit device synchronisation.
// b200_paged_decode asks such callers for a workspace; this entry point does
// not: the split-K partials live in a file-scope device array instead.
//
// The array is a fixed B200_DECODE_NOALLOC_SCRATCH_BYTES (16 MiB) per GPU that
// loads this library, held until the process exits.  The first call on a
// device looks up the array's device address (cudaGetSymbolAddress with that
// device current) and caches it; make that first call before any stream
// capture on the device.  Every call on a device shares it
// and it keeps the previous call's contents; nothing in it needs to start at
// zero, because every partial the merge reads was written earlier in the
// same call.  Two calls whose kernels overlap on the GPU (different streams
// without ordering) race on the array and must not be issued.
#include <mutex>

#include "common.cuh"

static __device__ __align__(256) unsigned char g_decode_scratch[B200_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr size_t kNoAllocScratchBytes = B200_DECODE_NOALLOC_SCRATCH_BYTES;

// Device address of g_decode_scratch per device.  The symbol's name in host
// code is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress with that device current.
constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B200_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || p == nullptr)
      return B200_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return B200_OK;
}

}  // namespace

extern "C" int b200_paged_decode_noalloc(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                         const void* k_pool, const void* v_pool,
                                         int64_t kv_stride_blk, int64_t kv_stride_h,
                                         int64_t kv_stride_slot, const int32_t* block_table,
                                         int64_t bt_stride_row, const int32_t* seq_lens,
                                         const int32_t* row_ids, void* out, int64_t out_stride_b,
                                         int64_t out_stride_h, int batch, int num_heads,
                                         int num_kv_heads, int head_dim, int block_size,
                                         int num_blocks, int max_pages, int max_requests,
                                         float scale, int pages_per_split, int32_t* dev_status,
                                         void* stream) {
  if (pages_per_split <= 0 && batch > 0 && num_kv_heads > 0 && max_pages > 0)
    pages_per_split = b200_paged_decode_default_split(batch, num_kv_heads, max_pages);
  const size_t need =
      b200_paged_decode_workspace_size(batch, num_heads, max_pages, pages_per_split);
  if (need > kNoAllocScratchBytes) return B200_ERR_WORKSPACE;  // beyond the static maximum
  void* scratch = nullptr;
  if (need > 0) {
    const int st = scratch_for_current_device(&scratch);
    if (st != B200_OK) return st;
  }
  return b200_paged_decode(q, q_stride_b, q_stride_h, k_pool, v_pool, kv_stride_blk, kv_stride_h,
                           kv_stride_slot, block_table, bt_stride_row, seq_lens, row_ids, out,
                           out_stride_b, out_stride_h, batch, num_heads, num_kv_heads, head_dim,
                           block_size, num_blocks, max_pages, max_requests, scale,
                           pages_per_split, scratch, need > 0 ? kNoAllocScratchBytes : 0,
                           dev_status, stream);
}
