// Allocation-free variant of the split-K paged decode entry point.
//
// Who needs it: callers that cannot allocate device memory at the moment they
// launch decode.  Examples are serving engines that hand (almost) all of HBM
// to the KV-cache pool up front and run their own fixed arena, plugins and
// foreign-language bindings (Go / Java / Rust FFI) that get raw device
// pointers but no device allocator to call, and latency-critical loops that
// must not take cudaMalloc's cost or its implicit device synchronisation.
// b200_paged_decode asks such callers for a workspace; this entry point does
// not: the split-K workspace lives in a file-scope device array instead.
//
// The array is a fixed B200_DECODE_NOALLOC_SCRATCH_BYTES (16 MiB) per GPU that
// loads this library, held until the process exits.  Its layout is the one of
// the caller workspace of b200_paged_decode: first one split-arrival counter
// per (request, kv head), then the per-split partials.  The counters MUST be
// zero when a launch starts -- the last split of a pair to arrive merges the
// pair and resets its counter.  Each call therefore clears the counters of the
// pairs it uses (one cudaMemsetAsync on the call's stream, before the kernel;
// this allocates nothing) instead of relying on the zero-initialised storage
// and the previous launch's resets alone: two calls whose kernels overlapped
// on the GPU could leave a counter non-zero, and without the clear every later
// call would merge too early or never write its output.  The partials need no
// clearing: every partial the merge reads was written earlier in the same
// launch.  Calls whose kernels overlap on the GPU (different streams without
// ordering) still race on the shared array and give wrong results for those
// calls; do not issue them.
//
// The array's device address is looked up (cudaGetSymbolAddress, with the
// device current) on the first call in each CUDA context and cached per
// device together with the context's id, so a context torn down and created
// again (cudaDeviceReset) gets a fresh lookup.  Make the first call on a
// device (and the first after a reset) before any stream capture on it.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

static __device__ __align__(256) unsigned char g_decode_scratch[B200_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr size_t kNoAllocScratchBytes = B200_DECODE_NOALLOC_SCRATCH_BYTES;

// Device address of g_decode_scratch per device, with the id of the context it
// was looked up in.  The symbol's name in host code is only a host-side
// stand-in, so the address must come from cudaGetSymbolAddress with that
// device current.
constexpr int kMaxDevices = 64;
struct ScratchEntry {
  void* ptr = nullptr;
  unsigned long long ctx_id = 0;
};
ScratchEntry g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_once;

// Id of the calling thread's current context; 0 if it cannot be read (the
// address is then looked up again on every call).
unsigned long long current_context_id() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  });
  if (g_ctx_current == nullptr || g_ctx_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int scratch_for_current_device(void** out) {
  int dev = -1;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return b200host::status_from_cuda(e);
  if (dev < 0 || dev >= kMaxDevices) return B200_ERR_CUDA;
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  ScratchEntry& s = g_scratch[dev];
  if (s.ptr == nullptr || ctx == 0 || s.ctx_id != ctx) {
    void* p = nullptr;
    const cudaError_t ge = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (ge != cudaSuccess) return b200host::status_from_cuda(ge);
    if (p == nullptr) return B200_ERR_CUDA;
    s.ptr = p;
    s.ctx_id = ctx;
  }
  *out = s.ptr;
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
  // the limit is checked against the split this call will use: the default
  // split for these shapes when pages_per_split <= 0 (not the worst case that
  // b200_paged_decode_workspace_size(..., 0) reports)
  if (pages_per_split <= 0 && batch > 0 && num_kv_heads > 0 && max_pages > 0)
    pages_per_split = b200_paged_decode_default_split(batch, num_kv_heads, max_pages);
  const size_t need =
      b200_paged_decode_workspace_size(batch, num_heads, max_pages, pages_per_split);
  if (need > kNoAllocScratchBytes) return B200_ERR_WORKSPACE;  // beyond the static maximum
  void* scratch = nullptr;
  if (need > 0) {
    const int st = scratch_for_current_device(&scratch);
    if (st != B200_OK) return st;
    // the split-arrival counters of the pairs this call uses start at zero.
    // The clear is enqueued only for calls that pass the pointer and shape
    // checks of the decode; one that the decode still refuses (alignment)
    // has cleared counters that must be zero anyway -- the library's own
    // memory, never the caller's.
    const int64_t pairs = static_cast<int64_t>(batch) * num_kv_heads;
    const bool launches = q && k_pool && v_pool && block_table && seq_lens && row_ids && out &&
                          head_dim == 128 && block_size == 16 && num_heads > 0 &&
                          num_heads % num_kv_heads == 0 && num_heads / num_kv_heads <= 8 &&
                          num_blocks > 0 && max_requests > 0 && bt_stride_row > 0;
    if (launches && pairs > 0 && pairs <= 65536) {
      const cudaError_t me = cudaMemsetAsync(scratch, 0, static_cast<size_t>(pairs) * sizeof(int32_t),
                                             static_cast<cudaStream_t>(stream));
      if (me != cudaSuccess) return b200host::status_from_cuda(me);
    }
  }
  return b200_paged_decode(q, q_stride_b, q_stride_h, k_pool, v_pool, kv_stride_blk, kv_stride_h,
                           kv_stride_slot, block_table, bt_stride_row, seq_lens, row_ids, out,
                           out_stride_b, out_stride_h, batch, num_heads, num_kv_heads, head_dim,
                           block_size, num_blocks, max_pages, max_requests, scale,
                           pages_per_split, scratch, need > 0 ? kNoAllocScratchBytes : 0,
                           dev_status, stream);
}
