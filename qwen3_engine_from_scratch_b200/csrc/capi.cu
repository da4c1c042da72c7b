// Library-wide C-ABI helpers: status text, ABI version, device queries and the
// driver entry point used to encode TMA tensor maps.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace b200host {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                      const cuuint32_t* box, const cuuint32_t* elem_strides,
                      CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2promo) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (g_encode == nullptr) return CUDA_ERROR_NOT_FOUND;
  return g_encode(map, dtype, rank, base, dims, strides_bytes, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, l2promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int sm_count(int device) {
  if (device < 0) return -1;
  if (device < kMaxDevices && g_sm_count[device] > 0) return g_sm_count[device];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  if (device < kMaxDevices) g_sm_count[device] = n;
  return n;
}

namespace {
thread_local cudaError_t g_last_cuda_error = cudaSuccess;
}

int status_from_cuda(cudaError_t e) {
  if (e == cudaSuccess) return B200_OK;
  g_last_cuda_error = e;
  return B200_ERR_CUDA;
}

cudaError_t last_cuda_error() { return g_last_cuda_error; }

}  // namespace b200host

namespace {

// One warp waits on an mbarrier that nothing completes, through the bounded
// wait every prefill pipeline wait uses: it gives up after limit_ns (or at
// once when dev_status already records a timeout elsewhere in the grid) and
// records B200_DEV_TIMEOUT, and the kernel returns normally.
__global__ void bounded_wait_probe_kernel(int32_t* dev_status, int32_t* result,
                                          uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = b200::smem_u32(&bar);
  if (threadIdx.x == 0) {
    b200::mbar_init(b, 1);
    b200::fence_mbar_init();
  }
  __syncthreads();
  const bool completed = b200::mbar_wait_abortable(b, 0, dev_status, limit_ns);
  if (threadIdx.x == 0) {
    if (!completed) b200::flag_error(dev_status, B200_DEV_TIMEOUT);
    result[0] = completed ? 1 : 0;
  }
}

constexpr uint64_t kMaxProbeWaitNs = 10000000000ull;  // 10 s

}  // namespace

extern "C" {

int b200_selftest_bounded_wait(int32_t* dev_status, int32_t* result, uint64_t limit_ns,
                               void* stream) {
  if (dev_status == nullptr || result == nullptr || limit_ns == 0 || limit_ns > kMaxProbeWaitNs)
    return B200_ERR_INVALID_ARGUMENT;
  bounded_wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dev_status, result,
                                                                             limit_ns);
  return b200host::status_from_cuda(cudaGetLastError());
}

const char* b200_status_string(int status) {
  switch (status) {
    case B200_OK: return "ok";
    case B200_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, size or stride)";
    case B200_ERR_UNSUPPORTED: return "unsupported shape (head_dim, block_size or GQA group)";
    case B200_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case B200_ERR_WORKSPACE: return "workspace missing or too small";
    case B200_ERR_CUDA: return "CUDA launch or driver error";
    case B200_ERR_TENSOR_MAP: return "TMA tensor map could not be encoded";
    default: return "unknown status";
  }
}

int b200_abi_version(void) { return 101; }

const char* b200_last_cuda_error_string(void) {
  const cudaError_t e = b200host::last_cuda_error();
  return e == cudaSuccess ? "no CUDA error recorded" : cudaGetErrorString(e);
}

int b200_device_sm_count(void) { return b200host::sm_count(b200host::current_device()); }

}  // extern "C"
