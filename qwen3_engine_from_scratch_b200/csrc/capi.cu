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

extern "C" {

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
