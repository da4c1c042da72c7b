// Varlen causal prefill attention (tcgen05 / TMEM / TMA) -- entry point.
#include "common.cuh"

extern "C" int b200_varlen_prefill(const void*, int64_t, int64_t, const void*, int64_t, int64_t,
                                   const void*, int64_t, int64_t, void*, int64_t, int64_t,
                                   const int32_t*, const int32_t*, int, int, int, int, int, int,
                                   float, int, int32_t*, void*) {
  return B200_ERR_UNSUPPORTED;
}
