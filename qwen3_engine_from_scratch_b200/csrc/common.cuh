// Shared device helpers for the sm_100a attention kernels: thin inline-PTX
// wrappers for mbarriers, TMA tensor loads, ldmatrix/movmatrix and the bf16
// mma.sync tile, plus host-side tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qwen3_b200_attn.h"

#define B200_DEVICE __device__ __forceinline__

namespace b200 {

// Upper bound on the polls of one pipeline wait.  A poll of try_wait can
// suspend the thread for a hardware-defined interval, so this bound is far
// beyond any legitimate wait, and it still ends a wait whose copy never lands.
constexpr uint32_t kMaxWaitPolls = 1u << 24;

B200_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

B200_DEVICE void flag_error(int32_t* dev_status, int32_t bits) {
  if (dev_status != nullptr) atomicOr(dev_status, bits);
}

// ---------------------------------------------------------------- mbarrier
B200_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

B200_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

B200_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// orders this thread's generic-proxy global stores before later async-proxy
// (TMA) accesses of the same memory
B200_DEVICE void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

B200_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

B200_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of the barrier to complete; false if it did not
// complete within kMaxWaitPolls polls.
B200_DEVICE bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMaxWaitPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

B200_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` with a wall-clock limit; also gives up as soon as
// another CTA has recorded a timeout in the device status word, so a broken
// pipeline ends the whole grid within about one limit.  Returns false on
// give-up.
B200_DEVICE bool mbar_wait_abortable(uint32_t bar, uint32_t parity, const int32_t* dev_status,
                                     uint64_t limit_ns) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (dev_status != nullptr &&
          (*reinterpret_cast<const volatile int32_t*>(dev_status) & B200_DEV_TIMEOUT))
        return false;
      const uint64_t t = globaltimer_ns();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > limit_ns) {
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
B200_DEVICE uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

B200_DEVICE void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled tensor load into this CTA's shared memory, completing on `bar`.
// No multicast: every load reads this GPU's own memory for this CTA only.
B200_DEVICE void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                             int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "l"(policy)
      : "memory");
}

// 4-D tiled tensor load without a cache hint (no multicast), completing on `bar`.
B200_DEVICE void tma_load_4d_nohint(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0,
                                    int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 3-D tiled tensor load (no multicast), completing on `bar`.
B200_DEVICE void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 3-D tiled tensor prefetch into L2 (no destination, no barrier).
B200_DEVICE void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// 3-D tiled tensor store from this CTA's shared memory (bulk-group completion).
B200_DEVICE void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
B200_DEVICE void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every committed bulk store of this thread has finished reading its shared-memory source
B200_DEVICE void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// every committed bulk store of this thread is complete
B200_DEVICE void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

B200_DEVICE void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// ---------------------------------------------------------------- named barriers
// barrier `id` over `count` threads (a multiple of 32)
B200_DEVICE void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// barrier `id` over `count` threads that also ANDs a predicate: every thread
// gets true only if all passed true, so a group of warps leaves a loop together
B200_DEVICE bool named_bar_and(uint32_t id, uint32_t count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %3, 0;\n\t"
      "barrier.red.and.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(id), "r"(count), "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------- warp MMA
B200_DEVICE void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                             uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

B200_DEVICE void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                   uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

B200_DEVICE uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// D = A(16x16, row) * B(16x8, col) + D, bf16 inputs, fp32 accumulate.
B200_DEVICE void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- numerics
// 2^x on the special-function unit (PTX ex2.approx.ftz.f32); 2^-inf = +0.
B200_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA/ALU pipes (no special-function unit), for x <= 126:
// x = j + f with j = round(x) obtained by adding 1.5 * 2^23 (the integer lands
// in the low mantissa bits), 2^f for f in [-0.5, 0.5] from a degree-3
// polynomial fitted here for minimum relative error (max 7.5e-5), and 2^j
// applied by adding j to the exponent field.  Inputs below -125 (and -inf)
// are clamped to -125 so the exponent field never underflows into the sign
// bit; the result, about 2^-125, is negligible next to the row maximum's 2^0.
B200_DEVICE float ex2_fma(float x) {
  x = fmaxf(x, -125.0f);
  const float t = x + 12582912.0f;
  const float j = t - 12582912.0f;
  const float f = x - j;
  const float p =
      fmaf(fmaf(fmaf(0.0551716685f, f, 0.2426111400f), f, 0.6932609677f), f, 0.9999280572f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// max of three floats in one instruction (sm_100 three-input max.f32)
B200_DEVICE float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

B200_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions: one issue for two lanes)
B200_DEVICE uint64_t f2_pack(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
B200_DEVICE void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
B200_DEVICE uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
B200_DEVICE uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
B200_DEVICE uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// ex2_fma on a pair with packed fp32 arithmetic: same method and result as
// ex2_fma lane by lane (2^j applied as t_bits * 2^23 + p_bits, which equals the
// shift-and-add of ex2_fma modulo 2^32).
B200_DEVICE uint64_t ex2_fma2(uint64_t y) {
  float a, b;
  f2_unpack(y, a, b);
  const uint64_t yc = f2_pack(fmaxf(a, -125.0f), fmaxf(b, -125.0f));
  const uint64_t t = f2_add(yc, f2_pack(12582912.0f, 12582912.0f));
  const uint64_t j = f2_add(t, f2_pack(-12582912.0f, -12582912.0f));
  const uint64_t f = f2_fma(j, f2_pack(-1.0f, -1.0f), yc);
  uint64_t p = f2_fma(f2_pack(0.0551716685f, 0.0551716685f), f,
                      f2_pack(0.2426111400f, 0.2426111400f));
  p = f2_fma(p, f, f2_pack(0.6932609677f, 0.6932609677f));
  p = f2_fma(p, f, f2_pack(0.9999280572f, 0.9999280572f));
  float t0, t1, p0, p1;
  f2_unpack(t, t0, t1);
  f2_unpack(p, p0, p1);
  return f2_pack(__int_as_float(__float_as_int(t0) * 8388608 + __float_as_int(p0)),
                 __int_as_float(__float_as_int(t1) * 8388608 + __float_as_int(p1)));
}

// 32-byte global store (sm_100 256-bit access); p must be 32-byte aligned.
B200_DEVICE void st_global_v8(void* p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]),
               "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

B200_DEVICE float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
B200_DEVICE float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// First statement of a kernel launched with b200host::launch_pdl: wait until
// the previous kernel on the stream has completed and its writes are visible
// (a no-op for an ordinary launch), then let the next programmatic dependent
// start launching (it waits the same way before touching memory).
B200_DEVICE void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace b200

// ------------------------------------------------------------------ host side
namespace b200host {

// cuTensorMapEncodeTiled, fetched once from the driver through the runtime
// (no link-time dependency on libcuda).
CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                      const cuuint32_t* box, const cuuint32_t* elem_strides,
                      CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2promo);

int current_device();
int sm_count(int device);
int status_from_cuda(cudaError_t e);  // records e for b200_last_cuda_error_string
cudaError_t last_cuda_error();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch as a programmatic dependent of the previous kernel on the stream:
// the grid may be scheduled while that kernel drains, which hides the launch
// latency between back-to-back kernels.  The kernel must begin with
// b200::pdl_begin() (nothing read or written before it).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace b200host
