// Varlen causal prefill attention for sm_100a on the 5th-generation tensor
// cores (tcgen05 + TMEM), fed by TMA.  Replaces flash_attention_varlen_kernel
// (qwen3/kernels/flash_attention_varlen.py:25-123) and its host entry (:126-194).
//
// One CTA computes a 128-query tile of one query head of one sequence:
//   warp 4      TMA producer: Q tile once, then K/V tiles of 128 keys into a
//               2-stage ring (two 64-column boxes per tile, 128-byte swizzle).
//   warp 5      MMA issuer (one thread): S = Q.K^T into one of two TMEM score
//               buffers (M=128, N=128, K=16 per instruction, 8 instructions),
//               O += P.V into the TMEM output accumulator; every group ends
//               with tcgen05.commit on an mbarrier.
//   warps 0-3   softmax: thread r owns query row r (TMEM lane r); it loads its
//               128 scores with tcgen05.ld, applies the causal / length mask,
//               updates the running max (base 2) and sum in fp32, writes P as
//               bf16 into a 128-byte-swizzled shared-memory tile (the A
//               operand of the P.V MMA), and rescales its O row in TMEM only
//               when the running max grew by more than 2^8 (otherwise the
//               stale max keeps every P <= 2^8, exact in fp32).
// KV tiles strictly above the diagonal are never loaded (the reference
// computes every KV block of the sequence, flash_attention_varlen.py:74-77).
//
// Operand layouts (UMMA canonical forms):
//   Q, K  (128 rows x 128 d)  K-major, 128B swizzle: two 16 KB blocks of
//         [row][64 d]; descriptor SBO = 1024 B (8 rows), start += 32 B per K
//         step inside a block, += 16 KB between blocks.
//   P     (128 rows x 128 keys) K-major, same form.
//   V     (128 keys x 128 d)  MN-major (d contiguous), 128B swizzle: LBO =
//         16 KB between the two 64-d blocks, SBO = 1024 B (8 keys), start +=
//         2 KB (16 keys) per K step.
//   TMEM  columns [0,128) S0, [128,256) S1, [256,384) O; lane = query row.
// Every mbarrier wait is bounded; TMEM is always freed before the CTA exits.
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr int kD = 128;
constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kStages = 2;
constexpr int kTileBytes = kBM * kD * 2;  // 32 KB
constexpr int kBlockBytes = kTileBytes / 2;  // 16 KB: one 64-column swizzled block
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffP = kOffV + kStages * kTileBytes;
constexpr int kSmemTiles = kOffP + kTileBytes;  // 192 KB
constexpr int kSmemBytes = kSmemTiles + 1024;
constexpr int kThreads = 192;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Of every kExpFmaPeriod columns, the first 2*kExpFmaPairs use ex2_fma.
constexpr int kExpFmaPeriod = 8;
constexpr int kExpFmaPairs = 2;
constexpr float kLog2e = 1.4426950408889634f;

struct PrefillArgs {
  const int32_t* cu;
  const int32_t* lens;  // nullable
  __nv_bfloat16* out;
  int64_t o_t, o_h;
  int num_seqs, num_heads, group, max_seqlen, zero_pad;
  float scale_log2;
  int32_t* dev_status;
};

struct __align__(8) Barriers {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t v_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint32_t tmem_base;
  int32_t error;
};

// ---------------------------------------------------------------- tcgen05
B200_DEVICE uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  // start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46), version 1 [46,48),
  // base offset 0, layout SWIZZLE_128B (2) at [61,64)
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M=128, N=128.
constexpr uint32_t idesc_bf16(bool b_mn_major) {
  return (1u << 4)                     // D format f32
         | (1u << 7)                   // A format bf16
         | (1u << 10)                  // B format bf16
         | (0u << 15)                  // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)
         | ((static_cast<uint32_t>(kBN) >> 3) << 17)   // N >> 3
         | ((static_cast<uint32_t>(kBM) >> 4) << 24);  // M >> 4
}

B200_DEVICE void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

B200_DEVICE void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

B200_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
B200_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this thread's lane into r[0..31].  The load is
// asynchronous: the registers are valid only after tmem_wait_ld(r) below.
B200_DEVICE void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// tcgen05.wait::ld that also "rewrites" r[0..31], so no use of the loaded
// registers can be scheduled above the wait.
B200_DEVICE void tmem_wait_ld(uint32_t* r) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
        "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
        "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
        "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
        "+r"(r[31])
      :
      : "memory");
}

B200_DEVICE void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

B200_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

B200_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per pipeline wait

// Bounded wait; on give-up record the error in the CTA and the device status
// (which makes every other CTA of the grid give up too).
B200_DEVICE bool wait_or_flag(uint32_t bar, uint32_t parity, Barriers* B, int32_t* dev_status) {
  if (b200::mbar_wait_abortable(bar, parity, dev_status, kWaitLimitNs)) return true;
  if (atomicExch(&B->error, 1) == 0) b200::flag_error(dev_status, B200_DEV_TIMEOUT);
  return false;
}

__global__ void __launch_bounds__(kThreads, 1)
    varlen_prefill_kernel(const __grid_constant__ CUtensorMap tmq,
                          const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Barriers B;

  const int tile = gridDim.x - 1 - blockIdx.x;  // heaviest (latest) tiles first
  const int h = blockIdx.y;
  const int seq = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (a.dev_status != nullptr &&
      (*reinterpret_cast<const volatile int32_t*>(a.dev_status) & B200_DEV_TIMEOUT))
    return;  // a pipeline already gave up: do not start new work until the host clears it
  const int start = a.cu[seq];
  const int len = a.lens != nullptr ? a.lens[seq] : a.cu[seq + 1] - start;
  const int m0 = tile * kBM;
  if (len < 0 || len > a.max_seqlen) {
    if (threadIdx.x == 0 && tile == 0 && h == 0) b200::flag_error(a.dev_status, B200_DEV_SEQ_OVERFLOW);
    return;
  }
  if (m0 >= len) {
    // tile entirely past the sequence: only the padded adapter wants zeros here
    if (a.zero_pad) {
      const int rows = min(kBM, a.max_seqlen - m0);
      for (int i = threadIdx.x; i < rows * (kD / 8); i += kThreads) {
        const int r = i / (kD / 8), c = i % (kD / 8);
        *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(start + m0 + r) * a.o_t +
                                  static_cast<int64_t>(h) * a.o_h + c * 8) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }
  const int hk = h / a.group;
  const int kv_end = min(len, m0 + kBM);        // causal: keys < m0 + 128
  const int n_kv = (kv_end + kBN - 1) / kBN;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = b200::smem_u32(smem);
  const uint32_t sQ = sbase + kOffQ, sK = sbase + kOffK, sV = sbase + kOffV, sP = sbase + kOffP;

  const uint32_t bar_q = b200::smem_u32(&B.q_full);
  auto bar_k = [&](int s) { return b200::smem_u32(&B.k_full[s]); };
  auto bar_v = [&](int s) { return b200::smem_u32(&B.v_full[s]); };
  auto bar_e = [&](int s) { return b200::smem_u32(&B.kv_empty[s]); };
  auto bar_sf = [&](int s) { return b200::smem_u32(&B.s_full[s]); };
  auto bar_sr = [&](int s) { return b200::smem_u32(&B.s_free[s]); };
  const uint32_t bar_p = b200::smem_u32(&B.p_full);
  const uint32_t bar_o = b200::smem_u32(&B.pv_done);

  if (threadIdx.x == 0) {
    b200::mbar_init(bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      b200::mbar_init(bar_k(s), 1);
      b200::mbar_init(bar_v(s), 1);
      b200::mbar_init(bar_e(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      b200::mbar_init(bar_sf(s), 1);
      b200::mbar_init(bar_sr(s), 128);
    }
    b200::mbar_init(bar_p, 128);
    b200::mbar_init(bar_o, 1);
    B.error = 0;
    b200::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     b200::smem_u32(&B.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B.tmem_base;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      b200::prefetch_tensormap(&tmq);
      b200::prefetch_tensormap(&tmk);
      b200::prefetch_tensormap(&tmv);
      b200::mbar_arrive_expect_tx(bar_q, kTileBytes);
      b200::tma_load_3d(sQ, &tmq, bar_q, 0, h, start + m0);
      b200::tma_load_3d(sQ + kBlockBytes, &tmq, bar_q, 64, h, start + m0);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j >= kStages && !wait_or_flag(bar_e(s), ((j >> 1) - 1) & 1, &B, a.dev_status)) break;
        const int row = start + j * kBN;
        const uint32_t dk = sK + s * kTileBytes, dv = sV + s * kTileBytes;
        b200::mbar_arrive_expect_tx(bar_k(s), kTileBytes);
        b200::tma_load_3d(dk, &tmk, bar_k(s), 0, hk, row);
        b200::tma_load_3d(dk + kBlockBytes, &tmk, bar_k(s), 64, hk, row);
        b200::mbar_arrive_expect_tx(bar_v(s), kTileBytes);
        b200::tma_load_3d(dv, &tmv, bar_v(s), 0, hk, row);
        b200::tma_load_3d(dv + kBlockBytes, &tmv, bar_v(s), 64, hk, row);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(false);
      constexpr uint32_t idO = idesc_bf16(true);
      bool ok = wait_or_flag(bar_q, 0, &B, a.dev_status);
      tc_fence_after();
      for (int j = 0; ok && j <= n_kv; ++j) {
        if (j < n_kv) {
          // ---- S(j) = Q . K_j^T into score buffer j & 1
          const int s = j & 1;
          ok = wait_or_flag(bar_k(s), (j >> 1) & 1, &B, a.dev_status);
          if (ok && j >= 2) ok = wait_or_flag(bar_sr(s), ((j >> 1) - 1) & 1, &B, a.dev_status);
          if (!ok) break;
          tc_fence_after();
          const uint32_t dS = tmem + kColS0 + s * kBN;
          const uint32_t kt = sK + s * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBlockBytes + (kk & 3) * 32;
            umma_bf16(dS, smem_desc(sQ + off, 16, 1024), smem_desc(kt + off, 16, 1024), idS,
                      kk > 0 ? 1u : 0u);
          }
          umma_commit(bar_sf(s));
        }
        if (j >= 1) {
          // ---- O += P(j-1) . V_{j-1}
          const int jp = j - 1;
          const int s = jp & 1;
          ok = wait_or_flag(bar_p, jp & 1, &B, a.dev_status);
          if (ok) ok = wait_or_flag(bar_v(s), (jp >> 1) & 1, &B, a.dev_status);
          if (!ok) break;
          tc_fence_after();
          const uint32_t vt = sV + s * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint32_t pa = sP + (kk >> 2) * kBlockBytes + (kk & 3) * 32;
            umma_bf16(tmem + kColO, smem_desc(pa, 16, 1024),
                      smem_desc(vt + kk * 16 * 128, kBlockBytes, 1024), idO,
                      (jp > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar_o);
          umma_commit(bar_e(s));
        }
      }
    }
  } else {
    // ---------------------------------------------------------- softmax
    const int r = threadIdx.x;  // query row in the tile == TMEM lane
    const int qpos = m0 + r;     // position within the sequence
    const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, wait_or_flag(bar_sf(s), (j >> 1) & 1, &B, a.dev_status));
      if (!ok) break;
      tc_fence_after();
      uint32_t xs[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tmem_ld32(tmem + lane_addr + kColS0 + s * kBN + c * 32, xs + c * 32);
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tmem_wait_ld(xs + c * 32);
      float x[kBN];
#pragma unroll
      for (int c = 0; c < kBN; ++c) x[c] = __uint_as_float(xs[c]);
      tc_fence_before();
      mbar_arrive(bar_sr(s));

      const int n0 = j * kBN;
      if (n0 + kBN - 1 > qpos || n0 + kBN > len) {
        const int lim = min(qpos + 1, len) - n0;  // keys [n0, n0 + lim) are visible
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (c >= lim) x[c] = -INFINITY;
      }
      float mx = x[0];
#pragma unroll
      for (int c = 1; c < kBN; ++c) mx = fmaxf(mx, x[c]);
      mx *= a.scale_log2;
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_used = mx;
      } else if (mx > m_used + kRescaleThreshold) {
        alpha = b200::ex2(m_used - mx);
        m_used = mx;
        rescale = true;
      }
      float rowsum = 0.f;
      uint32_t pk[kBN / 2];
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        // a fixed share of the exponentials runs on the FMA pipe so the
        // special-function unit is not the bottleneck of the tile
        const bool fma_pair = (c & (kExpFmaPeriod - 1)) < kExpFmaPairs * 2;
        const float y0 = fmaf(x[c], a.scale_log2, -m_used);
        const float y1 = fmaf(x[c + 1], a.scale_log2, -m_used);
        const float p0 = fma_pair ? b200::ex2_fma(y0) : b200::ex2(y0);
        const float p1 = fma_pair ? b200::ex2_fma(y1) : b200::ex2(y1);
        rowsum += p0 + p1;
        pk[c / 2] = b200::pack_bf16x2(p0, p1);
      }

      if (j >= 1) {
        // P buffer free and O updated by PV(j-1)
        ok = __all_sync(0xffffffffu, wait_or_flag(bar_o, (j - 1) & 1, &B, a.dev_status));
        if (!ok) break;
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: rescale the warp's rows together
        // (alpha == 1 for rows whose max did not move)
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t rr[32];
            tmem_ld32(tmem + lane_addr + kColO + c * 32, rr);
            tmem_wait_ld(rr);
#pragma unroll
            for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * alpha);
            tmem_st32(tmem + lane_addr + kColO + c * 32, rr);
          }
          tmem_wait_st();
        }
      }
      l = l * alpha + rowsum;
      // P row r into the swizzled K-major tile: 16-byte chunk g of the row
#pragma unroll
      for (int g = 0; g < kBN / 8; ++g) {
        const uint32_t addr = sP + (g >> 3) * kBlockBytes + r * 128 + (((g & 7) ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * g]),
                     "r"(pk[4 * g + 1]), "r"(pk[4 * g + 2]), "r"(pk[4 * g + 3])
                     : "memory");
      }
      b200::fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_p);
    }

    // ---- epilogue: O / l -> bf16 rows
    if (ok) ok = __all_sync(0xffffffffu, wait_or_flag(bar_o, (n_kv - 1) & 1, &B, a.dev_status));
    tc_fence_after();
    if (ok) {
      const bool live = qpos < len;
      const bool pad = !live && a.zero_pad && qpos < a.max_seqlen;
      const float inv = live ? 1.f / l : 0.f;
      __nv_bfloat16* orow =
          a.out + static_cast<int64_t>(start + qpos) * a.o_t + static_cast<int64_t>(h) * a.o_h;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_addr + kColO + c * 32, rr);
        tmem_wait_ld(rr);
        if (live || pad) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = b200::pack_bf16x2(__uint_as_float(rr[i]) * inv, __uint_as_float(rr[i + 1]) * inv);
            v.y = b200::pack_bf16x2(__uint_as_float(rr[i + 2]) * inv, __uint_as_float(rr[i + 3]) * inv);
            v.z = b200::pack_bf16x2(__uint_as_float(rr[i + 4]) * inv, __uint_as_float(rr[i + 5]) * inv);
            v.w = b200::pack_bf16x2(__uint_as_float(rr[i + 6]) * inv, __uint_as_float(rr[i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + i) = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

std::mutex g_attr_mu;
bool g_attr_done[64] = {false};

int ensure_smem_attr(int dev) {
  if (dev < 0) return B200_ERR_CUDA;
  if (dev < 64 && g_attr_done[dev]) return B200_OK;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (dev < 64 && g_attr_done[dev]) return B200_OK;
  if (cudaFuncSetAttribute(varlen_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kSmemBytes) != cudaSuccess)
    return B200_ERR_CUDA;
  if (dev < 64) g_attr_done[dev] = true;
  return B200_OK;
}

bool mult8(int64_t s) { return (s & 7) == 0; }

int encode_rows_map(CUtensorMap* map, const void* base, int heads, int tokens, int64_t stride_t,
                    int64_t stride_h) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(tokens)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_h) * 2,
                                 static_cast<cuuint64_t>(stride_t) * 2};
  const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kBM)};
  const cuuint32_t es[3] = {1, 1, 1};
  return b200host::encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
                                dims, strides, box, es, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B) == CUDA_SUCCESS
             ? B200_OK
             : B200_ERR_TENSOR_MAP;
}

}  // namespace

extern "C" int b200_varlen_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                                   const void* k, int64_t k_stride_t, int64_t k_stride_h,
                                   const void* v, int64_t v_stride_t, int64_t v_stride_h,
                                   void* out, int64_t o_stride_t, int64_t o_stride_h,
                                   const int32_t* cu_seqlens, const int32_t* seq_lens_opt,
                                   int num_seqs, int total_tokens, int max_seqlen, int num_heads,
                                   int num_kv_heads, int head_dim, float scale, int zero_pad_rows,
                                   int32_t* dev_status, void* stream) {
  if (num_seqs < 0 || total_tokens < 0 || max_seqlen < 0 || num_heads <= 0 || num_kv_heads <= 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || total_tokens == 0 || max_seqlen == 0) return B200_OK;
  if (!q || !k || !v || !out || !cu_seqlens) return B200_ERR_INVALID_ARGUMENT;
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (num_heads % num_kv_heads != 0) return B200_ERR_INVALID_ARGUMENT;
  if (num_heads > 65535 || num_seqs > 65535) return B200_ERR_INVALID_ARGUMENT;
  if (!b200host::aligned16(q) || !b200host::aligned16(k) || !b200host::aligned16(v) ||
      !b200host::aligned16(out))
    return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {q_stride_t, q_stride_h, k_stride_t, k_stride_h,
                             v_stride_t, v_stride_h, o_stride_t, o_stride_h};
  for (int64_t s : strides)
    if (!mult8(s)) return B200_ERR_ALIGNMENT;

  CUtensorMap tq, tk, tv;
  int st = encode_rows_map(&tq, q, num_heads, total_tokens, q_stride_t, q_stride_h);
  if (st == B200_OK) st = encode_rows_map(&tk, k, num_kv_heads, total_tokens, k_stride_t, k_stride_h);
  if (st == B200_OK) st = encode_rows_map(&tv, v, num_kv_heads, total_tokens, v_stride_t, v_stride_h);
  if (st != B200_OK) return st;

  PrefillArgs a;
  a.cu = cu_seqlens;
  a.lens = seq_lens_opt;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_t = o_stride_t;
  a.o_h = o_stride_h;
  a.num_seqs = num_seqs;
  a.num_heads = num_heads;
  a.group = num_heads / num_kv_heads;
  a.max_seqlen = max_seqlen;
  a.zero_pad = zero_pad_rows != 0;
  a.scale_log2 = scale * kLog2e;
  a.dev_status = dev_status;

  st = ensure_smem_attr(b200host::current_device());
  if (st != B200_OK) return st;
  dim3 grid(static_cast<unsigned>((max_seqlen + kBM - 1) / kBM), static_cast<unsigned>(num_heads),
            static_cast<unsigned>(num_seqs));
  varlen_prefill_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(tq, tk,
                                                                                            tv, a);
  return b200host::status_from_cuda(cudaGetLastError());
}
