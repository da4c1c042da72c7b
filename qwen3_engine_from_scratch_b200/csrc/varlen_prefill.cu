// Varlen causal prefill attention for sm_100a on the 5th-generation tensor
// cores (tcgen05 + TMEM), fed by TMA.  Replaces flash_attention_varlen_kernel
// (qwen3/kernels/flash_attention_varlen.py:25-123) and its host entry (:126-194).
//
// Persistent: two CTAs per SM (about 110 KB shared memory, 256 TMEM columns
// each) loop over work items -- a 128-query tile of one query head of one
// sequence.  Every CTA builds the same work list in shared memory: only the
// non-empty tiles, heaviest first (tile index descending, sequences sorted by
// length), and takes items from a global counter (dynamic balance) or, without
// one, in a fixed boustrophedon order.  One CTA's softmax overlaps the other's
// tensor-core work, and an item's Q load and epilogue overlap its neighbours'
// pipeline.
//   warp 4      TMA producer: lane 0 loads the Q tile once, then K tiles of
//               64 keys into a 2-stage ring, each stage refilled as soon as
//               its S = Q.K^T is done; lane 1 streams the V tiles, each stage
//               refilled after its P.V (two 64-column boxes per tile,
//               128-byte swizzle).
//   warp 5      MMA issuer (one thread): S = Q.K^T (M=128, N=64, K=16 per
//               instruction, 8 instructions) into one of two TMEM score
//               buffers, O += P.V (M=128, N=128, 4 instructions) with P read
//               from TMEM; each group ends with tcgen05.commit on an mbarrier.
//   warps 0-3   softmax: thread r owns query row r (TMEM lane r); it loads its
//               64 scores with tcgen05.ld, applies the causal / length mask,
//               updates the running max (base 2) and sum in fp32 with tree
//               reductions, and writes P as packed bf16 pairs over the first
//               32 columns of the same score buffer (tcgen05.st).  Its O row
//               in TMEM is rescaled only when the running max grew by more
//               than 2^8 (otherwise the stale max keeps every P <= 2^8).
// KV tiles strictly above the diagonal are never loaded (the reference
// computes every KV block of the sequence, flash_attention_varlen.py:74-77).
//
// Operand layouts (UMMA canonical forms):
//   Q (128 x 128 d), K (64 x 128 d)  K-major, 128B swizzle: two blocks of
//         [row][64 d]; descriptor SBO = 1024 B (8 rows), start += 32 B per K
//         step inside a block, += block size between blocks.
//   P     A operand in TMEM: lane = query row, column c = keys 2c, 2c+1.
//   V (64 keys x 128 d)  MN-major (d contiguous), 128B swizzle: LBO = 8 KB
//         between the two 64-d blocks, SBO = 1024 B (8 keys), start += 2 KB
//         (16 keys) per K step.
//   TMEM  columns [0,64) S0/P0, [64,128) S1/P1, [128,256) O; lane = query row.
// MMAs issued by the one MMA thread execute in order, so S(j+2) overwriting
// buffer j&1 follows the P.V that read P(j) from it.
// Every mbarrier wait is bounded; TMEM is always freed before the CTA exits.
#include <math.h>

#include <stdlib.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr int kD = 128;
constexpr int kBM = 128;
constexpr int kBN = 64;
constexpr int kStages = 2;
constexpr int kQBytes = kBM * kD * 2;       // 32 KB
constexpr int kQBlock = kQBytes / 2;        // 16 KB: [128 rows][64 d] swizzled block
constexpr int kKVBytes = kBN * kD * 2;      // 16 KB per K (or V) tile
constexpr int kKVBlock = kKVBytes / 2;      // 8 KB: [64 rows][64 d]
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;
constexpr int kOffV = kOffK + kStages * kKVBytes;
constexpr int kSmemTiles = kOffV + kStages * kKVBytes;  // 96 KB
constexpr int kSmemBytes = kSmemTiles + 1024;
constexpr int kThreads = 192;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS0 = 0, kColO = 2 * kBN;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Of every kExpFmaPeriod columns, the first 2 * FMA_PAIRS (kernel template
// parameter) use ex2_fma; the rest use the special-function unit.
constexpr int kExpFmaPeriod = 8;
constexpr int kDefaultExpFmaPairs = 0;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxSeqs = 256;               // sequences per launch (the host splits larger batches)
constexpr int kMaxTiles = 2048;             // 128-query tiles per sequence (max_seqlen <= 262144)
constexpr int kRing = 4;                    // item-index ring between the scheduler and the roles
constexpr int kRingConsumers = 2 + 128;     // V lane, MMA thread, softmax threads

struct PrefillArgs {
  const int32_t* cu;
  const int32_t* lens;  // nullable
  __nv_bfloat16* out;
  int64_t o_t, o_h;
  int num_seqs, num_heads, group, max_seqlen, zero_pad, total_tokens;
  int n_tiles;          // ceil(max_seqlen / 128)
  float scale_log2;
  int32_t* dev_status;
  int32_t* sched;       // nullable: [0] next item, [1] CTAs done (zero at launch, reset at exit)
};

// Work list shared by every CTA (each CTA builds the same one in shared
// memory): the non-empty (tile, sequence, head) items, heaviest first -- tile
// index descending (tile m attends to about 2m+2 K/V tiles of 64 keys),
// sequences in descending order of their tile count, so the sequences that
// reach tile m are a prefix of the sorted order.
struct WorkList {
  int len[kMaxSeqs];
  int start[kMaxSeqs];
  uint32_t key[kMaxSeqs];        // sorted: (kMaxTiles - 1 - tiles) << 16 | sequence
  int prefix[kMaxTiles + 1];     // items before step u (tile n_tiles - 1 - u)
  int pad_prefix[kMaxSeqs + 1];  // padded adapter: zero rows before sequence s (all heads)
  unsigned char pad_ok[kMaxSeqs];  // rows [len, max_seqlen) of sequence s lie inside the output
  int n_items;
  int ring[kRing];
};

struct Item {
  int start, len, m0, h, hk, n_kv;
};

B200_DEVICE Item decode_item(const PrefillArgs& a, const WorkList& W, int k) {
  int lo = 0, hi = a.n_tiles;  // step u: largest with prefix[u] <= k
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (W.prefix[mid] <= k) lo = mid; else hi = mid;
  }
  const int rem = k - W.prefix[lo];
  const int rank = rem / a.num_heads;
  Item it;
  it.h = rem - rank * a.num_heads;
  it.hk = it.h / a.group;
  const int seq = static_cast<int>(W.key[rank] & 0xFFFFu);
  it.start = W.start[seq];
  it.len = W.len[seq];
  it.m0 = (a.n_tiles - 1 - lo) * kBM;
  it.n_kv = (min(it.len, it.m0 + kBM) + kBN - 1) / kBN;  // causal: keys < m0 + 128
  return it;
}

// Every barrier below completes once per use of its slot.  A waiter asks for
// the n-th completion with parity (n >> 1) & 1 of slot n & 1 (or parity n & 1
// for single-slot barriers); the pipeline order guarantees that slot has not
// run two completions ahead of any waiter, so parities are unambiguous.
struct __align__(8) Barriers {
  uint64_t q_full, q_empty;   // Q tile loaded / all S of its item issued and done
  uint64_t k_full[kStages];
  uint64_t v_full[kStages];
  uint64_t k_empty[kStages];  // K stage free: its S = Q.K^T finished
  uint64_t v_empty[kStages];  // V stage free: its P.V finished
  uint64_t s_full[2];         // S(g) in TMEM buffer g & 1
  uint64_t p_full[2];         // P(g) written over S(g)
  uint64_t pv_done[2];        // P(g).V(g) finished
  uint64_t o_free;            // the item's O was read by the softmax warps
  uint64_t ring_full[kRing], ring_empty[kRing];
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

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M=128, N=n.
constexpr uint32_t idesc_bf16(uint32_t n, bool b_mn_major) {
  return (1u << 4)                     // D format f32
         | (1u << 7)                   // A format bf16
         | (1u << 10)                  // B format bf16
         | (0u << 15)                  // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)
         | ((n >> 3) << 17)                              // N >> 3
         | ((static_cast<uint32_t>(kBM) >> 4) << 24);    // M >> 4
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

// A operand from TMEM (lane = row, each column two K elements), B from smem.
B200_DEVICE void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
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

// Build the work list (every CTA computes the same one).  All threads call.
B200_DEVICE void build_work_list(const PrefillArgs& a, WorkList& W) {
  const int n = a.num_seqs;
  int p2 = 1;
  while (p2 < n) p2 <<= 1;
  for (int s = threadIdx.x; s < p2; s += kThreads) {
    if (s < n) {
      const int start = a.cu[s];
      int len = a.lens != nullptr ? a.lens[s] : a.cu[s + 1] - start;
      const int rows = a.zero_pad ? a.max_seqlen : len;  // rows this sequence writes
      const bool bad = len < 0 || len > a.max_seqlen || start < 0 ||
                       static_cast<int64_t>(start) + rows > a.total_tokens;
      if (bad) {
        b200::flag_error(a.dev_status, B200_DEV_SEQ_OVERFLOW);
        len = 0;
      }
      W.start[s] = start;
      W.len[s] = len;
      W.pad_ok[s] = bad ? 0 : 1;
      const int nt = (len + kBM - 1) / kBM;
      W.key[s] = (static_cast<uint32_t>(kMaxTiles - 1 - nt) << 16) | static_cast<uint32_t>(s);
    } else {
      W.key[s] = 0xFFFFFFFFu;
    }
  }
  __syncthreads();
  // bitonic sort, ascending key = descending tile count, then sequence id
  for (int k = 2; k <= p2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < p2; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint32_t x = W.key[i], y = W.key[ixj];
          if ((x > y) == ((i & k) == 0)) {
            W.key[i] = y;
            W.key[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    // prefix over steps u (tile m = n_tiles - 1 - u): sequences with more than
    // m tiles are the first `cnt` of the sorted order
    int cnt = 0, acc = 0;
    for (int u = 0; u < a.n_tiles; ++u) {
      const int m = a.n_tiles - 1 - u;
      while (cnt < n && static_cast<int>(kMaxTiles - 1 - (W.key[cnt] >> 16)) > m) ++cnt;
      W.prefix[u] = acc;
      acc += cnt * a.num_heads;
    }
    W.prefix[a.n_tiles] = acc;
    W.n_items = acc;
    int pad = 0;
    for (int s2 = 0; s2 < n; ++s2) {
      W.pad_prefix[s2] = pad;
      pad += a.zero_pad && W.pad_ok[s2] ? (a.max_seqlen - W.len[s2]) * a.num_heads : 0;
    }
    W.pad_prefix[n] = pad;
  }
  __syncthreads();
}

template <int FMA_PAIRS>
__global__ void __launch_bounds__(kThreads, 2)
    varlen_prefill_kernel(const __grid_constant__ CUtensorMap tmq,
                          const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Barriers B;
  __shared__ WorkList W;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // a pipeline already gave up: start no new work until the host clears the status
  const bool aborted =
      a.dev_status != nullptr &&
      (*reinterpret_cast<const volatile int32_t*>(a.dev_status) & B200_DEV_TIMEOUT);

  if (!aborted) {
  build_work_list(a, W);

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = b200::smem_u32(smem);
  const uint32_t sQ = sbase + kOffQ, sK = sbase + kOffK, sV = sbase + kOffV;

  const uint32_t bar_q = b200::smem_u32(&B.q_full);
  const uint32_t bar_qe = b200::smem_u32(&B.q_empty);
  auto bar_k = [&](int s) { return b200::smem_u32(&B.k_full[s]); };
  auto bar_v = [&](int s) { return b200::smem_u32(&B.v_full[s]); };
  auto bar_ke = [&](int s) { return b200::smem_u32(&B.k_empty[s]); };
  auto bar_ve = [&](int s) { return b200::smem_u32(&B.v_empty[s]); };
  auto bar_sf = [&](int g) { return b200::smem_u32(&B.s_full[g & 1]); };
  auto bar_p = [&](int g) { return b200::smem_u32(&B.p_full[g & 1]); };
  auto bar_o = [&](int g) { return b200::smem_u32(&B.pv_done[g & 1]); };
  const uint32_t bar_of = b200::smem_u32(&B.o_free);
  auto bar_rf = [&](int n) { return b200::smem_u32(&B.ring_full[n & (kRing - 1)]); };
  auto bar_re = [&](int n) { return b200::smem_u32(&B.ring_empty[n & (kRing - 1)]); };

  if (threadIdx.x == 0) {
    b200::mbar_init(bar_q, 1);
    b200::mbar_init(bar_qe, 1);
    for (int s = 0; s < kStages; ++s) {
      b200::mbar_init(bar_k(s), 1);
      b200::mbar_init(bar_v(s), 1);
      b200::mbar_init(bar_ke(s), 1);
      b200::mbar_init(bar_ve(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      b200::mbar_init(bar_sf(s), 1);
      b200::mbar_init(bar_p(s), 128);
      b200::mbar_init(bar_o(s), 1);
    }
    b200::mbar_init(bar_of, 128);
    for (int r = 0; r < kRing; ++r) {
      b200::mbar_init(bar_rf(r), 1);
      b200::mbar_init(bar_re(r), kRingConsumers);
    }
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

  // the roles read the n-th item of this CTA from the ring (-1 ends the list)
  auto next_item = [&](int n, bool& ok) -> int {
    ok = wait_or_flag(bar_rf(n), (n / kRing) & 1, &B, a.dev_status);
    const int k = ok ? W.ring[n & (kRing - 1)] : -1;
    mbar_arrive(bar_re(n));
    return k;
  };

  if (warp == kProducerWarp) {
    // lane 0 streams Q and the K tiles, lane 1 the V tiles: a K stage is
    // refilled as soon as its S = Q.K^T is done, without waiting for P.V
    if (lane == 0) {
      b200::prefetch_tensormap(&tmq);
      b200::prefetch_tensormap(&tmk);
      int kc = 0;
      bool ok = true;
      for (int n = 0; ok; ++n) {
        // scheduler: the next item from the global counter, or without one
        // the fixed boustrophedon order over the CTAs
        const int round = n / static_cast<int>(gridDim.x);
        int k = a.sched != nullptr
                    ? atomicAdd(&a.sched[0], 1)
                    : round * gridDim.x + ((round & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x);
        if (k >= W.n_items) k = -1;
        if (n >= kRing && !(ok = wait_or_flag(bar_re(n), ((n / kRing) - 1) & 1, &B, a.dev_status)))
          break;
        W.ring[n & (kRing - 1)] = k;
        mbar_arrive(bar_rf(n));
        if (k < 0) break;
        const Item it = decode_item(a, W, k);
        if (n > 0 && !(ok = wait_or_flag(bar_qe, (n - 1) & 1, &B, a.dev_status))) break;
        b200::mbar_arrive_expect_tx(bar_q, kQBytes);
        b200::tma_load_3d(sQ, &tmq, bar_q, 0, it.h, it.start + it.m0);
        b200::tma_load_3d(sQ + kQBlock, &tmq, bar_q, 64, it.h, it.start + it.m0);
        for (int j = 0; j < it.n_kv; ++j, ++kc) {
          const int s = kc & 1;
          if (kc >= kStages && !(ok = wait_or_flag(bar_ke(s), ((kc >> 1) - 1) & 1, &B, a.dev_status)))
            break;
          const uint32_t dk = sK + s * kKVBytes;
          b200::mbar_arrive_expect_tx(bar_k(s), kKVBytes);
          b200::tma_load_3d(dk, &tmk, bar_k(s), 0, it.hk, it.start + j * kBN);
          b200::tma_load_3d(dk + kKVBlock, &tmk, bar_k(s), 64, it.hk, it.start + j * kBN);
        }
      }
    } else if (lane == 1) {
      b200::prefetch_tensormap(&tmv);
      int vc = 0;
      bool ok = true;
      for (int n = 0; ok; ++n) {
        const int k = next_item(n, ok);
        if (!ok || k < 0) break;
        const Item it = decode_item(a, W, k);
        for (int j = 0; j < it.n_kv; ++j, ++vc) {
          const int s = vc & 1;
          if (vc >= kStages && !(ok = wait_or_flag(bar_ve(s), ((vc >> 1) - 1) & 1, &B, a.dev_status)))
            break;
          const uint32_t dv = sV + s * kKVBytes;
          b200::mbar_arrive_expect_tx(bar_v(s), kKVBytes);
          b200::tma_load_3d(dv, &tmv, bar_v(s), 0, it.hk, it.start + j * kBN);
          b200::tma_load_3d(dv + kKVBlock, &tmv, bar_v(s), 64, it.hk, it.start + j * kBN);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(kBN, false);
      constexpr uint32_t idO = idesc_bf16(kD, true);
      int g0 = 0;  // g = global index of S / P / P.V products in this CTA
      bool ok = true;
      for (int n_item = 0; ok; ++n_item) {
        const int k = next_item(n_item, ok);
        if (!ok || k < 0) break;
        const Item it = decode_item(a, W, k);
        if (!(ok = wait_or_flag(bar_q, n_item & 1, &B, a.dev_status))) break;
        tc_fence_after();
        for (int j = 0; j <= it.n_kv; ++j) {
          if (j < it.n_kv) {
            // ---- S(g) = Q . K^T into buffer g & 1 (it last held P(g-2), whose
            // P.V was issued before this point; MMAs execute in issue order)
            const int g = g0 + j;
            const int s = g & 1;
            if (!(ok = wait_or_flag(bar_k(s), (g >> 1) & 1, &B, a.dev_status))) break;
            tc_fence_after();
            const uint32_t dS = tmem + kColS0 + s * kBN;
            const uint32_t kt = sK + s * kKVBytes;
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t inblk = (kk & 3) * 32;
              umma_bf16(dS, smem_desc(sQ + (kk >> 2) * kQBlock + inblk, 16, 1024),
                        smem_desc(kt + (kk >> 2) * kKVBlock + inblk, 16, 1024), idS,
                        kk > 0 ? 1u : 0u);
            }
            umma_commit(bar_sf(g));
            umma_commit(bar_ke(s));
            if (j == it.n_kv - 1) umma_commit(bar_qe);
          }
          if (j >= 1) {
            // ---- O += P(g) . V(g), P from TMEM
            const int g = g0 + j - 1;
            const int s = g & 1;
            if (!(ok = wait_or_flag(bar_p(g), (g >> 1) & 1, &B, a.dev_status))) break;
            if (!(ok = wait_or_flag(bar_v(s), (g >> 1) & 1, &B, a.dev_status))) break;
            if (j == 1 && n_item > 0 &&
                !(ok = wait_or_flag(bar_of, (n_item - 1) & 1, &B, a.dev_status)))
              break;
            tc_fence_after();
            const uint32_t vt = sV + s * kKVBytes;
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk) {
              umma_bf16_ts(tmem + kColO, tmem + kColS0 + s * kBN + kk * 8,
                           smem_desc(vt + kk * 16 * 128, kKVBlock, 1024), idO,
                           (j > 1 || kk > 0) ? 1u : 0u);
            }
            umma_commit(bar_o(g));
            umma_commit(bar_ve(s));
          }
        }
        g0 += it.n_kv;
      }
    }
  } else {
    // ---------------------------------------------------------- softmax
    const int r = threadIdx.x;  // query row in the tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;

    // padded adapter: zero the rows past every sequence (spread over all CTAs)
    if (a.zero_pad) {
      const int total = W.pad_prefix[a.num_seqs];
      for (int z = blockIdx.x * 128 + r; z < total; z += gridDim.x * 128) {
        int lo = 0, hi = a.num_seqs;
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (W.pad_prefix[mid] <= z) lo = mid; else hi = mid;
        }
        const int rem = z - W.pad_prefix[lo];
        const int pad_rows = a.max_seqlen - W.len[lo];
        const int hh = rem / pad_rows;
        const int row = W.len[lo] + (rem - hh * pad_rows);
        __nv_bfloat16* orow = a.out + static_cast<int64_t>(W.start[lo] + row) * a.o_t +
                              static_cast<int64_t>(hh) * a.o_h;
#pragma unroll
        for (int c = 0; c < kD; c += 8)
          *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
      }
    }

    int g0 = 0;
    bool ok = true;
    for (int n = 0; ok; ++n) {
      const int k = next_item(n, ok);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || k < 0) break;
      const Item it = decode_item(a, W, k);
      const int qpos = it.m0 + r;  // position within the sequence
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j) {
        const int g = g0 + j;
        const int s = g & 1;
        ok = __all_sync(0xffffffffu, wait_or_flag(bar_sf(g), (g >> 1) & 1, &B, a.dev_status));
        if (!ok) break;
        tc_fence_after();
        const uint32_t sbuf = tmem + lane_addr + kColS0 + s * kBN;
        uint32_t xs[kBN];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_ld32(sbuf + c * 32, xs + c * 32);
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_wait_ld(xs + c * 32);
        float x[kBN];
#pragma unroll
        for (int c = 0; c < kBN; ++c) x[c] = __uint_as_float(xs[c]);

        const int n0 = j * kBN;
        if (n0 + kBN - 1 > qpos || n0 + kBN > it.len) {
          const int lim = min(qpos + 1, it.len) - n0;  // keys [n0, n0 + lim) are visible
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (c >= lim) x[c] = -INFINITY;
        }
        // tree max (8 independent chains)
        float mq[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mq[e] = x[e];
#pragma unroll
        for (int c = 8; c < kBN; ++c) mq[c & 7] = fmaxf(mq[c & 7], x[c]);
        const float mx = fmaxf(fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])),
                               fmaxf(fmaxf(mq[4], mq[5]), fmaxf(mq[6], mq[7]))) *
                         a.scale_log2;
        float alpha = 1.f;
        bool rescale = false;
        if (j == 0) {
          m_used = mx;
        } else if (mx > m_used + kRescaleThreshold) {
          alpha = b200::ex2(m_used - mx);
          m_used = mx;
          rescale = true;
        }
        float sq[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        uint32_t pk[kBN / 2];
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          // a fixed share of the exponentials runs on the FMA pipe
          const bool fma_pair = (c & (kExpFmaPeriod - 1)) < FMA_PAIRS * 2;
          const float y0 = fmaf(x[c], a.scale_log2, -m_used);
          const float y1 = fmaf(x[c + 1], a.scale_log2, -m_used);
          const float p0 = fma_pair ? b200::ex2_fma(y0) : b200::ex2(y0);
          const float p1 = fma_pair ? b200::ex2_fma(y1) : b200::ex2(y1);
          sq[(c >> 1) & 7] += p0 + p1;
          pk[c / 2] = b200::pack_bf16x2(p0, p1);
        }
        const float rowsum =
            ((sq[0] + sq[1]) + (sq[2] + sq[3])) + ((sq[4] + sq[5]) + (sq[6] + sq[7]));

        // P(g) over the first half of its own score buffer (S(g) is consumed)
        tmem_st32(sbuf, pk);
        if (__any_sync(0xffffffffu, rescale)) {
          // O must hold everything up to P(g-1).V(g-1) before it is rescaled;
          // tcgen05.ld/st are warp-collective, so the warp's rows rescale
          // together (alpha == 1 for rows whose max did not move)
          ok = __all_sync(0xffffffffu, wait_or_flag(bar_o(g - 1), ((g - 1) >> 1) & 1, &B,
                                                    a.dev_status));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t rr[32];
            tmem_ld32(tmem + lane_addr + kColO + c * 32, rr);
            tmem_wait_ld(rr);
#pragma unroll
            for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
            tmem_st32(tmem + lane_addr + kColO + c * 32, rr);
          }
        }
        l = l * alpha + rowsum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p(g));
      }
      if (!ok) break;

      // ---- epilogue: O / l -> bf16 rows; O is released before the stores
      const int glast = g0 + it.n_kv - 1;
      ok = __all_sync(0xffffffffu,
                      wait_or_flag(bar_o(glast), (glast >> 1) & 1, &B, a.dev_status));
      if (!ok) break;
      tc_fence_after();
      uint32_t ov[kD];
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) tmem_ld32(tmem + lane_addr + kColO + c * 32, ov + c * 32);
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) tmem_wait_ld(ov + c * 32);
      tc_fence_before();
      mbar_arrive(bar_of);
      if (qpos < it.len) {  // rows past the sequence are zeroed by the pass above
        const float inv = 1.f / l;
        __nv_bfloat16* orow = a.out + static_cast<int64_t>(it.start + qpos) * a.o_t +
                              static_cast<int64_t>(it.h) * a.o_h;
#pragma unroll
        for (int e = 0; e < kD; e += 8) {
          uint4 v;
          v.x = b200::pack_bf16x2(__uint_as_float(ov[e]) * inv, __uint_as_float(ov[e + 1]) * inv);
          v.y = b200::pack_bf16x2(__uint_as_float(ov[e + 2]) * inv, __uint_as_float(ov[e + 3]) * inv);
          v.z = b200::pack_bf16x2(__uint_as_float(ov[e + 4]) * inv, __uint_as_float(ov[e + 5]) * inv);
          v.w = b200::pack_bf16x2(__uint_as_float(ov[e + 6]) * inv, __uint_as_float(ov[e + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + e) = v;
        }
      }
      g0 += it.n_kv;
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
  }  // !aborted

  // the last CTA to finish leaves the schedule counter zeroed for the next launch
  if (a.sched != nullptr && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.sched[1], 1) == static_cast<int>(gridDim.x) - 1) {
      atomicExch(&a.sched[0], 0);
      atomicExch(&a.sched[1], 0);
    }
  }
}

std::mutex g_attr_mu;
bool g_attr_done[64] = {false};

template <int P>
cudaError_t set_smem_attr() {
  return cudaFuncSetAttribute(varlen_prefill_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSmemBytes);
}

int ensure_smem_attr(int dev) {
  if (dev < 0) return B200_ERR_CUDA;
  if (dev < 64 && g_attr_done[dev]) return B200_OK;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (dev < 64 && g_attr_done[dev]) return B200_OK;
  if (set_smem_attr<0>() != cudaSuccess || set_smem_attr<1>() != cudaSuccess ||
      set_smem_attr<2>() != cudaSuccess || set_smem_attr<3>() != cudaSuccess ||
      set_smem_attr<4>() != cudaSuccess)
    return B200_ERR_CUDA;
  if (dev < 64) g_attr_done[dev] = true;
  return B200_OK;
}

// Share of the softmax exponentials evaluated on the FMA pipe, in pairs of
// every 8 columns (0..4); B200_PREFILL_EXP_FMA_PAIRS overrides the default
// for tuning.
int exp_fma_pairs() {
  static const int v = [] {
    const char* e = getenv("B200_PREFILL_EXP_FMA_PAIRS");
    if (e == nullptr || *e < '0' || *e > '4' || e[1] != 0) return kDefaultExpFmaPairs;
    return *e - '0';
  }();
  return v;
}

bool mult8(int64_t s) { return (s & 7) == 0; }

int encode_rows_map(CUtensorMap* map, const void* base, int heads, int tokens, int64_t stride_t,
                    int64_t stride_h, int box_rows) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(tokens)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_h) * 2,
                                 static_cast<cuuint64_t>(stride_t) * 2};
  const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(box_rows)};
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
                                   int32_t* work_counter, int32_t* dev_status, void* stream) {
  if (num_seqs < 0 || total_tokens < 0 || max_seqlen < 0 || num_heads <= 0 || num_kv_heads <= 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || total_tokens == 0 || max_seqlen == 0) return B200_OK;
  if (!q || !k || !v || !out || !cu_seqlens) return B200_ERR_INVALID_ARGUMENT;
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (num_heads % num_kv_heads != 0) return B200_ERR_INVALID_ARGUMENT;
  const int n_tiles = (max_seqlen + kBM - 1) / kBM;
  if (n_tiles > kMaxTiles) return B200_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(n_tiles) * kMaxSeqs * num_heads > 0x7fffffff)
    return B200_ERR_INVALID_ARGUMENT;
  if (!b200host::aligned16(q) || !b200host::aligned16(k) || !b200host::aligned16(v) ||
      !b200host::aligned16(out))
    return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {q_stride_t, q_stride_h, k_stride_t, k_stride_h,
                             v_stride_t, v_stride_h, o_stride_t, o_stride_h};
  for (int64_t s : strides)
    if (!mult8(s)) return B200_ERR_ALIGNMENT;

  CUtensorMap tq, tk, tv;
  int st = encode_rows_map(&tq, q, num_heads, total_tokens, q_stride_t, q_stride_h, kBM);
  if (st == B200_OK)
    st = encode_rows_map(&tk, k, num_kv_heads, total_tokens, k_stride_t, k_stride_h, kBN);
  if (st == B200_OK)
    st = encode_rows_map(&tv, v, num_kv_heads, total_tokens, v_stride_t, v_stride_h, kBN);
  if (st != B200_OK) return st;

  st = ensure_smem_attr(b200host::current_device());
  if (st != B200_OK) return st;
  const int sms = b200host::sm_count(b200host::current_device());
  if (sms <= 0) return B200_ERR_CUDA;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int pairs = exp_fma_pairs();

  // sequences are independent: launch at most kMaxSeqs of them at a time
  for (int s0 = 0; s0 < num_seqs; s0 += kMaxSeqs) {
    PrefillArgs a;
    a.cu = cu_seqlens + s0;
    a.lens = seq_lens_opt != nullptr ? seq_lens_opt + s0 : nullptr;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.o_t = o_stride_t;
    a.o_h = o_stride_h;
    a.num_seqs = num_seqs - s0 < kMaxSeqs ? num_seqs - s0 : kMaxSeqs;
    a.num_heads = num_heads;
    a.group = num_heads / num_kv_heads;
    a.max_seqlen = max_seqlen;
    a.zero_pad = zero_pad_rows != 0;
    a.total_tokens = total_tokens;
    a.n_tiles = n_tiles;
    a.scale_log2 = scale * kLog2e;
    a.dev_status = dev_status;
    a.sched = work_counter;
    dim3 grid(static_cast<unsigned>(2 * sms));  // two persistent CTAs per SM
    switch (pairs) {
      case 0: varlen_prefill_kernel<0><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, a); break;
      case 2: varlen_prefill_kernel<2><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, a); break;
      case 3: varlen_prefill_kernel<3><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, a); break;
      case 4: varlen_prefill_kernel<4><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, a); break;
      default: varlen_prefill_kernel<1><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, a); break;
    }
    st = b200host::status_from_cuda(cudaGetLastError());
    if (st != B200_OK) return st;
  }
  return B200_OK;
}
