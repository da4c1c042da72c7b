// Varlen causal prefill attention for sm_100a on the 5th-generation tensor
// cores (tcgen05 + TMEM), fed by TMA.  Replaces flash_attention_varlen_kernel
// (qwen3/kernels/flash_attention_varlen.py:25-123) and its host entry (:126-194).
//
// Persistent, one CTA per SM (192 KB of tiles in shared memory, all 512 TMEM
// columns, 12 warps).  A work item is a PAIR of 128-row query tiles that read the same
// K/V rows: two query heads of one kv head at the same positions (GQA group
// even), or two consecutive row tiles of one head (group odd).  Each 128-key
// K/V tile is loaded once for both.  The two tiles ping-pong: while the
// softmax warps of one tile work on its scores, the tensor core computes the
// other tile's P.V and next S.
//   warps 0-3 / 4-7  softmax of tile 0 / tile 1: thread r owns query row r
//               (TMEM lane r); it loads its 128 scores with tcgen05.ld, applies
//               the causal / length mask, updates the running max (base 2) and
//               sum in fp32, and writes P as packed bf16 pairs over the first
//               64 columns of the same score buffer (tcgen05.st).  Its O row
//               is rescaled only when the running max grew by more than 2^8
//               (otherwise the stale max keeps every P <= 2^8).  After the
//               item's last tile the same warps normalise O: a full tile is
//               staged in the freed stage of the item's last K (tile 0) or V
//               (tile 1) tile for the store lane, the sequence's ragged last
//               tile (and every tile in paged mode) is stored row by row.
//   warp 8      MMA issuer (one thread): S_t = Q_t.K^T (M=128, N=128, K=16
//               per instruction, 8 instructions), O_t += P_t.V (M=128,
//               N=128, 8 instructions) with P_t read from TMEM; each group
//               ends with tcgen05.commit on an mbarrier.
//   warp 9      TMA producer (lane 0): takes the work items and loads both Q
//               tiles and the K tiles (2-stage ring)
//   warp 10     V tiles (lane 0)
//   warp 11     store lane (lane 0, not in paged mode): writes the staged
//               output tiles with TMA stores and returns their stages.
//               The loads and stores sit in warps of their own so that one
//               lane's waits never hold up another's (paged mode: 640 -> 702
//               TFLOP/s); the softmax warpgroups (warps 0-7) raise their
//               registers to 216 with setmaxnreg while warps 8-11 drop to 64
//               (256 x 216 + 128 x 64 = 63,488 of the 384 x 168 the block is
//               launched with), which keeps the softmax free of spills.
// Every CTA builds the same work list in shared memory: only the non-empty
// items, sequence-major (longest sequence first), heaviest tile first within
// a sequence; items are taken from a global counter (dynamic balance) or,
// without one, in a fixed boustrophedon order.  The scheduler lane decodes
// each item once and passes its fields to the other roles through a 4-slot
// ring in shared memory.  KV tiles strictly above the
// diagonal are never loaded (the reference computes every KV block of the
// sequence, flash_attention_varlen.py:74-77).
//
// Operand layouts (UMMA canonical forms):
//   Q (128 x 128 d), K (128 x 128 d)  K-major, 128B swizzle: two blocks of
//         [row][64 d]; descriptor SBO = 1024 B (8 rows), start += 32 B per K
//         step inside a block, += block size between blocks.
//   P     A operand in TMEM: lane = query row, column c = keys 2c, 2c+1.
//   V (128 keys x 128 d)  MN-major (d contiguous), 128B swizzle: LBO = 16 KB
//         between the two 64-d blocks, SBO = 1024 B (8 keys), start += 2 KB
//         (16 keys) per K step.  Paged mode: one 4 KB block per page
//         ([d half][16 keys][64 d]), LBO = 2 KB, start += 4 KB per K step.
//   TMEM  columns [0,128) S0/P0, [128,256) S1/P1, [256,384) O0, [384,512) O1;
//         lane = query row.
// MMAs issued by the one MMA thread execute in order, so S_t(j+1) overwriting
// P_t(j) follows the P_t(j).V that read it, and the commit that announces
// S_t(j+1) also covers that P.V (O_t is stable while its softmax rescales it).
// Every mbarrier wait is bounded; TMEM is always freed before the CTA exits.
#include <math.h>

#include <stdlib.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr int kD = 128;
constexpr int kBM = 128;                    // query rows per tile (one TMEM lane each)
constexpr int kBN = 128;                    // keys per K/V tile
constexpr int kStages = 2;                  // K (and V) tile ring depth
constexpr int kQBytes = kBM * kD * 2;       // 32 KB per Q tile
constexpr int kQBlock = kQBytes / 2;        // 16 KB: [128 rows][64 d] swizzled block
constexpr int kKVBytes = kBN * kD * 2;      // 32 KB per K (or V) tile
constexpr int kKVBlock = kKVBytes / 2;      // 16 KB: [128 keys][64 d]
constexpr int kOffQ = 0;                    // Q of tile 0, then tile 1
constexpr int kOffK = kOffQ + 2 * kQBytes;
constexpr int kOffV = kOffK + kStages * kKVBytes;
constexpr int kSmemTiles = kOffV + kStages * kKVBytes;  // 192 KB
constexpr int kSmemBytes = kSmemTiles + 1024;
constexpr int kThreads = 384;
constexpr int kSoftmaxThreads = 256;
constexpr int kMmaWarp = 8;
constexpr int kProducerWarp = 9;   // Q/K loads and the scheduler
constexpr int kVWarp = 10;          // V loads
constexpr int kStoreWarp = 11;      // output TMA stores
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 2 * kBN;  // + tile * 128
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Of every kExpFmaPeriod columns, the first 2 * FMA_PAIRS (kernel template
// parameter) use the FMA-pipe exp2; the rest use the special-function unit.
// In isolation a quarter on the FMA pipe is fastest, but inside this kernel
// the extra instructions delay the MMA warp that shares their SM sub-partition,
// so the default keeps every exponential on the special-function unit.
constexpr int kExpFmaPeriod = 16;
constexpr int kDefaultExpFmaPairs = 0;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxSeqs = 256;               // sequences per launch (the host splits larger batches)
constexpr int kMaxTiles = 2048;             // 128-row tiles per sequence (max_seqlen <= 262144)
constexpr int kRing = 4;                    // item-index ring between the scheduler and the roles
// V lane, store lane, MMA thread, softmax threads
constexpr int kRingConsumers = 3 + kSoftmaxThreads;

struct PrefillArgs {
  const int32_t* cu;
  const int32_t* lens;  // nullable
  __nv_bfloat16* out;
  int64_t o_t, o_h;
  int num_seqs, num_heads, group, max_seqlen, zero_pad, total_tokens;
  int pair_heads;       // 1: an item is query heads 2p, 2p+1 (group even); 0: two row tiles
  int out32;            // out rows 32-byte aligned (base and strides): 256-bit stores
  float scale_log2;
  int32_t* dev_status;
  int32_t* sched;       // nullable: [0] next item, [1] CTAs done (zero at launch, reset at exit)
  // paged mode (chunked prefill): the new tokens of sequence i sit at positions
  // ctx_i .. ctx_i + len_i - 1 after ctx_i = seq_lens[row_ids[i]] cached ones;
  // every key (cached and new) is read from the paged pool
  int paged;
  const int32_t* row_ids;
  const int32_t* seq_lens;
  const int32_t* block_table;
  int64_t bt_row;
  int num_blocks, max_pages, max_requests;
};

// Work list shared by every CTA (each CTA builds the same one in shared
// memory): the non-empty items, sequence-major -- sequences in descending
// order of their tile count, within a sequence the heaviest tiles first (a
// tile at row m0 attends to m0/128 + 1 K/V tiles), within a step the head
// pairs (or heads) in order.  The CTAs working at any moment then read the
// K/V of one or two sequences, which stay in L2, and the list still ends with
// its lightest items.
struct WorkList {
  int len[kMaxSeqs];
  int start[kMaxSeqs];
  int ctx[kMaxSeqs];             // cached positions before the new tokens (paged mode)
  int row[kMaxSeqs];             // pool row (paged mode)
  int qtiles[kMaxSeqs];          // 128-row query tiles of the new tokens
  uint32_t key[kMaxSeqs];        // sorted: (kMaxTiles - 1 - key tiles) << 16 | sequence
  int seq_prefix[kMaxSeqs + 1];  // items before the r-th sequence of the sorted order
  int pad_prefix[kMaxSeqs + 1];  // padded adapter: zero rows before sequence s (all heads)
  unsigned char pad_ok[kMaxSeqs];  // rows [len, max_seqlen) of sequence s lie inside the output
  int n_items;
  int ring[kRing];
};

struct Item {
  int start, len, hk, n_kv;
  int ctx, row;     // paged mode: cached positions, pool row
  int h[2], m0[2];  // query head and first row of tile 0 / tile 1
};

// Steps (heaviest first) a sequence of `tiles` row tiles contributes, and the
// items per step.
B200_DEVICE int seq_steps(const PrefillArgs& a, int tiles) {
  return a.pair_heads ? tiles : (tiles + 1) / 2;
}
B200_DEVICE int items_per_step(const PrefillArgs& a) {
  return a.pair_heads ? a.num_heads / 2 : a.num_heads;
}

B200_DEVICE Item decode_item(const PrefillArgs& a, const WorkList& W, int k) {
  int lo = 0, hi = a.num_seqs;  // rank: largest with seq_prefix[rank] <= k
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (W.seq_prefix[mid] <= k) lo = mid; else hi = mid;
  }
  const int per = items_per_step(a);
  const int rem = k - W.seq_prefix[lo];
  const int step = rem / per;
  const int p = rem - step * per;
  const int seq = static_cast<int>(W.key[lo] & 0xFFFFu);
  const int tiles = W.qtiles[seq];
  Item it;
  it.start = W.start[seq];
  it.len = W.len[seq];
  it.ctx = W.ctx[seq];
  it.row = W.row[seq];
  if (a.pair_heads) {
    it.h[0] = 2 * p;
    it.h[1] = 2 * p + 1;
    it.m0[0] = it.m0[1] = (tiles - 1 - step) * kBM;
  } else {
    it.h[0] = it.h[1] = p;
    it.m0[0] = (seq_steps(a, tiles) - 1 - step) * 2 * kBM;
    it.m0[1] = it.m0[0] + kBM;  // may lie past the sequence: computed, never stored
  }
  it.hk = it.h[0] / a.group;
  // causal: keys < ctx + m0 + 128
  it.n_kv = (it.ctx + min(it.len, it.m0[1] + kBM) + kBN - 1) / kBN;
  return it;
}

// Every barrier below completes once per use of its slot.  A waiter asks for
// the c-th completion of a slot with parity c & 1; the pipeline order
// guarantees that no slot runs two completions ahead of any of its waiters.
struct __align__(8) Barriers {
  uint64_t q_full, q_empty;   // both Q tiles loaded / every S of the item done
  uint64_t k_full[kStages], k_empty[kStages];  // K tile loaded / both S that read it done
  uint64_t v_full[kStages], v_empty[kStages];  // V tile loaded / both P.V that read it done
  uint64_t s_full[2];         // S_t(g) in TMEM (every earlier MMA of the CTA done too)
  uint64_t p_full[2];         // P_t(g) written over S_t(g), O_t rescaled
  uint64_t o_done[2];         // the item's last P_t.V done (O_t final)
  uint64_t o_free[2];         // the item's O_t was read by its softmax warps
  uint64_t staged[2][2];      // [tile][item parity]: the tile's output rows are in its stage
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

// 5-D tiled tensor load (no multicast), completing on `bar`.
B200_DEVICE void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                             int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(c4)
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

B200_DEVICE void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
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

// Paged mode: key tile j (keys [128j, 128j + 128)) of an item from the pool.
// K: 8 pages x two 64-column boxes of [16 slots][64 d] (2 KB each, stacked in
// the canonical [128 keys][64 d] blocks: the S MMA's B operand needs its
// 8-key groups at one stride across all 128 keys).  V (v_pages): one 4 KB box
// per page, [d half][16 slots][64 d], through a 5-D map whose d-half
// dimension (stride 128 B) comes after the slot dimension; each P.V MMA
// reads 16 keys, one page, so its descriptor starts at the page and steps
// 2 KB between the d halves.  Pages past the sequence repeat its last page,
// so masked keys read finite data; a bad table entry is flagged and replaced
// by block 0.
B200_DEVICE void load_kv_tile_paged(const PrefillArgs& a, const Item& it, const CUtensorMap* map,
                                    uint32_t dst, uint32_t bar, int j, bool v_pages = false) {
  const int last_page = (it.ctx + it.len - 1) / 16;
  const int32_t* bt = a.block_table + static_cast<int64_t>(it.row) * a.bt_row;
  int phys[kBN / 16];
#pragma unroll
  for (int i = 0; i < kBN / 16; ++i) {
    const int pg = min(j * (kBN / 16) + i, last_page);
    int ph = bt[pg];
    if (ph < 0 || ph >= a.num_blocks) {
      b200::flag_error(a.dev_status, B200_DEV_BAD_PAGE);
      ph = 0;
    }
    phys[i] = ph;
  }
  if (v_pages) {
#pragma unroll
    for (int i = 0; i < kBN / 16; ++i) tma_load_5d(dst + i * 4096, map, bar, 0, 0, 0, it.hk, phys[i]);
    return;
  }
#pragma unroll
  for (int i = 0; i < kBN / 16; ++i) {
    b200::tma_load_4d_nohint(dst + i * 2048, map, bar, 0, 0, it.hk, phys[i]);
    b200::tma_load_4d_nohint(dst + kKVBlock + i * 2048, map, bar, 64, 0, it.hk, phys[i]);
  }
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
      bool bad = len < 0 || len > a.max_seqlen || start < 0 ||
                 static_cast<int64_t>(start) + rows > a.total_tokens;
      int ctx = 0, row = 0;
      if (a.paged && !bad) {
        row = a.row_ids[s];
        if (row < 0 || row >= a.max_requests) {
          b200::flag_error(a.dev_status, B200_DEV_BAD_ROW);
          len = 0;
        } else {
          ctx = a.seq_lens[row];
          if (ctx < 0 || static_cast<int64_t>(ctx) + len > static_cast<int64_t>(a.max_pages) * 16 ||
              static_cast<int64_t>(ctx) + len > static_cast<int64_t>(kMaxTiles - 1) * kBN)
            bad = true;
        }
      }
      if (bad) {
        b200::flag_error(a.dev_status, B200_DEV_SEQ_OVERFLOW);
        len = 0;
        ctx = 0;
      }
      W.start[s] = start;
      W.len[s] = len;
      W.ctx[s] = ctx;
      W.row[s] = row;
      W.pad_ok[s] = bad ? 0 : 1;
      const int nt = (len + kBM - 1) / kBM;
      W.qtiles[s] = nt;
      // heaviest first: by the key tiles of the sequence's last query tile
      const int kt = len > 0 ? (ctx + len + kBN - 1) / kBN : 0;
      W.key[s] = (static_cast<uint32_t>(kMaxTiles - 1 - kt) << 16) | static_cast<uint32_t>(s);
    } else {
      W.key[s] = 0xFFFFFFFFu;
    }
  }
  __syncthreads();
  // bitonic sort, ascending key = descending tile count, then sequence id;
  // up to 32 sequences one warp sorts them in registers (no block barriers)
  const int lane = threadIdx.x & 31;
  if (p2 <= 32) {
    if (threadIdx.x < 32) {
      uint32_t v = lane < p2 ? W.key[lane] : 0xFFFFFFFFu;
      for (int k = 2; k <= 32; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
          const uint32_t o = __shfl_xor_sync(0xffffffffu, v, j);
          const bool lower = (lane & j) == 0, asc = (lane & k) == 0;
          v = (lower == asc) ? min(v, o) : max(v, o);
        }
      }
      if (lane < p2) W.key[lane] = v;
    }
  } else {
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
  }
  // items before each sequence of the sorted order, and the padded adapter's
  // zero rows before each sequence: prefix sums by one warp
  if (threadIdx.x < 32) {
    __syncwarp();
    const int per = items_per_step(a);
    int acc = 0, pad = 0;
    for (int r0 = 0; r0 < n; r0 += 32) {
      const int r = r0 + lane;
      const int v = r < n ? seq_steps(a, W.qtiles[W.key[r] & 0xFFFFu]) * per : 0;
      const int z = r < n && a.zero_pad && W.pad_ok[r] ? (a.max_seqlen - W.len[r]) * a.num_heads : 0;
      int iv = v, iz = z;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int yv = __shfl_up_sync(0xffffffffu, iv, o);
        const int yz = __shfl_up_sync(0xffffffffu, iz, o);
        if (lane >= o) {
          iv += yv;
          iz += yz;
        }
      }
      if (r < n) {
        W.seq_prefix[r] = acc + iv - v;
        W.pad_prefix[r] = pad + iz - z;
      }
      acc += __shfl_sync(0xffffffffu, iv, 31);
      pad += __shfl_sync(0xffffffffu, iz, 31);
    }
    if (lane == 0) {
      W.seq_prefix[n] = acc;
      W.n_items = acc;
      W.pad_prefix[n] = pad;
    }
  }
  __syncthreads();
}

template <int FMA_PAIRS>
__global__ void __launch_bounds__(kThreads, 1)
    varlen_prefill_kernel(const __grid_constant__ CUtensorMap tmq,
                          const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv,
                          const __grid_constant__ CUtensorMap tmo, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Barriers B;
  __shared__ WorkList W;
  __shared__ Item ring_item[kRing];  // the decoded items of the ring's slots

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
  auto bar_ke = [&](int s) { return b200::smem_u32(&B.k_empty[s]); };
  auto bar_v = [&](int s) { return b200::smem_u32(&B.v_full[s]); };
  auto bar_ve = [&](int s) { return b200::smem_u32(&B.v_empty[s]); };
  auto bar_sf = [&](int t) { return b200::smem_u32(&B.s_full[t]); };
  auto bar_p = [&](int t) { return b200::smem_u32(&B.p_full[t]); };
  auto bar_od = [&](int t) { return b200::smem_u32(&B.o_done[t]); };
  auto bar_of = [&](int t) { return b200::smem_u32(&B.o_free[t]); };
  auto bar_st = [&](int t, int n) { return b200::smem_u32(&B.staged[t][n & 1]); };
  auto bar_rf = [&](int n) { return b200::smem_u32(&B.ring_full[n & (kRing - 1)]); };
  auto bar_re = [&](int n) { return b200::smem_u32(&B.ring_empty[n & (kRing - 1)]); };

  if (threadIdx.x == 0) {
    b200::mbar_init(bar_q, 1);
    b200::mbar_init(bar_qe, 1);
    for (int s = 0; s < kStages; ++s) {
      b200::mbar_init(bar_k(s), 1);
      b200::mbar_init(bar_ke(s), 1);
      b200::mbar_init(bar_v(s), 1);
      b200::mbar_init(bar_ve(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      b200::mbar_init(bar_sf(t), 1);
      b200::mbar_init(bar_p(t), 128);
      b200::mbar_init(bar_od(t), 1);
      b200::mbar_init(bar_of(t), 128);
      b200::mbar_init(bar_st(t, 0), 128);
      b200::mbar_init(bar_st(t, 1), 128);
    }
    for (int r = 0; r < kRing; ++r) {
      b200::mbar_init(bar_rf(r), 1);
      // (paged mode: the store lane has no work and does not read the ring)
      b200::mbar_init(bar_re(r), a.paged ? kRingConsumers - 1 : kRingConsumers);
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


  // the roles read the n-th item of this CTA from the ring, index and fields
  // as the scheduler decoded them (-1 ends the list)
  auto next_item = [&](int n, bool& ok, Item& it) -> int {
    ok = wait_or_flag(bar_rf(n), (n / kRing) & 1, &B, a.dev_status);
    const int k = ok ? W.ring[n & (kRing - 1)] : -1;
    if (k >= 0) it = ring_item[n & (kRing - 1)];
    mbar_arrive(bar_re(n));
    return k;
  };

  // registers: the softmax warpgroups (warps 0-7) take 216, the MMA / load /
  // store warpgroup (warps 8-11) gives its share down to 64:
  // 256 x 216 + 128 x 64 = 63,488 <= 384 x 168 at launch
  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 64;" ::: "memory");
  if (warp == kProducerWarp) {
    // lane 0: scheduler, both Q tiles and the K tiles (the V tiles: warp 10).
    // A K (V) stage is refilled once both S (both P.V) that read it are done.
    if (lane == 0) {
      b200::prefetch_tensormap(&tmq);
      b200::prefetch_tensormap(&tmk);
      int kc = 0;
      bool ok = true;
      for (int n = 0; ok; ++n) {
        // scheduler: the next item from the global counter, or without one
        // the fixed boustrophedon order over the CTAs
        const int round = n / static_cast<int>(gridDim.x);
        // (with the counter, the first item of CTA b is item b and the counter
        // hands out the items from gridDim.x on: no atomic before the first loads)
        int k = a.sched != nullptr
                    ? (n == 0 ? static_cast<int>(blockIdx.x)
                              : atomicAdd(&a.sched[0], 1) + static_cast<int>(gridDim.x))
                    : round * static_cast<int>(gridDim.x) +
                          ((round & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x);
        if (k >= W.n_items) k = -1;
        if (n >= kRing && !(ok = wait_or_flag(bar_re(n), ((n / kRing) - 1) & 1, &B, a.dev_status)))
          break;
        Item it;
        if (k >= 0) {
          it = decode_item(a, W, k);
          ring_item[n & (kRing - 1)] = it;
        }
        W.ring[n & (kRing - 1)] = k;
        mbar_arrive(bar_rf(n));
        if (k < 0) break;
        if (n > 0 && !(ok = wait_or_flag(bar_qe, (n - 1) & 1, &B, a.dev_status))) break;
        b200::mbar_arrive_expect_tx(bar_q, 2 * kQBytes);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint32_t dq = sQ + t * kQBytes;
          b200::tma_load_3d(dq, &tmq, bar_q, 0, it.h[t], it.start + it.m0[t]);
          b200::tma_load_3d(dq + kQBlock, &tmq, bar_q, 64, it.h[t], it.start + it.m0[t]);
        }
        for (int j = 0; j < it.n_kv; ++j, ++kc) {
          const int s = kc & 1;
          if (kc >= kStages &&
              !(ok = wait_or_flag(bar_ke(s), ((kc >> 1) - 1) & 1, &B, a.dev_status)))
            break;
          const uint32_t dk = sK + s * kKVBytes;
          b200::mbar_arrive_expect_tx(bar_k(s), kKVBytes);
          if (a.paged) {
            load_kv_tile_paged(a, it, &tmk, dk, bar_k(s), j);
          } else {
            b200::tma_load_3d(dk, &tmk, bar_k(s), 0, it.hk, it.start + j * kBN);
            b200::tma_load_3d(dk + kKVBlock, &tmk, bar_k(s), 64, it.hk, it.start + j * kBN);
          }
        }
      }
    }
  } else if (warp == kStoreWarp) {
    if (lane == 0 && !a.paged) {
      // store lane (not in paged mode, whose epilogue writes rows directly
      // and whose stages the MMA thread releases): sends each finished tile's output (staged by its softmax
      // threads in the stage of the item's last K tile for tile 0, of its last
      // V tile for tile 1) to global memory with two TMA stores, and hands the
      // stage back to its producer once the stores have read it
      b200::prefetch_tensormap(&tmo);
      int gs = 0;  // steps of this CTA before the current item
      bool ok = true;
      for (int n = 0; ok; ++n) {
        Item it;
        const int k = next_item(n, ok, it);
        if (!ok || k < 0) break;
        const int g_last = gs + it.n_kv - 1;
        gs += it.n_kv;
        // The lead of the softmax over this lane is bounded: the stage this
        // lane returns for item n is the one the next item but one loads its
        // second K / V tile into, so the softmax cannot complete a tile of
        // item n + 2 before this lane has taken item n's.
        for (int t = 0; t < 2 && ok; ++t) {
          if (!(ok = wait_or_flag(bar_st(t, n), (n >> 1) & 1, &B, a.dev_status))) break;
          const uint32_t stage = (t == 0 ? sK : sV) + (g_last & 1) * kKVBytes;
          const int m0t = t == 0 ? it.m0[0] : it.m0[1];
          const int ht = t == 0 ? it.h[0] : it.h[1];
          if (m0t + kBM <= it.len) {
            b200::tma_store_3d(&tmo, stage, 0, ht, it.start + m0t);
            b200::tma_store_3d(&tmo, stage + kKVBlock, 64, ht, it.start + m0t);
            b200::bulk_commit_group();
            b200::bulk_wait_group_read0();
          }
          mbar_arrive(t == 0 ? bar_ke(g_last & 1) : bar_ve(g_last & 1));
        }
      }
      // the output stores are complete before the CTA ends
      b200::bulk_wait_group0();
    }
  } else if (warp == kVWarp) {
    if (lane == 0) {
      b200::prefetch_tensormap(&tmv);
      int vc = 0;
      bool ok = true;
      for (int n = 0; ok; ++n) {
        Item it;
        const int k = next_item(n, ok, it);
        if (!ok || k < 0) break;
        for (int j = 0; j < it.n_kv; ++j, ++vc) {
          const int s = vc & 1;
          if (vc >= kStages &&
              !(ok = wait_or_flag(bar_ve(s), ((vc >> 1) - 1) & 1, &B, a.dev_status)))
            break;
          const uint32_t dv = sV + s * kKVBytes;
          b200::mbar_arrive_expect_tx(bar_v(s), kKVBytes);
          if (a.paged) {
            load_kv_tile_paged(a, it, &tmv, dv, bar_v(s), j, true);
          } else {
            b200::tma_load_3d(dv, &tmv, bar_v(s), 0, it.hk, it.start + j * kBN);
            b200::tma_load_3d(dv + kKVBlock, &tmv, bar_v(s), 64, it.hk, it.start + j * kBN);
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(kBN, false);
      constexpr uint32_t idO = idesc_bf16(kD, true);
      // S_t = Q_t . K(s)^T into tile t's score buffer
      auto issue_s = [&](int t, int s) {
        const uint32_t q = sQ + t * kQBytes, kt = sK + s * kKVBytes;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t inblk = (kk & 3) * 32;
          umma_bf16(tmem + kColS + t * kBN, smem_desc(q + (kk >> 2) * kQBlock + inblk, 16, 1024),
                    smem_desc(kt + (kk >> 2) * kKVBlock + inblk, 16, 1024), idS,
                    kk > 0 ? 1u : 0u);
        }
        umma_commit(bar_sf(t));
      };
      // O_t (+)= P_t . V(s), P_t read from tile t's score buffer in TMEM
      auto issue_pv = [&](int t, int s, bool accumulate) {
        const uint32_t vt = sV + s * kKVBytes;
        // packed V: [d half][128 keys][64 d] (halves 16 KB apart); paged V:
        // [page][d half][16 keys][64 d] (4 KB per page, halves 2 KB apart)
        const uint32_t kstep = a.paged ? 4096u : 16u * 128u;
        const uint32_t lbo = a.paged ? 2048u : static_cast<uint32_t>(kKVBlock);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          umma_bf16_ts(tmem + kColO + t * kD, tmem + kColS + t * kBN + kk * 8,
                       smem_desc(vt + kk * kstep, lbo, 1024), idO,
                       (accumulate || kk > 0) ? 1u : 0u);
        }
      };
      int g = 0;  // K/V tiles consumed by this CTA before the current item
      bool ok = true;
      for (int n = 0; ok; ++n) {
        Item it;
        const int k = next_item(n, ok, it);
        if (!ok || k < 0) break;
        if (!(ok = wait_or_flag(bar_q, n & 1, &B, a.dev_status))) break;
        tc_fence_after();
        // step j issues P_t(j-1).V(j-1) then S_t(j) for t = 0, 1: S_t(j)
        // overwrites P_t(j-1), so its P.V goes first (MMAs run in order)
        for (int j = 0; ok && j <= it.n_kv; ++j) {
          const int gs = g + j, gp = gs - 1;  // tile of S(j) / of P(j-1)
          for (int t = 0; t < 2; ++t) {
            if (j > 0) {
              if (t == 0 && !(ok = wait_or_flag(bar_v(gp & 1), (gp >> 1) & 1, &B, a.dev_status)))
                break;
              if (!(ok = wait_or_flag(bar_p(t), gp & 1, &B, a.dev_status))) break;
              if (j == 1 && n > 0 &&
                  !(ok = wait_or_flag(bar_of(t), (n - 1) & 1, &B, a.dev_status)))
                break;
              tc_fence_after();
              issue_pv(t, gp & 1, j > 1);
              if (j == it.n_kv) umma_commit(bar_od(t));
            }
            if (j < it.n_kv) {
              if (t == 0 && !(ok = wait_or_flag(bar_k(gs & 1), (gs >> 1) & 1, &B, a.dev_status)))
                break;
              tc_fence_after();
              issue_s(t, gs & 1);
            }
          }
          if (!ok) break;
          // the stages of the item's last K and V tiles are released by the
          // store lane instead (the epilogue stages the output in them),
          // except in paged mode, whose epilogue writes rows directly
          if (j < it.n_kv - 1 || (a.paged && j < it.n_kv)) umma_commit(bar_ke(gs & 1));
          if (j == it.n_kv - 1) umma_commit(bar_qe);
          if (j > 0 && (j < it.n_kv || a.paged)) umma_commit(bar_ve(gp & 1));
        }
        g += it.n_kv;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory");
    // ---------------------------------------------------------- softmax
    const int t = warp >> 2;            // tile of this warpgroup
    const int r = threadIdx.x & 127;    // query row in the tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t sbuf = tmem + lane_addr + kColS + t * kBN;
    const uint32_t obuf = tmem + lane_addr + kColO + t * kD;

    // padded adapter: zero the rows past every sequence (spread over all CTAs)
    if (a.zero_pad) {
      const int total = W.pad_prefix[a.num_seqs];
      for (int z = blockIdx.x * kSoftmaxThreads + threadIdx.x; z < total;
           z += gridDim.x * kSoftmaxThreads) {
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

    int g = 0;
    bool ok = true;
    for (int n = 0; ok; ++n) {
      Item it;
      const int k = next_item(n, ok, it);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok || k < 0) break;
      // this tile's fields by selection, not by a runtime index (which would
      // put the item in local memory)
      const int m0t = t == 0 ? it.m0[0] : it.m0[1];
      const int ht = t == 0 ? it.h[0] : it.h[1];
      const int qpos = m0t + r;  // position within the sequence
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j, ++g) {
        ok = __all_sync(0xffffffffu, wait_or_flag(bar_sf(t), g & 1, &B, a.dev_status));
        if (!ok) break;
        tc_fence_after();
        uint32_t xs[kBN];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_ld32(sbuf + c * 32, xs + c * 32);
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_wait_ld(xs + c * 32);
        float* x = reinterpret_cast<float*>(xs);

        // key positions: cached ones first (paged mode), then the new tokens
        const int n0 = j * kBN;
        const int qabs = it.ctx + qpos, kend = it.ctx + it.len;
        if (n0 + kBN - 1 > qabs || n0 + kBN > kend) {
          const int lim = min(qabs + 1, kend) - n0;  // keys [n0, n0 + lim) are visible
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (c >= lim) x[c] = -INFINITY;
        }
        // tree max (8 independent chains of 3-input max)
        float mq[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mq[e] = b200::fmax3(x[e], x[e + 8], x[e + 16]);
#pragma unroll
        for (int c = 24; c + 16 <= kBN - 8; c += 16)
#pragma unroll
          for (int e = 0; e < 8; ++e) mq[e] = b200::fmax3(mq[e], x[c + e], x[c + e + 8]);
#pragma unroll
        for (int e = 0; e < 8; ++e) mq[e] = fmaxf(mq[e], x[kBN - 8 + e]);
        const float mx = b200::fmax3(b200::fmax3(mq[0], mq[1], mq[2]),
                                     b200::fmax3(mq[3], mq[4], mq[5]), fmaxf(mq[6], mq[7])) *
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
        // p = 2^(x * scale_log2 - m) on packed pairs; of every 16 columns the
        // first 2 * FMA_PAIRS take the FMA-pipe exp2, the rest the MUFU
        const uint64_t sc2 = b200::f2_pack(a.scale_log2, a.scale_log2);
        const uint64_t nm2 = b200::f2_pack(-m_used, -m_used);
        uint64_t sq[4] = {0, 0, 0, 0};
#pragma unroll
        for (int h = 0; h < kBN / 32; ++h) {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const uint64_t y = b200::f2_fma(b200::f2_pack(x[h * 32 + c], x[h * 32 + c + 1]), sc2, nm2);
            float p0, p1;
            if ((c & (kExpFmaPeriod - 1)) < FMA_PAIRS * 2) {
              b200::f2_unpack(b200::ex2_fma2(y), p0, p1);
            } else {
              float y0, y1;
              b200::f2_unpack(y, y0, y1);
              p0 = b200::ex2(y0);
              p1 = b200::ex2(y1);
            }
            sq[(c >> 1) & 3] = b200::f2_add(sq[(c >> 1) & 3], b200::f2_pack(p0, p1));
            pk[c / 2] = b200::pack_bf16x2(p0, p1);
          }
          // P over the first half of its own score buffer (S is in registers)
          tmem_st16(sbuf + h * 16, pk);
        }
        float s0, s1;
        b200::f2_unpack(b200::f2_add(b200::f2_add(sq[0], sq[1]), b200::f2_add(sq[2], sq[3])), s0, s1);
        const float rowsum = s0 + s1;

        if (__any_sync(0xffffffffu, rescale)) {
          // S_t(g) done implies every earlier P_t.V is done, and the next one
          // waits for this warp's arrival: O_t is stable here.  tcgen05.ld/st
          // are warp-collective, so the warp's rows rescale together (alpha ==
          // 1 for rows whose max did not move)
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t rr[32];
            tmem_ld32(obuf + c * 32, rr);
            tmem_wait_ld(rr);
#pragma unroll
            for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
            tmem_st32(obuf + c * 32, rr);
          }
        }
        l = l * alpha + rowsum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p(t));
      }
      if (!ok) break;

      // ---- epilogue: O_t / l -> bf16 rows; O_t is released before the stores
      ok = __all_sync(0xffffffffu, wait_or_flag(bar_od(t), n & 1, &B, a.dev_status));
      if (!ok) break;
      tc_fence_after();
      uint32_t ov[kD];
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) tmem_ld32(obuf + c * 32, ov + c * 32);
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) tmem_wait_ld(ov + c * 32);
      tc_fence_before();
      mbar_arrive(bar_of(t));
      // Staging buffer of this tile: the stage of the item's last K tile for
      // tile 0 (o_done of tile 0 covers every S of the item, tile 1's last
      // included), the stage of its last V tile for tile 1 (o_done of tile 1
      // covers both last P.V).  The store lane (warp 11) sends it
      // out with TMA stores and returns the stage to its producer; the stage's
      // next tile (the next item's second K / V tile) is needed only a step
      // later.
      const int g_last = g - 1;  // this CTA's step index of the item's last K/V tile
      const uint32_t stage = (t == 0 ? sK : sV) + (g_last & 1) * kKVBytes;
      // (paged mode: every tile row by row; its K/V stages, filled from 16
      // page boxes each, go back to their producers without waiting for this)
      if (!a.paged && m0t + kBM <= it.len) {
        // a full tile: rows staged in the swizzled [128 rows][64 d] x 2 layout
        // of a K/V tile (the TMA engine writes whole lines; the memory-
        // instruction queue that the other tile's softmax and the MMA thread
        // use carries a quarter of the requests of row-per-thread stores)
        const float inv = 1.f / l;
        const uint64_t inv2 = b200::f2_pack(inv, inv);
        auto norm2 = [&](int e) {  // O / l of columns e, e + 1 (one packed multiply) as bf16
          float lo, hi;
          b200::f2_unpack(b200::f2_mul(b200::f2_pack(__uint_as_float(ov[e]), __uint_as_float(ov[e + 1])),
                                       inv2),
                          lo, hi);
          return b200::pack_bf16x2(lo, hi);
        };
#pragma unroll
        for (int c = 0; c < kD / 8; ++c) {
          const int e = 8 * c;
          b200::st_shared_v4(stage + (c >> 3) * kKVBlock + r * 128 + (((c & 7) ^ (r & 7)) << 4),
                             norm2(e), norm2(e + 2), norm2(e + 4), norm2(e + 6));
        }
        b200::fence_proxy_async_smem();  // the rows, then the store lane's TMA stores
        mbar_arrive(bar_st(t, n));
      } else {
        // the sequence's ragged last tile: each thread writes its own row
        // (rows past the sequence are zeroed by the pass above, if asked)
        if (!a.paged) mbar_arrive(bar_st(t, n));  // nothing staged: the stage goes straight back
        if (qpos < it.len) {
        const float inv = 1.f / l;
        __nv_bfloat16* orow = a.out + static_cast<int64_t>(it.start + qpos) * a.o_t +
                              static_cast<int64_t>(ht) * a.o_h;
        if (a.out32) {
          // 32-byte stores: every row piece is a full sector
#pragma unroll
          for (int e = 0; e < kD; e += 16) {
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              w[i] = b200::pack_bf16x2(__uint_as_float(ov[e + 2 * i]) * inv,
                                       __uint_as_float(ov[e + 2 * i + 1]) * inv);
            b200::st_global_v8(orow + e, w);
          }
        } else {
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

// Launches the kernel over `num_seqs` sequences, at most kMaxSeqs per launch;
// `base` carries every field but the per-launch sequence slices.
int launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const CUtensorMap& to,
                   PrefillArgs base, const int32_t* cu_seqlens, const int32_t* lens_opt,
                   const int32_t* row_ids, int num_seqs, void* stream) {
  int st = ensure_smem_attr(b200host::current_device());
  if (st != B200_OK) return st;
  const int sms = b200host::sm_count(b200host::current_device());
  if (sms <= 0) return B200_ERR_CUDA;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int pairs = exp_fma_pairs();
  for (int s0 = 0; s0 < num_seqs; s0 += kMaxSeqs) {
    PrefillArgs a = base;
    a.cu = cu_seqlens + s0;
    a.lens = lens_opt != nullptr ? lens_opt + s0 : nullptr;
    a.row_ids = row_ids != nullptr ? row_ids + s0 : nullptr;
    a.num_seqs = num_seqs - s0 < kMaxSeqs ? num_seqs - s0 : kMaxSeqs;
    dim3 grid(static_cast<unsigned>(sms));  // one persistent CTA per SM
    switch (pairs) {
      case 0: varlen_prefill_kernel<0><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, to, a); break;
      case 2: varlen_prefill_kernel<2><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, to, a); break;
      case 3: varlen_prefill_kernel<3><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, to, a); break;
      case 4: varlen_prefill_kernel<4><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, to, a); break;
      default: varlen_prefill_kernel<1><<<grid, kThreads, kSmemBytes, cs>>>(tq, tk, tv, to, a); break;
    }
    st = b200host::status_from_cuda(cudaGetLastError());
    if (st != B200_OK) return st;
  }
  return B200_OK;
}

PrefillArgs base_args(void* out, int64_t o_stride_t, int64_t o_stride_h, int num_heads,
                      int num_kv_heads, int max_seqlen, int total_tokens, float scale,
                      int32_t* work_counter, int32_t* dev_status) {
  PrefillArgs a{};
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_t = o_stride_t;
  a.o_h = o_stride_h;
  a.num_heads = num_heads;
  a.group = num_heads / num_kv_heads;
  a.max_seqlen = max_seqlen;
  a.total_tokens = total_tokens;
  a.pair_heads = (a.group % 2) == 0 ? 1 : 0;
  a.out32 = (reinterpret_cast<uintptr_t>(out) & 31) == 0 && (o_stride_t & 15) == 0 &&
            (o_stride_h & 15) == 0;
  a.scale_log2 = scale * kLog2e;
  a.dev_status = dev_status;
  a.sched = work_counter;
  return a;
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

  PrefillArgs a = base_args(out, o_stride_t, o_stride_h, num_heads, num_kv_heads, max_seqlen,
                            total_tokens, scale, work_counter, dev_status);
  a.zero_pad = zero_pad_rows != 0;
  CUtensorMap to;  // the output, in the boxes of a Q load
  st = encode_rows_map(&to, out, num_heads, total_tokens, o_stride_t, o_stride_h, kBM);
  if (st != B200_OK) return st;
  return launch_prefill(tq, tk, tv, to, a, cu_seqlens, seq_lens_opt, nullptr, num_seqs, stream);
}

extern "C" int b200_paged_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                                  const void* k_pool, const void* v_pool, int64_t kv_stride_blk,
                                  int64_t kv_stride_h, int64_t kv_stride_slot,
                                  const int32_t* block_table, int64_t bt_stride_row,
                                  const int32_t* seq_lens, const int32_t* row_ids,
                                  const int32_t* cu_seqlens, void* out, int64_t o_stride_t,
                                  int64_t o_stride_h, int num_seqs, int total_tokens,
                                  int max_new_tokens, int num_heads, int num_kv_heads,
                                  int head_dim, int block_size, int num_blocks, int max_pages,
                                  int max_requests, float scale, int32_t* work_counter,
                                  int32_t* dev_status, void* stream) {
  if (num_seqs < 0 || total_tokens < 0 || max_new_tokens < 0 || num_heads <= 0 ||
      num_kv_heads <= 0 || num_blocks <= 0 || max_pages <= 0 || max_requests <= 0 ||
      bt_stride_row <= 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || total_tokens == 0 || max_new_tokens == 0) return B200_OK;
  if (!q || !k_pool || !v_pool || !block_table || !seq_lens || !row_ids || !cu_seqlens || !out)
    return B200_ERR_INVALID_ARGUMENT;
  if (head_dim != kD || block_size != 16) return B200_ERR_UNSUPPORTED;
  if (num_heads % num_kv_heads != 0) return B200_ERR_INVALID_ARGUMENT;
  const int n_tiles = (max_new_tokens + kBM - 1) / kBM;
  if (n_tiles > kMaxTiles) return B200_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(n_tiles) * kMaxSeqs * num_heads > 0x7fffffff)
    return B200_ERR_INVALID_ARGUMENT;
  if (!b200host::aligned16(q) || !b200host::aligned16(out) || !b200host::aligned16(k_pool) ||
      !b200host::aligned16(v_pool))
    return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {q_stride_t, q_stride_h, o_stride_t, o_stride_h,
                             kv_stride_blk, kv_stride_h, kv_stride_slot};
  for (int64_t s : strides)
    if (!mult8(s)) return B200_ERR_ALIGNMENT;

  CUtensorMap tq, tk, tv;
  int st = encode_rows_map(&tq, q, num_heads, total_tokens, q_stride_t, q_stride_h, kBM);
  if (st != B200_OK) return st;
  {
    // K, one layer of the pool: (d = 128, slot = 16, kv head, block), boxes of
    // half a page
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), 16u,
                                static_cast<cuuint64_t>(num_kv_heads),
                                static_cast<cuuint64_t>(num_blocks)};
    const cuuint64_t strides_b[3] = {static_cast<cuuint64_t>(kv_stride_slot) * 2,
                                     static_cast<cuuint64_t>(kv_stride_h) * 2,
                                     static_cast<cuuint64_t>(kv_stride_blk) * 2};
    const cuuint32_t box[4] = {64, 16, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (b200host::encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                               const_cast<void*>(k_pool), dims, strides_b, box, es,
                               CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B) != CUDA_SUCCESS)
      return B200_ERR_TENSOR_MAP;
    // V: one box per page, (d 64, slot 16, d half 2, kv head, block) -> smem
    // [d half][slot][64 d]
    const cuuint64_t dims5[5] = {64u, 16u, 2u, static_cast<cuuint64_t>(num_kv_heads),
                                 static_cast<cuuint64_t>(num_blocks)};
    const cuuint64_t strides5[4] = {static_cast<cuuint64_t>(kv_stride_slot) * 2, 128u,
                                    static_cast<cuuint64_t>(kv_stride_h) * 2,
                                    static_cast<cuuint64_t>(kv_stride_blk) * 2};
    const cuuint32_t box5[5] = {64, 16, 2, 1, 1};
    const cuuint32_t es5[5] = {1, 1, 1, 1, 1};
    if (b200host::encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5,
                               const_cast<void*>(v_pool), dims5, strides5, box5, es5,
                               CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B) != CUDA_SUCCESS)
      return B200_ERR_TENSOR_MAP;
  }

  PrefillArgs a = base_args(out, o_stride_t, o_stride_h, num_heads, num_kv_heads,
                            max_new_tokens, total_tokens, scale, work_counter, dev_status);
  a.paged = 1;
  a.seq_lens = seq_lens;
  a.block_table = block_table;
  a.bt_row = bt_stride_row;
  a.num_blocks = num_blocks;
  a.max_pages = max_pages;
  a.max_requests = max_requests;
  CUtensorMap to;  // the output, in the boxes of a Q load
  st = encode_rows_map(&to, out, num_heads, total_tokens, o_stride_t, o_stride_h, kBM);
  if (st != B200_OK) return st;
  return launch_prefill(tq, tk, tv, to, a, cu_seqlens, nullptr, row_ids, num_seqs, stream);
}
