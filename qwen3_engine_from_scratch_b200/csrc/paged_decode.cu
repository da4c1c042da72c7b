// Paged decode attention for sm_100a: split-K flash-decoding over the paged
// KV pool (the GPU-resident 2-D block table and row slots of
// qwen3/PagedKVcache.py), replacing paged_attn_decode_kernel
// (qwen3/kernels/paged_attention.py:27-129).
//
// Work decomposition
//   grid.x = request b x kv head hkv ("pair"), grid.y = split index.  A split
//   is `pages_per_split` consecutive 16-token pages of the pair's sequence;
//   CTAs whose split starts past the sequence exit at once, so the grid
//   depends on shapes only (CUDA-graph safe while seq_lens change).
//   A CTA has 4 warps.  Warp w takes pages w, w+4, ... of the split and keeps
//   its own online-softmax state; the 4 states are merged in shared memory at
//   the end.  A pair with one split writes the bf16 output directly; else the
//   split writes an fp32 partial (m, l, acc) to the workspace and bumps the
//   pair's arrival counter; the CTA that arrives last merges the partials
//   (they are in L2) and writes the output, then zeroes the counter, so the
//   counters are zero again after every launch.
//
// Data movement
//   Each page of one kv head is a contiguous 16 x 128 bf16 tile (4 KB) of K
//   and one of V.  Lane 0 of a warp stages them into a per-warp ring of 2
//   shared-memory slots with 4 TMA tensor loads (two 64-column boxes per
//   tensor, 128-byte swizzle, L2 evict-first) that complete on the slot's
//   mbarrier; all waits are bounded.  3 CTAs per SM (65 KB of slots each)
//   keep up to 192 KB of loads in flight per SM; with more CTAs of fewer
//   slots, one CTA's prologue or merge leaves less of the SM idle than with
//   2 CTAs of 3 slots (measured: the 28-layer config-2 step 2.61 -> 2.52 ms).
//
// Math (per page, per warp; G = num_heads / num_kv_heads <= 8)
//   S^T (16 tokens x 8 heads) = K (16 x 128) . Q^T (128 x 8): 8 x mma.m16n8k16,
//   tokens on the M side so the G query heads fill the N = 8 side (heads >= G
//   are zero).  K fragments come from ldmatrix on the swizzled tile.
//   Online softmax in base 2 on fp32 scores (max over the 16 tokens = 3 xor
//   shuffles), P rounded to bf16, transposed in registers with movmatrix into
//   the B operand of O^T (128 x 8) += V^T (128 x 16) . P (16 x 8): 8 more
//   mma with V^T fragments from ldmatrix.trans.  The rescale factor of a head
//   lives in the same lane as that head's accumulator columns, so no shuffle
//   is needed for it.
//
// Fused KV write (b200_paged_decode_kv_write)
//   The step's new K/V row of (request, kv head) belongs at position
//   seq_lens[row] of the pool, inside the sequence's last page.  The CTA whose
//   split holds that page stores the two 256-byte rows first (one 16-byte
//   chunk per thread, the range checks of the KV write kernel), orders the
//   stores before its own tensor loads with a generic-to-async proxy fence and
//   a CTA barrier, and then reads the page like any other.  No other CTA reads
//   that page, so one launch replaces the KV write launch and the decode.
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr int kD = 128;
constexpr int kBS = 16;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 2;
constexpr int kPageBytes = kBS * kD * 2;  // 4096
constexpr int kHalfBytes = kPageBytes / 2;
constexpr int kSlotBytes = 2 * kPageBytes;
constexpr int kMaxG = 8;
constexpr int kAccStride = 132;  // floats per head row of the merge buffer
constexpr int kMinDefaultPagesPerSplit = 16;
constexpr int kMaxPagesPerSplit = 32 * kWarps;  // a warp's page ids live one per lane
constexpr int kSmemBytes = kWarps * kStages * kSlotBytes + 1024;
constexpr float kLog2e = 1.4426950408889634f;
// The workspace starts with one split-arrival counter per (request, kv head),
// at a fixed place whatever the shapes, so one zeroed workspace can serve
// launches of any shape; the partials follow.
constexpr int kMaxPairs = 65536;
constexpr size_t kCounterBytes = kMaxPairs * sizeof(int32_t);

struct DecodeArgs {
  const __nv_bfloat16* q;
  int64_t q_b, q_h;
  const int32_t* block_table;
  int64_t bt_row;
  const int32_t* seq_lens;
  const int32_t* row_ids;
  __nv_bfloat16* out;
  int64_t o_b, o_h;
  int32_t* ws_done;  // [batch * num_kv_heads] split arrivals (zero at launch, zero at exit)
  float* ws_acc;     // [batch][num_heads][max_splits][128]
  float* ws_ml;      // [batch][num_heads][max_splits][2]
  int batch, num_heads, num_kv_heads, group, num_blocks, max_pages, max_requests;
  int pages_per_split, max_splits;
  float scale_log2;
  int32_t* dev_status;
  // fused KV write (k_new == nullptr: none)
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  int64_t kn_b, kn_h, vn_b, vn_h;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  int64_t kv_blk, kv_h, kv_slot;
};

// Visible pages of request b: L = seq_lens[row] + 1 tokens (the current token
// was written by the scatter first), clamped to the block table.  Returns the
// page count (0 for an invalid row) and sets L.
B200_DEVICE int request_pages(const DecodeArgs& a, int b, int& row, int& L, int& err) {
  err = 0;
  row = a.row_ids[b];
  if (row < 0 || row >= a.max_requests) {
    err = B200_DEV_BAD_ROW;
    L = 0;
    return 0;
  }
  L = a.seq_lens[row] + 1;
  if (L <= 0) {
    err = B200_DEV_SEQ_OVERFLOW;
    L = 0;
    return 0;
  }
  int npages = (L + kBS - 1) / kBS;
  if (npages > a.max_pages) {
    err = B200_DEV_SEQ_OVERFLOW;
    npages = a.max_pages;
    L = npages * kBS;
  }
  return npages;
}

__global__ void __launch_bounds__(kThreads, 3)
    paged_decode_split_kernel(const __grid_constant__ CUtensorMap kmap,
                              const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kWarps * kStages];
  __shared__ float s_ml[kWarps][kMaxG][2];

  // launched with b200host::launch_pdl: nothing read or written before this
  b200::pdl_begin();

  const int pair = blockIdx.x;
  const int split = blockIdx.y;
  const int b = pair / a.num_kv_heads;
  const int hkv = pair - b * a.num_kv_heads;
  const int G = a.group;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  int row, L, err;
  const int npages = request_pages(a, b, row, L, err);
  if (split == 0 && err != 0 && threadIdx.x == 0) b200::flag_error(a.dev_status, err);
  if (npages == 0) {
    // invalid row / empty sequence: split 0 writes zeros for this pair's heads
    if (split == 0) {
      for (int h = 0; h < G; ++h)
        a.out[b * a.o_b + (hkv * G + h) * a.o_h + threadIdx.x] = __float2bfloat16(0.f);
    }
    return;
  }
  const int p_begin = split * a.pages_per_split;
  if (p_begin >= npages) return;
  const int p_end = min(npages, p_begin + a.pages_per_split);
  const int nsplit = (npages + a.pages_per_split - 1) / a.pages_per_split;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem + warp * kStages * kSlotBytes;

  if (a.k_new != nullptr && p_end == npages && err == 0 && threadIdx.x < 32) {
    // fused KV write of this step's token (position L - 1, in the last page):
    // threads 0-15 store the K row, 16-31 the V row, 16 bytes each
    const int pos = L - 1;
    const int ph = a.block_table[static_cast<int64_t>(row) * a.bt_row + pos / kBS];
    if (ph < 0 || ph >= a.num_blocks) {
      if (threadIdx.x == 0) b200::flag_error(a.dev_status, B200_DEV_BAD_PAGE);
    } else {
      const int i = threadIdx.x & 15;
      const bool is_v = threadIdx.x >= 16;
      const __nv_bfloat16* src = is_v ? a.v_new + b * a.vn_b + hkv * a.vn_h
                                      : a.k_new + b * a.kn_b + hkv * a.kn_h;
      __nv_bfloat16* dst = (is_v ? a.v_pool : a.k_pool) + static_cast<int64_t>(ph) * a.kv_blk +
                           hkv * a.kv_h + (pos % kBS) * a.kv_slot;
      *reinterpret_cast<uint4*>(dst + 8 * i) = *reinterpret_cast<const uint4*>(src + 8 * i);
      // the stores above, then this CTA's tensor (async-proxy) loads of the page
      b200::fence_proxy_async_global();
    }
  }
  if (threadIdx.x == 0) {
    b200::prefetch_tensormap(&kmap);
    b200::prefetch_tensormap(&vmap);
    for (int i = 0; i < kWarps * kStages; ++i) b200::mbar_init(b200::smem_u32(&bars[i]), 1);
    b200::fence_mbar_init();
  }
  __syncthreads();

  // pages of this warp: p_begin + warp + kWarps * i, i < n_mine (<= 32)
  const int first = p_begin + warp;
  const int n_mine = first < p_end ? (p_end - first + kWarps - 1) / kWarps : 0;
  int my_phys = 0;
  if (lane < n_mine) {
    const int p = first + kWarps * lane;
    int ph = a.block_table[static_cast<int64_t>(row) * a.bt_row + p];
    if (ph < 0 || ph >= a.num_blocks) {
      b200::flag_error(a.dev_status, B200_DEV_BAD_PAGE);
      ph = 0;
    }
    my_phys = ph;
  }

  // Q^T fragments: lane (g, c) holds head g, dims 16ks + 2c (+1) and +8.
  const int g = lane >> 2;
  const int c = lane & 3;
  uint32_t qb[8][2];
  {
    const bool qv = g < G;
    const __nv_bfloat16* qrow = a.q + b * a.q_b + (hkv * G + (qv ? g : 0)) * a.q_h + 2 * c;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qb[ks][0] = qv ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks) : 0u;
      qb[ks][1] = qv ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8) : 0u;
    }
  }

  const uint64_t policy = b200::l2_policy_evict_first();
  const uint32_t bar0 = b200::smem_u32(&bars[warp * kStages]);
  const uint32_t ring_u32 = b200::smem_u32(ring);

  auto issue = [&](int i, int slot) {
    const int phys = __shfl_sync(0xffffffffu, my_phys, i);
    if (lane == 0) {
      const uint32_t bar = bar0 + 8 * slot;
      const uint32_t dst = ring_u32 + slot * kSlotBytes;
      b200::mbar_arrive_expect_tx(bar, kSlotBytes);
      b200::tma_load_4d(dst, &kmap, bar, 0, 0, hkv, phys, policy);
      b200::tma_load_4d(dst + kHalfBytes, &kmap, bar, 64, 0, hkv, phys, policy);
      b200::tma_load_4d(dst + kPageBytes, &vmap, bar, 0, 0, hkv, phys, policy);
      b200::tma_load_4d(dst + kPageBytes + kHalfBytes, &vmap, bar, 64, 0, hkv, phys, policy);
    }
  };

  // per-lane ldmatrix address terms (128-byte swizzle: chunk ^= row & 7)
  const int mi = lane >> 3;
  const int sw = lane & 7;
  const uint32_t k_row = static_cast<uint32_t>(((lane & 7) + ((mi & 1) << 3)) * 128);
  const int k_chunk_hi = mi >> 1;
  const uint32_t v_row = static_cast<uint32_t>(((lane & 7) + ((mi >> 1) << 3)) * 128);
  const int v_chunk_lo = mi & 1;

  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;

  int issued = 0;
  for (; issued < n_mine && issued < kStages; ++issued) issue(issued, issued);

  int consumed = 0;
  bool timed_out = false;
  for (; consumed < n_mine; ++consumed) {
    const int slot = consumed % kStages;
    const uint32_t parity = static_cast<uint32_t>((consumed / kStages) & 1);
    const bool ok = b200::mbar_wait_bounded(bar0 + 8 * slot, parity);
    if (__any_sync(0xffffffffu, !ok)) {
      timed_out = true;
      break;
    }
    const uint32_t kbase = ring_u32 + slot * kSlotBytes;
    const uint32_t vbase = kbase + kPageBytes;

    // ---- S^T = K . Q^T
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int chunk = ((ks & 3) << 1) + k_chunk_hi;
      const uint32_t addr = kbase + (ks >> 2) * kHalfBytes + k_row + ((chunk ^ sw) << 4);
      uint32_t a0, a1, a2, a3;
      b200::ldmatrix_x4(addr, a0, a1, a2, a3);
      b200::mma_bf16_16816(s, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
    }

    // ---- online softmax (base 2); lane holds tokens g, g+8 x heads 2c, 2c+1
    const int valid = L - (first + kWarps * consumed) * kBS;  // >= 1
    float x0 = s[0] * a.scale_log2, x1 = s[1] * a.scale_log2;
    float x2 = s[2] * a.scale_log2, x3 = s[3] * a.scale_log2;
    if (g >= valid) x0 = x1 = -INFINITY;
    if (g + 8 >= valid) x2 = x3 = -INFINITY;
    float pm0 = fmaxf(x0, x2), pm1 = fmaxf(x1, x3);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      pm0 = fmaxf(pm0, __shfl_xor_sync(0xffffffffu, pm0, o));
      pm1 = fmaxf(pm1, __shfl_xor_sync(0xffffffffu, pm1, o));
    }
    const float mn0 = fmaxf(m0, pm0), mn1 = fmaxf(m1, pm1);
    const float al0 = b200::ex2(m0 - mn0), al1 = b200::ex2(m1 - mn1);
    const uint32_t plo = b200::pack_bf16x2(b200::ex2(x0 - mn0), b200::ex2(x1 - mn1));
    const uint32_t phi = b200::pack_bf16x2(b200::ex2(x2 - mn0), b200::ex2(x3 - mn1));
    l0 = l0 * al0 + (b200::bf16_lo(plo) + b200::bf16_lo(phi));
    l1 = l1 * al1 + (b200::bf16_hi(plo) + b200::bf16_hi(phi));
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      acc[mt][0] *= al0;
      acc[mt][1] *= al1;
      acc[mt][2] *= al0;
      acc[mt][3] *= al1;
    }

    // ---- O^T += V^T . P
    const uint32_t pb0 = b200::movmatrix_trans(plo);
    const uint32_t pb1 = b200::movmatrix_trans(phi);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int chunk = ((mt & 3) << 1) + v_chunk_lo;
      const uint32_t addr = vbase + (mt >> 2) * kHalfBytes + v_row + ((chunk ^ sw) << 4);
      uint32_t a0, a1, a2, a3;
      b200::ldmatrix_x4_trans(addr, a0, a1, a2, a3);
      b200::mma_bf16_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
    }

    __syncwarp();
    if (issued < n_mine) {
      issue(issued, slot);
      ++issued;
    }
  }

  if (timed_out) {
    if (lane == 0) b200::flag_error(a.dev_status, B200_DEV_TIMEOUT);
    // let the copies this warp still has in flight land before the CTA exits
    for (int j = consumed; j < issued; ++j)
      b200::mbar_wait_bounded(bar0 + 8 * (j % kStages), static_cast<uint32_t>((j / kStages) & 1));
  }

#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }

  // ---- merge the 4 warp states (ring smem reused once every warp is done)
  __syncthreads();
  float* mbuf = reinterpret_cast<float*>(smem);
  {
    float* wbuf = mbuf + warp * kMaxG * kAccStride;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = 16 * mt + g;
      wbuf[(2 * c) * kAccStride + d] = acc[mt][0];
      wbuf[(2 * c + 1) * kAccStride + d] = acc[mt][1];
      wbuf[(2 * c) * kAccStride + d + 8] = acc[mt][2];
      wbuf[(2 * c + 1) * kAccStride + d + 8] = acc[mt][3];
    }
    if (g == 0) {
      s_ml[warp][2 * c][0] = m0;
      s_ml[warp][2 * c][1] = l0;
      s_ml[warp][2 * c + 1][0] = m1;
      s_ml[warp][2 * c + 1][1] = l1;
    }
  }
  __syncthreads();

  const int d = threadIdx.x;
  for (int h = 0; h < G; ++h) {
    float mt = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mt = fmaxf(mt, s_ml[w][h][0]);
    float o = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float sc = b200::ex2(s_ml[w][h][0] - mt);
      o += sc * mbuf[(w * kMaxG + h) * kAccStride + d];
      l += sc * s_ml[w][h][1];
    }
    const int hq = hkv * G + h;
    if (nsplit == 1) {
      a.out[b * a.o_b + hq * a.o_h + d] = __float2bfloat16(o / l);
    } else {
      const int64_t base = (static_cast<int64_t>(b) * a.num_heads + hq) * a.max_splits + split;
      a.ws_acc[base * kD + d] = o;
      if (d == 0) {
        a.ws_ml[base * 2] = mt;
        a.ws_ml[base * 2 + 1] = l;
      }
    }
  }
  if (nsplit == 1) return;

  // ---- arrival: the last split of the pair merges every partial of the pair
  __shared__ int s_last;
  __threadfence();  // this CTA's partials are visible device-wide before its arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&a.ws_done[pair], 1);
    s_last = prev == nsplit - 1;
    if (s_last) {
      __threadfence();             // order the partial reads after every arrival
      a.ws_done[pair] = 0;         // no other CTA of this launch touches it again
    }
  }
  __syncthreads();
  if (!s_last) return;
  for (int h = 0; h < G; ++h) {
    const int hq = hkv * G + h;
    const int64_t base = (static_cast<int64_t>(b) * a.num_heads + hq) * a.max_splits;
    const float* ml = a.ws_ml + base * 2;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(ml + 2 * sp));
    float o = 0.f, l = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float sc = b200::ex2(__ldcg(ml + 2 * sp) - M);
      l += sc * __ldcg(ml + 2 * sp + 1);
      o += sc * __ldcg(a.ws_acc + (base + sp) * kD + d);
    }
    a.out[b * a.o_b + hq * a.o_h + d] = __float2bfloat16(o / l);
  }
}

bool mult8(int64_t s) { return (s & 7) == 0; }

int max_splits_for(int max_pages, int pps) { return (max_pages + pps - 1) / pps; }

// Default split size: as many pages per CTA as possible (each split pays a
// prologue, an epilogue and a partial to merge), but enough CTAs for about 6
// per SM (two waves of the 3 resident ones) if the sequences fill half of the
// block table.  Measured on B200 (config 2: 512 pairs x 256 pages -> 73;
// config 4: 4096 pairs x 2048 pages -> 128): the 28-layer config-2 step at
// 6.40 TB/s against 6.30 with 110 pages (8 slots per SM), and config 4 at
// 7.07 TB/s.
int default_pages_per_split(int batch, int num_kv_heads, int max_pages) {
  const int sms = b200host::sm_count(b200host::current_device());
  const int64_t slots = 12 * static_cast<int64_t>(sms > 0 ? sms : 148);
  const int64_t pps =
      static_cast<int64_t>(batch) * num_kv_heads * static_cast<int64_t>(max_pages) / slots;
  return static_cast<int>(pps < kMinDefaultPagesPerSplit
                              ? kMinDefaultPagesPerSplit
                              : (pps > kMaxPagesPerSplit ? kMaxPagesPerSplit : pps));
}

std::mutex g_attr_mu;
bool g_attr_done[64] = {false};

int ensure_smem_attr(int dev) {
  if (dev < 0) return B200_ERR_CUDA;
  if (dev < 64 && g_attr_done[dev]) return B200_OK;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (dev < 64 && g_attr_done[dev]) return B200_OK;
  cudaError_t e = cudaFuncSetAttribute(paged_decode_split_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return B200_ERR_CUDA;
  if (dev < 64) g_attr_done[dev] = true;
  return B200_OK;
}

}  // namespace

extern "C" int b200_paged_decode_default_split(int batch, int num_kv_heads, int max_pages) {
  if (batch <= 0 || num_kv_heads <= 0 || max_pages <= 0) return kMinDefaultPagesPerSplit;
  return default_pages_per_split(batch, num_kv_heads, max_pages);
}

extern "C" size_t b200_paged_decode_workspace_size(int batch, int num_heads, int max_pages,
                                                   int pages_per_split) {
  if (batch <= 0 || num_heads <= 0 || max_pages <= 0) return 0;
  // <= 0: enough for any default split (the smallest one has the most partials)
  if (pages_per_split <= 0) pages_per_split = kMinDefaultPagesPerSplit;
  const int ms = max_splits_for(max_pages, pages_per_split);
  if (ms <= 1) return 0;
  // the counters, then the partials
  return kCounterBytes + static_cast<size_t>(batch) * num_heads * ms * (kD + 2) * sizeof(float);
}

namespace {

// Shared by the decode entry points; k_new == nullptr: no fused KV write.
int launch_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_new,
                  int64_t kn_stride_b, int64_t kn_stride_h, const void* v_new,
                  int64_t vn_stride_b, int64_t vn_stride_h, const void* k_pool,
                  const void* v_pool, int64_t kv_stride_blk, int64_t kv_stride_h,
                  int64_t kv_stride_slot, const int32_t* block_table, int64_t bt_stride_row,
                  const int32_t* seq_lens, const int32_t* row_ids, void* out,
                  int64_t out_stride_b, int64_t out_stride_h, int batch, int num_heads,
                  int num_kv_heads, int head_dim, int block_size, int num_blocks, int max_pages,
                  int max_requests, float scale, int pages_per_split, void* workspace,
                  size_t workspace_bytes, int32_t* dev_status, void* stream) {
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || max_pages <= 0 ||
      max_requests <= 0 || bt_stride_row <= 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (batch == 0) return B200_OK;
  if (!q || !k_pool || !v_pool || !block_table || !seq_lens || !row_ids || !out)
    return B200_ERR_INVALID_ARGUMENT;
  if (head_dim != kD || block_size != kBS) return B200_ERR_UNSUPPORTED;
  if (num_heads % num_kv_heads != 0) return B200_ERR_INVALID_ARGUMENT;
  const int G = num_heads / num_kv_heads;
  if (G > kMaxG) return B200_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(batch) * num_kv_heads > kMaxPairs) return B200_ERR_UNSUPPORTED;
  if (pages_per_split <= 0)
    pages_per_split = default_pages_per_split(batch, num_kv_heads, max_pages);
  if (pages_per_split > kMaxPagesPerSplit) return B200_ERR_INVALID_ARGUMENT;
  if (!b200host::aligned16(q) || !b200host::aligned16(out) || !b200host::aligned16(k_pool) ||
      !b200host::aligned16(v_pool))
    return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {q_stride_b, q_stride_h, out_stride_b, out_stride_h,
                             kv_stride_blk, kv_stride_h, kv_stride_slot};
  for (int64_t s : strides)
    if (!mult8(s)) return B200_ERR_ALIGNMENT;
  if (k_new != nullptr) {
    if (v_new == nullptr) return B200_ERR_INVALID_ARGUMENT;
    if (!b200host::aligned16(k_new) || !b200host::aligned16(v_new) || !mult8(kn_stride_b) ||
        !mult8(kn_stride_h) || !mult8(vn_stride_b) || !mult8(vn_stride_h))
      return B200_ERR_ALIGNMENT;
  }

  const int ms = max_splits_for(max_pages, pages_per_split);
  if (ms > 65535) return B200_ERR_INVALID_ARGUMENT;
  const size_t need =
      b200_paged_decode_workspace_size(batch, num_heads, max_pages, pages_per_split);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !b200host::aligned16(workspace)))
    return B200_ERR_WORKSPACE;

  // TMA maps over one layer of the pool: (d=128, slot=16, kv head, block)
  CUtensorMap kmap, vmap;
  {
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(kBS),
                                static_cast<cuuint64_t>(num_kv_heads),
                                static_cast<cuuint64_t>(num_blocks)};
    const cuuint64_t strides_b[3] = {static_cast<cuuint64_t>(kv_stride_slot) * 2,
                                     static_cast<cuuint64_t>(kv_stride_h) * 2,
                                     static_cast<cuuint64_t>(kv_stride_blk) * 2};
    const cuuint32_t box[4] = {64, kBS, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (b200host::encode_tiled(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                               const_cast<void*>(k_pool), dims, strides_b, box, es,
                               CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B) != CUDA_SUCCESS ||
        b200host::encode_tiled(&vmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                               const_cast<void*>(v_pool), dims, strides_b, box, es,
                               CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B) != CUDA_SUCCESS)
      return B200_ERR_TENSOR_MAP;
  }

  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_b = q_stride_b;
  a.q_h = q_stride_h;
  a.block_table = block_table;
  a.bt_row = bt_stride_row;
  a.seq_lens = seq_lens;
  a.row_ids = row_ids;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_b = out_stride_b;
  a.o_h = out_stride_h;
  a.ws_done = need > 0 ? static_cast<int32_t*>(workspace) : nullptr;
  a.ws_acc = need > 0 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes)
                      : nullptr;
  a.ws_ml = need > 0 ? a.ws_acc + static_cast<size_t>(batch) * num_heads * ms * kD : nullptr;
  a.batch = batch;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = G;
  a.num_blocks = num_blocks;
  a.max_pages = max_pages;
  a.max_requests = max_requests;
  a.pages_per_split = pages_per_split;
  a.max_splits = ms;
  a.scale_log2 = scale * kLog2e;
  a.dev_status = dev_status;
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.kn_b = kn_stride_b;
  a.kn_h = kn_stride_h;
  a.vn_b = vn_stride_b;
  a.vn_h = vn_stride_h;
  a.k_pool = static_cast<__nv_bfloat16*>(const_cast<void*>(k_pool));
  a.v_pool = static_cast<__nv_bfloat16*>(const_cast<void*>(v_pool));
  a.kv_blk = kv_stride_blk;
  a.kv_h = kv_stride_h;
  a.kv_slot = kv_stride_slot;

  int st = ensure_smem_attr(b200host::current_device());
  if (st != B200_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(static_cast<unsigned>(batch * num_kv_heads), static_cast<unsigned>(ms));
  // a programmatic dependent launch: the next layer's CTAs are launched while
  // this grid's last wave drains
  return b200host::status_from_cuda(b200host::launch_pdl(
      paged_decode_split_kernel, grid, dim3(kThreads), kSmemBytes, s, kmap, vmap, a));
}

}  // namespace

extern "C" int b200_paged_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                 const void* k_pool, const void* v_pool, int64_t kv_stride_blk,
                                 int64_t kv_stride_h, int64_t kv_stride_slot,
                                 const int32_t* block_table, int64_t bt_stride_row,
                                 const int32_t* seq_lens, const int32_t* row_ids, void* out,
                                 int64_t out_stride_b, int64_t out_stride_h, int batch,
                                 int num_heads, int num_kv_heads, int head_dim, int block_size,
                                 int num_blocks, int max_pages, int max_requests, float scale,
                                 int pages_per_split, void* workspace, size_t workspace_bytes,
                                 int32_t* dev_status, void* stream) {
  return launch_decode(q, q_stride_b, q_stride_h, nullptr, 0, 0, nullptr, 0, 0, k_pool, v_pool,
                       kv_stride_blk, kv_stride_h, kv_stride_slot, block_table, bt_stride_row,
                       seq_lens, row_ids, out, out_stride_b, out_stride_h, batch, num_heads,
                       num_kv_heads, head_dim, block_size, num_blocks, max_pages, max_requests,
                       scale, pages_per_split, workspace, workspace_bytes, dev_status, stream);
}

extern "C" int b200_paged_decode_kv_write(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_new,
    int64_t k_new_stride_b, int64_t k_new_stride_h, const void* v_new, int64_t v_new_stride_b,
    int64_t v_new_stride_h, void* k_pool, void* v_pool, int64_t kv_stride_blk,
    int64_t kv_stride_h, int64_t kv_stride_slot, const int32_t* block_table,
    int64_t bt_stride_row, const int32_t* seq_lens, const int32_t* row_ids, void* out,
    int64_t out_stride_b, int64_t out_stride_h, int batch, int num_heads, int num_kv_heads,
    int head_dim, int block_size, int num_blocks, int max_pages, int max_requests, float scale,
    int pages_per_split, void* workspace, size_t workspace_bytes, int32_t* dev_status,
    void* stream) {
  if (batch > 0 && (k_new == nullptr || v_new == nullptr)) return B200_ERR_INVALID_ARGUMENT;
  return launch_decode(q, q_stride_b, q_stride_h, k_new, k_new_stride_b, k_new_stride_h, v_new,
                       v_new_stride_b, v_new_stride_h, k_pool, v_pool, kv_stride_blk,
                       kv_stride_h, kv_stride_slot, block_table, bt_stride_row, seq_lens, row_ids,
                       out, out_stride_b, out_stride_h, batch, num_heads, num_kv_heads, head_dim,
                       block_size, num_blocks, max_pages, max_requests, scale, pages_per_split,
                       workspace, workspace_bytes, dev_status, stream);
}
