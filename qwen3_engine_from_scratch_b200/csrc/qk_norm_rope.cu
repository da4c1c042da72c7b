// Fused attention prologue: QK-RMSNorm + RoPE of q and k, and the KV-cache
// write of the roped k and of v, in one launch.  Replaces, per layer,
//   q = q_norm(q); k = k_norm(k)                      qwen3/attention.py:90-91,
//                                                     RMSNorm qwen3/norm.py:22-26
//   q, k = apply_rotary_pos_emb(q, k, cos, sin)       qwen3/attention.py:94-95,
//                                                     qwen3/rope.py:88-110
//   the KV write (update_kv_batch_triton, qwen3/kernels/paged_attention.py:292-377,
//   or PagedKVCache.update, qwen3/PagedKVcache.py:187-214)
// which the reference runs as separate elementwise launches.
//
// Rounding follows the reference's bf16 sequence exactly:
//   RMSNorm  y = bf16((x_f32 * rsqrt(mean(x_f32^2) + eps)) * w)
//   RoPE     c = bf16(cos), s = bf16(sin)           (.to(q.dtype), rope.py:106-107)
//            out = bf16(bf16(y * c) + bf16(rotate_half(y) * s))
// with rotate_half(y) = cat(-y[64:], y[:64]).  The cos/sin rows are the ones
// the reference's RotaryEmbedding gathered (fp32, (B, S, D)).
//
// One warp per token: it converts the token's cos/sin row and finds its pool
// slot once, then takes the token's rows 8 at a time (one warp per 8 rows cost
// every warp that per-token work: 129.3 -> 108.9 us on the C3 tokens).  With
// 16-byte aligned rows a half-warp holds a row, lane l of it elements
// 8l..8l+7, and a pass covers two rows; otherwise a warp holds a row, lane l
// elements 4l..4l+3.  The RoPE partner of a lane is the lane half a row away
// (l ^ 8, or l ^ 16).  A warp issues a group's 8 row loads before its math.  Rows of a
// token: the q heads, then the k heads, then (when a pool is given) the v
// heads.  A k row goes to k_out (optional) and to the pool slot of its
// position; a v row only to the pool.  Pool addressing is the rows mode of the KV write: position =
// seq_lens[row_ids[b]] + s.  Every index is range-checked; a bad one sets a
// dev_status bit and the row's pool write is skipped.
#include <type_traits>

#include "common.cuh"

namespace {

constexpr int kD = 128;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerWarp = 8;  // rows (q, k or v heads) of one token per load group

struct PrologueArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_b, q_h, q_s, k_b, k_h, k_s, v_b, v_h, v_s;
  const __nv_bfloat16* q_w;
  const __nv_bfloat16* k_w;
  float eps;
  const float* cos;
  const float* sin;
  int64_t cs_b, cs_s;
  __nv_bfloat16* q_out;
  int64_t qo_b, qo_h, qo_s;
  __nv_bfloat16* k_out;  // nullable
  int64_t ko_b, ko_h, ko_s;
  __nv_bfloat16* k_pool;  // nullable (no KV write)
  __nv_bfloat16* v_pool;
  int64_t kp_blk, kp_layer, kp_h, kp_slot, vp_blk, vp_layer, vp_h, vp_slot;
  const int32_t* seq_lens;
  const int32_t* block_table;
  int64_t bt_row;
  const int32_t* row_ids;
  int batch, n_tokens, num_heads, num_kv_heads, block_size, num_blocks, max_pages, max_requests,
      layer;
  int total_warps;  // batch * n_tokens: one warp per token (below 2^31)
  int32_t* dev_status;
};

// Pool slot of token (b, s): writes the element offset of (phys, layer, h=0,
// off) into *k_off / *v_off; false (and a status bit from lane 0) if an index
// is out of range.
B200_DEVICE bool pool_slot(const PrologueArgs& a, int b, int s, int lane, int64_t* k_off,
                           int64_t* v_off) {
  const int row = a.row_ids[b];
  if (row < 0 || row >= a.max_requests) {
    if (lane == 0) b200::flag_error(a.dev_status, B200_DEV_BAD_ROW);
    return false;
  }
  const int64_t pos = static_cast<int64_t>(a.seq_lens[row]) + s;
  const int64_t page = pos / a.block_size;
  if (pos < 0 || page >= a.max_pages) {
    if (lane == 0) b200::flag_error(a.dev_status, B200_DEV_SEQ_OVERFLOW);
    return false;
  }
  const int phys = a.block_table[row * a.bt_row + page];
  if (phys < 0 || phys >= a.num_blocks) {
    if (lane == 0) b200::flag_error(a.dev_status, B200_DEV_BAD_PAGE);
    return false;
  }
  const int64_t off = pos - page * a.block_size;
  *k_off = phys * a.kp_blk + a.layer * a.kp_layer + off * a.kp_slot;
  *v_off = phys * a.vp_blk + a.layer * a.vp_layer + off * a.vp_slot;
  return true;
}

// Packed bf16 pair arithmetic (one rounding of the exact result, as the
// reference's bf16 tensor ops round their fp32 result: for bf16 operands the
// fp32 product is exact, and an fp32 sum is either exact or rounds to the
// same bf16 value as the exact sum).
B200_DEVICE uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
B200_DEVICE uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// fp32 pair of the two bf16 halves of w
B200_DEVICE uint64_t bf2_to_f2(uint32_t w) {
  return b200::f2_pack(b200::bf16_lo(w), b200::bf16_hi(w));
}

// VEC elements of a row per lane: 8 (a row per half-warp, two rows per pass,
// 16-byte accesses; needs 16-byte aligned rows) or 4 (a row per warp, 8-byte
// accesses).  With 8 the per-row work of a lane (addresses, the reduction,
// the rsqrt, the weights) is spread over twice the elements.  After the
// normalisation every value is a packed bf16 pair: the RoPE partner is
// exchanged as pairs and the products and the sum are packed bf16 operations.
// The launch bound of 4 CTAs per SM keeps the kernel at 64 registers without
// spills: at 3 CTAs (67 registers) it was bound by the warps it could keep in
// flight.
template <int VEC>
__global__ void __launch_bounds__(kThreads, 4) qk_norm_rope_kv_write_kernel(const PrologueArgs a) {
  // launched with b200host::launch_pdl: nothing read or written before this
  b200::pdl_begin();
  constexpr int kLanesPerRow = kD / VEC;        // 16 or 32
  constexpr int kRowsPerPass = 32 / kLanesPerRow;
  constexpr int kPasses = kRowsPerWarp / kRowsPerPass;
  constexpr int kWords = VEC / 2;               // packed bf16 pairs per lane and row
  using Vec = typename std::conditional<VEC == 8, uint4, uint2>::type;
  const int lane = threadIdx.x & 31;
  const int heads = a.num_heads + (a.k_pool != nullptr ? 2 : 1) * a.num_kv_heads;
  // one warp per token: the token's cos/sin and pool slot once, then its rows
  // 8 at a time; the host keeps the warp count below 2^31 (32-bit indices)
  const int tok = static_cast<int>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (tok >= a.total_warps) return;
  const int b = tok / a.n_tokens;
  const int s = tok - b * a.n_tokens;
  const int sub = lane / kLanesPerRow;          // row of the pass this lane works on
  const int li = lane % kLanesPerRow;
  const int d = VEC * li;
  // cos / sin of this lane's elements as bf16 pairs (.to(q.dtype), rope.py:106-107)
  uint32_t c2[kWords], s2[kWords];
#pragma unroll
  for (int e = 0; e < VEC; e += 4) {
    const float4 c4 = *reinterpret_cast<const float4*>(a.cos + b * a.cs_b + s * a.cs_s + d + e);
    const float4 s4 = *reinterpret_cast<const float4*>(a.sin + b * a.cs_b + s * a.cs_s + d + e);
    c2[e / 2] = b200::pack_bf16x2(c4.x, c4.y);
    c2[e / 2 + 1] = b200::pack_bf16x2(c4.z, c4.w);
    s2[e / 2] = b200::pack_bf16x2(s4.x, s4.y);
    s2[e / 2 + 1] = b200::pack_bf16x2(s4.z, s4.w);
  }
  // rotate_half negates the partner for the first half of the row
  const uint32_t neg = li < kLanesPerRow / 2 ? 0x80008000u : 0u;

  int64_t k_off = 0, v_off = 0;
  bool write_pool = false, pool_done = false;

  for (int h0 = 0; h0 < heads; h0 += kRowsPerWarp) {
  const int nrows = min(kRowsPerWarp, heads - h0);
  // every row load of this group is issued before any math (memory-level parallelism)
  Vec raw[kPasses];
#pragma unroll
  for (int i = 0; i < kPasses; ++i) {
    const int hh = h0 + kRowsPerPass * i + sub;
    if (hh - h0 < nrows) {
      const __nv_bfloat16* src;
      if (hh < a.num_heads) {
        src = a.q + b * a.q_b + hh * a.q_h + s * a.q_s;
      } else if (hh < a.num_heads + a.num_kv_heads) {
        src = a.k + b * a.k_b + (hh - a.num_heads) * a.k_h + s * a.k_s;
      } else {
        src = a.v + b * a.v_b + (hh - a.num_heads - a.num_kv_heads) * a.v_h + s * a.v_s;
      }
      raw[i] = *reinterpret_cast<const Vec*>(src + d);
    }
  }
  if (!pool_done && h0 + nrows > a.num_heads) {
    // the token's pool slot, once, after the first rows that need it were requested
    write_pool = a.k_pool != nullptr && pool_slot(a, b, s, lane, &k_off, &v_off);
    pool_done = true;
  }
#pragma unroll
  for (int i = 0; i < kPasses; ++i) {
    if (kRowsPerPass * i >= nrows) break;
    const int hh = h0 + kRowsPerPass * i + sub;
    const bool live = hh - h0 < nrows;  // the pass's second row may lie past the chunk
    const bool is_q = hh < a.num_heads;
    const bool is_k = !is_q && hh < a.num_heads + a.num_kv_heads;
    if (h0 + kRowsPerPass * i >= a.num_heads + a.num_kv_heads) {
      // every row of this pass is a v row (the same for the whole warp): a copy
      if (live && write_pool)
        *reinterpret_cast<Vec*>(a.v_pool + v_off + (hh - a.num_heads - a.num_kv_heads) * a.vp_h +
                                d) = raw[i];
      continue;
    }
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(&raw[i]);
    // the reduction and the RoPE exchange are shuffles over the whole warp,
    // so every lane takes part; v rows and dead rows contribute zeros
    const bool norm = live && (is_q || is_k);
    // RMSNorm in fp32: mean of squares over the 128 elements of the row
    float ss = 0.f;
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
      const float x0 = b200::bf16_lo(rw[w]), x1 = b200::bf16_hi(rw[w]);
      ss = fmaf(x0, x0, ss);
      ss = fmaf(x1, x1, ss);
    }
    if (!norm) ss = 0.f;
#pragma unroll
    for (int o = kLanesPerRow / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rms = __frsqrt_rn(ss / static_cast<float>(kD) + a.eps);
    const uint64_t rms2 = b200::f2_pack(rms, rms);
    const __nv_bfloat16* wp = (is_q ? a.q_w : a.k_w) + d;
    const Vec wv = *reinterpret_cast<const Vec*>(wp);
    const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
    // y = bf16((x * rms) * w), then RoPE: bf16(bf16(y * c) + bf16(rot(y) * s))
    uint32_t out_w[kWords];
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
      float y0, y1;
      b200::f2_unpack(b200::f2_mul(b200::f2_mul(bf2_to_f2(rw[w]), rms2), bf2_to_f2(ww[w])), y0, y1);
      const uint32_t y2 = b200::pack_bf16x2(y0, y1);
      const uint32_t rot = __shfl_xor_sync(0xffffffffu, y2, kLanesPerRow / 2) ^ neg;
      out_w[w] = bf2_add(bf2_mul(y2, c2[w]), bf2_mul(rot, s2[w]));
    }
    const Vec out = *reinterpret_cast<const Vec*>(out_w);
    if (!live) continue;
    if (is_q) {
      *reinterpret_cast<Vec*>(a.q_out + b * a.qo_b + hh * a.qo_h + s * a.qo_s + d) = out;
    } else if (is_k) {
      const int h = hh - a.num_heads;
      if (a.k_out != nullptr)
        *reinterpret_cast<Vec*>(a.k_out + b * a.ko_b + h * a.ko_h + s * a.ko_s + d) = out;
      if (write_pool) *reinterpret_cast<Vec*>(a.k_pool + k_off + h * a.kp_h + d) = out;
    } else if (write_pool) {  // v row: a plain copy into the pool
      *reinterpret_cast<Vec*>(a.v_pool + v_off + (hh - a.num_heads - a.num_kv_heads) * a.vp_h +
                              d) = raw[i];
    }
  }
  }
}

bool mult8(int64_t s) { return (s & 7) == 0; }

}  // namespace

extern "C" int b200_qk_norm_rope_kv_write(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s, const void* k,
    int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s, const void* v,
    int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s, const void* q_weight,
    const void* k_weight, float eps, const float* cos, const float* sin, int64_t cs_stride_b,
    int64_t cs_stride_s, void* q_out, int64_t qo_stride_b, int64_t qo_stride_h,
    int64_t qo_stride_s, void* k_out, int64_t ko_stride_b, int64_t ko_stride_h,
    int64_t ko_stride_s, void* k_pool, void* v_pool, int64_t kp_stride_blk,
    int64_t kp_stride_layer, int64_t kp_stride_h, int64_t kp_stride_slot, int64_t vp_stride_blk,
    int64_t vp_stride_layer, int64_t vp_stride_h, int64_t vp_stride_slot,
    const int32_t* seq_lens, const int32_t* block_table, int64_t bt_stride_row,
    const int32_t* row_ids, int batch, int n_tokens, int num_heads, int num_kv_heads,
    int head_dim, int block_size, int num_blocks, int max_pages, int max_requests, int layer,
    int32_t* dev_status, void* stream) {
  if (batch < 0 || n_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0)
    return B200_ERR_INVALID_ARGUMENT;
  if (batch == 0 || n_tokens == 0) return B200_OK;
  if (head_dim != kD) return B200_ERR_UNSUPPORTED;
  if (!q || !k || !q_weight || !k_weight || !cos || !sin || !q_out)
    return B200_ERR_INVALID_ARGUMENT;
  const bool pool = k_pool != nullptr;
  if (pool) {
    if (!v || !v_pool || !seq_lens || !block_table || !row_ids || block_size <= 0 ||
        num_blocks <= 0 || max_pages <= 0 || max_requests <= 0 || bt_stride_row <= 0 ||
        layer < 0)
      return B200_ERR_INVALID_ARGUMENT;
  }
  // 8-byte row pieces for the bf16 rows, 16-byte pieces for the fp32 cos/sin rows
  const void* ptrs8[] = {q, k, q_weight, k_weight, q_out};
  for (const void* p : ptrs8)
    if ((reinterpret_cast<uintptr_t>(p) & 7) != 0) return B200_ERR_ALIGNMENT;
  if (!b200host::aligned16(cos) || !b200host::aligned16(sin)) return B200_ERR_ALIGNMENT;
  if ((cs_stride_b & 3) != 0 || (cs_stride_s & 3) != 0) return B200_ERR_ALIGNMENT;
  const int64_t strides[] = {q_stride_b, q_stride_h, q_stride_s, k_stride_b, k_stride_h,
                             k_stride_s, qo_stride_b, qo_stride_h, qo_stride_s};
  for (int64_t st : strides)
    if ((st & 3) != 0) return B200_ERR_ALIGNMENT;
  if (k_out != nullptr) {
    if ((reinterpret_cast<uintptr_t>(k_out) & 7) != 0 || (ko_stride_b & 3) != 0 ||
        (ko_stride_h & 3) != 0 || (ko_stride_s & 3) != 0)
      return B200_ERR_ALIGNMENT;
  }
  if (pool) {
    if ((reinterpret_cast<uintptr_t>(v) & 7) != 0 || !b200host::aligned16(k_pool) ||
        !b200host::aligned16(v_pool))
      return B200_ERR_ALIGNMENT;
    const int64_t ps[] = {v_stride_b, v_stride_h, v_stride_s, kp_stride_blk, kp_stride_layer,
                          kp_stride_h, kp_stride_slot, vp_stride_blk, vp_stride_layer,
                          vp_stride_h, vp_stride_slot};
    for (int64_t st : ps)
      if ((st & 3) != 0) return B200_ERR_ALIGNMENT;
  }
  const int heads = num_heads + (pool ? 2 : 1) * num_kv_heads;
  const int64_t warps = static_cast<int64_t>(batch) * n_tokens;  // one warp per token
  if (warps > 0x7fffffff - kWarps) return B200_ERR_INVALID_ARGUMENT;
  const int64_t blocks = (warps + kWarps - 1) / kWarps;

  PrologueArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.q_b = q_stride_b;
  a.q_h = q_stride_h;
  a.q_s = q_stride_s;
  a.k_b = k_stride_b;
  a.k_h = k_stride_h;
  a.k_s = k_stride_s;
  a.v_b = v_stride_b;
  a.v_h = v_stride_h;
  a.v_s = v_stride_s;
  a.q_w = static_cast<const __nv_bfloat16*>(q_weight);
  a.k_w = static_cast<const __nv_bfloat16*>(k_weight);
  a.eps = eps;
  a.cos = cos;
  a.sin = sin;
  a.cs_b = cs_stride_b;
  a.cs_s = cs_stride_s;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.qo_b = qo_stride_b;
  a.qo_h = qo_stride_h;
  a.qo_s = qo_stride_s;
  a.k_out = static_cast<__nv_bfloat16*>(k_out);
  a.ko_b = ko_stride_b;
  a.ko_h = ko_stride_h;
  a.ko_s = ko_stride_s;
  a.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  a.kp_blk = kp_stride_blk;
  a.kp_layer = kp_stride_layer;
  a.kp_h = kp_stride_h;
  a.kp_slot = kp_stride_slot;
  a.vp_blk = vp_stride_blk;
  a.vp_layer = vp_stride_layer;
  a.vp_h = vp_stride_h;
  a.vp_slot = vp_stride_slot;
  a.seq_lens = seq_lens;
  a.block_table = block_table;
  a.bt_row = bt_stride_row;
  a.row_ids = row_ids;
  a.batch = batch;
  a.n_tokens = n_tokens;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.max_pages = max_pages;
  a.max_requests = max_requests;
  a.layer = layer;
  a.total_warps = static_cast<int>(warps);
  a.dev_status = dev_status;
  // 16-byte row pieces when every row and the weights allow them
  bool v16 = b200host::aligned16(q) && b200host::aligned16(k) && b200host::aligned16(q_weight) &&
             b200host::aligned16(k_weight) && b200host::aligned16(q_out);
  for (int64_t st : strides) v16 = v16 && mult8(st);
  if (k_out != nullptr)
    v16 = v16 && b200host::aligned16(k_out) && mult8(ko_stride_b) && mult8(ko_stride_h) &&
          mult8(ko_stride_s);
  if (pool) {
    v16 = v16 && b200host::aligned16(v) && mult8(v_stride_b) && mult8(v_stride_h) &&
          mult8(v_stride_s) && mult8(kp_stride_blk) && mult8(kp_stride_layer) &&
          mult8(kp_stride_h) && mult8(kp_stride_slot) && mult8(vp_stride_blk) &&
          mult8(vp_stride_layer) && mult8(vp_stride_h) && mult8(vp_stride_slot);
  }
  const dim3 grid(static_cast<unsigned>(blocks));
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  return b200host::status_from_cuda(
      v16 ? b200host::launch_pdl(qk_norm_rope_kv_write_kernel<8>, grid, dim3(kThreads), 0, s, a)
          : b200host::launch_pdl(qk_norm_rope_kv_write_kernel<4>, grid, dim3(kThreads), 0, s, a));
}
