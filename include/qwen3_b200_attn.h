/*
 * qwen3_b200_attn.h -- C ABI of the B200 (sm_100a) attention hot path for the
 * Qwen3 inference engine (uphome/Qwen3-engine-from-scratch).
 *
 * Three operations, each a hand-written CUDA kernel behind a plain-C entry
 * point: raw device pointers, element strides, sizes, a CUDA stream.  No torch
 * types cross this boundary.  All entry points only enqueue work on `stream`
 * (no host synchronisation, no allocation, grid sizes derived from shapes
 * only), so they can be captured in a CUDA graph.  The decode, prologue and
 * KV-scatter kernels are launched as programmatic dependents of the previous
 * kernel on `stream` (their CTAs may be scheduled while it drains); each one
 * waits for that kernel's completion before its first memory access, so the
 * stream order callers see is that of an ordinary launch.
 *
 * Conventions
 *   - bf16 tensors are passed as `const void*` / `void*` (2-byte elements).
 *   - Strides are in ELEMENTS (like torch.Tensor.stride()), int64.
 *   - The innermost (head_dim) stride must be 1.
 *   - The KV pool has the reference layout
 *       (num_blocks, num_layers, num_kv_heads, block_size, head_dim)
 *     (qwen3/PagedKVcache.py:50-53); block_size must be 16, head_dim 128.
 *   - `dev_status` (nullable) points to one int32 in device memory; kernels
 *     OR B200_DEV_* bits into it when they meet an out-of-range index (the
 *     offending access is skipped, never performed).  Read it back with a
 *     plain device-to-host copy when convenient.
 *   - Return value: B200_OK (0) or a negative b200_status; nothing is
 *     launched when an argument check fails.  No entry point aborts/exits.
 */
#ifndef QWEN3_B200_ATTN_H
#define QWEN3_B200_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  B200_OK = 0,
  B200_ERR_INVALID_ARGUMENT = -1, /* null pointer, bad size or stride       */
  B200_ERR_UNSUPPORTED = -2,      /* head_dim / block_size / GQA group size  */
  B200_ERR_ALIGNMENT = -3,        /* pointer or stride not 16-byte aligned   */
  B200_ERR_WORKSPACE = -4,        /* workspace missing or too small          */
  B200_ERR_CUDA = -5,             /* launch / driver error                   */
  B200_ERR_TENSOR_MAP = -6        /* TMA descriptor could not be encoded     */
} b200_status;

/* Bits OR-ed into *dev_status by the kernels. */
#define B200_DEV_BAD_ROW 0x1      /* row_ids[b] outside [0, max_requests)       */
#define B200_DEV_BAD_PAGE 0x2     /* block-table entry outside [0, num_blocks)  */
#define B200_DEV_BAD_SLOT 0x4     /* slot_mapping entry past the pool           */
#define B200_DEV_SEQ_OVERFLOW 0x8 /* position needs a page past max_pages       */
#define B200_DEV_TIMEOUT 0x10     /* a bounded pipeline wait gave up            */
#define B200_DEV_BAD_PARAM 0x20   /* a per-row parameter outside its range      */

/* Human-readable text for a b200_status value. */
const char* b200_status_string(int status);

/* Text of the last CUDA error an entry point of this library met on the
 * calling thread (behind a B200_ERR_CUDA return). */
const char* b200_last_cuda_error_string(void);

/* Failure-detection self-test (no counterpart in the reference, whose Triton
 * kernels have no bounded waits): launches one warp on `stream` that waits on
 * an mbarrier nothing completes, through the same bounded wait every pipeline
 * wait of the prefill kernel uses.  The wait gives up after `limit_ns`
 * nanoseconds of device time (1 ns .. 10 s), or as soon as *dev_status already
 * holds B200_DEV_TIMEOUT (how one timed-out CTA ends the rest of its grid),
 * then ORs B200_DEV_TIMEOUT into *dev_status and writes 0 to *result (1 if the
 * wait had completed).  The kernel returns normally: the CUDA context stays
 * usable, and kernels that check the status word (the prefill) start no new
 * work until the caller clears it. */
int b200_selftest_bounded_wait(int32_t* dev_status, int32_t* result, uint64_t limit_ns,
                               void* stream);

/* ABI version of this library (major*100 + minor). */
int b200_abi_version(void);

/* Number of SMs of the current device (cached per device); <0 on error. */
int b200_device_sm_count(void);

/*
 * KV-cache write, row addressed.  For request b (0 <= b < batch) and token s
 * (0 <= s < n_tokens), head h:
 *     row  = row_ids[b];  pos = seq_lens[row] + s;
 *     phys = block_table[row * bt_stride_row + pos / 16];  off = pos % 16;
 *     k_pool[phys, layer, h, off, :] = k_new[b, h, s, :]   (same for v)
 * n_tokens == 1 replaces update_kv_batch_triton
 *   (qwen3/kernels/paged_attention.py:353-377, kernel :292-350) as called by
 *   KVCachePool.update_kv_batch (qwen3/PagedKVcache.py:99-114);
 * n_tokens  > 1 replaces the per-request prefill write of
 *   PagedKVCache.update (qwen3/PagedKVcache.py:187-214, called per request at
 *   qwen3/attention.py:160-161) for a whole right-padded batch in one launch.
 * k_new/v_new strides: (batch, head, token), head_dim stride 1.
 * Pool strides: (block, layer, head, slot), head_dim stride 1.
 */
int b200_kv_scatter_rows(const void* k_new, const void* v_new,
                         int64_t kn_stride_b, int64_t kn_stride_h, int64_t kn_stride_s,
                         int64_t vn_stride_b, int64_t vn_stride_h, int64_t vn_stride_s,
                         void* k_pool, void* v_pool,
                         int64_t kp_stride_blk, int64_t kp_stride_layer,
                         int64_t kp_stride_h, int64_t kp_stride_slot,
                         int64_t vp_stride_blk, int64_t vp_stride_layer,
                         int64_t vp_stride_h, int64_t vp_stride_slot,
                         const int32_t* seq_lens, const int32_t* block_table,
                         int64_t bt_stride_row, const int32_t* row_ids,
                         int batch, int n_tokens, int num_kv_heads, int head_dim,
                         int block_size, int num_blocks, int max_pages, int max_requests,
                         int layer, int32_t* dev_status, void* stream);

/*
 * KV-cache write, slot addressed (vLLM store_kvcache convention).  Token t:
 *     slot = slot_mapping[t]; if slot < 0: skip;
 *     k_pool[slot / 16, layer, h, slot % 16, :] = k[t, h, :]   (same for v)
 * The same pool addressing as PagedKVCache.update (qwen3/PagedKVcache.py:198-214)
 * with (phys, off) flattened; used by packed varlen prefill.
 * slot_mapping is int32 (slot_is_int64 == 0) or int64 (slot_is_int64 != 0).
 */
int b200_kv_scatter_slots(const void* k, const void* v,
                          int64_t k_stride_t, int64_t k_stride_h,
                          int64_t v_stride_t, int64_t v_stride_h,
                          void* k_pool, void* v_pool,
                          int64_t kp_stride_blk, int64_t kp_stride_layer,
                          int64_t kp_stride_h, int64_t kp_stride_slot,
                          int64_t vp_stride_blk, int64_t vp_stride_layer,
                          int64_t vp_stride_h, int64_t vp_stride_slot,
                          const void* slot_mapping, int slot_is_int64,
                          int n_tokens, int num_kv_heads, int head_dim, int block_size,
                          int num_blocks, int layer, int32_t* dev_status, void* stream);

/*
 * KV-cache write of one request from a host position: replaces the body of
 * PagedKVCache.update (qwen3/PagedKVcache.py:187-214), whose write position is
 * the handle's host-side seq_len.  Token s (0 <= s < n_tokens), head h:
 *     pos  = start_pos + s;  page = pos / 16;  (page < num_pages, else flagged
 *            B200_DEV_SEQ_OVERFLOW and skipped, where the reference's
 *            block_table_tensor[:num_pages][page] would raise)
 *     phys = block_table_row[page];  off = pos % 16;
 *     k_pool[phys, layer, h, off, :] = k_new[h, s, :]   (same for v)
 * block_table_row: the handle's row of the 2-D block table (num_pages entries
 * allocated); k_new/v_new (num_kv_heads, n_tokens, head_dim) with strides
 * (head, token), head_dim stride 1.  Pool strides as b200_kv_scatter_rows.
 */
int b200_kv_scatter_span(const void* k_new, const void* v_new,
                         int64_t kn_stride_h, int64_t kn_stride_s,
                         int64_t vn_stride_h, int64_t vn_stride_s,
                         void* k_pool, void* v_pool,
                         int64_t kp_stride_blk, int64_t kp_stride_layer,
                         int64_t kp_stride_h, int64_t kp_stride_slot,
                         int64_t vp_stride_blk, int64_t vp_stride_layer,
                         int64_t vp_stride_h, int64_t vp_stride_slot,
                         const int32_t* block_table_row, int num_pages, int start_pos,
                         int n_tokens, int num_kv_heads, int head_dim, int block_size,
                         int num_blocks, int layer, int32_t* dev_status, void* stream);

/*
 * Split-K paged decode: workspace bytes needed for `batch` requests, `num_heads`
 * query heads and a block table `max_pages` wide, with `pages_per_split`
 * pages per split.  <= 0 returns enough for any split the library may pick by
 * default (pass b200_paged_decode_default_split(...) to size it exactly).
 * Depends on shapes only.
 */
size_t b200_paged_decode_workspace_size(int batch, int num_heads, int max_pages,
                                        int pages_per_split);

/* The split size the library picks for these shapes when pages_per_split <= 0:
 * large splits (up to 128 pages), but enough CTAs for about 4 per SM when the
 * sequences fill half of the block table (depends on the current device's SM
 * count). */
int b200_paged_decode_default_split(int batch, int num_kv_heads, int max_pages);

/*
 * Paged decode attention (flash-decoding).  For request b, query head h:
 *     row = row_ids[b];  L = seq_lens[row] + 1;
 *     out[b,h,:] = softmax_j(scale * q[b,h,:].k_j) . v_j  over tokens j < L,
 * token j of the request at page block_table[row, j/16], slot j%16, kv head
 * h / (num_heads/num_kv_heads).  Replaces paged_attn_decode_kernel and
 * paged_attention_decode_triton (qwen3/kernels/paged_attention.py:27-178).
 * k_pool/v_pool point at the layer's first element (pool + layer*stride_layer),
 * strides (block, head, slot) in elements, head_dim stride 1.
 * q strides (batch, head); out strides (batch, head).  fp32 softmax, bf16 out.
 * `workspace` must hold b200_paged_decode_workspace_size(...) bytes (16-byte
 * aligned) when that size is non-zero.  Its first 256 KiB are split-arrival
 * counters (one per request x kv head, at most 65536 pairs): zero-fill the
 * workspace once when it is allocated; every launch leaves the counters zero,
 * so the same workspace serves later launches of any shape on one stream.
 * The rest carries the per-split partials, merged by the last split of each
 * (request, kv head) inside the same kernel.  Launches that may overlap on
 * the GPU need separate workspaces.
 */
int b200_paged_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                      const void* k_pool, const void* v_pool,
                      int64_t kv_stride_blk, int64_t kv_stride_h, int64_t kv_stride_slot,
                      const int32_t* block_table, int64_t bt_stride_row,
                      const int32_t* seq_lens, const int32_t* row_ids,
                      void* out, int64_t out_stride_b, int64_t out_stride_h,
                      int batch, int num_heads, int num_kv_heads, int head_dim,
                      int block_size, int num_blocks, int max_pages, int max_requests,
                      float scale, int pages_per_split,
                      void* workspace, size_t workspace_bytes,
                      int32_t* dev_status, void* stream);

/*
 * Decode step of one layer with the KV write fused in: replaces the pair
 * update_kv_batch_triton + paged_attention_decode_triton that
 * triton_paged_attention_decode_batch issues (qwen3/kernels/paged_attention.py:
 * 222-289, the write :292-377).  k_new / v_new (batch, num_kv_heads, head_dim)
 * bf16, strides (batch, head), are stored at position seq_lens[row_ids[b]] of
 * the pool (k_pool / v_pool: the layer's first element, writable) exactly as
 * b200_kv_scatter_rows with n_tokens == 1 stores them, and the decode then
 * attends over seq_lens[row] + 1 tokens, the new one included; one launch.
 * All other arguments, the workspace and the results as b200_paged_decode.
 * A bad block-table entry for the new position sets B200_DEV_BAD_PAGE and
 * skips the store.
 */
int b200_paged_decode_kv_write(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                               const void* k_new, int64_t k_new_stride_b, int64_t k_new_stride_h,
                               const void* v_new, int64_t v_new_stride_b, int64_t v_new_stride_h,
                               void* k_pool, void* v_pool,
                               int64_t kv_stride_blk, int64_t kv_stride_h, int64_t kv_stride_slot,
                               const int32_t* block_table, int64_t bt_stride_row,
                               const int32_t* seq_lens, const int32_t* row_ids,
                               void* out, int64_t out_stride_b, int64_t out_stride_h,
                               int batch, int num_heads, int num_kv_heads, int head_dim,
                               int block_size, int num_blocks, int max_pages, int max_requests,
                               float scale, int pages_per_split,
                               void* workspace, size_t workspace_bytes,
                               int32_t* dev_status, void* stream);

/*
 * Paged decode without a caller-provided workspace (allocation-free variant).
 * No counterpart in the reference: its Triton decode needs no workspace, and
 * the split-K design here does.  For callers that cannot allocate device
 * memory when they launch decode -- engines that give nearly all HBM to the KV
 * pool and run a fixed arena, FFI bindings holding raw device pointers but no
 * device allocator, loops that must not pay cudaMalloc's latency or its
 * implicit synchronisation.  Same arguments and results as b200_paged_decode
 * minus the workspace: the split workspace lives in a file-scope device array
 * of B200_DECODE_NOALLOC_SCRATCH_BYTES per GPU (held until process exit).
 * Returns B200_ERR_WORKSPACE when b200_paged_decode_workspace_size(batch,
 * num_heads, max_pages, s) exceeds that maximum, s being the split the call
 * uses: pages_per_split if > 0, else b200_paged_decode_default_split(batch,
 * num_kv_heads, max_pages) -- not the worst-case figure that
 * workspace_size(..., 0) reports, which can refuse shapes this entry accepts.
 * Calls no allocator.  The array starts with the split-arrival counters, which
 * must be zero at launch: every call clears those of its own pairs with one
 * cudaMemsetAsync on `stream` before the kernel.  The first call in a CUDA
 * context looks up the array's device address (cached per device and context
 * id); make it before any stream capture on that device, and again after a
 * device reset.  All calls on a device share the array: calls whose kernels
 * overlap on the GPU (unordered streams) race and must not be issued.
 */
#define B200_DECODE_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int b200_paged_decode_noalloc(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                              const void* k_pool, const void* v_pool,
                              int64_t kv_stride_blk, int64_t kv_stride_h, int64_t kv_stride_slot,
                              const int32_t* block_table, int64_t bt_stride_row,
                              const int32_t* seq_lens, const int32_t* row_ids,
                              void* out, int64_t out_stride_b, int64_t out_stride_h,
                              int batch, int num_heads, int num_kv_heads, int head_dim,
                              int block_size, int num_blocks, int max_pages, int max_requests,
                              float scale, int pages_per_split,
                              int32_t* dev_status, void* stream);

/*
 * Varlen causal prefill attention.  Sequence i owns rows
 * [cu_seqlens[i], cu_seqlens[i] + len_i) of the packed q/k/v/out tensors, with
 * len_i = cu_seqlens[i+1] - cu_seqlens[i] when seq_lens_opt is NULL (packed
 * varlen) or len_i = seq_lens_opt[i] (right-padded batch: cu_seqlens[i] =
 * i * S).  Query row m attends keys n <= m of its own sequence; q head h reads
 * kv head h / (num_heads/num_kv_heads); fp32 online softmax, bf16 output.
 * Replaces flash_attention_varlen_kernel / flash_attention_prefill
 * (qwen3/kernels/flash_attention_varlen.py:25-194) without its host sync:
 * `max_seqlen` (>= every len_i, <= 262144) sizes the work list.  With
 * zero_pad_rows != 0 the rows [cu_seqlens[i] + len_i, cu_seqlens[i] +
 * max_seqlen) of `out` are set to zero, as the padded-batch adapter does
 * (flash_attention_varlen.py:255-257).
 * q (T, H, D), k/v (T, Hkv, D): token and head strides in elements, head_dim
 * stride 1; out (T, H, D) with strides (token, head).  head_dim must be 128.
 * work_counter (nullable): two int32 in device memory, zero at launch; the
 * kernel hands out work items through them (balanced dynamically) and leaves
 * them zero when it finishes.  Launches that may overlap on the GPU need
 * separate counters.  NULL selects a fixed, slightly less balanced order.
 */
int b200_varlen_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                        const void* k, int64_t k_stride_t, int64_t k_stride_h,
                        const void* v, int64_t v_stride_t, int64_t v_stride_h,
                        void* out, int64_t o_stride_t, int64_t o_stride_h,
                        const int32_t* cu_seqlens, const int32_t* seq_lens_opt,
                        int num_seqs, int total_tokens, int max_seqlen,
                        int num_heads, int num_kv_heads, int head_dim,
                        float scale, int zero_pad_rows, int32_t* work_counter,
                        int32_t* dev_status, void* stream);

/*
 * Fused token sampling.  Replaces the reference's sample_tokens Triton path:
 * the batched torch.topk (qwen3/sampling.py:215-216) and _sample_topk_kernel
 * (qwen3/sampling.py:112-178), plus its greedy argmax (:253-254), in one launch.
 * logits (batch, vocab) fp32 (logits_bf16 = 0) or bf16, row stride in elements;
 * temperature / top_k / top_p: per-row device arrays, each nullable: NULL
 * gives every row the matching *_all value.  Per row:
 *   temperature <= 0: argmax (first index of the maximum);
 *   1 <= top_k <= 1024: the k largest logits (ties by ascending index),
 *     x = logit / temperature, softmax, keep rank 0 and every rank whose
 *     preceding probability mass is <= top_p, Gumbel-max with the uniform
 *     of Triton's tl.rand(seed, row * block_k + rank) (Philox4x32-10), as the
 *     reference kernel does (block_k = max(16, next power of two of the
 *     batch's largest top_k) reproduces its random stream);
 *   top_k == 0 and top_p >= 1: Gumbel-max over the whole row (uniforms at
 *     row * vocab + index).
 * Other top_k values are clamped to 1024 and flagged B200_DEV_BAD_PARAM.
 * Two launches: chunks of 8192 logits select their candidates into
 * `workspace` (b200_sample_workspace_size(batch, vocab, block_k) bytes,
 * 16-byte aligned, no initialisation needed), then one CTA per row merges
 * them and samples.  vocab <= 262144.  out: (batch,) int64 token ids.
 */
size_t b200_sample_workspace_size(int batch, int vocab, int block_k);
int b200_sample_tokens(const void* logits, int logits_bf16, int64_t stride_row, int batch,
                       int vocab, const float* temperature, const int32_t* top_k,
                       const float* top_p, float temperature_all, int top_k_all,
                       float top_p_all, uint64_t seed, int block_k, void* workspace,
                       size_t workspace_bytes, int64_t* out, int32_t* dev_status, void* stream);

/*
 * Chunked prefill over the paged KV cache (prefix continuation).  No
 * counterpart in the reference: its prefill ignores cached context
 * (qwen3/attention.py:109-120; chunked prefill and prefix caching are open
 * items of its ENGINE_COMPARISON.md).  Sequence i has ctx_i =
 * seq_lens[row_ids[i]] tokens cached and len_i = cu_seqlens[i+1] -
 * cu_seqlens[i] new tokens, rows [cu_seqlens[i], cu_seqlens[i+1]) of q/out;
 * the new tokens' K/V must already be in the pool at positions ctx_i ..
 * ctx_i + len_i - 1 (b200_kv_scatter_rows / b200_qk_norm_rope_kv_write write
 * there).  New token t attends causally to keys 0 .. ctx_i + t, all read from
 * the pool pages block_table[row, p] (the layout of b200_paged_decode:
 * k_pool/v_pool the layer's first element, strides (block, head, slot));
 * decode is the len_i == 1 case.  q (T, H, D), out (T, H, D): strides (token,
 * head).  max_new_tokens >= every len_i.  work_counter as in
 * b200_varlen_prefill.  Bad rows / table entries set dev_status bits.
 */
int b200_paged_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                       const void* k_pool, const void* v_pool,
                       int64_t kv_stride_blk, int64_t kv_stride_h, int64_t kv_stride_slot,
                       const int32_t* block_table, int64_t bt_stride_row,
                       const int32_t* seq_lens, const int32_t* row_ids,
                       const int32_t* cu_seqlens, void* out,
                       int64_t o_stride_t, int64_t o_stride_h,
                       int num_seqs, int total_tokens, int max_new_tokens,
                       int num_heads, int num_kv_heads, int head_dim, int block_size,
                       int num_blocks, int max_pages, int max_requests, float scale,
                       int32_t* work_counter, int32_t* dev_status, void* stream);

/*
 * Fused attention prologue: QK-RMSNorm + RoPE of q and k and the KV-cache
 * write of the roped k and of v, one launch.  Replaces qwen3/attention.py:90-95
 * (q_norm/k_norm, qwen3/norm.py:22-26; apply_rotary_pos_emb, qwen3/rope.py:88-110)
 * plus the KV write that follows (update_kv_batch_triton,
 * qwen3/kernels/paged_attention.py:292-377, or PagedKVCache.update,
 * qwen3/PagedKVcache.py:187-214), with the reference's bf16 rounding steps:
 *     y   = bf16((x * rsqrt(mean(x^2) + eps)) * weight)          (fp32 inside)
 *     out = bf16(bf16(y * bf16(cos)) + bf16(rotate_half(y) * bf16(sin)))
 * q (B, H, S, D), k and v (B, Hkv, S, D) bf16, strides (batch, head, token);
 * q_weight/k_weight (D,) bf16; cos/sin the fp32 rows the reference's
 * RotaryEmbedding gathered for these tokens, (B, S, D) with strides (batch,
 * token).  q_out (B, H, S, D) receives the roped q; k_out (nullable) the roped
 * k.  With k_pool != NULL, token s of request b is written (roped k, and v) at
 * position seq_lens[row_ids[b]] + s of the block table, as b200_kv_scatter_rows
 * does; k_pool == NULL skips the cache write (v may then be NULL).
 * head_dim must be 128.  Bad rows / pages / positions set dev_status bits and
 * skip that token's cache write.
 */
int b200_qk_norm_rope_kv_write(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
    const void* k, int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
    const void* v, int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
    const void* q_weight, const void* k_weight, float eps,
    const float* cos, const float* sin, int64_t cs_stride_b, int64_t cs_stride_s,
    void* q_out, int64_t qo_stride_b, int64_t qo_stride_h, int64_t qo_stride_s,
    void* k_out, int64_t ko_stride_b, int64_t ko_stride_h, int64_t ko_stride_s,
    void* k_pool, void* v_pool,
    int64_t kp_stride_blk, int64_t kp_stride_layer, int64_t kp_stride_h, int64_t kp_stride_slot,
    int64_t vp_stride_blk, int64_t vp_stride_layer, int64_t vp_stride_h, int64_t vp_stride_slot,
    const int32_t* seq_lens, const int32_t* block_table, int64_t bt_stride_row,
    const int32_t* row_ids,
    int batch, int n_tokens, int num_heads, int num_kv_heads, int head_dim, int block_size,
    int num_blocks, int max_pages, int max_requests, int layer,
    int32_t* dev_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QWEN3_B200_ATTN_H */
