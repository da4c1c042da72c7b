// Fused token sampling: top-k selection over the whole vocabulary plus the
// temperature / top-k / top-p / Gumbel-max step, one launch for the batch.
// Replaces the reference's batched torch.topk (qwen3/sampling.py:215-216)
// followed by _sample_topk_kernel (qwen3/sampling.py:112-178), and its greedy
// argmax (:253-254).
//
// Two launches, both graph-capturable:
//   chunk kernel  grid (chunks, rows): a chunk of 8192 logits of one row is
//       held in registers (16 consecutive per thread) as order-preserving
//       32-bit keys of its scores; the k-th largest key is found bit by bit
//       (count of keys at or above a candidate, summed with warp reductions),
//       the k_sel best (ties at the threshold by ascending index) are sorted
//       and written to the workspace.  Score = the logit, except for temperature-only rows
//       (top_k == 0, top_p >= 1: logit / T + Gumbel noise at offset row * V + j;
//       the reference draws these with torch.multinomial, :81-109, another
//       stream); k_sel = 1 for greedy and temperature-only rows, else top_k.
//       For k_sel <= 64 the bit-by-bit search is replaced by a lower bound
//       (the k-th largest of the threads' maxima), a compaction of the few
//       entries at or above it, and a direct ranking of those.
//   row kernel    grid (rows): the same selection over the chunks'
//       candidates, a bitonic sort by (score desc, index asc), and for top-k
//       rows the reference kernel's arithmetic on the sorted candidates
//       (sample_row_fast_kernel when every k of the batch is at most 64:
//       bound, compaction and ranking again, then one warp's scans):
//       x = logit / T, softmax, keep[0] | cumsum(p)[j-1] <= top_p, Gumbel-max
//       with the uniform of Triton's tl.rand(seed, row * block_k + j)
//       (Philox4x32-10, key = seed, counter = (offset, 0, 0, 0), first word to
//       float); greedy and temperature-only rows take the top candidate.
// top_k outside [0, 1024], or top_k == 0 with top_p < 1, is clamped to 1024
// and flagged (B200_DEV_BAD_PARAM).
#include "common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;

constexpr int kChunk = 8192;        // logits per chunk CTA (32 KB of keys in shared memory)
constexpr int kMaxChunks = 32;      // chunks per row (vocab <= 262144)

struct SampleArgs {
  const void* logits;
  int bf16;
  int64_t stride;
  int batch, vocab, block_k, chunks, chunk_len;
  const float* temperature;  // nullable: every row uses temperature_s
  const int32_t* top_k;      // nullable: top_k_s
  const float* top_p;        // nullable: top_p_s
  float temperature_s, top_p_s;
  int top_k_s;
  uint64_t seed;
  uint64_t* cand;   // workspace: [row][chunk][block_k] (key << 32 | ~index)
  int64_t* out;
  int32_t* dev_status;
};

enum RowMode { kGreedy = 0, kTopK = 1, kTempOnly = 2 };

B200_DEVICE float row_temperature(const SampleArgs& a, int row) {
  return a.temperature != nullptr ? a.temperature[row] : a.temperature_s;
}
B200_DEVICE float row_top_p(const SampleArgs& a, int row) {
  return a.top_p != nullptr ? a.top_p[row] : a.top_p_s;
}

// mode and number of candidates to select for row `row` (flags bad params once)
B200_DEVICE int row_mode(const SampleArgs& a, int row, int* k_sel, bool flag) {
  const float temp = row_temperature(a, row);
  int k = a.top_k != nullptr ? a.top_k[row] : a.top_k_s;
  if (!(temp > 0.f)) {
    *k_sel = 1;
    return kGreedy;
  }
  if (k == 0 && row_top_p(a, row) >= 1.f) {
    *k_sel = 1;
    return kTempOnly;
  }
  if (k <= 0 || k > kMaxK) {
    if (flag) b200::flag_error(a.dev_status, B200_DEV_BAD_PARAM);
    k = kMaxK;
  }
  *k_sel = min(k, a.vocab);
  return kTopK;
}

B200_DEVICE float logit_at(const SampleArgs& a, const void* row, int j) {
  return a.bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(row)[j])
                : static_cast<const float*>(row)[j];
}

// order-preserving: a > b as floats <=> key(a) > key(b) as unsigned
B200_DEVICE uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Philox4x32-10 (Salmon et al., SC 2011), first output word.
B200_DEVICE uint32_t philox_word0(uint64_t seed, uint32_t c0, uint32_t c1) {
  uint32_t c2 = 0, c3 = 0;
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    c0 = hi1 ^ c1 ^ k0;
    c2 = hi0 ^ c3 ^ k1;
    c1 = lo1;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

// uniform in [0, 1) exactly as Triton's uint_to_uniform_float on 32 bits
B200_DEVICE float uniform_of(uint32_t w) {
  int32_t x = static_cast<int32_t>(w);
  if (x < 0) x = -x - 1;
  return static_cast<float>(x) * 4.6566127342e-10f;
}

B200_DEVICE float gumbel(uint64_t seed, uint64_t offset) {
  const float u = fmaxf(uniform_of(philox_word0(seed, static_cast<uint32_t>(offset),
                                                static_cast<uint32_t>(offset >> 32))),
                        1.0e-7f);
  return -logf(-logf(u));
}

struct ArgMax {
  float v;
  int i;
};

B200_DEVICE ArgMax better(ArgMax x, ArgMax y) {
  // larger value; ties (and NaN-free equal values) to the smaller index
  if (y.v > x.v || (y.v == x.v && y.i < x.i)) return y;
  return x;
}

// block-wide argmax; every thread gets the result
template <int NT>
B200_DEVICE ArgMax block_argmax(ArgMax m, ArgMax* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax y;
    y.v = __shfl_xor_sync(0xffffffffu, m.v, o);
    y.i = __shfl_xor_sync(0xffffffffu, m.i, o);
    m = better(m, y);
  }
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < NT / 32 ? red[lane] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax y;
      y.v = __shfl_xor_sync(0xffffffffu, m.v, o);
      y.i = __shfl_xor_sync(0xffffffffu, m.i, o);
      m = better(m, y);
    }
    if (lane == 0) red[0] = m;
  }
  __syncthreads();
  const ArgMax r = red[0];
  __syncthreads();
  return r;
}

// ---- selection on keys held in registers: thread t holds positions
// t*PER .. t*PER+PER-1 (key 0 = empty; real keys of finite scores are > 0).

// Sum of v over the block (NT threads), returned to every thread.
template <int NT>
B200_DEVICE int block_sum(int v, int* red) {
  v = __reduce_add_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

// Exclusive prefix sum of v over the threads in order, and the total.
template <int NT>
B200_DEVICE int block_exclusive(int v, int* red, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red[warp] = x;
  __syncthreads();
  int before = 0, t = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) {
    const int r = red[w];
    if (w < warp) before += r;
    t += r;
  }
  __syncthreads();
  *total = t;
  return before + x - v;
}

// Top bits (key >> low) of the k-th largest key: bit-by-bit search for the
// largest T with count(key >= T) >= k.  Bits below `low` are constant across
// keys (bf16 scores: 16), so equal top bits mean equal keys.
template <int NT, int PER>
B200_DEVICE uint32_t kth_key(const uint32_t (&key)[PER], int k, int low, int* red) {
  // red holds 2 x NT/32 partial sums: step i writes half i & 1, so one barrier
  // per step suffices (a thread reads half i & 1 before it reaches the barrier
  // of step i + 1, and half i & 1 is written again only in step i + 2)
  uint32_t sk[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) sk[i] = key[i] >> low;
  const int lane = threadIdx.x & 31;
  uint32_t t = 0;
  int half = 0;
  for (int b = 31 - low; b >= 0; --b) {
    const uint32_t cand = t | (1u << b);
    int c = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) c += sk[i] >= cand ? 1 : 0;
    c = __reduce_add_sync(0xffffffffu, c);
    int* r = red + half * (NT / 32);
    if (lane == 0) r[threadIdx.x >> 5] = c;
    __syncthreads();
    const int total = __reduce_add_sync(0xffffffffu, lane < NT / 32 ? r[lane] : 0);
    if (total >= k) t = cand;
    half ^= 1;
  }
  __syncthreads();  // every partial read before red is reused
  return t;
}

// The k largest entries (ties at the threshold by ascending position) into
// dst[0..k) as (key << 32) | ~ident(position), unordered above the threshold.
template <int NT, int PER, typename Ident>
B200_DEVICE void select_k(const uint32_t (&key)[PER], int k, int low, Ident ident, uint64_t* dst,
                          int* red, int* s_count) {
  const uint32_t T = kth_key<NT, PER>(key, k, low, red);
  int gt = 0, eq = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const uint32_t top = key[i] >> low;
    gt += top > T ? 1 : 0;
    eq += top == T ? 1 : 0;
  }
  const int n_gt = block_sum<NT>(gt, red);
  int eq_total;
  const int eq_rank = block_exclusive<NT>(eq, red, &eq_total);
  if (threadIdx.x == 0) *s_count = 0;
  __syncthreads();
  int r = eq_rank;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const uint32_t top = key[i] >> low;
    const int pos = threadIdx.x * PER + i;
    if (top > T) {
      const int slot = atomicAdd(s_count, 1);
      dst[slot] = (static_cast<uint64_t>(key[i]) << 32) | static_cast<uint32_t>(~ident(pos));
    } else if (top == T) {
      if (r < k - n_gt)
        dst[n_gt + r] = (static_cast<uint64_t>(key[i]) << 32) | static_cast<uint32_t>(~ident(pos));
      ++r;
    }
  }
  __syncthreads();
}

// Bitonic sort of c[0..n) descending (n <= 1024, padded with 0 to a power of 2).
// Up to 64 entries one warp sorts them (warp barriers only).
template <int NT>
B200_DEVICE void sort_desc(uint64_t* c, int n) {
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int i = n + threadIdx.x; i < n2; i += NT) c[i] = 0;
  __syncthreads();
  if (n2 <= 64) {
    if (threadIdx.x < 32) {
      for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int i = threadIdx.x; i < n2; i += 32) {
            const int j = i ^ stride;
            if (j > i) {
              const uint64_t x = c[i], y = c[j];
              const bool desc = (i & size) == 0;
              if (desc ? (x < y) : (x > y)) {
                c[i] = y;
                c[j] = x;
              }
            }
          }
          __syncwarp();
        }
      }
    }
    __syncthreads();
    return;
  }
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n2; i += NT) {
        const int j = i ^ stride;
        if (j > i) {
          const uint64_t x = c[i], y = c[j];
          const bool desc = (i & size) == 0;
          if (desc ? (x < y) : (x > y)) {
            c[i] = y;
            c[j] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Block argmax of (key, position): the largest key, the smallest position on ties.
template <int NT, int PER>
B200_DEVICE uint64_t block_top1(const uint32_t (&key)[PER], uint64_t* red64) {
  uint64_t best = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const uint64_t v = (static_cast<uint64_t>(key[i]) << 32) |
                       static_cast<uint32_t>(~(threadIdx.x * PER + i));
    best = v > best ? v : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t y = __shfl_xor_sync(0xffffffffu, best, o);
    best = y > best ? y : best;
  }
  if ((threadIdx.x & 31) == 0) red64[threadIdx.x >> 5] = best;
  __syncthreads();
  uint64_t r = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) r = red64[w] > r ? red64[w] : r;
  __syncthreads();
  return r;
}

constexpr int kChunkThreads = 512;
constexpr int kChunkPer = kChunk / kChunkThreads;  // 16 logits per thread
// Rows selecting at most kFastK per chunk first bound the k-th largest key
// from below by the k-th largest of the threads' maxima (k distinct entries
// reach it), keep only the entries at or above that bound (the k best are
// among them; for k <= kFastK at most kFastK * kChunkPer = kMaxK unless the
// bound is tied) and rank those few directly: a handful of barriers instead
// of one per key bit.
constexpr int kFastK = kMaxK / kChunkPer;          // 64

// k-th largest of the block's per-thread values v (top bits only: values
// >> low), by one warp's bit-by-bit search over the kChunkThreads values in
// shared memory; warp reductions only.
B200_DEVICE uint32_t warp_kth_of(const uint32_t* v, int k, int low) {
  constexpr int kPerLane = kChunkThreads / 32;
  const int lane = threadIdx.x & 31;
  uint32_t x[kPerLane];
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) x[i] = v[lane * kPerLane + i];
  uint32_t t = 0;
  for (int b = 31 - low; b >= 0; --b) {
    const uint32_t cand = t | (1u << b);
    int c = 0;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) c += x[i] >= cand ? 1 : 0;
    if (__reduce_add_sync(0xffffffffu, c) >= k) t = cand;
  }
  return t;
}

// One chunk of one row: its k_sel best scores into the workspace.  Three CTAs
// per SM (40 registers; the few spills sit off the common path) keep more
// chunks in flight than two at 64 registers: 35 -> 33 us for top-k 50,
// 100 -> 94 us for top-k 200 on 64 x 151936 logits.
__global__ void __launch_bounds__(kChunkThreads, 3) sample_chunk_kernel(const SampleArgs a) {
  __shared__ __align__(16) uint64_t c[kMaxK];
  __shared__ uint64_t red64[kChunkThreads / 32];
  __shared__ int red[2 * kChunkThreads / 32];
  __shared__ int s_count;
  const int chunk = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
  int k_sel;
  const int mode = row_mode(a, row, &k_sel, chunk == 0 && tid == 0);
  const int j0 = chunk * a.chunk_len;
  const int n = min(a.chunk_len, a.vocab - j0);
  uint64_t* dst = a.cand + (static_cast<int64_t>(row) * a.chunks + chunk) * a.block_k;
  if (n <= 0) return;
  const float temp = row_temperature(a, row);

  // 16 consecutive logits per thread (vector loads when the row allows)
  float x[kChunkPer];
  const int first = tid * kChunkPer;
  if (a.bf16) {
    const __nv_bfloat16* lg = static_cast<const __nv_bfloat16*>(a.logits) + row * a.stride + j0;
    if ((a.stride & 7) == 0 && (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0 &&
        first + kChunkPer <= n) {
#pragma unroll
      for (int v = 0; v < kChunkPer / 8; ++v) {
        const uint4 u = *reinterpret_cast<const uint4*>(lg + first + 8 * v);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          x[8 * v + 2 * e] = b200::bf16_lo(w[e]);
          x[8 * v + 2 * e + 1] = b200::bf16_hi(w[e]);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < kChunkPer; ++i)
        x[i] = first + i < n ? __bfloat162float(lg[first + i]) : 0.f;
    }
  } else {
    const float* lg = static_cast<const float*>(a.logits) + row * a.stride + j0;
    if ((a.stride & 3) == 0 && (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0 &&
        first + kChunkPer <= n) {
#pragma unroll
      for (int v = 0; v < kChunkPer / 4; ++v) {
        const float4 u = *reinterpret_cast<const float4*>(lg + first + 4 * v);
        x[4 * v] = u.x;
        x[4 * v + 1] = u.y;
        x[4 * v + 2] = u.z;
        x[4 * v + 3] = u.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < kChunkPer; ++i) x[i] = first + i < n ? lg[first + i] : 0.f;
    }
  }
  uint32_t key[kChunkPer];
#pragma unroll
  for (int i = 0; i < kChunkPer; ++i) {
    float sc = x[i];
    if (mode == kTempOnly)
      sc = sc / temp +
           gumbel(a.seed, static_cast<uint64_t>(row) * a.vocab + static_cast<uint64_t>(j0 + first + i));
    key[i] = first + i < n ? order_key(sc) : 0u;
  }
  auto ident = [&](int pos) { return j0 + pos; };
  if (k_sel == 1) {
    const uint64_t b = block_top1<kChunkThreads, kChunkPer>(key, red64);
    if (tid == 0)
      dst[0] = (b & 0xFFFFFFFF00000000ull) |
               static_cast<uint32_t>(~ident(static_cast<int>(~static_cast<uint32_t>(b))));
    return;
  }
  const int k = min(k_sel, n);
  // bf16 scores leave the low 16 key bits constant (greedy / top-k rows)
  const int low = (a.bf16 && mode != kTempOnly) ? 16 : 0;
  if (k <= kFastK) {
    __shared__ uint32_t tmax[kChunkThreads];
    __shared__ uint32_t s_bound;
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < kChunkPer; ++i) m = max(m, key[i] >> low);
    tmax[tid] = m;
    if (tid == 0) s_count = 0;
    __syncthreads();
    if (tid < 32) {
      const uint32_t t0 = warp_kth_of(tmax, k, low);
      if (tid == 0) s_bound = t0;
    }
    __syncthreads();
    const uint32_t bound = s_bound;
    // entries at or above the bound (real keys only) into c[], one atomic per warp
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < kChunkPer; ++i) cnt += (key[i] != 0u && (key[i] >> low) >= bound) ? 1 : 0;
    const int lane = tid & 31;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int base = 0;
    if (lane == 31) base = atomicAdd(&s_count, incl);
    int pos = __shfl_sync(0xffffffffu, base, 31) + incl - cnt;
#pragma unroll
    for (int i = 0; i < kChunkPer; ++i) {
      if (key[i] != 0u && (key[i] >> low) >= bound) {
        if (pos < kMaxK)
          c[pos] = (static_cast<uint64_t>(key[i]) << 32) |
                   static_cast<uint32_t>(~ident(tid * kChunkPer + i));
        ++pos;
      }
    }
    __syncthreads();
    const int cn = s_count;
    if (cn <= kMaxK) {
      // rank of each entry among all of them, by (key desc, index asc): the
      // k best land sorted in dst[0..k)
      for (int i = tid; i < cn; i += kChunkThreads) {
        const uint64_t v = c[i];
        int r = 0;
        for (int j2 = 0; j2 < cn; ++j2) r += c[j2] > v ? 1 : 0;
        if (r < k) dst[r] = v;
      }
      // slots past the ranked entries hold no candidate (key 0)
      for (int i = min(cn, k) + tid; i < k_sel; i += kChunkThreads) dst[i] = 0;
      return;
    }
    // a bound tied across many threads: the general search below, once every
    // thread has read the count (the search resets it)
    __syncthreads();
  }
  select_k<kChunkThreads, kChunkPer>(key, k, low, ident, c, red, &s_count);
  // sorted by (score desc, index asc): the row kernel then meets equal scores
  // in ascending vocabulary order (chunks in order, each chunk sorted)
  sort_desc<kChunkThreads>(c, k);
  // rows whose k exceeds this chunk: the unused slots hold no candidate (key 0)
  for (int i = tid; i < k_sel; i += kChunkThreads) dst[i] = i < k ? c[i] : 0;
}

// One row: merge the chunks' candidates, sort the k best, sample.  kRowPer
// candidates per thread: the host picks the smallest power of two with
// kThreads * kRowPer >= chunks * block_k.
template <int kRowPer>
__global__ void __launch_bounds__(kThreads) sample_row_kernel(const SampleArgs a) {
  __shared__ __align__(16) uint64_t cand[kMaxK];   // (key << 32) | (~index): sorted descending
  __shared__ float prob[kMaxK];
  __shared__ uint64_t red64[kThreads / 32];
  __shared__ int red[2 * kThreads / 32];
  __shared__ ArgMax redm[32];
  __shared__ int s_count;
  const int row = blockIdx.x, tid = threadIdx.x;
  int k;
  const int mode = row_mode(a, row, &k, false);
  const uint64_t* src = a.cand + static_cast<int64_t>(row) * a.chunks * a.block_k;
  // candidate c = (chunk c / k, slot c % k): chunk-major, each chunk sorted
  const int n = a.chunks * k;
  auto ent = [&](int c) { return src[(c / k) * a.block_k + (c % k)]; };
  uint32_t key[kRowPer];
#pragma unroll
  for (int i = 0; i < kRowPer; ++i) {
    const int c = tid * kRowPer + i;
    key[i] = c < n ? static_cast<uint32_t>(ent(c) >> 32) : 0u;
  }
  if (k == 1) {
    const uint64_t b = block_top1<kThreads, kRowPer>(key, red64);
    if (tid == 0)
      a.out[row] = static_cast<int>(~static_cast<uint32_t>(ent(static_cast<int>(~static_cast<uint32_t>(b)))));
    return;
  }
  auto ident = [&](int c) { return static_cast<int>(~static_cast<uint32_t>(ent(c))); };
  const int low = a.bf16 ? 16 : 0;
  select_k<kThreads, kRowPer>(key, k, low, ident, cand, red, &s_count);
  sort_desc<kThreads>(cand, k);

  // ---- the reference kernel's step on the sorted candidates (thread j = rank j)
  const void* lg = a.bf16 ? static_cast<const void*>(static_cast<const __nv_bfloat16*>(a.logits) +
                                                     row * a.stride)
                          : static_cast<const void*>(static_cast<const float*>(a.logits) +
                                                     row * a.stride);
  const float temp = row_temperature(a, row);
  const float top_p = row_top_p(a, row);
  const int j = tid;
  const bool valid = j < k;
  const int idx = valid ? static_cast<int>(~static_cast<uint32_t>(cand[j])) : 0;
  const float x = valid ? logit_at(a, lg, idx) / temp : -INFINITY;
  const float m0 = logit_at(a, lg, static_cast<int>(~static_cast<uint32_t>(cand[0]))) / temp;
  const float e = valid ? expf(x - m0) : 0.f;
  // returns this thread's inclusive prefix sum; *last gets the total
  auto inclusive_scan = [&](float v, float* last) {
    prob[j] = v;
    __syncthreads();
    for (int o = 1; o < kThreads; o <<= 1) {
      const float add = j >= o ? prob[j - o] : 0.f;
      __syncthreads();
      prob[j] += add;
      __syncthreads();
    }
    const float r = prob[j];
    *last = prob[kThreads - 1];
    __syncthreads();
    return r;
  };
  float total, unused;
  inclusive_scan(e, &total);
  const float p = e / total;
  const float c = inclusive_scan(p, &unused);
  const bool keep = valid && (j == 0 || c - p <= top_p);
  const float score =
      keep ? x + gumbel(a.seed, static_cast<uint64_t>(row) * a.block_k + j) : -INFINITY;
  const ArgMax best = block_argmax<kThreads>(ArgMax{score, j}, redm);
  if (tid == 0) a.out[row] = static_cast<int>(~static_cast<uint32_t>(cand[best.i]));
  (void)mode;
}

// One row per CTA, for batches whose every k is at most kFastK: the same
// selection and arithmetic as sample_row_kernel with a handful of barriers.
// The chunks' lists are sorted, so the k-th largest of their first
// ceil(k / chunks) entries bounds the row's k-th largest candidate from below
// (k sampled entries reach it); the candidates at or above the bound are
// ranked directly in the total order (key desc, index asc), which puts the k
// best sorted in place; one warp then takes the reference kernel's step.
constexpr int kRowFastThreads = 256;
constexpr int kRowFastMax = kMaxChunks * kFastK;  // every candidate of a row

__global__ void __launch_bounds__(kRowFastThreads) sample_row_fast_kernel(const SampleArgs a) {
  __shared__ __align__(16) uint64_t sel[kRowFastMax];
  __shared__ __align__(16) uint64_t samp[kFastK + kMaxChunks];
  __shared__ __align__(16) uint64_t cand[kFastK];
  __shared__ uint64_t s_bound;
  __shared__ int s_count;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  int k;
  row_mode(a, row, &k, false);
  k = min(k, a.block_k);
  const uint64_t* src = a.cand + static_cast<int64_t>(row) * a.chunks * a.block_k;
  const int n = a.chunks * k;
  auto ent = [&](int c) { return src[(c / k) * a.block_k + (c % k)]; };
  if (k == 1) {
    if (tid < 32) {
      uint64_t best = 0;
      for (int c = lane; c < n; c += 32) {
        const uint64_t v = ent(c);
        best = v > best ? v : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const uint64_t y = __shfl_xor_sync(0xffffffffu, best, o);
        best = y > best ? y : best;
      }
      if (lane == 0) a.out[row] = static_cast<int>(~static_cast<uint32_t>(best));
    }
    return;
  }
  // the bound: the k-th largest of the first r entries of every chunk
  const int r = (k + a.chunks - 1) / a.chunks;
  const int ns = a.chunks * r;
  if (tid < ns) samp[tid] = src[(tid / r) * a.block_k + (tid % r)];
  if (tid == 0) {
    s_count = 0;
    // a chunk shorter than r leaves empty slots (0) among the samples; if the
    // k-th largest sample is one of those, no sample has rank k - 1 (the
    // empty slots tie) and the bound stays 0: every candidate is taken
    s_bound = 0;
  }
  __syncthreads();
  if (tid < ns) {
    const uint64_t v = samp[tid];
    int rk = 0;
    for (int j = 0; j < ns; ++j) rk += samp[j] > v ? 1 : 0;
    if (rk == k - 1 && v != 0) s_bound = v;
  }
  __syncthreads();
  const uint64_t bound = s_bound;
  // every candidate at or above the bound, one shared atomic per warp and pass
  for (int c0 = 0; c0 < n; c0 += kRowFastThreads) {
    const int c = c0 + tid;
    const uint64_t v = c < n ? ent(c) : 0;
    const bool take = c < n && v >= bound;
    const uint32_t bal = __ballot_sync(0xffffffffu, take);
    int base = 0;
    if (lane == 0 && bal != 0u) base = atomicAdd(&s_count, __popc(bal));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (take) sel[base + __popc(bal & ((1u << lane) - 1u))] = v;
  }
  __syncthreads();
  const int cn = s_count;
  for (int i = tid; i < cn; i += kRowFastThreads) {
    const uint64_t v = sel[i];
    int rk = 0;
    for (int j = 0; j < cn; ++j) rk += sel[j] > v ? 1 : 0;
    if (rk < k) cand[rk] = v;
  }
  __syncthreads();
  if (tid >= 32) return;

  // ---- the reference kernel's step on the sorted candidates (ranks lane, lane + 32)
  const void* lg = a.bf16 ? static_cast<const void*>(static_cast<const __nv_bfloat16*>(a.logits) +
                                                     row * a.stride)
                          : static_cast<const void*>(static_cast<const float*>(a.logits) +
                                                     row * a.stride);
  const float temp = row_temperature(a, row);
  const float top_p = row_top_p(a, row);
  float x[2], e[2];
  int idx[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int j = lane + 32 * h;
    idx[h] = j < k ? static_cast<int>(~static_cast<uint32_t>(cand[j])) : 0;
    x[h] = j < k ? logit_at(a, lg, idx[h]) / temp : -INFINITY;
  }
  const float m0 = __shfl_sync(0xffffffffu, x[0], 0);
#pragma unroll
  for (int h = 0; h < 2; ++h) e[h] = lane + 32 * h < k ? expf(x[h] - m0) : 0.f;
  // inclusive scan over the ranks (lane order, then the second half)
  auto scan2 = [&](const float (&v)[2], float (&out)[2]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float sum = v[h];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, sum, o);
        if (lane >= o) sum += y;
      }
      out[h] = sum;
    }
    out[1] += __shfl_sync(0xffffffffu, out[0], 31);
  };
  float ce[2];
  scan2(e, ce);
  const float total = __shfl_sync(0xffffffffu, ce[1], 31);
  float p[2], cp[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) p[h] = e[h] / total;
  scan2(p, cp);
  ArgMax best{-INFINITY, 0x7fffffff};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int j = lane + 32 * h;
    const bool keep = j < k && (j == 0 || cp[h] - p[h] <= top_p);
    const float score =
        keep ? x[h] + gumbel(a.seed, static_cast<uint64_t>(row) * a.block_k + j) : -INFINITY;
    best = better(best, ArgMax{score, j});
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax y;
    y.v = __shfl_xor_sync(0xffffffffu, best.v, o);
    y.i = __shfl_xor_sync(0xffffffffu, best.i, o);
    best = better(best, y);
  }
  const int bidx = __shfl_sync(0xffffffffu, best.i < 32 ? idx[0] : idx[1], best.i & 31);
  if (lane == 0) a.out[row] = bidx;
}

int chunks_for(int vocab) { return (vocab + kChunk - 1) / kChunk; }

}  // namespace

extern "C" size_t b200_sample_workspace_size(int batch, int vocab, int block_k) {
  if (batch <= 0 || vocab <= 0 || block_k <= 0) return 0;
  return static_cast<size_t>(batch) * chunks_for(vocab) * block_k * sizeof(uint64_t);
}

extern "C" int b200_sample_tokens(const void* logits, int logits_bf16, int64_t stride_row,
                                  int batch, int vocab, const float* temperature,
                                  const int32_t* top_k, const float* top_p,
                                  float temperature_all, int top_k_all, float top_p_all,
                                  uint64_t seed, int block_k, void* workspace,
                                  size_t workspace_bytes, int64_t* out, int32_t* dev_status,
                                  void* stream) {
  if (batch < 0 || vocab <= 0 || stride_row < vocab || block_k <= 0 || block_k > kMaxK)
    return B200_ERR_INVALID_ARGUMENT;
  if (batch == 0) return B200_OK;
  if (!logits || !out) return B200_ERR_INVALID_ARGUMENT;
  if (batch > 65535) return B200_ERR_INVALID_ARGUMENT;
  const int chunks = chunks_for(vocab);
  if (chunks > kMaxChunks) return B200_ERR_UNSUPPORTED;
  const size_t need = b200_sample_workspace_size(batch, vocab, block_k);
  if (workspace == nullptr || workspace_bytes < need || !b200host::aligned16(workspace))
    return B200_ERR_WORKSPACE;
  SampleArgs a;
  a.logits = logits;
  a.bf16 = logits_bf16 != 0;
  a.stride = stride_row;
  a.batch = batch;
  a.vocab = vocab;
  a.block_k = block_k;
  a.chunks = chunks;
  a.chunk_len = kChunk;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.temperature_s = temperature_all;
  a.top_k_s = top_k_all;
  a.top_p_s = top_p_all;
  a.seed = seed;
  a.cand = static_cast<uint64_t*>(workspace);
  a.out = out;
  a.dev_status = dev_status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  sample_chunk_kernel<<<dim3(chunks, batch), kChunkThreads, 0, s>>>(a);
  const int cand_per_row = chunks * block_k;
  if (block_k <= kFastK) {
    sample_row_fast_kernel<<<batch, kRowFastThreads, 0, s>>>(a);
  } else if (cand_per_row <= kThreads) {
    sample_row_kernel<1><<<batch, kThreads, 0, s>>>(a);
  } else if (cand_per_row <= 2 * kThreads) {
    sample_row_kernel<2><<<batch, kThreads, 0, s>>>(a);
  } else if (cand_per_row <= 4 * kThreads) {
    sample_row_kernel<4><<<batch, kThreads, 0, s>>>(a);
  } else if (cand_per_row <= 8 * kThreads) {
    sample_row_kernel<8><<<batch, kThreads, 0, s>>>(a);
  } else if (cand_per_row <= 16 * kThreads) {
    sample_row_kernel<16><<<batch, kThreads, 0, s>>>(a);
  } else {
    sample_row_kernel<32><<<batch, kThreads, 0, s>>>(a);
  }
  return b200host::status_from_cuda(cudaGetLastError());
}
