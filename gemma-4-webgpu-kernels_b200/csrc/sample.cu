// sample.cu — token sampling on the device: the reference's sampler
// (rust/src/sampler.rs:116-190) over logits that stay in HBM, so a decode step
// reads back one token id per sequence instead of a 1 MB logits row.
//
// Semantics follow sample():
//  * repetition penalty (sampler.rs:120-133): each distinct recent token < vocab,
//    x > 0 ? x / p : x * p, on a copy (the caller's logits are not modified);
//  * temperature <= 0: greedy, the first index of the largest value (NaN never wins);
//  * top_k = 0 and top_p >= 1: sample_all (sampler.rs:58-69) over the whole row:
//    r = u * sum(exp((l - max) / T)), the first index where the running r - exp(..)
//    reaches <= 0;
//  * otherwise the candidate path: the top_k largest (sorted by value, ties to the
//    smaller index), softmax_over them, the top-p cut (cum >= top_p keeps the
//    candidate that reaches it), softmax_over the kept ones, and the draw.
//    top_k = 0 with top_p < 1 (a nucleus over the whole sorted row) uses the
//    kSampleCap largest as candidates with the whole row's softmax denominator;
//    when they hold less than top_p of the mass the row's token is -1 and
//    GQ_DEVERR_SAMPLE_CAP is raised (the nucleus is larger than the device path
//    handles; the caller samples that row on the host).
//  * draws: one u = Rng::next_f64 per sampled (non-greedy) row from a per-row
//    splitmix64 state in device memory, advanced in place (sampler.rs:5-27), so a
//    seed gives the reference's stream and a step replays from a CUDA graph.
// Arithmetic: the candidate path runs the reference's sequential f32 softmax,
// cumulative sum and draw over the sorted candidates in one thread, in the same
// order; sums over the whole row (sample_all, the top-p-only denominator) are
// chunked reductions, so a draw that lands within rounding of a boundary between
// two tokens can pick the neighbour.
//
// Kernels: topk_chunk_kernel (one CTA per 4096-column chunk of a row: penalty,
// 64-bit keys (order-preserving value bits above the complemented column), the
// chunk's top K by a four-pass radix select of the K-th largest key, and its max;
// a full bitonic sort of the chunk measured 90 us for one row and 924 us for 64),
// chunk_expsum_kernel
// (per-chunk sum of exp((l - max) / T), only for the whole-row modes) and
// sample_row_kernel (one CTA per row: merge of the chunks' candidates by a second
// bitonic sort, then the reference's sequential candidate arithmetic, or the
// sample_all scan).
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "gq_internal.cuh"

namespace {

constexpr int kChunk = 4096;        // columns per chunk CTA
constexpr int kChunkThreads = 256;
constexpr int kRowThreads = 1024;
constexpr int kSampleCap = 256;     // largest candidate count (top_k, or the top-p-only cap)
constexpr int kMaxRecent = 4096;

// Order-preserving 32-bit key of a logit: NaN lowest (1), -0 as +0; 0 is padding.
__device__ __forceinline__ uint32_t vkey(float v) {
  if (v != v) return 1u;
  if (v == 0.0f) v = 0.0f;
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float vkey_value(uint32_t k) {
  if (k <= 1u) return __uint_as_float(0x7fc00000u);  // NaN (padding never reaches the arithmetic)
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// 64-bit candidate key: value key above the complemented column (ties: smaller column first)
__device__ __forceinline__ uint64_t ckey(float v, uint32_t col) {
  return ((uint64_t)vkey(v) << 32) | (uint64_t)(0xffffffffu - col);
}
__device__ __forceinline__ uint32_t ckey_col(uint64_t k) { return 0xffffffffu - (uint32_t)k; }

__device__ __forceinline__ float penalize(float x, float p) { return x > 0.0f ? __fdiv_rn(x, p) : __fmul_rn(x, p); }

// Descending bitonic sort of n (a power of two) keys in shared memory, all threads.
__device__ void bitonic_desc(uint64_t *k, int n) {
  for (int size = 2; size <= n; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = k[lo], b = k[hi];
        if ((a < b) == desc) {
          k[lo] = b;
          k[hi] = a;
        }
      }
    }
  __syncthreads();
}

// The k largest of n distinct-or-zero 64-bit keys in shared memory, all threads:
// radix select over eight 8-bit digits from the top (a histogram of the keys
// still matching the selected prefix, counts aggregated per warp with
// match.any, the bin holding the k-th largest found from the top by one warp's
// scan; once that bin holds at most kSurv keys they are compacted and the later
// passes scan only them), then every key above the k-th and enough copies of it
// go to out[0..k) unsorted. Zero keys (padding) are the only repeats and rank last.
constexpr int kSurv = 1024;  // select_top: keys still tied on the selected prefix, compacted

__device__ void select_top(const uint64_t *all_keys, int all_n, int k, uint64_t *out) {
  __shared__ uint32_t hist[2][256];  // double-buffered: pass p counts into hist[p & 1]
  __shared__ uint64_t surv[kSurv];
  __shared__ unsigned long long s_prefix;
  __shared__ uint32_t s_need, s_count, s_ties, s_bin_count, s_nsurv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint64_t prefix = 0ull, mask = 0ull;
  uint32_t need = (uint32_t)k;
  // the passes scan `keys`: all keys until the keys matching the selected prefix
  // fit the survivor buffer, then only those (the final gather scans all keys)
  const uint64_t *keys = all_keys;
  int n = all_n;
  bool compacted = false;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[0][i] = 0u;
  __syncthreads();
  for (int shift = 56, p = 0; shift >= 0; shift -= 8, ++p) {
    uint32_t *h = hist[p & 1];
    for (int base = warp * 32; base < n; base += nw * 32) {
      const int i = base + lane;
      const uint64_t kk = i < n ? keys[i] : 0ull;
      const bool live = i < n && (kk & mask) == prefix;
      const uint32_t bin = live ? (uint32_t)(kk >> shift) & 255u : 256u;
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (live && lane == __ffs(peers) - 1) atomicAdd(&h[bin], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l; counts from the top; the other
      // histogram is cleared for the next pass meanwhile
      uint32_t cnt[8], tot = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        cnt[q] = h[255 - 8 * lane - q];
        tot += cnt[q];
        hist[(p + 1) & 1][8 * lane + q] = 0u;
      }
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const uint32_t excl = incl - tot;
      if (excl < need && incl >= need) {
        uint32_t acc = excl;
        int q = 0;
        for (; q < 8; ++q) {
          if (acc + cnt[q] >= need) break;
          acc += cnt[q];
        }
        s_prefix = prefix | ((unsigned long long)(255u - 8u * lane - (uint32_t)q) << shift);
        s_need = need - acc;
        s_bin_count = cnt[q];
      }
      if (lane == 0) {
        s_nsurv = 0u;
        if (shift == 0) {
          s_count = 0u;
          s_ties = 0u;
        }
      }
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
    mask |= 255ull << shift;
    if (!compacted && shift > 0 && s_bin_count <= (uint32_t)kSurv) {  // uniform: read after the barrier
      for (int base = warp * 32; base < n; base += nw * 32) {
        const int i = base + lane;
        if (i < n && (keys[i] & mask) == prefix) surv[atomicAdd(&s_nsurv, 1u)] = keys[i];
      }
      __syncthreads();
      keys = surv;
      n = (int)s_nsurv;
      compacted = true;
    }
  }
  for (int i = threadIdx.x; i < all_n; i += blockDim.x) {
    const uint64_t kk = all_keys[i];
    bool take = kk > prefix;
    if (kk == prefix) take = atomicAdd(&s_ties, 1u) < need;
    if (take) {
      const uint32_t slot = atomicAdd(&s_count, 1u);
      if (slot < (uint32_t)k) out[slot] = kk;
    }
  }
  __syncthreads();
}

struct SampleArgs {
  const float *logits;
  int64_t m, n, ld;       // rows, columns, row stride (floats)
  int64_t idx_base;       // global id of column 0 (a vocab shard's first row)
  int k;                  // candidates kept per chunk / row (1 .. kSampleCap)
  int nchunks;
  float penalty;          // 1 = off
  const uint32_t *recent; // [m][recent_stride], ids >= idx_base + n ignored
  int64_t n_recent, recent_stride;
  uint64_t *ckeys;        // [m][nchunks][k] chunk candidates
  float *cmax;            // [m][nchunks] chunk max (NaN ignored)
  float *csum;            // [m][nchunks] chunk sum of exp((l - max) / T)
  float inv_t;
};

__device__ __forceinline__ float logit_at(const SampleArgs &a, int64_t row, int64_t col, const uint8_t *pen) {
  const float v = __ldg(a.logits + row * a.ld + col);
  return pen && pen[col & (kChunk - 1)] ? penalize(v, a.penalty) : v;
}

// Marks (in a per-chunk byte map) the recent tokens that fall in this chunk; each
// distinct token is marked once however often it repeats.
__device__ void mark_recent(const SampleArgs &a, int64_t row, int64_t c0, int64_t c1, uint8_t *pen) {
  for (int i = threadIdx.x; i < kChunk; i += blockDim.x) pen[i] = 0;
  __syncthreads();
  const uint32_t *rec = a.recent + row * a.recent_stride;
  for (int64_t j = threadIdx.x; j < a.n_recent; j += blockDim.x) {
    const int64_t col = (int64_t)__ldg(rec + j) - a.idx_base;
    if (col >= c0 && col < c1) pen[col - c0] = 1;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kChunkThreads) topk_chunk_kernel(const SampleArgs a) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  __shared__ uint64_t keys[kChunk];
  __shared__ uint8_t pen_s[kChunk];
  __shared__ float red[kChunkThreads / 32];
  const int64_t row = blockIdx.y;
  const int chunk = blockIdx.x;
  const int64_t c0 = (int64_t)chunk * kChunk, c1 = min(a.n, c0 + kChunk);
  const bool use_pen = a.penalty != 1.0f && a.n_recent > 0;
  if (use_pen) mark_recent(a, row, c0, c1, pen_s);
  const uint8_t *pen = use_pen ? pen_s : nullptr;
  float mx = -INFINITY;
  if (a.k == 1) {  // greedy: the chunk's best key by reduction
    uint64_t best = 0;
    for (int64_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
      const float v = logit_at(a, row, c, pen);
      mx = fmaxf(mx, v);
      const uint64_t kk = ckey(v, (uint32_t)(a.idx_base + c));
      best = kk > best ? kk : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t ob = __shfl_xor_sync(0xffffffffu, best, o);
      best = ob > best ? ob : best;
    }
    if ((threadIdx.x & 31) == 0) keys[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint64_t b = 0;
      for (int w = 0; w < kChunkThreads / 32; ++w) b = keys[w] > b ? keys[w] : b;
      a.ckeys[(row * a.nchunks + chunk)] = b;
    }
  } else {
    // The chunk's k largest keys by radix select: four 8-bit passes over the value
    // keys (histogram of the keys still matching the selected prefix, then the bin
    // holding the k-th largest from the top) give the k-th largest value key T; the
    // keys above T are taken, and of those equal to T the ones in the smallest
    // columns (a block scan in column order). The k candidates go out unsorted (the
    // row kernel sorts every chunk's candidates together). Thread t holds columns
    // c0 + 16t .. c0 + 16t + 15; columns past the row's end are padding (key 0).
    constexpr int PT = kChunk / kChunkThreads;  // 16 keys per thread
    uint32_t* hist = reinterpret_cast<uint32_t *>(keys);            // [256] (keys[] is free here)
    __shared__ uint32_t sel_prefix, sel_need, out_count, warp_ties[kChunkThreads / 32];
    uint32_t kv[PT];
#pragma unroll
    for (int j = 0; j < PT; ++j) {
      const int64_t c = c0 + (int64_t)threadIdx.x * PT + j;
      kv[j] = 0u;
      if (c < c1) {
        const float v = logit_at(a, row, c, pen);
        mx = fmaxf(mx, v);
        kv[j] = vkey(v);
      }
    }
    uint32_t prefix = 0u, mask = 0u, need = (uint32_t)a.k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
      __syncthreads();
#pragma unroll
      for (int j = 0; j < PT; ++j)
        if ((kv[j] & mask) == prefix) atomicAdd(&hist[(kv[j] >> shift) & 255u], 1u);
      __syncthreads();
      if (threadIdx.x < 32) {
        // lane l owns bins 255-8l .. 248-8l; counts from the top
        const int lane = threadIdx.x;
        uint32_t cnt[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          cnt[q] = hist[255 - 8 * lane - q];
          tot += cnt[q];
        }
        uint32_t incl = tot;  // inclusive prefix over lanes 0..l (higher bins first)
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const uint32_t excl = incl - tot;
        if (excl < need && incl >= need) {  // the bin of the need-th largest is in this lane
          uint32_t acc = excl;
          int q = 0;
          for (; q < 8; ++q) {
            if (acc + cnt[q] >= need) break;
            acc += cnt[q];
          }
          const uint32_t bin = 255u - 8u * lane - (uint32_t)q;
          sel_prefix = prefix | (bin << shift);
          sel_need = need - acc;
        }
      }
      __syncthreads();
      prefix = sel_prefix;
      need = sel_need;
      mask |= 255u << shift;
      __syncthreads();
    }
    // T = prefix: keys > T are taken; of the keys == T, the first `need` in column order
    uint32_t ties = 0;
#pragma unroll
    for (int j = 0; j < PT; ++j) ties += kv[j] == prefix;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = ties;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_ties[warp] = incl;
    if (threadIdx.x == 0) out_count = 0u;
    __syncthreads();
    uint32_t before = incl - ties;
    for (int w = 0; w < warp; ++w) before += warp_ties[w];
    uint64_t *out = a.ckeys + (row * a.nchunks + chunk) * a.k;
#pragma unroll
    for (int j = 0; j < PT; ++j) {
      bool take = kv[j] > prefix;
      if (kv[j] == prefix) {
        take = before < need;
        ++before;
      }
      if (take) {
        const uint32_t slot = atomicAdd(&out_count, 1u);
        if (slot < (uint32_t)a.k) {
          const uint32_t col = (uint32_t)(a.idx_base + c0 + (int64_t)threadIdx.x * PT + j);
          out[slot] = kv[j] ? (((uint64_t)kv[j] << 32) | (uint64_t)(0xffffffffu - col)) : 0ull;
        }
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m2 = -INFINITY;
    for (int w = 0; w < kChunkThreads / 32; ++w) m2 = fmaxf(m2, red[w]);
    a.cmax[row * a.nchunks + chunk] = m2;
  }
}

// Per-chunk sum of exp((l - rowmax) * inv_t) (penalised values), for the modes that
// need the whole row's softmax denominator.
__global__ void __launch_bounds__(kChunkThreads) chunk_expsum_kernel(const SampleArgs a) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  __shared__ uint8_t pen_s[kChunk];
  __shared__ float red[kChunkThreads / 32];
  const int64_t row = blockIdx.y;
  const int chunk = blockIdx.x;
  const int64_t c0 = (int64_t)chunk * kChunk, c1 = min(a.n, c0 + kChunk);
  const bool use_pen = a.penalty != 1.0f && a.n_recent > 0;
  if (use_pen) mark_recent(a, row, c0, c1, pen_s);
  const uint8_t *pen = use_pen ? pen_s : nullptr;
  float rmax = -INFINITY;
  for (int c = 0; c < a.nchunks; ++c) rmax = fmaxf(rmax, a.cmax[row * a.nchunks + c]);
  float s = 0.0f;
  for (int64_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) s += expf(__fmul_rn(logit_at(a, row, c, pen) - rmax, a.inv_t));
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < kChunkThreads / 32; ++w) t += red[w];
    a.csum[row * a.nchunks + chunk] = t;
  }
}

__device__ __forceinline__ double rng_next_f64(uint64_t *state) {
  uint64_t z = (*state += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  z ^= z >> 31;
  return (double)(z >> 11) / (double)(1ull << 53);
}

struct RowArgs {
  SampleArgs s;
  int mode;           // 0 greedy, 1 candidates (top-k and/or top-p), 2 sample_all
  int top_k;          // candidates taken from the merged list (mode 1)
  float top_p;
  int whole_denominator;  // mode 1 with top_k = 0: probabilities over the whole row
  uint64_t *rng;      // [m] splitmix64 states
  int32_t *tokens;    // [m]
  float *cand_val;    // optional [m][top_k] merged candidates (values), for the sharded exchange
  int64_t *cand_idx;  // optional [m][top_k] (global ids)
  uint32_t *err;
};

// One CTA per row: merge the chunks' candidate lists, then sample. Shared memory:
// the merge buffer (a power of two of keys) and one chunk's penalty map.
__global__ void __launch_bounds__(kRowThreads) sample_row_kernel(const RowArgs a) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float scan_r;
  __shared__ int scan_chunk;
  const SampleArgs &s = a.s;
  const int64_t row = blockIdx.x;
  const int total = s.nchunks * s.k;
  int n2 = 1;
  while (n2 < total) n2 <<= 1;
  uint64_t *keys = reinterpret_cast<uint64_t *>(smem);
  uint8_t *pen = smem + (size_t)n2 * 8;
  uint64_t *sel = reinterpret_cast<uint64_t *>(pen + kChunk);  // [kSampleCap]
  for (int i = threadIdx.x; i < n2; i += blockDim.x) keys[i] = i < total ? s.ckeys[row * total + i] : 0ull;
  // candidates in descending order: sort them all when few, else select the
  // top_k first and sort only those
  const int want = (a.mode == 1 || (a.cand_val && a.cand_idx)) ? a.top_k : 1;
  if (want >= 1 && want <= kSampleCap && total > 4 * want && total > 256) {
    __syncthreads();
    int w2 = 1;
    while (w2 < want) w2 <<= 1;
    for (int i = threadIdx.x; i < w2; i += blockDim.x) sel[i] = 0ull;
    __syncthreads();
    select_top(keys, total, want, sel);
    bitonic_desc(sel, w2);
    keys = sel;
    n2 = w2;
  } else if (n2 > 1) {
    bitonic_desc(keys, n2);
  }
  __syncthreads();
  if (a.cand_val && a.cand_idx) {  // merged candidates out (no sampling)
    for (int i = threadIdx.x; i < a.top_k; i += blockDim.x) {
      const uint64_t kk = keys[i];
      a.cand_val[row * a.top_k + i] = kk ? vkey_value((uint32_t)(kk >> 32)) : -INFINITY;
      a.cand_idx[row * a.top_k + i] = kk ? (int64_t)ckey_col(kk) : -1;
    }
    return;
  }
  if (a.mode == 2) {
    // sample_all: the draw scaled by the whole row's sum; the chunk (index order)
    // where the running remainder reaches <= 0; then the column inside it
    if (threadIdx.x == 0) {
      const double u = rng_next_f64(a.rng + row);
      float sum = 0.0f;
      for (int c = 0; c < s.nchunks; ++c) sum += s.csum[row * s.nchunks + c];
      float r = __fmul_rn((float)u, sum);
      int c = 0;
      for (; c < s.nchunks - 1; ++c) {
        const float cs = s.csum[row * s.nchunks + c];
        if (r - cs <= 0.0f) break;
        r -= cs;
      }
      scan_r = r;
      scan_chunk = c;
    }
    __syncthreads();
    const int c = scan_chunk;
    const int64_t c0 = (int64_t)c * kChunk, c1 = min(s.n, c0 + kChunk);
    const bool use_pen = s.penalty != 1.0f && s.n_recent > 0;
    if (use_pen) mark_recent(s, row, c0, c1, pen);
    if (threadIdx.x >= 32) return;
    float rmax = -INFINITY;
    for (int cc = 0; cc < s.nchunks; ++cc) rmax = fmaxf(rmax, s.cmax[row * s.nchunks + cc]);
    // warp scan: 32 consecutive columns per step, inclusive prefix of their exps
    const int lane = threadIdx.x;
    float r = scan_r;
    int32_t tok = (int32_t)(s.idx_base + c1 - 1);
    for (int64_t b = c0; b < c1; b += 32) {
      const int64_t col = b + lane;
      float e = 0.0f;
      if (col < c1) e = expf(__fmul_rn(logit_at(s, row, col, use_pen ? pen : nullptr) - rmax, s.inv_t));
      float pre = e;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += t;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, col < c1 && r - pre <= 0.0f);
      if (hit) {
        tok = (int32_t)(s.idx_base + b + (__ffs(hit) - 1));
        break;
      }
      r -= __shfl_sync(0xffffffffu, pre, 31);
    }
    if (lane == 0) a.tokens[row] = tok;
    return;
  }
  if (a.mode == 0) {
    if (threadIdx.x == 0) a.tokens[row] = keys[0] ? (int32_t)ckey_col(keys[0]) : -1;
    return;
  }
  // candidates, sorted; the reference's softmax_over / top-p / draw in its order.
  // Every candidate's exp is computed once, in parallel; the sums stay sequential.
  __shared__ float exs[kSampleCap];
  int nc = a.top_k < n2 ? a.top_k : n2;
  while (nc > 0 && keys[nc - 1] == 0ull) --nc;  // padding (rows or shards shorter than k)
  if (nc == 0) {
    if (threadIdx.x == 0) a.tokens[row] = -1;
    return;
  }
  const float mx = vkey_value((uint32_t)(keys[0] >> 32));
  for (int i = threadIdx.x; i < nc; i += blockDim.x)
    exs[i] = expf(__fmul_rn(vkey_value((uint32_t)(keys[i] >> 32)) - mx, s.inv_t));
  __syncthreads();
  if (threadIdx.x != 0) return;
  auto ex = [&](int i) { return exs[i]; };
  int keep = nc;
  if (a.top_p < 1.0f) {
    float denom = 0.0f;
    if (a.whole_denominator)
      for (int c = 0; c < s.nchunks; ++c) denom += s.csum[row * s.nchunks + c];
    else
      for (int i = 0; i < nc; ++i) denom += ex(i);
    float cum = 0.0f;
    keep = 0;
    for (int i = 0; i < nc; ++i) {
      keep = i + 1;
      cum += __fdiv_rn(ex(i), denom);
      if (cum >= a.top_p) break;
    }
    if (cum < a.top_p && a.whole_denominator && (int64_t)nc < s.n) {
      // the nucleus extends past the candidates the device keeps
      gqd::report(a.err, GQ_DEVERR_SAMPLE_CAP);
      (void)rng_next_f64(a.rng + row);
      a.tokens[row] = -1;
      return;
    }
  }
  float ksum = 0.0f;
  for (int i = 0; i < keep; ++i) ksum += ex(i);
  float r = (float)rng_next_f64(a.rng + row);
  int32_t tok = (int32_t)ckey_col(keys[keep - 1]);
  for (int i = 0; i < keep; ++i) {
    r -= __fdiv_rn(ex(i), ksum);
    if (r <= 0.0f) {
      tok = (int32_t)ckey_col(keys[i]);
      break;
    }
  }
  a.tokens[row] = tok;
}

// Candidate merge + sampling over given (value, id) pairs: [m][ncand] rows of a
// vocab-sharded model's per-shard candidates gathered from every rank.
__global__ void __launch_bounds__(kRowThreads) pairs_to_keys_kernel(const float *val, const int64_t *idx, int64_t m,
                                                                    int64_t ncand, uint64_t *keys) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t total = m * ncand;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    keys[i] = idx[i] < 0 ? 0ull : ckey(val[i], (uint32_t)idx[i]);
}

}  // namespace

// ---- host side ------------------------------------------------------------------------

namespace {
int sample_prepare(gq_ctx *ctx, const float *logits, int64_t m, int64_t n, int64_t ld, int64_t idx_base, int k,
                   float penalty, const uint32_t *recent, int64_t n_recent, int64_t recent_stride, float inv_t,
                   bool need_sums, SampleArgs *out) {
  SampleArgs a = {};
  a.logits = logits;
  a.m = m;
  a.n = n;
  a.ld = ld ? ld : n;
  a.idx_base = idx_base;
  a.k = k;
  a.nchunks = (int)((n + kChunk - 1) / kChunk);
  a.penalty = penalty;
  a.recent = recent;
  a.n_recent = recent ? n_recent : 0;
  a.recent_stride = recent_stride ? recent_stride : n_recent;
  a.inv_t = inv_t;
  const size_t nkeys = (size_t)m * a.nchunks * k;
  const size_t bytes = nkeys * 8 + 2 * (size_t)m * a.nchunks * 4 + 64;
  void *ws = nullptr;
  int rc = gq_workspace(ctx, bytes, &ws);
  if (rc != GQ_OK) return rc;
  a.ckeys = static_cast<uint64_t *>(ws);
  a.cmax = reinterpret_cast<float *>(a.ckeys + nkeys);
  a.csum = a.cmax + m * a.nchunks;
  const dim3 grid((unsigned)a.nchunks, (unsigned)m);
  GQ_CUDA_TRY(ctx, gq_launch(ctx, topk_chunk_kernel, grid, dim3(kChunkThreads), 0, a));
  if (need_sums) GQ_CUDA_TRY(ctx, gq_launch(ctx, chunk_expsum_kernel, grid, dim3(kChunkThreads), 0, a));
  *out = a;
  return GQ_OK;
}

size_t row_smem(const SampleArgs &a) {
  size_t n2 = 1;
  while (n2 < (size_t)a.nchunks * a.k) n2 <<= 1;
  return n2 * 8 + kChunk + kSampleCap * 8;
}

int launch_rows(gq_ctx *ctx, const RowArgs &r) {
  const size_t smem = row_smem(r.s);
  // (16 KB for the kernel's static shared memory: histograms, survivors, exps)
  if (smem + 16384 > ctx->smem_optin) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "sample: too many candidates per row");
  // the dynamic shared memory the kernel may use, raised per device as larger merges come
  static size_t attr_set[64] = {};
  const int dev = ctx->device & 63;
  // (set whenever the need grows: the kernel's static shared memory counts
  // toward the 48 KB a launch may use without it)
  if (smem > attr_set[dev]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(sample_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set[dev] = smem;
  }
  GQ_CUDA_TRY(ctx, gq_launch(ctx, sample_row_kernel, dim3((unsigned)r.s.m), dim3(kRowThreads), smem, r));
  return GQ_OK;
}

int check_opts(gq_ctx *ctx, const gq_sample_opts *o, int64_t n_recent, const uint32_t *recent) {
  if (!o) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "sample: null options");
  if (o->top_k < 0 || o->top_k > kSampleCap)
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "sample: top_k must be in 0..256 on the device");
  if (!(o->top_p == o->top_p) || !(o->temperature == o->temperature) || !(o->repetition_penalty > 0.0f))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "sample: NaN option or non-positive penalty");
  if (n_recent < 0 || n_recent > kMaxRecent || (n_recent > 0 && !recent))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "sample: 0..4096 recent tokens");
  return GQ_OK;
}
}  // namespace

extern "C" int gq_sample_rows(gq_ctx *ctx, const float *logits, int64_t m, int64_t vocab, int64_t ld,
                              const gq_sample_opts *opts, const uint32_t *recent, int64_t n_recent,
                              int64_t recent_stride, uint64_t *rng_state, int32_t *tokens) {
  if (!ctx) return GQ_ERR_INVALID_ARGUMENT;
  if (gq_enter_ctx(ctx) != GQ_OK) return GQ_ERR_CUDA;
  int rc = check_opts(ctx, opts, n_recent, recent);
  if (rc != GQ_OK) return rc;
  if (m < 0 || vocab <= 0 || vocab > (1ll << 31) || (ld != 0 && ld < vocab) || m > 65535)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "sample: 0 <= m <= 65535 rows of 1 .. 2^31 logits");
  if (m == 0) return GQ_OK;
  if (!logits || !tokens || !rng_state) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "sample: null pointer");
  const gq_sample_opts o = *opts;
  RowArgs r = {};
  r.tokens = tokens;
  r.rng = rng_state;
  r.err = ctx->dev_err;
  r.top_p = o.top_p;
  const float penalty = (o.repetition_penalty != 1.0f && n_recent > 0) ? o.repetition_penalty : 1.0f;
  int k;
  bool sums = false;
  if (o.temperature <= 0.0f) {
    r.mode = 0;
    k = 1;
  } else if (o.top_k == 0 && o.top_p >= 1.0f) {
    r.mode = 2;
    k = 1;
    sums = true;
  } else {
    r.mode = 1;
    k = o.top_k > 0 ? o.top_k : kSampleCap;
    if (k > vocab) k = (int)vocab;
    r.top_k = k;
    r.whole_denominator = o.top_k == 0;
    sums = r.whole_denominator;
  }
  rc = sample_prepare(ctx, logits, m, vocab, ld, 0, k, penalty, recent, n_recent, recent_stride,
                      o.temperature > 0.0f ? 1.0f / o.temperature : 0.0f, sums, &r.s);
  if (rc != GQ_OK) return rc;
  return launch_rows(ctx, r);
}

extern "C" int gq_topk_rows(gq_ctx *ctx, const float *logits, int64_t m, int64_t n, int64_t ld, int64_t idx_base,
                            int32_t k, float repetition_penalty, const uint32_t *recent, int64_t n_recent,
                            int64_t recent_stride, float *val, int64_t *idx) {
  if (!ctx) return GQ_ERR_INVALID_ARGUMENT;
  if (gq_enter_ctx(ctx) != GQ_OK) return GQ_ERR_CUDA;
  if (k < 1 || k > kSampleCap) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "topk_rows: k must be in 1..256");
  if (m < 0 || n <= 0 || m > 65535 || idx_base < 0 || idx_base + n > (1ll << 31) || (ld != 0 && ld < n))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "topk_rows: bad shape");
  if (n_recent < 0 || n_recent > kMaxRecent || (n_recent > 0 && !recent) || !(repetition_penalty > 0.0f))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "topk_rows: recent tokens / penalty");
  if (m == 0) return GQ_OK;
  if (!logits || !val || !idx) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "topk_rows: null pointer");
  RowArgs r = {};
  r.top_k = k;
  r.cand_val = val;
  r.cand_idx = idx;
  r.err = ctx->dev_err;
  const float penalty = (repetition_penalty != 1.0f && n_recent > 0) ? repetition_penalty : 1.0f;
  int rc = sample_prepare(ctx, logits, m, n, ld, idx_base, k, penalty, recent, n_recent, recent_stride, 1.0f, false,
                          &r.s);
  if (rc != GQ_OK) return rc;
  return launch_rows(ctx, r);
}

extern "C" int gq_sample_candidates(gq_ctx *ctx, const float *val, const int64_t *idx, int64_t m, int64_t ncand,
                                    const gq_sample_opts *opts, uint64_t *rng_state, int32_t *tokens) {
  if (!ctx) return GQ_ERR_INVALID_ARGUMENT;
  if (gq_enter_ctx(ctx) != GQ_OK) return GQ_ERR_CUDA;
  int rc = check_opts(ctx, opts, 0, nullptr);
  if (rc != GQ_OK) return rc;
  if (m < 0 || m > 65535 || ncand < 1 || ncand > 16 * kSampleCap)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "sample_candidates: 1..4096 candidates per row");
  const gq_sample_opts o = *opts;
  if (o.temperature > 0.0f && o.top_k == 0)
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED,
                   "sample_candidates: candidates alone sample only greedy or top-k (top_k > 0) rows");
  if (m == 0) return GQ_OK;
  if (!val || !idx || !tokens || !rng_state) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "sample_candidates: null pointer");
  void *ws = nullptr;
  rc = gq_workspace(ctx, (size_t)m * ncand * 8 + 64, &ws);
  if (rc != GQ_OK) return rc;
  uint64_t *keys = static_cast<uint64_t *>(ws);
  GQ_CUDA_TRY(ctx, gq_launch(ctx, pairs_to_keys_kernel, dim3((unsigned)std::min<int64_t>((m * ncand + 1023) / 1024, 1024)),
                             dim3(1024), 0, val, idx, m, ncand, keys));
  RowArgs r = {};
  r.s.m = m;
  r.s.n = ncand;
  r.s.k = (int)ncand;
  r.s.nchunks = 1;
  r.s.ckeys = keys;
  r.s.inv_t = o.temperature > 0.0f ? 1.0f / o.temperature : 0.0f;
  r.s.penalty = 1.0f;
  r.tokens = tokens;
  r.rng = rng_state;
  r.err = ctx->dev_err;
  r.top_p = o.top_p;
  if (o.temperature <= 0.0f) {
    r.mode = 0;
  } else {
    r.mode = 1;
    r.top_k = (int)std::min<int64_t>(o.top_k, ncand);
  }
  return launch_rows(ctx, r);
}
