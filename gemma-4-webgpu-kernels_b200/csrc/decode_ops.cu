// decode_ops.cu — the support ops a quantized decode step needs around MATMUL_Q:
// RMSNorm (plain, fused residual add + layer scalar), per-head norm + partial
// RoPE, grouped-query attention over a KV cache, the bf16-weight linear of the
// per-layer-input projection, elementwise add/mul/scale and strided row copies.
//
// Each op follows the reference's CPU semantics (rust/src/backend_cpu.rs) with
// the same operation order inside an element; only sums over a row or a key
// range are reduced in tree order (checked against the CPU oracle by tolerance).
//
// Layout choices for B200:
//  * one warp per normalised row, float4 loads, the row's sum of squares in a
//    warp butterfly; outputs can go to a strided destination, so a key or value
//    row is written straight into its KV-cache slot (no separate append);
//  * RoPE frequencies are computed on the host with the same f32 expression as
//    the CPU and passed by value in the kernel parameters (no table in memory,
//    nothing to allocate, graph-capturable);
//  * attention: a CTA owns one (query token, KV head) pair and a contiguous
//    chunk of the active key range (causal and window bounds found by binary
//    search when key positions are ascending, as a KV cache's are); every
//    thread owns 4 of the head_dim columns for all the query heads of the group
//    (MQA: 8 heads read each K/V element once), so K and V stream from HBM with
//    coalesced 16-byte loads and no shared-memory staging; score partials are
//    reduced by a transposing warp butterfly; chunk results (max, sum, output)
//    are merged by a second kernel when the range is split.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "gq_internal.cuh"

namespace {

constexpr int kNormThreads = 256;  // 8 warps, one row per warp
constexpr int kMaxGroup = 8;       // query heads served per KV head
constexpr int kKeyBatch = 8;       // keys scored per butterfly
constexpr int kMaxChunk = 256;     // keys per attention CTA
constexpr int kMaxHalfRot = 256;   // rotary_dim / 2

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Output row address: row r = (group, inner) with `per_group` rows per group.
struct RowMap {
  int64_t per_group, group_stride, inner_stride;
  __device__ __forceinline__ int64_t at(int64_t r) const {
    return (r / per_group) * group_stride + (r % per_group) * inner_stride;
  }
};

// Sum of squares of one row (warp-cooperative; every lane gets the total).
__device__ __forceinline__ float row_sumsq(const float *xr, int64_t d, int lane, bool vec) {
  float ss = 0.0f;
  if (vec) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
    for (int64_t i = lane; i < d / 4; i += 32) {
      const float4 v = x4[i];
      ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
      ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
      ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
      ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
    }
  } else {
    for (int64_t i = lane; i < d; i += 32) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
  }
  return warp_sum(ss);
}

// rust/src/backend_cpu.rs:149-172: inv = 1 / sqrt(ss / d + eps).
__device__ __forceinline__ float rms_inv(float ss, int64_t d, float eps) {
  return __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
}

// KIND 0: y = x * inv * w            (rms_norm; w may be null)
// KIND 1: y = (r + x * inv * w) * s  (add_rms_norm, rust/src/backend.rs:137-144; s may be null)
template <int KIND>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float *x, const float *r, const float *w,
                                                               const float *s, int64_t rows, int64_t d, float eps,
                                                               float *y, RowMap ymap) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float *xr = x + row * d;
  float *yr = y + ymap.at(row);
  const bool vec = (d % 4 == 0) && ((uintptr_t)x % 16 == 0) && ((uintptr_t)yr % 16 == 0) &&
                   (w == nullptr || (uintptr_t)w % 16 == 0) && (KIND == 0 || (uintptr_t)r % 16 == 0);
  const float inv = rms_inv(row_sumsq(xr, d, lane, vec), d, eps);
  const float sc = (KIND == 1 && s) ? *s : 1.0f;
  auto one = [&](float xv, float wv, float rv) {
    float n = __fmul_rn(xv, inv);
    if (w) n = __fmul_rn(n, wv);
    if (KIND == 1) {
      n = __fadd_rn(rv, n);
      if (s) n = __fmul_rn(n, sc);
    }
    return n;
  };
  if (vec) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    const float4 *r4 = reinterpret_cast<const float4 *>(KIND == 1 ? r + row * d : nullptr);
    float4 *y4 = reinterpret_cast<float4 *>(yr);
    for (int64_t i = lane; i < d / 4; i += 32) {
      const float4 v = x4[i];
      const float4 wv = w ? w4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
      const float4 rv = KIND == 1 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      y4[i] = make_float4(one(v.x, wv.x, rv.x), one(v.y, wv.y, rv.y), one(v.z, wv.z, rv.z), one(v.w, wv.w, rv.w));
    }
  } else {
    for (int64_t i = lane; i < d; i += 32)
      yr[i] = one(xr[i], w ? w[i] : 1.0f, KIND == 1 ? r[row * d + i] : 0.0f);
  }
}

struct RopeFreq {
  float f[kMaxHalfRot];
};

// rust/src/backend.rs:148-154 (NORM) / rust/src/backend_cpu.rs:248-268 (rope):
// per (token, head) row of head_dim values, optional weighted RMSNorm, then the
// half-split rotation of the first rotary_dim values. Rows are (token, head)
// with `heads` rows per token; positions[token].
template <bool NORM>
__global__ void __launch_bounds__(kNormThreads) head_rope_kernel(const float *x, const float *w, int64_t rows,
                                                                 int64_t heads, int64_t dh, float eps,
                                                                 const uint32_t *positions, int half,
                                                                 const __grid_constant__ RopeFreq fr, float *y,
                                                                 RowMap ymap) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float *xr = x + row * dh;
  float *yr = y + ymap.at(row);
  float inv = 1.0f;
  if (NORM) inv = rms_inv(row_sumsq(xr, dh, lane, (dh % 4 == 0) && ((uintptr_t)x % 16 == 0)), dh, eps);
  auto nrm = [&](int64_t i) {
    const float v = xr[i];
    return NORM ? __fmul_rn(__fmul_rn(v, inv), w[i]) : v;
  };
  const float pos = (float)positions[row / heads];
  for (int j = lane; j < half; j += 32) {
    const float ang = __fmul_rn(pos, fr.f[j]);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float a = nrm(j), b = nrm(j + half);
    yr[j] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
    yr[j + half] = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
  }
  for (int64_t i = 2 * half + lane; i < dh; i += 32) yr[i] = nrm(i);
}

// ---- attention --------------------------------------------------------------

struct AttnArgs {
  const float *q, *k, *v;
  const uint32_t *q_pos, *k_pos;
  float *out;      // [B*T, Hq*dh] (splits == 1) ...
  float *part_o;   // ... or [B*T*Hq, splits, dh] unnormalised chunk outputs
  float *part_ml;  // [B*T*Hq, splits, 2] chunk max and sum of exponentials
  int64_t T, Hq, Hkv, dh, S;
  int64_t kv_batch_stride;  // elements between sequences' K (and V) caches
  int64_t kpos_batch_stride;
  float scale, softcap;
  uint32_t window;
  int sorted, chunk, splits;
};

// First index in [0, n) whose key position exceeds `bound` (ascending positions).
__device__ __forceinline__ int64_t upper_bound_pos(const uint32_t *kp, int64_t n, uint32_t bound) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (kp[mid] <= bound) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// Grid: x = key chunk, y = (sequence, query token, KV head). Block: NT threads,
// thread t owns head_dim columns 4t .. 4t+3 for every query head of the group.
template <int NT>
__global__ void __launch_bounds__(NT) attn_chunk_kernel(const AttnArgs a) {
  constexpr int NWARP = NT / 32;
  __shared__ float sc[kMaxChunk][kMaxGroup];  // scores, then probabilities
  __shared__ float red[NWARP][kKeyBatch * kMaxGroup];
  __shared__ float hm[kMaxGroup], hl[kMaxGroup];
  __shared__ int64_t range[2];

  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = (int)(a.Hq / a.Hkv);
  const int64_t rowid = blockIdx.y;
  const int64_t bt = rowid / a.Hkv, kvh = rowid % a.Hkv;
  const int64_t b = bt / a.T;
  const uint32_t qpos = a.q_pos[bt];
  const uint32_t *kp = a.k_pos + b * a.kpos_batch_stride;
  const float *kb = a.k + b * a.kv_batch_stride + kvh * a.dh;
  const float *vb = a.v + b * a.kv_batch_stride + kvh * a.dh;
  const int64_t kv_row = a.Hkv * a.dh;

  if (tid == 0) {
    int64_t lo = 0, hi = a.S;
    if (a.sorted) {
      hi = upper_bound_pos(kp, a.S, qpos);
      if (a.window > 0 && qpos >= a.window) lo = upper_bound_pos(kp, hi, qpos - a.window);
    }
    const int64_t j0 = lo + (int64_t)blockIdx.x * a.chunk;
    range[0] = j0;
    range[1] = min(hi, j0 + (int64_t)a.chunk);
  }
  __syncthreads();
  const int64_t j0 = range[0], j1 = range[1];
  const int nkeys = j1 > j0 ? (int)(j1 - j0) : 0;

  const int col = 4 * tid;
  const bool colv = col < a.dh;
  float4 q[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    q[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g < G && colv)
      q[g] = *reinterpret_cast<const float4 *>(a.q + bt * a.Hq * a.dh + (kvh * G + g) * a.dh + col);
  }

  // ---- scores of the chunk, kKeyBatch keys at a time ----
  for (int jb = 0; jb < nkeys; jb += kKeyBatch) {
    float4 kv[kKeyBatch];
#pragma unroll
    for (int kk = 0; kk < kKeyBatch; ++kk) {
      kv[kk] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (jb + kk < nkeys && colv) kv[kk] = __ldg(reinterpret_cast<const float4 *>(kb + (j0 + jb + kk) * kv_row + col));
    }
    float p[kMaxGroup * kKeyBatch];  // index g * kKeyBatch + kk
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g)
#pragma unroll
      for (int kk = 0; kk < kKeyBatch; ++kk) {
        float t = __fmul_rn(q[g].x, kv[kk].x);
        t = __fmaf_rn(q[g].y, kv[kk].y, t);
        t = __fmaf_rn(q[g].z, kv[kk].z, t);
        t = __fmaf_rn(q[g].w, kv[kk].w, t);
        p[g * kKeyBatch + kk] = t;
      }
    // transposing butterfly: afterwards lane l holds the warp sums of entries 2l, 2l+1
#pragma unroll
    for (int o = 16, n = kMaxGroup * kKeyBatch; o >= 1; o >>= 1, n >>= 1) {
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = up ? p[i] : p[i + n / 2];
        const float keep = up ? p[i + n / 2] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    if (NWARP > 1) {
      red[warp][2 * lane] = p[0];
      red[warp][2 * lane + 1] = p[1];
      __syncthreads();
    }
    if (tid < kMaxGroup * kKeyBatch / (NWARP > 1 ? 1 : 2)) {
      // entries handled by this thread: NWARP > 1 -> one entry (tid); else two (2*lane, 2*lane+1)
      const int ne = NWARP > 1 ? 1 : 2;
      for (int e = 0; e < ne; ++e) {
        const int idx = NWARP > 1 ? tid : 2 * lane + e;
        float sum = NWARP > 1 ? 0.0f : p[e];
        if (NWARP > 1)
#pragma unroll
          for (int w2 = 0; w2 < NWARP; ++w2) sum += red[w2][idx];
        const int g = idx / kKeyBatch, kk = idx % kKeyBatch;
        const int jj = jb + kk;
        if (g < G && jj < nkeys) {
          const uint32_t kpos = kp[j0 + jj];
          float s = __fmul_rn(sum, a.scale);
          if (a.softcap > 0.0f) s = __fmul_rn(a.softcap, tanhf(__fdiv_rn(s, a.softcap)));
          if (kpos > qpos || (a.window > 0 && qpos - kpos >= a.window)) s = -INFINITY;
          sc[jj][g] = s;
        }
      }
    }
    __syncthreads();
  }

  // ---- per head: chunk max, probabilities, sum ----
  for (int g = warp; g < G; g += NWARP) {
    float m = -INFINITY;
    for (int j = lane; j < nkeys; j += 32) m = fmaxf(m, sc[j][g]);
    m = warp_max(m);
    float l = 0.0f;
    for (int j = lane; j < nkeys; j += 32) {
      const float s = sc[j][g];
      const float e = (s == -INFINITY) ? 0.0f : expf(__fsub_rn(s, m));
      sc[j][g] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      hm[g] = m;
      hl[g] = l;
    }
  }
  __syncthreads();

  // ---- P·V over the chunk ----
  float4 o[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int jb = 0; jb < nkeys; jb += 4) {
    float4 vv[4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      vv[kk] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (jb + kk < nkeys && colv) vv[kk] = __ldg(reinterpret_cast<const float4 *>(vb + (j0 + jb + kk) * kv_row + col));
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if (jb + kk >= nkeys) break;
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        const float pr = sc[jb + kk][g];
        o[g].x = __fmaf_rn(pr, vv[kk].x, o[g].x);
        o[g].y = __fmaf_rn(pr, vv[kk].y, o[g].y);
        o[g].z = __fmaf_rn(pr, vv[kk].z, o[g].z);
        o[g].w = __fmaf_rn(pr, vv[kk].w, o[g].w);
      }
    }
  }

  if (!colv) return;
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g >= G) break;
    const int64_t h = kvh * G + g;
    if (a.splits == 1) {
      const float inv = hl[g] > 0.0f ? __fdiv_rn(1.0f, hl[g]) : 0.0f;
      *reinterpret_cast<float4 *>(a.out + bt * a.Hq * a.dh + h * a.dh + col) =
          make_float4(__fmul_rn(o[g].x, inv), __fmul_rn(o[g].y, inv), __fmul_rn(o[g].z, inv), __fmul_rn(o[g].w, inv));
    } else {
      const int64_t prow = (bt * a.Hq + h) * a.splits + blockIdx.x;
      *reinterpret_cast<float4 *>(a.part_o + prow * a.dh + col) = o[g];
      if (tid == 0) {
        a.part_ml[2 * prow] = hm[g];
        a.part_ml[2 * prow + 1] = hl[g];
      }
    }
  }
}

// Merge the chunks of one (token, head) row: out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s.
__global__ void attn_combine_kernel(const float *part_o, const float *part_ml, int64_t rows, int64_t Hq, int64_t dh,
                                    int splits, float *out) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t row = blockIdx.x;  // (token, head)
  if (row >= rows) return;
  const float *ml = part_ml + row * splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ml[2 * s]);
  float L = 0.0f;
  for (int s = 0; s < splits; ++s)
    if (ml[2 * s] != -INFINITY) L += __fmul_rn(expf(__fsub_rn(ml[2 * s], M)), ml[2 * s + 1]);
  const float inv = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
  const int64_t bt = row / Hq, h = row % Hq;
  for (int64_t c = 4 * threadIdx.x; c < dh; c += 4 * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < splits; ++s) {
      if (ml[2 * s] == -INFINITY) continue;
      const float wgt = expf(__fsub_rn(ml[2 * s], M));
      const float4 v = *reinterpret_cast<const float4 *>(part_o + (row * splits + s) * dh + c);
      acc.x = __fmaf_rn(wgt, v.x, acc.x);
      acc.y = __fmaf_rn(wgt, v.y, acc.y);
      acc.z = __fmaf_rn(wgt, v.z, acc.z);
      acc.w = __fmaf_rn(wgt, v.w, acc.w);
    }
    *reinterpret_cast<float4 *>(out + bt * Hq * dh + h * dh + c) =
        make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
  }
}

// ---- bf16-weight linear (the per-layer-input model projection) ------------------
// y[m, n] = sum_k x[m, k] * w[n, k], w stored as bf16 [n, k]. One warp per weight
// row; the warp keeps a 2048-column slice of its row in registers and sweeps all
// m activation rows over it, so each weight byte is read once.
constexpr int kLinWarps = 8;
constexpr int kLinSlice = 2048;  // columns per register slice (8 per lane per 256)

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__global__ void __launch_bounds__(kLinWarps * 32) linear_bf16_kernel(const float *x, int64_t m, int64_t k,
                                                                     const uint16_t *w, int64_t n, float *y) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLinWarps + (threadIdx.x >> 5);
  if (row >= n) return;
  const uint16_t *wr = w + row * k;
  for (int64_t k0 = 0; k0 < k; k0 += kLinSlice) {
    const int64_t kl = min((int64_t)kLinSlice, k - k0);  // multiple of 8
    uint4 wv[kLinSlice / 256];
#pragma unroll
    for (int i = 0; i < kLinSlice / 256; ++i) {
      const int64_t c = k0 + 256 * i + 8 * lane;
      wv[i] = (256 * i + 8 * lane < kl) ? __ldg(reinterpret_cast<const uint4 *>(wr + c)) : make_uint4(0, 0, 0, 0);
    }
    for (int64_t mm = 0; mm < m; ++mm) {
      const float *xr = x + mm * k + k0;
      float acc = 0.0f;
#pragma unroll
      for (int i = 0; i < kLinSlice / 256; ++i) {
        const int c = 256 * i + 8 * lane;
        if (c < kl) {
          const float4 xa = __ldg(reinterpret_cast<const float4 *>(xr + c));
          const float4 xb = __ldg(reinterpret_cast<const float4 *>(xr + c + 4));
          acc = __fmaf_rn(xa.x, bf16lo(wv[i].x), acc);
          acc = __fmaf_rn(xa.y, bf16hi(wv[i].x), acc);
          acc = __fmaf_rn(xa.z, bf16lo(wv[i].y), acc);
          acc = __fmaf_rn(xa.w, bf16hi(wv[i].y), acc);
          acc = __fmaf_rn(xb.x, bf16lo(wv[i].z), acc);
          acc = __fmaf_rn(xb.y, bf16hi(wv[i].z), acc);
          acc = __fmaf_rn(xb.z, bf16lo(wv[i].w), acc);
          acc = __fmaf_rn(xb.w, bf16hi(wv[i].w), acc);
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) y[mm * n + row] = (k0 == 0) ? acc : __fadd_rn(y[mm * n + row], acc);
    }
  }
}

// Any shape: one thread per output, sequential k (the CPU's order).
__global__ void linear_bf16_scalar_kernel(const float *x, int64_t m, int64_t k, const uint16_t *w, int64_t n,
                                          float *y) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m * n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t mm = i / n, nn = i % n;
    float acc = 0.0f;
    for (int64_t kk = 0; kk < k; ++kk)
      acc = __fadd_rn(acc, __fmul_rn(x[mm * k + kk], __uint_as_float((uint32_t)w[nn * k + kk] << 16)));
    y[i] = acc;
  }
}

// ---- elementwise and row copies -------------------------------------------------
// op 0: a + b   op 1: a * b   op 2: a * s   op 3: a * sp[0]   (rust/src/backend_cpu.rs:224-235)
__global__ void ew_kernel(int op, const float *a, const float *b, float s, const float *sp, int64_t count, float *y) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const float f = (op == 3) ? *sp : s;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = a[i];
    y[i] = op == 0 ? __fadd_rn(v, b[i]) : op == 1 ? __fmul_rn(v, b[i]) : __fmul_rn(v, f);
  }
}

// dst[r * dst_stride + c] = src[r * src_stride + c], r < rows, c < cols.
__global__ void copy_rows_kernel(const float *src, int64_t rows, int64_t cols, int64_t src_stride, float *dst,
                                 int64_t dst_stride) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * cols; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    dst[r * dst_stride + c] = src[r * src_stride + c];
  }
}

unsigned blocks_for(gq_ctx *ctx, int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)ctx->num_sms * 16;
  return (unsigned)std::max<int64_t>(1, std::min(g, cap));
}

#define ENTER(ctx)                           \
  do {                                       \
    if (!(ctx)) return GQ_ERR_INVALID_ARGUMENT; \
    int _rc = gq_enter_ctx(ctx);             \
    if (_rc != GQ_OK) return _rc;            \
  } while (0)

int norm_launch(gq_ctx *ctx, int kind, const float *x, const float *r, const float *w, const float *s, int64_t rows,
                int64_t d, float eps, float *y, RowMap ym) {
  const dim3 grid((unsigned)((rows + kNormThreads / 32 - 1) / (kNormThreads / 32)));
  if (kind == 0)
    GQ_CUDA_TRY(ctx, gq_launch(ctx, rmsnorm_kernel<0>, grid, dim3(kNormThreads), 0, x, r, w, s, rows, d, eps, y, ym));
  else
    GQ_CUDA_TRY(ctx, gq_launch(ctx, rmsnorm_kernel<1>, grid, dim3(kNormThreads), 0, x, r, w, s, rows, d, eps, y, ym));
  return GQ_OK;
}

int rope_launch(gq_ctx *ctx, bool norm, const float *x, const float *w, int64_t t, int64_t heads, int64_t dh,
                float eps, const uint32_t *positions, float theta, int64_t rot, float *y, int64_t y_tok_stride) {
  if (t < 0 || heads <= 0 || dh <= 0 || rot < 0 || rot > dh || rot % 2 != 0)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "rope: need 0 <= rotary_dim <= head_dim, rotary_dim even");
  if (rot / 2 > kMaxHalfRot) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "rope: rotary_dim > 512");
  if (!x || !y || (t > 0 && !positions) || (norm && !w)) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "rope: null pointer");
  if (y_tok_stride < heads * dh) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "rope: output token stride too small");
  if (t == 0) return GQ_OK;
  RopeFreq fr;
  const int half = (int)(rot / 2);
  // the reference's frequency, same f32 expression (rust/src/backend_cpu.rs:258)
  for (int j = 0; j < half; ++j) fr.f[j] = powf(theta, -(2.0f * (float)j) / (float)rot);
  const int64_t rows = t * heads;
  const RowMap ym{heads, y_tok_stride, dh};
  const dim3 grid((unsigned)((rows + kNormThreads / 32 - 1) / (kNormThreads / 32)));
  if (norm)
    GQ_CUDA_TRY(ctx, gq_launch(ctx, head_rope_kernel<true>, grid, dim3(kNormThreads), 0, x, w, rows, heads, dh, eps,
                               positions, half, fr, y, ym));
  else
    GQ_CUDA_TRY(ctx, gq_launch(ctx, head_rope_kernel<false>, grid, dim3(kNormThreads), 0, x, w, rows, heads, dh, eps,
                               positions, half, fr, y, ym));
  return GQ_OK;
}

template <int NT>
cudaError_t attn_launch_nt(gq_ctx *ctx, dim3 grid, const AttnArgs &a) {
  return gq_launch(ctx, attn_chunk_kernel<NT>, grid, dim3(NT), 0, a);
}

}  // namespace

extern "C" {

int gq_rms_norm(gq_ctx *ctx, const float *x, int64_t rows, int64_t d, const float *w, float eps, float *y,
                int64_t y_stride) {
  ENTER(ctx);
  if (rows < 0 || d <= 0 || !x || !y) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "rms_norm: bad shape or null pointer");
  if (y_stride == 0) y_stride = d;
  if (y_stride < d) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "rms_norm: y_stride < d");
  if (rows == 0) return GQ_OK;
  return norm_launch(ctx, 0, x, nullptr, w, nullptr, rows, d, eps, y, RowMap{1, y_stride, 0});
}

int gq_add_rms_norm(gq_ctx *ctx, const float *residual, const float *x, int64_t rows, int64_t d, const float *w,
                    float eps, const float *scale_by, float *y) {
  ENTER(ctx);
  if (rows < 0 || d <= 0 || !x || !y || !residual || !w)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "add_rms_norm: bad shape or null pointer");
  if (rows == 0) return GQ_OK;
  return norm_launch(ctx, 1, x, residual, w, scale_by, rows, d, eps, y, RowMap{1, d, 0});
}

int gq_head_norm_rope(gq_ctx *ctx, const float *x, int64_t t, int64_t heads, int64_t head_dim, const float *w,
                      float eps, const uint32_t *positions, float theta, int64_t rotary_dim, float *y,
                      int64_t y_tok_stride) {
  ENTER(ctx);
  if (y_tok_stride == 0) y_tok_stride = heads * head_dim;
  return rope_launch(ctx, true, x, w, t, heads, head_dim, eps, positions, theta, rotary_dim, y, y_tok_stride);
}

int gq_rope(gq_ctx *ctx, const float *x, int64_t t, int64_t heads, int64_t head_dim, const uint32_t *positions,
            float theta, int64_t rotary_dim, float *y, int64_t y_tok_stride) {
  ENTER(ctx);
  if (y_tok_stride == 0) y_tok_stride = heads * head_dim;
  return rope_launch(ctx, false, x, nullptr, t, heads, head_dim, 0.0f, positions, theta, rotary_dim, y, y_tok_stride);
}

int gq_attention(gq_ctx *ctx, const float *q, int64_t batch, int64_t t, int64_t hq, int64_t head_dim, const float *k,
                 const float *v, int64_t s, int64_t hkv, int64_t kv_batch_stride, const uint32_t *q_pos,
                 const uint32_t *k_pos, int64_t kpos_batch_stride, float scale, uint32_t sliding_window,
                 float attn_softcap, uint32_t flags, float *out) {
  ENTER(ctx);
  if (batch < 0 || t < 0 || s < 0 || hq <= 0 || hkv <= 0 || hq % hkv != 0 || head_dim <= 0)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "attention: bad shape");
  if (hq / hkv > kMaxGroup) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "attention: more than 8 query heads per KV head");
  if (head_dim % 4 != 0 || head_dim > 4 * 256)
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "attention: head_dim must be a multiple of 4, at most 1024");
  if (batch * t == 0) return GQ_OK;
  if (!q || !out || !q_pos || (s > 0 && (!k || !v || !k_pos)))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "attention: null pointer");
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) % 16 != 0 || kv_batch_stride % 4 != 0)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT,
                   "attention: q, k, v and out must be 16-byte aligned, kv_batch_stride a multiple of 4");
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.q_pos = q_pos;
  a.k_pos = k_pos;
  a.out = out;
  a.T = t;
  a.Hq = hq;
  a.Hkv = hkv;
  a.dh = head_dim;
  a.S = s;
  a.kv_batch_stride = kv_batch_stride;
  a.kpos_batch_stride = kpos_batch_stride;
  a.scale = scale;
  a.softcap = attn_softcap;
  a.window = sliding_window;
  a.sorted = (flags & GQ_ATTN_KPOS_ASCENDING) ? 1 : 0;
  // keys a query can reach: the window bounds the range when positions ascend
  const int64_t active = (a.sorted && sliding_window > 0) ? std::min<int64_t>(s, sliding_window) : s;
  const int64_t rows = batch * t * hkv;
  int chunk = 32;
  while (chunk < kMaxChunk && rows * ((active + chunk - 1) / chunk) > 4 * (int64_t)ctx->num_sms * 4) chunk *= 2;
  a.chunk = chunk;
  a.splits = (int)std::max<int64_t>(1, (active + chunk - 1) / chunk);
  if (rows > 65535) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "attention: more than 65535 (token, kv head) rows");
  if (a.splits > 1) {
    const size_t orow = (size_t)(batch * t * hq) * a.splits;
    void *ws = nullptr;
    int rc = gq_workspace(ctx, orow * (size_t)head_dim * 4 + orow * 8 + 256, &ws);
    if (rc != GQ_OK) return rc;
    a.part_o = static_cast<float *>(ws);
    a.part_ml = a.part_o + orow * head_dim;
  }
  const dim3 grid((unsigned)a.splits, (unsigned)rows);
  const int nt = head_dim <= 128 ? 32 : head_dim <= 256 ? 64 : head_dim <= 512 ? 128 : 256;
  cudaError_t e;
  switch (nt) {
    case 32: e = attn_launch_nt<32>(ctx, grid, a); break;
    case 64: e = attn_launch_nt<64>(ctx, grid, a); break;
    case 128: e = attn_launch_nt<128>(ctx, grid, a); break;
    default: e = attn_launch_nt<256>(ctx, grid, a); break;
  }
  GQ_CUDA_TRY(ctx, e);
  if (a.splits > 1) {
    const int ct = (int)std::min<int64_t>(256, std::max<int64_t>(32, (head_dim / 4 + 31) / 32 * 32));
    GQ_CUDA_TRY(ctx, gq_launch(ctx, attn_combine_kernel, dim3((unsigned)(batch * t * hq)), dim3(ct), 0, a.part_o,
                               a.part_ml, batch * t * hq, hq, head_dim, a.splits, out));
  }
  return GQ_OK;
}

int gq_linear_bf16(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const uint16_t *w, int64_t n, float *y) {
  ENTER(ctx);
  if (m < 0 || k < 0 || n < 0) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_bf16: bad shape");
  if (m == 0 || n == 0) return GQ_OK;
  if (!x || !w || !y) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_bf16: null pointer");
  const bool vec = k % 8 == 0 && k > 0 && (uintptr_t)x % 16 == 0 && (uintptr_t)w % 16 == 0;
  if (vec) {
    GQ_CUDA_TRY(ctx, gq_launch(ctx, linear_bf16_kernel, dim3((unsigned)((n + kLinWarps - 1) / kLinWarps)),
                               dim3(kLinWarps * 32), 0, x, m, k, w, n, y));
  } else {
    GQ_CUDA_TRY(ctx, gq_launch(ctx, linear_bf16_scalar_kernel, dim3(blocks_for(ctx, m * n, 128)), dim3(128), 0, x, m,
                               k, w, n, y));
  }
  return GQ_OK;
}

static int ew(gq_ctx *ctx, int op, const float *a, const float *b, float s, const float *sp, int64_t n, float *y) {
  ENTER(ctx);
  if (n < 0) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "elementwise: negative count");
  if (n == 0) return GQ_OK;
  if (!a || !y || (op < 2 && !b) || (op == 3 && !sp)) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "elementwise: null pointer");
  GQ_CUDA_TRY(ctx, gq_launch(ctx, ew_kernel, dim3(blocks_for(ctx, n, 256)), dim3(256), 0, op, a, b, s, sp, n, y));
  return GQ_OK;
}

int gq_add(gq_ctx *ctx, const float *a, const float *b, int64_t n, float *y) { return ew(ctx, 0, a, b, 0.f, nullptr, n, y); }
int gq_mul(gq_ctx *ctx, const float *a, const float *b, int64_t n, float *y) { return ew(ctx, 1, a, b, 0.f, nullptr, n, y); }
int gq_scale(gq_ctx *ctx, const float *a, int64_t n, float s, float *y) { return ew(ctx, 2, a, nullptr, s, nullptr, n, y); }
int gq_scale_by_tensor(gq_ctx *ctx, const float *a, int64_t n, const float *s, float *y) {
  return ew(ctx, 3, a, nullptr, 0.f, s, n, y);
}

int gq_copy_rows(gq_ctx *ctx, const float *src, int64_t rows, int64_t cols, int64_t src_stride, float *dst,
                 int64_t dst_stride) {
  ENTER(ctx);
  if (rows < 0 || cols < 0 || src_stride < cols || dst_stride < cols)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "copy_rows: bad shape");
  if (rows * cols == 0) return GQ_OK;
  if (!src || !dst) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "copy_rows: null pointer");
  GQ_CUDA_TRY(ctx, gq_launch(ctx, copy_rows_kernel, dim3(blocks_for(ctx, rows * cols, 256)), dim3(256), 0, src, rows,
                             cols, src_stride, dst, dst_stride));
  return GQ_OK;
}

}  // extern "C"
