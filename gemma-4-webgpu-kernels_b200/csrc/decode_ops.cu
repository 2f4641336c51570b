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
//    chunk of the active key range (causal and window bounds computed directly
//    when key j sits at position j, as in a KV cache, or found by binary search
//    when positions only ascend); every thread owns 4 of the head_dim columns
//    for all the query heads of the group (MQA: 8 heads read each K/V element
//    once); score partials are reduced by a transposing warp butterfly; chunk
//    results (max, sum, output) are merged by a second kernel when the range is
//    split. With one KV head (rows contiguous) the chunk streams through a ring
//    of shared-memory stages filled by bulk copies (TMA engine), softmax online;
//    otherwise K and V are read with coalesced 16-byte loads straight from HBM.
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

// Register-resident variant of rmsnorm_kernel for rows of d <= 128 * VPL values
// (d % 4 == 0, 16-byte aligned rows): every lane issues all of its x, w and
// residual loads before the first use, so a row costs one memory round trip
// instead of one per strided loop iteration.
template <int KIND, int VPL>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_reg_kernel(const float *x, const float *r, const float *w,
                                                                   const float *s, int64_t rows, int64_t d,
                                                                   float eps, float *y, RowMap ymap) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int n4 = (int)(d / 4);
  const float4 *x4 = reinterpret_cast<const float4 *>(x + row * d);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  const float4 *r4 = reinterpret_cast<const float4 *>(KIND == 1 ? r + row * d : nullptr);
  const float sc = (KIND == 1 && s) ? __ldg(s) : 1.0f;
  float4 xv[VPL], wv[VPL], rv[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const bool in = c < n4;
    xv[i] = in ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    wv[i] = (in && w) ? __ldg(w4 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
    rv[i] = (KIND == 1 && in) ? r4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    ss = __fadd_rn(ss, __fmul_rn(xv[i].x, xv[i].x));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].y, xv[i].y));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].z, xv[i].z));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].w, xv[i].w));
  }
  const float inv = rms_inv(warp_sum(ss), d, eps);
  auto one = [&](float xx, float ww, float rr) {
    float n = __fmul_rn(xx, inv);
    if (w) n = __fmul_rn(n, ww);
    if (KIND == 1) {
      n = __fadd_rn(rr, n);
      if (s) n = __fmul_rn(n, sc);
    }
    return n;
  };
  float4 *y4 = reinterpret_cast<float4 *>(y + ymap.at(row));
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    if (c < n4)
      y4[c] = make_float4(one(xv[i].x, wv[i].x, rv[i].x), one(xv[i].y, wv[i].y, rv[i].y),
                          one(xv[i].z, wv[i].z, rv[i].z), one(xv[i].w, wv[i].w, rv[i].w));
  }
}

// add_rms_norm followed by rms_norm of its result, in one pass over the row:
// h = (r + rms_norm(x, w1)) * s, xn = rms_norm(h, w2). Every element and row sum
// is computed exactly as rmsnorm_reg_kernel computes it, so both outputs equal
// the two separate calls bit for bit. h may alias r.
template <int VPL>
__global__ void __launch_bounds__(kNormThreads) add_norm_norm_kernel(const float *x, const float *r, const float *w1,
                                                                     const float *s, const float *w2, int64_t rows,
                                                                     int64_t d, float eps, float *h, float *xn) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int n4 = (int)(d / 4);
  const float4 *x4 = reinterpret_cast<const float4 *>(x + row * d);
  const float4 *r4 = reinterpret_cast<const float4 *>(r + row * d);
  const float4 *w14 = reinterpret_cast<const float4 *>(w1);
  const float4 *w24 = reinterpret_cast<const float4 *>(w2);
  const float sc = s ? __ldg(s) : 1.0f;
  float4 xv[VPL], rv[VPL], wv[VPL], w2v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const bool in = c < n4;
    xv[i] = in ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    rv[i] = in ? r4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    wv[i] = in ? __ldg(w14 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
    w2v[i] = in ? __ldg(w24 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    ss = __fadd_rn(ss, __fmul_rn(xv[i].x, xv[i].x));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].y, xv[i].y));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].z, xv[i].z));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].w, xv[i].w));
  }
  const float inv = rms_inv(warp_sum(ss), d, eps);
  auto one = [&](float xx, float ww, float rr) {
    float n = __fadd_rn(rr, __fmul_rn(__fmul_rn(xx, inv), ww));
    if (s) n = __fmul_rn(n, sc);
    return n;
  };
  float ss2 = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    xv[i] = make_float4(one(xv[i].x, wv[i].x, rv[i].x), one(xv[i].y, wv[i].y, rv[i].y),
                        one(xv[i].z, wv[i].z, rv[i].z), one(xv[i].w, wv[i].w, rv[i].w));
    if (lane + 32 * i >= n4) xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    ss2 = __fadd_rn(ss2, __fmul_rn(xv[i].x, xv[i].x));
    ss2 = __fadd_rn(ss2, __fmul_rn(xv[i].y, xv[i].y));
    ss2 = __fadd_rn(ss2, __fmul_rn(xv[i].z, xv[i].z));
    ss2 = __fadd_rn(ss2, __fmul_rn(xv[i].w, xv[i].w));
  }
  const float inv2 = rms_inv(warp_sum(ss2), d, eps);
  float4 *h4 = reinterpret_cast<float4 *>(h + row * d);
  float4 *y4 = reinterpret_cast<float4 *>(xn + row * d);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    if (c < n4) {
      h4[c] = xv[i];
      y4[c] = make_float4(__fmul_rn(__fmul_rn(xv[i].x, inv2), w2v[i].x), __fmul_rn(__fmul_rn(xv[i].y, inv2), w2v[i].y),
                          __fmul_rn(__fmul_rn(xv[i].z, inv2), w2v[i].z), __fmul_rn(__fmul_rn(xv[i].w, inv2), w2v[i].w));
    }
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

// Register-resident head_rope_kernel for head_dim <= 128 * VPL (head_dim % 4 == 0,
// 16-byte aligned rows): the row and its weights are loaded up front, the
// normalised row goes through a per-warp shared-memory buffer so each lane can
// read the pair (j, j + half) it rotates.
template <bool NORM, int VPL>
__global__ void __launch_bounds__(kNormThreads) head_rope_reg_kernel(const float *x, const float *w, int64_t rows,
                                                                     int64_t heads, int64_t dh, float eps,
                                                                     const uint32_t *positions, int half,
                                                                     const __grid_constant__ RopeFreq fr, float *y,
                                                                     RowMap ymap) {
  __shared__ __align__(16) float buf[kNormThreads / 32][128 * VPL];
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + warp;
  if (row >= rows) return;
  const int n4 = (int)(dh / 4);
  const float4 *x4 = reinterpret_cast<const float4 *>(x + row * dh);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  const float pos = (float)__ldg(positions + row / heads);
  float4 xv[VPL], wv[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const bool in = c < n4;
    xv[i] = in ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    wv[i] = (NORM && in) ? __ldg(w4 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
  }
  float inv = 1.0f;
  if (NORM) {
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      ss = __fadd_rn(ss, __fmul_rn(xv[i].x, xv[i].x));
      ss = __fadd_rn(ss, __fmul_rn(xv[i].y, xv[i].y));
      ss = __fadd_rn(ss, __fmul_rn(xv[i].z, xv[i].z));
      ss = __fadd_rn(ss, __fmul_rn(xv[i].w, xv[i].w));
    }
    inv = rms_inv(warp_sum(ss), dh, eps);
  }
  float *b = buf[warp];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    if (c < n4) {
      float4 n = xv[i];
      if (NORM)
        n = make_float4(__fmul_rn(__fmul_rn(n.x, inv), wv[i].x), __fmul_rn(__fmul_rn(n.y, inv), wv[i].y),
                        __fmul_rn(__fmul_rn(n.z, inv), wv[i].z), __fmul_rn(__fmul_rn(n.w, inv), wv[i].w));
      reinterpret_cast<float4 *>(b)[c] = n;
    }
  }
  __syncwarp();
  float *yr = y + ymap.at(row);
  for (int j = lane; j < half; j += 32) {
    const float ang = __fmul_rn(pos, fr.f[j]);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float a = b[j], bb = b[j + half];
    yr[j] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(bb, sn));
    yr[j + half] = __fadd_rn(__fmul_rn(bb, cs), __fmul_rn(a, sn));
  }
  for (int64_t i = 2 * half + lane; i < dh; i += 32) yr[i] = b[i];
}

// The attention inputs of a KV layer in one launch (rust/src/model.rs:254-273):
// rows of the stacked projection output [t, (hq + 2 hkv) * dh] are, per token,
// hq query heads (weighted norm + RoPE), hkv key heads (weighted norm + RoPE) and
// hkv value heads (unweighted norm). One warp per (token, head) row with the
// arithmetic of head_rope_reg_kernel (the value norm is that kernel's with unit
// weights, the same products as rms_norm with no weight).
struct QkvArgs {
  const float *qkv;
  int64_t t, qkv_stride;
  int hq, hkv;
  int64_t dh;
  const float *qw, *kw;
  float eps;
  const uint32_t *positions;
  int half;
  float *q_out, *k_out, *v_out;
  int64_t q_stride, k_stride, v_stride;
};

template <int VPL>
__global__ void __launch_bounds__(kNormThreads) qkv_norm_rope_kernel(const QkvArgs a,
                                                                     const __grid_constant__ RopeFreq fr) {
  __shared__ __align__(16) float buf[kNormThreads / 32][128 * VPL];
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per_tok = a.hq + 2 * a.hkv;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + warp;
  if (row >= a.t * per_tok) return;
  const int64_t tok = row / per_tok;
  const int r = (int)(row - tok * per_tok);
  const int kind = r < a.hq ? 0 : (r < a.hq + a.hkv ? 1 : 2);  // q, k, v
  const float *w = kind == 0 ? a.qw : (kind == 1 ? a.kw : nullptr);
  float *yr = kind == 0 ? a.q_out + tok * a.q_stride + (int64_t)r * a.dh
            : kind == 1 ? a.k_out + tok * a.k_stride + (int64_t)(r - a.hq) * a.dh
                        : a.v_out + tok * a.v_stride + (int64_t)(r - a.hq - a.hkv) * a.dh;
  const int n4 = (int)(a.dh / 4);
  const float4 *x4 = reinterpret_cast<const float4 *>(a.qkv + tok * a.qkv_stride + (int64_t)r * a.dh);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  float4 xv[VPL], wv[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const bool in = c < n4;
    xv[i] = in ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    wv[i] = (w && in) ? __ldg(w4 + c) : make_float4(1.f, 1.f, 1.f, 1.f);
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    ss = __fadd_rn(ss, __fmul_rn(xv[i].x, xv[i].x));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].y, xv[i].y));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].z, xv[i].z));
    ss = __fadd_rn(ss, __fmul_rn(xv[i].w, xv[i].w));
  }
  const float inv = rms_inv(warp_sum(ss), a.dh, a.eps);
  float *b = buf[warp];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    if (c < n4) {
      const float4 n = xv[i];
      reinterpret_cast<float4 *>(b)[c] =
          make_float4(__fmul_rn(__fmul_rn(n.x, inv), wv[i].x), __fmul_rn(__fmul_rn(n.y, inv), wv[i].y),
                      __fmul_rn(__fmul_rn(n.z, inv), wv[i].z), __fmul_rn(__fmul_rn(n.w, inv), wv[i].w));
    }
  }
  __syncwarp();
  if (kind == 2) {
    for (int64_t i = lane; i < a.dh; i += 32) yr[i] = b[i];
    return;
  }
  const float pos = (float)__ldg(a.positions + tok);
  for (int j = lane; j < a.half; j += 32) {
    const float ang = __fmul_rn(pos, fr.f[j]);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float x0 = b[j], x1 = b[j + a.half];
    yr[j] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    yr[j + a.half] = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x0, sn));
  }
  for (int64_t i = 2 * a.half + lane; i < a.dh; i += 32) yr[i] = b[i];
}

// ---- row argmax (greedy decoding over a vocab shard) ----------------------------
// Per row: the largest value and the first column holding it, with NaN above
// every number (numpy.argmax semantics) and -0 equal to +0. Each block folds a
// column range to one 64-bit key, (order-preserving value bits << 32) | ~column,
// so the atomic max over keys keeps the largest value and, among equal values,
// the smallest column.
__device__ __forceinline__ uint32_t argmax_order(float v) {
  if (v != v) return 0xFFFFFFFFu;  // NaN
  uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kArgThreads = 256;

__global__ void __launch_bounds__(kArgThreads) argmax_rows_kernel(const float *x, int64_t n, int64_t ldx, int cols_per_block,
                                                                  unsigned long long *keys) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t row = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * cols_per_block;
  const int64_t c1 = min(n, c0 + cols_per_block);
  const float *xr = x + row * ldx;
  unsigned long long best = 0ull;
  for (int64_t c = c0 + threadIdx.x; c < c1; c += kArgThreads) {  // ascending per thread
    const unsigned long long k = ((unsigned long long)argmax_order(xr[c]) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)c);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ unsigned long long wbest[kArgThreads / 32];
  if ((threadIdx.x & 31) == 0) wbest[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgThreads / 32; ++w) best = wbest[w] > best ? wbest[w] : best;
    atomicMax(keys + row, best);
  }
}

__global__ void argmax_finish_kernel(const float *x, int64_t m, int64_t ldx, int64_t idx_base,
                                     const unsigned long long *keys, float *val, int64_t *idx) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= m) return;
  const int64_t c = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[row] & 0xFFFFFFFFull));
  val[row] = x[row * ldx + c];
  idx[row] = idx_base + c;
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
  int sorted, identity, chunk, splits;
  uint32_t *err;
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

  int64_t j0, j1;
  if (a.identity) {
    // key j sits at position j: the visible range is arithmetic
    const int64_t hi = min(a.S, (int64_t)qpos + 1);
    const int64_t lo = (a.window > 0 && qpos >= a.window) ? (int64_t)(qpos - a.window) + 1 : 0;
    j0 = lo + (int64_t)blockIdx.x * a.chunk;
    j1 = min(hi, j0 + (int64_t)a.chunk);
  } else {
    if (tid == 0) {
      int64_t lo = 0, hi = a.S;
      if (a.sorted) {
        hi = upper_bound_pos(kp, a.S, qpos);
        if (a.window > 0 && qpos >= a.window) lo = upper_bound_pos(kp, hi, qpos - a.window);
      }
      const int64_t jj0 = lo + (int64_t)blockIdx.x * a.chunk;
      range[0] = jj0;
      range[1] = min(hi, jj0 + (int64_t)a.chunk);
    }
    __syncthreads();
    j0 = range[0];
    j1 = range[1];
  }
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
          const uint32_t kpos = a.identity ? (uint32_t)(j0 + jj) : kp[j0 + jj];
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

// Single-KV-head attention over contiguous cache rows (the decode layout): the
// CTA streams its key chunk through a ring of kRingStages shared-memory stages,
// each holding kSubKeys key rows and the matching value rows, filled by two 1-D
// bulk copies (TMA engine) that complete on the stage's mbarrier; softmax is
// online across sub-tiles (running max, sum and output rescaled per head).
// Thread t owns head_dim columns 4t .. 4t+3 for all G query heads, as above.
constexpr int kSubKeys = 8;

template <int NT, int kRingStages>
__global__ void __launch_bounds__(NT) attn_ring_kernel(const AttnArgs a) {
  static_assert(NT >= kMaxGroup * kKeyBatch, "one thread per (head, key) entry of a sub-tile");
  constexpr int NWARP = NT / 32;
  extern __shared__ __align__(128) uint8_t smem_dyn[];
  float *ring = reinterpret_cast<float *>(smem_dyn);  // [stage][K|V][kSubKeys][dh]
  __shared__ __align__(8) uint64_t full[kRingStages];
  __shared__ float sc[kSubKeys][kMaxGroup];
  __shared__ float red[NWARP][kKeyBatch * kMaxGroup];
  __shared__ float m_run[kMaxGroup], l_run[kMaxGroup], corr[kMaxGroup];
  __shared__ int abort_flag;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = (int)a.Hq;  // one KV head
  const int64_t bt = blockIdx.y;
  const int64_t b = bt / a.T;
  const int dh = (int)a.dh;
  const uint32_t stage_floats = (uint32_t)(2 * kSubKeys * dh);
  if (tid == 0) {
    for (int i = 0; i < kRingStages; ++i) gqd::mbar_init(&full[i], 1);
    gqd::fence_mbar_init();
    abort_flag = 0;
  }
  if (tid < kMaxGroup) {
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.0f;
  }
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const uint32_t qpos = a.q_pos[bt];
  int64_t lo = 0, hi = a.S;
  if (a.identity) {
    hi = min(a.S, (int64_t)qpos + 1);
    lo = (a.window > 0 && qpos >= a.window) ? (int64_t)(qpos - a.window) + 1 : 0;
  } else {
    const uint32_t *kpb = a.k_pos + b * a.kpos_batch_stride;
    hi = upper_bound_pos(kpb, a.S, qpos);
    if (a.window > 0 && qpos >= a.window) lo = upper_bound_pos(kpb, hi, qpos - a.window);
  }
  const int64_t j0 = lo + (int64_t)blockIdx.x * a.chunk;
  const int64_t j1 = min(hi, j0 + (int64_t)a.chunk);
  const int nkeys = j1 > j0 ? (int)(j1 - j0) : 0;
  const int ntiles = (nkeys + kSubKeys - 1) / kSubKeys;
  const float *kb = a.k + b * a.kv_batch_stride;
  const float *vb = a.v + b * a.kv_batch_stride;
  const uint32_t *kp = a.identity ? nullptr : a.k_pos + b * a.kpos_batch_stride;
  __syncthreads();

  auto issue = [&](int t) {  // sub-tile t into stage t % kRingStages
    const int st = t % kRingStages;
    const int rows = min(kSubKeys, nkeys - t * kSubKeys);
    const uint32_t bytes = (uint32_t)rows * (uint32_t)dh * 4u;
    float *dst = ring + (size_t)st * stage_floats;
    gqd::mbar_arrive_expect_tx(&full[st], 2u * bytes);
    gqd::bulk_g2s(dst, kb + (j0 + (int64_t)t * kSubKeys) * dh, bytes, &full[st]);
    gqd::bulk_g2s(dst + kSubKeys * dh, vb + (j0 + (int64_t)t * kSubKeys) * dh, bytes, &full[st]);
  };
  if (tid == 0)
    for (int t = 0; t < min(ntiles, kRingStages); ++t) issue(t);

  const int col = 4 * tid;
  const bool colv = col < dh;
  float4 q[kMaxGroup], o[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    q[g] = (g < G && colv) ? *reinterpret_cast<const float4 *>(a.q + bt * a.Hq * a.dh + g * a.dh + col)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  int issued = min(ntiles, kRingStages);
  for (int t = 0; t < ntiles; ++t) {
    const int st = t % kRingStages;
    const bool ok = gqd::mbar_wait_bounded(&full[st], (uint32_t)(t / kRingStages) & 1u);
    if (!ok) abort_flag = 1;
    __syncthreads();
    if (abort_flag) break;
    const float *kt = ring + (size_t)st * stage_floats;
    const float *vt = kt + kSubKeys * dh;
    const int rows = min(kSubKeys, nkeys - t * kSubKeys);
    // scores of the sub-tile
    float p[kMaxGroup * kKeyBatch];
    {
      float4 kv[kKeyBatch];
#pragma unroll
      for (int kk = 0; kk < kKeyBatch; ++kk)
        kv[kk] = (colv && kk < rows) ? *reinterpret_cast<const float4 *>(kt + kk * dh + col) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g)
#pragma unroll
        for (int kk = 0; kk < kKeyBatch; ++kk) {
          float v = __fmul_rn(q[g].x, kv[kk].x);
          v = __fmaf_rn(q[g].y, kv[kk].y, v);
          v = __fmaf_rn(q[g].z, kv[kk].z, v);
          v = __fmaf_rn(q[g].w, kv[kk].w, v);
          p[g * kKeyBatch + kk] = v;
        }
    }
#pragma unroll
    for (int off = 16, n = kMaxGroup * kKeyBatch; off >= 1; off >>= 1, n >>= 1) {
      const bool up = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = up ? p[i] : p[i + n / 2];
        const float keep = up ? p[i + n / 2] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
    red[warp][2 * lane] = p[0];
    red[warp][2 * lane + 1] = p[1];
    __syncthreads();
    // online softmax: thread e < 64 owns entry (head g, key kk); 8 lanes per head
    if (tid < kMaxGroup * kKeyBatch) {
      const int g = tid / kKeyBatch, kk = tid % kKeyBatch;
      float sum = 0.0f;
#pragma unroll
      for (int w2 = 0; w2 < NWARP; ++w2) sum += red[w2][tid];
      float sv = -INFINITY;
      if (g < G && kk < rows) {
        const int64_t j = j0 + (int64_t)t * kSubKeys + kk;
        const uint32_t kpos = a.identity ? (uint32_t)j : kp[j];
        sv = __fmul_rn(sum, a.scale);
        if (a.softcap > 0.0f) sv = __fmul_rn(a.softcap, tanhf(__fdiv_rn(sv, a.softcap)));
        if (kpos > qpos || (a.window > 0 && qpos - kpos >= a.window)) sv = -INFINITY;
      }
      float mt = sv;
#pragma unroll
      for (int off = 4; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mo = m_run[g];
      const float mn = fmaxf(mo, mt);
      const float e = (sv == -INFINITY) ? 0.0f : expf(__fsub_rn(sv, mn));
      float lt = e;
#pragma unroll
      for (int off = 4; off >= 1; off >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
      sc[kk][g] = e;
      if (kk == 0) {
        const float cf = (mo == -INFINITY) ? 0.0f : expf(__fsub_rn(mo, mn));
        corr[g] = cf;
        l_run[g] = __fmaf_rn(l_run[g], cf, lt);
        m_run[g] = mn;
      }
    }
    __syncthreads();
    // P.V of the sub-tile, after rescaling the running output
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      const float cf = corr[g];
      o[g] = make_float4(__fmul_rn(o[g].x, cf), __fmul_rn(o[g].y, cf), __fmul_rn(o[g].z, cf), __fmul_rn(o[g].w, cf));
    }
#pragma unroll
    for (int kk = 0; kk < kKeyBatch; ++kk) {
      if (kk >= rows) break;
      const float4 vv = colv ? *reinterpret_cast<const float4 *>(vt + kk * dh + col) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        const float pr = sc[kk][g];
        o[g].x = __fmaf_rn(pr, vv.x, o[g].x);
        o[g].y = __fmaf_rn(pr, vv.y, o[g].y);
        o[g].z = __fmaf_rn(pr, vv.z, o[g].z);
        o[g].w = __fmaf_rn(pr, vv.w, o[g].w);
      }
    }
    __syncthreads();  // stage t and sc are free
    if (tid == 0 && issued < ntiles) {
      gqd::fence_proxy_async_smem();
      issue(issued);
      ++issued;
    }
  }

  if (abort_flag) {
    // drain the copies still in flight (bounded) before the CTA's shared memory goes away
    if (tid == 0) {
      for (int t = max(0, issued - kRingStages); t < issued; ++t)
        (void)gqd::mbar_wait_bounded(&full[t % kRingStages], (uint32_t)(t / kRingStages) & 1u, 100000000ull);
      gqd::report(a.err, GQ_DEVERR_WAIT_TIMEOUT);
    }
    return;
  }
  if (!colv) return;
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g >= G) break;
    if (a.splits == 1) {
      const float inv = l_run[g] > 0.0f ? __fdiv_rn(1.0f, l_run[g]) : 0.0f;
      *reinterpret_cast<float4 *>(a.out + bt * a.Hq * a.dh + g * a.dh + col) =
          make_float4(__fmul_rn(o[g].x, inv), __fmul_rn(o[g].y, inv), __fmul_rn(o[g].z, inv), __fmul_rn(o[g].w, inv));
    } else {
      const int64_t prow = (bt * a.Hq + g) * a.splits + blockIdx.x;
      *reinterpret_cast<float4 *>(a.part_o + prow * a.dh + col) = o[g];
      if (tid == 0) {
        a.part_ml[2 * prow] = m_run[g];
        a.part_ml[2 * prow + 1] = l_run[g];
      }
    }
  }
}

// Merge the chunks of one (token, head) row: out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s.
// Grid: x = (token, head) row, y = slice of 128 output columns. Block: 32 column
// threads (4 columns each) x 8 groups that split the chunks; the chunk weights are
// computed once in shared memory, the 8 group sums are added through shared memory.
constexpr int kMaxSplits = 256;
constexpr int kCombGroups = 8;
__global__ void __launch_bounds__(256) attn_combine_kernel(const float *part_o, const float *part_ml, int64_t rows,
                                                           int64_t Hq, int64_t dh, int splits, float *out) {
  __shared__ float wgt[kMaxSplits];
  __shared__ float wred[8], lred[8];
  __shared__ float4 acc_s[kCombGroups][32];
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t row = blockIdx.x;  // (token, head)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float *ml = part_ml + row * splits * 2;
  float m = -INFINITY, l = 0.0f;
  for (int s2 = tid; s2 < splits; s2 += blockDim.x) m = fmaxf(m, ml[2 * s2]);
  m = warp_max(m);
  if (lane == 0) wred[warp] = m;
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) M = fmaxf(M, wred[i]);
  for (int s2 = tid; s2 < splits; s2 += blockDim.x) {
    const float ms = ml[2 * s2];
    const float w = (ms == -INFINITY) ? 0.0f : expf(__fsub_rn(ms, M));
    wgt[s2] = w;
    l += __fmul_rn(w, ml[2 * s2 + 1]);
  }
  l = warp_sum(l);
  if (lane == 0) lred[warp] = l;
  __syncthreads();
  float L = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) L += lred[i];
  const float inv = L > 0.0f ? __fdiv_rn(1.0f, L) : 0.0f;
  const int64_t c = (int64_t)blockIdx.y * 128 + 4 * lane;  // this thread's 4 columns
  const int grp = warp;                                    // chunks grp, grp + 8, ...
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c < dh) {
    const float *po = part_o + row * splits * dh + c;
#pragma unroll 4
    for (int s2 = grp; s2 < splits; s2 += kCombGroups) {
      const float w = wgt[s2];
      const float4 v = *reinterpret_cast<const float4 *>(po + (int64_t)s2 * dh);
      acc.x = __fmaf_rn(w, v.x, acc.x);
      acc.y = __fmaf_rn(w, v.y, acc.y);
      acc.z = __fmaf_rn(w, v.z, acc.z);
      acc.w = __fmaf_rn(w, v.w, acc.w);
    }
  }
  acc_s[grp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < dh) {
    float4 t = acc_s[0][lane];
#pragma unroll
    for (int g2 = 1; g2 < kCombGroups; ++g2) {
      const float4 u = acc_s[g2][lane];
      t.x = __fadd_rn(t.x, u.x);
      t.y = __fadd_rn(t.y, u.y);
      t.z = __fadd_rn(t.z, u.z);
      t.w = __fadd_rn(t.w, u.w);
    }
    const int64_t bt = row / Hq, h = row % Hq;
    *reinterpret_cast<float4 *>(out + bt * Hq * dh + h * dh + c) =
        make_float4(__fmul_rn(t.x, inv), __fmul_rn(t.y, inv), __fmul_rn(t.z, inv), __fmul_rn(t.w, inv));
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

// M > 4 rows: a 64 (weight rows) x 64 (activation rows) output tile per CTA,
// K in chunks of 32 staged through shared memory (weights widened from bf16
// once per chunk and shared by all 64 activation rows), 4 x 4 outputs per thread.
constexpr int kLbT = 64, kLbK = 32;
__global__ void __launch_bounds__(256) linear_bf16_tiled_kernel(const float *x, int64_t m, int64_t k,
                                                                const uint16_t *w, int64_t n, float *y) {
  __shared__ float ws[kLbK][kLbT + 4];
  __shared__ float xs[kLbK][kLbT + 4];
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t n0 = (int64_t)blockIdx.x * kLbT, m0 = (int64_t)blockIdx.y * kLbT;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  const int lr = tid >> 2, lk = (tid & 3) * 8;  // loader: row lr, 8 columns from lk
  for (int64_t k0 = 0; k0 < k; k0 += kLbK) {
    {
      const int64_t nn = n0 + lr, kk = k0 + lk;
      float wv[8];
      if (nn < n && kk + 8 <= k) {
        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(w + nn * k + kk));
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          wv[2 * i] = bf16lo(q[i]);
          wv[2 * i + 1] = bf16hi(q[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          wv[i] = (nn < n && kk + i < k) ? __uint_as_float((uint32_t)w[nn * k + kk + i] << 16) : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ws[lk + i][lr] = wv[i];
      const int64_t mm = m0 + lr;
      float xv[8];
      if (mm < m && kk + 8 <= k) {
        const float4 a0 = __ldg(reinterpret_cast<const float4 *>(x + mm * k + kk));
        const float4 a1 = __ldg(reinterpret_cast<const float4 *>(x + mm * k + kk + 4));
        xv[0] = a0.x; xv[1] = a0.y; xv[2] = a0.z; xv[3] = a0.w;
        xv[4] = a1.x; xv[5] = a1.y; xv[6] = a1.z; xv[7] = a1.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[i] = (mm < m && kk + i < k) ? x[mm * k + kk + i] : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) xs[lk + i][lr] = xv[i];
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kLbK; ++kk) {
      const float4 a = *reinterpret_cast<const float4 *>(&ws[kk][4 * tx]);
      const float4 b = *reinterpret_cast<const float4 *>(&xs[kk][4 * ty]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(bv[j], av[i], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t mm = m0 + 4 * ty + j;
    if (mm >= m) continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t nn = n0 + 4 * tx + i;
      if (nn < n) y[mm * n + nn] = acc[i][j];
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

template <int KIND>
cudaError_t norm_reg_launch(gq_ctx *ctx, int vpl, dim3 grid, const float *x, const float *r, const float *w,
                            const float *s, int64_t rows, int64_t d, float eps, float *y, RowMap ym) {
  const dim3 blk(kNormThreads);
  switch (vpl) {
    case 1: return gq_launch(ctx, rmsnorm_reg_kernel<KIND, 1>, grid, blk, 0, x, r, w, s, rows, d, eps, y, ym);
    case 2: return gq_launch(ctx, rmsnorm_reg_kernel<KIND, 2>, grid, blk, 0, x, r, w, s, rows, d, eps, y, ym);
    case 4: return gq_launch(ctx, rmsnorm_reg_kernel<KIND, 4>, grid, blk, 0, x, r, w, s, rows, d, eps, y, ym);
    case 8: return gq_launch(ctx, rmsnorm_reg_kernel<KIND, 8>, grid, blk, 0, x, r, w, s, rows, d, eps, y, ym);
    case 12: return gq_launch(ctx, rmsnorm_reg_kernel<KIND, 12>, grid, blk, 0, x, r, w, s, rows, d, eps, y, ym);
    default: return gq_launch(ctx, rmsnorm_reg_kernel<KIND, 16>, grid, blk, 0, x, r, w, s, rows, d, eps, y, ym);
  }
}

// float4 per lane for a register-resident row of d values (0: use the strided kernel)
int reg_vpl(int64_t d) {
  const int64_t need = (d + 127) / 128;
  for (int v : {1, 2, 4, 8, 12, 16})
    if (need <= v) return v;
  return 0;
}

int norm_launch(gq_ctx *ctx, int kind, const float *x, const float *r, const float *w, const float *s, int64_t rows,
                int64_t d, float eps, float *y, RowMap ym) {
  const dim3 grid((unsigned)((rows + kNormThreads / 32 - 1) / (kNormThreads / 32)));
  const int vpl = reg_vpl(d);
  const bool aligned = d % 4 == 0 && ((uintptr_t)x | (uintptr_t)y | (uintptr_t)w | (uintptr_t)r) % 16 == 0 &&
                       (ym.group_stride % 4 == 0) && (ym.inner_stride % 4 == 0);
  if (vpl && aligned) {
    if (kind == 0)
      GQ_CUDA_TRY(ctx, norm_reg_launch<0>(ctx, vpl, grid, x, r, w, s, rows, d, eps, y, ym));
    else
      GQ_CUDA_TRY(ctx, norm_reg_launch<1>(ctx, vpl, grid, x, r, w, s, rows, d, eps, y, ym));
    return GQ_OK;
  }
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
  const int vpl = reg_vpl(dh);
  const bool aligned = dh % 4 == 0 && ((uintptr_t)x % 16 == 0) && (!norm || (uintptr_t)w % 16 == 0);
  if (aligned && vpl && vpl <= 4) {
    cudaError_t e;
    const dim3 blk(kNormThreads);
    if (norm) {
      e = vpl == 1 ? gq_launch(ctx, head_rope_reg_kernel<true, 1>, grid, blk, 0, x, w, rows, heads, dh, eps, positions, half, fr, y, ym)
        : vpl == 2 ? gq_launch(ctx, head_rope_reg_kernel<true, 2>, grid, blk, 0, x, w, rows, heads, dh, eps, positions, half, fr, y, ym)
                   : gq_launch(ctx, head_rope_reg_kernel<true, 4>, grid, blk, 0, x, w, rows, heads, dh, eps, positions, half, fr, y, ym);
    } else {
      e = vpl == 1 ? gq_launch(ctx, head_rope_reg_kernel<false, 1>, grid, blk, 0, x, w, rows, heads, dh, eps, positions, half, fr, y, ym)
        : vpl == 2 ? gq_launch(ctx, head_rope_reg_kernel<false, 2>, grid, blk, 0, x, w, rows, heads, dh, eps, positions, half, fr, y, ym)
                   : gq_launch(ctx, head_rope_reg_kernel<false, 4>, grid, blk, 0, x, w, rows, heads, dh, eps, positions, half, fr, y, ym);
    }
    GQ_CUDA_TRY(ctx, e);
    return GQ_OK;
  }
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

// Ring depth: three stages (96 KB at head_dim 512, two CTAs per SM). Measured on
// batch 64: two stages (three CTAs per SM) gave the same at head_dim 512, four
// stages lost 25 % at head_dim 256.
template <int NT>
constexpr int ring_stages() { return 3; }

template <int NT>
cudaError_t attn_ring_launch_nt(gq_ctx *ctx, dim3 grid, const AttnArgs &a) {
  constexpr int ST = ring_stages<NT>();
  const size_t smem = (size_t)2 * ST * kSubKeys * a.dh * 4;
  static bool attr_set[64] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_ring_kernel<NT, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(2 * ST * kSubKeys * 4 * NT * 4));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return gq_launch(ctx, attn_ring_kernel<NT, ST>, grid, dim3(NT), smem, a);
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

int gq_add_rms_norm_norm(gq_ctx *ctx, const float *residual, const float *x, int64_t rows, int64_t d, const float *w1,
                         float eps, const float *scale_by, const float *w2, float *h, float *xn) {
  ENTER(ctx);
  if (rows < 0 || d <= 0 || !x || !residual || !w1 || !w2 || !h || !xn)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "add_rms_norm_norm: bad shape or null pointer");
  if (rows == 0) return GQ_OK;
  const int vpl = reg_vpl(d);
  const bool aligned = d % 4 == 0 && ((uintptr_t)x | (uintptr_t)residual | (uintptr_t)w1 | (uintptr_t)w2 |
                                      (uintptr_t)h | (uintptr_t)xn) % 16 == 0;
  if (!vpl || vpl > 12 || !aligned) {  // the two calls it fuses
    int rc = norm_launch(ctx, 1, x, residual, w1, scale_by, rows, d, eps, h, RowMap{1, d, 0});
    if (rc != GQ_OK) return rc;
    return norm_launch(ctx, 0, h, nullptr, w2, nullptr, rows, d, eps, xn, RowMap{1, d, 0});
  }
  const dim3 grid((unsigned)((rows + kNormThreads / 32 - 1) / (kNormThreads / 32))), blk(kNormThreads);
  cudaError_t e;
  switch (vpl) {
    case 1: e = gq_launch(ctx, add_norm_norm_kernel<1>, grid, blk, 0, x, residual, w1, scale_by, w2, rows, d, eps, h, xn); break;
    case 2: e = gq_launch(ctx, add_norm_norm_kernel<2>, grid, blk, 0, x, residual, w1, scale_by, w2, rows, d, eps, h, xn); break;
    case 4: e = gq_launch(ctx, add_norm_norm_kernel<4>, grid, blk, 0, x, residual, w1, scale_by, w2, rows, d, eps, h, xn); break;
    case 8: e = gq_launch(ctx, add_norm_norm_kernel<8>, grid, blk, 0, x, residual, w1, scale_by, w2, rows, d, eps, h, xn); break;
    case 12: e = gq_launch(ctx, add_norm_norm_kernel<12>, grid, blk, 0, x, residual, w1, scale_by, w2, rows, d, eps, h, xn); break;
    default: e = gq_launch(ctx, add_norm_norm_kernel<12>, grid, blk, 0, x, residual, w1, scale_by, w2, rows, d, eps, h, xn); break;
  }
  GQ_CUDA_TRY(ctx, e);
  return GQ_OK;
}

int gq_head_norm_rope(gq_ctx *ctx, const float *x, int64_t t, int64_t heads, int64_t head_dim, const float *w,
                      float eps, const uint32_t *positions, float theta, int64_t rotary_dim, float *y,
                      int64_t y_tok_stride) {
  ENTER(ctx);
  if (y_tok_stride == 0) y_tok_stride = heads * head_dim;
  return rope_launch(ctx, true, x, w, t, heads, head_dim, eps, positions, theta, rotary_dim, y, y_tok_stride);
}

int gq_qkv_norm_rope(gq_ctx *ctx, const float *qkv, int64_t t, int64_t qkv_tok_stride, int64_t hq, int64_t hkv,
                     int64_t head_dim, const float *q_w, const float *k_w, float eps, const uint32_t *positions,
                     float theta, int64_t rotary_dim, float *q_out, int64_t q_tok_stride, float *k_out,
                     int64_t k_tok_stride, float *v_out, int64_t v_tok_stride) {
  ENTER(ctx);
  const int64_t dh = head_dim, rot = rotary_dim;
  if (t < 0 || hq <= 0 || hkv <= 0 || dh <= 0 || rot < 0 || rot > dh || rot % 2 != 0)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qkv_norm_rope: bad shape (rotary_dim even, <= head_dim)");
  if (!qkv || !q_w || !k_w || !q_out || !k_out || !v_out || (t > 0 && !positions))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qkv_norm_rope: null pointer");
  if (qkv_tok_stride == 0) qkv_tok_stride = (hq + 2 * hkv) * dh;
  if (q_tok_stride == 0) q_tok_stride = hq * dh;
  if (k_tok_stride == 0) k_tok_stride = hkv * dh;
  if (v_tok_stride == 0) v_tok_stride = hkv * dh;
  if (qkv_tok_stride < (hq + 2 * hkv) * dh || q_tok_stride < hq * dh || k_tok_stride < hkv * dh ||
      v_tok_stride < hkv * dh)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qkv_norm_rope: token stride too small");
  const int vpl = reg_vpl(dh);
  if (dh % 4 != 0 || qkv_tok_stride % 4 != 0 || (uintptr_t)qkv % 16 || (uintptr_t)q_w % 16 || (uintptr_t)k_w % 16 ||
      !vpl || vpl > 4)
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED,
                   "qkv_norm_rope: head_dim a multiple of 4 up to 512, 16-byte aligned rows and weights");
  if (rot / 2 > kMaxHalfRot) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "qkv_norm_rope: rotary_dim > 512");
  if (t == 0) return GQ_OK;
  RopeFreq fr;
  const int half = (int)(rot / 2);
  // the reference's frequency, same f32 expression as rope_launch (rust/src/backend_cpu.rs:258)
  for (int j = 0; j < half; ++j) fr.f[j] = powf(theta, -(2.0f * (float)j) / (float)rot);
  QkvArgs a{qkv, t, qkv_tok_stride, (int)hq, (int)hkv, dh, q_w, k_w, eps, positions, half,
            q_out, k_out, v_out, q_tok_stride, k_tok_stride, v_tok_stride};
  const int64_t rows = t * (hq + 2 * hkv);
  const dim3 grid((unsigned)((rows + kNormThreads / 32 - 1) / (kNormThreads / 32))), blk(kNormThreads);
  cudaError_t e = vpl == 1 ? gq_launch(ctx, qkv_norm_rope_kernel<1>, grid, blk, 0, a, fr)
                : vpl == 2 ? gq_launch(ctx, qkv_norm_rope_kernel<2>, grid, blk, 0, a, fr)
                           : gq_launch(ctx, qkv_norm_rope_kernel<4>, grid, blk, 0, a, fr);
  GQ_CUDA_TRY(ctx, e);
  return GQ_OK;
}

int gq_argmax_rows(gq_ctx *ctx, const float *x, int64_t m, int64_t n, int64_t ldx, int64_t idx_base, float *val,
                   int64_t *idx) {
  ENTER(ctx);
  if (m < 0 || n <= 0 || n > 0xFFFFFFFFll || (m > 0 && (!x || !val || !idx)))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "argmax_rows: bad shape or null pointer");
  if (ldx == 0) ldx = n;
  if (ldx < n) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "argmax_rows: ldx < n");
  if (m == 0) return GQ_OK;
  void *ws = nullptr;
  int rc = gq_workspace(ctx, (size_t)m * 8, &ws);
  if (rc != GQ_OK) return rc;
  unsigned long long *keys = static_cast<unsigned long long *>(ws);
  GQ_CUDA_TRY(ctx, cudaMemsetAsync(keys, 0, (size_t)m * 8, ctx->stream));
  // about two blocks per SM in all, at least 4096 columns per block
  int64_t blocks = std::max<int64_t>(1, (2 * (int64_t)ctx->num_sms + m - 1) / m);
  int64_t per = std::max<int64_t>(4096, (n + blocks - 1) / blocks);
  blocks = (n + per - 1) / per;
  GQ_CUDA_TRY(ctx, gq_launch(ctx, argmax_rows_kernel, dim3((unsigned)blocks, (unsigned)m), dim3(kArgThreads), 0, x, n,
                             ldx, (int)per, keys));
  GQ_CUDA_TRY(ctx, gq_launch(ctx, argmax_finish_kernel, dim3((unsigned)((m + 127) / 128)), dim3(128), 0, x, m, ldx,
                             idx_base, (const unsigned long long *)keys, val, idx));
  return GQ_OK;
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
  if (!q || !out || !q_pos || (s > 0 && (!k || !v || (!k_pos && !(flags & GQ_ATTN_KPOS_IDENTITY)))))
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
  a.identity = (flags & GQ_ATTN_KPOS_IDENTITY) ? 1 : 0;
  a.sorted = (a.identity || (flags & GQ_ATTN_KPOS_ASCENDING)) ? 1 : 0;
  // keys a query can reach: the window bounds the range when positions ascend
  a.err = ctx->dev_err;
  const int64_t active = (a.sorted && sliding_window > 0) ? std::min<int64_t>(s, sliding_window) : s;
  const int64_t rows = batch * t * hkv;
  if (rows > 65535) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "attention: more than 65535 (token, kv head) rows");
  // One KV head with its rows contiguous (kv row stride == head_dim): stream key
  // chunks through the shared-memory ring; chunks sized for ~4 CTAs per SM.
  const bool ring = hkv == 1 && a.sorted && head_dim <= 512;
  int chunk;
  if (ring) {
    const int64_t target = 4 * (int64_t)ctx->num_sms;
    int64_t per = (rows * active + target - 1) / target;  // keys per CTA for `target` CTAs
    per = std::max<int64_t>(32, (per + kSubKeys - 1) / kSubKeys * kSubKeys);
    per = std::max<int64_t>(per, (active + kMaxSplits - 1) / kMaxSplits);
    chunk = (int)std::min<int64_t>(per, 1 << 30);
  } else {
    chunk = 32;
    while (chunk < kMaxChunk && rows * ((active + chunk - 1) / chunk) > 4 * (int64_t)ctx->num_sms * 4) chunk *= 2;
    if ((active + chunk - 1) / chunk > kMaxSplits)
      return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "attention: key range too long for the generic kernel");
  }
  a.chunk = chunk;
  a.splits = (int)std::max<int64_t>(1, (active + chunk - 1) / chunk);
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
  if (ring) {
    // at least two warps: the softmax step gives one thread to each of the 64 (head, key) entries
    if (head_dim <= 256)
      e = attn_ring_launch_nt<64>(ctx, grid, a);
    else
      e = attn_ring_launch_nt<128>(ctx, grid, a);
  } else switch (nt) {
    case 32: e = attn_launch_nt<32>(ctx, grid, a); break;
    case 64: e = attn_launch_nt<64>(ctx, grid, a); break;
    case 128: e = attn_launch_nt<128>(ctx, grid, a); break;
    default: e = attn_launch_nt<256>(ctx, grid, a); break;
  }
  GQ_CUDA_TRY(ctx, e);
  if (a.splits > 1) {
    const dim3 cgrid((unsigned)(batch * t * hq), (unsigned)((head_dim + 127) / 128));
    GQ_CUDA_TRY(ctx, gq_launch(ctx, attn_combine_kernel, cgrid, dim3(256), 0, a.part_o, a.part_ml, batch * t * hq, hq,
                               head_dim, a.splits, out));
  }
  return GQ_OK;
}

int gq_linear_bf16(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const uint16_t *w, int64_t n, float *y) {
  ENTER(ctx);
  if (m < 0 || k < 0 || n < 0) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_bf16: bad shape");
  if (m == 0 || n == 0) return GQ_OK;
  if (!x || !w || !y) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_bf16: null pointer");
  const bool vec = k % 8 == 0 && k > 0 && (uintptr_t)x % 16 == 0 && (uintptr_t)w % 16 == 0;
  if (vec && m > 4) {
    const dim3 grid((unsigned)((n + kLbT - 1) / kLbT), (unsigned)((m + kLbT - 1) / kLbT));
    GQ_CUDA_TRY(ctx, gq_launch(ctx, linear_bf16_tiled_kernel, grid, dim3(256), 0, x, m, k, w, n, y));
  } else if (vec) {
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
