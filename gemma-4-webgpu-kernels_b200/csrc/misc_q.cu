// misc_q.cu — the generic MATMUL_Q_SCALAR path, per-row code sums, EMBED_Q and
// the elementwise ops the fused fallbacks compose with.
#include <cuda_runtime.h>
#include <math.h>

#include <type_traits>

#include <algorithm>

#include "gq_internal.cuh"

namespace {

constexpr int64_t kEmbedWarpsPerSm = 16;  // embed_row_kernel: row splitting stops above this

// Integer code of element [n, k]: rust/src/backend.rs:46-54 (offset binary for
// sub-byte and unsigned 8-bit payloads, two's complement for I8).
__device__ __forceinline__ int32_t code_at(const uint8_t *bytes, int64_t row_bytes, int bits,
                                           int signed_i8, int64_t n, int64_t k) {
  if (signed_i8) return (int32_t)(int8_t)bytes[n * row_bytes + k];
  const int per_byte = 8 / bits;
  const uint32_t b = bytes[n * row_bytes + k / per_byte];
  const uint32_t shift = (uint32_t)(k % per_byte) * (uint32_t)bits;
  return (int32_t)((b >> shift) & ((1u << bits) - 1u)) - (1 << (bits - 1));
}

struct QView {
  const uint8_t *bytes;
  const float *scales;
  int64_t n, k, row_bytes, scale_stride, group;
  int bits, signed_i8;
};

__device__ __forceinline__ float deq_at(const QView &q, int64_t n, int64_t k) {
  return __fmul_rn((float)code_at(q.bytes, q.row_bytes, q.bits, q.signed_i8, n, k),
                   q.scales[n * q.scale_stride + k / q.group]);
}

// MATMUL_Q_SCALAR semantics (rust/src/kernels/matmul_q_scalar.wgsl:1-35) with the
// CPU backend's exact operation order (rust/src/backend_cpu.rs:189-208): one
// thread per output, acc += x * (q * s), k ascending, no contraction. Handles
// any K, bit width, signedness and scale group. Used where the streaming GEMV
// does not apply (odd K, grouped scales).
__global__ void scalar_linear_kernel(const float *x, int64_t m_rows, QView q, float *y) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t total = m_rows * q.n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / q.n, n = i % q.n;
    const float *xr = x + m * q.k;
    float acc = 0.0f;
    for (int64_t k = 0; k < q.k; ++k) acc = __fadd_rn(acc, __fmul_rn(xr[k], deq_at(q, n, k)));
    y[m * q.n + n] = acc;
  }
}

// sum_k q[n, k] per row as f32 (exact: |sum| < 2^24 for K < 131072). Stored
// after the scales; the streaming GEMV's epilogue uses it.
__global__ void qsum_kernel(QView q, float *out) {
  const int64_t n = blockIdx.x * (int64_t)(blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= q.n) return;
  int64_t s = 0;
  for (int64_t k = lane; k < q.k; k += 32) s += code_at(q.bytes, q.row_bytes, q.bits, q.signed_i8, n, k);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[n] = (float)s;
}

// EMBED_Q: out[i, d] = (q(ids[i], d) * scale[ids[i]*ss + d/group]) * emb_scale,
// the operation order of rust/src/backend_cpu.rs:133 (deq, then * scale), so the
// result is bit-identical to the CPU reference. One thread per 4 consecutive
// values of an output row: a warp reads 32/64/128 contiguous packed bytes and
// writes 512 contiguous output bytes. Requires D % 4 == 0; an id >= rows zeroes
// the row and raises GQ_DEVERR_BAD_ID.
__global__ void embed_quad_kernel(QView q, const uint32_t *ids, int64_t t, float emb,
                                  float *out, uint32_t *err) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t quads_per_row = q.k >> 2;
  const int64_t total = t * quads_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / quads_per_row;
    const int64_t d0 = (i - row * quads_per_row) << 2;
    const uint32_t id = __ldg(ids + row);
    float4 v;
    if ((int64_t)id >= q.n) {
      v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (d0 == 0) gqd::report(err, GQ_DEVERR_BAD_ID);
    } else {
      const uint8_t *rp = q.bytes + (int64_t)id * q.row_bytes;
      int32_t c[4];
      if (q.signed_i8 || q.bits == 8) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(rp + d0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t b = (w >> (8 * j)) & 0xffu;
          c[j] = q.signed_i8 ? (int32_t)(int8_t)b : (int32_t)b - 128;
        }
      } else if (q.bits == 4) {
        const uint32_t w = *reinterpret_cast<const uint16_t *>(rp + (d0 >> 1));
#pragma unroll
        for (int j = 0; j < 4; ++j) c[j] = (int32_t)((w >> (4 * j)) & 0xfu) - 8;
      } else {
        const uint32_t w = rp[d0 >> 2];
#pragma unroll
        for (int j = 0; j < 4; ++j) c[j] = (int32_t)((w >> (2 * j)) & 0x3u) - 2;
      }
      const float *sr = q.scales + (int64_t)id * q.scale_stride;
      float r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        r[j] = __fmul_rn(__fmul_rn((float)c[j], __ldg(sr + (d0 + j) / q.group)), emb);
      v = make_float4(r[0], r[1], r[2], r[3]);
    }
    *reinterpret_cast<float4 *>(out + row * q.k + d0) = v;
  }
}

// EMBED_Q, one warp per output row (the row's id, packed row and scale row are
// looked up once). Lane l owns the four outputs 4l..4l+3 of every 128-column step,
// so each warp store writes 512 contiguous bytes (the output is 80 % of the bytes
// moved: a 16-byte store per lane at a 64-byte lane stride, as an earlier version
// did, spreads one store instruction over 32 sectors of 16 lines). The four codes
// of a lane are one 4-, 2- or 1-byte load (I8 / 4-bit / 2-bit), all U steps' loads
// are issued before the first store, and the stores stream past L2 (st.global.cs:
// an embedding row is not read again by this kernel). Arithmetic order
// (q * s) * emb as embed_quad_kernel and the CPU (bit-identical).
// Requires D % 4 == 0, group == D or a power of two >= 4, 16-byte aligned output
// rows, and packed rows aligned to one lane's load.
// A row may be split over wpr warps (contiguous ranges of spw 128-column steps), so
// that few rows (a decode step's one token, or 4096 rows on 148 SMs) still put
// enough warps and bytes in flight on every SM.
template <int BITS, bool SIGNED>
__global__ void __launch_bounds__(256) embed_row_kernel(QView q, const uint32_t *ids, int64_t t, float emb,
                                                        float *out, uint32_t *err, int wpr, int spw) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t row = gw / wpr;
  if (row >= t) return;
  const int part = (int)(gw - row * wpr);
  const uint32_t id = __ldg(ids + row);
  float *orow = out + row * q.k;
  const int64_t D = q.k;
  const int64_t cbeg = (int64_t)part * spw * 128, cend = min(D, cbeg + (int64_t)spw * 128);
  if ((int64_t)id >= q.n) {
    for (int64_t c = cbeg + 4 * lane; c < cend; c += 128)
      __stcs(reinterpret_cast<float4 *>(orow + c), make_float4(0.f, 0.f, 0.f, 0.f));
    if (lane == 0 && part == 0) gqd::report(err, GQ_DEVERR_BAD_ID);
    return;
  }
  const uint8_t *rp = q.bytes + (int64_t)id * q.row_bytes;
  const float *sr = q.scales + (int64_t)id * q.scale_stride;
  const int gshift = (q.group == q.k) ? 63 : (31 - __clz((int)q.group));  // group is a power of two here
  // 128-column steps per lane in flight: all loads first, then the stores. Config 4
  // (4096 rows of the PLE and token tables) measured 4620 / 4910 / 4890 / 3840 GB/s
  // at U = 8 / 16 / 24 / 32.
  constexpr int U = 16;
  for (int64_t c0 = cbeg + 4 * lane; c0 < cend; c0 += 128 * U) {
    uint32_t w[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = c0 + 128 * u;
      w[u] = 0;
      if (c < cend) {
        if constexpr (BITS == 8) w[u] = __ldg(reinterpret_cast<const uint32_t *>(rp + c));
        else if constexpr (BITS == 4) w[u] = __ldg(reinterpret_cast<const uint16_t *>(rp + (c >> 1)));
        else w[u] = __ldg(rp + (c >> 2));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = c0 + 128 * u;
      if (c >= cend) break;
      int32_t cd[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t b = (w[u] >> (BITS * i)) & ((1u << BITS) - 1u);
        if constexpr (BITS == 8) cd[i] = SIGNED ? (int32_t)(int8_t)b : (int32_t)b - 128;
        else cd[i] = (int32_t)b - (1 << (BITS - 1));
      }
      const float sc = __ldg(sr + (gshift == 63 ? 0 : (c >> gshift)));
      __stcs(reinterpret_cast<float4 *>(orow + c),
             make_float4(__fmul_rn(__fmul_rn((float)cd[0], sc), emb), __fmul_rn(__fmul_rn((float)cd[1], sc), emb),
                         __fmul_rn(__fmul_rn((float)cd[2], sc), emb), __fmul_rn(__fmul_rn((float)cd[3], sc), emb)));
    }
  }
}

// EMBED_Q for any D: one thread per output element.
__global__ void embed_scalar_kernel(QView q, const uint32_t *ids, int64_t t, float emb,
                                    float *out, uint32_t *err) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int64_t total = t * q.k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / q.k, d = i % q.k;
    const uint32_t id = ids[row];
    float v = 0.0f;
    if ((int64_t)id >= q.n) {
      if (d == 0) gqd::report(err, GQ_DEVERR_BAD_ID);
    } else {
      v = __fmul_rn(deq_at(q, id, d), emb);
    }
    out[i] = v;
  }
}

// op 0: softcap  y = cap * tanh(a / cap)          (rust/src/backend_cpu.rs:242-244)
// op 1: geglu    y = gelu(a) * b                  (rust/src/backend_cpu.rs:239-241)
// op 2: gelu * column slice: y[m, n] = gelu(a[m, n]) * b[m*stride + off + n]
__global__ void elementwise_kernel(int op, const float *a, const float *b, int64_t count,
                                   int64_t ncols, int64_t b_stride, int64_t b_off, float cap,
                                   float *y) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = a[i];
    float r;
    if (op == 0) {
      r = __fmul_rn(cap, tanhf(__fdiv_rn(v, cap)));
    } else if (op == 1) {
      r = __fmul_rn(gqd::gelu_tanh(v), b[i]);
    } else {
      const int64_t m = i / ncols, n = i % ncols;
      r = __fmul_rn(gqd::gelu_tanh(v), b[m * b_stride + b_off + n]);
    }
    y[i] = r;
  }
}

QView view_of(const gq_qweight *w) {
  QView q;
  q.bytes = w->bytes;
  q.scales = w->scales;
  q.n = w->n;
  q.k = w->k;
  q.row_bytes = w->row_bytes;
  q.scale_stride = w->scale_stride;
  q.group = w->group_size;
  q.bits = w->bits;
  q.signed_i8 = w->signed_i8;
  return q;
}

unsigned grid_for(gq_ctx *ctx, int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)ctx->num_sms * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

}  // namespace

int gq_scalar_linear_launch(gq_ctx *ctx, const float *x, int64_t m, const gq_qweight *w,
                            float *y) {
  const int64_t total = m * w->n;
  if (total == 0) return GQ_OK;
  GQ_CUDA_TRY(ctx, gq_launch(ctx, scalar_linear_kernel, dim3(grid_for(ctx, total, 128)), dim3(128), 0,
                             x, m, view_of(w), y));
  return GQ_OK;
}

int gq_qsum_launch(gq_ctx *ctx, const gq_qweight *w, float *out) {
  if (w->n == 0) return GQ_OK;
  const int rows_per_block = 8;
  const unsigned g = (unsigned)((w->n + rows_per_block - 1) / rows_per_block);
  qsum_kernel<<<g, rows_per_block * 32, 0, ctx->stream>>>(view_of(w), out);
  GQ_CUDA_TRY(ctx, cudaGetLastError());
  return GQ_OK;
}

int gq_embed_launch(gq_ctx *ctx, const gq_qweight *w, const uint32_t *ids, int64_t t, float emb,
                    float *out) {
  if (t == 0 || w->k == 0) return GQ_OK;
  const QView q = view_of(w);
  const int64_t g = w->group_size;
  const bool row_path = w->k % 4 == 0 && ((uintptr_t)out % 16 == 0) && (g == w->k || (g >= 4 && (g & (g - 1)) == 0)) &&
                        (uintptr_t)w->bytes % 4 == 0 && w->row_bytes % (w->signed_i8 || w->bits == 8 ? 4 : (w->bits == 4 ? 2 : 1)) == 0 &&
                        t <= (int64_t)0x7fffffff;
  if (row_path) {
    // warps per row: split a row only when the rows alone give fewer than ~16 warps
    // per SM (each warp keeps U = 8 steps of loads in flight; at 4096 rows of the
    // PLE table a second warp per row measured slower), each part keeping at
    // least two 128-column steps
    const int64_t steps = (w->k + 127) / 128;
    int64_t wpr = ((int64_t)ctx->num_sms * kEmbedWarpsPerSm + t - 1) / t;
    wpr = std::max<int64_t>(1, std::min<int64_t>(wpr, (steps + 1) / 2));
    const int spw = (int)((steps + wpr - 1) / wpr);
    wpr = (steps + spw - 1) / spw;  // no empty part
    const unsigned blocks = (unsigned)((t * wpr + 7) / 8);
    const int iw = (int)wpr;
    if (w->signed_i8)
      GQ_CUDA_TRY(ctx, gq_launch(ctx, embed_row_kernel<8, true>, dim3(blocks), dim3(256), 0, q, ids, t, emb, out,
                                 ctx->dev_err, iw, spw));
    else if (w->bits == 8)
      GQ_CUDA_TRY(ctx, gq_launch(ctx, embed_row_kernel<8, false>, dim3(blocks), dim3(256), 0, q, ids, t, emb, out,
                                 ctx->dev_err, iw, spw));
    else if (w->bits == 4)
      GQ_CUDA_TRY(ctx, gq_launch(ctx, embed_row_kernel<4, false>, dim3(blocks), dim3(256), 0, q, ids, t, emb, out,
                                 ctx->dev_err, iw, spw));
    else
      GQ_CUDA_TRY(ctx, gq_launch(ctx, embed_row_kernel<2, false>, dim3(blocks), dim3(256), 0, q, ids, t, emb, out,
                                 ctx->dev_err, iw, spw));
    return GQ_OK;
  }
  const bool quad = (w->k % 4 == 0) && ((uintptr_t)out % 16 == 0) &&
                    (w->signed_i8 || w->bits == 8 ? w->row_bytes % 4 == 0
                                                  : (w->bits == 4 ? w->row_bytes % 2 == 0 : true));
  if (quad) {
    const int64_t work = t * (w->k / 4);
    GQ_CUDA_TRY(ctx, gq_launch(ctx, embed_quad_kernel, dim3(grid_for(ctx, work, 256)), dim3(256), 0,
                               q, ids, t, emb, out, ctx->dev_err));
  } else {
    const int64_t work = t * w->k;
    GQ_CUDA_TRY(ctx, gq_launch(ctx, embed_scalar_kernel, dim3(grid_for(ctx, work, 256)), dim3(256),
                               0, q, ids, t, emb, out, ctx->dev_err));
  }
  return GQ_OK;
}

int gq_elementwise_launch(gq_ctx *ctx, int op, const float *a, const float *b, int64_t count,
                          int64_t ncols, int64_t b_stride, int64_t b_off, float cap, float *y) {
  if (count == 0) return GQ_OK;
  GQ_CUDA_TRY(ctx, gq_launch(ctx, elementwise_kernel, dim3(grid_for(ctx, count, 256)), dim3(256), 0,
                             op, a, b, count, ncols, b_stride, b_off, cap, y));
  return GQ_OK;
}
