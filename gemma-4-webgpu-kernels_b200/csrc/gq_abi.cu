// gq_abi.cu — the extern "C" boundary (include/gq.h): context, memory, weight
// upload and the dispatch of each Backend-trait op to its kernel.
//
// Dispatch mirrors the reference's decision order for quantized weights
// (rust/src/backend_wgpu.rs:768-806 and :808-835): the fast streaming kernel
// when the packed rows are whole 16-byte chunks with one scale per row, else
// the generic exact kernel, and for the fused ops a composition of the
// generic kernel with an elementwise epilogue.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <algorithm>
#include <string>

#include "gq_host.h"
#include "gq_internal.cuh"

// kernels (gemv_q.cu, misc_q.cu)
bool gq_gemv_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m, int nw);
int gq_gemv_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w,
                   const gq_qweight *w2, const float *bs, int64_t b_stride, int64_t b_off,
                   float cap, float *y, int64_t ldy, int64_t y_col0);
int gq_scalar_linear_launch(gq_ctx *ctx, const float *x, int64_t m, const gq_qweight *w, float *y);
int gq_gemv_pro_launch(gq_ctx *ctx, int mode, const float *o, const float *r, const float *w1, const float *s,
                       const float *w2n, float eps, float *h, const gq_qweight *w, const gq_qweight *wu,
                       const float *bs, int64_t b_off, float *y);
// gemv_tcx.cu
bool gq_gemv_tcx_supported(gq_ctx *ctx, const gq_qweight *w, const float *x, int64_t m, int nw);
int gq_gemv_tcx_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                       const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                       int64_t y_col0);
// gemv_tc.cu
bool gq_gemv_tc_supported(gq_ctx *ctx, const gq_qweight *w, const float *x, int64_t m, int nw);
int gq_gemv_tc_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                      const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                      int64_t y_col0);
bool gq_prefill_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m);
int gq_prefill_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                      const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                      int64_t y_col0);
int gq_qsum_launch(gq_ctx *ctx, const gq_qweight *w, float *out);
int gq_embed_launch(gq_ctx *ctx, const gq_qweight *w, const uint32_t *ids, int64_t t, float emb,
                    float *out);
int gq_elementwise_launch(gq_ctx *ctx, int op, const float *a, const float *b, int64_t count,
                          int64_t ncols, int64_t b_stride, int64_t b_off, float cap, float *y);

int gq_fail(gq_ctx *ctx, int status, const std::string &msg) {
  if (ctx) ctx->last_error = msg;
  return status;
}

int gq_cuda_fail(gq_ctx *ctx, cudaError_t e, const char *what) {
  (void)cudaGetLastError();  // clear a sticky launch error
  std::string msg = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return gq_fail(ctx, e == cudaErrorMemoryAllocation ? GQ_ERR_OUT_OF_MEMORY : GQ_ERR_CUDA, msg);
}

int gq_enter_ctx(gq_ctx *ctx) {
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != ctx->device) {
    GQ_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  }
  return GQ_OK;
}

int gq_workspace(gq_ctx *ctx, size_t bytes, void **out) {
  if (ctx->ws_cap < bytes) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    GQ_CUDA_TRY(ctx, cudaStreamIsCapturing(ctx->stream, &st));
    if (st != cudaStreamCaptureStatusNone)
      return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT,
                     "workspace must grow while the stream is being captured: run the call once before recording");
    if (ctx->ws) cudaFreeAsync(ctx->ws, ctx->stream);
    ctx->ws = nullptr;
    ctx->ws_cap = 0;
    GQ_CUDA_TRY(ctx, cudaMallocAsync(&ctx->ws, bytes, ctx->stream));
    ctx->ws_cap = bytes;
  }
  *out = ctx->ws;
  return GQ_OK;
}

namespace {

int enter(gq_ctx *ctx) { return gq_enter_ctx(ctx); }

#define GQ_ENTER(ctx)                                                            \
  do {                                                                           \
    if (!(ctx)) return GQ_ERR_INVALID_ARGUMENT;                                  \
    int _rc = enter(ctx);                                                        \
    if (_rc != GQ_OK) return _rc;                                                \
  } while (0)

bool valid_format(int32_t bits, int32_t signed_i8) {
  if (signed_i8) return bits == 8;
  return bits == 2 || bits == 4 || bits == 8;
}

// Workspace for the composed fallbacks (generic kernel + elementwise epilogue),
// grown on demand in stream order.
int scratch_get(gq_ctx *ctx, int slot, size_t floats, float **out) {
  if (ctx->scratch_cap[slot] < floats) {
    if (ctx->scratch[slot]) cudaFreeAsync(ctx->scratch[slot], ctx->stream);
    ctx->scratch[slot] = nullptr;
    ctx->scratch_cap[slot] = 0;
    GQ_CUDA_TRY(ctx, cudaMallocAsync(reinterpret_cast<void **>(&ctx->scratch[slot]),
                                     floats * sizeof(float), ctx->stream));
    ctx->scratch_cap[slot] = floats;
  }
  *out = ctx->scratch[slot];
  return GQ_OK;
}

}  // namespace

int gq_set_error(gq_ctx *ctx, int status, const std::string &msg) { return gq_fail(ctx, status, msg); }

extern "C" {

int gq_abi_version(void) { return GQ_ABI_VERSION; }

const char *gq_status_string(int status) {
  switch (status) {
    case GQ_OK: return "ok";
    case GQ_ERR_INVALID_ARGUMENT: return "invalid argument";
    case GQ_ERR_UNSUPPORTED: return "unsupported";
    case GQ_ERR_CUDA: return "CUDA error";
    case GQ_ERR_OUT_OF_MEMORY: return "out of memory";
    case GQ_ERR_DEVICE: return "device-reported error";
    default: return "unknown status";
  }
}

int gq_ctx_create(int device, gq_ctx **out) {
  if (!out) return GQ_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) return GQ_ERR_CUDA;
  if (device < 0 || device >= count) return GQ_ERR_INVALID_ARGUMENT;
  gq_ctx *ctx = new gq_ctx();
  ctx->device = device;
  int rc = GQ_OK;
  do {
    if ((e = cudaSetDevice(device)) != cudaSuccess) { rc = GQ_ERR_CUDA; break; }
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) { rc = GQ_ERR_CUDA; break; }
    if (prop.major < 10) {
      rc = GQ_ERR_UNSUPPORTED;  // built for sm_100a only
      break;
    }
    ctx->num_sms = prop.multiProcessorCount;
    ctx->smem_optin = prop.sharedMemPerBlockOptin;
    if ((e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking)) != cudaSuccess) {
      rc = GQ_ERR_CUDA;
      break;
    }
    ctx->stream = ctx->own_stream;
    if ((e = cudaMalloc(reinterpret_cast<void **>(&ctx->dev_err), sizeof(uint32_t))) != cudaSuccess) {
      rc = GQ_ERR_CUDA;
      break;
    }
    if ((e = cudaMemset(ctx->dev_err, 0, sizeof(uint32_t))) != cudaSuccess) { rc = GQ_ERR_CUDA; break; }
    const char *pdl = getenv("GQ_PDL");
    ctx->pdl = !(pdl && pdl[0] == '0');
  } while (0);
  if (rc != GQ_OK) {
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return rc;
  }
  *out = ctx;
  return GQ_OK;
}

int gq_ctx_destroy(gq_ctx *ctx) {
  if (!ctx) return GQ_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (int i = 0; i < 2; ++i)
    if (ctx->scratch[i]) cudaFree(ctx->scratch[i]);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return GQ_OK;
}

int gq_ctx_set_stream(gq_ctx *ctx, void *stream) {
  if (!ctx) return GQ_ERR_INVALID_ARGUMENT;
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  return GQ_OK;
}

void *gq_ctx_get_stream(gq_ctx *ctx) { return ctx ? static_cast<void *>(ctx->stream) : nullptr; }

int gq_ctx_num_sms(gq_ctx *ctx) { return ctx ? ctx->num_sms : 0; }

int gq_ctx_set_wait_limit(gq_ctx *ctx, uint64_t limit_ns) {
  if (!ctx || limit_ns < 1000000ull || limit_ns > 60000000000ull) return GQ_ERR_INVALID_ARGUMENT;
  ctx->wait_limit_ns = limit_ns;
  return GQ_OK;
}

const char *gq_last_error(gq_ctx *ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int gq_sync(gq_ctx *ctx) {
  GQ_ENTER(ctx);
  GQ_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
  uint32_t flags = 0;
  GQ_CUDA_TRY(ctx, cudaMemcpy(&flags, ctx->dev_err, sizeof(flags), cudaMemcpyDeviceToHost));
  if (flags) {
    GQ_CUDA_TRY(ctx, cudaMemset(ctx->dev_err, 0, sizeof(uint32_t)));
    std::string msg = "device error:";
    if (flags & GQ_DEVERR_BAD_ID) msg += " embedding id out of range;";
    if (flags & GQ_DEVERR_WAIT_TIMEOUT) msg += " pipeline wait timed out;";
    if (flags & GQ_DEVERR_SAMPLE_CAP) msg += " top-p nucleus larger than the device sampler's 256 candidates;";
    return gq_fail(ctx, GQ_ERR_DEVICE, msg);
  }
  return GQ_OK;
}

int gq_alloc(gq_ctx *ctx, size_t bytes, void **dptr) {
  GQ_ENTER(ctx);
  if (!dptr) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "gq_alloc: null out pointer");
  *dptr = nullptr;
  GQ_CUDA_TRY(ctx, cudaMalloc(dptr, bytes ? bytes : 16));
  return GQ_OK;
}

int gq_free(gq_ctx *ctx, void *dptr) {
  GQ_ENTER(ctx);
  if (dptr) GQ_CUDA_TRY(ctx, cudaFree(dptr));
  return GQ_OK;
}

int gq_memcpy_h2d(gq_ctx *ctx, void *dst, const void *src, size_t bytes) {
  GQ_ENTER(ctx);
  if (!bytes) return GQ_OK;
  if (!dst || !src) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "gq_memcpy_h2d: null pointer");
  GQ_CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return GQ_OK;
}

int gq_memcpy_d2h(gq_ctx *ctx, void *dst, const void *src, size_t bytes) {
  GQ_ENTER(ctx);
  if (!bytes) return GQ_OK;
  if (!dst || !src) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "gq_memcpy_d2h: null pointer");
  GQ_CUDA_TRY(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return GQ_OK;
}

int gq_memset(gq_ctx *ctx, void *dst, int value, size_t bytes) {
  GQ_ENTER(ctx);
  if (!bytes) return GQ_OK;
  if (!dst) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "gq_memset: null pointer");
  GQ_CUDA_TRY(ctx, cudaMemsetAsync(dst, value, bytes, ctx->stream));
  return GQ_OK;
}

int gq_readback(gq_ctx *ctx, float *dst, const float *src, size_t count) {
  int rc = gq_memcpy_d2h(ctx, dst, src, count * sizeof(float));
  if (rc != GQ_OK) return rc;
  return gq_sync(ctx);
}

static int qweight_upload_impl(gq_ctx *ctx, const uint8_t *qbytes, bool bytes_on_device, size_t nbytes,
                               const float *scales, size_t nscales, int64_t n, int64_t k, int32_t bits,
                               int32_t signed_i8, int64_t group_size, gq_qweight **out) {
  GQ_ENTER(ctx);
  if (!out) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qweight_upload: null out pointer");
  *out = nullptr;
  if (!valid_format(bits, signed_i8))
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "qweight_upload: bits must be 2, 4 or 8 (I8 is 8)");
  if (n < 0 || k < 0 || group_size <= 0)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qweight_upload: negative shape or group_size <= 0");
  const int64_t per_byte = signed_i8 ? 1 : 8 / bits;
  if (k % per_byte != 0)
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "qweight_upload: K is not a multiple of values per byte");
  const int64_t row_bytes = signed_i8 ? k : k / per_byte;
  const int64_t ss = (k + group_size - 1) / group_size;
  if ((int64_t)nbytes < n * row_bytes)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qweight_upload: qbytes shorter than n*row_bytes");
  if ((int64_t)nscales < n * ss)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qweight_upload: fewer scales than n*ceil(K/group)");
  if ((n * row_bytes > 0 && !qbytes) || (n * ss > 0 && !scales))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "qweight_upload: null payload");
  gq_qweight *w = new gq_qweight();
  w->ctx = ctx;
  w->device = ctx->device;
  w->n = n;
  w->k = k;
  w->bits = bits;
  w->signed_i8 = signed_i8;
  w->group_size = group_size;
  w->row_bytes = row_bytes;
  w->scale_stride = ss;
  w->nbytes = (size_t)(n * row_bytes);
  // Packed bytes padded to a 16-byte multiple (+16) so vector loads of the last
  // row never leave the allocation; scales followed by per-row code sums.
  const size_t byte_alloc = ((w->nbytes + 15) & ~size_t(15)) + 16;
  w->qsum_off = (n * ss + 3) & ~int64_t(3);
  const size_t scale_alloc = (size_t)(w->qsum_off + n + 8) * sizeof(float);
  cudaError_t e;
  if ((e = cudaMalloc(reinterpret_cast<void **>(&w->bytes), byte_alloc)) != cudaSuccess ||
      (e = cudaMalloc(reinterpret_cast<void **>(&w->scales), scale_alloc)) != cudaSuccess) {
    if (w->bytes) cudaFree(w->bytes);
    delete w;
    return gq_cuda_fail(ctx, e, "qweight_upload: cudaMalloc");
  }
  int rc = GQ_OK;
  do {
    if ((e = cudaMemsetAsync(w->bytes, 0, byte_alloc, ctx->stream)) != cudaSuccess) break;
    if (w->nbytes > 0 &&
        (e = cudaMemcpyAsync(w->bytes, qbytes, w->nbytes,
                             bytes_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                             ctx->stream)) != cudaSuccess)
      break;
    if ((e = cudaMemsetAsync(w->scales, 0, scale_alloc, ctx->stream)) != cudaSuccess) break;
    if (n * ss > 0 &&
        (e = cudaMemcpyAsync(w->scales, scales, (size_t)(n * ss) * sizeof(float), cudaMemcpyHostToDevice,
                             ctx->stream)) != cudaSuccess)
      break;
    rc = gq_qsum_launch(ctx, w, w->scales + w->qsum_off);
    if (rc != GQ_OK) break;
    // The host buffers may be freed by the caller as soon as we return.
    e = cudaStreamSynchronize(ctx->stream);
  } while (0);
  if (rc == GQ_OK && e != cudaSuccess) rc = gq_cuda_fail(ctx, e, "qweight_upload");
  if (rc != GQ_OK) {
    cudaFree(w->bytes);
    cudaFree(w->scales);
    delete w;
    return rc;
  }
  *out = w;
  return GQ_OK;
}

int gq_qweight_upload(gq_ctx *ctx, const uint8_t *qbytes, size_t nbytes, const float *scales,
                      size_t nscales, int64_t n, int64_t k, int32_t bits, int32_t signed_i8,
                      int64_t group_size, gq_qweight **out) {
  return qweight_upload_impl(ctx, qbytes, false, nbytes, scales, nscales, n, k, bits, signed_i8, group_size, out);
}

int gq_qweight_upload_device(gq_ctx *ctx, const uint8_t *qbytes_dev, size_t nbytes, const float *scales,
                             size_t nscales, int64_t n, int64_t k, int32_t bits, int32_t signed_i8,
                             int64_t group_size, gq_qweight **out) {
  return qweight_upload_impl(ctx, qbytes_dev, true, nbytes, scales, nscales, n, k, bits, signed_i8, group_size,
                             out);
}

int gq_qweight_free(gq_qweight *w) {
  if (!w) return GQ_OK;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != w->device) cudaSetDevice(w->device);
  cudaFree(w->bytes);
  cudaFree(w->scales);
  delete w;
  return GQ_OK;
}

int gq_qweight_info(const gq_qweight *w, int64_t *n, int64_t *k, int32_t *bits, int32_t *signed_i8,
                    int64_t *group_size) {
  if (!w) return GQ_ERR_INVALID_ARGUMENT;
  if (n) *n = w->n;
  if (k) *k = w->k;
  if (bits) *bits = w->bits;
  if (signed_i8) *signed_i8 = w->signed_i8;
  if (group_size) *group_size = w->group_size;
  return GQ_OK;
}

}  // extern "C"

namespace {

int check_linear_args(gq_ctx *ctx, const char *op, const float *x, int64_t m, int64_t k,
                      const gq_qweight *w, const float *y) {
  if (!w) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(op) + ": null weight");
  if (w->device != ctx->device)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(op) + ": weight lives on another device");
  if (m < 0 || k != w->k)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT,
                   std::string(op) + ": x is [" + std::to_string(m) + "," + std::to_string(k) +
                       "] but the weight has K=" + std::to_string(w->k));
  if (m > 0 && w->n > 0 && (!y || (k > 0 && !x)))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(op) + ": null activation/output");
  if (m > (1ll << 30)) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, std::string(op) + ": M too large");
  return GQ_OK;
}

// Rows of activations from which the bf16 tensor-core path is used (prefill).
// Below it the streaming CUDA-core kernel keeps f32 activations.
int64_t prefill_min_m() {
  static int64_t v = -1;
  if (v < 0) {
    const char *e = getenv("GQ_PREFILL_MIN_M");
    v = (e && *e) ? atoll(e) : 128;
    if (v < 16) v = 16;
  }
  return v;
}

bool use_prefill(gq_ctx *ctx, const float *x, int64_t m, const gq_qweight *w) {
  return m >= prefill_min_m() && ((uintptr_t)x % 16 == 0) && gq_prefill_supported(ctx, w, m);
}

// Decode rows (M <= 2): the tensor-core GEMV takes weights whose CTAs own at
// least 128 rows (vocab-sized projections), where it streams closest to
// the HBM roofline; the CUDA-core GEMV takes the small per-layer projections,
// where both are bound by launch and x-staging latency and it is the faster one.
// GQ_DECODE_TC=0 disables the tensor-core GEMV, =2 sends it every shape it
// supports (read per call, so tests can switch it).
bool use_gemv_tc(gq_ctx *ctx, const float *x, int64_t m, const gq_qweight *w, int nw) {
  const char *e = getenv("GQ_DECODE_TC");
  const int mode = (e && *e) ? (*e - '0') : 1;
  if (mode <= 0 || m > 2) return false;
  if (mode == 1 && (w->n + ctx->num_sms - 1) / ctx->num_sms < 128) return false;
  return gq_gemv_tc_supported(ctx, w, x, m, nw);
}

// 5 <= M <= 64 (3 <= M with GQ_DECODE_TC=2): the tensor-core GEMV with streamed
// limbs (weights read once for all rows); up to 4 rows the CUDA-core GEMV covers
// them in one pass and is faster (measured on the E2B layer sweep).
bool use_gemv_tcx(gq_ctx *ctx, const float *x, int64_t m, const gq_qweight *w, int nw) {
  const char *e = getenv("GQ_DECODE_TC");
  const int mode = (e && *e) ? (*e - '0') : 1;
  if (mode <= 0 || (mode == 1 && m < 5)) return false;
  return gq_gemv_tcx_supported(ctx, w, x, m, nw);
}

// More than 64 rows that the tensor-core prefill GEMM does not take (below its
// threshold, or a shape it does not support): the short-M GEMV in row blocks of
// at most 64 (equal blocks, so none falls under the GEMV's minimum), each block a
// launch over the same weights (L2 serves the later blocks of weights that fit).
// Exact integer dot products, so these rows keep the FFMA-path bound.
int64_t tcx_block_rows(int64_t m) {
  const int64_t nb = (m + 63) / 64;
  return (m + nb - 1) / nb;
}

bool use_gemv_tcx_blocked(gq_ctx *ctx, const float *x, int64_t m, const gq_qweight *w, int nw) {
  if (m <= 64 || w->k % 4 != 0) return false;  // row offsets of x stay 16-byte aligned
  if (ctx->peers.n > 0 || ctx->peers.signal) return false;  // one launch per call carries the peer stores
  return use_gemv_tcx(ctx, x, tcx_block_rows(m), w, nw);
}

int tcx_blocked_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                       const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                       int64_t y_col0) {
  const int64_t rb = tcx_block_rows(m);
  for (int64_t r0 = 0; r0 < m; r0 += rb) {
    const int64_t mb = std::min(rb, m - r0);
    const int rc = gq_gemv_tcx_launch(ctx, mode, x + r0 * w->k, mb, w, w2, bs ? bs + r0 * b_stride : nullptr, b_stride,
                                      b_off, cap, y + r0 * ldy, ldy, y_col0);
    if (rc != GQ_OK) return rc;
  }
  return GQ_OK;
}

}  // namespace

extern "C" {

int gq_linear(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w, float *y) {
  GQ_ENTER(ctx);
  int rc = check_linear_args(ctx, "linear", x, m, k, w, y);
  if (rc != GQ_OK || m == 0 || w->n == 0) return rc;
  if (use_prefill(ctx, x, m, w)) return gq_prefill_launch(ctx, 0, x, m, w, nullptr, nullptr, 0, 0, 0.0f, y, w->n, 0);
  if (use_gemv_tc(ctx, x, m, w, 1)) return gq_gemv_tc_launch(ctx, 0, x, m, w, nullptr, nullptr, 0, 0, 0.0f, y, w->n, 0);
  if (use_gemv_tcx(ctx, x, m, w, 1)) return gq_gemv_tcx_launch(ctx, 0, x, m, w, nullptr, nullptr, 0, 0, 0.0f, y, w->n, 0);
  if (use_gemv_tcx_blocked(ctx, x, m, w, 1))
    return tcx_blocked_launch(ctx, 0, x, m, w, nullptr, nullptr, 0, 0, 0.0f, y, w->n, 0);
  if (gq_gemv_supported(ctx, w, m, 1))
    return gq_gemv_launch(ctx, 0, x, m, w, nullptr, nullptr, 0, 0, 0.0f, y, w->n, 0);
  return gq_scalar_linear_launch(ctx, x, m, w, y);
}

int gq_linear_geglu(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *wg,
                    const gq_qweight *wu, float *y) {
  GQ_ENTER(ctx);
  int rc = check_linear_args(ctx, "linear_geglu", x, m, k, wg, y);
  if (rc == GQ_OK) rc = check_linear_args(ctx, "linear_geglu", x, m, k, wu, y);
  if (rc != GQ_OK) return rc;
  if (wg->n != wu->n) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_geglu: gate/up rows differ");
  if (m == 0 || wg->n == 0) return GQ_OK;
  const bool same = wg->bits == wu->bits && wg->signed_i8 == wu->signed_i8 &&
                    wg->group_size == wu->group_size;
  if (same && use_prefill(ctx, x, m, wg))
    return gq_prefill_launch(ctx, 1, x, m, wg, wu, nullptr, 0, 0, 0.0f, y, wg->n, 0);
  if (same && use_gemv_tc(ctx, x, m, wg, 2))
    return gq_gemv_tc_launch(ctx, 1, x, m, wg, wu, nullptr, 0, 0, 0.0f, y, wg->n, 0);
  if (same && use_gemv_tcx(ctx, x, m, wg, 2))
    return gq_gemv_tcx_launch(ctx, 1, x, m, wg, wu, nullptr, 0, 0, 0.0f, y, wg->n, 0);
  if (same && use_gemv_tcx_blocked(ctx, x, m, wg, 2))
    return tcx_blocked_launch(ctx, 1, x, m, wg, wu, nullptr, 0, 0, 0.0f, y, wg->n, 0);
  if (same && gq_gemv_supported(ctx, wg, m, 2))
    return gq_gemv_launch(ctx, 1, x, m, wg, wu, nullptr, 0, 0, 0.0f, y, wg->n, 0);
  // composition of rust/src/backend.rs:156-160
  const size_t cnt = (size_t)(m * wg->n);
  float *g = nullptr, *u = nullptr;
  if ((rc = scratch_get(ctx, 0, cnt, &g)) != GQ_OK) return rc;
  if ((rc = scratch_get(ctx, 1, cnt, &u)) != GQ_OK) return rc;
  if ((rc = gq_linear(ctx, x, m, k, wg, g)) != GQ_OK) return rc;
  if ((rc = gq_linear(ctx, x, m, k, wu, u)) != GQ_OK) return rc;
  return gq_elementwise_launch(ctx, 1, g, u, (int64_t)cnt, 0, 0, 0, 0.0f, y);
}

int gq_linear_gelu_mul_cols(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w,
                            const float *b, int64_t b_stride, int64_t b_offset, float *y) {
  GQ_ENTER(ctx);
  int rc = check_linear_args(ctx, "linear_gelu_mul_cols", x, m, k, w, y);
  if (rc != GQ_OK) return rc;
  if (b_offset < 0 || b_stride < 0 || b_offset + w->n > b_stride)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_gelu_mul_cols: offset + N exceeds b's row");
  if (m == 0 || w->n == 0) return GQ_OK;
  if (!b) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_gelu_mul_cols: null b");
  if (use_prefill(ctx, x, m, w))
    return gq_prefill_launch(ctx, 2, x, m, w, nullptr, b, b_stride, b_offset, 0.0f, y, w->n, 0);
  if (use_gemv_tc(ctx, x, m, w, 1))
    return gq_gemv_tc_launch(ctx, 2, x, m, w, nullptr, b, b_stride, b_offset, 0.0f, y, w->n, 0);
  if (use_gemv_tcx(ctx, x, m, w, 1))
    return gq_gemv_tcx_launch(ctx, 2, x, m, w, nullptr, b, b_stride, b_offset, 0.0f, y, w->n, 0);
  if (use_gemv_tcx_blocked(ctx, x, m, w, 1))
    return tcx_blocked_launch(ctx, 2, x, m, w, nullptr, b, b_stride, b_offset, 0.0f, y, w->n, 0);
  if (gq_gemv_supported(ctx, w, m, 1))
    return gq_gemv_launch(ctx, 2, x, m, w, nullptr, b, b_stride, b_offset, 0.0f, y, w->n, 0);
  // composition of rust/src/backend.rs:163-167
  const size_t cnt = (size_t)(m * w->n);
  float *g = nullptr;
  if ((rc = scratch_get(ctx, 0, cnt, &g)) != GQ_OK) return rc;
  if ((rc = gq_linear(ctx, x, m, k, w, g)) != GQ_OK) return rc;
  return gq_elementwise_launch(ctx, 2, g, b, (int64_t)cnt, w->n, b_stride, b_offset, 0.0f, y);
}

namespace {
bool ranges_overlap(const void *a, size_t na, const void *b, size_t nb) {
  const uintptr_t pa = (uintptr_t)a, pb = (uintptr_t)b;
  return na && nb && pa < pb + nb && pb < pa + na;
}
}  // namespace

int gq_add_norm_linear(gq_ctx *ctx, int32_t mode, const float *x, const float *residual, int64_t k,
                       const float *w_norm, float eps, const float *scale_by, const float *w_norm2, float *h_out,
                       const gq_qweight *w, const gq_qweight *w_up, const float *b, int64_t b_offset, float *y) {
  GQ_ENTER(ctx);
  const char *what = "add_norm_linear";
  if (mode < 0 || mode > 2) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(what) + ": mode not in 0..2");
  if (!x || !residual || !w_norm || !h_out || !w || !y)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(what) + ": null pointer");
  if (k != w->k || k <= 0) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(what) + ": k differs from the weight's K");
  if (mode == 1 && (!w_up || w_up->n != w->n || w_up->k != w->k || w_up->bits != w->bits ||
                    w_up->signed_i8 != w->signed_i8 || w_up->group_size != w_up->k))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(what) + ": geglu needs an up weight shaped as w");
  if (mode == 2 && (!b || b_offset < 0)) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(what) + ": null b");
  const size_t kb = (size_t)k * 4, yb = (size_t)w->n * 4;
  if (ranges_overlap(h_out, kb, x, kb) || ranges_overlap(h_out, kb, residual, kb) || ranges_overlap(y, yb, h_out, kb) ||
      ranges_overlap(y, yb, x, kb) || ranges_overlap(y, yb, residual, kb))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, std::string(what) + ": h_out and y must not overlap the inputs");
  if (w->n == 0) return GQ_OK;
  const bool fused = k % 4 == 0 && k <= 4096 &&
                     ((uintptr_t)x | (uintptr_t)residual | (uintptr_t)w_norm | (uintptr_t)h_out |
                      (uintptr_t)(w_norm2 ? w_norm2 : w_norm)) % 16 == 0 &&
                     gq_gemv_supported(ctx, w, 1, mode == 1 ? 2 : 1);
  if (!fused) {
    // the calls it fuses (the normalised row in the context workspace)
    int rc;
    const float *xn = h_out;
    if (w_norm2) {
      void *ws = nullptr;
      if ((rc = gq_workspace(ctx, kb, &ws)) != GQ_OK) return rc;
      if ((rc = gq_add_rms_norm_norm(ctx, residual, x, 1, k, w_norm, eps, scale_by, w_norm2, h_out,
                                     static_cast<float *>(ws))) != GQ_OK)
        return rc;
      xn = static_cast<const float *>(ws);
    } else if ((rc = gq_add_rms_norm(ctx, residual, x, 1, k, w_norm, eps, scale_by, h_out)) != GQ_OK) {
      return rc;
    }
    if (mode == 1) return gq_linear_geglu(ctx, xn, 1, k, w, w_up, y);
    if (mode == 2) return gq_linear_gelu_mul_cols(ctx, xn, 1, k, w, b, b_offset + w->n, b_offset, y);
    return gq_linear(ctx, xn, 1, k, w, y);
  }
  return gq_gemv_pro_launch(ctx, mode, x, residual, w_norm, scale_by, w_norm2, eps, h_out, w, mode == 1 ? w_up : nullptr,
                            b, b_offset, y);
}

namespace {
// One thread waits (bounded) until every rank's flag has reached this rank's
// epoch sync[1] (written by the signalling GEMV before this kernel in stream
// order); acquire, system scope. A peer one call ahead holds epoch + 1, so the
// test is a wrap-safe >=. On timeout it reports GQ_DEVERR_WAIT_TIMEOUT and returns.
__global__ void peer_wait_kernel(const uint32_t *flags, int world, const uint32_t *sync, uint64_t limit_ns,
                                 uint32_t *err) {
  gqd::griddep_wait();
  if (threadIdx.x != 0) return;
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t *>(sync + 1);
  const uint64_t t0 = gqd::globaltimer_ns();
  for (int r = 0; r < world; ++r) {
    for (uint32_t it = 0;; ++it) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if ((it & 255u) == 255u && gqd::globaltimer_ns() - t0 > limit_ns) {
        gqd::report(err, GQ_DEVERR_WAIT_TIMEOUT);
        return;
      }
      __nanosleep(64);
    }
  }
  gqd::griddep_launch_dependents();
}
}  // namespace

int gq_peer_wait(gq_ctx *ctx, const uint32_t *flags, int32_t world, const uint32_t *sync) {
  GQ_ENTER(ctx);
  if (!flags || !sync || world < 1 || world > kMaxPeerDst + 1)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "peer_wait: flags, sync word, 1..9 ranks");
  GQ_CUDA_TRY(ctx, gq_launch(ctx, peer_wait_kernel, dim3(1), dim3(32), 0, flags, (int)world, sync, ctx->wait_limit_ns,
                             ctx->dev_err));
  return GQ_OK;
}

static int softcap_peers_signal_impl(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w, float cap,
                                   float *y, int64_t ldy, int64_t y_col0, float *const *peer_y, int32_t npeers,
                                   uint32_t *const *flags, uint32_t *sync, int32_t rank, int fused_wait) {
  GQ_ENTER(ctx);
  if (!flags || !sync || rank < 0 || rank > npeers) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "peers_signal: flags, sync word, rank");
  for (int i = 0; i <= npeers && i <= kMaxPeerDst; ++i)
    if (!flags[i]) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "peers_signal: null flag array");
  ctx->peer_signal.sync = sync;
  ctx->peer_signal.rank = rank;
  for (int i = 0; i <= npeers && i <= kMaxPeerDst; ++i) ctx->peer_signal.flag[i] = flags[i];
  ctx->peer_signal.signal = 1;
  ctx->peer_signal.fused_wait = fused_wait;
  ctx->peer_signal.wait_limit_ns = ctx->wait_limit_ns;
  ctx->peer_signal.err = ctx->dev_err;
  const int rc = gq_linear_softcap_peers(ctx, x, m, k, w, cap, y, ldy, y_col0, peer_y, npeers);
  ctx->peer_signal = PeerDst{};
  return rc;
}

int gq_linear_softcap_peers_signal(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w, float cap,
                                   float *y, int64_t ldy, int64_t y_col0, float *const *peer_y, int32_t npeers,
                                   uint32_t *const *flags, uint32_t *sync, int32_t rank) {
  return softcap_peers_signal_impl(ctx, x, m, k, w, cap, y, ldy, y_col0, peer_y, npeers, flags, sync, rank, 0);
}

int gq_linear_softcap_peers_sync(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w, float cap,
                                 float *y, int64_t ldy, int64_t y_col0, float *const *peer_y, int32_t npeers,
                                 uint32_t *const *flags, uint32_t *sync, int32_t rank) {
  return softcap_peers_signal_impl(ctx, x, m, k, w, cap, y, ldy, y_col0, peer_y, npeers, flags, sync, rank, 1);
}

int gq_linear_softcap_peers(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w, float cap,
                            float *y, int64_t ldy, int64_t y_col0, float *const *peer_y, int32_t npeers) {
  GQ_ENTER(ctx);
  if (npeers < 0 || npeers > kMaxPeerDst || (npeers > 0 && !peer_y))
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_softcap_peers: 0..8 peer buffers");
  int rc = check_linear_args(ctx, "linear_softcap_peers", x, m, k, w, y);
  if (rc != GQ_OK) return rc;
  for (int i = 0; i < npeers; ++i)
    if (!peer_y[i]) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_softcap_peers: null peer buffer");
  // only the GEMV kernels carry the peer stores in their epilogue
  const bool gemv = !use_prefill(ctx, x, m, w) &&
                    (use_gemv_tc(ctx, x, m, w, 1) || use_gemv_tcx(ctx, x, m, w, 1) || gq_gemv_supported(ctx, w, m, 1));
  if (!gemv)
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "linear_softcap_peers: shape not served by a GEMV kernel (M < 128, whole rows)");
  ctx->peers = ctx->peer_signal;  // completion signal, when a caller set one
  ctx->peers.n = npeers;
  for (int i = 0; i < npeers; ++i) ctx->peers.p[i] = peer_y[i];
  rc = gq_linear_softcap(ctx, x, m, k, w, cap, y, ldy, y_col0);
  ctx->peers = PeerDst{};
  return rc;
}

int gq_ipc_get_handle(gq_ctx *ctx, void *dptr, uint8_t *handle64) {
  GQ_ENTER(ctx);
  if (!dptr || !handle64) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  GQ_CUDA_TRY(ctx, cudaIpcGetMemHandle(&h, dptr));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle64, &h, 64);
  return GQ_OK;
}

int gq_ipc_open(gq_ctx *ctx, const uint8_t *handle64, void **dptr) {
  GQ_ENTER(ctx);
  if (!dptr || !handle64) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  GQ_CUDA_TRY(ctx, cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess));
  return GQ_OK;
}

int gq_ipc_close(gq_ctx *ctx, void *dptr) {
  GQ_ENTER(ctx);
  if (!dptr) return GQ_OK;
  GQ_CUDA_TRY(ctx, cudaIpcCloseMemHandle(dptr));
  return GQ_OK;
}

int gq_linear_softcap(gq_ctx *ctx, const float *x, int64_t m, int64_t k, const gq_qweight *w,
                      float cap, float *y, int64_t ldy, int64_t y_col0) {
  GQ_ENTER(ctx);
  int rc = check_linear_args(ctx, "linear_softcap", x, m, k, w, y);
  if (rc != GQ_OK) return rc;
  if (ldy < 0 || y_col0 < 0 || y_col0 + w->n > ldy)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "linear_softcap: y_col0 + N exceeds ldy");
  if (m == 0 || w->n == 0) return GQ_OK;
  if (use_prefill(ctx, x, m, w)) return gq_prefill_launch(ctx, 3, x, m, w, nullptr, nullptr, 0, 0, cap, y, ldy, y_col0);
  if (use_gemv_tc(ctx, x, m, w, 1)) return gq_gemv_tc_launch(ctx, 3, x, m, w, nullptr, nullptr, 0, 0, cap, y, ldy, y_col0);
  if (use_gemv_tcx(ctx, x, m, w, 1))
    return gq_gemv_tcx_launch(ctx, 3, x, m, w, nullptr, nullptr, 0, 0, cap, y, ldy, y_col0);
  if (use_gemv_tcx_blocked(ctx, x, m, w, 1))
    return tcx_blocked_launch(ctx, 3, x, m, w, nullptr, nullptr, 0, 0, cap, y, ldy, y_col0);
  if (gq_gemv_supported(ctx, w, m, 1))
    return gq_gemv_launch(ctx, 3, x, m, w, nullptr, nullptr, 0, 0, cap, y, ldy, y_col0);
  // composition: generic linear into scratch, then soft-cap into the strided output
  const size_t cnt = (size_t)(m * w->n);
  float *g = nullptr;
  if ((rc = scratch_get(ctx, 0, cnt, &g)) != GQ_OK) return rc;
  if ((rc = gq_scalar_linear_launch(ctx, x, m, w, g)) != GQ_OK) return rc;
  for (int64_t r = 0; r < m; ++r) {
    float *dst = y + r * ldy + y_col0;
    const float *src = g + r * w->n;
    if (cap > 0.0f)
      rc = gq_elementwise_launch(ctx, 0, src, nullptr, w->n, 0, 0, 0, cap, dst);
    else
      rc = cudaMemcpyAsync(dst, src, (size_t)w->n * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream) ==
                   cudaSuccess
               ? GQ_OK
               : gq_fail(ctx, GQ_ERR_CUDA, "linear_softcap: copy");
    if (rc != GQ_OK) return rc;
  }
  return GQ_OK;
}

struct gq_graph {
  int device = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

int gq_graph_begin(gq_ctx *ctx) {
  GQ_ENTER(ctx);
  if (ctx->stream == nullptr || ctx->stream == cudaStreamLegacy || ctx->stream == cudaStreamPerThread)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "graph_begin: cannot record the default stream");
  GQ_CUDA_TRY(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  return GQ_OK;
}

int gq_graph_end(gq_ctx *ctx, gq_graph **out) {
  GQ_ENTER(ctx);
  if (!out) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "graph_end: null out pointer");
  *out = nullptr;
  cudaGraph_t g = nullptr;
  GQ_CUDA_TRY(ctx, cudaStreamEndCapture(ctx->stream, &g));
  cudaGraphExec_t ex = nullptr;
  cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    return gq_cuda_fail(ctx, e, "graph_end: cudaGraphInstantiate");
  }
  gq_graph *gr = new gq_graph();
  gr->device = ctx->device;
  gr->graph = g;
  gr->exec = ex;
  *out = gr;
  return GQ_OK;
}

int gq_graph_launch(gq_ctx *ctx, gq_graph *graph) {
  GQ_ENTER(ctx);
  if (!graph || graph->device != ctx->device)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "graph_launch: null graph or other device");
  GQ_CUDA_TRY(ctx, cudaGraphLaunch(graph->exec, ctx->stream));
  return GQ_OK;
}

int gq_graph_destroy(gq_graph *graph) {
  if (!graph) return GQ_OK;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != graph->device) cudaSetDevice(graph->device);
  if (graph->exec) cudaGraphExecDestroy(graph->exec);
  if (graph->graph) cudaGraphDestroy(graph->graph);
  delete graph;
  return GQ_OK;
}

int gq_embed_rows(gq_ctx *ctx, const gq_qweight *table, const uint32_t *ids, int64_t t, float scale,
                  float *out) {
  GQ_ENTER(ctx);
  if (!table) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "embed_rows: null table");
  if (table->device != ctx->device)
    return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "embed_rows: table lives on another device");
  if (t < 0) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "embed_rows: negative count");
  if (t == 0 || table->k == 0) return GQ_OK;
  if (!ids || !out) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "embed_rows: null ids/out");
  return gq_embed_launch(ctx, table, ids, t, scale, out);
}

int gq_softcap(gq_ctx *ctx, const float *x, int64_t n, float cap, float *y) {
  GQ_ENTER(ctx);
  if (n < 0) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "softcap: negative count");
  if (n == 0) return GQ_OK;
  if (!x || !y) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "softcap: null pointer");
  return gq_elementwise_launch(ctx, 0, x, nullptr, n, 0, 0, 0, cap, y);
}

int gq_geglu(gq_ctx *ctx, const float *gate, const float *up, int64_t n, float *y) {
  GQ_ENTER(ctx);
  if (n < 0) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "geglu: negative count");
  if (n == 0) return GQ_OK;
  if (!gate || !up || !y) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "geglu: null pointer");
  return gq_elementwise_launch(ctx, 1, gate, up, n, 0, 0, 0, 0.0f, y);
}

}  // extern "C"
