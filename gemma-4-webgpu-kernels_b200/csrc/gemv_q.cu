// gemv_q.cu — decode / short-M dequantizing GEMV (MATMUL_Q, CUDA-core path).
//
// Replaces the reference's MATMUL_Q shader (rust/src/kernels/matmul_q.wgsl:96-169,
// dispatched by rust/src/backend_wgpu.rs:646-695) for M <= 4 rows of activations:
//   y[m, n] = epilogue( scale[n] * sum_k x[m, k] * q[n, k] )
// with the MODE epilogues of matmul_q.wgsl:18-21 (0 plain, 1 GeGLU with a second
// weight, 2 gelu * column slice) plus MODE 3 (logit soft-cap).
//
// Design (B200, HBM-bound):
//  * Persistent CTAs, two per SM, each owning a contiguous range of weight rows.
//    Rows are contiguous in the packed layout, so a CTA's work is one contiguous
//    byte range, streamed into shared memory by the TMA engine with 1-D bulk
//    copies (cp.async.bulk) through a ring of mbarrier-tracked stages. Copies for
//    the first stages are issued before griddepcontrol.wait, so under
//    programmatic dependent launch the weight stream of this kernel overlaps the
//    tail of the kernel that produces x.
//  * Inside a stage the work is balanced at 16-byte-chunk granularity: thread t
//    takes chunks t, t+256, ... of the stage, whatever row they belong to, and
//    writes one partial sum per chunk; then one warp per row adds that row's
//    partials with shuffles and runs the epilogue.
//  * Dequantization costs one LOP3 + one FFMA per code. A code field masked in
//    place, (word & (mask << pos)), read as an f32 bit pattern is the subnormal
//    raw * 2^(pos-149); FFMA handles subnormal inputs at full rate and exactly.
//    x is pre-scaled in shared memory by 2^(S - pos) (a power of two, exact) so
//    every product equals x * raw * 2^(S-149) with a normal result. S is chosen
//    per activation row from max|x| so nothing overflows.
//  * Offset-binary codes are accumulated as raw = q + zp. To keep the zp*sum(x)
//    term small the per-row mean mu of x is subtracted first; the epilogue adds
//    back mu * sum_k q[n, k] (precomputed per weight row at upload) and removes
//    zp * sum_k (x - mu)_k exactly (double).
#include <cuda_runtime.h>
#include <math.h>

#include "gq_internal.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCtasPerSm = 2;  // one CTA's epilogue overlaps the other's stream
constexpr int kMaxStages = 4;

struct GemvArgs {
  const float *x;
  int64_t ldx;
  int M, K, N;
  const uint8_t *w;
  const float *s;
  const float *qsum;
  const uint8_t *w2;
  const float *s2;
  const float *qsum2;
  const float *bs;
  int64_t b_stride, b_off;
  float cap;
  float *y;
  int64_t ldy, y_col0;
  int row_bytes;    // bytes per packed row, multiple of 16
  int rows_per_cta; // contiguous rows per CTA
  int tile_rows;    // rows per pipeline stage
  int stages;       // pipeline depth
  uint32_t *err;
};

template <int BITS>
struct Fmt {
  static constexpr int kPerWord = 32 / BITS;      // codes per 32-bit word
  static constexpr int kPerChunk = 4 * kPerWord;  // codes per 16-byte chunk
  static constexpr int kPad = kPerChunk + 4;      // padded x floats per chunk
  static constexpr int kZp = 1 << (BITS - 1);     // offset-binary zero point
  // Codes [0, kSplit) are masked straight out of the word; the rest out of the
  // word shifted right by kShift, so every field stays inside f32 bits 0..22.
  static constexpr int kSplit = BITS == 4 ? 5 : (BITS == 2 ? 11 : 2);
  static constexpr int kShift = BITS == 4 ? 12 : 16;
};

// Bit position of code j of a word inside the 32-bit register it is masked from.
template <int BITS>
__host__ __device__ constexpr int code_pos(int j) {
  return j < Fmt<BITS>::kSplit ? j * BITS : j * BITS - Fmt<BITS>::kShift;
}

// ---- block reduction of (sum in double, max in float) in one pass --------------
__device__ __forceinline__ void block_sum_max(double &sum, float &mx, double *dscr, float *fscr) {
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) {
    dscr[warp] = sum;
    fscr[warp] = mx;
  }
  __syncthreads();
  sum = 0.0;
  mx = 0.0f;
  for (int i = 0; i < kWarps; ++i) {
    sum += dscr[i];
    mx = fmaxf(mx, fscr[i]);
  }
}

__device__ __forceinline__ float pow2f(int e) {  // exact 2^e for e in [-126, 127]
  return __int_as_float((e + 127) << 23);
}

// Shared-memory carve-up, identical on host (sizing) and device (addressing).
struct GemvSmem {
  size_t stage_off, xs_off, red_off, bar_off, dscr_off, fscr_off, par_off, total;
};
__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }
__host__ __device__ inline GemvSmem gemv_layout(int bits, int mt, int nw, int row_bytes,
                                                int tile_rows, int stages) {
  const int C = row_bytes / 16;
  const int per_chunk = 4 * (32 / bits);
  GemvSmem L;
  size_t o = 0;
  L.stage_off = o; o = align16(o + (size_t)stages * nw * tile_rows * row_bytes);
  L.xs_off = o;    o = align16(o + (size_t)mt * C * (per_chunk + 4) * sizeof(float));
  L.red_off = o;   o = align16(o + (size_t)nw * mt * tile_rows * C * sizeof(float));
  L.bar_off = o;   o = align16(o + kMaxStages * sizeof(uint64_t));
  L.dscr_off = o;  o = align16(o + kWarps * sizeof(double));
  L.fscr_off = o;  o = align16(o + kWarps * sizeof(float));
  L.par_off = o;   o = align16(o + (size_t)mt * (sizeof(double) + 2 * sizeof(float)));
  L.total = o;
  return L;
}

// ---- the kernel -----------------------------------------------------------------
template <int BITS, bool SIGNED, int MT, int MODE>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_q_kernel(const GemvArgs a) {
  using F = Fmt<BITS>;
  constexpr int NW = (MODE == 1) ? 2 : 1;  // weights streamed together
  constexpr int ACC = (MT == 1) ? 4 : (MT == 2 ? 2 : 1);
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  constexpr uint32_t kXor = (BITS == 8 && SIGNED) ? 0x80808080u : 0u;

  extern __shared__ __align__(128) uint8_t smem[];
  const int C = a.row_bytes >> 4;  // chunks per row
  const int stage_bytes = a.tile_rows * a.row_bytes;
  const int tile_chunks = a.tile_rows * C;
  const GemvSmem L = gemv_layout(BITS, MT, NW, a.row_bytes, a.tile_rows, a.stages);
  uint8_t *stage_buf = smem + L.stage_off;                        // [stages][NW][stage_bytes]
  float *xs = reinterpret_cast<float *>(smem + L.xs_off);         // [MT][C][kPad]
  float *red = reinterpret_cast<float *>(smem + L.red_off);       // [NW][MT][tile_chunks]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);  // [kMaxStages]
  double *dscr = reinterpret_cast<double *>(smem + L.dscr_off);   // [kWarps]
  float *fscr = reinterpret_cast<float *>(smem + L.fscr_off);     // [kWarps]
  double *pow2_s = reinterpret_cast<double *>(smem + L.par_off);  // [MT]
  float *mu_s = reinterpret_cast<float *>(pow2_s + MT);           // [MT]
  float *corr_s = mu_s + MT;                                      // [MT]

  const int tid = threadIdx.x;
  const int n_begin = blockIdx.x * a.rows_per_cta;
  const int n_end = min(a.N, n_begin + a.rows_per_cta);
  const int m0 = blockIdx.y * MT;
  const int nrows = n_end - n_begin;
  const int ntiles = nrows > 0 ? (nrows + a.tile_rows - 1) / a.tile_rows : 0;

  int issued = 0;  // tiles whose copies thread 0 has issued
  auto issue = [&](int t) {
    issued = t + 1;
    const int stage = t % a.stages;
    const int r0 = n_begin + t * a.tile_rows;
    const int rows = min(a.tile_rows, n_end - r0);
    const uint32_t bytes = (uint32_t)rows * (uint32_t)a.row_bytes;
    uint64_t *bar = &bars[stage];
    gqd::mbar_arrive_expect_tx(bar, bytes * NW);
    uint8_t *dst = stage_buf + (size_t)stage * NW * stage_bytes;
    gqd::bulk_g2s(dst, a.w + (size_t)r0 * a.row_bytes, bytes, bar);
    if (NW == 2) gqd::bulk_g2s(dst + stage_bytes, a.w2 + (size_t)r0 * a.row_bytes, bytes, bar);
  };

  if (tid == 0) {
    for (int i = 0; i < a.stages; ++i) gqd::mbar_init(&bars[i], 1);
    gqd::fence_mbar_init();
  }
  __syncthreads();
  // Weights are immutable after upload: start streaming before the dependency wait.
  if (tid == 0)
    for (int t = 0; t < min(a.stages, ntiles); ++t) issue(t);

  gqd::griddep_wait();

  // ---- stage x: x' = x - mu, scaled by 2^(S - pos) into the padded layout ----
  // mu and S come from one (sum, max|x|) reduction; S leaves one bit of headroom
  // for |x - mu| <= 2 max|x|. zp * sum(x') is taken as sum(x) - K*mu in double:
  // the per-element rounding of x - mu it ignores is below 2^-24 relative.
  for (int m = 0; m < MT; ++m) {
    const bool live = (m0 + m) < a.M;
    const float *xr = a.x + (size_t)(m0 + m) * a.ldx;
    double sx = 0.0;
    float mx = 0.0f;
    if (live)
      for (int k = tid * 4; k < a.K; k += kThreads * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + k);
        sx += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
    block_sum_max(sx, mx, dscr, fscr);
    const float mu = live && a.K > 0 ? (float)(sx / (double)a.K) : 0.0f;
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) frexpf(mx, &e);  // mx < 2^e, so |x - mu| < 2^(e+1)
    int S = 125 - e;
    S = max(-100, min(126, S));
    float *xm = xs + (size_t)m * C * F::kPad;
    for (int k = tid * 4; k < a.K; k += kThreads * 4) {
      float4 v = live ? *reinterpret_cast<const float4 *>(xr + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      float vv[4] = {__fsub_rn(v.x, mu), __fsub_rn(v.y, mu), __fsub_rn(v.z, mu), __fsub_rn(v.w, mu)};
      if (!live) vv[0] = vv[1] = vv[2] = vv[3] = 0.0f;
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = vv[i] * pow2f(S - code_pos<BITS>((k + i) % F::kPerWord));
      *reinterpret_cast<float4 *>(xm + (k / F::kPerChunk) * F::kPad + (k % F::kPerChunk)) =
          make_float4(o[0], o[1], o[2], o[3]);
    }
    if (tid == 0) {
      mu_s[m] = mu;
      const double sxp = live ? sx - (double)a.K * (double)mu : 0.0;
      corr_s[m] = (float)((double)F::kZp * sxp * ldexp(1.0, S - 149));
      pow2_s[m] = ldexp(1.0, 149 - S);
    }
  }
  __syncthreads();
  gqd::griddep_launch_dependents();

  bool failed = false;
  int t_fail = 0;
  for (int t = 0; t < ntiles; ++t) {
    const int stage = t % a.stages;
    const uint32_t parity = (uint32_t)(t / a.stages) & 1u;
    const bool ok = gqd::mbar_wait_bounded(&bars[stage], parity);
    if (__syncthreads_or(!ok)) {
      failed = true;
      t_fail = t;
      break;
    }
    const int r0 = n_begin + t * a.tile_rows;
    const int rows = min(a.tile_rows, n_end - r0);
    const int nch = rows * C;
    const uint8_t *buf = stage_buf + (size_t)stage * NW * stage_bytes;

    int r = tid / C, c = tid - (tid / C) * C;  // (row, chunk) of f, advanced without division
    const int dr = kThreads / C, dc = kThreads - (kThreads / C) * C;
    for (int f = tid; f < nch; f += kThreads) {
      uint4 wv[NW];
#pragma unroll
      for (int h = 0; h < NW; ++h)
        wv[h] = *reinterpret_cast<const uint4 *>(buf + h * stage_bytes + (size_t)r * a.row_bytes + c * 16);
      float acc[NW][MT][ACC];
#pragma unroll
      for (int h = 0; h < NW; ++h)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int q = 0; q < ACC; ++q) acc[h][m][q] = 0.0f;
      const float *xc = xs + (size_t)c * F::kPad;
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        uint32_t lo[NW], hi[NW];
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          const uint32_t word = (wi == 0 ? wv[h].x : wi == 1 ? wv[h].y : wi == 2 ? wv[h].z : wv[h].w) ^ kXor;
          lo[h] = word;
          hi[h] = word >> F::kShift;
        }
#pragma unroll
        for (int j4 = 0; j4 < F::kPerWord; j4 += 4) {
          float4 xv[MT];
#pragma unroll
          for (int m = 0; m < MT; ++m)
            xv[m] = *reinterpret_cast<const float4 *>(xc + (size_t)m * C * F::kPad + wi * F::kPerWord + j4);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int j = j4 + jj;
#pragma unroll
            for (int h = 0; h < NW; ++h) {
              const uint32_t src = (j < F::kSplit) ? lo[h] : hi[h];
              const float fld = __uint_as_float(src & (kMask << code_pos<BITS>(j)));
#pragma unroll
              for (int m = 0; m < MT; ++m) {
                const float xvj = jj == 0 ? xv[m].x : jj == 1 ? xv[m].y : jj == 2 ? xv[m].z : xv[m].w;
                acc[h][m][j % ACC] = __fmaf_rn(xvj, fld, acc[h][m][j % ACC]);
              }
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < NW; ++h)
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float v = acc[h][m][0];
#pragma unroll
          for (int q = 1; q < ACC; ++q) v += acc[h][m][q];
          red[((size_t)h * MT + m) * tile_chunks + f] = v;
        }
      r += dr;
      c += dc;
      if (c >= C) {
        c -= C;
        ++r;
      }
    }
    __syncthreads();  // partials written; stage buffer fully consumed
    if (tid == 0 && t + a.stages < ntiles) issue(t + a.stages);

    const int warp = tid >> 5, lane = tid & 31;
    for (int e = warp; e < rows * MT; e += kWarps) {  // one warp per (row, m)
      const int r2 = e / MT;
      const int m = e - r2 * MT;
      if (m0 + m >= a.M) continue;
      const int n = r0 + r2;
      float dsum[NW];
#pragma unroll
      for (int h = 0; h < NW; ++h) {
        const float *p = red + ((size_t)h * MT + m) * tile_chunks + (size_t)r2 * C;
        float v = 0.0f;
        for (int cc = lane; cc < C; cc += 32) v += p[cc];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        dsum[h] = v;
      }
      if (lane != 0) continue;
      const double mu = (double)mu_s[m];
      const double corr = (double)corr_s[m];
      const double p2 = pow2_s[m];
      const float v0 = (float)((((double)dsum[0] - corr) * p2 + mu * (double)a.qsum[n]) * (double)a.s[n]);
      float out;
      if (MODE == 1) {
        const float v1 = (float)((((double)dsum[NW - 1] - corr) * p2 + mu * (double)a.qsum2[n]) * (double)a.s2[n]);
        out = __fmul_rn(gqd::gelu_tanh(v0), v1);
      } else if (MODE == 2) {
        out = __fmul_rn(gqd::gelu_tanh(v0), a.bs[(size_t)(m0 + m) * a.b_stride + a.b_off + n]);
      } else if (MODE == 3) {
        out = a.cap > 0.0f ? __fmul_rn(a.cap, tanhf(__fdiv_rn(v0, a.cap))) : v0;
      } else {
        out = v0;
      }
      a.y[(size_t)(m0 + m) * a.ldy + a.y_col0 + n] = out;
    }
    // The partial buffer is rewritten by the next tile only after the barrier
    // at the top of the next iteration.
    __syncthreads();
  }

  if (failed) {
    if (tid == 0) {
      gqd::report(a.err, GQ_DEVERR_WAIT_TIMEOUT);
      // Drain copies still in flight (bounded) before the CTA's shared memory
      // is released: tiles [t_fail, issued) each own a distinct stage.
      for (int t = t_fail; t < issued; ++t)
        (void)gqd::mbar_wait_bounded(&bars[t % a.stages], (uint32_t)(t / a.stages) & 1u,
                                     100000000ull);
    }
    __syncthreads();
  }
}

template <int BITS, bool SIGNED, int MT, int MODE>
int launch_t(gq_ctx *ctx, const GemvArgs &a, dim3 grid, size_t smem) {
  auto kern = gemv_q_kernel<BITS, SIGNED, MT, MODE>;
  static bool attr_set[64] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)ctx->smem_optin));
    attr_set[dev] = true;
  }
  GQ_CUDA_TRY(ctx, gq_launch(ctx, kern, grid, dim3(kThreads), smem, a));
  return GQ_OK;
}

template <int BITS, bool SIGNED, int MT>
int launch_mode(gq_ctx *ctx, int mode, const GemvArgs &a, dim3 grid, size_t smem) {
  switch (mode) {
    case 0: return launch_t<BITS, SIGNED, MT, 0>(ctx, a, grid, smem);
    case 1: return launch_t<BITS, SIGNED, MT, 1>(ctx, a, grid, smem);
    case 2: return launch_t<BITS, SIGNED, MT, 2>(ctx, a, grid, smem);
    default: return launch_t<BITS, SIGNED, MT, 3>(ctx, a, grid, smem);
  }
}

template <int BITS, bool SIGNED>
int launch_mt(gq_ctx *ctx, int mt, int mode, const GemvArgs &a, dim3 grid, size_t smem) {
  if (mt == 1) return launch_mode<BITS, SIGNED, 1>(ctx, mode, a, grid, smem);
  if (mt == 2) return launch_mode<BITS, SIGNED, 2>(ctx, mode, a, grid, smem);
  return launch_mode<BITS, SIGNED, 4>(ctx, mode, a, grid, smem);
}

}  // namespace

// Shared memory the kernel needs for a configuration (bytes).
static size_t gemv_smem_bytes(int bits, int mt, int nw, int row_bytes, int tile_rows, int stages) {
  return gemv_layout(bits, mt, nw, row_bytes, tile_rows, stages).total;
}

// True when the CUDA-core GEMV handles this shape: whole 16-byte chunks per row,
// one scale per row (group == K), and x rows that fit in shared memory.
bool gq_gemv_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m, int nw) {
  if (w->group_size != w->k || w->k <= 0 || w->n <= 0 || m <= 0) return false;
  if (w->row_bytes % 16 != 0 || w->row_bytes > 65536) return false;
  if (w->n > (1ll << 30)) return false;
  const int mt = m <= 1 ? 1 : (m == 2 ? 2 : 4);
  if (w->k % 4 != 0) return false;
  return gemv_smem_bytes(w->bits, mt, nw, (int)w->row_bytes, 1, 2) <= ctx->smem_optin / kCtasPerSm - 1024;
}

// mode: 0 plain, 1 geglu (w2 = up), 2 gelu * bs slice, 3 soft-cap.
int gq_gemv_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w,
                   const gq_qweight *w2, const float *bs, int64_t b_stride, int64_t b_off,
                   float cap, float *y, int64_t ldy, int64_t y_col0) {
  const int nw = (mode == 1) ? 2 : 1;
  const int mt = m <= 1 ? 1 : (m == 2 ? 2 : 4);
  const int rb = (int)w->row_bytes;
  const int C = rb / 16;
  GemvArgs a = {};
  a.x = x;
  a.ldx = w->k;
  a.M = (int)m;
  a.K = (int)w->k;
  a.N = (int)w->n;
  a.w = w->bytes;
  a.s = w->scales;
  a.qsum = w->scales + w->n * w->scale_stride;  // qsum follows the scales
  if (w2) {
    a.w2 = w2->bytes;
    a.s2 = w2->scales;
    a.qsum2 = w2->scales + w2->n * w2->scale_stride;
  }
  a.bs = bs;
  a.b_stride = b_stride;
  a.b_off = b_off;
  a.cap = cap;
  a.y = y;
  a.ldy = ldy;
  a.y_col0 = y_col0;
  a.row_bytes = rb;
  a.err = ctx->dev_err;

  // Grid: kCtasPerSm CTAs per SM over contiguous row ranges.
  const int gx_max = ctx->num_sms * kCtasPerSm;
  int rows_per_cta = (int)((w->n + gx_max - 1) / gx_max);
  if (rows_per_cta < 1) rows_per_cta = 1;
  const int gx = (int)((w->n + rows_per_cta - 1) / rows_per_cta);
  // Stage size: about 1024 chunks (4 per thread) and <= 16 KB per weight.
  int tile_rows = max(1, 1024 / C);
  tile_rows = min(tile_rows, max(1, (16 * 1024) / rb));
  tile_rows = min(tile_rows, rows_per_cta);
  const int ntiles = (rows_per_cta + tile_rows - 1) / tile_rows;
  int stages = min(kMaxStages, ntiles);
  const size_t smem_cap = ctx->smem_optin / kCtasPerSm - 1024;
  size_t smem = gemv_smem_bytes(w->bits, mt, nw, rb, tile_rows, stages);
  while (smem > smem_cap && (stages > 1 || tile_rows > 1)) {
    if (stages > 2) --stages;
    else if (tile_rows > 1) tile_rows = (tile_rows + 1) / 2;
    else --stages;
    smem = gemv_smem_bytes(w->bits, mt, nw, rb, tile_rows, stages);
  }
  if (smem > smem_cap) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "gemv: shared memory");
  a.rows_per_cta = rows_per_cta;
  a.tile_rows = tile_rows;
  a.stages = stages;
  dim3 grid(gx, (unsigned)((m + mt - 1) / mt));
  if (w->bits == 4) return launch_mt<4, false>(ctx, mt, mode, a, grid, smem);
  if (w->bits == 2) return launch_mt<2, false>(ctx, mt, mode, a, grid, smem);
  if (w->signed_i8) return launch_mt<8, true>(ctx, mt, mode, a, grid, smem);
  return launch_mt<8, false>(ctx, mt, mode, a, grid, smem);
}
