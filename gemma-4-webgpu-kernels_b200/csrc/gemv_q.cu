// gemv_q.cu — decode / short-M dequantizing GEMV (MATMUL_Q, CUDA-core path).
//
// Replaces the reference's MATMUL_Q shader (rust/src/kernels/matmul_q.wgsl:96-169,
// dispatched by rust/src/backend_wgpu.rs:646-695) for M <= 4 rows of activations:
//   y[m, n] = epilogue( scale[n] * sum_k x[m, k] * q[n, k] )
// with the MODE epilogues of matmul_q.wgsl:18-21 (0 plain, 1 GeGLU with a second
// weight, 2 gelu * column slice) plus MODE 3 (logit soft-cap).
//
// Design (B200, HBM-bound):
//  * Persistent CTAs, one per SM, each owning a contiguous range of weight rows;
//    registers and shared memory are sized so the next kernel's CTA fits beside
//    it and prefetches its own weights under programmatic dependent launch.
//    Rows are contiguous in the packed layout, so a CTA's work is one contiguous
//    byte range, streamed into shared memory by the TMA engine with 1-D bulk
//    copies (cp.async.bulk) through a ring of mbarrier-tracked stages. Copies for
//    the first stages are issued before griddepcontrol.wait, so under
//    programmatic dependent launch the weight stream of this kernel overlaps the
//    tail of the kernel that produces x.
//  * Inside a stage each row belongs to a group of lanes of one warp, which
//    reduces its sum with shuffles and runs the epilogue; warps progress
//    independently (no block barrier per stage) and the last warp to finish a
//    stage issues its refill.
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

#include "gemv_core.cuh"
#include "gq_internal.cuh"

namespace {

constexpr int kThreads = 256;        // narrow variant (two CTAs fit per SM)
constexpr int kWideThreads = 512;    // wide variant for CTAs that own many rows
constexpr int kMaxWarps = kWideThreads / 32;
// One CTA per SM is launched, but registers and shared memory are sized so that
// two fit: the next kernel's CTA (programmatic dependent launch) becomes
// resident while this one streams, and prefetches its own weights.
constexpr int kResident = 2;
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
  PeerDst peers;  // extra output destinations (peer buffers); n = 0: none
  int64_t ldy, y_col0;
  int row_bytes;    // bytes per packed row, multiple of 16
  int rows_per_cta; // contiguous rows per CTA
  int tile_rows;    // rows per pipeline stage (a multiple of the rows one pass covers)
  int stages;       // pipeline depth
  int lanes;        // lanes per row (power of two dividing row_bytes/16)
  double inv_k;     // 1 / K
  uint32_t *err;
  // Norm prologue (kernels built with PRO, one activation row): x is not read
  // from memory but made in the CTA as the decode step's residual add + RMSNorm
  // would make it, h = (pr + po * inv(po) * pw1) [* *ps], written to ph by CTA 0,
  // and x = pw2 ? h * inv(h) * pw2 : h, with inv(v) = 1 / sqrt(sum(v^2) / K + peps).
  const float *po, *pr, *pw1, *ps, *pw2;
  float *ph;
  float peps;
};

using gqcore::Fmt;
using gqcore::code_pos;
using gqcore::pow2f;
using gqcore::mac_chunk;

// Shared-memory carve-up, identical on host (sizing) and device (addressing).
struct GemvSmem {
  size_t stage_off, xs_off, bar_off, cnt_off, dscr_off, fscr_off, par_off, pro_off, total;
};
__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }
// pro_k: floats per row buffer of the norm prologue (four buffers), 0 = none.
__host__ __device__ inline GemvSmem gemv_layout(int bits, int mt, int nw, int row_bytes,
                                                int tile_rows, int stages, int pro_k = 0) {
  const int C = row_bytes / 16;
  const int per_chunk = 4 * (32 / bits);
  GemvSmem L;
  size_t o = 0;
  // per stage: NW packed weight tiles, then NW x {scale, code sum} per row
  L.stage_off = o; o = align16(o + (size_t)stages * nw * ((size_t)tile_rows * row_bytes + 2 * tile_rows * sizeof(float)));
  L.xs_off = o;    o = align16(o + (size_t)mt * C * (per_chunk + 4) * sizeof(float));
  L.bar_off = o;   o = align16(o + kMaxStages * sizeof(uint64_t));
  L.cnt_off = o;   o = align16(o + kMaxStages * sizeof(uint32_t));
  L.dscr_off = o;  o = align16(o + (size_t)kMaxWarps * mt * sizeof(double));
  L.fscr_off = o;  o = align16(o + (size_t)kMaxWarps * mt * sizeof(float));
  L.par_off = o;   o = align16(o + (size_t)mt * (sizeof(double) + 2 * sizeof(float)));
  L.pro_off = o;   o = align16(o + (size_t)4 * pro_k * sizeof(float) + 2 * sizeof(float));
  L.total = o;
  return L;
}

// ---- the kernel -----------------------------------------------------------------
// Work mapping: a row of C 16-byte chunks belongs to LANES consecutive lanes of
// one warp (LANES a power of two dividing C); lane li of the group takes chunks
// li, li+LANES, ... so a stage's rows are read as contiguous 16*LANES-byte runs.
// A lane group holds R consecutive rows at once (the x value loaded for a code
// position feeds all R rows), a warp holds 32/LANES groups, and the CTA walks
// the stage's rows in passes of WARPS*R*32/LANES. Row sums are reduced with
// shuffles inside the lane group; no block barrier is needed per stage: the last
// warp to finish a stage refills it.
template <int BITS, bool SIGNED, int MT, int MODE, int THREADS, int R, bool PRO = false>
__global__ void __launch_bounds__(THREADS, THREADS == kThreads ? kResident : 1) gemv_q_kernel(const GemvArgs a) {
  static_assert(!PRO || MT == 1, "the norm prologue makes one activation row");
  using F = Fmt<BITS>;
  constexpr int WARPS = THREADS / 32;
  constexpr int NW = (MODE == 1) ? 2 : 1;  // weights streamed together
  constexpr int NR = NW * R;               // packed rows per lane group
  constexpr int ACC = (MT * NR == 1) ? 4 : ((MT * NR) == 2 ? 2 : 1);

  extern __shared__ __align__(128) uint8_t smem[];
  const int C = a.row_bytes >> 4;  // chunks per row
  const int stage_bytes = a.tile_rows * a.row_bytes;                    // one weight's tile
  const int stage_stride = NW * (stage_bytes + 2 * a.tile_rows * 4);    // weights + row operands
  const int pro_k = PRO ? ((a.K + 3) & ~3) : 0;
  const GemvSmem L = gemv_layout(BITS, MT, NW, a.row_bytes, a.tile_rows, a.stages, pro_k);
  uint8_t *stage_buf = smem + L.stage_off;                        // [stages][NW][stage_bytes]
  float *xs = reinterpret_cast<float *>(smem + L.xs_off);         // [MT][C][kPad]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);  // [kMaxStages]
  uint32_t *done = reinterpret_cast<uint32_t *>(smem + L.cnt_off);  // [kMaxStages]
  double *dscr = reinterpret_cast<double *>(smem + L.dscr_off);   // [WARPS][MT]
  float *fscr = reinterpret_cast<float *>(smem + L.fscr_off);     // [WARPS][MT]
  double *pow2_s = reinterpret_cast<double *>(smem + L.par_off);  // [MT]
  float *mu_s = reinterpret_cast<float *>(pow2_s + MT);           // [MT]
  float *corr_s = mu_s + MT;                                      // [MT]

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int n_begin = blockIdx.x * a.rows_per_cta;
  const int n_end = min(a.N, n_begin + a.rows_per_cta);
  const int m0 = blockIdx.y * MT;
  const int nrows = n_end - n_begin;
  const int ntiles = nrows > 0 ? (nrows + a.tile_rows - 1) / a.tile_rows : 0;
  const int xs_mstride = C * F::kPad;
  const int lanes = a.lanes;                 // lanes per row (power of two)
  const int li = lane & (lanes - 1);         // lane within the row group
  const int grp = lane / lanes;              // row group within the warp
  const int gpw = 32 / lanes;                // row groups per warp
  const int rows_per_pass = WARPS * gpw * R;
  const int cpl = C / lanes;                 // chunks per lane per row

  // One stage = the packed rows of the tile plus their scales and code sums
  // (contiguous per tile; r0 is a multiple of 4 so every copy is 16-byte
  // aligned, and the allocations are padded past the last row).
  auto issue = [&](int t) {
    const int stage = t % a.stages;
    const int r0 = n_begin + t * a.tile_rows;
    const int rows = min(a.tile_rows, n_end - r0);
    const uint32_t bytes = (uint32_t)rows * (uint32_t)a.row_bytes;
    const uint32_t obytes = ((uint32_t)rows * 4u + 15u) & ~15u;
    uint64_t *bar = &bars[stage];
    gqd::mbar_arrive_expect_tx(bar, NW * (bytes + 2 * obytes));
    uint8_t *dst = stage_buf + (size_t)stage * stage_stride;
    float *ops = reinterpret_cast<float *>(dst + NW * stage_bytes);
    gqd::bulk_g2s(dst, a.w + (size_t)r0 * a.row_bytes, bytes, bar);
    gqd::bulk_g2s(ops, a.s + r0, obytes, bar);
    gqd::bulk_g2s(ops + a.tile_rows, a.qsum + r0, obytes, bar);
    if (NW == 2) {
      gqd::bulk_g2s(dst + stage_bytes, a.w2 + (size_t)r0 * a.row_bytes, bytes, bar);
      gqd::bulk_g2s(ops + 2 * a.tile_rows, a.s2 + r0, obytes, bar);
      gqd::bulk_g2s(ops + 3 * a.tile_rows, a.qsum2 + r0, obytes, bar);
    }
  };

  if (tid == 0) {
    for (int i = 0; i < a.stages; ++i) {
      gqd::mbar_init(&bars[i], 1);
      done[i] = 0;
    }
    gqd::fence_mbar_init();
  }
  __syncthreads();
  // Weights are immutable after upload: start streaming before the dependency wait.
  if (tid == 0)
    for (int t = 0; t < min(a.stages, ntiles); ++t) issue(t);

  // Let the next kernel's CTAs launch now: they co-reside (the narrow variant's
  // registers and shared memory are sized for two CTAs per SM) and prefetch
  // their own weights while this grid streams; they wait for this grid's
  // results in griddepcontrol.wait.
  gqd::griddep_launch_dependents();
  gqd::griddep_wait();

  // ---- norm prologue: the activation row made here (PRO) ------------------------
  // The arithmetic of the row-norm kernels (decode_ops.cu: add_norm_norm_kernel,
  // rmsnorm_reg_kernel): lane l of warp 0 sums the squares of elements
  // 4(l + 32i) .. +3 for i = 0, 1, ... in that order, then a butterfly over the
  // warp, so x equals what those kernels write, bit for bit. The four rows come
  // in with one round trip by every thread.
  const float *xsrc = nullptr;
  if constexpr (PRO) {
    float *bo = reinterpret_cast<float *>(smem + L.pro_off), *br = bo + pro_k, *bw1 = br + pro_k, *bw2 = bw1 + pro_k;
    const int n4 = a.K >> 2;
    const float4 one4 = make_float4(1.f, 1.f, 1.f, 1.f);
    for (int c = tid; c < n4; c += THREADS) {
      reinterpret_cast<float4 *>(bo)[c] = __ldcg(reinterpret_cast<const float4 *>(a.po) + c);
      reinterpret_cast<float4 *>(br)[c] = __ldcg(reinterpret_cast<const float4 *>(a.pr) + c);
      reinterpret_cast<float4 *>(bw1)[c] = __ldg(reinterpret_cast<const float4 *>(a.pw1) + c);
      reinterpret_cast<float4 *>(bw2)[c] = a.pw2 ? __ldg(reinterpret_cast<const float4 *>(a.pw2) + c) : one4;
    }
    const float sc = a.ps ? __ldg(a.ps) : 1.0f;
    __syncthreads();
    // warp 0 alone forms the row (no block barrier between the two norms): lane l
    // handles float4 chunks l, l + 32, ... of every row, the order in which the
    // norm kernels accumulate their per-lane sums of squares
    if (warp == 0) {
      auto butterfly = [&](float v) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        return v;
      };
      auto inv_of = [&](float ss) { return __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.peps))); };
      float ss = 0.0f;
      for (int c = lane; c < n4; c += 32) {
        const float4 t = reinterpret_cast<const float4 *>(bo)[c];
        ss = __fadd_rn(ss, __fmul_rn(t.x, t.x));
        ss = __fadd_rn(ss, __fmul_rn(t.y, t.y));
        ss = __fadd_rn(ss, __fmul_rn(t.z, t.z));
        ss = __fadd_rn(ss, __fmul_rn(t.w, t.w));
      }
      const float inv = inv_of(butterfly(ss));
      auto one = [&](float xx, float ww, float rr) {
        float n = __fadd_rn(rr, __fmul_rn(__fmul_rn(xx, inv), ww));
        if (a.ps) n = __fmul_rn(n, sc);
        return n;
      };
      const bool writer = blockIdx.x == 0 && blockIdx.y == 0;
      float ss2 = 0.0f;
      for (int c = lane; c < n4; c += 32) {
        const float4 o4 = reinterpret_cast<const float4 *>(bo)[c];
        const float4 w4 = reinterpret_cast<const float4 *>(bw1)[c];
        const float4 r4 = reinterpret_cast<const float4 *>(br)[c];
        const float4 h4 = make_float4(one(o4.x, w4.x, r4.x), one(o4.y, w4.y, r4.y), one(o4.z, w4.z, r4.z),
                                      one(o4.w, w4.w, r4.w));
        reinterpret_cast<float4 *>(br)[c] = h4;
        if (writer) reinterpret_cast<float4 *>(a.ph)[c] = h4;
        ss2 = __fadd_rn(ss2, __fmul_rn(h4.x, h4.x));
        ss2 = __fadd_rn(ss2, __fmul_rn(h4.y, h4.y));
        ss2 = __fadd_rn(ss2, __fmul_rn(h4.z, h4.z));
        ss2 = __fadd_rn(ss2, __fmul_rn(h4.w, h4.w));
      }
      if (a.pw2) {
        const float inv2 = inv_of(butterfly(ss2));
        for (int c = lane; c < n4; c += 32) {
          const float4 h4 = reinterpret_cast<const float4 *>(br)[c];
          const float4 w4 = reinterpret_cast<const float4 *>(bw2)[c];
          reinterpret_cast<float4 *>(bo)[c] =
              make_float4(__fmul_rn(__fmul_rn(h4.x, inv2), w4.x), __fmul_rn(__fmul_rn(h4.y, inv2), w4.y),
                          __fmul_rn(__fmul_rn(h4.z, inv2), w4.z), __fmul_rn(__fmul_rn(h4.w, inv2), w4.w));
        }
      }
    }
    __syncthreads();
    xsrc = a.pw2 ? bo : br;
  }
  auto ldx4 = [&](const float *p) -> float4 {
    if constexpr (PRO) return *reinterpret_cast<const float4 *>(p);
    else return __ldg(reinterpret_cast<const float4 *>(p));
  };

  // ---- stage x: x' = x - mu, scaled by 2^(S - pos) into the padded layout ----
  // One global read of x (held in registers up to kXv float4 per thread and row),
  // one (sum, max|x|) reduction for all MT rows giving mu and S (S leaves one
  // bit of headroom for |x - mu| <= 2 max|x|), then the scaled write. zp*sum(x')
  // is taken as sum(x) - K*mu in double (the per-element rounding of x - mu it
  // ignores is below 2^-24 relative).
  {
    constexpr int kXv = (THREADS == kThreads ? 6 : 3) / MT > 0 ? (THREADS == kThreads ? 6 : 3) / MT : 1;
    float4 xv[MT][kXv];
    double sx[MT];
    float mx[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      sx[m] = 0.0;
      mx[m] = 0.0f;
      const bool live = m0 + m < a.M;
      const float *xr = PRO ? xsrc : a.x + (size_t)(m0 + m) * a.ldx;
#pragma unroll
      for (int i = 0; i < kXv; ++i) {
        const int k = (tid + i * THREADS) * 4;
        xv[m][i] = (live && k < a.K) ? ldx4(xr + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      for (int k = (tid + kXv * THREADS) * 4; live && k < a.K; k += THREADS * 4) {
        const float4 v = ldx4(xr + k);
        sx[m] += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
        mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
#pragma unroll
      for (int i = 0; i < kXv; ++i) {
        const float4 v = xv[m][i];
        sx[m] += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
        mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sx[m] += __shfl_xor_sync(0xffffffffu, sx[m], o);
        mx[m] = fmaxf(mx[m], __shfl_xor_sync(0xffffffffu, mx[m], o));
      }
      if (lane == 0) {
        dscr[warp * MT + m] = sx[m];
        fscr[warp * MT + m] = mx[m];
      }
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      double sum = 0.0;
      float mxx = 0.0f;
#pragma unroll
      for (int i = 0; i < WARPS; ++i) {
        sum += dscr[i * MT + m];
        mxx = fmaxf(mxx, fscr[i * MT + m]);
      }
      const bool live = (m0 + m) < a.M;
      const float mu = live ? (float)(sum * a.inv_k) : 0.0f;
      int e = 0;
      if (mxx > 0.0f && isfinite(mxx)) frexpf(mxx, &e);  // mx < 2^e, so |x - mu| < 2^(e+1)
      int S = 125 - e;
      S = max(22, min(126, S));  // 2^(149-S) stays a normal f32 for the epilogue
      float *xm = xs + (size_t)m * xs_mstride;
      const float *xr = PRO ? xsrc : a.x + (size_t)(m0 + m) * a.ldx;
      auto put = [&](int k, float4 v) {
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) {
          const float vv[4] = {__fsub_rn(v.x, mu), __fsub_rn(v.y, mu), __fsub_rn(v.z, mu), __fsub_rn(v.w, mu)};
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i] = vv[i] * pow2f(S - code_pos<BITS>((k + i) % F::kPerWord));
        }
        *reinterpret_cast<float4 *>(xm + (k / F::kPerChunk) * F::kPad + (k % F::kPerChunk)) =
            make_float4(o[0], o[1], o[2], o[3]);
      };
#pragma unroll
      for (int i = 0; i < kXv; ++i) {
        const int k = (tid + i * THREADS) * 4;
        if (k < a.K) put(k, xv[m][i]);
      }
      for (int k = (tid + kXv * THREADS) * 4; k < a.K; k += THREADS * 4)
        put(k, live ? ldx4(xr + k) : make_float4(0.f, 0.f, 0.f, 0.f));
      if (tid == 0) {
        mu_s[m] = mu;
        const double sxp = live ? sum - (double)a.K * (double)mu : 0.0;
        // 2^(S-149) and 2^(149-S) built exactly from their exponent bits
        corr_s[m] = (float)((double)F::kZp * sxp * __longlong_as_double((long long)(1023 + S - 149) << 52));
        pow2_s[m] = __longlong_as_double((long long)(1023 + 149 - S) << 52);
      }
    }
  }
  __syncthreads();

  float mu_r[MT], corr_r[MT], p2_r[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    mu_r[m] = mu_s[m];
    corr_r[m] = corr_s[m];
    p2_r[m] = (float)pow2_s[m];
  }

  bool failed = false;
  for (int t = 0; t < ntiles; ++t) {
    const int stage = t % a.stages;
    const int r0 = n_begin + t * a.tile_rows;
    const int rows = min(a.tile_rows, n_end - r0);
    const uint8_t *buf = stage_buf + (size_t)stage * stage_stride;
    const float *ops = reinterpret_cast<const float *>(buf + NW * stage_bytes);  // [NW][scale|qsum][tile_rows]
    if (!gqd::mbar_wait_bounded(&bars[stage], (uint32_t)(t / a.stages) & 1u)) {
      failed = true;
      break;
    }
    // rows rr0 .. rr0+R-1 of the stage belong to this lane group in this pass
    for (int rr0 = (warp * gpw + grp) * R, base = warp * gpw * R; base < rows; rr0 += rows_per_pass,
             base += rows_per_pass) {
      // epilogue operands: scales and code sums arrived with the stage; the
      // MODE-2 slice value is issued now and used after the rows' MAC work
      float sc[NR], qs[NR], bsv[R][MT];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int rr = rr0 + i, n = r0 + rr;
        const bool live_row = rr < rows;
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          sc[i * NW + h] = live_row ? ops[(2 * h) * a.tile_rows + rr] : 0.f;
          qs[i * NW + h] = live_row ? ops[(2 * h + 1) * a.tile_rows + rr] : 0.f;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m)
          bsv[i][m] = (MODE == 2 && live_row && (li & (lanes / R - 1)) == 0 && m0 + m < a.M)
                          ? a.bs[(size_t)(m0 + m) * a.b_stride + a.b_off + n]
                          : 0.f;
      }
      float acc[NR][MT][ACC];
#pragma unroll
      for (int h = 0; h < NR; ++h)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int q = 0; q < ACC; ++q) acc[h][m][q] = 0.0f;
      // rows past the stage's end read (stale but in-bounds) stage bytes; their
      // sums are discarded below
      const uint8_t *rowp = buf + (size_t)min(rr0, a.tile_rows - R) * a.row_bytes;
      int j = 0;
      for (; j + 1 < cpl; j += 2) {  // two chunks in flight
        const int ca = li + j * lanes, cb = ca + lanes;
        uint4 wa[NR], wb[NR];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int h = 0; h < NW; ++h) {
            const uint8_t *p = rowp + h * stage_bytes + (size_t)i * a.row_bytes;
            wa[i * NW + h] = *reinterpret_cast<const uint4 *>(p + ca * 16);
            wb[i * NW + h] = *reinterpret_cast<const uint4 *>(p + cb * 16);
          }
        mac_chunk<BITS, SIGNED, MT, NR, ACC>(wa, xs + (size_t)ca * F::kPad, xs_mstride, acc);
        mac_chunk<BITS, SIGNED, MT, NR, ACC>(wb, xs + (size_t)cb * F::kPad, xs_mstride, acc);
      }
      if (j < cpl) {
        const int ca = li + j * lanes;
        uint4 wa[NR];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int h = 0; h < NW; ++h)
            wa[i * NW + h] =
                *reinterpret_cast<const uint4 *>(rowp + h * stage_bytes + (size_t)i * a.row_bytes + ca * 16);
        mac_chunk<BITS, SIGNED, MT, NR, ACC>(wa, xs + (size_t)ca * F::kPad, xs_mstride, acc);
      }
      // Row sums. The first log2(R) butterfly steps are transposing: the lanes
      // with bit o set keep the upper half of the rows and send the lower half,
      // so each step halves the values per lane; after them a lane holds one
      // row's partial (row index from its o-bits) and the rest is a plain
      // xor-reduction. R rows cost the shuffles of one, and R lanes run the
      // epilogue in parallel.
      float v[R][NW * MT];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int h = 0; h < NW; ++h)
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            float sum = acc[i * NW + h][m][0];
#pragma unroll
            for (int q = 1; q < ACC; ++q) sum += acc[i * NW + h][m][q];
            v[i][h * MT + m] = sum;
          }
      int o = lanes >> 1;
      int row_sel = 0;  // row (within the group's R) this lane ends up holding
#pragma unroll
      for (int nv = R; nv > 1; nv >>= 1) {
        const bool upper = (li & o) != 0;
#pragma unroll
        for (int i = 0; i < nv / 2; ++i)
#pragma unroll
          for (int q = 0; q < NW * MT; ++q) {
            const float send = upper ? v[i][q] : v[i + nv / 2][q];
            const float keep = upper ? v[i + nv / 2][q] : v[i][q];
            v[i][q] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        if (upper) row_sel += nv / 2;
        o >>= 1;
      }
      for (; o > 0; o >>= 1)
#pragma unroll
        for (int q = 0; q < NW * MT; ++q) v[0][q] += __shfl_xor_sync(0xffffffffu, v[0][q], o);
      if ((li & (lanes / R - 1)) == 0) {
        const int i = row_sel;
        const int rr = rr0 + i, n = r0 + rr;
        if (rr < rows) {
          // the lane's operands for row i (registers indexed by a runtime row:
          // select from the R candidates)
          float sc0 = sc[0], qs0 = qs[0], sc1 = sc[NW - 1], qs1 = qs[NW - 1];
          float bsr[MT];
#pragma unroll
          for (int m = 0; m < MT; ++m) bsr[m] = bsv[0][m];
#pragma unroll
          for (int k = 1; k < R; ++k)
            if (k == i) {
              sc0 = sc[k * NW];
              qs0 = qs[k * NW];
              sc1 = sc[k * NW + NW - 1];
              qs1 = qs[k * NW + NW - 1];
#pragma unroll
              for (int m = 0; m < MT; ++m) bsr[m] = bsv[k][m];
            }
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            if (m0 + m >= a.M) break;
            // ((sum - zp*sum(x')) * 2^(149-S) + mu * sum(q)) * scale, in f32: the
            // power-of-two factor is exact and the two terms are of the size of
            // the result
            const float v0 = __fmul_rn(__fmaf_rn(mu_r[m], qs0, __fmul_rn(__fsub_rn(v[0][m], corr_r[m]), p2_r[m])), sc0);
            float out;
            if (MODE == 1) {
              const float v1 =
                  __fmul_rn(__fmaf_rn(mu_r[m], qs1, __fmul_rn(__fsub_rn(v[0][MT + m], corr_r[m]), p2_r[m])), sc1);
              out = __fmul_rn(gqd::gelu_tanh(v0), v1);
            } else if (MODE == 2) {
              out = __fmul_rn(gqd::gelu_tanh(v0), bsr[m]);
            } else if (MODE == 3) {
              out = a.cap > 0.0f ? __fmul_rn(a.cap, tanhf(__fdiv_rn(v0, a.cap))) : v0;
            } else {
              out = v0;
            }
            a.y[(size_t)(m0 + m) * a.ldy + a.y_col0 + n] = out;
          }
        }
      }
    }
    // This warp is done reading the stage; the last warp to finish refills it.
    __syncwarp();
    if (lane == 0) {
      const uint32_t prev = atomicAdd(&done[stage], 1u);
      if (prev == WARPS - 1) {
        atomicExch(&done[stage], 0u);
        if (t + a.stages < ntiles) issue(t + a.stages);
      }
    }
  }

  // A timed-out wait leaves this warp; report it and drain (bounded) the copies
  // this CTA may still have in flight before its shared memory is released.
  const bool any_failed = __syncthreads_or(failed);
  if (!any_failed && (a.peers.n > 0 || a.peers.signal))
    gqd::push_to_peers(a.y + (size_t)m0 * a.ldy, a.peers, min(MT, a.M - m0), a.ldy, a.y_col0 + n_begin,
                       a.y_col0 + n_end);
  if (any_failed) {
    if (tid == 0) {
      gqd::report(a.err, GQ_DEVERR_WAIT_TIMEOUT);
      for (int s = 0; s < a.stages; ++s) (void)gqd::mbar_wait_bounded(&bars[s], 0u, 50000000ull);
      for (int s = 0; s < a.stages; ++s) (void)gqd::mbar_wait_bounded(&bars[s], 1u, 50000000ull);
    }
    __syncthreads();
  }
}

template <int BITS, bool SIGNED, int MT, int MODE, int THREADS, int R, bool PRO>
int launch_t(gq_ctx *ctx, const GemvArgs &a, dim3 grid, size_t smem) {
  auto kern = gemv_q_kernel<BITS, SIGNED, MT, MODE, THREADS, R, PRO>;
  static bool attr_set[64] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)ctx->smem_optin));
    if (const char *c = getenv("GQ_CARVEOUT"))
      GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, atoi(c)));
    attr_set[dev] = true;
  }
  GQ_CUDA_TRY(ctx, gq_launch(ctx, kern, grid, dim3(THREADS), smem, a));
  return GQ_OK;
}

template <int BITS, bool SIGNED, int MT, int MODE, bool PRO>
int launch_v(gq_ctx *ctx, bool wide, const GemvArgs &a, dim3 grid, size_t smem) {
  if (wide) return launch_t<BITS, SIGNED, MT, MODE, kWideThreads, MT == 1 ? 2 : 1, PRO>(ctx, a, grid, smem);
  return launch_t<BITS, SIGNED, MT, MODE, kThreads, 1, PRO>(ctx, a, grid, smem);
}

template <int BITS, bool SIGNED, int MT, bool PRO = false>
int launch_mode(gq_ctx *ctx, int mode, bool wide, const GemvArgs &a, dim3 grid, size_t smem) {
  switch (mode) {
    case 0: return launch_v<BITS, SIGNED, MT, 0, PRO>(ctx, wide, a, grid, smem);
    case 1: return launch_v<BITS, SIGNED, MT, 1, PRO>(ctx, wide, a, grid, smem);
    case 2: return launch_v<BITS, SIGNED, MT, 2, PRO>(ctx, wide, a, grid, smem);
    default: return launch_v<BITS, SIGNED, MT, 3, PRO>(ctx, wide, a, grid, smem);
  }
}

template <int BITS, bool SIGNED>
int launch_mt(gq_ctx *ctx, int mt, int mode, bool wide, const GemvArgs &a, dim3 grid, size_t smem, bool pro) {
  if (pro) return launch_mode<BITS, SIGNED, 1, true>(ctx, mode, wide, a, grid, smem);
  if (mt == 1) return launch_mode<BITS, SIGNED, 1>(ctx, mode, wide, a, grid, smem);
  if (mt == 2) return launch_mode<BITS, SIGNED, 2>(ctx, mode, wide, a, grid, smem);
  return launch_mode<BITS, SIGNED, 4>(ctx, mode, wide, a, grid, smem);
}

}  // namespace

// Shared memory the kernel needs for a configuration (bytes).
static size_t gemv_smem_bytes(int bits, int mt, int nw, int row_bytes, int tile_rows, int stages, int pro_k = 0) {
  return gemv_layout(bits, mt, nw, row_bytes, tile_rows, stages, pro_k).total;
}

// True when the CUDA-core GEMV handles this shape: whole 16-byte chunks per row,
// one scale per row (group == K), and x rows that fit in shared memory.
// Activation rows per pass (grid row): 1, 2 or 4 (more rows take several passes;
// a single 8-row pass measured slower on the E2B projections than the short-M
// tensor-core GEMV that takes 5 or more rows by default).
static int gemv_mt(gq_ctx *, const gq_qweight *, int64_t m, int) { return m <= 1 ? 1 : (m == 2 ? 2 : 4); }

bool gq_gemv_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m, int nw) {
  if (w->group_size != w->k || w->k <= 0 || w->n <= 0 || m <= 0) return false;
  if (w->row_bytes % 16 != 0 || w->row_bytes > 65536) return false;
  if (w->n > (1ll << 30)) return false;
  const int mt = gemv_mt(ctx, w, m, nw);
  if (w->k % 4 != 0) return false;
  int lanes = 32;
  while ((w->row_bytes / 16) % lanes != 0) lanes >>= 1;
  // the wide variant has the SM's shared memory to itself
  return gemv_smem_bytes(w->bits, mt, nw, (int)w->row_bytes, (kThreads / 32) * (32 / lanes), 2) <=
         ctx->smem_optin - 1024;
}

bool gq_gemv_r1_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m, int nw);
int gq_gemv_r1_launch(gq_ctx *ctx, int mode, const float *x, const gq_qweight *w, const gq_qweight *w2,
                      const float *bs, int64_t b_off, float cap, float *y, int64_t y_col0);

// The norm prologue's inputs (one activation row; see GemvArgs::po).
struct GemvPro {
  const float *o, *r, *w1, *s, *w2;
  float *h;
  float eps;
};

// mode: 0 plain, 1 geglu (w2 = up), 2 gelu * bs slice, 3 soft-cap. pro: x made
// in the kernel by the norm prologue (m = 1, x unused).
static int gemv_launch_impl(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w,
                            const gq_qweight *w2, const float *bs, int64_t b_stride, int64_t b_off,
                            float cap, float *y, int64_t ldy, int64_t y_col0, const GemvPro *pro) {
  const int nw = (mode == 1) ? 2 : 1;
  // one activation row: the register-x kernel (gemv_r1.cu) where its shape rules hold
  if (!pro && m == 1 && (uintptr_t)x % 16 == 0 && gq_gemv_r1_supported(ctx, w, m, nw))
    return gq_gemv_r1_launch(ctx, mode, x, w, w2, bs, b_off, cap, y, y_col0);
  const int mt = pro ? 1 : gemv_mt(ctx, w, m, nw);
  const int pro_k = pro ? (int)((w->k + 3) & ~int64_t(3)) : 0;
  const int rb = (int)w->row_bytes;
  const int C = rb / 16;
  GemvArgs a = {};
  a.x = x;
  if (pro) {
    a.po = pro->o;
    a.pr = pro->r;
    a.pw1 = pro->w1;
    a.ps = pro->s;
    a.pw2 = pro->w2;
    a.ph = pro->h;
    a.peps = pro->eps;
  }
  a.ldx = w->k;
  a.M = (int)m;
  a.K = (int)w->k;
  a.N = (int)w->n;
  a.w = w->bytes;
  a.s = w->scales;
  a.qsum = w->scales + w->qsum_off;  // per-row code sums, 16-byte aligned after the scales
  if (w2) {
    a.w2 = w2->bytes;
    a.s2 = w2->scales;
    a.qsum2 = w2->scales + w2->qsum_off;
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
  a.peers = ctx->peers;

  // Grid: one CTA per SM over contiguous row ranges.
  // (a multiple of 4 rows, so each tile's scale copy starts 16-byte aligned)
  int rows_per_cta = (int)((w->n + ctx->num_sms - 1) / ctx->num_sms);
  rows_per_cta = (rows_per_cta + 3) & ~3;
  const int gx = (int)((w->n + rows_per_cta - 1) / rows_per_cta);
  int max_lanes = 32;
  while (C % max_lanes != 0) max_lanes >>= 1;

  // Two variants: narrow (256 threads, one row per lane group, sized so the next
  // kernel's CTA co-resides and prefetches under PDL) for CTAs that own < 8 rows;
  // wide (512 threads, two rows per lane group, the SM to itself)
  // otherwise, where latency hiding matters more.
  auto plan = [&](bool wide, int &lanes, int &tile_rows, int &stages, size_t &smem) -> bool {
    const int warps = (wide ? kWideThreads : kThreads) / 32;
    const int R = (wide && mt == 1) ? 2 : 1;
    const size_t cap = wide ? ctx->smem_optin - 1024 : ctx->smem_optin / kResident - 1024;
    // Lanes per row: a power of two dividing the chunk count. Fewer lanes per
    // row amortise the row's shuffle reduction and epilogue over more chunks per
    // lane and let row groups share the shared-memory reads of x; more lanes per
    // row keep all warps busy when a CTA owns few rows. Take the fewest lanes
    // (>= 4) whose passes fit a 48 KB stage and are at least 85% occupied.
    lanes = -1;
    for (int l = 4; l <= max_lanes; l <<= 1) {
      if (C % l != 0) continue;
      const int rpp = warps * (32 / l) * R;
      if ((size_t)rpp * rb * nw > 48 * 1024 || gemv_smem_bytes(w->bits, mt, nw, rb, rpp, 2, pro_k) > cap) continue;
      const int passes = (rows_per_cta + rpp - 1) / rpp;
      if (rows_per_cta >= (int)(0.85 * passes * rpp) || l == max_lanes) {
        lanes = l;
        break;
      }
    }
    if (lanes < 0) {  // nothing fits the 48 KB stage budget: one pass per stage at max lanes
      lanes = max_lanes;
      if (gemv_smem_bytes(w->bits, mt, nw, rb, warps * (32 / lanes) * R, 1, pro_k) > cap) return false;
    }
    const int rows_per_pass = warps * (32 / lanes) * R;
    // Stage size: whole passes, >= 24 KB per copy where the rows allow (large
    // bulk copies stream fastest), <= 48 KB per stage.
    int passes = 1;
    while ((passes + 1) * rows_per_pass * rb * nw <= 48 * 1024 && passes * rows_per_pass * rb < 24 * 1024) ++passes;
    tile_rows = passes * rows_per_pass;
    if (tile_rows > rows_per_cta) tile_rows = ((rows_per_cta + rows_per_pass - 1) / rows_per_pass) * rows_per_pass;
    const int ntiles = (rows_per_cta + tile_rows - 1) / tile_rows;
    stages = min(kMaxStages, ntiles);
    smem = gemv_smem_bytes(w->bits, mt, nw, rb, tile_rows, stages, pro_k);
    while (smem > cap && (stages > 1 || tile_rows > rows_per_pass)) {
      if (stages > 2 || (stages > 1 && tile_rows == rows_per_pass)) --stages;
      else tile_rows -= rows_per_pass;
      smem = gemv_smem_bytes(w->bits, mt, nw, rb, tile_rows, stages, pro_k);
    }
    return smem <= cap && tile_rows >= 1 && stages >= 1;
  };
  int lanes = 0, tile_rows = 0, stages = 0;
  size_t smem = 0;
  // Wide whenever a CTA owns a few row pairs: its 16 warps hide the dependent
  // LDS/FFMA chains far better than the co-resident narrow CTA gains from
  // prefetching under the previous kernel (measured on the E2B projections).
  // (for one activation row the wide variant holds 2 rows per >= 2-lane group)
  bool wide = rows_per_cta >= 8 && (mt > 1 || max_lanes >= 4);
  if (wide && !plan(true, lanes, tile_rows, stages, smem)) wide = false;
  if (!wide && !plan(false, lanes, tile_rows, stages, smem)) {
    // x rows too long for the narrow variant's half of the SM: the wide one
    wide = mt > 1 || max_lanes >= 4;
    if (!wide || !plan(true, lanes, tile_rows, stages, smem))
      return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "gemv: no stage configuration fits shared memory");
  }
  a.rows_per_cta = rows_per_cta;
  a.tile_rows = tile_rows;
  a.stages = stages;
  a.lanes = lanes;
  a.inv_k = 1.0 / (double)w->k;
  dim3 grid(gx, (unsigned)((m + mt - 1) / mt));
  const bool p = pro != nullptr;
  if (w->bits == 4) return launch_mt<4, false>(ctx, mt, mode, wide, a, grid, smem, p);
  if (w->bits == 2) return launch_mt<2, false>(ctx, mt, mode, wide, a, grid, smem, p);
  if (w->signed_i8) return launch_mt<8, true>(ctx, mt, mode, wide, a, grid, smem, p);
  return launch_mt<8, false>(ctx, mt, mode, wide, a, grid, smem, p);
}

int gq_gemv_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w,
                   const gq_qweight *w2, const float *bs, int64_t b_stride, int64_t b_off,
                   float cap, float *y, int64_t ldy, int64_t y_col0) {
  return gemv_launch_impl(ctx, mode, x, m, w, w2, bs, b_stride, b_off, cap, y, ldy, y_col0, nullptr);
}

// One activation row made by the norm prologue, then the streaming GEMV (modes 0-2;
// bs: the MODE-2 row, its columns from b_off). Arguments checked by the caller.
int gq_gemv_pro_launch(gq_ctx *ctx, int mode, const float *o, const float *r, const float *w1, const float *s,
                       const float *w2n, float eps, float *h, const gq_qweight *w, const gq_qweight *wu,
                       const float *bs, int64_t b_off, float *y) {
  const GemvPro pro = {o, r, w1, s, w2n, h, eps};
  return gemv_launch_impl(ctx, mode, nullptr, 1, w, wu, bs, 0, b_off, 0.0f, y, w->n, 0, &pro);
}
