// gemv_r1.cu — decode GEMV for one activation row (M = 1), x held in registers.
//
// Replaces the reference's MATMUL_Q shader at M = 1 (rust/src/kernels/matmul_q.wgsl:96-169,
// dispatched by rust/src/backend_wgpu.rs:646-695) for the per-layer projections of a
// decode step: y[n] = epilogue(scale[n] * sum_k x[k] * q[n, k]) with the MODE epilogues
// of matmul_q.wgsl:18-21 (0 plain, 1 GeGLU with a second weight, 2 gelu * column slice)
// plus MODE 3 (logit soft-cap).
//
// Why a second M = 1 kernel. A decode step is a chain of dependent launches of 0.4-9 MB
// projections; each costs a fixed ~2 us on B200 (the programmatic-dependent-launch
// release plus one L2 round trip for x, measured with an empty kernel of the same
// grid), so what matters is the time a launch adds on top. The shared-memory GEMV
// (gemv_q.cu) stages x through shared memory behind two block barriers and reads it
// back per weight chunk (for 4-bit codes 8 bytes of x per byte of weights), which
// leaves its warps stalled on shared-memory loads. Here:
//  * every warp reads the x values its lanes need straight from global memory into
//    registers (at most 64 per lane) and keeps them for all its rows: the only
//    shared-memory traffic of the MAC loop is the weights, one conflict-free 32-bit
//    load per lane per word;
//  * a CTA's whole row slice (weights, scales, code sums) fits in shared memory and
//    arrives by a few bulk copies issued before the dependency wait; the slice is
//    sized so two CTAs fit per SM, so the next kernel's CTA becomes resident early
//    (programmatic dependent launch) and streams its weights under this one;
//  * one block barrier per launch (the mean and max|x| of the row), plus one more
//    when a row's K range is split over several warps.
// Arithmetic is that of gemv_q.cu (exact power-of-two pre-scaling of x - mean, codes
// masked in place and read as f32 subnormals, LOP3 + FFMA per code, the zero point
// and the mean restored in the epilogue), so results agree with it to rounding of
// the accumulation order.
//
// Work mapping: a row is W 32-bit words. The K range is split into S segments
// (S in {1, 2, 4, 8}); warp w owns segment w % S of the rows g, g + G, ... with
// g = w / S and G = 8 / S; lane l of a warp owns words l, l + 32, ... of the segment,
// WPL words in all (a compile-time count), and holds the WPL * (32 / BITS) x values
// of those words.
#include <cuda_runtime.h>
#include <math.h>

#include "gq_internal.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxX = 64;  // x values held per lane

template <int BITS>
struct R1Fmt {
  static constexpr int kPerWord = 32 / BITS;   // codes per 32-bit word
  static constexpr int kZp = 1 << (BITS - 1);  // offset-binary zero point
  // codes [0, kSplit) are masked straight out of the word, the rest out of the word
  // shifted right by kShift, so every field stays inside f32 bits 0..22
  static constexpr int kSplit = BITS == 4 ? 5 : (BITS == 2 ? 11 : 2);
  static constexpr int kShift = BITS == 4 ? 12 : 16;
};

template <int BITS>
__host__ __device__ constexpr int r1_pos(int j) {
  return j < R1Fmt<BITS>::kSplit ? j * BITS : j * BITS - R1Fmt<BITS>::kShift;
}

__device__ __forceinline__ float r1_pow2f(int e) { return __int_as_float((e + 127) << 23); }

struct R1Args {
  const float *x;
  int K, N;
  const uint8_t *w;
  const float *s;
  const float *qsum;
  const uint8_t *w2;
  const float *s2;
  const float *qsum2;
  const float *bs;
  int64_t b_off;
  float cap;
  float *y;
  int64_t y_col0;
  int row_bytes;     // bytes per packed row, multiple of 128
  int rows_per_cta;  // multiple of 4
  int splits;        // K segments per row (warps sharing a row)
  double inv_k;
  uint32_t *err;
};

struct R1Smem {
  size_t w_off, ops_off, bar_off, red_off, part_off, total;
};

__host__ __device__ inline size_t r1_align16(size_t v) { return (v + 15) & ~size_t(15); }

__host__ __device__ inline R1Smem r1_layout(int nw, int rows_per_cta, int row_bytes, int splits) {
  R1Smem L;
  size_t o = 0;
  L.w_off = o;    o = r1_align16(o + (size_t)nw * rows_per_cta * row_bytes);
  L.ops_off = o;  o = r1_align16(o + (size_t)nw * 2 * rows_per_cta * sizeof(float));  // scale, code sum
  L.bar_off = o;  o = r1_align16(o + sizeof(uint64_t));
  L.red_off = o;  o = r1_align16(o + (size_t)kWarps * (sizeof(double) + sizeof(float)));
  L.part_off = o; o = r1_align16(o + (splits > 1 ? (size_t)nw * splits * rows_per_cta * sizeof(float) : 0));
  L.total = o;
  return L;
}

template <int BITS, bool SIGNED, int WPL, int MODE>
__global__ void __launch_bounds__(kThreads, 2) gemv_r1_kernel(const R1Args a) {
  using F = R1Fmt<BITS>;
  constexpr int CPW = F::kPerWord;
  constexpr int NX = WPL * CPW;  // x values per lane
  static_assert(NX <= kMaxX, "x slice exceeds the register budget");
  constexpr int NW = MODE == 1 ? 2 : 1;
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  constexpr uint32_t kXor = (BITS == 8 && SIGNED) ? 0x80808080u : 0u;
  constexpr int ACC = CPW >= 4 ? 2 : 1;  // independent FFMA chains per row

  extern __shared__ __align__(128) uint8_t smem[];
  const R1Smem L = r1_layout(NW, a.rows_per_cta, a.row_bytes, a.splits);
  const uint8_t *wsm = smem + L.w_off;                              // [NW][rows][row_bytes]
  float *ops = reinterpret_cast<float *>(smem + L.ops_off);         // [NW][scale | qsum][rows]
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  double *red_sum = reinterpret_cast<double *>(smem + L.red_off);   // [kWarps]
  float *red_max = reinterpret_cast<float *>(red_sum + kWarps);     // [kWarps]
  float *part = reinterpret_cast<float *>(smem + L.part_off);       // [NW][splits][rows]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * a.rows_per_cta;
  const int rows = min(a.N - n0, a.rows_per_cta);
  const int S = a.splits, G = kWarps / S;
  const int seg = warp % S, grp = warp / S;
  const int words = a.row_bytes >> 2;
  const int word0 = seg * (words / S);

  if (tid == 0) {
    gqd::mbar_init(bar, 1);
    gqd::fence_mbar_init();
  }
  __syncthreads();
  // Weights, scales and code sums are immutable after upload: fetch the CTA's whole
  // slice before the dependency wait (n0 is a multiple of 4, so every copy starts
  // 16-byte aligned; the allocations are padded past the last row).
  if (tid == 0) {
    const uint32_t wbytes = (uint32_t)rows * (uint32_t)a.row_bytes;
    const uint32_t obytes = ((uint32_t)rows * 4u + 15u) & ~15u;
    gqd::mbar_arrive_expect_tx(bar, NW * (wbytes + 2 * obytes));
    gqd::bulk_g2s(const_cast<uint8_t *>(wsm), a.w + (size_t)n0 * a.row_bytes, wbytes, bar);
    gqd::bulk_g2s(ops, a.s + n0, obytes, bar);
    gqd::bulk_g2s(ops + a.rows_per_cta, a.qsum + n0, obytes, bar);
    if (NW == 2) {
      gqd::bulk_g2s(const_cast<uint8_t *>(wsm) + (size_t)a.rows_per_cta * a.row_bytes,
                    a.w2 + (size_t)n0 * a.row_bytes, wbytes, bar);
      gqd::bulk_g2s(ops + 2 * a.rows_per_cta, a.s2 + n0, obytes, bar);
      gqd::bulk_g2s(ops + 3 * a.rows_per_cta, a.qsum2 + n0, obytes, bar);
    }
  }
  gqd::griddep_launch_dependents();
  gqd::griddep_wait();

  // ---- x: this lane's values of its segment, straight into registers ----------------
  float xr[NX];
#pragma unroll
  for (int j = 0; j < WPL; ++j) {
    const float4 *src = reinterpret_cast<const float4 *>(a.x + (size_t)(word0 + lane + 32 * j) * CPW);
#pragma unroll
    for (int q = 0; q < CPW / 4; ++q) {
      const float4 v = __ldg(src + q);
      xr[j * CPW + 4 * q + 0] = v.x;
      xr[j * CPW + 4 * q + 1] = v.y;
      xr[j * CPW + 4 * q + 2] = v.z;
      xr[j * CPW + 4 * q + 3] = v.w;
    }
  }
  // the row's sum (double) and max|x|: each segment's first warp contributes once
  {
    double sx = 0.0;
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < NX; i += 4) {
      sx += ((double)xr[i] + (double)xr[i + 1]) + ((double)xr[i + 2] + (double)xr[i + 3]);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(xr[i]), fabsf(xr[i + 1])), fmaxf(fabsf(xr[i + 2]), fabsf(xr[i + 3]))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sx += __shfl_xor_sync(0xffffffffu, sx, o);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0 && grp == 0) {
      red_sum[seg] = sx;
      red_max[seg] = mx;
    }
  }
  __syncthreads();
  double sum = 0.0;
  float mxx = 0.0f;
  for (int i = 0; i < S; ++i) {
    sum += red_sum[i];
    mxx = fmaxf(mxx, red_max[i]);
  }
  const float mu = (float)(sum * a.inv_k);
  int e = 0;
  if (mxx > 0.0f && isfinite(mxx)) frexpf(mxx, &e);  // max|x| < 2^e, so |x - mu| < 2^(e+1)
  const int Sx = max(22, min(126, 125 - e));          // 2^(149-Sx) stays a normal f32
  const double sxp = sum - (double)a.K * (double)mu;  // sum(x - mu) (rounding of x - mu below 2^-24 rel)
  const float corr = (float)((double)F::kZp * sxp * __longlong_as_double((long long)(1023 + Sx - 149) << 52));
  const float p2 = (float)__longlong_as_double((long long)(1023 + 149 - Sx) << 52);
#pragma unroll
  for (int i = 0; i < NX; ++i) xr[i] = __fmul_rn(__fsub_rn(xr[i], mu), r1_pow2f(Sx - r1_pos<BITS>(i % CPW)));

  // ---- the weights of the slice ---------------------------------------------------------
  const bool ok = gqd::mbar_wait_bounded(bar, 0u);

  auto epilogue = [&](int r, float v0raw, float v1raw) {
    const int n = n0 + r;
    const float v0 = __fmul_rn(__fmaf_rn(mu, ops[a.rows_per_cta + r], __fmul_rn(__fsub_rn(v0raw, corr), p2)), ops[r]);
    float out;
    if (MODE == 1) {
      const float v1 = __fmul_rn(__fmaf_rn(mu, ops[3 * a.rows_per_cta + r], __fmul_rn(__fsub_rn(v1raw, corr), p2)),
                                 ops[2 * a.rows_per_cta + r]);
      out = __fmul_rn(gqd::gelu_tanh(v0), v1);
    } else if (MODE == 2) {
      out = __fmul_rn(gqd::gelu_tanh(v0), a.bs[a.b_off + n]);
    } else if (MODE == 3) {
      out = a.cap > 0.0f ? __fmul_rn(a.cap, tanhf(__fdiv_rn(v0, a.cap))) : v0;
    } else {
      out = v0;
    }
    a.y[a.y_col0 + n] = out;
  };

  // Four rows of the warp at a time: their FFMA chains interleave, and their sums
  // are reduced together by a transposing butterfly (the first two steps halve the
  // values per lane, after which each lane holds one row), so four rows cost the
  // shuffles of one and four lanes run the epilogues.
  constexpr int R = 4;
  if (ok) {
    for (int j0 = 0; grp + G * j0 < rows; j0 += R) {
      float acc[R][NW][ACC];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int h = 0; h < NW; ++h)
#pragma unroll
          for (int q = 0; q < ACC; ++q) acc[i][h][q] = 0.0f;
#pragma unroll
      for (int h = 0; h < NW; ++h) {
        const uint32_t *wrow[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
          // rows past the slice's end read (stale, in-bounds) shared memory; their
          // sums are discarded below
          const int rl = min(grp + G * (j0 + i), a.rows_per_cta - 1);
          wrow[i] = reinterpret_cast<const uint32_t *>(wsm + ((size_t)h * a.rows_per_cta + rl) * a.row_bytes) +
                    word0 + lane;
        }
#pragma unroll
        for (int j = 0; j < WPL; ++j) {
          uint32_t wv[R];
#pragma unroll
          for (int i = 0; i < R; ++i) wv[i] = wrow[i][32 * j];
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const uint32_t lo = wv[i] ^ kXor;
            const uint32_t hi = lo >> F::kShift;
#pragma unroll
            for (int c = 0; c < CPW; ++c) {
              const float fld = __uint_as_float(((c < F::kSplit) ? lo : hi) & (kMask << r1_pos<BITS>(c)));
              acc[i][h][c % ACC] = __fmaf_rn(xr[j * CPW + c], fld, acc[i][h][c % ACC]);
            }
          }
        }
      }
      float v[R][NW];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          float t = acc[i][h][0];
#pragma unroll
          for (int q = 1; q < ACC; ++q) t += acc[i][h][q];
          v[i][h] = t;
        }
      const bool up16 = (lane & 16) != 0, up8 = (lane & 8) != 0;
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          const float send = up16 ? v[i][h] : v[i + 2][h];
          const float keep = up16 ? v[i + 2][h] : v[i][h];
          v[i][h] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
#pragma unroll
      for (int h = 0; h < NW; ++h) {
        const float send = up8 ? v[0][h] : v[1][h];
        const float keep = up8 ? v[1][h] : v[0][h];
        v[0][h] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) v[0][h] += __shfl_xor_sync(0xffffffffu, v[0][h], o);
      }
      const int r = grp + G * (j0 + (up16 ? 2 : 0) + (up8 ? 1 : 0));
      if ((lane & 7) == 0 && r < rows) {
        if (S == 1) {
          epilogue(r, v[0][0], v[0][NW - 1]);
        } else {
#pragma unroll
          for (int h = 0; h < NW; ++h) part[((size_t)h * S + seg) * a.rows_per_cta + r] = v[0][h];
        }
      }
    }
  }
  if (S > 1) {
    __syncthreads();
    if (ok)
      for (int r = tid; r < rows; r += kThreads) {
        float v[NW];
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          float t = 0.0f;
          for (int i = 0; i < S; ++i) t += part[((size_t)h * S + i) * a.rows_per_cta + r];
          v[h] = t;
        }
        epilogue(r, v[0], v[NW - 1]);
      }
  }
  if (!ok && tid == 0) {
    // a timed-out wait: report it and let the copy drain (bounded) before the
    // shared memory is released
    gqd::report(a.err, GQ_DEVERR_WAIT_TIMEOUT);
    (void)gqd::mbar_wait_bounded(bar, 0u, 50000000ull);
  }
}

template <int BITS, bool SIGNED, int WPL, int MODE>
int r1_launch_t(gq_ctx *ctx, const R1Args &a, dim3 grid, size_t smem) {
  auto kern = gemv_r1_kernel<BITS, SIGNED, WPL, MODE>;
  static bool attr_set[64] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ctx->smem_optin));
    // the largest shared-memory carveout, as the other decode GEMVs get from their
    // large dynamic shared memory, so consecutive launches need no SM reconfiguration
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          (int)cudaSharedmemCarveoutMaxShared));
    attr_set[dev] = true;
  }
  GQ_CUDA_TRY(ctx, gq_launch(ctx, kern, grid, dim3(kThreads), smem, a));
  return GQ_OK;
}

template <int BITS, bool SIGNED, int WPL>
int r1_launch_mode(gq_ctx *ctx, int mode, const R1Args &a, dim3 grid, size_t smem) {
  switch (mode) {
    case 0: return r1_launch_t<BITS, SIGNED, WPL, 0>(ctx, a, grid, smem);
    case 1: return r1_launch_t<BITS, SIGNED, WPL, 1>(ctx, a, grid, smem);
    case 2: return r1_launch_t<BITS, SIGNED, WPL, 2>(ctx, a, grid, smem);
    default: return r1_launch_t<BITS, SIGNED, WPL, 3>(ctx, a, grid, smem);
  }
}

// Words-per-lane counts compiled for each width (x values per lane <= 64).
template <int BITS, bool SIGNED>
int r1_launch_wpl(gq_ctx *ctx, int wpl, int mode, const R1Args &a, dim3 grid, size_t smem) {
  switch (wpl) {
    case 1: return r1_launch_mode<BITS, SIGNED, 1>(ctx, mode, a, grid, smem);
    case 2: return r1_launch_mode<BITS, SIGNED, 2>(ctx, mode, a, grid, smem);
    case 3: return r1_launch_mode<BITS, SIGNED, 3>(ctx, mode, a, grid, smem);
    case 4: return r1_launch_mode<BITS, SIGNED, 4>(ctx, mode, a, grid, smem);
    default: break;
  }
  if constexpr (BITS != 2) {
    if (wpl == 6) return r1_launch_mode<BITS, SIGNED, 6>(ctx, mode, a, grid, smem);
    if (wpl == 8) return r1_launch_mode<BITS, SIGNED, 8>(ctx, mode, a, grid, smem);
  }
  if constexpr (BITS == 8) {
    if (wpl == 12) return r1_launch_mode<BITS, SIGNED, 12>(ctx, mode, a, grid, smem);
    if (wpl == 16) return r1_launch_mode<BITS, SIGNED, 16>(ctx, mode, a, grid, smem);
  }
  return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "gemv_r1: no kernel for this row length");
}

bool r1_wpl_compiled(int bits, int wpl) {
  if (wpl >= 1 && wpl <= 4) return true;
  if ((wpl == 6 || wpl == 8) && bits != 2) return true;
  return (wpl == 12 || wpl == 16) && bits == 8;
}

struct R1Plan {
  int rows_per_cta = 0, gx = 0, splits = 0, wpl = 0;
  size_t smem = 0;
};

// Grid, K split and shared memory of a shape, or false when the kernel does not
// apply (the shared-memory GEMV takes it then).
bool r1_plan(const gq_ctx *ctx, const gq_qweight *w, int nw, R1Plan *p) {
  if (w->group_size != w->k || w->k <= 0 || w->n <= 0 || w->n > (1ll << 30)) return false;
  if (w->bits == 8 && !w->signed_i8) return false;  // U8 8-bit tables: the shared-memory GEMV
  if (w->row_bytes % 128 != 0 || w->row_bytes > 65536) return false;
  const int words = (int)(w->row_bytes / 4);
  const int cpw = 32 / w->bits;
  int rows = (int)((w->n + ctx->num_sms - 1) / ctx->num_sms);
  rows = (rows + 3) & ~3;
  // the cheapest K split: per-warp work in passes of four rows (ceil(rows * S / 8)
  // rows, rounded up to four) of words / S words, plus a small charge for the
  // partial-sum exchange of a split row; ties to fewer splits
  int best = 0;
  long best_cost = 0;
  for (int s = 1; s <= kWarps; s <<= 1) {
    if (words % (32 * s) != 0) continue;
    const int wpl = words / (32 * s);
    if (wpl * cpw > kMaxX || !r1_wpl_compiled(w->bits, wpl)) continue;
    const long per_warp = (rows * s + kWarps - 1) / kWarps;                  // rows per warp
    const long cost = ((per_warp + 3) / 4) * 4 * (words / s) + (s > 1 ? words / 8 : 0);  // four-row passes
    if (best == 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  if (best == 0) return false;
  const size_t smem = r1_layout(nw, rows, (int)w->row_bytes, best).total;
  // two CTAs per SM (the next kernel's CTA co-resides and prefetches) or at most one
  if (smem > ctx->smem_optin - 1024) return false;
  p->rows_per_cta = rows;
  p->gx = (int)((w->n + rows - 1) / rows);
  p->splits = best;
  p->wpl = words / (32 * best);
  p->smem = smem;
  return true;
}

// GQ_GEMV_R1=1 sends every supported M = 1 shape here, =0 none; by default the
// shapes whose CTAs have little MAC work (measured in the E2B decode chain: the
// per-layer-input gate [256, 1536] and projection [1536, 256], 2.6 -> 2.1 and
// 2.8 -> 2.3 us per launch), where the shared-memory GEMV's x staging dominates. With
// more work per CTA the shared-memory GEMV's 16 warps finish sooner (e.g. the 4-bit
// gate|up pair: 5.4 us there, 8.6 us here).
int r1_mode() {
  const char *e = getenv("GQ_GEMV_R1");
  return (e && *e) ? (e[0] == '1' ? 1 : 0) : 2;
}
constexpr int64_t kR1SmallWork = 8192;  // codes per CTA (rows x K x weights) below which it wins

}  // namespace

// True when the register-x GEMV takes this M = 1 shape (GQ_GEMV_R1 read per call,
// so tests compare both kernels).
bool gq_gemv_r1_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m, int nw) {
  const int mode = r1_mode();
  if (m != 1 || mode == 0 || ctx->peers.n > 0 || ctx->peers.signal) return false;
  R1Plan p;
  if (!r1_plan(ctx, w, nw, &p)) return false;
  return mode == 1 || (int64_t)p.rows_per_cta * w->k * nw <= kR1SmallWork;
}

// mode: 0 plain, 1 geglu (w2 = up), 2 gelu * bs slice, 3 soft-cap. One activation row.
int gq_gemv_r1_launch(gq_ctx *ctx, int mode, const float *x, const gq_qweight *w, const gq_qweight *w2,
                      const float *bs, int64_t b_off, float cap, float *y, int64_t y_col0) {
  const int nw = mode == 1 ? 2 : 1;
  R1Plan p;
  if (!r1_plan(ctx, w, nw, &p)) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "gemv_r1: shape not supported");
  if ((uintptr_t)x % 16 != 0) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "gemv_r1: x must be 16-byte aligned");
  R1Args a = {};
  a.x = x;
  a.K = (int)w->k;
  a.N = (int)w->n;
  a.w = w->bytes;
  a.s = w->scales;
  a.qsum = w->scales + w->qsum_off;
  if (w2) {
    a.w2 = w2->bytes;
    a.s2 = w2->scales;
    a.qsum2 = w2->scales + w2->qsum_off;
  }
  a.bs = bs;
  a.b_off = b_off;
  a.cap = cap;
  a.y = y;
  a.y_col0 = y_col0;
  a.row_bytes = (int)w->row_bytes;
  a.rows_per_cta = p.rows_per_cta;
  a.splits = p.splits;
  a.inv_k = 1.0 / (double)w->k;
  a.err = ctx->dev_err;
  const dim3 grid(p.gx);
  if (w->bits == 4) return r1_launch_wpl<4, false>(ctx, p.wpl, mode, a, grid, p.smem);
  if (w->bits == 2) return r1_launch_wpl<2, false>(ctx, p.wpl, mode, a, grid, p.smem);
  return r1_launch_wpl<8, true>(ctx, p.wpl, mode, a, grid, p.smem);
}
