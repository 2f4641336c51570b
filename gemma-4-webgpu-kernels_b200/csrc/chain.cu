// chain.cu — a decode chain: consecutive one-row MATMUL_Q calls in ONE
// persistent launch.
//
// The reference's wgpu backend records every op of a forward into one shared
// compute pass and submits it at flush (rust/src/backend_wgpu.rs:311-367); each
// MATMUL_Q dispatch there (rust/src/backend_wgpu.rs:768-835) waits for the one
// before it. On B200 a chain of separate kernels pays a dependent-launch
// round trip per call (about 2 us with programmatic dependent launch), which
// at one activation row is longer than streaming a projection's weights. This
// kernel runs a whole list of calls — Backend::linear, linear_geglu,
// linear_gelu_mul_cols (rust/src/backend.rs:105-167) and the soft-capped
// linear — with the same results as issuing them one after another:
//
//  * One CTA per SM for the whole list (a cooperative launch: every CTA is
//    resident). Op j's weight rows are split into one contiguous range per CTA.
//  * A producer warp streams each CTA's weight rows, op after op, into a ring
//    of shared-memory slots with 1-D bulk copies (cp.async.bulk, mbarrier
//    completion). Weights never depend on activations, so the stream runs up to
//    a ring ahead of the compute, across op boundaries: while op j waits for
//    its input, the weights of ops j+1, j+2, ... are already arriving.
//  * Sixteen consumer warps run op j: copy its descriptor into shared memory,
//    wait until every CTA has finished op j-1 (a device counter per op,
//    release/acquire at GPU scope; bounded wait), stage x (mean removal and
//    power-of-two pre-scaling, as the streaming GEMV), then the CTA's rows of
//    the op, all of its ring slots at once spread over every warp, with the
//    one-LOP3-one-FFMA dequant of gemv_core.cuh, the lane-group shuffle
//    reduction and the MODE epilogue. After its last row store the CTA adds one
//    to op j's counter (a release reduction).
//  * The counters return to zero at the end of every run (the last CTA to
//    finish the last op clears them), so a captured graph replays the chain.
//    Every wait is bounded (wall clock); a timeout sets an abort word that every
//    CTA polls, reports GQ_DEVERR_WAIT_TIMEOUT, drains its copies in flight and
//    returns. A chain that timed out needs gq_chain_reset before its next run.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <vector>

#include "gemv_core.cuh"
#include "gq_host.h"
#include "gq_internal.cuh"

using gqcore::code_pos;
using gqcore::Fmt;
using gqcore::mac_chunk;
using gqcore::pow2f;

namespace {

constexpr int kCW = 16;                  // consumer warps
constexpr int kCT = kCW * 32;            // consumer threads
constexpr int kThreads = kCT + 32;       // + one producer warp
constexpr int kMaxSlots = 8;
constexpr int kSlotBytes = 24 * 1024;    // one tile: weight rows + their scales and code sums
constexpr int kCounterStride = 32;       // 128 bytes between the per-op counters

// Weight formats: 2-bit, 4-bit, unsigned 8-bit, signed 8-bit.
enum { kFmt2 = 0, kFmt4 = 1, kFmtU8 = 2, kFmtI8 = 3 };

struct ChainOp {
  const uint8_t *w, *w2;    // packed rows (w2: the GeGLU up weight)
  const float *s, *s2;      // per-row scales (one group per row)
  const float *q, *q2;      // per-row code sums (precomputed at upload)
  const float *x;           // [K] input row
  float *y;                 // [N] output row
  const float *bs;          // MODE 2: y = gelu(.) * bs[b_off + n]
  int64_t b_off;
  float cap;                // MODE 3: soft-cap (<= 0: none)
  int kind;                 // format * 4 + mode
  int K, N, row_bytes;
  int lanes;                // lanes per row (power of two dividing row_bytes / 16)
  int tile_rows;            // rows per ring slot
  int ops_stride;           // floats per operand vector in a slot
  double inv_k;
};

constexpr int kBsCache = 256;  // MODE-2 column values staged with x (first rows of the CTA)

struct ChainShared {        // after the ring and the staged x
  ChainOp op;               // the current op's descriptor
  float bsc[kBsCache];
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  double dscr[kCW];
  float fscr[kCW];
  float mu, corr, p2;
  uint32_t issued[kMaxSlots];  // uses issued into each slot (producer)
  int abort;                // this CTA gave up (any warp)
  int go;                   // thread 0's verdict for the current op, read after a barrier
};

__device__ __forceinline__ void named_sync() {  // the consumer warps only
  asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(gqd::smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool aborted(const volatile int *sh_abort, const volatile uint32_t *g_abort) {
  return *sh_abort != 0 || *g_abort != 0u;
}
__device__ __forceinline__ void raise_abort(volatile int *sh_abort, uint32_t *g_abort, uint32_t *err) {
  *sh_abort = 1;
  atomicExch(g_abort, 1u);
  gqd::report(err, GQ_DEVERR_WAIT_TIMEOUT);
}

// Bounded mbarrier wait that also gives up when any CTA has aborted.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t *bar, uint32_t parity, uint64_t limit_ns,
                                                   const volatile int *sh_abort, const volatile uint32_t *g_abort) {
  if (gqd::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gqd::globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (gqd::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (aborted(sh_abort, g_abort)) return false;
      if (gqd::globaltimer_ns() - t0 > limit_ns) return false;
    }
  }
}

__device__ __forceinline__ void cta_rows(int N, int c, int G, int &r0, int &r1) {
  r0 = (int)(((int64_t)N * c) / G);
  r1 = (int)(((int64_t)N * (c + 1)) / G);
}

// ---- producer: the weight stream of every op, in chain order -----------------
__device__ void produce(const ChainOp *ops, int nops, uint8_t *slots, int nslots, ChainShared *sh,
                        uint32_t *g_abort, uint64_t limit_ns, uint32_t *err) {
  const int c = blockIdx.x, G = gridDim.x;
  uint32_t g = 0;
  for (int j = 0; j < nops; ++j) {
    const ChainOp &op = ops[j];
    const int nw = (op.kind & 3) == 1 ? 2 : 1;
    int r0, r1;
    cta_rows(op.N, c, G, r0, r1);
    const int rb = op.row_bytes;
    for (int rr = r0; rr < r1; rr += op.tile_rows, ++g) {
      if (aborted(&sh->abort, g_abort)) return;
      const int slot = (int)(g % (uint32_t)nslots);
      const uint32_t use = g / (uint32_t)nslots;
      if (use > 0 && !mbar_wait_or_abort(&sh->empty[slot], (use - 1) & 1u, limit_ns, &sh->abort, g_abort)) {
        if (!aborted(&sh->abort, g_abort)) raise_abort(&sh->abort, g_abort, err);
        return;
      }
      const int nr = min(op.tile_rows, r1 - rr);
      const int a4 = rr & ~3, e4 = (rr + nr + 3) & ~3;  // 16-byte aligned superset of the rows' operands
      const uint32_t bytes = (uint32_t)nr * (uint32_t)rb;
      const uint32_t ob = (uint32_t)(e4 - a4) * 4u;
      uint8_t *dst = slots + (size_t)slot * kSlotBytes;
      float *opb = reinterpret_cast<float *>(dst + (size_t)nw * op.tile_rows * rb);
      uint64_t *bar = &sh->full[slot];
      gqd::mbar_arrive_expect_tx(bar, (uint32_t)nw * (bytes + 2u * ob));
      gqd::bulk_g2s(dst, op.w + (size_t)rr * rb, bytes, bar);
      gqd::bulk_g2s(opb, op.s + a4, ob, bar);
      gqd::bulk_g2s(opb + op.ops_stride, op.q + a4, ob, bar);
      if (nw == 2) {
        gqd::bulk_g2s(dst + (size_t)op.tile_rows * rb, op.w2 + (size_t)rr * rb, bytes, bar);
        gqd::bulk_g2s(opb + 2 * op.ops_stride, op.s2 + a4, ob, bar);
        gqd::bulk_g2s(opb + 3 * op.ops_stride, op.q2 + a4, ob, bar);
      }
      sh->issued[slot] = use + 1;
    }
  }
}

// ---- consumers -----------------------------------------------------------------
// Stage op's x into the padded, pre-scaled layout of the streaming GEMV: one
// read of x through L2 (other CTAs wrote it during this launch, so never through
// the non-coherent path), one (sum, max|x|) reduction giving mu and S, then the
// scaled write; mu, the zp correction and 2^(149-S) go to shared memory.
template <int BITS>
__device__ void stage_x(const ChainOp &op, float *xs, ChainShared *sh) {
  using F = Fmt<BITS>;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = op.K;
  constexpr int kXv = 3;  // float4 per thread held in registers (K <= 6144 in one read)
  float4 xv[kXv];
  double sx = 0.0;
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < kXv; ++i) {
    const int k = (tid + i * kCT) * 4;
    xv[i] = k < K ? __ldcg(reinterpret_cast<const float4 *>(op.x + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int k = (tid + kXv * kCT) * 4; k < K; k += kCT * 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(op.x + k));
    sx += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int i = 0; i < kXv; ++i) {
    const float4 v = xv[i];
    sx += ((double)v.x + (double)v.y) + ((double)v.z + (double)v.w);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sx += __shfl_xor_sync(0xffffffffu, sx, o);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    sh->dscr[warp] = sx;
    sh->fscr[warp] = mx;
  }
  named_sync();
  double sum = 0.0;
  float mxx = 0.0f;
#pragma unroll
  for (int i = 0; i < kCW; ++i) {
    sum += sh->dscr[i];
    mxx = fmaxf(mxx, sh->fscr[i]);
  }
  const float mu = (float)(sum * op.inv_k);
  int e = 0;
  if (mxx > 0.0f && isfinite(mxx)) frexpf(mxx, &e);  // mx < 2^e, so |x - mu| < 2^(e+1)
  const int S = max(22, min(126, 125 - e));          // 2^(149-S) stays a normal f32
  auto put = [&](int k, float4 v) {
    const float vv[4] = {__fsub_rn(v.x, mu), __fsub_rn(v.y, mu), __fsub_rn(v.z, mu), __fsub_rn(v.w, mu)};
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = vv[i] * pow2f(S - code_pos<BITS>((k + i) % F::kPerWord));
    *reinterpret_cast<float4 *>(xs + (k / F::kPerChunk) * F::kPad + (k % F::kPerChunk)) =
        make_float4(o[0], o[1], o[2], o[3]);
  };
#pragma unroll
  for (int i = 0; i < kXv; ++i) {
    const int k = (tid + i * kCT) * 4;
    if (k < K) put(k, xv[i]);
  }
  for (int k = (tid + kXv * kCT) * 4; k < K; k += kCT * 4) put(k, __ldcg(reinterpret_cast<const float4 *>(op.x + k)));
  if (tid == 0) {
    sh->mu = mu;
    const double sxp = sum - (double)K * (double)mu;
    sh->corr = (float)((double)F::kZp * sxp * __longlong_as_double((long long)(1023 + S - 149) << 52));
    sh->p2 = (float)__longlong_as_double((long long)(1023 + 149 - S) << 52);
  }
  named_sync();
}

// The rows of a batch of ring slots: the CTA's rows [rr0, rr0 + nrows) of op,
// tile_rows to a slot, slots g0, g0+1, ... of the ring. Every warp takes rows of
// the whole batch (not slot by slot), so all sixteen warps work however the rows
// fall into slots. A row belongs to a group of `lanes` lanes of one warp; all
// lanes take part in every pass (rows past the end compute on a valid row and
// discard the result). bsc: the MODE-2 column values of the CTA's first rows,
// staged with x (nullptr: read them here).
template <int BITS, bool SIGNED, int MODE>
__device__ void run_rows(const ChainOp &op, const uint8_t *slots, int nslots, uint32_t g0, int rr0, int nrows,
                         int row_in_cta0, const float *xs, const ChainShared *sh) {
  using F = Fmt<BITS>;
  constexpr int NW = MODE == 1 ? 2 : 1;
  constexpr int ACC = NW == 1 ? 4 : 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = op.row_bytes, C = rb >> 4, lanes = op.lanes, tr = op.tile_rows;
  const int li = lane & (lanes - 1), grp = lane / lanes, gpw = 32 / lanes;
  const size_t wstride = (size_t)tr * rb;
  const float mu = sh->mu, corr = sh->corr, p2 = sh->p2;
  for (int base = warp * gpw; base < nrows; base += kCW * gpw) {
    const int row = base + grp;
    const bool live = row < nrows;
    const int rowc = live ? row : nrows - 1;
    const int t = rowc / tr, rin = rowc - t * tr;
    const uint8_t *buf = slots + (size_t)((g0 + (uint32_t)t) % (uint32_t)nslots) * kSlotBytes;
    const int rr = rr0 + t * tr;     // first row of the slot
    const int off = rr & 3;          // its place in the slot's aligned operand copy
    const float *opb = reinterpret_cast<const float *>(buf + NW * wstride);
    const int n = rr + rin;
    float bsv = 0.0f;
    if (MODE == 2 && live && li == 0) {
      const int ic = row_in_cta0 + row;
      bsv = ic < kBsCache ? sh->bsc[ic] : __ldcg(op.bs + op.b_off + n);
    }
    float acc[NW][1][ACC];
#pragma unroll
    for (int h = 0; h < NW; ++h)
#pragma unroll
      for (int q = 0; q < ACC; ++q) acc[h][0][q] = 0.0f;
    const uint8_t *rowp = buf + (size_t)rin * rb;
    int j = li;
    for (; j + lanes < C; j += 2 * lanes) {  // two chunks in flight
      uint4 wa[NW], wb[NW];
#pragma unroll
      for (int h = 0; h < NW; ++h) {
        wa[h] = *reinterpret_cast<const uint4 *>(rowp + h * wstride + (size_t)j * 16);
        wb[h] = *reinterpret_cast<const uint4 *>(rowp + h * wstride + (size_t)(j + lanes) * 16);
      }
      mac_chunk<BITS, SIGNED, 1, NW, ACC>(wa, xs + (size_t)j * F::kPad, 0, acc);
      mac_chunk<BITS, SIGNED, 1, NW, ACC>(wb, xs + (size_t)(j + lanes) * F::kPad, 0, acc);
    }
    if (j < C) {
      uint4 wa[NW];
#pragma unroll
      for (int h = 0; h < NW; ++h) wa[h] = *reinterpret_cast<const uint4 *>(rowp + h * wstride + (size_t)j * 16);
      mac_chunk<BITS, SIGNED, 1, NW, ACC>(wa, xs + (size_t)j * F::kPad, 0, acc);
    }
    float v[NW];
#pragma unroll
    for (int h = 0; h < NW; ++h) {
      float sum = acc[h][0][0];
#pragma unroll
      for (int q = 1; q < ACC; ++q) sum += acc[h][0][q];
      v[h] = sum;
    }
    for (int o = lanes >> 1; o > 0; o >>= 1)
#pragma unroll
      for (int h = 0; h < NW; ++h) v[h] += __shfl_xor_sync(0xffffffffu, v[h], o);
    if (live && li == 0) {
      const float sc0 = opb[off + rin], qs0 = opb[op.ops_stride + off + rin];
      // ((sum - zp*sum(x')) * 2^(149-S) + mu * sum(q)) * scale, as the streaming GEMV
      const float v0 = __fmul_rn(__fmaf_rn(mu, qs0, __fmul_rn(__fsub_rn(v[0], corr), p2)), sc0);
      float out;
      if (MODE == 1) {
        const float sc1 = opb[2 * op.ops_stride + off + rin], qs1 = opb[3 * op.ops_stride + off + rin];
        const float v1 = __fmul_rn(__fmaf_rn(mu, qs1, __fmul_rn(__fsub_rn(v[NW - 1], corr), p2)), sc1);
        out = __fmul_rn(gqd::gelu_tanh(v0), v1);
      } else if (MODE == 2) {
        out = __fmul_rn(gqd::gelu_tanh(v0), bsv);
      } else if (MODE == 3) {
        out = op.cap > 0.0f ? __fmul_rn(op.cap, tanhf(__fdiv_rn(v0, op.cap))) : v0;
      } else {
        out = v0;
      }
      op.y[n] = out;
    }
  }
}

__device__ __forceinline__ void stage_any(const ChainOp &op, float *xs, ChainShared *sh) {
  switch (op.kind >> 2) {
    case kFmt2: stage_x<2>(op, xs, sh); break;
    case kFmt4: stage_x<4>(op, xs, sh); break;
    default: stage_x<8>(op, xs, sh); break;
  }
}

template <int MODE>
__device__ __forceinline__ void rows_fmt(const ChainOp &op, const uint8_t *slots, int nslots, uint32_t g0, int rr0,
                                         int nrows, int ric, const float *xs, const ChainShared *sh) {
  switch (op.kind >> 2) {
    case kFmt2: run_rows<2, false, MODE>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
    case kFmt4: run_rows<4, false, MODE>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
    case kFmtU8: run_rows<8, false, MODE>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
    default: run_rows<8, true, MODE>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
  }
}

__device__ __forceinline__ void rows_any(const ChainOp &op, const uint8_t *slots, int nslots, uint32_t g0, int rr0,
                                         int nrows, int ric, const float *xs, const ChainShared *sh) {
  switch (op.kind & 3) {
    case 0: rows_fmt<0>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
    case 1: rows_fmt<1>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
    case 2: rows_fmt<2>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
    default: rows_fmt<3>(op, slots, nslots, g0, rr0, nrows, ric, xs, sh); break;
  }
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// ---- the kernel ------------------------------------------------------------------
// state: [0] abort word, [kCounterStride * (1 + j)] op j's count of finished CTAs.
__global__ void __launch_bounds__(kThreads, 1)
    chain_kernel(const ChainOp *ops, int nops, int nslots, int xs_floats, uint32_t *state, uint64_t limit_ns,
                 uint32_t *err) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *slots = smem;
  float *xs = reinterpret_cast<float *>(smem + (size_t)nslots * kSlotBytes);
  ChainShared *sh = reinterpret_cast<ChainShared *>(xs + xs_floats);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, G = gridDim.x;
  uint32_t *g_abort = state;

  if (tid == 0) {
    for (int s = 0; s < kMaxSlots; ++s) {
      gqd::mbar_init(&sh->full[s], 1);
      gqd::mbar_init(&sh->empty[s], kCW);
      sh->issued[s] = 0;
    }
    sh->abort = 0;
    gqd::fence_mbar_init();
  }
  __syncthreads();
  // the inputs of the first op (and the counters) come from earlier work on the stream
  gqd::griddep_wait();
  // a run after a timed-out one (no gq_chain_reset): every wait gives up at once;
  // say so again rather than leave stale outputs unreported
  if (tid == 0 && c == 0 && *(volatile uint32_t *)g_abort != 0u) gqd::report(err, GQ_DEVERR_WAIT_TIMEOUT);

  if (warp == kCW) {
    if (lane == 0) produce(ops, nops, slots, nslots, sh, g_abort, limit_ns, err);
  } else {
    uint32_t g = 0;  // ring position, in step with the producer
    for (int j = 0; j < nops; ++j) {
      // op j's descriptor into shared memory (its load overlaps the wait below)
      if (warp == 0 && lane < (int)(sizeof(ChainOp) / 8))
        reinterpret_cast<uint64_t *>(&sh->op)[lane] = reinterpret_cast<const uint64_t *>(ops + j)[lane];
      // every CTA has finished op j-1 (acquire: its outputs are visible after this)
      if (tid == 0 && j > 0 && !aborted(&sh->abort, g_abort)) {
        const uint32_t *cnt = state + kCounterStride * j;
        const uint64_t t0 = gqd::globaltimer_ns();
        for (uint32_t it = 0;; ++it) {
          if (ld_acquire(cnt) >= (uint32_t)G) break;
          if ((it & 63u) == 63u) {
            if (aborted(&sh->abort, g_abort)) break;
            if (gqd::globaltimer_ns() - t0 > limit_ns) {
              raise_abort(&sh->abort, g_abort, err);
              break;
            }
          }
        }
      }
      if (tid == 0) sh->go = !aborted(&sh->abort, g_abort);
      named_sync();
      const ChainOp &op = sh->op;
      const bool live = sh->go != 0;  // the same for every consumer thread (stage_x has barriers)
      int r0, r1;
      cta_rows(op.N, c, G, r0, r1);
      if (r1 > r0) {
        if (live && (op.kind & 3) == 2)  // the CTA's MODE-2 column values, loaded beside x
          for (int i = tid; i < min(kBsCache, r1 - r0); i += kCT) sh->bsc[i] = __ldcg(op.bs + op.b_off + r0 + i);
        if (live) stage_any(op, xs, sh);
        const int nt = (r1 - r0 + op.tile_rows - 1) / op.tile_rows;
        for (int t0 = 0; t0 < nt; t0 += nslots) {  // batches of up to a ring of slots
          const int nb = min(nslots, nt - t0);
          bool ok = live;
          for (int t = 0; t < nb && ok; ++t) {
            const uint32_t gg = g + (uint32_t)(t0 + t);
            ok = mbar_wait_or_abort(&sh->full[gg % (uint32_t)nslots], (gg / (uint32_t)nslots) & 1u, limit_ns,
                                    &sh->abort, g_abort);
          }
          if (ok) {
            const int rr0 = r0 + t0 * op.tile_rows;
            rows_any(op, slots, nslots, g + (uint32_t)t0, rr0, min(r1, rr0 + nb * op.tile_rows) - rr0,
                     t0 * op.tile_rows, xs, sh);
          } else if (live && lane == 0 && !aborted(&sh->abort, g_abort)) {
            raise_abort(&sh->abort, g_abort, err);
          }
          __syncwarp();
          if (lane == 0)
            for (int t = 0; t < nb; ++t) mbar_arrive(&sh->empty[(g + (uint32_t)(t0 + t)) % (uint32_t)nslots]);
        }
        g += (uint32_t)nt;
      }
      // the CTA's rows of op j are stored: count it finished (release at GPU scope)
      named_sync();
      if (tid == 0) {
        uint32_t *cnt = state + kCounterStride * (j + 1);
        if (j < nops - 1) {  // a release reduction: no round trip on this CTA's path
          asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(cnt), "r"(1u) : "memory");
        } else {
          __threadfence();
          const uint32_t prev = atomicAdd(cnt, 1u);
          if (prev == (uint32_t)G - 1u && !aborted(&sh->abort, g_abort)) {
            // every CTA is past all of its waits: clear the counters for the next run
            fence_acq_rel();
            for (int i = 1; i <= nops; ++i) state[kCounterStride * i] = 0u;
            __threadfence();
          }
        }
      }
    }
  }
  __syncthreads();
  gqd::griddep_launch_dependents();
  // Copies this CTA issued and nobody consumed (only after an abort): wait for
  // them (bounded) before the shared memory is released.
  if (tid == 0 && aborted(&sh->abort, g_abort)) {
    for (int s = 0; s < nslots; ++s)
      if (sh->issued[s] > 0) (void)gqd::mbar_wait_bounded(&sh->full[s], (sh->issued[s] - 1) & 1u, 50000000ull);
  }
  __syncthreads();
}

}  // namespace

// ---- host ------------------------------------------------------------------------
struct gq_chain {
  gq_ctx *ctx = nullptr;
  int n = 0;
  ChainOp *d_ops = nullptr;
  uint32_t *d_state = nullptr;
  size_t state_bytes = 0;
  int grid = 0, nslots = 0, xs_floats = 0;
  size_t smem = 0;
  bool coop = true;
};

namespace {

bool overlaps(const void *a, size_t na, const void *b, size_t nb) {
  const uintptr_t pa = (uintptr_t)a, pb = (uintptr_t)b;
  return pa < pb + nb && pb < pa + na;
}

int plan_op(gq_ctx *ctx, const gq_chain_op &in, int grid, int idx, ChainOp &op, int &xs_floats) {
  auto bad = [&](int status, const char *what) {
    return gq_fail(ctx, status, "chain op " + std::to_string(idx) + ": " + what);
  };
  if (in.mode < 0 || in.mode > 3) return bad(GQ_ERR_INVALID_ARGUMENT, "mode not in 0..3");
  const gq_qweight *w = in.w;
  if (!w || !in.x || !in.y) return bad(GQ_ERR_INVALID_ARGUMENT, "null weight, x or y");
  if (w->device != ctx->device) return bad(GQ_ERR_INVALID_ARGUMENT, "weight on another device");
  if (w->n <= 0 || w->k <= 0 || w->n > 0x7fffffff) return bad(GQ_ERR_INVALID_ARGUMENT, "empty or oversized weight");
  if (w->group_size != w->k) return bad(GQ_ERR_UNSUPPORTED, "grouped scales (one scale per row only)");
  if (w->row_bytes % 16 != 0 || w->k % 4 != 0) return bad(GQ_ERR_UNSUPPORTED, "row not a whole number of 16-byte chunks");
  if ((uintptr_t)in.x % 16 != 0) return bad(GQ_ERR_UNSUPPORTED, "x not 16-byte aligned");
  if (in.mode == 1) {
    const gq_qweight *u = in.w2;
    if (!u) return bad(GQ_ERR_INVALID_ARGUMENT, "geglu without the up weight");
    if (u->n != w->n || u->k != w->k || u->bits != w->bits || u->signed_i8 != w->signed_i8 ||
        u->row_bytes != w->row_bytes || u->group_size != u->k || u->device != w->device)
      return bad(GQ_ERR_INVALID_ARGUMENT, "gate and up weights differ in shape or format");
  }
  if (in.mode == 2 && (!in.b || in.b_offset < 0)) return bad(GQ_ERR_INVALID_ARGUMENT, "gelu_mul_cols without b");
  // in-place outputs would race with other CTAs still reading the op's inputs
  const size_t ybytes = (size_t)w->n * 4;
  if (overlaps(in.y, ybytes, in.x, (size_t)w->k * 4)) return bad(GQ_ERR_INVALID_ARGUMENT, "y overlaps x");
  if (in.mode == 2 && overlaps(in.y, ybytes, in.b + in.b_offset, ybytes))
    return bad(GQ_ERR_INVALID_ARGUMENT, "y overlaps b");
  const int nw = in.mode == 1 ? 2 : 1;
  const int rb = (int)w->row_bytes, C = rb / 16;
  const int fmt = w->bits == 2 ? kFmt2 : (w->bits == 4 ? kFmt4 : (w->signed_i8 ? kFmtI8 : kFmtU8));
  op = ChainOp{};
  op.w = w->bytes;
  op.s = w->scales;
  op.q = w->scales + w->qsum_off;
  if (nw == 2) {
    op.w2 = in.w2->bytes;
    op.s2 = in.w2->scales;
    op.q2 = in.w2->scales + in.w2->qsum_off;
  }
  op.x = in.x;
  op.y = in.y;
  op.bs = in.b;
  op.b_off = in.b_offset;
  op.cap = in.cap;
  op.kind = fmt * 4 + in.mode;
  op.K = (int)w->k;
  op.N = (int)w->n;
  op.row_bytes = rb;
  op.inv_k = 1.0 / (double)w->k;
  op.lanes = 32;
  while (C % op.lanes != 0) op.lanes >>= 1;
  // rows per slot: as many of the CTA's rows as fit, then evened out over the slots
  const int rows_max = (int)((w->n + grid - 1) / grid);
  auto slot_need = [&](int t) {
    const int stride = ((t + 3) & ~3) + 8;
    return (size_t)nw * t * rb + (size_t)nw * 2 * stride * 4;
  };
  int t = rows_max;
  while (t > 0 && slot_need(t) > (size_t)kSlotBytes) --t;
  if (t < 1) return bad(GQ_ERR_UNSUPPORTED, "a weight row does not fit a ring slot");
  const int ntiles = (rows_max + t - 1) / t;
  t = (rows_max + ntiles - 1) / ntiles;
  op.tile_rows = t;
  op.ops_stride = ((t + 3) & ~3) + 8;
  const int pad = 4 * (32 / w->bits) + 4;
  xs_floats = std::max(xs_floats, C * pad);
  return GQ_OK;
}

}  // namespace

int gq_chain_create(gq_ctx *ctx, const gq_chain_op *ops, int32_t n_ops, gq_chain **out) {
  if (!ctx || !out) return GQ_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int rc = gq_enter_ctx(ctx);
  if (rc != GQ_OK) return rc;
  if (!ops || n_ops < 1) return gq_fail(ctx, GQ_ERR_INVALID_ARGUMENT, "chain: no ops");
  const int grid = ctx->num_sms;
  std::vector<ChainOp> h((size_t)n_ops);
  int xs_floats = 0;
  for (int i = 0; i < n_ops; ++i)
    if ((rc = plan_op(ctx, ops[i], grid, i, h[i], xs_floats)) != GQ_OK) return rc;
  xs_floats = (xs_floats + 3) & ~3;
  const size_t fixed = (size_t)xs_floats * 4 + sizeof(ChainShared);
  if (fixed + 2 * (size_t)kSlotBytes > ctx->smem_optin)
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "chain: x of an op too long for shared memory");
  const int nslots = (int)std::min<size_t>(kMaxSlots, (ctx->smem_optin - fixed) / kSlotBytes);
  const size_t smem = (size_t)nslots * kSlotBytes + fixed;
  cudaError_t e = cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return gq_cuda_fail(ctx, e, "chain: shared memory attribute");
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_kernel, kThreads, smem);
  if (e != cudaSuccess) return gq_cuda_fail(ctx, e, "chain: occupancy");
  if (per_sm < 1) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "chain: kernel does not fit an SM");
  gq_chain *ch = new gq_chain();
  ch->ctx = ctx;
  ch->n = n_ops;
  ch->grid = grid;
  ch->nslots = nslots;
  ch->xs_floats = xs_floats;
  ch->smem = smem;
  if (const char *v = getenv("GQ_CHAIN_COOP")) ch->coop = atoi(v) != 0;
  ch->state_bytes = (size_t)(n_ops + 1) * kCounterStride * sizeof(uint32_t);
  if ((e = cudaMalloc(reinterpret_cast<void **>(&ch->d_ops), h.size() * sizeof(ChainOp))) != cudaSuccess ||
      (e = cudaMalloc(reinterpret_cast<void **>(&ch->d_state), ch->state_bytes)) != cudaSuccess ||
      (e = cudaMemcpy(ch->d_ops, h.data(), h.size() * sizeof(ChainOp), cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemset(ch->d_state, 0, ch->state_bytes)) != cudaSuccess) {
    if (ch->d_ops) cudaFree(ch->d_ops);
    if (ch->d_state) cudaFree(ch->d_state);
    delete ch;
    return gq_cuda_fail(ctx, e, "chain: device tables");
  }
  *out = ch;
  return GQ_OK;
}

int gq_chain_run(gq_chain *ch) {
  if (!ch) return GQ_ERR_INVALID_ARGUMENT;
  gq_ctx *ctx = ch->ctx;
  int rc = gq_enter_ctx(ctx);
  if (rc != GQ_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ch->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = ch->smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ch->coop ? 1 : 0;
  GQ_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, chain_kernel, (const ChainOp *)ch->d_ops, ch->n, ch->nslots,
                                     ch->xs_floats, ch->d_state, ctx->wait_limit_ns, ctx->dev_err));
  return GQ_OK;
}

int gq_chain_reset(gq_chain *ch) {
  if (!ch) return GQ_ERR_INVALID_ARGUMENT;
  int rc = gq_enter_ctx(ch->ctx);
  if (rc != GQ_OK) return rc;
  GQ_CUDA_TRY(ch->ctx, cudaMemsetAsync(ch->d_state, 0, ch->state_bytes, ch->ctx->stream));
  return GQ_OK;
}

int gq_chain_destroy(gq_chain *ch) {
  if (!ch) return GQ_OK;
  if (gq_enter_ctx(ch->ctx) == GQ_OK) {
    cudaFree(ch->d_ops);
    cudaFree(ch->d_state);
  }
  delete ch;
  return GQ_OK;
}
