// gemv_tcx.cu — short-M GEMV (3 <= M <= 64 activation rows) on the tensor cores.
//
// The same exact integer dot products as gemv_tc.cu (tcgen05.mma.kind::i8 on
// four signed byte limbs of x in 30-bit fixed point), for the M = 3..64 rows of
// a decode batch (rust/src/backend_wgpu.rs:646-695 sends M <= 15 to MATMUL_Q,
// rust/src/kernels/matmul_q.wgsl:96-169; BASELINE config 5 decodes 64 sequences):
//  * a pre-pass kernel (one block per activation row) writes the limbs of all M
//    rows once, as a [4*M, Kp] s8 matrix in global memory (row = token*4 + limb,
//    K permuted inside each 16-code group like the widened weights), plus each
//    row's exponent, sum of fixed-point values and a non-finite flag;
//  * the pre-pass lays the matrix out as the GEMV's swizzled shared-memory tiles
//    (64 / 128 / 256 limb rows x 128 bytes per K-block, zero rows past 4M), so the
//    GEMV fetches each K-block's A operand with one 1-D bulk copy: one M = 64 MMA for up to 16
//    tokens (accumulator row r in TMEM lane 32*(r/16) + r%16), else one or two
//    M = 128 MMAs (row r of half h in lane r of that half's accumulator);
//  * weights are the B operand exactly as in gemv_tc.cu (I8 rows straight from
//    TMA into the swizzled layout, sub-byte and U8 codes widened by 4 warps), one
//    tile of up to 256 rows per CTA, K-blocks dealt round-robin to up to three
//    issuing threads with separate accumulators; weights taller than one tile
//    per SM are processed as row slices, one launch each, sharing the limbs;
//  * the tile's scales come into shared memory by one bulk copy issued before
//    the grid dependency wait;
//  * all eight warps run the epilogue (warp w drains TMEM lane quarter w % 4),
//    recombine the limbs of each token in int64, remove the zero point exactly
//    and convert once: y = f32(T * 2^-s_m) * scale[n];
//  * long rows split K over a thread-block cluster whose CTAs add their exact
//    int64 partials over distributed shared memory (either operand layout; the
//    weights-as-A one, 128-row tiles as the MMA's A, serves one long weight at
//    M <= 16);
//  * optionally (GQ_TCX_XIN=1) each CTA makes its own limb tiles from x instead
//    of the pre-pass, bit for bit the same.
// The limb matrix is small and shared by every CTA, so after the first CTAs it
// streams from L2; the weights stream from HBM once for all M rows.
// Every wait is bounded (GQ_DEVERR_WAIT_TIMEOUT); TMA copies in flight are
// drained, outstanding MMAs committed and TMEM freed before the CTA exits.
#include <cuda_runtime.h>
#include <math.h>

#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "tc_common.cuh"

namespace {
using namespace gqt;

constexpr int kThreads = 256;  // warp 0 TMA, warps 1-3 MMA issue, warps 4-7 expanders + epilogue
constexpr int kKB = 128;       // codes per K-block
constexpr int kMaxRaw = 8;
constexpr int kMaxMma = 48;    // widened ring: up to every K-block of K = 6144
constexpr int kMaxXa = 24;     // A (limb) tile ring, all issuers together
constexpr int kMaxIss = 3;
constexpr int kExpWarps = 4;
constexpr int kMaxTok = 64;
constexpr int kMaxK = 8192;
constexpr int kXinSlots = 4;  // in-kernel limbs: 16-value groups a thread holds in registers

struct TcxArgs {
  int M, K, N;
  const float *s;
  const float *s2;
  const float *bs;
  int64_t b_stride, b_off;
  float cap;
  float *y;
  PeerDst peers;  // extra output destinations (peer buffers); n = 0: none
  int64_t ldy, y_col0;
  const int *xexp;        // [M] per-row exponent s_m (X = rint(x * 2^s_m))
  const long long *sumx;  // [M] sum_k X
  const uint32_t *bad;    // [M] non-finite x row
  const uint8_t *limbs;   // [kblocks][xa_rows][128 B] pre-swizzled A tiles (pre-pass)
  const float *x;         // [M, K] activations, read when xin
  int xin;                // 1: the CTA makes its own limb tiles from x (no pre-pass)
  int tile_rows;          // MMA N: multiple of 16
  int mh;                 // 0: one M=64 MMA (<= 16 tokens); 1 or 2: M=128 halves
  int wa;                 // 1: weights are the A operand (M = 128 rows), limb rows the B operand (N = lrows)
  int lrows;              // limb rows per tile when wa (4*M rounded up to 16, <= 256)
  int kblocks, kbr;
  int raw_stages, mma_stages, xa_stages, xi, xi_log2;
  int raw_bytes, mma_bytes, xa_tile;
  int issuers;
  int tmem_cols;
  int ksplit;             // K splits: the CTAs of one cluster (cluster rank = blockIdx.y)
  int kb_per;             // K-blocks per split (the last split may have fewer)
  uint32_t *err;
};

struct TcxSmem {
  uint32_t xa_off, raw_off, mma_off, sc_off, bar_off, misc_off, total;
};
__host__ __device__ inline TcxSmem tcx_layout(int xa_stages, int xa_tile, int raw_stages, int raw_bytes,
                                              int mma_stages, int mma_bytes, int sc_bytes) {
  TcxSmem L;
  uint32_t o = 0;
  L.xa_off = o;   o += (uint32_t)xa_stages * (uint32_t)xa_tile;
  L.raw_off = o;  o += (uint32_t)raw_stages * (uint32_t)raw_bytes;
  L.mma_off = o;  o += (uint32_t)mma_stages * (uint32_t)mma_bytes;
  L.sc_off = o;   o += (uint32_t)((sc_bytes + 127) & ~127);
  L.bar_off = o;  o += (2 * kMaxRaw + 2 * kMaxMma + 2 * kMaxXa + 2 * kMaxIss + 2) * 8;
  L.misc_off = o; o += 64 + kMaxTok * 36;
  L.total = o + 1024;
  return L;
}

template <int BITS>
__host__ __device__ constexpr int perm16(int p) {
  return BITS == 4 ? ((p & 8) | ((p & 3) << 1) | ((p >> 2) & 1))  // 0,2,4,6,1,3,5,7 per 8
         : BITS == 2 ? (((p & 3) << 2) | (p >> 2))               // 0,4,8,12,1,5,...
                     : p;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity) {
  return gqd::mbar_try_wait(bar, parity) || gqd::mbar_wait_bounded(bar, parity);
}
// all threads of every CTA of the cluster (release / acquire at cluster scope)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// the same barrier in two halves, so independent work can run between them
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
// the shared::cluster address of this CTA's shared-memory location p in cluster CTA `rank`
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(gqd::smem_u32(p)), "r"(rank));
  return ra;
}
// a 32-bit value at a shared::cluster address
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
// two 64-bit values at a shared::cluster address (16-byte aligned)
__device__ __forceinline__ void ld_cluster_v2s64(uint32_t addr, long long &v0, long long &v1) {
  asm volatile("ld.shared::cluster.v2.s64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "r"(addr) : "memory");
}

// ---- pre-pass: x row m -> 30-bit fixed point -> four s8 limb rows ------------
// Same arithmetic as the in-CTA staging of gemv_tc.cu: s = 30 - e with
// max|x| < 2^e, X = rint(x * 2^s), balanced base-256 digits from X + 0x808080.
// The limbs are written as the GEMV's shared-memory A tiles: K-block kb of limb
// row r at limbs + kb*xa_rows*128 + r*128, 16-byte chunk c stored at chunk
// c ^ (r % 8) (the 128-byte swizzle), so one K-block tile is one contiguous
// xa_rows*128-byte block that a 1-D bulk copy moves as is. Block M zero-fills
// the tile rows past 4*M.
template <int BITS>
__global__ void xlimbs_kernel(const float *x, int K, int Kp, int M, int xa_rows, uint8_t *limbs, int *xexp,
                              long long *sumx, uint32_t *bad) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (m == M) {  // zero rows 4M .. xa_rows-1 of every K-block tile
    const int pad = xa_rows - 4 * M, kbs = Kp / kKB;
    for (int i = tid; i < kbs * pad * 8; i += kThreads) {
      const int kb = i / (pad * 8), rem = i - kb * pad * 8;
      *reinterpret_cast<uint4 *>(limbs + ((size_t)kb * xa_rows + 4 * M) * 128 + (size_t)rem * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)m * K);
  __shared__ float wmax[8];
  __shared__ uint32_t wbad[8];
  __shared__ long long wsum[8];
  // each thread's 16-value groups (K <= 8192: at most two) stay in registers
  // from the max pass to the conversion
  constexpr int kG = kMaxK / 16 / kThreads;
  float4 v[kG][4];
  float mx = 0.0f;
  uint32_t b = 0;
#pragma unroll
  for (int j = 0; j < kG; ++j) {
    const int gi = tid + j * kThreads;
#pragma unroll
    for (int q = 0; q < 4; ++q) v[j][q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (gi * 16 < K) {
#pragma unroll
      for (int q = 0; q < 4; ++q) v[j][q] = __ldg(xr + gi * 4 + q);
    }
  }
#pragma unroll
  for (int j = 0; j < kG; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 u = v[j][q];
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))));
      b |= !(isfinite(u.x) && isfinite(u.y) && isfinite(u.z) && isfinite(u.w));
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    b |= __shfl_xor_sync(0xffffffffu, b, o);
  }
  if (lane == 0) {
    wmax[warp] = mx;
    wbad[warp] = b;
  }
  __syncthreads();
  mx = 0.0f;
  b = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mx = fmaxf(mx, wmax[i]);
    b |= wbad[i];
  }
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) frexpf(mx, &e);
  const int s = 30 - e;
  const float f1 = __int_as_float((s / 2 + 127) << 23), f2 = __int_as_float((s - s / 2 + 127) << 23);
  long long part = 0;
#pragma unroll
  for (int j = 0; j < kG; ++j) {
    const int gi = tid + j * kThreads;
    if (gi >= Kp / 16) break;
    int X[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      X[4 * q + 0] = __float2int_rn(__fmul_rn(__fmul_rn(v[j][q].x, f1), f2));
      X[4 * q + 1] = __float2int_rn(__fmul_rn(__fmul_rn(v[j][q].y, f1), f2));
      X[4 * q + 2] = __float2int_rn(__fmul_rn(__fmul_rn(v[j][q].z, f1), f2));
      X[4 * q + 3] = __float2int_rn(__fmul_rn(__fmul_rn(v[j][q].w, f1), f2));
    }
    uint32_t wv[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      const int xv = X[perm16<BITS>(p)];
      part += xv;
      wv[p] = ((uint32_t)xv + 0x00808080u) ^ 0x00808080u;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t t01a = prmt(wv[4 * q], wv[4 * q + 1], 0x5140), t23a = prmt(wv[4 * q + 2], wv[4 * q + 3], 0x5140);
      const uint32_t t01b = prmt(wv[4 * q], wv[4 * q + 1], 0x7362), t23b = prmt(wv[4 * q + 2], wv[4 * q + 3], 0x7362);
      wv[4 * q] = prmt(t01a, t23a, 0x5410);
      wv[4 * q + 1] = prmt(t01a, t23a, 0x7632);
      wv[4 * q + 2] = prmt(t01b, t23b, 0x5410);
      wv[4 * q + 3] = prmt(t01b, t23b, 0x7632);
    }
    const int kb = gi >> 3, c = gi & 7;
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const int r = 4 * m + l;
      *reinterpret_cast<uint4 *>(limbs + ((size_t)kb * xa_rows + r) * 128 + ((c ^ (r & 7)) << 4)) =
          make_uint4(wv[l], wv[4 + l], wv[8 + l], wv[12 + l]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) wsum[warp] = part;
  __syncthreads();
  if (tid == 0) {
    long long t = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += wsum[i];
    sumx[m] = t;
    xexp[m] = s;
    bad[m] = b;
  }
}

// ---- the GEMV -------------------------------------------------------------------
// Control flow is division-free in the steady state (ring slots and phases are
// stepped incrementally): the producer and issuer threads run one K-block every
// few tens of cycles, so they never pace the pipeline.
template <int BITS, bool SIGNED, int MODE, bool WA>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_tcx_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_w2,
                    const TcxArgs a) {
  constexpr int NW = (MODE == 1) ? 2 : 1;
  constexpr bool DIRECT = (BITS == 8 && SIGNED);
  constexpr int KB_BYTES = kKB * BITS / 8;
  constexpr int CPR = KB_BYTES / 16;
  constexpr long long ZP = (BITS == 8) ? 0 : (1 << (BITS - 1));
  constexpr int kBars = 2 * kMaxRaw + 2 * kMaxMma + 2 * kMaxXa + 2 * kMaxIss + 1;
  const int MH = a.mh > 0 ? a.mh : 1;  // accumulator halves
  // D = A * B^T: A = limb rows (s8, M = 64 or 128), B = weight rows (s8, N = tile_rows), D s32.
  const uint32_t idesc = WA ? ((2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.lrows >> 3) << 17) |
                                 ((uint32_t)(128 >> 4) << 24))
                              : ((2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.tile_rows >> 3) << 17) |
                                 ((uint32_t)((a.mh == 0 ? 64 : 128) >> 4) << 24));
  // accumulator columns per (issuer, weight): [NW][LR] when wa, [MH][NW][tile_rows] otherwise
  const int acc_cols = WA ? NW * a.lrows : MH * NW * a.tile_rows;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const TcxSmem L = tcx_layout(a.xa_stages, a.xa_tile, a.raw_stages, a.raw_bytes, a.mma_stages, a.mma_bytes,
                               NW * a.tile_rows * 4);
  uint8_t *xa = smem + L.xa_off;    // [xa_stages][xa_rows x 128 B], swizzled (TMA)
  uint8_t *raw = smem + L.raw_off;  // [raw_stages][raw_bytes]
  uint8_t *wid = smem + L.mma_off;  // [mma_stages][NW][tile_rows x 128 B], swizzled
  float *scb = reinterpret_cast<float *>(smem + L.sc_off);  // [NW][tile_rows]
  uint64_t *raw_full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *raw_empty = raw_full + kMaxRaw;
  uint64_t *mma_full = raw_empty + kMaxRaw;
  uint64_t *mma_empty = mma_full + kMaxMma;
  uint64_t *xa_full = mma_empty + kMaxMma;
  uint64_t *xa_empty = xa_full + kMaxXa;
  uint64_t *acc_full = xa_empty + kMaxXa;  // [kMaxIss]
  uint64_t *done_bar = acc_full + kMaxIss;  // [kMaxIss]
  uint64_t *sc_bar = done_bar + kMaxIss;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.misc_off);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  double *tok_pw = reinterpret_cast<double *>(smem + L.misc_off + 64);  // [kMaxTok] 2^-s
  long long *tok_zc = reinterpret_cast<long long *>(tok_pw + kMaxTok);  // [kMaxTok] ZP * sum X
  uint32_t *tok_bad = reinterpret_cast<uint32_t *>(tok_zc + kMaxTok);   // [kMaxTok]
  uint32_t *rmax = tok_bad + kMaxTok;                                     // [kMaxTok] max|x| bits (xin)
  int *tok_s = reinterpret_cast<int *>(rmax + kMaxTok);                   // [kMaxTok] exponent s (xin)
  long long *tok_zs = reinterpret_cast<long long *>(tok_s + kMaxTok);     // [kMaxTok] split's ZP * sum X
  // split-K partials [NW][M][tile_rows] (int64), over the rings once every MMA has completed
  long long *part = reinterpret_cast<long long *>(smem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_begin = blockIdx.x * a.tile_rows;
  const int n_end = min(a.N, n_begin + a.tile_rows);
  // split-K: this CTA (cluster rank sidx) owns K-blocks kbase .. kbase + kblocks - 1
  const int KS = a.ksplit, sidx = KS > 1 ? (int)blockIdx.y : 0;
  const int kbase = sidx * a.kb_per;
  const int kblocks = KS > 1 ? min(a.kb_per, a.kblocks - kbase) : a.kblocks;
  const int kbr = a.kbr, RS = a.raw_stages, MS = a.mma_stages;
  const int total_raw = (kblocks + kbr - 1) / kbr;
  // issuers with work: the last K split may own fewer work units than the plan's
  // issuer count (its rings then never wrap, so the slot ownership still holds)
  const int NI = max(1, min(a.issuers, DIRECT ? total_raw : kblocks)), XI = a.xi, XL = a.xi_log2;
  const int tile_bytes = a.tile_rows * 128;
  const uint32_t xa_tile = (uint32_t)a.xa_tile;

  // one barrier per thread (all the arrays are contiguous from raw_full)
  if (tid < kBars) {
    uint32_t cnt = 1;
    if (!DIRECT && tid >= kMaxRaw && tid < 2 * kMaxRaw) cnt = kExpWarps;  // raw_empty: each widening warp
    if (!DIRECT && tid >= 2 * kMaxRaw && tid < 2 * kMaxRaw + kMaxMma) cnt = kExpWarps;  // mma_full: likewise
    gqd::mbar_init(raw_full + tid, cnt);
    gqd::fence_mbar_init();
  }
  if (tid == 0) *abort_flag = 0;
  if (tid < kMaxTok) {  // in-kernel limbs: row maxima and sums start at zero
    rmax[tid] = 0u;
    tok_zs[tid] = 0;
  }
  __syncthreads();

  auto issue = [&](int r, int slot) {  // raw stage r (K-blocks r*kbr .. +kbr-1) into `slot`
    const int kb0 = r * kbr;
    uint8_t *dst = raw + slot * a.raw_bytes;
    if (DIRECT) {
      const int nkb = min(kbr, kblocks - kb0);
      gqd::mbar_arrive_expect_tx(&raw_full[slot], (uint32_t)(nkb * NW * tile_bytes));
      for (int j = 0; j < nkb; ++j)
        for (int h = 0; h < NW; ++h)
          tma_load_2d(dst + (j * NW + h) * tile_bytes, h ? &map_w2 : &map_w, (kbase + kb0 + j) * kKB, n_begin,
                      &raw_full[slot]);
    } else {
      gqd::mbar_arrive_expect_tx(&raw_full[slot], (uint32_t)(NW * a.tile_rows * kbr * KB_BYTES));
      for (int h = 0; h < NW; ++h)
        tma_load_2d(dst + h * a.tile_rows * kbr * KB_BYTES, h ? &map_w2 : &map_w, (kbase + kb0) * KB_BYTES, n_begin,
                    &raw_full[slot]);
    }
  };
  // The limb ring is split per issuer (XI slots each, a power of two) so every
  // slot is filled and consumed in order by one producer and one consumer: a
  // waiter then never asks for a phase two completions ahead of the barrier
  // (which an mbarrier parity wait would report as already complete).
  // K-block g belongs to issuer own(g) as its ord(g)-th K-block: whole raw
  // stages round-robin for I8 (stage u -> issuer u % NI), single K-blocks otherwise.
  auto x_owner = [&](int g, int &ord) {  // (abort path only; the loops step these incrementally)
    if (DIRECT) {
      const int u = g / kbr;
      ord = (u / NI) * kbr + g % kbr;
      return u % NI;
    }
    ord = g / NI;
    return g % NI;
  };
  auto issue_x = [&](int slot, int g) {  // limb tile of K-block g
    gqd::mbar_arrive_expect_tx(&xa_full[slot], xa_tile);
    gqd::bulk_g2s(xa + (size_t)slot * xa_tile, a.limbs + (size_t)(kbase + g) * xa_tile, xa_tile, &xa_full[slot]);
  };

  // ---- widening of sub-byte / U8 codes: the 4 warps widen one raw stage at a time ----
  // Stages are widened in order by all four warps together, so every wait is for
  // the next phase of its barrier (never two phases ahead).
  const int ew = warp - (kThreads / 32 - kExpWarps);  // expander warp index (valid for warps 4-7)
  const int et = tid - (kThreads - kExpWarps * 32);   // expander thread index
  int er = 0, erslot = 0, erk = 0;   // next raw stage to widen
  int emslot = 0, emk = 0;           // widened-ring slot of its first K-block and its use count
  // Widen raw stage er (warp-uniform; false on a timed-out wait).
  auto expand_stage = [&]() -> bool {
    const int g0 = er * kbr, nkb = min(kbr, kblocks - g0);
    if (!__all_sync(0xffffffffu, wait_phase(&raw_full[erslot], (uint32_t)erk & 1u))) return false;
    const int rstride = kbr * KB_BYTES;
    const uint8_t *src0 = raw + erslot * a.raw_bytes;
    for (int j = 0; j < nkb; ++j) {
      // the slot's previous K-block must have been consumed by its MMAs
      if (!__all_sync(0xffffffffu, emk == 0 || wait_phase(&mma_empty[emslot], (uint32_t)(emk - 1) & 1u)))
        return false;
#pragma unroll
      for (int h = 0; h < NW; ++h) {
        const uint8_t *src = src0 + h * a.tile_rows * rstride + j * KB_BYTES;
        uint8_t *dst = wid + emslot * a.mma_bytes + h * tile_bytes;
        for (int it = et; it < a.tile_rows * CPR; it += kExpWarps * 32) {
          const int row = it / CPR, ic = it % CPR;  // CPR is a compile-time power of two
          const uint4 in = *reinterpret_cast<const uint4 *>(src + row * rstride + ic * 16);
          if constexpr (BITS == 4) {
            const uint32_t m = 0x0F0F0F0Fu;
            *reinterpret_cast<uint4 *>(dst + sw128_off(row, 2 * ic)) =
                make_uint4(in.x & m, (in.x >> 4) & m, in.y & m, (in.y >> 4) & m);
            *reinterpret_cast<uint4 *>(dst + sw128_off(row, 2 * ic + 1)) =
                make_uint4(in.z & m, (in.z >> 4) & m, in.w & m, (in.w >> 4) & m);
          } else if constexpr (BITS == 2) {
            const uint32_t m = 0x03030303u;
            const uint32_t w4[4] = {in.x, in.y, in.z, in.w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4 *>(dst + sw128_off(row, 4 * ic + q)) =
                  make_uint4(w4[q] & m, (w4[q] >> 2) & m, (w4[q] >> 4) & m, (w4[q] >> 6) & m);
          } else {
            const uint32_t f = 0x80808080u;
            *reinterpret_cast<uint4 *>(dst + sw128_off(row, ic)) = make_uint4(in.x ^ f, in.y ^ f, in.z ^ f, in.w ^ f);
          }
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&mma_full[emslot]);
      if (++emslot == MS) { emslot = 0; ++emk; }
    }
    if (lane == 0) mbar_arrive(&raw_empty[erslot]);
    ++er;
    if (++erslot == RS) { erslot = 0; ++erk; }
    return true;
  };

  // TMEM before the dependency wait (warp 1 has nothing else to do here): it
  // can only wait on kernels that run ahead of this one, never on a dependent
  // (the dependents launch after this CTA's launch_dependents, which follows).
  // Measured: config-2 sweep at M = 8 2.29 -> 2.23 ms. (The same move in the
  // M <= 2 GEMV cost its lm_head 40 us inside the M = 1 decode step, so that one
  // allocates after the wait.)
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(gqd::smem_u32(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // ---- before the dependency wait: weights and scales only ----
  const int G_pre = DIRECT ? 0 : min(MS, kblocks);
  int issued = 0;
  if (warp == 0 && lane == 0) {
    // the tile's scales (rows rounded up to 16 bytes: the allocation extends past them)
    const uint32_t sbytes = (uint32_t)(((n_end - n_begin) * 4 + 15) & ~15);
    gqd::mbar_arrive_expect_tx(sc_bar, NW * sbytes);
    gqd::bulk_g2s(scb, a.s + n_begin, sbytes, sc_bar);
    if (NW == 2) gqd::bulk_g2s(scb + a.tile_rows, a.s2 + n_begin, sbytes, sc_bar);
    int rslot = 0, rk = 0;
    for (int r = 0; r < total_raw; ++r) {
      if (r >= RS) {
        const int last = min((r - RS + 1) * kbr, kblocks) - 1;
        if (DIRECT || last >= G_pre) break;
        if (!wait_phase(&raw_empty[rslot], (uint32_t)(rk - 1) & 1u)) {
          *abort_flag = 1;
          break;
        }
      }
      issue(r, rslot);
      issued = r + 1;
      if (++rslot == RS) { rslot = 0; ++rk; }
    }
  }
  bool exp_ok = true;
  if (!DIRECT && ew >= 0) {
    while (exp_ok && er < total_raw && min((er + 1) * kbr, kblocks) <= G_pre) exp_ok = expand_stage();
    if (!exp_ok) *abort_flag = 1;
  }
  gqd::griddep_launch_dependents();
  gqd::griddep_wait();  // the limbs come from the pre-pass
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- in-kernel limbs (xin): the CTA turns x into the resident A tiles of its
  // own K-blocks, with the pre-pass kernel's arithmetic and layout. The row
  // exponent needs max|x| over the whole row: each K split publishes its row
  // maxima in shared memory and reads the others' over the cluster. Zero points
  // are removed per split (exact integers), so the finalisation adds no term. ----
  if (a.xin) {
    // A row's groups (16 values each) occupy Gp lane slots: G rounded up to a power
    // of two below 32, to a multiple of 32 above, so every row starts an aligned
    // segment of S lanes and its maxima and sums reduce inside the segment. Thread
    // t holds slots t, t + 256, t + 512 and t + 768 (the planner keeps M * Gp <= 1024),
    // all loaded before the first use.
    const int G = kblocks * 8;
    const int Gp = G <= 8 ? 8 : G <= 16 ? 16 : (G + 31) & ~31;
    const int S = min(Gp, 32), ngp = a.M * Gp;
    const unsigned seg = S == 32 ? 0xffffffffu : (((1u << S) - 1u) << (lane & ~(S - 1)));
    const bool lead = (lane & (S - 1)) == 0;
    const int kx0 = kbase * kKB;
    float4 v[kXinSlots][4];
#pragma unroll
    for (int i = 0; i < kXinSlots; ++i) {
      const int slot = i * kThreads + tid, m = slot / Gp, j = slot - m * Gp, k = kx0 + j * 16;
      if (slot < ngp && j < G && k < a.K) {
        const float4 *src = reinterpret_cast<const float4 *>(a.x + (size_t)m * a.K + k);
#pragma unroll
        for (int q = 0; q < 4; ++q) v[i][q] = __ldg(src + q);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) v[i][q] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    // keep the loaded values in registers until pass 2 (no reload after the barriers)
#pragma unroll
    for (int i = 0; i < kXinSlots; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        asm volatile("" : "+f"(v[i][q].x), "+f"(v[i][q].y), "+f"(v[i][q].z), "+f"(v[i][q].w));
#pragma unroll
    for (int i = 0; i < kXinSlots; ++i) {
      const int slot = i * kThreads + tid;
      if (i * kThreads + warp * 32 >= ngp) break;  // warp-uniform: segments are whole
      uint32_t mx = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        mx = max(mx, max(max(__float_as_uint(v[i][q].x) & 0x7fffffffu, __float_as_uint(v[i][q].y) & 0x7fffffffu),
                         max(__float_as_uint(v[i][q].z) & 0x7fffffffu, __float_as_uint(v[i][q].w) & 0x7fffffffu)));
      mx = __reduce_max_sync(seg, mx);
      if (lead && slot < ngp) atomicMax(&rmax[slot / Gp], mx);  // ngp is a multiple of S: segments are whole
    }
    __syncthreads();
    if (KS > 1) cluster_sync_all();  // every split's row maxima are in place
    if (tid < a.M) {
      uint32_t mb = rmax[tid];
      for (int q = 0; q < KS; ++q)
        if (q != sidx) mb = max(mb, ld_cluster_u32(cluster_addr(&rmax[tid], (uint32_t)q)));
      int e = 0;
      if (mb != 0u && mb < 0x7f800000u) frexpf(__uint_as_float(mb), &e);
      tok_s[tid] = 30 - e;
      tok_bad[tid] = mb >= 0x7f800000u ? 1u : 0u;  // inf or NaN in the row
      tok_pw[tid] = __longlong_as_double((long long)(1023 - (30 - e)) << 52);  // 2^-s
    }
    __syncthreads();
    // pass 2: X = rint(x 2^s), four balanced byte digits, K permuted like the
    // widened codes, written as the swizzled A tiles; row sums of X
#pragma unroll
    for (int i = 0; i < kXinSlots; ++i) {
      const int slot = i * kThreads + tid, m = slot / Gp, j = slot - m * Gp;
      if (i * kThreads + warp * 32 >= ngp) break;
      long long part = 0;
      if (slot < ngp && j < G) {
        const int kb = j >> 3, c = j & 7;
        const int sx = tok_s[m];
        const float f1 = __int_as_float((sx / 2 + 127) << 23), f2 = __int_as_float((sx - sx / 2 + 127) << 23);
        int X[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          X[4 * q + 0] = __float2int_rn(__fmul_rn(__fmul_rn(v[i][q].x, f1), f2));
          X[4 * q + 1] = __float2int_rn(__fmul_rn(__fmul_rn(v[i][q].y, f1), f2));
          X[4 * q + 2] = __float2int_rn(__fmul_rn(__fmul_rn(v[i][q].z, f1), f2));
          X[4 * q + 3] = __float2int_rn(__fmul_rn(__fmul_rn(v[i][q].w, f1), f2));
        }
        uint32_t wv[16];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const int xv = X[perm16<BITS>(p)];
          part += xv;
          wv[p] = ((uint32_t)xv + 0x00808080u) ^ 0x00808080u;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t t01a = prmt(wv[4 * q], wv[4 * q + 1], 0x5140), t23a = prmt(wv[4 * q + 2], wv[4 * q + 3], 0x5140);
          const uint32_t t01b = prmt(wv[4 * q], wv[4 * q + 1], 0x7362), t23b = prmt(wv[4 * q + 2], wv[4 * q + 3], 0x7362);
          wv[4 * q] = prmt(t01a, t23a, 0x5410);
          wv[4 * q + 1] = prmt(t01a, t23a, 0x7632);
          wv[4 * q + 2] = prmt(t01b, t23b, 0x5410);
          wv[4 * q + 3] = prmt(t01b, t23b, 0x7632);
        }
        uint8_t *tile = xa + (size_t)kb * xa_tile;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
          const int r = 4 * m + l;
          *reinterpret_cast<uint4 *>(tile + r * 128 + ((c ^ (r & 7)) << 4)) =
              make_uint4(wv[l], wv[4 + l], wv[8 + l], wv[12 + l]);
        }
      }
      // |part| < 2^34: its 21-bit low and high halves sum exactly in 32 bits
      const int lo = __reduce_add_sync(seg, (int)(part & 0x1fffff));
      const int hi = __reduce_add_sync(seg, (int)(part >> 21));
      if (lead && slot < ngp)
        atomicAdd(reinterpret_cast<unsigned long long *>(&tok_zs[m]),
                  (unsigned long long)(((long long)hi << 21) + (long long)lo));
    }
    {  // limb rows past 4M read as zero
      const int pad = (int)(xa_tile >> 7) - 4 * a.M;
      for (int i = tid; i < kblocks * pad * 8; i += kThreads) {
        const int kb = i / (pad * 8), rem = i - kb * pad * 8;
        *reinterpret_cast<uint4 *>(xa + (size_t)kb * xa_tile + (size_t)(4 * a.M) * 128 + (size_t)rem * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
    }
    fence_proxy_async();  // the tiles are read by the tensor cores (async proxy)
    __syncthreads();
    if (tid < a.M) {
      const long long z = ZP * tok_zs[tid];
      tok_zc[tid] = KS > 1 ? 0 : z;   // unsplit: removed in the epilogue
      tok_zs[tid] = KS > 1 ? z : 0;   // split: removed from this split's partials
    }
  }

  if (warp == 0) {
    // ---- TMA producer: limb tiles and weight refills, in K-block order ----
    if (lane == 0 && !*abort_flag) {
      int xi = 0;
      bool ok = true;
      int jj = 0, r = 0, rslot = 0, rk = 0;  // position of K-block g in the raw stages
      int own = 0, ord = 0, base_ord = 0;    // limb-ring owner of K-block g
      for (int g = 0; g < kblocks; ++g) {
        if (jj == 0 && r >= issued) {
          if (!wait_phase(&raw_empty[rslot], (uint32_t)(rk - 1) & 1u)) {
            ok = false;
            break;
          }
          issue(r, rslot);
          issued = r + 1;
        }
        if (DIRECT) ord = base_ord + jj;
        if (!a.xin) {
          const int xslot = own * XI + (ord & (XI - 1));
          if (ord >= XI && !wait_phase(&xa_empty[xslot], (uint32_t)((ord >> XL) - 1) & 1u)) {
            ok = false;
            break;
          }
          issue_x(xslot, g);
          xi = g + 1;
        }
        if (++jj == kbr) {
          jj = 0;
          ++r;
          if (++rslot == RS) { rslot = 0; ++rk; }
          if (DIRECT && ++own == NI) { own = 0; base_ord += kbr; }
        }
        if (!DIRECT && ++own == NI) { own = 0; ++ord; }
      }
      if (!ok) *abort_flag = 1;
      if (*abort_flag) {
        // bounded drain of the copies still in flight before shared memory is released
        for (int rr = issued > RS ? issued - RS : 0; rr < issued; ++rr)
          (void)gqd::mbar_wait_bounded(&raw_full[rr % RS], (uint32_t)(rr / RS) & 1u, 100000000ull);
        for (int gg = 0; gg < xi; ++gg) {
          int o2;
          const int ow = x_owner(gg, o2);
          (void)gqd::mbar_wait_bounded(&xa_full[ow * XI + (o2 & (XI - 1))], (uint32_t)(o2 >> XL) & 1u, 100000000ull);
        }
        (void)gqd::mbar_wait_bounded(sc_bar, 0u, 100000000ull);
      }
    }
  } else if (warp <= kMaxIss) {
    // ---- MMA issue: K-blocks dealt round-robin to the issuers ----
    const int iss = warp - 1;
    if (lane == 0 && iss < NI) {
      const uint32_t dcol = tmem + (uint32_t)(iss * acc_cols);
      bool ok = !*abort_flag, first = true;
      int ord = 0;  // K-blocks this issuer has consumed (its limb-ring position)
      const int S = DIRECT ? RS : MS;
      const int units = DIRECT ? total_raw : kblocks;
      int slot = iss, par = 0;
      while (slot >= S) { slot -= S; par ^= 1; }
      const uint64_t xa_desc0 = sw128_desc(gqd::smem_u32(xa), 1024);
      const uint64_t w_desc0 = sw128_desc(gqd::smem_u32(DIRECT ? raw : wid), 1024);
      const uint32_t w_stride = (uint32_t)(DIRECT ? a.raw_bytes : a.mma_bytes);
      for (int u = iss; u < units && ok; u += NI) {
        const int ng = DIRECT ? min(kbr, kblocks - u * kbr) : 1;
        ok = wait_phase(DIRECT ? &raw_full[slot] : &mma_full[slot], (uint32_t)par);
        for (int j = 0; j < ng && ok; ++j) {
          // limb tile of this K-block: resident tile g (xin) or the issuer's ring slot
          const int xslot = a.xin ? (DIRECT ? u * kbr + j : u) : iss * XI + (ord & (XI - 1));
          if (!a.xin) ok = wait_phase(&xa_full[xslot], (uint32_t)(ord >> XL) & 1u);
          ++ord;
          if (!ok) break;
          tc_fence_after();
          const uint64_t ad = xa_desc0 + (uint64_t)(((uint32_t)xslot * xa_tile) >> 4);
          const uint64_t bd0 = w_desc0 + (uint64_t)((slot * w_stride + (DIRECT ? j * NW * tile_bytes : 0)) >> 4);
#pragma unroll
          for (int h = 0; h < NW; ++h) {
            const uint64_t bd = bd0 + (uint64_t)((h * tile_bytes) >> 4);
            if constexpr (WA) {  // D[weight row][limb row] = W . L^T
              const uint32_t d = dcol + (uint32_t)(h * a.lrows);
              tc_mma_i8(d, bd, ad, idesc, first ? 0u : 1u);
              tc_mma_i8(d, bd + 2, ad + 2, idesc, 1u);
              tc_mma_i8(d, bd + 4, ad + 4, idesc, 1u);
              tc_mma_i8(d, bd + 6, ad + 6, idesc, 1u);
            } else {
              for (int hh = 0; hh < MH; ++hh) {
                const uint32_t d = dcol + (uint32_t)((hh * NW + h) * a.tile_rows);
                const uint64_t ah = ad + (uint64_t)(hh * (16384 >> 4));  // rows 128*hh.. of the limb tile
                tc_mma_i8(d, ah, bd, idesc, first ? 0u : 1u);
                tc_mma_i8(d, ah + 2, bd + 2, idesc, 1u);
                tc_mma_i8(d, ah + 4, bd + 4, idesc, 1u);
                tc_mma_i8(d, ah + 6, bd + 6, idesc, 1u);
              }
            }
          }
          first = false;
          if (!a.xin) tc_commit(&xa_empty[xslot]);
        }
        if (!ok) break;
        tc_commit(DIRECT ? &raw_empty[slot] : &mma_empty[slot]);
        slot += NI;
        while (slot >= S) { slot -= S; par ^= 1; }
      }
      if (ok) tc_commit(&acc_full[iss]);
      if (!ok) *abort_flag = 1;
      tc_commit(&done_bar[iss]);
      if (!gqd::mbar_wait_bounded(&done_bar[iss], 0)) *abort_flag = 1;
    }
  } else if (!DIRECT) {
    // ---- warps 4-7: the rest of the widening ----
    bool ok = exp_ok && !*abort_flag;
    while (ok && er < total_raw) ok = expand_stage();
    if (!ok) *abort_flag = 1;
  }

  // ---- epilogue: all eight warps. Warp w reads TMEM lane quarter w % 4; the two
  // warps of a quarter take alternate column (or token) groups, and each group's
  // TMEM loads are all issued before one wait. ----
  if (!a.xin && tid < a.M) {
    tok_pw[tid] = __longlong_as_double((long long)(1023 - a.xexp[tid]) << 52);  // 2^-s
    tok_zc[tid] = ZP * a.sumx[tid];
    tok_bad[tid] = a.bad[tid];
    tok_zs[tid] = 0;
  }
  __syncthreads();
  // y of token tok, tile row nl (column n) from its exact sums (t0v: the weight, t1v: the up weight)
  auto finish = [&](long long t0v, long long t1v, int tok, int nl, int n) -> float {
    if (tok_bad[tok]) return __int_as_float(0x7fc00000);
    const double pwt = tok_pw[tok];
    const long long zct = tok_zc[tok];
    const float v0 = __fmul_rn((float)((double)(t0v - zct) * pwt), scb[nl]);
    if (MODE == 1) {
      const float v1 = __fmul_rn((float)((double)(t1v - zct) * pwt), scb[a.tile_rows + nl]);
      return __fmul_rn(gqd::gelu_tanh(v0), v1);
    } else if (MODE == 2) {
      return __fmul_rn(gqd::gelu_tanh(v0), a.bs[(size_t)tok * a.b_stride + a.b_off + n]);
    } else if (MODE == 3) {
      return a.cap > 0.0f ? __fmul_rn(a.cap, tanhf(__fdiv_rn(v0, a.cap))) : v0;
    }
    return v0;
  };
  {
    const int quarter = warp & 3, half = warp >> 2;
    bool ok = !*abort_flag && wait_phase(sc_bar, 0u);
    for (int i = 0; i < NI; ++i) ok = ok && wait_phase(&acc_full[i], 0u);
    if (WA && __all_sync(0xffffffffu, ok)) {
      // Thread (quarter, lane) owns weight row nl (TMEM lane nl); columns 4*tok + limb
      // hold the limb dot products of token tok, recombined here in int64. The two
      // warps of a quarter take alternate groups of 8 tokens.
      tc_fence_after();
      const int nl = quarter * 32 + lane, n = n_begin + nl;
      const bool nok = n < n_end;
      for (int t0 = 8 * half; t0 < a.M; t0 += 16) {
        long long T[NW][2][4];
#pragma unroll
        for (int h = 0; h < NW; ++h)
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int t = 0; t < 4; ++t) T[h][j][t] = 0;
        for (int i = 0; i < NI; ++i) {
          uint32_t d[NW][2][16];
#pragma unroll
          for (int h = 0; h < NW; ++h)
#pragma unroll
            for (int j = 0; j < 2; ++j)
              if (t0 + 4 * j < a.M)
                tmem_ld16_nowait(tmem + (uint32_t)(i * acc_cols + h * a.lrows + 4 * (t0 + 4 * j)) +
                                     ((uint32_t)(quarter * 32) << 16),
                                 d[h][j]);
#pragma unroll
          for (int h = 0; h < NW; ++h)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              tmem_wait_ld16(d[h][j]);
#pragma unroll
              for (int t = 0; t < 4; ++t)
#pragma unroll
                for (int l = 0; l < 4; ++l) T[h][j][t] += (long long)(int32_t)d[h][j][4 * t + l] << (8 * l);
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int tok = t0 + 4 * j + t;
            if (!nok || tok >= a.M) continue;
            if (KS > 1) {  // this split's exact partial sums, finalised after the cluster barrier
#pragma unroll
              for (int h = 0; h < NW; ++h) part[((size_t)h * a.M + tok) * a.tile_rows + nl] = T[h][j][t] - tok_zs[tok];
              continue;
            }
            a.y[(size_t)tok * a.ldy + a.y_col0 + n] = finish(T[0][j][t], T[NW - 1][j][t], tok, nl, n);
          }
      }
    } else if (!WA && __all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const int limb = lane & 3;
      const bool b1 = (lane & 1) != 0, b2 = (lane & 2) != 0;
      for (int hh = 0; hh < MH; ++hh) {
        // M=64: lane quarter q holds limb rows 16q.. in lanes 0-15 (tokens 4q..4q+3);
        // M=128: lane quarter q of half hh holds limb rows 128hh + 32q + lane.
        const int tok = a.mh == 0 ? 4 * quarter + ((lane >> 2) & 3) : 32 * hh + 8 * quarter + (lane >> 2);
        const bool lane_ok = (a.mh != 0 || lane < 16) && tok < a.M;
        for (int c0 = 8 * half; c0 < a.tile_rows; c0 += 16) {
          long long T[NW][2];
#pragma unroll
          for (int h = 0; h < NW; ++h) {
            uint32_t d[kMaxIss][8];
            const uint32_t col = (uint32_t)((hh * NW + h) * a.tile_rows + c0) + ((uint32_t)(quarter * 32) << 16);
#pragma unroll
            for (int i = 0; i < kMaxIss; ++i)
              if (i < NI) tmem_ld8_nowait(tmem + col + (uint32_t)(i * MH * NW * a.tile_rows), d[i]);
            uint32_t r[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) r[c] = 0;
#pragma unroll
            for (int i = 0; i < kMaxIss; ++i)
              if (i < NI) {
                tmem_wait_ld8(d[i]);
#pragma unroll
                for (int c = 0; c < 8; ++c) r[c] += d[i][c];
              }
            // The four lanes of a token hold limbs 0-3 of rows c0..c0+7: two 4x4
            // transposes inside the lane group leave lane `limb` with the four limb
            // sums of rows c0 + limb (r[0..3]) and c0 + 4 + limb (r[4..7]).
#pragma unroll
            for (int q = 0; q < 8; q += 4) {
              uint32_t t;
              t = __shfl_xor_sync(0xffffffffu, b1 ? r[q] : r[q + 1], 1);
              if (b1) r[q] = t; else r[q + 1] = t;
              t = __shfl_xor_sync(0xffffffffu, b1 ? r[q + 2] : r[q + 3], 1);
              if (b1) r[q + 2] = t; else r[q + 3] = t;
              t = __shfl_xor_sync(0xffffffffu, b2 ? r[q] : r[q + 2], 2);
              if (b2) r[q] = t; else r[q + 2] = t;
              t = __shfl_xor_sync(0xffffffffu, b2 ? r[q + 1] : r[q + 3], 2);
              if (b2) r[q + 1] = t; else r[q + 3] = t;
            }
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
              long long v = 0;
#pragma unroll
              for (int l = 0; l < 4; ++l) v += (long long)(int32_t)r[4 * hr + l] << (8 * l);
              T[h][hr] = v;
            }
          }
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const int nl = c0 + 4 * hr + limb;
            const int n = n_begin + nl;
            if (!lane_ok || n >= n_end) continue;
            if (KS > 1) {  // this split's exact partial sums, finalised after the cluster barrier
#pragma unroll
              for (int h = 0; h < NW; ++h) part[((size_t)h * a.M + tok) * a.tile_rows + nl] = T[h][hr] - tok_zs[tok];
              continue;
            }
            a.y[(size_t)tok * a.ldy + a.y_col0 + n] = finish(T[0][hr], T[NW - 1][hr], tok, nl, n);
          }
        }
      }
    } else {
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  int c_lo = n_begin, c_hi = n_end;  // output columns this CTA completes
  if (KS > 1) {
    // Every CTA of the cluster holds its split's partials; CTA sidx finalises
    // rows [r_lo, r_hi) of the tile for every token: the partials are summed in
    // int64 (exact, fixed order) over the cluster's shared memory.
    cluster_sync_all();
    const int per = ((a.tile_rows + KS - 1) / KS + 3) & ~3;
    const int r_lo = min(n_end - n_begin, sidx * per), r_hi = min(n_end - n_begin, r_lo + per);
    c_lo = n_begin + r_lo;
    c_hi = n_begin + r_hi;
    const int nr = r_hi - r_lo;
    if (!*abort_flag && nr > 0) {
      uint32_t rbase[8];  // the partials' base in every cluster CTA
#pragma unroll
      for (int q = 0; q < 8; ++q) rbase[q] = cluster_addr(part, (uint32_t)(q < KS ? q : 0));
      const int np = (nr + 1) >> 1;  // pairs of adjacent rows (r_lo is even, partial rows are 16-byte pairs)
      for (int idx = tid; idx < a.M * np; idx += kThreads) {
        const int tok = idx / np, nl = r_lo + 2 * (idx - tok * np);
        long long T[NW][2];
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          const uint32_t off = (uint32_t)((((size_t)h * a.M + tok) * a.tile_rows + nl) * 8);
          long long v[8][2];
#pragma unroll
          for (int q = 0; q < 8; ++q)  // all loads issued before the sums
            if (q < KS) ld_cluster_v2s64(rbase[q] + off, v[q][0], v[q][1]);
          T[h][0] = T[h][1] = 0;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (q < KS) {
              T[h][0] += v[q][0];
              T[h][1] += v[q][1];
            }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int nle = nl + e, n = n_begin + nle;
          if (nle >= r_hi) break;
          a.y[(size_t)tok * a.ldy + a.y_col0 + n] = finish(T[0][e], T[NW - 1][e], tok, nle, n);
        }
      }
    }
    __syncthreads();
  }
  // No CTA leaves (releasing its shared memory) while a cluster peer may still
  // read it: every thread has finished its reads of the peers' partials here, so
  // it arrives now and waits only at the exit, after the rest of the tail.
  if (KS > 1) cluster_arrive();
  if (!*abort_flag && (a.peers.n > 0 || a.peers.signal)) gqd::push_to_peers(a.y, a.peers, a.M, a.ldy, a.y_col0 + c_lo, a.y_col0 + c_hi);
  if (*abort_flag) {
    if (tid == 0) gqd::report(a.err, GQ_DEVERR_WAIT_TIMEOUT);
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
  }
  if (KS > 1) cluster_wait();
}

}  // namespace

namespace {

template <int BITS, bool SIGNED, int MODE>
int launch_x(gq_ctx *ctx, const CUtensorMap &m1, const CUtensorMap &m2, const TcxArgs &a, dim3 grid, size_t smem) {
  auto kern = a.wa ? gemv_tcx_kernel<BITS, SIGNED, MODE, true> : gemv_tcx_kernel<BITS, SIGNED, MODE, false>;
  static bool attr_set[64][2] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev][a.wa]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ctx->smem_optin));
    attr_set[dev][a.wa] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ctx->pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (a.ksplit > 1) {  // the split CTAs of one tile form a cluster (grid y = split index)
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = (unsigned)a.ksplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  GQ_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, m1, m2, a));
  return GQ_OK;
}

template <int BITS, bool SIGNED>
int launch_xm(gq_ctx *ctx, int mode, const CUtensorMap &m1, const CUtensorMap &m2, const TcxArgs &a, dim3 grid,
              size_t smem) {
  switch (mode) {
    case 0: return launch_x<BITS, SIGNED, 0>(ctx, m1, m2, a, grid, smem);
    case 1: return launch_x<BITS, SIGNED, 1>(ctx, m1, m2, a, grid, smem);
    case 2: return launch_x<BITS, SIGNED, 2>(ctx, m1, m2, a, grid, smem);
    default: return launch_x<BITS, SIGNED, 3>(ctx, m1, m2, a, grid, smem);
  }
}

struct TcxPlan {
  int wa, lrows;
  int tile_rows, mh, gx, slice_rows, kblocks, kbr, raw_stages, mma_stages, xa_stages, xi, raw_bytes, mma_bytes,
      xa_tile, issuers, tmem_cols;
  int ksplit, kb_per;
  int xin;  // limb tiles made in the GEMV (all of a CTA's K-blocks resident), no pre-pass
  size_t smem;
};

int mh_of(int64_t m) { return m <= 16 ? 0 : (m <= 32 ? 1 : 2); }

int tcx_max_tile(int64_t m, int nw, bool wa) {
  const int MH = (wa || mh_of(m) == 0) ? 1 : mh_of(m);
  return wa ? 128 : std::min(256 / nw, 512 / (MH * nw)) / 16 * 16;
}

// One tile of weight rows per CTA (tile_rows <= 0: the default, N / num_sms
// rounded up to 16). Weights taller than num_sms tiles run as row slices of
// num_sms * tile_rows rows. ks > 1 splits the K-blocks over a cluster of ks
// CTAs per tile (one slice only, either operand layout). Rings sized to the SM's
// shared memory for the CTA's own K-blocks: the limb ring gets up to ~half of
// it, the weight rings the rest.
bool tcx_plan_with(const gq_ctx *ctx, const gq_qweight *w, int64_t m, int nw, bool wa, int tile_rows, int ks,
                   TcxPlan &p) {
  const bool direct = (w->bits == 8 && w->signed_i8);
  const int kb_bytes = kKB * w->bits / 8;
  p.wa = wa;
  p.mh = wa ? 0 : mh_of(m);
  p.lrows = (int)((4 * m + 15) / 16 * 16);
  const int MH = (wa || p.mh == 0) ? 1 : p.mh;
  const int xa_rows = wa ? p.lrows : (p.mh == 0 ? 64 : 128 * p.mh);
  p.xa_tile = xa_rows * 128;
  const int max_tile = tcx_max_tile(m, nw, wa);
  const int64_t rows0 = (w->n + ctx->num_sms - 1) / ctx->num_sms;
  if (tile_rows <= 0) tile_rows = (int)std::min<int64_t>(max_tile, std::max<int64_t>(16, (rows0 + 15) / 16 * 16));
  if (wa) tile_rows = 128;
  if (tile_rows % 16 != 0 || tile_rows < 16 || tile_rows > max_tile) return false;
  p.tile_rows = tile_rows;
  const int acc_cols = wa ? nw * p.lrows : MH * nw * p.tile_rows;
  p.slice_rows = (int)std::min<int64_t>(w->n, (int64_t)ctx->num_sms * p.tile_rows);
  p.gx = (int)((p.slice_rows + p.tile_rows - 1) / p.tile_rows);
  p.kblocks = (int)((w->k + kKB - 1) / kKB);
  // split-K: a cluster of ks CTAs per tile, every split non-empty, one slice
  if (ks < 1 || ks > 8 || (ks > 1 && (p.slice_rows < w->n || (int64_t)p.gx * ks > ctx->num_sms))) return false;
  p.ksplit = ks;
  p.kb_per = (p.kblocks + ks - 1) / ks;
  if (ks > 1 && (int64_t)(ks - 1) * p.kb_per >= p.kblocks) return false;
  const int kbl = p.kb_per;  // K-blocks of one CTA (rings are sized for these)
  const int tile_bytes = p.tile_rows * 128;
  const int sc_bytes = nw * p.tile_rows * 4;
  const size_t budget = ctx->smem_optin - 1024;
  // issuers: TMEM columns, work units; then the limb ring: XI >= 2 slots each
  const int units_hint = direct ? kbl : kbl;
  p.issuers = wa ? 1 : std::max(1, std::min(std::min(kMaxIss, units_hint), 512 / acc_cols));
  const size_t xa_budget = std::min<size_t>(budget / 2 + 16384, 131072);
  while (p.issuers > 1 && (size_t)p.issuers * 2 * p.xa_tile > xa_budget) --p.issuers;
  p.xi = (int)std::max<size_t>(2, std::min<size_t>(kMaxXa / p.issuers, xa_budget / ((size_t)p.issuers * p.xa_tile)));
  p.xi = std::min(p.xi, std::max(2, (kbl + p.issuers - 1) / p.issuers));
  if (direct) {
    p.kbr = std::max(1, std::min(kbl, (8192 + nw * tile_bytes - 1) / (nw * tile_bytes)));
    p.raw_bytes = p.kbr * nw * tile_bytes;
    p.mma_bytes = 0;
    p.mma_stages = 0;
  } else {
    // K-blocks per packed stage: up to 256-byte TMA rows, stages of at most ~32 KB
    p.kbr = std::max(1, std::min(std::min(kbl, 256 / kb_bytes), 32768 / (nw * p.tile_rows * kb_bytes)));
    p.raw_bytes = (nw * p.tile_rows * p.kbr * kb_bytes + 1023) / 1024 * 1024;
    p.mma_bytes = nw * tile_bytes;
  }
  const int total_raw = (kbl + p.kbr - 1) / p.kbr;
  for (;;) {
    p.xa_stages = p.issuers * p.xi;
    if (!direct) {
      const TcxSmem L0 = tcx_layout(p.xa_stages, p.xa_tile, 2, p.raw_bytes, 0, p.mma_bytes, sc_bytes);
      const int fit = L0.total <= budget ? (int)((budget - L0.total) / p.mma_bytes) : 0;
      p.mma_stages = std::min(std::min(kMaxMma, kbl), fit);
    }
    const TcxSmem L1 = tcx_layout(p.xa_stages, p.xa_tile, 0, p.raw_bytes, p.mma_stages, p.mma_bytes, sc_bytes);
    const int fit = L1.total <= budget ? (int)((budget - L1.total) / p.raw_bytes) : 0;
    p.raw_stages = std::min(std::min(kMaxRaw, total_raw), fit);
    const bool ok = p.raw_stages >= std::min(2, total_raw) && (direct || p.mma_stages >= 2);
    if (ok) break;
    if (p.xi > 2) {
      --p.xi;
    } else if (p.issuers > 1) {
      --p.issuers;
      p.xi = 2;
    } else {
      return false;
    }
  }
  const int units = direct ? total_raw : kbl;
  p.issuers = std::min(p.issuers, std::max(1, units));
  // A ring that wraps must hand each slot back to the same issuer (slots are
  // consumed round-robin): its depth is then a multiple of the issuer count.
  if (direct && p.raw_stages < total_raw) {
    while (p.issuers > 1 && p.raw_stages < p.issuers) --p.issuers;
    p.raw_stages -= p.raw_stages % p.issuers;
  }
  if (!direct && p.mma_stages < kbl) {
    while (p.issuers > 1 && p.mma_stages < p.issuers) --p.issuers;
    p.mma_stages -= p.mma_stages % p.issuers;
  }
  while (p.xi & (p.xi - 1)) --p.xi;  // a power of two (slots and phases by mask and shift)
  p.xa_stages = p.issuers * p.xi;
  if (p.xa_stages > kMaxXa || p.xi < 2) return false;
  const int cols = p.issuers * acc_cols;
  p.tmem_cols = 32;
  while (p.tmem_cols < cols) p.tmem_cols <<= 1;
  p.smem = tcx_layout(p.xa_stages, p.xa_tile, p.raw_stages, p.raw_bytes, p.mma_stages, p.mma_bytes, sc_bytes).total;
  if (ks > 1) {  // the partials [nw][m][tile_rows] int64 overlay the rings
    const TcxSmem L = tcx_layout(p.xa_stages, p.xa_tile, p.raw_stages, p.raw_bytes, p.mma_stages, p.mma_bytes,
                                 sc_bytes);
    if ((size_t)nw * (size_t)m * (size_t)p.tile_rows * 8 > L.sc_off) return false;
  }
  p.xin = 0;
  if (p.tmem_cols > 512 || p.smem > budget) return false;
  // In-kernel limbs (GQ_TCX_XIN=1) when a CTA's share of x fits its threads'
  // registers (four 16-value groups each): its K-blocks' limb tiles all stay
  // resident (the weight rings shrink to make room) and the pre-pass launch goes
  // away. Measured slower on B200 than the pre-pass (config-2 sweep at M = 8:
  // 2.63 against 2.38 ms): a %globaltimer trace puts ~0.5 us on each converted
  // group slot in the run-once conversion code, more than the launch it saves.
  const char *xe = getenv("GQ_TCX_XIN");
  const int gk = kbl * 8, gp = gk <= 8 ? 8 : gk <= 16 ? 16 : (gk + 31) / 32 * 32;  // lane slots of a row
  if (xe && *xe == '1' && m * gp <= kThreads * kXinSlots) {
    TcxPlan q = p;
    q.xa_stages = kbl;
    for (;;) {
      const TcxSmem Lq = tcx_layout(q.xa_stages, q.xa_tile, q.raw_stages, q.raw_bytes, q.mma_stages, q.mma_bytes,
                                    sc_bytes);
      if (Lq.total <= budget && (ks == 1 || (size_t)nw * (size_t)m * (size_t)q.tile_rows * 8 <= Lq.sc_off)) {
        q.smem = Lq.total;
        q.xin = 1;
        p = q;
        break;
      }
      // shrink a weight ring, keeping every ring that wraps a multiple of the issuer count
      int nm = q.mma_stages - 1;
      nm -= nm % q.issuers;
      if (!direct && nm >= std::max(2, q.issuers)) {
        q.mma_stages = nm;
        continue;
      }
      int nr = q.raw_stages - 1;
      if (direct && nr < total_raw) nr -= nr % q.issuers;
      if (nr >= std::min(2, total_raw) && (!direct || nr >= total_raw || nr >= q.issuers)) {
        q.raw_stages = nr;
        continue;
      }
      break;  // does not fit: keep the pre-pass plan
    }
  }
  return true;
}

// Plan choice. The per-CTA cost grows with its K-block count (each K-block is
// a limb tile fetch and a few small MMAs), so long rows split K over a cluster:
// measured on the E2B projections (graph-replayed, M = 8 / 64, one B200):
//   K = 6144 (2-bit down)      25.6 -> 12.4 / 29.2 -> 15.9 us with 4 splits, 64-row tiles
//   K = 4096 (global o_proj)   14.0 -> 10.9 / 20.3 -> 13.9 us with 4 splits, 64-row tiles
//   K = 2048 (local o_proj)     9.2 ->  8.9 / 13.3 -> 11.5 us with 2 splits, 32-row tiles
//   N = 256, K = 1536 (PLE gate) 8.5 -> 7.6 / 12.1 ->  9.3 us with 4 splits, 32-row tiles
// and no gain for K = 1536 with N >= 2048 (q|k|v, gate|up) or K = 256. The first
// candidate that fits is taken. GQ_TCX_SPLIT="S" or "S:tile" forces a split
// count (and tile) when that plan fits.
bool tcx_plan(const gq_ctx *ctx, const gq_qweight *w, int64_t m, int nw, bool wa, TcxPlan &p) {
  const char *e = getenv("GQ_TCX_SPLIT");
  if (e && *e) {
    int ks = atoi(e), tile = 0;
    const char *c = strchr(e, ':');
    if (c) tile = atoi(c + 1);
    if (ks >= 1 && tcx_plan_with(ctx, w, m, nw, wa, tile, ks, p)) return true;
  } else if (wa) {
    // weights as A (128-row tiles): split K until the clusters cover the SMs
    const int64_t gx = (w->n + 127) / 128;
    for (int ks = (int)std::min<int64_t>(8, std::max<int64_t>(1, ctx->num_sms / gx)); ks > 1; --ks)
      if (tcx_plan_with(ctx, w, m, nw, wa, 128, ks, p)) return true;
  } else {
    const int kb = (int)((w->k + kKB - 1) / kKB);
    if (kb >= 24) {
      if (tcx_plan_with(ctx, w, m, nw, wa, 64, 4, p) || tcx_plan_with(ctx, w, m, nw, wa, 32, 2, p)) return true;
    } else if (kb >= 16) {
      if (tcx_plan_with(ctx, w, m, nw, wa, 32, 2, p)) return true;
    } else if (kb >= 8 && w->n <= 1024) {
      if (tcx_plan_with(ctx, w, m, nw, wa, 32, 4, p)) return true;
    }
  }
  return tcx_plan_with(ctx, w, m, nw, wa, 0, 1, p);
}

CUresult encode_w(CUtensorMap *map, const gq_qweight *w, const TcxPlan &p) {
  const bool direct = (w->bits == 8 && w->signed_i8);
  cuuint64_t dims[2] = {(cuuint64_t)w->row_bytes, (cuuint64_t)w->n};
  cuuint64_t strides[1] = {(cuuint64_t)w->row_bytes};
  cuuint32_t box[2] = {direct ? 128u : (cuuint32_t)(p.kbr * kKB * w->bits / 8), (cuuint32_t)p.tile_rows};
  cuuint32_t estr[2] = {1, 1};
  return gq_encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->bytes, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, direct ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int BITS>
cudaError_t launch_limbs(gq_ctx *ctx, const float *x, int64_t m, int64_t k, int64_t kp, int xa_rows, uint8_t *limbs,
                         int *xexp, long long *sumx, uint32_t *bad) {
  // m blocks write the token rows, one more zero-fills the tile rows past 4*m
  return gq_launch(ctx, xlimbs_kernel<BITS>, dim3((unsigned)(m + (4 * m < xa_rows ? 1 : 0))), dim3(kThreads), 0, x,
                   (int)k, (int)kp, (int)m, xa_rows, limbs, xexp, sumx, bad);
}

// Operand layout. Limb rows as A (M = 64 / 128) with weight tiles of 16..256
// rows as N, one tile per SM; or weights as A (128-row tiles, limb rows as N up
// to 256) with K split over a cluster so the grid still covers the SMs. Measured
// per E2B projection (graph-replayed chains, one B200): the weights-as-A split
// wins for one weight with long rows at small M (M = 8: 2-bit down 15.6 -> 12.5 us,
// o_proj 12.6 -> 10.6 us; M = 16 likewise) and loses for the fused gate|up pair
// (14.7 -> 24.7 us) and at M >= 32 (M = 64 gate|up 20.6 -> 39.1 us). GQ_TCX_WA=1|0
// forces either layout.
bool tcx_weights_as_a(int64_t m, const gq_qweight *w, int nw) {
  const char *e = getenv("GQ_TCX_WA");
  if (e && *e) return *e == '1';
  return nw == 1 && m <= 16 && w->k >= 2048;
}

// Rows [r0, r0 + n) of a weight as a weight of its own (same layout).
gq_qweight row_slice(const gq_qweight *w, int64_t r0, int64_t n) {
  gq_qweight v = *w;
  v.bytes = w->bytes + r0 * w->row_bytes;
  v.scales = w->scales + r0 * w->scale_stride;
  v.n = n;
  return v;
}

}  // namespace

// 3 <= M <= 64 activation rows, one scale per weight row, K a multiple of 16 up
// to 8192, 16-byte aligned x and packed rows.
bool gq_gemv_tcx_supported(gq_ctx *ctx, const gq_qweight *w, const float *x, int64_t m, int nw) {
  if (m < 3 || m > kMaxTok || w->group_size != w->k || w->k <= 0 || w->n <= 0) return false;
  if (w->k % 16 != 0 || w->k > kMaxK || w->n > (1ll << 30)) return false;
  if (w->row_bytes % 16 != 0 || (uintptr_t)w->bytes % 16 != 0 || (uintptr_t)x % 16 != 0) return false;
  if (gq_encode_fn() == nullptr) return false;
  TcxPlan p;
  return tcx_plan(ctx, w, m, nw, tcx_weights_as_a(m, w, nw), p);
}

int gq_gemv_tcx_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                       const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                       int64_t y_col0) {
  const int nw = (mode == 1) ? 2 : 1;
  TcxPlan p;
  if (!tcx_plan(ctx, w, m, nw, tcx_weights_as_a(m, w, nw), p))
    return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "gemv_tcx: no stage configuration fits");
  int rc = GQ_OK;
  uint8_t *limbs = nullptr;
  long long *sumx = nullptr;
  int *xexp = nullptr;
  uint32_t *bad = nullptr;
  if (!p.xin) {  // the limb pre-pass: one launch before the GEMV
    const int64_t kp = (int64_t)p.kblocks * kKB;
    const int xa_rows = p.xa_tile / 128;
    const size_t limb_bytes = ((size_t)p.kblocks * p.xa_tile + 255) & ~size_t(255);
    void *wsp = nullptr;
    rc = gq_workspace(ctx, limb_bytes + (size_t)m * 16 + 256, &wsp);
    if (rc != GQ_OK) return rc;
    limbs = static_cast<uint8_t *>(wsp);
    sumx = reinterpret_cast<long long *>(limbs + limb_bytes);
    xexp = reinterpret_cast<int *>(sumx + m);
    bad = reinterpret_cast<uint32_t *>(xexp + m);
    if (w->bits == 4) {
      GQ_CUDA_TRY(ctx, launch_limbs<4>(ctx, x, m, w->k, kp, xa_rows, limbs, xexp, sumx, bad));
    } else if (w->bits == 2) {
      GQ_CUDA_TRY(ctx, launch_limbs<2>(ctx, x, m, w->k, kp, xa_rows, limbs, xexp, sumx, bad));
    } else {
      GQ_CUDA_TRY(ctx, launch_limbs<8>(ctx, x, m, w->k, kp, xa_rows, limbs, xexp, sumx, bad));
    }
  }
  for (int64_t r0 = 0; r0 < w->n; r0 += p.slice_rows) {
    const int64_t rows = std::min<int64_t>(p.slice_rows, w->n - r0);
    const gq_qweight ws = row_slice(w, r0, rows);
    const gq_qweight ws2 = row_slice(w2 ? w2 : w, r0, rows);
    CUtensorMap m1, m2;
    if (encode_w(&m1, &ws, p) != CUDA_SUCCESS || encode_w(&m2, &ws2, p) != CUDA_SUCCESS)
      return gq_fail(ctx, GQ_ERR_CUDA, "gemv_tcx: weight tensor map");
    TcxArgs a = {};
    a.M = (int)m;
    a.K = (int)w->k;
    a.N = (int)rows;
    a.s = ws.scales;
    a.s2 = w2 ? ws2.scales : nullptr;
    a.bs = bs;
    a.b_stride = b_stride;
    a.b_off = b_off + r0;
    a.cap = cap;
    a.y = y;
    a.ldy = ldy;
    a.y_col0 = y_col0 + r0;
    a.xexp = xexp;
    a.sumx = sumx;
    a.bad = bad;
    a.limbs = limbs;
    a.x = x;
    a.xin = p.xin;
    a.tile_rows = p.tile_rows;
    a.mh = p.mh;
    a.wa = p.wa;
    a.lrows = p.lrows;
    a.kblocks = p.kblocks;
    a.kbr = p.kbr;
    a.raw_stages = p.raw_stages;
    a.mma_stages = p.mma_stages;
    a.xa_stages = p.xa_stages;
    a.xi = p.xi;
    a.xi_log2 = __builtin_ctz((unsigned)p.xi);
    a.raw_bytes = p.raw_bytes;
    a.mma_bytes = p.mma_bytes;
    a.xa_tile = p.xa_tile;
    a.issuers = p.issuers;
    a.tmem_cols = p.tmem_cols;
    a.ksplit = p.ksplit;
    a.kb_per = p.kb_per;
    a.err = ctx->dev_err;
    a.peers = ctx->peers;
    a.peers.signal = ctx->peers.signal && (r0 + p.slice_rows >= w->n);  // the launch that completes y
    const dim3 grid((unsigned)((rows + p.tile_rows - 1) / p.tile_rows), (unsigned)p.ksplit);
    if (w->bits == 4) rc = launch_xm<4, false>(ctx, mode, m1, m2, a, grid, p.smem);
    else if (w->bits == 2) rc = launch_xm<2, false>(ctx, mode, m1, m2, a, grid, p.smem);
    else if (w->signed_i8) rc = launch_xm<8, true>(ctx, mode, m1, m2, a, grid, p.smem);
    else rc = launch_xm<8, false>(ctx, mode, m1, m2, a, grid, p.smem);
    if (rc != GQ_OK) return rc;
  }
  return GQ_OK;
}
