// gemv_tc.cu — decode GEMV (M = 1 or 2 activation rows) on the tensor cores.
//
// Replaces the reference's MATMUL_Q shader (rust/src/kernels/matmul_q.wgsl:96-169,
// dispatched by rust/src/backend_wgpu.rs:646-695) for decode:
//   y[m, n] = epilogue( scale[n] * sum_k x[m, k] * q[n, k] )
// with the MODE epilogues of matmul_q.wgsl:18-21 (0 plain, 1 GeGLU with a second
// weight, 2 gelu * column slice) plus MODE 3 (logit soft-cap).
//
// The dot products are exact integer arithmetic on tcgen05.mma.kind::i8:
//  * x row m is turned into 30-bit fixed point, X = rint(x * 2^s_m) with s_m
//    chosen from max|x| so |X| < 2^30, and X is split into four signed bytes
//    X = L0 + 2^8 L1 + 2^16 L2 + 2^24 L3 (balanced digits, |L3| <= 64).
//  * The limbs are the MMA's A operand (rows = token*4 + limb, K-major,
//    128-byte swizzle). Only 8 rows exist: the descriptor's 8-row-group stride
//    is 0, so the M=64 MMA reads the same 1 KB atom eight times; an M=64
//    accumulator row r sits in TMEM lane 32*(r/16) + r%16, so lanes 0-15 of
//    every lane quarter hold two copies of the 8 limb rows.
//  * The weight rows are the B operand (MMA N = up to 256 rows). I8 rows go from
//    HBM straight into the swizzled operand layout by TMA: no instruction
//    touches them. 4-bit / 2-bit / U8 codes come in packed by TMA and 4
//    expander warps widen them to bytes (2 or 3 logic ops per 8 or 16 codes);
//    the K order inside each 16-code group is permuted the way the widening
//    falls out, and the limbs are written in the same permuted order.
//  * TMEM accumulates sum_k raw * L_l in s32 (|raw| <= 255, |L| <= 128,
//    K <= 8192: no overflow). A CTA with one tile splits its K-blocks over up
//    to three issuing threads with separate accumulators (one thread issuing
//    small MMAs is latency-bound); the epilogue adds them, recombines the limbs
//    in int64, removes the offset-binary zero point (zp * sum_k X, exact) and
//    converts once: y = f32(T * 2^-s_m) * scale[n]. The result is the exact dot
//    product of the codes with x rounded to 30 significant bits relative to
//    max|x|, rounded once, so it sits within float rounding of the reference's
//    CPU loop (rust/src/backend_cpu.rs:194-206).
//
// Overlap: one CTA per SM over a contiguous row range, sized so two CTAs fit per
// SM. Weight copies are issued, and sub-byte codes widened, before
// griddepcontrol.wait as far as the rings allow, so under programmatic dependent
// launch a kernel's weight stream runs under the tail of the kernel before it;
// only the x staging, the MMAs and the epilogue wait for the producer of x.
// Every wait is bounded (GQ_DEVERR_WAIT_TIMEOUT); TMA copies in flight are
// drained, outstanding MMAs committed and TMEM freed before the CTA exits.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "tc_common.cuh"

namespace {
using namespace gqt;

constexpr int kThreads = 256;  // warp 0 TMA, warps 1-3 MMA issue, warps 4-7 expanders + epilogue
constexpr int kKB = 128;       // codes per K-block: one 128-byte swizzle row of s8
constexpr int kMaxRaw = 8;     // packed / I8 stage ring
constexpr int kMaxMma = 16;    // widened stage ring (sub-byte and U8 codes)
constexpr int kMaxIss = 3;     // MMA issuing threads (warps 1-3), each with its own accumulator
constexpr int kExpWarps = 4;   // warps 4-7
constexpr int kMaxK = 8192;    // s32 accumulators: 255 * 128 * 8192 < 2^31

struct TcArgs {
  const float *x;
  int M, K, N;
  const float *s;
  const float *s2;
  const float *bs;
  int64_t b_stride, b_off;
  float cap;
  float *y;
  PeerDst peers;  // extra output destinations (peer buffers); n = 0: none
  int64_t ldy, y_col0;
  int rows_per_cta;  // whole tiles
  int tile_rows;     // MMA N: multiple of 16, <= 256
  int kblocks;       // ceil(K / 128)
  int kbr;           // K-blocks per raw stage
  int raw_stages, mma_stages;
  int raw_bytes, mma_bytes;
  int issuers;       // 1..3 (1 when a CTA owns several tiles)
  int tmem_cols;
  uint32_t *err;
};

struct TcSmem {
  uint32_t x_off, raw_off, mma_off, bar_off, misc_off, total;
};
__host__ __device__ inline TcSmem tc_layout(int kblocks, int raw_stages, int raw_bytes, int mma_stages,
                                            int mma_bytes) {
  TcSmem L;
  uint32_t o = 0;
  L.x_off = o;    o += (uint32_t)kblocks * 1024u;
  L.raw_off = o;  o += (uint32_t)raw_stages * (uint32_t)raw_bytes;
  L.mma_off = o;  o += (uint32_t)mma_stages * (uint32_t)mma_bytes;
  L.bar_off = o;  o += (2 * kMaxRaw + 2 * kMaxMma + 4 + 2 + kMaxIss) * 8;
  L.misc_off = o; o += 192;
  L.total = o + 1024;  // alignment slack for the 1024-byte swizzle atoms
  return L;
}

// Byte order of the codes the expanders produce inside a 16-code group
// (position p holds code perm16(p)); the limbs of x are laid out the same way.
template <int BITS>
__device__ __forceinline__ int perm16(int p) {
  if constexpr (BITS == 4) return (p & 8) | ((p & 3) << 1) | ((p >> 2) & 1);  // 0,2,4,6,1,3,5,7 per 8
  else if constexpr (BITS == 2) return ((p & 3) << 2) | (p >> 2);          // 0,4,8,12,1,5,...
  else return p;
}

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }  // e in [-126, 127]

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// One-poll fast path before the bounded wait (the common case: already complete).
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity) {
  return gqd::mbar_try_wait(bar, parity) || gqd::mbar_wait_bounded(bar, parity);
}

template <int BITS, bool SIGNED, int MT, int MODE>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_w2,
                   const TcArgs a) {
  constexpr int NW = (MODE == 1) ? 2 : 1;
  constexpr bool DIRECT = (BITS == 8 && SIGNED);  // I8: TMA lands the MMA operand itself
  constexpr int KB_BYTES = kKB * BITS / 8;        // packed bytes of one K-block of one row
  constexpr int CPR = KB_BYTES / 16;              // 16-byte packed chunks per row per K-block
  constexpr long long ZP = (BITS == 8) ? 0 : (1 << (BITS - 1));  // U8 is flipped to s8 when widened
  // D = A * B^T with A = the 8 limb rows (s8) read as M = 64 (eight aliased 8-row
  // groups), B = weight rows (s8, N = tile_rows), D s32. An M = 64 accumulator
  // row r lives in TMEM lane 32 * (r / 16) + r % 16: lanes 0-15 of every lane
  // quarter hold two copies of the 8 limb rows.
  const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.tile_rows >> 3) << 17) |
                         ((uint32_t)(64 >> 4) << 24);

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const TcSmem L = tc_layout(a.kblocks, a.raw_stages, a.raw_bytes, a.mma_stages, a.mma_bytes);
  uint8_t *xs = smem + L.x_off;    // [kblocks][8 limb rows x 128 B], swizzled
  uint8_t *raw = smem + L.raw_off;  // [raw_stages][raw_bytes]
  uint8_t *wid = smem + L.mma_off;  // [mma_stages][NW][tile_rows x 128 B], swizzled
  uint64_t *raw_full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *raw_empty = raw_full + kMaxRaw;
  uint64_t *mma_full = raw_empty + kMaxRaw;
  uint64_t *mma_empty = mma_full + kMaxMma;
  uint64_t *acc_full = mma_empty + kMaxMma;  // [4]: per issuer (one tile) or per TMEM buffer (several)
  uint64_t *acc_empty = acc_full + 4;        // [2]
  uint64_t *done_bar = acc_empty + 2;        // [kMaxIss]
  uint32_t *misc = reinterpret_cast<uint32_t *>(smem + L.misc_off);
  uint32_t *tmem_slot = misc;
  volatile uint32_t *abort_flag = misc + 1;
  uint32_t *bad_x = misc + 2;                                 // [2] non-finite x row
  int *xexp = reinterpret_cast<int *>(misc + 4);              // [2]
  long long *sumx = reinterpret_cast<long long *>(misc + 6);  // [2]
  float *maxs = reinterpret_cast<float *>(misc + 10);         // [2][8 warps]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_begin = blockIdx.x * a.rows_per_cta;
  const int n_end = min(a.N, n_begin + a.rows_per_cta);
  const int ntiles = n_end > n_begin ? (n_end - n_begin + a.tile_rows - 1) / a.tile_rows : 0;
  const int kblocks = a.kblocks, kbr = a.kbr, RS = a.raw_stages, MS = a.mma_stages, NI = a.issuers;
  const int spt = (kblocks + kbr - 1) / kbr;  // raw stages per tile
  const int total_raw = ntiles * spt;
  const int total_kb = ntiles * kblocks;
  const int tile_bytes = a.tile_rows * 128;   // one weight's widened K-block
  const bool multi = NI == 1 && a.rows_per_cta > a.tile_rows;

  if (tid == 0) {
    for (int i = 0; i < kMaxRaw; ++i) {
      gqd::mbar_init(&raw_full[i], 1);
      gqd::mbar_init(&raw_empty[i], DIRECT ? 1 : kExpWarps);
    }
    for (int i = 0; i < kMaxMma; ++i) {
      gqd::mbar_init(&mma_full[i], kExpWarps);
      gqd::mbar_init(&mma_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) gqd::mbar_init(&acc_full[i], 1);
    for (int i = 0; i < 2; ++i) gqd::mbar_init(&acc_empty[i], kExpWarps);
    for (int i = 0; i < kMaxIss; ++i) gqd::mbar_init(&done_bar[i], 1);
    *abort_flag = 0;
    bad_x[0] = bad_x[1] = 0;
    sumx[0] = sumx[1] = 0;
    gqd::fence_mbar_init();
  }
  __syncthreads();

  // raw stage r = (tile r / spt, K-blocks kb0 .. kb0 + kbr - 1 of it)
  auto issue = [&](int r) {
    const int slot = r % RS;
    const int t = r / spt, kb0 = (r % spt) * kbr;
    const int row0 = n_begin + t * a.tile_rows;
    uint8_t *dst = raw + slot * a.raw_bytes;
    if (DIRECT) {
      const int nkb = min(kbr, kblocks - kb0);
      gqd::mbar_arrive_expect_tx(&raw_full[slot], (uint32_t)(nkb * NW * tile_bytes));
      for (int j = 0; j < nkb; ++j)
        for (int h = 0; h < NW; ++h)
          tma_load_2d(dst + (j * NW + h) * tile_bytes, h ? &map_w2 : &map_w, (kb0 + j) * kKB, row0, &raw_full[slot]);
    } else {
      gqd::mbar_arrive_expect_tx(&raw_full[slot], (uint32_t)(NW * a.tile_rows * kbr * KB_BYTES));
      for (int h = 0; h < NW; ++h)
        tma_load_2d(dst + h * a.tile_rows * kbr * KB_BYTES, h ? &map_w2 : &map_w, kb0 * KB_BYTES, row0,
                    &raw_full[slot]);
    }
  };

  // Widen K-block g (index over this CTA's tiles) into widened slot g % MS.
  // Warp-uniform; returns false on a timed-out wait.
  auto expand = [&](int g) -> bool {
    const int et = tid - (kThreads - kExpWarps * 32);
    const int t = g / kblocks, kb = g % kblocks;
    const int r = t * spt + kb / kbr, rslot = r % RS, j = kb % kbr;
    const int mslot = g % MS;
    bool ok = !*abort_flag && wait_phase(&raw_full[rslot], (uint32_t)(r / RS) & 1u);
    ok = ok && (g < MS || wait_phase(&mma_empty[mslot], (uint32_t)((g / MS) - 1) & 1u));
    if (!__all_sync(0xffffffffu, ok)) return false;
    const int rstride = kbr * KB_BYTES;  // packed row stride inside the raw stage
    const int items = NW * a.tile_rows * CPR;
    for (int it = et; it < items; it += kExpWarps * 32) {
      const int h = it / (a.tile_rows * CPR);
      const int rem = it - h * (a.tile_rows * CPR);
      const int row = rem / CPR, ic = rem - row * CPR;
      const uint4 in = *reinterpret_cast<const uint4 *>(raw + rslot * a.raw_bytes + h * a.tile_rows * rstride +
                                                         row * rstride + j * KB_BYTES + ic * 16);
      uint8_t *dst = wid + mslot * a.mma_bytes + h * tile_bytes;
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
      } else {  // U8: offset binary -> two's complement
        const uint32_t f = 0x80808080u;
        *reinterpret_cast<uint4 *>(dst + sw128_off(row, ic)) = make_uint4(in.x ^ f, in.y ^ f, in.z ^ f, in.w ^ f);
      }
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&mma_full[mslot]);
      if (j == kbr - 1 || kb == kblocks - 1) mbar_arrive(&raw_empty[rslot]);
    }
    return true;
  };

  // ---- before the dependency wait: weights only (immutable after upload) ----
  // Sub-byte codes: K-blocks [0, G_pre) are widened before the wait, and a raw
  // stage whose K-blocks all lie there is refilled before the wait too (its
  // release needs only the expanders). I8 stages are released by the MMAs.
  const int G_pre = DIRECT ? 0 : min(MS, total_kb);
  auto last_kb = [&](int r) { return (r / spt) * kblocks + min((r % spt + 1) * kbr, kblocks) - 1; };
  int issued = 0;
  if (warp == 0 && lane == 0) {
    for (int r = 0; r < total_raw; ++r) {
      if (r >= RS) {
        if (DIRECT || last_kb(r - RS) >= G_pre) break;
        if (!wait_phase(&raw_empty[r % RS], (uint32_t)((r / RS) - 1) & 1u)) {
          *abort_flag = 1;
          break;
        }
      }
      issue(r);
      issued = r + 1;
    }
  }
  int g_exp = 0;
  bool exp_ok = true;
  if (!DIRECT && warp >= kThreads / 32 - kExpWarps) {
    while (exp_ok && g_exp < G_pre) exp_ok = expand(g_exp++);
    if (!exp_ok) *abort_flag = 1;
  }
  gqd::griddep_launch_dependents();
  gqd::griddep_wait();

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(gqd::smem_u32(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // ---- x -> 30-bit fixed point -> four signed byte limbs (A operand) ----
  // Pass 1 reads x from global memory (max|x|); pass 2 re-reads it from L1.
  {
    const int ngroups = kblocks * 8;  // 16-code groups, zero past K
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float mx = 0.0f;
      uint32_t bad = 0;
      if (m < a.M) {
        const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)m * a.K);
        for (int k4 = tid; k4 < a.K / 4; k4 += kThreads) {
          const float4 v = __ldg(xr + k4);
          mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
          bad |= !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
      }
      if (lane == 0) {
        maxs[m * 8 + warp] = mx;
        if (bad) atomicOr(&bad_x[m], 1u);
      }
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const bool live = m < a.M;
      const float4 *xr = reinterpret_cast<const float4 *>(a.x + (size_t)m * a.K);
      float bm = 0.0f;
#pragma unroll
      for (int i = 0; i < kThreads / 32; ++i) bm = fmaxf(bm, maxs[m * 8 + i]);
      int e = 0;
      if (bm > 0.0f && isfinite(bm)) frexpf(bm, &e);  // max|x| < 2^e
      const int s = 30 - e;                             // |x| * 2^s < 2^30
      const float f1 = pow2f(s / 2), f2 = pow2f(s - s / 2);
      long long part = 0;
      for (int gi = tid; gi < ngroups; gi += kThreads) {
        int X[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (live && gi * 16 < a.K) v = __ldg(xr + gi * 4 + q);
          X[4 * q + 0] = __float2int_rn(__fmul_rn(__fmul_rn(v.x, f1), f2));
          X[4 * q + 1] = __float2int_rn(__fmul_rn(__fmul_rn(v.y, f1), f2));
          X[4 * q + 2] = __float2int_rn(__fmul_rn(__fmul_rn(v.z, f1), f2));
          X[4 * q + 3] = __float2int_rn(__fmul_rn(__fmul_rn(v.w, f1), f2));
        }
        // Balanced base-256 digits of X in one add and one xor: with X' = X + 0x808080
        // the low three bytes of X' ^ 0x808080 read as s8 are the digits (carries
        // included) and the top byte is the signed leading digit (|.| <= 64).
        uint32_t wv[16];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const int v = X[perm16<BITS>(p)];
          part += v;
          wv[p] = ((uint32_t)v + 0x00808080u) ^ 0x00808080u;
        }
        uint32_t limb[4][4];  // [limb][word of the 16-byte chunk]: 4x4 byte transposes
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t t01a = prmt(wv[4 * q], wv[4 * q + 1], 0x5140), t23a = prmt(wv[4 * q + 2], wv[4 * q + 3], 0x5140);
          const uint32_t t01b = prmt(wv[4 * q], wv[4 * q + 1], 0x7362), t23b = prmt(wv[4 * q + 2], wv[4 * q + 3], 0x7362);
          limb[0][q] = prmt(t01a, t23a, 0x5410);
          limb[1][q] = prmt(t01a, t23a, 0x7632);
          limb[2][q] = prmt(t01b, t23b, 0x5410);
          limb[3][q] = prmt(t01b, t23b, 0x7632);
        }
        uint8_t *atom = xs + (gi >> 3) * 1024;
#pragma unroll
        for (int l = 0; l < 4; ++l)
          *reinterpret_cast<uint4 *>(atom + sw128_off(m * 4 + l, gi & 7)) =
              make_uint4(limb[l][0], limb[l][1], limb[l][2], limb[l][3]);
        if (MT == 1)  // rows 4-7 of the atom are read by the MMA: keep them zero
#pragma unroll
          for (int l = 0; l < 4; ++l)
            *reinterpret_cast<uint4 *>(atom + sw128_off(4 + l, gi & 7)) = make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) atomicAdd(reinterpret_cast<unsigned long long *>(&sumx[m]), (unsigned long long)part);
      if (tid == 0) xexp[m] = s;
    }
  }
  fence_proxy_async();  // limbs written by the generic proxy, read by tcgen05.mma
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer: refill raw stages as they are released ----
    if (lane == 0) {
      for (int r = issued; r < total_raw; ++r) {
        const int slot = r % RS;
        if (*abort_flag || !wait_phase(&raw_empty[slot], (uint32_t)((r / RS) - 1) & 1u)) {
          *abort_flag = 1;
          break;
        }
        issue(r);
        issued = r + 1;
      }
    }
  } else if (warp <= kMaxIss) {
    // ---- MMA issue: issuer i = warp - 1 (lane 0) ----
    const int iss = warp - 1;
    if (lane == 0 && iss < NI) {
      const uint32_t xs_addr = gqd::smem_u32(xs);
      const uint64_t ad0 = sw128_desc(xs_addr, 0);  // 8 limb rows, group stride 0
      bool ok = true;
      if (!multi) {
        // one tile: the K-blocks are dealt round-robin to the issuers, each into its own accumulator
        const uint32_t dcol = tmem + (uint32_t)(iss * NW * a.tile_rows);
        bool first = true;
        if (DIRECT) {
          for (int r = iss; r < total_raw && ok; r += NI) {
            const int slot = r % RS, kb0 = r * kbr, nkb = min(kbr, kblocks - kb0);
            ok = !*abort_flag && wait_phase(&raw_full[slot], (uint32_t)(r / RS) & 1u);
            if (!ok) break;
            tc_fence_after();
            const uint32_t sbase = gqd::smem_u32(raw + slot * a.raw_bytes);
            for (int j = 0; j < nkb; ++j) {
              const uint64_t ad = ad0 + (uint64_t)(((kb0 + j) * 1024) >> 4);
#pragma unroll
              for (int h = 0; h < NW; ++h) {
                const uint64_t bd = sw128_desc(sbase + (j * NW + h) * tile_bytes, 1024);
                const uint32_t d = dcol + h * a.tile_rows;
                tc_mma_i8(d, ad, bd, idesc, first ? 0u : 1u);
                tc_mma_i8(d, ad + 2, bd + 2, idesc, 1u);
                tc_mma_i8(d, ad + 4, bd + 4, idesc, 1u);
                tc_mma_i8(d, ad + 6, bd + 6, idesc, 1u);
              }
              first = false;
            }
            tc_commit(&raw_empty[slot]);
          }
        } else {
          for (int g = iss; g < total_kb && ok; g += NI) {
            const int slot = g % MS;
            ok = !*abort_flag && wait_phase(&mma_full[slot], (uint32_t)(g / MS) & 1u);
            if (!ok) break;
            tc_fence_after();
            const uint64_t ad = ad0 + (uint64_t)((g * 1024) >> 4);
            const uint32_t sbase = gqd::smem_u32(wid + slot * a.mma_bytes);
#pragma unroll
            for (int h = 0; h < NW; ++h) {
              const uint64_t bd = sw128_desc(sbase + h * tile_bytes, 1024);
              const uint32_t d = dcol + h * a.tile_rows;
              tc_mma_i8(d, ad, bd, idesc, first ? 0u : 1u);
              tc_mma_i8(d, ad + 2, bd + 2, idesc, 1u);
              tc_mma_i8(d, ad + 4, bd + 4, idesc, 1u);
              tc_mma_i8(d, ad + 6, bd + 6, idesc, 1u);
            }
            first = false;
            tc_commit(&mma_empty[slot]);
          }
        }
        if (ok) tc_commit(&acc_full[iss]);
      } else {
        // several tiles, one issuer, two TMEM buffers (the epilogue drains one while the other fills)
        for (int t = 0; t < ntiles && ok; ++t) {
          const int buf = t & 1;
          if (t >= 2 && !(ok = !*abort_flag && wait_phase(&acc_empty[buf], (uint32_t)((t / 2) - 1) & 1u))) break;
          tc_fence_after();
          const uint32_t dcol = tmem + (uint32_t)(buf * NW * a.tile_rows);
          for (int kb = 0; kb < kblocks && ok; ++kb) {
            uint32_t bbase;
            int slot, j = 0;
            if (DIRECT) {
              const int r = t * spt + kb / kbr;
              slot = r % RS;
              j = kb % kbr;
              if (j == 0 && !(ok = !*abort_flag && wait_phase(&raw_full[slot], (uint32_t)(r / RS) & 1u))) break;
              bbase = gqd::smem_u32(raw + slot * a.raw_bytes + j * NW * tile_bytes);
            } else {
              const int g = t * kblocks + kb;
              slot = g % MS;
              if (!(ok = !*abort_flag && wait_phase(&mma_full[slot], (uint32_t)(g / MS) & 1u))) break;
              bbase = gqd::smem_u32(wid + slot * a.mma_bytes);
            }
            tc_fence_after();
            const uint64_t ad = ad0 + (uint64_t)((kb * 1024) >> 4);
#pragma unroll
            for (int h = 0; h < NW; ++h) {
              const uint64_t bd = sw128_desc(bbase + h * tile_bytes, 1024);
              const uint32_t d = dcol + h * a.tile_rows;
              tc_mma_i8(d, ad, bd, idesc, kb != 0 ? 1u : 0u);
              tc_mma_i8(d, ad + 2, bd + 2, idesc, 1u);
              tc_mma_i8(d, ad + 4, bd + 4, idesc, 1u);
              tc_mma_i8(d, ad + 6, bd + 6, idesc, 1u);
            }
            if (DIRECT) {
              if (j == kbr - 1 || kb == kblocks - 1) tc_commit(&raw_empty[slot]);
            } else {
              tc_commit(&mma_empty[slot]);
            }
          }
          if (ok) tc_commit(&acc_full[buf]);
        }
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued has completed once this fires
      tc_commit(&done_bar[iss]);
      if (!gqd::mbar_wait_bounded(&done_bar[iss], 0)) *abort_flag = 1;
    }
  } else {
    // ---- warps 4-7: the rest of the widening, then the epilogue ----
    if (!DIRECT) {
      bool ok = exp_ok && !*abort_flag;
      for (int g = g_exp; ok && g < total_kb; ++g) ok = expand(g);
      if (!ok) *abort_flag = 1;
    }
    const int quarter = warp & 3;
    const int lrow = lane & 7;              // limb row this lane's TMEM lane holds (lanes 0-15)
    const int tok = lrow >> 2, limb = lrow & 3;
    const int cp = (lane >> 3) & 1;         // which of the quarter's two copies
    const bool lane_ok = lane < 16;
    double pw[MT];
    long long zc[MT];
    bool badr[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      pw[m] = __longlong_as_double((long long)(1023 - xexp[m]) << 52);  // 2^-s
      zc[m] = ZP * sumx[m];
      badr[m] = bad_x[m] != 0;
    }
    const double pwt = (MT == 2 && tok) ? pw[MT - 1] : pw[0];
    const long long zct = (MT == 2 && tok) ? zc[MT - 1] : zc[0];
    const bool badt = (MT == 2 && tok) ? badr[MT - 1] : badr[0];
    const int nacc = multi ? 1 : NI;
    constexpr int KC = 8;  // 8-column chunks per warp per tile: tile_rows <= 256 = 4 warps x 8 x 8
    for (int t = 0; t < ntiles; ++t) {
      const int buf = multi ? (t & 1) : 0;
      const int row0 = n_begin + t * a.tile_rows;
      // epilogue operands do not depend on the MMAs: fetch them before waiting
      float sc[KC], sc2[KC], bsv[KC];
#pragma unroll
      for (int k = 0; k < KC; ++k) {
        const int c0 = 8 * quarter + 32 * k;
        const int n = row0 + c0 + 4 * cp + limb;
        const bool live = c0 < a.tile_rows && lane_ok && tok < MT && tok < a.M && n < n_end;
        sc[k] = live ? __ldg(a.s + n) : 0.0f;
        sc2[k] = (MODE == 1 && live) ? __ldg(a.s2 + n) : 0.0f;
        bsv[k] = (MODE == 2 && live) ? a.bs[(size_t)tok * a.b_stride + a.b_off + n] : 0.0f;
      }
      bool ok = !*abort_flag;
      if (multi) {
        ok = ok && wait_phase(&acc_full[buf], (uint32_t)(t / 2) & 1u);
      } else {
        for (int i = 0; i < NI; ++i) ok = ok && wait_phase(&acc_full[i], 0u);
      }
      if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform: tcgen05.ld and shuffles need the whole warp
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < KC; ++k) {
        const int c0 = 8 * quarter + 32 * k;
        if (c0 >= a.tile_rows) break;
        // 8 columns: lane (copy cp, limb) finishes column c0 + 4 * cp + limb
        long long T[NW];
#pragma unroll
        for (int h = 0; h < NW; ++h) {
          uint32_t d[kMaxIss][8];
          const uint32_t col = (uint32_t)(h * a.tile_rows + c0) + ((uint32_t)(quarter * 32) << 16);
#pragma unroll
          for (int i = 0; i < kMaxIss; ++i)
            if (i < nacc) tmem_ld8_nowait(tmem + col + (uint32_t)((multi ? buf : i) * NW * a.tile_rows), d[i]);
          int32_t dsum[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) dsum[c] = 0;
#pragma unroll
          for (int i = 0; i < kMaxIss; ++i)
            if (i < nacc) {
              tmem_wait_ld8(d[i]);
#pragma unroll
              for (int c = 0; c < 8; ++c) dsum[c] += (int32_t)d[i][c];
            }
          // recombine the limbs: lanes limb 0..3 of a token hold sum_k raw * L_limb
          T[h] = 0;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            long long v = (long long)dsum[c] << (8 * limb);
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            if (c == 4 * cp + limb) T[h] = v;
          }
        }
        const int n = row0 + c0 + 4 * cp + limb;
        if (lane_ok && tok < MT && tok < a.M && n < n_end) {
          float o;
          if (badt) {
            o = __int_as_float(0x7fc00000);
          } else {
            const float v0 = __fmul_rn((float)((double)(T[0] - zct) * pwt), sc[k]);
            if (MODE == 1) {
              const float v1 = __fmul_rn((float)((double)(T[NW - 1] - zct) * pwt), sc2[k]);
              o = __fmul_rn(gqd::gelu_tanh(v0), v1);
            } else if (MODE == 2) {
              o = __fmul_rn(gqd::gelu_tanh(v0), bsv[k]);
            } else if (MODE == 3) {
              o = a.cap > 0.0f ? __fmul_rn(a.cap, tanhf(__fdiv_rn(v0, a.cap))) : v0;
            } else {
              o = v0;
            }
          }
          a.y[(size_t)tok * a.ldy + a.y_col0 + n] = o;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (multi && lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (!*abort_flag && (a.peers.n > 0 || a.peers.signal))
    gqd::push_to_peers(a.y, a.peers, a.M, a.ldy, a.y_col0 + n_begin, a.y_col0 + n_end);
  if (*abort_flag) {
    if (tid == 0) gqd::report(a.err, GQ_DEVERR_WAIT_TIMEOUT);
    if (warp == 0 && lane == 0) {
      // bounded drain of the copies still in flight before shared memory is released
      for (int r = issued > RS ? issued - RS : 0; r < issued; ++r)
        (void)gqd::mbar_wait_bounded(&raw_full[r % RS], (uint32_t)(r / RS) & 1u, 100000000ull);
    }
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols) : "memory");
  }
}

template <int BITS, bool SIGNED, int MT, int MODE>
int launch_t(gq_ctx *ctx, const CUtensorMap &m1, const CUtensorMap &m2, const TcArgs &a, dim3 grid, size_t smem) {
  auto kern = gemv_tc_kernel<BITS, SIGNED, MT, MODE>;
  static bool attr_set[64] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ctx->smem_optin / 2 - 1024));
    attr_set[dev] = true;
  }
  GQ_CUDA_TRY(ctx, gq_launch(ctx, kern, grid, dim3(kThreads), smem, m1, m2, a));
  return GQ_OK;
}

template <int BITS, bool SIGNED, int MT>
int launch_mode(gq_ctx *ctx, int mode, const CUtensorMap &m1, const CUtensorMap &m2, const TcArgs &a, dim3 grid,
                size_t smem) {
  switch (mode) {
    case 0: return launch_t<BITS, SIGNED, MT, 0>(ctx, m1, m2, a, grid, smem);
    case 1: return launch_t<BITS, SIGNED, MT, 1>(ctx, m1, m2, a, grid, smem);
    case 2: return launch_t<BITS, SIGNED, MT, 2>(ctx, m1, m2, a, grid, smem);
    default: return launch_t<BITS, SIGNED, MT, 3>(ctx, m1, m2, a, grid, smem);
  }
}

template <int BITS, bool SIGNED>
int launch_mt(gq_ctx *ctx, int mt, int mode, const CUtensorMap &m1, const CUtensorMap &m2, const TcArgs &a,
              dim3 grid, size_t smem) {
  if (mt == 1) return launch_mode<BITS, SIGNED, 1>(ctx, mode, m1, m2, a, grid, smem);
  return launch_mode<BITS, SIGNED, 2>(ctx, mode, m1, m2, a, grid, smem);
}

struct TcPlan {
  int rows_per_cta, tile_rows, kblocks, kbr, raw_stages, mma_stages, raw_bytes, mma_bytes, issuers, tmem_cols, gx;
  bool chained;  // widened ring smaller than a CTA's K-blocks: widening waits on MMA progress
  size_t smem;
};

bool tc_plan(const gq_ctx *ctx, const gq_qweight *w, int nw, TcPlan &p) {
  const bool direct = (w->bits == 8 && w->signed_i8);
  const int kb_bytes = kKB * w->bits / 8;
  const int max_tile = nw == 2 ? 128 : 256;  // two TMEM buffers of nw x tile columns within 512
  const int64_t rows0 = (w->n + ctx->num_sms - 1) / ctx->num_sms;
  const int ntc = (int)((rows0 + max_tile - 1) / max_tile);
  p.tile_rows = (int)((((rows0 + ntc - 1) / ntc) + 15) / 16 * 16);
  p.rows_per_cta = ntc * p.tile_rows;
  p.gx = (int)((w->n + p.rows_per_cta - 1) / p.rows_per_cta);
  p.kblocks = (int)((w->k + kKB - 1) / kKB);
  const int tile_bytes = p.tile_rows * 128;
  // two CTAs per SM (programmatic dependent launch); 1 KB per CTA is reserved
  const size_t budget = ctx->smem_optin / 2 - 1024;
  p.chained = false;
  if (direct) {
    p.kbr = std::max(1, std::min(p.kblocks, (8192 + nw * tile_bytes - 1) / (nw * tile_bytes)));
    p.raw_bytes = p.kbr * nw * tile_bytes;  // multiple of 1024 (tile_rows % 8 == 0)
    p.mma_bytes = 0;
    p.mma_stages = 0;
  } else {
    p.kbr = std::max(1, std::min(p.kblocks, 256 / kb_bytes));  // TMA box inner extent <= 256 bytes
    p.raw_bytes = (nw * p.tile_rows * p.kbr * kb_bytes + 1023) / 1024 * 1024;
    p.mma_bytes = nw * tile_bytes;
    // widened ring: every K-block of the CTA when it fits next to two raw stages
    const int total_kb = ntc * p.kblocks;
    const TcSmem L0 = tc_layout(p.kblocks, std::min(2, ntc * ((p.kblocks + p.kbr - 1) / p.kbr)), p.raw_bytes, 0,
                                p.mma_bytes);
    const int fit = L0.total <= budget ? (int)((budget - L0.total) / p.mma_bytes) : 0;
    p.mma_stages = std::min(std::min(kMaxMma, total_kb), fit);
    p.chained = p.mma_stages < total_kb;
    if (p.mma_stages < 2) return false;
  }
  const int spt = (p.kblocks + p.kbr - 1) / p.kbr;
  const int total_raw = ntc * spt;
  const TcSmem L1 = tc_layout(p.kblocks, 0, p.raw_bytes, p.mma_stages, p.mma_bytes);
  const int fit = L1.total <= budget ? (int)((budget - L1.total) / p.raw_bytes) : 0;
  p.raw_stages = std::min(std::min(kMaxRaw, total_raw), fit);
  if (p.raw_stages < std::min(2, total_raw)) return false;
  // One tile per CTA: up to three issuers split the K-blocks, each into its own
  // accumulator (a single issuing thread is latency-bound on small MMAs).
  // Several tiles: one issuer and two accumulator buffers.
  if (ntc == 1) {
    const int units = direct ? total_raw : p.kblocks;
    p.issuers = std::max(1, std::min(std::min(kMaxIss, units), 512 / (nw * p.tile_rows)));
    // Slots of a ring that wraps must return to the same issuer (units are dealt
    // round-robin; an mbarrier parity wait cannot tell a phase two completions
    // ahead from a completed one): the depth is then a multiple of the issuers.
    if (direct && p.raw_stages < total_raw) {
      while (p.issuers > 1 && p.raw_stages < p.issuers) --p.issuers;
      p.raw_stages -= p.raw_stages % p.issuers;
    }
    if (!direct && p.mma_stages < p.kblocks) {
      while (p.issuers > 1 && p.mma_stages < p.issuers) --p.issuers;
      p.mma_stages -= p.mma_stages % p.issuers;
    }
  } else {
    p.issuers = 1;
  }
  const int cols = (ntc > 1 ? 2 : p.issuers) * nw * p.tile_rows;
  p.tmem_cols = 32;
  while (p.tmem_cols < cols) p.tmem_cols <<= 1;
  p.smem = tc_layout(p.kblocks, p.raw_stages, p.raw_bytes, p.mma_stages, p.mma_bytes).total;
  return p.tmem_cols <= 512 && p.smem <= budget;
}

CUresult encode_map(CUtensorMap *map, const gq_qweight *w, const TcPlan &p) {
  const bool direct = (w->bits == 8 && w->signed_i8);
  cuuint64_t dims[2] = {(cuuint64_t)w->row_bytes, (cuuint64_t)w->n};
  cuuint64_t strides[1] = {(cuuint64_t)w->row_bytes};
  cuuint32_t box[2] = {direct ? 128u : (cuuint32_t)(p.kbr * kKB * w->bits / 8), (cuuint32_t)p.tile_rows};
  cuuint32_t estr[2] = {1, 1};
  return gq_encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->bytes, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, direct ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace

// The tensor-core decode GEMV takes M <= 2 activation rows, one scale per weight
// row, K a multiple of 16 up to 8192, 16-byte aligned x and packed rows.
bool gq_gemv_tc_supported(gq_ctx *ctx, const gq_qweight *w, const float *x, int64_t m, int nw) {
  if (m < 1 || m > 2 || w->group_size != w->k || w->k <= 0 || w->n <= 0) return false;
  if (w->k % 16 != 0 || w->k > kMaxK || w->n > (1ll << 30)) return false;
  if (w->row_bytes % 16 != 0 || (uintptr_t)w->bytes % 16 != 0 || (uintptr_t)x % 16 != 0) return false;
  if (gq_encode_fn() == nullptr) return false;
  TcPlan p;
  if (!tc_plan(ctx, w, nw, p)) return false;
  // One CTA's codes widened in a ring smaller than its K-blocks make the
  // widening wait on MMA progress; for one small tile per CTA the CUDA-core
  // GEMV is faster, for many large tiles the ring streams fine.
  return !(p.chained && p.rows_per_cta <= p.tile_rows);
}

int gq_gemv_tc_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                      const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                      int64_t y_col0) {
  const int nw = (mode == 1) ? 2 : 1;
  TcPlan p;
  if (!tc_plan(ctx, w, nw, p)) return gq_fail(ctx, GQ_ERR_UNSUPPORTED, "gemv_tc: no stage configuration fits");
  CUtensorMap m1, m2;
  if (encode_map(&m1, w, p) != CUDA_SUCCESS || encode_map(&m2, w2 ? w2 : w, p) != CUDA_SUCCESS)
    return gq_fail(ctx, GQ_ERR_CUDA, "gemv_tc: weight tensor map");
  TcArgs a = {};
  a.x = x;
  a.M = (int)m;
  a.K = (int)w->k;
  a.N = (int)w->n;
  a.s = w->scales;
  a.s2 = w2 ? w2->scales : nullptr;
  a.bs = bs;
  a.b_stride = b_stride;
  a.b_off = b_off;
  a.cap = cap;
  a.y = y;
  a.ldy = ldy;
  a.y_col0 = y_col0;
  a.rows_per_cta = p.rows_per_cta;
  a.tile_rows = p.tile_rows;
  a.kblocks = p.kblocks;
  a.kbr = p.kbr;
  a.raw_stages = p.raw_stages;
  a.mma_stages = p.mma_stages;
  a.raw_bytes = p.raw_bytes;
  a.mma_bytes = p.mma_bytes;
  a.issuers = p.issuers;
  a.tmem_cols = p.tmem_cols;
  a.err = ctx->dev_err;
  a.peers = ctx->peers;
  const int mt = m <= 1 ? 1 : 2;
  const dim3 grid((unsigned)p.gx);
  if (w->bits == 4) return launch_mt<4, false>(ctx, mt, mode, m1, m2, a, grid, p.smem);
  if (w->bits == 2) return launch_mt<2, false>(ctx, mt, mode, m1, m2, a, grid, p.smem);
  if (w->signed_i8) return launch_mt<8, true>(ctx, mt, mode, m1, m2, a, grid, p.smem);
  return launch_mt<8, false>(ctx, mt, mode, m1, m2, a, grid, p.smem);
}
