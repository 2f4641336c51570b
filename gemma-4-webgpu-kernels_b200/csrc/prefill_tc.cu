// prefill_tc.cu — prefill dequantizing GEMM on the 5th-generation tensor cores.
//
// Replaces the reference's MATMUL_Q_TILED shader (rust/src/kernels/matmul_q_tiled.wgsl:
// 39-126, chosen for M >= 16 at rust/src/backend_wgpu.rs:663-673), whose W tile is
// dequantized to f32 in workgroup memory and multiplied with f32 FMAs. Here:
//   C[m, n] = epilogue( s[n] * 2^-e[m] * sum_k f16(x[m, k] * 2^e[m]) * q[n, k] )
// with f16 operands and fp32 accumulation in tensor memory (TMEM):
//  * a cast kernel scales each activation row by a power of two chosen from its
//    max|x| (so |x * 2^e| < 2^14, far inside the f16 range; the scaling is exact
//    and undone in the epilogue) and rounds it to f16 — 11 significant bits, 3
//    more than bf16. It also permutes K inside every 8 / 16-code group into the
//    order the weight widening below produces, so no instruction reorders codes;
//  * the MMA is D[weight rows, tokens] = W[128 rows, K] x X[NT tokens, K]^T: the
//    weights are the A operand and live in TMEM, x is the B operand in shared
//    memory. One thread issues TMA copies of the f16 x tile (NT x 64, 128-byte
//    swizzle) and of the packed weight tile (128 rows x 64 codes) into a load
//    ring;
//  * 8 producer warps (two groups of four, alternate stages) widen the packed
//    codes of their lane's weight row to f16 and write them into a TMEM A ring
//    with tcgen05.st: a code masked into the mantissa of f16 1024 (0x6400 | n) is
//    exactly 1024 + n, so one LOP3 per code pair and one HSUB2/HFMA2 give the
//    signed codes (9 instructions per 8 nibbles, 17 per 16 crumbs, 5 per 4
//    bytes). The widened weights never touch shared memory: per stage the
//    shared-memory traffic is the x tile (TMA write + MMA read) and the packed
//    codes, which keeps the tensor pipe, not shared-memory bandwidth, the limit;
//  * one elected thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=NT,
//    K=16, A from TMEM) into an fp32 TMEM accumulator and commits each consumed
//    stage back to both rings, then the accumulator to the epilogue;
//  * the 8 producer warps read the accumulator back with tcgen05.ld (lane = weight
//    row, so every store instruction writes 32 consecutive outputs of one token
//    row), apply the row and weight scales and the MODE epilogue (0 plain, 1
//    GeGLU, 2 gelu * column slice, 3 soft-cap).
// For MODE 1 the 128 weight rows of a tile are 64 gate rows followed by the same
// 64 up rows; the up halves go through shared memory to the gate warps.
//
// Every wait is bounded (2 s); a timeout sets GQ_DEVERR_WAIT_TIMEOUT, drains,
// frees TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "tc_common.cuh"

namespace {

constexpr int MW = 128;        // weight rows per tile (MMA M)
constexpr int NT_MAX = 256;    // tokens per tile (MMA N): 256, or 128 for short prefills
constexpr int BK = 64;         // K per stage: one 128-byte swizzle row of f16
constexpr int kThreads = 320;  // warp 0: TMA, warp 1: MMA + TMEM, warps 2-9: producers, then epilogue
constexpr int kProdWarps = 8;
constexpr int AS = 4;                         // TMEM A ring stages
constexpr uint32_t A_COLS = BK / 2;           // 64 f16 per row = 32 TMEM columns per stage
constexpr uint32_t TMEM_COLS = 512;           // accumulator (NT columns) + A ring
constexpr uint32_t A_COL0 = NT_MAX;           // the A ring sits after the accumulator
constexpr uint32_t X_STAGE = NT_MAX * BK * 2;  // 32 KB

// Load-ring depth per code width (x tile + packed weight tile per stage).
template <int BITS>
struct Ring {
  static constexpr uint32_t PW = MW * BK * BITS / 8;  // packed bytes per stage
  static constexpr int LS = BITS == 8 ? 5 : 6;
  static constexpr size_t kSmem =
      1024 + (size_t)LS * (X_STAGE + PW) + (2 * LS + 2 * AS + 1) * 8 + 16 + 2 * NT_MAX * sizeof(float);
};

struct PrefillArgs {
  int M, N, K;
  int nt;           // tokens per tile (MMA N): 128 or 256
  int ksplit;       // K splits: the CTAs of one cluster (cluster rank = blockIdx.z), 1 = none
  int kt_per;       // stages (BK each) per split
  const float *s;
  const float *s2;
  const int *xexp;  // per activation row: the power of two e[m] applied by the cast
  const float *bs;
  int64_t b_stride, b_off;
  float cap;
  float *y;
  int64_t ldy, y_col0;
  uint32_t *err;
};

using namespace gqt;

// Instruction descriptor: f16 x f16 -> f32, K-major, M=128, N=nt.
__device__ __forceinline__ uint32_t idesc_f16(int nt) {
  return (1u << 4) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(MW >> 4) << 24);
}
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// all threads of every CTA of the cluster (release / acquire at cluster scope)
__device__ __forceinline__ void pf_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// the shared::cluster address of this CTA's shared-memory location p in cluster CTA `rank`
__device__ __forceinline__ uint32_t pf_cluster_addr(const void *p, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(gqd::smem_u32(p)), "r"(rank));
  return ra;
}
// four f32 at a shared::cluster address (16-byte aligned)
__device__ __forceinline__ float4 pf_ld_cluster4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// 32 lanes x 32 bits, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- widening of packed codes to f16 (signed code values, exact) ----------------
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
constexpr uint32_t kMag = 0x64006400u;  // f16 1024 in both halves

// 4-bit: one word = codes 0..7 (nibble j at bits 4j, offset binary, zp 8) ->
// f16 pairs (n0,n4) (n1,n5) (n2,n6) (n3,n7).
__device__ __forceinline__ uint4 widen4(uint32_t w) {
  const uint32_t w8 = w >> 8;
  uint4 r;
  r.x = hsub2((w & 0x000F000Fu) | kMag, 0x64086408u);                // 1024+n - 1032
  r.y = hfma2((w & 0x00F000F0u) | kMag, 0x2C002C00u, 0xD480D480u);   // (1024+16n)/16 - 72
  r.z = hsub2((w8 & 0x000F000Fu) | kMag, 0x64086408u);
  r.w = hfma2((w8 & 0x00F000F0u) | kMag, 0x2C002C00u, 0xD480D480u);
  return r;
}
// 2-bit: one word = codes 0..15 (crumb j at bits 2j, zp 2); the low byte of each
// half gives f16 pairs (c0,c8) (c1,c9) (c2,c10) (c3,c11), the word shifted by 8
// gives (c4,c12) (c5,c13) (c6,c14) (c7,c15).
__device__ __forceinline__ uint4 widen2_half(uint32_t w) {
  uint4 r;
  r.x = hsub2((w & 0x00030003u) | kMag, 0x64026402u);               // 1024+c - 1026
  r.y = hfma2((w & 0x000C000Cu) | kMag, 0x34003400u, 0xDC08DC08u);  // (1024+4c)/4 - 258
  r.z = hfma2((w & 0x00300030u) | kMag, 0x2C002C00u, 0xD420D420u);  // (1024+16c)/16 - 66
  r.w = hfma2((w & 0x00C000C0u) | kMag, 0x24002400u, 0xCC80CC80u);  // (1024+64c)/64 - 18
  return r;
}
// 8-bit: two words = codes 0..7 in natural order. u = byte (U8) or byte ^ 0x80
// (I8) is offset binary with zp 128: 1024 + u - 1152 is the code.
template <bool SIGNED>
__device__ __forceinline__ uint4 widen8(uint32_t w0, uint32_t w1) {
  const uint32_t f = SIGNED ? 0x80808080u : 0u;
  const uint32_t u0 = w0 ^ f, u1 = w1 ^ f;
  uint4 r;
  r.x = hsub2(prmt(u0, 0x64646464u, 0x5140), 0x64806480u);
  r.y = hsub2(prmt(u0, 0x64646464u, 0x7362), 0x64806480u);
  r.z = hsub2(prmt(u1, 0x64646464u, 0x5140), 0x64806480u);
  r.w = hsub2(prmt(u1, 0x64646464u, 0x7362), 0x64806480u);
  return r;
}

// Position p of a K group holds code kperm(p) (the activations follow it).
template <int BITS>
__host__ __device__ constexpr int kperm(int p) {
  return BITS == 4 ? ((p & 8) | ((p & 1) << 2) | ((p >> 1) & 3))  // 0,4,1,5,2,6,3,7 per 8
         : BITS == 2 ? (((p & 1) << 3) | (p >> 1))                // 0,8,1,9,...,7,15
                     : p;
}

// ---- the kernel -----------------------------------------------------------------
template <int BITS, bool SIGNED, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_w2, const PrefillArgs a) {
  using R = Ring<BITS>;
  constexpr int LS = R::LS;
  constexpr int OW = (MODE == 1) ? MW / 2 : MW;  // output columns (weight rows) per tile
  constexpr int PK = BK * BITS / 8;              // packed bytes per weight row per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sX = smem;                 // [LS][NT x BK f16], swizzled (TMA)
  uint8_t *sP = sX + LS * X_STAGE;    // [LS][MW rows x PK packed bytes] (TMA)
  uint64_t *l_full = reinterpret_cast<uint64_t *>(sP + LS * R::PW);
  uint64_t *l_empty = l_full + LS;
  uint64_t *a_full = l_empty + LS;
  uint64_t *a_empty = a_full + AS;
  uint64_t *acc_full = a_empty + AS;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  float *rs_tab = reinterpret_cast<float *>(tmem_slot + 4);  // [2][NT_MAX]: 2^-e of each token row, two factors

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = a.nt;
  const int m0 = blockIdx.x * nt;   // first token of the tile
  const int n0 = blockIdx.y * OW;   // first output column (weight row) of the tile
  // split-K: this CTA (cluster rank blockIdx.z) owns stages kt0 .. kt0 + KT - 1 of the K range
  const int KS = a.ksplit, sidx = KS > 1 ? (int)blockIdx.z : 0;
  const int kt0 = sidx * a.kt_per;
  const int KT = KS > 1 ? min(a.kt_per, a.K / BK - kt0) : a.K / BK;
  const uint32_t x_bytes = (uint32_t)nt * BK * 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < LS; ++i) {
      gqd::mbar_init(&l_full[i], 1);
      gqd::mbar_init(&l_empty[i], 1 + kProdWarps / 2);  // the MMA's commit (x) + the stage's 4 producer warps
    }
    for (int i = 0; i < AS; ++i) {
      gqd::mbar_init(&a_full[i], kProdWarps / 2);
      gqd::mbar_init(&a_empty[i], 1);
    }
    gqd::mbar_init(acc_full, 1);
    *abort_flag = 0;
    gqd::fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(gqd::smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // The packed weights are immutable: the first ring's worth of weight tiles is
  // requested before the dependency wait, so under programmatic dependent launch
  // their HBM latency overlaps the cast kernel; their stages' x tiles follow the
  // wait (x, the f16 workspace, comes from the cast).
  const int pre = min(LS, KT);
  auto load_w = [&](int kt, int s) {
    if (MODE == 1) {  // gate rows then the same up rows
      tma_load_2d(sP + s * R::PW, &tmap_w, (kt0 + kt) * PK, n0, &l_full[s]);
      tma_load_2d(sP + s * R::PW + (MW / 2) * PK, &tmap_w2, (kt0 + kt) * PK, n0, &l_full[s]);
    } else {
      tma_load_2d(sP + s * R::PW, &tmap_w, (kt0 + kt) * PK, n0, &l_full[s]);
    }
  };
  if (warp == 0 && lane == 0)
    for (int kt = 0; kt < pre; ++kt) {
      gqd::mbar_arrive_expect_tx(&l_full[kt], x_bytes + MW * PK);
      load_w(kt, kt);
    }
  gqd::griddep_wait();

  if (warp == 0) {
    // ---- TMA: x tile + packed weight tile per stage ----
    if (lane == 0) {
      int issued = 0;
      for (int kt = 0; kt < KT && !*abort_flag; ++kt) {
        const int s = kt % LS;
        if (kt >= LS && !gqd::mbar_wait_bounded(&l_empty[s], ((kt / LS) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        if (kt >= pre) gqd::mbar_arrive_expect_tx(&l_full[s], x_bytes + MW * PK);
        tma_load_2d(sX + s * X_STAGE, &tmap_x, (kt0 + kt) * BK, m0, &l_full[s]);
        if (kt >= pre) load_w(kt, s);
        issued = kt + 1;
      }
      if (issued < pre) issued = pre;  // weight tiles of stages whose x never came: drained below
      if (*abort_flag) {
        // bounded drain of the loads still in flight before shared memory is released
        for (int kt = issued > LS ? issued - LS : 0; kt < issued; ++kt)
          (void)gqd::mbar_wait_bounded(&l_full[kt % LS], (kt / LS) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue (one thread) ----
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(nt);
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % LS, q = kt % AS;
        if (*abort_flag || !gqd::mbar_wait_bounded(&l_full[s], (kt / LS) & 1) ||
            !gqd::mbar_wait_bounded(&a_full[q], (kt / AS) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint64_t bd = sw128_desc(gqd::smem_u32(sX + s * X_STAGE));
        const uint32_t at = tmem + A_COL0 + (uint32_t)q * A_COLS;
        tc_mma_f16_ts(tmem, at, bd, idesc, kt != 0);
        tc_mma_f16_ts(tmem, at + 8, bd + 2, idesc, 1u);  // 16 f16: 8 TMEM columns, 32 bytes of x
        tc_mma_f16_ts(tmem, at + 16, bd + 4, idesc, 1u);
        tc_mma_f16_ts(tmem, at + 24, bd + 6, idesc, 1u);
        tc_commit(&l_empty[s]);
        tc_commit(&a_empty[q]);
      }
      tc_commit(acc_full);  // fires once every MMA issued above has completed
    }
  } else {
    // ---- producers: widen this lane's weight row into the TMEM A ring ----
    // Warps 2-5 take the even stages, 6-9 the odd ones; warp w writes TMEM lane
    // quarter w % 4, i.e. weight rows 32 * (w % 4) .. + 31.
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    for (int kt = grp; kt < KT; kt += 2) {
      const int s = kt % LS, q = kt % AS;
      bool ok = !*abort_flag && gqd::mbar_wait_bounded(&l_full[s], (kt / LS) & 1);
      ok = ok && (kt < AS || gqd::mbar_wait_bounded(&a_empty[q], ((kt / AS) - 1) & 1));
      if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform: tcgen05.st and the syncs below
        *abort_flag = 1;
        break;
      }
      const uint8_t *src = sP + s * R::PW + row * PK;
      uint32_t r[32];
      if constexpr (BITS == 4) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 in = *reinterpret_cast<const uint4 *>(src + 16 * h);
          const uint32_t w4[4] = {in.x, in.y, in.z, in.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint4 o = widen4(w4[t]);
            r[16 * h + 4 * t] = o.x;
            r[16 * h + 4 * t + 1] = o.y;
            r[16 * h + 4 * t + 2] = o.z;
            r[16 * h + 4 * t + 3] = o.w;
          }
        }
      } else if constexpr (BITS == 2) {
        const uint4 in = *reinterpret_cast<const uint4 *>(src);
        const uint32_t w4[4] = {in.x, in.y, in.z, in.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const uint4 o0 = widen2_half(w4[t]), o1 = widen2_half(w4[t] >> 8);
          r[8 * t] = o0.x;
          r[8 * t + 1] = o0.y;
          r[8 * t + 2] = o0.z;
          r[8 * t + 3] = o0.w;
          r[8 * t + 4] = o1.x;
          r[8 * t + 5] = o1.y;
          r[8 * t + 6] = o1.z;
          r[8 * t + 7] = o1.w;
        }
      } else {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint4 in = *reinterpret_cast<const uint4 *>(src + 16 * h);
          const uint4 o0 = widen8<SIGNED>(in.x, in.y), o1 = widen8<SIGNED>(in.z, in.w);
          r[8 * h] = o0.x;
          r[8 * h + 1] = o0.y;
          r[8 * h + 2] = o0.z;
          r[8 * h + 3] = o0.w;
          r[8 * h + 4] = o1.x;
          r[8 * h + 5] = o1.y;
          r[8 * h + 6] = o1.z;
          r[8 * h + 7] = o1.w;
        }
      }
      tmem_st32(tmem + ((uint32_t)(quarter * 32) << 16) + A_COL0 + (uint32_t)q * A_COLS, r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[q]);
        mbar_arrive(&l_empty[s]);  // the packed codes of this stage are consumed
      }
    }
    // ---- epilogue: warps 2..9 read the accumulator back ----
    // Warp w reads TMEM lane quarter w % 4 (weight rows 32*(w%4) .. +31), warps
    // 2-5 the first half of the tile's tokens and warps 6-9 the second. Lane =
    // weight row, so each store writes 32 consecutive outputs of one token row.
    {
      // the tile's token-row scales 2^-e (two exact factors each), staged once
      {
        const int t = threadIdx.x - 64;  // 0..255
        const int m = m0 + t;
        const int ex = (t < nt && m < a.M) ? a.xexp[m] : 0;
        rs_tab[t] = __int_as_float((127 - ex / 2) << 23);
        rs_tab[NT_MAX + t] = __int_as_float((127 - (ex - ex / 2)) << 23);
      }
      // uniform over the 8 epilogue warps (also publishes rs_tab; MODE 1 pairs
      // them on named barrier 1 below)
      const bool mine = !*abort_flag && gqd::mbar_wait_bounded(acc_full, 0);
      uint32_t all_ok;
      asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, 1, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                   : "=r"(all_ok)
                   : "r"((uint32_t)mine), "r"(kProdWarps * 32)
                   : "memory");
      const bool ok = all_ok != 0;
      if (!ok) *abort_flag = 1;
      tc_fence_after();
      if (KS > 1) {
        // Split-K: this CTA's fp32 partial tile goes to its shared memory as
        // part[token][weight row] (the load ring is idle now); after a cluster
        // barrier CTA sidx finalises output columns [sidx*per, (sidx+1)*per) of the
        // tile for every token, adding the KS partials read over distributed shared
        // memory in cluster-rank order, then applies the epilogue. The final cluster
        // barrier (after the join below) keeps every partial alive until its peers
        // have read it.
        float *part = reinterpret_cast<float *>(sX);
        if (ok) {
          for (int c0 = grp * (nt / 2); c0 < (grp + 1) * (nt / 2); c0 += 32) {
            uint32_t d0[16], d1[16];
            const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
            tmem_ld16_nowait(taddr, d0);
            tmem_ld16_nowait(taddr + 16, d1);
            tmem_wait_ld16(d0);
            tmem_wait_ld16(d1);
#pragma unroll
            for (int j = 0; j < 32; ++j) part[(c0 + j) * MW + row] = __uint_as_float(j < 16 ? d0[j] : d1[j - 16]);
          }
        }
        tc_fence_before();
      } else {
      const int half = grp;
      const int tcount = nt / 2;
      // weight row of this lane -> output column n
      const int n = n0 + (MODE == 1 ? (row & (OW - 1)) : row);
      const bool col_ok = n < a.N;
      const float sn = col_ok ? (MODE == 1 && quarter >= 2 ? a.s2[n] : a.s[n]) : 0.0f;
      // MODE 1: the up rows (quarters 2, 3) hand their values to the gate rows
      float *up = reinterpret_cast<float *>(sX);  // [nt tokens][OW] (the load ring is idle now)
      float *yc = a.y + a.y_col0 + n;
      if (ok) {
        for (int c0 = half * tcount; c0 < (half + 1) * tcount; c0 += 32) {
          uint32_t d0[16], d1[16];
          const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0;
          tmem_ld16_nowait(taddr, d0);
          tmem_ld16_nowait(taddr + 16, d1);
          tmem_wait_ld16(d0);
          tmem_wait_ld16(d1);
          float o[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float v = __uint_as_float(j < 16 ? d0[j] : d1[j - 16]);
            o[j] = __fmul_rn(__fmul_rn(__fmul_rn(v, rs_tab[c0 + j]), rs_tab[NT_MAX + c0 + j]), sn);
          }
          if (MODE == 1) {
            if (quarter >= 2) {
#pragma unroll
              for (int j = 0; j < 32; ++j) up[(c0 + j) * OW + (row & (OW - 1))] = o[j];
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kProdWarps * 32) : "memory");
            if (quarter < 2 && col_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int m = m0 + c0 + j;
                if (m < a.M)
                  yc[(size_t)m * a.ldy] = __fmul_rn(gqd::gelu_tanh(o[j]), up[(c0 + j) * OW + (row & (OW - 1))]);
              }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kProdWarps * 32) : "memory");
          } else if (col_ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = m0 + c0 + j;
              if (m >= a.M) continue;
              float r = o[j];
              if (MODE == 2) {
                r = __fmul_rn(gqd::gelu_tanh(r), a.bs[(size_t)m * a.b_stride + a.b_off + n]);
              } else if (MODE == 3) {
                if (a.cap > 0.0f) r = __fmul_rn(a.cap, tanhf(__fdiv_rn(r, a.cap)));
              }
              yc[(size_t)m * a.ldy] = r;
            }
          }
        }
      }
      tc_fence_before();
      }  // KS == 1
    }
  }

  if (KS > 1) {
    // every CTA of the cluster reaches both barriers (abort or not), so none waits
    // for a peer that left; the second one keeps the partials alive for the readers
    pf_cluster_sync();
    if (!*abort_flag && threadIdx.x >= 64) {
      // groups of four columns: one 16-byte distributed-shared-memory load per peer,
      // all KS loads of a group issued before they are added (in rank order)
      constexpr int kMaxKs = 8;
      const float *part = reinterpret_cast<const float *>(sX);
      const int per = ((OW + KS - 1) / KS + 3) & ~3;
      const int c_lo = sidx * per, c_hi = min(OW, c_lo + per), ng = (c_hi - c_lo) / 4;
      for (int i = threadIdx.x - 64; ng > 0 && i < nt * ng; i += kThreads - 64) {
        const int t = i / ng, col = c_lo + 4 * (i % ng);  // consecutive threads: consecutive column groups
        const int m = m0 + t;
        if (m >= a.M) continue;
        float4 p0[kMaxKs], p1[kMaxKs];
#pragma unroll
        for (int p = 0; p < kMaxKs; ++p)
          if (p < KS) {
            p0[p] = pf_ld_cluster4(pf_cluster_addr(part + t * MW + col, (uint32_t)p));
            if (MODE == 1) p1[p] = pf_ld_cluster4(pf_cluster_addr(part + t * MW + col + MW / 2, (uint32_t)p));
          }
        float4 v0 = p0[0], v1 = MODE == 1 ? p1[0] : v0;
#pragma unroll
        for (int p = 1; p < kMaxKs; ++p)
          if (p < KS) {
            v0.x += p0[p].x; v0.y += p0[p].y; v0.z += p0[p].z; v0.w += p0[p].w;
            if (MODE == 1) { v1.x += p1[p].x; v1.y += p1[p].y; v1.z += p1[p].z; v1.w += p1[p].w; }
          }
        const float a0[4] = {v0.x, v0.y, v0.z, v0.w}, a1[4] = {v1.x, v1.y, v1.z, v1.w};
        const float r0 = rs_tab[t], r1 = rs_tab[NT_MAX + t];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int n = n0 + col + c;
          if (n >= a.N) break;
          float r = __fmul_rn(__fmul_rn(__fmul_rn(a0[c], r0), r1), a.s[n]);
          if (MODE == 1) {
            r = __fmul_rn(gqd::gelu_tanh(r), __fmul_rn(__fmul_rn(__fmul_rn(a1[c], r0), r1), a.s2[n]));
          } else if (MODE == 2) {
            r = __fmul_rn(gqd::gelu_tanh(r), a.bs[(size_t)m * a.b_stride + a.b_off + n]);
          } else if (MODE == 3) {
            if (a.cap > 0.0f) r = __fmul_rn(a.cap, tanhf(__fdiv_rn(r, a.cap)));
          }
          a.y[(size_t)m * a.ldy + a.y_col0 + n] = r;
        }
      }
    }
    pf_cluster_sync();
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) gqd::report(a.err, GQ_DEVERR_WAIT_TIMEOUT);
  if (warp == 1) {
    if (*abort_flag) {
      // Outstanding MMAs (if any) signal acc_full through the final commit.
      (void)gqd::mbar_wait_bounded(acc_full, 0, 100000000ull);
    }
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// f32 -> f16 with a power of two per row: e[m] = 14 - ceil-exponent of max|x[m]|
// (so |x * 2^e| < 2^14), K permuted inside each group of G codes as kperm<BITS>.
// One block per row; the row is read twice (the second time from L1/L2).
template <int BITS>
__global__ void cast_f16_kernel(const float *x, __half *xh, int *xexp, int K) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  constexpr int G = BITS == 2 ? 16 : 8;
  const int m = blockIdx.x;
  const float *xr = x + (size_t)m * K;
  __shared__ float red[32];
  float mx = 0.0f;
  for (int k4 = threadIdx.x; k4 < K / 4; k4 += blockDim.x) {
    const float4 v = reinterpret_cast<const float4 *>(xr)[k4];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) frexpf(mx, &e);  // max|x| < 2^e
  const int s = 14 - e;
  const float f1 = __int_as_float((s / 2 + 127) << 23), f2 = __int_as_float((s - s / 2 + 127) << 23);
  if (threadIdx.x == 0) xexp[m] = s;
  __half *hr = xh + (size_t)m * K;
  for (int gi = threadIdx.x; gi < K / G; gi += blockDim.x) {
    float v[G];
#pragma unroll
    for (int q = 0; q < G / 4; ++q) {
      const float4 t = reinterpret_cast<const float4 *>(xr + gi * G)[q];
      v[4 * q] = t.x;
      v[4 * q + 1] = t.y;
      v[4 * q + 2] = t.z;
      v[4 * q + 3] = t.w;
    }
#pragma unroll
    for (int c = 0; c < G / 8; ++c) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a0 = __fmul_rn(__fmul_rn(v[kperm<BITS>(8 * c + 2 * j)], f1), f2);
        const float a1 = __fmul_rn(__fmul_rn(v[kperm<BITS>(8 * c + 2 * j + 1)], f1), f2);
        const __half2 h = __floats2half2_rn(a0, a1);
        o[j] = *reinterpret_cast<const uint32_t *>(&h);
      }
      reinterpret_cast<uint4 *>(hr + gi * G)[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return gq_encode_fn(); }

template <int BITS, bool SIGNED, int MODE>
int launch_t(gq_ctx *ctx, const CUtensorMap &map, const CUtensorMap &mw, const CUtensorMap &mw2,
             const PrefillArgs &a, dim3 grid) {
  auto kern = prefill_tc_kernel<BITS, SIGNED, MODE>;
  static bool attr_set[64] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Ring<BITS>::kSmem));
    attr_set[dev] = true;
  }
  // the K splits of one output tile form a cluster along z
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Ring<BITS>::kSmem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ctx->pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (a.ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = (unsigned)a.ksplit;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  GQ_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kern, map, mw, mw2, a));
  return GQ_OK;
}

template <int BITS, bool SIGNED>
int launch_mode(gq_ctx *ctx, int mode, const CUtensorMap &map, const CUtensorMap &mw, const CUtensorMap &mw2,
                const PrefillArgs &a, dim3 grid) {
  switch (mode) {
    case 0: return launch_t<BITS, SIGNED, 0>(ctx, map, mw, mw2, a, grid);
    case 1: return launch_t<BITS, SIGNED, 1>(ctx, map, mw, mw2, a, grid);
    case 2: return launch_t<BITS, SIGNED, 2>(ctx, map, mw, mw2, a, grid);
    default: return launch_t<BITS, SIGNED, 3>(ctx, map, mw, mw2, a, grid);
  }
}

// Tensor map over a packed weight [n rows, row_bytes] (uint8), box = one stage:
// the packed bytes of BK codes for `rows` rows.
CUresult encode_weight_map(CUtensorMap *map, const uint8_t *w, int64_t n, int64_t row_bytes, int bits, int rows) {
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)n};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(BK * bits / 8), (cuuint32_t)rows};
  cuuint32_t estr[2] = {1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(w), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Tensor map over the f16 activations [m, k], box nt rows x 64 halves, 128-byte swizzle.
// Tokens per tile (the MMA N, a multiple of 64: the epilogue drains 32 columns
// per half). 128 for short prefills. For longer ones a tile's time is mostly
// fixed cost, so fewer idle SMs win: where 256-token tiles fill less than half
// the SMs (the K-split regime), a smaller tile that fills half to all of them in
// one wave without a split, else 256 with K split over clusters; otherwise the
// smallest of 128 / 192 / 256 that needs no more waves than 256. Measured on B200
// (µs per call incl. the cast): 4-bit gate [6144, 1536] at M = 512 21.2 -> 20.1
// (192), fused gate+up 51.9 -> 46.2 (192), M = 1024 40.0 -> 37.7 (192), M = 256
// 19.6 (256, K in 2) -> 17.2 (128); the 2-bit down [1536, 6144] at M = 512 stays at
// 256 with K in 4 (24.6; 33.9 at 128, 38.4 at 192), as does M = 2048 (three waves).
// GQ_PREFILL_NT (64, 128, 192 or 256) overrides the choice for tuning and tests.
int token_tile(int64_t m, int64_t wtiles, int kt_all, int num_sms) {
  if (const char *e = getenv("GQ_PREFILL_NT")) {
    const int v = atoi(e);
    if (v == 64 || v == 128 || v == 192 || v == 256) return v;
  }
  if (m <= 128) return 128;
  auto tiles = [&](int nt) { return ((m + nt - 1) / nt) * wtiles; };
  if (tiles(NT_MAX) * 2 <= num_sms && kt_all / 2 >= 3) {
    for (int nt : {128, 192})
      if (tiles(nt) * 2 >= num_sms && tiles(nt) <= num_sms) return nt;
    return NT_MAX;  // K split over clusters
  }
  auto waves = [&](int nt) { return (tiles(nt) + num_sms - 1) / num_sms; };
  for (int nt : {128, 192})
    if (waves(nt) <= waves(NT_MAX)) return nt;
  return NT_MAX;
}

CUresult encode_x_map(CUtensorMap *map, const __half *xh, int64_t m, int64_t k, int nt) {
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  cuuint32_t box[2] = {BK, (cuuint32_t)nt};
  cuuint32_t estr[2] = {1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(xh), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int BITS>
cudaError_t launch_cast(cudaStream_t stream, bool pdl, const float *x, __half *xh, int *xexp, int64_t m, int64_t k) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((unsigned)m);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, cast_f16_kernel<BITS>, x, xh, xexp, (int)k);
}

cudaError_t cast_any(int bits, cudaStream_t stream, bool pdl, const float *x, __half *xh, int *xexp, int64_t m,
                     int64_t k) {
  if (bits == 4) return launch_cast<4>(stream, pdl, x, xh, xexp, m, k);
  if (bits == 2) return launch_cast<2>(stream, pdl, x, xh, xexp, m, k);
  return launch_cast<8>(stream, pdl, x, xh, xexp, m, k);
}

size_t smem_for(int bits) {
  return bits == 4 ? Ring<4>::kSmem : (bits == 2 ? Ring<2>::kSmem : Ring<8>::kSmem);
}

}  // namespace

// The tensor-core path applies to M >= 16 rows with K a multiple of 64 (so every
// packed row is a whole number of 16-byte TMA units), one scale per row and a
// 16-byte aligned packed weight.
bool gq_prefill_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m) {
  if (m < 16 || w->group_size != w->k || w->k % BK != 0 || w->k <= 0 || w->n <= 0) return false;
  if (m > (1ll << 30) || w->n > (1ll << 30) || w->k > (1 << 24)) return false;
  if ((w->n + MW / 2 - 1) / (MW / 2) > 65535) return false;  // grid.y = weight tiles (GeGLU: MW/2 rows)
  if ((uintptr_t)w->bytes % 16 != 0) return false;  // the packed tiles come in by TMA
  return smem_for(w->bits) <= ctx->smem_optin && encode_fn() != nullptr;
}


int gq_prefill_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                      const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                      int64_t y_col0) {
  const int64_t K = w->k;
  const size_t xh_bytes = ((size_t)(m * K) * 2 + 255) & ~size_t(255);
  void *wsp = nullptr;
  int rc = gq_workspace(ctx, xh_bytes + (size_t)m * sizeof(int), &wsp);
  if (rc != GQ_OK) return rc;
  __half *xh = static_cast<__half *>(wsp);
  int *xexp = reinterpret_cast<int *>(static_cast<uint8_t *>(wsp) + xh_bytes);
  GQ_CUDA_TRY(ctx, cast_any(w->bits, ctx->stream, ctx->pdl, x, xh, xexp, m, K));
  const int ow_sel = (mode == 1) ? MW / 2 : MW;
  const int nt = token_tile(m, (w->n + ow_sel - 1) / ow_sel, (int)(K / BK), ctx->num_sms);
  CUtensorMap map;
  if (encode_x_map(&map, xh, m, K, nt) != CUDA_SUCCESS)
    return gq_fail(ctx, GQ_ERR_CUDA, "prefill: activation tensor map");
  PrefillArgs a = {};
  a.nt = nt;
  a.M = (int)m;
  a.N = (int)w->n;
  a.K = (int)K;
  a.s = w->scales;
  a.s2 = w2 ? w2->scales : nullptr;
  a.xexp = xexp;
  a.bs = bs;
  a.b_stride = b_stride;
  a.b_off = b_off;
  a.cap = cap;
  a.y = y;
  a.ldy = ldy;
  a.y_col0 = y_col0;
  a.err = ctx->dev_err;
  const int ow = (mode == 1) ? MW / 2 : MW;
  CUtensorMap mw, mw2;
  if (encode_weight_map(&mw, w->bytes, w->n, w->row_bytes, w->bits, ow) != CUDA_SUCCESS ||
      encode_weight_map(&mw2, w2 ? w2->bytes : w->bytes, w->n, w->row_bytes, w->bits, ow) != CUDA_SUCCESS)
    return gq_fail(ctx, GQ_ERR_CUDA, "prefill: weight tensor map");
  dim3 grid((unsigned)((m + nt - 1) / nt), (unsigned)((w->n + ow - 1) / ow));
  // Split K over a cluster of 2, 4 or 8 CTAs when the output tiles leave SMs idle
  // (the 2-bit down projection of config 3 has 24 tiles on 148 SMs): the largest
  // power of two that keeps the grid within one wave and >= 3 stages per split.
  // Measured on B200 at the E2B shapes (M = 128..512): one wave beats two, and
  // clusters of 3, 5 or 6 CTAs run slower than the power of two below them. The
  // splits' fp32 partials are added over distributed shared memory in a fixed
  // order (deterministic).
  const int kt_all = (int)(K / BK);
  const int tiles = (int)(grid.x * grid.y);
  int ks = 1;
  while (ks < 8 && (int64_t)tiles * ks * 2 <= ctx->num_sms && kt_all / (ks * 2) >= 3) ks *= 2;
  if (const char *e = getenv("GQ_PREFILL_KSPLIT")) {  // explicit split (tuning and tests): 1..8
    const int v = atoi(e);
    if (v >= 1 && v <= 8) ks = std::min(v, kt_all);
  }
  a.kt_per = (kt_all + ks - 1) / ks;
  a.ksplit = (kt_all + a.kt_per - 1) / a.kt_per;  // no empty split
  grid.z = (unsigned)a.ksplit;
  if (w->bits == 4) return launch_mode<4, false>(ctx, mode, map, mw, mw2, a, grid);
  if (w->bits == 2) return launch_mode<2, false>(ctx, mode, map, mw, mw2, a, grid);
  if (w->signed_i8) return launch_mode<8, true>(ctx, mode, map, mw, mw2, a, grid);
  return launch_mode<8, false>(ctx, mode, map, mw, mw2, a, grid);
}

// ---- allocation-free variant ---------------------------------------------------
// For callers that cannot allocate device memory at call time: a serving process
// that reserves its whole HBM budget at start-up and treats any later cudaMalloc
// as an error, or an embedder whose buffers all come from its own arena. The
// scratch this path needs (the f16 copy of the activations and one exponent per
// row) lives in these file-scope arrays instead of a context workspace; every
// GPU that loads the library holds them until the process exits.
namespace {
constexpr int64_t kStaticScratchElems = int64_t(4) << 20;  // 4 Mi f16 (8 MiB): M*K <= 4,194,304
constexpr int64_t kStaticRows = kStaticScratchElems / BK;   // K >= 64, so M <= 65,536
constexpr int64_t kStaticMaxN = int64_t(65535) * MW;        // grid.y = N / 128 weight tiles
static __device__ __align__(256) __half g_prefill_scratch[kStaticScratchElems];
static __device__ __align__(256) int g_prefill_xexp[kStaticRows];
// GQ_DEVERR_* bits of the calls on this device (a bounded wait that gave up),
// read and cleared by gq_linear_prefill_static_status.
static __device__ __align__(16) uint32_t g_prefill_status;

// Host-side device addresses of the arrays, one per device. Host code must not
// pass the symbols themselves to a kernel: in host code they name host-side
// stand-ins, not device memory. The look-up runs once per device under a lock
// (two host threads making their first call on one device do not race on it);
// `ready` is published with release order and read with acquire order.
struct StaticSetup {
  void *scratch = nullptr;
  void *xexp = nullptr;
  uint32_t *status = nullptr;
  int smem_optin = 0;
  std::atomic<bool> ready{false};
};
StaticSetup g_static_setup[64];
std::mutex g_static_mu;

cudaError_t static_setup(int dev, StaticSetup **out) {
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  StaticSetup &st = g_static_setup[dev];
  if (!st.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!st.ready.load(std::memory_order_relaxed)) {
      void *scratch = nullptr, *xexp = nullptr, *status = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&scratch, g_prefill_scratch);
      if (e != cudaSuccess) return e;
      e = cudaGetSymbolAddress(&xexp, g_prefill_xexp);
      if (e != cudaSuccess) return e;
      e = cudaGetSymbolAddress(&status, g_prefill_status);
      if (e != cudaSuccess) return e;
      if (scratch == nullptr || xexp == nullptr || status == nullptr) return cudaErrorInvalidSymbol;
      int optin = 0;
      e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
      if (e != cudaSuccess) return e;
      st.scratch = scratch;
      st.xexp = xexp;
      st.status = static_cast<uint32_t *>(status);
      st.smem_optin = optin;
      st.ready.store(true, std::memory_order_release);
    }
  }
  *out = &st;
  return cudaSuccess;
}

template <int BITS, bool SIGNED>
cudaError_t static_launch(cudaStream_t stream, const CUtensorMap &map, const CUtensorMap &mw, const PrefillArgs &a,
                          dim3 grid) {
  auto kern = prefill_tc_kernel<BITS, SIGNED, 0>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Ring<BITS>::kSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Ring<BITS>::kSmem;
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, kern, map, mw, mw, a);
}
}  // namespace

extern "C" int gq_linear_prefill_static(void *cuda_stream, const float *x, int64_t m, int64_t k,
                                        const uint8_t *qbytes, const float *scales, int64_t n, int32_t bits,
                                        int32_t signed_i8, float *y) {
  if (m < 0 || n < 0 || k <= 0) return GQ_ERR_INVALID_ARGUMENT;
  if (m == 0 || n == 0) return GQ_OK;
  if (!x || !qbytes || !scales || !y) return GQ_ERR_INVALID_ARGUMENT;
  if (signed_i8 ? bits != 8 : (bits != 2 && bits != 4 && bits != 8)) return GQ_ERR_UNSUPPORTED;
  if (k % BK != 0) return GQ_ERR_UNSUPPORTED;
  if (m > kStaticScratchElems / k) return GQ_ERR_INVALID_ARGUMENT;  // M*K beyond the static scratch
  if (n > kStaticMaxN) return GQ_ERR_UNSUPPORTED;  // more weight tiles than a grid dimension holds
  if ((uintptr_t)x % 16 != 0 || (uintptr_t)qbytes % 16 != 0 || (uintptr_t)scales % 4 != 0)
    return GQ_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQ_ERR_CUDA;
  StaticSetup *st = nullptr;
  if (static_setup(dev, &st) != cudaSuccess) return GQ_ERR_CUDA;
  if ((size_t)st->smem_optin < smem_for(bits) || encode_fn() == nullptr) return GQ_ERR_UNSUPPORTED;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  __half *xh = static_cast<__half *>(st->scratch);
  int *xexp = static_cast<int *>(st->xexp);
  if (cast_any(bits, stream, false, x, xh, xexp, m, k) != cudaSuccess) return GQ_ERR_CUDA;
  // no SM count here and no K split: 256 (128 for short prefills) unless overridden
  const int nt = token_tile(m, int64_t(1) << 30, (int)(k / BK), 1);
  CUtensorMap map;
  if (encode_x_map(&map, xh, m, k, nt) != CUDA_SUCCESS) return GQ_ERR_CUDA;
  PrefillArgs a = {};
  a.nt = nt;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.s = scales;
  a.xexp = xexp;
  a.y = y;
  a.ldy = n;
  a.y_col0 = 0;
  a.err = st->status;  // a timed-out wait: gq_linear_prefill_static_status reports it
  const dim3 grid((unsigned)((m + nt - 1) / nt), (unsigned)((n + MW - 1) / MW));
  CUtensorMap mw;
  if (encode_weight_map(&mw, qbytes, n, signed_i8 ? k : k * bits / 8, bits, MW) != CUDA_SUCCESS) return GQ_ERR_CUDA;
  cudaError_t e;
  if (bits == 4) e = static_launch<4, false>(stream, map, mw, a, grid);
  else if (bits == 2) e = static_launch<2, false>(stream, map, mw, a, grid);
  else if (signed_i8) e = static_launch<8, true>(stream, map, mw, a, grid);
  else e = static_launch<8, false>(stream, map, mw, a, grid);
  return e == cudaSuccess ? GQ_OK : GQ_ERR_CUDA;
}

extern "C" int gq_linear_prefill_static_status(void *cuda_stream, uint32_t *status_bits) {
  if (!status_bits) return GQ_ERR_INVALID_ARGUMENT;
  *status_bits = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQ_ERR_CUDA;
  StaticSetup *st = nullptr;
  if (static_setup(dev, &st) != cudaSuccess) return GQ_ERR_CUDA;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  if (cudaStreamSynchronize(stream) != cudaSuccess) return GQ_ERR_CUDA;
  uint32_t bits = 0;
  if (cudaMemcpy(&bits, st->status, sizeof(bits), cudaMemcpyDeviceToHost) != cudaSuccess) return GQ_ERR_CUDA;
  if (bits != 0 && cudaMemset(st->status, 0, sizeof(uint32_t)) != cudaSuccess) return GQ_ERR_CUDA;
  *status_bits = bits;
  return bits ? GQ_ERR_DEVICE : GQ_OK;
}
