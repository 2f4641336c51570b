// prefill_tc.cu — prefill dequantizing GEMM on the 5th-generation tensor cores.
//
// Replaces the reference's MATMUL_Q_TILED shader (rust/src/kernels/matmul_q_tiled.wgsl:
// 39-126, chosen for M >= 16 at rust/src/backend_wgpu.rs:663-673), whose W tile is
// dequantized to f32 in workgroup memory and multiplied with f32 FMAs. Here:
//   C[m, n] = epilogue( s[n] * sum_k bf16(x[m, k]) * q[n, k] )
// with bf16 operands and fp32 accumulation in tensor memory (TMEM):
//  * x is cast to bf16 once per call (a [M, K] workspace) and loaded tile by tile
//    with TMA (cp.async.bulk.tensor, 128-byte swizzle);
//  * 8 producer warps dequantize the packed weight rows straight into shared
//    memory in the K-major 128-byte-swizzled layout tcgen05.mma reads (codes are
//    exact in bf16; the per-row scale is applied in the epilogue);
//  * one elected thread issues tcgen05.mma (M=128 tokens, N=256 weight rows,
//    K=16) into a 128x256 fp32 accumulator in TMEM; tcgen05.commit releases
//    each shared-memory stage and finally signals the epilogue;
//  * the 8 producer warps then read the accumulator back with tcgen05.ld, apply
//    the scale and the MODE epilogue (0 plain, 1 GeGLU, 2 gelu * column slice,
//    3 soft-cap) and store f32 rows through a shared-memory transpose.
// For MODE 1 the 256 MMA columns hold 128 gate rows followed by the same 128 up
// rows, so one MMA computes both projections of a 128-wide output tile.
//
// Every wait is bounded (2 s); a timeout sets GQ_DEVERR_WAIT_TIMEOUT, drains,
// frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>

#include "tc_common.cuh"

namespace {

constexpr int BM = 128;        // tokens per tile (MMA M)
constexpr int BN = 256;        // MMA N (weight rows, or gate+up halves)
constexpr int BK = 64;         // K per stage: one 128-byte swizzle row of bf16
constexpr int STAGES = 3;
constexpr int kThreads = 320;  // warp 0: TMA(A), warp 1: MMA + TMEM, warps 2-9: B producers
constexpr int kProducers = 256;
constexpr uint32_t A_STAGE = BM * BK * 2;  // 16 KB
constexpr uint32_t B_STAGE = BN * BK * 2;  // 32 KB
constexpr uint32_t P_STAGE = BN * BK;      // packed weight tile, <= 16 KB (8-bit)
constexpr uint32_t TMEM_COLS = 256;

struct PrefillArgs {
  int M, N, K;
  const uint8_t *w;
  const float *s;
  const uint8_t *w2;
  const float *s2;
  int row_bytes;
  const float *bs;
  int64_t b_stride, b_off;
  float cap;
  float *y;
  int64_t ldy, y_col0;
  uint32_t *err;
};

using namespace gqt;

// Instruction descriptor: bf16 x bf16 -> f32, both K-major, M=128, N=256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

// ---- dequantization of 8 consecutive codes to 8 bf16 (natural K order) -------
// Sub-byte codes use the bf16 pattern 0x4300|n (= 128 + n, exact), then subtract
// 128 + zero point. Two codes at bit offsets a (low half) and a+16 (high half)
// come out of one masked word; PRMT then pairs neighbours into natural order.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ uint32_t bsub(uint32_t v, uint32_t c2) {  // bf16x2 v - c2 (exact here)
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&v);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&c2);
  __nv_bfloat162 r = __hsub2(a, b);
  return *reinterpret_cast<uint32_t *>(&r);
}

// 4-bit: one 32-bit word = codes 0..7 (nibble j at bits 4j, offset binary).
__device__ __forceinline__ uint4 deq8_b4(uint32_t w) {
  const uint32_t A = (w & 0x000F000Fu) | 0x43004300u;          // (c0, c4)
  const uint32_t B = ((w >> 4) & 0x000F000Fu) | 0x43004300u;   // (c1, c5)
  const uint32_t C = ((w >> 8) & 0x000F000Fu) | 0x43004300u;   // (c2, c6)
  const uint32_t D = ((w >> 12) & 0x000F000Fu) | 0x43004300u;  // (c3, c7)
  const uint32_t zp = 0x43084308u;                              // 136 = 128 + 8
  uint4 r;
  r.x = bsub(prmt(A, B, 0x5410), zp);  // (c0, c1)
  r.y = bsub(prmt(C, D, 0x5410), zp);  // (c2, c3)
  r.z = bsub(prmt(A, B, 0x7632), zp);  // (c4, c5)
  r.w = bsub(prmt(C, D, 0x7632), zp);  // (c6, c7)
  return r;
}
// 2-bit: 16 bits = codes 0..7 (crumb j at bits 2j).
__device__ __forceinline__ uint4 deq8_b2(uint32_t h) {
  // E_j holds code j (low half) and code j+4 (high half)
  const uint32_t v = (h & 0xFFu) | ((h & 0xFF00u) << 8);  // codes 0-3 at bits 0-7, codes 4-7 at bits 16-23
  const uint32_t E0 = (v & 0x00030003u) | 0x43004300u;
  const uint32_t E1 = ((v >> 2) & 0x00030003u) | 0x43004300u;
  const uint32_t E2 = ((v >> 4) & 0x00030003u) | 0x43004300u;
  const uint32_t E3 = ((v >> 6) & 0x00030003u) | 0x43004300u;
  const uint32_t zp = 0x43024302u;  // 130 = 128 + 2
  uint4 r;
  r.x = bsub(prmt(E0, E1, 0x5410), zp);  // (c0, c1)
  r.y = bsub(prmt(E2, E3, 0x5410), zp);  // (c2, c3)
  r.z = bsub(prmt(E0, E1, 0x7632), zp);  // (c4, c5)
  r.w = bsub(prmt(E2, E3, 0x7632), zp);  // (c6, c7)
  return r;
}
// 8-bit: two words = codes 0..7. u = byte ^ XOR is offset binary (zp 128); the f32
// 2^23 + u minus 2^23 + 128 is the exact code, and its upper half is its bf16.
template <bool SIGNED>
__device__ __forceinline__ uint32_t deq2_b8(uint32_t u, int j0) {
  const uint32_t magic = 0x4B000000u;
  const float f0 = __uint_as_float(prmt(u, magic, 0x7440u + j0)) - 8388736.0f;
  const float f1 = __uint_as_float(prmt(u, magic, 0x7440u + j0 + 1)) - 8388736.0f;
  return prmt(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
}
template <bool SIGNED>
__device__ __forceinline__ uint4 deq8_b8(uint2 q) {
  const uint32_t x = SIGNED ? 0x80808080u : 0u;
  const uint32_t u0 = q.x ^ x, u1 = q.y ^ x;
  uint4 r;
  r.x = deq2_b8<SIGNED>(u0, 0);
  r.y = deq2_b8<SIGNED>(u0, 2);
  r.z = deq2_b8<SIGNED>(u1, 0);
  r.w = deq2_b8<SIGNED>(u1, 2);
  return r;
}

// Packed bytes of 8 consecutive codes.
template <int BITS>
struct Pack8 {
  using T = typename std::conditional<BITS == 8, uint2, typename std::conditional<BITS == 4, uint32_t, uint16_t>::type>::type;
};

template <int BITS, bool SIGNED>
__device__ __forceinline__ uint4 deq8(typename Pack8<BITS>::T p) {
  if constexpr (BITS == 4) return deq8_b4(p);
  else if constexpr (BITS == 2) return deq8_b2(p);
  else return deq8_b8<SIGNED>(p);
}

template <int BITS>
__device__ __forceinline__ typename Pack8<BITS>::T load8(const uint8_t *row, int k) {
  using T = typename Pack8<BITS>::T;
  return *reinterpret_cast<const T *>(row + (size_t)k * BITS / 8);
}

// ---- the kernel -----------------------------------------------------------------
template <int BITS, bool SIGNED, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_w2, const PrefillArgs a) {
  using P8 = typename Pack8<BITS>::T;
  constexpr int OW = (MODE == 1) ? BN / 2 : BN;  // output columns per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = smem;                                       // [STAGES][BM x BK bf16], swizzled
  uint8_t *sB = smem + STAGES * A_STAGE;                    // [STAGES][BN x BK bf16], swizzled
  uint8_t *sP = sB + STAGES * B_STAGE;                      // [STAGES][BN rows x BK codes packed]
  uint64_t *full_a = reinterpret_cast<uint64_t *>(sP + STAGES * P_STAGE);
  uint64_t *full_b = full_a + STAGES;
  uint64_t *empty = full_b + STAGES;
  uint64_t *acc_full = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int n0 = blockIdx.y * OW;
  const int KT = a.K / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      gqd::mbar_init(&full_a[i], 1);
      gqd::mbar_init(&full_b[i], kProducers);
      gqd::mbar_init(&empty[i], 1);
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

  gqd::griddep_wait();  // x (the bf16 workspace) comes from the preceding cast kernel

  if (warp == 0) {
    // ---- A: TMA loads of the bf16 activation tile ----
    if (lane == 0) {
      int issued = 0;
      for (int kt = 0; kt < KT && !*abort_flag; ++kt) {
        const int s = kt % STAGES;
        if (kt >= STAGES && !gqd::mbar_wait_bounded(&empty[s], ((kt / STAGES) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        constexpr uint32_t pk = BK * BITS / 8;  // packed bytes of one row per stage
        gqd::mbar_arrive_expect_tx(&full_a[s], A_STAGE + BN * pk);
        tma_load_2d(sA + s * A_STAGE, &tmap_a, kt * BK, m0, &full_a[s]);
        if (MODE == 1) {  // gate rows then the same up rows
          tma_load_2d(sP + s * P_STAGE, &tmap_w, kt * (int)pk, n0, &full_a[s]);
          tma_load_2d(sP + s * P_STAGE + (BN / 2) * pk, &tmap_w2, kt * (int)pk, n0, &full_a[s]);
        } else {
          tma_load_2d(sP + s * P_STAGE, &tmap_w, kt * (int)pk, n0, &full_a[s]);
        }
        issued = kt + 1;
      }
      if (*abort_flag) {
        // bounded drain of the loads still in flight before shared memory is released
        for (int kt = issued > STAGES ? issued - STAGES : 0; kt < issued; ++kt)
          (void)gqd::mbar_wait_bounded(&full_a[kt % STAGES], (kt / STAGES) & 1, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue (one thread) ----
    if (lane == 0) {
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (*abort_flag || !gqd::mbar_wait_bounded(&full_a[s], ph) || !gqd::mbar_wait_bounded(&full_b[s], ph)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(gqd::smem_u32(sA + s * A_STAGE));
        const uint64_t bd = sw128_desc(gqd::smem_u32(sB + s * B_STAGE));
#pragma unroll
        for (int j = 0; j < BK / 16; ++j)  // 16 bf16 = 32 bytes per MMA along K
          tc_mma_f16(tmem, ad + (uint64_t)(2 * j), bd + (uint64_t)(2 * j), kIdesc, (kt | j) != 0);
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);  // fires once every MMA issued above has completed
    }
  } else {
    // ---- B: dequantize the TMA-staged packed rows into the swizzled K-major tile ----
    const int pt = threadIdx.x - 64;  // 0..255
    constexpr int pk = BK * BITS / 8;  // packed bytes per row per stage
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES && (*abort_flag || !gqd::mbar_wait_bounded(&empty[s], ((kt / STAGES) - 1) & 1))) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag || !gqd::mbar_wait_bounded(&full_a[s], (kt / STAGES) & 1)) {
        *abort_flag = 1;
        break;
      }
      uint8_t *dst = sB + s * B_STAGE;
      const uint8_t *src = sP + s * P_STAGE;
#pragma unroll
      for (int it = 0; it < (BN * 8) / kProducers; ++it) {
        const int item = pt + it * kProducers;
        const int r = item >> 3;  // tile row 0..255 (rows past N arrive zero-filled; discarded later)
        const int c = item & 7;   // 16-byte chunk (8 codes) within the 128-byte row
        const uint4 v = deq8<BITS, SIGNED>(*reinterpret_cast<const P8 *>(src + r * pk + c * (8 * BITS / 8)));
        *reinterpret_cast<uint4 *>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async();  // make the generic-proxy stores visible to the tensor core
      mbar_arrive(&full_b[s]);
    }
    // ---- epilogue: warps 2..9 read the accumulator back ----
    // Warp w may only touch TMEM lanes 32*(w%4)..+31 (its row quarter); warps
    // 2-5 take the first half of the output columns and warps 6-9 the second.
    // Each 32x32 block goes through a padded shared-memory tile so that the
    // global stores are whole 128-byte row segments, not one row per lane.
    {
      const int q = warp & 3;
      const int half = (warp - 2) >> 2;
      constexpr int HALF_W = OW / 2;  // 128 (MODE 0/2/3) or 64 (MODE 1)
      const bool ok = gqd::mbar_wait_bounded(acc_full, 0);
      if (!ok) *abort_flag = 1;
      tc_fence_after();
      if (ok) {
        // every MMA has completed, so the pipeline buffers are free for staging
        float *stg = reinterpret_cast<float *>(sB) + (warp - 2) * (32 * 33);
        const int row0 = m0 + q * 32;
        for (int c0 = half * HALF_W; c0 < (half + 1) * HALF_W; c0 += 32) {
          float v[32], u[32];
          const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + c0;
          tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
          tmem_ld16(taddr + 16, *reinterpret_cast<float(*)[16]>(v + 16));
          if (MODE == 1) {
            tmem_ld16(taddr + BN / 2, *reinterpret_cast<float(*)[16]>(u));
            tmem_ld16(taddr + BN / 2 + 16, *reinterpret_cast<float(*)[16]>(u + 16));
          }
          // lane = row: scale and the row-independent part of the MODE epilogue
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = min(n0 + c0 + j, a.N - 1);  // columns past N are computed, never stored
            float o = __fmul_rn(v[j], a.s[n]);
            if (MODE == 1) {
              o = __fmul_rn(gqd::gelu_tanh(o), __fmul_rn(u[j], a.s2[n]));
            } else if (MODE == 2) {
              o = gqd::gelu_tanh(o);
            } else if (MODE == 3) {
              if (a.cap > 0.0f) o = __fmul_rn(a.cap, tanhf(__fdiv_rn(o, a.cap)));
            }
            stg[lane * 33 + j] = o;
          }
          __syncwarp();
          // lane = column: one 128-byte row segment per store instruction
          const int n = n0 + c0 + lane;
          if (n < a.N) {
            for (int r = 0; r < 32; ++r) {
              const int m = row0 + r;
              if (m >= a.M) break;
              float o = stg[r * 33 + lane];
              if (MODE == 2) o = __fmul_rn(o, a.bs[(size_t)m * a.b_stride + a.b_off + n]);
              a.y[(size_t)m * a.ldy + a.y_col0 + n] = o;
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
    }
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

// f32 -> bf16 (round to nearest even), [M, K] row-major, K % 4 == 0.
__global__ void cast_bf16_kernel(const float *x, __nv_bfloat16 *xb, int64_t n4) {
  gqd::griddep_wait();
  gqd::griddep_launch_dependents();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4 *>(x)[i];
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t *>(&lo);
    o.y = *reinterpret_cast<uint32_t *>(&hi);
    reinterpret_cast<uint2 *>(xb)[i] = o;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return gq_encode_fn(); }

template <int BITS, bool SIGNED, int MODE>
int launch_t(gq_ctx *ctx, const CUtensorMap &map, const CUtensorMap &mw, const CUtensorMap &mw2,
             const PrefillArgs &a, dim3 grid, size_t smem) {
  auto kern = prefill_tc_kernel<BITS, SIGNED, MODE>;
  static bool attr_set[64] = {};
  const int dev = ctx->device & 63;
  if (!attr_set[dev]) {
    GQ_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set[dev] = true;
  }
  GQ_CUDA_TRY(ctx, gq_launch(ctx, kern, grid, dim3(kThreads), smem, map, mw, mw2, a));
  return GQ_OK;
}

template <int BITS, bool SIGNED>
int launch_mode(gq_ctx *ctx, int mode, const CUtensorMap &map, const CUtensorMap &mw, const CUtensorMap &mw2,
                const PrefillArgs &a, dim3 grid, size_t smem) {
  switch (mode) {
    case 0: return launch_t<BITS, SIGNED, 0>(ctx, map, mw, mw2, a, grid, smem);
    case 1: return launch_t<BITS, SIGNED, 1>(ctx, map, mw, mw2, a, grid, smem);
    case 2: return launch_t<BITS, SIGNED, 2>(ctx, map, mw, mw2, a, grid, smem);
    default: return launch_t<BITS, SIGNED, 3>(ctx, map, mw, mw2, a, grid, smem);
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

constexpr size_t kSmemBytes = 1024 + STAGES * (A_STAGE + B_STAGE + P_STAGE) + (3 * STAGES + 1) * 8 + 16;

}  // namespace

// The tensor-core path applies to M >= 16 rows with K a multiple of 64 (so every
// packed row is a whole number of 16-byte TMA units), one scale per row and a
// 16-byte aligned packed weight.
bool gq_prefill_supported(gq_ctx *ctx, const gq_qweight *w, int64_t m) {
  if (m < 16 || w->group_size != w->k || w->k % BK != 0 || w->k <= 0 || w->n <= 0) return false;
  if (m > (1ll << 30) || w->n > (1ll << 30) || w->k > (1 << 24)) return false;
  if ((uintptr_t)w->bytes % 16 != 0) return false;  // the packed tiles come in by TMA
  return kSmemBytes <= ctx->smem_optin && encode_fn() != nullptr;
}

// Workspace for the bf16 copy of x (grown on demand, stream-ordered).
static int ws_get(gq_ctx *ctx, size_t bytes, void **out) {
  if (ctx->ws_cap < bytes) {
    if (ctx->ws) cudaFreeAsync(ctx->ws, ctx->stream);
    ctx->ws = nullptr;
    ctx->ws_cap = 0;
    GQ_CUDA_TRY(ctx, cudaMallocAsync(&ctx->ws, bytes, ctx->stream));
    ctx->ws_cap = bytes;
  }
  *out = ctx->ws;
  return GQ_OK;
}

int gq_prefill_launch(gq_ctx *ctx, int mode, const float *x, int64_t m, const gq_qweight *w, const gq_qweight *w2,
                      const float *bs, int64_t b_stride, int64_t b_off, float cap, float *y, int64_t ldy,
                      int64_t y_col0) {
  const int64_t K = w->k;
  void *wsp = nullptr;
  int rc = ws_get(ctx, (size_t)(m * K) * 2, &wsp);
  if (rc != GQ_OK) return rc;
  __nv_bfloat16 *xb = static_cast<__nv_bfloat16 *>(wsp);
  {
    const int64_t n4 = m * K / 4;
    int64_t g = (n4 + 255) / 256;
    if (g > (int64_t)ctx->num_sms * 8) g = (int64_t)ctx->num_sms * 8;
    GQ_CUDA_TRY(ctx, gq_launch(ctx, cast_bf16_kernel, dim3((unsigned)g), dim3(256), 0, x, xb, n4));
  }
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)m};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {BK, BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult cr = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xb, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return gq_fail(ctx, GQ_ERR_CUDA, "prefill: cuTensorMapEncodeTiled failed");
  PrefillArgs a = {};
  a.M = (int)m;
  a.N = (int)w->n;
  a.K = (int)K;
  a.w = w->bytes;
  a.s = w->scales;
  if (w2) {
    a.w2 = w2->bytes;
    a.s2 = w2->scales;
  }
  a.row_bytes = (int)w->row_bytes;
  a.bs = bs;
  a.b_stride = b_stride;
  a.b_off = b_off;
  a.cap = cap;
  a.y = y;
  a.ldy = ldy;
  a.y_col0 = y_col0;
  a.err = ctx->dev_err;
  const int ow = (mode == 1) ? BN / 2 : BN;
  CUtensorMap mw, mw2;
  if (encode_weight_map(&mw, w->bytes, w->n, w->row_bytes, w->bits, ow) != CUDA_SUCCESS ||
      encode_weight_map(&mw2, w2 ? w2->bytes : w->bytes, w->n, w->row_bytes, w->bits, ow) != CUDA_SUCCESS)
    return gq_fail(ctx, GQ_ERR_CUDA, "prefill: weight tensor map");
  dim3 grid((unsigned)((m + BM - 1) / BM), (unsigned)((w->n + ow - 1) / ow));
  if (w->bits == 4) return launch_mode<4, false>(ctx, mode, map, mw, mw2, a, grid, kSmemBytes);
  if (w->bits == 2) return launch_mode<2, false>(ctx, mode, map, mw, mw2, a, grid, kSmemBytes);
  if (w->signed_i8) return launch_mode<8, true>(ctx, mode, map, mw, mw2, a, grid, kSmemBytes);
  return launch_mode<8, false>(ctx, mode, map, mw, mw2, a, grid, kSmemBytes);
}

// ---- allocation-free variant ---------------------------------------------------
// For callers that cannot allocate device memory at call time: a serving process
// that reserves its whole HBM budget at start-up and treats any later cudaMalloc
// as an error, or an embedder whose buffers all come from its own arena. The
// scratch this path needs (the bf16 copy of the activations) lives in this
// file-scope array instead of a context workspace; every GPU that loads the
// library holds it until the process exits.
namespace {
constexpr int64_t kStaticScratchElems = int64_t(4) << 20;  // 4 Mi bf16 (8 MiB): M*K <= 4,194,304
static __device__ __align__(256) __nv_bfloat16 g_prefill_scratch[kStaticScratchElems];

// Host-side device addresses of the array, one per device. Host code must not
// pass the symbol itself to a kernel: in host code it names a host-side
// stand-in, not device memory.
struct StaticSetup {
  void *scratch = nullptr;
  int smem_optin = 0;
  bool ready = false;
};
StaticSetup g_static_setup[64];

cudaError_t static_setup(int dev, StaticSetup **out) {
  StaticSetup &st = g_static_setup[dev & 63];
  if (!st.ready) {
    cudaError_t e = cudaGetSymbolAddress(&st.scratch, g_prefill_scratch);
    if (e != cudaSuccess) return e;
    if (st.scratch == nullptr) return cudaErrorInvalidSymbol;
    e = cudaDeviceGetAttribute(&st.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    st.ready = true;
  }
  *out = &st;
  return cudaSuccess;
}

template <int BITS, bool SIGNED>
cudaError_t static_launch(cudaStream_t stream, const CUtensorMap &map, const CUtensorMap &mw, const PrefillArgs &a,
                          dim3 grid) {
  auto kern = prefill_tc_kernel<BITS, SIGNED, 0>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
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
  if (n > (int64_t(1) << 30)) return GQ_ERR_UNSUPPORTED;
  if ((uintptr_t)x % 16 != 0 || (uintptr_t)qbytes % 16 != 0 || (uintptr_t)scales % 4 != 0)
    return GQ_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQ_ERR_CUDA;
  StaticSetup *st = nullptr;
  if (static_setup(dev, &st) != cudaSuccess) return GQ_ERR_CUDA;
  if ((size_t)st->smem_optin < kSmemBytes || encode_fn() == nullptr) return GQ_ERR_UNSUPPORTED;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  __nv_bfloat16 *xb = static_cast<__nv_bfloat16 *>(st->scratch);
  {
    const int64_t n4 = m * k / 4;
    const unsigned g = (unsigned)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    cast_bf16_kernel<<<g, 256, 0, stream>>>(x, xb, n4);
    if (cudaGetLastError() != cudaSuccess) return GQ_ERR_CUDA;
  }
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
  cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  cuuint32_t box[2] = {BK, BM};
  cuuint32_t estr[2] = {1, 1};
  if (encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xb, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return GQ_ERR_CUDA;
  PrefillArgs a = {};
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.w = qbytes;
  a.s = scales;
  a.row_bytes = (int)(signed_i8 ? k : k * bits / 8);
  a.y = y;
  a.ldy = n;
  a.y_col0 = 0;
  a.err = nullptr;  // no context: a timed-out wait is still bounded, but not reported
  const dim3 grid((unsigned)((m + BM - 1) / BM), (unsigned)((n + BN - 1) / BN));
  CUtensorMap mw;
  if (encode_weight_map(&mw, qbytes, n, a.row_bytes, bits, BN) != CUDA_SUCCESS) return GQ_ERR_CUDA;
  cudaError_t e;
  if (bits == 4) e = static_launch<4, false>(stream, map, mw, a, grid);
  else if (bits == 2) e = static_launch<2, false>(stream, map, mw, a, grid);
  else if (signed_i8) e = static_launch<8, true>(stream, map, mw, a, grid);
  else e = static_launch<8, false>(stream, map, mw, a, grid);
  return e == cudaSuccess ? GQ_OK : GQ_ERR_CUDA;
}
