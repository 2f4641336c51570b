// gq_internal.cuh — shared definitions of libgq.so: the context and weight
// objects behind the C ABI, and the sm_100a PTX helpers the kernels use
// (mbarrier, bulk async copy, programmatic dependent launch, bounded waits).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/gq.h"

// Extra destinations of a GEMV's output: peer GPUs' buffers mapped into this
// device's address space (CUDA IPC). Every output element is also stored at
// p[i] + (its offset in y). n = 0 is the plain single output.
constexpr int kMaxPeerDst = 8;
struct PeerDst {
  float *p[kMaxPeerDst];
  int n;
  // completion signal (optional): sync = {CTA counter, epoch}, zeroed at set-up,
  // on this device. The last CTA of the grid (after every CTA's pushes) resets
  // the counter, increments the epoch and stores it at flag[i] + rank for every
  // rank i (own flags first, then the peers'). The epoch lives in device memory
  // so a captured graph replays with fresh epochs.
  uint32_t *flag[kMaxPeerDst + 1];
  uint32_t *sync;
  int rank;
  int signal;  // 1 on the launch that completes the output (the last row slice)
  // fused completion wait: after publishing, the last CTA also waits (bounded by
  // wait_limit_ns, timeout reported in *err) until every rank's flag in this rank's
  // own array (flag[0][0 .. n]) has reached the epoch, so the grid completes only
  // when the full logits are on this rank
  int fused_wait;
  uint64_t wait_limit_ns;
  uint32_t *err;
};

struct gq_ctx {
  int device = 0;
  int num_sms = 0;
  size_t smem_optin = 0;       // max dynamic shared memory per block
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  uint32_t *dev_err = nullptr; // device status word (GQ_DEVERR_*)
  bool pdl = true;             // launch with programmatic stream serialization
  uint64_t wait_limit_ns = 2000000000ull;  // bound of the cross-GPU waits (gq_peer_wait)
  std::string last_error;
  // temporaries of the composed fallbacks (generic kernel + elementwise epilogue)
  float *scratch[2] = {nullptr, nullptr};
  size_t scratch_cap[2] = {0, 0};
  // workspace of the tensor-core prefill path (f16 copy of the activations, row exponents)
  void *ws = nullptr;
  size_t ws_cap = 0;
  // set by gq_linear_softcap_peers(_signal) for the duration of one call
  PeerDst peers = {};
  PeerDst peer_signal = {};
};

struct gq_qweight {
  gq_ctx *ctx = nullptr;
  int device = 0;
  uint8_t *bytes = nullptr;    // packed rows, reference layout, padded allocation
  float *scales = nullptr;     // [n, scale_stride]
  int64_t n = 0, k = 0;
  int32_t bits = 0;
  int32_t signed_i8 = 0;
  int64_t group_size = 0;
  int64_t row_bytes = 0;       // bytes per packed row
  int64_t scale_stride = 0;    // scale entries per row
  int64_t qsum_off = 0;        // float offset of the per-row code sums (16-byte aligned)
  size_t nbytes = 0;
};

// ---- status helpers (host) ------------------------------------------------
int gq_fail(gq_ctx *ctx, int status, const std::string &msg);
// Make the context's device current for the calling host thread.
int gq_enter_ctx(gq_ctx *ctx);
// The context workspace, grown on demand with stream-ordered allocation. Growth
// is refused while the stream is being captured (the allocation would belong to
// the graph): run a call once eagerly before recording it.
int gq_workspace(gq_ctx *ctx, size_t bytes, void **out);
int gq_cuda_fail(gq_ctx *ctx, cudaError_t e, const char *what);
#define GQ_CUDA_TRY(ctx, expr)                                   \
  do {                                                           \
    cudaError_t _e = (expr);                                     \
    if (_e != cudaSuccess) return gq_cuda_fail((ctx), _e, #expr); \
  } while (0)

// Launch with optional programmatic dependent launch (PDL) on ctx->stream.
template <typename Kern, typename... Args>
static inline cudaError_t gq_launch(gq_ctx *ctx, Kern kernel, dim3 grid, dim3 block, size_t smem,
                                    Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ctx->pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---- device helpers ----------------------------------------------------------
namespace gqd {

// Programmatic dependent launch: wait for the upstream grid's results / let the
// downstream grid start its prologue. No-ops when launched without PDL.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: gives up after `limit_ns` of wall time
// (checked every 1024 polls) and returns false. Never spins forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// 1-D bulk async copy global -> shared (TMA engine), completion counted on bar.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Order this thread's earlier shared-memory accesses before later async-proxy
// (bulk copy) writes to the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Push this CTA's finished outputs (token rows 0..m-1, columns [c0, c1) of the
// [m, ldy] output) from its local buffer to every peer destination with
// coalesced 16-byte NVLink stores, then fence: call after a block barrier that
// follows the CTA's local output stores (bar.sync makes them visible to the
// block), by all threads of the block. One thread's system-scope fence after a
// second barrier orders every store of the CTA (fences are cumulative).
__device__ __forceinline__ void push_to_peers(const float *y, const PeerDst &pd, int m, int64_t ldy, int64_t c0,
                                              int64_t c1) {
  const int tid = threadIdx.x, nt = blockDim.x;
  if (pd.n == 0 && !pd.signal) return;
  // a CTA with no columns still counts towards the completion signal
  for (int r = 0; r < m && c1 > c0 && pd.n > 0; ++r) {
    const int64_t base = (int64_t)r * ldy;
    int64_t a = c0, b = c1;
    // ragged head and tail element by element, the aligned middle as float4
    while (a < b && ((base + a) & 3)) {
      if (tid == 0)
        for (int i = 0; i < pd.n; ++i) pd.p[i][base + a] = y[base + a];
      ++a;
    }
    while (b > a && ((base + b) & 3)) {
      --b;
      if (tid == 0)
        for (int i = 0; i < pd.n; ++i) pd.p[i][base + b] = y[base + b];
    }
    const int64_t n4 = (b - a) / 4;
    const float4 *src = reinterpret_cast<const float4 *>(y + base + a);
    for (int64_t j = tid; j < n4; j += nt) {
      const float4 v = src[j];
      for (int i = 0; i < pd.n; ++i) reinterpret_cast<float4 *>(pd.p[i] + base + a)[j] = v;
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    if (pd.signal && pd.sync) {
      // the last CTA to finish publishes the next epoch to every rank (release, system scope)
      const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
      if (atomicAdd(pd.sync, 1u) == total - 1) {
        __threadfence_system();
        volatile uint32_t *sy = pd.sync;
        sy[0] = 0u;
        const uint32_t e = sy[1] + 1u;
        sy[1] = e;
        for (int i = 0; i <= pd.n; ++i)
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(pd.flag[i] + pd.rank), "r"(e) : "memory");
        if (pd.fused_wait) {
          const uint64_t t0 = globaltimer_ns();
          bool timed_out = false;
          for (int r = 0; r <= pd.n && !timed_out; ++r) {
            for (uint32_t it = 0;; ++it) {
              uint32_t v;
              asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(pd.flag[0] + r) : "memory");
              if ((int32_t)(v - e) >= 0) break;
              if ((it & 255u) == 255u && globaltimer_ns() - t0 > pd.wait_limit_ns) {
                if (pd.err) atomicOr(pd.err, GQ_DEVERR_WAIT_TIMEOUT);
                timed_out = true;
                break;
              }
              __nanosleep(32);
            }
          }
        }
      }
    }
  }
}

__device__ __forceinline__ void report(uint32_t *err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

// tanh-approximated GELU of rust/src/backend_cpu.rs:55-58, same operation order
// (0.5*v) * (1 + tanh(c * (v + ((0.044715*v)*v)*v))). tanhf is CUDA's accurate
// single-precision tanh.
__device__ __forceinline__ float gelu_tanh(float v) {
  // c = sqrtf(2.0f / (float)pi) exactly as the f32 expression evaluates on the
  // CPU (0x3F4C4229), one ulp below the correctly rounded sqrt(2/pi).
  const float c = __int_as_float(0x3F4C4229);
  float inner = __fmul_rn(c, __fadd_rn(v, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v)));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}

}  // namespace gqd
