// chain_latency.cu — the latency floor of a chain of dependent phases on B200: the
// measurement behind the per-launch figures of the decode GEMV chain. A "phase" is
// what a decode-step op does besides its own work: wait for the previous op, read
// its 1536-float output (6 KB, from L2) with 148 CTAs x 512 threads, write a slice.
//  * launch chain: 210 such kernels captured in a CUDA graph, with and without
//    programmatic dependent launch (griddepcontrol.wait for the previous grid);
//  * persistent chain: the same 210 phases in one cooperative kernel, phases
//    separated by a grid barrier (one release-add per CTA, acquire polling).
// Prints us per phase; every wait is bounded (an iteration limit sets an error
// flag). Built and run by tests/test_chain_latency_gpu.py.
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdint>
#include <vector>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("ERR %s at %d: %s\n", #x, __LINE__, cudaGetErrorString(e)); return 1; } } while (0)

constexpr int K = 1536;

__device__ __forceinline__ uint64_t gtime() { uint64_t t; asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t)); return t; }

// one phase as its own launch: wait for the previous grid, read x (K floats), write a slice of y
__global__ void __launch_bounds__(512) phase_kernel(const float *x, float *y, int pdl) {
  __shared__ float red[16];
  if (pdl) { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); asm volatile("griddepcontrol.wait;" ::: "memory"); }
  float s = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) s += x[k];
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(~0u, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 16) {
    float v = red[threadIdx.x];
    for (int o = 8; o; o >>= 1) v += __shfl_xor_sync(0xffffu, v, o);
    if (threadIdx.x == 0) { for (int j = 0; j < 11; ++j) y[(blockIdx.x * 11 + j) % K] = v * 1e-3f + j; }
  }
}

// all phases in one persistent kernel with a grid barrier between phases
__global__ void __launch_bounds__(512) chain_kernel(float *buf, int phases, unsigned *counter, unsigned *err, unsigned long long *tsum) {
  __shared__ float red[16];
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  uint64_t t_wait = 0, t_read = 0;
  for (int p = 0; p < phases; ++p) {
    const float *x = buf + (p & 1) * K;
    float *y = buf + ((p + 1) & 1) * K;
    uint64_t t0 = gtime();
    float s = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) s += __ldcg(x + k);
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(~0u, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    uint64_t t1 = gtime();
    if (threadIdx.x < 16) {
      float v = red[threadIdx.x];
      for (int o = 8; o; o >>= 1) v += __shfl_xor_sync(0xffffu, v, o);
      if (threadIdx.x == 0) { for (int j = 0; j < 11; ++j) __stcg(y + (blockIdx.x * 11 + j) % K, v * 1e-3f + j); }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned target = (unsigned)(p + 1) * gridDim.x;
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(counter), "r"(1u) : "memory");
      unsigned v = 0; long it = 0;
      do {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
        if (++it > 4000000) { atomicOr(err, 1u); bad = 1; break; }
      } while ((int)(v - target) < 0);
    }
    __syncthreads();
    uint64_t t2 = gtime();
    t_read += t1 - t0; t_wait += t2 - t1;
    if (bad) break;
  }
  if (threadIdx.x == 0 && blockIdx.x == 0) { tsum[0] = t_read; tsum[1] = t_wait; }
}

int main() {
  int nsm = 0; CK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, 0));
  float *buf; CK(cudaMalloc(&buf, 2 * K * sizeof(float))); CK(cudaMemset(buf, 0, 2 * K * sizeof(float)));
  unsigned *counter, *err; unsigned long long *tsum;
  CK(cudaMalloc(&counter, 4)); CK(cudaMalloc(&err, 4)); CK(cudaMalloc(&tsum, 16));
  cudaStream_t st; CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  cudaEvent_t a, b; CK(cudaEventCreate(&a)); CK(cudaEventCreate(&b));
  const int N = 210;
  for (int pdl = 0; pdl < 2; ++pdl) {
    cudaGraph_t g; cudaGraphExec_t ge;
    CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeGlobal));
    for (int i = 0; i < N; ++i) {
      cudaLaunchConfig_t cfg = {}; cfg.gridDim = dim3(nsm); cfg.blockDim = dim3(512); cfg.stream = st;
      cudaLaunchAttribute at[1]; at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      at[0].val.programmaticStreamSerializationAllowed = 1; cfg.attrs = at; cfg.numAttrs = pdl;
      CK(cudaLaunchKernelEx(&cfg, phase_kernel, (const float *)(buf + (i & 1) * K), buf + ((i + 1) & 1) * K, pdl));
    }
    CK(cudaStreamEndCapture(st, &g)); CK(cudaGraphInstantiate(&ge, g, 0));
    for (int w = 0; w < 5; ++w) CK(cudaGraphLaunch(ge, st));
    CK(cudaStreamSynchronize(st));
    CK(cudaEventRecord(a, st));
    for (int r = 0; r < 20; ++r) CK(cudaGraphLaunch(ge, st));
    CK(cudaEventRecord(b, st)); CK(cudaEventSynchronize(b));
    float ms; CK(cudaEventElapsedTime(&ms, a, b));
    printf("launch chain pdl=%d: %.3f us per launch\n", pdl, ms * 1000.f / (20 * N));
  }
  for (int rep = 0; rep < 3; ++rep) {
    CK(cudaMemset(counter, 0, 4)); CK(cudaMemset(err, 0, 4));
    int phases = N;
    void *args[] = {&buf, &phases, &counter, &err, &tsum};
    CK(cudaEventRecord(a, st));
    CK(cudaLaunchCooperativeKernel((void *)chain_kernel, dim3(nsm), dim3(512), args, 0, st));
    CK(cudaEventRecord(b, st)); CK(cudaEventSynchronize(b));
    float ms; CK(cudaEventElapsedTime(&ms, a, b));
    unsigned errv = 0; unsigned long long ts[2];
    CK(cudaMemcpy(&errv, err, 4, cudaMemcpyDeviceToHost)); CK(cudaMemcpy(ts, tsum, 16, cudaMemcpyDeviceToHost));
    printf("persistent chain: %.3f us per phase (err=%u; cta0 read %.3f us, barrier %.3f us per phase)\n",
           ms * 1000.f / N, errv, ts[0] / 1000.0 / N, ts[1] / 1000.0 / N);
  }
  return 0;
}
