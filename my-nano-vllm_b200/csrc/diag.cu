// Diagnostics entry points (no counterpart in the reference): they exercise, on the GPU, the
// library's own device-side mechanisms in isolation, so tests can check them directly.
//   fp8attn_diag_wait_timeout  the bounded mbarrier wait every engine uses, on a barrier that
//                              nothing ever arrives on: the wait must give up after its limit,
//                              record kDevErrWaitTimeout in the error word and let the launch end
//                              with the control block's work counters back at zero;
//   fp8attn_diag_exp2          the FMA-pipe exp2 of the prefill softmax (exp2_poly_x2) next to
//                              the MUFU ex2.approx, element by element.
#include "../../include/fp8attn.h"
#include "common.cuh"
#include "kernels.h"

namespace fp8attn {
namespace {

constexpr int kDiagThreads = 64;

// Every CTA claims one work item from ctrl[1] like the persistent engines do, then its first
// warp waits (bounded by limit_ns) on an mbarrier whose expected arrival never happens; the
// teardown is the engines' own (release_work_counters).
__global__ void __launch_bounds__(kDiagThreads) wait_timeout_kernel(int* ctrl,
                                                                   unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none is ever made
    fence_mbar_init();
    atomicAdd(ctrl + 1, 1);
  }
  __syncthreads();
  if (threadIdx.x < 32) mbar_wait_for(&bar, 0, ctrl, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0) release_work_counters(ctrl);
}

__global__ void exp2_kernel(const float* __restrict__ x, float* __restrict__ poly,
                            float* __restrict__ mufu, int64_t n) {
  const int64_t i = 2 * (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i], x1 = i + 1 < n ? x[i + 1] : 0.f;
  float p0, p1;
  exp2_poly_x2(x0, x1, p0, p1);
  poly[i] = p0;
  mufu[i] = ex2(x0);
  if (i + 1 < n) {
    poly[i + 1] = p1;
    mufu[i + 1] = ex2(x1);
  }
}

}  // namespace
}  // namespace fp8attn

extern "C" {

int fp8attn_diag_wait_timeout(void* workspace, int64_t limit_ns, int num_ctas, void* stream) {
  if (workspace == nullptr || limit_ns < 0 || num_ctas < 1 || num_ctas > 1024) return FP8ATTN_EINVAL;
  fp8attn::wait_timeout_kernel<<<num_ctas, fp8attn::kDiagThreads, 0,
                                 static_cast<cudaStream_t>(stream)>>>(
      static_cast<int*>(workspace), static_cast<unsigned long long>(limit_ns));
  return cudaGetLastError() == cudaSuccess ? FP8ATTN_OK : FP8ATTN_ECUDA;
}

int fp8attn_diag_exp2(const float* x, float* poly, float* mufu, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (x == nullptr || poly == nullptr || mufu == nullptr)))
    return FP8ATTN_EINVAL;
  if (n == 0) return FP8ATTN_OK;
  const int64_t pairs = (n + 1) / 2;
  const int threads = 256;
  fp8attn::exp2_kernel<<<static_cast<unsigned>((pairs + threads - 1) / threads), threads, 0,
                         static_cast<cudaStream_t>(stream)>>>(x, poly, mufu, n);
  return cudaGetLastError() == cudaSuccess ? FP8ATTN_OK : FP8ATTN_ECUDA;
}

}  // extern "C"
