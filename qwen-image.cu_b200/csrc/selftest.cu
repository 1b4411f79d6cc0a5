// selftest.cu -- exercises the bounded-wait error path without faulting.
//
// Every spin-wait in the tensor-core kernels gives up after a time limit,
// writes an error word and returns, so a stuck pipeline surfaces as
// QI_ERR_DEVICE from qi_ctx_check instead of a hung or trapped GPU.  This
// kernel waits on an mbarrier that nothing arrives on, with a short limit,
// and must take that path; the context stays usable afterwards.
#include "qi_internal.h"
#include "sm100.cuh"

namespace qi {
namespace {
__global__ void wait_timeout_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait_limit(&bar, 0, &abort_flag, limit_ns)) atomicCAS(err, 0, kErrTimeoutSelftest);
  }
}
}  // namespace

int selftest_wait_timeout(int* err, int limit_us, cudaStream_t stream) {
  if (limit_us <= 0 || limit_us > 2000000) return QI_ERR_ARG;
  wait_timeout_kernel<<<1, 32, 0, stream>>>(err, static_cast<uint64_t>(limit_us) * 1000ull);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}
}  // namespace qi
