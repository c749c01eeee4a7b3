// selftest.cu -- exercises the bounded-wait error path of the kernels on the
// device without faulting it: one warp waits, through the same mbar_wait the
// decode and prefill pipelines use, on an mbarrier that nothing arrives on.
// The wait gives up after limit_ns, the kernel sets B200_DEV_WAIT_TIMEOUT in
// the status word and returns normally, so the context stays usable.
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace b200 {

__global__ void bounded_wait_selftest_kernel(int32_t* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  // Phase 0 of `bar` never completes: no thread arrives on it.
  const bool ok = mbar_wait(&bar, 0, limit_ns);
  if (!__all_sync(0xffffffffu, ok) && threadIdx.x == 0) report(status, B200_DEV_WAIT_TIMEOUT);
}

int launch_bounded_wait_selftest(int32_t* status, int64_t limit_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(status, static_cast<uint64_t>(limit_ns));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bounded-wait selftest launch");
  return B200_OK;
}

}  // namespace b200
