// eb_selftest.cu -- eb_selftest_wait_timeout: exercises the failure path of
// the bounded waits every tcgen05 kernel here uses (eb_common.cuh mbar_wait):
// a one-CTA kernel waits on an mbarrier that nothing arrives on, with a
// short limit; the wait gives up, sets kErrTimeoutSelftest in the device
// error word and the kernel returns. Nothing faults or hangs, and the
// context stays usable, so a caller (or a test) can check that a stuck
// pipeline is reported through eb_get_device_error on its own deployment.
#include "../../include/eyebrowse_attn.h"
#include "eb_common.cuh"
#include "eb_kernels.cuh"

namespace eb {

__global__ void wait_timeout_selftest_kernel(unsigned* err, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // phase 0 never completes: no thread arrives and no copy is issued
  if (threadIdx.x == 0)
    (void)mbar_wait(smem_u32(&bar), 0, &abort_flag, err, kErrTimeoutSelftest, timeout_ns);
}

cudaError_t launch_wait_timeout_selftest(unsigned* err, unsigned long long timeout_ns,
                                         cudaStream_t st) {
  wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(err, timeout_ns);
  return cudaGetLastError();
}

}  // namespace eb
