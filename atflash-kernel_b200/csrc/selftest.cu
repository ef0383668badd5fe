// Self-test of the bounded device waits every kernel of this library uses: one
// thread waits on an mbarrier that nothing ever arrives on. The wait gives up
// after its time limit (kWaitLimitNs), writes kDevErrTimeout to the caller's
// error flag and the kernel returns, leaving the context usable. No GPU fault,
// trap or unbounded wait is involved.
#include "atf_internal.h"
#include "atf_ptx.cuh"

namespace atf {
namespace selftest {

__global__ void wait_timeout_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  const AbortCtl ab{reinterpret_cast<volatile int*>(&s_abort), err};
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, ab, kDevErrTimeout);
}

}  // namespace selftest
}  // namespace atf

using namespace atf;

extern "C" int atf_selftest_wait_timeout(int* error_flag, atf_stream_t stream) {
  if (error_flag == nullptr) return ATF_ERR_INVALID_ARG;
  int dev = 0;
  int rc = check_device(&dev);
  if (rc != ATF_OK) return rc;
  selftest::wait_timeout_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(error_flag);
  return cudaGetLastError() == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
}
