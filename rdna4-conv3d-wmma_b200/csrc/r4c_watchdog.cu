// r4c_watchdog.cu — self-test of the kernels' bounded waits.
//
// Every pipeline wait in the library's kernels is bounded (bounded_wait in
// r4c_sm100.cuh): a wait that lasts longer than its limit sets the device
// error flag that r4c_device_error() reads, and the kernel winds down instead
// of hanging the GPU. This kernel runs that same wait on an mbarrier that
// nothing ever arrives at, with a caller-chosen limit, so a test can make a
// wait run out on purpose and check that the kernel returns, that the flag is
// set, and that the context stays usable. No reference counterpart (the
// reference's Triton kernels have no device-side waits).
#include "r4c_internal.h"
#include "r4c_sm100.cuh"

namespace r4c {
namespace watchdog {

using namespace r4c::sm100;

__global__ void selftest_kernel(uint64_t limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);   // one arrival expected; none is ever made
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) bounded_wait(&bar, 0, limit_ns, &abort_flag, err, 3, 0);
  __syncthreads();
}

}  // namespace watchdog
}  // namespace r4c

extern "C" int r4c_watchdog_selftest(uint64_t limit_ns, r4c_stream_t stream) {
  if (limit_ns == 0 || limit_ns > 2000000000ull) return R4C_ERR_INVALID;
  int* err = r4c::tc::device_error_flag();
  if (!err) return R4C_ERR_NO_DEVICE;
  r4c::watchdog::selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns, err);
  r4c::note_launches(1);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}
