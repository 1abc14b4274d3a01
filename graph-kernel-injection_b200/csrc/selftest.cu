// Self-test of the failure path every tensor-core kernel relies on: a wait on
// an mbarrier phase that never completes gives up after its limit, records
// the timeout in the library's status word and returns, leaving the CUDA
// context usable.  Nothing here faults or hangs: the only wait is bounded.
#include "tc_prims.cuh"

namespace sbfa {
namespace {

__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(tc::smem_u32(&bar), 1);
    abort_flag = 0;
    tc::mbar_init_fence();
  }
  __syncthreads();
  // nothing ever arrives: phase 0 never completes and the wait must give up
  tc::wait_bar(tc::smem_u32(&bar), 0, &abort_flag, status, limit_ns);
}

}  // namespace
}  // namespace sbfa

extern "C" int sbfa_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  using namespace sbfa;
  if (limit_ns < 1000000 || limit_ns > 1000000000)
    return fail(SBFA_ERR_INVALID, "limit_ns must be in [1e6, 1e9]");
  cudaStream_t s = (cudaStream_t)stream;
  LaunchScope ls("wait_timeout_selftest_kernel", s);
  wait_timeout_selftest_kernel<<<1, 32, 0, s>>>((uint64_t)limit_ns, device_status_ptr());
  return check_launch("wait_timeout_selftest_kernel");
}
