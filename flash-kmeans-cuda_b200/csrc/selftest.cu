// Test of the device-side failure path without a fault: a one-warp kernel
// waits, with the same bounded mbarrier wait the assignment pipeline uses, on
// a barrier that nothing ever arrives on. After the deadline the wait gives
// up, the kernel records a site code in the device error word (as an expired
// pipeline wait does) and returns; fkc_device_status() then reports
// FKC_ETIMEOUT and the context stays usable.
#include <cuda_runtime.h>

#include "fkc_internal.h"
#include "fkc_launch.cuh"
#include "fkc_ptx.cuh"

namespace fkc {
namespace {

constexpr int kErrSelfTest = 199;

__global__ void wait_selftest_kernel(int* err, uint64_t deadline_ns) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&bar), 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    // Phase 0 never completes: the wait can only end at its deadline.
    if (!ptx::mbar_wait(ptx::smem_u32(&bar), 0u, &abort_flag, deadline_ns))
      atomicCAS(err, 0, kErrSelfTest);
  }
}

}  // namespace
}  // namespace fkc

extern "C" FKC_CAPI_EXPORT int fkc_selftest_wait_timeout(uint32_t timeout_us,
                                                         fkc_stream_t stream) {
  fkc::clear_error();
  FKC_REQUIRE(timeout_us >= 1 && timeout_us <= 10000000u,
              "timeout_us must be in [1, 10^7] (got %u)", timeout_us);
  int* err = fkc::device_error_word();
  FKC_REQUIRE(err != nullptr, "no device error word on the current device");
  fkc::wait_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      err, static_cast<uint64_t>(timeout_us) * 1000ull);
  FKC_CUDA_TRY(cudaGetLastError());
  fkc::count_launches(1);
  return FKC_OK;
}
