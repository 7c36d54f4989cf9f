// selftest.cu — exercise the kernels' failure path without a GPU fault.
//
// One CTA waits, with the same bounded wait every pipeline uses, on an
// mbarrier that nothing ever arrives on. The wait gives up after `limit_ns`,
// sets the CTA's abort flag and the engine's wait-timeout error bit, and the
// kernel returns normally: the context stays usable and the host learns of the
// failure through rb_check_device_errors.
#include <cstdint>

#include "sm100.cuh"
#include "kernels.h"

namespace rb {

__global__ void wait_timeout_probe_kernel(uint32_t* err, uint64_t limit_ns, uint32_t* waited) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_timer_ns();
    const bool ok = mbar_wait_limit(&bar, 0, err, &abort_flag, limit_ns);
    waited[0] = ok ? 0u : static_cast<uint32_t>((global_timer_ns() - t0) / 1000u);  // microseconds
  }
}

int launch_wait_timeout_probe(uint32_t* err, int64_t limit_ns, uint32_t* waited, cudaStream_t st) {
  if (limit_ns <= 0 || limit_ns > 1000000000ll) return RB_E_SHAPE;  // at most 1 s
  wait_timeout_probe_kernel<<<1, 32, 0, st>>>(err, static_cast<uint64_t>(limit_ns), waited);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_E_DEVICE;
}

}  // namespace rb
