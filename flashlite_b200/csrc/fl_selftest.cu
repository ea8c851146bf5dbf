// Self-test of the bounded-wait failure path (fl_selftest_bounded_wait).
//
// Every mbarrier wait in this library's kernels goes through
// mbar_wait_hinted (fl_ptx.cuh): a wait that runs past its limit raises the
// CTA's abort flag and ORs kDevErrWaitTimeout into the device error word, and
// the CTA's other waiting roles see the flag and return instead of waiting
// out their own limits. This kernel runs exactly that protocol on barriers
// that nothing ever arrives on, with a short limit on one of them, so the
// failure path can be tested without a fault, a trap or an endless loop.

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/flashlite_b200.h"
#include "fl_internal.h"
#include "fl_ptx.cuh"

namespace fl {
namespace {

__global__ void __launch_bounds__(64, 1) selftest_wait_kernel(uint64_t limit_ns, uint64_t* out,
                                                              unsigned int* err) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars[0]), 1);  // expects one arrival; none ever comes
    mbar_init(smem_u32(&bars[1]), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t t0 = globaltimer_ns();
  const bool ok = mbar_wait_hinted(smem_u32(&bars[warp]), 0, abort_flag, err, FL_WAIT_HINT_NS,
                                   warp == 0 ? limit_ns : FL_WAIT_LIMIT_NS);
  const bool all = __all_sync(0xffffffffu, ok);
  const uint64_t t1 = globaltimer_ns();
  if ((threadIdx.x & 31) == 0) {
    out[2 * warp] = all ? 1u : 0u;
    out[2 * warp + 1] = t1 - t0;
  }
  __syncthreads();
}

}  // namespace
}  // namespace fl

extern "C" int fl_selftest_bounded_wait(uint64_t limit_ns, uint64_t* out, void* stream) {
  if (out == nullptr || limit_ns == 0 || limit_ns > 1000000000ull) {
    fl::set_last_error("fl_selftest_bounded_wait: out must be non-null and limit_ns in [1, 1e9]");
    return FL_ERR_INVALID_ARGUMENT;
  }
  if (!fl::prepare_current_device()) {
    fl::set_last_error("fl_selftest_bounded_wait: device initialisation failed");
    return FL_ERR_NO_DEVICE;
  }
  fl::selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, out,
                                                                             fl::device_error_word());
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fl::set_last_error(std::string("fl_selftest_bounded_wait: ") + cudaGetErrorString(e));
    return FL_ERR_CUDA;
  }
  return FL_OK;
}
