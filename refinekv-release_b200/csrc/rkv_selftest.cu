// rkv_selftest_wait_timeout: exercises the bounded-wait path every kernel of
// this library relies on, without a fault.  One warp initialises an mbarrier
// that nothing will ever complete, waits on it through the same warp-uniform
// bounded wait the kernels use (with a short limit instead of 1 s), records
// RKV_DEVICE_TIMEOUT in the status word as the kernels do, and returns.  The
// context stays usable and the call is graph-capturable.
#include <string>

#include "refinekv_b200.h"
#include "rkv_device.cuh"

namespace rkv {
void set_last_error(const std::string& message);
}

namespace {

__global__ void __launch_bounds__(32) wait_timeout_kernel(int* status,
                                                          unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    rkv::mbar_init(&bar, 1);
    rkv::mbar_fence_init();
  }
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, rkv::mbar_wait(&bar, 0, limit_ns));
  if (!ok && threadIdx.x == 0) atomicOr(status, rkv::kStatusTimeout);
}

}  // namespace

extern "C" {

int rkv_selftest_wait_timeout(int32_t* status, int64_t limit_ns, void* stream) {
  if (status == nullptr || limit_ns <= 0 || limit_ns > 1000000000LL) {
    rkv::set_last_error("rkv_selftest_wait_timeout: status must be non-null and 0 < limit_ns <= 1e9");
    return RKV_ERR_INVALID_ARGUMENT;
  }
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<unsigned long long>(limit_ns));
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    rkv::set_last_error(std::string("wait_timeout_kernel launch: ") + cudaGetErrorString(err));
    return RKV_ERR_CUDA;
  }
  return RKV_OK;
}

}  // extern "C"
