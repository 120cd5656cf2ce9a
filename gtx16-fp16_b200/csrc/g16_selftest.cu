// Failure-detection self-test (g16_selftest_wait_timeout): exercises the bounded-wait path that
// every pipeline kernel in this library relies on, without any pipeline bug and without faulting
// or hanging the GPU.
//
// One CTA of two warps. Each warp's elected lane waits on its own mbarrier in shared memory, and
// nothing ever arrives on either. Warp 0 waits with the caller's short limit; when it expires it
// raises the CTA's abort flag and records G16_ERR_TIMEOUT in the device status word, exactly as a
// pipeline role does. Warp 1 waits with the library's full limit (kWaitLimitNs, 1 s) but returns
// as soon as it sees the abort flag, the way the other roles of a pipeline unwind after one role
// timed out. The kernel therefore ends shortly after the short limit, the context stays usable,
// and the host reads the status with g16_device_status.
#include <cuda_runtime.h>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

namespace g16 {
namespace {

__global__ void __launch_bounds__(64, 1) wait_timeout_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_flag;
  const uint32_t warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (elect_one()) {
    volatile int* flag = &abort_flag;
    if (warp == 0) {
      if (!mbar_wait_limit(&bars[0], 0, flag, limit_ns)) {
        *flag = 1;
        atomicExch(status, G16_ERR_TIMEOUT);
      }
    } else {
      // Unblocked by the abort flag long before its own 1 s limit.
      if (!mbar_wait(&bars[1], 0, flag) && *flag == 0) atomicExch(status, G16_ERR_TIMEOUT);
    }
  }
  __syncwarp();
  __syncthreads();
}

}  // namespace
}  // namespace g16

using namespace g16;

extern "C" int g16_selftest_wait_timeout(int limit_us, void* stream) {
  if (limit_us < 1 || limit_us > 1000000) return G16_ERR_ARG;
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  int* status = device_status_ptr();
  if (status == nullptr) return G16_ERR_CUDA;
  wait_timeout_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(status, 1000ull * limit_us);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}
