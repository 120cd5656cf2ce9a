// Column-sharded GEMM with the output all-gather and the completion barrier both fused into the
// kernel (g16_gemm_allgather_mc): no host collective on the call path.
//
// Every rank runs the CTA-pair GEMM on its column shard. The epilogue writes each 128-byte output
// row segment once through the NVLink multicast address of the ranks' output buffers
// (multimem.st), and the switch delivers it to every GPU. After its last store each CTA fences and
// adds 1, with release semantics, to a counter that lives behind a second multicast address, so
// every GPU's copy of the counter counts the CTAs, of all ranks, that have finished. A one-thread
// kernel then waits on this GPU's counter (acquire loads, bounded by a time limit) until it reaches
// the caller's target: from then on, work later on the stream sees every rank's tiles.
//
// Counters only grow (mod 2^32). A caller keeps the running target: the previous one plus the sum,
// over the ranks, of g16_gemm_allgather_signals for the call's shape. Two calls in a row must not
// write the same output buffer (a peer may start call i + 1 while this rank still reads the result
// of call i); alternating two buffers is enough when each rank reads a result before its next
// call: a peer's call i + 1 starts only after this rank's kernel of call i has finished, so after
// this rank's stream has passed its reads of the result of call i - 1, which used the same buffer.
#include <cuda_runtime.h>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

namespace g16 {
namespace {

__global__ void wait_signals_kernel(const uint32_t* flag, uint32_t target, int* status, uint64_t limit_ns) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    const uint32_t v = ld_acquire_sys_u32(flag);
    if (static_cast<int32_t>(v - target) >= 0) return;
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicExch(status, G16_ERR_TIMEOUT);
      return;
    }
    __nanosleep(128);
  }
}

}  // namespace
}  // namespace g16

using namespace g16;

extern "C" int g16_gemm_allgather_signals(int M, int K, int N) {
  if (M < 0 || K <= 0 || N < 0) return -G16_ERR_ARG;
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return -st;
  if (!gemm_pair_available()) return -G16_ERR_UNSUPPORTED;
  return gemm_pair_ctas(M, N, *dev);
}

extern "C" int g16_gemm_allgather_mc(const uint16_t* a16, const uint16_t* b16, void* mc_out, int out_dtype,
                                     const float* bias, const float* rscale, int M, int K, int N, long long ldc,
                                     int col0, void* mc_flag, const uint32_t* flag, uint32_t target,
                                     int wait_limit_us, void* stream) {
  if (mc_out == nullptr || mc_flag == nullptr || flag == nullptr) return G16_ERR_ARG;
  if (M < 0 || K <= 0 || N < 0 || col0 < 0 || ldc < static_cast<long long>(col0) + N) return G16_ERR_ARG;
  if (out_dtype != G16_F32 && out_dtype != G16_F16) return G16_ERR_ARG;
  if (wait_limit_us < 1 || wait_limit_us > 60 * 1000 * 1000) return G16_ERR_ARG;
  if (K % 8 != 0 || N % 8 != 0 || col0 % 8 != 0 || ldc % 8 != 0) return G16_ERR_UNSUPPORTED;
  if (a16 == nullptr || b16 == nullptr) return G16_ERR_ARG;
  if (!aligned16(a16) || !aligned16(b16) || !aligned16(mc_out) || (bias != nullptr && !aligned16(bias)))
    return G16_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(mc_flag) & 3u) != 0 || (reinterpret_cast<uintptr_t>(flag) & 3u) != 0)
    return G16_ERR_ALIGN;
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  if (!gemm_pair_available()) return G16_ERR_UNSUPPORTED;
  int* status = device_status_ptr();
  if (status == nullptr) return G16_ERR_CUDA;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M > 0 && N > 0) {
    st = launch_gemm_pair_multimem(a16, b16, mc_out, out_dtype, bias, rscale, M, K, N, ldc, col0, s, *dev, mc_flag);
    if (st != G16_OK) return st;
  }
  // Also with nothing to compute here: the peers' tiles still have to land before the caller goes on.
  wait_signals_kernel<<<1, 32, 0, s>>>(flag, target, status, 1000ull * static_cast<uint64_t>(wait_limit_us));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}
