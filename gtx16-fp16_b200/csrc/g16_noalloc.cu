// Split-K GEMM entry point that allocates nothing (g16_gemm_static_scratch).
//
// Who needs it: callers that cannot allocate device memory when they call the GEMM. Typical
// examples are inference servers that reserve all of a GPU's memory for their own pools when they
// start (so a later cudaMalloc fails, or would bypass their accounting), and hosts that forbid
// cudaMalloc/cudaFree on latency-critical threads because those calls can synchronise the device.
// Such callers cannot provide the workspace that g16_gemm needs for its split-K partial tiles.
//
// This variant runs g16_gemm's own plan. Most plans need no scratch at all; the ones that do (the
// small-problem grid split, and the split into fp32 partial tiles reduced by a second kernel)
// keep their partial tiles in one fixed array in device memory instead of a workspace:
// g16_static_scratch below, 8 MiB, i.e. at most 64 partial tiles of 128 x 256 fp32. Every GPU that
// loads this library holds the array until the process exits. An explicit split whose partials do
// not fit is rejected with G16_ERR_TOO_LARGE; in the automatic plan the grid split gives way to the
// cluster plan when its partials do not fit, and a partial-tile split is lowered until they fit.
//
// The array is shared by every call on a device and keeps whatever the last call wrote. Nothing in
// it has to start at zero: each call writes every partial tile it later reads. Two calls whose
// work overlaps on the GPU (for example on two streams) race on the array and may return wrong
// results; callers must order them.
#include <cuda_runtime.h>

#include <mutex>

#include "g16_internal.cuh"

namespace g16 {
namespace {

constexpr size_t kStaticScratchBytes = static_cast<size_t>(G16_STATIC_SCRATCH_BYTES);

// The scratch array. In host code the name g16_static_scratch is only a host-side stand-in for the
// device symbol, not a device address; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g16_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g16_static_scratch on the current device. Looked up once per device, with
// that device current, on the first call there.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return G16_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g16_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e);
    if (p == nullptr) return G16_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return G16_OK;
}

size_t partials_bytes(int M, int K, int N, int ksplit) { return gemm_workspace_bytes(M, K, N, ksplit); }

}  // namespace
}  // namespace g16

using namespace g16;

// The plan is g16_gemm's own: launch_gemm is called with the static array as its workspace. Most
// plans need no workspace at all (the medium-M kernel, the small-problem cluster plan and the
// in-cluster split, single passes); the grid split runs only where its partials fit the array
// (else the cluster plan), and the partial-tile split (ksplit > 16, or a split whose cluster cannot
// be resident) is checked to fit before anything is launched (G16_ERR_WORKSPACE, nothing
// enqueued). So the same arguments give the same kernel and the same bits as g16_gemm given an
// 8 MiB workspace.
extern "C" int g16_gemm_static_scratch(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype,
                                       const float* bias, const float* rscale, int M, int K, int N, int ksplit,
                                       void* stream) {
  if (M < 0 || K < 0 || N < 0 || ksplit < 0 || (out_dtype != G16_F32 && out_dtype != G16_F16)) return G16_ERR_ARG;
  if (K % 8 != 0 || N % 8 != 0) return G16_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return G16_OK;
  if (K == 0 || a16 == nullptr || b16 == nullptr || out == nullptr) return G16_ERR_ARG;
  if (!aligned16(a16) || !aligned16(b16) || !aligned16(out)) return G16_ERR_ALIGN;
  if (bias != nullptr && !aligned16(bias)) return G16_ERR_ALIGN;
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  void* scratch = nullptr;
  st = scratch_address(&scratch);
  if (st != G16_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = launch_gemm(a16, b16, out, out_dtype, bias, rscale, M, K, N, ksplit, scratch, kStaticScratchBytes, s, *dev);
  if (st == G16_ERR_WORKSPACE && ksplit == 0) {
    // The automatic plan fell through to the partial-tile split and its partials do not fit:
    // lower that split until they do (down to a single pass) and run it explicitly.
    int ks = gemm_auto_ksplit(M, K, N, *dev);
    while (ks > 1 && partials_bytes(M, K, N, ks) > kStaticScratchBytes) --ks;
    st = launch_gemm(a16, b16, out, out_dtype, bias, rscale, M, K, N, ks, scratch, kStaticScratchBytes, s, *dev);
  }
  return st == G16_ERR_WORKSPACE ? G16_ERR_TOO_LARGE : st;
}
