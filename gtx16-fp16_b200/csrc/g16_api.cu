// C-ABI entry points (include/g16.h): argument checks, per-device state and the dispatch that the
// reference performs in Python in mm_t (src/gtx16_fp16/ops.py:65-108).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

namespace g16 {

// One status word per device (each device holds its own copy of module-scope device variables).
__device__ int g16_status_word = 0;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceInfo g_info[kMaxDevices];
bool g_info_ok[kMaxDevices] = {};
int* g_status_ptr[kMaxDevices] = {};
std::atomic<uint64_t> g_launches{0};
thread_local int t_last_cuda = 0;

__global__ void fill_rows_kernel(void* out, int out_f16, const float* bias, int M, int N, int act) {
  const size_t total = static_cast<size_t>(M) * N;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = apply_act(bias != nullptr ? bias[i % N] : 0.f, act);
    if (out_f16)
      reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
    else
      reinterpret_cast<float*>(out)[i] = v;
  }
}

int current_device(int* dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (*dev < 0 || *dev >= kMaxDevices) return G16_ERR_DEVICE;
  return G16_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// fp32 activations in g16_mm_t: the row rescale as its own pass (rowscale writes the fp16 copy of x
// that the GEMM reads). G16_FUSED_RESCALE=1 (a build option) makes g16_mm_t use the form fused into
// the GEMM's A operand instead, wherever that applies (g16_mm_t_fused_rescale): on B200 the fused
// form measured slower on every shape tried, so it is not the default.
#ifndef G16_FUSED_RESCALE
#define G16_FUSED_RESCALE 0
#endif

// Workspace layout of g16_mm_t: [split-K partials | x16 | rscale | rscale_inv], each part 256-byte
// aligned. fp32 x: x16 (the fp16 copy of x) with the rowscale pass, rscale_inv with the fused one.
struct MmLayout {
  size_t partials_bytes = 0, x16_off = 0, rscale_off = 0, rscale_inv_off = 0, total = 0;
  int ksplit = 1;
  bool fused_rescale = false;
};

MmLayout mm_layout(int M, int K, int N, int x_dtype, const DeviceInfo& dev) {
  MmLayout L;
  if (M <= G16_SKINNY_MAX_M || K == 0) return L;
  L.ksplit = gemm_auto_ksplit(M, K, N, dev);
  size_t off = 0;
  const size_t partials = gemm_auto_workspace_bytes(M, K, N, dev);
  if (partials > 0) {
    L.partials_bytes = align_up(partials, 256);
    off += L.partials_bytes;
  }
  if (x_dtype == G16_F32) {
    L.fused_rescale = G16_FUSED_RESCALE && gemm_auto_uses_pair(M, K, N, dev);
    if (!L.fused_rescale) {
      L.x16_off = off;
      off += align_up(static_cast<size_t>(M) * K * 2, 256);
    }
    L.rscale_off = off;
    off += align_up(static_cast<size_t>(M) * 4, 256);
    if (L.fused_rescale) {
      L.rscale_inv_off = off;
      off += align_up(static_cast<size_t>(M) * 4, 256);
    }
  }
  L.total = off;
  return L;
}

int check_common(const void* x, int x_dtype, const void* w, const void* out, int out_dtype, int M, int K, int N) {
  if (M < 0 || K < 0 || N < 0) return G16_ERR_ARG;
  if ((x_dtype != G16_F32 && x_dtype != G16_F16) || (out_dtype != G16_F32 && out_dtype != G16_F16)) return G16_ERR_ARG;
  if (K % 8 != 0 || N % 8 != 0) return G16_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return G16_OK;
  if (out == nullptr || (K > 0 && (x == nullptr || w == nullptr))) return G16_ERR_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return G16_ERR_ALIGN;
  return G16_OK;
}

}  // namespace

int cuda_fail(cudaError_t e) {
  t_last_cuda = static_cast<int>(e);
  return G16_ERR_CUDA;
}

void note_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

const DeviceInfo* device_info(int* status) {
  int dev = 0;
  int st = current_device(&dev);
  if (st != G16_OK) {
    *status = st;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_info_ok[dev]) {
    DeviceInfo d;
    cudaError_t e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) {
      *status = cuda_fail(e);
      return nullptr;
    }
    g_info[dev] = d;
    g_info_ok[dev] = true;
  }
  if (g_info[dev].cc_major != 10) {  // kernels are built for sm_100a only
    *status = G16_ERR_DEVICE;
    return nullptr;
  }
  *status = G16_OK;
  return &g_info[dev];
}

int* device_status_ptr() {
  int dev = 0;
  if (current_device(&dev) != G16_OK) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g16_status_word);
    if (e != cudaSuccess) {
      cuda_fail(e);
      return nullptr;
    }
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

}  // namespace g16

using namespace g16;

extern "C" {

int g16_version(void) { return 100; }

uint64_t g16_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int g16_last_cuda_error(void) { return t_last_cuda; }

const char* g16_strerror(int status) {
  switch (status) {
    case G16_OK: return "ok";
    case G16_ERR_ARG: return "invalid argument (size, dtype code or null pointer)";
    case G16_ERR_UNSUPPORTED: return "unsupported shape: K and N must be multiples of 8";
    case G16_ERR_ALIGN: return "pointer not 16-byte aligned (workspace: 256-byte)";
    case G16_ERR_WORKSPACE: return "workspace missing or too small";
    case G16_ERR_CUDA: return t_last_cuda != 0 ? cudaGetErrorString(static_cast<cudaError_t>(t_last_cuda)) : "CUDA error";
    case G16_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case G16_ERR_TIMEOUT: return "a kernel's bounded device-side wait expired";
    case G16_ERR_TOO_LARGE: return "split-K partial tiles exceed the fixed 8 MiB scratch array of g16_gemm_static_scratch";
    default: return "unknown g16 status";
  }
}

size_t g16_mm_t_workspace_bytes(int M, int K, int N, int x_dtype) {
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return 0;
  return mm_layout(M, K, N, x_dtype, *dev).total;
}

size_t g16_gemm_workspace_bytes(int M, int K, int N, int ksplit) {
  if (ksplit == 0) {
    int st = G16_OK;
    const DeviceInfo* dev = device_info(&st);
    if (dev == nullptr) return 0;
    return gemm_auto_workspace_bytes(M, K, N, *dev);
  }
  return gemm_workspace_bytes(M, K, N, ksplit);
}

int g16_gemm_auto_ksplit(int M, int K, int N) {
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return -st;
  return gemm_auto_ksplit(M, K, N, *dev);
}

namespace {

int mm_t_impl(const void* x, int x_dtype, const void* w_t, const float* bias, void* out, int out_dtype, int M, int K,
              int N, void* workspace, size_t workspace_bytes, void* stream, int act) {
  int st = check_common(x, x_dtype, w_t, out, out_dtype, M, K, N);
  if (st != G16_OK) return st;
  if (M == 0 || N == 0) return G16_OK;
  if (bias != nullptr && !aligned16(bias)) return G16_ERR_ALIGN;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) {  // empty reduction: every row is the bias (or zero), like the reference's kernels
    fill_rows_kernel<<<dev->sm_count * 4, 256, 0, s>>>(out, out_dtype == G16_F16, bias, M, N, act);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    note_launch();
    return G16_OK;
  }
  if (M <= G16_SKINNY_MAX_M)
    return launch_skinny(x, x_dtype, static_cast<const uint16_t*>(w_t), bias, out, out_dtype, M, K, N, s, *dev, act);

  const MmLayout L = mm_layout(M, K, N, x_dtype, *dev);
  if (L.total > 0) {
    if (workspace == nullptr || workspace_bytes < L.total) return G16_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return G16_ERR_ALIGN;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const uint16_t* a16 = static_cast<const uint16_t*>(x);
  const float* rscale = nullptr;
  if (x_dtype == G16_F32 && L.fused_rescale) {
    float* rs = reinterpret_cast<float*>(ws + L.rscale_off);
    float* rsi = reinterpret_cast<float*>(ws + L.rscale_inv_off);
    st = launch_rowamax(static_cast<const float*>(x), rs, rsi, M, K, G16_ROW_SCALE_THRESHOLD, s);
    if (st != G16_OK) return st;
    return launch_gemm_pair_f32a(static_cast<const float*>(x), static_cast<const uint16_t*>(w_t), out, out_dtype,
                                 bias, rs, rsi, M, K, N, s, *dev, act);
  }
  if (x_dtype == G16_F32) {
    uint16_t* x16 = reinterpret_cast<uint16_t*>(ws + L.x16_off);
    float* rs = reinterpret_cast<float*>(ws + L.rscale_off);
    st = launch_rowscale(x, G16_F32, x16, rs, M, K, G16_ROW_SCALE_THRESHOLD, s);
    if (st != G16_OK) return st;
    a16 = x16;
    rscale = rs;
  }
  // fp16 activations need no rescale here: products accumulate in fp32 TMEM and cannot overflow
  // the way the reference's fp16 partial sums could.
  // ksplit 0: the automatic plan (L.ksplit sized the workspace for its fallback).
  return launch_gemm(a16, static_cast<const uint16_t*>(w_t), out, out_dtype, bias, rscale, M, K, N, 0,
                     L.partials_bytes > 0 ? ws : nullptr, L.partials_bytes, s, *dev, act);
}

}  // namespace

int g16_mm_t(const void* x, int x_dtype, const void* w_t, const float* bias, void* out, int out_dtype, int M, int K,
             int N, void* workspace, size_t workspace_bytes, void* stream) {
  return mm_t_impl(x, x_dtype, w_t, bias, out, out_dtype, M, K, N, workspace, workspace_bytes, stream, G16_ACT_NONE);
}

int g16_mm_t_act(const void* x, int x_dtype, const void* w_t, const float* bias, void* out, int out_dtype, int M,
                 int K, int N, int act, void* workspace, size_t workspace_bytes, void* stream) {
  if (act != G16_ACT_NONE && act != G16_ACT_GELU) return G16_ERR_ARG;
  return mm_t_impl(x, x_dtype, w_t, bias, out, out_dtype, M, K, N, workspace, workspace_bytes, stream, act);
}

size_t g16_mm_t_fused_rescale_workspace_bytes(int M) {
  return M > 0 ? 2 * align_up(static_cast<size_t>(M) * 4, 256) : 0;
}

int g16_mm_t_fused_rescale(const float* x, const void* w_t, const float* bias, void* out, int out_dtype, int M,
                           int K, int N, int act, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_common(x, G16_F32, w_t, out, out_dtype, M, K, N);
  if (st != G16_OK) return st;
  if (act != G16_ACT_NONE && act != G16_ACT_GELU) return G16_ERR_ARG;
  if (M == 0 || N == 0) return G16_OK;
  if (K == 0) return G16_ERR_UNSUPPORTED;
  if (bias != nullptr && !aligned16(bias)) return G16_ERR_ALIGN;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  if (M <= G16_SKINNY_MAX_M || !gemm_pair_available()) return G16_ERR_UNSUPPORTED;
  const size_t need = g16_mm_t_fused_rescale_workspace_bytes(M);
  if (workspace == nullptr || workspace_bytes < need) return G16_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return G16_ERR_ALIGN;
  float* rs = static_cast<float*>(workspace);
  float* rsi = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + need / 2);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = launch_rowamax(x, rs, rsi, M, K, G16_ROW_SCALE_THRESHOLD, s);
  if (st != G16_OK) return st;
  return launch_gemm_pair_f32a(x, static_cast<const uint16_t*>(w_t), out, out_dtype, bias, rs, rsi, M, K, N, s, *dev,
                               act);
}

int g16_skinny(const void* x, int x_dtype, const uint16_t* w_t, const float* bias, void* out, int out_dtype, int M,
               int K, int N, void* stream) {
  int st = check_common(x, x_dtype, w_t, out, out_dtype, M, K, N);
  if (st != G16_OK) return st;
  if (M == 0 || N == 0) return G16_OK;
  if (M > G16_SKINNY_MAX_M) return G16_ERR_ARG;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  return launch_skinny(x, x_dtype, w_t, bias, out, out_dtype, M, K, N, static_cast<cudaStream_t>(stream), *dev);
}

int g16_rowscale(const void* x, int x_dtype, uint16_t* y16, float* rscale, int M, int K, float thresh, void* stream) {
  if (M < 0 || K < 0 || (x_dtype != G16_F32 && x_dtype != G16_F16)) return G16_ERR_ARG;
  if (K % 8 != 0) return G16_ERR_UNSUPPORTED;
  if (M == 0) return G16_OK;
  if (x == nullptr || y16 == nullptr || rscale == nullptr) return G16_ERR_ARG;
  if (!aligned16(x) || !aligned16(y16)) return G16_ERR_ALIGN;
  if (!(thresh > 0.f)) return G16_ERR_ARG;
  int st = G16_OK;
  if (device_info(&st) == nullptr) return st;
  return launch_rowscale(x, x_dtype, y16, rscale, M, K, thresh, static_cast<cudaStream_t>(stream));
}

int g16_gemm(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
             const float* rscale, int M, int K, int N, int ksplit, void* workspace, size_t workspace_bytes,
             void* stream) {
  int st = check_common(a16, G16_F16, b16, out, out_dtype, M, K, N);
  if (st != G16_OK) return st;
  if (M == 0 || N == 0) return G16_OK;
  if (K == 0 || ksplit < 0) return G16_ERR_ARG;
  if (bias != nullptr && !aligned16(bias)) return G16_ERR_ALIGN;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  return launch_gemm(a16, b16, out, out_dtype, bias, rscale, M, K, N, ksplit, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), *dev);
}

int g16_gemm_scatter(const uint16_t* a16, const uint16_t* b16, void* const* dst, int ndst, int out_dtype,
                     const float* bias, const float* rscale, int M, int K, int N, long long ldc, int col0,
                     int flags, void* stream) {
  if (dst == nullptr || ndst < 1 || ndst > G16_SCATTER_MAX_DST) return G16_ERR_ARG;
  if (flags != G16_SCATTER_DEFAULT && flags != G16_SCATTER_STORES && flags != G16_SCATTER_TMA &&
      flags != G16_SCATTER_PAIRS && flags != G16_SCATTER_MULTIMEM)
    return G16_ERR_ARG;
  if (flags == G16_SCATTER_MULTIMEM && ndst != 1) return G16_ERR_ARG;
  if (M < 0 || K <= 0 || N < 0 || col0 < 0 || ldc < static_cast<long long>(col0) + N) return G16_ERR_ARG;
  if (out_dtype != G16_F32 && out_dtype != G16_F16) return G16_ERR_ARG;
  if (K % 8 != 0 || N % 8 != 0 || col0 % 8 != 0 || ldc % 8 != 0) return G16_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return G16_OK;
  if (a16 == nullptr || b16 == nullptr) return G16_ERR_ARG;
  if (!aligned16(a16) || !aligned16(b16) || (bias != nullptr && !aligned16(bias))) return G16_ERR_ALIGN;
  for (int d = 0; d < ndst; ++d) {
    if (dst[d] == nullptr) return G16_ERR_ARG;
    if (!aligned16(dst[d])) return G16_ERR_ALIGN;
  }
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  return launch_gemm_scatter(a16, b16, dst, ndst, out_dtype, bias, rscale, M, K, N, ldc, col0, flags,
                             static_cast<cudaStream_t>(stream), *dev);
}

int g16_ipc_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return G16_ERR_ARG;
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e);
  return G16_OK;
}

int g16_ipc_free(void* ptr) {
  if (ptr == nullptr) return G16_ERR_ARG;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? G16_OK : cuda_fail(e);
}

int g16_ipc_get_handle(void* ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == G16_IPC_HANDLE_BYTES, "IPC handle size");
  if (ptr == nullptr || handle == nullptr) return G16_ERR_ARG;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e);
  std::memcpy(handle, &h, sizeof(h));
  return G16_OK;
}

int g16_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return G16_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e);
  return G16_OK;
}

int g16_ipc_close(void* ptr) {
  if (ptr == nullptr) return G16_ERR_ARG;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? G16_OK : cuda_fail(e);
}

int g16_gemm_plan(int M, int K, int N, int* info) {
  if (info == nullptr || M <= 0 || K <= 0 || N <= 0) return G16_ERR_ARG;
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  const int ranks = gemm_midm_ranks(M, K, N, *dev);
  if (ranks > 0) {
    info[0] = 2;
    info[1] = 128;
    info[2] = ranks;
    return G16_OK;
  }
  const SmallPlan p = plan_gemm_small(M, K, N, *dev);
  if (p.bn != 0 && p.gs_split > 1) {
    info[0] = 3;
    info[1] = p.gs_bn;
    info[2] = p.gs_split;
    return G16_OK;
  }
  info[0] = p.bn != 0 ? 1 : 0;
  info[1] = p.bn != 0 ? p.bn : kBN;
  info[2] = p.bn != 0 ? p.csize : gemm_auto_ksplit(M, K, N, *dev);
  return G16_OK;
}

int g16_skinny_plan(int M, int K, int N, int x_dtype, int* info) {
  if (info == nullptr || K <= 0 || N <= 0 || (x_dtype != G16_F32 && x_dtype != G16_F16)) return G16_ERR_ARG;
  int st = G16_OK;
  const DeviceInfo* dev = device_info(&st);
  if (dev == nullptr) return st;
  return skinny_plan_info(M, K, N, x_dtype, info, *dev);
}

int g16_device_status(int* status_out, int clear, void* stream) {
  if (status_out == nullptr) return G16_ERR_ARG;
  int* p = device_status_ptr();
  if (p == nullptr) return G16_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(p, 0, sizeof(int), s);
  if (e == cudaSuccess && clear) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e);
  *status_out = v;
  return G16_OK;
}

}  // extern "C"
