// TEST INFRASTRUCTURE ONLY - the reference's own CUDA kernels as a GPU-side checker.
//
// oracle/build_ref.py extracts the CUDA C source string of the reference (_SRC in
// src/gtx16_fp16/kernels.py:19-251) into a temporary file at build time and compiles this file
// with -DREF_KERNELS="<that file>" and the reference's NVRTC options (--use_fast_math,
// -std=c++17; kernels.py:352-353) for sm_100a into oracle/_ref/libg16ref_gpu.so. The reference
// source is never stored in this repository; only the built library lands in oracle/_ref/ (ignored
// by git, shipped to the GPU box with the snapshot).
//
// The launchers below restate the reference's host dispatch (src/gtx16_fp16/ops.py:45-108):
// grid shapes, skinny_config, split-K ksplit/kchunk, the zero/bias prefill and the fp16 cast.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include REF_KERNELS

namespace {

__global__ void f32_to_f16_kernel(const float* in, __half* out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(in[i]);  // torch's .to(float16) rounds to nearest even
}

__global__ void prefill_kernel(float* out, const float* bias, int M, int N) {
  const size_t total = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
    out[i] = bias ? bias[i % N] : 0.f;  // _prefilled, ops.py:54-62
}

int err() { return (int)cudaGetLastError(); }

}  // namespace

extern "C" {

// skinny_config (ops.py:45-51)
int g16ref_skinny_config(int N, int K, int sms, int* nbx, int* ksplit) {
  *nbx = (N + 255) / 256;
  int ks = (4 * sms + *nbx - 1) / *nbx;
  if (K / 64 < ks) ks = K / 64;
  if (ks < 1) ks = 1;
  const int kchunk = ((K + ks - 1) / ks + 7) / 8 * 8;
  *ksplit = (K + kchunk - 1) / kchunk;
  return kchunk;
}

int g16ref_rowscale(const void* x, int x_is_f16, __half* y, float* S, int M, int K, float thresh, cudaStream_t s) {
  if (x_is_f16)
    rowscale_f16<<<M, 256, 0, s>>>((const __half*)x, y, S, K, thresh);
  else
    rowscale_f32<<<M, 256, 0, s>>>((const float*)x, y, S, K, thresh);
  return err();
}

int g16ref_hgemm(const __half* a, const __half* b, void* out, int out_is_f16, const float* bias, const float* rscale,
                 int M, int N, int K, cudaStream_t s) {
  const dim3 grid((N + 127) / 128, (M + 127) / 128, 1);
  if (out_is_f16)
    hgemm_f16out<<<grid, 256, 0, s>>>(a, b, (__half*)out, bias, rscale, M, N, K);
  else
    hgemm_f32out<<<grid, 256, 0, s>>>(a, b, (float*)out, bias, rscale, M, N, K);
  return err();
}

// C (fp32) must already hold the prefill.
int g16ref_hgemm_splitk(const __half* a, const __half* b, float* C, const float* rscale, int M, int N, int K,
                        int kchunk, cudaStream_t s) {
  const int ksplit = (K + kchunk - 1) / kchunk;
  const dim3 grid((N + 127) / 128, (M + 127) / 128, ksplit);
  hgemm_splitk<<<grid, 256, 0, s>>>(a, b, C, rscale, M, N, K, kchunk);
  return err();
}

// C (fp32) must be zeroed.
int g16ref_skinny(const void* x, int x_is_f16, const __half* w, float* C, const float* bias, int M, int N, int K,
                  int sms, cudaStream_t s) {
  int nbx, ksplit;
  const int kchunk = g16ref_skinny_config(N, K, sms, &nbx, &ksplit);
  const dim3 grid(nbx, ksplit, 1);
  if (x_is_f16)
    skinny_f16in<<<grid, 256, 0, s>>>((const __half*)x, w, C, bias, M, N, K, kchunk);
  else
    skinny_f32in<<<grid, 256, 0, s>>>((const float*)x, w, C, bias, M, N, K, kchunk);
  return err();
}

// Scratch the reference allocates per call (ops.py:79,87-88,98): bytes for x16 + rscale + fp32 C.
size_t g16ref_mm_t_scratch_bytes(int M, int K, int N) {
  return (size_t)M * K * 2 + 256 + (size_t)M * 4 + 256 + (size_t)M * N * 4;
}

// mm_t (ops.py:65-108) with the reference's kernels. `scratch` must hold g16ref_mm_t_scratch_bytes.
int g16ref_mm_t(const void* x, int x_is_f16, const __half* w, const float* bias, void* out, int out_is_f16, int M,
                int K, int N, int sms, void* scratch, cudaStream_t s) {
  char* p = (char*)scratch;
  __half* x16 = (__half*)p;
  p += ((size_t)M * K * 2 + 255) / 256 * 256;
  float* rscale = (float*)p;
  p += ((size_t)M * 4 + 255) / 256 * 256;
  float* c32 = (float*)p;
  const size_t n = (size_t)M * N;
  if (M <= 8) {
    float* C = out_is_f16 ? c32 : (float*)out;
    cudaMemsetAsync(C, 0, n * 4, s);  // torch.zeros, ops.py:79
    int e = g16ref_skinny(x, x_is_f16, w, C, bias, M, N, K, sms, s);
    if (e) return e;
    if (out_is_f16) f32_to_f16_kernel<<<256, 256, 0, s>>>(C, (__half*)out, n);
    return err();
  }
  int e = g16ref_rowscale(x, x_is_f16, x16, rscale, M, K, 1024.0f, s);
  if (e) return e;
  const int tiles = ((N + 127) / 128) * ((M + 127) / 128);
  if (tiles < 2 * sms && K >= 256) {
    int ksplit = (2 * sms + tiles - 1) / tiles;
    if (K / 128 < ksplit) ksplit = K / 128;
    const int kchunk = ((K + ksplit - 1) / ksplit + 15) / 16 * 16;
    float* C = out_is_f16 ? c32 : (float*)out;
    prefill_kernel<<<256, 256, 0, s>>>(C, bias, M, N);
    e = g16ref_hgemm_splitk(x16, w, C, rscale, M, N, K, kchunk, s);
    if (e) return e;
    if (out_is_f16) f32_to_f16_kernel<<<256, 256, 0, s>>>(C, (__half*)out, n);
    return err();
  }
  return g16ref_hgemm(x16, w, out, out_is_f16, bias, rscale, M, N, K, s);
}

}  // extern "C"
