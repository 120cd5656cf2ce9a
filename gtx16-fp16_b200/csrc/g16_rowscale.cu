// Per-row overflow rescale before the fp16 cast of the GEMM path.
//
// Reference behaviour replaced: rowscale_body / rowscale_f32 / rowscale_f16
// (src/gtx16_fp16/kernels.py:227-250), launched by mm_t for every M > 8 call (ops.py:86-90):
//   amax = max_k |x[row,k]|
//   S[row] = 2^ceil(log2(amax / thresh)) if amax > thresh else 1
//   y[row,k] = fp16_rn(x[row,k] / S[row])
// The reference evaluates the exponent with fast-math log2f/exp2f; here ceil(log2(r)) is read
// exactly from the IEEE-754 exponent and mantissa fields of r = amax / thresh (no transcendental
// call), so S is always the smallest power of two with amax / S <= thresh.
//
// Rows up to 3072 (fp32) or 4096 (fp16) elements: one warp per row, the row held in registers
// between the |max| reduction and the scaled cast (read from HBM once, 16-byte coalesced loads,
// a persistent grid of warps walking the rows). Longer rows: one CTA per row, the second pass
// hitting L1/L2.
#include <cuda_fp16.h>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

namespace g16 {
namespace {

constexpr int kThreads = 256;

// Smallest power of two S with amax / S <= thresh (S = 1 when amax <= thresh). Returns the
// scale and writes its exact reciprocal.
__device__ __forceinline__ float pow2_row_scale(float amax, float thresh, float* inv) {
  if (!(amax > thresh)) {
    *inv = 1.f;
    return 1.f;
  }
  const float r = amax / thresh;  // exact when thresh is a power of two
  const uint32_t b = __float_as_uint(r);
  const int e = static_cast<int>((b >> 23) & 0xFFu);
  if (e == 0xFF) {  // amax = inf: the reference's exp2f(inf) gives S = inf, 1/S = 0
    *inv = 0.f;
    return __uint_as_float(0x7F800000u);
  }
  // r >= 1 here, so r is a normal number: log2(r) = (e - 127) + log2(1.mantissa).
  const int c = (e - 127) + ((b & 0x7FFFFFu) != 0u ? 1 : 0);  // ceil(log2(r)), 0 <= c <= 128
  if (c >= 128) {
    *inv = 0.f;
    return __uint_as_float(0x7F800000u);
  }
  *inv = __uint_as_float(static_cast<uint32_t>(127 - c) << 23);  // 2^-c, normal for c <= 126
  return __uint_as_float(static_cast<uint32_t>(127 + c) << 23);  // 2^c
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

// K % 8 == 0 and 16-byte aligned rows (K % 8 == 0 with a 16-byte aligned base) are required.
__global__ void __launch_bounds__(kThreads) rowscale_f32_kernel(const float* __restrict__ x, __half* __restrict__ y,
                                                                float* __restrict__ S, int K, float thresh) {
  __shared__ float red[kThreads / 32];
  const size_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * K);
  const int nv = K / 4;
  if (threadIdx.x == 0) grid_launch_dependents();  // as in rowscale_warp_kernel
  grid_dependency_wait();
  float m = 0.f;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    const float4 v = xr[i];
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  const float amax = block_max(m, red);
  float inv;
  const float sc = pow2_row_scale(amax, thresh, &inv);
  uint2* yr = reinterpret_cast<uint2*>(y + row * K);
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float4 v = xr[i];
    if (sc != 1.f) { v.x *= inv; v.y *= inv; v.z *= inv; v.w *= inv; }
    const __half2 h0 = __floats2half2_rn(v.x, v.y);
    const __half2 h1 = __floats2half2_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&h0);
    o.y = *reinterpret_cast<const uint32_t*>(&h1);
    yr[i] = o;
  }
  if (threadIdx.x == 0) S[row] = sc;
}

__global__ void __launch_bounds__(kThreads) rowscale_f16_kernel(const __half* __restrict__ x, __half* __restrict__ y,
                                                                float* __restrict__ S, int K, float thresh) {
  __shared__ float red[kThreads / 32];
  const size_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
  const int nv = K / 8;
  if (threadIdx.x == 0) grid_launch_dependents();  // as in rowscale_warp_kernel
  grid_dependency_wait();
  float m = 0.f;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    const uint4 v = xr[i];
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  const float amax = block_max(m, red);
  float inv;
  const float sc = pow2_row_scale(amax, thresh, &inv);
  uint4* yr = reinterpret_cast<uint4*>(y + row * K);
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    uint4 v = xr[i];
    if (sc != 1.f) {
      __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        h[j] = __floats2half2_rn(f.x * inv, f.y * inv);
      }
    }
    yr[i] = v;
  }
  if (threadIdx.x == 0) S[row] = sc;
}

// Warp per row: NV 16-byte vectors per lane (row length <= 32 * NV vectors); kVec elements each.
template <typename TX, int NV>
__global__ void __launch_bounds__(kThreads) rowscale_warp_kernel(const TX* __restrict__ x, __half* __restrict__ y,
                                                                 float* __restrict__ S, int M, int K, float thresh) {
  constexpr int kVec = 16 / sizeof(TX);  // elements per 16-byte vector
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (kThreads / 32);
  const int nvec = K / kVec;  // K % 8 == 0
  // Programmatic dependent launch: the next kernel (the GEMM reading y) may start its set-up now;
  // x, y and S are touched only once the preceding kernel has completed.
  if (threadIdx.x == 0) grid_launch_dependents();
  grid_dependency_wait();
  for (int row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < M; row += warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * K);
    uint4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + 32 * i;
      v[i] = j < nvec ? __ldcs(xr + j) : make_uint4(0u, 0u, 0u, 0u);  // read once: evict first
    }
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if constexpr (sizeof(TX) == 4) {
        m = fmaxf(m, fmaxf(fmaxf(fabsf(__uint_as_float(v[i].x)), fabsf(__uint_as_float(v[i].y))),
                           fmaxf(fabsf(__uint_as_float(v[i].z)), fabsf(__uint_as_float(v[i].w)))));
      } else {
        const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(h[q]);
          m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float inv;
    const float sc = pow2_row_scale(m, thresh, &inv);
    __half* yr = y + static_cast<size_t>(row) * K;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + 32 * i;
      if (j >= nvec) break;
      if constexpr (sizeof(TX) == 4) {
        float a = __uint_as_float(v[i].x), b = __uint_as_float(v[i].y), c = __uint_as_float(v[i].z),
              d = __uint_as_float(v[i].w);
        if (sc != 1.f) { a *= inv; b *= inv; c *= inv; d *= inv; }
        const __half2 h0 = __floats2half2_rn(a, b), h1 = __floats2half2_rn(c, d);
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&h0);
        o.y = *reinterpret_cast<const uint32_t*>(&h1);
        reinterpret_cast<uint2*>(yr)[j] = o;
      } else {
        uint4 o = v[i];
        if (sc != 1.f) {
          __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(h[q]);
            h[q] = __floats2half2_rn(f.x * inv, f.y * inv);
          }
        }
        reinterpret_cast<uint4*>(yr)[j] = o;
      }
    }
    if (lane == 0) S[row] = sc;
  }
}

template <typename TX, int NV>
cudaError_t launch_rowscale_warp(const void* x, uint16_t* y16, float* rscale, int M, int K, float thresh,
                                 cudaStream_t s) {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int rows_per_block = kThreads / 32;
  int blocks = (M + rows_per_block - 1) / rows_per_block;
  const int cap = sms * 8;  // 64 warps per SM, each with NV loads in flight
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rowscale_warp_kernel<TX, NV>, static_cast<const TX*>(x),
                            reinterpret_cast<__half*>(y16), rscale, M, K, thresh);
}

template <typename TX>
cudaError_t launch_rowscale_warp_any(const void* x, uint16_t* y16, float* rscale, int M, int K, float thresh,
                                     cudaStream_t s) {
  const int nvec = K / (16 / static_cast<int>(sizeof(TX)));
  if (nvec <= 32 * 4) return launch_rowscale_warp<TX, 4>(x, y16, rscale, M, K, thresh, s);
  if (nvec <= 32 * 8) return launch_rowscale_warp<TX, 8>(x, y16, rscale, M, K, thresh, s);
  if constexpr (sizeof(TX) == 2) {
    return launch_rowscale_warp<TX, 16>(x, y16, rscale, M, K, thresh, s);
  } else {
    if (nvec <= 32 * 16) return launch_rowscale_warp<TX, 16>(x, y16, rscale, M, K, thresh, s);
    return launch_rowscale_warp<TX, 24>(x, y16, rscale, M, K, thresh, s);
  }
}

// Row scale only, for a GEMM that converts fp32 activations itself: S[row] and its exact reciprocal
// Sinv[row], the same values rowscale computes; x is read once and nothing else is written (x stays
// in L2 for the GEMM when it fits). Warp per row, NV 16-byte loads in flight per lane.
template <int NV>
__global__ void __launch_bounds__(kThreads) rowamax_f32_kernel(const float* __restrict__ x, float* __restrict__ S,
                                                               float* __restrict__ Sinv, int M, int K,
                                                               float thresh) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (kThreads / 32);
  const int nvec = K / 4;  // K % 8 == 0
  for (int row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < M; row += warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * K);
    float m = 0.f;
    for (int j0 = 0; j0 < nvec; j0 += 32 * NV) {
      float4 v[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int j = j0 + lane + 32 * i;
        v[i] = j < nvec ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < NV; ++i)
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) {
      float inv;
      S[row] = pow2_row_scale(m, thresh, &inv);
      Sinv[row] = inv;
    }
  }
}

}  // namespace

int launch_rowamax(const float* x, float* rscale, float* rscale_inv, int M, int K, float thresh, cudaStream_t s) {
  if (M <= 0) return G16_OK;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e);
  const int rows_per_block = kThreads / 32;
  int blocks = (M + rows_per_block - 1) / rows_per_block;
  if (blocks > sms * 8) blocks = sms * 8;
  rowamax_f32_kernel<8><<<blocks, kThreads, 0, s>>>(x, rscale, rscale_inv, M, K, thresh);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

int launch_rowscale(const void* x, int x_dtype, uint16_t* y16, float* rscale, int M, int K, float thresh,
                    cudaStream_t s) {
  if (M <= 0) return G16_OK;
  const int nvec = K / (x_dtype == G16_F32 ? 4 : 8);
  if (nvec <= 32 * (x_dtype == G16_F32 ? 24 : 16)) {  // the row fits a warp's registers
    const cudaError_t e = x_dtype == G16_F32 ? launch_rowscale_warp_any<float>(x, y16, rscale, M, K, thresh, s)
                                             : launch_rowscale_warp_any<__half>(x, y16, rscale, M, K, thresh, s);
    if (e != cudaSuccess) return cuda_fail(e);
    note_launch();
    return G16_OK;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(M), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      x_dtype == G16_F32
          ? cudaLaunchKernelEx(&cfg, rowscale_f32_kernel, static_cast<const float*>(x), reinterpret_cast<__half*>(y16),
                               rscale, K, thresh)
          : cudaLaunchKernelEx(&cfg, rowscale_f16_kernel, static_cast<const __half*>(x),
                               reinterpret_cast<__half*>(y16), rscale, K, thresh);
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

}  // namespace g16
