// Skinny GEMM for M <= 8 (token-by-token decode): out[M,N] = x[M,K] @ w[K,N] + bias[N].
//
// Reference behaviour replaced: skinny_body / skinny_f32in / skinny_f16in
// (src/gtx16_fp16/kernels.py:163-219) launched by mm_t (src/gtx16_fp16/ops.py:78-84). The reference
// splits K over gridDim.y and adds partial sums into a zeroed output with fp32 atomics, then casts
// to fp16 with a separate kernel. Here:
//   * the weight matrix is streamed from HBM exactly once with 128-bit non-allocating loads, eight
//     loads in flight per thread (the kernel is HBM-bound: 2*K*N bytes dominate);
//   * arithmetic is fp32 FMA on (x, w) pairs using sm_100a packed FFMA2;
//   * K is split across the CTAs of one thread-block cluster (<= 8) that share a 128-column strip;
//     partial sums are reduced in a fixed order inside the CTA (shared memory) and then across
//     the cluster through distributed shared memory, so the result is bitwise reproducible and no
//     zero-filled output or atomic is needed; bias add and the fp16 cast are fused.
#include <cuda_fp16.h>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

namespace g16 {
namespace {

constexpr int kColGroups = 16;                 // 8 fp16 columns (16 bytes) per group
constexpr int kRowLanes = 16;                  // rows handled in parallel inside a CTA
constexpr int kStrip = kColGroups * 8;         // 128 output columns per cluster
constexpr int kThreads = kColGroups * kRowLanes;  // 256
constexpr int kUnroll = 8;                     // 128-bit weight loads in flight per thread
constexpr int kPieceMax = 2048;                // rows of x staged in shared memory at a time

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <int M>
struct MPad {
  static constexpr int v = (M <= 1) ? 1 : (M <= 2) ? 2 : (M <= 4) ? 4 : 8;
};

// acc[m][j] += x[m] * w[j] for the 8 columns of one 16-byte weight vector.
template <int M>
__device__ __forceinline__ void fma_row(float2 (&acc)[M][4], const uint4& wv, const float* __restrict__ xk) {
  const __half2* wh = reinterpret_cast<const __half2*>(&wv);
  float2 wf[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) wf[j] = __half22float2(wh[j]);
  constexpr int MP = MPad<M>::v;
  float xr[MP];
  if constexpr (MP >= 4) {
#pragma unroll
    for (int q = 0; q < MP / 4; ++q) {
      const float4 t = reinterpret_cast<const float4*>(xk)[q];
      xr[4 * q + 0] = t.x; xr[4 * q + 1] = t.y; xr[4 * q + 2] = t.z; xr[4 * q + 3] = t.w;
    }
  } else if constexpr (MP == 2) {
    const float2 t = reinterpret_cast<const float2*>(xk)[0];
    xr[0] = t.x; xr[1] = t.y;
  } else {
    xr[0] = xk[0];
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const float2 xm = make_float2(xr[m], xr[m]);
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[m][j] = ffma2(xm, wf[j], acc[m][j]);
  }
}

// grid = (C, strips); cluster = (C, 1, 1); blockIdx.x is the CTA's rank inside its cluster and
// selects the K chunk [rank*kchunk, min(K, (rank+1)*kchunk)).
template <int M, typename TX, bool OUT_F16>
__global__ void __launch_bounds__(kThreads, 2)
skinny_kernel(const TX* __restrict__ x, const __half* __restrict__ w, const float* __restrict__ bias,
              void* __restrict__ out, int K, int N, int kchunk, int piece, int red_floats) {
  constexpr int MP = MPad<M>::v;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                  // [piece][MP] fp32, during the main loop
  float* red = smem;                 // [kRowLanes][M][kStrip], after the main loop (aliases xs)
  float* part = smem + red_floats;   // [M][kStrip]: this CTA's partial, read by the whole cluster

  const int tid = threadIdx.x;
  const int cg = tid % kColGroups;
  const int rl = tid / kColGroups;
  const int rank = blockIdx.x;
  const int csize = gridDim.x;
  const int n0 = blockIdx.y * kStrip;
  const int col = n0 + cg * 8;
  const bool col_ok = col < N;  // N % 8 == 0: a group of 8 columns is entirely in or out
  const int kb = rank * kchunk;
  const int ke = min(K, kb + kchunk);

  float2 acc[M][4];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[m][j] = make_float2(0.f, 0.f);

  for (int p0 = kb; p0 < ke; p0 += piece) {
    const int plen = min(piece, ke - p0);
    // Stage x[:, p0 : p0+plen] as fp32 [k][MP] (rows m >= M are zero).
    for (int i = tid; i < plen * MP; i += kThreads) {
      const int m = i / plen, k = i - m * plen;
      xs[k * MP + m] = (m < M) ? to_f32(x[static_cast<size_t>(m) * K + p0 + k]) : 0.f;
    }
    __syncthreads();
    if (col_ok) {
      const __half* wp = w + static_cast<size_t>(p0 + rl) * N + col;
      const size_t step = static_cast<size_t>(kRowLanes) * N;
      int k = rl;
      for (; k + (kUnroll - 1) * kRowLanes < plen; k += kUnroll * kRowLanes) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = ldg_stream(wp + u * step);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) fma_row<M>(acc, v[u], xs + (k + u * kRowLanes) * MP);
        wp += kUnroll * step;
      }
      for (; k < plen; k += kRowLanes) {
        const uint4 v = ldg_stream(wp);
        fma_row<M>(acc, v, xs + k * MP);
        wp += step;
      }
    }
    __syncthreads();
  }

  // Reduce the 16 row lanes of this CTA in a fixed order.
#pragma unroll
  for (int m = 0; m < M; ++m) {
    float4* dst = reinterpret_cast<float4*>(red + (rl * M + m) * kStrip + cg * 8);
    dst[0] = make_float4(acc[m][0].x, acc[m][0].y, acc[m][1].x, acc[m][1].y);
    dst[1] = make_float4(acc[m][2].x, acc[m][2].y, acc[m][3].x, acc[m][3].y);
  }
  __syncthreads();
  for (int i = tid; i < M * kStrip; i += kThreads) {
    const int m = i / kStrip, c = i - m * kStrip;
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kRowLanes; ++r) s += red[(r * M + m) * kStrip + c];
    part[i] = s;
  }

  // Reduce across the cluster in rank order; CTA `rank` finalises a contiguous share of outputs.
  cluster_sync();
  const int total = M * kStrip;
  const int share = (total + csize - 1) / csize;
  const int i0 = rank * share;
  const int i1 = min(total, i0 + share);
  const uint32_t part_addr = smem_u32(part);
  for (int i = i0 + tid; i < i1; i += kThreads) {
    const int m = i / kStrip, c = i - m * kStrip;
    const int n = n0 + c;
    float s = 0.f;
    for (int q = 0; q < csize; ++q) s += ld_cluster_f32(map_cluster(part_addr + 4u * i, q));
    if (n < N) {
      if (bias != nullptr) s += bias[n];
      if constexpr (OUT_F16) {
        reinterpret_cast<__half*>(out)[static_cast<size_t>(m) * N + n] = __float2half_rn(s);
      } else {
        reinterpret_cast<float*>(out)[static_cast<size_t>(m) * N + n] = s;
      }
    }
  }
  cluster_sync();  // keep this CTA's `part` alive until every peer has read it
}

struct SkinnyPlan {
  int csize, strips, kchunk, piece;
  size_t smem_bytes;
  int red_floats;
};

SkinnyPlan plan_skinny(int M, int K, int N, int sm_count) {
  SkinnyPlan p{};
  p.strips = (N + kStrip - 1) / kStrip;
  // Aim for about two CTAs per SM; every CTA should still stream a useful number of rows.
  int c = (2 * sm_count + p.strips - 1) / p.strips;
  c = c < 1 ? 1 : (c > 8 ? 8 : c);
  const int max_by_k = K / 64 > 0 ? K / 64 : 1;
  if (c > max_by_k) c = max_by_k;
  int kchunk = (K + c - 1) / c;
  kchunk = (kchunk + kRowLanes - 1) / kRowLanes * kRowLanes;
  if (kchunk <= 0) kchunk = kRowLanes;
  c = (K + kchunk - 1) / kchunk;
  if (c < 1) c = 1;
  p.csize = c;
  p.kchunk = kchunk;
  p.piece = kchunk < kPieceMax ? kchunk : kPieceMax;
  const int mp = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  const int xs_floats = p.piece * mp;
  const int red_floats = kRowLanes * M * kStrip;
  p.red_floats = xs_floats > red_floats ? xs_floats : red_floats;
  p.smem_bytes = static_cast<size_t>(p.red_floats + M * kStrip) * sizeof(float);
  return p;
}

template <int M, typename TX, bool OUT_F16>
int launch_skinny_t(const void* x, const uint16_t* w, const float* bias, void* out, int K, int N, cudaStream_t s,
                    const DeviceInfo& dev) {
  const SkinnyPlan p = plan_skinny(M, K, N, dev.sm_count);
  auto kern = skinny_kernel<M, TX, OUT_F16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(p.smem_bytes));
  if (e != cudaSuccess) return cuda_fail(e);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.csize, p.strips, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, static_cast<const TX*>(x), reinterpret_cast<const __half*>(w), bias, out, K, N,
                         p.kchunk, p.piece, p.red_floats);
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

template <int M>
int dispatch_types(const void* x, int x_dtype, const uint16_t* w, const float* bias, void* out, int out_dtype, int K,
                   int N, cudaStream_t s, const DeviceInfo& dev) {
  if (x_dtype == G16_F32) {
    return out_dtype == G16_F16 ? launch_skinny_t<M, float, true>(x, w, bias, out, K, N, s, dev)
                                : launch_skinny_t<M, float, false>(x, w, bias, out, K, N, s, dev);
  }
  return out_dtype == G16_F16 ? launch_skinny_t<M, __half, true>(x, w, bias, out, K, N, s, dev)
                              : launch_skinny_t<M, __half, false>(x, w, bias, out, K, N, s, dev);
}

}  // namespace

int launch_skinny(const void* x, int x_dtype, const uint16_t* w, const float* bias, void* out, int out_dtype, int M,
                  int K, int N, cudaStream_t s, const DeviceInfo& dev) {
  switch (M) {
    case 1: return dispatch_types<1>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    case 2: return dispatch_types<2>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    case 3: return dispatch_types<3>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    case 4: return dispatch_types<4>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    case 5: return dispatch_types<5>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    case 6: return dispatch_types<6>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    case 7: return dispatch_types<7>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    case 8: return dispatch_types<8>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev);
    default: return G16_ERR_ARG;
  }
}

}  // namespace g16
