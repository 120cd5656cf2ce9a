// Skinny GEMM for M <= 8 (token-by-token decode): out[M,N] = x[M,K] @ w[K,N] + bias[N].
//
// Reference behaviour replaced: skinny_body / skinny_f32in / skinny_f16in
// (src/gtx16_fp16/kernels.py:163-219) launched by mm_t (src/gtx16_fp16/ops.py:78-84). The reference
// splits K over gridDim.y and adds partial sums into a zeroed output with fp32 atomics, then casts
// to fp16 with a separate kernel. Here the kernel is built for HBM streaming:
//   * the weight matrix (2*K*N bytes, the dominant traffic) is read exactly once by TMA: a producer
//     warp keeps a 12-stage ring of [16 rows x 256 columns] boxes (8 KiB each) in flight from the
//     first cycle, ~96 KiB per SM, enough to cover HBM latency at full bandwidth;
//   * 8 consumer warps multiply the boxes against x (staged once in shared memory as fp32) with
//     packed FFMA2, fp32 accumulation;
//   * K is split across the CTAs of one thread-block cluster (up to 16) that share a 256-column
//     strip; partial sums are reduced in a fixed order inside the CTA (shared memory) and across
//     the cluster (distributed shared memory), so the result is bitwise reproducible and needs no
//     zero-filled output or atomics; bias add and the fp16 cast are fused.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <atomic>
#include <mutex>
#include <unordered_map>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

namespace g16 {
namespace {

constexpr int kStrip = 256;                  // output columns per cluster (one TMA box row: 512 B)
constexpr int kBoxRows = 16;                 // weight rows per pipeline stage
constexpr int kStages = 12;
constexpr int kStageBytes = kBoxRows * kStrip * 2;  // 8 KiB
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;    // + one producer warp
constexpr int kRowLanes = kConsumerWarps;    // warp w handles rows w, w+8 of every stage
constexpr int kPieceMax = 2048;              // rows of x staged in shared memory at a time
constexpr int kMaxCluster = 16;
constexpr int kStageBatch = 2;               // x-staging k-batches per thread (x M loads in flight)

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

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

struct SkinnyArgs {
  const void* x;
  const float* bias;
  void* out;
  int* status;
  int K, N, kchunk, piece;
};

// grid = (C, strips); cluster = (C, 1, 1); blockIdx.x is the CTA's rank in its cluster and selects
// the K chunk [rank*kchunk, min(K, (rank+1)*kchunk)).
// Shared memory: [ring: kStages x 8 KiB | xs: piece x MP fp32 | part: M x kStrip fp32 | barriers].
template <int M, typename TX, bool OUT_F16>
__global__ void __launch_bounds__(kThreads, 1)
skinny_kernel(const __grid_constant__ CUtensorMap tmap_w, const SkinnyArgs args) {
  constexpr int MP = MPad<M>::v;
  extern __shared__ uint8_t smem_raw[];
  // Align by pointer arithmetic on the __shared__ array (an integer round trip would turn
  // every access into a generic-address load).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  float* xs = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  float* part = xs + args.piece * MP;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(part + M * kStrip);
  uint64_t* empty_bar = full_bar + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty_bar + kStages);
  float* red = reinterpret_cast<float*>(ring);  // [kRowLanes][M][kStrip], after the main loop
  // Self-check: the layout must end inside the launch's dynamic shared memory (uniform for the
  // whole grid, so every CTA returns before any barrier or shared-memory access).
  const uint32_t layout_end = static_cast<uint32_t>(reinterpret_cast<const volatile uint8_t*>(abort_flag + 1) - smem_raw);
  if (layout_end > dynamic_smem_bytes()) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicExch(args.status, G16_ERR_ARG);
    return;
  }

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rank = blockIdx.x;
  const int csize = gridDim.x;
  const int n0 = blockIdx.y * kStrip;
  const int kb = rank * args.kchunk;
  const int ke = min(args.K, kb + args.kchunk);
  const int nrows = max(0, ke - kb);
  const int nstages = (nrows + kBoxRows - 1) / kBoxRows;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer: stream this CTA's weight rows through the ring ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      uint32_t phase = 0;
      int stage = 0;
      bool armed[kStages];
      uint32_t armed_phase[kStages];
      for (int s = 0; s < kStages; ++s) { armed[s] = false; armed_phase[s] = 0; }
      bool ok = true;
      for (int t = 0; t < nstages; ++t) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
        armed[stage] = true;
        armed_phase[stage] = phase;
        tma_load_2d(ring + stage * kStageBytes, &tmap_w, &full_bar[stage], n0, kb + t * kBoxRows);
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
        for (int s = 0; s < kStages; ++s)
          if (armed[s]) mbar_wait(&full_bar[s], armed_phase[s], nullptr);
      }
    }
  } else {
    // ---------------- consumers ----------------
    const int cg = lane;             // 8-column group
    const int rl = warp;             // row lane
    const TX* x = static_cast<const TX*>(args.x);
    float2 acc[M][4];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[m][j] = make_float2(0.f, 0.f);

    // Every consumer warp executes the same sequence of named barriers whether or not a wait
    // expired (a hardware barrier cannot time out); after an expiry the remaining stages are
    // skipped without waiting.
    uint32_t phase = 0;
    int stage = 0;
    int t = 0;
    bool ok = true;
    for (int p0 = 0; p0 < nrows; p0 += args.piece) {
      const int plen = min(args.piece, nrows - p0);
      if (p0 > 0) consumer_sync();  // everyone is done with the previous piece of x
      // Stage x[:, piece] transposed to [k][MP] fp32 (rows m >= M are zero). The row index is a
      // compile-time loop, so there is no per-element division, and each thread keeps
      // M x kStageBatch loads in flight: one memory latency per batch.
      for (int k0 = tid; k0 < plen; k0 += kConsumers * kStageBatch) {
        float v[M][kStageBatch];
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
          for (int u = 0; u < kStageBatch; ++u) {
            const int k = k0 + u * kConsumers;
            v[m][u] = k < plen ? to_f32(x[static_cast<size_t>(m) * args.K + kb + p0 + k]) : 0.f;
          }
#pragma unroll
        for (int u = 0; u < kStageBatch; ++u) {
          const int k = k0 + u * kConsumers;
          if (k < plen) {
#pragma unroll
            for (int m = 0; m < MP; ++m) xs[k * MP + m] = m < M ? v[m < M ? m : 0][u] : 0.f;
          }
        }
      }
      consumer_sync();
      const int t_end = (p0 + plen + kBoxRows - 1) / kBoxRows;
      for (; t < t_end; ++t) {
        if (!ok) continue;
        bool got = mbar_wait(&full_bar[stage], phase, abort_flag);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          ok = false;
          if (lane == 0) { *abort_flag = 1; atomicExch(args.status, G16_ERR_TIMEOUT); }
          continue;
        }
        const uint8_t* sbuf = ring + stage * kStageBytes;
#pragma unroll
        for (int rr = 0; rr < kBoxRows / kRowLanes; ++rr) {
          const int r = rl + rr * kRowLanes;      // row inside the box
          const int krow = t * kBoxRows + r;      // row inside this CTA's chunk
          if (krow < p0 + plen && krow >= p0) {
            const uint4 wv = *reinterpret_cast<const uint4*>(sbuf + r * (kStrip * 2) + cg * 16);
            fma_row<M>(acc, wv, xs + (krow - p0) * MP);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[stage]);
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
    consumer_sync();  // ring no longer read: reuse it for the row-lane reduction
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float4* dst = reinterpret_cast<float4*>(red + (rl * M + m) * kStrip + cg * 8);
      dst[0] = make_float4(acc[m][0].x, acc[m][0].y, acc[m][1].x, acc[m][1].y);
      dst[1] = make_float4(acc[m][2].x, acc[m][2].y, acc[m][3].x, acc[m][3].y);
    }
    consumer_sync();
    for (int i = tid; i < M * kStrip; i += kConsumers) {
      const int m = i / kStrip, c = i - m * kStrip;
      float s = 0.f;
#pragma unroll
      for (int r = 0; r < kRowLanes; ++r) s += red[(r * M + m) * kStrip + c];
      part[i] = s;
    }
  }

  // Reduce across the cluster in rank order; CTA `rank` finalises a contiguous share of outputs.
  cluster_sync();
  if (warp < kConsumerWarps) {
    const int total = M * kStrip;
    const int share = (total + csize - 1) / csize;
    const int i0 = rank * share;
    const int i1 = min(total, i0 + share);
    const uint32_t part_addr = smem_u32(part);
    for (int i = i0 + tid; i < i1; i += kConsumers) {
      const int m = i / kStrip, c = i - m * kStrip;
      const int n = n0 + c;
      if (n < args.N) {
        // all remote loads in flight first, then the fixed-order sum
        float pv[kMaxCluster];
#pragma unroll
        for (int q = 0; q < kMaxCluster; ++q)
          pv[q] = q < csize ? ld_cluster_f32(map_cluster(part_addr + 4u * i, q)) : 0.f;
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < kMaxCluster; ++q)
          if (q < csize) s += pv[q];
        if (args.bias != nullptr) s += args.bias[n];
        if constexpr (OUT_F16) {
          reinterpret_cast<__half*>(args.out)[static_cast<size_t>(m) * args.N + n] = __float2half_rn(s);
        } else {
          reinterpret_cast<float*>(args.out)[static_cast<size_t>(m) * args.N + n] = s;
        }
      }
    }
  }
  cluster_sync();  // keep this CTA's `part` alive until every peer has read it
}

struct SkinnyPlan {
  int csize, strips, kchunk, piece;
  size_t smem_bytes;
};

size_t skinny_smem_bytes(int M, int piece) {
  const int mp = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  return 1024 + static_cast<size_t>(kStages) * kStageBytes + static_cast<size_t>(piece) * mp * 4 +
         static_cast<size_t>(M) * kStrip * 4 + 2 * kStages * 8 + 16;
}

SkinnyPlan plan_skinny(int M, int K, int N, int sm_count) {
  SkinnyPlan p{};
  p.strips = (N + kStrip - 1) / kStrip;
  // One CTA per SM: split K across as many cluster ranks as fill the GPU (at most 16), keeping
  // at least four boxes of rows per CTA.
  int c = sm_count / p.strips;
  if (c < 1) c = 1;
  if (c > kMaxCluster) c = kMaxCluster;
  const int max_by_k = K / (4 * kBoxRows) > 0 ? K / (4 * kBoxRows) : 1;
  if (c > max_by_k) c = max_by_k;
  int kchunk = (K + c - 1) / c;
  kchunk = (kchunk + 7) / 8 * 8;
  if (kchunk <= 0) kchunk = 8;
  c = (K + kchunk - 1) / kchunk;
  if (c < 1) c = 1;
  p.csize = c;
  p.kchunk = kchunk;
  p.piece = kchunk < kPieceMax ? kchunk : kPieceMax;
  p.smem_bytes = skinny_smem_bytes(M, p.piece);
  return p;
}

template <typename F>
cudaError_t ensure_attrs(F* kern, std::atomic<uint64_t>& done, int smem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Largest dynamic shared memory any skinny launch requests (set once per kernel and device).
constexpr int kSmemAttrBytes = 1024 + kStages * kStageBytes + kPieceMax * 8 * 4 + 8 * kStrip * 4 + 2 * kStages * 8 + 16;

cudaLaunchConfig_t make_cfg(const SkinnyPlan& p, cudaStream_t s, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.csize, p.strips, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// The plan for (K, N) on this device: the largest cluster size whose clusters are all resident at
// once (cudaOccupancyMaxActiveClusters), so the grid runs in a single wave. Cached per instantiation.
template <typename F>
int plan_for(F* kern, int M, int K, int N, const DeviceInfo& dev, SkinnyPlan* out) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, SkinnyPlan> cache;
  int devid = 0;
  cudaError_t e = cudaGetDevice(&devid);
  if (e != cudaSuccess) return cuda_fail(e);
  // Every instantiation shares this cache (same kernel function type), and the layout depends on M.
  const uint64_t key = (static_cast<uint64_t>(devid) << 58) ^ (static_cast<uint64_t>(M) << 54) ^
                       (static_cast<uint64_t>(K) << 27) ^ static_cast<uint64_t>(N);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return G16_OK;
    }
  }
  SkinnyPlan p = plan_skinny(M, K, N, dev.sm_count);
  while (true) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(p, nullptr, attr);
    int active = 0;
    e = cudaOccupancyMaxActiveClusters(&active, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e);
    if (active >= p.strips || p.csize == 1) break;
    // Shrink the cluster until every cluster fits at once.
    const int c = p.csize - 1;
    p = plan_skinny(M, K, N, c * p.strips);
    if (p.csize > c) p = plan_skinny(M, K, N, c * p.strips);
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = p;
  *out = p;
  return G16_OK;
}

template <int M, typename TX, bool OUT_F16>
int launch_skinny_t(const void* x, const uint16_t* w, const float* bias, void* out, int K, int N, cudaStream_t s,
                    const DeviceInfo& dev) {
  static std::atomic<uint64_t> attr_done{0};
  auto kern = skinny_kernel<M, TX, OUT_F16>;
  cudaError_t e = ensure_attrs(kern, attr_done, kSmemAttrBytes);
  if (e != cudaSuccess) return cuda_fail(e);
  SkinnyPlan p;
  int st0 = plan_for(kern, M, K, N, dev, &p);
  if (st0 != G16_OK) return st0;
  if (p.smem_bytes < skinny_smem_bytes(M, p.piece) || p.smem_bytes > static_cast<size_t>(kSmemAttrBytes))
    return G16_ERR_ARG;
  CUtensorMap tmap;
  int st = make_tmap_2d(&tmap, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                        kBoxRows, kStrip, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != G16_OK) return st;
  SkinnyArgs a{};
  a.x = x;
  a.bias = bias;
  a.out = out;
  a.status = device_status_ptr();
  if (a.status == nullptr) return G16_ERR_CUDA;
  a.K = K;
  a.N = N;
  a.kchunk = p.kchunk;
  a.piece = p.piece;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(p, s, attr);
  e = cudaLaunchKernelEx(&cfg, kern, tmap, a);
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
