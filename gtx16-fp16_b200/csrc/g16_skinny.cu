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

#include <algorithm>
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

__device__ __forceinline__ void consumer_sync() { named_bar_sync(1, kConsumers); }

struct SkinnyArgs {
  const void* x;
  const float* bias;
  void* out;
  int* status;
  int K, N, kchunk, piece;
  int stages;  // tensor-core variant: weight ring depth
  int rows;    // tensor-core variant: weight rows per stage (32, 64 or 128)
  int act;     // epilogue activation (G16_ACT_*)
};

// grid = (C, strips); cluster = (C, 1, 1); blockIdx.x is the CTA's rank in its cluster and selects
// the K chunk [rank*kchunk, min(K, (rank+1)*kchunk)).
// Shared memory: [ring: kStages x 8 KiB | xs: piece x MP fp32 | part: M x kStrip fp32 | barriers].
template <int M, typename TX, bool OUT_F16>
__global__ void __launch_bounds__(kThreads, 1)
skinny_fma_kernel(const __grid_constant__ CUtensorMap tmap_w, const SkinnyArgs args) {
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
        s = apply_act(s, args.act);
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
  int active_first = -1;  // resident clusters at the first cluster size tried
  int active = -1;        // resident clusters at the chosen cluster size
  int tc = 0;             // 1: tensor-core variant
  int stages = 0;         // tensor-core variant: weight ring depth
  int rows = 0;           // tensor-core variant: weight rows per stage
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
  // Carve the whole unified L1 as shared memory, so two CTAs (and cluster peers) fit per SM.
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
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
int launch_skinny_fma_t(const void* x, const uint16_t* w, const float* bias, void* out, int K, int N, cudaStream_t s,
                        const DeviceInfo& dev, int act) {
  static std::atomic<uint64_t> attr_done{0};
  auto kern = skinny_fma_kernel<M, TX, OUT_F16>;
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
  a.act = act;
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

// =============================================================================================
// Tensor-core variant (used whenever the CTA's K chunk fits: kchunk <= kTcMaxChunk).
//
// The fp32 FMA work of M <= 8 rows (M FMAs per weight element) is moved to the tensor core without
// losing fp32 accuracy: each CTA scales its chunk of every x row by a power of two s (so the row's
// |max| lands in [2^14, 2^15)), splits x*s = hi + lo into two fp16 values (hi = fp16(x*s),
// lo = fp16(x*s - hi); hi + lo carries 22 significant bits, products with fp16 weights are exact,
// sums are fp32), and computes out^T[n][m'] = sum_k W[k][n] * xhl[m'][k] with
// tcgen05.mma kind::f16, M=128 (weight columns), N=16 (m' < 8: hi rows, m' >= 8: lo rows), K=16.
// W is the MN-major A operand, streamed by TMA in 128-byte swizzled [32 rows x 64 columns] boxes
// (the layout the GEMM uses for its B operand); xhl is a K-major B operand built in shared memory.
// The partial for (m, n) is (D[n][m] + D[n][m+8]) / s. Work per 32-row stage is two MMAs whatever
// M is.
//
// Reduction over the K chunks: rank r of the cluster finalises columns [r*slice, (r+1)*slice) of
// the strip (slice = ceil(128 / csize)). Every rank pushes its partials for those columns into the
// owner's shared memory with st.async, which completes bytes on the owner's mbarrier; the owner
// sums the csize partials in rank order (deterministic) and stores. No cluster-wide barrier sits
// on this path; one split arrive/wait pair at the start publishes the barriers' initialisation.
//
// A kernel that allocates tensor memory runs one CTA per SM, and a cluster must fit inside one
// GPC, so strips are 128 columns wide (4096 columns -> 32 clusters of 4 CTAs on 148 SMs) rather
// than the FMA variant's 256. Shared memory left over by x is all weight ring (up to 24 stages,
// 192 KiB), and the producer fills the ring before the CTA-wide barrier, so the weight stream
// starts while x is still being prepared.
// =============================================================================================
constexpr int kTcStrip = 128;                           // output columns per cluster (UMMA M)
constexpr int kTcMinRows = 32;                          // stage heights: 128, 64 or 32 weight rows
constexpr int kTcMaxRows = 128;
constexpr int kTcMaxStages = 24;                        // layout limit of the ring depth
constexpr int kTcBoxCols = 64;                          // one 128-byte swizzle row of fp16
__host__ __device__ constexpr int tc_box_bytes(int rows) { return rows * kTcBoxCols * 2; }  // [rows x 64]
__host__ __device__ constexpr int tc_stage_bytes(int rows) { return 2 * tc_box_bytes(rows); }  // [rows x 128]
constexpr int kTcThreads = 192;  // warps 0-3: x prep + epilogue, warp 4: TMEM + MMA, warp 5: TMA
constexpr int kTcXRows = 16;     // UMMA N: x_hi rows 0..7, x_lo rows 8..15
// x_hi / x_lo, the K-major B operand (128-byte swizzle), per 64-wide K block of the chunk:
//   M <= 4 ("packed"): one 8-row group [hi rows 0..M-1 | lo rows M..2M-1 | zero rows] (1 KiB); the
//     operand's second 8-row group is a single shared 1 KiB zero block after the last K block,
//     reached through a per-K-block stride-byte-offset (SBO) in the descriptor;
//   M > 4: hi rows 0..7 then lo rows 8..15, zero rows past M (2 KiB).
template <int M>
struct XhlLayout {
  static constexpr bool kPacked = M <= 4;
  static constexpr int kBlockBytes = kPacked ? 1024 : 2048;
  static constexpr int kLoRow = kPacked ? M : 8;  // first lo row = accumulator column of lo(x[0])
};
__host__ __device__ constexpr int tc_xhl_bytes(int M, int nkb) { return M <= 4 ? (nkb + 1) * 1024 : nkb * 2048; }
constexpr int kTcMaxChunk = 2048;                       // xhl <= 64 KiB of shared memory
constexpr int kTcRedBytes = (kTcStrip + kMaxCluster) * 8 * 4;  // pushed partials: csize x slice x MP fp32
constexpr int kTcSmemLimit = 227 * 1024;
// Consecutive 16-wide K steps go round-robin to kTcAcc independent [128 x 16] accumulators: a
// dependent chain of N=16 MMAs into one accumulator runs at the MMA's latency (~0.1 us each),
// far slower than the weight stream; independent ones overlap. Summed in fixed order at the end.
constexpr int kTcAcc = 8;
constexpr uint32_t kTcTmemCols = kTcAcc * kTcXRows;     // 128 columns (a power of two >= 32)

__device__ __forceinline__ void epi_sync() { named_bar_sync(2, 128); }
constexpr uint32_t kStartBar = 1;     // warp 5 arrives, warps 0-4 wait: start-up done
constexpr uint32_t kTmemFreeBar = 3;  // warps 0-4: the epilogue has read the accumulator
constexpr uint64_t kPushWaitLimitNs = 3ull * kWaitLimitNs;  // > any chain of waits before a peer pushes

// Eight consecutive values from shared memory as fp32 (16-byte aligned source).
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
  const uint4 u = reinterpret_cast<const uint4*>(p)[0];
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(h[j]);
    v[2 * j] = f.x; v[2 * j + 1] = f.y;
  }
}

// Power-of-two scale that maps |max| into [2^14, 2^15) (2^125 for zero rows); writes its reciprocal.
__device__ __forceinline__ float split_scale(float amax, float* inv) {
  const int ef = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu);  // biased exponent
  int e = 141 - ef;                                                       // 15 - unbiased(frexp)
  e = e < -125 ? -125 : (e > 125 ? 125 : e);
  *inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
  return __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
}

template <int M, typename TX, bool OUT_F16>
__global__ void __launch_bounds__(kTcThreads, 1)
skinny_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const SkinnyArgs args) {
  constexpr int MP = MPad<M>::v;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = args.stages;                                      // ring depth
  const int R = args.rows;                                        // weight rows per stage
  const int box_bytes = tc_box_bytes(R);
  const int stage_bytes = tc_stage_bytes(R);
  using XL = XhlLayout<M>;
  uint8_t* ring = smem;                                           // S x [2 boxes of R x 64]
  const int nkb = (args.kchunk + 63) / 64;                        // 64-wide K blocks of x
  const int kpad = nkb * 64;
  // x as loaded, [M][kpad], overlays the ring's last stages: they are filled only after x_hi/x_lo
  // are built (the producer issues stage 0 alone before then).
  const int xst_stages = (M * kpad * static_cast<int>(sizeof(TX)) + stage_bytes - 1) / stage_bytes;
  TX* xst = reinterpret_cast<TX*>(ring + (S - xst_stages) * stage_bytes);
  uint8_t* xhl = ring + S * stage_bytes;                          // x_hi / x_lo, 1 KiB aligned
  float* red = reinterpret_cast<float*>(xhl + tc_xhl_bytes(M, nkb));  // [csize][slice][MP]: pushed partials
  float* amax_w = red + kTcRedBytes / 4;                          // [4 warps][8]
  float* scale_inv = amax_w + 32;                                 // [8]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(scale_inv + 8);
  uint64_t* empty_bar = full_bar + kTcMaxStages;
  uint64_t* xready_bar = empty_bar + kTcMaxStages;
  uint64_t* done_bar = xready_bar + 1;
  uint64_t* red_bar = done_bar + 1;
  uint64_t* xfull_bar = red_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Self-check: the layout must end inside the launch's dynamic shared memory (uniform for the
  // grid, so every CTA returns before any barrier, TMEM allocation or shared-memory access).
  if (S < 1 || S > kTcMaxStages || (R != 32 && R != 64 && R != 128) || xst_stages > S - 1 ||
      static_cast<uint32_t>(reinterpret_cast<const volatile uint8_t*>(abort_flag + 1) - smem_raw) >
          dynamic_smem_bytes()) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) {
      grid_dependency_wait();
      atomicExch(args.status, G16_ERR_ARG);
    }
    return;
  }

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rank = blockIdx.x;
  const int csize = gridDim.x;
  const int n0 = blockIdx.y * kTcStrip;
  const int kb = rank * args.kchunk;
  const int ke = min(args.K, kb + args.kchunk);
  const int nrows = max(0, ke - kb);
  const int nstages = (nrows + R - 1) / R;
  // The next kernel may start its set-up on free SMs now; it reads nothing this one writes before
  // its own grid_dependency_wait.
  if (tid == 0) grid_launch_dependents();
  const int slice = (kTcStrip + csize - 1) / csize;  // strip columns each rank finalises
  const int own0 = rank * slice;
  const int own_cnt = max(0, min(kTcStrip - own0, slice));
  const int pre = min(S, nstages);                   // ring fill: stages issued without waiting
  const TX* x = static_cast<const TX*>(args.x);

  // Start-up. The producer never waits on a CTA-wide barrier: TMA issue blocks while the TMA
  // unit's queue is full, and a barrier behind it would hold back x and the tensor core.
  // kStartBar (warp 5 arrives, warps 0-4 wait): barriers initialised, TMEM allocated. x is one
  // bulk copy per row, issued right after barrier initialisation, and the first weight stage(s)
  // follow it at once (x's requests go first); the rest of the ring waits until x_hi/x_lo are
  // built (xready_bar), since x as loaded overlays the ring's last stages and a long burst of TMA
  // issues would stall the shared-memory accesses of the x preparation behind it.
  if (warp == 5) {
    if (lane == 0) {
      for (int st = 0; st < S; ++st) {
        mbar_init(&full_bar[st], 1);
        mbar_init(&empty_bar[st], 1);
      }
      mbar_init(xready_bar, 1);
      mbar_init(done_bar, 1);
      mbar_init(red_bar, 1);
      mbar_init(xfull_bar, 1);
      *abort_flag = 0;
      fence_barrier_init();  // cluster scope: peers push into red_bar after the cluster barrier
      mbar_arrive_expect_tx(red_bar, static_cast<uint32_t>(csize * own_cnt * MP * 4));
      grid_dependency_wait();  // x, W: written by the preceding kernel, possibly
      // x chunk: one bulk copy per row (16-byte aligned: x is, K % 8 == 0 and kb % 32 == 0).
      const uint32_t xrow_bytes = static_cast<uint32_t>(nrows * sizeof(TX));
      mbar_arrive_expect_tx(xfull_bar, M * xrow_bytes);
      if (xrow_bytes > 0) {
#pragma unroll
        for (int m = 0; m < M; ++m)
          bulk_load(xst + m * kpad, x + static_cast<size_t>(m) * args.K + kb, xrow_bytes, xfull_bar);
      }
    }
    named_bar_arrive(kStartBar, 192);
    cluster_arrive();  // every thread, once; the epilogue waits before its first remote store
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      bool ok = true;
      uint32_t armed = 0;        // stages holding an issued load
      uint32_t armed_phase = 0;  // its phase parity, one bit per stage
      // Stages issued right behind x, before x_hi/x_lo exist: those not overlaid by x as loaded.
      // Measured on B200 (4096 x 4096, CUDA graph): all of them for M >= 4 (M = 8: 10.75 ->
      // 9.97 us, M = 4: 9.67 -> 9.45 us); only the first for smaller M (M = 1: 9.03 -> 8.96 us; all
      // of them gave 9.19 us), the x preparation then stalling less behind the TMA issues.
      const int early = M >= 4 ? S - xst_stages : 1;
      // Fill the ring: never-used stages, no empty-barrier wait.
      for (int t = 0; t < pre && ok; ++t) {
        if (t == early && !mbar_wait(xready_bar, 0, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[t], stage_bytes);
        armed |= 1u << t;
#pragma unroll
        for (int j = 0; j < kTcStrip / kTcBoxCols; ++j)
          tma_load_2d(ring + t * stage_bytes + j * box_bytes, &tmap_w, &full_bar[t], n0 + j * kTcBoxCols, kb + t * R);
      }
      int stage = pre;
      uint32_t phase = 0;
      if (stage == S) { stage = 0; phase = 1u; }
      for (int t = pre; t < nstages && ok; ++t) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
        uint8_t* dst = ring + stage * stage_bytes;
        mbar_arrive_expect_tx(&full_bar[stage], stage_bytes);
        armed |= 1u << stage;
        armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
#pragma unroll
        for (int j = 0; j < kTcStrip / kTcBoxCols; ++j)
          tma_load_2d(dst + j * box_bytes, &tmap_w, &full_bar[stage], n0 + j * kTcBoxCols, kb + t * R);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
        // No copy may still land in shared memory once the CTA leaves: x, then the armed stages.
        mbar_wait(xfull_bar, 0, nullptr);
        for (int st = 0; st < S; ++st)
          if ((armed >> st) & 1u) mbar_wait(&full_bar[st], (armed_phase >> st) & 1u, nullptr);
      }
    }
    return;
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  } else {
    // Zero the shared zero block of the packed layout while x is in flight.
    if constexpr (XL::kPacked) {
      if (tid < 64) reinterpret_cast<uint4*>(xhl + nkb * 1024)[tid] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  grid_dependency_wait();  // bias, out, status
  tc_fence_before();
  named_bar_sync(kStartBar, 192);
  tc_fence_after();
  cluster_arrive();  // every thread, once; the epilogue waits before its first remote store
  const uint32_t tmem = *tmem_slot;
  if (warp == 4) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // D[n][m'] += W[k][n] * xhl[m'][k]: A = W (MN-major), B = xhl (K-major), M=128, N=16, K=16.
      constexpr uint32_t idesc = idesc_f16_f32(128, kTcXRows, /*b_mn_major=*/false, /*a_mn_major=*/true);
      bool ok = mbar_wait(xready_bar, 0, abort_flag);
      uint32_t phase = 0;
      int stage = 0;
      for (int t = 0; t < nstages && ok; ++t) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(ring + stage * stage_bytes);
        for (int j = 0; j < R / kUmmaK; ++j) {
          const int ks = t * (R / kUmmaK) + j;  // 16-wide K step within the chunk
          // A: rows [16j, 16j + 16) of the stage: 2 KiB in; the two 64-column boxes are box_bytes
          // apart (LBO), 8-row k groups 1 KiB apart (SBO).
          const uint64_t adesc = smem_desc_sw128(sa + j * (kUmmaK * 128), box_bytes, 1024);
          // B: K step ks of x_hi / x_lo; the second 8-row group is SBO bytes on (the zero block
          // when packed).
          const uint32_t sbo = XL::kPacked ? static_cast<uint32_t>(nkb - (ks >> 2)) * 1024u : 1024u;
          const uint64_t bdesc =
              smem_desc_sw128(smem_u32(xhl) + (ks >> 2) * XL::kBlockBytes + (ks & 3) * 32, 16, sbo);
          umma_f16(tmem + static_cast<uint32_t>((ks % kTcAcc) * kTcXRows), adesc, bdesc, idesc,
                   ks >= kTcAcc ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
      }
      umma_commit(done_bar);  // also the drain: arrives once every issued MMA has completed
      mbar_wait(done_bar, 0, nullptr);
    }
    __syncwarp();
    named_bar_sync(kTmemFreeBar, 160);  // the epilogue has read the accumulator
    __syncwarp();                        // tcgen05.dealloc is .sync.aligned
    tc_fence_after();
    tmem_dealloc(tmem, kTcTmemCols);
  } else {
    // ---------------- warps 0-3: build xhl, then the epilogue ----------------
    // xst rows hold [0, nrows) of the chunk; k >= nrows is masked below (nrows % 8 == 0).
    if (!mbar_wait(xfull_bar, 0, abort_flag) && tid == 0) {
      *abort_flag = 1;
      atomicExch(args.status, G16_ERR_TIMEOUT);
    }
    // 1. per-row |max| over the chunk (8 values per 16 bytes read)
    float am[M];
#pragma unroll
    for (int m = 0; m < M; ++m) am[m] = 0.f;
    for (int k = tid * 8; k < nrows; k += 128 * 8) {  // zeros past nrows do not change |max|
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float v[8];
        load8(xst + m * kpad + k, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) am[m] = fmaxf(am[m], fabsf(v[j]));
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) am[m] = fmaxf(am[m], __shfl_xor_sync(0xffffffffu, am[m], o));
      if (lane == 0) amax_w[warp * 8 + m] = am[m];
    }
    epi_sync();  // amax_w complete
    float sc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float a = fmaxf(fmaxf(amax_w[m], amax_w[8 + m]), fmaxf(amax_w[16 + m], amax_w[24 + m]));
      float inv;
      sc[m] = split_scale(a, &inv);
      if (tid == 0) scale_inv[m] = inv;
    }
    // 2. x*s = hi + lo into x_hi / x_lo (every row of the block written, zero rows included): one
    //    16-byte chunk of 8 k values per row and step, 128-byte swizzled K-major layout (chunk
    //    index ^ (row & 7)).
    for (int k = tid * 8; k < kpad; k += 128 * 8) {
      uint8_t* kblk = xhl + (k >> 6) * XL::kBlockBytes;
      const int c16 = (k & 63) >> 3;
      auto put = [&](int row, uint4 v) {
        *reinterpret_cast<uint4*>(kblk + (row >> 3) * 1024 + (row & 7) * 128 + ((c16 ^ (row & 7)) << 4)) = v;
      };
      const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (XL::kPacked) {
#pragma unroll
        for (int row = 2 * M; row < 8; ++row) put(row, zero);
      } else {
#pragma unroll
        for (int row = M; row < 8; ++row) {
          put(row, zero);
          put(8 + row, zero);
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float v[8];
        if (k < nrows) {
          load8(xst + m * kpad + k, v);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = 0.f;
        }
        uint32_t hp[4], lp[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a0 = v[2 * j] * sc[m], a1 = v[2 * j + 1] * sc[m];
          const __half2 h = __floats2half2_rn(a0, a1);
          const float2 hf = __half22float2(h);
          const __half2 l = __floats2half2_rn(a0 - hf.x, a1 - hf.y);
          hp[j] = *reinterpret_cast<const uint32_t*>(&h);
          lp[j] = *reinterpret_cast<const uint32_t*>(&l);
        }
        put(m, make_uint4(hp[0], hp[1], hp[2], hp[3]));
        put(XL::kLoRow + m, make_uint4(lp[0], lp[1], lp[2], lp[3]));
      }
    }
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
    epi_sync();
    if (tid == 0) mbar_arrive(xready_bar);

    // 3. wait for the last MMA, read the kTcAcc [128 x 16] accumulators (lane = weight column)
    //    and add those that were written, in accumulator order
    bool got = mbar_wait(done_bar, 0, abort_flag);
    got = __all_sync(0xffffffffu, got);
    if (!got && lane == 0) {
      *abort_flag = 1;
      atomicExch(args.status, G16_ERR_TIMEOUT);
    }
    tc_fence_after();
    const int used = min(kTcAcc, nstages * (R / kUmmaK));
    float acc16[kTcXRows];
#pragma unroll
    for (int i = 0; i < kTcXRows; ++i) acc16[i] = 0.f;
    __syncwarp();
#pragma unroll
    for (int q = 0; q < kTcAcc / 2; ++q) {
      uint32_t d[32];
      __syncwarp();  // tcgen05.ld is .sync.aligned
      tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(q * 32), d);
      tmem_ld_wait();
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (2 * q + h < used) {
#pragma unroll
          for (int i = 0; i < kTcXRows; ++i) acc16[i] += __uint_as_float(d[h * kTcXRows + i]);
        }
    }
    tc_fence_before();
    named_bar_arrive(kTmemFreeBar, 160);
    const bool live = nstages > 0 && got;
    float v[MP];
#pragma unroll
    for (int m = 0; m < MP; ++m)
      v[m] = (m < M && live) ? (acc16[m] + acc16[XL::kLoRow + m]) * scale_inv[m] : 0.f;

    // 4. push column `tid` to the rank that owns it (every path pushes: owners wait for all bytes)
    const int owner = tid / slice;
    const int j = tid - owner * slice;
    cluster_wait();  // peers' barriers are initialised
    const uint32_t dst = map_cluster(smem_u32(red + (rank * slice + j) * MP), static_cast<uint32_t>(owner));
    const uint32_t rbar = map_cluster(smem_u32(red_bar), static_cast<uint32_t>(owner));
    if constexpr (MP == 1) {
      st_async_b32(dst, v[0], rbar);
    } else if constexpr (MP == 2) {
      st_async_v2(dst, v[0], v[1], rbar);
    } else {
#pragma unroll
      for (int q = 0; q < MP / 4; ++q)
        st_async_v4(dst + 16u * q, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3], rbar);
    }

    // 5. finalise the owned columns: sum the csize partials in rank order, add bias, store
    if (!mbar_wait_cluster(red_bar, 0, kPushWaitLimitNs)) {
      if (tid == 0) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
      }
      return;
    }
    for (int i = tid; i < M * own_cnt; i += 128) {
      const int m = i / own_cnt, jj = i - m * own_cnt;
      const int n = n0 + own0 + jj;
      if (n < args.N) {
        float acc = 0.f;
        for (int q = 0; q < csize; ++q) acc += red[(q * slice + jj) * MP + m];
        if (args.bias != nullptr) acc += args.bias[n];
        acc = apply_act(acc, args.act);
        if constexpr (OUT_F16) {
          reinterpret_cast<__half*>(args.out)[static_cast<size_t>(m) * args.N + n] = __float2half_rn(acc);
        } else {
          reinterpret_cast<float*>(args.out)[static_cast<size_t>(m) * args.N + n] = acc;
        }
      }
    }
  }
}

// Ring stages that x (as loaded) overlays.
int tc_xst_stages(int M, int kchunk, int x_bytes, int rows) {
  const int kpad = (kchunk + 63) / 64 * 64;
  return (M * kpad * x_bytes + tc_stage_bytes(rows) - 1) / tc_stage_bytes(rows);
}

size_t skinny_tc_smem_bytes(int M, int kchunk, int rows, int stages) {
  const int nkb = (kchunk + 63) / 64;
  return 1024 + static_cast<size_t>(stages) * tc_stage_bytes(rows) + tc_xhl_bytes(M, nkb) + kTcRedBytes + 32 * 4 +
         8 * 4 + (2 * kTcMaxStages + 4) * 8 + 8;
}

// The largest layout (8 fp32 rows, the longest chunk, 128-row stages) must still hold x in the
// ring's last stages and leave one stage before them.
static_assert(1024 + 3 * tc_stage_bytes(kTcMaxRows) + tc_xhl_bytes(8, kTcMaxChunk / 64) + kTcRedBytes + 32 * 4 +
                      8 * 4 + (2 * kTcMaxStages + 4) * 8 + 8 <=
                  kTcSmemLimit &&
                  8 * kTcMaxChunk * 4 <= 2 * tc_stage_bytes(kTcMaxRows),
              "tensor-core skinny layout exceeds shared memory");
static_assert(kTcMaxStages <= 32, "armed-stage bit masks are 32 bits wide");

// Column strips of kTcStrip; K split over up to 16 cluster ranks with chunks that are whole
// stages of `rows` weight rows, at least two stages per rank.
SkinnyPlan plan_tc_rows(int M, int K, int N, int ctas, int x_bytes, int rows) {
  SkinnyPlan p{};
  p.strips = (N + kTcStrip - 1) / kTcStrip;
  int c = ctas / p.strips;
  if (c < 1) c = 1;
  if (c > kMaxCluster) c = kMaxCluster;
  const int max_by_k = K / (2 * rows) > 0 ? K / (2 * rows) : 1;
  if (c > max_by_k) c = max_by_k;
  int kchunk = (K + c - 1) / c;
  kchunk = (kchunk + rows - 1) / rows * rows;
  c = (K + kchunk - 1) / kchunk;
  if (c < 1) c = 1;
  p.csize = c;
  p.kchunk = kchunk;
  p.piece = kchunk;
  p.rows = rows;
  // Ring depth: measured on B200 (4096 x 4096), 3 stages of 128 rows beat 2, 4, 5 and 6: the
  // bandwidth is there with 96 KiB in flight per CTA, and deeper rings queue more TMA issues in
  // front of the MMA issues. x as loaded overlays the last stages, so at least one precedes them.
  const size_t fixed = skinny_tc_smem_bytes(M, kchunk, rows, 0);
  int stages = fixed < static_cast<size_t>(kTcSmemLimit)
                   ? static_cast<int>((static_cast<size_t>(kTcSmemLimit) - fixed) / tc_stage_bytes(rows))
                   : 0;
  const int xst_stages = tc_xst_stages(M, kchunk, x_bytes, rows);
  const int preferred = rows == 128 ? 3 : rows == 64 ? 4 : 8;
  stages = std::min(stages, kTcMaxStages);
  stages = std::min(stages, std::max(std::min(preferred, kchunk / rows), xst_stages + 1));
  p.stages = stages;
  p.smem_bytes = skinny_tc_smem_bytes(M, kchunk, rows, stages);
  p.tc = (kchunk <= kTcMaxChunk && stages >= 2 && stages >= xst_stages + 1) ? 1 : 0;
  return p;
}

// Each stage costs the MMA issuer a commit and a barrier round trip whatever its height, so the
// tallest stage wins unless a shorter one puts more CTAs to work.
SkinnyPlan plan_tc(int M, int K, int N, int ctas, int x_bytes) {
  SkinnyPlan best = plan_tc_rows(M, K, N, ctas, x_bytes, kTcMinRows);
  for (int rows = kTcMaxRows; rows > kTcMinRows; rows /= 2) {
    const SkinnyPlan p = plan_tc_rows(M, K, N, ctas, x_bytes, rows);
    if (p.tc && (!best.tc || p.csize >= best.csize)) {
      best = p;
      break;
    }
  }
  return best;
}

// The largest cluster whose clusters are all resident at once (one CTA per SM with tensor memory).
template <typename F>
int plan_tc_for(F* kern, int M, int K, int N, int x_bytes, const DeviceInfo& dev, SkinnyPlan* out) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, SkinnyPlan> cache;
  int devid = 0;
  cudaError_t e = cudaGetDevice(&devid);
  if (e != cudaSuccess) return cuda_fail(e);
  const uint64_t key = (static_cast<uint64_t>(devid) << 58) ^ (static_cast<uint64_t>(M) << 54) ^
                       (static_cast<uint64_t>(x_bytes) << 51) ^ (static_cast<uint64_t>(K) << 26) ^
                       static_cast<uint64_t>(N);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return G16_OK;
    }
  }
  SkinnyPlan p = plan_tc(M, K, N, dev.sm_count, x_bytes);
  int first = -1;
  while (p.tc) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(p, nullptr, attr);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    int active = 0;
    e = cudaOccupancyMaxActiveClusters(&active, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e);
    if (first < 0) first = active;
    p.active = active;
    if (active >= p.strips || p.csize == 1) break;
    p = plan_tc(M, K, N, (p.csize - 1) * p.strips, x_bytes);
  }
  p.active_first = first;
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = p;
  *out = p;
  return G16_OK;
}

template <int M, typename TX, bool OUT_F16>
int launch_skinny_tc_t(const void* x, const uint16_t* w, const float* bias, void* out, int K, int N, cudaStream_t s,
                       const DeviceInfo& dev, int act) {
  static std::atomic<uint64_t> attr_done{0};
  auto kern = skinny_tc_kernel<M, TX, OUT_F16>;
  cudaError_t e = ensure_attrs(kern, attr_done, kTcSmemLimit);
  if (e != cudaSuccess) return cuda_fail(e);
  SkinnyPlan p;
  int st = plan_tc_for(kern, M, K, N, static_cast<int>(sizeof(TX)), dev, &p);
  if (st != G16_OK) return st;
  if (!p.tc) return launch_skinny_fma_t<M, TX, OUT_F16>(x, w, bias, out, K, N, s, dev, act);
  if (p.stages < 2 || p.stages > kTcMaxStages ||
      p.smem_bytes != skinny_tc_smem_bytes(M, p.kchunk, p.rows, p.stages) ||
      p.stages < tc_xst_stages(M, p.kchunk, static_cast<int>(sizeof(TX)), p.rows) + 1 ||
      p.smem_bytes > static_cast<size_t>(kTcSmemLimit))
    return G16_ERR_ARG;
  CUtensorMap tmap;
  st = make_tmap_2d(&tmap, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                    p.rows, kTcBoxCols, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  SkinnyArgs a{};
  a.act = act;
  a.x = x;
  a.bias = bias;
  a.out = out;
  a.status = device_status_ptr();
  if (a.status == nullptr) return G16_ERR_CUDA;
  a.K = K;
  a.N = N;
  a.kchunk = p.kchunk;
  a.piece = p.kchunk;
  a.stages = p.stages;
  a.rows = p.rows;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = make_cfg(p, s, attr);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  // Programmatic dependent launch: back-to-back calls overlap one launch's set-up with the
  // previous one's tail (the kernel waits for its predecessor before any global access).
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, tmap, a);
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

// The tensor-core variant whenever its K chunk fits in shared memory, else the FMA variant.
template <int M, typename TX, bool OUT_F16>
int launch_skinny_t(const void* x, const uint16_t* w, const float* bias, void* out, int K, int N, cudaStream_t s,
                    const DeviceInfo& dev, int act) {
  return launch_skinny_tc_t<M, TX, OUT_F16>(x, w, bias, out, K, N, s, dev, act);
}

template <int M>
int dispatch_types(const void* x, int x_dtype, const uint16_t* w, const float* bias, void* out, int out_dtype, int K,
                   int N, cudaStream_t s, const DeviceInfo& dev, int act) {
  if (x_dtype == G16_F32) {
    return out_dtype == G16_F16 ? launch_skinny_t<M, float, true>(x, w, bias, out, K, N, s, dev, act)
                                : launch_skinny_t<M, float, false>(x, w, bias, out, K, N, s, dev, act);
  }
  return out_dtype == G16_F16 ? launch_skinny_t<M, __half, true>(x, w, bias, out, K, N, s, dev, act)
                              : launch_skinny_t<M, __half, false>(x, w, bias, out, K, N, s, dev, act);
}

}  // namespace

int launch_skinny(const void* x, int x_dtype, const uint16_t* w, const float* bias, void* out, int out_dtype, int M,
                  int K, int N, cudaStream_t s, const DeviceInfo& dev, int act) {
  switch (M) {
    case 1: return dispatch_types<1>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    case 2: return dispatch_types<2>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    case 3: return dispatch_types<3>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    case 4: return dispatch_types<4>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    case 5: return dispatch_types<5>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    case 6: return dispatch_types<6>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    case 7: return dispatch_types<7>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    case 8: return dispatch_types<8>(x, x_dtype, w, bias, out, out_dtype, K, N, s, dev, act);
    default: return G16_ERR_ARG;
  }
}

int skinny_plan_info(int M, int K, int N, int x_dtype, int* info, const DeviceInfo& dev) {
  if (M < 1 || M > 8) return G16_ERR_ARG;
  SkinnyPlan p;
  int st;
  if (x_dtype == G16_F32) {
    static std::atomic<uint64_t> attr_done{0};
    auto kern = skinny_tc_kernel<1, float, false>;
    cudaError_t e = ensure_attrs(kern, attr_done, kTcSmemLimit);
    if (e != cudaSuccess) return cuda_fail(e);
    st = plan_tc_for(kern, M, K, N, 4, dev, &p);
  } else {
    static std::atomic<uint64_t> attr_done{0};
    auto kern = skinny_tc_kernel<1, __half, false>;
    cudaError_t e = ensure_attrs(kern, attr_done, kTcSmemLimit);
    if (e != cudaSuccess) return cuda_fail(e);
    st = plan_tc_for(kern, M, K, N, 2, dev, &p);
  }
  if (st != G16_OK) return st;
  info[0] = p.tc;
  info[1] = p.csize;
  info[2] = p.strips;
  info[3] = p.kchunk;
  info[4] = static_cast<int>(p.smem_bytes);
  info[5] = p.active_first;
  info[6] = p.active;
  return G16_OK;
}

}  // namespace g16
