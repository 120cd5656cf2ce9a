// Tensor-core GEMM for problems with fewer output tiles than SMs: out[M,N] = (A @ B) * rscale[row]
// + bias[col], A [M,K] fp16 K-major, B [K,N] fp16 N-major, fp32 accumulation in TMEM.
//
// One CTA per (tile, K chunk), no persistence. Tiles are 128 x BN (BN = 64, 128 or 256: narrower tiles
// put more CTAs to work when M is small). When K is split into C chunks, the C CTAs of a tile form
// a thread-block cluster and reduce in distributed shared memory instead of through HBM:
//   * rank r owns rows [r*rpo, (r+1)*rpo) of the tile (rpo = ceil(128 / C));
//   * once every rank's mainloop has drained (split cluster barrier), each epilogue warp reads its
//     32 TMEM lanes (rows) and pushes them with st.async into the owner's shared memory (its freed
//     TMA ring), completing bytes on the owner's mbarrier;
//   * the owner sums the C partials of its rows in rank order (p0 + p1 + ... in fp32, the same
//     order and chunk boundaries as the workspace split-K reduction, so results are bitwise
//     identical to it), applies the unscale and bias and stores.
// No atomics, no workspace, bitwise reproducible. Roles: warp 0 TMA producer, warp 1 TMEM
// allocation + MMA issue, warps 2-5 epilogue. Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <unordered_map>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

// 64-wide tiles in the automatic plan (a build option for measuring them against 128-wide ones).
#ifndef G16_SMALL_BN64
#define G16_SMALL_BN64 1
#endif

namespace g16 {
namespace {

constexpr int kSmThreads = 192;
constexpr int kSmStagesDefault = 4;
constexpr uint32_t kSmABytes = kBM * kBK * 2;      // 16 KiB
constexpr uint32_t kSmBBoxBytes = kBK * 64 * 2;    // one [64 k x 64 n] box: 8 KiB
constexpr int kSmMaxCluster = 16;
constexpr uint64_t kSmPushWaitNs = 3ull * kWaitLimitNs;  // > any chain of waits before a peer pushes

template <int BN>
struct SmallGeo {
  static constexpr uint32_t kBBytes = kBK * BN * 2;
  static constexpr uint32_t kStageBytes = kSmABytes + kBBytes;
  // 64-wide tiles: a deeper ring, which also keeps the CTA at one per SM (two would share its
  // bandwidth)
  static constexpr int kStages = BN == 64 ? 6 : kSmStagesDefault;
  static constexpr uint32_t kRingBytes = kStages * kStageBytes;
  // partials received by an owner: C x rpo rows x BN fp32, at most (128 + C - 1) rows
  static constexpr uint32_t kRecvBytes = (kBM + kSmMaxCluster) * BN * 4;
  static_assert(kRecvBytes <= kRingBytes, "the freed ring must hold an owner's partials");
  static constexpr size_t kSmemBytes = 1024 + kRingBytes + 256;
};

struct SmallArgs {
  void* out;
  const float* bias;
  const float* rscale;
  int* status;
  int M, N, K;
  int n_tiles;           // tiles along N
  int kblocks, kb_per_split;
  int act;  // epilogue activation (G16_ACT_*)
};

template <bool OUT_F16>
__device__ __forceinline__ void store4(const SmallArgs& a, int row, int col, float o0, float o1, float o2, float o3) {
  const size_t off = static_cast<size_t>(row) * a.N + col;
  o0 = apply_act(o0, a.act);
  o1 = apply_act(o1, a.act);
  o2 = apply_act(o2, a.act);
  o3 = apply_act(o3, a.act);
  if constexpr (OUT_F16) {
    const __half2 h0 = __floats2half2_rn(o0, o1), h1 = __floats2half2_rn(o2, o3);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&h0);
    u.y = *reinterpret_cast<const uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(a.out) + off) = u;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + off) = make_float4(o0, o1, o2, o3);
  }
}

// grid = (C, tiles); cluster (C, 1, 1) when C > 1. blockIdx.x = K chunk = rank in the cluster.
template <bool OUT_F16, int BN>
__global__ void __launch_bounds__(kSmThreads, 1)
gemm_small_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                  const SmallArgs args) {
  using G = SmallGeo<BN>;
  constexpr int kSmStages = G::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  float* recv = reinterpret_cast<float*>(smem);  // after the mainloop: [C][rpo][BN] partials
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + G::kRingBytes);
  uint64_t* empty_bar = full_bar + kSmStages;
  uint64_t* done_bar = empty_bar + kSmStages;
  uint64_t* red_bar = done_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  if (static_cast<uint32_t>(reinterpret_cast<const volatile uint8_t*>(abort_flag + 1) - smem_raw) >
      dynamic_smem_bytes()) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) {
      grid_dependency_wait();
      atomicExch(args.status, G16_ERR_ARG);
    }
    return;
  }

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int csize = gridDim.x;
  const int rank = blockIdx.x;
  const int tile = blockIdx.y;
  const int mt = tile / args.n_tiles;
  const int nt = tile - mt * args.n_tiles;
  const int kb0 = rank * args.kb_per_split;
  const int kb1 = min(args.kblocks, kb0 + args.kb_per_split);
  const int rpo = (kBM + csize - 1) / csize;                      // rows each rank finalises
  const int own0 = rank * rpo;
  const int own_rows = max(0, min(kBM - own0, rpo));
  // The next kernel may start its set-up now; it reads nothing this one writes before its own
  // grid dependency wait.
  if (threadIdx.x == 0) grid_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSmStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(red_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();  // cluster scope: peers push into red_bar after the cluster barrier
    if (csize > 1) mbar_arrive_expect_tx(red_bar, static_cast<uint32_t>(csize * own_rows * BN * 4));
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
      grid_dependency_wait();  // A, B: possibly written by the preceding kernel
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
        uint8_t* sa = ring + stage * G::kStageBytes;
        uint8_t* sb = sa + kSmABytes;
        mbar_arrive_expect_tx(&full_bar[stage], G::kStageBytes);
        armed |= 1u << stage;
        armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
        tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * kBK, mt * kBM);
#pragma unroll
        for (int j = 0; j < BN / 64; ++j)
          tma_load_2d(sb + j * kSmBBoxBytes, &tmap_b, &full_bar[stage], nt * BN + 64 * j, kb * kBK);
        if (++stage == kSmStages) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
        for (int s = 0; s < kSmStages; ++s)
          if ((armed >> s) & 1u) mbar_wait(&full_bar[s], (armed_phase >> s) & 1u, nullptr);
      }
    }
    if (csize > 1) cluster_arrive();  // every thread of the cluster arrives once
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN, /*b_mn_major=*/true);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(ring + stage * G::kStageBytes);
        const uint32_t sb = sa + kSmABytes;
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k) {
          // A: K-major, 128-byte rows, 8-row atoms 1024 B apart (SBO); K steps of 32 B.
          const uint64_t adesc = smem_desc_sw128(sa + k * (kUmmaK * 2), 16, 1024);
          // B: N-major, 64-column boxes 8 KiB apart (LBO), 8-row k groups 1024 B apart (SBO).
          const uint64_t bdesc = smem_desc_sw128(sb + k * (kUmmaK * 128), kSmBBoxBytes, 1024);
          umma_f16(tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == kSmStages) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
      }
      umma_commit(done_bar);  // also the drain: arrives once every issued MMA has completed
      mbar_wait(done_bar, 0, nullptr);
    }
    __syncwarp();
    if (csize > 1) cluster_arrive();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;                 // TMEM lane quarter this warp may access
    const int r_local = quarter * 32 + lane;      // tile row of this lane
    const int row = mt * kBM + r_local;
    grid_dependency_wait();  // bias, rscale, out
    bool got = mbar_wait(done_bar, 0, abort_flag);
    got = __all_sync(0xffffffffu, got);
    if (!got && lane == 0) {
      *abort_flag = 1;
      atomicExch(args.status, G16_ERR_TIMEOUT);
    }
    const bool live = got && kb1 > kb0;
    tc_fence_after();
    if (csize == 1) {
      const float rs = (args.rscale != nullptr && row < args.M) ? __ldg(args.rscale + row) : 1.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(c * 32), r);
        tmem_ld_wait();
        const int col0 = nt * BN + c * 32;
        if (row < args.M) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int col = col0 + 4 * g;
            if (col < args.N) {  // N % 8 == 0: whole quads are in or out
              float v[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) v[j] = live ? __uint_as_float(r[4 * g + j]) : 0.f;
              const float4 b = args.bias != nullptr ? __ldg(reinterpret_cast<const float4*>(args.bias + col))
                                                    : make_float4(0.f, 0.f, 0.f, 0.f);
              store4<OUT_F16>(args, row, col, fmaf(v[0], rs, b.x), fmaf(v[1], rs, b.y), fmaf(v[2], rs, b.z),
                              fmaf(v[3], rs, b.w));
            }
          }
        }
      }
    } else {
      // Every rank's tensor core and TMA are done with its ring before anyone overwrites it.
      cluster_arrive();
      cluster_wait();
      const int owner = r_local / rpo;
      const int rr = r_local - owner * rpo;
      const uint32_t rbar = map_cluster(smem_u32(red_bar), static_cast<uint32_t>(owner));
      const uint32_t dst_row =
          map_cluster(smem_u32(recv + (static_cast<size_t>(rank) * rpo + rr) * BN), static_cast<uint32_t>(owner));
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(c * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 8; ++q)
          st_async_v4(dst_row + static_cast<uint32_t>((c * 32 + 4 * q) * 4),
                      live ? __uint_as_float(r[4 * q]) : 0.f, live ? __uint_as_float(r[4 * q + 1]) : 0.f,
                      live ? __uint_as_float(r[4 * q + 2]) : 0.f, live ? __uint_as_float(r[4 * q + 3]) : 0.f, rbar);
      }
      // Sum this rank's rows over the cluster in rank order, then unscale, bias, store.
      if (mbar_wait_cluster(red_bar, 0, kSmPushWaitNs)) {
        const int et = threadIdx.x - 64;  // 0..127
        const int quads = own_rows * (BN / 4);
        for (int i = et; i < quads; i += 128) {
          const int orr = i / (BN / 4);
          const int col_l = (i - orr * (BN / 4)) * 4;
          const int orow = mt * kBM + own0 + orr;
          const int col = nt * BN + col_l;
          if (orow < args.M && col < args.N) {
            float4 acc = *reinterpret_cast<const float4*>(recv + static_cast<size_t>(orr) * BN + col_l);
            for (int s = 1; s < csize; ++s) {
              const float4 v = *reinterpret_cast<const float4*>(recv + (static_cast<size_t>(s) * rpo + orr) * BN + col_l);
              acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
            const float rs = args.rscale != nullptr ? __ldg(args.rscale + orow) : 1.f;
            const float4 b = args.bias != nullptr ? __ldg(reinterpret_cast<const float4*>(args.bias + col))
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            store4<OUT_F16>(args, orow, col, fmaf(acc.x, rs, b.x), fmaf(acc.y, rs, b.y), fmaf(acc.z, rs, b.z),
                            fmaf(acc.w, rs, b.w));
          }
        }
      } else if (threadIdx.x == 64) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, BN);
  }
}

template <typename F>
cudaError_t ensure_small_attrs(F* kern, std::atomic<uint64_t>& done, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

template <bool OUT_F16, int BN>
int launch_small_t(const uint16_t* a16, const uint16_t* b16, void* out, const float* bias, const float* rscale, int M,
                   int K, int N, int csize, cudaStream_t s, int act) {
  static std::atomic<uint64_t> attr_done{0};
  auto kern = gemm_small_kernel<OUT_F16, BN>;
  cudaError_t e = ensure_small_attrs(kern, attr_done, static_cast<int>(SmallGeo<BN>::kSmemBytes));
  if (e != cudaSuccess) return cuda_fail(e);
  SmallArgs args{};
  args.act = act;
  args.out = out;
  args.bias = bias;
  args.rscale = rscale;
  args.status = device_status_ptr();
  if (args.status == nullptr) return G16_ERR_CUDA;
  args.M = M;
  args.N = N;
  args.K = K;
  const int m_tiles = (M + kBM - 1) / kBM;
  args.n_tiles = (N + BN - 1) / BN;
  args.kblocks = (K + kBK - 1) / kBK;
  args.kb_per_split = (args.kblocks + csize - 1) / csize;
  csize = (args.kblocks + args.kb_per_split - 1) / args.kb_per_split;  // no empty chunks
  CUtensorMap ta, tb;
  int st = make_tmap_2d(&ta, a16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(M),
                        static_cast<uint64_t>(K), kBM, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  st = make_tmap_2d(&tb, b16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                    kBK, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(csize), static_cast<unsigned>(m_tiles * args.n_tiles), 1);
  cfg.blockDim = dim3(kSmThreads, 1, 1);
  cfg.dynamicSmemBytes = SmallGeo<BN>::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: a launch's set-up overlaps the previous kernel's tail.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, args);
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

// Clusters of `c` CTAs of this kernel that can be resident at once (0 if none).
template <int BN>
int active_clusters(int c, int tiles) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;  // (device, cluster size) -> resident clusters
  int devid = 0;
  if (cudaGetDevice(&devid) != cudaSuccess) return 0;
  const uint64_t key = (static_cast<uint64_t>(devid) << 32) | static_cast<uint32_t>(c);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  static std::atomic<uint64_t> attr_done{0};
  auto kern = gemm_small_kernel<true, BN>;  // both output types have the same resources
  if (ensure_small_attrs(kern, attr_done, static_cast<int>(SmallGeo<BN>::kSmemBytes)) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(c), static_cast<unsigned>(tiles), 1);
  cfg.blockDim = dim3(kSmThreads, 1, 1);
  cfg.dynamicSmemBytes = SmallGeo<BN>::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(c);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int active = 0;
  if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    active = 0;
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = active;
  return active;
}

int active_clusters_bn(int bn, int c, int tiles) {
  return bn == 64 ? active_clusters<64>(c, tiles)
                  : bn == 128 ? active_clusters<128>(c, tiles) : active_clusters<256>(c, tiles);
}

}  // namespace

// Plan for the small-problem kernel: BN and cluster size, or bn = 0 when the problem has enough
// tiles for the persistent kernel. Measured on B200 (eager launches, operands from HBM):
// 128-wide tiles beat 256-wide ones whenever the output has few tiles (more CTAs; these
// problems are bound by operand reads from L2 and HBM, not by the tensor core), and splitting K
// pays only when the output is tiny and K long (128x16384x1024: 10 chunks 18.9 us vs 20.7 us via
// the workspace; 1024^3 and 2048x3072x1024: no split is fastest). So: 128-wide tiles, K split
// towards one CTA per SM while every chunk keeps >= 16 k-blocks (>= 4 when the output has fewer
// than 32 tiles), then shrunk until every cluster is resident at once (a second wave would double
// the time). Cached per (device, M, K, N).
SmallPlan plan_gemm_small(int M, int K, int N, const DeviceInfo& dev) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, SmallPlan> cache;
  SmallPlan p{};
  const int m_tiles = (M + kBM - 1) / kBM;
  const int kblocks = (K + kBK - 1) / kBK;
  const int t256 = m_tiles * ((N + 255) / 256);
  if (t256 * 2 > dev.sm_count) return p;  // persistent kernel
  int devid = 0;
  if (cudaGetDevice(&devid) != cudaSuccess) return p;
  const uint64_t key = (static_cast<uint64_t>(devid) << 58) ^ (static_cast<uint64_t>(M) << 38) ^
                       (static_cast<uint64_t>(K) << 19) ^ static_cast<uint64_t>(N);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  // K chunks for `tiles` tiles of width bn: towards one CTA per SM, chunks of >= kmin k-blocks,
  // every cluster resident at once; 0 if not even one cluster of one CTA fits.
  auto chunks = [&](int bn, int tiles) {
    const int kmin = tiles < 32 ? 4 : 16;
    int c = std::min(std::min(dev.sm_count / tiles, kSmMaxCluster), std::max(1, kblocks / kmin));
    c = std::max(c, 1);
    for (; c > 1; --c)
      if (active_clusters_bn(bn, c, tiles) >= tiles) break;
    return (c > 1 || active_clusters_bn(bn, 1, tiles) >= 1) ? c : 0;
  };
  const int tiles = m_tiles * ((N + 127) / 128);
  if (tiles <= dev.sm_count) {
    const int c = chunks(128, tiles);
    if (c > 0) {
      p.bn = 128;
      p.csize = c;
    }
    // 64-wide tiles when the 128-wide plan leaves more than a quarter of the SMs idle (the cluster
    // size, at most 16 and further limited by residency, caps the K split) and they put at least
    // 1.5x as many CTAs to work. Measured on B200 (CUDA graphs, operands rotated through HBM),
    // 128-wide -> 64-wide: 1024^3 9.56 -> 8.32 us (64 -> 128 CTAs), 200 x 1032 x 136 9.59 -> 6.74
    // (16 -> 24); but 128 x 16384 x 1024 17.88 -> 18.51 and 256 x 16384 x 512 17.23 -> 18.20, where
    // residency cuts the 64-wide clusters to 6 chunks (80 -> 96 CTAs).
    const int tiles64 = m_tiles * ((N + 63) / 64);
    if (4 * tiles * c < 3 * dev.sm_count && tiles64 <= dev.sm_count && G16_SMALL_BN64) {
      const int c64 = chunks(64, tiles64);
      if (c64 > 0 && 2 * tiles64 * c64 >= 3 * tiles * c) {
        p.bn = 64;
        p.csize = c64;
      }
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = p;
  return p;
}

int launch_gemm_small(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                      const float* rscale, int M, int K, int N, int bn, int csize, bool exact, cudaStream_t s,
                      int act) {
  if (csize < 1 || csize > kSmMaxCluster || (bn != 64 && bn != 128 && bn != 256)) return G16_ERR_ARG;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  int c = csize;
  while (c > 1 && active_clusters_bn(bn, c, tiles) < 1) --c;  // a cluster must fit at all
  if (exact && c != csize) return G16_ERR_UNSUPPORTED;        // the caller asked for csize K chunks
  if (bn == 64)
    return out_dtype == G16_F16 ? launch_small_t<true, 64>(a16, b16, out, bias, rscale, M, K, N, c, s, act)
                                : launch_small_t<false, 64>(a16, b16, out, bias, rscale, M, K, N, c, s, act);
  if (out_dtype == G16_F16) {
    return bn == 128 ? launch_small_t<true, 128>(a16, b16, out, bias, rscale, M, K, N, c, s, act)
                     : launch_small_t<true, 256>(a16, b16, out, bias, rscale, M, K, N, c, s, act);
  }
  return bn == 128 ? launch_small_t<false, 128>(a16, b16, out, bias, rscale, M, K, N, c, s, act)
                   : launch_small_t<false, 256>(a16, b16, out, bias, rscale, M, K, N, c, s, act);
}

}  // namespace g16
