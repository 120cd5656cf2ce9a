// Medium-M GEMM: out[M,N] = (x16[M,K] @ W[K,N]) * rscale[row] + bias[col] for M <= 64 rows of
// activations (the reference's tiled/split-K kernels, src/gtx16_fp16/ops.py:89-108, serve these
// shapes on its GPU). Such a GEMM streams W (2KN bytes) and does little math per byte, so it is
// HBM bound; a 128-row tensor-core tile with the activations as its M operand would be mostly
// zero rows. Here the operands swap roles: out^T = W^T x^T, so the 128 weight columns of a strip
// are the MMA's M and the activation rows the MMA's N (16, 32 or 64):
//   * W is the MN-major A operand ([64 k x 64 n] 128-byte-swizzled boxes, two per 64-wide K step),
//     x the K-major B operand (one [MX rows x 64 k] box per K step; rows past M read as zero);
//   * grid = 128-column strips x cluster ranks; rank r of a cluster takes K rows
//     [r*kchunk, (r+1)*kchunk) of its strip; one CTA per SM (TMEM);
//   * consecutive K steps go round-robin to NACC accumulators ([128 x MX] fp32 each): a chain of
//     dependent narrow MMAs into one accumulator would run at MMA latency, not at the weight
//     stream's rate; they are summed in fixed order;
//   * K ranks reduce through distributed shared memory: once every rank's MMAs are done (one split
//     cluster barrier), each epilogue thread (one weight column = one TMEM lane) pushes its
//     partial row with st.async into the owning rank's freed ring; the owner's 128 epilogue
//     threads add the partials in rank order (deterministic), apply rscale and bias and store
//     fp32 or fp16.
// Measured on B200 against the 128-row-tile kernels (CUDA graph, weights rotated through HBM):
// 4096 x 4096 at M = 16 / 32 / 64: 9.7 / 10.7 / 12.8 us (15.6 / 16.7 / 16.7); 1024 x 3072 at
// M = 8 / 32: 5.7 / 6.6 us (11.0 / 12.3). At M = 128 the result was mixed (faster at 4096 x 11008,
// slower at 768 x 3072 and 16384 x 1024), so M > 64 stays on the 128-row tiles.
// Warp 0 TMA producer, warp 1 TMEM allocation + MMA issue, warps 2-5 epilogue. Programmatic
// dependent launch; every mbarrier wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <atomic>
#include <mutex>
#include <unordered_map>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

// K steps (of 64 rows) each rank of the medium-M cluster keeps at least. Measured on B200 (CUDA
// graphs, weights rotated through HBM), 4 -> 2 -> 1: 64 x 1024 x 1024 7.6 -> 6.8 -> 6.8 us (2 -> 8
// ranks; 16 requested at 1, lowered to 8 by the residency check), 16 x 1024 x 1024 5.0 -> 4.7 ->
// 4.7, 64 x 768 x 768 9.1 -> 7.1 -> 6.3; shapes with long K unchanged (their ranks are capped by
// the CTAs that fit).
#ifndef G16_MIDM_MIN_STEPS
#define G16_MIDM_MIN_STEPS 1
#endif

namespace g16 {
namespace {

constexpr int kMdThreads = 192;
constexpr int kMdStrip = 128;                        // weight columns per CTA (UMMA M)
constexpr int kMdMaxCluster = 16;
constexpr uint32_t kMdWBoxBytes = kBK * 64 * 2;      // [64 k x 64 n] fp16 = 8 KiB
constexpr uint32_t kMdWBytes = 2 * kMdWBoxBytes;     // one K step of the strip: 16 KiB
constexpr int kMdMaxStages = 16;
constexpr uint32_t kMdTmemFreeBar = 1;               // warp 1 + epilogue warps: TMEM read
constexpr uint64_t kMdPushWaitNs = 3ull * kWaitLimitNs;  // > any chain of waits before a peer pushes

__host__ __device__ constexpr uint32_t md_stage_bytes(int mx) { return kMdWBytes + static_cast<uint32_t>(mx) * 128u; }
__host__ __device__ constexpr int md_nacc(int mx) { return 8; }  // 8 x MX <= 512 TMEM columns
__host__ __device__ constexpr uint32_t md_tmem_cols(int mx) {
  return md_nacc(mx) * mx <= 32 ? 32u : md_nacc(mx) * mx <= 64 ? 64u : md_nacc(mx) * mx <= 128 ? 128u
         : md_nacc(mx) * mx <= 256 ? 256u : 512u;
}
// Pushed partials: [csize][slice][MX + 4] fp32 per owner (the 16-byte pad keeps the owner's row
// reads free of bank conflicts); 128 rows in all.
__host__ __device__ constexpr uint32_t md_red_bytes(int mx) { return kMdStrip * (mx + 4) * 4u; }
__host__ __device__ constexpr size_t md_smem_bytes(int mx, int stages) {
  return 1024 + static_cast<size_t>(stages) * md_stage_bytes(mx) + (2 * kMdMaxStages + 4) * 8 + 16;
}

struct MidArgs {
  void* out;
  const float* bias;
  const float* rscale;
  int* status;
  int M, N, K;
  int kchunk;  // K rows per cluster rank (a multiple of 64)
  int stages;  // ring depth
  int act;     // epilogue activation (G16_ACT_*)
};

template <int MX, bool OUT_F16>
__global__ void __launch_bounds__(kMdThreads, 1)
gemm_midm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const MidArgs args) {
  constexpr int NACC = md_nacc(MX);
  constexpr uint32_t kStage = md_stage_bytes(MX);
  constexpr uint32_t kTmemCols = md_tmem_cols(MX);
  constexpr int kRow = MX + 4;  // pushed row stride (floats)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = args.stages;
  uint8_t* ring = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(S) * kStage);
  uint64_t* empty_bar = full_bar + kMdMaxStages;
  uint64_t* done_bar = empty_bar + kMdMaxStages;
  uint64_t* red_bar = done_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int csize = gridDim.x;
  // Uniform over the grid: every CTA returns before any barrier, TMEM allocation or shared access.
  if (S < 2 || S > kMdMaxStages || kMdStrip % csize != 0 ||
      static_cast<uint32_t>(S) * kStage < (csize > 1 ? md_red_bytes(MX) : 0u) ||
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
  const int rank = blockIdx.x;  // cluster rank: clusters run along x
  const int n0 = blockIdx.y * kMdStrip;
  const int kb0 = rank * args.kchunk;
  const int ke = min(args.K, kb0 + args.kchunk);
  const int nst = ke > kb0 ? (ke - kb0 + kBK - 1) / kBK : 0;
  const int slice = kMdStrip / csize;  // strip columns each rank finalises
  if (tid == 0) grid_launch_dependents();

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(red_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();  // cluster scope: peers complete bytes on red_bar
    if (csize > 1) mbar_arrive_expect_tx(red_bar, static_cast<uint32_t>(csize * slice * MX * 4));
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      grid_dependency_wait();  // x, W: possibly written by the preceding kernel
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_phase = 0;
      bool ok = true;
      for (int t = 0; t < nst; ++t) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[stage], kStage);
        armed |= 1u << stage;
        armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
        uint8_t* sw = ring + static_cast<size_t>(stage) * kStage;
        const int k = kb0 + t * kBK;
        tma_load_2d(sw, &tmap_w, &full_bar[stage], n0, k);
        tma_load_2d(sw + kMdWBoxBytes, &tmap_w, &full_bar[stage], n0 + 64, k);
        tma_load_2d(sw + kMdWBytes, &tmap_x, &full_bar[stage], k, 0);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
        for (int s = 0; s < S; ++s)
          if ((armed >> s) & 1u) mbar_wait(&full_bar[s], (armed_phase >> s) & 1u, nullptr);
      }
    }
    __syncwarp();
    if (csize > 1) cluster_arrive();  // every thread once: this role is done with the ring
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // D[n][m] += W[k][n] * x[m][k]: A = W (MN-major), B = x (K-major), M = 128, N = MX, K = 16.
      constexpr uint32_t idesc = idesc_f16_f32(kMdStrip, MX, /*b_mn_major=*/false, /*a_mn_major=*/true);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = 0; t < nst; ++t) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sw = smem_u32(ring + static_cast<size_t>(stage) * kStage);
        const uint32_t sx = sw + kMdWBytes;
#pragma unroll
        for (int j = 0; j < kBK / kUmmaK; ++j) {
          const int ks = t * (kBK / kUmmaK) + j;
          // A: K rows [16j, 16j + 16) of the two boxes (LBO = one box), 8-row groups 1 KiB apart.
          const uint64_t adesc = smem_desc_sw128(sw + j * (kUmmaK * 128), kMdWBoxBytes, 1024);
          // B: 128-byte rows of x, 8-row atoms 1 KiB apart, K steps of 32 bytes.
          const uint64_t bdesc = smem_desc_sw128(sx + j * (kUmmaK * 2), 16, 1024);
          umma_f16(tmem + static_cast<uint32_t>((ks % NACC) * MX), adesc, bdesc, idesc, ks >= NACC ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
      }
      umma_commit(done_bar);  // arrives once every issued MMA has completed
      // TMEM is freed below: every issued MMA must have finished writing it first (bounded).
      mbar_wait(done_bar, 0, nullptr);
    }
    __syncwarp();
    if (csize > 1) cluster_arrive();
    named_bar_sync(kMdTmemFreeBar, 160);  // the epilogue has read the accumulators
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  } else {
    // ---------------- epilogue: warps 2-5, thread = weight column nl = TMEM lane ----------------
    const int quarter = warp & 3;  // TMEM lanes [32 * (warp % 4), +32) belong to this warp
    const int nl = quarter * 32 + lane;
    grid_dependency_wait();  // rscale, bias, out
    bool got = mbar_wait(done_bar, 0, abort_flag);
    got = __all_sync(0xffffffffu, got);
    if (!got && lane == 0) {
      *abort_flag = 1;
      atomicExch(args.status, G16_ERR_TIMEOUT);
    }
    tc_fence_after();
    if (csize > 1) {
      cluster_arrive();  // this CTA's MMAs are done: its ring may take the peers' partials
      cluster_wait();
    }
    const int used = min(NACC, nst * (kBK / kUmmaK));  // accumulators that were written
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int owner = nl / slice;
    const int j = nl - owner * slice;
    const uint32_t rbar = map_cluster(smem_u32(red_bar), static_cast<uint32_t>(owner));
    const uint32_t rdst =
        map_cluster(smem_u32(reinterpret_cast<float*>(ring) + (rank * slice + j) * kRow), static_cast<uint32_t>(owner));
    const int n = n0 + nl;
    constexpr int kChunks = MX >= 32 ? MX / 32 : 1;
#pragma unroll 1
    for (int c = 0; c < kChunks; ++c) {
      float v[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = 0.f;
      if (got) {
        if constexpr (MX >= 32) {
          // two accumulators per wait (warp-uniform condition), added in accumulator order
#pragma unroll 1
          for (int a = 0; a < NACC; a += 2) {
            if (a >= used) break;
            const bool two = a + 1 < used;
            uint32_t d0[32], d1[32];
            __syncwarp();
            tmem_ld_32x32b_x32(t_lane + static_cast<uint32_t>(a * MX + c * 32), d0);
            if (two) tmem_ld_32x32b_x32(t_lane + static_cast<uint32_t>((a + 1) * MX + c * 32), d1);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] += __uint_as_float(d0[e]);
            if (two) {
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] += __uint_as_float(d1[e]);
            }
          }
        } else {
          // MX = 16: one load covers accumulators a and a + 1
#pragma unroll 1
          for (int a = 0; a < NACC; a += 2) {
            if (a >= used) break;
            uint32_t d[32];
            __syncwarp();
            tmem_ld_32x32b_x32(t_lane + static_cast<uint32_t>(a * MX), d);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] += __uint_as_float(d[e]);
            if (a + 1 < used) {
#pragma unroll
              for (int e = 0; e < 16; ++e) v[e] += __uint_as_float(d[16 + e]);
            }
          }
        }
      }
      constexpr int kCols = MX >= 32 ? 32 : 16;
      if (csize == 1) {
        // this CTA holds the whole K range: rows m across the warp's lanes are consecutive columns
        if (n < args.N) {
          const float b = args.bias != nullptr ? __ldg(args.bias + n) : 0.f;
#pragma unroll
          for (int e = 0; e < kCols; ++e) {
            const int m = c * 32 + e;
            if (m < args.M) {
              const float rs = args.rscale != nullptr ? __ldg(args.rscale + m) : 1.f;
              const float o = apply_act(fmaf(v[e], rs, b), args.act);
              if constexpr (OUT_F16) {
                reinterpret_cast<__half*>(args.out)[static_cast<size_t>(m) * args.N + n] = __float2half_rn(o);
              } else {
                reinterpret_cast<float*>(args.out)[static_cast<size_t>(m) * args.N + n] = o;
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < kCols / 4; ++q)
          st_async_v4(rdst + 4u * static_cast<uint32_t>(c * 32 + 4 * q), v[4 * q], v[4 * q + 1], v[4 * q + 2],
                      v[4 * q + 3], rbar);
      }
    }
    tc_fence_before();
    named_bar_arrive(kMdTmemFreeBar, 160);
    if (csize > 1) {
      // Finalise the owned columns [own0, own0 + slice): all 128 epilogue threads share the work,
      // thread t takes column jj = t % slice and every csize-th group of 4 rows from t / slice.
      const int t = tid - 64;
      const int jj = t % slice;
      const int grp = t / slice;  // 0 .. csize - 1
      const bool in = mbar_wait_cluster(red_bar, 0, kMdPushWaitNs);
      const int nn = n0 + rank * slice + jj;
      if (!in) {
        if (t == 0) {
          *abort_flag = 1;
          atomicExch(args.status, G16_ERR_TIMEOUT);
        }
      } else if (nn < args.N) {
        const float* red = reinterpret_cast<const float*>(ring);
        const float b = args.bias != nullptr ? __ldg(args.bias + nn) : 0.f;
#pragma unroll 1
        for (int m4 = grp; 4 * m4 < args.M; m4 += csize) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int q = 0; q < csize; ++q) {  // rank order: deterministic
            const float4 p = *reinterpret_cast<const float4*>(red + (q * slice + jj) * kRow + 4 * m4);
            acc.x += p.x;
            acc.y += p.y;
            acc.z += p.z;
            acc.w += p.w;
          }
          const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = 4 * m4 + e;
            if (m < args.M) {
              const float rs = args.rscale != nullptr ? __ldg(args.rscale + m) : 1.f;
              const float o = apply_act(fmaf(a4[e], rs, b), args.act);
              if constexpr (OUT_F16) {
                reinterpret_cast<__half*>(args.out)[static_cast<size_t>(m) * args.N + nn] = __float2half_rn(o);
              } else {
                reinterpret_cast<float*>(args.out)[static_cast<size_t>(m) * args.N + nn] = o;
              }
            }
          }
        }
      }
      // Every epilogue thread waited for this CTA's full set of pushed bytes above, so no peer
      // still writes into it when it leaves.
    }
  }
}

template <typename F>
cudaError_t md_ensure_attrs(F* kern, std::atomic<uint64_t>& done, int smem) {
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

struct MidPlan {
  int mx = 0, csize = 1, strips = 0, kchunk = 0, stages = 0;
  size_t smem = 0;
};

#ifndef G16_MIDM_STAGES
#define G16_MIDM_STAGES 6
#endif

MidPlan md_plan_shape(int M, int K, int N, int ctas) {
  MidPlan p;
  p.mx = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  p.strips = (N + kMdStrip - 1) / kMdStrip;
  // K ranks: a power of two (the 128 strip columns split evenly among owners), at most 16, with
  // at least G16_MIDM_MIN_STEPS K steps each, and strips x ranks within the CTAs that fit at once.
  int c = 1;
  while (2 * c <= kMdMaxCluster && 2 * c * p.strips <= ctas && K >= 2 * c * G16_MIDM_MIN_STEPS * kBK) c *= 2;
  int kchunk = (K + c - 1) / c;
  kchunk = (kchunk + kBK - 1) / kBK * kBK;
  p.csize = c;
  p.kchunk = kchunk;
  const uint32_t stage = md_stage_bytes(p.mx);
  int s = G16_MIDM_STAGES;
  while (s > 2 && md_smem_bytes(p.mx, s) > 227u * 1024u) --s;
  while (c > 1 && static_cast<uint32_t>(s) * stage < md_red_bytes(p.mx)) ++s;  // the ring takes the partials
  p.stages = s;
  p.smem = md_smem_bytes(p.mx, s);
  return p;
}

cudaLaunchConfig_t md_cfg(const MidPlan& p, cudaStream_t s, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(p.csize), static_cast<unsigned>(p.strips), 1);
  cfg.blockDim = dim3(kMdThreads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

// Plan for (M-class, K, N) on this device: halve the K ranks until every cluster is resident at
// once. Cached.
template <typename F>
int md_plan_for(F* kern, int M, int K, int N, const DeviceInfo& dev, MidPlan* out) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, MidPlan> cache;
  int devid = 0;
  cudaError_t e = cudaGetDevice(&devid);
  if (e != cudaSuccess) return cuda_fail(e);
  MidPlan p = md_plan_shape(M, K, N, dev.sm_count);
  const uint64_t key = (static_cast<uint64_t>(devid) << 58) ^ (static_cast<uint64_t>(p.mx) << 50) ^
                       (static_cast<uint64_t>(K) << 25) ^ static_cast<uint64_t>(N);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return G16_OK;
    }
  }
  while (true) {
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = md_cfg(p, nullptr, attr);
    int active = 0;
    e = cudaOccupancyMaxActiveClusters(&active, kern, &cfg);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      active = 0;
    }
    if (active >= p.strips || p.csize == 1) break;
    p = md_plan_shape(M, K, N, (p.csize / 2) * p.strips);
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = p;
  *out = p;
  return G16_OK;
}

template <int MX, bool OUT_F16>
int md_launch_t(const uint16_t* x16, const uint16_t* w, void* out, const float* bias, const float* rscale, int M,
                int K, int N, cudaStream_t s, const DeviceInfo& dev, int act) {
  static std::atomic<uint64_t> attr_done{0};
  auto kern = gemm_midm_kernel<MX, OUT_F16>;
  cudaError_t e = md_ensure_attrs(kern, attr_done, 227 * 1024);
  if (e != cudaSuccess) return cuda_fail(e);
  MidPlan p;
  int st = md_plan_for(kern, M, K, N, dev, &p);
  if (st != G16_OK) return st;
  if (p.mx != MX || p.smem > 227u * 1024u) return G16_ERR_ARG;
  CUtensorMap tx, tw;
  st = make_tmap_2d(&tx, x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(M), static_cast<uint64_t>(K),
                    MX, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  st = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                    kBK, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  MidArgs a{};
  a.out = out;
  a.bias = bias;
  a.rscale = rscale;
  a.status = device_status_ptr();
  if (a.status == nullptr) return G16_ERR_CUDA;
  a.M = M;
  a.N = N;
  a.K = K;
  a.kchunk = p.kchunk;
  a.stages = p.stages;
  a.act = act;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = md_cfg(p, s, attr);
  e = cudaLaunchKernelEx(&cfg, kern, tx, tw, a);
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

template <int MX>
int md_launch_m(const uint16_t* x16, const uint16_t* w, void* out, int out_dtype, const float* bias,
                const float* rscale, int M, int K, int N, cudaStream_t s, const DeviceInfo& dev, int act) {
  return out_dtype == G16_F16 ? md_launch_t<MX, true>(x16, w, out, bias, rscale, M, K, N, s, dev, act)
                              : md_launch_t<MX, false>(x16, w, out, bias, rscale, M, K, N, s, dev, act);
}

}  // namespace

int gemm_midm_ranks(int M, int K, int N, const DeviceInfo& dev) {
  if (M <= 0 || M > kMidMaxM || K <= 0 || N <= 0) return 0;
  return md_plan_shape(M, K, N, dev.sm_count).csize;
}

int launch_gemm_midm(const uint16_t* x16, const uint16_t* w, void* out, int out_dtype, const float* bias,
                     const float* rscale, int M, int K, int N, cudaStream_t s, const DeviceInfo& dev, int act) {
  if (M <= 0 || N <= 0) return G16_OK;
  if (M > kMidMaxM || K <= 0) return G16_ERR_UNSUPPORTED;
  if (M <= 16) return md_launch_m<16>(x16, w, out, out_dtype, bias, rscale, M, K, N, s, dev, act);
  if (M <= 32) return md_launch_m<32>(x16, w, out, out_dtype, bias, rscale, M, K, N, s, dev, act);
  return md_launch_m<64>(x16, w, out, out_dtype, bias, rscale, M, K, N, s, dev, act);
}

}  // namespace g16
