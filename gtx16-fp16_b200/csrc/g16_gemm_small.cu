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
//
// Grid split (GS, automatic plan with a workspace): a cluster holds at most 16 CTAs, and at most
// one cluster of 10 fits in a GPC, so an output of a handful of tiles with a long K
// (128 x 16384 x 1024: 8 tiles of 128 x 128) keeps most SMs idle under the cluster plan. In GS the
// S K chunks of a tile are independent CTAs of one wave (at most one CTA per SM, all resident):
//   * each writes its fp32 partial tile to the workspace, P[tile][chunk][128][BN], with TMA stores
//     of [32 x 32] boxes staged in shared memory, waits for them to complete and fences;
//   * then publishes a flag F[tile][chunk] (its own 128-byte line) carrying the tile's call tag
//     E[tile] + 1;
//   * lane s of one warp waits (acquire, bounded) until chunk s's flag carries the tag and then
//     fetches chunk s's part of this CTA's share (a contiguous 1/S of the tile's quads) with a bulk
//     copy; the CTA adds the S parts in chunk order (the same order and chunk bounds as the cluster
//     and workspace reductions, so the same bits), applies the epilogue and stores;
//   * chunk 0 then advances E[tile], so the next call's tag differs from every flag written so far.
// Tags make the workspace need no initial contents: stale flags never carry the current tag. The
// waits rely on all S CTAs of a tile being resident together (the plan checks the occupancy); a
// grid held back for longer than the wait limit, by another stream's kernels occupying SMs, ends
// with G16_ERR_TIMEOUT in the status word rather than hanging.
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
// The grid split in the automatic plan when a workspace is given (a build option for measuring it
// against the cluster plan).
#ifndef G16_SMALL_GS
#define G16_SMALL_GS 1
#endif
// Ring depth of the 128-wide tiles. Measured on B200 (CUDA graphs, operands rotated through HBM),
// 4 -> 5 stages: 128 x 16384 x 1024 13.8 -> 13.3 us, 2048 x 3072 x 1024 19.8 -> 19.3, 128 x 4096 x
// 4096 15.6 -> 15.0, 512 x 8192 x 1024 19.2 -> 18.8; 6 stages within the run-to-run spread of 5.
#ifndef G16_SMALL_STAGES128
#define G16_SMALL_STAGES128 5
#endif

namespace g16 {
namespace {

constexpr int kSmThreads = 192;
constexpr int kSmStagesDefault = 4;
constexpr uint32_t kSmABytes = kBM * kBK * 2;      // 16 KiB
constexpr uint32_t kSmBBoxBytes = kBK * 64 * 2;    // one [64 k x 64 n] box: 8 KiB
constexpr int kSmMaxCluster = 16;
constexpr uint64_t kSmPushWaitNs = 3ull * kWaitLimitNs;  // > any chain of waits before a peer pushes
// Grid split: workspace header of call tags E[kGsMaxTiles] (64-bit words) and chunk flags
// F[kGsMaxTiles][kGsMaxSplit], each flag a 64-bit word alone in a 128-byte line (the S CTAs of a
// tile poll every flag of the tile; flags sharing lines measured slower), then the partial tiles.
constexpr int kGsMaxTiles = 64;
constexpr int kGsMaxSplit = 32;  // one lane per chunk polls the flags
constexpr int kGsFlagWords = 16; // 128 bytes per flag
constexpr size_t kGsTagBytes = static_cast<size_t>(kGsMaxTiles) * 8;
constexpr size_t kGsHeaderBytes = kGsTagBytes + static_cast<size_t>(kGsMaxTiles) * kGsMaxSplit * kGsFlagWords * 8;
static_assert(kGsTagBytes % 128 == 0 && kGsHeaderBytes % 256 == 0, "flags in whole lines, partials 256-byte aligned");
// Flags store tag ^ salt, so memory left by other uses of the workspace (zeros, fills, float data)
// does not read as a current flag.
constexpr uint64_t kGsSalt = 0x9E3779B97F4A7C15ull;

template <int BN>
struct SmallGeo {
  static constexpr uint32_t kBBytes = kBK * BN * 2;
  static constexpr uint32_t kStageBytes = kSmABytes + kBBytes;
  // 64-wide tiles: a deeper ring, which also keeps the CTA at one per SM (two would share its
  // bandwidth)
  static constexpr int kStages = BN == 64 ? 6 : BN == 128 ? G16_SMALL_STAGES128 : kSmStagesDefault;
  static constexpr uint32_t kRingBytes = kStages * kStageBytes;
  // partials received by an owner: C x rpo rows x BN fp32, at most (128 + C - 1) rows
  static constexpr uint32_t kRecvBytes = (kBM + kSmMaxCluster) * BN * 4;
  static_assert(kRecvBytes <= kRingBytes, "the freed ring must hold an owner's partials");
  static constexpr size_t kSmemBytes = 1024 + kRingBytes + 256;
  // grid split, after the mainloop: staging buffers, then one tile's worth of partial quads
  static_assert(kBM * BN * 4 + kGsMaxSplit * 16 <= kRingBytes,
                "the freed ring must hold the grid split's staged tile and received quads");
};

struct SmallArgs {
  void* out;
  const float* bias;
  const float* rscale;
  float* partials;  // grid split: [tiles][S][128][BN] fp32
  uint64_t* tags;   // grid split: E[kGsMaxTiles], then the flags F[kGsMaxTiles][kGsMaxSplit]
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

// Grid-split epilogue, run by the four epilogue warps (threads 64..191) once the MMAs have drained.
// smem: the freed ring (1024-byte aligned); bar: an mbarrier initialised with count S; go: a shared
// word for the decision to reduce, so that all 128 threads take the same branch.
template <bool OUT_F16, int BN>
__device__ __forceinline__ void gs_epilogue(const SmallArgs& args, const CUtensorMap* tmap_p, uint8_t* smem,
                                            uint64_t* bar, volatile int* abort_flag, volatile int* go, uint32_t tmem,
                                            bool live, int warp, int lane, int S, int rank, int tile, int mt, int nt,
                                            uint64_t tag) {
  constexpr int kQ = kBM * BN / 4;  // float4 quads of one partial tile
  const int quarter = warp & 3;
  const int et = threadIdx.x - 64;
  // 1. Partial tile -> P[tile][rank] (row-major [128][BN] fp32) by TMA stores of [32 x 32] boxes.
  //    After each TMEM load a lane holds 32 columns of its row; it writes them as one 128-byte row
  //    of the box, 16-byte chunks in the 128-byte swizzle order (conflict-free), into the warp's own
  //    staging area (the whole tile fits the freed ring, so no buffer is reused).
  uint8_t* stg = smem + (warp - 2) * (BN * 128);  // this warp's 32 rows: BN / 32 boxes of 4 KiB
  const int prow = (tile * S + rank) * kBM + quarter * 32;
  // Two 32-column TMEM loads per wait (one round trip for both).
#pragma unroll 1
  for (int c = 0; c < BN / 32; c += 2) {
    uint32_t r[2][32];
    __syncwarp();
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(c * 32);
    tmem_ld_32x32b_x32(taddr, r[0]);
    tmem_ld_32x32b_x32(taddr + 32, r[1]);
    tmem_ld_wait();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint8_t* buf = stg + (c + h) * 4096;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 v = live ? make_uint4(r[h][4 * j], r[h][4 * j + 1], r[h][4 * j + 2], r[h][4 * j + 3])
                             : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = v;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmap_p, stg + c * 4096, c * 32, prow);
      tma_store_2d(tmap_p, stg + (c + 1) * 4096, (c + 1) * 32, prow);
      bulk_commit_group();
    }
  }
  // The stores are complete (not only read from shared memory) and visible at GPU scope before the
  // flag goes out (fence by the issuing thread, then the barrier; the flag store follows both).
  if (lane == 0) {
    bulk_wait_group0();
    fence_proxy_async_global();
    __threadfence();
  }
  named_bar_sync(1, 128);
  // 2. Publish this chunk's flag. Lane s then waits for chunk s's flag and at once fetches chunk
  //    s's share of this CTA's quads [q0, q1) with a bulk copy, so the hand-over overlaps the
  //    transfers; every lane s < S arrives on `bar` exactly once (with the bytes it expects).
  const int q0 = static_cast<int>(static_cast<long long>(rank) * kQ / S);
  const int q1 = static_cast<int>(static_cast<long long>(rank + 1) * kQ / S);
  const int nq = q1 - q0;
  float4* red = reinterpret_cast<float4*>(smem);  // [S][nq]; the staging areas are free again
  uint64_t* flags = args.tags + kGsMaxTiles + static_cast<size_t>(tile) * kGsMaxSplit * kGsFlagWords;
  if (warp == 2) {
    const uint64_t want = tag ^ kGsSalt;
    if (lane == 0) st_relaxed_gpu_u64(flags + rank * kGsFlagWords, want);
    bool ok = true;
    if (lane < S) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_gpu_u64(flags + lane * kGsFlagWords) != want) {
        if (globaltimer_ns() - t0 > kSmPushWaitNs) {
          ok = false;
          break;
        }
        __nanosleep(32);
      }
      if (ok && nq > 0) {
        fence_proxy_async_global();
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nq * 16));
        bulk_load(red + lane * nq,
                  reinterpret_cast<const float4*>(args.partials) + (static_cast<size_t>(tile) * S + lane) * kQ + q0,
                  static_cast<uint32_t>(nq * 16), bar);
      } else {
        mbar_arrive(bar);
      }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (lane == 0) {
      // Every chunk has read the tag (its flag carries it): advance it for the next call.
      if (rank == 0) st_relaxed_gpu_u64(args.tags + tile, tag);
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
      }
      *go = ok ? 1 : 0;
    }
  }
  named_bar_sync(1, 128);
  // Copies in flight land before anyone leaves, whatever the decision.
  const bool landed = mbar_wait(bar, 0, nullptr);
  if (!landed && et == 0) {
    *abort_flag = 1;
    atomicExch(args.status, G16_ERR_TIMEOUT);
  }
  if (*go == 0 || !landed) return;
  // 3. Add the S partials of each quad in chunk order; unscale, bias, activation, store.
  for (int i = et; i < nq; i += 128) {
    const int q = q0 + i;
    const int rl = q / (BN / 4);
    const int cl = (q - rl * (BN / 4)) * 4;
    const int orow = mt * kBM + rl;
    const int col = nt * BN + cl;
    if (orow >= args.M || col >= args.N) continue;
    float4 acc = red[i];
    int s = 1;
    for (; s + 8 <= S; s += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = red[(s + j) * nq + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
      }
    }
    for (; s < S; ++s) {
      const float4 v = red[s * nq + i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const float rs = args.rscale != nullptr ? __ldg(args.rscale + orow) : 1.f;
    const float4 b = args.bias != nullptr ? __ldg(reinterpret_cast<const float4*>(args.bias + col))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
    store4<OUT_F16>(args, orow, col, fmaf(acc.x, rs, b.x), fmaf(acc.y, rs, b.y), fmaf(acc.z, rs, b.z),
                    fmaf(acc.w, rs, b.w));
  }
}

// grid = (C, tiles); cluster (C, 1, 1) when C > 1 (GS: no cluster). blockIdx.x = K chunk = rank.
template <bool OUT_F16, int BN, bool GS>
__global__ void __launch_bounds__(kSmThreads, 1)
gemm_small_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                  const __grid_constant__ CUtensorMap tmap_p, const SmallArgs args) {
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
  volatile int* gs_go = abort_flag + 1;
  if (static_cast<uint32_t>(reinterpret_cast<const volatile uint8_t*>(gs_go + 1) - smem_raw) >
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
  const bool in_cluster = !GS && csize > 1;  // the K chunks of the tile reduce in the cluster
  // The next kernel may start its set-up now; it reads nothing this one writes before its own
  // grid dependency wait. Except for a grid split with row scales (fp32 activations, so the next
  // kernel is most likely the next row-rescale pass): measured on B200 (CUDA graphs of fp32
  // mm_t calls), an early start there cost 128 x 16384 x 1024 21.8 against 18.3 us, 256 x 8192 x
  // 512 16.4 against 13.8; back-to-back fp16 grid splits gain from it (10.6 -> 10.0 us).
  if (threadIdx.x == 0 && (!GS || args.rscale == nullptr)) grid_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSmStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(red_bar, GS ? csize : 1);  // GS: one arrival per chunk's bulk copy
    *abort_flag = 0;
    fence_barrier_init();  // cluster scope: peers push into red_bar after the cluster barrier
    if (in_cluster) mbar_arrive_expect_tx(red_bar, static_cast<uint32_t>(csize * own_rows * BN * 4));
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
    if (in_cluster) cluster_arrive();  // every thread of the cluster arrives once
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
    if (in_cluster) cluster_arrive();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;                 // TMEM lane quarter this warp may access
    const int r_local = quarter * 32 + lane;      // tile row of this lane
    const int row = mt * kBM + r_local;
    grid_dependency_wait();  // bias, rscale, out
    // Grid split: this call's tag for the tile, read while the mainloop runs (warp 2 publishes it).
    uint64_t gs_tag = 0;
    if (GS && warp == 2) {
      if (lane == 0) gs_tag = ld_relaxed_gpu_u64(args.tags + tile) + 1;
      gs_tag = __shfl_sync(0xffffffffu, gs_tag, 0);
    }
    bool got = mbar_wait(done_bar, 0, abort_flag);
    got = __all_sync(0xffffffffu, got);
    if (!got && lane == 0) {
      *abort_flag = 1;
      atomicExch(args.status, G16_ERR_TIMEOUT);
    }
    const bool live = got && kb1 > kb0;
    tc_fence_after();
    if constexpr (GS) {
      gs_epilogue<OUT_F16, BN>(args, &tmap_p, smem, red_bar, abort_flag, gs_go, tmem, live, warp, lane, csize, rank,
                               tile, mt, nt, gs_tag);
    } else if (csize == 1) {
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

// gs_ws != nullptr: grid split over csize chunks with the workspace gs_ws (header, then partials);
// otherwise clusters of csize.
template <bool OUT_F16, int BN>
int launch_small_t(const uint16_t* a16, const uint16_t* b16, void* out, const float* bias, const float* rscale, int M,
                   int K, int N, int csize, cudaStream_t s, int act, void* gs_ws) {
  static std::atomic<uint64_t> attr_done{0}, attr_done_gs{0};
  const bool gs = gs_ws != nullptr;
  auto kern = gs ? gemm_small_kernel<OUT_F16, BN, true> : gemm_small_kernel<OUT_F16, BN, false>;
  cudaError_t e = ensure_small_attrs(kern, gs ? attr_done_gs : attr_done, static_cast<int>(SmallGeo<BN>::kSmemBytes));
  if (e != cudaSuccess) return cuda_fail(e);
  SmallArgs args{};
  if (gs) {
    args.tags = static_cast<uint64_t*>(gs_ws);
    args.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(gs_ws) + kGsHeaderBytes);
  }
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
  // Grid split: the partial tiles P as a [tiles * S * 128, BN] fp32 matrix, stored in [32 x 32]
  // boxes with the 128-byte swizzle. Unused otherwise (B's map stands in).
  CUtensorMap tp = tb;
  if (gs) {
    st = make_tmap_2d(&tp, args.partials, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                      static_cast<uint64_t>(m_tiles) * args.n_tiles * csize * kBM, static_cast<uint64_t>(BN), 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != G16_OK) return st;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(csize), static_cast<unsigned>(m_tiles * args.n_tiles), 1);
  cfg.blockDim = dim3(kSmThreads, 1, 1);
  cfg.dynamicSmemBytes = SmallGeo<BN>::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  // Programmatic dependent launch: a launch's set-up overlaps the previous kernel's tail.
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(csize);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = gs ? 1 : 2;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tp, args);
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
  auto kern = gemm_small_kernel<true, BN, false>;  // both output types have the same resources
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

// CTAs of the grid-split kernel that can be resident at once on this device (0 if none).
template <int BN>
int gs_resident_ctas(const DeviceInfo& dev) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;  // device -> resident CTAs
  int devid = 0;
  if (cudaGetDevice(&devid) != cudaSuccess) return 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(devid);
    if (it != cache.end()) return it->second;
  }
  static std::atomic<uint64_t> attr_done{0};
  auto kern = gemm_small_kernel<true, BN, true>;
  int per_sm = 0;
  if (ensure_small_attrs(kern, attr_done, static_cast<int>(SmallGeo<BN>::kSmemBytes)) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kSmThreads, SmallGeo<BN>::kSmemBytes) !=
          cudaSuccess) {
    (void)cudaGetLastError();
    per_sm = 0;
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[devid] = per_sm * dev.sm_count;
  return per_sm * dev.sm_count;
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
  // Grid split (used when the caller gives a workspace): the K chunks as independent CTAs of one
  // resident wave, towards one CTA per SM with chunks of >= kmin k-blocks, 128-wide tiles unless
  // 64-wide ones put 1.25x as many CTAs to work; taken when that is at least 1.25x the cluster
  // plan's CTAs.
  // Measured on B200 (CUDA graphs, operands rotated through HBM), cluster plan -> grid split:
  // 128 x 16384 x 1024 17.9 -> 13.7 us, 256 x 8192 x 512 13.2 -> 10.1, 96 x 12288 x 768
  // 13.5 -> 10.9, 128 x 16384 x 256 (64-wide) 10.4 -> 9.8.
  if (G16_SMALL_GS && p.bn != 0) {
    auto gs_chunks = [&](int gbn) {
      const int gtiles = m_tiles * ((N + gbn - 1) / gbn);
      if (gtiles > kGsMaxTiles) return 0;
      const int kmin = gtiles < 32 ? 4 : 16;
      int S = std::min(std::min(kGsMaxSplit, dev.sm_count / gtiles), std::max(1, kblocks / kmin));
      if (S < 2) return 0;
      const int per = (kblocks + S - 1) / S;
      S = (kblocks + per - 1) / per;  // no empty chunks
      const int resident = gbn == 64 ? gs_resident_ctas<64>(dev) : gs_resident_ctas<128>(dev);
      return (S >= 2 && gtiles * S <= resident) ? S : 0;
    };
    const int s128 = gs_chunks(128), s64 = G16_SMALL_BN64 ? gs_chunks(64) : 0;
    const int c128 = s128 * m_tiles * ((N + 127) / 128), c64 = s64 * m_tiles * ((N + 63) / 64);
    const int gbn = 4 * c64 >= 5 * c128 ? 64 : 128;  // 64-wide tiles re-read A twice as often
    const int S = gbn == 64 ? s64 : s128;
    const int ctas = p.csize * m_tiles * ((N + p.bn - 1) / p.bn);
    if (S >= 2 && 4 * std::max(c64, c128) >= 5 * ctas) {
      p.gs_bn = gbn;
      p.gs_split = S;
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = p;
  return p;
}

size_t small_gs_workspace_bytes(const SmallPlan& p, int M, int N) {
  if (p.gs_split < 2) return 0;
  const size_t tiles = static_cast<size_t>((M + kBM - 1) / kBM) * ((N + p.gs_bn - 1) / p.gs_bn);
  return kGsHeaderBytes + tiles * p.gs_split * kBM * p.gs_bn * sizeof(float);
}

int launch_gemm_small_gs(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                         const float* rscale, int M, int K, int N, const SmallPlan& p, void* ws, size_t ws_bytes,
                         cudaStream_t s, int act) {
  if (p.gs_split < 2 || p.gs_split > kGsMaxSplit) return G16_ERR_UNSUPPORTED;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + p.gs_bn - 1) / p.gs_bn);
  if (tiles > kGsMaxTiles) return G16_ERR_UNSUPPORTED;
  if (ws == nullptr || ws_bytes < small_gs_workspace_bytes(p, M, N)) return G16_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return G16_ERR_ALIGN;
  const int S = p.gs_split;
  if (p.gs_bn == 64)
    return out_dtype == G16_F16 ? launch_small_t<true, 64>(a16, b16, out, bias, rscale, M, K, N, S, s, act, ws)
                                : launch_small_t<false, 64>(a16, b16, out, bias, rscale, M, K, N, S, s, act, ws);
  if (p.gs_bn == 128)
    return out_dtype == G16_F16 ? launch_small_t<true, 128>(a16, b16, out, bias, rscale, M, K, N, S, s, act, ws)
                                : launch_small_t<false, 128>(a16, b16, out, bias, rscale, M, K, N, S, s, act, ws);
  if (p.gs_bn == 256)
    return out_dtype == G16_F16 ? launch_small_t<true, 256>(a16, b16, out, bias, rscale, M, K, N, S, s, act, ws)
                                : launch_small_t<false, 256>(a16, b16, out, bias, rscale, M, K, N, S, s, act, ws);
  return G16_ERR_UNSUPPORTED;
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
    return out_dtype == G16_F16 ? launch_small_t<true, 64>(a16, b16, out, bias, rscale, M, K, N, c, s, act, nullptr)
                                : launch_small_t<false, 64>(a16, b16, out, bias, rscale, M, K, N, c, s, act, nullptr);
  if (out_dtype == G16_F16) {
    return bn == 128 ? launch_small_t<true, 128>(a16, b16, out, bias, rscale, M, K, N, c, s, act, nullptr)
                     : launch_small_t<true, 256>(a16, b16, out, bias, rscale, M, K, N, c, s, act, nullptr);
  }
  return bn == 128 ? launch_small_t<false, 128>(a16, b16, out, bias, rscale, M, K, N, c, s, act, nullptr)
                   : launch_small_t<false, 256>(a16, b16, out, bias, rscale, M, K, N, c, s, act, nullptr);
}

}  // namespace g16
