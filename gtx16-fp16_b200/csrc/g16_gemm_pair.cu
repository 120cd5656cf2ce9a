// Tensor-core GEMM on CTA pairs: out[M,N] = (A @ B) * rscale[row] + bias[col], A [M,K] fp16
// K-major, B [K,N] fp16 N-major, fp32 accumulation in TMEM. Persistent, one cluster of 2 CTAs
// (2 SMs) per 256 x 256 output tile:
//   * each CTA of the pair loads its 128 rows of A and its 128-column half of B per 64-wide K step
//     (32 KiB, against 48 KiB for a 128 x 256 tile on one SM: the operand bytes per FLOP drop by a
//     third, and the single-SM kernel is close to the per-SM operand-load limit);
//   * the leader CTA (rank 0 of the pair) issues tcgen05.mma.cta_group::2 (M = 256, N = 256,
//     K = 16), which reads A and B from both CTAs' shared memory and accumulates each CTA's 128
//     rows in its own TMEM; commits arrive on both CTAs' barriers (tcgen05.commit multicast);
//   * every TMA load completes its bytes on the leader's barrier (the .cta_group::2 form of the
//     tensor load, no multicast); each CTA's epilogue reads its own TMEM and releases the
//     accumulator on the leader's barrier.
// Roles per CTA: warp 0 TMA producer, warp 1 TMEM allocation (collective for the pair) and, in the
// leader, the MMA issuer; warps 2-5 epilogue. Two 256-column accumulators double-buffer the
// epilogue against the next tile's MMAs. The epilogue stages each warp's 32 rows x 128 bytes
// (32 fp32 or 64 fp16 columns) in a 128-byte-swizzled shared buffer (two per warp, alternating) and
// writes it with a TMA tile store, so global writes are whole lines and ragged edges are clipped
// by the tensor map. Every mbarrier wait is bounded. Results are bitwise equal to the single-CTA
// kernel's (same K order per output element).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <atomic>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

#ifndef G16_PAIR_BN
#define G16_PAIR_BN 256
#endif
#ifndef G16_PAIR_EPIW
#define G16_PAIR_EPIW 0
#endif

namespace g16 {
namespace {

constexpr int kPrThreads = 192;
constexpr uint32_t kPrABytes = kBM * kBK * 2;       // this CTA's 128 rows x 64 k: 16 KiB
constexpr uint32_t kPrBBoxBytes = kBK * 64 * 2;     // [64 k x 64 n]: 8 KiB
// Rasterisation: 8 pair-rows (2048 rows) per group. Measured against 4 and 16 at 16384^3,
// 8192 x 8192 x 16384, 4096 x 4096 x 16384 and 16384 x 16384 x 8192: best or within the
// run-to-run spread on each.
constexpr int kPrGroupM = 8;
// Programmatic dependent launch of plain-output calls (a build option while it is measured).
#ifndef G16_PAIR_PDL
#define G16_PAIR_PDL 1
#endif
constexpr uint32_t kPrEpiBufBytes = 32 * 128;             // one warp's 32 rows x 128 bytes

// Tile width BN (the MMA's N): 256 (the default: fewest operand bytes per FLOP) or 128 (twice the
// tiles, for outputs whose 256 x 256 tiles would leave most SMs idle). Each CTA of the pair holds
// BN / 2 columns of B per K step; the ring keeps about the same bytes in flight at either width.
//
// fp32 activations (A_F32): A is fp32 in global memory and every CTA converts its own rows. TMA
// loads each K step's [128 x 64] fp32 block (two [128 x 32] boxes, 128-byte swizzle) into a
// three-deep staging ring; four converter warps (one thread per row) scale it by the row's exact
// power-of-two reciprocal 1/S (from the row-amax pre-pass), round it to fp16 exactly as the
// rowscale kernel does, and write the 128-byte-swizzled K-major operand into a two-deep ring of
// its own, then arrive on the leader's barrier; B has its own TMA ring. The fp16 copy of x never
// exists in global memory, and the operand bits equal rowscale's, so results equal the two-pass
// form bit for bit.
//
// Epilogue width EPIW: 4 warps (one per TMEM lane quarter) or 8 (two per quarter, each taking half
// of the tile's columns), for tiles whose few K steps leave too little mainloop time to hide a
// 4-warp epilogue (short K, fp32 output).
template <int BN, bool A_F32 = false, int EPIW = 4>
struct PairGeo {
  static_assert(BN == 128 || BN == 256, "pair tile width");
  static_assert(EPIW == 4 || (EPIW == 8 && !A_F32), "epilogue warps");
  static constexpr int kThreads = 64 + 32 * EPIW + (A_F32 ? 128 : 0);  // + 4 converter warps
  static constexpr uint32_t kEpiBytes = EPIW * 2 * kPrEpiBufBytes;     // two buffers per epilogue warp
  static constexpr int kBBoxes = BN / 128;                         // [64 k x 64 n] boxes per CTA
  static constexpr uint32_t kBBytes = kBBoxes * kPrBBoxBytes;      // this CTA's half of B
  // TMA ring stage: A and B (fp16 A), or B alone (fp32 A: the converted A has a ring of its own)
  static constexpr uint32_t kStageBytes = A_F32 ? kBBytes : kPrABytes + kBBytes;
  static constexpr int kStages = A_F32 ? (BN == 256 ? 4 : 8) : (BN == 256 ? (EPIW == 8 ? 5 : 6) : 8);
  static constexpr int kA16Stages = A_F32 ? 4 : 0;                 // converted fp16 A ring
  static constexpr int kStgStages = A_F32 ? 2 : 0;                 // fp32 A staging ring
  static constexpr uint32_t kStgBytes = 2 * kBM * 32 * 4;          // [128 x 64] fp32: 32 KiB
  static constexpr uint32_t kTmemCols = 2 * BN;                    // two accumulators
  static constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + kA16Stages * kPrABytes +
                                       kStgStages * kStgBytes + kEpiBytes + 256;
  static_assert(kSmemBytes <= 227 * 1024, "pair GEMM shared memory");
};

// Output tensor maps: one for a plain GEMM, or one per destination of the multi-GPU scatter (each
// [M, col0 + N] of a [.., ldc] buffer; this GEMM's tile lands at column col0 of every one).
constexpr int kPrMaxDst = G16_SCATTER_MAX_DST;
struct PairDst {
  CUtensorMap m[kPrMaxDst];
  int ndst;
  int col0;
  // NVLink multicast mode (ndst == 0): the output rows [M, ldc] behind one multicast address; each
  // 128-byte row segment is written once with multimem.st and reaches every GPU's copy.
  uint64_t mc;
  long long ldc;
  // Multicast mode only, optional (0: none): a 32-bit counter behind an NVLink multicast address.
  // Each CTA adds 1 to it on every GPU once all its stores are issued and fenced, so a GPU whose
  // counter has grown by (CTAs per rank x ranks) holds every rank's tiles.
  uint64_t mc_flag;
};

struct PairArgs {
  void* out;
  const float* bias;
  const float* rscale;
  const float* rscale_inv;  // A_F32 only: 1 / rscale, the factor the converters apply
  int* status;
  int M, N, K;
  int m2_tiles, n_tiles, units, kblocks;  // tiles of 256 x BN
  int act;                                // epilogue activation (G16_ACT_*)
};

__device__ __forceinline__ void pair_coords(const PairArgs& a, int u, int* mt2, int* nt) {
  const int per_group = kPrGroupM * a.n_tiles;
  const int g = u / per_group;
  const int first = g * kPrGroupM;
  const int gsize = min(kPrGroupM, a.m2_tiles - first);
  const int in_g = u - g * per_group;
  *mt2 = first + in_g % gsize;
  *nt = in_g / gsize;
}

// Epilogue math for 32 accumulator columns of one row: acc * rscale + bias, packed as 4 (fp16) or
// 8 (fp32) 16-byte chunks of the row segment.
template <bool OUT_F16>
__device__ __forceinline__ void pair_pack32(const PairArgs& a, int col0, float rs, const uint32_t (&r)[32], uint4* out) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int col = col0 + 8 * g;
    float o[8];
    if (a.bias != nullptr && col < a.N) {  // N % 8 == 0: 8 columns are all in or all out
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(a.bias + col));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(a.bias + col + 4));
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = fmaf(__uint_as_float(r[8 * g + j]), rs, bb[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __uint_as_float(r[8 * g + j]) * rs;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = apply_act(o[j], a.act);
    if constexpr (OUT_F16) {
      __half2 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
      out[g] = *reinterpret_cast<const uint4*>(h);
    } else {
      out[2 * g] = make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3]));
      out[2 * g + 1] =
          make_uint4(__float_as_uint(o[4]), __float_as_uint(o[5]), __float_as_uint(o[6]), __float_as_uint(o[7]));
    }
  }
}

// grid = 2 * pairs CTAs, clusters of 2 along x: CTA 2p + q is rank q of pair p.
template <bool OUT_F16, int BN, bool A_F32, int EPIW>
__global__ void __launch_bounds__(PairGeo<BN, A_F32, EPIW>::kThreads, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 const __grid_constant__ PairDst dst,
                 const PairArgs args) {
  using G = PairGeo<BN, A_F32, EPIW>;
  constexpr int kPrStages = G::kStages;
  constexpr uint32_t kPrStageBytes = G::kStageBytes;
  constexpr int kStg = G::kStgStages;
  constexpr int kA16 = G::kA16Stages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;                                    // all offsets below 1024-byte aligned
  uint8_t* a16r = smem + kPrStages * kPrStageBytes;        // converted A ring (A_F32)
  uint8_t* stg = a16r + kA16 * kPrABytes;                  // fp32 A staging (A_F32)
  uint8_t* epi_stage = stg + kStg * G::kStgBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_stage + G::kEpiBytes);
  uint64_t* empty_bar = full_bar + kPrStages;
  uint64_t* tfull_bar = empty_bar + kPrStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* stg_full = drain_bar + 1;                      // kStg each (A_F32)
  uint64_t* stg_empty = stg_full + kStg;
  uint64_t* a16_full = stg_empty + kStg;                   // kA16 each (A_F32)
  uint64_t* a16_empty = a16_full + kA16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a16_empty + kA16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Uniform over the grid: every CTA returns before any barrier, cluster barrier or allocation.
  if (static_cast<uint32_t>(reinterpret_cast<const volatile uint8_t*>(abort_flag + 1) - smem_raw) >
      dynamic_smem_bytes()) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
      grid_dependency_wait();
      atomicExch(args.status, G16_ERR_ARG);
    }
    return;
  }
  // The next kernel may start its set-up now; it reads nothing this one writes before its own wait.
  // No early griddepcontrol.launch_dependents: the next kernel starts only when this one ends.
  // Letting it start early measured slower where a rowscale pass follows (its CTAs then take the
  // SMs the last wave frees): fp32 mm_t 65536 x 768 x 768 128.0 -> 135.3 us.

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t q = cluster_ctarank();  // rank in the pair (cluster of 2)
  const bool leader = q == 0;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  constexpr uint16_t kPairMask = 0x3;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPrStages; ++s) {
      mbar_init(&full_bar[s], 1);   // the leader's producer arrives (expecting both CTAs' TMA bytes)
      mbar_init(&empty_bar[s], 1);  // the leader's MMA commit
    }
    for (int j = 0; j < kStg; ++j) {
      mbar_init(&stg_full[j], 1);   // this CTA's producer (fp32 A bytes)
      mbar_init(&stg_empty[j], 4);  // this CTA's converter warps
    }
    for (int j = 0; j < kA16; ++j) {
      mbar_init(&a16_full[j], 2 * 4);  // the converter warps of both CTAs (the leader's is used)
      mbar_init(&a16_empty[j], 1);     // the leader's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * EPIW);  // both CTAs' epilogue warps (the leader's is used)
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    for (int d = 0; d < dst.ndst; ++d) tma_prefetch_desc(&dst.m[d]);  // none in multicast mode
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, G::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barrier initialisation and the pair's TMEM allocation, visible to both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch (plain outputs): the set-up above may overlap the preceding
  // kernel's tail; no global memory is touched before it has completed.
  grid_dependency_wait();

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_phase = 0;
      int sj = 0;                  // A_F32: staging slot
      uint32_t sphase = 0;
      uint32_t sarmed = 0, sarmed_phase = 0;
      bool ok = true;
      for (int u = pair; u < args.units && ok; u += pairs) {
        int mt2, nt;
        pair_coords(args, u, &mt2, &nt);
        const int row0 = mt2 * 2 * kBM + static_cast<int>(q) * kBM;
        for (int kb = 0; kb < args.kblocks; ++kb) {
          if constexpr (A_F32) {
            // this CTA's fp32 rows of the K step, two [128 x 32] boxes, on its own staging barrier
            if (!mbar_wait(&stg_empty[sj], sphase ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&stg_full[sj], G::kStgBytes);
            sarmed |= 1u << sj;
            sarmed_phase = (sarmed_phase & ~(1u << sj)) | (sphase << sj);
            uint8_t* sdst = stg + sj * G::kStgBytes;
            tma_load_2d(sdst, &tmap_a, &stg_full[sj], kb * kBK, row0);
            tma_load_2d(sdst + G::kStgBytes / 2, &tmap_a, &stg_full[sj], kb * kBK + 32, row0);
            if (++sj == kStg) { sj = 0; sphase ^= 1u; }
          }
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) {
            mbar_arrive_expect_tx(&full_bar[stage], 2 * kPrStageBytes);
            armed |= 1u << stage;
            armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t bar = map_cluster(smem_u32(&full_bar[stage]), 0);
          uint8_t* sa = ring + stage * kPrStageBytes;
          uint8_t* sb = A_F32 ? sa : sa + kPrABytes;
          if constexpr (!A_F32) tma_load_2d_pair(sa, &tmap_a, bar, kb * kBK, row0);
#pragma unroll
          for (int j = 0; j < G::kBBoxes; ++j)
            tma_load_2d_pair(sb + j * kPrBBoxBytes, &tmap_b, bar, nt * BN + static_cast<int>(q) * (BN / 2) + 64 * j,
                             kb * kBK);
          if (++stage == kPrStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
        // The leader's full barriers count both CTAs' bytes: wait for every armed stage, so no
        // copy is still landing when the pair passes its final cluster barrier; the same for this
        // CTA's armed fp32 staging slots.
        for (int j = 0; j < kStg; ++j)
          if ((sarmed >> j) & 1u) mbar_wait(&stg_full[j], (sarmed_phase >> j) & 1u, nullptr);
        for (int s = 0; s < kPrStages; ++s)
          if ((armed >> s) & 1u) mbar_wait(&full_bar[s], (armed_phase >> s) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * kBM, BN, /*b_mn_major=*/true);
      int stage = 0;
      uint32_t phase = 0;
      int ai = 0;                  // A_F32: converted-A slot
      uint32_t aphase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = pair; u < args.units && ok; u += pairs) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < args.kblocks; ++kb) {
          bool full = mbar_wait(&full_bar[stage], phase, abort_flag);
          // A_F32: the converters of both CTAs arrive with release.cluster after writing the operand
          if constexpr (A_F32) full = full && mbar_wait_acq_cluster(&a16_full[ai], aphase, abort_flag);
          if (!full) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = A_F32 ? smem_u32(a16r + ai * kPrABytes) : smem_u32(ring + stage * kPrStageBytes);
          const uint32_t sb = A_F32 ? smem_u32(ring + stage * kPrStageBytes) : sa + kPrABytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // A: K-major, 128-byte rows, 8-row atoms 1024 B apart (SBO); K steps of 32 B.
            const uint64_t adesc = smem_desc_sw128(sa + k * (kUmmaK * 2), 16, 1024);
            // B: N-major, 64-column boxes 8 KiB apart (LBO), 8-row k groups 1024 B (SBO).
            const uint64_t bdesc = smem_desc_sw128(sb + k * (kUmmaK * 128), kPrBBoxBytes, 1024);
            umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty_bar[stage], kPairMask);
          if (++stage == kPrStages) { stage = 0; phase ^= 1u; }
          if constexpr (A_F32) {
            umma_commit_pair(&a16_empty[ai], kPairMask);
            if (++ai == kA16) { ai = 0; aphase ^= 1u; }
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull_bar[acc], kPairMask);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(args.status, G16_ERR_TIMEOUT);
      }
      umma_commit_pair(drain_bar, kPairMask);  // every issued MMA complete, in both CTAs
    }
  } else if (warp < 2 + EPIW) {
    // ---------------- epilogue (warps 2 .. 1 + EPIW, both CTAs) ----------------
    const int quarter = warp & 3;
    // with 8 warps, the two warps of a lane quarter take one half of the tile's columns each
    constexpr int kSpan = BN / (EPIW / 4);
    const int cbeg = ((warp - 2) >> 2) * kSpan;
    const int r_local = quarter * 32 + lane;
    const uint32_t tempty_leader[2] = {map_cluster(smem_u32(&tempty_bar[0]), 0),
                                       map_cluster(smem_u32(&tempty_bar[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t nbuf = 0;  // staging buffers used so far by this warp (alternating)
    uint8_t* my_stage = epi_stage + (warp - 2) * 2 * kPrEpiBufBytes;
    constexpr int kCols = OUT_F16 ? 64 : 32;  // columns per 128-byte row segment
    for (int u = pair; u < args.units; u += pairs) {
      int mt2, nt;
      pair_coords(args, u, &mt2, &nt);
      bool got = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag);
      got = __all_sync(0xffffffffu, got);
      if (!got) {
        if (lane == 0) {
          *abort_flag = 1;
          atomicExch(args.status, G16_ERR_TIMEOUT);
        }
        break;
      }
      tc_fence_after();
      const int row = mt2 * 2 * kBM + static_cast<int>(q) * kBM + r_local;
      const float rs = (args.rscale != nullptr && row < args.M) ? __ldg(args.rscale + row) : 1.f;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int y = mt2 * 2 * kBM + static_cast<int>(q) * kBM + quarter * 32;  // the warp's first row
#pragma unroll 1
      for (int c0 = cbeg; c0 < cbeg + kSpan; c0 += kCols, ++nbuf) {
        const int gcol = nt * BN + c0;
        uint4 packed[8];
#pragma unroll
        for (int h = 0; h < kCols / 32; ++h) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_row + c0 + h * 32, r);
          tmem_ld_wait();
          pair_pack32<OUT_F16>(args, gcol + h * 32, rs, r, packed + (OUT_F16 ? 4 : 8) * h);
        }
        uint8_t* buf = my_stage + (nbuf & 1u) * kPrEpiBufBytes;
        if (lane == 0) bulk_wait_group_read1();  // the store that last read `buf` has read it
        __syncwarp();
        // this lane's row: 8 chunks of 16 bytes, swizzled by row (the tensor map's 128-byte swizzle)
#pragma unroll
        for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = packed[j];
        if (dst.ndst > 0) {
          fence_proxy_async_smem();  // staged rows -> visible to the TMA engine
          __syncwarp();
          if (lane == 0) {
            if (y < args.M && gcol < args.N)
              for (int d = 0; d < dst.ndst; ++d) tma_store_2d(&dst.m[d], buf, dst.col0 + gcol, y);
            bulk_commit_group();
          }
        } else {
          // Multicast: 8 lanes per 128-byte row segment, 4 rows per instruction, 8 passes.
          __syncwarp();
          constexpr int kElems = OUT_F16 ? 8 : 4;  // elements per 16-byte chunk
          constexpr int kEsz = OUT_F16 ? 2 : 4;
          const int c = lane & 7;
          const int col = gcol + c * kElems;  // N % 8 == 0: a chunk is wholly inside or outside
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3);
            const uint4 v = *reinterpret_cast<const uint4*>(buf + r * 128 + ((c ^ (r & 7)) << 4));
            const int grow = y + r;
            if (grow < args.M && col < args.N)
              multimem_st_v4(dst.mc + (static_cast<uint64_t>(grow) * static_cast<uint64_t>(dst.ldc) +
                                       static_cast<uint64_t>(dst.col0 + col)) * kEsz, v);
          }
          __syncwarp();  // the buffer is read before the next pass rewrites it
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  if constexpr (A_F32) {
    if (warp >= 2 + EPIW) {
      // ---------------- converters (warps 6..9, both CTAs): fp32 A -> scaled fp16 operand ----------------
      const int ct = threadIdx.x - (2 + EPIW) * 32;  // this thread's row of the CTA's 128
      const uint32_t rsw = static_cast<uint32_t>(ct & 7);
      const uint32_t a16_full_leader0 = map_cluster(smem_u32(&a16_full[0]), 0);
      int ai = 0, sj = 0;
      uint32_t aphase = 0, sphase = 0;
      for (int u = pair; u < args.units; u += pairs) {
        int mt2, nt;
        pair_coords(args, u, &mt2, &nt);
        const int row = mt2 * 2 * kBM + static_cast<int>(q) * kBM + ct;
        const float inv = row < args.M ? __ldg(args.rscale_inv + row) : 1.f;
        bool ok = true;
        for (int kb = 0; kb < args.kblocks; ++kb) {
          ok = mbar_wait(&stg_full[sj], sphase, abort_flag) && mbar_wait(&a16_empty[ai], aphase ^ 1u, abort_flag);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          // row ct: staged as two [128 x 32] fp32 boxes, chunk c (4 floats) of a row at
          // ((c ^ (row & 7)) << 4); the operand row holds 8 chunks of 8 fp16 at ((c ^ (row & 7)) << 4)
          const uint8_t* srow = stg + sj * G::kStgBytes + ct * 128;
          uint8_t* drow = a16r + ai * kPrABytes + ct * 128;
#pragma unroll
          for (int c16 = 0; c16 < 8; ++c16) {
            const uint8_t* sbox = srow + (c16 >> 2) * (G::kStgBytes / 2);
            const uint32_t f0 = 2u * static_cast<uint32_t>(c16 & 3);
            float4 lo = *reinterpret_cast<const float4*>(sbox + ((f0 ^ rsw) << 4));
            float4 hi = *reinterpret_cast<const float4*>(sbox + (((f0 + 1u) ^ rsw) << 4));
            if (inv != 1.f) {  // the rowscale kernel's arithmetic: x * (1/S), then round to fp16
              lo.x *= inv; lo.y *= inv; lo.z *= inv; lo.w *= inv;
              hi.x *= inv; hi.y *= inv; hi.z *= inv; hi.w *= inv;
            }
            const __half2 h0 = __floats2half2_rn(lo.x, lo.y), h1 = __floats2half2_rn(lo.z, lo.w);
            const __half2 h2 = __floats2half2_rn(hi.x, hi.y), h3 = __floats2half2_rn(hi.z, hi.w);
            uint4 o;
            o.x = *reinterpret_cast<const uint32_t*>(&h0);
            o.y = *reinterpret_cast<const uint32_t*>(&h1);
            o.z = *reinterpret_cast<const uint32_t*>(&h2);
            o.w = *reinterpret_cast<const uint32_t*>(&h3);
            *reinterpret_cast<uint4*>(drow + ((static_cast<uint32_t>(c16) ^ rsw) << 4)) = o;
          }
          // the operand (this CTA's shared memory, generic-proxy writes) is read by the tensor core
          // through the async proxy; the release.cluster arrive below orders it for the leader
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_cluster(a16_full_leader0 + 8u * static_cast<uint32_t>(ai));
            mbar_arrive(&stg_empty[sj]);
          }
          if (++ai == kA16) { ai = 0; aphase ^= 1u; }
          if (++sj == kStg) { sj = 0; sphase ^= 1u; }
        }
        if (!ok) {
          if (lane == 0) {
            *abort_flag = 1;
            atomicExch(args.status, G16_ERR_TIMEOUT);
          }
          break;
        }
      }
    }
  }

  // Every tile store has completed (and, for peer destinations, is visible system-wide) before the
  // grid ends. In multicast mode every lane stored, so every lane fences.
  if (warp >= 2 && warp < 2 + EPIW) {
    if (lane == 0) bulk_wait_group0();
    if (dst.ndst == 0 || (dst.ndst > 1 && lane == 0)) __threadfence_system();
  }
  // TMEM is released only after every MMA of the pair has completed and both CTAs are done.
  if (warp == 1) {
    if (lane == 0) mbar_wait(drain_bar, 0, nullptr);
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  // Completion signal (multicast mode): the cluster barrier above orders every thread's fenced
  // stores before this release, which reaches every GPU's counter through the switch.
  if (threadIdx.x == 0 && dst.mc_flag != 0) {
    __threadfence_system();
    multimem_red_add_release_u32(dst.mc_flag, 1u);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem, G::kTmemCols);
  }
}

template <typename F>
cudaError_t ensure_pair_attr(F* kern, std::atomic<uint64_t>& done, size_t bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// cudaFuncSetAttribute once per (kernel variant, device), then the launch.
template <bool OUT_F16, int BN, bool A_F32, int EPIW>
cudaError_t launch_pair_variant(cudaLaunchConfig_t cfg, const CUtensorMap& ta, const CUtensorMap& tb,
                                const PairDst& dmaps, const PairArgs& args) {
  using G = PairGeo<BN, A_F32, EPIW>;
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t e = ensure_pair_attr(gemm_pair_kernel<OUT_F16, BN, A_F32, EPIW>, attr_done, G::kSmemBytes);
  if (e != cudaSuccess) return e;
  cfg.blockDim = dim3(G::kThreads, 1, 1);
  cfg.dynamicSmemBytes = G::kSmemBytes;
  return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<OUT_F16, BN, A_F32, EPIW>, ta, tb, dmaps, args);
}

template <bool A_F32>
cudaError_t launch_pair_any(int out_dtype, int bn, int epiw, const cudaLaunchConfig_t& cfg, const CUtensorMap& ta,
                            const CUtensorMap& tb, const PairDst& dmaps, const PairArgs& args) {
  const bool f16 = out_dtype == G16_F16;
#if G16_PAIR_BN == 128
  if (bn == 128)
    return f16 ? launch_pair_variant<true, 128, A_F32, 4>(cfg, ta, tb, dmaps, args)
               : launch_pair_variant<false, 128, A_F32, 4>(cfg, ta, tb, dmaps, args);
#else
  (void)bn;
#endif
  if constexpr (!A_F32) {
    if (epiw == 8)
      return f16 ? launch_pair_variant<true, 256, false, 8>(cfg, ta, tb, dmaps, args)
                 : launch_pair_variant<false, 256, false, 8>(cfg, ta, tb, dmaps, args);
  }
  return f16 ? launch_pair_variant<true, 256, A_F32, 4>(cfg, ta, tb, dmaps, args)
             : launch_pair_variant<false, 256, A_F32, 4>(cfg, ta, tb, dmaps, args);
}

// Tile width of the pair kernel: 256. G16_PAIR_BN=128 (a build option) selects 128-wide tiles,
// which put twice as many pairs to work on outputs with few 256 x 256 tiles. Measured on B200
// (CUDA graphs, operands rotated through HBM): a 128-wide K step costs about as much as a 256-wide
// one, so the narrow tiles lost wherever they applied: 2048 x 3072 x 1024 22.7 us (the small-problem
// kernel 19.9, 256-wide pairs 23.7), 1024^3 12.2 (9.6, 13.8), 2048 x 4096 x 2048 47.5 (31.2 with
// 256-wide pairs).
int pair_tile_width(int, int, int) { return G16_PAIR_BN == 128 ? 128 : 256; }

// Epilogue warps for an output: 8 when a tile's K loop is short (at most 16 K steps of 64) and
// the output fp32, the case where a 4-warp epilogue outlasts the next tile's mainloop; else 4.
// Measured on B200 (CUDA graphs, operands rotated through HBM, fp32 out), 4 -> 8 warps:
// 65536 x 768 x 768 91.4 -> 85.3 us, 65536 x 768 x 2304 250.7 -> 233.5, 65536 x 768 x 3072
// 334.9 -> 310.8, 16384 x 1024 x 4096 176.1 -> 124.2; but 65536 x 3072 x 768 236.2 -> 251.2 and
// fp16-output shapes level or slower (the ring loses a stage to the second set of staging buffers).
// G16_PAIR_EPIW (a build option, 0 = this rule) forces 4 or 8.
int pair_epilogue_warps(int K, int out_dtype) {
  if (G16_PAIR_EPIW == 4 || G16_PAIR_EPIW == 8) return G16_PAIR_EPIW;
  return (out_dtype == G16_F32 && K <= 16 * kBK) ? 8 : 4;
}

}  // namespace

// Whether a cluster of two pair-GEMM CTAs can be resident on the current device (cached).
bool gemm_pair_available() {
  static std::atomic<uint64_t> known{0}, ok{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const uint64_t bit = 1ull << (dev & 63);
  if (known.load(std::memory_order_acquire) & bit) return (ok.load(std::memory_order_acquire) & bit) != 0;
  static std::atomic<uint64_t> attr_probe{0};
  bool good =
      ensure_pair_attr(gemm_pair_kernel<true, 256, false, 4>, attr_probe, PairGeo<256>::kSmemBytes) == cudaSuccess;
  if (good) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kPrThreads, 1, 1);
    cfg.dynamicSmemBytes = PairGeo<256>::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int active = 0;
    good = cudaOccupancyMaxActiveClusters(&active, gemm_pair_kernel<true, 256, false, 4>, &cfg) == cudaSuccess &&
           active >= 1;
    (void)cudaGetLastError();
  }
  if (good) ok.fetch_or(bit, std::memory_order_acq_rel);
  known.fetch_or(bit, std::memory_order_acq_rel);
  return good;
}

namespace {

// a: fp16 A (a_f32 false) or fp32 A with the row scales' reciprocals in rscale_inv (a_f32 true).
int launch_pair_impl(const void* a, bool a_f32, const uint16_t* b16, const PairDst& dmaps, int out_dtype,
                     const float* bias, const float* rscale, const float* rscale_inv, int M, int K, int N,
                     cudaStream_t s, const DeviceInfo& dev, int act) {
  if (M <= 0 || N <= 0) return G16_OK;
  if (a_f32 && (rscale_inv == nullptr || dmaps.ndst != 1)) return G16_ERR_ARG;
  PairArgs args{};
  args.act = act;
  args.bias = bias;
  args.rscale = rscale;
  args.rscale_inv = rscale_inv;
  args.status = device_status_ptr();
  if (args.status == nullptr) return G16_ERR_CUDA;
  args.M = M;
  args.N = N;
  args.K = K;
  const int max_pairs = dev.sm_count / 2;
  const int bn = pair_tile_width(M, N, max_pairs);
  args.m2_tiles = (M + 2 * kBM - 1) / (2 * kBM);
  args.n_tiles = (N + bn - 1) / bn;
  args.units = args.m2_tiles * args.n_tiles;
  args.kblocks = (K + kBK - 1) / kBK;
  if (args.kblocks < 1) return G16_ERR_ARG;
  CUtensorMap ta, tb;
  // A: fp16 [128 x 64] boxes, or fp32 [128 x 32] boxes (two per K step); 128-byte swizzle either way.
  int st = a_f32 ? make_tmap_2d(&ta, a, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, static_cast<uint64_t>(M),
                                static_cast<uint64_t>(K), kBM, 32, CU_TENSOR_MAP_SWIZZLE_128B)
                 : make_tmap_2d(&ta, a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(M),
                                static_cast<uint64_t>(K), kBM, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  st = make_tmap_2d(&tb, b16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                    kBK, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  const int pairs = args.units < max_pairs ? args.units : max_pairs;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch for a plain output (the multi-GPU variants keep stream order).
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dmaps.ndst == 1 && G16_PAIR_PDL ? 2 : 1;
  const int epiw = a_f32 ? 4 : pair_epilogue_warps(K, out_dtype);
  const cudaError_t e = a_f32 ? launch_pair_any<true>(out_dtype, bn, epiw, cfg, ta, tb, dmaps, args)
                              : launch_pair_any<false>(out_dtype, bn, epiw, cfg, ta, tb, dmaps, args);
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

}  // namespace

int launch_gemm_pair(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                     const float* rscale, int M, int K, int N, cudaStream_t s, const DeviceInfo& dev, int act) {
  if (M <= 0 || N <= 0) return G16_OK;
  // Output: [32 rows x 128 bytes] boxes (32 fp32 or 64 fp16 columns), 128-byte swizzle.
  PairDst dmaps{};
  const bool f16 = out_dtype == G16_F16;
  int st = make_tmap_2d(&dmaps.m[0], out, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        f16 ? 2 : 4, static_cast<uint64_t>(M), static_cast<uint64_t>(N), 32, f16 ? 64 : 32,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  dmaps.ndst = 1;
  dmaps.col0 = 0;
  return launch_pair_impl(a16, false, b16, dmaps, out_dtype, bias, rscale, nullptr, M, K, N, s, dev, act);
}

int launch_gemm_pair_f32a(const float* x, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                          const float* rscale, const float* rscale_inv, int M, int K, int N, cudaStream_t s,
                          const DeviceInfo& dev, int act) {
  if (M <= 0 || N <= 0) return G16_OK;
  PairDst dmaps{};
  const bool f16 = out_dtype == G16_F16;
  int st = make_tmap_2d(&dmaps.m[0], out, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                        f16 ? 2 : 4, static_cast<uint64_t>(M), static_cast<uint64_t>(N), 32, f16 ? 64 : 32,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  dmaps.ndst = 1;
  dmaps.col0 = 0;
  return launch_pair_impl(x, true, b16, dmaps, out_dtype, bias, rscale, rscale_inv, M, K, N, s, dev, act);
}

int launch_gemm_pair_multimem(const uint16_t* a16, const uint16_t* b16, void* mc, int out_dtype, const float* bias,
                              const float* rscale, int M, int K, int N, long long ldc, int col0, cudaStream_t s,
                              const DeviceInfo& dev, void* mc_flag) {
  if (mc == nullptr) return G16_ERR_ARG;
  if (M <= 0 || N <= 0) return G16_OK;
  PairDst dmaps{};
  dmaps.ndst = 0;
  dmaps.col0 = col0;
  dmaps.mc = reinterpret_cast<uint64_t>(mc);
  dmaps.ldc = ldc;
  dmaps.mc_flag = reinterpret_cast<uint64_t>(mc_flag);
  return launch_pair_impl(a16, false, b16, dmaps, out_dtype, bias, rscale, nullptr, M, K, N, s, dev, G16_ACT_NONE);
}

int gemm_pair_ctas(int M, int N, const DeviceInfo& dev) {
  if (M <= 0 || N <= 0) return 0;
  const int max_pairs = dev.sm_count / 2;
  const int bn = pair_tile_width(M, N, max_pairs);
  const int units = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + bn - 1) / bn);
  return 2 * (units < max_pairs ? units : max_pairs);
}

int launch_gemm_pair_scatter(const uint16_t* a16, const uint16_t* b16, void* const* dst, int ndst, int out_dtype,
                             const float* bias, const float* rscale, int M, int K, int N, long long ldc, int col0,
                             cudaStream_t s, const DeviceInfo& dev) {
  if (ndst < 1 || ndst > kPrMaxDst) return G16_ERR_ARG;
  if (M <= 0 || N <= 0) return G16_OK;
  PairDst dmaps{};
  const bool f16 = out_dtype == G16_F16;
  for (int d = 0; d < ndst; ++d) {
    if (dst[d] == nullptr) return G16_ERR_ARG;
    // [M, col0 + N] of each destination: columns past this rank's shard are outside the map, so a
    // partial last box cannot spill into a neighbour's columns.
    const int st = make_tmap_2d_strided(&dmaps.m[d], dst[d],
                                        f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                        f16 ? 2 : 4, static_cast<uint64_t>(M),
                                        static_cast<uint64_t>(col0) + static_cast<uint64_t>(N),
                                        static_cast<uint64_t>(ldc), 32, f16 ? 64 : 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != G16_OK) return st;
  }
  dmaps.ndst = ndst;
  dmaps.col0 = col0;
  return launch_pair_impl(a16, false, b16, dmaps, out_dtype, bias, rscale, nullptr, M, K, N, s, dev, G16_ACT_NONE);
}

}  // namespace g16
