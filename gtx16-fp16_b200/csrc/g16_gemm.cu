// Tensor-core GEMM for the M > 8 path: out[M,N] = (A[M,K] @ B[K,N]) * rscale[row] + bias[col].
//
// Reference behaviour replaced: hgemm_body / hgemm_f32out / hgemm_f16out / hgemm_splitk
// (src/gtx16_fp16/kernels.py:35-151) and the split-K host logic of mm_t (ops.py:92-107). The
// reference is a 128x128 SIMT tile with packed-fp16 FMA over 16-wide K slices folded into fp32;
// its split-K variant adds partial tiles into a prefilled fp32 output with atomics.
//
// B200 design (sm_100a):
//   * persistent kernel, one CTA per SM, static round-robin over work units; a unit is one
//     128x256 output tile (or one K chunk of it in split-K mode);
//   * warp 0: TMA producer (one elected thread) filling a 4-stage shared-memory ring with 128-byte
//     swizzled tiles: A [128 x 64] K-major, B [64 x 256] N-major (w_t is [K, N] row-major);
//   * warp 1: allocates 512 TMEM columns (two 128x256 fp32 accumulators) and issues
//     tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) from one thread; tcgen05.commit
//     releases smem stages and publishes finished accumulators;
//   * warps 2-5: epilogue; each reads its 32 TMEM lanes with tcgen05.ld, applies the per-row
//     power-of-two unscale and fp32 bias, converts and stores, overlapping the next tile's MMAs;
//   * split-K (few output tiles): each unit writes its fp32 partial tile to the workspace; a
//     second, fully parallel kernel (launched with programmatic dependent launch so its launch
//     overlaps the GEMM's tail) sums the partials of every output in split order and applies the
//     same epilogue. No atomics and no waiting: results are bitwise reproducible.
// Every wait is bounded; on expiry the kernel records G16_ERR_TIMEOUT in the device status word,
// drains its in-flight copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <atomic>
#include <mutex>

#include "g16_internal.cuh"
#include "g16_ptx.cuh"

#ifndef G16_MIDM_DISPATCH
#define G16_MIDM_DISPATCH 1
#endif

namespace g16 {
namespace {

constexpr int kStages = 4;
constexpr int kThreads = 192;  // 6 warps
constexpr int kEpiThreads = 128;
constexpr uint32_t kABytes = kBM * kBK * 2;     // 16 KiB
constexpr uint32_t kBBoxBytes = kBK * 64 * 2;   // one [64 k x 64 n] box: 8 KiB
constexpr uint32_t kBBytes = kBK * kBN * 2;     // 32 KiB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 2 * kBN;         // double-buffered accumulator
constexpr int kGroupM = 8;                      // tile rasterisation: 8 tile-rows per group
constexpr size_t kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + 256 /*barriers etc.*/;
// Scatter epilogue: each epilogue warp transposes its 32 rows x 128 bytes through shared memory so
// that every store instruction writes whole 128-byte row segments (8 lanes per row).
constexpr int kMaxDst = 8;
constexpr uint32_t kEpiStageBytes = (kEpiThreads / 32) * 32 * 128;  // 16 KiB
constexpr size_t kSmemBytesScatter = kSmemBytes + kEpiStageBytes;

struct GemmArgs {
  void* out;
  void* dst[kMaxDst];  // scatter: destination buffers, each [M, ldc]; the tile lands at column col0 + n
  int ndst;
  long long ldc;
  int col0;
  const float* bias;
  const float* rscale;
  float* partials;  // [m_tiles * n_tiles][ksplit][kBM][kBN] fp32 (split-K only), tile = mt * n_tiles + nt
  int* status;      // device status word
  int M, N, K;
  int m_tiles, n_tiles, tiles;
  int ksplit, kblocks, kb_per_split, units;
  // Tail split (ksplit == 1): units >= full_units are 128-column halves of the last tiles, so a
  // last partial wave of T tiles runs as 2T half-tiles on the idle SMs (full K, no reduction).
  int full_units, split_tail;
  int act;  // epilogue activation (G16_ACT_*)
};

// Scatter epilogue modes.
constexpr int kScatterNone = 0;
constexpr int kScatterStores = 1;  // 16-byte stores by the epilogue warps
constexpr int kScatterTma = 2;     // TMA tile stores of the staged rows, one per destination

// Destination tensor maps of the TMA scatter epilogue: [M rows, col0 + N columns] of dst[d] with
// row stride ldc, [32 x 128-byte] boxes, 128-byte swizzle (the staging layout).
struct DstMaps {
  CUtensorMap m[kMaxDst];
};

struct Unit {
  int tile, mt, nt, split, kb0, kb1;
  int col0, ncols;  // first output column and width of the unit (kBN, or 128 for a tail half)
};

__device__ __forceinline__ Unit unit_coords(const GemmArgs& a, int u) {
  Unit r;
  int half = -1;
  if (a.split_tail && u >= a.full_units) {
    const int h = u - a.full_units;
    r.tile = a.full_units + (h >> 1);
    r.split = 0;
    half = h & 1;
  } else {
    r.tile = u / a.ksplit;
    r.split = u - r.tile * a.ksplit;
  }
  // Grouped rasterisation: walk kGroupM tile-rows together so B column panels stay in L2.
  const int per_group = kGroupM * a.n_tiles;
  const int g = r.tile / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(kGroupM, a.m_tiles - first_m);
  const int in_g = r.tile - g * per_group;
  r.mt = first_m + in_g % gsize;
  r.nt = in_g / gsize;
  r.kb0 = r.split * a.kb_per_split;
  r.kb1 = min(a.kblocks, r.kb0 + a.kb_per_split);
  r.col0 = r.nt * kBN + (half > 0 ? kBN / 2 : 0);
  r.ncols = half >= 0 ? kBN / 2 : kBN;
  return r;
}

__device__ __forceinline__ void report_timeout(int* status, volatile int* abort_flag) {
  *abort_flag = 1;
  atomicExch(status, G16_ERR_TIMEOUT);
}

// Store 32 consecutive fp32 results (one row, columns col0..col0+31) with unscale and bias.
template <bool OUT_F16>
__device__ __forceinline__ void store_row32(const GemmArgs& a, int row, int col0, float rs, const float (&v)[32]) {
  if (row >= a.M) return;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int col = col0 + 8 * g;
    if (col >= a.N) break;  // N % 8 == 0: whole 8-column groups are in or out
    float o[8];
    if (a.bias != nullptr) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(a.bias + col));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(a.bias + col + 4));
      o[0] = fmaf(v[8 * g + 0], rs, b0.x); o[1] = fmaf(v[8 * g + 1], rs, b0.y);
      o[2] = fmaf(v[8 * g + 2], rs, b0.z); o[3] = fmaf(v[8 * g + 3], rs, b0.w);
      o[4] = fmaf(v[8 * g + 4], rs, b1.x); o[5] = fmaf(v[8 * g + 5], rs, b1.y);
      o[6] = fmaf(v[8 * g + 6], rs, b1.z); o[7] = fmaf(v[8 * g + 7], rs, b1.w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[8 * g + j] * rs;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = apply_act(o[j], a.act);
    const size_t off = static_cast<size_t>(row) * a.N + col;
    if constexpr (OUT_F16) {
      __half2 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.out) + off) = *reinterpret_cast<const uint4*>(h);
    } else {
      float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + off);
      dst[0] = make_float4(o[0], o[1], o[2], o[3]);
      dst[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
  }
}

// One 128-byte row segment per lane-octet: the scatter epilogue's coalesced store of a warp's
// staged [32 rows x 128 bytes] (16-byte chunk j of row r sits at chunk j ^ (r & 7)).
template <bool OUT_F16>
__device__ __forceinline__ void scatter_rows(const GemmArgs& a, const uint8_t* stage, int row0, int col_first,
                                             int lane) {
  constexpr int kElem = OUT_F16 ? 2 : 4;
  constexpr int kPerChunk = 16 / kElem;  // elements per 16-byte chunk
  const int c = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {  // 4 rows (8 lanes each) per instruction
    const int r = i * 4 + (lane >> 3);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128 + ((c ^ (r & 7)) << 4));
    const int row = row0 + r;
    const int col = col_first + c * kPerChunk;  // local column
    if (row < a.M && col < a.N) {                // N % 8 == 0: whole chunks are in or out
      const long long off = (static_cast<long long>(row) * a.ldc + a.col0 + col) * kElem;
      for (int d = 0; d < a.ndst; ++d)
        *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.dst[d]) + off) = v;
    }
  }
}

template <bool OUT_F16, int SCATTER>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
            const GemmArgs args, const __grid_constant__ DstMaps dmaps) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  // Align by pointer arithmetic on the __shared__ array (an integer round trip would turn
  // every access into a generic-address load).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stage_base = smem;
  uint8_t* epi_stage = smem + kStages * kStageBytes;  // scatter only: kEpiStageBytes, 1 KiB aligned
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi_stage + (SCATTER != kScatterNone ? kEpiStageBytes : 0));
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* tfull_bar = empty_bar + kStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  // Self-check: the layout must end inside the launch's dynamic shared memory (uniform for the
  // whole grid: every CTA returns before any barrier, TMEM allocation or shared-memory access).
  if (static_cast<uint32_t>(reinterpret_cast<const volatile uint8_t*>(abort_flag + 1) - smem_raw) > dynamic_smem_bytes()) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(args.status, G16_ERR_ARG);
    return;
  }

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], kEpiThreads / 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_phase[kStages];
      bool armed[kStages];
      for (int s = 0; s < kStages; ++s) { armed[s] = false; armed_phase[s] = 0; }
      bool ok = true;
      for (int u = blockIdx.x; u < args.units && ok; u += gridDim.x) {
        const Unit w = unit_coords(args, u);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = stage_base + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          const int nbox = w.ncols / 64;
          mbar_arrive_expect_tx(&full_bar[stage], kABytes + nbox * kBBoxBytes);
          armed[stage] = true;
          armed_phase[stage] = phase;
          tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * kBK, w.mt * kBM);
          for (int j = 0; j < nbox; ++j)
            tma_load_2d(sb + j * kBBoxBytes, &tmap_b, &full_bar[stage], w.col0 + 64 * j, kb * kBK);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        report_timeout(args.status, abort_flag);
        // Drain: never leave the CTA with bulk copies still landing in its shared memory.
        for (int s = 0; s < kStages; ++s)
          if (armed[s]) mbar_wait(&full_bar[s], armed_phase[s], nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_full = idesc_f16_f32(kBM, kBN, /*b_mn_major=*/true);
      constexpr uint32_t idesc_half = idesc_f16_f32(kBM, kBN / 2, /*b_mn_major=*/true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < args.units && ok; u += gridDim.x) {
        const Unit w = unit_coords(args, u);
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        const uint32_t idesc = w.ncols == kBN ? idesc_full : idesc_half;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(stage_base + stage * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // A: K-major, rows of 128 B, 8-row atoms 1024 B apart (SBO); step K by 32 B.
            const uint64_t adesc = smem_desc_sw128(sa + k * (kUmmaK * 2), 16, 1024);
            // B: N-major, 64-column blocks 8 KiB apart (LBO), 8-row k-groups 1024 B apart (SBO);
            // step K by 16 rows of 128 B.
            const uint64_t bdesc = smem_desc_sw128(sb + k * (kUmmaK * 128), kBBoxBytes, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb > w.kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok) report_timeout(args.status, abort_flag);
      // Wait for every issued MMA before TMEM is released.
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0, nullptr);
    }
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int r_local = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < args.units; u += gridDim.x) {
      const Unit w = unit_coords(args, u);
      // Every lane waits; the outcome is made warp-uniform (and the warp reconverged) before any
      // .sync.aligned tcgen05 instruction.
      bool got = mbar_wait(&tfull_bar[acc], acc_phase, abort_flag);
      got = __all_sync(0xffffffffu, got);
      if (!got && lane == 0) report_timeout(args.status, abort_flag);
      const int row = w.mt * kBM + r_local;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kBN);
      if constexpr (SCATTER != kScatterNone) {
        // ksplit == 1 (enforced by the launcher). 128 bytes per row per pass: 64 fp16 or 32 fp32
        // columns; every destination gets each row segment once.
        if (!got) break;
        tc_fence_after();
        const float rs = (args.rscale != nullptr && row < args.M) ? __ldg(args.rscale + row) : 1.f;
        constexpr int kCols = OUT_F16 ? 64 : 32;
        uint8_t* my_stage = epi_stage + quarter * (32 * 128);
#pragma unroll 1
        for (int c0 = 0; c0 < w.ncols; c0 += kCols) {
          const int gcol = w.col0 + c0;  // local column of the pass
          uint4 packed[8];
#pragma unroll
          for (int h = 0; h < kCols / 32; ++h) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld_32x32b_x32(t_row + c0 + h * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int col = gcol + h * 32 + 8 * g;
              float o[8];
              if (args.bias != nullptr && col < args.N) {
                const float4 b0 = __ldg(reinterpret_cast<const float4*>(args.bias + col));
                const float4 b1 = __ldg(reinterpret_cast<const float4*>(args.bias + col + 4));
                const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = fmaf(__uint_as_float(r[8 * g + j]), rs, bb[j]);
              } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = __uint_as_float(r[8 * g + j]) * rs;
              }
              if constexpr (OUT_F16) {
                __half2 hh[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) hh[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
                packed[h * 4 + g] = *reinterpret_cast<const uint4*>(hh);
              } else {
                packed[h * 8 + 2 * g] = make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]),
                                                   __float_as_uint(o[2]), __float_as_uint(o[3]));
                packed[h * 8 + 2 * g + 1] = make_uint4(__float_as_uint(o[4]), __float_as_uint(o[5]),
                                                       __float_as_uint(o[6]), __float_as_uint(o[7]));
              }
            }
          }
          // this lane's row: 8 chunks of 16 bytes, swizzled by row (the 128-byte TMA swizzle)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(my_stage + lane * 128 + ((j ^ (lane & 7)) << 4)) = packed[j];
          if constexpr (SCATTER == kScatterTma) {
            fence_proxy_async_smem();  // staged rows -> visible to the TMA engine
            __syncwarp();
            const int y = w.mt * kBM + quarter * 32;
            if (lane == 0 && y < args.M && gcol < args.N) {
              for (int d = 0; d < args.ndst; ++d) tma_store_2d(&dmaps.m[d], my_stage, args.col0 + gcol, y);
              bulk_commit_group();
              bulk_wait_group_read0();  // the engine has read the stage: it may be rewritten
            }
            __syncwarp();
          } else {
            __syncwarp();
            scatter_rows<OUT_F16>(args, my_stage, w.mt * kBM + quarter * 32, gcol, lane);
            __syncwarp();  // the stage is rewritten by the next pass
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      } else if (args.ksplit == 1) {
        if (!got) break;
        tc_fence_after();
        const float rs = (args.rscale != nullptr && row < args.M) ? __ldg(args.rscale + row) : 1.f;
#pragma unroll 1
        for (int c = 0; c < w.ncols / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          store_row32<OUT_F16>(args, row, w.col0 + c * 32, rs, v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      } else {
        if (!got) break;
        tc_fence_after();
        const int tile_rm = w.mt * args.n_tiles + w.nt;
        float* my_part = args.partials + (static_cast<size_t>(tile_rm) * args.ksplit + w.split) * (kBM * kBN) +
                         static_cast<size_t>(r_local) * kBN;
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait();
          float4* dst = reinterpret_cast<float4*>(my_part + c * 32);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(dst + j, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                        __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  // Scatter: stores into peer memory (NVLink) are complete and visible system-wide before the grid
  // ends.
  if constexpr (SCATTER == kScatterTma) {
    if (warp >= 2 && lane == 0) bulk_wait_group0();
  }
  if constexpr (SCATTER != kScatterNone) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Split-K reduction: out = (sum over splits s = 0..ksplit-1, in order, of partial[tile][s]) * rscale
// + bias. One thread per 4 consecutive output columns of one row; launched with programmatic
// dependent launch, so it waits here for the GEMM grid's partial stores.
template <bool OUT_F16>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmArgs args) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int kQuads = kBN / 4;
  const size_t total = static_cast<size_t>(args.m_tiles) * args.n_tiles * kBM * kQuads;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int q = static_cast<int>(i % kQuads);
    const size_t t1 = i / kQuads;
    const int r = static_cast<int>(t1 % kBM);
    const size_t tile = t1 / kBM;
    const int mt = static_cast<int>(tile / args.n_tiles);
    const int nt = static_cast<int>(tile % args.n_tiles);
    const int row = mt * kBM + r;
    const int col = nt * kBN + 4 * q;
    if (row >= args.M || col >= args.N) continue;
    const float* p = args.partials + tile * args.ksplit * static_cast<size_t>(kBM * kBN) + r * kBN + 4 * q;
    float4 acc = __ldcg(reinterpret_cast<const float4*>(p));
    int s = 1;
    for (; s + 3 < args.ksplit; s += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcg(reinterpret_cast<const float4*>(p + static_cast<size_t>(s + u) * (kBM * kBN)));
#pragma unroll
      for (int u = 0; u < 4; ++u) { acc.x += v[u].x; acc.y += v[u].y; acc.z += v[u].z; acc.w += v[u].w; }
    }
    for (; s < args.ksplit; ++s) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(p + static_cast<size_t>(s) * (kBM * kBN)));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const float rs = args.rscale != nullptr ? __ldg(args.rscale + row) : 1.f;
    float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
    if (args.bias != nullptr) b = __ldg(reinterpret_cast<const float4*>(args.bias + col));
    const float o0 = apply_act(fmaf(acc.x, rs, b.x), args.act), o1 = apply_act(fmaf(acc.y, rs, b.y), args.act),
                o2 = apply_act(fmaf(acc.z, rs, b.z), args.act), o3 = apply_act(fmaf(acc.w, rs, b.w), args.act);
    const size_t off = static_cast<size_t>(row) * args.N + col;
    if constexpr (OUT_F16) {
      const __half2 h0 = __floats2half2_rn(o0, o1), h1 = __floats2half2_rn(o2, o3);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&h0);
      u.y = *reinterpret_cast<const uint32_t*>(&h1);
      *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(args.out) + off) = u;
    } else {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + off) = make_float4(o0, o1, o2, o3);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
size_t partial_bytes(int tiles, int ksplit) {
  return static_cast<size_t>(tiles) * ksplit * kBM * kBN * sizeof(float);
}

int tiles_of(int M, int N) { return ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN); }

}  // namespace

int gemm_auto_ksplit(int M, int K, int N, const DeviceInfo& dev) {
  const int tiles = tiles_of(M, N);
  const int kblocks = (K + kBK - 1) / kBK;
  if (tiles * 2 > dev.sm_count || kblocks < 8) return 1;
  int ks = dev.sm_count / tiles;
  const int by_k = kblocks / 4;  // keep at least 4 k-blocks (256 of K) per split
  if (ks > by_k) ks = by_k;
  return ks < 1 ? 1 : ks;
}

bool gemm_auto_uses_pair(int M, int K, int N, const DeviceInfo& dev) {
  if (M <= kMidMaxM || K <= 0 || N <= 0) return false;           // medium-M kernel
  if (plan_gemm_small(M, K, N, dev).bn != 0) return false;        // small-problem kernel
  if (gemm_auto_ksplit(M, K, N, dev) > 1) return false;           // split K
  return gemm_pair_available();
}

size_t gemm_workspace_bytes(int M, int K, int N, int ksplit) {
  if (ksplit <= 1) return 0;
  const int kblocks = (K + kBK - 1) / kBK;
  if (ksplit > kblocks) ksplit = kblocks;
  return partial_bytes(tiles_of(M, N), ksplit);
}

size_t gemm_auto_workspace_bytes(int M, int K, int N, const DeviceInfo& dev) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  const size_t split = gemm_workspace_bytes(M, K, N, gemm_auto_ksplit(M, K, N, dev));
  if (M <= kMidMaxM && G16_MIDM_DISPATCH && gemm_midm_ranks(M, K, N, dev) > 0) return split;
  const size_t gs = small_gs_workspace_bytes(plan_gemm_small(M, K, N, dev), M, N);
  return gs > split ? gs : split;
}

namespace {

// cudaFuncSetAttribute once per (kernel, device): the call costs microseconds on the host.
template <typename F>
cudaError_t ensure_smem_attr(F* kern, std::atomic<uint64_t>& done, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// A last partial wave of at most half the SMs runs as 128-column halves (see GemmArgs).
void set_tail_split(GemmArgs& a, const DeviceInfo& dev) {
  a.full_units = a.units;
  a.split_tail = 0;
  if (a.ksplit != 1 || a.tiles <= dev.sm_count) return;
  const int tail = a.tiles % dev.sm_count;
  if (tail == 0 || 2 * tail > dev.sm_count) return;
  a.split_tail = 1;
  a.full_units = a.tiles - tail;
  a.units = a.full_units + 2 * tail;
}

std::atomic<uint64_t> g_attr_f16{0}, g_attr_f32{0}, g_attr_sc16{0}, g_attr_sc32{0}, g_attr_tm16{0}, g_attr_tm32{0};

template <bool OUT_F16>
cudaError_t launch_reduce(const GemmArgs& args, cudaStream_t s, const DeviceInfo& dev) {
  const size_t total = static_cast<size_t>(args.m_tiles) * args.n_tiles * kBM * (kBN / 4);
  size_t blocks = (total + 255) / 256;
  const size_t cap = static_cast<size_t>(dev.sm_count) * 8;
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, splitk_reduce_kernel<OUT_F16>, args);
}

}  // namespace

int launch_gemm(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                const float* rscale, int M, int K, int N, int ksplit, void* ws, size_t ws_bytes, cudaStream_t s,
                const DeviceInfo& dev, int act) {
  if (M <= 0 || N <= 0) return G16_OK;
  const int kblocks = (K + kBK - 1) / kBK;
  // Automatic plan, M <= 64: the swapped-operand kernel (weight columns as the MMA's M).
  if (ksplit == 0 && M <= kMidMaxM && G16_MIDM_DISPATCH) {
    const int st = launch_gemm_midm(a16, b16, out, out_dtype, bias, rscale, M, K, N, s, dev, act);
    if (st != G16_ERR_UNSUPPORTED) return st;
  }
  if (ksplit == 0) {
    const SmallPlan p = plan_gemm_small(M, K, N, dev);
    if (p.bn != 0) {
      // The grid split when the workspace holds it, else the cluster plan (no workspace).
      if (p.gs_split > 1 && ws != nullptr && ws_bytes >= small_gs_workspace_bytes(p, M, N) &&
          (reinterpret_cast<uintptr_t>(ws) & 255u) == 0) {
        const int st = launch_gemm_small_gs(a16, b16, out, out_dtype, bias, rscale, M, K, N, p, ws, ws_bytes, s, act);
        if (st != G16_ERR_UNSUPPORTED) return st;
      }
      const int st = launch_gemm_small(a16, b16, out, out_dtype, bias, rscale, M, K, N, p.bn, p.csize, false, s, act);
      if (st != G16_ERR_UNSUPPORTED) return st;
    }
    ksplit = gemm_auto_ksplit(M, K, N, dev);
  }
  if (ksplit > kblocks) ksplit = kblocks;
  if (ksplit > 1 && ksplit <= 16) {
    const int st = launch_gemm_small(a16, b16, out, out_dtype, bias, rscale, M, K, N, 256, ksplit, true, s, act);
    if (st != G16_ERR_UNSUPPORTED) return st;
  }
  if (ksplit < 1) ksplit = 1;
  // A single pass runs on CTA pairs (256 x 256 tiles, a third fewer operand bytes per FLOP; the
  // same bits as the single-CTA kernel below). Measured on B200 with the pair kernel's TMA-store
  // epilogue: 4096^3 +9 %, 16384^3 +4-10 %, 8192 x 8192 x 16384 +7-14 %, 4096 x 4096 x 16384
  // +17-23 % over the single-CTA kernel, which keeps the multi-destination scatter epilogue.
  if (ksplit == 1 && gemm_pair_available())
    return launch_gemm_pair(a16, b16, out, out_dtype, bias, rscale, M, K, N, s, dev, act);
  GemmArgs args{};
  args.out = out;
  args.bias = bias;
  args.rscale = rscale;
  args.act = act;
  args.status = device_status_ptr();
  if (args.status == nullptr) return G16_ERR_CUDA;
  args.M = M;
  args.N = N;
  args.K = K;
  args.m_tiles = (M + kBM - 1) / kBM;
  args.n_tiles = (N + kBN - 1) / kBN;
  args.tiles = args.m_tiles * args.n_tiles;
  args.kblocks = kblocks;
  args.kb_per_split = (kblocks + ksplit - 1) / ksplit;
  ksplit = (kblocks + args.kb_per_split - 1) / args.kb_per_split;  // no empty splits
  args.ksplit = ksplit;
  args.units = args.tiles * ksplit;
  set_tail_split(args, dev);
  if (ksplit > 1) {
    const size_t need = partial_bytes(args.tiles, ksplit);
    if (ws == nullptr || ws_bytes < need) return G16_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return G16_ERR_ALIGN;
    args.partials = static_cast<float*>(ws);
  }

  CUtensorMap ta, tb;
  // A: [M, K] K-major, [128 x 64] boxes; B: [K, N] N-major, [64 x 64] boxes; 128-byte swizzle.
  int st = make_tmap_2d(&ta, a16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(M),
                        static_cast<uint64_t>(K), kBM, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  st = make_tmap_2d(&tb, b16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                    kBK, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;

  const int grid = args.units < dev.sm_count ? args.units : dev.sm_count;
  cudaError_t e;
  static const DstMaps kNoMaps{};
  if (out_dtype == G16_F16) {
    e = ensure_smem_attr(gemm_kernel<true, kScatterNone>, g_attr_f16, static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return cuda_fail(e);
    gemm_kernel<true, kScatterNone><<<grid, kThreads, kSmemBytes, s>>>(ta, tb, args, kNoMaps);
  } else {
    e = ensure_smem_attr(gemm_kernel<false, kScatterNone>, g_attr_f32, static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return cuda_fail(e);
    gemm_kernel<false, kScatterNone><<<grid, kThreads, kSmemBytes, s>>>(ta, tb, args, kNoMaps);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  if (ksplit > 1) {
    e = out_dtype == G16_F16 ? launch_reduce<true>(args, s, dev) : launch_reduce<false>(args, s, dev);
    if (e != cudaSuccess) return cuda_fail(e);
    note_launch();
  }
  return G16_OK;
}

int launch_gemm_scatter(const uint16_t* a16, const uint16_t* b16, void* const* dst, int ndst, int out_dtype,
                        const float* bias, const float* rscale, int M, int K, int N, long long ldc, int col0,
                        int flags, cudaStream_t s, const DeviceInfo& dev) {
  if (ndst < 1 || ndst > kMaxDst) return G16_ERR_ARG;
  if (M <= 0 || N <= 0) return G16_OK;
  // Default: CTA pairs. Measured at 2 GPUs (16384^3 N-sharded, interleaved repetitions, median):
  // pairs 3.66 ms per step (the local shard GEMM alone took 3.68 ms: the exchange is hidden),
  // single-CTA 16-byte stores 4.18 ms, single-CTA TMA stores 4.31 ms.
  if (flags == G16_SCATTER_MULTIMEM) {
    if (ndst != 1) return G16_ERR_ARG;
    if (!gemm_pair_available()) return G16_ERR_UNSUPPORTED;
    return launch_gemm_pair_multimem(a16, b16, dst[0], out_dtype, bias, rscale, M, K, N, ldc, col0, s, dev);
  }
  if (flags == G16_SCATTER_DEFAULT) flags = G16_SCATTER_PAIRS;
  if (flags == G16_SCATTER_PAIRS) {
    if (gemm_pair_available())
      return launch_gemm_pair_scatter(a16, b16, dst, ndst, out_dtype, bias, rscale, M, K, N, ldc, col0, s, dev);
    flags = G16_SCATTER_TMA;
  }
  GemmArgs args{};
  for (int d = 0; d < ndst; ++d) {
    if (dst[d] == nullptr) return G16_ERR_ARG;
    args.dst[d] = dst[d];
  }
  args.ndst = ndst;
  args.ldc = ldc;
  args.col0 = col0;
  args.bias = bias;
  args.rscale = rscale;
  args.status = device_status_ptr();
  if (args.status == nullptr) return G16_ERR_CUDA;
  args.M = M;
  args.N = N;
  args.K = K;
  args.m_tiles = (M + kBM - 1) / kBM;
  args.n_tiles = (N + kBN - 1) / kBN;
  args.tiles = args.m_tiles * args.n_tiles;
  args.kblocks = (K + kBK - 1) / kBK;
  args.kb_per_split = args.kblocks;
  args.ksplit = 1;
  args.units = args.tiles;
  set_tail_split(args, dev);

  CUtensorMap ta, tb;
  int st = make_tmap_2d(&ta, a16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(M),
                        static_cast<uint64_t>(K), kBM, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  st = make_tmap_2d(&tb, b16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                    kBK, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != G16_OK) return st;
  const bool tma = flags == G16_SCATTER_TMA;
  DstMaps maps{};
  if (tma) {
    // [M, col0 + N] of each destination: columns past this rank's shard are outside the map, so a
    // partial last box cannot spill into a neighbour's columns.
    for (int d = 0; d < ndst; ++d) {
      st = make_tmap_2d_strided(&maps.m[d], dst[d],
                                out_dtype == G16_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                out_dtype == G16_F16 ? 2 : 4, static_cast<uint64_t>(M),
                                static_cast<uint64_t>(col0) + static_cast<uint64_t>(N), static_cast<uint64_t>(ldc), 32,
                                out_dtype == G16_F16 ? 64 : 32, CU_TENSOR_MAP_SWIZZLE_128B);
      if (st != G16_OK) return st;
    }
  }
  const int grid = args.units < dev.sm_count ? args.units : dev.sm_count;
  cudaError_t e;
  if (out_dtype == G16_F16) {
    if (tma) {
      e = ensure_smem_attr(gemm_kernel<true, kScatterTma>, g_attr_tm16, static_cast<int>(kSmemBytesScatter));
      if (e != cudaSuccess) return cuda_fail(e);
      gemm_kernel<true, kScatterTma><<<grid, kThreads, kSmemBytesScatter, s>>>(ta, tb, args, maps);
    } else {
      e = ensure_smem_attr(gemm_kernel<true, kScatterStores>, g_attr_sc16, static_cast<int>(kSmemBytesScatter));
      if (e != cudaSuccess) return cuda_fail(e);
      gemm_kernel<true, kScatterStores><<<grid, kThreads, kSmemBytesScatter, s>>>(ta, tb, args, maps);
    }
  } else {
    if (tma) {
      e = ensure_smem_attr(gemm_kernel<false, kScatterTma>, g_attr_tm32, static_cast<int>(kSmemBytesScatter));
      if (e != cudaSuccess) return cuda_fail(e);
      gemm_kernel<false, kScatterTma><<<grid, kThreads, kSmemBytesScatter, s>>>(ta, tb, args, maps);
    } else {
      e = ensure_smem_attr(gemm_kernel<false, kScatterStores>, g_attr_sc32, static_cast<int>(kSmemBytesScatter));
      if (e != cudaSuccess) return cuda_fail(e);
      gemm_kernel<false, kScatterStores><<<grid, kThreads, kSmemBytesScatter, s>>>(ta, tb, args, maps);
    }
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  note_launch();
  return G16_OK;
}

}  // namespace g16
