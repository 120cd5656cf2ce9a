// Internal declarations shared by the kernel translation units and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "../../include/g16.h"

namespace g16 {

// Device status word (G16_OK or G16_ERR_TIMEOUT), one per device, defined in g16_api.cu.
// Kernels compiled in other translation units receive its address as a parameter.
int* device_status_ptr();  // host: device address of the current device's status word

// Records the CUDA error and returns G16_ERR_CUDA (host).
int cuda_fail(cudaError_t e);

// Per-device facts cached on first use (host).
struct DeviceInfo {
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int max_smem_optin = 0;
};
const DeviceInfo* device_info(int* status);  // current device; nullptr + status on failure

void note_launch(uint64_t n = 1);

// ---- launchers (host), each returns a g16_status code ----
int launch_skinny(const void* x, int x_dtype, const uint16_t* w, const float* bias, void* out, int out_dtype, int M,
                  int K, int N, cudaStream_t s, const DeviceInfo& dev, int act = 0);

// Launch plan of the skinny kernel for (M, K, N): info[0] tensor-core variant (1) or FMA (0),
// [1] cluster size, [2] strips, [3] K chunk, [4] dynamic shared memory, [5] resident clusters at the
// first cluster size tried, [6] at the chosen one.
int skinny_plan_info(int M, int K, int N, int x_dtype, int* info, const DeviceInfo& dev);

int launch_rowscale(const void* x, int x_dtype, uint16_t* y16, float* rscale, int M, int K, float thresh,
                    cudaStream_t s);
// fp32 activations only: the row scales of launch_rowscale (rscale) and their reciprocals, without
// writing an fp16 copy of x (for a GEMM that converts x itself).
int launch_rowamax(const float* x, float* rscale, float* rscale_inv, int M, int K, float thresh, cudaStream_t s);

// Tensor-core GEMM. ksplit = 0: automatic plan (the small-problem kernel when the output has too
// few tiles for the persistent one: its grid split when ws holds gemm_auto_workspace_bytes(), else
// its cluster plan; ws must hold gemm_workspace_bytes(M, K, N, gemm_auto_ksplit(...)) for the
// fallback). ksplit 2..16: that many K chunks reduced in a cluster (same chunks and order as the
// workspace path, which runs when such a cluster cannot be resident or ksplit > 16; ws must then
// hold gemm_workspace_bytes(M, K, N, ksplit)).
int launch_gemm(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                const float* rscale, int M, int K, int N, int ksplit, void* ws, size_t ws_bytes, cudaStream_t s,
                const DeviceInfo& dev, int act = 0);
size_t gemm_workspace_bytes(int M, int K, int N, int ksplit);
// Workspace of the automatic plan (ksplit = 0): its fallback split and the grid split, if any.
size_t gemm_auto_workspace_bytes(int M, int K, int N, const DeviceInfo& dev);
// Sharded GEMM whose fp16/fp32 output tiles go to ndst buffers [M, ldc] at column col0 (no split-K).
int launch_gemm_scatter(const uint16_t* a16, const uint16_t* b16, void* const* dst, int ndst, int out_dtype,
                        const float* bias, const float* rscale, int M, int K, int N, long long ldc, int col0,
                        int flags, cudaStream_t s, const DeviceInfo& dev);
int gemm_auto_ksplit(int M, int K, int N, const DeviceInfo& dev);
// Whether launch_gemm's automatic plan (ksplit = 0) is a single pass on the CTA-pair kernel.
bool gemm_auto_uses_pair(int M, int K, int N, const DeviceInfo& dev);

// GEMM on CTA pairs (g16_gemm_pair.cu): persistent, 256 x 256 tiles, tcgen05.mma.cta_group::2.
int launch_gemm_pair(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                     const float* rscale, int M, int K, int N, cudaStream_t s, const DeviceInfo& dev, int act = 0);
bool gemm_pair_available();
// The same GEMM with fp32 activations: each CTA converts its rows of x to fp16 as x * rscale_inv[row]
// (rounded like launch_rowscale) in shared memory; the epilogue multiplies by rscale[row]. Both
// come from launch_rowamax.
int launch_gemm_pair_f32a(const float* x, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                          const float* rscale, const float* rscale_inv, int M, int K, int N, cudaStream_t s,
                          const DeviceInfo& dev, int act = 0);
// The same kernel storing every output tile into ndst buffers [M, ldc] at column col0 (TMA tile
// stores; peer buffers for the multi-GPU exchange).
// The same with every tile written once through an NVLink multicast address covering all ranks'
// [M, ldc] outputs (multimem.st; the switch replicates it).
// mc_flag (optional): multicast address of a 32-bit counter every CTA adds 1 to after its stores.
int launch_gemm_pair_multimem(const uint16_t* a16, const uint16_t* b16, void* mc, int out_dtype, const float* bias,
                              const float* rscale, int M, int K, int N, long long ldc, int col0, cudaStream_t s,
                              const DeviceInfo& dev, void* mc_flag = nullptr);
// CTAs the pair kernel launches for an [M, N] output (each signals once in multicast mode).
int gemm_pair_ctas(int M, int N, const DeviceInfo& dev);
int launch_gemm_pair_scatter(const uint16_t* a16, const uint16_t* b16, void* const* dst, int ndst, int out_dtype,
                             const float* bias, const float* rscale, int M, int K, int N, long long ldc, int col0,
                             cudaStream_t s, const DeviceInfo& dev);

// Medium-M GEMM (g16_gemm_midm.cu): M <= kMidMaxM activation rows, operands swapped so the
// weight columns are the MMA's M and the rows its N; K split over a cluster, reduced in DSMEM.
constexpr int kMidMaxM = 64;
int launch_gemm_midm(const uint16_t* x16, const uint16_t* w, void* out, int out_dtype, const float* bias,
                     const float* rscale, int M, int K, int N, cudaStream_t s, const DeviceInfo& dev, int act = 0);
// Cluster size (K ranks) of the medium-M plan for this shape, 0 when it does not apply.
int gemm_midm_ranks(int M, int K, int N, const DeviceInfo& dev);

// Small-problem GEMM (g16_gemm_small.cu): one CTA per (tile, K chunk), K chunks of a tile reduced
// inside a thread-block cluster. bn = 0: the problem has enough tiles for the persistent kernel.
struct SmallPlan {
  int bn = 0;     // 64, 128 or 256 (N width of a tile)
  int csize = 1;  // K chunks = cluster size
  // Grid split, used instead when the caller gives a workspace of small_gs_workspace_bytes():
  // gs_split (>= 2) K chunks of gs_bn-wide tiles as independent CTAs, reduced through the workspace.
  int gs_bn = 0;
  int gs_split = 0;
};
SmallPlan plan_gemm_small(int M, int K, int N, const DeviceInfo& dev);
size_t small_gs_workspace_bytes(const SmallPlan& p, int M, int N);  // 0 without a grid split
int launch_gemm_small_gs(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                         const float* rscale, int M, int K, int N, const SmallPlan& p, void* ws, size_t ws_bytes,
                         cudaStream_t s, int act = 0);
// exact: fail with G16_ERR_UNSUPPORTED rather than run fewer K chunks than csize.
int launch_gemm_small(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                      const float* rscale, int M, int K, int N, int bn, int csize, bool exact, cudaStream_t s, int act = 0);

// 2-D TMA tensor map over a row-major [rows, cols] matrix with a [box_rows, box_cols] box (g16_tmap.cu).
int make_tmap_2d_strided(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes,
                         uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_rows, uint32_t box_cols,
                         CUtensorMapSwizzle swz);
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes, uint64_t rows,
                 uint64_t cols, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// GEMM tile geometry (also used for workspace sizing on the host).
constexpr int kBM = 128;   // UMMA M (one CTA, cta_group::1)
constexpr int kBN = 256;   // UMMA N
constexpr int kBK = 64;    // K per pipeline stage: one 128-byte swizzle row of fp16
constexpr int kUmmaK = 16; // K per tcgen05.mma for 16-bit inputs

}  // namespace g16
