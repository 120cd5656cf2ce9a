/*
 * g16.h - C ABI of the B200 (sm_100a) fp16 matmul hot path.
 *
 * Drop-in for the kernel layer of gtx16_fp16: the reference compiles seven CUDA C kernels with
 * NVRTC and launches them through ctypes cuLaunchKernel (src/gtx16_fp16/kernels.py:299-338).
 * This library replaces that layer with hand-written sm_100a kernels behind plain C entry points:
 * raw device pointers, int sizes, a dtype code and the caller's cudaStream_t passed as void*.
 *
 * Ownership: the caller owns every buffer (inputs, output, workspace). The library never
 * allocates, frees or synchronises; inputs are never written. All work is enqueued on `stream`
 * on the current CUDA device. Every entry point returns a g16_status code; none throws.
 *
 * Numerics (all paths): fp32 accumulation. GEMM path: fp16 x fp16 products on the tcgen05
 * tensor cores; fp32 activations are first cast to fp16 with the reference's per-row
 * power-of-two overflow rescale (rows with |max| > thresh). Skinny path (M <= 8): fp32 FMA of the
 * fp32/fp16 activations against fp16 weights. Results are bitwise reproducible run to run on the
 * same device (no floating-point atomics).
 */
#ifndef G16_H
#define G16_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element type codes (the reference accepts exactly these two, src/gtx16_fp16/ops.py:29-35,70-71). */
enum g16_dtype { G16_F32 = 0, G16_F16 = 1 };

enum g16_status {
  G16_OK = 0,
  G16_ERR_ARG = 1,         /* bad size, dtype code or null pointer                               */
  G16_ERR_UNSUPPORTED = 2, /* shape outside the gate of ops.py:29-35 (K % 8, N % 8)              */
  G16_ERR_ALIGN = 3,       /* a pointer is not 16-byte aligned                                    */
  G16_ERR_WORKSPACE = 4,   /* workspace missing or smaller than g16_mm_t_workspace_bytes()        */
  G16_ERR_CUDA = 5,        /* a CUDA runtime call failed; see g16_last_cuda_error()               */
  G16_ERR_DEVICE = 6,      /* the current device is not sm_100 (B200-class)                       */
  G16_ERR_TIMEOUT = 7,     /* a kernel's bounded device-side wait expired (pipeline fault)        */
  G16_ERR_TOO_LARGE = 8    /* g16_gemm_static_scratch: partials exceed its fixed scratch array    */
};

/* Largest M served by the skinny (GEMV) path: SKINNY_MAX_M, src/gtx16_fp16/kernels.py:253. */
#define G16_SKINNY_MAX_M 8
/* Rows whose |max| exceeds this are scaled by a power of two before the fp16 cast:
 * ROW_SCALE_THRESHOLD, src/gtx16_fp16/ops.py:14-16. */
#define G16_ROW_SCALE_THRESHOLD 1024.0f

/*
 * out[M,N] = x[M,K] @ w_t[K,N] + bias[N], dispatched like the reference's mm_t
 * (src/gtx16_fp16/ops.py:65-108): M <= 8 -> skinny GEMV; otherwise rowscale (fp32 x only) and the
 * tensor-core GEMM, with a deterministic split-K reduction when the output has too few tiles to
 * fill the GPU (replaces hgemm_splitk's fp32 atomics, ops.py:92-101).
 *   x        [M,K] row-major, dtype x_dtype (G16_F32 or G16_F16), 16-byte aligned
 *   w_t      [K,N] row-major fp16, 16-byte aligned
 *   bias     [N] fp32 or NULL
 *   out      [M,N] row-major, dtype out_dtype, 16-byte aligned, must not alias any input
 *   workspace/workspace_bytes: scratch of at least g16_mm_t_workspace_bytes(M,K,N,x_dtype) bytes,
 *            256-byte aligned, no initial contents required; may be NULL when that size is 0.
 *            Calls that may overlap on the GPU (different streams) need separate workspaces.
 * Requires K % 8 == 0, N % 8 == 0, M >= 0 (M == 0 is a no-op).
 */
int g16_mm_t(const void* x, int x_dtype, const void* w_t, const float* bias, void* out, int out_dtype, int M, int K,
             int N, void* workspace, size_t workspace_bytes, void* stream);

/* g16_mm_t with an activation applied by the epilogue after the bias: out = act(x @ w_t + bias)
 * (no counterpart in the reference; `patch(..., fuse=True)` folds a Linear's GELU into its GEMM
 * with it). act: G16_ACT_NONE or G16_ACT_GELU (exact erf form, x * 0.5 * (1 + erf(x / sqrt(2)))
 * in fp32 before the output cast). Same workspace as g16_mm_t; G16_ERR_ARG for another act. */
enum g16_act { G16_ACT_NONE = 0, G16_ACT_GELU = 1 };
int g16_mm_t_act(const void* x, int x_dtype, const void* w_t, const float* bias, void* out, int out_dtype, int M,
                 int K, int N, int act, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace g16_mm_t needs for this problem on the current device (0 when none). */
size_t g16_mm_t_workspace_bytes(int M, int K, int N, int x_dtype);

/*
 * g16_mm_t for fp32 activations with the per-row overflow rescale fused into the GEMM's A operand
 * (no counterpart in the reference, whose rowscale is always a separate pass, kernels.py:227-250 /
 * ops.py:86-90). A read-only pass computes each row's scale S (the rowscale rule) and 1/S without
 * writing an fp16 copy of x; the CTA-pair GEMM then loads fp32 tiles of x with TMA and converter
 * warps round x * (1/S) to fp16 in shared memory, the operand the tensor core reads; the epilogue
 * multiplies by S. The operand bits equal rowscale's, so the result equals g16_mm_t's two-pass form
 * (rowscale, then the same GEMM) bit for bit. Measured on B200 it is slower than that form (the
 * conversion, not the bytes, bounds it), so g16_mm_t does not use it. M > 8; the workspace holds
 * g16_mm_t_fused_rescale_workspace_bytes(M) bytes, 256-byte aligned; act as g16_mm_t_act;
 * G16_ERR_UNSUPPORTED where the CTA-pair kernel cannot run.
 */
int g16_mm_t_fused_rescale(const float* x, const void* w_t, const float* bias, void* out, int out_dtype, int M, int K,
                           int N, int act, void* workspace, size_t workspace_bytes, void* stream);
size_t g16_mm_t_fused_rescale_workspace_bytes(int M);

/*
 * Skinny path alone, M in [1, 8]: out[M,N] = x[M,K] @ w_t[K,N] + bias (fp32 accumulate).
 * Replaces skinny_f32in / skinny_f16in (src/gtx16_fp16/kernels.py:163-219) plus the zero-fill and
 * fp16 cast around them (ops.py:78-84). K is split across the CTAs of a thread-block cluster and
 * reduced in a fixed order through distributed shared memory, so no zeroed output is needed.
 */
int g16_skinny(const void* x, int x_dtype, const uint16_t* w_t, const float* bias, void* out, int out_dtype, int M,
               int K, int N, void* stream);

/*
 * Per-row overflow rescale: S[row] = 2^ceil(log2(amax/thresh)) if amax > thresh else 1;
 * y16 = fp16(x / S). Replaces rowscale_f32 / rowscale_f16 (src/gtx16_fp16/kernels.py:227-250).
 */
int g16_rowscale(const void* x, int x_dtype, uint16_t* y16, float* rscale, int M, int K, float thresh, void* stream);

/*
 * Tensor-core GEMM: out[M,N] = (a16[M,K] @ b16[K,N]) * rscale[row] + bias[col], fp32 accumulate in
 * TMEM, fused epilogue. Replaces hgemm_f32out / hgemm_f16out / hgemm_splitk
 * (src/gtx16_fp16/kernels.py:139-151). rscale and bias may be NULL. ksplit = 0 picks the plan
 * automatically: for M <= 64 a kernel with the operands swapped (128 weight columns per CTA as
 * the MMA's M, the rows as its N, K split over a cluster and reduced in shared memory); else,
 * when the output has too few 128 x 256 tiles to fill the GPU, a kernel with one CTA per (tile,
 * K chunk), 64-, 128- or 256-wide tiles and the K chunks of a tile reduced inside a thread-block
 * cluster (no workspace used) or, for a handful of tiles with a long K and a workspace of
 * g16_gemm_workspace_bytes(M,K,N,0) given, as independent CTAs reduced through the workspace (the
 * "grid split"; the workspace needs no initial contents, and calls that may overlap on the GPU
 * need separate workspaces); otherwise the persistent kernels. ksplit = 1 forces a
 * single pass; ksplit > 1 forces that many K chunks: 2..16 are reduced in a cluster when one can
 * be resident, else (and for ksplit > 16) through the workspace, which must hold
 * g16_gemm_workspace_bytes(M,K,N,ksplit). Both reductions add the chunks' fp32 partials in chunk
 * order, so a given ksplit gives the same bits either way.
 */
int g16_gemm(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
             const float* rscale, int M, int K, int N, int ksplit, void* workspace, size_t workspace_bytes,
             void* stream);

/* Workspace bytes for g16_gemm with the given ksplit (0 = automatic choice). */
size_t g16_gemm_workspace_bytes(int M, int K, int N, int ksplit);

/* The K split of the workspace fallback of the automatic plan (sizes its workspace). */
int g16_gemm_auto_ksplit(int M, int K, int N);

/*
 * No counterpart in the reference: an entry point for callers that cannot allocate device memory
 * at call time (e.g. servers that reserve all GPU memory for their own pools at start-up, or hosts
 * that keep cudaMalloc/cudaFree, which can synchronise the device, off latency-critical threads).
 * Same operation, arguments and launch plan as g16_gemm given a workspace of
 * G16_STATIC_SCRATCH_BYTES: the plans that need none (medium-M, small-problem and in-cluster split
 * kernels, single passes) run as they do there; the plans that need one (the small-problem grid
 * split when its partials fit, and the partial-tile split: ksplit > 16, or a split whose cluster
 * cannot be resident) keep their fp32 partial tiles in a fixed array in device memory of
 * G16_STATIC_SCRATCH_BYTES (8 MiB, 64 partial tiles of 128 x 256), held by every GPU that loads
 * the library until exit. An explicit split whose partials do not fit returns G16_ERR_TOO_LARGE
 * with nothing launched; with ksplit = 0 the grid split gives way to the cluster plan when its
 * partials do not fit, and a partial-tile split is lowered until they do (so the bits equal those
 * of g16_gemm with an 8 MiB workspace, and can differ from g16_gemm with a larger one).
 * Allocates nothing. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before any stream capture.
 * All calls on a device share the array: nothing in it needs to start at zero, but calls that
 * overlap on the GPU race on it.
 */
#define G16_STATIC_SCRATCH_BYTES (8u * 1024u * 1024u)
int g16_gemm_static_scratch(const uint16_t* a16, const uint16_t* b16, void* out, int out_dtype, const float* bias,
                            const float* rscale, int M, int K, int N, int ksplit, void* stream);

/* Launch plan the skinny path would use for (M, K, N) on the current device (introspection for
 * tests and tuning; the reference has no equivalent, its plan is skinny_config, ops.py:45-51):
 * info[0] = 1 tensor-core variant / 0 FMA variant, [1] cluster size (CTAs splitting K), [2] column
 * strips, [3] K rows per CTA, [4] dynamic shared memory bytes, [5] clusters resident at once at the
 * first cluster size tried, [6] at the chosen size. info must hold 7 ints. */
int g16_skinny_plan(int M, int K, int N, int x_dtype, int* info);

/*
 * No counterpart in the reference (it has no multi-GPU path): the column-sharded GEMM with the
 * output all-gather fused into the epilogue. This rank computes C = (a16[M,K] @ b16[K,N]) *
 * rscale[row] + bias[col] for its N columns and stores every tile into each of the ndst buffers
 * dst[d] (its own and its peers' full outputs, e.g. g16_ipc_open mappings over NVLink) at
 * dst[d][row * ldc + col0 + col], in whole 128-byte row segments (no multicast). No split-K. The caller orders the call against its peers: every rank must
 * be done with its destination buffer before any peer's call starts, and a peer's stores are
 * complete once that peer's kernel has completed (the grid ends with a system-scope fence).
 * Requires 1 <= ndst <= G16_SCATTER_MAX_DST, K % 8 == 0, N % 8 == 0, col0 + N <= ldc, col0 and
 * ldc multiples of 8, all pointers 16-byte aligned.
 */
#define G16_SCATTER_MAX_DST 8
/* flags: how the tiles reach the destinations. G16_SCATTER_DEFAULT picks the measured best;
 * G16_SCATTER_STORES: 16-byte stores by the epilogue warps; G16_SCATTER_TMA: one TMA tile store
 * (cp.async.bulk.tensor, shared -> global) per destination from the staged rows; G16_SCATTER_PAIRS:
 * the CTA-pair kernel (256 x 256 tiles on two SMs) with the same TMA tile stores (falls back to
 * G16_SCATTER_TMA where a pair cluster cannot be resident); G16_SCATTER_MULTIMEM: ndst must be 1
 * and dst[0] an NVLink multicast (NVLS) address bound to every rank's [.., ldc] output buffer (e.g.
 * torch symmetric memory's multicast_ptr): the CTA-pair kernel writes each 128-byte row segment
 * once with multimem.st and the switch delivers it to every GPU (G16_ERR_UNSUPPORTED where a pair
 * cluster cannot be resident; any other address in dst[0] is the caller's error and undefined, as
 * the library cannot tell a multicast address from another). All give the same bits. */
#define G16_SCATTER_DEFAULT 0
#define G16_SCATTER_STORES 1
#define G16_SCATTER_TMA 2
#define G16_SCATTER_PAIRS 3
#define G16_SCATTER_MULTIMEM 4
int g16_gemm_scatter(const uint16_t* a16, const uint16_t* b16, void* const* dst, int ndst, int out_dtype,
                     const float* bias, const float* rscale, int M, int K, int N, long long ldc, int col0,
                     int flags, void* stream);

/*
 * No counterpart in the reference (it has no multi-GPU path): the column-sharded GEMM with both the
 * output all-gather and the completion barrier fused into the kernel, so a call needs no host
 * collective. mc_out: NVLink multicast address bound to every rank's [M, ldc] output buffer (as for
 * G16_SCATTER_MULTIMEM); this rank's tiles land at column col0 of every copy. mc_flag: multicast
 * address of a 32-bit counter bound on every rank; flag: this GPU's copy of it. After its last
 * store each CTA of every rank adds 1 to the counter on every GPU (multimem.red.release.sys); a
 * one-thread kernel, enqueued after the GEMM, then waits until this GPU's counter reaches `target`
 * (compared mod 2^32), so later work on `stream` sees every rank's tiles. The caller keeps the
 * running target: previous target + the sum over all ranks of g16_gemm_allgather_signals(M, K, N)
 * (counters start at 0 on every GPU before the first call). The wait is bounded by wait_limit_us
 * (1 .. 60,000,000): on expiry it records G16_ERR_TIMEOUT in the device status word
 * (g16_device_status) and returns. Consecutive calls must use different output buffers (a peer may
 * start call i + 1 while this rank still reads the result of call i); alternating two buffers is
 * enough when each rank reads a result on `stream` before its next call, because a peer's call
 * i + 1 starts only after this rank's kernel of call i, and so its reads of the result of call
 * i - 1 enqueued before it, has finished. Requirements as g16_gemm_scatter;
 * G16_ERR_UNSUPPORTED where a CTA-pair cluster cannot be resident.
 */
int g16_gemm_allgather_mc(const uint16_t* a16, const uint16_t* b16, void* mc_out, int out_dtype, const float* bias,
                          const float* rscale, int M, int K, int N, long long ldc, int col0, void* mc_flag,
                          const uint32_t* flag, uint32_t target, int wait_limit_us, void* stream);
/* Counter increments one g16_gemm_allgather_mc call of this rank makes on every GPU (its CTAs), or
 * minus a g16_status code. */
int g16_gemm_allgather_signals(int M, int K, int N);

/*
 * No counterpart in the reference: device buffers shared between the processes of one node with
 * CUDA IPC, the destinations of g16_gemm_scatter. g16_ipc_alloc allocates `bytes` on the current
 * device (cudaMalloc, so the buffer starts an allocation of its own and its handle maps it
 * exactly); g16_ipc_get_handle writes its G16_IPC_HANDLE_BYTES-byte handle; another process opens
 * it with g16_ipc_open (peer access enabled on first use) and releases it with g16_ipc_close
 * before the owner calls g16_ipc_free.
 */
#define G16_IPC_HANDLE_BYTES 64
int g16_ipc_alloc(size_t bytes, void** ptr);
int g16_ipc_free(void* ptr);
int g16_ipc_get_handle(void* ptr, void* handle);
int g16_ipc_open(const void* handle, void** ptr);
int g16_ipc_close(void* ptr);

/* Plan g16_gemm uses for ksplit = 0 on the current device (introspection for tests and tuning; no
 * counterpart in the reference, whose choice is the split-K rule of ops.py:92-101): info[0] = 2 the
 * medium-M kernel (M <= 64: weight columns as the MMA's M, 128-column strips) / 3 the
 * small-problem kernel's grid split (K chunks as independent CTAs reduced through the workspace;
 * without a workspace the cluster plan of kind 1 runs instead) / 1 the small-problem kernel (one
 * CTA per tile and K chunk, chunks reduced in a cluster) / 0 the persistent kernels, [1] tile width
 * (64, 128 or 256; the strip width for kind 2), [2] K chunks (cluster size; for the persistent kernel
 * the workspace split). info must hold 3 ints. */
int g16_gemm_plan(int M, int K, int N, int* info);

/* Device-side status word of the current device: G16_OK, or G16_ERR_TIMEOUT if a kernel's
 * bounded wait expired since the last clear. Synchronises `stream`. clear != 0 resets it. */
int g16_device_status(int* status_out, int clear, void* stream);

/* No counterpart in the reference (its failure surface is the launch error of kernels.py:300-302):
 * a failure-detection self-test. Launches one small kernel whose bounded device-side waits run out
 * on purpose: one role waits limit_us microseconds (1 .. 1,000,000) on an mbarrier nothing arrives
 * on, then records G16_ERR_TIMEOUT in the device status word and raises its CTA's abort flag; a
 * second role, waiting with the library's full 1 s limit, leaves as soon as it sees the flag. No
 * fault, no trap, no hang: the kernel ends shortly after limit_us and the context stays usable.
 * Read (and clear) the result with g16_device_status. Returns G16_ERR_ARG for limit_us out of range. */
int g16_selftest_wait_timeout(int limit_us, void* stream);

/* Number of kernels this library has launched in this process (all devices). */
uint64_t g16_launch_count(void);

/* Human-readable text for a g16_status code; the last CUDA error text for G16_ERR_CUDA. */
const char* g16_strerror(int status);
int g16_last_cuda_error(void);

/* Library ABI version (major * 10000 + minor * 100 + patch). */
int g16_version(void);

#ifdef __cplusplus
}
#endif

#endif /* G16_H */
