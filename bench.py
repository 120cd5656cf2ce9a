"""Benchmark of the gtx16_fp16 hot path on B200 (prints one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (a "step" is one call of the hot path on one batch of synthetic input):
  gemm4096   gtx16_fp16.matmul, fp16 4096x4096x4096 -> fp16 (config 3; the headline metric)   [default]
  gemm1024   gtx16_fp16.matmul, fp16 1024^3 (config 1 on the GPU)
  skinny*    mm_t M in {1,4,8} at K=N=4096 and M in {1,4} at K=1024, N=3072; fp32 x, fp16 w_t,
             fp32 bias/out (config 2)
  splitk*    mm_t 128x16384x1024 and 64x1024x1024 fp16 -> fp16 (config 3, split-K shapes)
  rescale    mm_t 2048x3072x1024 fp32 x with 1% rows x [100,200] (config 4)
  bert*      BERT-base, 256 x 256 tokens, every Linear patched (config 5); variants with fp16
             activations and with the GELU/QKV fusion
  decode16   16 FastLinear(4096, 4096) layers at M=1 per step, replayed from a CUDA graph
             (gtx16_fp16.graphs); decode16_eager calls the same layers from Python
The top-level line is the chosen workload as N independent replicas (no exchange step for these
shapes; scaling "weak"), value = sum over ranks (max-over-ranks time). `sub` (N=1 only) measures the
other workloads briefly. `collective` holds the blocks every rank runs at every N: `gemm16384`
(16384^3 with w_t N-sharded over the ranks and the all-gather fused into the GEMM epilogue; strong
scaling, fp64 parity on 256 sampled rows, efficiency against the same run's 1-GPU 16384^3) and
`bert` (data parallel over the 256 sequences, cosine against fp32 over all of them).

Timing: W untimed warm-up steps, then K steps between barrier + synchronize, timed with CUDA events
on the launching stream. Inputs rotate over several sets whose total exceeds the 126 MB L2, so every
step reads its operands from HBM. Clocks and throttle reasons are sampled with NVML during the timed
region. `e2e` repeats the step through the public API from pinned host memory (H2D of the inputs and
D2H of the result inside the timed region). `cpu_baseline` times the reference's CPU path
(oracle/cpu_path.py: torch fp32 matmul) on a bounded sample on the host cores (rank 0, N=1 only).
Each roofline is the binding one of its shape: FLOPs at the measured bf16 peak or algorithmic bytes
at the measured copy bandwidth, whichever takes longer.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "gtx16-fp16_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def load_profile_traffic():
    """Per-launch DRAM bytes of each workload's dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except ValueError:
            return {}
    return {}


# ---------------------------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device_index: int, interval_s: float = 0.005):
        self.interval = interval_s
        self.samples: list[tuple[int, int]] = []
        self.sm_max = None
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            uuid = None
            try:
                uuid = torch.cuda.get_device_properties(device_index).uuid
            except Exception:
                pass
            self.h = None
            if uuid is not None:
                try:
                    self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(uuid)).encode())
                except Exception:
                    self.h = None
            if self.h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[device_index]) if vis and vis.split(",")[0].isdigit() else device_index
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.sm_max = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.ok = True
        except Exception as e:  # no NVML: report that instead of clocks
            self.err = str(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = int(self._reasons_fn(self.h))
                self.samples.append((sm, rs))
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"error": getattr(self, "err", "nvml unavailable")}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.sm_max, "reasons": [], "samples": 0}
        sms = sorted(s for s, _ in self.samples)
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [name for bit, name in self.REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": self.sm_max, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------------
class Workload:
    name = ""
    metric = ""
    unit = ""
    bound = "tensor"
    graphable = True
    scaling = "weak"

    def __init__(self, dev):
        self.dev = dev

    def flops(self) -> float:
        return 0.0

    def alg_bytes(self) -> float:
        return 0.0

    def close(self):
        """Release collective resources (every rank calls it, in the same order)."""

    # Double-buffered end-to-end steps (workloads whose step is one call on a few input tensors):
    # e2e_compute(g16, dev_inputs) -> the step's device result.
    e2e_compute = None


def _rotating_sets(nbytes_per_set: int) -> int:
    return max(3, int(2 * L2_BYTES // max(nbytes_per_set, 1)) + 1)


def binding_bound(flops: float, nbytes: float, peaks: dict) -> str:
    """"tensor" or "hbm": whichever roofline takes longer for this much work (FLOPs at the measured
    bf16 peak against algorithmic bytes at the measured copy bandwidth)."""
    t_tensor = flops / (peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]) * 1e12)
    t_hbm = nbytes / (peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]) * 1e9)
    return "tensor" if t_tensor >= t_hbm else "hbm"


class Gemm(Workload):
    """gtx16_fp16.matmul: fp16 A[M,K] @ fp16 B[K,N] -> fp16."""

    def __init__(self, dev, M, K, N, name):
        super().__init__(dev)
        self.M, self.K, self.N = M, K, N
        self.name = name
        self.bound = binding_bound(self.flops(), self.alg_bytes(), load_peaks()[0])
        self.metric = f"GEMM TFLOPS (fp16 {M}x{K}x{N}, gtx16_fp16.matmul)"
        self.unit = "TFLOPS"
        per = (M * K + K * N + M * N) * 2
        self.nsets = _rotating_sets(per)
        g = torch.Generator(device=dev).manual_seed(0)
        self.A = [torch.randn(M, K, device=dev, generator=g).half() for _ in range(self.nsets)]
        self.B = [(torch.randn(K, N, device=dev, generator=g) * K ** -0.5).half() for _ in range(self.nsets)]
        self.i = 0

    def config(self):
        return {"workload": self.name, "M": self.M, "K": self.K, "N": self.N, "in": "fp16", "out": "fp16",
                "inputs": "A~N(0,1), B~N(0,1/sqrt(K)) fp16, seed 0 (BASELINE config 3)",
                "l2": f"{self.nsets} rotating input sets ({self.nsets * (self.M * self.K + self.K * self.N) * 2 >> 20} MiB) > 126 MB L2"}

    def flops(self):
        return 2.0 * self.M * self.N * self.K

    def alg_bytes(self):
        return 2.0 * (self.M * self.K + self.K * self.N + self.M * self.N)

    def step(self, g16):
        j = self.i % self.nsets
        self.i += 1
        return g16.matmul(self.A[j], self.B[j])

    # e2e through the public API from pinned host memory
    def host_inputs(self):
        return [self.A[0].cpu().pin_memory(), self.B[0].cpu().pin_memory()]

    def host_out(self):
        return torch.empty(self.M, self.N, dtype=torch.float16).pin_memory()

    def e2e_step(self, g16, hin, hout):
        a = hin[0].to(self.dev, non_blocking=True)
        b = hin[1].to(self.dev, non_blocking=True)
        hout.copy_(g16.matmul(a, b), non_blocking=True)

    def e2e_compute(self, g16, dev_in):
        return g16.matmul(dev_in[0], dev_in[1])

    def cpu_sample(self):
        """The reference CPU path on a bounded sample: fp32 torch.matmul of 512 rows x full B."""
        rows = min(self.M, 512)
        a = self.A[0][:rows].float().cpu()
        b = self.B[0].float().cpu()
        return (lambda: torch.matmul(a, b)), 2.0 * rows * self.N * self.K, f"fp32 torch.matmul {rows}x{self.K}x{self.N} (rows of the workload)"


class MmT(Workload):
    """gtx16_fp16.mm_t(x, w_t, bias, out_dtype) (BASELINE configs 2 and 4)."""

    def __init__(self, dev, M, K, N, name, xdt, out_dtype, wstd, bias_std, rescale=False):
        super().__init__(dev)
        self.M, self.K, self.N = M, K, N
        self.name = name
        self.xdt, self.out_dtype = xdt, out_dtype
        self.skinny = M <= 8
        self.bound = "hbm" if self.skinny else binding_bound(self.flops(), self.alg_bytes(), load_peaks()[0])
        self.metric = (f"skinny mm_t HBM GB/s (M={M}, {K}x{N})" if self.skinny else
                       f"mm_t TFLOPS ({M}x{K}x{N}{', overflow rescale' if rescale else ''})")
        self.unit = "GB/s" if self.skinny else "TFLOPS"
        xs = 4 if xdt == torch.float32 else 2
        per = M * K * xs + K * N * 2 + M * N * 4
        self.nsets = _rotating_sets(per)
        g = torch.Generator(device=dev).manual_seed(0)
        self.X, self.W = [], []
        for _ in range(self.nsets):
            x = torch.randn(M, K, device=dev, generator=g)
            if rescale:
                rows = torch.randperm(M, device=dev, generator=g)[: max(1, M // 100)]
                f = torch.exp(torch.empty(len(rows), device=dev).uniform_(4.6051702, 5.2983174, generator=g))
                x[rows] *= f[:, None]
            self.X.append(x.to(xdt))
            self.W.append((torch.randn(K, N, device=dev, generator=g) * wstd).half())
        self.b = torch.randn(N, device=dev, generator=g) * bias_std if bias_std else torch.zeros(N, device=dev)
        self.rescale = rescale
        self.i = 0

    def config(self):
        return {"workload": self.name, "M": self.M, "K": self.K, "N": self.N,
                "in": "fp32" if self.xdt == torch.float32 else "fp16", "w": "fp16",
                "out": "fp32" if self.out_dtype == torch.float32 else "fp16",
                "l2": f"{self.nsets} rotating input sets > 126 MB L2"}

    def flops(self):
        return 2.0 * self.M * self.N * self.K

    def alg_bytes(self):
        xs = 4 if self.xdt == torch.float32 else 2
        os_ = 4 if self.out_dtype == torch.float32 else 2
        return float(2 * self.K * self.N + xs * self.M * self.K + 4 * self.N + os_ * self.M * self.N)

    def step(self, g16):
        j = self.i % self.nsets
        self.i += 1
        return g16.mm_t(self.X[j], self.W[j], self.b, self.out_dtype)

    def host_inputs(self):
        return [self.X[0].cpu().pin_memory(), self.W[0].cpu().pin_memory()]

    def host_out(self):
        return torch.empty(self.M, self.N, dtype=self.out_dtype).pin_memory()

    def e2e_step(self, g16, hin, hout):
        x = hin[0].to(self.dev, non_blocking=True)
        w = hin[1].to(self.dev, non_blocking=True)
        hout.copy_(g16.mm_t(x, w, self.b, self.out_dtype), non_blocking=True)

    def e2e_compute(self, g16, dev_in):
        return g16.mm_t(dev_in[0], dev_in[1], self.b, self.out_dtype)

    def cpu_sample(self):
        rows = min(self.M, 512)
        x = self.X[0][:rows].float().cpu()
        w = self.W[0].float().cpu()
        b = self.b.cpu()
        from oracle import cpu_path
        return (lambda: cpu_path.mm_t_fp32(x, w.half(), b)), 2.0 * rows * self.N * self.K, \
            f"fp32 F.linear {rows}x{self.K}x{self.N} (reference linear.py fallback)"


class FusedRescale(MmT):
    """fp32-activation GEMM with the row rescale fused into the GEMM's A operand
    (g16_mm_t_fused_rescale: row-amax pass + CTA-pair GEMM converting fp32 tiles in shared memory),
    measured beside mm_t's default two-pass form (rowscale, then the GEMM) on the same inputs."""

    def __init__(self, dev, M, K, N, name, rescale):
        super().__init__(dev, M, K, N, name, torch.float32, torch.float32, 0.02, 0.0, rescale=rescale)
        self.metric = f"fused-rescale GEMM TFLOPS ({M}x{K}x{N}, fp32 x, g16_mm_t_fused_rescale)"
        from gtx16_fp16 import _native
        self._L = _native.lib()
        n = int(self._L.g16_mm_t_fused_rescale_workspace_bytes(M))
        self.ws = torch.empty(max(n, 256), dtype=torch.uint8, device=dev)
        self.O = torch.empty(M, N, device=dev)

    def config(self):
        return dict(super().config(), path="row-amax pass + CTA-pair GEMM with fp32-A converter warps")

    def step(self, g16):
        from gtx16_fp16 import _native
        j = self.i % self.nsets
        self.i += 1
        st = self._L.g16_mm_t_fused_rescale(self.X[j].data_ptr(), self.W[j].data_ptr(), self.b.data_ptr(),
                                            self.O.data_ptr(), _native.G16_F32, self.M, self.K, self.N,
                                            _native.ACT_NONE, self.ws.data_ptr(), self.ws.numel(),
                                            _native.stream_handle(self.dev.index or 0))
        _native.check(st, "g16_mm_t_fused_rescale")
        return self.O


class ShardedGemm(Workload):
    """16384^3 fp16 GEMM with w_t split by columns over the ranks (1/2/4/8 GPUs):
    each rank holds A (replicated) and its column shard of B and computes its output columns; the
    GEMM epilogue stores every output tile into each rank's full C (gtx16_fp16.dist.ShardedMatmul,
    CUDA IPC over NVLink), so the all-gather overlaps the math. A step ends with the full C on
    every rank. Total work is fixed: strong scaling."""
    bound = "tensor"
    graphable = False
    multicast = None  # ShardedMatmul.multicast: None = NVLink multicast where supported, False = peer stores

    def __init__(self, dev, world, rank, M=16384, K=16384, N=16384, sample_rows=0, keep_full_b=False):
        super().__init__(dev)
        from gtx16_fp16.dist import ShardedMatmul, shard_bounds
        self.M, self.K, self.N, self.world, self.rank = M, K, N, world, rank
        self._exchange = None
        self.name = "gemm16384"
        self.metric = f"GEMM TFLOPS (fp16 {M}x{K}x{N}, N-sharded over GPUs, all-gather fused into the epilogue)"
        self.unit = "TFLOPS"
        self.scaling = "strong"
        g = torch.Generator(device=dev).manual_seed(0)
        self.A = torch.randn(M, K, device=dev, generator=g).half()
        n0, n1 = shard_bounds(N, world, rank)
        b = torch.empty(K, n1 - n0, device=dev, dtype=torch.float16)
        self.B_full = torch.empty(K, N, device=dev, dtype=torch.float16) if keep_full_b else None
        # fp64 truth for `sample_rows` seeded rows of the full output: A[rows] @ B, panel by panel
        self.rows = None
        if sample_rows:
            self.rows = torch.randperm(M, generator=torch.Generator().manual_seed(1))[:sample_rows].sort().values
            a_s = self.A[self.rows.to(dev)].double()
            self.ref_rows = torch.empty(sample_rows, N, device=dev, dtype=torch.float64)
            self.mag_rows = torch.empty(sample_rows, N, device=dev, dtype=torch.float64)
        # B ~ N(0, 1/sqrt(K)) generated in 2048-column panels so every rank draws the same B
        for c0 in range(0, N, 2048):
            panel = (torch.randn(K, min(2048, N - c0), device=dev, generator=g) * K ** -0.5).half()
            c1 = c0 + panel.shape[1]
            lo, hi = max(c0, n0), min(c1, n1)
            if lo < hi:
                b[:, lo - n0:hi - n0] = panel[:, lo - c0:hi - c0]
            if self.B_full is not None:
                self.B_full[:, c0:c1] = panel
            if sample_rows:
                p64 = panel.double()
                self.ref_rows[:, c0:c1] = a_s @ p64
                self.mag_rows[:, c0:c1] = a_s.abs() @ p64.abs()
                del p64
            del panel
        if sample_rows:
            del a_s
        self.B = b
        self.sm = ShardedMatmul(self.B, N, out_dtype=torch.float16, multicast=self.multicast)

    def check_rows(self, out):
        """(norm-wise, component-wise) relative error of the sampled rows of the full output against
        fp64: ||y - ref|| / ||ref|| and max |y - ref| / (|A| @ |B|)."""
        y = out[self.rows.to(out.device)].double()
        d = y - self.ref_rows
        norm = float(d.norm() / self.ref_rows.norm())
        comp = float((d.abs() / self.mag_rows.clamp_min(1e-300)).max())
        finite = bool(torch.isfinite(y).all())
        return norm, comp, finite

    def config(self):
        return {"workload": self.name, "M": self.M, "K": self.K, "N": self.N, "in": "fp16", "out": "fp16",
                "shard": f"w_t columns [{self.sm.n0}, {self.sm.n1}) on rank {self.rank}",
                "exchange": self._exchange or self.exchange(),
                "inputs": "A~N(0,1), B~N(0,1/sqrt(K)) fp16, seed 0 (BASELINE config 3)",
                "l2": "A alone is 512 MiB > 126 MB L2"}

    def flops(self):
        return 2.0 * self.M * self.N * self.K / self.world  # per rank (value sums over ranks)

    def alg_bytes(self):
        return 2.0 * (self.M * self.K + self.K * self.N / self.world + self.M * self.N)

    def step(self, g16):
        return self.sm(self.A)

    def local_step(self, g16):
        return self.sm.local(self.A)

    def exchange(self):
        from gtx16_fp16.dist import MulticastBuffer
        if self.world == 1:
            return "none (one rank)"
        bufs = list(self.sm._bufs.values())
        if not bufs:
            return "not run"
        return ("NVLink multicast stores (multimem.st) from the GEMM epilogue; completion signalled by the "
                "kernel through a multicast counter, no host collective per call"
                if isinstance(bufs[0], MulticastBuffer) else
                "peer TMA stores from the GEMM epilogue (CUDA IPC); two NCCL all-reduces per call order buffer reuse")

    def close(self):
        self._exchange = self.exchange()
        self.sm.close()

    def host_inputs(self):
        return [self.A.cpu().pin_memory(), self.B.cpu().pin_memory()]

    def host_out(self):
        return torch.empty(self.M, self.N, dtype=torch.float16).pin_memory()

    def e2e_step(self, g16, hin, hout):
        a = hin[0].to(self.dev, non_blocking=True)
        self.B.copy_(hin[1], non_blocking=True)
        hout.copy_(self.sm(a), non_blocking=True)

    def cpu_sample(self):
        rows = 256
        a = self.A[:rows].float().cpu()
        b = self.B[:, : min(2048, self.B.shape[1])].float().cpu()
        return (lambda: torch.matmul(a, b)), 2.0 * rows * b.shape[1] * self.K, \
            f"fp32 torch.matmul {rows}x{self.K}x{b.shape[1]} (a block of the workload)"


class Decode(Workload):
    """Token-by-token decode through FastLinear: x [1, 4096] fp32 through 16 FastLinear(4096, 4096)
    layers per step (BASELINE config 2's skinny shape, the reference's batch-1 usage measured by
    its bench/overhead.py). graphed: the step is captured once with gtx16_fp16.graphs.capture and
    replayed (input copy, one graph launch, output clone per step); eager: the 16 layers are
    called from Python each step, host cost included. The 16 weights (512 MiB) exceed L2, so every
    step streams them from HBM."""
    bound = "hbm"
    graphable = False  # the graphed variant replays its own graph; the eager one measures Python

    def __init__(self, dev, graphed, layers=16, K=4096, M=1):
        super().__init__(dev)
        import torch.nn as nn

        import gtx16_fp16 as g16
        self.graphed, self.layers, self.K, self.M = graphed, layers, K, M
        self.name = "decode16" if graphed else "decode16_eager"
        self.metric = (f"FastLinear decode step HBM GB/s ({layers} x {K}x{K} layers, M={M}, "
                       f"{'CUDA graph via gtx16_fp16.graphs' if graphed else 'eager Python calls'})")
        self.unit = "GB/s"
        g = torch.Generator(device=dev).manual_seed(0)
        mods = []
        for _ in range(layers):
            fl = g16.FastLinear(K, K, bias=True, device=dev)
            with torch.no_grad():
                fl.weight_t.copy_((torch.randn(K, K, device=dev, generator=g) * 0.02).half())
                fl.bias.copy_(torch.randn(K, device=dev, generator=g) * 0.01)
            mods.append(fl)
        self.model = nn.Sequential(*mods).eval()
        self.x = torch.randn(M, K, device=dev, generator=g)
        self.graph_step = g16.graphs.capture(self.model, self.x) if graphed else None

    def config(self):
        return {"workload": self.name, "layers": self.layers, "M": self.M, "K": self.K, "N": self.K,
                "in": "fp32", "w": "fp16", "out": "fp32", "mode": "graph replay" if self.graphed else "eager",
                "l2": f"{self.layers} weights = {self.layers * self.K * self.K * 2 >> 20} MiB > 126 MB L2"}

    def alg_bytes(self):
        per = 2 * self.K * self.K + 4 * self.M * self.K + 4 * self.K + 4 * self.M * self.K
        return float(self.layers * per)

    def flops(self):
        return 2.0 * self.layers * self.M * self.K * self.K

    def step(self, g16):
        with torch.no_grad():
            return self.graph_step(self.x) if self.graphed else self.model(self.x)

    def host_inputs(self):
        return [self.x.cpu().pin_memory()]

    def host_out(self):
        return torch.empty(self.M, self.K, dtype=torch.float32).pin_memory()

    def e2e_step(self, g16, hin, hout):
        x = hin[0].to(self.dev, non_blocking=True)
        with torch.no_grad():
            y = self.graph_step(x) if self.graphed else self.model(x)
        hout.copy_(y, non_blocking=True)

    def cpu_sample(self):
        from oracle import cpu_path
        ws = [m.weight_t.cpu() for m in self.model[:4]]
        bs = [m.bias.cpu() for m in self.model[:4]]
        x = self.x.cpu()

        def run():
            y = x
            for w, b in zip(ws, bs):
                y = cpu_path.mm_t_fp32(y, w, b)
            return y
        return run, 2.0 * 4 * self.M * self.K * self.K, "fp32 F.linear through 4 of the 16 layers (reference linear.py fallback)"


class Bert(Workload):
    """BERT-base encoder inference with every Linear patched to FastLinear:
    random init (seed 0), fp32 activations, 256 sequences x 256 tokens, ids uniform in
    [1000, 30521], full attention mask. Data parallel: rank r runs its slice of the 256 sequences;
    value = 256 / (max-rank step time). The CLS embeddings are L2-normalised and compared with the
    unpatched fp32 model (cosine >= 0.9999)."""
    bound = "tensor"
    graphable = False

    def __init__(self, dev, world, rank, batch=256, seq=256, reference=False, half=False, fuse=False):
        super().__init__(dev)
        import copy
        import gtx16_fp16 as g16
        from gtx16_fp16.dist import batch_slice
        from transformers import BertConfig, BertModel
        self.half, self.fuse = half, fuse
        self.name = ("bert16" if half else "bert") + ("_fused" if fuse else "")
        opts = ", ".join(o for o, on in (("fp16 activations", half), ("GELU/QKV fused", fuse)) if on)
        self.metric = (f"BERT-base texts/s (256 x 256 tokens, FastLinear{', ' + opts + ' (opt-in)' if opts else ''}, "
                       "data parallel)")
        self.unit = "texts/s"
        self.scaling = "strong"
        self.world, self.rank, self.batch, self.seq = world, rank, batch, seq
        cfg = BertConfig(vocab_size=30522, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                         intermediate_size=3072, hidden_act="gelu", max_position_embeddings=512,
                         attn_implementation="sdpa")
        self.cfg = cfg
        self.n_patched = 0
        if not reference:  # the reference arm only runs the CPU model (cpu_sample)
            torch.manual_seed(0)
            model = BertModel(cfg).eval()
            self.ref_model = copy.deepcopy(model).to(dev)
            self.model = model.to(dev)
            self.n_patched = g16.patch(self.model, force=True, activations=torch.float16 if half else None, fuse=fuse)
        gen = torch.Generator().manual_seed(0)
        ids = torch.randint(1000, 30522, (batch, seq), generator=gen)
        sl = batch_slice(batch, world, rank)
        self.local_batch = sl.stop - sl.start
        self.ids_host = ids[sl].contiguous()
        self.ids = self.ids_host.to(dev) if not reference else None
        self.mask = torch.ones_like(self.ids) if not reference else None
        self.cos_min = None

    def config(self):
        return {"workload": self.name, "model": "BERT-base (12 x 768, 12 heads, FFN 3072, random init seed 0)",
                "global_batch": self.batch, "seq_len": self.seq, "local_batch": self.local_batch,
                "patched_linears": self.n_patched, "activations": "fp16" if self.half else "fp32",
                "fused": "GELU into the FFN GEMM, one QKV GEMM" if self.fuse else "none",
                "attention": f"torch sdpa ({'fp16' if self.half else 'fp32'})",
                "cosine_min_vs_fp32": self.cos_min, "l2": "activations 200+ MB per layer > 126 MB L2"}

    def flops(self):  # Linear FLOPs of this rank's slice (the part that runs on libg16)
        tokens = self.local_batch * self.seq
        return 2.0 * tokens * 12 * (4 * 768 * 768 + 2 * 768 * 3072) + 2.0 * self.local_batch * 768 * 768

    def alg_bytes(self):
        return 0.0

    def step(self, g16):
        with torch.no_grad():
            return self.model(input_ids=self.ids, attention_mask=self.mask).last_hidden_state[:, 0]

    def check_cosine(self):
        with torch.no_grad():
            ref = self.ref_model(input_ids=self.ids, attention_mask=self.mask).last_hidden_state[:, 0]
            got = self.step(None)
        ref = torch.nn.functional.normalize(ref.float(), dim=-1)
        got = torch.nn.functional.normalize(got.float(), dim=-1)
        self.cos_min = round(float((ref * got).sum(-1).min()), 7)
        del self.ref_model
        torch.cuda.empty_cache()
        return self.cos_min

    def host_inputs(self):
        return [self.ids_host.pin_memory()]

    def host_out(self):
        return torch.empty(self.local_batch, 768, dtype=torch.float32).pin_memory()

    def e2e_step(self, g16, hin, hout):
        ids = hin[0].to(self.dev, non_blocking=True)
        with torch.no_grad():
            cls = self.model(input_ids=ids, attention_mask=torch.ones_like(ids)).last_hidden_state[:, 0]
        hout.copy_(torch.nn.functional.normalize(cls, dim=-1), non_blocking=True)

    def cpu_sample(self):
        """The reference CPU path for this model: the unpatched fp32 model on the host (4 sequences)."""
        import copy
        from transformers import BertConfig, BertModel
        torch.manual_seed(0)
        cpu_model = BertModel(self.cfg).eval()
        ids = self.ids_host[:4]
        mask = torch.ones_like(ids)

        def run():
            with torch.no_grad():
                cpu_model(input_ids=ids, attention_mask=mask)
        return run, 4.0, "unpatched fp32 BERT-base forward, 4 x 256 tokens on the host"


WORKLOADS = {
    "gemm4096": lambda dev, w, r: Gemm(dev, 4096, 4096, 4096, "gemm4096"),
    "gemm1024": lambda dev, w, r: Gemm(dev, 1024, 1024, 1024, "gemm1024"),
    "splitk": lambda dev, w, r: Gemm(dev, 128, 16384, 1024, "splitk"),
    "splitk64": lambda dev, w, r: Gemm(dev, 64, 1024, 1024, "splitk64"),
    "gemm16384": lambda dev, w, r: ShardedGemm(dev, w, r),
    "skinny": lambda dev, w, r: MmT(dev, 8, 4096, 4096, "skinny", torch.float32, torch.float32, 0.02, 0.01),
    "skinny1": lambda dev, w, r: MmT(dev, 1, 4096, 4096, "skinny1", torch.float32, torch.float32, 0.02, 0.01),
    "skinny4": lambda dev, w, r: MmT(dev, 4, 4096, 4096, "skinny4", torch.float32, torch.float32, 0.02, 0.01),
    "skinny1x3072": lambda dev, w, r: MmT(dev, 1, 1024, 3072, "skinny1x3072", torch.float32, torch.float32, 0.02, 0.01),
    "skinny4x3072": lambda dev, w, r: MmT(dev, 4, 1024, 3072, "skinny4x3072", torch.float32, torch.float32, 0.02, 0.01),
    "rescale": lambda dev, w, r: MmT(dev, 2048, 3072, 1024, "rescale", torch.float32, torch.float32, 0.02, 0.0,
                                     rescale=True),
    "rescale_fused": lambda dev, w, r: FusedRescale(dev, 2048, 3072, 1024, "rescale_fused", True),
    "linear768": lambda dev, w, r: MmT(dev, 65536, 768, 768, "linear768", torch.float32, torch.float32, 0.02, 0.0),
    "linear768_fused": lambda dev, w, r: FusedRescale(dev, 65536, 768, 768, "linear768_fused", False),
    "bert": lambda dev, w, r: Bert(dev, w, r),
    "bert_fused": lambda dev, w, r: Bert(dev, w, r, fuse=True),
    "bert16": lambda dev, w, r: Bert(dev, w, r, half=True),
    "bert16_fused": lambda dev, w, r: Bert(dev, w, r, half=True, fuse=True),
    "decode16": lambda dev, w, r: Decode(dev, True),
    "decode16_eager": lambda dev, w, r: Decode(dev, False),
}


# ---------------------------------------------------------------------------------------------
def timed_loop(wl, g16, steps, stream, graph=None):
    """Device milliseconds for `steps` consecutive steps, CUDA events on the launching stream.

    With `graph` (a CUDA graph holding exactly `steps` captured steps) the steps are replayed from
    the graph, so host launch overhead does not stretch microsecond-scale steps."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replay() and the steps launch on the current stream
        start.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for _ in range(steps):
                wl.step(g16)
        end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def capture_steps(wl, g16, steps, stream):
    """(graph, launches): a CUDA graph of `steps` consecutive steps captured on `stream` (warmed up
    on it first) and the number of libg16 kernel launches it holds."""
    from gtx16_fp16 import _native
    with torch.cuda.stream(stream):
        for _ in range(3):
            wl.step(g16)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    l0 = _native.launch_count()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(steps):
            wl.step(g16)
    launches = _native.launch_count() - l0
    stream.synchronize()
    return graph, launches


def run_ours(args, rank, world, dev):
    import gtx16_fp16 as g16
    from gtx16_fp16 import _native

    peaks, peak_src = load_peaks()
    wl = WORKLOADS[args.workload](dev, world, rank)
    if isinstance(wl, Bert):
        wl.check_cosine()
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        wl.step(g16)
    torch.cuda.synchronize(dev)
    graph = None
    if args.graph and wl.graphable:
        gstream = torch.cuda.Stream(dev)
        graph, launches = capture_steps(wl, g16, args.steps, gstream)
        stream = gstream
        with torch.cuda.stream(stream):
            graph.replay()  # one untimed replay: the warm-up of the captured work
        torch.cuda.synchronize(dev)

    sampler = ClockSampler(dev.index or 0)
    barrier(world)
    torch.cuda.synchronize(dev)
    if graph is None:
        l0 = _native.launch_count()
    with sampler:
        ms = timed_loop(wl, g16, args.steps, stream, graph)
    torch.cuda.synchronize(dev)
    if graph is None:
        launches = _native.launch_count() - l0
    barrier(world)
    ms_max = reduce_max(ms, world, dev)
    ms_step = ms_max / args.steps

    if wl.unit == "TFLOPS":
        per_rank_units = wl.flops() / 1e12
    elif wl.unit == "texts/s":
        per_rank_units = float(wl.local_batch)
    else:
        per_rank_units = wl.alg_bytes() / 1e9
    value = world * per_rank_units / (ms_step * 1e-3)
    if wl.unit == "texts/s":
        value = wl.batch / (ms_step * 1e-3)  # the whole batch per max-rank step time

    # e2e through the public API with host buffers
    stream = torch.cuda.current_stream(dev)
    hin, hout = wl.host_inputs(), wl.host_out()
    e2e_steps = max(3, min(args.steps, 50))
    if wl.e2e_compute is not None:
        pipe = E2EPipeline(wl, g16, hin, hout, dev)
        pipe.run(max(2, args.warmup // 4))
        torch.cuda.synchronize(dev)
        barrier(world)
        e2e_ms = reduce_max(pipe.run(e2e_steps), world, dev) / e2e_steps
        e2e_mode = "double-buffered: H2D of step i+1, compute of step i and D2H of step i-1 on three streams"
    else:
        for _ in range(max(2, args.warmup // 4)):
            wl.e2e_step(g16, hin, hout)
        torch.cuda.synchronize(dev)
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(e2e_steps):
            wl.e2e_step(g16, hin, hout)
        e.record(stream)
        e.synchronize()
        e2e_ms = reduce_max(s.elapsed_time(e), world, dev) / e2e_steps
        e2e_mode = "serial: H2D, compute, D2H per step on one stream"
    h2d = sum(t.numel() * t.element_size() for t in hin)
    d2h = hout.numel() * hout.element_size()
    wl.close()

    # roofline of the dominant kernel (the only libg16 kernel per step for fp16 GEMM workloads)
    if wl.bound == "tensor":
        peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
        achieved = wl.flops() / (ms_step * 1e-3) / 1e12
        unit = "TFLOP/s"
    else:
        peak = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
        achieved = wl.alg_bytes() / (ms_step * 1e-3) / 1e9
        unit = "GB/s"
    traffic = load_profile_traffic().get(args.workload)
    roof = {"bound": wl.bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "peak_source": f"{peak_src} ({'bf16_tflops burst' if wl.bound == 'tensor' else 'hbm_gbs copy'})",
            "basis": (f"Linear FLOPs of the rank's slice = {wl.flops():.4g} per step (rate over the whole step)"
                      if wl.unit == "texts/s" else
                      f"2*M*N*K = {wl.flops():.4g} FLOP per launch" if wl.bound == "tensor" else
                      f"2KN+xMK+4N+oMN = {wl.alg_bytes():.4g} B per launch"),
            "launches_per_step": launches / max(args.steps, 1)}

    line = {"metric": wl.metric, "value": round(value, 3), "unit": wl.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": wl.scaling, "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)", "data": "synthetic",
            "config": dict(wl.config(), parallelism=(f"replicas x{world}" if wl.scaling == "weak" else
                                                     (f"dp{world}" if wl.unit == "texts/s" else f"n-shard{world}"))),
            "e2e": {"value": round((wl.batch if wl.unit == "texts/s" else world * per_rank_units) / (e2e_ms * 1e-3), 3),
                    "unit": wl.unit,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 4), "api": "gtx16_fp16 public API, pinned host buffers",
                    "schedule": e2e_mode},
            "roofline": roof, "gpu_launches": int(launches), "clocks": sampler.summary(), "impl": "ours",
            "timing": "CUDA graph of the K steps, replayed once" if graph is not None else "eager launches"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl)
    del wl
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and args.extra:
        line["sub"] = sub_metrics(args, dev, g16, peaks)
    if args.blocks:
        line["collective"] = {name: BLOCKS[name](args, rank, world, dev, peaks)
                              for name in args.blocks.split(",") if name}
    return line


class E2EPipeline:
    """End-to-end steps through the public API with every step's inputs copied host -> device and
    its result copied device -> host inside the timed region, double-buffered over three streams:
    the inputs of step i+1 upload while step i computes and step i-1's result downloads (PCIe is
    full duplex). Each step reads its own device copy of the inputs (two slots, reused once the
    compute two steps back has finished with them)."""

    def __init__(self, wl, g16, hin, hout, dev):
        self.wl, self.g16, self.hin, self.hout, self.dev = wl, g16, hin, hout, dev
        self.slots = [[torch.empty_like(t, device=dev) for t in hin] for _ in range(2)]
        self.s_in, self.s_comp, self.s_out = (torch.cuda.Stream(dev) for _ in range(3))
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.freed = [torch.cuda.Event() for _ in range(2)]

    def run(self, steps):
        """Device milliseconds for `steps` steps (events on the caller's stream around all three)."""
        main = torch.cuda.current_stream(self.dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(main)
        for st in (self.s_in, self.s_comp, self.s_out):
            st.wait_stream(main)
        for i in range(steps):
            k = i % 2
            self.s_in.wait_event(self.freed[k])
            with torch.cuda.stream(self.s_in):
                for dst, src in zip(self.slots[k], self.hin):
                    dst.copy_(src, non_blocking=True)
                self.ready[k].record(self.s_in)
            self.s_comp.wait_event(self.ready[k])
            with torch.cuda.stream(self.s_comp):
                y = self.wl.e2e_compute(self.g16, self.slots[k])
                self.freed[k].record(self.s_comp)
            y.record_stream(self.s_out)
            self.s_out.wait_stream(self.s_comp)
            with torch.cuda.stream(self.s_out):
                self.hout.copy_(y, non_blocking=True)
        for st in (self.s_in, self.s_comp, self.s_out):
            main.wait_stream(st)
        end.record(main)
        end.synchronize()
        return start.elapsed_time(end)


def sub_metrics(args, dev, g16, peaks):
    """Short measurements of the other BASELINE configs (same timing rules), for context."""
    out = {}
    for name in [n for n in args.extra.split(",") if n and n != args.workload]:
        wl = WORKLOADS[name](dev, 1, 0)
        for _ in range(5):
            wl.step(g16)
        torch.cuda.synchronize(dev)
        steps = 50 if name != "gemm16384" else 10
        graph, stream = None, torch.cuda.current_stream(dev)
        if args.graph and wl.graphable:
            stream = torch.cuda.Stream(dev)
            graph, _ = capture_steps(wl, g16, steps, stream)
            with torch.cuda.stream(stream):
                graph.replay()
            torch.cuda.synchronize(dev)
        cos = wl.check_cosine() if isinstance(wl, Bert) else None
        ms = timed_loop(wl, g16, steps, stream, graph) / steps
        if wl.unit == "texts/s":
            v = wl.batch / (ms * 1e-3)
        elif wl.unit == "TFLOPS":
            v = wl.flops() / (ms * 1e-3) / 1e12
        else:
            v = wl.alg_bytes() / (ms * 1e-3) / 1e9
        if wl.bound == "tensor":
            frac = wl.flops() / (ms * 1e-3) / 1e12 / peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
        else:
            frac = wl.alg_bytes() / (ms * 1e-3) / 1e9 / peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
        out[name] = {"value": round(v, 2), "unit": wl.unit, "us_per_step": round(ms * 1e3, 2),
                     "bound": wl.bound, "frac_of_measured_peak": round(frac, 4),
                     "basis": ("2*M*N*K FLOP at the bf16 burst peak" if wl.bound == "tensor" else
                               "algorithmic bytes at the measured copy bandwidth"),
                     "config": wl.config()}
        if cos is not None:
            out[name]["cosine_min_vs_fp32"] = cos
        del wl
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------------------------
# Collective blocks: every rank takes part, at every N (the strong-scaling evidence of the line)
# ---------------------------------------------------------------------------------------------
def timed_eager(fn, steps, world, dev):
    """Max-over-ranks device milliseconds per step of `fn` (CUDA events, barrier + sync around)."""
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    barrier(world)
    return reduce_max(start.elapsed_time(end), world, dev) / steps


def block_gemm16384(args, rank, world, dev, peaks):
    """16384^3 fp16 GEMM, w_t N-sharded over all ranks with the all-gather fused into the GEMM
    epilogue (gtx16_fp16.dist.ShardedMatmul); TFLOPS of the whole job, max-over-ranks time.
    Parity: 256 seeded rows of the full gathered output on every rank against fp64 (norm-wise and
    component-wise, worst rank). Efficiency: against the same run's 1-GPU 16384^3 (the full
    unsharded GEMM through gtx16_fp16.matmul on each rank's GPU; the fastest GPU is the baseline)."""
    import gtx16_fp16 as g16
    from gtx16_fp16 import _native
    wl = ShardedGemm(dev, world, rank, sample_rows=256, keep_full_b=world > 1)
    steps = args.block_steps
    for _ in range(3):
        wl.step(g16)
    l0 = _native.launch_count()
    ms = timed_eager(lambda: wl.step(g16), steps, world, dev)
    launches = (_native.launch_count() - l0) / steps
    flops = 2.0 * wl.M * wl.N * wl.K
    tflops = flops / (ms * 1e-3) / 1e12
    out = wl.step(g16)
    torch.cuda.synchronize(dev)
    norm, comp, finite = wl.check_rows(out)
    norm, comp = reduce_max(norm, world, dev), reduce_max(comp, world, dev)
    finite = reduce_max(0.0 if finite else 1.0, world, dev) == 0.0
    exchange = wl.exchange()
    wl.close()
    if world > 1:
        a, b = wl.A, wl.B_full
        for _ in range(3):
            g16.matmul(a, b)
        torch.cuda.synchronize(dev)
        stream = torch.cuda.current_stream(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            g16.matmul(a, b)
        e.record(stream)
        e.synchronize()
        one_ms = -reduce_max(-s.elapsed_time(e) / steps, world, dev)  # fastest GPU
        barrier(world)
    else:
        one_ms = ms
    one_tflops = flops / (one_ms * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    res = {"value": round(tflops, 2), "unit": "TFLOPS", "ms_per_step": round(ms, 4), "steps": steps,
           "n_gpus": world, "scaling": "strong", "exchange": exchange,
           "one_gpu_tflops": round(one_tflops, 2),
           "efficiency_vs_1gpu": round(tflops / (world * one_tflops), 4),
           "per_gpu_frac_of_measured_peak": round(tflops / world / peak, 4),
           "parity": {"rows": int(wl.rows.numel()), "norm_rel_err_vs_fp64": norm,
                      "componentwise_rel_err_vs_fp64": comp, "finite": finite,
                      "tolerance": 1e-3, "pass": bool(finite and norm <= 1e-3 and comp <= 1e-3),
                      "checked_on": "every rank (worst rank reported)"},
           "gpu_launches_per_step": launches,
           "config": dict(wl.config(), parallelism=f"n-shard{world}",
                          timing="eager steps, CUDA events, max over ranks",
                          one_gpu_baseline="gtx16_fp16.matmul 16384^3 on each GPU of this run, fastest GPU")}
    del wl
    torch.cuda.empty_cache()
    return res


def block_bert(args, rank, world, dev, peaks):
    """BERT-base (config 5), data parallel over the 256 sequences; texts/s = 256 / max-rank step
    time. Cosine of the CLS embeddings against the unpatched fp32 model on every rank's slice, so
    all 256 sequences are checked; the worst one is reported."""
    import gtx16_fp16 as g16
    from gtx16_fp16 import _native
    wl = Bert(dev, world, rank)
    cos = -reduce_max(-wl.check_cosine(), world, dev)
    for _ in range(3):
        wl.step(g16)
    l0 = _native.launch_count()
    ms = timed_eager(lambda: wl.step(g16), args.bert_steps, world, dev)
    launches = (_native.launch_count() - l0) / args.bert_steps
    linear_tflops = world * wl.flops() / (ms * 1e-3) / 1e12  # approximate: slices differ by <= 1 sequence
    res = {"value": round(wl.batch / (ms * 1e-3), 2), "unit": "texts/s", "ms_per_step": round(ms, 3),
           "steps": args.bert_steps, "n_gpus": world, "scaling": "strong",
           "cosine_min_vs_fp32": round(cos, 7), "cosine_target": 0.9999, "sequences_checked": wl.batch,
           "linear_tflops": round(linear_tflops, 2),
           "linear_frac_of_measured_peak": round(linear_tflops / world /
                                                 peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]), 4),
           "gpu_launches_per_step": launches,
           "config": dict(wl.config(), parallelism=f"dp{world}", cosine_min_vs_fp32=round(cos, 7),
                          timing="eager steps, CUDA events, max over ranks")}
    del wl
    torch.cuda.empty_cache()
    return res


BLOCKS = {"gemm16384": block_gemm16384, "bert": block_bert}


def cpu_baseline(wl):
    from oracle import cpu_path
    cores = cpu_path.use_all_cores()
    fn, units, sample = wl.cpu_sample()
    fn()
    t0 = time.perf_counter()
    n = 0
    while True:
        fn()
        n += 1
        if time.perf_counter() - t0 > 3.0 or n >= 20:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(cpu_value(wl, units, dt), 5), "unit": wl.unit, "cores": cores, "kind": "port",
            "sample": sample, "seconds_per_sample": round(dt, 4)}


def cpu_value(wl, units, dt):
    """Convert a CPU sample (units of work in dt seconds) to the workload's metric unit."""
    if wl.unit == "TFLOPS":
        return units / dt / 1e12
    if wl.unit == "texts/s":
        return units / dt
    return wl.alg_bytes() * (units / wl.flops()) / dt / 1e9  # GB/s of the same algorithmic bytes


def run_reference(args, rank, world, dev):
    """The reference's CPU implementation of the path (torch fp32 fallback) on the host cores."""
    if rank != 0:
        return None
    from oracle import cpu_path
    wl = (Bert(dev, 1, 0, reference=True) if args.workload.startswith("bert")
          else WORKLOADS[args.workload](dev, 1, 0))
    cores = cpu_path.use_all_cores()
    fn, units, sample = wl.cpu_sample()
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    v = cpu_value(wl, units, dt)
    return {"metric": wl.metric, "value": round(v, 5), "unit": wl.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": wl.scaling,
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "config": dict(wl.config(), parallelism="cpu"),
            "impl": "reference",
            "cpu_baseline": {"value": round(v, 5), "unit": wl.unit, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 5), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------------------------
def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_max(v, world, dev):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="gemm4096", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--extra", default=("gemm1024,skinny1,skinny4,skinny,skinny1x3072,skinny4x3072,splitk,splitk64,"
                                        "rescale,rescale_fused,linear768,linear768_fused,decode16,decode16_eager,bert_fused,bert16"),
                    help="comma list of other workloads measured briefly into 'sub' (N=1 only); '' to skip")
    ap.add_argument("--blocks", default="gemm16384,bert",
                    help="comma list of collective blocks every rank runs at every N ('collective'); '' to skip")
    ap.add_argument("--block-steps", type=int, default=10, help="timed steps of the gemm16384 block")
    ap.add_argument("--bert-steps", type=int, default=5, help="timed steps of the bert block")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--graph", type=int, default=1, help="1: time a CUDA graph of the K steps (default); 0: eager")
    ap.add_argument("--exchange", default="auto", choices=["auto", "peer"],
                    help="gemm16384 on N > 1 GPUs: NVLink multicast where supported (auto) or peer stores")
    args = ap.parse_args()
    ShardedGemm.multicast = None if args.exchange == "auto" else False
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and rank != 0:
        return  # the reference arm is the host CPU path: rank 0 alone runs and prints it
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist
        # NCCL's own collectives are small (barrier all-reduces, result gathers), so NCCL runs without
        # NVLS; the sharded GEMM's exchange binds its output to a multicast object of its own
        # (torch symmetric memory) where the GPUs support it.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    try:
        if args.impl == "reference":
            line = run_reference(args, rank, world, dev)
        else:
            line = run_ours(args, rank, world, dev)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
