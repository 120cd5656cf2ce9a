"""TEST INFRASTRUCTURE ONLY: the checker for the gtx16_fp16 B200 hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package. The product
library never links, imports or calls it.

Three oracles, all on the host CPU:

* ``fp64_*``: exact ground truth, an fp64 matmul of the (already fp16/fp32) inputs.
* ``ref_*``: a C restatement (g16_oracle.c) of the arithmetic of the reference's CUDA kernels in
  src/gtx16_fp16/kernels.py and of the dispatch in src/gtx16_fp16/ops.py (hybrid fp16 FMA over
  16-wide K slices folded into fp32, the skinny fp32-FMA path, the per-row power-of-two rescale).
* ``cpu_path``: the reference's own CPU code path (torch matmul fallbacks, ops.py:119 and
  linear.py:188-189), which is the timed CPU baseline.

Pinning: see tests/test_oracle.py (known answers and golden vectors from the reference's test suite
and from running the importable reference in the build container, tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libg16_oracle.so")
_lib = None

ROW_SCALE_THRESHOLD = 1024.0  # src/gtx16_fp16/ops.py:16
SKINNY_MAX_M = 8  # src/gtx16_fp16/kernels.py:253


def build() -> str:
    """Compile the C oracle with the Makefile beside this file; returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.g16o_h2f.argtypes, L.g16o_h2f.restype = [ctypes.c_uint16], F
        L.g16o_d2h.argtypes, L.g16o_d2h.restype = [ctypes.c_double], ctypes.c_uint16
        L.g16o_rowscale.argtypes = [P, I, P, P, I, I, F]
        L.g16o_hgemm_accf.argtypes = [P, P, I, I, I, I, I, P]
        L.g16o_hgemm.argtypes = [P, P, P, I, P, P, I, I, I]
        L.g16o_hgemm_splitk.argtypes = [P, P, P, P, P, I, I, I, I]
        L.g16o_skinny.argtypes = [P, I, P, P, P, I, I, I, I]
        L.g16o_skinny_config.argtypes = [I, I, I, P, P]
        L.g16o_skinny_config.restype = I
        L.g16o_mm_t.argtypes = [P, I, P, P, P, I, I, I, I, I]
        L.g16o_num_threads.restype = I
        for f in ("g16o_rowscale", "g16o_hgemm_accf", "g16o_hgemm", "g16o_hgemm_splitk", "g16o_skinny", "g16o_mm_t"):
            getattr(L, f).restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _f16bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    if a.dtype == np.uint16:
        return a
    raise TypeError(f"expected float16 array, got {a.dtype}")


def threads() -> int:
    return _load().g16o_num_threads()


# ---------------------------------------------------------------------------------------------
# Ground truth
# ---------------------------------------------------------------------------------------------
def fp64_mm(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """Exact-enough reference: x @ w (+ bias) in float64 on the given (fp16/fp32) values."""
    y = x.astype(np.float64) @ w.astype(np.float64)
    if bias is not None:
        y += bias.astype(np.float64)
    return y


def rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """Norm-wise relative error ||y - ref|| / ||ref|| (the reference's metric, tests/test_correctness.py:10-11)."""
    ref = ref.astype(np.float64)
    d = np.linalg.norm(y.astype(np.float64) - ref)
    return float(d / max(np.linalg.norm(ref), 1e-300))


# ---------------------------------------------------------------------------------------------
# Restatement of the reference kernels (src/gtx16_fp16/kernels.py)
# ---------------------------------------------------------------------------------------------
def ref_rowscale(x: np.ndarray, thresh: float = ROW_SCALE_THRESHOLD) -> tuple[np.ndarray, np.ndarray]:
    """rowscale_f32 / rowscale_f16 (kernels.py:227-250): returns (fp16 x/S, S)."""
    L = _load()
    M, K = x.shape
    is16 = x.dtype == np.float16
    xx = _f16bits(x) if is16 else np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty((M, K), dtype=np.uint16)
    S = np.empty(M, dtype=np.float32)
    L.g16o_rowscale(_ptr(xx), int(is16), _ptr(y), _ptr(S), M, K, float(thresh))
    return y.view(np.float16), S


def ref_hgemm(a16: np.ndarray, b16: np.ndarray, bias: np.ndarray | None = None, rscale: np.ndarray | None = None,
              out_dtype=np.float32) -> np.ndarray:
    """hgemm_f32out / hgemm_f16out (kernels.py:35-151): hybrid fp16-slice accumulation, fused epilogue."""
    L = _load()
    M, K = a16.shape
    N = b16.shape[1]
    A, B = _f16bits(a16), _f16bits(b16)
    out16 = out_dtype == np.float16
    out = np.empty((M, N), dtype=np.uint16 if out16 else np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rscale = None if rscale is None else np.ascontiguousarray(rscale, dtype=np.float32)
    L.g16o_hgemm(_ptr(A), _ptr(B), _ptr(out), int(out16), _ptr(bias), _ptr(rscale), M, N, K)
    return out.view(np.float16) if out16 else out


def ref_hgemm_accf(a16: np.ndarray, b16: np.ndarray, k0: int = 0, klen: int | None = None) -> np.ndarray:
    """Raw fp32 accumulator of hgemm_body over K range [k0, k0+klen) (kernels.py:77-104)."""
    L = _load()
    M, K = a16.shape
    N = b16.shape[1]
    klen = K - k0 if klen is None else klen
    out = np.empty((M, N), dtype=np.float32)
    L.g16o_hgemm_accf(_ptr(_f16bits(a16)), _ptr(_f16bits(b16)), M, N, K, k0, klen, _ptr(out))
    return out


def ref_hgemm_splitk(a16, b16, bias=None, rscale=None, kchunk: int = 128) -> np.ndarray:
    """hgemm_splitk + _prefilled (kernels.py:143-147, ops.py:54-62,92-101), chunks added in order."""
    L = _load()
    M, K = a16.shape
    N = b16.shape[1]
    out = np.empty((M, N), dtype=np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rscale = None if rscale is None else np.ascontiguousarray(rscale, dtype=np.float32)
    L.g16o_hgemm_splitk(_ptr(_f16bits(a16)), _ptr(_f16bits(b16)), _ptr(out), _ptr(bias), _ptr(rscale), M, N, K, kchunk)
    return out


def skinny_config(N: int, K: int, sms: int) -> tuple[tuple[int, int, int], int]:
    """ops.py:45-51 restated in C; returns ((nbx, ksplit, 1), kchunk) like the reference."""
    L = _load()
    nbx, ks = ctypes.c_int(), ctypes.c_int()
    kchunk = L.g16o_skinny_config(N, K, sms, ctypes.byref(nbx), ctypes.byref(ks))
    return (nbx.value, ks.value, 1), kchunk


def ref_skinny(x: np.ndarray, w16: np.ndarray, bias: np.ndarray | None = None, sms: int = 148,
               kchunk: int | None = None) -> np.ndarray:
    """skinny_f32in / skinny_f16in (kernels.py:163-219) with skinny_config's K chunks; fp32 [M,N]."""
    L = _load()
    M, K = x.shape
    N = w16.shape[1]
    if kchunk is None:
        kchunk = skinny_config(N, K, sms)[1]
    is16 = x.dtype == np.float16
    xx = _f16bits(x) if is16 else np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((M, N), dtype=np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    L.g16o_skinny(_ptr(xx), int(is16), _ptr(_f16bits(w16)), _ptr(bias), _ptr(out), M, N, K, kchunk)
    return out


def ref_mm_t(x: np.ndarray, w16: np.ndarray, bias: np.ndarray | None = None, out_dtype=np.float32,
             sms: int = 148) -> np.ndarray:
    """mm_t (ops.py:65-108) on a GPU with `sms` SMs, every kernel restated on the CPU."""
    L = _load()
    M, K = x.shape
    N = w16.shape[1]
    is16 = x.dtype == np.float16
    xx = _f16bits(x) if is16 else np.ascontiguousarray(x, dtype=np.float32)
    out16 = out_dtype == np.float16
    out = np.empty((M, N), dtype=np.uint16 if out16 else np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    L.g16o_mm_t(_ptr(xx), int(is16), _ptr(_f16bits(w16)), _ptr(bias), _ptr(out), int(out16), M, K, N, sms)
    return out.view(np.float16) if out16 else out
