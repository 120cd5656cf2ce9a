"""Host-side ops: the reference's Python surface (src/gtx16_fp16/ops.py) over the sm_100a C ABI.

Same names, arguments, defaults, dtypes and error behaviour as the reference:
  * ``mm_t(x2d, w_t, bias=None, out_dtype=torch.float32)``   (ops.py:65-108)
  * ``matmul(a, b, out_dtype=None)``                          (ops.py:111-119)
  * ``supported(x2d, w_t)``                                   (ops.py:29-35)
  * ``is_affected(device=None)``                              (ops.py:19-26)
  * ``skinny_config(N, K, sms)``                              (ops.py:45-51)
  * ``ROW_SCALE_THRESHOLD``, ``SKINNY_MAX_M``                  (ops.py:16, kernels.py:253)
One ctypes call per mm_t; the three-way dispatch (skinny / rowscale + tensor-core GEMM /
deterministic split-K) happens inside libg16 (g16_mm_t).
"""
from __future__ import annotations

import re

import torch

from . import _native
from ._native import G16Error, dtype_code, stream_handle

# Device names of the tensor-core-less Turing parts the reference targets (the same pattern as
# its ops.py:11, so is_affected answers the same on every device name).
_AFFECTED = re.compile(r"GTX 16\d\d|MX ?450|MX ?550|\bT400\b|\bT600\b|\bT1000\b|T1200", re.I)

# GEMM path only: an fp32 activation row whose largest magnitude is above this value is divided by
# a power of two before it is rounded to fp16, and the product is multiplied back in the epilogue.
ROW_SCALE_THRESHOLD = 1024.0
# Activations with at most this many rows take the HBM-streaming GEMV kernel instead of the GEMM.
SKINNY_MAX_M = 8

_ws_cache: dict[tuple[int, int, int, int, int], int] = {}


def is_affected(device: torch.device | int | None = None) -> bool:
    """Whether ``device`` (default: the current one) is one of the cc 7.5 GTX 16xx-class parts the
    reference was written for. Same answer as the reference for every device; on a B200 it is
    False, which is why ``patch`` is called with ``force=True`` there."""
    if not torch.cuda.is_available():
        return False
    idx = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    if torch.cuda.get_device_capability(idx) != (7, 5):
        return False
    return bool(_AFFECTED.search(torch.cuda.get_device_name(idx)))


def supported(x2d: torch.Tensor, w_t: torch.Tensor) -> bool:
    """Whether mm_t accepts this pair: a 2-D contiguous CUDA activation in fp16 or fp32 whose
    width equals the weight's K, and a contiguous fp16 weight [K, N] starting on a 16-byte boundary,
    with both K and N multiples of 8. The predicate is the reference's (ops.py:29-35) term for term."""
    K, N = w_t.shape
    return (x2d.is_cuda and x2d.dim() == 2 and x2d.dtype in (torch.float16, torch.float32)
            and w_t.dtype == torch.float16 and x2d.is_contiguous() and w_t.is_contiguous()
            and x2d.shape[1] == K and K % 8 == 0 and N % 8 == 0 and w_t.data_ptr() % 16 == 0)


def skinny_config(N: int, K: int, sms: int) -> tuple[tuple[int, int, int], int]:
    """The reference's launch geometry for its skinny kernel (ops.py:45-51), kept for API
    compatibility. libg16 plans its own cluster split (g16_skinny.cu) and does not use it."""
    nbx = (N + 255) // 256
    ksplit = max(1, min((4 * sms + nbx - 1) // nbx, K // 64))
    kchunk = ((K + ksplit - 1) // ksplit + 7) // 8 * 8
    ksplit = (K + kchunk - 1) // kchunk
    return (nbx, ksplit, 1), kchunk


def _aligned(t: torch.Tensor) -> torch.Tensor:
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _ws_bytes(dev_index: int, M: int, K: int, N: int, xcode: int) -> int:
    key = (dev_index, M, K, N, xcode)
    n = _ws_cache.get(key)
    if n is None:
        n = int(_native.lib().g16_mm_t_workspace_bytes(M, K, N, xcode))
        _ws_cache[key] = n
    return n


_ACTS = {None: _native.ACT_NONE, "gelu": _native.ACT_GELU}


def mm_t(x2d: torch.Tensor, w_t: torch.Tensor, bias: torch.Tensor | None = None,
         out_dtype: torch.dtype = torch.float32, *, act: str | None = None) -> torch.Tensor:
    """out[M,N] = x2d[M,K] @ w_t[K,N] + bias[N].

    x2d fp16 or fp32 (fp32 rows with |max| > 1024 are rescaled by a power of two before the fp16
    cast on the GEMM path); w_t fp16; bias fp32 or None; out fp32 or fp16, always a fresh tensor.
    Check supported() first: unlike the reference, an unsupported input raises ValueError.
    act="gelu" (keyword, not in the reference) applies the exact GELU in the epilogue:
    gelu(x2d @ w_t + bias), computed in fp32 before the output cast."""
    if act not in _ACTS:
        raise ValueError(f"act must be None or 'gelu', got {act!r}")
    if out_dtype not in (torch.float32, torch.float16):
        raise ValueError(f"out_dtype must be float32 or float16, got {out_dtype}")
    if not supported(x2d, w_t):
        raise ValueError("mm_t: inputs not supported (see gtx16_fp16.supported)")
    M, K = x2d.shape
    N = w_t.shape[1]
    dev = x2d.device
    idx = dev.index or 0
    if w_t.device != dev:
        raise ValueError("mm_t: x2d and w_t are on different devices")
    out = torch.empty(M, N, device=dev, dtype=out_dtype)
    if M == 0 or N == 0:
        return out
    x = _aligned(x2d)
    b = None
    if bias is not None:
        b = _aligned(bias.to(device=dev, dtype=torch.float32).contiguous())
    lib = _native.lib()
    xcode = dtype_code(x.dtype)
    if idx != torch.cuda.current_device():
        with torch.cuda.device(idx):
            return _mm_t_launch(lib, x, w_t, b, out, xcode, M, K, N, dev, idx, _ACTS[act])
    return _mm_t_launch(lib, x, w_t, b, out, xcode, M, K, N, dev, idx, _ACTS[act])


def _mm_t_launch(lib, x, w_t, b, out, xcode, M, K, N, dev, idx, act=_native.ACT_NONE):
    stream = stream_handle(idx)
    need = _ws_bytes(idx, M, K, N, xcode)
    ws, wsn = _native.workspace(dev, stream, need)
    bp = None if b is None else b.data_ptr()
    if act == _native.ACT_NONE:
        st = lib.g16_mm_t(x.data_ptr(), xcode, w_t.data_ptr(), bp, out.data_ptr(), dtype_code(out.dtype), M, K, N,
                          ws or None, wsn, stream)
    else:
        st = lib.g16_mm_t_act(x.data_ptr(), xcode, w_t.data_ptr(), bp, out.data_ptr(), dtype_code(out.dtype), M, K, N,
                              act, ws or None, wsn, stream)
    if st != _native.OK:
        raise G16Error(st, "g16_mm_t")
    return out


def matmul(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """a @ b for two 2-D fp16 CUDA matrices on libg16's tensor-core GEMM, fp16 result unless
    ``out_dtype`` says otherwise. Anything mm_t does not accept (CPU tensors, other dtypes or ranks,
    K or N not a multiple of 8) is computed by torch.matmul and cast, as in the reference (ops.py:119)."""
    out_dtype = out_dtype or torch.float16
    if a.dim() == 2 and b.dim() == 2 and a.dtype == b.dtype == torch.float16 and a.is_cuda:
        a_c, b_c = a.contiguous(), b.contiguous()
        if supported(a_c, b_c):
            return mm_t(a_c, b_c, None, out_dtype)
    return torch.matmul(a, b).to(out_dtype)
