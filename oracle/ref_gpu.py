"""TEST INFRASTRUCTURE ONLY: ctypes binding of oracle/_ref/libg16ref_gpu.so, the reference's own
CUDA kernels (src/gtx16_fp16/kernels.py:19-251) compiled for sm_100a by oracle/build_ref.py, with
launchers that restate the reference's host dispatch (src/gtx16_fp16/ops.py:45-108).

Used by the GPU parity tests to run the reference on the same B200 and the same inputs.
"""
from __future__ import annotations

import ctypes
import os

import torch

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libg16ref_gpu.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def _load():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB)
        P, I, F, Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
        L.g16ref_mm_t.argtypes = [P, I, P, P, P, I, I, I, I, I, P, P]
        L.g16ref_mm_t_scratch_bytes.argtypes, L.g16ref_mm_t_scratch_bytes.restype = [I, I, I], Z
        L.g16ref_hgemm.argtypes = [P, P, P, I, P, P, I, I, I, P]
        L.g16ref_rowscale.argtypes = [P, I, P, P, I, I, F, P]
        L.g16ref_skinny.argtypes = [P, I, P, P, P, I, I, I, I, P]
        L.g16ref_hgemm_splitk.argtypes = [P, P, P, P, I, I, I, I, P]
        for f in ("g16ref_mm_t", "g16ref_hgemm", "g16ref_rowscale", "g16ref_skinny", "g16ref_hgemm_splitk"):
            getattr(L, f).restype = I
        _lib = L
    return _lib


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _check(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"{what}: CUDA error {rc}")


def mm_t(x: torch.Tensor, w_t: torch.Tensor, bias: torch.Tensor | None = None, out_dtype=torch.float32) -> torch.Tensor:
    """The reference's mm_t on this GPU (its kernels, its dispatch)."""
    L = _load()
    M, K = x.shape
    N = w_t.shape[1]
    sms = torch.cuda.get_device_properties(x.device).multi_processor_count
    out = torch.empty(M, N, device=x.device, dtype=out_dtype)
    scratch = torch.empty(int(L.g16ref_mm_t_scratch_bytes(M, K, N)), dtype=torch.uint8, device=x.device)
    b = None if bias is None else bias.float().contiguous()
    _check(L.g16ref_mm_t(x.data_ptr(), int(x.dtype == torch.float16), w_t.data_ptr(), _p(b), out.data_ptr(),
                         int(out_dtype == torch.float16), M, K, N, sms, scratch.data_ptr(), _stream(x)), "g16ref_mm_t")
    return out


def hgemm(a16, b16, bias=None, rscale=None, out_dtype=torch.float32) -> torch.Tensor:
    """hgemm_f32out / hgemm_f16out alone (deterministic: no atomics)."""
    L = _load()
    M, K = a16.shape
    N = b16.shape[1]
    out = torch.empty(M, N, device=a16.device, dtype=out_dtype)
    _check(L.g16ref_hgemm(a16.data_ptr(), b16.data_ptr(), out.data_ptr(), int(out_dtype == torch.float16), _p(bias),
                          _p(rscale), M, N, K, _stream(a16)), "g16ref_hgemm")
    return out


def rowscale(x, thresh: float = 1024.0):
    """rowscale_f32 / rowscale_f16 alone: (fp16 x/S, S)."""
    L = _load()
    M, K = x.shape
    y = torch.empty(M, K, device=x.device, dtype=torch.float16)
    S = torch.empty(M, device=x.device, dtype=torch.float32)
    _check(L.g16ref_rowscale(x.data_ptr(), int(x.dtype == torch.float16), y.data_ptr(), S.data_ptr(), M, K,
                             float(thresh), _stream(x)), "g16ref_rowscale")
    return y, S
