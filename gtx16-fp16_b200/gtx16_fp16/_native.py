"""ctypes binding of libg16.so (the C ABI declared in include/g16.h).

Replaces the reference's kernel-launch plumbing (src/gtx16_fp16/kernels.py:253-355: NVRTC compile
cache, ctypes cuLaunchKernel, PreparedLaunch). The library is built in-tree for sm_100a; if it is
missing, every CUDA entry point raises instead of silently falling back to torch.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libg16.so")

G16_F32 = 0
G16_F16 = 1

OK = 0
ERR_ARG, ERR_UNSUPPORTED, ERR_ALIGN, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE, ERR_TIMEOUT, ERR_TOO_LARGE = range(1, 9)

_lib = None
_lock = threading.Lock()

# Every exported symbol of include/g16.h with its ctypes signature (restype, argtypes).
_P, _I, _F, _Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
IPC_HANDLE_BYTES = 64       # G16_IPC_HANDLE_BYTES
SCATTER_MAX_DST = 8         # G16_SCATTER_MAX_DST
SCATTER_DEFAULT, SCATTER_STORES, SCATTER_TMA, SCATTER_PAIRS, SCATTER_MULTIMEM = 0, 1, 2, 3, 4  # G16_SCATTER_*
ACT_NONE, ACT_GELU = 0, 1   # G16_ACT_*: activation applied by the GEMM epilogue (g16_mm_t_act)
SIGNATURES = {
    "g16_mm_t": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "g16_mm_t_workspace_bytes": (_Z, [_I, _I, _I, _I]),
    "g16_mm_t_act": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P, _Z, _P]),
    "g16_mm_t_fused_rescale": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _Z, _P]),
    "g16_mm_t_fused_rescale_workspace_bytes": (_Z, [_I]),
    "g16_skinny": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P]),
    "g16_rowscale": (_I, [_P, _I, _P, _P, _I, _I, _F, _P]),
    "g16_gemm": (_I, [_P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "g16_gemm_workspace_bytes": (_Z, [_I, _I, _I, _I]),
    "g16_gemm_auto_ksplit": (_I, [_I, _I, _I]),
    "g16_gemm_static_scratch": (_I, [_P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P]),
    "g16_gemm_scatter": (_I, [_P, _P, ctypes.POINTER(_P), _I, _I, _P, _P, _I, _I, _I, ctypes.c_longlong, _I, _I,
                              _P]),
    "g16_gemm_allgather_mc": (_I, [_P, _P, _P, _I, _P, _P, _I, _I, _I, ctypes.c_longlong, _I, _P, _P,
                                   ctypes.c_uint32, _I, _P]),
    "g16_gemm_allgather_signals": (_I, [_I, _I, _I]),
    "g16_ipc_alloc": (_I, [_Z, ctypes.POINTER(_P)]),
    "g16_ipc_free": (_I, [_P]),
    "g16_ipc_get_handle": (_I, [_P, _P]),
    "g16_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "g16_ipc_close": (_I, [_P]),
    "g16_gemm_plan": (_I, [_I, _I, _I, ctypes.POINTER(_I)]),
    "g16_skinny_plan": (_I, [_I, _I, _I, _I, ctypes.POINTER(_I)]),
    "g16_device_status": (_I, [ctypes.POINTER(_I), _I, _P]),
    "g16_selftest_wait_timeout": (_I, [_I, _P]),
    "g16_launch_count": (ctypes.c_uint64, []),
    "g16_strerror": (ctypes.c_char_p, [_I]),
    "g16_last_cuda_error": (_I, []),
    "g16_version": (_I, []),
}


class G16Error(RuntimeError):
    """A libg16 entry point returned a non-zero status."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {strerror(status)} (g16 status {status})")


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use). Raises ImportError when it was never built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"gtx16_fp16: native library {LIB_PATH} is not built; run "
                        "`make -C gtx16-fp16_b200/csrc` (or __graft_entry__.build())")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    f = getattr(L, name)
                    f.restype, f.argtypes = res, args
                _lib = L
    return _lib


def strerror(status: int) -> str:
    try:
        return lib().g16_strerror(status).decode()
    except ImportError:
        return f"status {status}"


def check(status: int, where: str) -> None:
    if status != OK:
        raise G16Error(status, where)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return G16_F32
    if dt == torch.float16:
        return G16_F16
    raise ValueError(f"unsupported dtype {dt}")


def stream_handle(device_index: int) -> int:
    """Raw handle of torch's current CUDA stream on the device (same accessor as kernels.py:294-296)."""
    return torch._C._cuda_getCurrentRawStream(device_index)


# ---------------------------------------------------------------------------------------------
# Workspace: one buffer per (device, stream), grown on demand. It holds split-K partial tiles and the
# fp16 copy of fp32 activations; no initial contents are needed. Calls on the same stream are
# ordered, so sharing it across calls is safe. A buffer that is outgrown is retired, not freed: a
# CUDA graph captured earlier on that stream still holds its address and writes it on replay.
# ---------------------------------------------------------------------------------------------
_ws: dict[tuple[int, int], torch.Tensor] = {}
_ws_retired: list[torch.Tensor] = []
_ws_lock = threading.Lock()


def workspace(device: torch.device, stream: int, nbytes: int) -> tuple[int, int]:
    """(pointer, size) of a workspace of at least nbytes for this device and stream."""
    if nbytes <= 0:
        return 0, 0
    key = (device.index or 0, stream)
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        with _ws_lock:
            buf = _ws.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 0 if buf is None else 2 * buf.numel())
                if buf is not None:
                    _ws_retired.append(buf)
                buf = torch.empty(size, dtype=torch.uint8, device=device)
                _ws[key] = buf
    return buf.data_ptr(), buf.numel()


def launch_count() -> int:
    """Kernels launched by libg16 in this process."""
    return int(lib().g16_launch_count())


def device_status(clear: bool = False) -> int:
    """The current device's status word (OK, or ERR_TIMEOUT after an expired device-side wait)."""
    v = ctypes.c_int(0)
    dev = torch.cuda.current_device()
    check(lib().g16_device_status(ctypes.byref(v), int(clear), stream_handle(dev)), "g16_device_status")
    return v.value
