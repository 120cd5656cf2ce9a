"""The C ABI library loads and exports exactly what include/g16.h declares (no GPU needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "g16.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(g16_[a-z0-9_]+)\s*\(", src)))


def header_enum(name):
    src = open(HEADER).read()
    body = re.search(r"enum\s+%s\s*\{(.*?)\}" % name, src, flags=re.S).group(1)
    return {k: int(v) for k, v in re.findall(r"(G16_[A-Z0-9_]+)\s*=\s*(\d+)", body)}


def test_library_exports_every_declared_symbol():
    from gtx16_fp16 import _native
    L = _native.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), f"libg16.so does not export {n}"
    # and the ctypes table covers exactly the declared set
    assert sorted(_native.SIGNATURES) == names


def test_status_codes_match_header():
    from gtx16_fp16 import _native
    st = header_enum("g16_status")
    assert st["G16_OK"] == _native.OK
    assert st["G16_ERR_ARG"] == _native.ERR_ARG
    assert st["G16_ERR_UNSUPPORTED"] == _native.ERR_UNSUPPORTED
    assert st["G16_ERR_ALIGN"] == _native.ERR_ALIGN
    assert st["G16_ERR_WORKSPACE"] == _native.ERR_WORKSPACE
    assert st["G16_ERR_CUDA"] == _native.ERR_CUDA
    assert st["G16_ERR_DEVICE"] == _native.ERR_DEVICE
    assert st["G16_ERR_TIMEOUT"] == _native.ERR_TIMEOUT
    assert st["G16_ERR_TOO_LARGE"] == _native.ERR_TOO_LARGE
    dt = header_enum("g16_dtype")
    assert dt == {"G16_F32": _native.G16_F32, "G16_F16": _native.G16_F16}


def test_host_only_entry_points():
    from gtx16_fp16 import _native
    L = _native.lib()
    assert L.g16_version() == 100
    for code in range(0, 9):
        assert len(L.g16_strerror(code)) > 0
    assert L.g16_strerror(99) == b"unknown g16 status"
    assert L.g16_launch_count() == 0


def test_argument_checks_return_codes_without_launching():
    # rejected before any CUDA call: bad dtype code, K % 8 != 0, negative sizes, misalignment
    from gtx16_fp16 import _native
    L = _native.lib()
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.addressof(buf)
    p16 = (p + 15) // 16 * 16
    assert L.g16_mm_t(p16, 7, p16, None, p16, 0, 4, 8, 8, None, 0, None) == _native.ERR_ARG
    assert L.g16_mm_t(p16, 0, p16, None, p16, 0, 4, 12, 8, None, 0, None) == _native.ERR_UNSUPPORTED
    assert L.g16_mm_t(p16, 0, p16, None, p16, 0, -1, 8, 8, None, 0, None) == _native.ERR_ARG
    assert L.g16_mm_t(p16 + 4, 0, p16, None, p16, 0, 4, 8, 8, None, 0, None) == _native.ERR_ALIGN
    assert L.g16_mm_t(p16, 0, p16, None, p16, 0, 0, 8, 8, None, 0, None) == _native.OK  # M == 0: no-op
    assert L.g16_skinny(p16, 0, p16, None, p16, 0, 9, 8, 8, None) == _native.ERR_ARG
    assert L.g16_rowscale(p16, 0, p16, p16, 2, 12, 1024.0, None) == _native.ERR_UNSUPPORTED
    dsts = (ctypes.c_void_p * 1)(p16)
    assert L.g16_gemm_scatter(p16, p16, dsts, 0, 1, None, None, 16, 8, 8, 8, 0, 0, None) == _native.ERR_ARG
    assert L.g16_gemm_scatter(p16, p16, dsts, 1, 1, None, None, 16, 12, 8, 8, 0, 0, None) == _native.ERR_UNSUPPORTED
    assert L.g16_gemm_scatter(p16, p16, dsts, 1, 1, None, None, 16, 8, 8, 8, 8, 0, None) == _native.ERR_ARG
    assert L.g16_gemm_scatter(p16, p16, dsts, 1, 1, None, None, 16, 8, 8, 8, 0, 5, None) == _native.ERR_ARG
    assert L.g16_ipc_alloc(0, None) == _native.ERR_ARG
    assert L.g16_ipc_open(None, None) == _native.ERR_ARG
    assert L.g16_selftest_wait_timeout(0, None) == _native.ERR_ARG
    assert L.g16_selftest_wait_timeout(1000001, None) == _native.ERR_ARG
    assert L.g16_launch_count() == 0


def test_oracle_libraries_present_for_gpu_box():
    # built by __graft_entry__.build(); the GPU box uses these prebuilt files
    assert os.path.exists(os.path.join(ROOT, "oracle", "_build", "libg16_oracle.so"))
