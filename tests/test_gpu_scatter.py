"""g16_gemm_scatter on one GPU: the sharded GEMM's epilogue writes each tile into several [M, ldc]
buffers at column col0 (on a single GPU, two local buffers stand in for the ranks' outputs). Every
destination must hold exactly what g16_gemm with ksplit = 1 computes (same kernel, same K order),
at the right offset, and nothing outside [col0, col0 + N) may be touched."""
import ctypes

import pytest
import torch

from gtx16_fp16 import _native

from _tol import assert_close_fp64

pytestmark = pytest.mark.gpu


def _gemm_ksplit1(a, b, bias, out_dtype):
    L = _native.lib()
    M, K = a.shape
    N = b.shape[1]
    out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    st = L.g16_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype),
                    None if bias is None else bias.data_ptr(), None, M, K, N, 1, None, 0, _native.stream_handle(0))
    _native.check(st, "g16_gemm")
    return out


@pytest.mark.parametrize("M,K,N,ldc,col0", [(1024, 2048, 2048, 4096, 2048), (1000, 1024, 2056, 4104, 0),
                                             (129, 520, 264, 1024, 528), (4096, 4096, 512, 4096, 3584),
                                             (2048, 256, 5120, 6144, 1024)])  # last: split tail
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("flags", [0, 1, 2, 3])
def test_scatter_matches_gemm(cuda_ok, M, K, N, ldc, col0, out_dtype, with_bias, flags):
    gen = torch.Generator(device="cuda").manual_seed(M + N + col0)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    bias = torch.randn(N, device="cuda", generator=gen) if with_bias else None
    sentinel = -7.0
    dsts = [torch.full((M, ldc), sentinel, dtype=out_dtype, device="cuda") for _ in range(2)]
    ptrs = (ctypes.c_void_p * 2)(*[d.data_ptr() for d in dsts])
    st = _native.lib().g16_gemm_scatter(a.data_ptr(), b.data_ptr(), ptrs, 2, _native.dtype_code(out_dtype),
                                        None if bias is None else bias.data_ptr(), None, M, K, N, ldc, col0,
                                        flags, _native.stream_handle(0))
    _native.check(st, "g16_gemm_scatter")
    ref = _gemm_ksplit1(a, b, bias, out_dtype)
    torch.cuda.synchronize()
    for d in dsts:
        assert torch.equal(d[:, col0:col0 + N], ref)
        assert bool((d[:, :col0] == sentinel).all()) and bool((d[:, col0 + N:] == sentinel).all())
    assert_close_fp64(dsts[0][:, col0:col0 + N], a, b, bias, out_dtype, "scatter")


def test_scatter_rejects_bad_arguments(cuda_ok):
    L = _native.lib()
    a = torch.empty(256, 64, dtype=torch.float16, device="cuda")
    b = torch.empty(64, 64, dtype=torch.float16, device="cuda")
    d = torch.empty(256, 128, dtype=torch.float16, device="cuda")
    one = (ctypes.c_void_p * 1)(d.data_ptr())
    s = _native.stream_handle(0)
    f16 = _native.G16_F16
    assert L.g16_gemm_scatter(a.data_ptr(), b.data_ptr(), one, 0, f16, None, None, 256, 64, 64, 128, 0, 0, s) == _native.ERR_ARG
    assert L.g16_gemm_scatter(a.data_ptr(), b.data_ptr(), one, 9, f16, None, None, 256, 64, 64, 128, 0, 0, s) == _native.ERR_ARG
    assert L.g16_gemm_scatter(a.data_ptr(), b.data_ptr(), one, 1, f16, None, None, 256, 64, 64, 128, 68, 0, s) == _native.ERR_ARG
    assert L.g16_gemm_scatter(a.data_ptr(), b.data_ptr(), one, 1, f16, None, None, 256, 64, 64, 128, 4, 0, s) == \
        _native.ERR_UNSUPPORTED
    mis = (ctypes.c_void_p * 1)(d.data_ptr() + 8)
    assert L.g16_gemm_scatter(a.data_ptr(), b.data_ptr(), mis, 1, f16, None, None, 256, 64, 64, 128, 0, 0, s) == _native.ERR_ALIGN
    assert L.g16_gemm_scatter(a.data_ptr(), b.data_ptr(), one, 1, f16, None, None, 256, 64, 64, 128, 0, 5, s) == _native.ERR_ARG
    two = (ctypes.c_void_p * 2)(d.data_ptr(), d.data_ptr())  # multicast mode takes exactly one address
    assert L.g16_gemm_scatter(a.data_ptr(), b.data_ptr(), two, 2, f16, None, None, 256, 64, 64, 128, 0, 4, s) == _native.ERR_ARG
