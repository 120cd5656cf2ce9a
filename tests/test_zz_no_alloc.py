"""g16_gemm_static_scratch, the GEMM entry point for callers that cannot allocate device memory at
call time (for example a server that reserved all GPU memory for its own pools at start-up). It
keeps its split-K partial tiles in a fixed 8 MiB array inside libg16 instead of a caller workspace.

Checked through the C ABI against the workspace-based g16_gemm with the same K split, on two calls
in a row (the second on new inputs, so whatever the first call left in the shared array must not
leak into the result). This file is collected last on purpose."""
import pytest
import torch

from gtx16_fp16 import _native

from _tol import assert_close_fp64, rel_err, GEMM_NORM

pytestmark = pytest.mark.gpu


def _gemm_with_workspace(a, b, bias, out_dtype, ksplit):
    L = _native.lib()
    M, K = a.shape
    N = b.shape[1]
    nws = int(L.g16_gemm_workspace_bytes(M, K, N, ksplit))
    ws = torch.empty(max(nws, 256), dtype=torch.uint8, device=a.device)
    out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    st = L.g16_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype),
                    None if bias is None else bias.data_ptr(), None, M, K, N, ksplit, ws.data_ptr(), ws.numel(),
                    _native.stream_handle(a.device.index or 0))
    assert st == _native.OK, _native.strerror(st)
    return out


def _gemm_static(a, b, bias, out_dtype, ksplit):
    L = _native.lib()
    M, K = a.shape
    N = b.shape[1]
    out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    st = L.g16_gemm_static_scratch(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype),
                                   None if bias is None else bias.data_ptr(), None, M, K, N, ksplit,
                                   _native.stream_handle(a.device.index or 0))
    assert st == _native.OK, _native.strerror(st)
    return out


@pytest.mark.parametrize("M,K,N,ksplit", [(64, 1024, 1024, 4), (128, 16384, 1024, 16), (200, 1032, 136, 3),
                                          (129, 2048, 264, 8)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_static_scratch_matches_workspace_gemm(cuda_ok, M, K, N, ksplit, out_dtype):
    for call in range(2):  # two calls in a row, new inputs each time
        gen = torch.Generator(device="cuda").manual_seed(1000 * call + M + K + N)
        a = torch.randn(M, K, device="cuda", generator=gen).half()
        b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
        bias = torch.randn(N, device="cuda", generator=gen)
        ref = _gemm_with_workspace(a, b, bias, out_dtype, ksplit)
        got = _gemm_static(a, b, bias, out_dtype, ksplit)
        torch.cuda.synchronize()
        assert rel_err(got, ref.double()) <= GEMM_NORM
        assert torch.equal(got, ref)  # same kernel, same K split: identical bits
        assert_close_fp64(got, a, b, bias, out_dtype, f"static scratch call {call}")


def test_static_scratch_automatic_split_fits(cuda_ok):
    # ksplit = 0: the usual split (37 on 148 SMs here) is lowered until 4 tiles x ksplit fit in 8 MiB
    gen = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(128, 16384, device="cuda", generator=gen).half()
    b = (torch.randn(16384, 1024, device="cuda", generator=gen) * 16384 ** -0.5).half()
    for _ in range(2):
        got = _gemm_static(a, b, None, torch.float16, 0)
        assert_close_fp64(got, a, b, None, torch.float16, "static scratch, automatic split")


def test_static_scratch_rejects_problems_that_do_not_fit(cuda_ok):
    # 1024 x 4096 output = 128 tiles; two K chunks need 128 x 2 x 128 KiB = 32 MiB > 8 MiB
    L = _native.lib()
    a = torch.empty(1024, 4096, device="cuda", dtype=torch.float16)
    b = torch.empty(4096, 4096, device="cuda", dtype=torch.float16)
    out = torch.empty(1024, 4096, device="cuda", dtype=torch.float16)
    st = L.g16_gemm_static_scratch(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.G16_F16, None, None,
                                   1024, 4096, 4096, 2, _native.stream_handle(0))
    assert st == _native.ERR_TOO_LARGE
    assert "8 MiB" in _native.strerror(st)
