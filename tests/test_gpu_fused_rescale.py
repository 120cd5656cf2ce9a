"""The row rescale fused into the GEMM's A operand (north-star subsystem 3), g16_mm_t_fused_rescale.

A read-only row-amax pass computes the scale S of each row (the rule of the reference's rowscale,
kernels.py:227-250) and 1/S; the CTA-pair GEMM's converter warps turn each staged fp32 tile into the
fp16 operand x * (1/S) in shared memory, so the fp16 copy of x never reaches global memory. The
operand bits are rowscale's, so the result must equal the two-pass form (g16_rowscale, then
g16_gemm with the same tiling; also what mm_t runs) bit for bit, with rows that are rescaled
(|max| > 1024, up to the reference's 179,940 spike) and rows that are not, and match fp64 within
the GEMM tolerance."""
import pytest
import torch

import gtx16_fp16 as g
from gtx16_fp16 import _native

from _tol import assert_close_fp64

pytestmark = pytest.mark.gpu


def _two_pass(x, w, bias, out_dtype, act=_native.ACT_NONE):
    """rowscale -> fp16 copy + S, then the single-pass GEMM (same CTA-pair kernel and tiling)."""
    L = _native.lib()
    M, K = x.shape
    N = w.shape[1]
    st = _native.stream_handle(x.device.index or 0)
    x16 = torch.empty(M, K, dtype=torch.float16, device=x.device)
    S = torch.empty(M, dtype=torch.float32, device=x.device)
    _native.check(L.g16_rowscale(x.data_ptr(), _native.G16_F32, x16.data_ptr(), S.data_ptr(), M, K, 1024.0, st),
                  "g16_rowscale")
    out = torch.empty(M, N, dtype=out_dtype, device=x.device)
    assert act == _native.ACT_NONE
    _native.check(L.g16_gemm(x16.data_ptr(), w.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype),
                             None if bias is None else bias.data_ptr(), S.data_ptr(), M, K, N, 1, None, 0, st),
                  "g16_gemm")
    return out


def _inputs(M, K, N, seed, spikes):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=gen)
    if spikes:
        rows = torch.randperm(M, device="cuda", generator=gen)[: max(1, M // 50)]
        f = torch.exp(torch.empty(len(rows), device="cuda").uniform_(4.6, 5.3, generator=gen))
        x[rows] *= f[:, None]          # |max| ~ 800 .. 1000 x 4 sigma: many rows above 1024
        x[rows[0], 7] = 179940.0       # the reference's spike: beyond fp16 without the rescale
        x[rows[-1], 100] = -120000.0
    w = (torch.randn(K, N, device="cuda", generator=gen) * 0.02).half()
    b = torch.randn(N, device="cuda", generator=gen) * 0.1
    return x, w, b


def _fused(x, w, bias, out_dtype, act=_native.ACT_NONE):
    """g16_mm_t_fused_rescale through the C ABI."""
    L = _native.lib()
    M, K = x.shape
    N = w.shape[1]
    ws = torch.empty(max(int(L.g16_mm_t_fused_rescale_workspace_bytes(M)), 256), dtype=torch.uint8, device=x.device)
    out = torch.empty(M, N, dtype=out_dtype, device=x.device)
    _native.check(L.g16_mm_t_fused_rescale(x.data_ptr(), w.data_ptr(), None if bias is None else bias.data_ptr(),
                                           out.data_ptr(), _native.dtype_code(out_dtype), M, K, N, act,
                                           ws.data_ptr(), ws.numel(), _native.stream_handle(x.device.index or 0)),
                  "g16_mm_t_fused_rescale")
    return out


def _uses_fused_path(M, K, N):
    """g16_gemm's automatic plan is a single pass on the persistent kernels (the CTA pairs)."""
    import ctypes
    info = (ctypes.c_int * 3)()
    _native.check(_native.lib().g16_gemm_plan(M, K, N, info), "g16_gemm_plan")
    return M > 64 and info[0] == 0 and info[2] <= 1


@pytest.mark.parametrize("M,K,N", [(2048, 768, 3072), (1000, 1032, 4104), (4096, 256, 2304), (8192, 3072, 768)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("spikes", [False, True])
def test_fused_rescale_equals_two_pass(cuda_ok, M, K, N, out_dtype, spikes):
    assert _uses_fused_path(M, K, N)  # the shapes where mm_t's GEMM is the CTA-pair kernel
    x, w, b = _inputs(M, K, N, M + K + N, spikes)
    got = _fused(x, w, b, out_dtype)
    want = _two_pass(x, w, b, out_dtype)
    default = g.mm_t(x, w, b, out_dtype)  # mm_t's own path: the two-pass form
    torch.cuda.synchronize()
    assert torch.isfinite(got).all()
    assert torch.equal(got, want)
    assert torch.equal(default, want)
    sample = torch.randperm(M, generator=torch.Generator().manual_seed(0))[:256].cuda()
    assert_close_fp64(got[sample], x[sample], w, b, out_dtype, f"fused rescale {M}x{K}x{N}")


def test_fused_rescale_with_gelu_epilogue(cuda_ok):
    x, w, b = _inputs(2048, 768, 3072, 5, True)
    got = _fused(x, w, b, torch.float32, act=_native.ACT_GELU)
    want = torch.nn.functional.gelu(_two_pass(x, w, b, torch.float32))
    torch.cuda.synchronize()
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)


def test_fused_rescale_is_deterministic_and_reads_no_stale_scales(cuda_ok):
    """Two different inputs in a row: each result equals its own two-pass form (the second call's
    scales, not the first's), and repeating a call gives the same bits."""
    for seed in (1, 2):
        x, w, b = _inputs(2048, 768, 3072, seed, seed == 1)
        a1 = _fused(x, w, b, torch.float32)
        a2 = _fused(x, w, b, torch.float32)
        want = _two_pass(x, w, b, torch.float32)
        torch.cuda.synchronize()
        assert torch.equal(a1, a2) and torch.equal(a1, want)
