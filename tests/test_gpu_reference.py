"""Parity against the reference itself on the B200.

oracle/_ref/libg16ref_gpu.so holds the reference's own CUDA kernels (src/gtx16_fp16/kernels.py:19-251,
compiled by oracle/build_ref.py with its NVRTC options) and launchers restating its dispatch
(ops.py:45-108). These tests:
  1. pin the CPU restatement (oracle/g16_oracle.c) bit-for-bit against those kernels where the
     reference is deterministic (hgemm_f32out / hgemm_f16out, rowscale), and to fp32 atomics order
     where it is not (skinny, split-K);
  2. run every BASELINE configuration through both the reference and this package on the same
     seeded inputs and check both against fp64, and against each other.
"""
import numpy as np
import pytest
import torch

import gtx16_fp16 as g
import oracle
from oracle import ref_gpu

from _tol import assert_close_fp64, rel_err

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_gpu.available(), reason="oracle/_ref not built (oracle/build_ref.py)")]


def f16np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("M,K,N", [(128, 128, 128), (200, 1032, 136), (129, 136, 8), (64, 1024, 96)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_oracle_hgemm_bitexact_vs_reference_kernel(cuda_ok, M, K, N, out_dtype):
    torch.manual_seed(M + K + N)
    a = (torch.randn(M, K, device="cuda") * 0.5).half()
    b = (torch.randn(K, N, device="cuda") * 0.5).half()
    bias = torch.randn(N, device="cuda")
    rs = torch.where(torch.rand(M, device="cuda") < 0.2, 4.0, 1.0).float()
    y_ref = ref_gpu.hgemm(a, b, bias, rs, out_dtype)
    y_or = oracle.ref_hgemm(f16np(a), f16np(b), f16np(bias), f16np(rs),
                            np.float16 if out_dtype == torch.float16 else np.float32)
    assert np.array_equal(f16np(y_ref).view(np.uint16 if out_dtype == torch.float16 else np.uint32),
                          np.ascontiguousarray(y_or).view(np.uint16 if out_dtype == torch.float16 else np.uint32))


@pytest.mark.parametrize("xdt", [torch.float32, torch.float16])
def test_oracle_rowscale_bitexact_vs_reference_kernel(cuda_ok, xdt):
    torch.manual_seed(2)
    x = torch.randn(96, 520, device="cuda") * 3
    x[5, 7] = 179940.0 if xdt == torch.float32 else 60000.0
    x[6, 1] = -1500.0
    x[8, 0] = 2048.5
    x = x.to(xdt)
    y_ref, s_ref = ref_gpu.rowscale(x)
    y_or, s_or = oracle.ref_rowscale(f16np(x))
    assert np.array_equal(f16np(s_ref), s_or)
    assert np.array_equal(f16np(y_ref).view(np.uint16), y_or.view(np.uint16))
    # this package's rowscale gives the same bits
    from gtx16_fp16 import _native
    y = torch.empty_like(y_ref)
    s = torch.empty_like(s_ref)
    assert _native.lib().g16_rowscale(x.data_ptr(), _native.dtype_code(xdt), y.data_ptr(), s.data_ptr(), 96, 520,
                                      1024.0, _native.stream_handle(0)) == 0
    assert torch.equal(y, y_ref) and torch.equal(s, s_ref)


@pytest.mark.parametrize("M,K,N", [(1, 1024, 3072), (4, 4096, 512), (8, 520, 136)])
def test_oracle_skinny_vs_reference_kernel(cuda_ok, M, K, N):
    torch.manual_seed(M * K)
    x = torch.randn(M, K, device="cuda")
    w = (torch.randn(K, N, device="cuda") * 0.02).half()
    bias = torch.randn(N, device="cuda") * 0.01
    y_ref = ref_gpu.mm_t(x, w, bias, torch.float32)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    y_or = oracle.ref_skinny(f16np(x), f16np(w), f16np(bias), sms=sms)
    # same per-chunk arithmetic; only the order of the fp32 atomics across K chunks differs
    np.testing.assert_allclose(f16np(y_ref), y_or, rtol=1e-6, atol=1e-6)


def _cfg2(M, K, N, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=gen)
    w = (torch.randn(K, N, device="cuda", generator=gen) * 0.02).half()
    b = torch.randn(N, device="cuda", generator=gen) * 0.01
    return x, w, b


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (4, 4096, 4096), (8, 4096, 4096), (1, 1024, 3072), (4, 1024, 3072)])
def test_config2_skinny_vs_reference(cuda_ok, M, K, N):
    x, w, b = _cfg2(M, K, N)
    r64 = x.double() @ w.double() + b.double()
    y = g.mm_t(x, w, b, torch.float32)
    y_ref = ref_gpu.mm_t(x, w, b, torch.float32)
    assert_close_fp64(y, x, w, b, torch.float32, "ours", ref=r64)
    assert_close_fp64(y_ref, x, w, b, torch.float32, "reference", ref=r64)
    assert rel_err(y, y_ref.double()) < 2e-5


def _cfg3(M, K, N, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    return a, b


@pytest.mark.parametrize("M,K,N", [(4096, 4096, 4096), (64, 1024, 1024), (128, 16384, 1024), (1024, 1024, 1024)])
def test_config3_gemm_vs_reference(cuda_ok, M, K, N):
    a, b = _cfg3(M, K, N)
    r64 = a.double() @ b.double()
    y = g.matmul(a, b)
    y_ref = ref_gpu.mm_t(a, b, None, torch.float16)
    assert y.dtype == torch.float16
    e = assert_close_fp64(y, a, b, None, torch.float16, "ours", ref=r64)
    e_ref = rel_err(y_ref, r64)
    assert e_ref < 2e-3  # the reference's hybrid fp16 accumulation (README.md:36-38: ~6e-4)
    assert e <= e_ref + 1e-5  # fp32 tensor-core accumulation is at least as accurate
    assert rel_err(y, y_ref.double()) < 2e-3


def _cfg4(seed=0, spike=True):
    M, K, N = 2048, 3072, 1024
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=gen)
    rows = torch.randperm(M, device="cuda", generator=gen)[: M // 100]
    f = torch.exp(torch.empty(len(rows), device="cuda").uniform_(np.log(100.0), np.log(200.0), generator=gen))
    x[rows] *= f[:, None]
    if spike:  # the reference test's massive activation (tests/test_correctness.py:119-120) on those rows
        x[rows, 7] = 179940.0
        x[rows[0], 100] = -120000.0
    w = (torch.randn(K, N, device="cuda", generator=gen) * 0.02).half()
    b = torch.zeros(N, device="cuda")
    return x, w, b, rows


@pytest.mark.parametrize("spike", [False, True])
def test_config4_overflow_rescale_vs_reference(cuda_ok, spike):
    x, w, b, rows = _cfg4(spike=spike)
    r64 = x.double() @ w.double()
    y = g.mm_t(x, w, b, torch.float32)
    y_ref = ref_gpu.mm_t(x, w, b, torch.float32)
    assert torch.isfinite(y).all() and torch.isfinite(y_ref).all()
    assert_close_fp64(y, x, w, b, torch.float32, "ours", ref=r64)
    assert rel_err(y_ref, r64) < 2e-3
    assert rel_err(y[rows], r64[rows]) < 1e-3  # the rescaled rows themselves
