"""GPU parity of the sm_100a kernels: the reference's test suite (tests/test_correctness.py) ported to
this package, with the fp64 product as ground truth and the tolerances of tests/_tol.py, plus bitwise
determinism, forced split-K, the C ABI called directly, and the native-path-was-used check."""
import ctypes

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import gtx16_fp16 as g
from gtx16_fp16 import _native

from _tol import GEMM_NORM, assert_close_fp64, bounds, ref64, rel_err

pytestmark = pytest.mark.gpu

SHAPES = [  # (M, K, N): tile-aligned, ragged edges, skinny (M <= 8), tiny (tests/test_correctness.py:14-18)
    (128, 128, 128), (256, 512, 384), (1000, 1032, 776), (129, 136, 8), (3, 4096, 4096),
    (1, 1024, 3072), (8, 2048, 520), (9, 64, 64), (4096, 4096, 1024), (17, 8, 4104),
    (64, 1024, 1024), (33, 4096, 768),  # medium-M path (M <= 64, swapped operands)
    (200, 1032, 136),  # split-K path
]


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("with_bias", [False, True])
def test_mm_t_matches_fp64(cuda_ok, M, K, N, out_dtype, with_bias):
    torch.manual_seed(M * 7 + K * 3 + N)
    x = (torch.randn(M, K, device="cuda") * 0.5).half()
    w = (torch.randn(K, N, device="cuda") * 0.5).half()
    b = torch.randn(N, device="cuda") if with_bias else None
    assert g.supported(x, w)
    y = g.mm_t(x, w, b, out_dtype)
    assert y.dtype == out_dtype and y.shape == (M, N)
    assert_close_fp64(y, x, w, b, out_dtype, f"{M}x{K}x{N}")
    # the reference's own bound against an fp32 reference (tests/test_correctness.py:35)
    assert rel_err(y, x.float() @ w.float() + (b if with_bias else 0)) < (2e-3 if out_dtype == torch.float16 else 1.5e-3)


@pytest.mark.parametrize("M", [1, 3, 8, 9, 64, 300])
def test_fp32_activations_match_fp64(cuda_ok, M):
    torch.manual_seed(M)
    K, N = 1024, 768
    x = torch.randn(M, K, device="cuda")
    w = (torch.randn(K, N, device="cuda") * 0.05).half()
    b = torch.randn(N, device="cuda") * 0.1
    y = g.mm_t(x, w, b, torch.float32)
    assert_close_fp64(y, x, w, b, torch.float32, f"fp32 x M={M}")


@pytest.mark.parametrize("M", [1, 2, 8, 64, 1000])
def test_bias_and_inputs_are_not_modified(cuda_ok, M):
    x = torch.randn(M, 512, device="cuda").half()
    w = torch.randn(512, 768, device="cuda").half()
    b = torch.randn(768, device="cuda")
    x0, w0, b0 = x.clone(), w.clone(), b.clone()
    for _ in range(3):
        g.mm_t(x, w, b, torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(x, x0) and torch.equal(w, w0) and torch.equal(b, b0)


@pytest.mark.parametrize("M,K,N", [(1, 1024, 768), (8, 4096, 4096), (64, 1024, 1024), (128, 16384, 1024),
                                   (1000, 1032, 776), (2048, 3072, 1024)])
@pytest.mark.parametrize("xdt", [torch.float32, torch.float16])
def test_bitwise_deterministic(cuda_ok, M, K, N, xdt):
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda").to(xdt)
    w = (torch.randn(K, N, device="cuda") * 0.02).half()
    b = torch.randn(N, device="cuda")
    outs = [g.mm_t(x, w, b, torch.float32) for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_fast_linear_is_deterministic_across_calls(cuda_ok):
    lin = nn.Linear(1024, 768).cuda()
    fl = g.FastLinear.from_linear(lin)
    x = torch.randn(1, 1024, device="cuda")
    with torch.no_grad():
        outs = [fl(x) for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])  # stronger than the reference's rel < 1e-6


def test_matmul_fallback_for_odd_shapes(cuda_ok):
    a = torch.randn(33, 13, device="cuda").half()  # K % 8 != 0 -> torch fallback
    b = torch.randn(13, 7, device="cuda").half()
    assert not g.supported(a, b)
    torch.testing.assert_close(g.matmul(a, b), (a @ b), rtol=1e-2, atol=1e-2)


def test_matmul_uses_native_kernels(cuda_ok):
    a = torch.randn(256, 512, device="cuda").half()
    b = (torch.randn(512, 384, device="cuda") * 0.05).half()
    before = _native.launch_count()
    y = g.matmul(a, b)
    torch.cuda.synchronize()
    assert _native.launch_count() > before
    assert y.dtype == torch.float16
    assert_close_fp64(y, a, b, None, torch.float16, "matmul")


def test_fast_linear_matches_nn_linear(cuda_ok):
    torch.manual_seed(0)
    lin = nn.Linear(1024, 768).cuda()
    fl = g.FastLinear.from_linear(lin)
    for shape in [(4, 50, 1024), (1, 1, 1024), (2, 1024), (7, 1024)]:
        x = torch.randn(*shape, device="cuda")
        with torch.no_grad():
            ref, y = lin(x), fl(x)
        assert y.dtype == torch.float32 and y.shape == ref.shape
        assert rel_err(y, ref) < 3e-3


def test_fast_linear_fp16_input_gives_fp16(cuda_ok):
    lin = nn.Linear(512, 256).cuda()
    fl = g.FastLinear.from_linear(lin)
    x = torch.randn(3, 20, 512, device="cuda").half()
    with torch.no_grad():
        y = fl(x)
    assert y.dtype == torch.float16 and y.shape == (3, 20, 256)
    assert rel_err(y, lin(x.float())) < 3e-3


def test_fast_linear_falls_back_when_grad_needed(cuda_ok):
    lin = nn.Linear(256, 256).cuda()
    fl = g.FastLinear.from_linear(lin)
    x = torch.randn(4, 256, device="cuda", requires_grad=True)
    fl(x).sum().backward()
    assert x.grad is not None


def test_patch_replaces_linear_layers(cuda_ok):
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(512, 1024), nn.GELU(), nn.Linear(1024, 512), nn.Linear(512, 10)).cuda().eval()
    x = torch.randn(64, 512, device="cuda")
    with torch.no_grad():
        ref = model(x)
    assert g.patch(model, min_features=256) == 0  # B200 is not an affected GPU
    n = g.patch(model, min_features=256, force=True)
    assert n == 2  # the 512->10 head is below min_features
    assert isinstance(model[0], g.FastLinear) and isinstance(model[3], nn.Linear)
    with torch.no_grad():
        y = model(x)
    assert rel_err(y, ref) < 3e-3


def test_patch_skip(cuda_ok):
    model = nn.Sequential(nn.Linear(512, 512), nn.Linear(512, 512)).cuda()
    assert g.patch(model, force=True, skip=("1",)) == 1
    assert isinstance(model[0], g.FastLinear) and isinstance(model[1], nn.Linear)


def test_large_outputs_do_not_overflow_with_fp32_out(cuda_ok):
    x = torch.full((128, 4096), 16.0, device="cuda").half()
    w = torch.full((4096, 128), 16.0, device="cuda").half()
    y = g.mm_t(x, w, None, torch.float32)
    assert torch.isfinite(y).all()
    assert torch.all(y == 16 * 16 * 4096)  # exact in fp32 accumulation


@pytest.mark.parametrize("M", [1, 5, 8, 9, 64, 300])
@pytest.mark.parametrize("in_dtype", [torch.float32, torch.float16])
def test_massive_activations_do_not_overflow(cuda_ok, M, in_dtype):
    """The reference's massive-activation case (tests/test_correctness.py:112-126): a column at
    179,940 and one element at -120,000. The skinny path (M <= 8, fp32 out) is held to its own
    1e-5 bound against fp64, the GEMM path to 1e-3 (both norm-wise and component-wise)."""
    torch.manual_seed(1)
    K, N = 3072, 1024
    x = torch.randn(M, K, device="cuda")
    x[:, 7] = 179940.0 if in_dtype == torch.float32 else 60000.0
    x[0, 100] = -120000.0 if in_dtype == torch.float32 else -50000.0
    x = x.to(in_dtype)
    w = (torch.randn(K, N, device="cuda") * 0.3).half()
    y = g.mm_t(x, w, None, torch.float32)
    assert torch.isfinite(y).all()
    assert rel_err(y, x.float() @ w.float()) < 2e-3
    norm, rtol = bounds(M, torch.float32)
    assert rel_err(y, ref64(x, w)) < norm
    assert_close_fp64(y, x, w, None, torch.float32, f"massive activations M={M}")


def test_is_affected_reports_bool(cuda_ok):
    assert isinstance(g.is_affected(), bool)
    assert g.is_affected() is False  # sm_100


@pytest.mark.parametrize("M,K,N", [(64, 1024, 1024), (128, 16384, 1024), (300, 4096, 256), (129, 2048, 8)])
@pytest.mark.parametrize("ksplit", [1, 2, 3, 5, 7, 13, 16, 20])
def test_forced_split_k_through_c_abi(cuda_ok, M, K, N, ksplit):
    """g16_gemm with a forced K split (2..16: chunks reduced inside a thread-block cluster; 20: through
    the workspace): deterministic, matches fp64."""
    torch.manual_seed(ksplit)
    a = torch.randn(M, K, device="cuda").half()
    b = (torch.randn(K, N, device="cuda") * K ** -0.5).half()
    bias = torch.randn(N, device="cuda")
    L = _native.lib()
    stream = _native.stream_handle(0)
    nws = int(L.g16_gemm_workspace_bytes(M, K, N, ksplit))
    ws = torch.full((max(nws, 1),), 0xFF, dtype=torch.uint8, device="cuda")  # no initial contents needed
    outs = []
    for _ in range(2):
        out = torch.empty(M, N, device="cuda", dtype=torch.float32)
        st = L.g16_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.G16_F32, bias.data_ptr(), None, M, K, N,
                        ksplit, ws.data_ptr() if nws else None, nws, stream)
        assert st == 0, _native.strerror(st)
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    assert_close_fp64(outs[0], a, b, bias, torch.float32, f"split {ksplit}")


def _gemm_c(a, b, bias, rscale, out_dtype, ksplit):
    L = _native.lib()
    M, K = a.shape
    N = b.shape[1]
    nws = int(L.g16_gemm_workspace_bytes(M, K, N, ksplit))
    ws = torch.empty(max(nws, 256), dtype=torch.uint8, device="cuda")
    out = torch.empty(M, N, device="cuda", dtype=out_dtype)
    st = L.g16_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype),
                    None if bias is None else bias.data_ptr(), None if rscale is None else rscale.data_ptr(),
                    M, K, N, ksplit, ws.data_ptr(), ws.numel(), _native.stream_handle(0))
    assert st == 0, _native.strerror(st)
    return out


@pytest.mark.parametrize("M,K,N", [(128, 16384, 1024), (2048, 3072, 1024), (1000, 4096, 392), (250, 8192, 2000),
                                   (64, 1024, 1024), (384, 512, 136)])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_automatic_small_problem_plan(cuda_ok, M, K, N, out_dtype):
    """ksplit = 0 on outputs with few tiles: one CTA per (tile, K chunk), chunks reduced in a cluster.
    Deterministic, and within the GEMM tolerance of fp64 (with bias and per-row unscale), as is the
    forced single pass on the same inputs."""
    gen = torch.Generator(device="cuda").manual_seed(M + N)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    bias = torch.randn(N, device="cuda", generator=gen)
    rscale = torch.where(torch.rand(M, device="cuda", generator=gen) < 0.1, 4.0, 1.0)
    y0 = _gemm_c(a, b, bias, rscale, out_dtype, 0)
    y1 = _gemm_c(a, b, bias, rscale, out_dtype, 0)
    assert torch.equal(y0, y1)
    single = _gemm_c(a, b, bias, rscale, out_dtype, 1)
    ref = (a.double() @ b.double()) * rscale.double()[:, None] + bias.double()
    for y, what in ((y0, "automatic"), (single, "single pass")):
        assert torch.isfinite(y).all()
        assert ((y.double() - ref).norm() / ref.norm()).item() < GEMM_NORM, what


@pytest.mark.parametrize("M,K,N", [(4096, 1024, 4096), (2048, 512, 5120), (1000, 520, 5000), (512, 256, 12288),
                                   (1000, 776, 12296)])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_persistent_gemm_single_pass(cuda_ok, M, K, N, out_dtype):
    """Explicit single-pass GEMMs (ksplit = 1) run on CTA pairs (256 x 256 tiles, every tile over the
    whole K), N = 12288 and 12296 included. Deterministic, bitwise equal to the single-CTA kernel
    (reached through the one-destination scatter entry point, whose last partial wave runs as
    128-column halves when it fits in half the SMs: 512 x 12288 has 192 tiles on 148 SMs, the last
    44 as 88 halves), within the GEMM tolerance, bias on every column including ragged last tiles."""
    gen = torch.Generator(device="cuda").manual_seed(M + K + N)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    bias = torch.randn(N, device="cuda", generator=gen)
    y0 = _gemm_c(a, b, bias, None, out_dtype, 1)
    y1 = _gemm_c(a, b, bias, None, out_dtype, 1)
    assert torch.equal(y0, y1)
    single = torch.empty_like(y0)
    ptrs = (ctypes.c_void_p * 1)(single.data_ptr())
    st = _native.lib().g16_gemm_scatter(a.data_ptr(), b.data_ptr(), ptrs, 1, _native.dtype_code(out_dtype),
                                        bias.data_ptr(), None, M, K, N, N, 0, 0, _native.stream_handle(0))
    _native.check(st, "g16_gemm_scatter")
    assert torch.equal(y0, single)
    assert_close_fp64(y0, a, b, bias, out_dtype, "split tail")


MEDIUM_M = [(1, 1024, 768), (9, 64, 64), (16, 4096, 4096), (17, 1032, 776), (32, 768, 3072), (33, 4096, 768),
            (48, 16384, 1024), (64, 1024, 1024), (64, 520, 4104), (40, 8, 136)]


@pytest.mark.parametrize("M,K,N", MEDIUM_M)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_medium_m_kernel(cuda_ok, M, K, N, out_dtype):
    """Automatic plan for M <= 64: the swapped-operand kernel (128 weight columns per CTA as the
    MMA's M, the rows as its N padded to 16/32/64, K split over a cluster and the partials added in
    rank order). Reported by g16_gemm_plan; deterministic; within the GEMM tolerance of fp64 with
    bias and per-row unscale, ragged M, N and K (K = 8 and K = 520 leave a partial 64-wide step)."""
    L = _native.lib()
    info = (ctypes.c_int * 3)()
    assert L.g16_gemm_plan(M, K, N, info) == 0
    assert info[0] == 2 and info[1] == 128 and info[2] >= 1
    gen = torch.Generator(device="cuda").manual_seed(M * 31 + K + N)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    bias = torch.randn(N, device="cuda", generator=gen)
    rscale = torch.where(torch.rand(M, device="cuda", generator=gen) < 0.25, 8.0, 1.0)
    y0 = _gemm_c(a, b, bias, rscale, out_dtype, 0)
    y1 = _gemm_c(a, b, bias, rscale, out_dtype, 0)
    assert torch.equal(y0, y1)
    ref = (a.double() @ b.double()) * rscale.double()[:, None] + bias.double()
    assert torch.isfinite(y0).all()
    assert ((y0.double() - ref).norm() / ref.norm()).item() < GEMM_NORM
    single = _gemm_c(a, b, bias, rscale, out_dtype, 1)  # the 128-row-tile kernels
    assert ((y0.double() - single.double()).norm() / ref.norm()).item() < GEMM_NORM


def test_medium_m_plan_boundary(cuda_ok):
    L = _native.lib()
    info = (ctypes.c_int * 3)()
    assert L.g16_gemm_plan(64, 4096, 4096, info) == 0 and info[0] == 2
    assert L.g16_gemm_plan(65, 4096, 4096, info) == 0 and info[0] != 2


@pytest.mark.parametrize("M", [9, 24, 64])
def test_medium_m_fp32_activations_with_rescale(cuda_ok, M):
    """mm_t with fp32 activations, 8 < M <= 64: rowscale (rows above |1024| scaled by a power of two)
    then the medium-M kernel with the unscale in its epilogue; a row with a 1.2e5 spike stays finite
    and accurate."""
    torch.manual_seed(M)
    x = torch.randn(M, 3072, device="cuda")
    x[M // 2, 17] = 120000.0
    w = (torch.randn(3072, 1024, device="cuda") * 0.02).half()
    b = torch.randn(1024, device="cuda")
    y = g.mm_t(x, w, b, torch.float32)
    ref = x.double() @ w.double() + b.double()
    assert torch.isfinite(y).all()
    assert ((y.double() - ref).norm() / ref.norm()).item() < GEMM_NORM
    assert torch.equal(y, g.mm_t(x, w, b, torch.float32))


def test_rowscale_through_c_abi(cuda_ok):
    torch.manual_seed(5)
    M, K = 64, 1024
    x = torch.randn(M, K, device="cuda")
    x[3, 11] = 179940.0
    x[7, 0] = -2048.0
    x[9, 5] = 1024.0
    y = torch.empty(M, K, device="cuda", dtype=torch.float16)
    S = torch.empty(M, device="cuda")
    L = _native.lib()
    st = L.g16_rowscale(x.data_ptr(), _native.G16_F32, y.data_ptr(), S.data_ptr(), M, K, 1024.0, _native.stream_handle(0))
    assert st == 0
    assert S[3].item() == 256.0 and S[7].item() == 2.0 and S[9].item() == 1.0 and S[0].item() == 1.0
    torch.testing.assert_close(y.float(), (x / S[:, None]).half().float(), rtol=0, atol=0)


def _expected_row_scale(x):
    """S = smallest power of two with amax / S <= 1024 (1 when amax <= 1024), computed exactly."""
    amax = x.float().abs().amax(dim=1).double().cpu()
    r = amax / 1024.0
    m, e = torch.frexp(r)  # r = m * 2^e, m in [0.5, 1)
    c = torch.where(m == 0.5, e - 1, e)  # ceil(log2(r))
    return torch.where(amax > 1024.0, torch.pow(2.0, c.double()), torch.ones_like(amax)).float()


@pytest.mark.parametrize("xdt,K", [(torch.float32, 8), (torch.float32, 768), (torch.float32, 3072),
                                   (torch.float32, 3080), (torch.float32, 8192), (torch.float16, 4096),
                                   (torch.float16, 4104)])
def test_rowscale_row_lengths(cuda_ok, xdt, K):
    """Rows that fit a warp's registers (fp32 K <= 3072, fp16 K <= 4096) and longer rows (one CTA
    per row) give the same scale rule and the same bits as x / S cast to fp16."""
    torch.manual_seed(K)
    M = 300
    x = torch.randn(M, K, device="cuda") * 4
    x[0, K - 1] = 5000.0 if xdt == torch.float16 else 179940.0
    x[1, 0] = -1025.0
    x[2, K // 2] = 1024.0
    x = x.to(xdt)
    y = torch.empty(M, K, device="cuda", dtype=torch.float16)
    S = torch.empty(M, device="cuda")
    st = _native.lib().g16_rowscale(x.data_ptr(), _native.dtype_code(xdt), y.data_ptr(), S.data_ptr(), M, K, 1024.0,
                                    _native.stream_handle(0))
    assert st == 0
    exp_s = _expected_row_scale(x)
    assert torch.equal(S.cpu(), exp_s)
    assert S[1].item() == 2.0 and S[2].item() == 1.0
    assert torch.equal(y, (x.float() / S[:, None]).half())


# shapes reaching each epilogue: skinny (M <= 8, fp32 x), medium-M, small-problem (one chunk at
# 256 x 768 x 3072; the grid split at 128 x 16384 x 1024, where mm_t gives a workspace), CTA pairs
# (N = 12288 included), and the empty reduction
GELU_SHAPES = [(1, 1024, 3072), (4, 4096, 512), (16, 1024, 3072), (64, 768, 3072), (256, 768, 3072),
               (128, 16384, 1024), (4096, 768, 3072), (512, 256, 12288), (40, 0, 136)]


@pytest.mark.parametrize("M,K,N", GELU_SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_mm_t_gelu_epilogue(cuda_ok, M, K, N, out_dtype):
    """mm_t(..., act="gelu") applies the exact GELU to the fp32 epilogue value: it equals torch's
    F.gelu of the plain result (fp32 output) to an ulp, and the fp16 output is that value rounded."""
    torch.manual_seed(M + K + N)
    x = torch.randn(M, K, device="cuda")
    w = (torch.randn(K, N, device="cuda") * (max(K, 1) ** -0.5)).half()
    b = torch.randn(N, device="cuda")
    plain = g.mm_t(x, w, b, torch.float32)
    ref = F.gelu(plain)
    y = g.mm_t(x, w, b, out_dtype, act="gelu")
    if out_dtype == torch.float32:
        torch.testing.assert_close(y, ref, rtol=2e-6, atol=2e-7)
    else:
        torch.testing.assert_close(y.float(), ref.half().float(), rtol=1e-3, atol=1e-3)
    with pytest.raises(ValueError):
        g.mm_t(x, w, b, out_dtype, act="relu")


def test_mm_t_act_rejects_unknown_code(cuda_ok):
    L = _native.lib()
    x = torch.randn(16, 64, device="cuda")
    w = torch.randn(64, 64, device="cuda").half()
    out = torch.empty(16, 64, device="cuda")
    st = L.g16_mm_t_act(x.data_ptr(), _native.G16_F32, w.data_ptr(), None, out.data_ptr(), _native.G16_F32, 16, 64,
                        64, 7, None, 0, _native.stream_handle(0))
    assert st == _native.ERR_ARG


def test_k_zero_gives_bias(cuda_ok):
    x = torch.empty(16, 0, device="cuda").half()
    w = torch.empty(0, 64, device="cuda").half()
    b = torch.randn(64, device="cuda")
    y = g.mm_t(x, w, b, torch.float32)
    assert torch.equal(y, b.expand(16, 64))


def test_device_status_clean_after_suite(cuda_ok):
    assert _native.device_status(clear=False) == _native.OK


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("K,N", [(8, 64), (136, 8), (520, 1032), (1032, 776), (4096, 4096), (65536, 512)])
def test_skinny_all_m(cuda_ok, M, K, N):
    """Every M of the skinny path, ragged K (not a multiple of the 16-row box), K split over up to 16
    cluster ranks, and K large enough that x is staged in several pieces."""
    torch.manual_seed(M * 1000 + K + N)
    x = torch.randn(M, K, device="cuda")
    w = (torch.randn(K, N, device="cuda") * K ** -0.5).half()
    b = torch.randn(N, device="cuda") * 0.1
    y = g.mm_t(x, w, b, torch.float32)
    assert_close_fp64(y, x, w, b, torch.float32, f"skinny M={M} K={K} N={N}")
    y2 = g.mm_t(x, w, b, torch.float32)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("M", [1, 8])
def test_skinny_fp16_in_and_out(cuda_ok, M):
    torch.manual_seed(M)
    K, N = 2048, 520
    x = torch.randn(M, K, device="cuda").half()
    w = (torch.randn(K, N, device="cuda") * 0.05).half()
    b = torch.randn(N, device="cuda")
    y32 = g.mm_t(x, w, b, torch.float32)
    y16 = g.mm_t(x, w, b, torch.float16)
    assert_close_fp64(y32, x, w, b, torch.float32, "fp16 x -> fp32")
    assert_close_fp64(y16, x, w, b, torch.float16, "fp16 x -> fp16")
    assert torch.equal(y16, y32.half())  # the fused cast rounds the same fp32 sum
