"""g16_gemm_static_scratch, the GEMM entry point for callers that cannot allocate device memory at
call time (for example a server that reserved all GPU memory for its own pools at start-up). It runs
g16_gemm's plan, but the one plan that needs scratch memory, the split into fp32 partial tiles,
keeps them in a fixed 8 MiB array inside libg16 instead of a caller workspace.

Checked through the C ABI against the workspace-based g16_gemm with the same arguments (for the
automatic plan, with a workspace no larger than the array), on two calls in a row (the second on
new inputs, so whatever the first call left in the shared array must not leak into the result).
The cases with ksplit > 16 run the partial-tile split and 128 x 3840 x 1024 the grid split, the
plans that read and write the array; the others check that the plans needing no scratch are
g16_gemm's own. This file is collected last on purpose."""
import pytest
import torch

from gtx16_fp16 import _native

from _tol import assert_close_fp64, rel_err, GEMM_NORM

pytestmark = pytest.mark.gpu


STATIC_BYTES = 8 << 20  # G16_STATIC_SCRATCH_BYTES


def _gemm_with_workspace(a, b, bias, out_dtype, ksplit):
    """g16_gemm with a workspace of at most the static array's size: the automatic plan then takes
    the same branches as g16_gemm_static_scratch (the grid split only where its partials fit)."""
    L = _native.lib()
    M, K = a.shape
    N = b.shape[1]
    nws = int(L.g16_gemm_workspace_bytes(M, K, N, ksplit))
    if ksplit == 0:
        nws = min(nws, STATIC_BYTES)
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
    out = torch.full((M, N), float("nan"), dtype=out_dtype, device=a.device)
    st = L.g16_gemm_static_scratch(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype),
                                   None if bias is None else bias.data_ptr(), None, M, K, N, ksplit,
                                   _native.stream_handle(a.device.index or 0))
    assert st == _native.OK, _native.strerror(st)
    return out


def _inputs(M, K, N, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    bias = torch.randn(N, device="cuda", generator=gen)
    return a, b, bias


@pytest.mark.parametrize("M,K,N,ksplit", [
    # partial-tile split through the static array (ksplit > 16)
    (128, 16384, 256, 32),   # 1 tile x 32 chunks = 4 MiB of partials
    (200, 8192, 256, 20),    # 2 tiles x 20 chunks = 5 MiB
    (100, 4096, 264, 17),    # 2 tiles, 64 k-blocks: 16 chunks of 4 = 4 MiB, still the partials path
    (64, 16384, 512, 32),    # 2 tiles x 32 = 8 MiB, the whole array
    # plans without scratch: in-cluster split, automatic plan (medium-M, small-problem; the grid
    # split's partials exceed the array at 128 x 16384 x 1024, so the cluster plan runs there)
    (64, 1024, 1024, 4), (128, 16384, 1024, 16), (200, 1032, 136, 3), (1024, 4096, 4096, 2),
    (48, 4096, 768, 0), (2048, 3072, 1024, 0), (128, 16384, 1024, 0),
    # automatic plan with the grid split inside the array (8 tiles x 15 chunks = 7.5 MiB)
    (128, 3840, 1024, 0),
])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_static_scratch_matches_workspace_gemm(cuda_ok, M, K, N, ksplit, out_dtype):
    for call in range(2):  # two calls in a row, new inputs each time
        a, b, bias = _inputs(M, K, N, 1000 * call + M + K + N + ksplit)
        ref = _gemm_with_workspace(a, b, bias, out_dtype, ksplit)
        got = _gemm_static(a, b, bias, out_dtype, ksplit)
        torch.cuda.synchronize()
        assert rel_err(got, ref.double()) <= GEMM_NORM
        assert torch.equal(got, ref)  # same plan, same K split: identical bits
        assert_close_fp64(got, a, b, bias, out_dtype, f"static scratch call {call}")


def test_static_scratch_array_does_not_leak_between_calls(cuda_ok):
    """A large-split call fills the array; a following call with another shape and split that reads
    fewer partials gets exactly g16_gemm's result."""
    a, b, bias = _inputs(64, 16384, 512, 1)
    _gemm_static(a, b, bias, torch.float32, 32)  # 8 MiB of partials
    a, b, bias = _inputs(128, 8192, 256, 2)
    ref = _gemm_with_workspace(a, b, bias, torch.float32, 24)
    got = _gemm_static(a, b, bias, torch.float32, 24)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


def test_static_scratch_rejects_splits_that_do_not_fit(cuda_ok):
    # 1024 x 4096 output = 128 tiles; 20 K chunks need 128 x 20 x 128 KiB = 320 MiB > 8 MiB
    L = _native.lib()
    a = torch.zeros(1024, 4096, device="cuda", dtype=torch.float16)
    b = torch.zeros(4096, 4096, device="cuda", dtype=torch.float16)
    out = torch.full((1024, 4096), 7.0, device="cuda", dtype=torch.float16)
    st = L.g16_gemm_static_scratch(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.G16_F16, None, None,
                                   1024, 4096, 4096, 20, _native.stream_handle(0))
    assert st == _native.ERR_TOO_LARGE
    assert "8 MiB" in _native.strerror(st)
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched
