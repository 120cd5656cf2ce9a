"""The small-problem GEMM's grid split (automatic plan kind 3: the K chunks of a few output tiles as
independent CTAs of one resident wave, reduced through the caller's workspace with per-tile call
tags). It replaces the reference's split-K for tiny outputs with long K (hgemm_splitk,
src/gtx16_fp16/kernels.py:143-147, chosen at ops.py:92-101), as the in-cluster reduction does when
no workspace is given.

Checked through the C ABI: against fp64; bitwise run to run; against the same K chunks reduced
through the workspace split-K path; with workspaces that start as zeros, all-ones bits or stale
data of other shapes; across interleaved shapes sharing one workspace; inside a replayed CUDA
graph; and the cluster plan taking over when no workspace is given."""
import ctypes

import pytest
import torch

import gtx16_fp16 as g
from gtx16_fp16 import _native

from _tol import assert_close_fp64

pytestmark = pytest.mark.gpu

GS_SHAPES = [(128, 16384, 1024), (256, 16384, 512), (128, 8192, 2048), (100, 12288, 776), (200, 6144, 264)]


def _plan(M, K, N):
    info = (ctypes.c_int * 3)()
    assert _native.lib().g16_gemm_plan(M, K, N, info) == _native.OK
    return tuple(info)


def _inputs(M, K, N, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    bias = torch.randn(N, device="cuda", generator=gen)
    return a, b, bias


def _gemm(a, b, bias, out_dtype, ksplit, ws, rscale=None):
    M, K = a.shape
    N = b.shape[1]
    out = torch.full((M, N), float("nan"), dtype=out_dtype, device=a.device)
    st = _native.lib().g16_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype),
                                None if bias is None else bias.data_ptr(),
                                None if rscale is None else rscale.data_ptr(), M, K, N, ksplit,
                                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                                _native.stream_handle(a.device.index or 0))
    assert st == _native.OK, _native.strerror(st)
    return out


def _workspace(M, K, N, ksplit=0, fill=None):
    n = int(_native.lib().g16_gemm_workspace_bytes(M, K, N, ksplit))
    ws = torch.empty(max(n, 256), dtype=torch.uint8, device="cuda")
    if fill is not None:
        ws.fill_(fill)
    return ws


@pytest.mark.parametrize("M,K,N", GS_SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_grid_split_matches_fp64_and_workspace_split(cuda_ok, M, K, N, out_dtype):
    kind, bn, chunks = _plan(M, K, N)
    assert kind == 3 and 2 <= chunks <= 32, (kind, bn, chunks)
    ws = _workspace(M, K, N)
    for call in range(2):
        a, b, bias = _inputs(M, K, N, 10 * call + M + N)
        y = _gemm(a, b, bias, out_dtype, 0, ws)
        assert_close_fp64(y, a, b, bias, out_dtype, f"grid split {M}x{K}x{N} call {call}")
        assert torch.equal(_gemm(a, b, bias, out_dtype, 0, ws), y)  # bitwise run to run
        # the same K chunks added in the same order through the workspace split-K path
        forced = _gemm(a, b, bias, out_dtype, chunks, _workspace(M, K, N, chunks))
        assert torch.equal(forced, y)


@pytest.mark.parametrize("fill", [0, 255, 0x3F])
def test_grid_split_needs_no_initial_workspace_contents(cuda_ok, fill):
    M, K, N = 128, 16384, 1024
    a, b, bias = _inputs(M, K, N, 5)
    ref = _gemm(a, b, bias, torch.float32, 0, _workspace(M, K, N))
    for _ in range(3):
        ws = _workspace(M, K, N, fill=fill)
        assert torch.equal(_gemm(a, b, bias, torch.float32, 0, ws), ref)


def test_grid_split_shapes_interleaved_on_one_workspace(cuda_ok):
    """Calls of other shapes (other tile counts and chunk counts, and the workspace split-K path,
    whose partials overwrite the tags) between grid-split calls on the same workspace."""
    shapes = [(128, 16384, 1024), (256, 16384, 512), (200, 6144, 264), (128, 8192, 2048)]
    need = max(int(_native.lib().g16_gemm_workspace_bytes(M, K, N, k)) for (M, K, N) in shapes for k in (0, 24))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    data = {s: _inputs(*s, seed=sum(s)) for s in shapes}
    refs = {s: _gemm(*data[s], torch.float32, 0, _workspace(*s)) for s in shapes}
    for rep in range(3):
        for s in shapes + shapes[::-1]:
            assert torch.equal(_gemm(*data[s], torch.float32, 0, ws), refs[s]), (rep, s)
        a, b, bias = data[shapes[0]]
        _gemm(a, b, bias, torch.float32, 24, ws)  # partial-tile split over the same bytes


def test_grid_split_in_cuda_graph(cuda_ok):
    M, K, N = 128, 16384, 1024
    sets = [_inputs(M, K, N, 50 + i) for i in range(3)]
    ws = _workspace(M, K, N)
    refs = [_gemm(a, b, bias, torch.float16, 0, _workspace(M, K, N)) for (a, b, bias) in sets]
    outs = [torch.empty(M, N, dtype=torch.float16, device="cuda") for _ in sets]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    L = _native.lib()

    def step():
        for (a, b, bias), o in zip(sets, outs):
            st = L.g16_gemm(a.data_ptr(), b.data_ptr(), o.data_ptr(), _native.G16_F16, bias.data_ptr(), None, M, K,
                            N, 0, ws.data_ptr(), ws.numel(), s.cuda_stream)
            assert st == _native.OK

    with torch.cuda.stream(s):
        step()
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        step()
    for _ in range(4):
        for o in outs:
            o.fill_(float("nan"))
        with torch.cuda.stream(s):
            graph.replay()
        s.synchronize()
        for o, r in zip(outs, refs):
            assert torch.equal(o, r)
    assert _native.device_status(clear=True) == _native.OK
    del graph


def test_without_workspace_the_cluster_plan_runs(cuda_ok):
    M, K, N = 128, 16384, 1024
    a, b, bias = _inputs(M, K, N, 9)
    launches = _native.launch_count()
    y = _gemm(a, b, bias, torch.float32, 0, None)
    assert _native.launch_count() == launches + 1
    assert_close_fp64(y, a, b, bias, torch.float32, "cluster plan")
    assert torch.equal(_gemm(a, b, bias, torch.float32, 0, None), y)


def test_grid_split_with_row_scales_and_mm_t(cuda_ok):
    """fp32 activations through mm_t: rowscale, then the grid split with the unscale in its
    reduction (the workspace from the package's per-stream cache)."""
    M, K, N = 128, 16384, 1024
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(M, K, device="cuda", generator=gen)
    x[5] *= 4000.0  # a row above the rescale threshold
    w = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    bias = torch.randn(N, device="cuda", generator=gen)
    y = g.mm_t(x, w, bias, torch.float32)
    assert_close_fp64(y, x, w, bias, torch.float32, "mm_t grid split")
    assert torch.equal(g.mm_t(x, w, bias, torch.float32), y)
    assert _native.device_status(clear=True) == _native.OK
