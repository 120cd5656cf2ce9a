"""CUDA-graph capture of FastLinear steps (gtx16_fp16.graphs) on the GPU: a patched layer stack
replayed from a graph gives the same bits as eager calls, at batch sizes that take the skinny
kernel (M <= 8) and the rowscale + tensor-core GEMM path (M = 16, fp32 activations with a row
above the rescale threshold); the graph holds the libg16 kernels (launch counter), outputs of
earlier calls are not overwritten, and mismatched inputs are refused."""
import pytest
import torch
import torch.nn as nn

import gtx16_fp16 as g
from gtx16_fp16 import _native

pytestmark = pytest.mark.gpu


def _stack(seed):
    torch.manual_seed(seed)
    model = nn.Sequential(nn.Linear(1024, 3072), nn.GELU(), nn.Linear(3072, 1024), nn.GELU(),
                          nn.Linear(1024, 1024)).cuda().eval()
    assert g.patch(model, force=True) == 3
    return model


@pytest.mark.parametrize("M", [1, 4, 16])
def test_graphed_stack_matches_eager(cuda_ok, M):
    model = _stack(M)
    gen = torch.Generator(device="cuda").manual_seed(M)
    x0 = torch.randn(M, 1024, device="cuda", generator=gen)
    l0 = _native.launch_count()
    step = g.graphs.capture(model, x0)
    per_call = (_native.launch_count() - l0) // 4  # 3 warm-up calls + the captured one
    assert per_call >= 3  # one libg16 kernel per layer at least (rowscale + GEMM at M = 16)
    outs = []
    for i in range(3):
        x = torch.randn(M, 1024, device="cuda", generator=gen)
        if M == 16:
            x[3] *= 3000.0  # |max| above 1024: the row is rescaled before the fp16 cast
        y = step(x)
        with torch.no_grad():
            ref = model(x)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), i
        outs.append((y, ref))
    for y, ref in outs:  # clones: later replays did not overwrite earlier results
        assert torch.equal(y, ref)
    step.close()


def test_graphed_step_static_outputs_and_checks(cuda_ok):
    model = _stack(7)
    x = torch.randn(1, 1024, device="cuda")
    step = g.graphs.capture(model, x)
    a = step(x, clone=False)
    b = step(x * 2, clone=False)
    assert a.data_ptr() == b.data_ptr() == step.static_outputs[0].data_ptr()
    with torch.no_grad():
        assert torch.equal(b, model(x * 2))
    with pytest.raises(ValueError, match="does not match"):
        step(torch.randn(2, 1024, device="cuda"))
    with pytest.raises(ValueError, match="expected 1 inputs"):
        step(x, x)
    step.close()


def test_graphed_mm_t_with_workspace(cuda_ok):
    """mm_t on fp32 activations takes a workspace (fp16 copy + row scales) from the capture
    stream's cache. A larger call on that same stream afterwards grows the cache: the buffer the
    graph holds is retired, not freed, so later replays stay correct."""
    torch.manual_seed(3)
    w = (torch.randn(2048, 1024, device="cuda") * 0.02).half()
    bias = torch.randn(1024, device="cuda")
    x = torch.randn(512, 2048, device="cuda")
    step = g.graphs.capture(lambda t: g.mm_t(t, w, bias, torch.float32), x)
    big = torch.randn(4096, 2048, device="cuda")
    side = step._stream
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        g.mm_t(big, w, bias, torch.float32)  # grows the capture stream's workspace
        filler = torch.full((64 << 20,), 7, dtype=torch.uint8, device="cuda")  # reuse freed memory, if any
    torch.cuda.current_stream().wait_stream(side)
    del filler
    for _ in range(2):
        x2 = torch.randn(512, 2048, device="cuda") * 10
        assert torch.equal(step(x2), g.mm_t(x2, w, bias, torch.float32))
    step.close()
