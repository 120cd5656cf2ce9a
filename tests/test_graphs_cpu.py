"""Host-side logic of CUDA-graph support, on a CPU-only host: the step capture helper's argument
checks, and the workspace cache that must never free a buffer a captured graph may still use."""
import pytest
import torch

from gtx16_fp16 import _native, graphs


def test_capture_rejects_non_cuda_inputs():
    with pytest.raises(ValueError, match="CUDA device"):
        graphs.capture(lambda x: x * 2, torch.zeros(4))
    with pytest.raises(ValueError, match="at least one"):
        graphs.GraphedStep(lambda: None, [])


def test_outgrown_workspace_is_retired_not_freed():
    # device "cpu" stands in for a GPU: the cache logic is the same; stream ids are plain keys
    dev = torch.device("cpu")
    stream = 0x5eed
    p1, n1 = _native.workspace(dev, stream, 1000)
    assert n1 >= 1000
    p_same, _ = _native.workspace(dev, stream, 500)
    assert p_same == p1  # a smaller request reuses the buffer
    before = len(_native._ws_retired)
    p2, n2 = _native.workspace(dev, stream, 5000)
    assert n2 >= 5000
    assert len(_native._ws_retired) == before + 1
    assert _native._ws_retired[-1].data_ptr() == p1  # the old buffer is still alive
    assert _native.workspace(dev, stream + 1, 10)[0] not in (p1, p2)  # per-stream buffers
    assert _native.workspace(dev, stream, 0) == (0, 0)


def test_flatten_outputs():
    t = torch.ones(2)
    ts, rebuild = graphs._flatten(t)
    assert ts == [t] and rebuild(ts) is t
    ts, rebuild = graphs._flatten((t, t + 1))
    assert isinstance(rebuild(ts), tuple) and len(rebuild(ts)) == 2
    with pytest.raises(TypeError):
        graphs._flatten({"y": t})
