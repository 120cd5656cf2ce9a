"""CUDA-graph capture of inference steps built on gtx16_fp16 (FastLinear, mm_t, matmul).

At batch 1 (token-by-token generation) a Linear of 4096 x 4096 streams 32 MiB of fp16 weights in
~9 us, while an eager FastLinear call costs tens of microseconds of Python, allocator and launch
work on the host (the reference measures it with bench/overhead.py; its PreparedLaunch,
src/gtx16_fp16/kernels.py:324-338, only trims the argument packing). Capturing a whole step
once and replaying it removes the host cost altogether: every libg16 entry point is capturable
(it never allocates, frees or synchronises; workspaces come from torch's caching allocator), and
the skinny kernels launch with programmatic dependent launch, which a graph keeps, so consecutive
layers overlap one kernel's start-up with the previous one's tail.

    step = gtx16_fp16.graphs.capture(model_step, x_example)   # warm-up + capture
    y = step(x)                                               # copy in, replay, return outputs

The step function must be a pure function of its tensor arguments (no host-side branching on
tensor values, no host synchronisation); shapes and dtypes are fixed at capture.
"""
from __future__ import annotations

from typing import Any, Callable, Sequence

import torch


def _flatten(out: Any) -> tuple[list[torch.Tensor], Callable[[list[torch.Tensor]], Any]]:
    """Tensors of a step's output (a tensor, or a tuple/list of tensors) and a rebuilder."""
    if isinstance(out, torch.Tensor):
        return [out], lambda ts: ts[0]
    if isinstance(out, (tuple, list)) and all(isinstance(t, torch.Tensor) for t in out):
        kind = type(out)
        return list(out), lambda ts: kind(ts)
    raise TypeError("a captured step must return a tensor or a tuple/list of tensors")


class GraphedStep:
    """A step function captured in a CUDA graph with static input and output tensors.

    Calling it copies the new inputs into the static inputs on the current stream, replays the
    graph there and returns the outputs (fresh clones by default, so results of earlier calls are
    never overwritten; ``clone=False`` returns the static outputs themselves, valid until the
    next call). Inputs must match the captured shapes, dtypes and device.
    """

    def __init__(self, fn: Callable[..., Any], example_inputs: Sequence[torch.Tensor], warmup: int = 3):
        if not example_inputs:
            raise ValueError("capture needs at least one example input tensor")
        dev = example_inputs[0].device
        if dev.type != "cuda" or any(t.device != dev for t in example_inputs):
            raise ValueError("capture: every example input must be on the same CUDA device")
        self.device = dev
        self.static_inputs = [t.detach().clone() for t in example_inputs]
        self._stream = torch.cuda.Stream(dev)
        self._graph = torch.cuda.CUDAGraph()
        cur = torch.cuda.current_stream(dev)
        self._stream.wait_stream(cur)
        with torch.no_grad(), torch.cuda.device(dev), torch.cuda.stream(self._stream):
            # Warm-up on the capture stream: one-time host work (kernel attributes, launch plans,
            # this stream's workspace) happens here, outside the capture.
            for _ in range(max(1, warmup)):
                fn(*self.static_inputs)
            self._stream.synchronize()
            with torch.cuda.graph(self._graph, stream=self._stream):
                out = fn(*self.static_inputs)
        cur.wait_stream(self._stream)
        self.static_outputs, self._rebuild = _flatten(out)

    def __call__(self, *inputs: torch.Tensor, clone: bool = True) -> Any:
        if len(inputs) != len(self.static_inputs):
            raise ValueError(f"expected {len(self.static_inputs)} inputs, got {len(inputs)}")
        for dst, src in zip(self.static_inputs, inputs):
            if src.shape != dst.shape or src.dtype != dst.dtype or src.device != dst.device:
                raise ValueError(f"input {tuple(src.shape)} {src.dtype} {src.device} does not match the captured "
                                 f"{tuple(dst.shape)} {dst.dtype} {dst.device}")
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src)
        self.replay()
        outs = [t.clone() for t in self.static_outputs] if clone else self.static_outputs
        return self._rebuild(outs)

    def replay(self) -> None:
        """Replay on the current stream with whatever the static inputs hold."""
        with torch.cuda.device(self.device):
            self._graph.replay()

    def close(self) -> None:
        """Release the graph (and with it the graph's memory pool)."""
        self._graph.reset()


def capture(fn: Callable[..., Any], *example_inputs: torch.Tensor, warmup: int = 3) -> GraphedStep:
    """Warm up ``fn(*example_inputs)`` and capture it in a CUDA graph (see GraphedStep)."""
    return GraphedStep(fn, example_inputs, warmup=warmup)
