"""nn.Linear replacement storing fp16 weights and computing with the sm_100a kernels.

Mirrors src/gtx16_fp16/linear.py: same class name, constructor, buffers (``weight_t`` fp16
[in, out], ``bias`` fp32 [out]) and so the same state_dict keys, the ``from_linear`` constructor,
the ``.weight`` view, the forward branches and ``patch``.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native
from ._native import G16_F32, G16Error, stream_handle
from .ops import SKINNY_MAX_M, is_affected, mm_t, supported


class FastLinear(nn.Module):
    """Inference-only linear layer backed by libg16.

    - Weight stored once as fp16, transposed to [in, out] (half the memory of fp32).
    - Small batches (<= 8 rows, e.g. token-by-token generation) compute in fp32 from fp32 inputs
      on the HBM-streaming skinny kernel (one C call, no zero-fill).
    - Larger batches run the tcgen05 tensor-core GEMM: fp32 inputs are cast to fp16 with the per-row
      power-of-two rescale of rows with |max| > 1024, products accumulate in fp32, and the unscale
      and fp32 bias are fused into the epilogue.
    - Output dtype follows the input dtype (fp32 in -> fp32 out).
    - When autograd is needed or the shape is unsupported, falls back to F.linear (linear.py:45-46,69-70).
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.register_buffer("weight_t", torch.empty(in_features, out_features, dtype=torch.float16, device=device))
        self.register_buffer("bias", torch.empty(out_features, dtype=torch.float32, device=device) if bias else None)

    @classmethod
    def from_linear(cls, lin: nn.Linear) -> "FastLinear":
        m = cls(lin.in_features, lin.out_features, lin.bias is not None, device=lin.weight.device)
        with torch.no_grad():
            m.weight_t.copy_(lin.weight.detach().t().to(torch.float16))
            if lin.bias is not None:
                m.bias.copy_(lin.bias.detach().float())
        return m

    @property
    def weight(self) -> torch.Tensor:  # some model code reads .weight (e.g. for dtype/device)
        return self.weight_t.t()

    def _apply(self, fn, recurse=True):
        """Device moves apply as usual, but the storage formats the kernels read stay fixed:
        weight_t fp16 and bias fp32, so model.half() / .float() / .to(dtype) cannot hand the kernels
        a buffer of another type. A dtype change is dropped, not applied and undone, so no value
        loses precision on the way."""
        for name, want in (("weight_t", torch.float16), ("bias", torch.float32)):
            t = self._buffers.get(name)
            if t is None:
                continue
            moved = fn(t)
            if moved.dtype != want:
                moved = t.to(device=moved.device, dtype=want)
            self._buffers[name] = moved
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out_dtype = x.dtype if x.dtype in (torch.float32, torch.float16) else torch.float32
        if torch.is_grad_enabled() and x.requires_grad:
            return F.linear(x, self.weight_t.t().to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
        shape = x.shape
        # Small-batch fast path (generation): one C call, minimal Python per call.
        if x.is_cuda and x.dtype == torch.float32 and x.is_contiguous() and x.data_ptr() % 16 == 0:
            K, N = self.in_features, self.out_features
            M = x.numel() // K if shape[-1] == K else -1
            if 0 < M <= SKINNY_MAX_M and K % 8 == 0 and N % 8 == 0 and self.weight_t.data_ptr() % 16 == 0:
                idx = x.device.index or 0
                out = torch.empty(*shape[:-1], N, device=x.device, dtype=torch.float32)
                b = self.bias
                if idx != torch.cuda.current_device():
                    with torch.cuda.device(idx):
                        st = self._skinny(x, b, out, M, K, N, idx)
                else:
                    st = self._skinny(x, b, out, M, K, N, idx)
                if st != _native.OK:
                    raise G16Error(st, "g16_skinny")
                return out
        x2 = x.reshape(-1, self.in_features)
        if x2.dtype not in (torch.float16, torch.float32):
            x2 = x2.float()
        x2 = x2.contiguous()  # fp32 stays fp32: the kernels cast (and rescale large rows) themselves
        if x2.shape[0] == 0 or not supported(x2, self.weight_t):
            y = F.linear(x2.float(), self.weight_t.t().float(), self.bias)
        else:
            y = mm_t(x2, self.weight_t, self.bias, torch.float32 if out_dtype == torch.float32 else torch.float16)
        return y.reshape(*shape[:-1], self.out_features).to(out_dtype)

    def _skinny(self, x, b, out, M, K, N, idx) -> int:
        return _native.lib().g16_skinny(x.data_ptr(), G16_F32, self.weight_t.data_ptr(),
                                        None if b is None else b.data_ptr(), out.data_ptr(), G16_F32, M, K, N,
                                        stream_handle(idx))

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


def patch(model: nn.Module, min_features: int = 256, force: bool = False,
          skip: tuple[str, ...] = (), *, activations: torch.dtype | None = None) -> int:
    """Replace nn.Linear layers in-place with FastLinear. Returns the number replaced.

    Same selection rules as the reference (linear.py:79-99): only on affected GPUs unless
    force=True (B200 is not "affected", so pass force=True there); CUDA weights only; in and out
    features >= min_features and multiples of 8; qualified names containing any string in `skip`
    are left alone (e.g. skip=("lm_head",) keeps an output head in fp32).

    activations=torch.float16 (opt-in, not in the reference) also converts the rest of the model
    to fp16 after the swap, so activations stay fp16 between layers: each FastLinear then reads
    fp16 activations with no rescale pass and writes fp16, and the layers in between (attention,
    norms, activation functions) run in torch's fp16 kernels. FastLinear keeps its own formats
    (weight_t fp16, bias fp32). Inputs must then be fp16 (or integer ids). Accuracy follows fp16
    activations rather than the fp32 reference semantics (linear.py:44), which is why it is opt-in.
    """
    if activations not in (None, torch.float16, torch.float32):
        raise ValueError(f"activations must be None, torch.float16 or torch.float32, got {activations}")
    if not force and not any(is_affected(p.device) for p in model.parameters() if p.is_cuda):
        return 0
    n = 0
    for name, mod in list(model.named_modules()):
        for child_name, child in list(mod.named_children()):
            full = f"{name}.{child_name}" if name else child_name
            if (isinstance(child, nn.Linear) and child.weight.is_cuda
                    and min(child.in_features, child.out_features) >= min_features
                    and child.in_features % 8 == 0 and child.out_features % 8 == 0
                    and not any(s in full for s in skip)):
                setattr(mod, child_name, FastLinear.from_linear(child))
                n += 1
    if activations is torch.float16:
        model.half()
    elif activations is torch.float32:
        model.float()
    return n
