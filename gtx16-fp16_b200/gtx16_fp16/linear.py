"""nn.Linear replacement storing fp16 weights and computing with the sm_100a kernels.

Mirrors src/gtx16_fp16/linear.py: same class name, constructor, buffers (``weight_t`` fp16
[in, out], ``bias`` fp32 [out]) and so the same state_dict keys, the ``from_linear`` constructor,
the ``.weight`` view, the forward branches and ``patch``.
"""
from __future__ import annotations

import weakref

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native
from ._native import G16_F32, G16Error, stream_handle
from .ops import SKINNY_MAX_M, is_affected, mm_t, supported


class FastLinear(nn.Module):
    """An nn.Linear for inference whose matmuls run in libg16.

    - The weight is kept once, in fp16 and already transposed: ``weight_t`` is [in, out], so the
      layer holds half the bytes of an fp32 nn.Linear.
    - Up to 8 rows of fp32 input (decoding one token at a time, say) go to the skinny GEMV kernel,
      which multiplies and accumulates in fp32 with one C call and no zero-filled output.
    - More rows go to the tcgen05 GEMM: fp32 rows are rounded to fp16 (rows above 1024 in magnitude
      are first divided by a power of two), products accumulate in fp32 and the epilogue undoes the
      row scale and adds the fp32 bias.
    - The result has the input's dtype: fp16 in gives fp16 out, fp32 in gives fp32 out.
    - Inputs that need a gradient, and shapes mm_t does not accept, are computed with F.linear, the
      reference's own fallback (linear.py:45-46,69-70).
    - ``activation = "gelu"`` (set by ``patch(..., fuse=True)``, not in the reference) applies the
      exact GELU in the GEMM epilogue; a layer in a shared-input group (attention's query/key/value)
      computes the group's fused GEMM once per input and returns its column slice.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.activation: str | None = None
        self._group: _SharedInputGroup | None = None
        self._group_index = 0
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
    def weight(self) -> torch.Tensor:  # for callers that inspect .weight (its dtype, device, shape)
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
            y = F.linear(x, self.weight_t.t().to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
            return F.gelu(y) if self.activation == "gelu" else y
        if self._group is not None and x.is_cuda:
            return self._group.output(self._group_index, x)
        shape = x.shape
        # Small-batch fast path (generation): one C call, minimal Python per call.
        if (self.activation is None and x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
                and x.data_ptr() % 16 == 0):
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
        x2 = x2.contiguous()  # no cast here: libg16 rounds fp32 rows to fp16 (with the row rescale)
        if x2.shape[0] == 0 or not supported(x2, self.weight_t):
            y = F.linear(x2.float(), self.weight_t.t().float(), self.bias)
            if self.activation == "gelu":
                y = F.gelu(y)
        else:
            y = mm_t(x2, self.weight_t, self.bias, torch.float32 if out_dtype == torch.float32 else torch.float16,
                     act=self.activation)
        return y.reshape(*shape[:-1], self.out_features).to(out_dtype)

    def _skinny(self, x, b, out, M, K, N, idx) -> int:
        return _native.lib().g16_skinny(x.data_ptr(), G16_F32, self.weight_t.data_ptr(),
                                        None if b is None else b.data_ptr(), out.data_ptr(), G16_F32, M, K, N,
                                        stream_handle(idx))

    def extra_repr(self) -> str:
        r = f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"
        if self.activation is not None:
            r += f", activation={self.activation}"
        if self._group is not None:
            r += f", fused_group={self._group_index}/{len(self._group.members)}"
        return r


class _SharedInputGroup:
    """FastLinear layers that read the same input, e.g. attention's query / key / value: one GEMM
    over their concatenated weights ([K, sum N], a single rowscale pass for fp32 input) instead of
    one per layer. The first member called with an input computes the fused result; each other
    member called next with the same tensor (same object, same version, same stream) takes its
    column slice of it. A member called with another input recomputes. The concatenated weight is a
    copy (the members keep their own buffers, so state_dict is unchanged); it is rebuilt if a
    member's weight_t or bias changed (a load_state_dict, a device move)."""

    def __init__(self, members: list[FastLinear]):
        self.members = members
        self._w = None
        self._b = None
        self._src = None
        self._key = None
        self._out = None
        self._pending: set[int] = set()
        for i, m in enumerate(members):
            m._group, m._group_index = self, i

    def _weights(self):
        src = tuple((m.weight_t.data_ptr(), m.weight_t._version,
                     None if m.bias is None else (m.bias.data_ptr(), m.bias._version)) for m in self.members)
        if src != self._src:
            with torch.no_grad():
                self._w = torch.cat([m.weight_t for m in self.members], dim=1).contiguous()
                if all(m.bias is None for m in self.members):
                    self._b = None
                else:
                    self._b = torch.cat([m.bias if m.bias is not None else
                                         torch.zeros(m.out_features, device=m.weight_t.device) for m in self.members])
            self._src = src
        return self._w, self._b

    def output(self, index: int, x: torch.Tensor) -> torch.Tensor:
        key = (x.data_ptr(), x._version, tuple(x.shape), x.stride(), x.dtype, x.device,
               torch.cuda.current_stream(x.device).cuda_stream)
        ref = self._key[0]() if self._key is not None else None
        if ref is x and self._key[1] == key and index in self._pending:
            self._pending.discard(index)
            out = self._out
            if not self._pending:
                self._key, self._out = None, None
            return self._slice(out, index)
        m0 = self.members[0]
        w, b = self._weights()
        K = m0.in_features
        out_dtype = x.dtype if x.dtype in (torch.float32, torch.float16) else torch.float32
        x2 = x.reshape(-1, K)
        if x2.dtype not in (torch.float16, torch.float32):
            x2 = x2.float()
        x2 = x2.contiguous()
        if x2.shape[0] == 0 or not supported(x2, w):
            y = F.linear(x2.float(), w.t().float(), b).to(out_dtype)
        else:
            y = mm_t(x2, w, b, torch.float32 if out_dtype == torch.float32 else torch.float16)
        y = y.reshape(*x.shape[:-1], w.shape[1])
        self._key = (weakref.ref(x), key)
        self._out = y
        self._pending = set(range(len(self.members))) - {index}
        return self._slice(y, index)

    def _slice(self, y: torch.Tensor, index: int) -> torch.Tensor:
        n0 = sum(m.out_features for m in self.members[:index])
        return y[..., n0:n0 + self.members[index].out_features]


def _is_exact_gelu(fn) -> bool:
    if isinstance(fn, nn.GELU):
        return fn.approximate == "none"
    # transformers' GELUActivation (hidden_act="gelu") wraps the exact torch.nn.functional.gelu
    return type(fn).__name__ == "GELUActivation" and getattr(fn, "act", None) is F.gelu


def _fuse(model: nn.Module) -> tuple[int, int]:
    """Fold exact GELUs that follow a FastLinear into its epilogue, and group query/key/value
    FastLinears of one module. Returns (GELUs folded, groups formed)."""
    gelus = groups = 0
    for mod in model.modules():
        # x -> dense -> intermediate_act_fn (transformers' BertIntermediate and alike)
        dense, act = getattr(mod, "dense", None), getattr(mod, "intermediate_act_fn", None)
        if isinstance(dense, FastLinear) and dense.activation is None and _is_exact_gelu(act):
            dense.activation = "gelu"
            mod.intermediate_act_fn = nn.Identity()
            gelus += 1
        # nn.Sequential(..., FastLinear, GELU, ...)
        if isinstance(mod, nn.Sequential):
            names = list(mod._modules.keys())
            for a, b in zip(names, names[1:]):
                lin, act = mod._modules[a], mod._modules[b]
                if isinstance(lin, FastLinear) and lin.activation is None and _is_exact_gelu(act):
                    lin.activation = "gelu"
                    mod._modules[b] = nn.Identity()
                    gelus += 1
        qkv = [getattr(mod, n, None) for n in ("query", "key", "value")]
        if (all(isinstance(m, FastLinear) for m in qkv) and len({m.in_features for m in qkv}) == 1
                and all(m._group is None and m.activation is None for m in qkv)
                and len({m.weight_t.device for m in qkv}) == 1):
            _SharedInputGroup(qkv)
            groups += 1
    return gelus, groups


def patch(model: nn.Module, min_features: int = 256, force: bool = False,
          skip: tuple[str, ...] = (), *, activations: torch.dtype | None = None, fuse: bool = False) -> int:
    """Swap the model's eligible nn.Linear children for FastLinear copies, in place, and return
    how many were swapped.

    A layer is eligible under the reference's rules (linear.py:79-99): the model has a parameter on
    an affected GPU, or force=True (a B200 is never affected, so pass force=True there); the layer's
    weight is on a CUDA device; both feature counts are at least min_features and divisible by 8;
    and no string in `skip` occurs in its dotted name (skip=("lm_head",), for example, leaves a
    model's output head as an fp32 nn.Linear).

    activations=torch.float16 (opt-in, not in the reference) also converts the rest of the model
    to fp16 after the swap, so activations stay fp16 between layers: each FastLinear then reads
    fp16 activations with no rescale pass and writes fp16, and the layers in between (attention,
    norms, activation functions) run in torch's fp16 kernels. FastLinear keeps its own formats
    (weight_t fp16, bias fp32). Inputs must then be fp16 (or integer ids). Accuracy follows fp16
    activations rather than the fp32 reference semantics (linear.py:44), which is why it is opt-in.

    fuse=True (opt-in, not in the reference) rewrites two patterns after the swap: an exact GELU
    right after a patched layer (a module's `dense` + `intermediate_act_fn`, as in transformers'
    BertIntermediate, or consecutive entries of an nn.Sequential) is folded into that layer's GEMM
    epilogue and replaced by nn.Identity; a module's `query` / `key` / `value` layers share one
    GEMM over their concatenated weights per input. The returned count is still the number of
    layers swapped.
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
    if fuse:
        _fuse(model)
    return n
