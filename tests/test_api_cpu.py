"""The drop-in Python surface on a CPU-only host: same names, constants, gates and CPU fallbacks as
the reference (golden values recorded from the reference package by tests/golden/make_golden.py)."""
import json
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

import gtx16_fp16 as g

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLD, "reference_cpu.npz")), json.load(open(os.path.join(GOLD, "reference_meta.json")))


def test_public_names_and_constants(golden):
    _, meta = golden
    assert g.__all__ == meta["reference_all"]
    assert g.ROW_SCALE_THRESHOLD == meta["ROW_SCALE_THRESHOLD"]
    assert g.SKINNY_MAX_M == meta["SKINNY_MAX_M"]
    for name in g.__all__:
        assert callable(getattr(g, name))


def test_skinny_config_is_reference_compatible(golden):
    arr, _ = golden
    for N, K, sms, g0, g1, g2, kchunk in arr["skinny_config"]:
        assert g.skinny_config(int(N), int(K), int(sms)) == ((g0, g1, g2), kchunk)


def test_cpu_decisions(golden):
    _, meta = golden
    a = torch.randn(32, 64).half()
    b = torch.randn(64, 48).half()
    assert g.supported(a, b) == meta["supported_cpu"]
    assert g.is_affected() == meta["is_affected"]
    model = nn.Sequential(nn.Linear(512, 1024), nn.GELU(), nn.Linear(1024, 512))
    assert g.patch(model, min_features=256, force=True) == meta["patch_cpu_force"]
    assert g.patch(model) == meta["patch_cpu_noforce"]


def test_mm_t_rejects_bad_out_dtype(golden):
    _, meta = golden
    a = torch.randn(32, 64).half()
    b = torch.randn(64, 48).half()
    with pytest.raises(ValueError) as e:
        g.mm_t(a, b, None, torch.bfloat16)
    assert str(e.value) == meta["mm_t_bad_dtype"]


def test_matmul_cpu_fallback_matches_reference(golden):
    arr, _ = golden
    gen = torch.Generator().manual_seed(3)
    a = torch.randn(32, 64, generator=gen).half()
    b = (torch.randn(64, 48, generator=gen) * 64 ** -0.5).half()
    prev = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        y = g.matmul(a, b)
        y32 = g.matmul(a, b, torch.float32)
    finally:
        torch.set_num_threads(prev)
    assert y.dtype == torch.float16 and y32.dtype == torch.float32
    np.testing.assert_allclose(y.float().numpy(), arr["small_matmul"].astype(np.float32), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(y32.numpy(), arr["small_matmul_f32"], rtol=1e-5, atol=1e-5)


def test_fast_linear_cpu_matches_reference(golden):
    arr, meta = golden
    gen = torch.Generator().manual_seed(0)
    w = torch.randn(768, 1024, generator=gen) * 0.03
    bias = torch.randn(768, generator=gen) * 0.1
    x = torch.randn(2, 8, 1024, generator=gen)
    lin = nn.Linear(1024, 768)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(bias)
    fl = g.FastLinear.from_linear(lin)
    info = meta["fastlinear_cpu"]
    assert sorted(fl.state_dict().keys()) == info["state_dict_keys"]
    assert str(fl.weight_t.dtype) == info["weight_t_dtype"] and str(fl.bias.dtype) == info["bias_dtype"]
    assert fl.extra_repr() == info["extra_repr"]
    assert fl.weight.shape == (768, 1024) and fl.weight.dtype == torch.float16
    with torch.no_grad():
        y = fl(x)
    assert str(y.dtype) == info["dtype"] and list(y.shape) == info["shape"]
    np.testing.assert_allclose(y.numpy(), arr["fastlinear_cpu"], rtol=1e-5, atol=1e-5)


def test_fast_linear_grad_fallback_on_cpu():
    lin = nn.Linear(256, 256)
    fl = g.FastLinear.from_linear(lin)
    x = torch.randn(4, 256, requires_grad=True)
    fl(x).sum().backward()
    assert x.grad is not None


def test_state_dict_round_trip():
    lin = nn.Linear(64, 32)
    fl = g.FastLinear.from_linear(lin)
    fl2 = g.FastLinear(64, 32)
    fl2.load_state_dict(fl.state_dict())
    assert torch.equal(fl2.weight_t, fl.weight_t) and torch.equal(fl2.bias, fl.bias)
    nb = g.FastLinear(64, 32, bias=False)
    assert nb.bias is None and "bias" not in dict(nb.named_buffers())


def test_fast_linear_keeps_its_storage_formats_under_dtype_casts():
    """model.half() / .float() / .double() leave weight_t fp16 and bias fp32 (the formats the kernels
    read); the bias keeps its full fp32 value through the casts."""
    lin = nn.Linear(64, 48)
    with torch.no_grad():
        lin.bias[0] = 1.0 + 2.0 ** -20  # not representable in fp16
    m = g.FastLinear.from_linear(lin)
    seq = nn.Sequential(m, nn.LayerNorm(48))
    for cast in (seq.half, seq.float, seq.double, lambda: seq.to(torch.bfloat16)):
        cast()
        assert m.weight_t.dtype == torch.float16 and m.bias.dtype == torch.float32
        assert m.bias[0].item() == 1.0 + 2.0 ** -20
    seq.half()
    assert seq[1].weight.dtype == torch.float16  # other modules do change
    sd = m.state_dict()
    assert sd["weight_t"].dtype == torch.float16 and sd["bias"].dtype == torch.float32


def test_patch_rejects_unknown_activation_dtype():
    with pytest.raises(ValueError, match="activations"):
        g.patch(nn.Sequential(nn.Linear(8, 8)), force=True, activations=torch.bfloat16)


class _Intermediate(nn.Module):  # the shape of transformers' BertIntermediate
    def __init__(self):
        super().__init__()
        import transformers.activations as ta
        self.dense = g.FastLinear(64, 128)
        self.intermediate_act_fn = ta.ACT2FN["gelu"]

    def forward(self, x):
        return self.intermediate_act_fn(self.dense(x))


class _Attention(nn.Module):
    def __init__(self):
        super().__init__()
        self.query, self.key, self.value = g.FastLinear(64, 64), g.FastLinear(64, 64), g.FastLinear(64, 32)

    def forward(self, x):
        return self.query(x), self.key(x), self.value(x)


def _init(m):
    torch.manual_seed(0)
    for mod in m.modules():
        if isinstance(mod, g.FastLinear):
            with torch.no_grad():
                mod.weight_t.copy_((torch.randn(mod.in_features, mod.out_features) * 0.1).half())
                mod.bias.copy_(torch.randn(mod.out_features))
    return m


def test_fuse_rewrites_gelu_and_groups_qkv_on_cpu():
    """patch(fuse=True)'s rewrite: the exact GELU after `dense` (and after a FastLinear inside an
    nn.Sequential) moves into the layer (activation='gelu', the GELU module becomes Identity); the
    query/key/value layers form one shared-input group; a tanh-approximate GELU is left alone.
    The CPU fallback computes the same function before and after."""
    from gtx16_fp16.linear import _fuse
    inter = _init(_Intermediate())
    seq = _init(nn.Sequential(g.FastLinear(64, 64), nn.GELU(), g.FastLinear(64, 64), nn.GELU(approximate="tanh")))
    att = _init(_Attention())
    model = nn.ModuleDict({"inter": inter, "seq": seq, "att": att})
    x = torch.randn(5, 64)
    with torch.no_grad():
        before = [inter(x), seq(x), *att(x)]
    assert _fuse(model) == (2, 1)
    assert inter.dense.activation == "gelu" and isinstance(inter.intermediate_act_fn, nn.Identity)
    assert seq[0].activation == "gelu" and isinstance(seq[1], nn.Identity)
    assert seq[2].activation is None and isinstance(seq[3], nn.GELU)
    assert att.query._group is att.key._group is att.value._group is not None
    assert "fused_group=2/3" in repr(att.value)
    with torch.no_grad():
        after = [inter(x), seq(x), *att(x)]
    for a, b in zip(before, after):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)
    assert _fuse(model) == (0, 0)  # idempotent
