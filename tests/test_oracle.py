"""Pins the CPU oracle (oracle/g16_oracle.c, oracle/cpu_path.py) before it is trusted as the checker.

Evidence used:
  * golden vectors recorded from the reference package itself (tests/golden/make_golden.py):
    skinny_config, the CPU matmul fallback of BASELINE config 1, the FastLinear CPU fallback;
  * the reference test suite's known answers (tests/test_correctness.py:103-109 and 112-126);
  * the error figures the reference publishes for its kernels (README.md:33-38), reproduced by the
    restatement on the same input distribution (randn * 0.5);
  * exactness of the emulated fp16 FMA against rational arithmetic.
The bit-exact pin of the restatement against the reference's own kernels running on a B200 is in
tests/test_gpu_reference.py.
"""
import json
import os
from fractions import Fraction

import numpy as np
import pytest
import torch

import oracle
from oracle import cpu_path

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def golden():
    arr = np.load(os.path.join(GOLD, "reference_cpu.npz"))
    meta = json.load(open(os.path.join(GOLD, "reference_meta.json")))
    return arr, meta


def config1_inputs(M=1024, K=1024, N=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).half()
    b = (torch.randn(K, N, generator=g) * K ** -0.5).half()
    return a, b


def test_skinny_config_matches_reference(golden):
    arr, _ = golden
    for N, K, sms, g0, g1, g2, kchunk in arr["skinny_config"]:
        grid, kc = oracle.skinny_config(int(N), int(K), int(sms))
        assert grid == (g0, g1, g2) and kc == kchunk, (N, K, sms)


def test_cpu_matmul_path_matches_reference_golden(golden):
    arr, meta = golden
    prev = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        a, b = config1_inputs()
        y = cpu_path.matmul(a, b)
        a_s, b_s = config1_inputs(32, 64, 48, seed=3)
        ys = cpu_path.matmul(a_s, b_s)
        ys32 = cpu_path.matmul(a_s, b_s, torch.float32)
    finally:
        torch.set_num_threads(prev)
    assert str(y.dtype) == meta["config1"]["dtype"]
    np.testing.assert_allclose(y[:8].float().numpy(), arr["config1_rows0_7"].astype(np.float32), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(ys.float().numpy(), arr["small_matmul"].astype(np.float32), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(ys32.numpy(), arr["small_matmul_f32"], rtol=1e-5, atol=1e-5)
    # config 1 on the CPU path stays within the GEMM tolerance of the fp64 product
    ref = oracle.fp64_mm(a.numpy(), b.numpy())
    assert oracle.rel_err(y.float().numpy(), ref) < 1e-3


def test_cpu_linear_fallback_matches_reference_golden(golden):
    arr, _ = golden
    g = torch.Generator().manual_seed(0)
    w = torch.randn(768, 1024, generator=g) * 0.03
    bias = torch.randn(768, generator=g) * 0.1
    x = torch.randn(2, 8, 1024, generator=g)
    w_t = w.t().contiguous().half()
    y = cpu_path.mm_t_fp32(x.reshape(-1, 1024), w_t, bias).reshape(2, 8, 768)
    np.testing.assert_allclose(y.numpy(), arr["fastlinear_cpu"], rtol=1e-5, atol=1e-5)


def test_known_answer_large_outputs():
    # tests/test_correctness.py:103-109: 16 * 16 * 4096 = 1,048,576 exactly, above fp16 max
    x = np.full((8, 4096), 16, np.float16)
    w = np.full((4096, 8), 16, np.float16)
    y = oracle.ref_hgemm(x, w)
    assert np.all(y == 16 * 16 * 4096)
    ym = oracle.ref_mm_t(x.astype(np.float32), w, None, np.float32)
    assert np.all(np.isfinite(ym)) and abs(ym[0, 0] - 1048576) / 1048576 < 1e-3


@pytest.mark.parametrize("M", [1, 5, 64, 300])
@pytest.mark.parametrize("in16", [False, True])
def test_massive_activations_oracle(M, in16):
    # tests/test_correctness.py:112-126 restated on the oracle (reduced K to keep the CPU test fast)
    rng = np.random.default_rng(1)
    K, N = 3072, 64
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[:, 7] = 60000.0 if in16 else 179940.0
    x[0, 100] = -50000.0 if in16 else -120000.0
    if in16:
        x = x.astype(np.float16)
    w = (rng.standard_normal((K, N)) * 0.3).astype(np.float16)
    y = oracle.ref_mm_t(x, w, None, np.float32)
    assert np.all(np.isfinite(y))
    assert oracle.rel_err(y, oracle.fp64_mm(x, w)) < 2e-3


def test_published_error_figures_reproduced():
    # README.md:36-38: hybrid accumulation gives 6.0e-4 .. 6.1e-4 norm-wise (randn*0.5 inputs);
    # README.md:33-35: skinny path 2.2e-7 .. 3.2e-7 against an fp32 reference.
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((64, 1024)) * 0.5).astype(np.float16)
    w = (rng.standard_normal((1024, 96)) * 0.5).astype(np.float16)
    e = oracle.rel_err(oracle.ref_hgemm(x, w), x.astype(np.float32) @ w.astype(np.float32))
    assert 5.0e-4 < e < 7.2e-4, e
    x1 = (rng.standard_normal((1, 4096)) * 0.5).astype(np.float16)
    w1 = (rng.standard_normal((4096, 512)) * 0.5).astype(np.float16)
    es = oracle.rel_err(oracle.ref_skinny(x1, w1), x1.astype(np.float32) @ w1.astype(np.float32))
    assert 5e-8 < es < 1e-6, es


def _all_f16_positive():
    return np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)


def _rne16(fr: Fraction, table):
    s = -1.0 if fr < 0 else 1.0
    a = abs(fr)
    if a >= Fraction(65520):
        return s * np.inf
    i = int(np.searchsorted(table, float(a)))
    cands = [table[j] for j in (i - 1, i, i + 1) if 0 <= j < len(table)]
    best = min(cands, key=lambda v: (abs(Fraction(v) - a), int(np.float16(v).view(np.uint16)) & 1))
    return s * best


def test_fp16_fma_chain_is_exact():
    table = _all_f16_positive()
    rng = np.random.default_rng(0)
    for _ in range(400):
        v = [np.float16(rng.standard_normal() * rng.choice([1e-4, 1.0, 30.0])) for _ in range(4)]
        A = np.array([[v[0], v[2]]], np.float16)
        B = np.array([[v[1]], [v[3]]], np.float16)
        got = float(oracle.ref_hgemm_accf(A, B)[0, 0])
        c = _rne16(Fraction(float(v[0])) * Fraction(float(v[1])), table)
        exp = _rne16(Fraction(float(v[2])) * Fraction(float(v[3])) + Fraction(float(c)), table)
        assert got == exp


def test_rowscale_scale_rule():
    # S = 2^ceil(log2(amax/1024)) when amax > 1024 (kernels.py:242), exact at powers of two
    amax = np.array([0.5, 1024.0, 1024.0001, 2048.0, 2049.0, 65504.0, 179940.0, 3.0e38], np.float32)
    x = np.zeros((len(amax), 8), np.float32)
    x[:, 3] = -amax
    y, S = oracle.ref_rowscale(x)
    expect = [1, 1, 2, 2, 4, 64, 256, 2.0 ** 118]
    np.testing.assert_array_equal(S, np.array(expect, np.float32))
    np.testing.assert_array_equal(y[:, 3].astype(np.float32), (-amax / S).astype(np.float16).astype(np.float32))
