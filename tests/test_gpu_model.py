"""Model-level GPU checks: BERT-base patched with FastLinear against the unpatched fp32 model
(BASELINE config 5 at a reduced batch), and the column-sharded matmul on one GPU."""
import copy

import pytest
import torch

import gtx16_fp16 as g
from gtx16_fp16.dist import ShardedMatmul, shard_bounds

pytestmark = pytest.mark.gpu


def test_bert_base_patched_cosine(cuda_ok):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.BertConfig(vocab_size=30522, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                                  intermediate_size=3072, hidden_act="gelu", max_position_embeddings=512,
                                  attn_implementation="sdpa")
    torch.manual_seed(0)
    model = transformers.BertModel(cfg).eval()
    ref_model = copy.deepcopy(model).cuda()
    model = model.cuda()
    assert g.patch(model, force=True) == 73  # 12 x (q, k, v, attn-out, intermediate, output) + pooler
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30522, (16, 256), generator=gen).cuda()
    mask = torch.ones_like(ids)
    with torch.no_grad():
        ref = ref_model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0]
        got = model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0]
    ref = torch.nn.functional.normalize(ref.float(), dim=-1)
    got = torch.nn.functional.normalize(got.float(), dim=-1)
    cos = (ref * got).sum(-1)
    assert cos.min().item() >= 0.9999, cos.min().item()


def test_bert_base_patched_cosine_full_batch(cuda_ok):
    """BASELINE config 5 at its full size: 256 sequences x 256 tokens through the patched model
    (73 FastLinear layers, fp32 activations), CLS cosine >= 0.9999 against the unpatched fp32 model
    for every one of the 256 sequences."""
    transformers = pytest.importorskip("transformers")
    cfg = transformers.BertConfig(vocab_size=30522, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                                  intermediate_size=3072, hidden_act="gelu", max_position_embeddings=512,
                                  attn_implementation="sdpa")
    torch.manual_seed(0)
    model = transformers.BertModel(cfg).eval()
    ref_model = copy.deepcopy(model).cuda()
    model = model.cuda()
    assert g.patch(model, force=True) == 73
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30522, (256, 256), generator=gen).cuda()
    mask = torch.ones_like(ids)
    with torch.no_grad():
        ref = ref_model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0]
        got = model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0]
    assert torch.isfinite(got).all()
    cos = (torch.nn.functional.normalize(ref.float(), dim=-1) * torch.nn.functional.normalize(got.float(), dim=-1)).sum(-1)
    assert cos.numel() == 256
    assert cos.min().item() >= 0.9999, cos.min().item()


def test_gemm_16384_cubed_sampled_rows_vs_fp64(cuda_ok):
    """BASELINE config 3's 16384^3 on one GPU (the single-pass CTA-pair kernel), A ~ N(0,1),
    B ~ N(0, 1/sqrt(K)), fp16 out: 256 seeded rows of the output against fp64, norm-wise and
    component-wise within 1e-3, no inf/NaN anywhere in the 16384 x 16384 output."""
    from _tol import GEMM_NORM, GEMM_RTOL
    M = K = N = 16384
    gen = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(M, K, device="cuda", generator=gen).half()
    b = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
    y = g.matmul(a, b)
    assert y.dtype == torch.float16 and y.shape == (M, N)
    assert torch.isfinite(y).all()
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(1))[:256].sort().values.cuda()
    a_s = a[rows].double()
    ys = y[rows].double()
    d2 = r2 = 0.0
    comp = 0.0
    for c0 in range(0, N, 2048):
        p = b[:, c0:c0 + 2048].double()
        ref = a_s @ p
        mag = a_s.abs() @ p.abs()
        d = ys[:, c0:c0 + 2048] - ref
        d2 += float((d * d).sum())
        r2 += float((ref * ref).sum())
        comp = max(comp, float((d.abs() / mag).max()))
    norm = (d2 / r2) ** 0.5
    assert norm <= GEMM_NORM, norm
    assert comp <= GEMM_RTOL, comp
    # bitwise reproducible at this size too
    assert torch.equal(g.matmul(a, b)[rows], y[rows])


def test_bert_base_fp16_activations_mode(cuda_ok):
    """patch(..., activations=torch.float16): the whole model runs with fp16 activations (opt-in;
    the reference's FastLinear keeps fp32 activations). FastLinear keeps weight_t fp16 and bias
    fp32 through model.half(); the CLS embeddings stay close to the unpatched fp32 model's."""
    transformers = pytest.importorskip("transformers")
    cfg = transformers.BertConfig(vocab_size=30522, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                                  intermediate_size=3072, hidden_act="gelu", max_position_embeddings=512,
                                  attn_implementation="sdpa")
    torch.manual_seed(0)
    model = transformers.BertModel(cfg).eval()
    ref_model = copy.deepcopy(model).cuda()
    model = model.cuda()
    assert g.patch(model, force=True, activations=torch.float16) == 73
    fl = model.encoder.layer[0].attention.self.query
    assert isinstance(fl, g.FastLinear) and fl.weight_t.dtype == torch.float16 and fl.bias.dtype == torch.float32
    assert model.embeddings.word_embeddings.weight.dtype == torch.float16
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30522, (16, 256), generator=gen).cuda()
    mask = torch.ones_like(ids)
    with torch.no_grad():
        ref = ref_model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0]
        got = model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0]
    assert got.dtype == torch.float16 and torch.isfinite(got).all()
    ref = torch.nn.functional.normalize(ref.float(), dim=-1)
    got = torch.nn.functional.normalize(got.float(), dim=-1)
    cos = (ref * got).sum(-1)
    assert cos.min().item() >= 0.9999, cos.min().item()  # measured 0.9999987 on B200


@pytest.mark.parametrize("half", [False, True])
def test_bert_base_fused_patch(cuda_ok, half):
    """patch(..., fuse=True): the 12 intermediate GELUs fold into their GEMMs and each attention's
    query/key/value share one GEMM. Same CLS embeddings as the unfused patch (up to rounding) and
    the fp32 model's within cosine 0.9999; in fp32 mode 12 x 2 fewer rowscale passes and 12 fewer
    GELU launches."""
    transformers = pytest.importorskip("transformers")
    cfg = transformers.BertConfig(vocab_size=30522, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                                  intermediate_size=3072, hidden_act="gelu", max_position_embeddings=512,
                                  attn_implementation="sdpa")
    torch.manual_seed(0)
    model = transformers.BertModel(cfg).eval()
    ref_model = copy.deepcopy(model).cuda()
    plain = copy.deepcopy(model).cuda()
    model = model.cuda()
    act = torch.float16 if half else None
    assert g.patch(plain, force=True, activations=act) == 73
    assert g.patch(model, force=True, activations=act, fuse=True) == 73
    layer = model.encoder.layer[0]
    assert layer.intermediate.dense.activation == "gelu"
    assert isinstance(layer.intermediate.intermediate_act_fn, torch.nn.Identity)
    assert layer.attention.self.query._group is layer.attention.self.value._group is not None
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30522, (8, 256), generator=gen).cuda()
    mask = torch.ones_like(ids)
    with torch.no_grad():
        ref = ref_model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0].float()
        unf = plain(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0].float()
        got = model(input_ids=ids, attention_mask=mask).last_hidden_state[:, 0].float()
    torch.testing.assert_close(got, unf, rtol=1e-2 if half else 1e-4, atol=1e-2 if half else 1e-4)
    cos = (torch.nn.functional.normalize(ref, dim=-1) * torch.nn.functional.normalize(got, dim=-1)).sum(-1)
    assert cos.min().item() >= 0.9999, cos.min().item()


@pytest.mark.parametrize("M,K,N", [(512, 1024, 2048), (300, 512, 776)])
def test_sharded_matmul_single_gpu(cuda_ok, M, K, N):
    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda").half()
    w = (torch.randn(K, N, device="cuda") * K ** -0.5).half()
    n0, n1 = shard_bounds(N, 1, 0)
    sm = ShardedMatmul(w[:, n0:n1].contiguous(), N)
    y = sm(a)
    assert torch.equal(y, g.mm_t(a, w, None, torch.float16))
