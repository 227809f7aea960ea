"""``jaxml_b200.nn`` building blocks on the GPU against the oracle's restatement of the reference ops
(``oracle/jaxml_oracle.py``: rmsnorm / layernorm / gemma_rmsnorm, dense, apply_rope, mha)."""
import pytest
import torch

from jaxml_b200 import nn
from jaxml_b200.cache import KVCache
from jaxml_b200.config import ModelConfig
from oracle import jaxml_oracle as O

pytestmark = pytest.mark.gpu


def _close_bf16(y, ref):
    """within one bfloat16 rounding of the reference (plus float32 accumulation-order noise)"""
    y, ref = y.float().cpu(), ref.float().cpu()
    bad = (y - ref).abs() > ref.abs() * 2.0 ** -7 + 1e-3
    assert not bad.any(), ((y - ref).abs().max().item(), int(bad.sum()))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 1000, 4096])
def test_norms_match_oracle(dtype, d):
    g = torch.Generator().manual_seed(d)
    x = (3 * torch.randn(3, 5, d, generator=g)).to(dtype)
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(dtype)
    b = (0.1 * torch.randn(d, generator=g)).to(dtype)
    cases = [(nn.RMSNorm(hidden_size=d, eps=1e-5, dtype=dtype), {"weight": w}, O.rmsnorm(x, w, 1e-5)),
             (nn.GemmaRMSNorm(hidden_size=d, eps=1e-6, dtype=dtype), {"weight": w}, O.gemma_rmsnorm(x, w, 1e-6)),
             (nn.LayerNorm(hidden_size=d, eps=1e-5, dtype=dtype), {"weight": w, "bias": b},
              O.layernorm(x, w, b, 1e-5))]
    for m, p, ref in cases:
        y = m.apply({"params": {k: t.cuda() for k, t in p.items()}}, x.cuda())
        assert y.dtype == dtype and y.shape == x.shape
        if dtype == torch.float32:
            torch.testing.assert_close(y.cpu(), ref, rtol=1e-5, atol=1e-5)
        else:
            _close_bf16(y, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [100, 4096])
def test_embed_gather_is_exact(dtype, d):
    e = nn.Embed(num_embeddings=50, features=d, dtype=dtype)
    v = e.init(0, torch.tensor([1]))
    ids = torch.tensor([[0, 7, 49], [3, 3, 12]])
    y = e.apply(v, ids.cuda())
    assert y.shape == (2, 3, d) and y.dtype == dtype
    assert torch.equal(y.cpu(), v["params"]["embedding"].to(dtype).cpu()[ids])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,features,axis", [((2, 3, 256), (4, 16), -1), ((2, 100, 256), 384, -1),
                                                  ((2, 3, 4, 64), 200, (-2, -1))])
def test_dense_general_matches_oracle(dtype, shape, features, axis):
    nin = 1 if isinstance(axis, int) else len(axis)
    axes = tuple(f"a{i}" for i in range(nin + (1 if isinstance(features, int) else len(features))))
    m = nn.DenseGeneral(features=features, axis=axis, dtype=dtype, kernel_axes=axes, use_bias=True)
    x = torch.randn(*shape, generator=torch.Generator().manual_seed(1))
    v = m.init(3, x)
    v["params"]["bias"] = 0.5 * torch.randn(v["params"]["bias"].shape, generator=torch.Generator().manual_seed(2)).cuda()
    y = m.apply(v, x.cuda())
    ref = O.dense(x, v["params"]["kernel"].cpu(), v["params"]["bias"].cpu(), dtype, n_in=nin)
    assert y.shape == ref.shape and y.dtype == dtype
    if dtype == torch.float32:
        torch.testing.assert_close(y.cpu(), ref, rtol=1e-4, atol=1e-4)
    else:
        _close_bf16(y, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("hd,pct", [(128, 1.0), (64, 0.25), (256, 1.0)])
def test_apply_rotary_pos_emb_is_exact(dtype, hd, pct):
    g = torch.Generator().manual_seed(hd)
    B, S = 2, 7
    q = torch.randn(B, S, 4, hd, generator=g).to(dtype)
    k = torch.randn(B, S, 2, hd, generator=g).to(dtype)
    cos, sin = O.rope_tables(hd, pct, 10000.0, 1.0, 64, dtype)
    for pos in (torch.randint(0, 64, (B, S), generator=g), torch.arange(S)[None]):
        qo, ko = nn.RotaryEmbedding.apply_rotary_pos_emb(q.cuda(), k.cuda(), cos.cuda(), sin.cuda(), pos.cuda())
        rq, rk = O.apply_rope(q, k, cos, sin, pos.expand(B, S))
        assert torch.equal(qo.cpu(), rq) and torch.equal(ko.cpu(), rk)


def _cfg():
    return ModelConfig(head_dim=32, hidden_size=128, num_heads=4, num_kv_heads=2, num_layers=1,
                       max_position_embeddings=256, vocab_size=100, norm_eps=1e-5)


def _oracle_attention(p, x, cos, sin, pos, mask, cfg, dtype, window=None):
    q = O.dense(x, p["q_proj"]["kernel"].cpu(), None, dtype)
    k = O.dense(x, p["k_proj"]["kernel"].cpu(), None, dtype)
    v = O.dense(x, p["v_proj"]["kernel"].cpu(), None, dtype)
    q, k = O.apply_rope(q, k, cos, sin, pos)
    n_rep = cfg.num_heads // cfg.num_key_value_heads
    out = O.mha(q, O.repeat_kv(k, n_rep), O.repeat_kv(v, n_rep), mask, True, window, cfg.attn_scale)
    return O.dense(out.reshape(out.shape[:2] + (-1,)), p["o_proj"]["kernel"].cpu(), None, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_attention_with_rope_prefill_and_decode_match_oracle(dtype):
    """Prefill of a right-padded batch into a KVCache, then one decode step, against the oracle's full
    attention over the same tokens."""
    cfg = _cfg()
    B, S = 2, 9
    m = nn.AttentionWithRoPE(config=cfg, dtype=dtype, weight_dtype=dtype)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(B, S + 1, cfg.hidden_size, generator=g).to(dtype)
    v = m.init(0, x[:, :S])
    rope = nn.RotaryEmbedding(dim=cfg.head_dim, max_length=cfg.max_position_embeddings, dtype=dtype)
    rv = rope.init(0, x)
    cos, sin = rope.apply(rv, x.cuda())
    mask = torch.ones(B, S, dtype=torch.bool)
    mask[1, 6:] = False                                   # row 1 has 6 valid prompt tokens
    cache = KVCache.init(32, dtype=dtype)
    out = m.apply(v, x[:, :S].cuda(), (cos, sin), attention_mask=mask.cuda(), kv_cache=cache)
    ref = _oracle_attention(v["params"], x[:, :S], cos.cpu(), sin.cpu(), torch.arange(S)[None].expand(B, S),
                            mask, cfg, dtype)
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(out.attention_output.cpu().float(), ref.float(), **tol)
    # decode: the next token of each row lands at its own next position
    cache = out.kv_cache
    step = m.apply(v, x[:, S:].cuda(), (cos, sin), kv_cache=cache)
    for b, n in ((0, S), (1, 6)):
        xs = torch.cat([x[b:b + 1, :n], x[b:b + 1, S:]], dim=1)
        full = _oracle_attention(v["params"], xs, cos.cpu(), sin.cpu(), torch.arange(n + 1)[None],
                                 torch.ones(1, n + 1, dtype=torch.bool), cfg, dtype)
        torch.testing.assert_close(step.attention_output[b, 0].cpu().float(), full[0, -1].float(), **tol)
    assert step.kv_cache.pos_id[:, 0].tolist() == [S, 6]


def test_attention_without_cache_and_sliding_window_matches_oracle():
    cfg = _cfg()
    B, S = 2, 12
    m = nn.Attention(config=cfg, dtype=torch.float32)
    x = torch.randn(B, S, cfg.hidden_size, generator=torch.Generator().manual_seed(8))
    v = m.init(1, x)
    for window in (None, 4):
        out = m.apply(v, x.cuda(), sliding_window=window)
        p = v["params"]
        q = O.dense(x, p["q_proj"]["kernel"].cpu(), None, torch.float32)
        k = O.dense(x, p["k_proj"]["kernel"].cpu(), None, torch.float32)
        vv = O.dense(x, p["v_proj"]["kernel"].cpu(), None, torch.float32)
        o = O.mha(q, O.repeat_kv(k, 2), O.repeat_kv(vv, 2), torch.ones(B, S, dtype=torch.bool), True, window,
                  cfg.attn_scale)
        ref = O.dense(o.reshape(B, S, -1), p["o_proj"]["kernel"].cpu(), None, torch.float32)
        torch.testing.assert_close(out.attention_output.cpu(), ref, rtol=1e-4, atol=1e-4)


def _attn1(**kw):
    base = dict(head_dim=1, hidden_size=1, num_heads=1, num_layers=1, max_position_embeddings=8, vocab_size=8,
                attn_scale=1.0, use_rope=False)
    base.update(kw)
    return nn.Attention(ModelConfig(**base))


def test_mha_known_answers():
    """``Attention.mha`` with weights (the reference's ``tests/test_attention.py:108-240`` cases): a decode
    sliding window without and with a padded cache mask, an all-masked row, an integer mask."""
    attn = _attn1()
    q = torch.zeros(1, 1, 1, 1, device="cuda")
    out, w = attn.apply({}, q, torch.zeros(1, 5, 1, 1, device="cuda"),
                        torch.arange(5.0, device="cuda").reshape(1, 5, 1, 1) * 10, sliding_window=2,
                        output_attentions=True, method=nn.Attention.mha)
    assert torch.allclose(out.cpu(), torch.tensor([[[[35.0]]]]))
    assert torch.allclose(w.cpu(), torch.tensor([[[[0.0, 0.0, 0.0, 0.5, 0.5]]]]))
    mask = torch.tensor([[True, True, True, True, False, False, False, False]], device="cuda")
    out, w = attn.apply({}, q, torch.zeros(1, 8, 1, 1, device="cuda"),
                        torch.arange(8.0, device="cuda").reshape(1, 8, 1, 1) * 10, attention_mask=mask,
                        sliding_window=2, output_attentions=True, method="mha")
    assert torch.allclose(out.cpu(), torch.tensor([[[[25.0]]]]))
    assert torch.allclose(w.cpu(), torch.tensor([[[[0.0, 0.0, 0.5, 0.5, 0.0, 0.0, 0.0, 0.0]]]]))
    out, w = attn.apply({}, q, torch.zeros(1, 2, 1, 1, device="cuda"),
                        torch.tensor([[[[2.0]], [[4.0]]]], device="cuda"),
                        attention_mask=torch.tensor([[False, False]], device="cuda"), output_attentions=True,
                        method=nn.Attention.mha)
    assert torch.isfinite(out).all() and torch.allclose(out.cpu(), torch.tensor([[[[3.0]]]]))
    assert torch.allclose(w.cpu(), torch.tensor([[[[0.5, 0.5]]]]))
    v = torch.arange(3.0, device="cuda").reshape(1, 3, 1, 1)
    o1, w1 = attn.apply({}, q, torch.zeros(1, 3, 1, 1, device="cuda"), v,
                        attention_mask=torch.tensor([[1, 1, 0]], dtype=torch.int32), output_attentions=True,
                        method=nn.Attention.mha)
    o2, w2 = attn.apply({}, q, torch.zeros(1, 3, 1, 1, device="cuda"), v,
                        attention_mask=torch.tensor([[True, True, False]]), output_attentions=True,
                        method=nn.Attention.mha)
    assert torch.equal(o1, o2) and torch.equal(w1, w2)
    o3, w3 = attn.apply({}, q, torch.zeros(1, 3, 1, 1, device="cuda"), v, method=nn.Attention.mha)
    assert w3 is None and tuple(o3.shape) == (1, 1, 1, 1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("S,T,causal,window,padded", [(6, 6, True, None, False), (6, 6, True, 3, True),
                                                      (1, 9, True, None, True), (1, 9, True, 4, True),
                                                      (1, 9, False, 4, False), (4, 4, False, None, True)])
def test_mha_matches_oracle(dtype, S, T, causal, window, padded):
    """``Attention.mha`` output and weights against the oracle's ``mha`` (prefill and decode shapes,
    causal, sliding window, right-padded masks)."""
    H, hd = 4, 16
    attn = _attn1(head_dim=hd, hidden_size=H * hd, num_heads=H, attn_scale=hd ** -0.5)
    g = torch.Generator().manual_seed(S * 31 + T)
    q = torch.randn(2, S, H, hd, generator=g).to(dtype)
    k = torch.randn(2, T, H, hd, generator=g).to(dtype)
    v = torch.randn(2, T, H, hd, generator=g).to(dtype)
    mask = None
    if padded:
        mask = torch.ones(2, T, dtype=torch.bool)
        mask[1, T - 2:] = False
    out, w = attn.apply({}, q.cuda(), k.cuda(), v.cuda(), attention_mask=None if mask is None else mask.cuda(),
                        causal=causal, sliding_window=window, output_attentions=True, method=nn.Attention.mha)
    ref, ref_w = O.mha(q, k, v, mask, causal, window, hd ** -0.5, return_weights=True)
    assert out.dtype == dtype and tuple(w.shape) == (2, H, S, T)
    if dtype == torch.float32:
        torch.testing.assert_close(out.cpu(), ref, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(w.cpu(), ref_w, rtol=1e-5, atol=1e-6)
    else:
        _close_bf16(out, ref)
        _close_bf16(w, ref_w)
