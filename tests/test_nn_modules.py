"""CPU checks of the ``jaxml_b200.nn`` building blocks: field and input validation (the reference's
``tests/test_modules.py`` / ``test_rope.py`` cases), parameter names and shapes, RoPE tables, and that
``apply`` refuses CPU tensors (there is no CPU path)."""
import numpy as np
import pytest
import torch

from jaxml_b200 import nn
from jaxml_b200.cache import KVCache
from jaxml_b200.config import ModelConfig
from oracle import jaxml_oracle as O


def test_norm_fields_and_params():
    v = nn.RMSNorm(hidden_size=4).init(0, torch.ones(2, 4))
    assert list(v["params"]) == ["weight"] and torch.equal(v["params"]["weight"].cpu(), torch.ones(4))
    v = nn.LayerNorm(hidden_size=4).init(0, torch.ones(2, 4))
    assert sorted(v["params"]) == ["bias", "weight"]
    v = nn.LayerNorm(hidden_size=4, use_bias=False).init(0, torch.ones(2, 4))
    assert list(v["params"]) == ["weight"]
    v = nn.GemmaRMSNorm(hidden_size=4).init(0, torch.ones(1, 4))
    assert torch.equal(v["params"]["weight"].cpu(), torch.zeros(4))


@pytest.mark.parametrize("kw,exc,msg", [
    (dict(hidden_size=0), ValueError, "hidden_size must be positive"),
    (dict(hidden_size=True), TypeError, "hidden_size must be an integer"),
    (dict(hidden_size=4, eps=0.0), ValueError, "eps must be positive"),
    (dict(hidden_size=4, upcast=1), TypeError, "upcast must be a boolean"),
    (dict(hidden_size=4, dtype=None), TypeError, "dtype must be a valid"),
])
def test_norm_field_validation(kw, exc, msg):
    with pytest.raises(exc, match=msg):
        nn.RMSNorm(**kw).init(0, torch.ones(1, 4))


def test_norm_input_validation():
    m = nn.RMSNorm(hidden_size=4)
    with pytest.raises(ValueError, match="hidden dimension mismatch"):
        m.init(0, torch.ones(2, 3))
    with pytest.raises(TypeError, match="floating point"):
        m.init(0, torch.ones(2, 4, dtype=torch.int32))
    with pytest.raises(ValueError, match="at least one dimension"):
        m.init(0, torch.tensor(1.0))
    with pytest.raises(ValueError, match="finite"):
        m.init(0, torch.tensor([[1.0, float("nan"), 0.0, 0.0]]))
    with pytest.raises(ValueError, match="empty axes"):
        m.init(0, torch.ones(0, 4))


def test_layernorm_use_bias_must_be_bool():
    with pytest.raises(TypeError, match="use_bias must be a boolean"):
        nn.LayerNorm(hidden_size=4, use_bias=1).init(0, torch.ones(1, 4))


def test_embed_validation_and_params():
    e = nn.Embed(num_embeddings=np.int64(8), features=np.int64(4))
    v = e.init(0, torch.tensor([0, 1]))
    assert v["params"]["embedding"].shape == (8, 4)
    with pytest.raises(ValueError, match="non-negative"):
        e.init(0, torch.tensor([-1]))
    with pytest.raises(ValueError, match="less than num_embeddings=8"):
        e.init(0, torch.tensor([8]))
    with pytest.raises(ValueError, match="integer or unsigned integer"):
        e.init(0, torch.tensor([1.0]))
    with pytest.raises(ValueError, match="at least one token id"):
        e.init(0, torch.zeros(0, dtype=torch.int64))
    with pytest.raises(TypeError, match="one_hot must be a boolean"):
        nn.Embed(num_embeddings=8, features=4, one_hot=1).init(0, torch.tensor([1]))
    with pytest.raises(ValueError, match="num_embeddings must be positive"):
        nn.Embed(num_embeddings=0, features=4).init(0, torch.tensor([0]))
    with pytest.raises(TypeError, match="unexpected field"):
        nn.Embed(num_embeddings=8, features=4, bogus=1)


def test_dense_general_kernel_shapes_and_init_scale():
    d = nn.DenseGeneral(features=(4, 16), axis=-1, kernel_axes=("embed", "heads", "head_states"), use_bias=True)
    v = d.init(1, torch.randn(2, 3, 32))
    assert v["params"]["kernel"].shape == (32, 4, 16) and v["params"]["bias"].shape == (4, 16)
    # variance_scaling(1, fan_in, truncated_normal): std 1/sqrt(32)
    assert abs(float(v["params"]["kernel"].float().std()) - 32 ** -0.5) < 0.02
    # two contracted axes
    d2 = nn.DenseGeneral(features=8, axis=(-2, -1), kernel_axes=("heads", "head_states", "embed"))
    assert d2.init(0, torch.randn(2, 3, 4, 16))["params"]["kernel"].shape == (4, 16, 8)
    # same key -> same values
    a = d.init(5, torch.randn(2, 3, 32))["params"]["kernel"]
    b = d.init(5, torch.randn(2, 3, 32))["params"]["kernel"]
    assert torch.equal(a, b)


@pytest.mark.parametrize("kw,x,exc,msg", [
    (dict(features=0, kernel_axes=("a", "b")), torch.ones(2, 4), ValueError, "features values must be positive"),
    (dict(features=4, axis=3, kernel_axes=("a", "b")), torch.ones(2, 4), ValueError, "out of bounds"),
    (dict(features=4, axis=(-1, 1), kernel_axes=("a", "b", "c")), torch.ones(2, 4), ValueError, "unique"),
    (dict(features=4, kernel_axes=("a", "b")), torch.ones(2, 4, dtype=torch.int32), TypeError, "floating point"),
    (dict(features=4), torch.ones(2, 4), ValueError, "Kernel axes must be specified"),
    (dict(features=4, kernel_axes="ab"), torch.ones(2, 4), TypeError, "not a string"),
])
def test_dense_general_validation(kw, x, exc, msg):
    with pytest.raises(exc, match=msg):
        nn.DenseGeneral(**kw).init(0, x)


def test_rotary_tables_match_the_oracle_restatement():
    r = nn.RotaryEmbedding(dim=64, max_length=128, base=500000.0, dtype=torch.bfloat16)
    v = r.init(0, torch.ones(1, 4, 64))
    cos, sin = O.rope_tables(64, 1.0, 500000.0, 1.0, 128, torch.bfloat16)
    assert torch.equal(v["cache"]["cos_cached"].cpu(), cos) and torch.equal(v["cache"]["sin_cached"].cpu(), sin)
    c, s = r.apply(v, torch.ones(1, 4, 64, dtype=torch.bfloat16))
    assert c.shape == (128, 64) and c.dtype == torch.bfloat16
    with pytest.raises(ValueError, match="only cover max_length=128"):
        r.apply(v, torch.ones(1, 4, 64), seq_len=129)
    # partial rotary (GPT-NeoX 0.25)
    r2 = nn.RotaryEmbedding(dim=64, rotary_pct=0.25, max_length=16)
    assert r2.init(0, torch.ones(1, 2, 64))["cache"]["cos_cached"].shape == (16, 16)


@pytest.mark.parametrize("kw,msg", [
    (dict(dim=0), "dim must be positive"),
    (dict(dim=8, max_length=0), "max_length must be positive"),
    (dict(dim=8, base=0.0), "base must be positive"),
    (dict(dim=8, rope_scale=0.5), "rope scale"),
    (dict(dim=8, rotary_pct=1.5), "rotary_pct"),
    (dict(dim=6, rotary_pct=0.5), "odd"),
    (dict(dim=2, rotary_pct=0.1), "less than or equal to 0"),
])
def test_rotary_field_validation(kw, msg):
    with pytest.raises(ValueError, match=msg):
        nn.RotaryEmbedding(**kw).init(0, torch.ones(1, 2, 8))


def test_apply_rotary_pos_emb_validation():
    q = torch.ones(1, 2, 2, 8)
    cos, sin = O.rope_tables(8, 1.0, 10000.0, 1.0, 4, torch.float32)
    f = nn.RotaryEmbedding.apply_rotary_pos_emb
    with pytest.raises(ValueError, match="4D"):
        f(q[0], q, cos, sin, torch.zeros(1, 2, dtype=torch.int32))
    with pytest.raises(ValueError, match="within rotary table length 4"):
        f(q, q, cos, sin, torch.tensor([[0, 4]]))
    with pytest.raises(ValueError, match="non-negative"):
        f(q, q, cos, sin, torch.tensor([[0, -1]]))
    with pytest.raises(TypeError, match="integer positions"):
        f(q, q, cos, sin, torch.tensor([[0.0, 1.0]]))
    with pytest.raises(ValueError, match="broadcastable"):
        f(q, q, cos, sin, torch.zeros(2, 3, dtype=torch.int32))
    with pytest.raises(ValueError, match="cannot exceed"):
        f(q, q, torch.ones(4, 16), torch.ones(4, 16), torch.zeros(1, 2, dtype=torch.int32))


def _cfg(**kw):
    args = dict(head_dim=16, hidden_size=64, num_heads=4, num_kv_heads=2, num_layers=1, max_position_embeddings=64,
                vocab_size=100)
    return ModelConfig(**(args | kw))


def test_attention_params_and_validation():
    a = nn.AttentionWithRoPE(config=_cfg(use_bias=True))
    v = a.init(0, torch.randn(2, 5, 64))
    p = v["params"]
    assert p["q_proj"]["kernel"].shape == (64, 4, 16) and p["k_proj"]["kernel"].shape == (64, 2, 16)
    assert p["o_proj"]["kernel"].shape == (64, 64) and p["q_proj"]["bias"].shape == (4, 16)
    qk = nn.Attention(config=_cfg(), qk_norm_cls_and_args=(nn.GemmaRMSNorm, dict(hidden_size=16)))
    assert sorted(qk.init(0, torch.randn(1, 3, 64))["params"]) == ["k_norm", "k_proj", "o_proj", "q_norm", "q_proj", "v_proj"]
    with pytest.raises(ValueError, match="fused_qkv requires"):
        nn.Attention(config=_cfg(), fused_qkv=True).init(0, torch.randn(1, 2, 64))
    fused = nn.Attention(config=_cfg(num_kv_heads=4), fused_qkv=True)
    assert fused.init(0, torch.randn(1, 2, 64))["params"]["qkv_proj"]["kernel"].shape == (64, 3, 4, 16)
    with pytest.raises(ValueError, match="3D"):
        a.init(0, torch.randn(5, 64))
    with pytest.raises(TypeError, match="config must be a ModelConfig"):
        nn.Attention(config=None).init(0, torch.randn(1, 2, 64))


def test_apply_refuses_cpu_tensors():
    m = nn.RMSNorm(hidden_size=4)
    v = m.init(0, torch.ones(1, 4))
    v = {"params": {k: t.cpu() for k, t in v["params"].items()}}
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        m.apply(v, torch.ones(1, 4))


def _attn1(**kw):
    from jaxml_b200 import ModelConfig
    from jaxml_b200.nn import Attention

    base = dict(head_dim=1, hidden_size=1, num_heads=1, num_layers=1, max_position_embeddings=8, vocab_size=8,
                attn_scale=1.0, use_rope=False)
    base.update(kw)
    return Attention(ModelConfig(**base))


def test_repeat_kv_on_cpu():
    """nn/attention.py:294-319 (``tests/test_attention.py:245-340`` cases): the grouped heads repeated."""
    from jaxml_b200.nn import Attention

    attn = _attn1(head_dim=2, hidden_size=4, num_heads=2, num_kv_heads=1, attn_scale=2 ** -0.5)
    k = torch.tensor([[[[1.0, 2.0]], [[3.0, 4.0]]]])
    keys, values = attn.apply({}, k, k + 10, method=Attention.repeat_kv)
    assert tuple(keys.shape) == (1, 2, 2, 2) and tuple(values.shape) == (1, 2, 2, 2)
    assert torch.equal(keys[:, :, 1], k[:, :, 0]) and torch.equal(values[:, :, 1], k[:, :, 0] + 10)
    z = torch.zeros
    for kw, exc, match in (({"key_states": z(1, 2, 1)}, ValueError, "key_states must be a 4D array"),
                           ({"key_states": z(0, 2, 1, 2)}, ValueError, "batch axis must be non-empty"),
                           ({"key_states": z(1, 0, 1, 2)}, ValueError, "sequence axis must be non-empty"),
                           ({"key_states": z(1, 2, 0, 2)}, ValueError, "head axis must be non-empty"),
                           ({"key_states": z(1, 2, 1, 0)}, ValueError, "head_dim axis must be non-empty"),
                           ({"value_states": z(1, 2, 1, 2, dtype=torch.int32)}, TypeError,
                            "value_states must contain floating"),
                           ({"value_states": z(1, 3, 1, 2)}, ValueError, "key_states and value_states"),
                           ({"key_states": z(1, 2, 2, 2), "value_states": z(1, 2, 2, 2)}, ValueError,
                            "num_key_value_heads"),
                           ({"key_states": z(1, 2, 1, 3), "value_states": z(1, 2, 1, 3)}, ValueError,
                            "config.head_dim")):
        args = {"key_states": z(1, 2, 1, 2), "value_states": z(1, 2, 1, 2)}
        args.update(kw)
        with pytest.raises(exc, match=match):
            attn.apply({}, method="repeat_kv", **args)
    for field in ("key_states", "value_states"):
        args = {"key_states": z(1, 2, 1, 2), "value_states": z(1, 2, 1, 2)}
        args[field][0, 0, 0, 0] = float("nan")
        with pytest.raises(ValueError, match=f"{field} must contain only finite values"):
            attn.apply({}, method=Attention.repeat_kv, **args)
    with pytest.raises(ValueError, match="no method"):
        attn.apply({}, method="_attend")


def test_mha_argument_checks_on_cpu():
    """nn/attention.py:321-356 (``tests/test_attention.py:340-780`` cases): raised before any device work;
    the options the kernel does not take raise NotImplementedError."""
    from jaxml_b200.nn import Attention

    attn = _attn1()
    z = torch.zeros
    base = {"query_states": z(1, 1, 1, 1), "key_states": z(1, 3, 1, 1), "value_states": z(1, 3, 1, 1)}
    cases = [({"query_states": z(1, 1, 1)}, ValueError, "query_states must be a 4D array"),
             ({"key_states": z(1, 3, 1)}, ValueError, "key_states must be a 4D array"),
             ({"query_states": z(0, 1, 1, 1)}, ValueError, "batch axis must be non-empty"),
             ({"query_states": z(1, 1, 1, 0)}, ValueError, "head_dim axis must be non-empty"),
             ({"value_states": z(1, 0, 1, 1)}, ValueError, "sequence axis must be non-empty"),
             ({"key_states": z(1, 3, 1, 1, dtype=torch.int32)}, TypeError, "key_states must contain floating"),
             ({"value_states": z(1, 2, 1, 1)}, ValueError, "key_states and value_states"),
             ({"query_states": z(2, 1, 1, 1)}, ValueError, "matching batch"),
             ({"query_states": z(1, 1, 2, 1)}, ValueError, "matching batch"),
             ({"causal": 1}, TypeError, "causal must be a boolean"),
             ({"softmax_fp32": "yes"}, TypeError, "softmax_fp32 must be a boolean"),
             ({"output_attentions": None}, TypeError, "output_attentions must be a boolean"),
             ({"sliding_window": True}, TypeError, "sliding_window must be an integer when set"),
             ({"sliding_window": 0}, ValueError, "sliding_window must be positive when set"),
             ({"attention_mask": torch.ones(1, 2, dtype=torch.bool)}, ValueError, "attention batch and key length"),
             ({"attention_mask": torch.ones(1, 3)}, TypeError, "attention_mask must be boolean or integer"),
             ({"attention_mask": torch.tensor([[1, 2, 0]])}, ValueError, "integer values must be 0 or 1"),
             ({"alibi_slope": z(1, 1)}, ValueError, "alibi_slope must be a 1D array"),
             ({"alibi_slope": z(2)}, ValueError, "alibi_slope must contain 1 values"),
             ({"alibi_slope": z(1, dtype=torch.int32)}, TypeError, "alibi_slope must contain floating"),
             ({"alibi_slope": torch.tensor([float("inf")])}, ValueError, "alibi_slope must contain only finite"),
             ({"alibi_slope": z(1)}, NotImplementedError, "ALiBi"),
             ({"softmax_fp32": False}, NotImplementedError, "softmax_fp32"),
             ({"attention_mask": torch.tensor([[False, True, True]])}, NotImplementedError, "right-padded")]
    for kw, exc, match in cases:
        args = dict(base)
        args.update(kw)
        with pytest.raises(exc, match=match):
            attn.apply({}, method=Attention.mha, **args)
    for field in ("query_states", "key_states", "value_states"):
        args = {k: v.clone() for k, v in base.items()}
        args[field][0, 0, 0, 0] = float("inf")
        with pytest.raises(ValueError, match=f"{field} must contain only finite values"):
            attn.apply({}, method=Attention.mha, **args)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        attn.apply({}, method=Attention.mha, **base)


def test_init_keys_made_from_different_seeds_draw_differently():
    e = nn.Embed(num_embeddings=8, features=4)
    t = [e.init(k, [0])["params"]["embedding"] for k in (np.array([0, 1], dtype=np.uint32),
                                                        np.array([0, 2], dtype=np.uint32), 1)]
    assert not torch.equal(t[0], t[1]) and torch.equal(t[0], t[2])


def test_apply_kv_cache_method():
    from jaxml_b200 import ModelConfig

    cfg = ModelConfig(head_dim=2, hidden_size=4, num_heads=2, num_kv_heads=1, num_layers=1,
                      max_position_embeddings=8, vocab_size=8, use_rope=False)
    attn = nn.Attention(cfg)
    k = torch.ones(1, 3, 1, 2)
    keys, values, mask, cache = attn.apply({}, k, k + 1, None, KVCache.init(6), method=nn.Attention.apply_kv_cache)
    assert tuple(keys.shape) == (1, 6, 1, 2) and mask.tolist() == [[True] * 3 + [False] * 3]
    assert cache.pos_id.tolist() == [[2]]
    same = attn.apply({}, k, k, None, None, method="apply_kv_cache")
    assert same[0] is k and same[3] is None
    with pytest.raises(TypeError, match="kv_cache must be a KVCache"):
        attn.apply({}, k, k, None, object(), method="apply_kv_cache")
