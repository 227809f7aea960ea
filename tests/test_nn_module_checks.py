"""Field and input checks of ``jaxml_b200.nn``'s norms, ``Embed`` and ``DenseGeneral`` at ``init`` (no
device work), case by case as the reference's ``tests/test_modules.py:120-680`` states them."""
import numpy as np
import pytest
import torch

from jaxml_b200.nn import DenseGeneral, Embed, GemmaRMSNorm, LayerNorm, RMSNorm

X = torch.ones(1, 2, 4)


def test_gemma_rms_norm_requires_upcast():
    with pytest.raises(ValueError, match="upcast=True"):
        GemmaRMSNorm(hidden_size=4, upcast=False).init(0, X)


@pytest.mark.parametrize("cls", [RMSNorm, LayerNorm, GemmaRMSNorm])
def test_norm_input_checks(cls):
    with pytest.raises(ValueError, match="hidden dimension mismatch"):
        cls(hidden_size=4).init(0, torch.ones(1, 2, 3))
    with pytest.raises(ValueError, match="at least one dimension"):
        cls(hidden_size=4).init(0, torch.tensor(1.0))
    for x in (torch.ones(0, 2, 4), torch.ones(1, 0, 4), torch.ones(1, 2, 0)):
        with pytest.raises(ValueError, match="empty axes"):
            cls(hidden_size=4).init(0, x)
    with pytest.raises(TypeError, match="floating point"):
        cls(hidden_size=4).init(0, torch.ones(1, 2, 4, dtype=torch.int32))
    for v in (float("nan"), float("inf"), -float("inf")):
        x = X.clone()
        x[0, 0, 0] = v
        with pytest.raises(ValueError, match="input must contain only finite values"):
            cls(hidden_size=4).init(0, x)


@pytest.mark.parametrize("cls", [RMSNorm, LayerNorm])
@pytest.mark.parametrize("kwargs,exc,match", [
    ({"hidden_size": True}, TypeError, "hidden_size must be an integer"),
    ({"hidden_size": np.bool_(True)}, TypeError, "hidden_size must be an integer"),
    ({"hidden_size": 1.5}, TypeError, "hidden_size must be an integer"),
    ({"hidden_size": 0}, ValueError, "hidden_size must be positive"),
    ({"eps": True}, TypeError, "eps must be a real number"),
    ({"eps": "1e-6"}, TypeError, "eps must be a real number"),
    ({"eps": float("nan")}, ValueError, "eps must be finite"),
    ({"eps": 0.0}, ValueError, "eps must be positive"),
    ({"upcast": 1}, TypeError, "upcast must be a boolean"),
    ({"dtype": None}, TypeError, "dtype must be a valid"),
    ({"dtype": "not-a-dtype"}, TypeError, "dtype must be a valid"),
])
def test_norm_field_checks(cls, kwargs, exc, match):
    with pytest.raises(exc, match=match):
        cls(**({"hidden_size": 4} | kwargs)).init(0, X)


def test_norm_numpy_fields_and_layer_norm_bias_flag():
    for cls in (RMSNorm, LayerNorm):
        v = cls(hidden_size=np.int64(4), eps=np.float64(1e-6), upcast=np.bool_(True), dtype=np.float32).init(0, X)
        assert v["params"]["weight"].dtype == torch.float32
    with pytest.raises(TypeError, match="use_bias must be a boolean"):
        LayerNorm(hidden_size=4, use_bias=1).init(0, X)
    assert set(LayerNorm(hidden_size=4, use_bias=False).init(0, X)["params"]) == {"weight"}


@pytest.mark.parametrize("kwargs,exc,match", [
    ({"num_embeddings": True, "features": 4}, TypeError, "num_embeddings must be an integer"),
    ({"num_embeddings": np.bool_(True), "features": 4}, TypeError, "num_embeddings must be an integer"),
    ({"num_embeddings": 1.5, "features": 4}, TypeError, "num_embeddings must be an integer"),
    ({"num_embeddings": 0, "features": 4}, ValueError, "num_embeddings must be positive"),
    ({"num_embeddings": 8, "features": True}, TypeError, "features must be an integer"),
    ({"num_embeddings": 8, "features": 1.5}, TypeError, "features must be an integer"),
    ({"num_embeddings": 8, "features": 0}, ValueError, "features must be positive"),
    ({"num_embeddings": 8, "features": 4, "one_hot": 1}, TypeError, "one_hot must be a boolean"),
    ({"num_embeddings": 8, "features": 4, "dtype": None}, TypeError, "dtype must be a valid"),
    ({"num_embeddings": 8, "features": 4, "dtype": "not-a-dtype"}, TypeError, "dtype must be a valid"),
])
def test_embed_field_checks(kwargs, exc, match):
    with pytest.raises(exc, match=match):
        Embed(**kwargs).init(0, torch.tensor([0, 1], dtype=torch.int32))


def test_embed_inputs():
    v = Embed(num_embeddings=np.int64(8), features=np.int64(4), one_hot=np.bool_(True)).init(0, [0, 1])
    assert tuple(v["params"]["embedding"].shape) == (8, 4)
    for x in (torch.zeros(0, dtype=torch.int32), torch.zeros(1, 0, dtype=torch.int32)):
        with pytest.raises(ValueError, match="at least one token id"):
            Embed(num_embeddings=8, features=4).init(0, x)
    for x, match in ((torch.tensor([0, 8]), "less than num_embeddings=8"), (torch.tensor([-1, 0]), "non-negative")):
        with pytest.raises(ValueError, match=match):
            Embed(num_embeddings=8, features=4).init(0, x)


def _dense(**kw):
    base = dict(features=4, axis=-1, kernel_axes=("embed", "features"))
    base.update(kw)
    return DenseGeneral(**base)


X3 = torch.ones(1, 2, 3)


@pytest.mark.parametrize("kw,exc,match", [
    ({"axis": (-1, -1)}, ValueError, "unique"),
    ({"axis": 3}, ValueError, "out of bounds"),
    ({"axis": 1.5}, TypeError, "integers"),
    ({"axis": True}, TypeError, "integers"),
    ({"axis": np.bool_(True)}, TypeError, "integers"),
    ({"with_logical_partitioning": 1}, TypeError, "with_logical_partitioning must be a boolean"),
    ({"kernel_axes": ()}, ValueError, "Kernel axes must be specified"),
    ({"kernel_axes": ("embed",)}, ValueError, "one axis name per kernel dimension"),
    ({"kernel_axes": "embed"}, TypeError, "kernel_axes must be a tuple"),
    ({"kernel_axes": ("embed", 1)}, TypeError, "kernel_axes entries"),
    ({"features": True}, TypeError, "features values must be integers"),
    ({"features": np.bool_(True)}, TypeError, "features values must be integers"),
    ({"features": 1.5}, TypeError, "features values must be integers"),
    ({"features": 0}, ValueError, "features values must be positive"),
    ({"features": (4, True)}, TypeError, "features values must be integers"),
    ({"features": (4, 0)}, ValueError, "features values must be positive"),
    ({"dtype": None}, TypeError, "dtype must be a valid"),
    ({"dtype": "not-a-dtype"}, TypeError, "dtype must be a valid"),
    ({"weight_dtype": None}, TypeError, "weight_dtype must be a valid"),
    ({"weight_dtype": "not-a-dtype"}, TypeError, "weight_dtype must be a valid"),
    ({"use_bias": 1}, TypeError, "use_bias must be a boolean"),
])
def test_dense_general_field_checks(kw, exc, match):
    with pytest.raises(exc, match=match):
        _dense(**kw).init(0, X3)


def test_dense_general_inputs_and_parameter_shapes():
    with pytest.raises(TypeError, match="floating point"):
        _dense().init(0, torch.ones(1, 2, 3, dtype=torch.int32))
    for v in (float("nan"), float("inf")):
        x = X3.clone()
        x[0, 0, 0] = v
        with pytest.raises(ValueError, match="DenseGeneral inputs must contain only finite values"):
            _dense().init(0, x)
    for x in (torch.ones(0, 2, 3), torch.ones(1, 0, 3), torch.ones(1, 2, 0)):
        with pytest.raises(ValueError, match="empty axes"):
            _dense().init(0, x)
    assert tuple(_dense(axis=np.int64(-1)).init(0, X3)["params"]["kernel"].shape) == (3, 4)
    p = _dense(features=(np.int64(4), np.int64(2)), kernel_axes=("embed", "a", "b")).init(0, X3)["params"]
    assert tuple(p["kernel"].shape) == (3, 4, 2)
    p = _dense(use_bias=np.bool_(True), dtype=np.float32, weight_dtype=np.float32).init(0, X3)["params"]
    assert tuple(p["bias"].shape) == (4,) and p["kernel"].dtype == torch.float32
    for axes in ("embed", ("embed",), (1,)):
        p = _dense(kernel_axes=axes, use_bias=True, with_logical_partitioning=False).init(0, X3)["params"]
        assert tuple(p["bias"].shape) == (4,)
    p = _dense(features=(4, 2), kernel_axes=("embed", "a", "b"), use_bias=True,
               with_logical_partitioning=np.bool_(True)).init(0, X3)["params"]
    assert tuple(p["bias"].shape) == (4, 2)


def _attn_cfg(use_rope, **kw):
    from jaxml_b200 import ModelConfig

    base = dict(head_dim=2 if use_rope else 1, hidden_size=2 if use_rope else 1, num_heads=1, num_layers=1,
                max_position_embeddings=8, vocab_size=8, attn_scale=1.0, use_rope=use_rope)
    base.update(kw)
    return ModelConfig(**base)


def _cos_sin(n):
    return torch.ones(n, 2), torch.zeros(n, 2)


def test_attention_construction_checks():
    from jaxml_b200.nn import Attention

    cfg = _attn_cfg(False, head_dim=4, hidden_size=16, num_heads=4, num_kv_heads=2)
    with pytest.raises(ValueError, match="fused_qkv"):
        Attention(cfg, fused_qkv=True).init(0, torch.zeros(1, 2, 16))
    for kw, match in (({"dtype": None}, "dtype must be a valid"), ({"dtype": "not-a-dtype"}, "dtype must be a valid"),
                      ({"weight_dtype": None}, "weight_dtype must be a valid"),
                      ({"with_logical_partitioning": 1}, "with_logical_partitioning must be a boolean")):
        with pytest.raises(TypeError, match=match):
            Attention(_attn_cfg(False), **kw).init(0, torch.zeros(1, 2, 1))
    p = Attention(_attn_cfg(False), dtype=np.float32, weight_dtype=torch.bfloat16,
                  with_logical_partitioning=np.bool_(False)).init(0, torch.zeros(1, 2, 1))["params"]
    assert all(p[n]["kernel"].dtype == torch.bfloat16 for n in ("q_proj", "k_proj", "v_proj", "o_proj"))


@pytest.mark.parametrize("use_rope", [False, True], ids=["Attention", "AttentionWithRoPE"])
def test_attention_call_checks_before_projections(use_rope):
    """Flags, the flash request, the cache type, hidden states and (with RoPE) the cos / sin pair are
    checked before any projection (the reference's ``tests/test_attention.py:455-680`` cases)."""
    from jaxml_b200.nn import Attention, AttentionWithRoPE

    cfg = _attn_cfg(use_rope)
    attn = (AttentionWithRoPE if use_rope else Attention)(cfg)
    h = torch.zeros(1, 2, cfg.hidden_size)
    kw = {"cos_sin": _cos_sin(8)} if use_rope else {}
    v = attn.init(0, h, **kw)
    for extra, match in (({"output_attentions": 1}, "output_attentions must be a boolean"),
                         ({"use_flash": 1}, "use_flash must be a boolean")):
        with pytest.raises(TypeError, match=match):
            attn.apply(v, h, **kw, **extra)
    with pytest.raises(NotImplementedError, match="flash attention is not enabled"):
        attn.apply(v, h, use_flash=True, **({} if use_rope else {"kv_cache": object()}))
    with pytest.raises(TypeError, match="kv_cache must be a KVCache"):
        attn.apply(v, h, **kw, kv_cache=object())
    for bad, exc, match in ((torch.zeros(1, 2), ValueError, "hidden_states must be a 3D array"),
                            (torch.zeros(1, 2, 1, 1), ValueError, "hidden_states must be a 3D array"),
                            (torch.zeros(0, 2, 1), ValueError, "empty axes"),
                            (torch.zeros(1, 2, 1, dtype=torch.int32), TypeError, "hidden_states must contain floating")):
        with pytest.raises(exc, match=match):
            attn.apply(v, bad, **kw)
    x = h.clone()
    x[0, 0, 0] = float("nan")
    with pytest.raises(ValueError, match="hidden_states must contain only finite values"):
        attn.apply(v, x, **kw)


def test_attention_with_rope_cos_sin_checks():
    from jaxml_b200.nn import AttentionWithRoPE

    cfg = _attn_cfg(True, attn_scale=2 ** -0.5)
    attn = AttentionWithRoPE(cfg)
    h = torch.zeros(1, 2, 2)
    v = attn.init(0, h, cos_sin=_cos_sin(8))
    with pytest.raises(ValueError, match="requires cos_sin"):
        attn.apply(v, h)
    for cs, exc, match in (((), ValueError, "exactly two arrays"),
                           ((torch.ones(2, 2),), ValueError, "exactly two arrays"),
                           ((torch.ones(2, 2), torch.zeros(2, 2), torch.ones(2, 2)), ValueError, "exactly two arrays"),
                           (torch.ones(2, 2), TypeError, "not a single array"),
                           (np.ones((2, 2), dtype=np.float32), TypeError, "not a single array"),
                           (object(), TypeError, "cos_sin must be a pair")):
        with pytest.raises(exc, match=match):
            attn.apply(v, h, cos_sin=cs)
