"""HF state dict -> reference parameter tree conversion checks (the reference's
``tests/test_hf_utils.py`` conversion cases), CPU only."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from jaxml_b200.hf_utils import to_gemma_jax_params, to_llama_jax_params, to_neox_jax_params


class _Fake:
    def __init__(self, config, states=None):
        self.config = config
        self.states = states if states is not None else {
            f"{n}.weight": torch.arange(32, dtype=torch.float32).reshape(4, 8) for n in ("q_proj", "k_proj", "v_proj")}

    def state_dict(self):
        return self.states


def test_head_dim_fallbacks():
    p = to_llama_jax_params(_Fake(SimpleNamespace(hidden_size=8, num_attention_heads=2)))
    assert p["params"]["q_proj"]["kernel"].shape == (8, 1, 4)
    p = to_gemma_jax_params(_Fake(SimpleNamespace(hidden_size=8, num_attention_heads=2, head_dim=None)))
    assert p["params"]["k_proj"]["kernel"].shape == (8, 1, 4)
    p = to_llama_jax_params(_Fake(SimpleNamespace(hidden_size=8, num_attention_heads=2, head_dim=np.int64(4))))
    assert p["params"]["q_proj"]["kernel"].shape == (8, 1, 4)
    p = to_neox_jax_params(_Fake(SimpleNamespace(hidden_size=8, num_attention_heads=2, head_dim=None)))
    assert p["params"]["q_proj"]["kernel"].shape == (8, 1, 4)


def test_model_surface_is_checked():
    with pytest.raises(ValueError, match="Llama model to expose a config"):
        to_llama_jax_params(SimpleNamespace(state_dict=lambda: {}))
    cfg = SimpleNamespace(hidden_size=8, num_attention_heads=2)
    with pytest.raises(TypeError, match="callable state_dict"):
        to_llama_jax_params(SimpleNamespace(config=cfg))
    with pytest.raises(TypeError, match="state_dict must be a mapping"):
        to_llama_jax_params(SimpleNamespace(config=cfg, state_dict=lambda: []))
    with pytest.raises(ValueError, match="state dict must contain at least one tensor"):
        to_llama_jax_params(SimpleNamespace(config=cfg, state_dict=lambda: {}))


@pytest.mark.parametrize("head_dim,exc,match", [(0, ValueError, "head_dim must be positive"),
                                                (-1, ValueError, "head_dim must be positive"),
                                                (True, TypeError, "head_dim must be an integer"),
                                                (np.bool_(True), TypeError, "head_dim must be an integer"),
                                                (1.5, TypeError, "head_dim must be an integer")])
def test_invalid_head_dim(head_dim, exc, match):
    with pytest.raises(exc, match=match):
        to_llama_jax_params(_Fake(SimpleNamespace(hidden_size=8, num_attention_heads=2, head_dim=head_dim)))


@pytest.mark.parametrize("cfg,match", [
    (SimpleNamespace(hidden_size=10, num_attention_heads=3), "hidden_size must be divisible"),
    (SimpleNamespace(hidden_size=8.0, num_attention_heads=2), "hidden_size must be an integer"),
    (SimpleNamespace(hidden_size=8, num_attention_heads=True), "num_attention_heads must be an integer"),
    (SimpleNamespace(hidden_size=0, num_attention_heads=2), "hidden_size must be positive"),
    (SimpleNamespace(hidden_size=8, num_attention_heads=0), "num_attention_heads must be positive"),
])
def test_invalid_head_dim_fallback(cfg, match):
    with pytest.raises((TypeError, ValueError), match=match):
        to_llama_jax_params(_Fake(cfg))


def test_neox_renames_without_mutating_and_rejects_collisions():
    cfg = SimpleNamespace(hidden_size=8, num_attention_heads=2, head_dim=None)
    model = _Fake(cfg, {"gpt_neox.embed_in.weight": torch.arange(32, dtype=torch.float32).reshape(4, 8),
                        "gpt_neox.final_layer_norm.weight": torch.arange(8, dtype=torch.float32)})
    p = to_neox_jax_params(model)
    assert "embed_tokens" in p["params"]["gpt_neox"] and "norm" in p["params"]["gpt_neox"]
    assert set(model.states) == {"gpt_neox.embed_in.weight", "gpt_neox.final_layer_norm.weight"}
    clash = _Fake(cfg, {"gpt_neox.layers.0.attention.dense.weight": torch.zeros(8, 8),
                        "gpt_neox.layers.0.self_attn.o_proj.weight": torch.zeros(8, 8)})
    with pytest.raises(ValueError, match="map to the same jaxml destination"):
        to_neox_jax_params(clash)


@pytest.mark.parametrize("name,exc,match", [("", ValueError, "non-empty"), ("   ", ValueError, "non-empty"),
                                            (123, TypeError, "string or path-like")])
def test_load_model_from_hf_rejects_invalid_names_before_loading(name, exc, match):
    from jaxml_b200.hf_utils import load_model_from_hf

    with pytest.raises(exc, match=match):
        load_model_from_hf(name)


@pytest.mark.parametrize("dtype,exc,match", [(np.float32, TypeError, "Expected dtype"),
                                             ("bad", ValueError, "Unsupported dtype"),
                                             (torch.int32, ValueError, "Unsupported dtype")])
def test_load_model_from_hf_rejects_invalid_dtypes_before_loading(dtype, exc, match):
    from jaxml_b200.hf_utils import load_model_from_hf

    with pytest.raises(exc, match=match):
        load_model_from_hf("some/model", dtype=dtype)


def test_load_model_from_hf_architecture_argument():
    from jaxml_b200.hf_utils import load_model_from_hf

    with pytest.raises(ValueError, match="Unsupported"):
        load_model_from_hf("some/model", architecture="mamba")
    with pytest.raises(TypeError, match="architecture must be a string"):
        load_model_from_hf("some/model", architecture=3)


def _fake_auto_model(monkeypatch, make):
    import transformers

    class _Auto:
        @classmethod
        def from_pretrained(cls, *a, **k):
            return make()

    monkeypatch.setattr(transformers, "AutoModelForCausalLM", _Auto)


def _refuse(monkeypatch, *names):
    import jaxml_b200.hf_utils as H

    calls = []

    def _no(*a, **k):
        calls.append(a)
        raise AssertionError("must not be reached")

    for n in names:
        monkeypatch.setattr(H, n, _no)
    return calls


def test_direct_loaders_check_arguments_before_loading(monkeypatch):
    """hf_utils.py:184-250 (the reference's ``tests/test_hf_utils.py:222-270`` cases)."""
    from jaxml_b200.hf_utils import load_llama_from_hf

    _fake_auto_model(monkeypatch, lambda: (_ for _ in ()).throw(AssertionError("loaded")))
    with pytest.raises(TypeError, match="Expected dtype"):
        load_llama_from_hf("some/model", dtype=np.float32)
    for name, exc, match in (("", ValueError, "non-empty"), ("   ", ValueError, "non-empty"),
                             (123, TypeError, "string or path-like")):
        with pytest.raises(exc, match=match):
            load_llama_from_hf(name)


@pytest.mark.parametrize("loader,model_type,match", [("load_llama_from_hf", "gpt_neox", "Llama model_type"),
                                                     ("load_neox_from_hf", "llama", "GPT-NeoX model_type")])
def test_direct_loaders_check_the_model_type_before_converting(monkeypatch, loader, model_type, match):
    import jaxml_b200.hf_utils as H

    _fake_auto_model(monkeypatch, lambda: SimpleNamespace(config=SimpleNamespace(model_type=model_type),
                                                          state_dict=lambda: {}))
    calls = _refuse(monkeypatch, "to_llama_jax_params", "to_neox_jax_params")
    with pytest.raises(ValueError, match=match):
        getattr(H, loader)("some/model")
    assert calls == []


@pytest.mark.parametrize("loader,match", [("load_llama_from_hf", "Llama model to expose a config"),
                                          ("load_neox_from_hf", "GPT-NeoX model to expose a config")])
def test_direct_loaders_need_a_config(monkeypatch, loader, match):
    import jaxml_b200.hf_utils as H

    _fake_auto_model(monkeypatch, lambda: SimpleNamespace(state_dict=lambda: {}))
    calls = _refuse(monkeypatch, "to_llama_jax_params", "to_neox_jax_params")
    with pytest.raises(ValueError, match=match):
        getattr(H, loader)("some/model")
    assert calls == []


def test_gemma_loader_checks(monkeypatch):
    """The wrapper's model type and config, its language model, and the text model's type and config are
    checked before any conversion (the reference's ``tests/test_hf_utils.py:329-422`` cases)."""
    from jaxml_b200.hf_utils import load_gemma_from_hf

    calls = _refuse(monkeypatch, "to_gemma_jax_params")
    _fake_auto_model(monkeypatch, lambda: SimpleNamespace(config=SimpleNamespace(model_type="llama")))
    with pytest.raises(ValueError, match="Gemma model_type"):
        load_gemma_from_hf("some/model")
    _fake_auto_model(monkeypatch, lambda: SimpleNamespace(config=SimpleNamespace(model_type="gemma3")))
    with pytest.raises(ValueError, match="language_model"):
        load_gemma_from_hf("some/model")

    class _Exploding:
        @property
        def language_model(self):
            raise AssertionError("language_model read before the wrapper config was checked")

    _fake_auto_model(monkeypatch, _Exploding)
    with pytest.raises(ValueError, match="Gemma model to expose a config"):
        load_gemma_from_hf("some/model")
    _fake_auto_model(monkeypatch, lambda: SimpleNamespace(
        config=SimpleNamespace(model_type="gemma3"),
        language_model=SimpleNamespace(config=SimpleNamespace(model_type="llama"), state_dict=lambda: {})))
    with pytest.raises(ValueError, match="Gemma text model_type"):
        load_gemma_from_hf("some/model")
    _fake_auto_model(monkeypatch, lambda: SimpleNamespace(config=SimpleNamespace(model_type="gemma3"),
                                                          language_model=SimpleNamespace(state_dict=lambda: {})))
    with pytest.raises(ValueError, match="Gemma text model to expose a config"):
        load_gemma_from_hf("some/model")
    assert calls == []


def test_load_model_from_hf_dispatch(monkeypatch):
    """``auto`` reads the config's model type (gemma3_text included) and forwards the loader kwargs; a bad
    dtype is refused before the config is read."""
    import transformers

    import jaxml_b200.hf_utils as H

    seen = []

    class _AutoConfig:
        @classmethod
        def from_pretrained(cls, *a, **k):
            return SimpleNamespace(model_type="gemma3_text")

    def _gemma(name, dtype, **kw):
        seen.append((name, dtype, kw))
        return "model", {"params": {}}

    monkeypatch.setattr(transformers, "AutoConfig", _AutoConfig)
    monkeypatch.setattr(H, "load_gemma_from_hf", _gemma)
    assert H.load_model_from_hf("some/model", dtype="float32", local_files_only=True) == ("model", {"params": {}})
    assert seen == [("some/model", "float32", {"local_files_only": True})]
    calls = _refuse(monkeypatch, "_infer_hf_architecture")
    for dtype, exc, match in ((np.float32, TypeError, "Expected dtype"), ("bad", ValueError, "Unsupported dtype"),
                              (torch.int32, ValueError, "Unsupported dtype")):
        with pytest.raises(exc, match=match):
            H.load_model_from_hf("some/model", dtype=dtype)
    assert calls == []


def test_converter_default_dtypes_follow_the_reference():
    """hf_utils.py:57-70: float16 for Llama and GPT-NeoX, bfloat16 for Gemma, unless asked otherwise."""
    cfg = SimpleNamespace(hidden_size=8, num_attention_heads=2, head_dim=None)
    assert to_llama_jax_params(_Fake(cfg))["params"]["q_proj"]["kernel"].dtype == torch.float16
    assert to_neox_jax_params(_Fake(cfg))["params"]["q_proj"]["kernel"].dtype == torch.float16
    assert to_gemma_jax_params(_Fake(cfg))["params"]["q_proj"]["kernel"].dtype == torch.bfloat16
    assert to_llama_jax_params(_Fake(cfg), dtype=torch.float32)["params"]["q_proj"]["kernel"].dtype == torch.float32
