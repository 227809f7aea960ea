"""Engine argument validation on CPU: the errors are raised before any device work, with the messages
the reference's own tests match (``tests/test_generation.py:117-1182``), and ``max_new_tokens=0``
returns the prompt without touching a GPU."""
import numpy as np
import pytest
import torch

from jaxml_b200 import Engine, InferenceConfig, LlamaModelWithHead, ModelConfig
from jaxml_b200.models import random_params


@pytest.fixture(scope="module")
def engine():
    cfg = ModelConfig(head_dim=8, hidden_size=32, num_heads=4, num_kv_heads=2, num_layers=1,
                      max_position_embeddings=64, vocab_size=100)
    model = LlamaModelWithHead(cfg)
    return Engine(model, InferenceConfig(), random_params("llama", cfg, seed=0))


def test_negative_max_new_tokens_is_rejected_first(engine):
    with pytest.raises(ValueError, match="max_new_tokens must be non-negative"):
        engine.generate(torch.ones(1, 2, 3), max_new_tokens=-1, temperature=float("nan"))


@pytest.mark.parametrize("value", [True, 1.5])
def test_non_integer_max_new_tokens(engine, value):
    with pytest.raises(TypeError, match="max_new_tokens must be an integer"):
        engine.generate(torch.ones(1, 4, dtype=torch.int32), max_new_tokens=value)


@pytest.mark.parametrize("seed", [True, np.bool_(True), 1.5])
def test_non_integer_seed(engine, seed):
    with pytest.raises(TypeError, match="seed must be an integer"):
        engine.generate(torch.ones(1, 4, dtype=torch.int32), max_new_tokens=0, seed=seed)


@pytest.mark.parametrize("kwargs,match", [({"include_prompt": 1}, "include_prompt must be a boolean"),
                                          ({"fuse_decoding": 1}, "fuse_decoding must be a boolean")])
def test_non_boolean_control_flags(engine, kwargs, match):
    with pytest.raises(TypeError, match=match):
        engine.generate(torch.ones(1, 4, dtype=torch.int32), max_new_tokens=0, **kwargs)


def test_numpy_scalar_control_arguments_and_zero_tokens(engine):
    out = engine.generate(np.ones((1, 4), dtype=np.int32), seed=np.int64(0), max_new_tokens=np.int64(0),
                          include_prompt=np.bool_(False), fuse_decoding=np.bool_(False))
    assert tuple(out.shape) == (1, 0)
    out = engine.generate(np.arange(4, dtype=np.int32), max_new_tokens=0, include_prompt=True)
    assert tuple(out.shape) == (1, 4) and out.dtype == torch.int32 and out[0].tolist() == [0, 1, 2, 3]
    out = engine.generate(np.arange(4, dtype=np.int32), attention_mask=np.ones(4, dtype=bool), max_new_tokens=0)
    assert tuple(out.shape) == (1, 4)


@pytest.mark.parametrize("kwargs,exc,match", [({"top_p": True}, TypeError, "top_p must be a real number"),
                                              ({"min_p": "0.1"}, TypeError, "min_p must be a real number"),
                                              ({"temperature": float("nan")}, ValueError, "must be finite")])
def test_invalid_sampling_values(engine, kwargs, exc, match):
    with pytest.raises(exc, match=match):
        engine.generate(torch.ones(1, 4, dtype=torch.int32), max_new_tokens=0, **kwargs)


@pytest.mark.parametrize("ids,match", [(torch.ones(1, 2, 3, dtype=torch.int32), "1D or 2D array"),
                                       (torch.ones(0, 1, dtype=torch.int32), "at least one batch row"),
                                       (torch.ones(1, 0, dtype=torch.int32), "at least one token")])
def test_invalid_prompt_shapes(engine, ids, match):
    with pytest.raises(ValueError, match=match):
        engine.generate(ids, max_new_tokens=0)


def test_prompt_tokens_must_be_integers_in_the_vocabulary(engine):
    with pytest.raises(TypeError, match="integer token ids"):
        engine.generate(torch.ones(1, 4), max_new_tokens=0)
    for tok in (-1, 100):
        with pytest.raises(ValueError, match=r"prompt_tokens token ids must be within"):
            engine.generate(torch.tensor([[tok]], dtype=torch.int32), max_new_tokens=0)


def test_attention_mask_validation(engine):
    ids = torch.ones(2, 4, dtype=torch.int32)
    with pytest.raises(ValueError, match="attention_mask shape must match"):
        engine.generate(ids, attention_mask=torch.ones(1, 4, dtype=torch.bool), max_new_tokens=0)
    with pytest.raises(TypeError, match="attention_mask must be boolean or integer"):
        engine.generate(ids[:1], attention_mask=torch.ones(1, 4), max_new_tokens=0)
    for bad in ([[1, 2, 1, 1]], [[1, -1, 0, 0]]):
        with pytest.raises(ValueError, match="integer values must be 0 or 1"):
            engine.generate(ids[:1], attention_mask=torch.tensor(bad, dtype=torch.int32), max_new_tokens=0)
    with pytest.raises(ValueError, match="at least one valid token"):
        engine.generate(ids, attention_mask=torch.tensor([[1, 0, 0, 0], [0, 0, 0, 0]], dtype=torch.bool),
                        max_new_tokens=0)
    with pytest.raises(ValueError, match="right padded"):
        engine.generate(ids[:1], attention_mask=torch.tensor([[0, 1, 1, 1]], dtype=torch.bool), max_new_tokens=0)
    # integer masks of 0 / 1 are accepted
    out = engine.generate(ids[:1], attention_mask=torch.tensor([[1, 1, 0, 0]], dtype=torch.int32), max_new_tokens=0)
    assert tuple(out.shape) == (1, 4)


def test_engine_construction_validation(engine):
    cfg = engine.model.config
    with pytest.raises(TypeError, match="config must be an InferenceConfig"):
        Engine(engine.model, None, engine.params)
    with pytest.raises(ValueError, match="cache_stride must be positive"):
        Engine(engine.model, InferenceConfig(), engine.params, cache_stride=0)
    for bad in (True, 2.5):
        with pytest.raises(TypeError, match="cache_stride must be an integer"):
            Engine(engine.model, InferenceConfig(), engine.params, cache_stride=bad)
    assert Engine(engine.model, InferenceConfig(), engine.params, cache_stride=np.int64(128)).cache_stride == 128
    with pytest.raises(ValueError, match="requires .* devices"):
        Engine(engine.model, InferenceConfig(tp_size=64), engine.params)
    assert cfg.vocab_size == 100


def test_init_params_validates_weights_before_device_work(engine):
    with pytest.raises(TypeError, match="weights must be a mapping"):
        engine.init_params(weights=[1, 2])
    with pytest.raises(ValueError, match="'params'"):
        engine.init_params(weights={"model": {}})
    with pytest.raises(TypeError, match=r"weights\['params'\] must be a mapping"):
        engine.init_params(weights={"params": 3})
    with pytest.raises(TypeError, match="use_tpu must be a boolean"):
        engine.init_params(use_tpu=1)
    with pytest.raises(TypeError, match="reinit_weight must be a boolean"):
        engine.init_params(reinit_weight="yes")


def test_init_cache(engine):
    """engine.py:110-121: one empty cache per layer in the engine's dtype (the reference's
    ``tests/test_generation.py:1119-1160`` cases)."""
    caches = engine.init_cache(max_seq_len=np.int64(8))
    assert len(caches) == engine.model.config.num_layers
    assert all(c.max_seq_len == 8 and c.k is None and c.dtype == engine.dtype for c in caches)
    for bad in (True, 1.5):
        with pytest.raises(TypeError, match="max_seq_len must be an integer"):
            engine.init_cache(max_seq_len=bad)
    for bad in (0, -1):
        with pytest.raises(ValueError, match="max_seq_len must be positive"):
            engine.init_cache(max_seq_len=bad)

    class _NoConfig:
        config = object()

    class _Cfg:
        def __init__(self, n):
            self.num_layers = n

    class _Model:
        def __init__(self, n):
            self.config = _Cfg(n)

    with pytest.raises(TypeError, match="config.num_layers"):
        Engine(_NoConfig(), InferenceConfig(), {"params": {}}).init_cache(8)
    for n, exc, match in ((True, TypeError, "model.config.num_layers must be an integer"),
                          (1.5, TypeError, "model.config.num_layers must be an integer"),
                          (0, ValueError, "model.config.num_layers must be positive")):
        with pytest.raises(exc, match=match):
            Engine(_Model(n), InferenceConfig(), {"params": {}}).init_cache(8)


def test_prepare_input(engine):
    """engine.py:320-353: 2D leaves of one batch size, cast to ``dtype`` (the reference's
    ``tests/test_generation.py:297-485`` cases)."""
    out = engine.prepare_input({"input_ids": np.array([[1, 2, 3]], dtype=np.int32)}, dtype=np.float32)
    assert set(out) == {"input_ids"} and out["input_ids"].dtype == torch.float32
    assert out["input_ids"].cpu().tolist() == [[1.0, 2.0, 3.0]]
    out = engine.prepare_input([np.ones((2, 2), dtype=np.int64), torch.zeros(2, 5, dtype=torch.int32)])
    assert isinstance(out, list) and out[1].dtype == torch.int32
    for inputs, exc, match in ((object(), TypeError, "array-like"),
                               (np.ones(3, dtype=np.int32), ValueError, "2D arrays"),
                               (np.ones((1, 2, 3), dtype=np.int32), ValueError, "2D arrays"),
                               ({}, ValueError, "at least one array leaf"),
                               ({"x": np.ones((0, 2), dtype=np.int32)}, ValueError, "at least one batch row"),
                               ({"x": np.ones((1, 0), dtype=np.int32)}, ValueError, "at least one token"),
                               ({"a": np.ones((1, 2)), "b": np.ones((2, 2))}, ValueError, "same batch size")):
        with pytest.raises(exc, match=match):
            engine.prepare_input(inputs)
    with pytest.raises(TypeError, match="valid"):
        engine.prepare_input(np.ones((1, 2), dtype=np.int32), dtype="not-a-dtype")


def test_prepare_input_batch_divisible_by_dp_size(engine, monkeypatch):
    import jaxml_b200.engine as E

    monkeypatch.setattr(E, "_device_count", lambda: 2)
    eng = Engine(engine.model, InferenceConfig(dp_size=2), engine.params)
    assert tuple(eng.prepare_input({"x": np.array([[1, 2], [3, 4]])})["x"].shape) == (2, 2)
    with pytest.raises(ValueError, match="divisible by dp_size=2"):
        eng.prepare_input({"x": np.array([[1, 2], [3, 4], [5, 6]])})


def test_inference_config_checks():
    """engine.py:59-82 (the reference's ``tests/test_generation.py:1206-1240`` cases)."""
    for kw in ({"tp_size": 0}, {"tp_size": -1}, {"dp_size": 0}, {"dp_size": -1}):
        with pytest.raises(ValueError, match=next(iter(kw))):
            InferenceConfig(**kw)
    for kw, match in (({"tp_size": True}, "tp_size must be an integer"), ({"tp_size": 1.5}, "tp_size must be an integer"),
                      ({"dp_size": True}, "dp_size must be an integer"), ({"dp_size": 1.5}, "dp_size must be an integer")):
        with pytest.raises(TypeError, match=match):
            InferenceConfig(**kw)
    c = InferenceConfig(tp_size=np.int64(1), dp_size=np.int64(1))
    assert c.tp_size == 1 and c.dp_size == 1 and type(c.tp_size) is int


def test_engine_dtype_and_config_arguments(engine):
    for bad in (None, "not-a-dtype", object()):
        with pytest.raises(TypeError, match="dtype must be a valid"):
            Engine(engine.model, InferenceConfig(), engine.params, dtype=bad)
    for dt, want in ((torch.float32, torch.float32), (np.float32, torch.float32), ("bfloat16", torch.bfloat16)):
        assert Engine(engine.model, InferenceConfig(), engine.params, dtype=dt).dtype == want
    for bad in (None, {"tp_size": 1}, object()):
        with pytest.raises(TypeError, match="config must be an InferenceConfig"):
            Engine(engine.model, bad, engine.params)


def test_init_params_checks_explicit_weights_before_touching_the_model():
    """engine.py:225-240: malformed weights are rejected before the model is asked for anything."""
    from types import MappingProxyType

    class _Untouchable:
        def __getattr__(self, name):
            raise AssertionError(f"the model was used ({name}) before the weights were checked")

    eng = Engine(_Untouchable(), InferenceConfig(), {"params": {}})
    for weights, exc, match in ((("params", {}), TypeError, "weights must be a mapping"),
                                ({}, ValueError, "'params'"),
                                ({"cache": {}}, ValueError, "'params'"),
                                (MappingProxyType({"cache": {}}), ValueError, "'params'"),
                                ({"params": []}, TypeError, r"weights\['params'\] must be a mapping"),
                                (MappingProxyType({"params": []}), TypeError, r"weights\['params'\] must be a mapping")):
        with pytest.raises(exc, match=match):
            eng.init_params(weights=weights, use_tpu=False)
    for kw, match in (({"use_tpu": 1}, "use_tpu must be a boolean"), ({"reinit_weight": 1}, "reinit_weight must be a boolean")):
        with pytest.raises(TypeError, match=match):
            eng.init_params(**kw)


def test_prepare_generation_inputs_is_static_and_canonicalises():
    ids, mask = Engine._prepare_generation_inputs(np.arange(4, dtype=np.int32), np.array([1, 1, 0, 0], dtype=np.int32))
    assert tuple(ids.shape) == (1, 4) and mask.dtype == torch.bool and mask.tolist() == [[True, True, False, False]]
    for bad in ([[1, 2, 0, 0]], [[1, -1, 0, 0]]):
        with pytest.raises(ValueError, match="integer values must be 0 or 1"):
            Engine._prepare_generation_inputs(np.ones((1, 4), dtype=np.int32), np.array(bad, dtype=np.int32))
    ids, mask = Engine._prepare_generation_inputs(torch.ones(2, 3, dtype=torch.int64), None)
    assert mask is None and tuple(ids.shape) == (2, 3)
