"""GenerationConfig / TextGenerationPipeline (text_generation.py of the reference): validation and the
tokenize -> generate -> decode plumbing, with a fake engine and tokenizer (no GPU)."""
import numpy as np
import pytest

from jaxml_b200 import GenerationConfig, TextGenerationPipeline


class _Tok:
    """Character-level tokenizer: ids = ord(c) % 97 + 3, right padding with 0."""

    def __call__(self, texts, return_tensors="np", padding=True, **kw):
        ids = [[ord(c) % 97 + 3 for c in t] for t in texts]
        n = max(len(x) for x in ids)
        arr = np.zeros((len(ids), n), dtype=np.int64)
        mask = np.zeros((len(ids), n), dtype=np.int64)
        for i, x in enumerate(ids):
            arr[i, :len(x)] = x
            mask[i, :len(x)] = 1
        return {"input_ids": arr, "attention_mask": mask}

    def batch_decode(self, tokens, skip_special_tokens=True):
        return ["".join(chr(int(t) + 60) for t in row) for row in tokens]


class _Engine:
    def __init__(self):
        self.calls = []

    def generate(self, prompt_tokens, attention_mask=None, **kw):
        self.calls.append((np.asarray(prompt_tokens), attention_mask, kw))
        B, P = np.asarray(prompt_tokens).shape
        new = np.full((B, kw["max_new_tokens"]), 7, dtype=np.int32)
        return np.concatenate([prompt_tokens, new], 1) if kw["include_prompt"] else new


def test_generation_config_validates_like_the_reference():
    c = GenerationConfig(seed=np.int64(3), max_new_tokens=5, top_p=1)
    assert c.seed == 3 and isinstance(c.seed, int) and c.top_p == 1.0
    with pytest.raises(TypeError, match="seed must be an integer"):
        GenerationConfig(seed=True)
    with pytest.raises(ValueError, match="max_new_tokens must be non-negative"):
        GenerationConfig(max_new_tokens=-1)
    with pytest.raises(ValueError, match="top_k must be non-negative"):
        GenerationConfig(top_k=-2)
    with pytest.raises(ValueError, match="temperature must be finite"):
        GenerationConfig(temperature=float("inf"))
    with pytest.raises(TypeError, match="top_p must be a real number"):
        GenerationConfig(top_p="0.5")
    with pytest.raises(TypeError, match="include_prompt must be a boolean"):
        GenerationConfig(include_prompt=1)


def test_pipeline_tokenize_generate_decode():
    eng = _Engine()
    pipe = TextGenerationPipeline(eng, _Tok())
    out = pipe.generate_text(["ab", "xyz"], max_new_tokens=2, temperature=0.0)
    assert isinstance(out, list) and len(out) == 2
    ids, mask, kw = eng.calls[-1]
    assert ids.shape == (2, 3) and mask.dtype == bool and not mask[0, 2]
    assert kw["max_new_tokens"] == 2 and kw["temperature"] == 0.0 and kw["include_prompt"] is True
    single = pipe.generate_text("hi", GenerationConfig(max_new_tokens=1), include_prompt=False)
    assert isinstance(single, str) and len(single) == 1
    toks = pipe.generate_tokens("hi", max_new_tokens=3)
    assert toks.shape == (1, 5)


def test_pipeline_rejects_bad_inputs():
    with pytest.raises(TypeError, match="engine must provide a callable generate"):
        TextGenerationPipeline(object(), _Tok())
    with pytest.raises(TypeError, match="batch_decode"):
        TextGenerationPipeline(_Engine(), lambda x: x)
    pipe = TextGenerationPipeline(_Engine(), _Tok())
    with pytest.raises(ValueError, match="at least one prompt"):
        pipe.generate_text([])
    with pytest.raises(TypeError, match="prompts must be a string"):
        pipe.generate_text([1, 2])
    with pytest.raises(TypeError, match="generation_config must be a GenerationConfig"):
        pipe.generate_tokens("a", generation_config={"seed": 1})

    class _BadEngine(_Engine):
        def generate(self, prompt_tokens, attention_mask=None, **kw):
            return np.zeros((1, 1), dtype=np.int32)
    with pytest.raises(ValueError, match="token length must match"):
        TextGenerationPipeline(_BadEngine(), _Tok()).generate_tokens("abc", max_new_tokens=4)


class _Static:
    """Tokenizer returning a fixed encoding (records calls)."""

    def __init__(self, encoded):
        self.encoded, self.calls = encoded, 0

    def __call__(self, texts, **kw):
        self.calls += 1
        return self.encoded

    def batch_decode(self, tokens, **kw):
        return ["x"] * len(tokens)


@pytest.mark.parametrize("kwargs,exc,match", [
    ({"max_new_tokens": True}, TypeError, "max_new_tokens must be an integer"),
    ({"max_new_tokens": -1}, ValueError, "max_new_tokens must be non-negative"),
    ({"top_k": -1}, ValueError, "top_k must be non-negative"),
    ({"include_prompt": 1}, TypeError, "include_prompt must be a boolean"),
    ({"seed": True}, TypeError, "seed must be an integer"),
    ({"temperature": np.nan}, ValueError, "temperature must be finite"),
    ({"fuse_decoding": 1}, TypeError, "fuse_decoding must be a boolean"),
    ({"unknown_option": 1}, TypeError, "unexpected keyword argument"),
])
def test_generation_overrides_are_validated_before_tokenizing(kwargs, exc, match):
    tok, eng = _Static({"input_ids": np.ones((1, 2), dtype=np.int32)}), _Engine()
    pipe = TextGenerationPipeline(eng, tok)
    for fn in (pipe.generate_tokens, pipe.generate_text):
        with pytest.raises(exc, match=match):
            fn("hello", **kwargs)
    assert tok.calls == 0 and eng.calls == []


def test_kwargs_mappings_are_validated_before_tokenizing():
    tok, eng = _Static({"input_ids": np.ones((1, 2), dtype=np.int32)}), _Engine()
    pipe = TextGenerationPipeline(eng, tok)
    with pytest.raises(TypeError, match="tokenize_kwargs must be a mapping"):
        pipe.generate_tokens("hello", tokenize_kwargs=["padding"])
    with pytest.raises(TypeError, match="decode_kwargs must be a mapping"):
        pipe.generate_text("hello", decode_kwargs=["skip_special_tokens"])
    assert tok.calls == 0 and eng.calls == []


@pytest.mark.parametrize("encoded,exc,match", [
    ({"input_ids": np.ones((2,), dtype=np.int32)}, ValueError, "input_ids must be a 2D array"),
    ({"input_ids": np.ones((1, 2), dtype=np.float32)}, TypeError, "integer token ids"),
    ({"input_ids": np.ones((0, 2), dtype=np.int32)}, ValueError, "at least one batch row"),
    ({"input_ids": np.ones((1, 0), dtype=np.int32)}, ValueError, "at least one token"),
    ({"input_ids": np.array([[1, -1]], dtype=np.int32)}, ValueError, "token ids must be non-negative"),
    ({"input_ids": np.ones((1, 2), dtype=np.int32), "attention_mask": np.ones((2,), dtype=np.int32)},
     ValueError, "attention_mask must be a 2D array"),
    ({"input_ids": np.ones((1, 2), dtype=np.int32), "attention_mask": np.ones((1, 2), dtype=np.float32)},
     TypeError, "attention_mask must be boolean or integer"),
    ({"input_ids": np.ones((1, 2), dtype=np.int32), "attention_mask": np.ones((1, 3), dtype=np.int32)},
     ValueError, "attention_mask shape must match"),
    ({"input_ids": np.ones((1, 2), dtype=np.int32), "attention_mask": np.zeros((1, 2), dtype=np.int32)},
     ValueError, "at least one valid token"),
    ({"input_ids": np.ones((1, 2), dtype=np.int32), "attention_mask": np.array([[1, 2]], dtype=np.int32)},
     ValueError, "integer values must be 0 or 1"),
    ({}, ValueError, "tokenizer output must contain 'input_ids'"),
])
def test_tokenizer_arrays_are_validated_before_generation(encoded, exc, match):
    tok, eng = _Static(encoded), _Engine()
    with pytest.raises(exc, match=match):
        TextGenerationPipeline(eng, tok).generate_tokens("hello")
    assert tok.calls == 1 and eng.calls == []


def _no_loading(monkeypatch):
    """Tokenizer and model loaders that record and refuse any call."""
    import transformers

    import jaxml_b200.text_generation as T

    calls = []

    class _AutoTok:
        @classmethod
        def from_pretrained(cls, *a, **k):
            calls.append("tokenizer")
            raise AssertionError("the tokenizer must not be loaded")

    def _load(*a, **k):
        calls.append("model")
        raise AssertionError("the model must not be loaded")

    monkeypatch.setattr(transformers, "AutoTokenizer", _AutoTok)
    monkeypatch.setattr(T, "load_model_from_hf", _load)
    return calls


def test_from_hf_wires_loader_engine_and_tokenizer(monkeypatch):
    """text_generation.py:204-262 (the reference's ``tests/test_text_generation.py:577-620``): the loader,
    the engine and the tokenizer get the arguments as given."""
    import torch

    import jaxml_b200.text_generation as T
    from jaxml_b200 import InferenceConfig

    calls = {}

    class _FakeEngine:
        def __init__(self, model, config, params, dtype, cache_stride):
            calls["engine"] = (model, config, params, dtype, cache_stride)

        def init_params(self, use_tpu):
            calls["use_tpu"] = use_tpu

        def generate(self, *a, **k):
            raise AssertionError("from_hf does not generate")

    def _load(name, architecture, dtype, **kw):
        calls["load"] = (name, architecture, dtype, kw)
        return "model", {"params": "params"}

    monkeypatch.setattr(T, "Engine", _FakeEngine)
    monkeypatch.setattr(T, "load_model_from_hf", _load)
    tok = _Tok()
    cfg = InferenceConfig()
    pipe = TextGenerationPipeline.from_hf("some/model", architecture="llama", model_dtype="bfloat16",
                                          engine_dtype="float32", inference_config=cfg, use_tpu=np.bool_(True),
                                          cache_stride=128, tokenizer=tok, model_kwargs={"trust_remote_code": True})
    assert pipe.tokenizer is tok
    assert calls["load"] == ("some/model", "llama", "bfloat16", {"trust_remote_code": True})
    assert calls["engine"] == ("model", cfg, {"params": "params"}, torch.float32, 128)
    assert calls["use_tpu"] is True


@pytest.mark.parametrize("name,exc,match", [("", ValueError, "non-empty"), ("   ", ValueError, "non-empty"),
                                            (123, TypeError, "string or path-like")])
def test_from_hf_rejects_invalid_names_before_loading(monkeypatch, name, exc, match):
    calls = _no_loading(monkeypatch)
    with pytest.raises(exc, match=match):
        TextGenerationPipeline.from_hf(name)
    assert calls == []


@pytest.mark.parametrize("kwargs,exc,match", [
    ({"architecture": None}, TypeError, "architecture must be a string"),
    ({"architecture": "unknown"}, ValueError, "Unsupported Hugging Face architecture"),
    ({"model_dtype": np.float32}, TypeError, "Expected dtype"),
    ({"model_dtype": "bad"}, ValueError, "Unsupported dtype"),
    ({"engine_dtype": None}, TypeError, "engine_dtype must be a valid"),
    ({"engine_dtype": "not-a-dtype"}, TypeError, "engine_dtype must be a valid"),
    ({"use_tpu": 1}, TypeError, "use_tpu must be a boolean"),
    ({"inference_config": {"tp_size": 1}}, TypeError, "inference_config must be an InferenceConfig"),
    ({"tokenizer_kwargs": [1]}, TypeError, "tokenizer_kwargs must be a mapping"),
    ({"model_kwargs": "x"}, TypeError, "model_kwargs must be a mapping"),
    ({"cache_stride": 0}, ValueError, "cache_stride must be positive"),
    ({"cache_stride": True}, TypeError, "cache_stride must be an integer"),
    ({"tokenizer": object()}, TypeError, "tokenizer must be callable"),
])
def test_from_hf_rejects_invalid_arguments_before_loading(monkeypatch, kwargs, exc, match):
    calls = _no_loading(monkeypatch)
    with pytest.raises(exc, match=match):
        TextGenerationPipeline.from_hf("some/model", **kwargs)
    assert calls == []


def test_from_hf_pathlike_name(monkeypatch, tmp_path):
    import jaxml_b200.text_generation as T

    seen = {}

    class _FakeEngine:
        def __init__(self, *a, **k):
            pass

        def init_params(self, use_tpu):
            pass

        def generate(self, *a, **k):
            raise AssertionError

    def _load(name, architecture, dtype, **kw):
        seen["name"] = name
        return "model", {"params": {}}

    monkeypatch.setattr(T, "Engine", _FakeEngine)
    monkeypatch.setattr(T, "load_model_from_hf", _load)
    TextGenerationPipeline.from_hf(tmp_path, tokenizer=_Tok())
    assert seen["name"] == str(tmp_path)


class _Fixed:
    """An engine returning a fixed token array."""

    def __init__(self, out):
        self.out = out

    def generate(self, *a, **k):
        return self.out


def test_pipeline_construction_checks_and_default_copies():
    """text_generation.py:194-230 (the reference's ``tests/test_text_generation.py:157-200`` cases)."""
    for kw, match in (({"default_tokenize_kwargs": ["padding"]}, "default_tokenize_kwargs must be a mapping"),
                      ({"default_decode_kwargs": ["x"]}, "default_decode_kwargs must be a mapping")):
        with pytest.raises(TypeError, match=match):
            TextGenerationPipeline(engine=_Engine(), tokenizer=_Tok(), **kw)

    class _NoDecode:
        def __call__(self, *a, **k):
            return {}

    for eng, tok, match in ((object(), _Tok(), "engine must provide a callable generate method"),
                            (_Engine(), object(), "tokenizer must be callable"),
                            (_Engine(), _NoDecode(), "batch_decode")):
        with pytest.raises(TypeError, match=match):
            TextGenerationPipeline(engine=eng, tokenizer=tok)
    tk, dk = {"padding": True}, {"skip_special_tokens": True}
    pipe = TextGenerationPipeline(engine=_Engine(), tokenizer=_Tok(), default_tokenize_kwargs=tk,
                                  default_decode_kwargs=dk)
    tk["padding"] = "longest"
    dk["skip_special_tokens"] = False
    assert pipe.default_tokenize_kwargs == {"padding": True}
    assert pipe.default_decode_kwargs == {"skip_special_tokens": True}


@pytest.mark.parametrize("ids,mask,exc,match", [
    (np.ones(2, dtype=np.int32), None, ValueError, "input_ids must be a 2D array"),
    (np.ones((1, 2), dtype=np.float32), None, TypeError, "integer token ids"),
    (np.ones((0, 2), dtype=np.int32), None, ValueError, "at least one batch row"),
    (np.ones((1, 0), dtype=np.int32), None, ValueError, "at least one token"),
    (np.array([[1, -1]], dtype=np.int32), None, ValueError, "token ids must be non-negative"),
    (np.ones((1, 2), dtype=np.int32), np.ones(2, dtype=np.int32), ValueError, "attention_mask must be a 2D array"),
    (np.ones((1, 2), dtype=np.int32), np.ones((1, 2), dtype=np.float32), TypeError, "boolean or integer"),
    (np.ones((1, 2), dtype=np.int32), np.ones((1, 3), dtype=np.int32), ValueError, "attention_mask shape must match"),
    (np.ones((1, 2), dtype=np.int32), np.array([[1, 2]]), ValueError, "integer values must be 0 or 1"),
    (np.ones((1, 2), dtype=np.int32), np.zeros((1, 2), dtype=bool), ValueError, "at least one valid token"),
])
def test_token_arrays_checked_before_the_engine(ids, mask, exc, match):
    eng = _Engine()
    with pytest.raises(exc, match=match):
        TextGenerationPipeline(eng, _Tok())._generate_tokens_from_arrays(ids, mask)
    assert eng.calls == []


def test_integer_mask_reaches_the_engine_as_booleans():
    eng = _Engine()
    TextGenerationPipeline(eng, _Tok())._generate_tokens_from_arrays(np.ones((1, 2), dtype=np.int32),
                                                                     np.array([[1, 0]], dtype=np.int32),
                                                                     max_new_tokens=1)
    mask = eng.calls[0][1]
    assert np.asarray(mask).dtype == np.bool_ and np.asarray(mask).tolist() == [[True, False]]


def test_engine_output_checked_before_decoding():
    ids = "ab"
    for out, exc, match in ((np.ones(3, dtype=np.int32), ValueError, "2D token array"),
                            (np.ones((1, 2), dtype=np.float32), TypeError, "integer token ids"),
                            (np.array([[-1]], dtype=np.int32), ValueError, "token ids must be non-negative"),
                            (np.ones((2, 3), dtype=np.int32), ValueError, "token batch size must match input batch size")):
        with pytest.raises(exc, match=match):
            TextGenerationPipeline(_Fixed(out), _Tok()).generate_text(ids, max_new_tokens=1, include_prompt=False)
    for include, out, expected in ((False, np.ones((1, 0), dtype=np.int32), 1),
                                   (False, np.ones((1, 2), dtype=np.int32), 1),
                                   (True, np.ones((1, 1), dtype=np.int32), 3),
                                   (True, np.ones((1, 4), dtype=np.int32), 3)):
        with pytest.raises(ValueError, match=f"got {out.shape[1]} and expected {expected}"):
            TextGenerationPipeline(_Fixed(out), _Tok()).generate_text(ids, max_new_tokens=1, include_prompt=include)


@pytest.mark.parametrize("decoded,exc,match", [("decoded", TypeError, "sequence of strings"),
                                               (["first", "second"], ValueError, "output batch size must match"),
                                               ([1], TypeError, "sequence of strings")])
def test_decoded_output_checks(decoded, exc, match):
    class _Tok2(_Tok):
        def batch_decode(self, tokens, **kw):
            return decoded

    with pytest.raises(exc, match=match):
        TextGenerationPipeline(_Engine(), _Tok2()).generate_text("ab", max_new_tokens=1)
