"""``*ModelWithHead.apply`` input checks (the reference's ``tests/test_model_inputs.py`` cases): all
raised before any device work, so they run on CPU."""
import numpy as np
import pytest
import torch

from jaxml_b200 import GemmaModelWithHead, GPTNeoXModelWithHead, LlamaModelWithHead, ModelConfig
from jaxml_b200.models import random_params


def _models():
    cfg = ModelConfig(head_dim=8, hidden_size=32, num_heads=4, num_kv_heads=4, num_layers=1,
                      max_position_embeddings=64, vocab_size=50)
    return [(cls(cfg), random_params(fam, cfg)) for cls, fam in ((LlamaModelWithHead, "llama"),
                                                                 (GPTNeoXModelWithHead, "neox"),
                                                                 (GemmaModelWithHead, "gemma3"))]


MODELS = _models()


@pytest.mark.parametrize("mp", MODELS, ids=["llama", "neox", "gemma3"])
@pytest.mark.parametrize("ids,exc,match", [
    (torch.arange(4, dtype=torch.int32), ValueError, "input_ids must be a 2D array"),
    (torch.ones(1, 2, 1, dtype=torch.int32), ValueError, "input_ids must be a 2D array"),
    (torch.ones(1, 4), TypeError, "integer token ids"),
    (torch.ones(0, 4, dtype=torch.int32), ValueError, "at least one batch row"),
    (torch.ones(1, 0, dtype=torch.int32), ValueError, "at least one token"),
    (torch.tensor([[0, 50]], dtype=torch.int32), ValueError, "less than vocab_size"),
    (torch.tensor([[-100, -100]], dtype=torch.int32), ValueError, "at least one non-negative token"),
])
def test_invalid_input_ids(mp, ids, exc, match):
    model, params = mp
    with pytest.raises(exc, match=match):
        model.apply(params, ids)


@pytest.mark.parametrize("mask,exc,match", [
    (torch.ones(4, dtype=torch.bool), ValueError, "attention_mask must be a 2D array"),
    (torch.ones(1, 2, 1, dtype=torch.bool), ValueError, "attention_mask must be a 2D array"),
    (torch.ones(1, 3, dtype=torch.bool), ValueError, "attention_mask shape must match"),
    (torch.ones(1, 4), TypeError, "attention_mask must be boolean or integer"),
    (torch.tensor([[1, 2, 1, 1]], dtype=torch.int32), ValueError, "integer values must be 0 or 1"),
    (torch.tensor([[1, -1, 1, 1]], dtype=torch.int32), ValueError, "integer values must be 0 or 1"),
])
def test_invalid_attention_mask(mask, exc, match):
    model, params = MODELS[0]
    with pytest.raises(exc, match=match):
        model.apply(params, torch.arange(4, dtype=torch.int32)[None], attention_mask=mask)


def test_mask_contents():
    model, params = MODELS[0]
    ids = torch.arange(4, dtype=torch.int32)[None].repeat(2, 1)
    with pytest.raises(ValueError, match="at least one valid token"):
        model.apply(params, ids, attention_mask=torch.tensor([[1, 1, 0, 0], [0, 0, 0, 0]], dtype=torch.bool))
    with pytest.raises(ValueError, match="must not mark negative placeholder"):
        model.apply(params, torch.tensor([[1, -100]], dtype=torch.int32), attention_mask=np.array([[1, 1]]))
    # placeholders before the tokens make a left-padded mask, which the kernels do not take
    with pytest.raises(NotImplementedError, match="right-padded"):
        model.apply(params, torch.tensor([[-100, 1]], dtype=torch.int32))


def test_flag_types():
    model, params = MODELS[0]
    ids = torch.ones(1, 3, dtype=torch.int32)
    for kw, match in (({"use_cache": 1}, "use_cache must be a boolean"),
                      ({"use_cache": None}, "use_cache must be a boolean"),
                      ({"output_attentions": 1}, "output_attentions must be a boolean"),
                      ({"output_hidden_states": "true"}, "output_hidden_states must be a boolean")):
        with pytest.raises(TypeError, match=match):
            model.apply(params, ids, **kw)
    for keep, exc, match in ((True, TypeError, "keep_last_n_logits must be an integer"),
                             (np.bool_(True), TypeError, "keep_last_n_logits must be an integer"),
                             (1.5, TypeError, "keep_last_n_logits must be an integer"),
                             (-1, ValueError, "keep_last_n_logits must be non-negative")):
        with pytest.raises(exc, match=match):
            model.apply(params, ids, keep_last_n_logits=keep)


@pytest.mark.parametrize("pos,exc,match", [
    (torch.arange(4, dtype=torch.int32), ValueError, "position_ids must be a 2D array"),
    (torch.ones(1, 4), TypeError, "integer positions"),
    (torch.ones(1, 3, dtype=torch.int32), ValueError, "position_ids shape must be broadcastable"),
    (torch.tensor([[-1, 0, 1, 2]], dtype=torch.int32), ValueError, "non-negative positions"),
    (torch.tensor([[0, 1, 2, 64]], dtype=torch.int32), ValueError, "less than max_position_embeddings=64"),
])
def test_invalid_position_ids(pos, exc, match):
    model, params = MODELS[0]
    with pytest.raises(exc, match=match):
        model.apply(params, torch.arange(4, dtype=torch.int32)[None], position_ids=pos)


def _populated(B=1, T=8, n=2, mask_dtype=torch.bool):
    from jaxml_b200.cache import KVCache

    k = torch.randn(B, n, 4, 8)
    return KVCache.init(T, k=k, v=torch.randn_like(k), mask=torch.ones(B, n, dtype=mask_dtype))


def test_kv_cache_argument_checks():
    """models/_utils.py:99-177 checks on the caches, raised before any device work (the reference's
    ``tests/test_model_inputs.py`` cases)."""
    from jaxml_b200.cache import KVCache

    model, params = MODELS[0]
    ids = torch.tensor([[2]], dtype=torch.int32)
    with pytest.raises(ValueError, match="one cache per layer"):
        model.apply(params, ids, kv_caches=())
    with pytest.raises(TypeError, match="kv_caches must be a sequence"):
        model.apply(params, ids, kv_caches=3)
    with pytest.raises(TypeError, match="KVCache instances or None"):
        model.apply(params, ids, kv_caches=(object(),))
    bad = KVCache(k=None, v=torch.zeros(1), max_seq_len=8, mask=None)
    with pytest.raises(ValueError, match="k is empty"):
        model.apply(params, ids, kv_caches=(bad,))
    c = _populated()
    with pytest.raises(TypeError, match="Cached mask must be boolean"):
        model.apply(params, ids, kv_caches=(c.replace(mask=c.mask.to(torch.int32)),))
    # a populated cache carries the mask: a token-shaped mask no longer fits
    with pytest.raises(ValueError, match="populated KV cache mask shape"):
        model.apply(params, ids, attention_mask=torch.ones(1, 1, dtype=torch.bool), kv_caches=(c,))
    with pytest.raises(ValueError, match="attention_mask is not token-shaped"):
        model.apply(params, torch.tensor([[-100]], dtype=torch.int32), attention_mask=c.mask, kv_caches=(c,))
    with pytest.raises(ValueError, match="using populated KV caches"):
        model.apply(params, torch.tensor([[-100]], dtype=torch.int32), kv_caches=(c,))
    with pytest.raises(ValueError, match="share input_ids batch size"):
        model.apply(params, torch.ones(2, 1, dtype=torch.int32), kv_caches=(c,))


def test_kv_cache_mask_shapes_must_agree():
    from jaxml_b200.models import _prepare_model_inputs

    cfg = ModelConfig(head_dim=8, hidden_size=32, num_heads=4, num_layers=2, max_position_embeddings=64,
                      vocab_size=50)
    with pytest.raises(ValueError, match="share attention mask shape"):
        _prepare_model_inputs(cfg, torch.ones(1, 1, dtype=torch.int32), None, (_populated(T=8), _populated(T=9)))
    from jaxml_b200.decoders import _cached_sequence_length

    with pytest.raises(ValueError, match="share cached sequence length"):
        _cached_sequence_length((_populated(T=8), _populated(T=9)))
    assert _cached_sequence_length((None, _populated(T=9))) == 9
    # populated caches supply the mask: none is built from the ids
    ids, mask, caches, pos = _prepare_model_inputs(cfg, torch.ones(1, 1, dtype=torch.int32), None,
                                                   (_populated(), None))
    assert mask is None and len(caches) == 2 and pos is None
    # empty caches keep the default mask (ids >= 0)
    ids, mask, _, _ = _prepare_model_inputs(cfg, torch.tensor([[3, -1]]), None, (None, None))
    assert mask.tolist() == [[True, False]] and ids.tolist() == [[3, 0]]


@pytest.mark.parametrize("fam", ["llama", "neox", "gemma3"])
def test_stack_model_init_and_input_checks(fam):
    """``*Model`` (the stack without the head) takes the body subtree and applies the same input checks."""
    from jaxml_b200.models import GemmaModel, GPTNeoXModel, LlamaModel

    cls = {"llama": LlamaModel, "neox": GPTNeoXModel, "gemma3": GemmaModel}[fam]
    cfg = ModelConfig(head_dim=8, hidden_size=32, num_heads=4, num_kv_heads=4, num_layers=1,
                      max_position_embeddings=64, vocab_size=50)
    model = cls(cfg)
    params = model.init(0)
    assert "embed_tokens" in params["params"] and "lm_head" not in params["params"]
    body = "gpt_neox" if fam == "neox" else "model"
    full = random_params(fam, cfg, seed=0)["params"][body]
    for k in full["embed_tokens"]:
        assert torch.equal(torch.as_tensor(params["params"]["embed_tokens"][k]), torch.as_tensor(full["embed_tokens"][k]))
    tree = model._full_tree(params)
    assert set(tree["params"]) == {body, "lm_head"}
    assert tuple(tree["params"]["lm_head"]["kernel"].shape) == (32, 50)
    with pytest.raises(ValueError, match="input_ids must be a 2D array"):
        model.apply(params, torch.arange(4, dtype=torch.int32))
    with pytest.raises(ValueError, match="less than vocab_size"):
        model.apply(params, torch.tensor([[0, 50]], dtype=torch.int32))
    with pytest.raises(TypeError, match="output_attentions must be a boolean"):
        model.apply(params, torch.ones(1, 4, dtype=torch.int32), output_attentions=1)
    with pytest.raises(ValueError, match="one cache per layer"):
        model.apply(params, torch.ones(1, 4, dtype=torch.int32), kv_caches=(None, None))


def test_model_init_takes_a_seed_or_a_key_and_checks_example_ids():
    model, _ = MODELS[0]
    a = model.init(0)
    b = model.init(np.array([0, 0], dtype=np.uint32))
    c = model.init(np.array([0, 7], dtype=np.uint32), torch.ones(1, 4, dtype=torch.int32))
    d = model.init(7)
    k = "model"
    emb = [t["params"][k]["embed_tokens"]["embedding"] for t in (a, b, c, d)]
    assert torch.equal(emb[0], emb[1]) and torch.equal(emb[2], emb[3]) and not torch.equal(emb[0], emb[2])
    with pytest.raises(ValueError, match="input_ids must be a 2D array"):
        model.init(0, torch.arange(4, dtype=torch.int32))
    with pytest.raises(ValueError, match="less than vocab_size"):
        model.init(0, torch.tensor([[0, 50]], dtype=torch.int32))


@pytest.mark.parametrize("fam", ["llama", "neox", "gemma3"])
def test_init_holds_the_rotary_tables_in_the_model_dtype(fam):
    """The reference's ``tests/test_model_inputs.py:294-320`` case: the ``cache`` collection of ``init``
    holds the rotary tables (and Gemma's local ones) in the model dtype."""
    from jaxml_b200.models import GemmaModel, GPTNeoXModel, LlamaModel

    cfg = ModelConfig(head_dim=8, hidden_size=32, num_heads=4, num_kv_heads=4, num_layers=2,
                      max_position_embeddings=64, vocab_size=50, **({"sliding_window": 4, "sliding_window_pattern": 2}
                                                                     if fam == "gemma3" else {}))
    cls = {"llama": LlamaModel, "neox": GPTNeoXModel, "gemma3": GemmaModel}[fam]
    v = cls(cfg, dtype=torch.bfloat16).init(0, torch.tensor([[0, 1]], dtype=torch.int32))
    names = ["rotary_emb"] + (["rotary_emb_local"] if fam == "gemma3" else [])
    assert sorted(v["cache"]) == names
    for n in names:
        assert v["cache"][n]["cos_cached"].dtype == torch.bfloat16 and v["cache"][n]["sin_cached"].dtype == torch.bfloat16
        assert tuple(v["cache"][n]["cos_cached"].shape) == (64, 8)
    head = {"llama": LlamaModelWithHead, "neox": GPTNeoXModelWithHead, "gemma3": GemmaModelWithHead}[fam]
    w = head(cfg).init(0)
    assert set(w) == {"params", "cache"} and set(w["cache"]) == {"gpt_neox" if fam == "neox" else "model"}


def test_block_properties():
    model, _ = MODELS[0]
    cfg = model.config
    assert (model.num_layers, model.head_dim, model.hidden_size, model.num_heads) == (
        cfg.num_layers, cfg.head_dim, cfg.hidden_size, cfg.num_heads)
    assert (model.intermediate_size, model.norm_eps, model.use_bias, model.attn_scale) == (
        cfg.intermediate_size, cfg.norm_eps, cfg.use_bias, cfg.attn_scale)
