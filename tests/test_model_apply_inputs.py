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


def test_unsupported_options():
    model, params = MODELS[0]
    ids = torch.ones(1, 3, dtype=torch.int32)
    for kw in ({"use_cache": True}, {"kv_caches": ()}, {"position_ids": torch.zeros(1, 3, dtype=torch.int32)}):
        with pytest.raises(NotImplementedError):
            model.apply(params, ids, **kw)
    for kw in ({"output_attentions": True}, {"output_hidden_states": True}):
        with pytest.raises(NotImplementedError):
            model.apply(params, ids, **kw)
    with pytest.raises(TypeError, match="use_cache must be a boolean"):
        model.apply(params, ids, use_cache=1)
    with pytest.raises(ValueError, match="keep_last_n_logits must be non-negative"):
        model.apply(params, ids, keep_last_n_logits=-1)


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
    with pytest.raises(NotImplementedError, match="KV caches"):
        model.apply(params, torch.ones(1, 4, dtype=torch.int32), use_cache=True)
    with pytest.raises(NotImplementedError, match="hidden states"):
        model.apply(params, torch.ones(1, 4, dtype=torch.int32), output_hidden_states=True)
