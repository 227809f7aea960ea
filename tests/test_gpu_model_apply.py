"""``*ModelWithHead.apply`` (the reference's model call without a cache) on the GPU kernels against the
oracle: all-position logits, the last-n slice, and a right-padded mask."""
import pytest
import torch

from jaxml_b200 import GemmaModelWithHead, GPTNeoXModelWithHead, LlamaModelWithHead
from oracle import jaxml_oracle as O

pytestmark = pytest.mark.gpu

CLASSES = {"llama": LlamaModelWithHead, "neox": GPTNeoXModelWithHead, "gemma3": GemmaModelWithHead}


def _close(got, want, dtype):
    got, want = got.float().cpu(), want.float().cpu()
    if dtype == torch.float32:
        assert torch.allclose(got, want, rtol=1e-4, atol=1e-5), (got - want).abs().max().item()
    else:
        assert (got - want).abs().max().item() <= 2e-2, (got - want).abs().max().item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_model_apply_matches_oracle(family, dtype, hf_models):
    _, cfg, params = hf_models[family]
    model = CLASSES[family](cfg, dtype=dtype)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (3, 9), generator=g, dtype=torch.int32)
    want = O.forward(family, cfg, params, ids, dtype).logits
    out = model.apply(params, ids)
    assert tuple(out.logits.shape) == (3, 9, cfg.vocab_size) and out.logits.dtype == dtype
    _close(out.logits, want, dtype)
    last = model.apply(params, ids, keep_last_n_logits=2).logits
    assert tuple(last.shape) == (3, 2, cfg.vocab_size)
    _close(last, want[:, -2:], dtype)
    if dtype == torch.float32:
        mask = torch.ones(3, 9, dtype=torch.bool)
        mask[1, 6:] = False
        got = model.apply(params, ids, attention_mask=mask).logits
        ref = O.forward(family, cfg, params, ids, dtype, attention_mask=mask).logits
        _close(got[0], ref[0], dtype)
        _close(got[1, :6], ref[1, :6], dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_stack_model_apply_matches_oracle(family, dtype, hf_models):
    """``*Model.apply``: the final-norm hidden states of every position against the oracle's."""
    from jaxml_b200.models import GemmaModel, GPTNeoXModel, LlamaModel

    _, cfg, params = hf_models[family]
    cls = {"llama": LlamaModel, "neox": GPTNeoXModel, "gemma3": GemmaModel}[family]
    body = "gpt_neox" if family == "neox" else "model"
    model = cls(cfg, dtype=dtype)
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, cfg.vocab_size, (2, 11), generator=g, dtype=torch.int32)
    want = O.forward(family, cfg, params, ids, dtype).last_hidden_state
    out = model.apply({"params": params["params"][body]}, ids).last_hidden_state
    assert tuple(out.shape) == (2, 11, cfg.hidden_size) and out.dtype == dtype
    _close(out, want, dtype)
