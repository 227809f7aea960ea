"""The decoder building blocks (``LlamaMLP`` / ``LlamaDecoder`` and siblings) on CPU: fields, parameter
names and shapes from ``init``, and the input checks of models/_utils.py:37-49 (``validate_mlp_input``)
and the block ``setup`` methods.  ``apply`` runs on the GPU kernels (``test_gpu_model_apply.py``)."""
import numpy as np
import pytest
import torch

from jaxml_b200 import ModelConfig
from jaxml_b200.models import (GemmaDecoder, GemmaMLP, GPTNeoXDecoder, GPTNeoXMLP, LlamaDecoder, LlamaMLP)


def _cfg(**kw):
    base = dict(head_dim=8, hidden_size=32, num_heads=4, num_kv_heads=2, num_layers=1, intermediate_ratio=(3, 2),
                max_position_embeddings=64, vocab_size=50)
    base.update(kw)
    return ModelConfig(**base)


@pytest.mark.parametrize("cls,names", [(LlamaMLP, {"gate_proj", "up_proj", "down_proj"}),
                                       (GemmaMLP, {"gate_proj", "up_proj", "down_proj"}),
                                       (GPTNeoXMLP, {"up_proj", "down_proj"})])
def test_mlp_init_parameter_tree(cls, names):
    v = cls(_cfg()).init(0, torch.zeros(1, 3, 32))
    p = v["params"]
    assert set(p) == names
    assert tuple(p["up_proj"]["kernel"].shape) == (32, 48)
    assert tuple(p["down_proj"]["kernel"].shape) == (48, 32)
    if "gate_proj" in p:
        assert tuple(p["gate_proj"]["kernel"].shape) == (32, 48)
    assert all("bias" not in p[n] for n in p)
    pb = cls(_cfg(use_bias=True)).init(0, torch.zeros(1, 3, 32))["params"]
    assert all(tuple(pb[n]["bias"].shape) == (pb[n]["kernel"].shape[1],) for n in pb)


@pytest.mark.parametrize("cls", [LlamaMLP, GemmaMLP, GPTNeoXMLP])
@pytest.mark.parametrize("x,exc,match", [
    (torch.zeros(3, 32), ValueError, "input must be a 3D array"),
    (torch.zeros(1, 3, 32, dtype=torch.int32), TypeError, "floating point"),
    (torch.zeros(1, 0, 32), ValueError, "empty axes"),
    (torch.zeros(1, 3, 16), ValueError, "hidden dimension mismatch"),
    (torch.full((1, 3, 32), float("nan")), ValueError, "only finite values"),
])
def test_mlp_input_checks(cls, x, exc, match):
    m = cls(_cfg())
    with pytest.raises(exc, match=match):
        m.init(0, x)
    with pytest.raises(exc, match=cls.__name__):
        m.apply({"params": {}}, x)


def test_mlp_custom_activation_is_not_implemented():
    with pytest.raises(NotImplementedError, match="act_fn"):
        LlamaMLP(_cfg(), act_fn=lambda x: x).init(0, torch.zeros(1, 1, 32))


@pytest.mark.parametrize("cls,norms,attn", [
    (LlamaDecoder, {"input_layernorm", "post_attention_layernorm"}, {"q_proj", "k_proj", "v_proj", "o_proj"}),
    (GemmaDecoder, {"input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                    "post_feedforward_layernorm"}, {"q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"}),
])
def test_decoder_init_parameter_tree(cls, norms, attn):
    p = cls(_cfg()).init(0, torch.zeros(1, 3, 32))["params"]
    assert set(p) == norms | {"self_attn", "mlp"}
    assert set(p["self_attn"]) == attn
    assert tuple(p["self_attn"]["k_proj"]["kernel"].shape) == (32, 2, 8)
    for n in norms:
        assert tuple(p[n]["weight"].shape) == (32,)
    if cls is GemmaDecoder:
        assert tuple(p["self_attn"]["q_norm"]["weight"].shape) == (8,)
        assert float(p["input_layernorm"]["weight"].abs().sum()) == 0.0   # Gemma norms start at zero


def test_neox_decoder_init_parameter_tree():
    cfg = _cfg(num_kv_heads=4, use_bias=True)
    p = GPTNeoXDecoder(cfg).init(0, torch.zeros(1, 3, 32))["params"]
    assert set(p["self_attn"]) == {"qkv_proj", "o_proj"}
    assert tuple(p["self_attn"]["qkv_proj"]["kernel"].shape) == (32, 3, 4, 8)
    assert set(p["input_layernorm"]) == {"weight", "bias"}
    assert set(p["mlp"]) == {"up_proj", "down_proj"}


def test_decoder_setup_checks():
    with pytest.raises(ValueError, match="Llama hidden_size must equal num_heads \\* head_dim"):
        LlamaDecoder(_cfg(hidden_size=40)).init(0, torch.zeros(1, 1, 40))
    with pytest.raises(ValueError, match="GPT-NeoX hidden_size must equal"):
        GPTNeoXDecoder(_cfg(hidden_size=40, num_kv_heads=4)).init(0, torch.zeros(1, 1, 40))
    with pytest.raises(ValueError, match="fused_qkv requires num_heads to equal num_key_value_heads"):
        GPTNeoXDecoder(_cfg()).init(0, torch.zeros(1, 1, 32))
    with pytest.raises(ValueError, match="Gemma3 decoder requires use_rope=True"):
        GemmaDecoder(_cfg(use_rope=False)).init(0, torch.zeros(1, 1, 32))
    with pytest.raises(TypeError, match="use_sliding must be a boolean"):
        GemmaDecoder(_cfg(), use_sliding=1).init(0, torch.zeros(1, 1, 32))
    # Gemma's head dim is free of the hidden size (no hidden_size == heads * head_dim rule)
    GemmaDecoder(_cfg(hidden_size=40)).init(0, torch.zeros(1, 1, 40))
    with pytest.raises(TypeError, match="config must be a ModelConfig"):
        LlamaDecoder(None).init(0, torch.zeros(1, 1, 32))
    with pytest.raises(ValueError, match="input must be a 3D array"):
        LlamaDecoder(_cfg()).init(0, np.zeros((1, 32), dtype=np.float32))
