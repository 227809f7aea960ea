"""``torch_to_jax_states`` (utils.py:197-371) on CPU: the reference's layout rules and argument checks,
case by case as its ``tests/test_modules.py:725-916`` states them."""
from types import MappingProxyType

import numpy as np
import pytest
import torch

from jaxml_b200.hf_utils import torch_to_jax_states


@pytest.mark.parametrize("dtype", ["bad", torch.int32])
def test_unsupported_dtype(dtype):
    with pytest.raises(ValueError, match="Unsupported dtype"):
        torch_to_jax_states({"weight": torch.ones(1)}, dtype=dtype)


def test_dtype_must_be_a_name_or_torch_dtype():
    with pytest.raises(TypeError, match="Expected dtype"):
        torch_to_jax_states({"weight": torch.ones(1)}, dtype=np.float32)


def test_mapping_and_module_inputs():
    p = torch_to_jax_states(MappingProxyType({"weight": torch.arange(6, dtype=torch.float32).reshape(2, 3)}))
    assert tuple(p["params"]["kernel"].shape) == (3, 2)
    assert torch.equal(p["params"]["kernel"], torch.arange(6, dtype=torch.float32).reshape(2, 3).T)
    with pytest.raises(TypeError, match="PyTorch module or a mapping"):
        torch_to_jax_states([("weight", torch.ones(1))])
    with pytest.raises(ValueError, match="state dict must contain at least one tensor"):
        torch_to_jax_states({})
    with pytest.raises(ValueError, match="state dict must contain at least one tensor"):
        torch_to_jax_states(torch.nn.Identity())
    lin = torch.nn.Linear(3, 2)
    p = torch_to_jax_states(lin)
    assert tuple(p["params"]["kernel"].shape) == (3, 2) and tuple(p["params"]["bias"].shape) == (2,)


@pytest.mark.parametrize("head_dim", [True, np.bool_(True), 1.5])
def test_non_integer_head_dim(head_dim):
    with pytest.raises(TypeError, match="head_dim must be an integer"):
        torch_to_jax_states({"weight": torch.ones(1)}, head_dim=head_dim)


@pytest.mark.parametrize("head_dim", [0, -1])
def test_non_positive_head_dim(head_dim):
    with pytest.raises(ValueError, match="head_dim must be positive"):
        torch_to_jax_states({"weight": torch.ones(1)}, head_dim=head_dim)


def test_projection_layouts():
    p = torch_to_jax_states({"q_proj.weight": torch.ones((4, 8))}, head_dim=np.int64(4))
    assert tuple(p["params"]["q_proj"]["kernel"].shape) == (8, 1, 4)
    w = torch.arange(48, dtype=torch.float32).reshape(6, 8)
    b = torch.arange(6, dtype=torch.float32)
    p = torch_to_jax_states({"qkv_proj.weight": w, "qkv_proj.bias": b})
    assert tuple(p["params"]["qkv_proj"]["kernel"].shape) == (8, 3, 2)
    assert tuple(p["params"]["qkv_proj"]["bias"].shape) == (3, 2)
    # with head_dim: [d, heads, 3, hd] grouping of the fused rows, moved to [d, 3, heads, hd]
    w = torch.arange(12 * 8, dtype=torch.float32).reshape(12, 8)
    p = torch_to_jax_states({"qkv_proj.weight": w}, head_dim=2)
    k = p["params"]["qkv_proj"]["kernel"]
    assert tuple(k.shape) == (8, 3, 2, 2)
    # output row r = (head h, part j, element e) with r = (h * 3 + j) * 2 + e
    assert torch.equal(k[:, 1, 0, 1], w[(0 * 3 + 1) * 2 + 1])
    assert torch.equal(k[:, 2, 1, 0], w[(1 * 3 + 2) * 2 + 0])
    p = torch_to_jax_states({"embed_tokens.weight": torch.ones(5, 3), "model.norm.weight": torch.ones(3)})
    assert tuple(p["params"]["embed_tokens"]["embedding"].shape) == (5, 3)
    assert tuple(p["params"]["model"]["norm"]["weight"].shape) == (3,)


@pytest.mark.parametrize("state,match", [
    ({"qkv_proj.weight": torch.ones((5, 8))}, "Fused QKV projection output dimension"),
    ({"qkv_proj.bias": torch.ones(5)}, "Fused QKV projection bias length"),
])
def test_fused_qkv_not_divisible_by_three(state, match):
    with pytest.raises(ValueError, match=match):
        torch_to_jax_states(state)


@pytest.mark.parametrize("state,match", [
    ({"q_proj.weight": torch.ones((5, 8))}, "Q/K/V projection output dimension"),
    ({"k_proj.bias": torch.ones(5)}, "Q/K/V projection bias length"),
    ({"qkv_proj.weight": torch.ones((10, 8))}, "Fused QKV projection output dimension"),
    ({"qkv_proj.bias": torch.ones(10)}, "Fused QKV projection bias length"),
])
def test_projection_shapes_incompatible_with_head_dim(state, match):
    with pytest.raises(ValueError, match=match):
        torch_to_jax_states(state, head_dim=4)


def test_state_value_checks():
    with pytest.raises(TypeError, match="State value for key 'weight'"):
        torch_to_jax_states({"weight": np.ones(1)})
    for dt in (torch.bool, torch.int32, torch.int64):
        with pytest.raises(TypeError, match="must contain floating point values"):
            torch_to_jax_states({"weight": torch.ones((2, 3), dtype=dt)})
    for v in (float("nan"), float("inf"), -float("inf")):
        with pytest.raises(ValueError, match="must contain only finite values"):
            torch_to_jax_states({"weight": torch.tensor([[0.0, v]])})
    for state in ({"bias": torch.empty(0)}, {"weight": torch.empty((0, 4))}, {"q_proj.weight": torch.empty((4, 0))}):
        with pytest.raises(ValueError, match="must not be empty"):
            torch_to_jax_states(state)


def test_grad_and_bfloat16_sources():
    p = torch_to_jax_states({"bias": torch.tensor([1.0, 2.0], requires_grad=True)})
    assert not p["params"]["bias"].requires_grad and p["params"]["bias"].tolist() == [1.0, 2.0]
    p = torch_to_jax_states({"bias": torch.tensor([1.0, 2.0], dtype=torch.bfloat16)}, dtype="bfloat16")
    assert p["params"]["bias"].dtype == torch.bfloat16 and p["params"]["bias"].float().tolist() == [1.0, 2.0]


def test_state_keys():
    with pytest.raises(TypeError, match="State key must be a string"):
        torch_to_jax_states({1: torch.ones(1)})
    for key in ("", ".weight", "stack..weight", "stack.weight."):
        with pytest.raises(ValueError, match="State key"):
            torch_to_jax_states({key: torch.ones(1)})
    p = torch_to_jax_states({"encoder.0.block.1.weight": torch.ones((2, 3))})
    assert tuple(p["params"]["encoder_0"]["block_1"]["kernel"].shape) == (3, 2)
    p = torch_to_jax_states({"stack.0.1.weight": torch.ones((2, 3))})
    assert tuple(p["params"]["stack_0_1"]["kernel"].shape) == (3, 2)
    with pytest.raises(ValueError, match="Multiple state keys map"):
        torch_to_jax_states({"stack.0.weight": torch.ones((2, 3)), "stack_0.weight": torch.ones((2, 3))})
    with pytest.raises(ValueError, match="conflicts with existing leaf"):
        torch_to_jax_states({"stack.bias": torch.ones((2, 3)), "stack.bias.extra": torch.ones((2, 3))})
