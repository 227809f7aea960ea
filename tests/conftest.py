import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built native library")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


def _hf_configs():
    from transformers import Gemma3TextConfig, GPTNeoXConfig, LlamaConfig

    # The reference's tiny test configurations (tests/conftest.py:54-110 of the reference).
    llama = LlamaConfig(hidden_size=48, intermediate_size=144, num_hidden_layers=2, max_position_embeddings=256,
                        vocab_size=1024, num_attention_heads=6, num_key_value_heads=3, hidden_act="silu",
                        rms_norm_eps=1e-6, attn_implementation="eager")
    neox = GPTNeoXConfig(hidden_size=48, intermediate_size=144, num_hidden_layers=2, max_position_embeddings=256,
                         vocab_size=1024, num_attention_heads=6, hidden_act="gelu", layer_norm_eps=1e-6,
                         rotary_emb_base=10000.0, rotary_pct=0.5, use_parallel_residual=True,
                         attn_implementation="eager", attention_bias=True)
    gemma = Gemma3TextConfig(hidden_size=48, head_dim=8, intermediate_size=144, num_hidden_layers=4,
                             max_position_embeddings=256, vocab_size=1024, num_attention_heads=6,
                             num_key_value_heads=3, rope_scaling={"factor": 8.0, "rope_type": "linear"},
                             sliding_window=32, sliding_window_pattern=2, use_parallel_residual=True,
                             attn_implementation="eager")
    return {"llama": llama, "neox": neox, "gemma3": gemma}


@pytest.fixture(scope="session")
def hf_models():
    """HF eager torch models with random init (seed 0) and their Flax-layout parameter trees."""
    import torch
    from transformers import Gemma3ForCausalLM, GPTNeoXForCausalLM, LlamaForCausalLM

    from jaxml_b200.config import ModelConfig
    from jaxml_b200.hf_utils import to_gemma_jax_params, to_llama_jax_params, to_neox_jax_params

    cfgs = _hf_configs()
    out = {}
    for family, cls, conv in (("llama", LlamaForCausalLM, to_llama_jax_params),
                              ("neox", GPTNeoXForCausalLM, to_neox_jax_params),
                              ("gemma3", Gemma3ForCausalLM, to_gemma_jax_params)):
        torch.manual_seed(0)
        model = cls(cfgs[family]).eval()
        if family == "gemma3":
            # Random norm weights make the (1 + w) scaling visible in the comparison.
            with torch.no_grad():
                for name, p in model.named_parameters():
                    if "norm" in name:
                        p.normal_(0.0, 0.1)
        params = conv(model, dtype=torch.float32)
        if "lm_head" not in params["params"]:
            emb = params["params"]["model"]["embed_tokens"]["embedding"]
            params["params"]["lm_head"] = {"kernel": emb.T.contiguous()}
        out[family] = (model, ModelConfig.from_hf(cfgs[family]), params)
    return out
