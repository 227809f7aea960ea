"""Generates ``hf_tiny.npz``: golden logits and greedy tokens of tiny HF transformers models (Llama,
GPT-NeoX, Gemma3; float32, eager attention, random init with seed 0), with their parameters in the
reference's Flax layout, so the oracle (and the float32 runtime) can be checked against them without
HF at test time.  The reference pins jaxml the same way (``tests/test_llama.py:82-134``,
``tests/test_neox.py:17-90``, ``tests/test_gemma.py:71-122``: HF eager models, ``atol=1e-5``, greedy
tokens identical).

Run from the repository root: ``python tests/golden/make_golden.py`` (needs ``transformers``).
"""
import dataclasses
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "hf_tiny.npz")


def configs():
    from transformers import Gemma3TextConfig, GPTNeoXConfig, LlamaConfig

    llama = LlamaConfig(hidden_size=32, intermediate_size=64, num_hidden_layers=2, max_position_embeddings=64,
                        vocab_size=128, num_attention_heads=4, num_key_value_heads=2, hidden_act="silu",
                        rms_norm_eps=1e-6, rope_theta=10000.0, attn_implementation="eager")
    neox = GPTNeoXConfig(hidden_size=32, intermediate_size=64, num_hidden_layers=2, max_position_embeddings=64,
                         vocab_size=128, num_attention_heads=4, hidden_act="gelu", layer_norm_eps=1e-5,
                         rotary_emb_base=10000.0, rotary_pct=0.25, use_parallel_residual=True,
                         attn_implementation="eager", attention_bias=True)
    gemma = Gemma3TextConfig(hidden_size=32, head_dim=8, intermediate_size=64, num_hidden_layers=2,
                             max_position_embeddings=64, vocab_size=128, num_attention_heads=4,
                             num_key_value_heads=2, sliding_window=4, sliding_window_pattern=2,
                             attn_implementation="eager")
    return {"llama": llama, "neox": neox, "gemma3": gemma}


def flatten(tree, prefix=""):
    out = {}
    for k, v in tree.items():
        key = f"{prefix}/{k}" if prefix else k
        if isinstance(v, dict):
            out.update(flatten(v, key))
        else:
            out[key] = np.asarray(v.detach().cpu() if isinstance(v, torch.Tensor) else v, dtype=np.float32)
    return out


def main():
    from transformers import Gemma3ForCausalLM, GPTNeoXForCausalLM, LlamaForCausalLM

    from jaxml_b200.config import ModelConfig
    from jaxml_b200.hf_utils import to_gemma_jax_params, to_llama_jax_params, to_neox_jax_params

    arrays = {}
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 127, (2, 7), generator=g, dtype=torch.int64)
    arrays["input_ids"] = ids.numpy().astype(np.int32)
    for family, cls, conv in (("llama", LlamaForCausalLM, to_llama_jax_params),
                              ("neox", GPTNeoXForCausalLM, to_neox_jax_params),
                              ("gemma3", Gemma3ForCausalLM, to_gemma_jax_params)):
        torch.manual_seed(0)
        cfg = configs()[family]
        model = cls(cfg).eval()
        if family == "gemma3":
            with torch.no_grad():
                for name, p in model.named_parameters():
                    if "norm" in name:
                        p.normal_(0.0, 0.1)
        params = conv(model, dtype=torch.float32)
        if "lm_head" not in params["params"]:
            emb = params["params"]["model"]["embed_tokens"]["embedding"]
            params["params"]["lm_head"] = {"kernel": emb.T.contiguous()}
        for k, v in flatten(params).items():
            arrays[f"{family}:param:{k}"] = v
        with torch.no_grad():
            logits = model(ids).logits[:, -1].float()
            toks = ids.clone()
            for _ in range(8):
                nxt = model(input_ids=toks).logits[:, -1].argmax(-1, keepdim=True)
                toks = torch.cat([toks, nxt], dim=-1)
        arrays[f"{family}:logits_last"] = logits.numpy().astype(np.float32)
        arrays[f"{family}:greedy"] = toks.numpy().astype(np.int32)
        mc = ModelConfig.from_hf(cfg)
        fields = {f.name: getattr(mc, f.name) for f in dataclasses.fields(mc)}
        arrays[f"{family}:model_config"] = np.frombuffer(json.dumps(fields).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT}: {os.path.getsize(OUT)} bytes, {len(arrays)} arrays")


if __name__ == "__main__":
    main()
