"""The oracle against committed golden outputs of HF transformers' eager models (``tests/golden``,
made by ``tests/golden/make_golden.py``): last-position logits within ``atol=1e-5`` and identical greedy
tokens in float32, as the reference pins jaxml (``tests/test_llama.py:82-134``, ``test_neox.py:17-90``,
``test_gemma.py:71-122``).  Needs no HF at test time."""
import json
import os

import numpy as np
import pytest
import torch

from jaxml_b200.config import ModelConfig
from oracle import jaxml_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "hf_tiny.npz")


def load_family(family):
    """(ModelConfig, Flax-layout params as torch tensors, input ids, golden last logits, golden greedy ids)."""
    z = np.load(GOLDEN)
    fields = json.loads(bytes(z[f"{family}:model_config"]).decode())
    if isinstance(fields.get("intermediate_ratio"), list):
        fields["intermediate_ratio"] = tuple(fields["intermediate_ratio"])
    cfg = ModelConfig(**fields)
    params = {}
    prefix = f"{family}:param:"
    for key in z.files:
        if not key.startswith(prefix):
            continue
        node = params
        parts = key[len(prefix):].split("/")
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        node[parts[-1]] = torch.from_numpy(z[key].copy())
    ids = torch.from_numpy(z["input_ids"].copy())
    return cfg, params, ids, torch.from_numpy(z[f"{family}:logits_last"].copy()), torch.from_numpy(z[f"{family}:greedy"].copy())


@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_oracle_matches_golden_hf_outputs(family):
    cfg, params, ids, logits, greedy = load_family(family)
    out = O.forward(family, cfg, params, ids, torch.float32)
    assert np.allclose(out.logits[:, -1].numpy(), logits.numpy(), atol=1e-5)
    toks = O.generate(family, cfg, params, ids, torch.float32, max_new_tokens=greedy.shape[1] - ids.shape[1],
                      temperature=0.0)
    assert torch.equal(toks.to(torch.int32), greedy)
