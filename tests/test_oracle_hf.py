"""Pins the CPU oracle against HF transformers, the way the reference pins jaxml.

Same models, tolerance (``atol=1e-5``, float32) and greedy-token identity as the reference's
``tests/test_llama.py:82-134``, ``tests/test_neox.py:17-90`` and ``tests/test_gemma.py:71-122``.
"""
import numpy as np
import pytest
import torch

from oracle import jaxml_oracle as O

FAMILIES = ["llama", "neox", "gemma3"]


def _ids(cfg, bs=4, seq=10, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab_size - 1, (bs, seq), generator=g, dtype=torch.int32)


@pytest.mark.parametrize("family", FAMILIES)
def test_oracle_model_matches_hf(family, hf_models):
    model, cfg, params = hf_models[family]
    x = _ids(cfg)
    out = O.forward(family, cfg, params, x, torch.float32)
    with torch.no_grad():
        ref = model(x.to(torch.int64), output_hidden_states=True)
    assert np.allclose(out.logits.numpy(), ref.logits.numpy(), atol=1e-5)
    for a, b in zip(out.hidden_states, ref.hidden_states):
        assert np.allclose(a.numpy(), b.numpy(), atol=1e-5)


@pytest.mark.parametrize("family", FAMILIES)
def test_oracle_greedy_generation_matches_hf(family, hf_models):
    model, cfg, params = hf_models[family]
    x = _ids(cfg)
    y = O.generate(family, cfg, params, x, torch.float32, max_new_tokens=10, temperature=0.0)
    with torch.no_grad():
        y2 = x.to(torch.int64)
        for _ in range(10):
            logits = model(input_ids=y2).logits[:, -1]
            y2 = torch.cat([y2, logits.argmax(-1, keepdim=True)], dim=-1)
    assert np.array_equal(y.numpy(), y2.numpy())


@pytest.mark.parametrize("family", FAMILIES)
def test_oracle_kv_cache_rollback_consistency(family, hf_models):
    """Prefill, roll back one token, re-decode it: same hidden state (reference ``test_llama.py:137-154``)."""
    _, cfg, params = hf_models[family]
    x = _ids(cfg)
    caches = tuple(O.OracleKVCache(20, torch.float32) for _ in range(cfg.num_layers))
    y = O.forward(family, cfg, params, x, torch.float32, kv_caches=caches)
    rolled = tuple(c.rollback(1) for c in y.kv_caches)
    y2 = O.forward(family, cfg, params, x[:, -1:], torch.float32, kv_caches=rolled)
    assert np.allclose(y.last_hidden_state[:, -1:].numpy(), y2.last_hidden_state.numpy(), atol=1e-6)


def test_oracle_chunked_generation_matches_single_chunk(hf_models):
    """A tiny cache stride forces resize chunks; tokens must equal the one-chunk run."""
    _, cfg, params = hf_models["llama"]
    x = _ids(cfg, bs=2, seq=5)
    a = O.generate("llama", cfg, params, x, torch.float32, max_new_tokens=9, temperature=0.0, cache_stride=4)
    b = O.generate("llama", cfg, params, x, torch.float32, max_new_tokens=9, temperature=0.0, cache_stride=256)
    assert np.array_equal(a.numpy(), b.numpy())


def test_oracle_temperature_chunks_continue_rng(hf_models):
    """RNG continues across cache-resize chunks (reference ``tests/test_generation.py:630-675``)."""
    _, cfg, params = hf_models["llama"]
    x = _ids(cfg, bs=2, seq=5)
    a = O.generate("llama", cfg, params, x, torch.float32, max_new_tokens=9, temperature=0.8, seed=3, cache_stride=4)
    b = O.generate("llama", cfg, params, x, torch.float32, max_new_tokens=9, temperature=0.8, seed=3, cache_stride=256)
    assert np.array_equal(a.numpy(), b.numpy())
