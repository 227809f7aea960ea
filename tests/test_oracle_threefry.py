"""Pins the oracle's PRNG and the reference's known-answer tests for masks and caches."""
import numpy as np
import torch

from oracle import jaxml_oracle as O
from oracle import threefry as T


def test_threefry_random123_known_answers():
    # Random123 threefry2x32_20 known-answer vectors (kat_vectors of the Random123 distribution).
    cases = [
        ((0x00000000, 0x00000000), (0x00000000, 0x00000000), (0x6B200159, 0x99BA4EFE)),
        ((0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF), (0x1CB996FC, 0xBB002BE7)),
        ((0x13198A2E, 0x03707344), (0x243F6A88, 0x85A308D3), (0xC4923A9C, 0x483DF7A0)),
    ]
    for key, x, want in cases:
        got = T.threefry2x32(key, np.uint32(x[0]), np.uint32(x[1]))
        assert (int(got[0]), int(got[1])) == want


def test_legacy_split_of_key_zero():
    # jax.random.split(jax.random.PRNGKey(0)) under the legacy (non-partitionable) scheme.
    got = T.split_legacy(T.prng_key(0))
    assert got.tolist() == [[4146024105, 967050713], [2718843009, 1272950319]]


def test_prng_key_layout():
    assert T.prng_key(0).tolist() == [0, 0]
    assert T.prng_key(123).tolist() == [0, 123]


def test_bf16_uniform_and_gumbel_table():
    u = T.uniform_bits_to_u_bf16(np.arange(256))
    assert u.min() == np.float32(2.0 ** -126) and u.max() == np.float32(127 / 128)
    g = T.gumbel_table_bf16()
    # values are bfloat16-representable and monotone in the draw
    assert np.all(g.view(np.uint32) & 0xFFFF == 0)
    assert np.all(np.diff(g[::2]) > 0)


def test_categorical_first_index_tie_break():
    logits = np.zeros((1, 1, 8), dtype=np.float32)
    logits[0, 0, 3] = 100.0
    logits[0, 0, 5] = 100.0
    out = T.categorical_bf16(T.prng_key(0), logits, 1.0)
    assert out.shape == (1, 1) and out[0, 0] in (3, 5)


# ---- the reference's known-answer tests (tests/test_attention.py:108-264, tests/test_cache.py:593-606) ----
def _mha(q, k, v, mask=None, sw=None):
    return O.mha(q, k, v, mask, True, sw, 1.0, return_weights=True)


def test_sliding_window_decode_masks_old_keys():
    q = torch.zeros(1, 1, 1, 1)
    k = torch.zeros(1, 5, 1, 1)
    v = torch.arange(5, dtype=torch.float32).reshape(1, 5, 1, 1) * 10
    out, w = _mha(q, k, v, sw=2)
    assert np.allclose(out.numpy(), [[[[35.0]]]])
    assert np.allclose(w.numpy(), [[[[0, 0, 0, 0.5, 0.5]]]])


def test_sliding_window_decode_respects_padded_cache_mask():
    q = torch.zeros(1, 1, 1, 1)
    k = torch.zeros(1, 8, 1, 1)
    v = torch.arange(8, dtype=torch.float32).reshape(1, 8, 1, 1) * 10
    mask = torch.tensor([[True, True, True, True, False, False, False, False]])
    out, w = _mha(q, k, v, mask=mask, sw=2)
    assert np.allclose(out.numpy(), [[[[25.0]]]])
    assert np.allclose(w.numpy(), [[[[0, 0, 0.5, 0.5, 0, 0, 0, 0]]]])


def test_attention_all_masked_rows_remain_finite():
    q = torch.zeros(1, 1, 1, 1)
    k = torch.zeros(1, 2, 1, 1)
    v = torch.tensor([[[[2.0]], [[4.0]]]])
    out, w = _mha(q, k, v, mask=torch.tensor([[False, False]]))
    assert np.allclose(out.numpy(), [[[[3.0]]]])
    assert np.allclose(w.numpy(), [[[[0.5, 0.5]]]])


def test_repeat_kv_repeats_grouped_key_values():
    k = torch.tensor([[[[1.0, 2.0]], [[3.0, 4.0]]]])
    r = O.repeat_kv(k, 2)
    assert r.shape == (1, 2, 2, 2)
    assert torch.equal(r[:, :, 0], k[:, :, 0]) and torch.equal(r[:, :, 1], k[:, :, 0])


def test_kv_cache_decode_extends_cached_mask():
    k = torch.ones(2, 2, 1, 1)
    cache = O.OracleKVCache(4, torch.float32).update(k, k, torch.tensor([[True, True], [True, False]]))
    cache = cache.update(torch.full((2, 1, 1, 1), 3.0), torch.full((2, 1, 1, 1), 3.0), None)
    assert cache.mask.tolist() == [[True, True, True, False], [True, True, False, False]]
    assert cache.pos_id.tolist() == [[2], [1]]
    assert cache.k[1, 1, 0, 0] == 3.0 and cache.k[0, 2, 0, 0] == 3.0
