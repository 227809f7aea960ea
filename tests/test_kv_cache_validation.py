"""KVCache validation on CPU tensors: the reference's ``tests/test_cache.py`` cases (messages matched
the same way), against ``jaxml_b200.cache.KVCache``."""
import numpy as np
import pytest
import torch

from jaxml_b200.cache import KVCache


def _kv(batch=2, seq_len=1, heads=1, hd=2, value=1.0):
    k = torch.full((batch, seq_len, heads, hd), value, dtype=torch.float32)
    return k, k + 1.0


@pytest.mark.parametrize("field", ["k", "v"])
def test_update_rejects_non_floating_values(field):
    k, v = _kv()
    if field == "k":
        k = k.to(torch.int32)
    else:
        v = v.to(torch.int32)
    with pytest.raises(TypeError, match=f"{field} must contain floating point"):
        KVCache.init(4).update(k, v, mask=None)


@pytest.mark.parametrize("value", [float("nan"), float("inf"), -float("inf")])
@pytest.mark.parametrize("field", ["k", "v"])
def test_update_rejects_non_finite_values(field, value):
    for prefill in (True, False):
        k, v = _kv(seq_len=2)
        cache = KVCache.init(4)
        if not prefill:
            cache = cache.update(k, v, mask=torch.ones(2, 2, dtype=torch.bool))
            k, v = _kv(seq_len=1)
        (k if field == "k" else v)[0, 0, 0, 0] = value
        with pytest.raises(ValueError, match=f"{field} must contain only finite values"):
            cache.update(k, v, mask=None)


def test_integer_initial_mask_is_canonicalised():
    k, v = _kv(seq_len=3)
    cache = KVCache.init(4).update(k, v, mask=torch.tensor([[1, 1, 0], [1, 0, 0]], dtype=torch.int32))
    assert cache.mask.dtype == torch.bool
    assert cache.mask.tolist() == [[True, True, False, False], [True, False, False, False]]
    assert cache.pos_id.tolist() == [[1], [0]]


@pytest.mark.parametrize("mask", [[[1, 2, 0], [1, 0, 0]], [[1, -1, 0], [1, 0, 0]]])
def test_non_binary_integer_initial_mask(mask):
    k, v = _kv(seq_len=3)
    with pytest.raises(ValueError, match="mask integer values must be 0 or 1"):
        KVCache.init(4).update(k, v, mask=torch.tensor(mask, dtype=torch.int32))


def test_float_initial_mask():
    k, v = _kv(seq_len=3)
    with pytest.raises(TypeError, match="mask must be boolean or integer"):
        KVCache.init(4).update(k, v, mask=torch.ones(2, 3))


@pytest.mark.parametrize("shape", [(2, 1), (2, 1, 2)])
def test_non_4d_values(shape):
    t = torch.ones(shape)
    with pytest.raises(ValueError, match="4D"):
        KVCache.init(4).update(t, t, mask=None)


@pytest.mark.parametrize("shape,match", [((0, 1, 1, 2), "batch axis must be non-empty"),
                                         ((1, 0, 1, 2), "sequence axis must be non-empty"),
                                         ((1, 1, 0, 2), "head axis must be non-empty"),
                                         ((1, 1, 1, 0), "head_dim axis must be non-empty")])
def test_empty_axes(shape, match):
    t = torch.zeros(shape)
    with pytest.raises(ValueError, match=match):
        KVCache.init(4).update(t, t, mask=None)


def test_capacity_and_mask_contents():
    k, v = _kv(seq_len=3)
    with pytest.raises(ValueError, match="Cannot cache 3 tokens"):
        KVCache.init(2).update(k, v, mask=torch.ones(2, 3, dtype=torch.bool))
    with pytest.raises(ValueError, match="at least one valid token"):
        KVCache.init(4).update(k, v, mask=torch.tensor([[True, False, False], [False, False, False]]))
    k1, v1 = _kv(batch=1, seq_len=3)
    with pytest.raises(ValueError, match="right padded"):
        KVCache.init(4).update(k1, v1, mask=torch.tensor([[True, False, True]]))


def test_decode_checks():
    k, v = _kv(seq_len=2)
    cache = KVCache.init(4).update(k, v, mask=torch.tensor([[True, True], [True, False]]))
    nk, nv = _kv(seq_len=1, value=3.0)
    with pytest.raises(ValueError, match="exactly one token"):
        cache.update(k, v, mask=None)
    with pytest.raises(ValueError, match="Decode cache mask shape must match"):
        cache.update(nk, nv, mask=torch.ones(2, 1, dtype=torch.bool))
    with pytest.raises(ValueError, match="must match current cached mask state"):
        cache.update(nk, nv, mask=torch.ones(2, 4, dtype=torch.bool))
    for bad in ([[1, 2, 0, 0], [1, 0, 0, 0]], [[1, -1, 0, 0], [1, 0, 0, 0]]):
        with pytest.raises(ValueError, match="Decode cache mask integer values must be 0 or 1"):
            cache.update(nk, nv, mask=torch.tensor(bad, dtype=torch.int32))
    # the current mask (bool or 0/1 integers) is accepted and the decode lands at pos_id + 1 per row
    for m in (cache.mask, cache.mask.to(torch.int32)):
        nxt = cache.update(nk, nv, mask=m)
        assert nxt.pos_id.tolist() == [[2], [1]]
        assert nxt.mask.tolist() == [[True, True, True, False], [True, True, False, False]]
        assert torch.equal(nxt.k[0, 2], nk[0, 0]) and torch.equal(nxt.k[1, 1], nk[1, 0])
    full = KVCache.init(2).update(k, v, mask=torch.ones(2, 2, dtype=torch.bool))
    with pytest.raises(ValueError, match="max_seq_len=2"):
        full.update(nk, nv, mask=None)


def test_dtype_and_capacity_arguments():
    assert KVCache.init(np.int64(4)).max_seq_len == 4
    for bad in (True, 2.5):
        with pytest.raises(TypeError, match="max_seq_len must be an integer"):
            KVCache.init(bad)
    with pytest.raises(ValueError, match="max_seq_len must be positive"):
        KVCache.init(-1)
    c = KVCache.init(4, dtype="bfloat16")
    assert c.dtype == torch.bfloat16
    k, v = _kv(seq_len=2)
    assert c.update(k, v).k.dtype == torch.bfloat16


def test_rollback_and_resize_arguments():
    k, v = _kv(seq_len=3)
    cache = KVCache.init(6).update(k, v, mask=None)
    for bad in (True, 1.5):
        with pytest.raises(TypeError, match="n must be an integer"):
            cache.rollback(bad)
    with pytest.raises(ValueError, match="Cannot roll back past the beginning"):
        cache.rollback(3)
    r = cache.rollback(np.int64(1))
    assert r.pos_id.tolist() == [[1], [1]] and r.mask[:, 2].tolist() == [False, False]
    with pytest.raises(ValueError, match="below the highest cached position"):
        cache.resize(2)
    for bad in (True, 2.5):
        with pytest.raises(TypeError, match="new_size must be an integer"):
            cache.resize(bad)
    grown = cache.resize(np.int64(10))
    assert grown.max_seq_len == 10 and grown.k.shape[1] == 10 and torch.equal(grown.k[:, :6], cache.k)
    empty = KVCache.init(4).resize(8)
    assert empty.max_seq_len == 8 and empty.k is None


def _state(k_shape=(1, 4, 1, 2), v_shape=None, k_dtype=torch.float32, v_dtype=None, mask=None, pos=None,
           dtype=torch.float32, T=4):
    k = torch.zeros(k_shape, dtype=k_dtype)
    v = torch.zeros(v_shape or k_shape, dtype=v_dtype or k_dtype)
    B = k_shape[0]
    mask = torch.ones(B, k_shape[1] if len(k_shape) > 1 else 4, dtype=torch.bool) if mask is None else mask
    pos = torch.full((B, 1), (mask.shape[1] - 1) if B else 0, dtype=torch.int32) if pos is None else pos
    return KVCache(k=k, v=v, max_seq_len=T, mask=mask, dtype=dtype, pos_id=pos)


def _nonfinite(field, value):
    c = _state()
    t = (c.k if field == "k" else c.v).clone()
    t[0, 0, 0, 0] = value
    return c.replace(**{field: t})


@pytest.mark.parametrize("cache,exc,match", [
    (_state(v_shape=(1, 3, 1, 2)), ValueError, "same shape"),
    (_state(k_shape=(1, 4, 2), mask=torch.ones(1, 4, dtype=torch.bool)), ValueError, "4D arrays"),
    (_state(k_shape=(0, 4, 1, 2), mask=torch.ones(0, 4, dtype=torch.bool)), ValueError, "batch axis must be non-empty"),
    (_state(k_shape=(1, 3, 1, 2)), ValueError, "sequence axis must match"),
    (_state(k_shape=(1, 4, 0, 2)), ValueError, "head axis must be non-empty"),
    (_state(k_shape=(1, 4, 1, 0)), ValueError, "head_dim axis must be non-empty"),
    (_state(k_dtype=torch.int32, v_dtype=torch.float32), TypeError, "Cached k must contain floating"),
    (_state(k_dtype=torch.float32, v_dtype=torch.bfloat16, dtype=torch.bfloat16), TypeError,
     "Cached k dtype must match cache dtype"),
    (_state(v_dtype=torch.int32), TypeError, "Cached v must contain floating"),
    (_nonfinite("k", float("nan")), ValueError, "Cached k must contain only finite values"),
    (_nonfinite("v", float("inf")), ValueError, "Cached v must contain only finite values"),
    (_state(v_dtype=torch.bfloat16), TypeError, "Cached v dtype must match cache dtype"),
    (_state(mask=torch.ones(1, 3, dtype=torch.bool)), ValueError, "Cached mask shape"),
    (_state(mask=torch.ones(1, 4, dtype=torch.int32)), TypeError, "Cached mask must be boolean"),
    (_state(mask=torch.zeros(1, 4, dtype=torch.bool)), ValueError, "at least one valid token"),
    (_state(mask=torch.tensor([[True, False, True, False]]), pos=torch.tensor([[2]], dtype=torch.int32)), ValueError,
     "right padded"),
    (_state(pos=torch.zeros(1, 2, dtype=torch.int32)), ValueError, "Cached pos_id shape"),
    (_state(pos=torch.zeros(1, 1)), TypeError, "Cached pos_id must contain integer"),
    (_state(pos=torch.full((1, 1), 4, dtype=torch.int32)), ValueError, r"within \[0, 4\)"),
    (_state(pos=torch.zeros(1, 1, dtype=torch.int32)), ValueError, "last valid token position"),
])
def test_validate_state_rejects_invalid_populated_state(cache, exc, match):
    """Each malformed populated cache of the reference's ``tests/test_cache.py:345-590`` table, checked
    by ``validate_state`` and before any ``update``."""
    with pytest.raises(exc, match=match):
        cache.validate_state()
    k = torch.zeros(cache.k.shape[0], 1, 1, 2) if cache.k.ndim == 4 else torch.zeros(1, 1, 1, 2)
    with pytest.raises((TypeError, ValueError)):
        cache.update(k, k.clone())


def test_static_fields_and_initial_state():
    """The reference's ``tests/test_cache.py:16-140`` cases: static fields checked by ``validate_state``
    and before any update, a complete initial state padded and positioned, partial ones refused."""
    for cache, exc, match in ((KVCache(k=None, v=None, max_seq_len=0, mask=None), ValueError,
                               "max_seq_len must be positive"),
                              (KVCache(k=None, v=None, max_seq_len=True, mask=None), TypeError,
                               "max_seq_len must be an integer"),
                              (KVCache(k=None, v=None, max_seq_len=4, mask=None, dtype=None), TypeError,
                               "dtype must be a valid"),
                              (KVCache(k=None, v=None, max_seq_len=4, mask=None, dtype="not-a-dtype"), TypeError,
                               "dtype must be a valid")):
        with pytest.raises(exc, match=match):
            cache.validate_state()
        k, v = _kv(batch=1)
        with pytest.raises(exc, match=match):
            cache.update(k, v, mask=None)
    k, v = _kv(seq_len=2)
    c = KVCache.init(4, k=k, v=v, mask=torch.tensor([[1, 1], [1, 0]], dtype=torch.int32))
    assert tuple(c.k.shape) == (2, 4, 1, 2) and c.mask.dtype == torch.bool
    assert c.mask.tolist() == [[True, True, False, False], [True, False, False, False]]
    assert c.pos_id.tolist() == [[1], [0]]
    c = KVCache.init(4, k=k, v=v, mask=None, dtype=torch.bfloat16)
    assert c.k.dtype == torch.bfloat16 and c.v.dtype == torch.bfloat16 and c.dtype == torch.bfloat16
    c = KVCache.init(4).update(k, v, mask=None)
    assert c.mask.tolist() == [[True, True, False, False]] * 2 and c.pos_id.tolist() == [[1], [1]]
    one_k, one_v = _kv(seq_len=1)
    for kw in ({"k": one_k}, {"v": one_v}, {"mask": torch.ones(2, 1, dtype=torch.bool)},
               {"k": one_k, "mask": torch.ones(2, 1, dtype=torch.bool)}):
        with pytest.raises(ValueError, match="requires both k and v"):
            KVCache.init(4, **kw)
    partial = KVCache(k=None, v=None, max_seq_len=4, mask=None, pos_id=torch.zeros(1, 1, dtype=torch.int32))
    with pytest.raises(ValueError, match="k is empty"):
        partial.update(*_kv(batch=1), mask=None)
