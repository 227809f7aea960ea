"""KVCache (cache.py:69-282 of the reference): prefill padding, decode appends, rollback, resize and the
validation messages; cross-checked against the oracle's cache restatement."""
import pytest
import torch

from jaxml_b200.cache import KVCache, get_default_pos_ids
from oracle import jaxml_oracle as O


def _kv(B, S, H=2, hd=4, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, S, H, hd, generator=g), torch.randn(B, S, H, hd, generator=g)


def test_default_pos_ids_right_padding():
    mask = torch.tensor([[1, 1, 1, 0, 0], [1, 0, 0, 0, 0]], dtype=torch.bool)
    assert get_default_pos_ids(mask).tolist() == [[2], [0]]


def test_prefill_decode_rollback_resize_match_the_oracle():
    k, v = _kv(2, 3)
    mask = torch.tensor([[1, 1, 1], [1, 1, 0]], dtype=torch.bool)
    c = KVCache.init(8, k, v, mask, dtype=torch.float32)
    o = O.OracleKVCache(8, torch.float32).update(k, v, mask)
    assert c.k.shape == (2, 8, 2, 4) and c.pos_id.tolist() == [[2], [1]]
    assert torch.equal(c.k, o.k) and torch.equal(c.mask, o.mask)
    for step in range(3):
        k1, v1 = _kv(2, 1, seed=10 + step)
        c2 = c.update(k1, v1, c.next_mask)
        o = o.update(k1, v1, None)
        assert torch.equal(c2.k, o.k) and torch.equal(c2.v, o.v) and torch.equal(c2.mask, o.mask)
        assert torch.equal(c2.pos_id.to(torch.int64), o.pos_id.to(torch.int64))
        assert not torch.equal(c.k, c2.k)          # functional: the old cache is unchanged
        c = c2
    r = c.rollback(2)
    orr = o.rollback(2)
    assert torch.equal(r.k, orr.k) and torch.equal(r.mask, orr.mask) and r.pos_id.tolist() == [[3], [2]]
    big = r.resize(12)
    assert big.k.shape[1] == 12 and big.validate_state() is big
    small = r.resize(6)
    assert small.k.shape[1] == 6 and torch.equal(small.k, r.k[:, :6])


def test_cache_errors():
    with pytest.raises(ValueError, match="max_seq_len must be positive"):
        KVCache.init(0)
    with pytest.raises(TypeError, match="max_seq_len must be an integer"):
        KVCache.init(True)
    k, v = _kv(1, 4)
    with pytest.raises(ValueError, match="Cannot cache 4 tokens in max_seq_len=3"):
        KVCache.init(3, k, v)
    with pytest.raises(ValueError, match="requires both k and v"):
        KVCache.init(8, k=k)
    with pytest.raises(ValueError, match="right padded"):
        KVCache.init(8, k, v, torch.tensor([[1, 0, 1, 1]]))
    with pytest.raises(ValueError, match="integer values must be 0 or 1"):
        KVCache.init(8, k, v, torch.tensor([[1, 2, 1, 1]]))
    c = KVCache.init(5, k, v)
    with pytest.raises(ValueError, match="exactly one token"):
        c.update(*_kv(1, 2))
    c = c.update(*_kv(1, 1))
    with pytest.raises(ValueError, match="Cannot decode past max_seq_len=5"):
        c.update(*_kv(1, 1))
    with pytest.raises(ValueError, match="Cannot roll back past the beginning"):
        c.rollback(5)
    with pytest.raises(ValueError, match="below the highest cached position"):
        c.resize(4)
    with pytest.raises(ValueError, match="Cannot get next position ids"):
        KVCache.init(4).next_pos_id


@pytest.mark.gpu
def test_cache_stays_on_the_gpu():
    k, v = _kv(2, 3)
    c = KVCache.init(8, k.cuda(), v.cuda(), dtype=torch.bfloat16)
    c = c.update(*(t.cuda() for t in _kv(2, 1, seed=3)))
    assert c.k.is_cuda and c.mask.is_cuda and c.k.dtype == torch.bfloat16 and c.pos_id.tolist() == [[3], [3]]
