"""min-p / top-k / top-p filtering: the reference's known-answer cases (tests/test_sampling.py:57-252 of
the reference, same inputs and expected kept tokens) for the oracle restatement and for the device
filter (run here on CPU tensors), plus agreement of the two on random logits."""
import pytest
import torch

from jaxml_b200.sampling import filter_logits_
from oracle import jaxml_oracle as O


def _both(logits, top_k=0, top_p=1.0, min_p=0.0):
    want = O.filter_logits(logits, top_k, top_p, min_p)
    got = filter_logits_(logits, torch.empty_like(logits), top_k, top_p, min_p)
    return torch.isfinite(want), torch.isfinite(got)


LOGITS4 = torch.tensor([[0.0, 1.0, 5.0, 2.0], [4.0, 1.0, 0.0, 3.0]])


def test_top_k_keeps_top_tokens_per_row():
    for kept in _both(LOGITS4, top_k=2):
        assert kept.tolist() == [[False, False, True, True], [True, False, False, True]]


def test_top_k_caps_k_to_vocab_and_keeps_ties():
    for kept in _both(LOGITS4, top_k=10):
        assert kept.all()
    for kept in _both(torch.tensor([[3.0, 3.0, 1.0, 0.0]]), top_k=1):
        assert kept.tolist() == [[True, True, False, False]]


def test_top_p_uses_the_sorted_cutoff_per_row():
    for kept in _both(LOGITS4, top_p=0.7):
        assert kept.tolist() == [[False, False, True, False], [True, False, False, True]]


def test_min_p_falls_back_per_row_when_no_token_qualifies():
    logits = torch.tensor([[10.0, 0.0, 0.0], [0.0, 0.0, 0.0]])
    for kept in _both(logits, min_p=0.9):
        assert kept.tolist() == [[True, False, False], [True, True, True]]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_device_filter_matches_the_oracle_on_random_logits(dtype):
    g = torch.Generator().manual_seed(0)
    logits = (torch.randn(4, 5000, generator=g) * 3).to(dtype)
    for top_k, top_p, min_p in ((40, 1.0, 0.0), (0, 0.9, 0.0), (0, 1.0, 0.01), (50, 0.8, 0.02)):
        want = O.filter_logits(logits, top_k, top_p, min_p)
        got = filter_logits_(logits, torch.empty_like(logits), top_k, top_p, min_p)
        assert torch.equal(want, got), (top_k, top_p, min_p)
