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


# ---- parameter normalisation and method selection (the reference's tests/test_sampling.py cases) ----
import numpy as np  # noqa: E402

from jaxml_b200.sampling import SamplingMethod, normalize_sampling_params  # noqa: E402


def test_normalize_sampling_params_clips_bounds():
    p = normalize_sampling_params(top_k=-3, top_p=1.5, min_p=-0.5, temp=-1.0)
    assert (p.top_k, p.top_p, p.min_p, p.temp) == (0, 1.0, 0.0, 0.0)


@pytest.mark.parametrize("top_k", [True, np.bool_(True), 1.5])
def test_normalize_sampling_params_rejects_non_integer_top_k(top_k):
    with pytest.raises(TypeError, match="top_k must be an integer"):
        normalize_sampling_params(top_k=top_k, top_p=1.0, min_p=0.0, temp=1.0)


@pytest.mark.parametrize("name", ["top_p", "min_p", "temp"])
@pytest.mark.parametrize("value", [True, np.bool_(True), "1.0"])
def test_normalize_sampling_params_rejects_non_real_values(name, value):
    kw = {"top_k": 0, "top_p": 1.0, "min_p": 0.0, "temp": 1.0, name: value}
    with pytest.raises(TypeError, match=f"{name} must be a real number"):
        normalize_sampling_params(**kw)


@pytest.mark.parametrize("name", ["top_p", "min_p", "temp"])
@pytest.mark.parametrize("value", [np.nan, np.inf, -np.inf])
def test_normalize_sampling_params_rejects_non_finite_values(name, value):
    kw = {"top_k": 0, "top_p": 1.0, "min_p": 0.0, "temp": 1.0, name: value}
    with pytest.raises(ValueError, match=f"{name} must be finite"):
        normalize_sampling_params(**kw)


def test_sampling_method_flags():
    m = SamplingMethod(use_top_k=np.bool_(True), use_top_p=np.bool_(False), use_min_p=np.bool_(False),
                       use_greedy=np.bool_(False))
    assert (m.use_top_k, m.use_top_p, m.use_min_p, m.use_greedy) == (True, False, False, False)
    for field in ("use_top_k", "use_top_p", "use_min_p", "use_greedy"):
        for value in (1, 0, "true"):
            kw = {"use_top_k": False, "use_top_p": False, "use_min_p": False, "use_greedy": True, field: value}
            with pytest.raises(TypeError, match=f"{field} must be a boolean"):
                SamplingMethod(**kw)


@pytest.mark.parametrize("kw,greedy,filters", [
    (dict(top_k=0, top_p=1.0, min_p=0.0, temp=0.0), True, False),      # temperature 0 -> greedy
    (dict(top_k=1, top_p=1.0, min_p=0.0, temp=0.8), True, False),      # top_k == 1 -> greedy
    (dict(top_k=0, top_p=0.0, min_p=0.0, temp=0.8), True, False),      # top_p == 0 -> greedy
    (dict(top_k=0, top_p=1.0, min_p=0.0, temp=0.8), False, False),     # plain temperature sampling
    (dict(top_k=20, top_p=0.9, min_p=0.05, temp=0.8), False, True),    # all three filters
])
def test_sampling_method_from_values(kw, greedy, filters):
    m = SamplingMethod.from_values(**kw)
    assert m.use_greedy == greedy and m.uses_filters == filters
