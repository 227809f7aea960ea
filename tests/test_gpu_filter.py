"""The min-p / top-k / top-p filter kernel (jx_filter_logits) against the oracle.

The reference's known-answer cases (its tests/test_sampling.py inputs and kept tokens) in float32 and
bfloat16; random rows at the oracle's exact agreement sizes (5000 columns: top-k is exact, and the
float32 cumulative sum of the oracle's top-p stays far from top_p at the cutoff); and full-vocabulary
rows (Llama-3's 128256 columns, Gemma 3's 262144) through the defining property of each filter, since
there a float32 cumulative sum over ~10^5 entries is itself off by more than the gap between two sorted
probabilities:
  top-k  exactly the entries >= the k-th largest value (ties kept), compared with torch.topk;
  top-p  the kept set is {x >= t} for a row value t with G(t) >= top_p > G(next larger value), G the
         float64 sum of the dtype-rounded probabilities over the entries >= a value, within 1e-5;
  min-p  exactly the oracle's set, except entries whose probability is within one dtype ulp of min_p.
"""
import pytest
import torch

from oracle import jaxml_oracle as O

pytestmark = pytest.mark.gpu


def _kernel(logits, top_k=0, top_p=1.0, min_p=0.0, out=None):
    from jaxml_b200.sampling import filter_logits_

    x = logits.cuda()
    o = torch.empty_like(x) if out is None else out
    return filter_logits_(x, o, top_k, top_p, min_p).cpu()


LOGITS4 = torch.tensor([[0.0, 1.0, 5.0, 2.0], [4.0, 1.0, 0.0, 3.0]])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_known_answers(dtype):
    x = LOGITS4.to(dtype)
    assert torch.isfinite(_kernel(x, top_k=2)).tolist() == [[False, False, True, True], [True, False, False, True]]
    assert torch.isfinite(_kernel(x, top_k=10)).all()
    ties = torch.tensor([[3.0, 3.0, 1.0, 0.0]], dtype=dtype)
    assert torch.isfinite(_kernel(ties, top_k=1)).tolist() == [[True, True, False, False]]
    assert torch.isfinite(_kernel(x, top_p=0.7)).tolist() == [[False, False, True, False], [True, False, False, True]]
    mp = torch.tensor([[10.0, 0.0, 0.0], [0.0, 0.0, 0.0]], dtype=dtype)
    assert torch.isfinite(_kernel(mp, min_p=0.9)).tolist() == [[True, False, False], [True, True, True]]
    # kept entries are the inputs themselves
    got = _kernel(x, top_k=2)
    keep = torch.isfinite(got)
    assert torch.equal(got[keep], x[keep])


def test_negative_zero_ties_positive_zero():
    x = torch.tensor([[1.0, -0.0, 0.0, -1.0, 2.0]])
    # the 3rd largest value is 0.0; -0.0 compares equal to it, so both zeros stay
    assert torch.isfinite(_kernel(x, top_k=3)).tolist() == [[True, True, True, False, True]]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_random_rows_match_the_oracle(dtype):
    g = torch.Generator().manual_seed(0)
    logits = (torch.randn(6, 5000, generator=g) * 3).to(dtype)
    logits[2, 100:110] = logits[2].max()           # ties at the maximum
    logits[3, :4000] = float("-inf")               # masked columns
    for top_k, top_p, min_p in ((40, 1.0, 0.0), (0, 0.9, 0.0), (0, 1.0, 0.01), (50, 0.8, 0.02), (4999, 0.5, 0.0),
                                (1, 1.0, 0.0), (0, 0.05, 0.0), (7, 0.99, 0.001)):
        want = O.filter_logits(logits, top_k, top_p, min_p)
        got = _kernel(logits, top_k, top_p, min_p)
        assert torch.equal(torch.isfinite(got), torch.isfinite(want)), (top_k, top_p, min_p)
        assert torch.equal(got, want), (top_k, top_p, min_p)


def test_in_place_and_strided_rows():
    g = torch.Generator().manual_seed(1)
    base = torch.randn(3, 6000, generator=g).cuda()
    rows = base[:, :5000]                           # leading dimension 6000
    want = O.filter_logits(rows.cpu(), 30, 0.9, 0.0)
    got = _kernel(rows, 30, 0.9, 0.0)
    assert torch.equal(got, want)
    x = torch.randn(2, 5000, generator=g).to(torch.bfloat16).cuda()
    ref = O.filter_logits(x.cpu(), 0, 0.8, 0.0)
    from jaxml_b200.sampling import filter_logits_

    filter_logits_(x, x, 0, 0.8, 0.0)               # out aliases logits
    assert torch.equal(x.cpu(), ref)


def _probs64(x):
    """The oracle's dtype-rounded probabilities, as float64."""
    return O._probs(x).double()


def _check_top_p_property(x, got, top_p):
    keep = torch.isfinite(got)
    for r in range(x.shape[0]):
        xr = x[r].float()
        t = xr[keep[r]].min()
        assert torch.equal(keep[r], xr >= t), r
        q = _probs64(x[r:r + 1])[0]
        G_t = q[xr >= t].sum().item()
        above = xr[xr > t]
        G_next = q[xr >= above.min()].sum().item() if above.numel() else 0.0
        assert G_t >= top_p - 1e-5 and G_next < top_p + 1e-5, (r, G_t, G_next)


@pytest.mark.parametrize("V", [128256, 262144])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_full_vocabulary_rows(V, dtype):
    g = torch.Generator().manual_seed(V)
    B = 16
    logits = (torch.randn(B, V, generator=g) * 2.5).to(dtype)
    logits[1, 5:50] = logits[1].max()
    # top-k: exact
    for k in (1, 50, 1000, V - 1):
        got = _kernel(logits, top_k=k)
        cut = torch.topk(logits.float(), k, dim=-1).values[:, -1:]
        assert torch.equal(torch.isfinite(got), logits.float() >= cut), k
    # top-p: the defining property
    for p in (0.5, 0.9, 0.95):
        _check_top_p_property(logits, _kernel(logits, top_p=p), p)
    # min-p: the oracle's set up to entries within one ulp of the threshold
    min_p = 2e-4
    got = torch.isfinite(_kernel(logits, min_p=min_p))
    want = torch.isfinite(O.filter_logits(logits, 0, 1.0, min_p))
    diff = got != want
    if diff.any():
        q = _probs64(logits)
        ulp = min_p * (2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -23)
        assert ((q[diff] - min_p).abs() <= 2 * ulp).all()
    # all three in the reference's order: top-k's exact set after min-p, top-p's property after both
    k, p = 200, 0.9
    got = _kernel(logits, k, p, min_p)
    after_mk = _kernel(logits, k, 1.0, min_p)
    assert not (torch.isfinite(got) & ~torch.isfinite(after_mk)).any()
    _check_top_p_property(after_mk, got, p)
