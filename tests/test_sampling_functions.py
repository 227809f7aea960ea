"""The reference's public sampling functions (inference_engine/sampling.py:18-188): ``top_k_filtering``,
``top_p_filtering``, ``min_p_filtering``, ``greedy_fn`` and ``SamplingMethod.get_sampling_fn``, on CPU
tensors (the filters and the checks; the categorical draw itself runs on the GPU), case by case as the
reference's ``tests/test_sampling.py:57-341`` states them."""
import numpy as np
import pytest
import torch

from jaxml_b200.sampling import (SamplingMethod, greedy_fn, min_p_filtering, top_k_filtering, top_p_filtering)

KEY = np.array([0, 0], dtype=np.uint32)


def _kept(x):
    return torch.isfinite(x).numpy()


def test_top_k_filtering():
    logits = torch.tensor([[[0.0, 1.0, 5.0, 2.0]], [[4.0, 1.0, 0.0, 3.0]]])
    assert (_kept(top_k_filtering(KEY, logits, 2, 1.0, 0.0, 1.0))
            == np.array([[[False, False, True, True]], [[True, False, False, True]]])).all()
    one = logits[:1]
    assert _kept(top_k_filtering(KEY, one, 8, 1.0, 0.0, 1.0)).all()
    assert (_kept(top_k_filtering(KEY, one, np.int64(2), 1.0, 0.0, 1.0)) == [[[False, False, True, True]]]).all()
    assert torch.equal(top_k_filtering(KEY, one, 0, 1.0, 0.0, 1.0), one)
    for k in (True, np.bool_(True), 1.5):
        with pytest.raises(TypeError, match="top_k must be an integer"):
            top_k_filtering(KEY, one, k, 1.0, 0.0, 1.0)


@pytest.mark.parametrize("fn", [top_k_filtering, top_p_filtering, min_p_filtering, greedy_fn])
@pytest.mark.parametrize("logits,exc,match", [(torch.tensor(1.0), ValueError, "vocabulary axis"),
                                              (torch.ones(1, 1, 0), ValueError, "non-empty vocabulary"),
                                              (torch.ones(1, 1, 4, dtype=torch.int32), TypeError, "floating point")])
def test_invalid_logits(fn, logits, exc, match):
    with pytest.raises(exc, match=match):
        fn(KEY, logits, 2, 0.9, 0.1, 1.0)


@pytest.mark.parametrize("fn", [top_p_filtering, min_p_filtering, greedy_fn])
def test_invalid_logit_values_and_masks(fn):
    for logits, match in ((torch.tensor([[[0.0, float("nan")]]]), "NaN or positive infinity"),
                          (torch.tensor([[[0.0, float("inf")]]]), "NaN or positive infinity"),
                          (torch.tensor([[[-float("inf"), -float("inf")]]]), "at least one finite value")):
        with pytest.raises(ValueError, match=match):
            fn(KEY, logits, 2, 0.9, 0.1, 1.0)
    x = torch.tensor([[[0.0, -float("inf"), 1.0]]])
    out = fn(KEY, x, 2, 0.9, 0.1, 1.0)
    assert tuple(out.shape) == (tuple(x.shape[:-1]) if fn is greedy_fn else tuple(x.shape))


def test_top_p_filtering():
    logits = torch.tensor([[[0.0, 1.0, 5.0, 2.0]], [[4.0, 1.0, 0.0, 3.0]]])
    assert (_kept(top_p_filtering(KEY, logits, 0, 0.7, 0.0, 1.0))
            == np.array([[[False, False, True, False]], [[True, False, False, True]]])).all()
    one = logits[:1]
    assert torch.equal(top_p_filtering(KEY, one, 0, 1.5, 0.0, 1.0), one)
    assert (_kept(top_p_filtering(KEY, torch.tensor([[[0.0, 5.0, 5.0, 2.0]]]), 0, 0.0, 0.0, 1.0))
            == [[[False, True, True, False]]]).all()
    for p, exc, match in ((True, TypeError, "top_p must be a real number"),
                          (np.bool_(True), TypeError, "top_p must be a real number"),
                          ("0.9", TypeError, "top_p must be a real number"),
                          (float("nan"), ValueError, "top_p must be finite")):
        with pytest.raises(exc, match=match):
            top_p_filtering(KEY, one, 0, p, 0.0, 1.0)


def test_min_p_filtering():
    logits = torch.tensor([[[10.0, 0.0, 0.0]], [[0.0, 0.0, 0.0]]])
    assert (_kept(min_p_filtering(KEY, logits, 0, 1.0, 0.9, 1.0))
            == np.array([[[True, False, False]], [[True, True, True]]])).all()
    for p, exc, match in ((True, TypeError, "min_p must be a real number"),
                          (np.bool_(True), TypeError, "min_p must be a real number"),
                          ("0.1", TypeError, "min_p must be a real number"),
                          (float("nan"), ValueError, "min_p must be finite")):
        with pytest.raises(exc, match=match):
            min_p_filtering(KEY, logits, 0, 1.0, p, 1.0)


def test_greedy_first_index_of_the_maximum():
    assert greedy_fn(KEY, torch.tensor([[1.0, 3.0, 3.0, 0.0], [2.0, 2.0, 1.0, 2.0]])).tolist() == [1, 0]
    fn = SamplingMethod.from_values(top_k=1, top_p=1.0, min_p=0.0, temp=1.0).get_sampling_fn()
    assert fn is greedy_fn


def test_sampling_fn_checks_before_drawing():
    fn = SamplingMethod.from_values(top_k=2, top_p=0.9, min_p=0.0, temp=1.0).get_sampling_fn()
    with pytest.raises(TypeError, match="floating point"):
        fn(KEY, torch.ones(1, 1, 4, dtype=torch.int32), 2, 0.9, 0.0, 1.0)
    for logits, match in ((torch.tensor([[[0.0, float("nan")]]]), "NaN or positive infinity"),
                          (torch.tensor([[[-float("inf"), -float("inf")]]]), "at least one finite value")):
        with pytest.raises(ValueError, match=match):
            fn(KEY, logits, 2, 0.9, 0.0, 1.0)
    fn = SamplingMethod(use_top_k=True, use_top_p=False, use_min_p=False, use_greedy=False).get_sampling_fn()
    with pytest.raises(ValueError, match="temp must be positive"):
        fn(KEY, torch.tensor([[[0.0, 1.0, 5.0, 2.0]]]), 2, 1.0, 0.0, 0.0)
    with pytest.raises(RuntimeError, match="CUDA logits only"):
        fn(KEY, torch.tensor([[[0.0, 1.0, 5.0, 2.0]]]), 2, 1.0, 0.0, 1.0)
