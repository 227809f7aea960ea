"""``SamplingMethod.get_sampling_fn`` on the sampling kernel against the oracle's categorical draw
(threefry Gumbel-max, bit-exact tokens) with and without the min-p / top-k / top-p filters."""
import numpy as np
import pytest
import torch

from jaxml_b200.prng import prng_key, split
from jaxml_b200.sampling import SamplingMethod
from oracle import jaxml_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("kw", [dict(top_k=0, top_p=1.0, min_p=0.0), dict(top_k=40, top_p=0.9, min_p=0.0),
                                dict(top_k=0, top_p=1.0, min_p=0.02)], ids=["plain", "topk_topp", "minp"])
def test_sampling_fn_matches_oracle(dtype, kw):
    g = torch.Generator().manual_seed(3)
    logits = (2.0 * torch.randn(5, 1, 5000, generator=g)).to(dtype)
    fn = SamplingMethod.from_values(temp=0.8, **kw).get_sampling_fn()
    key = prng_key(11)
    for _ in range(4):
        key, sub = split(key)
        got = fn(sub, logits.cuda(), kw["top_k"], kw["top_p"], kw["min_p"], 0.8)
        want = O.sample(logits, sub, 0.8, False, **kw)
        assert got.dtype == torch.int32 and tuple(got.shape) == (5, 1)
        assert torch.equal(got.cpu(), want)


def test_sampling_fn_respects_the_filters():
    """The reference's pipeline cases (``tests/test_sampling.py:254-280``): batched rows never draw a
    filtered token; a top-k larger than the vocabulary keeps every token."""
    logits = torch.tensor([[[0.0, 1.0, 5.0, 2.0]], [[4.0, 1.0, 0.0, 3.0]]], device="cuda")
    fn = SamplingMethod.from_values(top_k=2, top_p=0.9, min_p=0.0, temp=1.0).get_sampling_fn()
    for seed in range(16):
        out = fn(np.array([0, seed], dtype=np.uint32), logits, 2, 0.9, 0.0, 1.0).cpu()
        assert tuple(out.shape) == (2, 1) and int(out[0, 0]) != 0 and int(out[1, 0]) != 1
    fn = SamplingMethod.from_values(top_k=8, top_p=1.0, min_p=0.0, temp=1.0).get_sampling_fn()
    out = fn(np.array([0, 0], dtype=np.uint32), logits[:1], 8, 1.0, 0.0, 1.0)
    assert tuple(out.shape) == (1, 1) and 0 <= int(out[0, 0]) < 4
