"""The float32 runtime (libjxb200 kernels) against committed golden outputs of HF transformers' eager
models (``tests/golden/hf_tiny.npz``): last-position logits within 1e-4 relative (1e-5 absolute floor)
and identical greedy tokens, for Llama, GPT-NeoX and Gemma3."""
import pytest
import torch

from oracle import threefry as TF
from tests.test_oracle_golden import load_family

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_runtime_f32_matches_golden_hf_outputs(family):
    from jaxml_b200.runtime import DecoderRuntime, ModelWeights

    cfg, params, ids, logits, greedy = load_family(family)
    B, P = ids.shape
    n = greedy.shape[1] - P
    rt = DecoderRuntime(ModelWeights(family, cfg, params, torch.float32, "cuda:0"), B, 64)
    mask = torch.ones(B, P, dtype=torch.bool, device="cuda")
    key, sub = TF.split(TF.prng_key(0))
    rt.reset(mask, key, sub, n)
    rt.prefill(ids.cuda(), greedy=True, temp=1.0)
    torch.cuda.synchronize()
    rt.check_status()
    got = rt.logits_buf()[:B].float().cpu()
    assert torch.allclose(got, logits, rtol=1e-4, atol=1e-5), (got - logits).abs().max().item()
    toks = rt.generate(ids.cuda(), mask, n, True, 1.0, 0).cpu()
    rt.check_status()
    assert torch.equal(toks, greedy[:, P:])
