"""Helpers of the step-by-step GPU parity tests (not a test module).

``steps`` drives a decoder runtime through a prefill and decode steps the way generation does: the
first decode step eagerly, the rest as replays of the captured CUDA graph.  ``check_sampled_step``
checks one temperature-sampled step of bfloat16 logits against the oracle's threefry/Gumbel sampler.
"""
import numpy as np
import torch

from oracle import jaxml_oracle as O
from oracle import threefry as TF


def steps(rt, n_steps, greedy, temp):
    """Yields "prefill", then "eager" after the first decode step and "replay" after each of the other
    n_steps - 1 (each a replay of the captured decode graph)."""
    yield "prefill"
    if n_steps < 1:
        return
    rt.decode_step(greedy, temp)
    torch.cuda.synchronize()
    rt.check_status()
    yield "eager"
    g = rt.capture_decode(greedy, temp)
    for _ in range(n_steps - 1):
        g.replay()
        torch.cuda.synchronize()
        rt.check_status()
        yield "replay"


def check_sampled_step(got_logits, want_logits, tok, sub, temp, logits_tol):
    """One temperature step, bfloat16 logits [B, 1, V] on the CPU.

    * the device's tokens ``tok`` [B] equal the oracle's categorical draw on the device's own logits
      with the step's key ``sub`` (the sampler is bit-exact);
    * they equal the oracle's draw on the oracle's logits unless that draw is a near-tie: the perturbed
      score of the device's token is within the logits tolerance (scaled by 1/temp) plus two bf16 ulps
      of the best perturbed score.
    Returns the fraction of rows whose token equals the oracle's own draw."""
    assert torch.equal(tok, O.sample(got_logits, sub, temp, False)[:, 0])
    own = O.sample(want_logits, sub, temp, False)[:, 0]
    t16 = TF._bf16_round(np.array([temp], np.float32))[0]
    scaled = TF._bf16_round(want_logits.float().numpy() / t16)
    bits = TF.random_bits32(sub, scaled.size).reshape(scaled.shape)
    total = TF._bf16_round(TF.gumbel_table_bf16()[bits & np.uint32(0xFF)] + scaled)[:, 0]
    rows = np.arange(total.shape[0])
    gap = total[rows, own.numpy()] - total[rows, tok.numpy()]
    bound = 2 * logits_tol / temp + 2 * np.exp2(np.floor(np.log2(np.abs(total.max(-1)) + 1e-30)) - 7)
    assert bool(np.all((own.numpy() == tok.numpy()) | (gap <= bound))), (gap, bound)
    return float((own == tok).float().mean())
