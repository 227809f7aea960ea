"""The persistent decode-step kernel (jx_decode_step) against the oracle and the per-op decode path.

Small Llama-shaped bf16 models with head size 128 (the kernel's) so the oracle stays fast; they
exercise projections with fewer iterations than CTAs (most CTAs have no share of a phase), rows of
different lengths (right-padded prompts: different key-split counts per row), several 128-key splits,
both attention forms (split items over 128-key ranges with a grid barrier between scores and P.V, and
single-pass items per (row, KV head) when those fill half the grid), one and sixteen batch rows, and repeated replays of the captured step (the grid barrier counter, the
split-K and attention arrival counters must reset every step).  Norm weights are random so their loads
count.  Logits within max(2e-2, 4 bf16 ulps of the largest logit) of the oracle with a mean error below
half an ulp of the largest logit (measured: a quarter; a wrong index or rounding point shows as errors
of the logits' own size), and the per-op path's logits and caches agree with the persistent kernel's to
the same bounds.
"""
import pytest
import torch

from oracle import jaxml_oracle as O
from oracle import threefry as TF
from tests.stepwise import steps

pytestmark = pytest.mark.gpu


def _cfg(d=512, H=4, Hkv=2, L=2, V=1000):
    from jaxml_b200.config import ModelConfig

    return ModelConfig(hidden_size=d, head_dim=128, num_heads=H, num_kv_heads=Hkv, num_layers=L,
                       intermediate_ratio=(7, 2), max_position_embeddings=2048, vocab_size=V, norm_eps=1e-5,
                       rope_theta=500000.0)


def _runtime(cfg, params, B, T, persistent):
    from jaxml_b200.runtime import DecoderRuntime, ModelWeights

    old = DecoderRuntime.persistent_decode
    DecoderRuntime.persistent_decode = persistent
    try:
        rt = DecoderRuntime(ModelWeights("llama", cfg, params, torch.bfloat16, "cuda:0"), B, T)
    finally:
        DecoderRuntime.persistent_decode = old
    assert (rt.fused_step is not None) == persistent
    return rt


CASES = [
    # (B, P, lens of the right-padded prompt rows, n decode steps, model)
    (3, 37, [37, 20, 5], 6, dict()),
    (16, 300, [300 - 7 * i for i in range(16)], 4, dict()),
    (1, 130, [130], 5, dict(H=8, Hkv=1)),
    (5, 200, [200, 199, 129, 128, 127], 4, dict(d=1024, H=16, Hkv=4, L=3, V=3000)),
    # 16 rows x 8 KV heads: one single-pass attention item per (row, KV head), ragged key counts
    (16, 260, [260 - 17 * i for i in range(16)], 4, dict(d=512, H=32, Hkv=8)),
]


@pytest.mark.parametrize("B,P,lens,n_steps,model", CASES)
def test_persistent_decode_matches_oracle_and_per_op_path(B, P, lens, n_steps, model):
    cfg = _cfg(**model)
    params = O.init_params("llama", cfg, seed=3, dtype=torch.bfloat16)
    gw = torch.Generator().manual_seed(9)
    body = params["params"]["model"]
    for lp in [body["norm"]] + [body[f"layers_{i}"][n] for i in range(cfg.num_layers)
                                for n in ("input_layernorm", "post_attention_layernorm")]:
        lp["weight"] = (1 + 0.1 * torch.randn(cfg.hidden_size, generator=gw)).to(torch.bfloat16)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=g, dtype=torch.int32)
    mask = torch.arange(P)[None, :] < torch.tensor(lens)[:, None]
    T = (P // 256 + 1) * 256
    rts = {name: _runtime(cfg, params, B, T, name == "persistent") for name in ("persistent", "per-op")}
    key, sub = TF.split(TF.prng_key(0))
    gens = {}
    for name, rt in rts.items():
        rt.reset(mask.cuda(), key, sub, n_steps + 1)
        rt.prefill(ids.cuda(), True, 1.0)
        torch.cuda.synchronize()
        rt.check_status()
        gens[name] = steps(rt, n_steps, True, 1.0)
    caches = tuple(O.OracleKVCache(T, torch.bfloat16) for _ in range(cfg.num_layers))
    out = O.forward("llama", cfg, params, ids, torch.bfloat16, attention_mask=mask, kv_caches=caches,
                    keep_last_n_logits=1)
    for i in range(n_steps + 1):
        for gen in gens.values():
            next(gen)
        rp, ro = rts["persistent"], rts["per-op"]
        lp, lo = rp.logits_buf()[:B].float().cpu(), ro.logits_buf()[:B].float().cpu()
        want = out.logits[:, -1].float()
        ulp = 2.0 ** (torch.floor(torch.log2(want.abs().max())).item() - 7)
        tol, tol_mean = max(2e-2, 4 * ulp), max(2e-3, 0.5 * ulp)
        for other in (want, lo):
            err = (lp - other).abs()
            assert err.max().item() <= tol and err.mean().item() <= tol_mean, (i, err.max().item(), err.mean().item(), tol)
        tp, to = rp.tokens_out[:, i].cpu(), ro.tokens_out[:, i].cpu()
        assert torch.equal(tp, torch.argmax(lp, -1).to(torch.int32))
        if i == n_steps:
            break
        # both runtimes continue from the persistent kernel's tokens (the per-op one is fed the same)
        ro.next_ids.copy_(rp.next_ids)
        ro.tokens_out[:, i].copy_(rp.tokens_out[:, i])
        out = O.forward("llama", cfg, params, tp[:, None], torch.bfloat16, kv_caches=out.kv_caches,
                        keep_last_n_logits=1)
    for name in ("persistent", "per-op"):
        assert int(rts[name].status[0].item()) == 0
    rp, ro = rts["persistent"], rts["per-op"]
    assert int(rp.gemv_counters.abs().sum().item()) == 0 and int(rp.attn_counters.abs().sum().item()) == 0
    assert int(rp.fused_step.sync[1].item()) == 0
    assert torch.equal(rp.pos_id, ro.pos_id)
    c = out.kv_caches
    for li in range(cfg.num_layers):
        for got, other, want in ((rp.k_cache[li], ro.k_cache[li], c[li].k), (rp.v_cache[li], ro.v_cache[li], c[li].v)):
            got, other = got.float().cpu(), other.float().cpu()
            ulp = 2.0 ** (torch.floor(torch.log2(want.float().abs().max())).item() - 7)
            for ref in (want.float(), other):
                err = (got - ref).abs()
                assert err.max().item() <= max(2e-2, 4 * ulp) and err.mean().item() <= max(2e-3, 0.5 * ulp), (li, err.max().item())


def test_persistent_decode_rejects_unsupported_shapes():
    """The C ABI checks the sizes it covers before launching anything."""
    from jaxml_b200 import _native as N

    a = N.JxStepArgs()
    a.M, a.L, a.d, a.Hq, a.Hkv, a.hd = 17, 1, 512, 4, 2, 128
    assert N.load().jx_decode_step(a, None) == N.JX_ERR_SHAPE
    a.M, a.hd = 4, 64
    assert N.load().jx_decode_step(a, None) == N.JX_ERR_SHAPE


def test_norm_tail_decode_step_is_bit_identical():
    """The per-op decode step with the norms in the o_proj / down tails (DecoderRuntime.tail_norm) gives
    the same logits, tokens and caches, bit for bit, as with separate jx_norm launches, and launches two
    kernels fewer per layer."""
    from jaxml_b200.runtime import DecoderRuntime, ModelWeights

    cfg = _cfg(d=512, H=4, Hkv=2, L=3, V=1000)
    params = O.init_params("llama", cfg, seed=4, dtype=torch.bfloat16)
    gw = torch.Generator().manual_seed(10)
    body = params["params"]["model"]
    for lp in [body[f"layers_{i}"][n] for i in range(cfg.num_layers)
               for n in ("input_layernorm", "post_attention_layernorm")]:
        lp["weight"] = (1 + 0.1 * torch.randn(cfg.hidden_size, generator=gw)).to(torch.bfloat16)
    B, P, T, n = 7, 45, 256, 5
    g = torch.Generator().manual_seed(8)
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=g, dtype=torch.int32)
    mask = torch.arange(P)[None, :] < torch.tensor([45, 40, 33, 45, 12, 30, 44])[:, None]
    runs = {}
    old = DecoderRuntime.tail_norm
    try:
        for on in (True, False):
            DecoderRuntime.tail_norm = on
            rt = DecoderRuntime(ModelWeights("llama", cfg, params, torch.bfloat16, "cuda:0"), B, T)
            key, sub = TF.split(TF.prng_key(0))
            rt.reset(mask.cuda(), key, sub, n + 1)
            rt.prefill(ids.cuda(), True, 1.0)
            logits = [rt.logits_buf()[:B].clone()]
            for _ in range(n):
                rt.decode_step(True, 1.0)
                logits.append(rt.logits_buf()[:B].clone())
            torch.cuda.synchronize()
            rt.check_status()
            runs[on] = (logits, rt.tokens_out[:, :n + 1].clone(), rt.k_cache.clone(), rt.v_cache.clone(),
                        rt.count_launches_per_decode_step())
    finally:
        DecoderRuntime.tail_norm = old
    a, b = runs[True], runs[False]
    for la, lb in zip(a[0], b[0]):
        assert torch.equal(la, lb)
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])
    assert a[4] == b[4] - 2 * cfg.num_layers + 1   # no norm after o_proj; none after down except the last
