"""GPU tests of the tensor-core prefill attention (C ABI) and of whole models whose head size takes the
tensor-core attention paths in both prefill and decode."""
import pytest
import torch

from oracle import jaxml_oracle as O
from oracle import threefry as TF
from tests.test_gpu_kernels import _n, _rup, _stream

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hd,Hq,Hkv,window,S", [(128, 8, 2, 0, 150), (256, 4, 2, 0, 70), (256, 4, 2, 33, 130),
                                                 (64, 4, 4, 0, 64), (128, 8, 8, 20, 100)])
def test_prefill_attention_matches_oracle(hd, Hq, Hkv, window, S):
    """Causal + window + right-padding masks over the cache, including query rows with no visible key
    (padding and window together), against Attention.mha of the oracle."""
    N = _n()
    torch.manual_seed(7)
    B, T, L = 3, 256, 2
    lens = torch.tensor([S, S - 37, 5], dtype=torch.int32)         # valid prompt tokens per row
    kc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16)
    vc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16)
    kc[:, :, S:] = 0
    vc[:, :, S:] = 0
    q = torch.randn(B, S, Hq, hd).to(torch.bfloat16)
    layer = 1
    scale = hd ** -0.5
    Mp = _rup(B * S, 128)
    Kp = _rup(Hq * hd, 128)
    out = torch.zeros(Mp * Kp, dtype=torch.bfloat16, device="cuda")
    qd = q.reshape(B * S, Hq * hd).contiguous().cuda()
    kd, vd = kc.cuda(), vc.cuda()
    pos = (lens - 1).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = N.JxPAttnArgs()
    a.B, a.S, a.Hq, a.Hkv, a.hd, a.T, a.window = B, S, Hq, Hkv, hd, T, window
    a.cache_rows, a.layer_row0 = L * B * T, layer * B * T
    a.q, a.k_base, a.v_base = qd.data_ptr(), kd.data_ptr(), vd.data_ptr()
    a.len_ptr, a.len_add, a.scale = pos.data_ptr(), 1, scale
    a.out, a.out_rp, a.status = out.data_ptr(), Mp, status.data_ptr()
    N.call("jx_prefill_attention", a, 1, _stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = torch.empty(B * S, Hq * hd, dtype=torch.bfloat16, device="cuda")
    N.call("jx_unpack_k128", out.data_ptr(), B * S, Hq * hd, Mp, got.data_ptr(), N.JX_BF16, Hq * hd, _stream())
    got = got.float().cpu().reshape(B, S, Hq, hd)
    mask = torch.arange(T)[None, :] < lens[:, None]
    n_rep = Hq // Hkv
    want = O.mha(q, O.repeat_kv(kc[layer], n_rep), O.repeat_kv(vc[layer], n_rep), mask, True,
                 window if window else None, scale).float()
    err = (got - want).abs()
    ulp = torch.exp2(torch.floor(torch.log2(want.abs().clamp_min(1e-30))) - 7)
    assert err.max().item() <= 4e-3, err.max().item()
    assert (err <= ulp + 1e-6).float().mean().item() >= 0.99


def _shape_cfg(family):
    from jaxml_b200.config import ModelConfig

    if family == "llama":
        return ModelConfig(head_dim=128, hidden_size=1024, num_heads=8, num_kv_heads=2, num_layers=2,
                           max_position_embeddings=1024, vocab_size=2048, intermediate_ratio=(11, 4), norm_eps=1e-5,
                           rope_theta=500000.0)
    return ModelConfig(head_dim=256, hidden_size=640, num_heads=4, num_kv_heads=2, num_layers=4,
                       max_position_embeddings=1024, vocab_size=2048, intermediate_ratio=(4, 1), norm_eps=1e-6,
                       rope_theta=1e6, rope_scale=8.0, sliding_window=24, sliding_window_pattern=2,
                       attn_scale=256 ** -0.5)


@pytest.mark.parametrize("family", ["llama", "gemma3"])
def test_model_with_tensor_core_attention_matches_oracle(family):
    """A bf16 model with head_dim 128 (Llama) / 256 (Gemma3, sliding window 24 on alternate layers):
    padded prefill then decode steps, logits within 2e-2 of the oracle."""
    from jaxml_b200.runtime import DecoderRuntime, ModelWeights

    cfg = _shape_cfg(family)
    params = O.init_params(family, cfg, seed=1)
    B, P, T = 3, 40, 256
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=g, dtype=torch.int32)
    mask = torch.ones(B, P, dtype=torch.bool)
    mask[1, 31:] = False
    rt = DecoderRuntime(ModelWeights(family, cfg, params, torch.bfloat16, "cuda:0"), B, T)
    assert rt.fast_attn
    key, sub = TF.split(TF.prng_key(0))
    rt.reset(mask.cuda(), key, sub, 8)
    rt.prefill(ids.cuda(), greedy=True, temp=1.0)
    torch.cuda.synchronize()
    rt.check_status()
    caches = tuple(O.OracleKVCache(T, torch.bfloat16) for _ in range(cfg.num_layers))
    out = O.forward(family, cfg, params, ids, torch.bfloat16, attention_mask=mask, kv_caches=caches,
                    keep_last_n_logits=1)
    err = (rt.logits_buf()[:B].float().cpu() - out.logits[:, 0].float()).abs().max().item()
    assert err <= 2e-2, err
    tok = rt.tokens_out[:, 0].cpu()
    caches = out.kv_caches
    for _ in range(3):
        rt.decode_step(True, 1.0)
        torch.cuda.synchronize()
        rt.check_status()
        out = O.forward(family, cfg, params, tok[:, None], torch.bfloat16, kv_caches=caches, keep_last_n_logits=1)
        caches = out.kv_caches
        err = (rt.logits_buf()[:B].float().cpu() - out.logits[:, 0].float()).abs().max().item()
        assert err <= 2e-2, err
        tok = rt.next_ids.cpu()


@pytest.mark.parametrize("kind", ["rms", "gemma", "layer"])
@pytest.mark.parametrize("d,ldh,k128,M", [(4096, 4096, True, 600), (3840, 3840, False, 600), (2048, 2112, True, 600),
                                          (256, 256, False, 600), (2048, 2048, True, 603)])
def test_prefill_norm_rows_match_the_per_row_kernel(kind, d, ldh, k128, M):
    """jx_norm at prefill row counts (one warp per row) writes the bits of the same rows normalised in
    calls of fewer rows (one CTA per row), into row-major and K128 outputs, with a row stride above d and
    a row count that is not a multiple of the rows per CTA."""
    N = _n()
    torch.manual_seed(23)
    chunk = 100
    knd = {"rms": N.JX_NORM_RMS, "gemma": N.JX_NORM_GEMMA, "layer": N.JX_NORM_LAYER}[kind]
    h = (2 * torch.randn(M, ldh, device="cuda") + 0.3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16)
    b = (0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16) if kind == "layer" else None
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def call(r0, rows, out, ldo, out_rp):
        a = N.JxNormArgs()
        a.M, a.d, a.eps, a.kind = rows, d, 1e-5, knd
        a.h, a.ldh = h[r0:].data_ptr(), ldh
        a.w, a.b = w.data_ptr(), None if b is None else b.data_ptr()
        a.out, a.ldo, a.out_rp, a.status = out, ldo, out_rp, status.data_ptr()
        N.call("jx_norm", a, N.JX_BF16, 1, _stream())

    ref = torch.empty(M, d, dtype=torch.bfloat16, device="cuda")
    for r0 in range(0, M, chunk):
        call(r0, min(chunk, M - r0), ref[r0:].data_ptr(), d, 0)
    got = torch.empty(M, d, dtype=torch.bfloat16, device="cuda")
    if k128:
        Mp = _rup(M, 128)
        xk = torch.zeros(Mp * d, dtype=torch.bfloat16, device="cuda")
        call(0, M, xk.data_ptr(), d, Mp)
        N.call("jx_unpack_k128", xk.data_ptr(), M, d, Mp, got.data_ptr(), N.JX_BF16, d, _stream())
    else:
        call(0, M, got.data_ptr(), d, 0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(got, ref)
    # against the oracle's norm (float32 statistics in another summation order: within two bf16 ulps)
    x, wc = h[:, :d].cpu(), w.cpu()
    want = {"rms": lambda: O.rmsnorm(x, wc, 1e-5), "gemma": lambda: O.gemma_rmsnorm(x, wc, 1e-5),
            "layer": lambda: O.layernorm(x, wc, b.cpu(), 1e-5)}[kind]().float()
    diff = (got.float().cpu() - want).abs()
    assert bool((diff <= 2.0 ** -6 * want.abs() + 1e-3).all()), diff.max().item()


@pytest.mark.parametrize("hd,Hq,Hkv,rd", [(128, 32, 8, 128), (64, 8, 8, 16), (128, 16, 2, 64), (256, 8, 4, 256)])
def test_prefill_rope_append_rows_match_the_per_head_kernel(hd, Hq, Hkv, rd):
    """jx_qkv_rope_append at prefill row counts (one CTA per token row, 16-byte vectors) writes the bits
    that the same prompts appended one sequence at a time (fewer rows: one warp per head) write: q and
    the K / V cache."""
    N = _n()
    torch.manual_seed(29)
    B, S, T, max_pos = 4, 96, 128, 256
    M, nq = B * S, (Hq + 2 * Hkv) * hd
    qkv = torch.randn(M, nq, device="cuda").to(torch.bfloat16)
    cos, sin = (t.cuda() for t in O.rope_tables(hd, rd / hd, 10000.0, 1.0, max_pos, torch.bfloat16))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def run(m0, rows, q, kc, vc):
        qa = N.JxQkvArgs()
        qa.M, qa.S, qa.Hq, qa.Hkv, qa.hd, qa.rd = rows, S, Hq, Hkv, hd, rd
        qa.qkv, qa.ld_qkv, qa.qn_w, qa.kn_w, qa.eps = qkv[m0:].data_ptr(), nq, None, None, 1e-6
        qa.max_pos, qa.cos, qa.sin, qa.pos_id, qa.decode, qa.T = max_pos, cos.data_ptr(), sin.data_ptr(), None, 0, T
        qa.q_out, qa.k_cache, qa.v_cache, qa.status = q, kc, vc, status.data_ptr()
        N.call("jx_qkv_rope_append", qa, N.JX_BF16, 1, _stream())

    q1 = torch.zeros(M, Hq * hd, dtype=torch.bfloat16, device="cuda")
    k1 = torch.zeros(B, T, Hkv, hd, dtype=torch.bfloat16, device="cuda")
    v1 = torch.zeros_like(k1)
    run(0, M, q1.data_ptr(), k1.data_ptr(), v1.data_ptr())
    q2, k2, v2 = torch.zeros_like(q1), torch.zeros_like(k1), torch.zeros_like(v1)
    for b in range(B):
        run(b * S, S, q2[b * S:].data_ptr(), k2[b].data_ptr(), v2[b].data_ptr())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(q1, q2) and torch.equal(k1, k2) and torch.equal(v1, v2)
    # against the oracle's rotation (q and k rotated in the model dtype: the same bits), v copied
    x = qkv.cpu().view(B, S, Hq + 2 * Hkv, hd)
    pos = torch.arange(S).expand(B, S)
    want_q, want_k = O.apply_rope(x[:, :, :Hq], x[:, :, Hq:Hq + Hkv], cos.cpu(), sin.cpu(), pos)
    assert torch.equal(q1.cpu().view(B, S, Hq, hd), want_q)
    assert torch.equal(k1[:, :S].cpu(), want_k)
    assert torch.equal(v1[:, :S].cpu(), x[:, :, Hq + Hkv:])
    assert not k1[:, S:].any() and not v1[:, S:].any()
