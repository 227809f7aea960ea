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
