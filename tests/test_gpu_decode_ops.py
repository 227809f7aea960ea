"""GPU tests of the decode-step kernels through the C ABI: both decode projection kernels (tcgen05 and
mma.sync) with their fused epilogues, and the tensor-core decode attention."""
import pytest
import torch

from tests.test_gpu_kernels import _assert_rounded_dot, _epi, _n, _pack, _rup, _stream

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[2, 1], ids=["tcgen05", "mma_sync"])
def impl(request):
    N = _n()
    N.call("jx_set_decode_linear_impl", request.param)
    yield request.param
    N.call("jx_set_decode_linear_impl", 0)


def _ws(N, Np):
    n = N.LL()
    N.check(N.load().jx_linear_decode_workspace(148, 64, n), "ws")
    return (torch.zeros(n.value, dtype=torch.float32, device="cuda"),
            torch.zeros(Np // 64 + 1, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("M,Nn,K", [(1, 6144, 4096), (16, 6144, 4096), (16, 4096, 14336), (16, 28672, 4096),
                                    (33, 512, 1024), (64, 1000, 384), (5, 100, 48), (16, 128256, 4096)])
def test_linear_decode_store(impl, M, Nn, K):
    N = _n()
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
    Mp = 16 if M <= 16 else (32 if M <= 32 else 64)
    Np, Kp = _rup(Nn, 128), _rup(K, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, w, Np, Kp)
    out = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
    ws, cnt = _ws(N, Np)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    e = _epi(N, N.JX_EPI_STORE, M, Nn, out, Nn)
    for grid in (148, 13):
        out.zero_()
        N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Np, Kp, M, e, ws.data_ptr(), ws.numel(),
               cnt.data_ptr(), status.data_ptr(), grid, 1, _stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert int(cnt.abs().sum().item()) == 0
        _assert_rounded_dot(out, x, w)


@pytest.mark.parametrize("M,Nn,K", [(33, 512, 8192), (64, 640, 14336)])
def test_linear_decode_long_k_by_shape(M, Nn, K):
    """By shape, more than 16 token rows over K >= 8192 take the tcgen05 kernel: its results equal the
    float64 dot rounded once, over the full grid and a partial one."""
    N = _n()
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
    Mp = 64 if M > 32 else 32
    Np, Kp = _rup(Nn, 128), _rup(K, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, w, Np, Kp)
    out = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
    ws, cnt = _ws(N, Np)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    e = _epi(N, N.JX_EPI_STORE, M, Nn, out, Nn)
    for grid in (148, 13):
        out.zero_()
        N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Np, Kp, M, e, ws.data_ptr(), ws.numel(),
               cnt.data_ptr(), status.data_ptr(), grid, 1, _stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and int(cnt.abs().sum().item()) == 0
        _assert_rounded_dot(out, x, w)


@pytest.mark.parametrize("M", [3, 16, 40])
def test_linear_decode_glu_resid_bias(impl, M):
    """GLU (SiLU) into a K128 output, then a residual projection with bias, both fused."""
    N = _n()
    torch.manual_seed(1)
    F, K, D = 200, 256, 384
    Mp = 16 if M <= 16 else (32 if M <= 32 else 64)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    g = (torch.randn(F, K, device="cuda") * 0.05).to(torch.bfloat16)
    u = (torch.randn(F, K, device="cuda") * 0.05).to(torch.bfloat16)
    F32 = _rup(F, 32)
    gp = torch.zeros(F32, K, dtype=torch.bfloat16, device="cuda")
    up = torch.zeros_like(gp)
    gp[:F], up[:F] = g, u
    wgu = torch.stack([gp.reshape(-1, 32, K), up.reshape(-1, 32, K)], 1).reshape(2 * F32, K)
    Kp, Np = _rup(K, 128), _rup(2 * F32, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, wgu, Np, Kp)
    act = torch.zeros(Mp * _rup(F, 128), dtype=torch.bfloat16, device="cuda")
    ws, cnt = _ws(N, max(Np, 4096))
    e = _epi(N, N.JX_EPI_GLU_SILU, M, F, act, 0, out_rp=Mp)
    N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Np, Kp, M, e, ws.data_ptr(), ws.numel(),
           cnt.data_ptr(), None, 148, 1, _stream())
    got = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    N.call("jx_unpack_k128", act.data_ptr(), M, F, Mp, got.data_ptr(), N.JX_BF16, F, _stream())
    gg = (x.double() @ g.double().T).to(torch.bfloat16).double()
    uu = (x.double() @ u.double().T).to(torch.bfloat16).double()
    a = (gg * torch.sigmoid(gg)).to(torch.bfloat16).double()
    ref = (a * uu).to(torch.bfloat16).double()
    # inputs of the activation may differ by one bf16 ulp (accumulation order)
    assert (got.double() - ref).abs().max().item() <= 0.03 * ref.abs().max().item()
    # down projection with bias and residual, reading the K128 activations
    wd = (torch.randn(D, F, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(_rup(D, 128), device="cuda") * 0.1).to(torch.bfloat16)
    h = torch.randn(M, D, device="cuda").to(torch.bfloat16)
    h0 = h.clone()
    Npd, Kpd = _rup(D, 128), _rup(F, 128)
    wdp = _pack(N, wd, Npd, Kpd)
    e2 = _epi(N, N.JX_EPI_RESID, M, D, h, D, res=h, ldr=D, bias=bias)
    N.call("jx_linear_decode", wdp.data_ptr(), act.data_ptr(), Npd, Kpd, M, e2, ws.data_ptr(), ws.numel(),
           cnt.data_ptr(), None, 148, 1, _stream())
    torch.cuda.synchronize()
    y = (got.double() @ wd.double().T).to(torch.bfloat16).double()
    y = (y + bias[:D].double()).to(torch.bfloat16).double()
    ref2 = (y + h0.double()).to(torch.bfloat16).double()
    assert (h.double() - ref2).abs().max().item() <= 0.05 * ref2.abs().max().item()


@pytest.fixture(params=[2, 1, 3, 4, 5], ids=["cluster", "split", "column", "cluster-split", "queue"])
def attn_form(request):
    N = _n()
    N.call("jx_set_decode_attention_impl", request.param)
    yield request.param
    N.call("jx_set_decode_attention_impl", 0)


@pytest.mark.parametrize("hd,Hq,Hkv,window,B", [(128, 32, 8, 0, 3), (256, 16, 8, 0, 3), (256, 16, 8, 100, 3),
                                                 (64, 8, 8, 0, 3), (128, 16, 1, 0, 3), (128, 64, 8, 0, 3),
                                                 (128, 32, 8, 0, 20)])
def test_decode_attention_matches_oracle(attn_form, hd, Hq, Hkv, window, B):
    """Tensor-core decode attention (single-pass cluster form; split scores with the split or the column
    pv; the cluster-split form; the queue form) vs the oracle's Attention.mha on a padded cache.

    The kernel rounds at the reference's points (scores, scale, probabilities, output), so results agree
    to about one bf16 ulp.  A q.k accumulated in a different order can round to the neighbouring bf16
    value (|q.k| ~ 40 here, where one ulp is 0.25), which moves that key's probability by a few percent;
    such flips are rare, so the bound is one ulp for 99% of the outputs and 2e-3 absolute for all."""
    from oracle import jaxml_oracle as O

    N = _n()
    torch.manual_seed(5)
    T, L = 768, 2
    # valid keys after the append (B=20: 160 head groups, one CTA per group in the cluster form)
    lens = torch.tensor(([513, 200, 767] * 7)[:B], dtype=torch.int32)
    kc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16)
    vc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16)
    q = torch.randn(B, Hq, hd).to(torch.bfloat16)
    scale = hd ** -0.5
    layer = 1
    kd, vd, qd = kc.cuda(), vc.cuda(), q.cuda()
    pos = (lens - 2).cuda()
    Mp = _rup(B, 16)          # output rows of the K128 layout: every batch row must fit
    Kp = _rup(Hq * hd, 128)
    out = torch.zeros(Mp * Kp, dtype=torch.bfloat16, device="cuda")
    nb = N.LL()
    N.check(N.load().jx_decode_attention_workspace(B, Hq, hd, T, window, nb), "ws")
    ws = torch.zeros(nb.value // 4 + 1, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = N.JxDAttnArgs()
    a.B, a.Hq, a.Hkv, a.hd, a.T, a.window = B, Hq, Hkv, hd, T, window
    a.cache_rows, a.layer_row0 = L * B * T, layer * B * T
    a.q, a.k_base, a.v_base = qd.data_ptr(), kd.data_ptr(), vd.data_ptr()
    a.len_ptr, a.len_add, a.scale = pos.data_ptr(), 2, scale
    a.out, a.out_rp = out.data_ptr(), Mp
    a.ws, a.ws_bytes, a.counters, a.status = ws.data_ptr(), ws.numel() * 4, cnt.data_ptr(), status.data_ptr()
    mask = torch.arange(T)[None, :] < lens[:, None]
    want = O.mha(q[:, None], O.repeat_kv(kc[layer], Hq // Hkv), O.repeat_kv(vc[layer], Hq // Hkv), mask, True,
                 window if window else None, scale)[:, 0].float()
    ulp = torch.exp2(torch.floor(torch.log2(want.abs().clamp_min(1e-30))) - 7)
    for _ in range(2):   # twice: the split counters must reset themselves
        N.call("jx_decode_attention", a, 1, _stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and int(cnt.abs().sum().item()) == 0
        # the queue form's counters (the workspace's last 2 + B * Hq ints) are back at zero
        tail = ws.view(torch.int32)[(nb.value // 4) - (2 + B * Hq):nb.value // 4]
        assert int(tail.abs().sum().item()) == 0
        got = torch.empty(B, Hq * hd, dtype=torch.bfloat16, device="cuda")
        N.call("jx_unpack_k128", out.data_ptr(), B, Hq * hd, Mp, got.data_ptr(), N.JX_BF16, Hq * hd, _stream())
        got = got.float().cpu().reshape(B, Hq, hd)
        err = (got - want).abs()
        assert err.max().item() <= 2e-3, err.max().item()
        assert (err <= ulp + 1e-6).float().mean().item() >= 0.99


def _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, q, kd, vd, pos, fused=None):
    """jx_decode_attention (split form) on cache `kd` / `vd`; `fused` = (qkv, cos, sin, rd, max_pos) reads q,
    k and v from the projection output and appends instead of `q`.  Returns the [B, Hq*hd] output."""
    Mp, Kp = _rup(B, 16), _rup(Hq * hd, 128)
    out = torch.zeros(Mp * Kp, dtype=torch.bfloat16, device="cuda")
    nb = N.LL()
    N.check(N.load().jx_decode_attention_workspace(B, Hq, hd, T, 0, nb), "ws")
    ws = torch.zeros(nb.value // 4 + 1, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = N.JxDAttnArgs()
    a.B, a.Hq, a.Hkv, a.hd, a.T, a.window = B, Hq, Hkv, hd, T, 0
    a.cache_rows, a.layer_row0 = L * B * T, layer * B * T
    a.q, a.k_base, a.v_base = (None if q is None else q.data_ptr()), kd.data_ptr(), vd.data_ptr()
    a.len_ptr, a.len_add, a.scale = pos.data_ptr(), 2, hd ** -0.5
    a.out, a.out_rp = out.data_ptr(), Mp
    a.ws, a.ws_bytes, a.counters, a.status = ws.data_ptr(), ws.numel() * 4, cnt.data_ptr(), status.data_ptr()
    if fused is not None:
        qkv, cos, sin, rd, max_pos = fused
        a.qkv, a.ld_qkv, a.cos, a.sin, a.rd, a.max_pos = qkv.data_ptr(), qkv.shape[1], cos.data_ptr(), sin.data_ptr(), rd, max_pos
    N.call("jx_decode_attention", a, 1, _stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = torch.empty(B, Hq * hd, dtype=torch.bfloat16, device="cuda")
    N.call("jx_unpack_k128", out.data_ptr(), B, Hq * hd, Mp, got.data_ptr(), N.JX_BF16, Hq * hd, _stream())
    torch.cuda.synchronize()
    return got


@pytest.mark.parametrize("hd,Hq,Hkv,rd,B", [(128, 32, 8, 128, 3), (64, 8, 8, 16, 5), (128, 16, 2, 128, 20),
                                             (256, 16, 8, 256, 3)])
def test_decode_attention_fused_rope_matches_separate_kernels(hd, Hq, Hkv, rd, B):
    """RoPE + cache append fused into the decode attention: the same output bits and the same cache as
    jx_qkv_rope_append followed by the attention on its q."""
    from oracle import jaxml_oracle as O

    N = _n()
    torch.manual_seed(7)
    T, L, layer, max_pos = 768, 2, 1, 1024
    lens = torch.tensor(([513, 200, 767, 64, 1] * 4)[:B], dtype=torch.int32)   # valid keys after the append
    kc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16).cuda()
    vc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16).cuda()
    qkv = torch.randn(B, (Hq + 2 * Hkv) * hd).to(torch.bfloat16).cuda()
    cos, sin = (t.cuda() for t in O.rope_tables(hd, rd / hd, 10000.0, 1.0, max_pos, torch.bfloat16))
    pos = (lens - 2).cuda()
    # separate kernels
    k1, v1 = kc.clone(), vc.clone()
    q = torch.empty(B, Hq * hd, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    qa = N.JxQkvArgs()
    qa.M, qa.S, qa.Hq, qa.Hkv, qa.hd, qa.rd = B, 1, Hq, Hkv, hd, rd
    qa.qkv, qa.ld_qkv, qa.qn_w, qa.kn_w, qa.eps = qkv.data_ptr(), qkv.shape[1], None, None, 1e-6
    qa.max_pos, qa.cos, qa.sin, qa.pos_id, qa.decode, qa.T = max_pos, cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), 1, T
    qa.q_out, qa.k_cache, qa.v_cache, qa.status = q.data_ptr(), k1[layer].data_ptr(), v1[layer].data_ptr(), status.data_ptr()
    N.call("jx_qkv_rope_append", qa, N.JX_BF16, 0, _stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    out1 = _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, q, k1, v1, pos)
    # fused
    k2, v2 = kc.clone(), vc.clone()
    out2 = _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, None, k2, v2, pos, fused=(qkv, cos, sin, rd, max_pos))
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    assert torch.equal(out1, out2)
    # the queue form: the split form's bits, fused or not, and twice (its claim counters reset themselves)
    N.call("jx_set_decode_attention_impl", 5)
    try:
        for _ in range(2):
            k3, v3 = kc.clone(), vc.clone()
            out3 = _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, None, k3, v3, pos, fused=(qkv, cos, sin, rd, max_pos))
            assert torch.equal(k1, k3) and torch.equal(v1, v3)
            assert torch.equal(out1, out3)
            assert torch.equal(out1, _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, q, k1, v1, pos))
    finally:
        N.call("jx_set_decode_attention_impl", 0)
    # the other forms do not take the fused inputs
    for form in (2, 3, 4):
        N.call("jx_set_decode_attention_impl", form)
        try:
            with pytest.raises(RuntimeError):
                _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, None, k2, v2, pos, fused=(qkv, cos, sin, rd, max_pos))
        finally:
            N.call("jx_set_decode_attention_impl", 0)


@pytest.mark.parametrize("kind", ["rms", "gemma", "layer"])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_linear_decode_norm_prologue(impl, kind, M):
    """Normalisation prologue of the decode projection (jx_epilogue.pn_*): the activation rows it writes
    match jx_norm's (same arithmetic, another float32 summation order: at most one bf16 ulp on a few
    elements), the projection of them matches the projection of jx_norm's output, and the epoch and
    arrival counters advance and reset over back-to-back calls."""
    N = _n()
    torch.manual_seed(11)
    d, Nn, Mp = 4096, 6144, 16
    knd = {"rms": N.JX_NORM_RMS, "gemma": N.JX_NORM_GEMMA, "layer": N.JX_NORM_LAYER}[kind]
    h = (2 * torch.randn(M, d, device="cuda")).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16)
    b = (0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16) if kind == "layer" else None
    wt = (torch.randn(Nn, d, device="cuda") * 0.02).to(torch.bfloat16)
    wp = _pack(N, wt, Nn, d)
    ws, cnt = _ws(N, Nn)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # reference: jx_norm into the K128 activations, then the projection
    xn_ref = torch.zeros(Mp * d, dtype=torch.bfloat16, device="cuda")
    a = N.JxNormArgs()
    a.M, a.d, a.eps, a.kind = M, d, 1e-5, knd
    a.h, a.ldh, a.w, a.b = h.data_ptr(), d, w.data_ptr(), None if b is None else b.data_ptr()
    a.out, a.ldo, a.out_rp, a.status = xn_ref.data_ptr(), d, Mp, status.data_ptr()
    N.call("jx_norm", a, N.JX_BF16, 0, _stream())
    out_ref = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
    e = _epi(N, N.JX_EPI_STORE, M, Nn, out_ref, Nn)
    N.call("jx_linear_decode", wp.data_ptr(), xn_ref.data_ptr(), Nn, d, M, e, ws.data_ptr(), ws.numel(),
           cnt.data_ptr(), status.data_ptr(), 148, 1, _stream())
    # prologue
    sync = torch.zeros(18, dtype=torch.int32, device="cuda")
    xn = torch.zeros(Mp * d, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
    e2 = _epi(N, N.JX_EPI_STORE, M, Nn, out, Nn)
    e2.pn_h, e2.pn_ldh, e2.pn_w, e2.pn_b = h.data_ptr(), d, w.data_ptr(), None if b is None else b.data_ptr()
    e2.pn_sync, e2.pn_kind, e2.pn_d, e2.pn_eps = sync.data_ptr(), knd, d, 1e-5
    for rep in range(3):
        xn.zero_()
        N.call("jx_linear_decode", wp.data_ptr(), xn.data_ptr(), Nn, d, M, e2, ws.data_ptr(), ws.numel(),
               cnt.data_ptr(), status.data_ptr(), 148, 1, _stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert sync[0].item() == rep + 1 and sync[1].item() == 0 and int(cnt.abs().sum().item()) == 0
        got = torch.empty(M, d, dtype=torch.bfloat16, device="cuda")
        ref = torch.empty(M, d, dtype=torch.bfloat16, device="cuda")
        N.call("jx_unpack_k128", xn.data_ptr(), M, d, Mp, got.data_ptr(), N.JX_BF16, d, _stream())
        N.call("jx_unpack_k128", xn_ref.data_ptr(), M, d, Mp, ref.data_ptr(), N.JX_BF16, d, _stream())
        torch.cuda.synchronize()
        diff = (got.float() - ref.float()).abs()
        ulp = torch.exp2(torch.floor(torch.log2(ref.float().abs().clamp_min(1e-30))) - 7)
        assert bool((diff <= ulp + 1e-12).all()) and (diff > 0).float().mean().item() <= 0.01
        err = (out.float() - out_ref.float()).abs().max().item()
        assert err <= 2e-2 * max(1.0, out_ref.float().abs().max().item()), err
        if bool((diff == 0).all()):
            assert torch.equal(out, out_ref)


@pytest.mark.parametrize("form", [0, 3, 5], ids=["split", "column", "queue"])
@pytest.mark.parametrize("T,lens", [(4096, [4096, 2085, 129]), (32768, [32768, 16421])])
def test_decode_attention_long_context_matches_oracle(form, T, lens):
    """Decode attention at 4k and 32k-key caches (Llama-3-8B heads): the key-split count grows with the
    buffer length (32 and 256 splits of 128 keys), and rows of one batch have different lengths."""
    from oracle import jaxml_oracle as O

    N = _n()
    N.call("jx_set_decode_attention_impl", form)
    try:
        torch.manual_seed(13)
        B, Hq, Hkv, hd, L, layer = len(lens), 32, 8, 128, 1, 0
        lens_t = torch.tensor(lens, dtype=torch.int32)
        kc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16)
        vc = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16)
        q = torch.randn(B, Hq, hd).to(torch.bfloat16)
        got = _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, q.reshape(B, -1).cuda(), kc.cuda(), vc.cuda(),
                          (lens_t - 2).cuda()).float().cpu().reshape(B, Hq, hd)
        for b in range(B):   # one row at a time keeps the oracle's repeated K/V small
            mask = torch.arange(T)[None, :] < lens_t[b:b + 1, None]
            want = O.mha(q[b:b + 1, None], O.repeat_kv(kc[layer, b:b + 1], Hq // Hkv),
                         O.repeat_kv(vc[layer, b:b + 1], Hq // Hkv), mask, True, None, hd ** -0.5)[0, 0].float()
            ulp = torch.exp2(torch.floor(torch.log2(want.abs().clamp_min(1e-30))) - 7)
            err = (got[b] - want).abs()
            assert err.max().item() <= 2e-3, (b, err.max().item())
            assert (err <= ulp + 1e-6).float().mean().item() >= 0.99
    finally:
        N.call("jx_set_decode_attention_impl", 0)


@pytest.mark.parametrize("M,Nn,K", [(1, 6144, 4096), (16, 6144, 4096), (16, 4096, 14336), (16, 4096, 4096),
                                    (7, 512, 1024), (16, 4608, 384)])
def test_linear_decode_row_split(M, Nn, K):
    """The row-split decode projection (jx_set_decode_linear_impl(3)): each CTA takes 32 or 48 output rows
    over the whole K; plain store, then a residual epilogue with bias, against a float64 dot."""
    N = _n()
    N.call("jx_set_decode_linear_impl", 3)
    try:
        torch.manual_seed(2)
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
        Kp = _rup(K, 128)
        xp, wp = _pack(N, x, 16, Kp), _pack(N, w, Nn, Kp)
        out = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
        ws, cnt = _ws(N, Nn)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        e = _epi(N, N.JX_EPI_STORE, M, Nn, out, Nn)
        for _ in range(2):
            out.zero_()
            N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Nn, Kp, M, e, ws.data_ptr(), ws.numel(),
                   cnt.data_ptr(), status.data_ptr(), 148, 1, _stream())
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            _assert_rounded_dot(out, x, w)
        bias = (torch.randn(Nn, device="cuda") * 0.1).to(torch.bfloat16)
        h = torch.randn(M, Nn, device="cuda").to(torch.bfloat16)
        h0 = h.clone()
        e2 = _epi(N, N.JX_EPI_RESID, M, Nn, h, Nn, res=h, ldr=Nn, bias=bias)
        N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Nn, Kp, M, e2, ws.data_ptr(), ws.numel(),
               cnt.data_ptr(), status.data_ptr(), 148, 1, _stream())
        torch.cuda.synchronize()
        y = (x.double() @ w.double().T).to(torch.bfloat16).double()
        y = (y + bias.double()).to(torch.bfloat16).double()
        ref = (y + h0.double()).to(torch.bfloat16).double()
        assert (h.double() - ref).abs().max().item() <= 0.05 * ref.abs().max().item()
        # a grid below the row count's needs is refused, not run
        with pytest.raises(RuntimeError):
            N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Nn, Kp, M, e, ws.data_ptr(), ws.numel(),
                   cnt.data_ptr(), status.data_ptr(), 4, 1, _stream())
    finally:
        N.call("jx_set_decode_linear_impl", 0)


@pytest.mark.parametrize("form", [1, 5], ids=["split", "queue"])
def test_decode_attention_back_to_back_launches(form):
    """Launches on consecutive layers with programmatic dependent launch and no synchronisation between
    them, sharing one workspace and counter array (as a captured decode step replays them): each output
    equals a separately synchronised call's, and the counters are zero afterwards.  The queue form's
    next launch starts while the previous one runs, so its shared counters must not be touched before
    its wait."""
    N = _n()
    torch.manual_seed(17)
    B, Hq, Hkv, hd, T, L = 16, 32, 8, 128, 768, 4
    lens = torch.tensor([640 - 9 * i for i in range(B)], dtype=torch.int32)
    kd = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16).cuda()
    vd = torch.randn(L, B, T, Hkv, hd).to(torch.bfloat16).cuda()
    q = torch.randn(B, Hq * hd).to(torch.bfloat16).cuda()
    pos = (lens - 2).cuda()
    Mp, Kp = _rup(B, 16), _rup(Hq * hd, 128)
    nb = N.LL()
    N.check(N.load().jx_decode_attention_workspace(B, Hq, hd, T, 0, nb), "ws")
    ws = torch.zeros(nb.value // 4 + 1, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = [torch.zeros(Mp * Kp, dtype=torch.bfloat16, device="cuda") for _ in range(L)]
    a = N.JxDAttnArgs()
    a.B, a.Hq, a.Hkv, a.hd, a.T, a.window, a.cache_rows = B, Hq, Hkv, hd, T, 0, L * B * T
    a.q, a.k_base, a.v_base = q.data_ptr(), kd.data_ptr(), vd.data_ptr()
    a.len_ptr, a.len_add, a.scale = pos.data_ptr(), 2, hd ** -0.5
    a.out_rp, a.ws, a.ws_bytes, a.counters, a.status = Mp, ws.data_ptr(), ws.numel() * 4, cnt.data_ptr(), status.data_ptr()
    N.call("jx_set_decode_attention_impl", form)
    try:
        for rep in range(3):
            for layer in range(L):
                a.layer_row0, a.out = layer * B * T, outs[layer].data_ptr()
                N.call("jx_decode_attention", a, 1, _stream())
            torch.cuda.synchronize()
            assert int(status.item()) == 0 and int(cnt.abs().sum().item()) == 0
            tail = ws.view(torch.int32)[(nb.value // 4) - (2 + B * Hq):nb.value // 4]
            assert int(tail.abs().sum().item()) == 0
    finally:
        N.call("jx_set_decode_attention_impl", 0)
    for layer in range(L):
        want = _dattn_call(N, B, Hq, Hkv, hd, T, L, layer, q, kd, vd, pos)
        got = torch.empty(B, Hq * hd, dtype=torch.bfloat16, device="cuda")
        N.call("jx_unpack_k128", outs[layer].data_ptr(), B, Hq * hd, Mp, got.data_ptr(), N.JX_BF16, Hq * hd, _stream())
        torch.cuda.synchronize()
        assert torch.equal(got, want), layer


@pytest.mark.parametrize("kind", ["rms", "gemma", "layer"])
@pytest.mark.parametrize("M,d,K", [(16, 4096, 4096), (1, 4096, 14336), (5, 2048, 1024), (16, 512, 384)])
def test_linear_decode_norm_tail(kind, M, d, K):
    """Normalisation tail of the row-split projection (jx_epilogue.tn_*): the residual stream it writes and
    the normalised activations its last CTA writes are bit-identical to the projection without the tail
    followed by jx_norm, over back-to-back calls (the arrival counter resets itself); a tail on another
    decode kernel is refused before any launch."""
    N = _n()
    torch.manual_seed(19)
    Mp = 16
    knd = {"rms": N.JX_NORM_RMS, "gemma": N.JX_NORM_GEMMA, "layer": N.JX_NORM_LAYER}[kind]
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    wt = (torch.randn(d, K, device="cuda") * 0.02).to(torch.bfloat16)
    Kp = _rup(K, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, wt, d, Kp)
    nw = (1 + 0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16)
    nb = (0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16) if kind == "layer" else None
    h0 = (2 * torch.randn(M, d, device="cuda")).to(torch.bfloat16)
    ws, cnt = _ws(N, d)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    sync = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.call("jx_set_decode_linear_impl", 3)
    try:
        # reference: the projection's residual add, then jx_norm into the K128 activations
        h_ref = h0.clone()
        e = _epi(N, N.JX_EPI_RESID, M, d, h_ref, d, res=h_ref, ldr=d)
        N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), d, Kp, M, e, ws.data_ptr(), ws.numel(),
               cnt.data_ptr(), status.data_ptr(), 148, 1, _stream())
        xn_ref = torch.zeros(Mp * d, dtype=torch.bfloat16, device="cuda")
        a = N.JxNormArgs()
        a.M, a.d, a.eps, a.kind = M, d, 1e-5, knd
        a.h, a.ldh, a.w, a.b = h_ref.data_ptr(), d, nw.data_ptr(), None if nb is None else nb.data_ptr()
        a.out, a.ldo, a.out_rp, a.status = xn_ref.data_ptr(), d, Mp, status.data_ptr()
        N.call("jx_norm", a, N.JX_BF16, 1, _stream())
        torch.cuda.synchronize()
        for rep in range(3):
            h = h0.clone()
            xn = torch.zeros(Mp * d, dtype=torch.bfloat16, device="cuda")
            e2 = _epi(N, N.JX_EPI_RESID, M, d, h, d, res=h, ldr=d)
            e2.tn_x, e2.tn_rp, e2.tn_w, e2.tn_b = xn.data_ptr(), Mp, nw.data_ptr(), None if nb is None else nb.data_ptr()
            e2.tn_sync, e2.tn_kind, e2.tn_eps = sync.data_ptr(), knd, 1e-5
            N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), d, Kp, M, e2, ws.data_ptr(), ws.numel(),
                   cnt.data_ptr(), status.data_ptr(), 148, 1, _stream())
            torch.cuda.synchronize()
            assert int(status.item()) == 0 and int(sync.item()) == 0
            assert torch.equal(h, h_ref)
            assert torch.equal(xn, xn_ref), rep
        N.call("jx_set_decode_linear_impl", 1)
        assert N.load().jx_linear_decode(wp.data_ptr(), xp.data_ptr(), d, Kp, M, e2, ws.data_ptr(), ws.numel(),
                                         cnt.data_ptr(), status.data_ptr(), 148, 1, _stream()) == N.JX_ERR_UNSUPPORTED
    finally:
        N.call("jx_set_decode_linear_impl", 0)
