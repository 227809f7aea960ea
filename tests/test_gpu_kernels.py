"""Kernel-level GPU tests through the C ABI: layout packing, projections, sampling."""
import numpy as np
import pytest
import torch

from oracle import threefry as TF

pytestmark = pytest.mark.gpu


def _n():
    from jaxml_b200 import _native as N

    N.load()
    return N


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _rup(x, m):
    return (x + m - 1) // m * m


def _assert_rounded_dot(out, x, w):
    """out == bf16 rounding of x @ w.T up to half a bf16 ulp plus float32 accumulation noise."""
    ref = x.double() @ w.double().T
    err = (out.double() - ref).abs()
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 7)
    # tensor-core float32 accumulation: allow 2^-16 of the absolute-value sum for ordering / alignment
    acc = 2.0 ** -16 * ((x.double().abs() @ w.double().abs().T))
    bad = err > 0.5 * ulp + acc
    assert not bad.any(), (err[bad].max().item(), ref[bad][:4].tolist(), out.double()[bad][:4].tolist())


def _pack(N, w_nk, rp, kp):
    """[rows, K] float tensor -> K128 bf16."""
    out = torch.empty(rp * kp, dtype=torch.bfloat16, device="cuda")
    src = w_nk.contiguous()
    dt = N.JX_BF16 if src.dtype == torch.bfloat16 else N.JX_F32
    N.call("jx_pack_k128", src.data_ptr(), dt, src.shape[0], src.shape[1], src.shape[1], 0, out.data_ptr(), rp, kp,
           _stream())
    return out


def test_pack_unpack_roundtrip():
    N = _n()
    x = torch.randn(37, 300, device="cuda").to(torch.bfloat16)
    p = _pack(N, x, 40, 384)
    y = torch.empty(37, 300, dtype=torch.bfloat16, device="cuda")
    N.call("jx_unpack_k128", p.data_ptr(), 37, 300, 40, y.data_ptr(), N.JX_BF16, 300, _stream())
    assert torch.equal(x, y)
    # the layout formula, checked element by element on a small case
    pc = p.cpu().float()
    xc = x.cpu().float()
    for r, k in [(0, 0), (5, 7), (8, 9), (36, 299), (17, 130)]:
        off = ((k // 128) * (40 // 8) + r // 8) * 1024 + ((k % 128) // 8) * 64 + (r % 8) * 8 + k % 8
        assert pc[off] == xc[r, k]


def _epi(N, kind, M, n_valid, out, ldo, out_rp=0, res=None, ldr=0, bias=None):
    e = N.JxEpilogue()
    e.kind, e.M, e.N = kind, M, n_valid
    e.out, e.ldo, e.out_rp = out.data_ptr(), ldo, out_rp
    e.res = None if res is None else res.data_ptr()
    e.ldr = ldr
    e.bias = None if bias is None else bias.data_ptr()
    return e


@pytest.mark.parametrize("M,Nn,K", [(1, 6144, 4096), (16, 6144, 4096), (16, 4096, 14336), (33, 512, 1024),
                                    (64, 1000, 384), (5, 100, 48)])
def test_linear_decode_matches_torch(M, Nn, K):
    N = _n()
    torch.manual_seed(0)
    x = (torch.randn(M, K, device="cuda")).to(torch.bfloat16)
    w = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
    Mp = 16 if M <= 16 else (32 if M <= 32 else 64)
    Np, Kp = _rup(Nn, 64), _rup(K, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, w, Np, Kp)
    out = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
    ws_n = N.LL()
    N.check(N.load().jx_linear_decode_workspace(148, 64, ws_n), "ws")
    ws = torch.zeros(ws_n.value, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(Np // 64 + 1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    e = _epi(N, N.JX_EPI_STORE, M, Nn, out, Nn)
    for grid in (148, 7):
        N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Np, Kp, M, e, ws.data_ptr(), ws.numel(),
               cnt.data_ptr(), status.data_ptr(), grid, 0, _stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert int(cnt.abs().sum().item()) == 0   # split-K counters reset themselves
        _assert_rounded_dot(out, x, w)


def test_linear_decode_glu_and_resid():
    N = _n()
    torch.manual_seed(1)
    M, F, K = 16, 96, 256
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    g = (torch.randn(F, K, device="cuda") * 0.05).to(torch.bfloat16)
    u = (torch.randn(F, K, device="cuda") * 0.05).to(torch.bfloat16)
    # interleave in 32-row groups: 32 gate rows then the same 32 up rows
    wgu = torch.stack([g.reshape(-1, 32, K), u.reshape(-1, 32, K)], 1).reshape(2 * F, K)
    Kp = _rup(K, 128)
    xp, wp = _pack(N, x, 16, Kp), _pack(N, wgu, _rup(2 * F, 64), Kp)
    out = torch.zeros(16 * _rup(F, 128), dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(148 * 2 * 64 * 64, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(64, dtype=torch.int32, device="cuda")
    e = _epi(N, N.JX_EPI_GLU_SILU, M, F, out, 0, out_rp=16)
    N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), _rup(2 * F, 64), Kp, M, e, ws.data_ptr(), ws.numel(),
           cnt.data_ptr(), None, 148, 0, _stream())
    got = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    N.call("jx_unpack_k128", out.data_ptr(), M, F, 16, got.data_ptr(), N.JX_BF16, F, _stream())
    gg = (x.float() @ g.float().T).to(torch.bfloat16).float()
    uu = (x.float() @ u.float().T).to(torch.bfloat16).float()
    a = (gg * torch.sigmoid(gg)).to(torch.bfloat16).float()
    ref = (a * uu).to(torch.bfloat16).float()
    assert (got.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item()


@pytest.fixture(params=[2, 1], ids=["tcgen05", "mma_sync"])
def prefill_impl(request):
    N = _n()
    N.call("jx_set_prefill_linear_impl", request.param)
    yield request.param
    N.call("jx_set_prefill_linear_impl", 0)


@pytest.mark.parametrize("M,Nn,K", [(300, 384, 512), (1024, 6144, 4096), (128, 128, 128), (520, 1280, 2048)])
def test_linear_prefill_matches_torch(prefill_impl, M, Nn, K):
    """Prefill projection (tcgen05 and mma.sync kernels), including a 128-token last block (M=300, 520)."""
    N = _n()
    torch.manual_seed(2)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
    Mp, Np, Kp = _rup(M, 128), _rup(Nn, 128), _rup(K, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, w, Np, Kp)
    out = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    e = _epi(N, N.JX_EPI_STORE, M, Nn, out, Nn)
    N.call("jx_linear_prefill", xp.data_ptr(), wp.data_ptr(), Mp, Np, Kp, e, status.data_ptr(), 0, _stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    _assert_rounded_dot(out, x, w)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("greedy", [True, False])
def test_sample_kernel_bit_exact(dtype, greedy):
    N = _n()
    from jaxml_b200.runtime import gumbel_table_bf16

    B, V = 4, 128256
    torch.manual_seed(3)
    logits = (torch.randn(B, V) * 2).to(dtype)
    key = TF.prng_key(7)
    key, sub = TF.split(key)
    rng = torch.from_numpy(np.array([key[0], key[1], sub[0], sub[1]], dtype=np.uint32).view(np.int32).copy()).cuda()
    lg = logits.cuda()
    chunk = 4096
    nchunks = (V + chunk - 1) // chunk
    ws = torch.zeros(B * nchunks, dtype=torch.int64, device="cuda")
    cnt = torch.zeros(B + 1, dtype=torch.int32, device="cuda")
    toks = torch.zeros(B, 2, dtype=torch.int32, device="cuda")
    step = torch.zeros(1, dtype=torch.int32, device="cuda")
    nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
    tab = gumbel_table_bf16().cuda()
    s = N.JxSampleArgs()
    s.B, s.V, s.logits, s.ld = B, V, lg.data_ptr(), V
    s.dtype = N.JX_BF16 if dtype == torch.bfloat16 else N.JX_F32
    s.greedy, s.temp, s.chunk = (1 if greedy else 0), 0.8, chunk
    s.vocab_offset, s.vocab_total = 0, V
    s.rng, s.gumbel_tab, s.ws, s.counters = rng.data_ptr(), tab.data_ptr(), ws.data_ptr(), cnt.data_ptr()
    s.finalize, s.ld_tok, s.tokens_out, s.step, s.next_ids = 1, 2, toks.data_ptr(), step.data_ptr(), nxt.data_ptr()
    s.advance_rng = 1
    N.call("jx_sample", s, 0, _stream())
    torch.cuda.synchronize()
    arr = logits.float().numpy()[:, None, :]
    if greedy:
        want = np.argmax(arr[:, 0], -1)
    elif dtype == torch.bfloat16:
        want = TF.categorical_bf16(sub, arr, 0.8)[:, 0]
    else:
        want = TF.categorical_f32(sub, arr, 0.8)[:, 0]
    assert toks[:, 0].cpu().numpy().tolist() == want.tolist()
    assert nxt.cpu().numpy().tolist() == want.tolist()
    assert int(step.item()) == 1
    k2, s2 = TF.split(key)
    assert rng.cpu().numpy().view(np.uint32).tolist() == [k2[0], k2[1], s2[0], s2[1]]
    assert int(cnt.abs().sum().item()) == 0



def test_linear_prefill_glu_bias_resid(prefill_impl):
    """Prefill projection epilogues: SwiGLU into the K128 layout, then a residual add with bias."""
    N = _n()
    torch.manual_seed(3)
    M, F, K = 300, 192, 256
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    g = (torch.randn(F, K, device="cuda") * 0.05).to(torch.bfloat16)
    u = (torch.randn(F, K, device="cuda") * 0.05).to(torch.bfloat16)
    wgu = torch.stack([g.reshape(-1, 32, K), u.reshape(-1, 32, K)], 1).reshape(2 * F, K)
    Mp, Kp = _rup(M, 128), _rup(K, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, wgu, _rup(2 * F, 128), Kp)
    Fp = _rup(F, 128)
    act = torch.zeros(Mp * Fp, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    e = _epi(N, N.JX_EPI_GLU_SILU, M, F, act, 0, out_rp=Mp)
    N.call("jx_linear_prefill", xp.data_ptr(), wp.data_ptr(), Mp, _rup(2 * F, 128), Kp, e, status.data_ptr(), 0,
           _stream())
    got = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    N.call("jx_unpack_k128", act.data_ptr(), M, F, Mp, got.data_ptr(), N.JX_BF16, F, _stream())
    gg = (x.float() @ g.float().T).to(torch.bfloat16).float()
    uu = (x.float() @ u.float().T).to(torch.bfloat16).float()
    a = (gg * torch.sigmoid(gg)).to(torch.bfloat16).float()
    ref = (a * uu).to(torch.bfloat16).float()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert (got.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item()
    # down-style projection of the activations with bias and residual: out = bf16(bf16(a.Wd + b) + res)
    D = 160
    wd = (torch.randn(D, F, device="cuda") * 0.05).to(torch.bfloat16)
    bias = (torch.randn(D, device="cuda") * 0.1).to(torch.bfloat16)
    res = torch.randn(M, D, device="cuda").to(torch.bfloat16)
    wdp = _pack(N, wd, _rup(D, 128), Fp)
    out = torch.zeros(M, D, dtype=torch.bfloat16, device="cuda")
    e2 = _epi(N, N.JX_EPI_RESID, M, D, out, D)
    e2.bias, e2.res, e2.ldr = bias.data_ptr(), res.data_ptr(), D
    N.call("jx_linear_prefill", act.data_ptr(), wdp.data_ptr(), Mp, _rup(D, 128), Fp, e2, status.data_ptr(), 0,
           _stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    y = (got.float() @ wd.float().T).to(torch.bfloat16).float()
    want = ((y + bias.float()).to(torch.bfloat16).float() + res.float()).to(torch.bfloat16).float()
    err = (out.float() - want).abs()
    assert err.max().item() <= 0.02 * want.abs().max().item(), err.max().item()
