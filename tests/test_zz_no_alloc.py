"""The allocation-free decode projection, checked against the regular one through the C ABI.

jx_linear_decode_noalloc serves callers that cannot allocate device memory (a handler inside a host
framework's custom-call hook, or any plugin that must not call cudaMalloc): its split-K scratch is a
fixed array inside the library.  Its results must equal those of jx_linear_decode, which uses a
caller-provided workspace, on two calls in a row (the shared array keeps the previous call's contents).
This file sorts last so that a run stopping at the first failure has run every other test first.
"""
import pytest
import torch

from tests.test_gpu_kernels import _epi, _n, _pack, _rup, _stream

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,Nn,K,kind", [(16, 6144, 4096, "store"), (5, 128256, 4096, "store"),
                                         (16, 2 * 14336, 4096, "glu"), (1, 4096, 14336, "resid")])
def test_noalloc_matches_workspace_version(M, Nn, K, kind):
    N = _n()
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
    Mp, Np, Kp = 16, _rup(Nn, 128), _rup(K, 128)
    xp, wp = _pack(N, x, Mp, Kp), _pack(N, w, Np, Kp)
    res = torch.randn(M, Nn, device="cuda").to(torch.bfloat16)

    def make_out():
        if kind == "glu":
            return torch.zeros(Mp * _rup(Nn // 2, 128), dtype=torch.bfloat16, device="cuda")
        return res.clone() if kind == "resid" else torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")

    def epi(out):
        if kind == "glu":
            return _epi(N, N.JX_EPI_GLU_SILU, M, Nn // 2, out, 0, out_rp=Mp)
        if kind == "resid":
            return _epi(N, N.JX_EPI_RESID, M, Nn, out, Nn, res=out, ldr=Nn)
        return _epi(N, N.JX_EPI_STORE, M, Nn, out, Nn)

    # reference: the workspace version
    ref = make_out()
    nws = N.LL()
    N.check(N.load().jx_linear_decode_workspace(148, M, nws), "ws")
    ws = torch.zeros(nws.value, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(Np // 64 + 1, dtype=torch.int32, device="cuda")
    N.call("jx_linear_decode", wp.data_ptr(), xp.data_ptr(), Np, Kp, M, epi(ref), ws.data_ptr(), ws.numel(),
           cnt.data_ptr(), None, 148, 1, _stream())
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(2):
        out = make_out()
        N.call("jx_linear_decode_noalloc", wp.data_ptr(), xp.data_ptr(), Np, Kp, M, epi(out), status.data_ptr(),
               148, 1, _stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        # same kernel, same deterministic split-K order: identical bits
        assert torch.equal(out, ref)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    N = _n()
    lib = N.load()
    e = N.JxEpilogue()
    dummy = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    assert lib.jx_linear_decode_noalloc(dummy.data_ptr(), dummy.data_ptr(), 128, 128, 17, e, None, 148, 0,
                                        _stream()) == N.JX_ERR_SHAPE
    assert b"M must be in [1, 16]" in lib.jx_last_error()
    assert lib.jx_linear_decode_noalloc(dummy.data_ptr(), dummy.data_ptr(), 4096 * 64, 128, 16, e, None, 148, 0,
                                        _stream()) == N.JX_ERR_SHAPE
