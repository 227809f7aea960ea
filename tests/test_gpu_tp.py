"""Tensor parallelism on 2 GPUs (NCCL): per-rank logits shards and tokens against the oracle.

Skipped when fewer than two GPUs are visible.  Each rank runs in its own process (one process per GPU),
exactly like the production path.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg():
    from jaxml_b200.config import ModelConfig

    return ModelConfig(head_dim=128, hidden_size=1024, num_heads=8, num_kv_heads=2, num_layers=2,
                       max_position_embeddings=1024, vocab_size=2048, intermediate_ratio=(11, 4), norm_eps=1e-5,
                       rope_theta=500000.0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, ids, q):
    import datetime

    import torch.distributed as dist

    from jaxml_b200.engine import TPComm
    from jaxml_b200.runtime import DecoderRuntime, ModelWeights
    from oracle import jaxml_oracle as O
    from oracle import threefry as TF

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        cfg = _cfg()
        params = O.init_params("llama", cfg, seed=1)
        B, P = ids.shape
        w = ModelWeights("llama", cfg, params, torch.bfloat16, f"cuda:{rank}", tp_rank=rank, tp_size=world)
        comm = TPComm()
        runs = []
        # decode's row-parallel projections: push form (fused with the exchange), then the pull all-reduce
        for push in (True, False):
            rt = DecoderRuntime(w, B, 256, comm=comm)
            rt.peer_push = push
            key, sub = TF.split(TF.prng_key(0))
            rt.reset(torch.ones(B, P, dtype=torch.bool, device="cuda"), key, sub, 8)
            rt.prefill(ids.cuda(), True, 1.0)
            torch.cuda.synchronize()
            logits = [rt.logits_buf()[:B].float().cpu()]
            toks = [rt.tokens_out[:, 0].cpu()]
            for _ in range(2):
                rt.decode_step(True, 1.0)
                torch.cuda.synchronize()
                logits.append(rt.logits_buf()[:B].float().cpu())
                toks.append(rt.next_ids.cpu())
            rt.check_status()
            # filtered temperature sampling over the gathered vocabulary (CUDA-graph decode): every rank
            # must draw the same tokens
            rt.filters = (20, 0.9, 0.01)
            ftoks = rt.generate(ids.cuda(), torch.ones(B, P, dtype=torch.bool, device="cuda"), 6, False, 0.8,
                                3).cpu()
            rt.check_status()
            rt.graph = None
            toks.append(ftoks)
            runs.append((logits, toks))
            del rt
        comm.close()
        logits, toks = runs[0]
        same = all(torch.equal(a, b) for a, b in zip(runs[0][0], runs[1][0])) and all(
            torch.equal(a, b) for a, b in zip(runs[0][1], runs[1][1]))
        toks = toks + [torch.tensor([1 if same else 0])]
        q.put((rank, logits, toks, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, None, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_logit_shards_and_tokens_match_oracle():
    from oracle import jaxml_oracle as O

    cfg = _cfg()
    B, P = 3, 24
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=torch.Generator().manual_seed(4), dtype=torch.int32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ids, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, logits, toks, err = q.get(timeout=240)
        assert err is None, f"rank {rank}: {err}"
        res[rank] = (logits, toks)
    for p in procs:
        p.join(timeout=60)
    # both ranks agree on every sampled token
    for a, b in zip(res[0][1], res[1][1]):
        assert torch.equal(a, b)
    # the push form gives bit-identical logits and tokens to the pull all-reduce, on every rank
    assert int(res[0][1][-1][0]) == 1 and int(res[1][1][-1][0]) == 1
    params = O.init_params("llama", cfg, seed=1)
    caches = tuple(O.OracleKVCache(256, torch.bfloat16) for _ in range(cfg.num_layers))
    out = O.forward("llama", cfg, params, ids, torch.bfloat16, kv_caches=caches, keep_last_n_logits=1)
    half = cfg.vocab_size // 2
    for step in range(3):
        full = torch.cat([res[0][0][step], res[1][0][step]], dim=1)
        err = (full - out.logits[:, 0].float()).abs().max().item()
        assert err <= 2e-2, (step, err)
        if step < 2:
            tok = res[0][1][step]
            out = O.forward("llama", cfg, params, tok[:, None], torch.bfloat16, kv_caches=out.kv_caches,
                            keep_last_n_logits=1)
    assert half == res[0][0][0].shape[1]


def _allreduce_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from jaxml_b200.engine import TPComm

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        comm = TPComm()
        dev = torch.device("cuda", rank)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        assert comm.prepare_peer(dev) is not None
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        out = torch.empty(TPComm.PEER_MAX_FLOATS, device=dev)

        def reference(x):   # the rank-order sum of every rank's input
            parts = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(parts, x)
            want = parts[0].clone()
            for r in range(1, world):
                want += parts[r]
            return want

        results = []
        for n in (4, 16 * 4096, 1 * 4096, TPComm.PEER_MAX_FLOATS, 64 * 128, 8):
            x = torch.randn(n, device=dev, generator=g)
            src = comm.partial_buffer(n)
            src.copy_(x)
            want = reference(x)
            comm.all_reduce_partial(src, out[:n], status)
            torch.cuda.synchronize()
            results.append((n, bool(torch.equal(out[:n], want)), out[:n].sum().item()))
        # two calls (both buffers) captured in one CUDA graph and replayed: the call counter lives on
        # the device and the buffers alternate
        n = 16 * 4096
        x = torch.randn(n, device=dev, generator=g)
        srcs = [comm.partial_buffer(n)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        out2 = torch.empty(n, device=dev)
        with torch.cuda.graph(graph, stream=s):
            comm.all_reduce_partial(srcs[0], out[:n], status)
            srcs.append(comm.partial_buffer(n))
            comm.all_reduce_partial(srcs[1], out2, status)
        for rep in range(5):
            srcs[0].copy_(x * (rep + 1))
            srcs[1].copy_(x * (rep + 2))
            torch.cuda.synchronize()
            dist.barrier()
            graph.replay()
            torch.cuda.synchronize()
            ok = torch.equal(out[:n], reference(x * (rep + 1))) and torch.equal(out2, reference(x * (rep + 2)))
            results.append((f"graph{rep}", bool(ok), out2.sum().item()))
        del graph
        st = int(status.item())
        comm.close()
        q.put((rank, results, st, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, None, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_peer_allreduce_matches_rank_order_sum():
    """NVLink peer all-reduce (jx_allreduce_f32): bit-identical to the rank-order sum on every rank, for
    several sizes and across CUDA-graph replays."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_allreduce_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, results, st, err = q.get(timeout=240)
        assert err is None, f"rank {rank}: {err}"
        assert st == 0, f"rank {rank}: status {st}"
        res[rank] = results
    for p in procs:
        p.join(timeout=60)
    for (n0, ok0, s0), (n1, ok1, s1) in zip(res[0], res[1]):
        assert ok0 and ok1, n0
        assert s0 == s1, n0            # every rank holds the same values


def _push_worker(rank, world, port, q):
    """Row-parallel decode projection with the push epilogue + the consuming norm, against the same
    projection stored locally (JX_EPI_STORE_F32), summed in rank order and fed to the same norm."""
    import datetime

    import torch.distributed as dist

    from jaxml_b200 import _native as N
    from jaxml_b200.engine import TPComm

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        lib = N.load()
        comm = TPComm()
        dev = torch.device("cuda", rank)
        peer = comm.prepare_peer(dev)
        assert peer is not None
        stream = torch.cuda.current_stream().cuda_stream
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        g = torch.Generator(device=dev).manual_seed(300 + rank)
        d, K, Mp = 1024, 512, 16
        ws_n = N.LL()
        N.check(lib.jx_linear_decode_workspace(148, 64, ws_n), "ws")
        ws = torch.zeros(ws_n.value, dtype=torch.float32, device=dev)
        cnt = torch.zeros(d // 64 + 1, dtype=torch.int32, device=dev)
        nw = (1.0 + 0.1 * torch.randn(d, device=dev, generator=torch.Generator(device=dev).manual_seed(7)))
        nw = nw.to(torch.bfloat16)

        def pack(t, rp, kp):
            out = torch.empty(rp * kp, dtype=torch.bfloat16, device=dev)
            N.check(lib.jx_pack_k128(t.data_ptr(), N.JX_BF16, t.shape[0], t.shape[1], t.shape[1], 0, out.data_ptr(),
                                     rp, kp, stream), "pack")
            return out

        results = []
        for impl in (1, 2):
            N.check(lib.jx_set_decode_linear_impl(impl), "impl")
            for M in (16, 5):
                x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
                w = (0.05 * torch.randn(d, K, device=dev, generator=g)).to(torch.bfloat16)
                bias = torch.randn(d, device=dev, generator=g).to(torch.bfloat16) if rank == 0 else None
                xp, wp = pack(x, Mp, K), pack(w, d, K)
                part = torch.zeros(M, d, dtype=torch.float32, device=dev)
                # the residual stream is replicated: the same on every rank
                hg = torch.Generator(device=dev).manual_seed(11 + M + 100 * impl)
                h0 = torch.randn(M, d, device=dev, generator=hg).to(torch.bfloat16)

                def linear(push):
                    e = N.JxEpilogue()
                    e.kind, e.M, e.N = N.JX_EPI_STORE_F32, M, d
                    e.out, e.ldo = part.data_ptr(), d
                    e.bias = None if bias is None else bias.data_ptr()
                    if push:
                        peer.push_epilogue(e, d)
                        e.out = None
                    N.check(lib.jx_linear_decode(wp.data_ptr(), xp.data_ptr(), d, K, M, e, ws.data_ptr(), ws.numel(),
                                                 cnt.data_ptr(), status.data_ptr(), 148, 1, stream), "linear")

                def norm(push, h, out, a=None):
                    args = N.JxNormArgs()
                    args.M, args.d, args.eps, args.kind = M, d, 1e-5, N.JX_NORM_RMS
                    args.h, args.ldh, args.w = h.data_ptr(), d, nw.data_ptr()
                    args.out, args.ldo = out.data_ptr(), d
                    args.status = status.data_ptr()
                    if push:
                        peer.push_norm(args, d, d)
                    else:
                        args.a, args.a_f32, args.lda = a.data_ptr(), 1, d
                    N.check(lib.jx_norm(args, N.JX_BF16, 1, stream), "norm")

                def expected():
                    linear(False)
                    parts = [torch.empty_like(part) for _ in range(world)]
                    dist.all_gather(parts, part)
                    tot = parts[0].clone()
                    for r in range(1, world):
                        tot += parts[r]
                    h, out = h0.clone(), torch.zeros(M, d, dtype=torch.bfloat16, device=dev)
                    norm(False, h, out, tot)
                    torch.cuda.synchronize()
                    return h, out

                def check(tag, h, out):
                    want_h, want_out = expected()
                    results.append((f"{impl}/{M}/{tag}", bool(torch.equal(h, want_h) and torch.equal(out, want_out)),
                                    out.float().sum().item()))

                # eager, twice (both slot sets)
                for rep in range(2):
                    h, out = h0.clone(), torch.zeros(M, d, dtype=torch.bfloat16, device=dev)
                    linear(True)
                    norm(True, h, out)
                    torch.cuda.synchronize()
                    check(f"eager{rep}", h, out)
                # one push per graph (odd): replays alternate sets by the device-side epoch
                h, out = h0.clone(), torch.zeros(M, d, dtype=torch.bfloat16, device=dev)
                s = torch.cuda.Stream(device=dev)
                s.wait_stream(torch.cuda.current_stream())
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    stream = s.cuda_stream
                    linear(True)
                    norm(True, h, out)
                stream = torch.cuda.current_stream().cuda_stream
                for rep in range(5):
                    x.copy_(torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16))
                    xp.copy_(pack(x, Mp, K))
                    h.copy_(h0)
                    torch.cuda.synchronize()
                    dist.barrier()
                    graph.replay()
                    torch.cuda.synchronize()
                    check(f"graph{rep}", h.clone(), out.clone())
                del graph
        N.check(lib.jx_set_decode_linear_impl(0), "impl")
        st = int(status.item())
        comm.close()
        q.put((rank, results, st, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, None, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_push_projection_matches_pull_sum():
    """JX_EPI_PUSH_F32 decode projection + push-mode norm: bit-identical to the locally stored partials
    summed in rank order and normalised, for both decode kernels, eager and across CUDA-graph replays of
    an odd number of pushes."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_push_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, results, st, err = q.get(timeout=240)
        assert err is None, f"rank {rank}: {err}"
        assert st == 0, f"rank {rank}: status {st}"
        res[rank] = results
    for p in procs:
        p.join(timeout=60)
    for (n0, ok0, s0), (n1, ok1, s1) in zip(res[0], res[1]):
        assert ok0 and ok1, n0
        assert s0 == s1, n0            # every rank holds the same values
