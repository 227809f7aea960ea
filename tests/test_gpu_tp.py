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
        rt = DecoderRuntime(w, B, 256, comm=TPComm())
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
