"""Tensor-parallel host logic on CPU: per-rank weight shards and the collectives of TPComm (gloo)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from jaxml_b200.config import ModelConfig
from jaxml_b200.models import random_params
from jaxml_b200.runtime import ModelWeights


def _cfg(family):
    if family == "gemma3":
        return ModelConfig(head_dim=8, hidden_size=48, num_heads=4, num_kv_heads=2, num_layers=2,
                           max_position_embeddings=64, vocab_size=96, intermediate_ratio=(3, 1),
                           sliding_window=8, sliding_window_pattern=2)
    return ModelConfig(head_dim=8, hidden_size=32, num_heads=4, num_kv_heads=4 if family == "neox" else 2,
                       num_layers=2, max_position_embeddings=64, vocab_size=96, intermediate_ratio=(3, 1),
                       rotary_pct=0.5 if family == "neox" else 1.0)


@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_tp_shards_reassemble_the_full_weights(family):
    cfg = _cfg(family)
    params = random_params(family, cfg, seed=0)
    full = ModelWeights(family, cfg, params, torch.float32, "cpu")
    shards = [ModelWeights(family, cfg, params, torch.float32, "cpu", tp_rank=r, tp_size=2) for r in range(2)]
    hd = cfg.head_dim
    for li in range(cfg.num_layers):
        fl = full.layers[li]
        sl = [s.layers[li] for s in shards]
        # column-parallel QKV: each shard holds its q heads, then its k heads, then its v heads
        Hq, Hkv = full.Hq, full.Hkv
        fq, fk, fv = fl.wqkv[:, :Hq * hd], fl.wqkv[:, Hq * hd:(Hq + Hkv) * hd], fl.wqkv[:, (Hq + Hkv) * hd:]
        q = torch.cat([s.wqkv[:, :Hq // 2 * hd] for s in sl], 1)
        k = torch.cat([s.wqkv[:, Hq // 2 * hd:(Hq // 2 + Hkv // 2) * hd] for s in sl], 1)
        v = torch.cat([s.wqkv[:, (Hq // 2 + Hkv // 2) * hd:] for s in sl], 1)
        assert torch.equal(q, fq) and torch.equal(k, fk) and torch.equal(v, fv)
        # row-parallel o_proj and down: shards stack along K
        assert torch.equal(torch.cat([s.wo for s in sl], 0), fl.wo)
        F = full.F
        assert torch.equal(torch.cat([s.wd[:F // 2] for s in sl], 0), fl.wd[:F])
        # bias of a row-parallel projection is added once (rank 0)
        if fl.bo is not None:
            assert sl[0].bo is not None and sl[1].bo is None
    # vocabulary-parallel head
    assert torch.equal(torch.cat([s.lm_head for s in shards], 1), full.lm_head)
    assert [s.vocab_offset for s in shards] == [0, cfg.vocab_size // 2]


def test_tp_rejects_indivisible_sizes():
    cfg = _cfg("llama")
    with pytest.raises(ValueError, match="tp_size=3 must divide"):
        ModelWeights("llama", cfg, random_params("llama", cfg), torch.float32, "cpu", tp_rank=0, tp_size=3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from jaxml_b200.engine import TPComm

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = TPComm()
    t = torch.full((3, 4), float(rank + 1))
    comm.all_reduce(t)
    keys = torch.tensor([10 * rank + 1, 10 * rank + 2], dtype=torch.int64)
    g = comm.all_gather_keys(keys)
    q.put((rank, t.tolist(), g.tolist(), comm.size, comm.rank))
    dist.destroy_process_group()


def test_tp_comm_collectives_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=60) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, t, g, size, r in out:
        assert size == 2 and r == rank
        assert t == [[3.0] * 4] * 3
        assert g == [[1, 2], [11, 12]]
