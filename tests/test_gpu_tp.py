"""Tensor-parallel LM head on two GPUs: with the head's rows split over two
processes, greedy decoding produces the same tokens as one GPU and each rank's
logits shard equals the same rows of the unsharded logits (bit-exact: the
shard's tiles are the same computation). Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling
    from xpose_b200.tp import shard_lm_head
    cfg = DecodeConfig(n_layers=3, vocab=32768, max_seq=128)
    s = DecodeSession.random(cfg, Sampling(greedy=True), seed=9, device=rank)
    prompt = np.arange(10, dtype=np.uint32) * 997 % cfg.vocab
    s.prefill(prompt)
    ref_logits = s.last_logits()
    ref_toks, _ = s.generate(6)
    s.reset()
    shard_lm_head(s)
    s.prefill(prompt)
    logits = s.last_logits()
    toks, _ = s.generate(6)
    units = cfg.vocab // 64
    u0, u1 = units * rank // world, units * (rank + 1) // world
    same_shard = bool(np.array_equal(logits[u0 * 64:u1 * 64], ref_logits[u0 * 64:u1 * 64]))
    q.put((rank, list(map(int, ref_toks)), list(map(int, toks)), same_shard, s.error_word()))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_lm_head_matches_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ref, got, same_shard, err in res:
        assert err == 0
        assert got == ref, (rank, ref, got)
        assert same_shard
