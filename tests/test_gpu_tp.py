"""Tensor parallelism on two GPUs: with the LM head's rows split over two
processes (and, in the second mode, the FFN's gate|up columns and down-proj
rows too, the down-proj sums exchanged between the ranks in int64), greedy
decoding produces the same tokens as one GPU and each rank's logits shard
equals the same rows of the unsharded logits (bit-exact: the shard's tiles
are the same computation, and the per-unit int64 down-proj sums do not depend
on their order; the FFN mode's one-GPU reference is the same kernel attached
at one rank).
Sampled decoding (top-k 64 / top-p 0.95) gathers every shard's candidate
lists over peer memory and draws the same tokens as one GPU. Prefill
(launches without logits) and decode both run sharded. Skipped with fewer
than two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _worker(rank, world, port, q, shard_ffn, greedy):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling
    from xpose_b200.tp import shard_lm_head
    cfg = DecodeConfig(n_layers=3, vocab=32768, max_seq=128)
    sp = Sampling(greedy=True) if greedy else Sampling(greedy=False, temperature=1.0, top_k=64, top_p=0.95, seed=5)
    s = DecodeSession.random(cfg, sp, seed=9, device=rank)
    prompt = np.arange(10, dtype=np.uint32) * 997 % cfg.vocab
    # the tensor-parallel kernel at one rank: the bit-exact reference
    s.tp_attach(0, 1, [s.tp_handle()], shard_ffn=True)
    s.prefill(prompt)
    ref_logits = s.last_logits()
    ref_toks, _ = s.generate(12)
    s.reset()
    shard_lm_head(s, shard_ffn=shard_ffn)
    s.prefill(prompt)
    logits = s.last_logits()
    toks, _ = s.generate(12)
    units = cfg.vocab // 64
    u0, u1 = units * rank // world, units * (rank + 1) // world
    same_shard = bool(np.array_equal(logits[u0 * 64:u1 * 64], ref_logits[u0 * 64:u1 * 64]))
    q.put((rank, list(map(int, ref_toks)), list(map(int, toks)), same_shard, s.error_word()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("shard_ffn,greedy", [(False, True), (True, True), (True, False)])
def test_sharded_decode_matches_one_gpu(shard_ffn, greedy):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, shard_ffn, greedy)) for r in range(2)]
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
