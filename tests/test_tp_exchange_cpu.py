"""Host side of the tensor-parallel LM head (xpose_b200.tp.shard_lm_head):
two gloo ranks on CPU exchange their handles and each attaches with every
rank's handle in rank order. The device side needs two GPUs
(tests/test_gpu_tp.py)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


class FakeSession:
    def __init__(self, rank):
        self.rank = rank
        self.attached = None

    def tp_handle(self):
        return bytes([self.rank]) * 64

    def tp_attach(self, rank, world, handles, shard_ffn=False):
        self.attached = (rank, world, list(handles))
        self.shard_ffn = shard_ffn


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from xpose_b200.tp import shard_lm_head
    s = FakeSession(rank)
    shard_lm_head(s)
    q.put(s.attached)
    dist.destroy_process_group()


def test_handles_exchanged_in_rank_order():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, (r, world, handles) in enumerate(got):
        assert (r, world) == (rank, 2)
        assert handles == [bytes([0]) * 64, bytes([1]) * 64]
