"""Tensor parallelism over torch.distributed ranks (one GPU each).

Every rank holds the same weights and decodes the same tokens; the LM head's
rows are split evenly and the token kernel exchanges each rank's argmax over
NVLink (xp_session_tp_attach). Optionally the FFN is split too: gate|up
columns and the matching down-proj rows per rank, the down-proj sums
exchanged over NVLink inside the same launch. torch.distributed only carries the 64-byte IPC
handles at set-up (any backend, gloo included)."""


def shard_lm_head(session, group=None, shard_ffn=False):
    """Collective: every rank of `group` calls it with its own session. With
    shard_ffn the FFN's gate|up columns and down-proj rows are split too."""
    import torch.distributed as dist
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    handles = [None] * world
    dist.all_gather_object(handles, session.tp_handle(), group=group)
    session.tp_attach(rank, world, handles, shard_ffn=shard_ffn)
    dist.barrier(group)
    return rank, world
