"""Tensor-parallel LM head over torch.distributed ranks (one GPU each).

Every rank holds the same weights and decodes the same tokens; the LM head's
rows are split evenly and the token kernel exchanges each rank's argmax over
NVLink (xp_session_tp_attach). torch.distributed only carries the 64-byte IPC
handles at set-up (any backend, gloo included)."""


def shard_lm_head(session, group=None):
    """Collective: every rank of `group` calls it with its own session."""
    import torch.distributed as dist
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    handles = [None] * world
    dist.all_gather_object(handles, session.tp_handle(), group=group)
    session.tp_attach(rank, world, handles)
    dist.barrier(group)
    return rank, world
