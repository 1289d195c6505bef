"""Expert parallelism over the GPUs of one node: host-side plumbing.

Experts are dealt round robin: expert e lives on rank e % world.  Every rank
runs the whole decode step for every client; only the expert GEMVs are split,
and each rank writes its experts' output rows into every rank's exchange
buffer over NVLink (peer memory mapped by CUDA IPC).  This module exchanges
the IPC handles through torch.distributed -- the only collective the path
needs, once per session.
"""
from __future__ import annotations


def owned_experts(experts: int, world: int, rank: int) -> list[int]:
    """The experts rank `rank` holds and computes."""
    if not 1 <= world <= 8 or not 0 <= rank < world:
        raise ValueError("expert parallel: 1 to 8 ranks")
    return list(range(rank, experts, world))


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' handles in rank order (torch.distributed all_gather_object)."""
    import torch.distributed as dist

    if len(handle) != 64:
        raise ValueError("CUDA IPC handles are 64 bytes")
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


def connect(session, group=None) -> None:
    """Map every rank's exchange buffer into `session` (call on every rank)."""
    session.ep_connect(exchange_handles(session.ep_handle(), group))
