"""Expert parallelism over the GPUs of one node: host-side plumbing.

Experts are dealt round robin: expert e lives on rank e % world.  Clients
are dealt in contiguous blocks: rank r owns clients r*n/world ..
(r+1)*n/world - 1, runs their attention block over their KV cache (on its
GPU only) and stores the post-attention rows into every rank's states over
NVLink; every rank then routes every client and runs its own experts for
them, writing the expert output rows into every rank's exchange buffer; each
rank combines, runs the LM head and picks for its own clients only, and the
picks are gathered by peer stores.  All of it is peer memory mapped by CUDA
IPC.  This module exchanges the IPC handles through torch.distributed -- the
only collective the path needs, once per session.
"""
from __future__ import annotations


def owned_experts(experts: int, world: int, rank: int) -> list[int]:
    """The experts rank `rank` holds and computes."""
    if not 1 <= world <= 8 or not 0 <= rank < world:
        raise ValueError("expert parallel: 1 to 8 ranks")
    return list(range(rank, experts, world))


def owned_clients(clients: int, world: int, rank: int) -> list[int]:
    """The clients whose attention block, KV cache, LM head and pick rank
    `rank` holds (the engine's split: a contiguous block of clients/world)."""
    if not 1 <= world <= 8 or not 0 <= rank < world:
        raise ValueError("expert parallel: 1 to 8 ranks")
    if clients % world:
        raise ValueError("expert parallel: the client count must be a multiple of the ranks")
    per = clients // world
    return list(range(rank * per, (rank + 1) * per))


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
