"""Expert-parallel host plumbing on CPU: the expert partition, and the IPC
handle exchange between two gloo ranks (no GPU)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from emufpga_b200 import ep


def test_experts_are_dealt_round_robin_and_cover_every_expert_once():
    for experts, world in [(64, 2), (128, 8), (8, 3), (128, 1)]:
        seen = []
        for rank in range(world):
            own = ep.owned_experts(experts, world, rank)
            assert all(e % world == rank for e in own)
            seen += own
        assert sorted(seen) == list(range(experts))
    with pytest.raises(ValueError):
        ep.owned_experts(64, 9, 0)
    with pytest.raises(ValueError):
        ep.owned_experts(64, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    handle = bytes([rank]) * 64
    got = ep.exchange_handles(handle)
    q.put((rank, got))
    dist.barrier()
    dist.destroy_process_group()


def test_handles_are_exchanged_in_rank_order_between_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert out[r] == [bytes([0]) * 64, bytes([1]) * 64]


def test_exchange_refuses_a_short_handle():
    with pytest.raises(ValueError):
        ep.exchange_handles(b"x" * 10)
