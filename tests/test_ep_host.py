"""Expert-parallel host plumbing on CPU: the expert and client partitions,
the IPC handle exchange between two gloo ranks, and the step's exchange
bookkeeping modelled on 2 and 4 gloo ranks (no GPU)."""
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


# ---- the expert-parallel step's bookkeeping, modelled on gloo ranks ----
#
# One routed layer of the engine's expert-parallel step, with numpy stand-ins
# for the kernels and gloo all-gathers for the peer stores: rank r runs the
# "attention block" of its own clients, every rank receives every client's
# post-attention row, routes every client (the oracle's softmax and top-K,
# moe.rs:17-35), computes the selected (client, expert) products of its own
# experts only, and every rank receives every rank's expert rows; each rank
# then combines its own clients in ascending expert id and picks their
# greedy tokens, and the picks are gathered.  The result must equal the
# same layer run in one process, bit for bit, and every selected
# (client, expert) product must be computed by exactly one rank.

_N, _E, _K, _D, _V = 8, 16, 4, 32, 48


def _layer_weights():
    import numpy as np

    rng = np.random.default_rng(20240611)
    x = rng.standard_normal((_N, _D), dtype=np.float32)
    wa = rng.standard_normal((_D, _D), dtype=np.float32) * np.float32(0.1)
    wr = rng.standard_normal((_E, _D), dtype=np.float32)
    we = rng.standard_normal((_E, _D, _D), dtype=np.float32) * np.float32(0.1)
    wl = rng.standard_normal((_V, _D), dtype=np.float32)
    return x, wa, wr, we, wl


def _attention_block(x, wa):
    import numpy as np

    return x + np.tanh((wa * x[None, :]).sum(axis=1, dtype=np.float32))


def _expert(we, e, h):
    return (we[e] * h[None, :]).sum(axis=1)


def _route(wr, h):
    from oracle import oracle as O

    return O.top_k(O.softmax_route((wr * h[None, :]).sum(axis=1)), _K)


def _combine(h, sel, rows):
    """h plus the selected experts' weighted rows, ascending expert id."""
    import numpy as np

    y = h.copy()
    for e, w in sorted(sel):
        y = y + np.float32(w) * rows[e]
    return y


def _pick(wl, y):
    from oracle import oracle as O

    return O.argmax_last((wl * y[None, :]).sum(axis=1))


def _layer_one_process():
    x, wa, wr, we, wl = _layer_weights()
    h = [_attention_block(x[c], wa) for c in range(_N)]
    out, picks, used = [], [], set()
    for c in range(_N):
        sel = _route(wr, h[c])
        used |= {e for e, _ in sel}
        y = _combine(h[c], sel, {e: _expert(we, e, h[c]) for e, _ in sel})
        out.append(y)
        picks.append(_pick(wl, y))
    return out, picks, used


def _ep_layer_rank(rank, world, port, q):
    import numpy as np
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, wa, wr, we, wl = _layer_weights()
        mine = ep.owned_clients(_N, world, rank)
        experts = set(ep.owned_experts(_E, world, rank))
        # 1. attention block of this rank's clients; rows to every rank
        h_mine = torch.from_numpy(np.stack([_attention_block(x[c], wa) for c in mine]))
        got = [torch.empty_like(h_mine) for _ in range(world)]
        dist.all_gather(got, h_mine)
        h = torch.cat(got).numpy()
        # 2. every client routed on every rank; this rank's experts only
        routes = [_route(wr, h[c]) for c in range(_N)]
        rows = np.zeros((_E, _N, _D), np.float32)
        computed = torch.zeros((_E, _N), dtype=torch.int32)
        for c, sel in enumerate(routes):
            for e, _ in sel:
                if e in experts:
                    rows[e, c] = _expert(we, e, h[c])
                    computed[e, c] += 1
        dist.all_reduce(computed)
        xbuf = [torch.empty(_E, _N, _D) for _ in range(world)]
        dist.all_gather(xbuf, torch.from_numpy(rows))
        # 3. combine this rank's clients, rows read from each expert's owner
        out = {c: _combine(h[c], routes[c], {e: xbuf[e % world][e, c].numpy() for e, _ in routes[c]})
               for c in mine}
        picks = torch.tensor([_pick(wl, out[c]) for c in mine], dtype=torch.int64)
        allp = [torch.empty_like(picks) for _ in range(world)]
        dist.all_gather(allp, picks)
        want = np.zeros((_E, _N), np.int32)
        for c, sel in enumerate(routes):
            for e, _ in sel:
                want[e, c] = 1
        q.put((rank, {c: out[c].tobytes() for c in mine}, torch.cat(allp).tolist(),
               bool(np.array_equal(computed.numpy(), want))))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_layer_bookkeeping_on_gloo_ranks(world):
    import numpy as np

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_layer_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want_out, want_picks, used = _layer_one_process()
    # every rank's experts take part, so every rank's rows cross the exchange
    assert all(used & set(ep.owned_experts(_E, world, r)) for r in range(world))
    rows = {}
    for rank, out, picks, once in res:
        assert once, f"rank {rank}: a selected (client, expert) product was not computed exactly once"
        assert picks == want_picks
        assert sorted(out) == ep.owned_clients(_N, world, rank)
        rows.update(out)
    assert sorted(rows) == list(range(_N))
    for c in range(_N):
        assert rows[c] == want_out[c].tobytes(), f"client {c}"


def test_clients_are_dealt_in_contiguous_blocks():
    for clients, world in [(8, 1), (8, 2), (8, 4), (8, 8), (4, 2)]:
        blocks = [ep.owned_clients(clients, world, r) for r in range(world)]
        assert sum(blocks, []) == list(range(clients))
        assert {len(b) for b in blocks} == {clients // world}
    with pytest.raises(ValueError, match="multiple of the ranks"):
        ep.owned_clients(6, 4, 0)
    with pytest.raises(ValueError):
        ep.owned_clients(8, 9, 0)
