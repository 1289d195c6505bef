"""Expert parallel decode on two GPUs against the oracle and the single-GPU
path.  Each rank runs the attention block of its own clients (rank k of W:
clients k*n/W .. (k+1)*n/W - 1) and the experts it owns for every client;
the greedy picks are gathered, so every rank returns all n of them.

Checked per step: every rank's greedy picks equal the oracle's for all
clients, the routes equal the oracle's, and the logits of the rank's own
clients lie within 1e-3 * max|logit| of the oracle's and of one GPU's.
Needs two GPUs (skipped with fewer)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import emufpga_b200 as eb
from emufpga_b200 import configs, ep
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = [("qwen3moe-q5_k", 8), ("olmoe-q2_k", 8), ("qwen3moe-q5_k", 2)]
TOL = 1e-3


def _tokens(step, n, vocab):
    return [(step * 31 + i * 19) % vocab for i in range(n)]


def _rank(rank, world, port, name, n, steps, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = configs.TINY[name]
        m = eb.Model(eb.synth_gguf(r), r.shape, device=rank, ep=(world, rank))
        sess = eb.Session(m, n, 16)
        ep.connect(sess)
        dist.barrier()
        out = []
        for step in range(steps):
            best, logits = sess.decode_step(_tokens(step, n, r.shape.vocab), want_logits=True)
            out.append((best, logits.copy(), sess.routes(n).copy()))
            dist.barrier()  # ranks leave only between steps
        q.put((rank, out))
        sess.close()
        m.close()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _close(got, want):
    return float(np.abs(got - want).max()) <= TOL * float(np.abs(want).max())


@pytest.mark.parametrize("name,n", CASES)
def test_expert_parallel_on_two_gpus_matches_the_oracle(cuda, name, n):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    steps, world = 4, 2
    r = configs.TINY[name]
    img = eb.synth_gguf(r)
    m = eb.Model(img, r.shape)
    sess = eb.Session(m, n, 16)
    osess = O.OracleModel(img, r.shape).session(n, 16)
    single = []
    for step in range(steps):
        toks = _tokens(step, n, r.shape.vocab)
        best, logits = sess.decode_step(toks, want_logits=True)
        want, oroutes = osess.step(toks, routes=True)
        single.append((best, logits.copy(), want, oroutes))
    sess.close()
    m.close()

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(k, world, port, name, n, steps, q)) for k in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    per = n // world
    for k in range(world):
        assert not isinstance(got[k], str), got[k]
        own = slice(k * per, (k + 1) * per)
        for step in range(steps):
            best, logits, routes = got[k][step]
            sbest, slogits, want, oroutes = single[step]
            assert best == [O.argmax_last(want[i]) for i in range(n)], (k, step)
            assert best == sbest, (k, step)
            assert np.array_equal(routes, oroutes), (k, step)
            assert _close(logits[own], want[own]), (k, step)
            assert _close(logits[own], slogits[own]), (k, step)


def test_client_count_must_divide_among_the_ranks(cuda):
    r = configs.TINY["qwen3moe-q5_k"]
    m = eb.Model(eb.synth_gguf(r), r.shape, ep=(2, 0))
    s = eb.Session(m, 4, 8)
    with pytest.raises(eb.SpmError) as e:
        s.decode_step([1, 2, 3])
    assert e.value.name == "SPM_E_ARG"
    s.close()
    m.close()
