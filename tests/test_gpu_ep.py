"""Expert parallel decode on two GPUs against the single-GPU path and the
oracle: logits bit-for-bit equal to one GPU's on every rank, routes equal to
the oracle's, greedy tokens identical.  Needs two GPUs (skipped with fewer)."""
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

NAMES = ["qwen3moe-q5_k", "olmoe-q2_k"]


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


@pytest.mark.parametrize("name", NAMES)
def test_expert_parallel_on_two_gpus_equals_one_gpu(cuda, name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n, steps, world = 8, 4, 2
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
        single.append((best, logits.copy(), sess.routes(n).copy(), oroutes))
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
    for k in range(world):
        assert not isinstance(got[k], str), got[k]
        for step in range(steps):
            best, logits, routes = got[k][step]
            sbest, slogits, sroutes, oroutes = single[step]
            assert best == sbest, (k, step)
            assert np.array_equal(routes, oroutes), (k, step)
            assert np.array_equal(logits.view(np.uint32), slogits.view(np.uint32)), (k, step)
