"""A device wait on another rank that nothing answers gives up, reports
SPM_E_TIMEOUT, and leaves the CUDA context usable.

One process, one GPU: the model is rank 0 of an expert-parallel pair, and the
session's rank-1 slot is pointed back at its own exchange buffer, so rank 1's
flags are never raised.  The waits are shortened to 1 ms; every routed
layer's router (for rank 1's rows) and combine (for rank 1's expert rows), and
the gather of the greedy picks, then wait that long on a missing flag, flag
the session's status word and go on (no trap, no fault).  The same context then serves a
single-GPU model whose step matches the oracle.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_exchange_wait_runs_out_and_the_context_stays_usable(cuda):
    r = configs.TINY["qwen3moe-q5_k"]
    sh = r.shape
    img = eb.synth_gguf(r)
    ep = eb.Model(img, sh, ep=(2, 0))
    s = eb.Session(ep, 2, 8)
    own = s.ep_handle()
    s.ep_connect([own, own])  # rank 1 is never there: its flag stays down
    s.set_wait_limit(1_000_000)  # 1 ms
    with pytest.raises(eb.SpmError) as e:
        s.decode_step([3, 17])
    assert e.value.name == "SPM_E_TIMEOUT"
    # the status word was cleared: the session reports the next run-out again
    with pytest.raises(eb.SpmError) as e:
        s.decode_step([5, 9])
    assert e.value.name == "SPM_E_TIMEOUT"
    s.close()
    ep.close()
    # the context still computes: a normal step on the same device matches the oracle
    m = eb.Model(img, sh)
    t = eb.Session(m, 2, 8)
    want = O.OracleModel(img, sh).session(2, 8).step([3, 17])
    best, got = t.decode_step([3, 17], want_logits=True)
    assert float(np.abs(got - want).max()) <= 1e-3 * float(np.abs(want).max())
    assert best == [O.argmax_last(want[i]) for i in range(2)]
    t.close()
    m.close()


def test_wait_limit_must_be_positive(cuda):
    r = configs.TINY["qwen3moe-q5_k"]
    m = eb.Model(eb.synth_gguf(r), r.shape)
    s = eb.Session(m, 1, 4)
    with pytest.raises(eb.SpmError):
        s.set_wait_limit(0)
    s.close()
    m.close()
