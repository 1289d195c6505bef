"""Full runs of the benchmark workloads on the device against the oracle's
full runs (tests/golden/runs/*.npz, made by tests/golden/make_runs.py).

The schedule is serve-demo's lockstep (spm-batch/examples/serve-demo.rs:
59-91): every tick one decode step for every client, prompt tokens fed one
per tick, then the greedy picks.  The device follows the oracle's run: its
next token is the oracle's pick, so one tick's result cannot move the
following ticks off the oracle's path.  At every tick of the whole run --
prompt ticks included -- the device's greedy pick must equal the oracle's,
and its logits at the oracle's eight largest must lie within
1e-3 * max|logit| of the oracle's values.  The one exception is a near tie:
where the oracle's best and the device's pick lie within TIE * max|logit| in
the oracle's own logits (the order of the fp32 sums decides between them;
the golden files hold a handful of such ticks among thousands), either is
accepted.  Routed models add a second kind of near tie: where, on the
device, a client's K-th routing probability and the next one lie within
ROUTE_TIE of each other, the two sides may route that client through
different experts in that layer; that tick's logits are then held to
ROUTE_SLACK * max|logit|, and fewer than one client-tick in a thousand may
need it.  The synthetic model is made here from its seeded recipe; the
golden file records a digest of the bytes it was made from.
"""
import dataclasses
from pathlib import Path

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs

pytestmark = pytest.mark.gpu

RUNS = Path(__file__).resolve().parent / "golden" / "runs"
LOGIT_TOL = 1e-3
TIE = 1e-4
# Routed models: where a client's routing on the device had a near tie (the
# K-th and the next routing probability within ROUTE_TIE of each other,
# relatively) the device may pick the other expert set; that tick's logits
# are held to ROUTE_SLACK instead, and such ticks must stay rare.
ROUTE_TIE = 1e-4
ROUTE_SLACK = 1e-2


def _digest(img):
    import sys

    sys.path.insert(0, str(RUNS.parent))
    from make_runs import image_digest

    return image_digest(img)


def _load(name):
    path = RUNS / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"no golden run for {name}")
    return np.load(path)


def _check_tick(t, best, logits, g, route_tie=None, gaps=None):
    """Returns (near ties the device decided the other way, clients exempted
    for a routing near tie).  route_tie[i]: in this tick client i's routing
    had a near tie in some layer on the device (spm_session_route_gaps)."""
    ids, vals, scale = g["top_ids"][t], g["top_vals"][t], g["maxabs"][t]
    ties = exempt = 0
    for i in range(len(best)):
        rt = route_tie is not None and bool(route_tie[i])
        bound = ROUTE_SLACK if rt else TIE
        want = int(g["argmax"][t][i])
        if best[i] != want:
            where = np.nonzero(ids[i] == best[i])[0]
            assert where.size and vals[i][0] - vals[i][where[0]] <= bound * scale[i], \
                f"tick {t} client {i}: greedy pick {best[i]} != {want} (not a near tie)"
            ties += 1
        err = np.abs(logits[i, ids[i]] - vals[i]).max()
        if err > LOGIT_TOL * scale[i]:
            # an expert set that differs from the oracle's at a routing near tie
            gap = None if gaps is None else float(gaps[i])
            assert rt and err <= ROUTE_SLACK * scale[i], (t, i, float(err), float(scale[i]), gap)
            exempt += 1
    return ties, exempt


def _model(name):
    w = configs.WORKLOADS[name]
    recipe = configs.RECIPES[w["recipe"]]
    img = eb.synth_gguf(recipe)
    return w, recipe, img


@pytest.mark.parametrize("name", ["qwen3-8b-b1", "qwen3-8b-b4", "olmoe-q6_k-b8", "olmoe-q2_k-b8", "qwen3-30b-b8"])
def test_full_run_matches_the_oracle(cuda, name):
    g = _load(name)
    w, recipe, img = _model(name)
    assert _digest(img) == str(g["digest"]), "the synthetic model differs from the one the golden run used"
    prompts = configs.workload_prompts(name)
    m = eb.Model(img, recipe.shape)
    del img
    n, longest = len(prompts), max(len(p) for p in prompts)
    ticks = longest + w["steps"] - 1
    assert g["argmax"].shape == (ticks, n)
    s = eb.Session(m, n, longest + w["steps"] + 1)
    toks = [p[0] for p in prompts]
    ties = exempt = 0
    for t in range(ticks):
        best, logits = s.decode_step(toks, want_logits=True)
        gaps = s.route_gaps(n).min(axis=0) if recipe.shape.moe else None
        a, b = _check_tick(t, best, logits, g, None if gaps is None else gaps < ROUTE_TIE, gaps)
        ties, exempt = ties + a, exempt + b
        oracle = g["argmax"][t].tolist()
        toks = [p[t + 1] if t + 1 < len(p) else oracle[i] for i, p in enumerate(prompts)]
    s.close()
    m.close()
    near = int((g["margin"] <= TIE * g["maxabs"]).sum())
    print(f"{name}: {ticks * n} client-ticks, {ties} greedy near ties decided the other way, "
          f"{exempt} logit checks at routing near ties")
    assert ties <= near + exempt, (ties, near, exempt)
    assert exempt <= 0.001 * ticks * n, exempt


def test_full_run_with_tensor_core_prompts(cuda):
    """Qwen3-30B-A3B b8 with every client's prompt (but its last token) run by
    spm_prefill on the tensor cores: from the prompt's last tick on, the
    greedy picks and logits match the oracle's token-by-token run."""
    name = "qwen3-30b-b8"
    g = _load(name)
    w, recipe, img = _model(name)
    prompts = configs.workload_prompts(name)
    m = eb.Model(img, recipe.shape)
    del img
    n, L = len(prompts), len(prompts[0])
    assert all(len(p) == L for p in prompts)
    s = eb.Session(m, n, L + w["steps"] + 1)
    for i, p in enumerate(prompts):
        s.prefill(i, p[:-1])
    toks = [p[-1] for p in prompts]
    for t in range(L - 1, L + w["steps"] - 1):
        best, logits = s.decode_step(toks, want_logits=True)
        _check_tick(t, best, logits, g, s.route_gaps(n).min(axis=0) < ROUTE_TIE)
        toks = g["argmax"][t].tolist()
    s.close()
    m.close()

