"""Full runs of the benchmark workloads on the device against the oracle's
full runs (tests/golden/runs/*.npz, made by tests/golden/make_runs.py).

The schedule is serve-demo's lockstep (spm-batch/examples/serve-demo.rs:
59-91): every tick one decode step for every client, prompt tokens fed one
per tick, then the greedy picks.  The device follows the oracle's run: its
next token is the oracle's pick, so one tick's result cannot move the
following ticks off the oracle's path.  Every tick of the whole run --
prompt ticks included -- is held to the rule of tests/fullrun_check.py:
equal greedy picks except at near ties, logits at the oracle's eight
largest within 1e-3 * max|logit|, and for routed models a wider allowance
from a client's first routing near tie on (on the device or in the
oracle), used by few client-ticks.  The synthetic model is made here from
its seeded recipe; the golden file records a digest of the bytes it was
made from.
"""
from pathlib import Path

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from tests.fullrun_check import RunCheck

pytestmark = pytest.mark.gpu

RUNS = Path(__file__).resolve().parent / "golden" / "runs"


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
    check = RunCheck(g, n)
    for t in range(ticks):
        best, logits = s.decode_step(toks, want_logits=True)
        gaps = s.route_gaps(n).min(axis=0) if recipe.shape.moe else None
        check.tick(t, best, logits, gaps)
        oracle = g["argmax"][t].tolist()
        toks = [p[t + 1] if t + 1 < len(p) else oracle[i] for i, p in enumerate(prompts)]
    s.close()
    m.close()
    print(f"{name}: {check.finish()}")


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
    check = RunCheck(g, n)
    for t in range(L - 1):
        check.note_prompt(t)
    toks = [p[-1] for p in prompts]
    for t in range(L - 1, L + w["steps"] - 1):
        best, logits = s.decode_step(toks, want_logits=True)
        check.tick(t, best, logits, s.route_gaps(n).min(axis=0))
        toks = g["argmax"][t].tolist()
    s.close()
    m.close()
    print(f"{name} with tensor-core prompts: {check.summary()}")

