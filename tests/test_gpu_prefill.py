"""Prompts on the tensor cores (spm_prefill) against the oracle's prompt fed
one token per step (spm-batch/examples/serve-demo.rs:84-89).

After a prefill of prompt[:-1] the prompt's last token goes through the
decode step: its logits must be within max|delta| <= 1e-3 * max|logit| of the
oracle's, its greedy pick identical, and the greedy tokens after it too.
"""
import dataclasses

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def close(got, want):
    return float(np.abs(got - want).max()) <= LOGIT_TOL * float(np.abs(want).max())


def prefill_run(recipe, prompts, steps, context=None):
    """Prefill every client's prompt but its last token, then lockstep greedy
    decode on the device; the oracle runs the same prompts one token per
    step.  Returns per-step (device logits, oracle logits)."""
    sh = recipe.shape
    img = eb.synth_gguf(recipe)
    m = eb.Model(img, sh)
    om = O.OracleModel(img, sh)
    n, L = len(prompts), len(prompts[0])
    context = context or L + steps + 2
    s = eb.Session(m, n, context)
    osess = om.session(n, context)
    for i, p in enumerate(prompts):
        s.prefill(i, p[:-1])
        assert s.length(i) == L - 1
    for t in range(L - 1):
        osess.step([p[t] for p in prompts])
    toks = [p[-1] for p in prompts]
    out = []
    for _ in range(steps):
        best, got = s.decode_step(toks, want_logits=True)
        want = osess.step(toks)
        out.append((best, got, want))
        toks = [O.argmax_last(want[i]) for i in range(n)]
        assert best == toks
    s.close()
    m.close()
    return out


@pytest.mark.parametrize("name", list(configs.TINY))
def test_prefill_then_decode_matches_the_oracle(cuda, name):
    r = configs.TINY[name]
    prompts = [configs.prompt_tokens(21, i, 40, r.shape.vocab) for i in range(2)]
    for step, (best, got, want) in enumerate(prefill_run(r, prompts, 6)):
        assert close(got, want), (name, step, float(np.abs(got - want).max()))


def test_prefill_longer_than_one_chunk(cuda):
    # 1100 positions: two chunks of the 1024-row prompt buffers; the second
    # chunk's attention reads the first chunk's keys and values from the cache
    r = configs.TINY["qwen3-q6_k"]
    prompts = [configs.prompt_tokens(22, 0, 1100, r.shape.vocab)]
    for best, got, want in prefill_run(r, prompts, 3):
        assert close(got, want)


@pytest.mark.parametrize("recipe,clients,length", [("qwen3-30b-a3b-q5_k", 8, 160), ("qwen3-8b-q6_k", 1, 300),
                                                   ("olmoe-q2_k", 4, 130), ("smollm2-q8_0", 2, 100)])
def test_prefill_at_benchmark_shapes(cuda, recipe, clients, length):
    # two layers of the benchmark models: real widths, 128 or 64 experts with
    # skewed routing (grouped expert products), Q5_K / Q6_K / Q2_K / Q8_0
    r = configs.RECIPES[recipe]
    r = r.replace(shape=dataclasses.replace(r.shape, layers=2))
    prompts = [configs.prompt_tokens(23, i, length, r.shape.vocab) for i in range(clients)]
    for best, got, want in prefill_run(r, prompts, 3):
        assert close(got, want)


def test_prefill_after_decoded_tokens_and_edge_cases(cuda):
    r = configs.TINY["qwen3moe-q5_k"]
    sh = r.shape
    img = eb.synth_gguf(r)
    m = eb.Model(img, sh)
    om = O.OracleModel(img, sh)
    s = eb.Session(m, 1, 48)
    osess = om.session(1, 48)
    s.prefill(0, [])  # nothing to do
    assert s.length(0) == 0
    # a prefill continues a client that already decoded some tokens
    head = configs.prompt_tokens(24, 0, 5, sh.vocab)
    for t in head:
        s.decode_step([t])
        osess.step([t])
    more = configs.prompt_tokens(25, 0, 20, sh.vocab)
    s.prefill(0, more[:-1])
    for t in more[:-1]:
        osess.step([t])
    best, got = s.decode_step([more[-1]], want_logits=True)
    want = osess.step([more[-1]])
    assert close(got, want) and best[0] == O.argmax_last(want[0])
    with pytest.raises(eb.SpmError) as e:
        s.prefill(0, [sh.vocab])
    assert e.value.name == "SPM_E_ARG"
    with pytest.raises(eb.SpmError) as e:
        s.prefill(0, [1] * 40)
    assert e.value.name == "SPM_E_CONTEXT"
    s.close()
    m.close()
