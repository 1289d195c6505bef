"""The whole token loop on the device against the oracle's CPU token loop.

Bars: greedy tokens identical over the run; logits within
max|delta| <= 1e-3 * max|logit| (fp32 accumulation); weight bytes per step
independent of the client count; batched clients get what they get alone.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
DENSE = ["llama-q8_0", "llama-q6_k", "qwen3-q6_k", "qwen3-q5_k", "qwen3-q2_k", "qwen3-g8-q6_k", "qwen3-g4-q5_k"]


def logits_close(got, want):
    bound = LOGIT_TOL * float(np.abs(want).max())
    return float(np.abs(got - want).max()) <= bound


@pytest.fixture(scope="module")
def models():
    cache = {}

    def get(name):
        if name not in cache:
            r = configs.TINY[name]
            img = eb.synth_gguf(r)
            cache[name] = (r, img, eb.Model(img, r.shape), O.OracleModel(img, r.shape))
        return cache[name]

    yield get
    for r, img, m, om in cache.values():
        m.close()


@pytest.mark.parametrize("name", DENSE)
def test_stepwise_logits_match_the_oracle(cuda, models, name):
    # Teacher-forced: both sides see the same token every step.
    r, img, m, om = models(name)
    n, steps = 3, 6
    sess = eb.Session(m, n, 16)
    osess = om.session(n, 16)
    for step in range(steps):
        toks = [(step * 37 + i * 11) % r.shape.vocab for i in range(n)]
        best, got = sess.decode_step(toks, want_logits=True)
        want = osess.step(toks)
        assert logits_close(got, want), (step, float(np.abs(got - want).max()), float(np.abs(want).max()))
        assert best == [O.argmax_last(want[i]) for i in range(n)]
    sess.close()


@pytest.mark.parametrize("name", DENSE)
def test_greedy_serving_matches_the_oracle(cuda, models, name):
    r, img, m, om = models(name)
    prompts = [configs.prompt_tokens(11, i, ln, r.shape.vocab) for i, ln in enumerate([3, 5, 8])]
    want, wl = om.serve(prompts, 10)
    got, gl = eb.serve(m, prompts, 10, want_logits=True)
    assert got == want
    assert logits_close(gl, wl)


def test_batched_clients_get_what_they_get_alone(cuda, models):
    # spm-batch/tests/batching.rs:128-145 on the device
    r, img, m, om = models("qwen3-q6_k")
    prompts = [configs.prompt_tokens(5, i, ln, r.shape.vocab) for i, ln in enumerate([2, 4, 6, 3, 5])]
    together, _ = eb.serve(m, prompts, 6)
    longest = max(len(p) for p in prompts)
    for i, p in enumerate(prompts):
        alone, _ = eb.serve(m, [p], 6 + longest - len(p))
        assert alone[0] == together[i]


def test_weight_bytes_do_not_depend_on_client_count(cuda, models):
    # spm-batch/tests/batching.rs:147-217: bytes per sweep come from the
    # descriptors, not from the clients.
    r, img, m, om = models("llama-q8_0")
    s = r.shape
    per_layer = 2 * s.hidden * s.q_width + 2 * s.hidden * s.kv_width + 3 * s.hidden * s.intermediate
    expect = (s.layers * per_layer + s.vocab * s.hidden) * 34 // 32
    assert m.weight_bytes == expect
    for n in (1, 2, 5):
        sess = eb.Session(m, n, 8)
        sess.decode_step([1] * n)
        assert m.weight_bytes == expect
        sess.close()


def test_context_exhaustion_is_an_error_not_a_fault(cuda, models):
    r, img, m, om = models("llama-q8_0")
    sess = eb.Session(m, 1, 3)
    for _ in range(3):
        sess.decode_step([1])
    with pytest.raises(eb.SpmError) as e:
        sess.decode_step([1])
    assert e.value.name == "SPM_E_CONTEXT"
    sess.reset(0)
    assert sess.length(0) == 0
    sess.decode_step([1])
    sess.close()


def test_graph_and_eager_steps_agree_bit_for_bit(cuda, models):
    r, img, m, om = models("qwen3-q5_k")
    a = eb.Session(m, 2, 8, graphs=True)
    b = eb.Session(m, 2, 8, graphs=False)
    for t in range(4):
        _, la = a.decode_step([t, t + 1], want_logits=True)
        _, lb = b.decode_step([t, t + 1], want_logits=True)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    assert a.launches_per_step(2) > 0


def test_launch_profile_times_every_kernel_and_changes_no_result(cuda, models):
    # the profiled (eager, event-bracketed) step computes what the graph step does
    r, img, m, om = models("qwen3moe-q5_k")
    sh = r.shape
    a = eb.Session(m, 3, 8, graphs=True)
    b = eb.Session(m, 3, 8)
    b.set_profile(True)
    for t in range(2):
        _, la = a.decode_step([t, t + 1, t + 2], want_logits=True)
        _, lb = b.decode_step([t, t + 1, t + 2], want_logits=True)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    prof = b.profile()
    kinds = [eb.Session.KERNEL_KINDS[k] for k in prof["kind"]]
    # embed; per routed layer QKV, attention, O, router with routing (one
    # launch on one GPU), expert gate/up, expert down, combine; head, argmax, advance
    per_step = 1 + sh.layers * 7 + 1 + 2
    assert len(kinds) == 2 * per_step
    assert kinds.count("attention") == 2 * sh.layers and kinds.count("gemv_head") == 2
    assert (prof["ms"] > 0).all()
    gemv = prof["kind"] < len(eb.Session.GEMV_KINDS)
    assert (prof["bytes"][gemv] > 0).all() and (prof["bytes"][~gemv] == 0).all()
    # expert launches count the plan's active experts: gate+up stream twice the down bytes per expert
    routes = b.routes(3)
    active = [len(set(routes[l].ravel().tolist())) for l in range(sh.layers)]
    one = m.stream_info(m.stream_index("blk.0.ffn_down_exps.weight"))["bytes"] // sh.experts
    down = [int(x) for x, k in zip(prof["bytes"], kinds) if k == "gemv_expert_down"][-sh.layers:]
    assert down == [u * one for u in active]
    b.set_profile(False)
    assert b.profile()["ms"].size == 0
    a.close()
    b.close()


def test_bad_token_is_refused(cuda, models):
    r, img, m, om = models("llama-q8_0")
    sess = eb.Session(m, 1, 4)
    with pytest.raises(eb.SpmError):
        sess.decode_step([r.shape.vocab])
    sess.close()


# ---- benchmark model shapes ----
def test_smollm2_b5_full_run_matches_the_oracle(cuda):
    """Config 2 (SmolLM2 Q8_0, 5 clients, prompts 16/24/32/48/64, 128 greedy
    tokens each, lockstep): every greedy token identical over the full run."""
    w = configs.WORKLOADS["smollm2-b5"]
    r = configs.RECIPES[w["recipe"]]
    img = eb.synth_gguf(r)
    prompts = configs.workload_prompts("smollm2-b5")
    om = O.OracleModel(img, r.shape)
    want, wl = om.serve(prompts, w["steps"])
    m = eb.Model(img, r.shape)
    got, gl = eb.serve(m, prompts, w["steps"], want_logits=True)
    m.close()
    assert [len(g) for g in got] == [len(x) for x in want]
    assert got == want
    assert logits_close(gl, wl)


def test_smollm2_b1_full_run_matches_the_oracle(cuda):
    """Config 1 (SmolLM2 Q8_0, one 32-token prompt, 64 greedy tokens)."""
    w = configs.WORKLOADS["smollm2-b1"]
    r = configs.RECIPES[w["recipe"]]
    img = eb.synth_gguf(r)
    prompts = configs.workload_prompts("smollm2-b1")
    want, wl = O.OracleModel(img, r.shape).serve(prompts, w["steps"])
    m = eb.Model(img, r.shape)
    got, gl = eb.serve(m, prompts, w["steps"], want_logits=True)
    m.close()
    assert got == want
    assert logits_close(gl, wl)


def test_qwen3_8b_shape_two_layers_matches_the_oracle(cuda):
    """Qwen3-8B dimensions (hidden 4096, ffn 12288, 32/8 heads of 128, vocab
    151936, Q6_K) with 2 of its 36 layers: stepwise logits and tokens."""
    base = configs.RECIPES["qwen3-8b-q6_k"]
    import dataclasses

    r = base.replace(shape=dataclasses.replace(base.shape, layers=2))
    img = eb.synth_gguf(r)
    om = O.OracleModel(img, r.shape)
    m = eb.Model(img, r.shape)
    n = 4
    sess = eb.Session(m, n, 8)
    osess = om.session(n, 8)
    for step in range(3):
        toks = configs.prompt_tokens(3 + step, 0, n, r.shape.vocab)
        best, got = sess.decode_step(toks, want_logits=True)
        want = osess.step(toks)
        assert logits_close(got, want)
        assert best == [O.argmax_last(want[i]) for i in range(n)]
    sess.close()
    m.close()


@pytest.mark.parametrize("name,n", [("llama-q8_0", 2), ("qwen3-q6_k", 2), ("qwen3-g8-q6_k", 2), ("qwen3-g8-q6_k", 8),
                                    ("qwen3-g4-q5_k", 8)])
def test_long_context_attention_matches_the_oracle(cuda, models, name, n):
    # a client's prefix splits over several CTAs whose softmax partials are
    # combined (qwen3-g8-q6_k and qwen3-g4-q5_k with 8 clients: 16 kv head x
    # client pairs, the tensor-core kernel at head_dim 128 and 64; otherwise
    # the CUDA-core kernel)
    r, img, m, om = models(name)
    steps = 600
    sess = eb.Session(m, n, steps)
    osess = om.session(n, steps)
    for step in range(steps):
        toks = [(step * 13 + i * 7) % r.shape.vocab for i in range(n)]
        best, got = sess.decode_step(toks, want_logits=step % 50 == 49)
        want = osess.step(toks)
        if got is not None:
            assert logits_close(got, want), step
        assert best == [O.argmax_last(want[i]) for i in range(n)], step
    sess.close()


MOE = ["olmoe-q6_k", "olmoe-q2_k", "qwen3moe-q5_k"]


@pytest.mark.parametrize("name", MOE)
def test_routed_layers_match_the_oracle(cuda, models, name):
    # router softmax -> top-k -> renormalised expert mixture
    # (spm-granite-moe/src/moe.rs:17-35, layout.rs:244-333)
    r, img, m, om = models(name)
    n, steps = 4, 5
    sess = eb.Session(m, n, 16)
    osess = om.session(n, 16)
    for step in range(steps):
        toks = [(step * 29 + i * 17) % r.shape.vocab for i in range(n)]
        best, got = sess.decode_step(toks, want_logits=True)
        want, oroutes = osess.step(toks, routes=True)
        assert np.array_equal(sess.routes(n), oroutes), step
        assert logits_close(got, want), (step, float(np.abs(got - want).max()), float(np.abs(want).max()))
        assert best == [O.argmax_last(want[i]) for i in range(n)]
    sess.close()


@pytest.mark.parametrize("name", MOE)
def test_routed_greedy_serving_matches_the_oracle(cuda, models, name):
    r, img, m, om = models(name)
    prompts = [configs.prompt_tokens(21, i, ln, r.shape.vocab) for i, ln in enumerate([3, 6, 4, 5, 2, 7, 3, 4])]
    want, wl = om.serve(prompts, 8)
    got, gl = eb.serve(m, prompts, 8, want_logits=True)
    assert got == want
    assert logits_close(gl, wl)


def test_olmoe_shape_two_layers_matches_the_oracle(cuda):
    """OLMoE-1B-7B dimensions (hidden 2048, 16 heads of 128, 64 experts of
    1024, top-8, vocab 50304) with 2 of its 16 layers, Q2_K experts, 8 clients."""
    import dataclasses

    base = configs.RECIPES["olmoe-q2_k"]
    r = base.replace(shape=dataclasses.replace(base.shape, layers=2))
    img = eb.synth_gguf(r)
    om = O.OracleModel(img, r.shape)
    m = eb.Model(img, r.shape)
    n = 8
    sess = eb.Session(m, n, 8)
    osess = om.session(n, 8)
    for step in range(3):
        toks = configs.prompt_tokens(30 + step, 0, n, r.shape.vocab)
        best, got = sess.decode_step(toks, want_logits=True)
        want, oroutes = osess.step(toks, routes=True)
        assert np.array_equal(sess.routes(n), oroutes)
        assert logits_close(got, want)
        assert best == [O.argmax_last(want[i]) for i in range(n)]
    sess.close()
    m.close()


def test_qwen3_30b_shape_two_layers_matches_the_oracle(cuda):
    """Qwen3-30B-A3B dimensions (hidden 2048, 32/4 heads of 128, 128 experts
    of 768, top-8, vocab 151936, Q5_K) with 2 of its 48 layers, 8 clients."""
    import dataclasses

    base = configs.RECIPES["qwen3-30b-a3b-q5_k"]
    r = base.replace(shape=dataclasses.replace(base.shape, layers=2))
    img = eb.synth_gguf(r)
    om = O.OracleModel(img, r.shape)
    m = eb.Model(img, r.shape)
    n = 8
    sess = eb.Session(m, n, 8)
    osess = om.session(n, 8)
    for step in range(3):
        toks = configs.prompt_tokens(40 + step, 0, n, r.shape.vocab)
        best, got = sess.decode_step(toks, want_logits=True)
        want, oroutes = osess.step(toks, routes=True)
        assert np.array_equal(sess.routes(n), oroutes)
        assert logits_close(got, want)
        assert best == [O.argmax_last(want[i]) for i in range(n)]
    sess.close()
    m.close()


def test_continuous_batching_matches_the_oracle_served_alone(cuda, models):
    """Requests join free slots mid-flight and leave when done: each one's
    tokens equal the oracle's for that request served alone."""
    from emufpga_b200.scheduler import Request, serve_continuous

    r, img, m, om = models("qwen3-q6_k")
    v = r.shape.vocab
    reqs = [Request(configs.prompt_tokens(50 + i, 0, ln, v), new, arr)
            for i, (ln, new, arr) in enumerate([(3, 6, 0), (5, 4, 0), (2, 7, 1), (4, 5, 3), (6, 3, 4), (1, 8, 9)])]
    for prefill in (False, True):
        sess = eb.Session(m, 3, 24)
        got = serve_continuous(sess, reqs, prefill=prefill)
        sess.close()
        for q, g in zip(reqs, got):
            want, _ = om.serve([list(q.prompt)], q.max_new)
            assert g == want[0], (prefill, q)


@pytest.mark.parametrize("name", ["qwen3-q5_k", "olmoe-q2_k"])
def test_packed_image_file_opens_the_same_model(cuda, models, tmp_path, name):
    """A model opened from its packed image file (one upload, no re-packing)
    decodes bit-for-bit like the one packed from the GGUF."""
    r, img, m, om = models(name)
    path = tmp_path / "m.spmimg"
    eb.pack_image(img, str(path), r.shape)
    mi = eb.Model.from_image(str(path), r.shape)
    assert mi.weight_bytes == m.weight_bytes
    n = 3
    a, b = eb.Session(m, n, 8), eb.Session(mi, n, 8)
    for t in range(4):
        toks = [(t * 5 + i * 3) % r.shape.vocab for i in range(n)]
        _, la = a.decode_step(toks, want_logits=True)
        _, lb = b.decode_step(toks, want_logits=True)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    a.close()
    b.close()
    mi.close()
