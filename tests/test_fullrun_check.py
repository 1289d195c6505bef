"""The full-run parity rule (tests/fullrun_check.py) on made-up golden runs:
what it accepts, what it refuses, and the drift allowance after a routing
near tie.  CPU only; the GPU test feeds the same rule the device's run."""
import numpy as np
import pytest

from tests.fullrun_check import DRIFT_SHARE, LOGIT_TOL, ROUTE_SLACK, ROUTE_TIE, TIE, RunCheck

TICKS, N, VOCAB = 40, 4, 64


def _golden(route=True, seed=0):
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((TICKS, N, VOCAB)).astype(np.float32) * 4
    ids = np.argsort(-logits, axis=2, kind="stable")[:, :, :8].astype(np.int32)
    vals = np.take_along_axis(logits, ids, axis=2)
    s = np.sort(logits, axis=2)
    g = {
        "argmax": ids[:, :, 0].copy(),
        "top_ids": ids,
        "top_vals": vals,
        "margin": s[:, :, -1] - s[:, :, -2],
        "maxabs": np.abs(logits).max(axis=2),
    }
    if route:
        g["route_margin"] = np.full((TICKS, N), 0.3, np.float32)
    return g, logits


def _run(check, g, logits, gaps=None, upto=TICKS):
    for t in range(upto):
        check.tick(t, g["argmax"][t], logits[t], None if gaps is None else gaps[t])


def test_the_oracles_own_run_passes_with_nothing_exempted():
    g, logits = _golden()
    c = RunCheck(g, N)
    _run(c, g, logits, gaps=np.full((TICKS, N), 0.5))
    c.finish()
    assert (c.ties, c.exempt_now, c.exempt_drift) == (0, 0, 0)
    assert c.drift_since == [None] * N


def test_logits_within_the_tolerance_pass_and_beyond_it_fail():
    g, logits = _golden(route=False)
    scale = g["maxabs"][7, 2]
    ok = logits.copy()
    ok[7, 2, g["top_ids"][7, 2, 3]] += 0.9 * LOGIT_TOL * scale
    _run(RunCheck(g, N), g, ok)
    bad = logits.copy()
    bad[7, 2, g["top_ids"][7, 2, 3]] += 1.5 * LOGIT_TOL * scale
    with pytest.raises(AssertionError, match="tick 7 client 2"):
        _run(RunCheck(g, N), g, bad)


def test_a_different_pick_passes_only_at_a_near_tie():
    g, logits = _golden(route=False)
    t, i = 5, 1
    second = int(g["top_ids"][t, i, 1])
    best = g["argmax"][t].copy()
    best[i] = second
    # far apart in the oracle's logits: refused
    g["top_vals"][t, i, 1] = g["top_vals"][t, i, 0] - 10 * TIE * g["maxabs"][t, i]
    with pytest.raises(AssertionError, match="not a near tie"):
        RunCheck(g, N).tick(t, best, logits[t])
    # within TIE * max|logit|: accepted and counted against the oracle's near margins
    g["top_vals"][t, i, 1] = g["top_vals"][t, i, 0] - 0.5 * TIE * g["maxabs"][t, i]
    g["margin"][t, i] = g["top_vals"][t, i, 0] - g["top_vals"][t, i, 1]
    logits[t, i, second] = g["top_vals"][t, i, 1]
    c = RunCheck(g, N)
    c.tick(t, best, logits[t])
    assert c.ties == 1
    c.finish()


def test_a_device_routing_near_tie_allows_the_slack_at_that_tick():
    g, logits = _golden()
    t, i = 9, 3
    off = logits.copy()
    off[t, i, g["top_ids"][t, i, 0]] += 5 * LOGIT_TOL * g["maxabs"][t, i]
    gaps = np.full((TICKS, N), 0.2)
    with pytest.raises(AssertionError):
        _run(RunCheck(g, N), g, off, gaps)
    gaps[t, i] = 0.5 * ROUTE_TIE
    c = RunCheck(g, N)
    _run(c, g, off, gaps)
    assert (c.exempt_now, c.exempt_drift, c.drift_since[i]) == (1, 0, t)


def test_drift_after_an_oracle_routing_near_tie_is_allowed_from_that_tick_on():
    """The case that an order-of-sums change met: the near tie at an earlier
    tick (in the oracle's routing), the logits off at a later one."""
    g, logits = _golden()
    tie_at, off_at, i = 12, 16, 1
    off = logits.copy()
    for t in range(off_at, off_at + 3):
        off[t, i, g["top_ids"][t, i, 2]] += 4 * LOGIT_TOL * g["maxabs"][t, i]
    # no near tie anywhere: refused at the first off tick
    with pytest.raises(AssertionError, match=f"tick {off_at} client {i}"):
        _run(RunCheck(g, N), g, off)
    # a near tie after the off ticks does not excuse them
    late = {k: v.copy() for k, v in g.items()}
    late["route_margin"][off_at + 5, i] = 0.1 * ROUTE_TIE
    with pytest.raises(AssertionError, match=f"tick {off_at} client {i}"):
        _run(RunCheck(late, N), late, off)
    # a near tie of another client does not either
    other = {k: v.copy() for k, v in g.items()}
    other["route_margin"][tie_at, i + 1] = 0.1 * ROUTE_TIE
    with pytest.raises(AssertionError, match=f"tick {off_at} client {i}"):
        _run(RunCheck(other, N), other, off)
    # the client's own near tie before them: allowed, counted as drift
    g["route_margin"][tie_at, i] = 0.1 * ROUTE_TIE
    c = RunCheck(g, N)
    _run(c, g, off)
    assert (c.exempt_now, c.exempt_drift, c.drift_since[i]) == (0, 3, tie_at)
    c.finish()


def test_the_allowance_has_a_ceiling():
    g, logits = _golden()
    g["route_margin"][0, 0] = 0.0
    t, i = 20, 0
    off = logits.copy()
    off[t, i, g["top_ids"][t, i, 0]] += 1.5 * ROUTE_SLACK * g["maxabs"][t, i]
    with pytest.raises(AssertionError, match=f"tick {t} client {i}"):
        _run(RunCheck(g, N), g, off)


def test_near_ties_in_unchecked_prompt_ticks_count():
    """Prompts run by spm_prefill are not checked tick by tick, but the
    oracle's routing near ties inside them still start the allowance."""
    g, logits = _golden()
    g["route_margin"][3, 2] = 0.5 * ROUTE_TIE
    c = RunCheck(g, N)
    for t in range(10):
        c.note_prompt(t)
    assert c.drift_since == [None, None, 3, None]
    off = logits.copy()
    off[10, 2, g["top_ids"][10, 2, 0]] += 3 * LOGIT_TOL * g["maxabs"][10, 2]
    for t in range(10, TICKS):
        c.tick(t, g["argmax"][t], off[t])
    assert c.exempt_drift == 1


def test_the_counts_are_bounded_over_the_run():
    g, logits = _golden()
    g["route_margin"][0, :] = 0.0
    off = logits + (3 * LOGIT_TOL * g["maxabs"])[:, :, None]
    off[0] = logits[0]
    c = RunCheck(g, N)
    _run(c, g, off)
    # every cell after the near ties of tick 0 drifted: far above the share allowed
    assert c.exempt_now == 0
    assert c.exempt_drift == (TICKS - 1) * N > DRIFT_SHARE * TICKS * N
    with pytest.raises(AssertionError, match=str(c.exempt_drift)):
        c.finish()


def test_dense_golden_runs_have_no_routing_margins_and_need_none():
    g, logits = _golden(route=False)
    c = RunCheck(g, N)
    assert c.route_margin is None
    _run(c, g, logits)
    c.finish()


def test_committed_routed_golden_runs_carry_routing_margins():
    from pathlib import Path

    runs = Path(__file__).resolve().parent / "golden" / "runs"
    for name in ("olmoe-q6_k-b8", "olmoe-q2_k-b8"):
        g = np.load(runs / f"{name}.npz")
        assert "route_margin" in g.files, name
        rm = g["route_margin"]
        assert rm.shape == g["argmax"].shape and np.all((rm >= 0) & (rm <= 1)), name
