"""The full-run parity rule: a device run checked tick by tick against the
oracle's golden full run (tests/golden/runs/*.npz).  Pure numpy, so the rule
itself is tested on the CPU (tests/test_fullrun_check.py) and the GPU test
(tests/test_gpu_fullrun.py) only feeds it the device's picks and logits.

The schedule is serve-demo's lockstep (spm-batch/examples/serve-demo.rs:
59-91).  The device follows the oracle's run (its next token is the oracle's
pick), so at every tick:

- its greedy pick equals the oracle's, unless the two lie within
  TIE * max|logit| in the oracle's own logits (a near tie: the order of the
  fp32 sums decides between them); the number of picks decided the other way
  may not exceed the number of such oracle margins;
- its logits at the oracle's eight largest lie within LOGIT_TOL * max|logit|
  of the oracle's values.

Routed models add the router's top-K selection.  Where a client's K-th and
(K+1)-th routing probabilities lie within ROUTE_TIE of each other
(relatively), on the device (spm_session_route_gaps) or in the oracle (the
golden file's route_margin), the two sides may send that client through
different experts in that layer.  That decision is written into the KV
cache at that position, so the client can stay off the oracle's values at
later ticks too (moe.rs:17-35 selects by those probabilities; a changed
expert set at one position moves every later attention over it).  So from
the first tick with such a near tie on, the client is held to the routing
allowance: logits within ROUTE_SLACK * max|logit| and picks within the same
near-tie bound.  Checks that needed the allowance are counted two ways:

- at the tick of the near tie itself: fewer than ROUTE_SHARE of the
  client-ticks;
- at later ticks (drift from an earlier near tie): fewer than DRIFT_SHARE.

A run whose logits never leave LOGIT_TOL uses neither count; the rule is the
earlier per-tick rule widened only where that one would have failed.
"""
from __future__ import annotations

import numpy as np

LOGIT_TOL = 1e-3
TIE = 1e-4
ROUTE_TIE = 1e-4
ROUTE_SLACK = 1e-2
ROUTE_SHARE = 1e-3
DRIFT_SHARE = 5e-2


class RunCheck:
    """Checks one device run against golden run `g` (an npz mapping) for
    `n` clients.  Call note_prompt() for ticks the device ran without
    checking (prompts run by spm_prefill), tick() for checked ticks, then
    finish()."""

    def __init__(self, g, n: int):
        self.g = g
        self.n = n
        files = getattr(g, "files", g.keys())
        self.route_margin = g["route_margin"] if "route_margin" in files else None
        self.drift_since: list[int | None] = [None] * n
        self.ticks = 0
        self.ties = 0
        self.exempt_now = 0
        self.exempt_drift = 0

    def _near_tie(self, t: int, i: int, device_gaps) -> bool:
        if device_gaps is not None and float(device_gaps[i]) < ROUTE_TIE:
            return True
        return self.route_margin is not None and float(self.route_margin[t][i]) < ROUTE_TIE

    def note_prompt(self, t: int) -> None:
        """Tick t ran on the device unchecked: only the oracle's routing
        margins are known for it."""
        for i in range(self.n):
            if self.drift_since[i] is None and self._near_tie(t, i, None):
                self.drift_since[i] = t

    def tick(self, t: int, best, logits: np.ndarray, device_gaps=None) -> None:
        """Checks tick t: `best` the device's picks, `logits` [n, vocab],
        `device_gaps` each client's smallest routing margin over the layers
        at this tick on the device (routed models) or None."""
        g = self.g
        ids, vals, scale = g["top_ids"][t], g["top_vals"][t], g["maxabs"][t]
        self.ticks += 1
        for i in range(self.n):
            now = self._near_tie(t, i, device_gaps)
            if now and self.drift_since[i] is None:
                self.drift_since[i] = t
            allowed = self.drift_since[i] is not None
            bound = ROUTE_SLACK if allowed else TIE
            want = int(g["argmax"][t][i])
            if int(best[i]) != want:
                where = np.nonzero(ids[i] == int(best[i]))[0]
                assert where.size and vals[i][0] - vals[i][where[0]] <= bound * scale[i], \
                    f"tick {t} client {i}: greedy pick {int(best[i])} != {want} (not a near tie)"
                self.ties += 1
            err = float(np.abs(logits[i, ids[i]] - vals[i]).max())
            if err > LOGIT_TOL * scale[i]:
                gap = None if device_gaps is None else float(device_gaps[i])
                assert allowed and err <= ROUTE_SLACK * scale[i], \
                    (f"tick {t} client {i}: logits {err / scale[i]:.2e}*max|logit| off", gap,
                     "routing near tie since tick", self.drift_since[i])
                if now:
                    self.exempt_now += 1
                else:
                    self.exempt_drift += 1

    def finish(self) -> str:
        """The run's counts against their limits (a whole run's ticks)."""
        g, cells = self.g, self.ticks * self.n
        near = int((g["margin"] <= TIE * g["maxabs"]).sum())
        assert self.ties <= near + self.exempt_now + self.exempt_drift, (self.ties, near)
        assert self.exempt_now <= ROUTE_SHARE * cells, self.exempt_now
        assert self.exempt_drift <= DRIFT_SHARE * cells, self.exempt_drift
        return self.summary()

    def summary(self) -> str:
        cells = self.ticks * self.n
        drifted = sum(d is not None for d in self.drift_since)
        return (f"{cells} client-ticks, {self.ties} greedy near ties decided the other way, "
                f"{self.exempt_now} logit checks at routing near ties, {self.exempt_drift} after one "
                f"({drifted} clients met a routing near tie)")
