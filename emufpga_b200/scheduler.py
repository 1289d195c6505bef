"""Continuous batching over one decode session.

The reference serves a fixed batch in lockstep (spm-batch/examples/
serve-demo.rs:45-91): every client starts at tick 0 and the batch ends with
its longest client.  Here requests join free client slots while other
clients are decoding and leave as soon as they are done, so the weight sweep
of every step is shared by whichever requests are in flight.  Each request
follows serve-demo's per-client rule on its own clock: it feeds its prompt
one token per step, then feeds back its greedy pick, and produces `max_new`
tokens -- the same tokens it would produce served alone.

A step runs clients 0..n-1 where n-1 is the highest busy slot; a free slot
below that decodes a filler token and is reset before a request takes it
(or when its cache would otherwise fill).

With `prefill=True` a joining request's prompt, all but its last token, runs
at once through the session's `prefill` (the tensor-core prompt path) when
it takes its slot; it then feeds its last prompt token in the next step and
decodes from there -- the batched prefill for late joiners that the
reference's lockstep server lacks (docs/results.md:1189-1191).
"""
from __future__ import annotations

import dataclasses
from typing import Protocol, Sequence


@dataclasses.dataclass(frozen=True)
class Request:
    prompt: Sequence[int]
    max_new: int
    arrival: int = 0  # first step at which the request may start


class DecodeSession(Protocol):
    """What the scheduler needs from a session (engine.Session has it)."""

    max_clients: int
    context: int

    def reset(self, client: int) -> None: ...

    def length(self, client: int) -> int: ...

    def decode_step(self, tokens: Sequence[int], want_logits: bool = False): ...

    # only with prefill=True: run tokens for `client` at its next positions
    def prefill(self, client: int, tokens: Sequence[int]) -> None: ...


def serve_continuous(session: DecodeSession, requests: Sequence[Request], filler: int = 0,
                     prefill: bool = False) -> list[list[int]]:
    """Serve `requests` on `session`; returns each request's produced tokens.

    Requests start in arrival order (ties in list order) as slots free up.
    With prefill, a starting request's prompt but its last token is run at
    once by session.prefill.  Raises ValueError when a request cannot fit the
    session's context."""
    for r in requests:
        if not r.prompt or r.max_new < 1:
            raise ValueError("a request needs a prompt and at least one new token")
        if len(r.prompt) + r.max_new > session.context:
            raise ValueError("a request does not fit the session's context")
    waiting = sorted(range(len(requests)), key=lambda i: (requests[i].arrival, i))
    out: list[list[int]] = [[] for _ in requests]
    active: dict[int, list[int]] = {}  # slot -> [request, local step, next token]
    step = 0
    while waiting or active:
        for s in range(session.max_clients):
            if not waiting or requests[waiting[0]].arrival > step:
                break
            if s in active:
                continue
            r = waiting.pop(0)
            session.reset(s)
            prompt = requests[r].prompt
            if prefill and len(prompt) > 1:
                session.prefill(s, list(prompt[:-1]))
                active[s] = [r, len(prompt) - 1, prompt[-1]]
            else:
                active[s] = [r, 0, prompt[0]]
        if not active:
            step = requests[waiting[0]].arrival
            continue
        n = max(active) + 1
        for s in range(n):
            if s not in active and session.length(s) + 1 >= session.context:
                session.reset(s)
        best, _ = session.decode_step([active[s][2] if s in active else filler for s in range(n)])
        for s in list(active):
            st = active[s]
            r, k = st[0], st[1]
            prompt = requests[r].prompt
            if k + 1 < len(prompt):
                st[2] = prompt[k + 1]
            else:
                out[r].append(best[s])
                st[2] = best[s]
            st[1] = k + 1
            if len(out[r]) >= requests[r].max_new:
                del active[s]
        step += 1
    return out
