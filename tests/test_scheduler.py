"""Continuous batching host logic on CPU with a toy session whose greedy
pick depends only on the client's own history since its last reset (as in
the real engine, where clients share weights but nothing else)."""
import hashlib

import pytest

from emufpga_b200.scheduler import Request, serve_continuous


class ToySession:
    def __init__(self, max_clients, context, vocab=50):
        self.max_clients, self.context, self.vocab = max_clients, context, vocab
        self.hist = [[] for _ in range(max_clients)]
        self.steps = []
        self.prefills = []

    def reset(self, client):
        self.hist[client] = []

    def length(self, client):
        return len(self.hist[client])

    def prefill(self, client, tokens):
        # the prompt path: the same history as feeding the tokens one per step
        self.prefills.append((client, len(tokens)))
        self.hist[client].extend(tokens)

    def decode_step(self, tokens, want_logits=False):
        self.steps.append(len(tokens))
        best = []
        for i, t in enumerate(tokens):
            if len(self.hist[i]) >= self.context:
                raise RuntimeError("context exhausted")
            self.hist[i].append(t)
            h = hashlib.sha256(repr(self.hist[i]).encode()).digest()
            best.append(h[0] % self.vocab)
        return best, None


def alone(req, context=64):
    return serve_continuous(ToySession(1, context), [Request(req.prompt, req.max_new)])[0]


def test_each_request_gets_what_it_gets_alone():
    reqs = [Request([1, 2, 3], 5), Request([7], 9, arrival=2), Request([4, 4, 4, 4], 3, arrival=2),
            Request([9, 8], 6, arrival=5), Request([3, 1, 4, 1, 5], 4, arrival=6), Request([2], 2, arrival=30)]
    sess = ToySession(3, 64)
    got = serve_continuous(sess, reqs)
    for r, g in zip(reqs, got):
        assert g == alone(r)
        assert len(g) == r.max_new
    # never more clients in a step than slots, and slots were reused
    assert max(sess.steps) <= 3
    assert len(sess.steps) < sum(len(r.prompt) + r.max_new - 1 for r in reqs)


def test_single_request_matches_the_lockstep_rule():
    # serve-demo: prompt of L tokens, S generated tokens -> L + S - 1 steps
    sess = ToySession(1, 64)
    out = serve_continuous(sess, [Request([5, 6, 7, 8], 6)])
    assert len(out[0]) == 6
    assert len(sess.steps) == 4 + 6 - 1


def test_idle_slots_below_busy_ones_never_exhaust_the_context():
    # slot 0 finishes quickly; slot 1 runs long; slot 0 idles under it
    reqs = [Request([1], 1), Request([2, 3], 14)]
    got = serve_continuous(ToySession(2, 16), reqs)
    assert got[1] == alone(reqs[1], 16)


def test_requests_that_cannot_fit_are_refused():
    with pytest.raises(ValueError):
        serve_continuous(ToySession(2, 8), [Request([1] * 5, 4)])
    with pytest.raises(ValueError):
        serve_continuous(ToySession(2, 8), [Request([], 2)])


def test_prefill_of_joining_requests_changes_no_token():
    reqs = [Request([1, 2, 3, 9, 9], 5), Request([7], 9, arrival=2), Request([4, 4, 4, 4], 3, arrival=2),
            Request([5, 6, 7, 8, 1, 2], 4, arrival=6)]
    plain = ToySession(2, 32)
    fast = ToySession(2, 32)
    assert serve_continuous(fast, reqs, prefill=True) == serve_continuous(plain, reqs)
    # every prompt longer than one token went through prefill, all but its last token
    assert sorted(n for _, n in fast.prefills) == sorted(len(r.prompt) - 1 for r in reqs if len(r.prompt) > 1)
    assert len(fast.steps) < len(plain.steps)
