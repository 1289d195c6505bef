"""The default consumption order never makes a decode step seek backward
(spm-order/tests/no_seek.rs:50-100 for the reference's order files): the
streams a step demands, in the engine's launch order, walk the rotating
region in increasing index order once per step, with one rewind between
steps; the resident region holds what is read once (the untied LM head)."""
import os

import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from emufpga_b200._lib import LLAMA


def parse(text):
    rot, res, sec = [], [], None
    for line in text.splitlines():
        line = line.strip()
        if not line or line.startswith("#"):
            continue
        if line == "[rotating]":
            sec = rot
        elif line == "[resident]":
            sec = res
        else:
            sec.append(line)
    return rot, res


def demands(shape):
    """Matrices one decode step streams, in launch order (engine.cu enqueue_step)."""
    out = []
    for l in range(shape.layers):
        p = f"blk.{l}."
        out += [p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight", p + "attn_output.weight"]
        if shape.experts:
            out += [p + "ffn_gate_inp.weight", p + "ffn_gate_exps.weight", p + "ffn_up_exps.weight",
                    p + "ffn_down_exps.weight"]
        else:
            out += [p + "ffn_gate.weight", p + "ffn_up.weight", p + "ffn_down.weight"]
    if not shape.tied:
        out.append("output.weight")
    return out


@pytest.mark.parametrize("name", sorted(configs.TINY))
def test_a_decode_step_never_moves_backward(name):
    r = configs.TINY[name]
    rot, res = parse(eb.default_order(r.shape, eb.synth_gguf(r)))
    index = {n: i for i, n in enumerate(rot)}
    steps, prev, rewinds = 3, None, 0
    for _ in range(steps):
        for n in demands(r.shape):
            at = index[n]
            if prev is not None and at <= prev:
                assert at == 0 and prev == len(index) - 1, (n, at, prev)
                rewinds += 1
            prev = at
    assert rewinds == steps - 1
    # every rotating matrix is demanded once per step
    assert sorted(demands(r.shape)) == sorted(rot)
    assert "token_embd.weight" in res
    if r.shape.tied:
        assert "output.weight" not in res + rot


@pytest.mark.parametrize("name", sorted(configs.TINY))
def test_packed_streams_are_the_rotating_region_and_the_embedding(name, tmp_path):
    """The host-packed device image holds one stream per rotating matrix plus
    the token embedding (the gather table, and the LM head when tied)."""
    r = configs.TINY[name]
    image = eb.synth_gguf(r)
    rot, _ = parse(eb.default_order(r.shape, image))
    path = os.fspath(tmp_path / "model.spmimg")
    eb.pack_image(image, path, r.shape)
    _, streams = eb.image_probe(path)
    assert streams == len(rot) + 1


def test_alphabetical_order_would_have_seeked_backward():
    r = configs.TINY["qwen3-q6_k"]
    rot, _ = parse(eb.default_order(r.shape, eb.synth_gguf(r)))
    alphabetical = sorted(rot)
    assert alphabetical != rot
    # the first thing a layer wants (attn_q) comes after attn_output alphabetically
    assert alphabetical.index("blk.0.attn_output.weight") < alphabetical.index("blk.0.attn_q.weight")
