"""Host-side logic without a GPU: GGUF bounds (spm-gguf/tests/safety.rs),
.order rules (spm-order), the synthetic-model writer and encoders."""
import struct

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from oracle import oracle as O


def header(tensors, metadata):
    return b"GGUF" + struct.pack("<IQQ", 3, tensors, metadata)


def product_error(img: bytes) -> str:
    with pytest.raises(eb.SpmError) as e:
        eb.gguf_probe(np.frombuffer(img, dtype=np.uint8).copy())
    return str(e.value)


# ---- spm-gguf/tests/safety.rs:16-73 ----
def test_rejects_bad_magic():
    assert "magic" in product_error(b"NOPE")
    assert "magic" in O.gguf_parse_error(np.frombuffer(b"NOPE", dtype=np.uint8))


def test_rejects_unbounded_counts():
    img = header(0, 1_000_001)
    assert "metadata count" in product_error(img)
    assert "metadata count" in O.gguf_parse_error(np.frombuffer(img, dtype=np.uint8))


def test_rejects_unbounded_strings_before_allocation():
    img = header(0, 1) + struct.pack("<Q", 16 * 1024 * 1024 + 1)
    assert "string length" in product_error(img)
    assert "string length" in O.gguf_parse_error(np.frombuffer(img, dtype=np.uint8))


def tiny_tensor(offset):
    v = header(1, 0) + struct.pack("<Q", 1) + b"x" + struct.pack("<I", 1) + struct.pack("<Q", 32)
    v += struct.pack("<I", 0) + struct.pack("<Q", offset)
    return v.ljust(64, b"\0")


def test_rejects_tensor_ranges_beyond_the_file():
    img = tiny_tensor(4096)
    assert "beyond file" in product_error(img)
    assert "beyond file" in O.gguf_parse_error(np.frombuffer(img, dtype=np.uint8))


def test_reads_a_tiny_aligned_fixture():
    img = tiny_tensor(0).ljust(64 + 32 * 4, b"\x01")
    arr = np.frombuffer(img, dtype=np.uint8).copy()
    assert eb.gguf_probe(arr) == (1, 64)
    t = eb.gguf_find(arr, "x")
    assert t["nbytes"] == 128 and t["offset"] == 64 and t["dtype"] == 0
    assert O.gguf_parse_error(arr) is None


def test_rejects_unknown_dtype_and_overlap():
    v = header(2, 0)
    for name, off in ((b"a", 0), (b"b", 0)):
        v += struct.pack("<Q", 1) + name + struct.pack("<I", 1) + struct.pack("<Q", 32) + struct.pack("<IQ", 0, off)
    img = v.ljust(96, b"\0").ljust(96 + 256, b"\0")
    assert "overlapping" in product_error(img)
    v = header(1, 0) + struct.pack("<Q", 1) + b"x" + struct.pack("<I", 1) + struct.pack("<Q", 32) + struct.pack("<IQ", 99, 0)
    assert "dtype" in product_error(v.ljust(256, b"\0"))


# ---- synthetic models ----
TINY = configs.TINY["llama-q8_0"]


def test_synth_is_deterministic_and_thread_independent():
    a = eb.synth_gguf(TINY, threads=1)
    b = eb.synth_gguf(TINY, threads=4)
    assert np.array_equal(a, b)
    c = eb.synth_gguf(TINY.replace(seed=TINY.seed + 1))
    assert not np.array_equal(a, c)


@pytest.mark.parametrize("name", sorted(configs.TINY))
def test_synth_images_parse_in_both_parsers(name):
    r = configs.TINY[name]
    img = eb.synth_gguf(r)
    count, _ = eb.gguf_probe(img)
    assert O.gguf_parse_error(img) is None
    order = eb.default_order(r.shape, img)
    eb.order_check(order, img)
    names = [ln for ln in order.splitlines() if ln and not ln.startswith("#") and not ln.startswith("[")]
    assert len(names) == count


def test_synth_weights_have_the_requested_spread():
    r = configs.TINY["qwen3-q6_k"]
    img = eb.synth_gguf(r)
    t = eb.gguf_find(img, "blk.0.ffn_up.weight")
    w = eb.decode_q6_k(img[t["offset"]: t["offset"] + t["nbytes"]])
    assert abs(float(w.std()) - 0.02) < 0.002 and abs(float(w.mean())) < 0.002
    g = eb.gguf_find(img, "blk.0.attn_norm.weight")
    gains = eb.decode_f32(img[g["offset"]: g["offset"] + g["nbytes"]])
    assert abs(float(gains.mean()) - 1.0) < 0.05  # gain_sigma 0.1 in the tiny recipes


@pytest.mark.parametrize("dtype", [O.Q8_0, O.Q6_K, O.Q5_K, O.Q2_K])
def test_encoders_write_valid_blocks(dtype):
    # N(0, 0.02) values quantized by this library's encoders decode to finite
    # weights with about the requested spread.
    r = configs.TINY["qwen3-q6_k"].replace(layer_type=dtype, embed_type=dtype, head_type=dtype)
    img = eb.synth_gguf(r)
    t = eb.gguf_find(img, "blk.0.attn_q.weight")
    w = eb.decode_blocks(dtype, img[t["offset"]: t["offset"] + t["nbytes"]])
    assert np.isfinite(w).all()
    assert 0.5 * 0.02 < float(w.std()) < 1.6 * 0.02


def test_zipf_router_bias_is_a_log_probability_per_layer():
    r = configs.TINY["olmoe-q6_k"]
    img = eb.synth_gguf(r)
    for layer in range(r.shape.layers):
        t = eb.gguf_find(img, f"blk.{layer}.exp_probs_b.bias")
        b = eb.decode_f32(img[t["offset"]: t["offset"] + t["nbytes"]]).astype(np.float64)
        assert abs(np.exp(b).sum() - 1.0) < 1e-5
        ranks = np.argsort(-b)
        p = np.exp(b[ranks])
        expect = np.arange(1, len(b) + 1, dtype=np.float64) ** -1.1
        assert np.allclose(p, expect / expect.sum(), rtol=1e-5)


# ---- spm-order (no_seek.rs rules) ----
def test_order_refuses_missing_and_unlisted_names():
    img = eb.synth_gguf(TINY)
    order = eb.default_order(TINY.shape)
    with pytest.raises(eb.SpmError) as e:
        eb.order_check(order.replace("blk.0.attn_q.weight\n", ""), img)
    assert "not named in the order file" in str(e.value)
    with pytest.raises(eb.SpmError) as e:
        eb.order_check(order + "blk.99.attn_q.weight\n", img)
    assert "not in the checkpoint" in str(e.value)
    with pytest.raises(eb.SpmError) as e:
        eb.order_check("blk.0.attn_q.weight\n" + order, img)
    assert "before any" in str(e.value)


def test_oracle_serves_a_tiny_model_deterministically():
    r = configs.TINY["llama-q8_0"]
    img = eb.synth_gguf(r)
    m = O.OracleModel(img, r.shape)
    prompts = [configs.prompt_tokens(1, i, 3 + i, r.shape.vocab) for i in range(3)]
    a, la = m.serve(prompts, 4, threads=1)
    b, lb = m.serve(prompts, 4, threads=4)
    assert a == b and np.array_equal(la, lb)
    # THE CLAIM (spm-batch/tests/batching.rs:128-145): batched == alone.
    for i, p in enumerate(prompts):
        alone, _ = m.serve([p], 4 + len(prompts[-1]) - len(p), threads=2)
        assert alone[0][: len(a[i])] == a[i][: len(alone[0])]


def test_oracle_records_routing_margins():
    """The oracle's per-layer routing margin (p_K - p_K+1) / p_K of each
    client: in [0, 1], the same on any thread count, 1 for a dense model."""
    r = configs.TINY["olmoe-q6_k"]
    img = eb.synth_gguf(r)
    m = O.OracleModel(img, r.shape)
    a, b = m.session(3, 8), m.session(3, 8)
    for t in range(3):
        toks = [(t * 7 + i * 5) % r.shape.vocab for i in range(3)]
        _, ra = a.step(toks, threads=1, routes=True)
        b.step(toks, threads=4)
        ma, mb = a.route_margins(), b.route_margins()
        assert ma.shape == (r.shape.layers, 3)
        assert np.array_equal(ma, mb)
        assert ((ma >= 0) & (ma <= 1)).all() and (ma < 1).any()
        assert ra.shape[0] == r.shape.layers
    d = configs.TINY["llama-q8_0"]
    dm = O.OracleModel(eb.synth_gguf(d), d.shape).session(2, 4)
    dm.step([1, 2])
    assert (dm.route_margins() == 1).all()
