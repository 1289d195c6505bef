"""The reference's own known-answer tests, run against the C oracle.

Each test names the reference test it restates (paths inside the emufpga tree).
"""
import struct

import numpy as np
import pytest

from oracle import oracle as O


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


# ---- spm-gguf/tests/decode.rs ----
def test_f32_known_values_and_rejects_partial_value():
    data = bytes([0, 0, 128, 63, 0, 0, 32, 192])
    assert list(O.decode(O.F32, data)) == [1.0, -2.5]
    with pytest.raises(ValueError):
        O.decode(O.F32, data[:7])


def test_q6_k_zero_code_with_unit_scale_is_minus_32():
    block = bytearray(210)
    block[192:208] = b"\x01" * 16
    block[208:210] = (0x3C00).to_bytes(2, "little")
    assert list(O.decode(O.Q6_K, bytes(block))) == [-32.0] * 256


def test_q6_k_lane_bit_packing_matches_reference_layout():
    block = bytearray(210)
    block[192:208] = b"\x01" * 16
    block[208:210] = (0x4000).to_bytes(2, "little")
    block[0] = 0xA5
    block[32] = 0xC7
    block[128] = 0b11_10_01_00
    d = O.decode(O.Q6_K, bytes(block))
    got = [f32_bits(d[i]) for i in (0, 32, 64, 96)]
    assert got == [f32_bits(v) for v in (-54.0, -18.0, 20.0, 56.0)]


def test_q6_k_rejects_partial_block():
    with pytest.raises(ValueError):
        O.decode(O.Q6_K, bytes(209))


def test_q5_k_known_low_nibbles_and_rejects_partial_block():
    block = bytearray(176)
    block[0:2] = (0x3C00).to_bytes(2, "little")
    block[4] = 1
    block[5] = 1
    block[48:80] = b"\x32" * 32
    d = O.decode(O.Q5_K, bytes(block))
    assert list(d[:32]) == [2.0] * 32
    assert list(d[32:64]) == [3.0] * 32
    with pytest.raises(ValueError):
        O.decode(O.Q5_K, bytes(block[:175]))


def test_q8_0_signed_values_and_rejects_partial_block():
    block = bytearray(34)
    block[0:2] = (0x3800).to_bytes(2, "little")
    block[2] = 4
    block[3] = (-6) & 0xFF
    d = O.decode(O.Q8_0, bytes(block))
    assert abs(d[0] - 2.0) < np.finfo(np.float32).eps
    assert abs(d[1] + 3.0) < np.finfo(np.float32).eps
    with pytest.raises(ValueError):
        O.decode(O.Q8_0, bytes(block[:33]))


def test_f16_conversion_is_exact_for_every_bit_pattern():
    # spm-gguf/src/tensor.rs:82-98 handles subnormals exactly; numpy's half
    # conversion is exact, so every one of the 65536 patterns must agree.
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.f16_to_f32(int(b)) for b in bits[::1]], dtype=np.float32)
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all()


# ---- spm-qwen3-slice/src/attention.rs:85-131 ----
def test_rope_identity_and_known_pair():
    head = np.arange(128, dtype=np.float32)
    assert np.array_equal(O.rope_slice(head, 0, 1e6), head)
    head = np.zeros(128, dtype=np.float32)
    head[0] = 1.0
    r = O.rope_slice(head, 1, 1e6)
    assert abs(r[0] - np.cos(np.float32(1.0))) < 1e-6
    assert abs(r[64] - np.sin(np.float32(1.0))) < 1e-6


def test_softmax_of_equal_scores_is_exact_half():
    # spm-qwen3-slice/src/attention.rs:96-98 and spm-granite-moe/src/math.rs:44-45
    p = O.softmax_route(np.array([1000.0, 1000.0], dtype=np.float32))
    assert [f32_bits(v) for v in p] == [f32_bits(0.5)] * 2


def test_causal_gqa_maps_four_query_heads_to_each_kv_head():
    q = np.zeros(32 * 128, dtype=np.float32)
    k = np.zeros(8 * 128, dtype=np.float32)
    v = np.concatenate([np.full(128, h, dtype=np.float32) for h in range(8)])
    out = O.attend("slice", q, k, v, 1, 32, 8, 128)
    for h in range(32):
        assert abs(out[h * 128] - h // 4) < np.finfo(np.float32).eps


def test_later_key_cannot_affect_earlier_output():
    # one query at position 0 sees only position 0's value
    q = np.zeros(32 * 128, dtype=np.float32)
    keys = np.zeros((2, 8 * 128), dtype=np.float32)
    values = np.ones((2, 8 * 128), dtype=np.float32)
    values[1] = 99.0
    out = O.attend("slice", q, keys, values, 1, 32, 8, 128)
    assert np.array_equal(out, np.ones(32 * 128, dtype=np.float32))


# ---- spm-smol-ops/tests/attention.rs:5-60 (the cached form in spm-kv) ----
def test_the_causal_mask_includes_the_diagonal():
    out = O.attend("smol", [1.0, 0.0], [1.0, 0.0], [7.0, -3.0], 1, 1, 1, 2)
    assert list(out) == [7.0, -3.0]


def test_query_heads_share_their_key_value_head():
    q = [1.0, 0.0] * 4
    out = O.attend("smol", q, [1.0, 0.0, 1.0, 0.0], [5.0, 5.0, 9.0, 9.0], 1, 4, 2, 2)
    assert list(out) == [5.0, 5.0, 5.0, 5.0, 9.0, 9.0, 9.0, 9.0]


def test_a_later_position_cannot_see_an_earlier_one_only_the_reverse():
    q = [1.0, 0.0]
    k = [1.0, 0.0, 1.0, 0.0]
    first0 = O.attend("smol", q, k[:2], [1.0, 1.0], 1, 1, 1, 2)
    second0 = O.attend("smol", q, k[:2], [1.0, 1.0], 1, 1, 1, 2)
    assert np.array_equal(first0, second0)
    first1 = O.attend("smol", q, k, [1.0, 1.0, 2.0, 2.0], 2, 1, 1, 2)
    second1 = O.attend("smol", q, k, [1.0, 1.0, 99.0, 99.0], 2, 1, 1, 2)
    assert not np.array_equal(first1, second1)


# ---- spm-qwen3-slice/src/math.rs:54-60, spm-granite-moe/src/math.rs:38-47 ----
def test_rms_norm_known_vector():
    r = O.rms_norm_slice(np.array([3.0, 4.0]), np.array([1.0, 2.0]), 1e-6)
    assert abs(r[0] - 0.848528) < 1e-5
    assert abs(r[1] - 2.2627416) < 1e-5


def test_matvec_known_matrix():
    w = np.array([1.0, 2.0, 3.0, 4.0], dtype=np.float32).view(np.uint8)
    y = O.gemv_dot(O.F32, w, 2, 2, np.array([5.0, 6.0], dtype=np.float32), 1)
    assert list(y[0]) == [17.0, 39.0]


def test_routing_is_stable():
    assert O.top_k(np.array([1.0, 3.0, 3.0, 2.0]), 3) == [(1, 3.0), (2, 3.0), (3, 2.0)]


# ---- spm-granite-moe/src/moe.rs:182-191 ----
def test_olmoe_route_has_eight_of_sixty_four_experts():
    p = O.softmax_route(np.arange(64, dtype=np.float32))
    assert [i for i, _ in O.top_k(p, 8)] == [63, 62, 61, 60, 59, 58, 57, 56]


def test_serial_order_is_expert_id_order():
    # moe.rs:165-180: the union of routes, visited in ascending id order.
    logits = np.array([v % 9 for v in range(32)], dtype=np.float32)
    ids = sorted({i for i, _ in O.top_k(O.softmax_route(logits), 8)})
    assert all(a < b for a, b in zip(ids, ids[1:]))


# ---- greedy selection, spm-batch/examples/serve-demo.rs:72-79 ----
def test_greedy_tie_goes_to_the_last_index():
    assert O.argmax_last(np.array([1.0, 3.0, 3.0, 2.0])) == 2
    assert O.argmax_last(np.array([5.0])) == 0


# ---- spm-linear: the FMA chain ----
def test_gemv_is_a_fused_multiply_add_chain():
    # spm-linear/src/resident.rs:135 uses mul_add: out = fma(w, x, out).
    # acc = -1, then fma((1+2^-23), (1+2^-22), -1) keeps the 2^-45 term that
    # a separate multiply would round away.
    w = np.array([-1.0, 1.0 + 2.0**-23], dtype=np.float32)
    x = np.array([1.0, 1.0 + 2.0**-22], dtype=np.float32)
    y = O.gemv_fma(O.F32, w.view(np.uint8), 1, 2, x, 1)[0, 0]
    assert y == np.float32(3 * 2.0**-23 + 2.0**-45)
    # the logits path (spm-batch/src/inner.rs:89-105, finish) is multiply-then-add
    y2 = O.gemv_dot(O.F32, w.view(np.uint8), 1, 2, x, 1)[0, 0]
    assert y2 == np.float32(3 * 2.0**-23)
