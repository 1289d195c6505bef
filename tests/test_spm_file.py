""".spm files and the ternary oracle on the CPU.

Mirrors the reference's format tests (spm-file/tests/golden.rs, errors.rs;
spm-header/tests/wire.rs; spm-layout/tests/wire.rs) against the library's
host reader and this repo's writer, and pins the ternary oracle against the
reference's gemv-ref tests (spm-gemv-ref/tests/correctness.rs,
batch_and_metrics.rs).  The device upload's refusals happen on the host
before any device call, so they are checked here too.
"""
import struct
from pathlib import Path

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import spmfile as sf
from emufpga_b200 import ternary as T
from oracle import oracle as O
from tests.spm_cases import generate, random_file, reference_gemv

GOLDEN = (Path(__file__).resolve().parent / "golden" / "tiny_ternary.spm").read_bytes()
SPM_E_ARG, SPM_E_ACTIVATION_LEN, SPM_E_TRUNCATED, SPM_E_STREAM, SPM_E_ENCODING = -1, -2, -3, -4, -5
SPM_E_NO_DEVICE = -10


def tiny_writer():
    w = sf.SpmWriter([(3, 2, 4)])
    w.write_group(1.0, [1, 0, -1, 1])
    w.write_group(0.5, [-1, 0])
    return w


def status(fn, *args):
    try:
        fn(*args)
    except eb.SpmError as e:
        return e.code, str(e)
    return 0, ""


# ---- format (spm-file/tests/golden.rs) ----

def test_the_writer_reproduces_the_fixture_byte_for_byte():
    assert tiny_writer().finish() == GOLDEN
    codes = sf.ternary_codes([1, 0, -1, 1, -1, 0])
    assert sf.ternary_file(3, 2, 4, codes, np.array([1.0, 0.5], np.float32)) == GOLDEN


def test_the_fixture_matches_the_documented_offsets():
    assert GOLDEN[:8] == bytes([0x89, ord("S"), ord("P"), ord("M"), 0x0D, 0x0A, 0x1A, 0x0A])
    assert GOLDEN[16:20] == struct.pack("<I", 1)
    assert GOLDEN[32:44] == struct.pack("<III", 3, 2, 4)
    assert GOLDEN[44] == 1
    assert GOLDEN[64:68] == struct.pack("<f", 1.0)
    assert GOLDEN[68] == 0b01_11_00_01
    assert GOLDEN[69:73] == struct.pack("<f", 0.5)
    assert GOLDEN[73] == 0b00_11


def test_the_library_reads_the_fixture_back():
    assert T.file_probe(GOLDEN) == (1, 0, 1)
    s = T.file_stream(GOLDEN, 0)
    assert (s.rows, s.cols, s.group_size, s.encoding, s.lane_count) == (3, 2, 4, 1, 1)
    assert (s.groups, s.offset, s.bytes) == (2, 64, 10)
    assert O.spm_describe(GOLDEN) == {"streams": 1, "rows": 3, "cols": 2, "group_size": 4, "encoding": 1}


def test_the_fixture_computes_its_known_answer():
    # y0 = +x0 + x1 (scale 1), y1 = -0.5 x1, y2 = -x0
    x = np.array([[3.0, 5.0], [1.0, -2.0]], np.float32)
    np.testing.assert_array_equal(O.spm_run_gemv(GOLDEN, x), [[8.0, -2.5, -3.0], [-1.0, 1.0, -1.0]])


# ---- header and descriptor wire rules (spm-header/tests/wire.rs, spm-layout/tests/wire.rs) ----

def test_header_and_descriptor_reserved_bytes_are_zero():
    h = sf.render_header(7)
    assert len(h) == 32 and h[13:16] == bytes(3) and h[20:32] == bytes(12)
    d = sf.render_descriptor(512, 256, 64, sf.TERNARY, 8)
    assert len(d) == 32 and d[13] == 0 and d[16:32] == bytes(16)
    assert struct.unpack_from("<IIIBxH", d) == (512, 256, 64, 1, 8)


def test_encoding_codes_keep_their_block_sizes():
    assert (sf.TERNARY, sf.F32, sf.BF16, sf.Q6_K, sf.Q5_K, sf.Q8_0) == (1, 2, 3, 4, 5, 6)
    assert sf.bytes_for(sf.Q6_K, 256) == 210
    assert sf.bytes_for(sf.Q5_K, 256) == 176
    assert sf.bytes_for(sf.Q8_0, 32) == 34
    assert sf.bytes_for(sf.TERNARY, 5) == 2


def malformed():
    good = bytearray(GOLDEN)
    cases = {}
    b = bytearray(good); b[0] = 0
    cases["bad magic"] = (bytes(b), SPM_E_STREAM, "bad magic")
    cases["short header"] = (bytes(good[:8]), SPM_E_TRUNCATED, "header truncated: 8 bytes available, need 32")
    b = bytearray(good); b[8] = 99
    cases["newer major"] = (bytes(b), SPM_E_STREAM, "unsupported .spm major version 99: this build reads up to 1")
    b = bytearray(good); b[12] = 3
    cases["endianness"] = (bytes(b), SPM_E_STREAM, "unknown endianness discriminant 3")
    b = bytearray(good); b[44] = 200
    cases["unknown encoding"] = (bytes(b), SPM_E_ENCODING, "unknown .spm encoding profile 200")
    b = bytearray(good); b[40:44] = bytes(4)
    cases["zero group"] = (bytes(b), SPM_E_STREAM, "group_size must be at least 1")
    cases["short directory"] = (bytes(good[:48]), SPM_E_TRUNCATED, "descriptor truncated: 16 bytes, need 32")
    b = bytearray(good[:64]); b[16:20] = struct.pack("<I", 0xFFFFFFFF)
    cases["hostile stream count"] = (bytes(b), SPM_E_TRUNCATED, "descriptor truncated: 0 bytes, need 32")
    return cases


@pytest.mark.parametrize("name", sorted(malformed()))
def test_malformed_files_fail_loudly_and_alike(name):
    data, code, msg = malformed()[name]
    got, text = status(T.file_probe, data)
    assert got == code and msg in text
    # the oracle reads the same bytes to the same refusal
    with pytest.raises(O.SpmError) as e:
        O.spm_describe(data)
    assert e.value.code == code and msg in str(e.value)


def test_a_truncated_payload_is_detected_rather_than_read_past():
    code, text = status(T.file_stream, GOLDEN[:-1], 0)
    assert code == SPM_E_TRUNCATED and "group needs 5 bytes, 4 remain" in text
    with pytest.raises(O.SpmError) as e:
        O.spm_run_gemv(GOLDEN[:-1], np.zeros((1, 2), np.float32))
    assert e.value.code == SPM_E_TRUNCATED and "group needs 5 bytes, 4 remain" in str(e.value)


# ---- writer refusals (spm-file/tests/errors.rs) ----

def test_finishing_with_unwritten_streams_fails():
    w = sf.SpmWriter([(3, 2, 4)])
    w.write_group(1.0, [1] * 4)
    with pytest.raises(ValueError, match="only 0 of 1 streams were written"):
        w.finish()


def test_a_group_of_the_wrong_length_is_refused():
    with pytest.raises(ValueError, match="group expects 4 weights, got 3"):
        sf.SpmWriter([(3, 2, 4)]).write_group(1.0, [1] * 3)


def test_writing_past_the_last_declared_stream_is_refused():
    w = tiny_writer()
    with pytest.raises(ValueError, match="only 1 of 1 streams were written"):
        w.write_group(1.0, [1] * 4)


def test_a_value_that_is_not_ternary_is_refused():
    with pytest.raises(ValueError, match="value 2 is not ternary"):
        sf.ternary_codes([1, 2])


# ---- streams: placement, empty streams, several streams ----

def test_streams_are_placed_in_order_and_empty_ones_hold_no_groups():
    w = sf.SpmWriter([(3, 2, 4), (0, 5, 3), (2, 3, 3, sf.F32)])
    w.write_group(1.0, [1, 0, -1, 1])
    w.write_group(0.5, [-1, 0])
    w.write_raw_group(1.0, struct.pack("<3f", 1, 2, 3), 3)
    w.write_raw_group(1.0, struct.pack("<3f", 4, 5, 6), 3)
    data = w.finish()
    assert T.file_probe(data) == (1, 0, 3)
    s1, s2 = T.file_stream(data, 1), T.file_stream(data, 2)
    assert (s1.groups, s1.bytes, s1.offset) == (0, 0, 32 + 3 * 32 + 10)
    assert (s2.groups, s2.bytes, s2.offset, s2.encoding) == (2, 32, s1.offset, sf.F32)
    # the next stream's first group is read by the reference's scan before it
    # stops, so cutting it makes the first stream's GEMV fail too
    with pytest.raises(O.SpmError) as e:
        O.spm_run_gemv(data[:-20], np.zeros((1, 2), np.float32))
    assert e.value.code == SPM_E_TRUNCATED
    assert status(T.TernaryMatrix, data[:-20])[0] == SPM_E_TRUNCATED
    assert O.spm_run_gemv(data[:-16], np.ones((1, 2), np.float32)).shape == (1, 3)


# ---- the ternary oracle against the reference's gemv-ref tests ----

CORRECTNESS = [(3, 2, 4), (8, 4, 8), (8, 4, 3), (16, 5, 16), (7, 3, 64), (1, 1, 64)]


@pytest.mark.parametrize("index,shape", list(enumerate(CORRECTNESS)))
def test_oracle_matches_the_f64_reference_across_shapes_and_group_sizes(index, shape):
    case = generate(index + 1, *shape)
    got = O.spm_run_gemv(case.spm(), case.activations[None, :])[0].astype(np.float64)
    want = reference_gemv(case)
    assert np.abs(got - want).max(initial=0.0) <= 2e-3
    if np.any(got) and np.any(want):
        cos = got @ want / (np.linalg.norm(got) * np.linalg.norm(want))
        assert cos > 0.999_999


def test_generator_follows_the_reference_draw_order():
    # draw.rs: weights first, then scales, then activations, all from one state
    case = generate(21, 16, 5, 8)
    assert case.weights.size == 80 and case.scales.size == 10 and case.activations.size == 5
    assert set(np.unique(case.weights)) <= {-1, 0, 1}
    assert np.all((case.scales * 16 - 1) % 1 == 0) and case.scales.min() >= 0.0625
    assert np.all((case.activations * 16) % 1 == 0) and case.activations.min() >= -2.0
    assert generate(21, 16, 5, 8).spm() == case.spm()


def test_oracle_every_lane_agrees_when_every_lane_holds_the_same_activations():
    case = generate(21, 16, 5, 8)
    one = O.spm_run_gemv(case.spm(), case.activations[None, :])
    eight = O.spm_run_gemv(case.spm(), np.tile(case.activations, (8, 1)))
    for lane in range(8):
        np.testing.assert_array_equal(eight[lane], one[0])


def test_oracle_zero_weight_matrix_and_missing_activations():
    case = generate(11, 0, 4, 8)
    assert O.spm_run_gemv(case.spm(), case.activations[None, :]).shape == (1, 0)
    case = generate(13, 8, 4, 8)
    with pytest.raises(O.SpmError, match="need 4 activations per lane, got 2"):
        O.spm_run_gemv(case.spm(), case.activations[None, :2])


def test_oracle_reserved_codes_are_no_ops_like_the_datapath():
    rng = np.random.default_rng(3)
    data, codes, scales = random_file(rng, 9, 7, 5, reserved=0.3)
    assert (codes == 2).any()
    cleared = sf.ternary_file(9, 7, 5, np.where(codes == 2, 0, codes), scales)
    x = rng.standard_normal((2, 7)).astype(np.float32)
    np.testing.assert_array_equal(O.spm_run_gemv(data, x), O.spm_run_gemv(cleared, x))


# ---- the device upload refuses on the host before touching a device ----

def test_upload_refuses_non_ternary_streams_and_empty_files():
    w = sf.SpmWriter([(2, 3, 3, sf.F32)])
    w.write_raw_group(1.0, struct.pack("<3f", 1, 2, 3), 3)
    w.write_raw_group(1.0, struct.pack("<3f", 4, 5, 6), 3)
    code, text = status(T.TernaryMatrix, w.finish())
    assert code == SPM_E_ENCODING and "not ternary" in text
    code, text = status(T.TernaryMatrix, sf.render_header(0))
    assert code == SPM_E_ARG and "declares no operations" in text
    code, _ = status(T.TernaryMatrix, GOLDEN, 1)
    assert code == SPM_E_ARG


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the refusal without a device")
def test_upload_without_a_device_fails_loudly():
    assert status(T.TernaryMatrix, GOLDEN)[0] == SPM_E_NO_DEVICE
