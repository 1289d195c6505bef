"""spm_linear::streamed for dense .spm streams: the oracle on the CPU.

Mirrors spm-linear/tests/agreement.rs (streamed == resident bit for bit on
the reference's own shapes, consecutive streams, a group size that does not
divide, a stream that ends early, batching) and the error kinds of
stream.rs:63-100 / spm-codec-any/src/decode.rs.  The device upload's
refusals happen on the host before any device call, so they are checked here.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import linear as L
from emufpga_b200 import spmfile as sf
from oracle import oracle as O
from tests.spm_cases import sixteenths


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("index,shape", list(enumerate([(1536, 512), (512, 512), (3072, 512), (512, 1536)])))
def test_streamed_and_resident_agree_bit_for_bit(index, shape):
    rows, cols = shape
    matrix = sixteenths(index + 1, rows * cols)
    x = sixteenths(1000 + index, cols)
    data = sf.dense_file([shape], 1024, [matrix])
    np.testing.assert_array_equal(bits(O.spm_streamed(data, x, 1)), bits(O.resident(matrix, rows, cols, x, 1)))


def test_consecutive_streams_are_consumed_in_order():
    shapes = [(8, 4), (4, 8), (16, 2)]
    matrices = [sixteenths(i + 7, r * c) for i, (r, c) in enumerate(shapes)]
    data = sf.dense_file(shapes, 16, matrices)
    for index, (rows, cols) in enumerate(shapes):
        x = sixteenths(500 + index, cols)
        np.testing.assert_array_equal(bits(O.spm_streamed(data, x, 1, index)),
                                      bits(O.resident(matrices[index], rows, cols, x, 1)))


def test_a_group_size_that_does_not_divide_still_agrees():
    matrix, x = sixteenths(42, 35), sixteenths(43, 5)
    data = sf.dense_file([(7, 5)], 16, [matrix])  # groups of 16, 16 and 3
    np.testing.assert_array_equal(bits(O.spm_streamed(data, x, 1)), bits(O.resident(matrix, 7, 5, x, 1)))


def test_a_stream_that_ends_early_is_refused():
    data = sf.dense_file([(8, 4)], 16, [sixteenths(9, 32)])
    with pytest.raises(O.SpmError, match="stream ended after 32 of 64 weights"):
        O.spm_streamed(data, sixteenths(10, 4), 1, shape=(16, 4))


def test_batching_reuses_each_weight_without_changing_any_answer():
    rows, cols, positions = 16, 8, 5
    matrix = sixteenths(77, rows * cols)
    batch = np.concatenate([sixteenths(100 + p, cols) for p in range(positions)])
    got = O.spm_streamed(sf.dense_file([(rows, cols)], 32, [matrix]), batch, positions)
    for p in range(positions):
        alone = O.resident(matrix, rows, cols, batch[p * cols:(p + 1) * cols], 1)
        np.testing.assert_array_equal(bits(got[p]), bits(alone[0]))


def test_bf16_streams_decode_by_widening():
    rng = np.random.default_rng(2)
    w = rng.standard_normal(6 * 5).astype(np.float32)
    x = rng.standard_normal(5).astype(np.float32)
    widened = (sf.bf16_round(w).astype(np.uint32) << 16).view(np.float32)
    data = sf.dense_file([(6, 5)], 8, [w], sf.BF16)
    np.testing.assert_array_equal(bits(O.spm_streamed(data, x, 1)), bits(O.resident(widened, 6, 5, x, 1)))


def test_bf16_rounding_ties_to_even_and_keeps_nan_quiet():
    v = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.nan], np.float32)
    assert sf.bf16_round(v).tolist() == [0x3F80, 0x3F80, 0x3F82, 0xC020, 0x7FC0]


def test_too_few_activations_fail_before_the_scan():
    data = sf.dense_file([(3, 4)], 8, [sixteenths(1, 12)])
    with pytest.raises(O.SpmError, match="need 12 activations, got 11"):
        O.spm_streamed(data, np.zeros(11, np.float32), 3)


@pytest.mark.parametrize("encoding,name", [(sf.TERNARY, "Ternary2F32I32"), (sf.Q8_0, "Q8_0")])
def test_profiles_without_a_dense_decoder_are_refused(encoding, name):
    w = sf.SpmWriter([(2, 16, 32, encoding)])
    w.write_raw_group(1.0, bytes(sf.bytes_for(encoding, 32)), 32)
    data = w.finish()
    msg = f"parameter stream: {name} needs a scale-aware engine"
    with pytest.raises(O.SpmError, match=msg):
        O.spm_streamed(data, np.zeros(16, np.float32), 1)
    with pytest.raises(eb.SpmError, match=msg) as e:
        L.DenseMatrix(data)
    assert e.value.code == -4


def test_upload_refuses_a_cut_stream_and_a_missing_index():
    data = sf.dense_file([(4, 4)], 8, [sixteenths(3, 16)])
    with pytest.raises(eb.SpmError) as e:
        L.DenseMatrix(data[:-1])
    assert e.value.code == -3
    with pytest.raises(eb.SpmError) as e:
        L.DenseMatrix(data, 1)
    assert e.value.code == -1
