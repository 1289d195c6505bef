"""Ternary GEMV on the B200 against the oracle: bit-identical results.

Every comparison is on the raw bits (a +0/-0 or last-bit difference fails).
Cases follow the reference's gemv-ref tests (spm-gemv-ref/tests/
correctness.rs, batch_and_metrics.rs) plus shapes and group sizes that
exercise the device layout: rows not a multiple of 32, columns not a multiple
of 16, groups smaller than, equal to and spanning columns, reserved codes,
extra activations, empty matrices, and row counts that select every
lanes-per-thread variant of the kernel.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import spmfile as sf
from emufpga_b200 import ternary as T
from oracle import oracle as O
from tests.spm_cases import generate, random_file, reference_gemv

pytestmark = pytest.mark.gpu


def bits_equal(a, b):
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def device_gemv(data, x, cuda, index=0):
    import torch

    with T.TernaryMatrix(data, index) as m:
        y = m.gemv(torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(cuda))
        torch.cuda.synchronize()
        return y.cpu().numpy(), m


def test_the_fixture_computes_its_known_answer(cuda):
    w = sf.SpmWriter([(3, 2, 4)])
    w.write_group(1.0, [1, 0, -1, 1])
    w.write_group(0.5, [-1, 0])
    out = T.run_gemv(w.finish(), T.Activations.per_lane(2, 2, [3.0, 5.0, 1.0, -2.0]))
    np.testing.assert_array_equal(out.bank.data, [[8.0, -2.5, -3.0], [-1.0, 1.0, -1.0]])
    assert out.bank.lane(1).tolist() == [-1.0, 1.0, -1.0]


@pytest.mark.parametrize("index,shape", list(enumerate([(3, 2, 4), (8, 4, 8), (8, 4, 3), (16, 5, 16),
                                                         (7, 3, 64), (1, 1, 64)])))
def test_matches_the_reference_across_shapes_and_group_sizes(cuda, index, shape):
    case = generate(index + 1, *shape)
    out = T.run_gemv(case.spm(), T.Activations.broadcast(1, case.activations))
    assert bits_equal(out.bank.data, O.spm_run_gemv(case.spm(), case.activations[None, :]))
    assert np.abs(out.bank.lane(0) - reference_gemv(case)).max(initial=0.0) <= 2e-3


def test_every_lane_agrees_when_every_lane_holds_the_same_activations(cuda):
    case = generate(21, 16, 5, 8)
    single = T.run_gemv(case.spm(), T.Activations.broadcast(1, case.activations))
    batched = T.run_gemv(case.spm(), T.Activations.broadcast(8, case.activations))
    for lane in range(8):
        assert bits_equal(batched.bank.lane(lane), single.bank.lane(0))


def test_scan_productivity_equals_the_batch_size(cuda):
    case = generate(23, 16, 4, 8)
    for lanes in (1, 2, 4, 8, 16, 32):
        out = T.run_gemv(case.spm(), T.Activations.broadcast(lanes, case.activations))
        assert out.metrics.scan_productivity() == lanes
        assert out.metrics.parameter_bytes_read == (16 * 4 + 3) // 4
        assert out.metrics.weights_decoded == 64
        assert out.metrics.weight_applications == 64 * lanes


SHAPES = [(3, 2, 4), (1, 1, 1), (33, 17, 33), (33, 17, 1), (33, 17, 5), (64, 16, 64), (31, 47, 31 * 47),
          (100, 40, 7), (5, 100, 500), (40, 33, 16), (96, 35, 192), (257, 19, 100), (32, 1, 2), (1000, 300, 1000),
          (70, 1000, 70), (9, 2049, 5)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("lanes,extra", [(1, 0), (3, 2), (8, 0), (17, 1)])
def test_bit_identical_to_the_oracle(cuda, shape, lanes, extra):
    rows, cols, group = shape
    rng = np.random.default_rng(rows * 7919 + cols * 31 + group + lanes)
    data, codes, _ = random_file(rng, rows, cols, group)
    x = (rng.standard_normal((lanes, cols + extra)) * 10).astype(np.float32)
    y, m = device_gemv(data, x, cuda)
    assert m.reserved_codes == int((codes == 2).sum())
    assert bits_equal(y, O.spm_run_gemv(data, x))


@pytest.mark.parametrize("rows,group", [(16384, 16384), (32768, 5), (65536, 1000)])
def test_every_lanes_per_thread_variant(cuda, rows, group):
    # with 8 lanes these row counts pick 2, 4 and 8 lanes per thread on 148 SMs
    rng = np.random.default_rng(rows)
    data, _, _ = random_file(rng, rows, 37, group)
    for lanes in (8, 7):
        x = rng.standard_normal((lanes, 37)).astype(np.float32)
        y, _ = device_gemv(data, x, cuda)
        assert bits_equal(y, O.spm_run_gemv(data, x))


def test_a_large_matrix_at_one_scale_per_column(cuda):
    # group_size == rows: the configuration the reference recommends
    rng = np.random.default_rng(5)
    data, _, _ = random_file(rng, 4096, 4096, 4096, reserved=0.0)
    x = rng.standard_normal((8, 4096)).astype(np.float32)
    y, m = device_gemv(data, x, cuda)
    assert m.payload_bytes == 4096 * 4096 // 4
    assert bits_equal(y, O.spm_run_gemv(data, x))


def test_empty_matrices_and_zero_lanes(cuda):
    import torch

    for rows, cols in ((0, 5), (5, 0)):
        data = sf.ternary_file(rows, cols, 3, np.zeros(0, np.uint8), np.zeros(0, np.float32))
        x = np.ones((2, cols), np.float32)
        y, _ = device_gemv(data, x, cuda)
        assert bits_equal(y, O.spm_run_gemv(data, x)) and y.shape == (2, rows)
    with T.TernaryMatrix(generate(3, 8, 4, 8).spm()) as m:
        assert tuple(m.gemv(torch.empty((0, 4), device=cuda)).shape) == (0, 8)


def test_too_few_activations_fail_before_the_scan(cuda):
    import torch

    case = generate(13, 8, 4, 8)
    with pytest.raises(eb.SpmError, match="need 4 activations per lane, got 2") as e:
        T.run_gemv(case.spm(), T.Activations.broadcast(1, case.activations[:2]))
    assert e.value.code == -2
    with T.TernaryMatrix(case.spm()) as m:
        with pytest.raises(eb.SpmError) as e:
            m.gemv(torch.zeros((1, 3), device=cuda))
        assert e.value.code == -2


def test_a_later_stream_and_a_cuda_stream(cuda):
    import torch

    rng = np.random.default_rng(11)
    first, _, _ = random_file(rng, 6, 5, 4)
    second_codes = rng.integers(0, 4, 70 * 9).astype(np.uint8)
    second_scales = rng.standard_normal(-(-630 // 13)).astype(np.float32)
    data = (sf.render_header(2) + sf.render_descriptor(6, 5, 4) + sf.render_descriptor(70, 9, 13)
            + first[64:] + sf.ternary_stream_bytes(second_codes, second_scales, 13))
    only_second = sf.ternary_file(70, 9, 13, second_codes, second_scales)
    x = rng.standard_normal((3, 9)).astype(np.float32)
    s = torch.cuda.Stream()
    with T.TernaryMatrix(data, 1) as m:
        xd = torch.from_numpy(x).to(cuda)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            y = m.gemv(xd, stream=s)
        s.synchronize()
        assert bits_equal(y.cpu().numpy(), O.spm_run_gemv(only_second, x))
