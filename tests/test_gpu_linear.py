"""Dense .spm streamed GEMV on the B200: bit-identical to the oracle.

The reference's agreement tests (spm-linear/tests/agreement.rs) run on the
device, plus F32 and Bf16 streams of shapes that exercise the layout (rows
not a multiple of 32, columns not a multiple of 16, groups smaller than,
equal to and spanning columns), weights spread over six decades (so only the
reference's order of fused multiply-adds reproduces the results), every
positions-per-thread variant, a later stream of a multi-stream file, empty
shapes and a 4096 x 4096 stream.  Raw bits are compared.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import linear as L
from emufpga_b200 import spmfile as sf
from oracle import oracle as O
from tests.spm_cases import sixteenths

pytestmark = pytest.mark.gpu


def bits_equal(a, b):
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("index,shape", list(enumerate([(1536, 512), (512, 512), (3072, 512), (512, 1536)])))
def test_streamed_and_resident_agree_bit_for_bit(cuda, index, shape):
    rows, cols = shape
    matrix = sixteenths(index + 1, rows * cols)
    x = sixteenths(1000 + index, cols)
    got = L.streamed(sf.dense_file([shape], 1024, [matrix]), 0, x, 1)
    assert bits_equal(got, O.resident(matrix, rows, cols, x, 1))


def test_consecutive_streams_and_batching(cuda):
    shapes = [(8, 4), (4, 8), (16, 2)]
    matrices = [sixteenths(i + 7, r * c) for i, (r, c) in enumerate(shapes)]
    data = sf.dense_file(shapes, 16, matrices)
    for index, (rows, cols) in enumerate(shapes):
        batch = np.concatenate([sixteenths(500 + index + 10 * p, cols) for p in range(5)])
        assert bits_equal(L.streamed(data, index, batch, 5), O.resident(matrices[index], rows, cols, batch, 5))


SHAPES = [(1, 1, 1), (7, 5, 16), (33, 17, 33), (33, 17, 5), (31, 47, 1000), (100, 40, 7), (40, 300, 96),
          (9, 2049, 64), (257, 19, 100), (1000, 300, 1000)]


@pytest.mark.parametrize("encoding", [sf.F32, sf.BF16])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("positions", [1, 3, 8])
def test_bit_identical_to_the_oracle(cuda, encoding, shape, positions):
    rows, cols, group = shape
    rng = np.random.default_rng(rows * 7919 + cols * 31 + group + positions + encoding)
    w = (rng.standard_normal(rows * cols) * rng.choice([1e-3, 1.0, 1e3], rows * cols)).astype(np.float32)
    x = (rng.standard_normal(positions * cols) * 10).astype(np.float32)
    data = sf.dense_file([(rows, cols)], group, [w], encoding)
    assert bits_equal(L.streamed(data, 0, x, positions), O.spm_streamed(data, x, positions))


@pytest.mark.parametrize("rows", [16384, 32768])
def test_every_positions_per_thread_variant(cuda, rows):
    # with 8 positions these row counts pick 2 and 4 positions per thread on 148 SMs
    rng = np.random.default_rng(rows)
    w = rng.standard_normal(rows * 21).astype(np.float32)
    data = sf.dense_file([(rows, 21)], rows, [w])
    for positions in (8, 7):
        x = rng.standard_normal(positions * 21).astype(np.float32)
        assert bits_equal(L.streamed(data, 0, x, positions), O.spm_streamed(data, x, positions))


def test_a_large_stream(cuda):
    rng = np.random.default_rng(9)
    w = (rng.standard_normal(4096 * 4096) * 0.02).astype(np.float32)
    x = rng.standard_normal(8 * 4096).astype(np.float32)
    data = sf.dense_file([(4096, 4096)], 4096, [w])
    with L.DenseMatrix(data) as m:
        assert m.payload_bytes == 4096 * 4096 * 4
        import torch

        y = m.streamed(torch.from_numpy(x).to(cuda), 8).cpu().numpy()
    assert bits_equal(y, O.spm_streamed(data, x, 8))


def test_a_later_stream_on_a_side_cuda_stream(cuda):
    import torch

    rng = np.random.default_rng(4)
    first, second = rng.standard_normal(6 * 4).astype(np.float32), rng.standard_normal(20 * 11).astype(np.float32)
    data = (sf.render_header(2) + sf.render_descriptor(6, 4, 8, sf.BF16) + sf.render_descriptor(20, 11, 8, sf.BF16)
            + sf.dense_stream_bytes(first, 8, sf.BF16) + sf.dense_stream_bytes(second, 8, sf.BF16))
    x = rng.standard_normal(3 * 11).astype(np.float32)
    s = torch.cuda.Stream()
    with L.DenseMatrix(data, 1) as m:
        xd = torch.from_numpy(x).to(cuda)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            y = m.streamed(xd, 3, stream=s)
        s.synchronize()
        assert bits_equal(y.cpu().numpy(), O.spm_streamed(data, x, 3, 1))


def test_empty_shapes_and_too_few_activations(cuda):
    import torch

    for rows, cols in ((0, 5), (5, 0)):
        data = sf.dense_file([(rows, cols)], 4, [np.zeros(0, np.float32)])
        x = np.ones(2 * cols, np.float32)
        assert bits_equal(L.streamed(data, 0, x, 2), O.spm_streamed(data, x, 2))
    data = sf.dense_file([(3, 4)], 8, [sixteenths(1, 12)])
    with L.DenseMatrix(data) as m:
        with pytest.raises(eb.SpmError, match="need 12 activations, got 11") as e:
            m.streamed(torch.zeros(11, device=cuda), 3)
        assert e.value.code == -2
        assert tuple(m.streamed(torch.zeros(4, device=cuda), 0).shape) == (0, 3)
