"""Block-profile .spm streams (Q8_0, Q6K, Q5K) on the B200: the outputs of
q6_operation / stream_matrix bit-identical to the oracle, for whole tensors,
for shapes whose rows start and end inside blocks, for several input counts
and every positions-per-thread variant."""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import qblocks as Q
from emufpga_b200 import spmfile as sf
from oracle import oracle as O
from tests.test_qblocks import tensor_blocks

pytestmark = pytest.mark.gpu


def bits_equal(a, b):
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("enc", [sf.Q8_0, sf.Q6_K, sf.Q5_K])
@pytest.mark.parametrize("reshape", [None, 1, 3, 12])
@pytest.mark.parametrize("inputs", [1, 3, 8])
def test_bit_identical_to_the_oracle(cuda, enc, reshape, inputs):
    blocks, rows, cols = tensor_blocks(enc)
    if reshape is not None:  # six blocks read as `reshape` rows
        bv, bb = sf.BLOCK[enc]
        blocks = blocks[: 6 * bb]
        rows, cols = reshape, 6 * bv // reshape
    data = sf.qblock_file(rows, cols, enc, blocks)
    rng = np.random.default_rng(enc * 100 + (reshape or 0) + inputs)
    xs = [(rng.standard_normal(cols) * 4).astype(np.float32) for _ in range(inputs)]
    got = Q.q_operation(data, 0, xs)
    want = O.spm_qblocks(data, np.concatenate(xs), inputs)
    assert bits_equal(np.stack(got), want)


@pytest.mark.parametrize("rows", [16384, 32768])
def test_every_positions_per_thread_variant(cuda, rows):
    import torch

    rng = np.random.default_rng(rows)
    blk = bytearray(rng.integers(0, 256, rows * 34, dtype=np.uint8).tobytes())
    for i in range(rows):  # a normal f16 scale in every block
        blk[i * 34:i * 34 + 2] = (0x2c00 | int(rng.integers(0, 0x3ff))).to_bytes(2, "little")
    data = sf.qblock_file(rows, 32, sf.Q8_0, bytes(blk))
    with Q.QBlockMatrix(data) as m:
        for positions in (8, 7):
            x = rng.standard_normal(positions * 32).astype(np.float32)
            y = m.gemv(torch.from_numpy(x).to(cuda), positions).cpu().numpy()
            assert bits_equal(y, O.spm_qblocks(data, x, positions))


def test_too_few_activations_and_no_inputs(cuda):
    import torch

    blocks, rows, cols = tensor_blocks(sf.Q8_0)
    data = sf.qblock_file(rows, cols, sf.Q8_0, blocks)
    assert Q.q_operation(data, 0, []) == []
    with Q.QBlockMatrix(data) as m:
        with pytest.raises(eb.SpmError) as e:
            m.gemv(torch.zeros(cols - 1, device=cuda), 1)
        assert e.value.code == -2
