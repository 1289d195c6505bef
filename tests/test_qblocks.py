"""The block profiles of .spm files (Q8_0, Q6K, Q5K) on the CPU: the oracle's
restatement of q6_operation / stream_matrix (spm-granite-moe/src/
layout.rs:208-242, gemma_smoke.rs:201-236) pinned against its FMA-chain GEMV
over the same blocks and a hand-computed answer, and the refusals the device
upload makes on the host."""
import ctypes as C
import struct

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs
from emufpga_b200 import qblocks as Q
from emufpga_b200 import spmfile as sf
from oracle import oracle as O

GGML = {sf.Q8_0: 8, sf.Q6_K: 14, sf.Q5_K: 13}
SOURCE = {sf.Q8_0: "llama-q8_0", sf.Q6_K: "llama-q6_k", sf.Q5_K: "qwen3-q5_k"}


def tensor_blocks(enc, name="blk.0.ffn_down.weight"):
    img = eb.synth_gguf(configs.TINY[SOURCE[enc]])
    t = eb.gguf_find(img, name)
    assert t["dtype"] == GGML[enc]
    return bytes(img[t["offset"]:t["offset"] + t["nbytes"]]), t["dims"][1], t["dims"][0]


@pytest.mark.parametrize("enc", [sf.Q8_0, sf.Q6_K, sf.Q5_K])
def test_restatement_matches_the_fma_chain_gemv(enc):
    blocks, rows, cols = tensor_blocks(enc)
    x = np.random.default_rng(enc).standard_normal(3 * cols).astype(np.float32)
    got = O.spm_qblocks(sf.qblock_file(rows, cols, enc, blocks), x, 3)
    buf = np.frombuffer(blocks, np.uint8).copy()
    want = np.empty(3 * rows, np.float32)
    assert O.lib().or_gemv_fma(GGML[enc], buf.ctypes.data, rows, cols, x.ctypes.data_as(C.POINTER(C.c_float)), 3,
                               want.ctypes.data_as(C.POINTER(C.c_float)), 1) == 0
    np.testing.assert_array_equal(got.view(np.uint32).ravel(), want.view(np.uint32))


def test_q8_0_known_answer_with_rows_inside_a_block():
    # one Q8_0 block, d = 0.5, q = 1..32, read as 4 rows of 8: row r holds
    # 0.5 * (8r+1 .. 8r+8); with x = 1..8 each row sums 0.5 * sum((8r+c) * c)
    blk = struct.pack("<e", 0.5) + bytes(range(1, 33))
    x = np.arange(1, 9, dtype=np.float32)
    got = O.spm_qblocks(sf.qblock_file(4, 8, sf.Q8_0, blk), x, 1)[0]
    want = [0.5 * sum((8 * r + c) * c for c in range(1, 9)) for r in range(4)]
    np.testing.assert_array_equal(got, np.array(want, np.float32))


def refusals():
    blocks, _, _ = tensor_blocks(sf.Q6_K)
    one = blocks[:210]
    two = blocks[:420]
    cases = {
        # two blocks in one group of 512 values
        "group of two blocks": (sf.render_header(1) + sf.render_descriptor(2, 256, 512, sf.Q6_K)
                                + struct.pack("<f", 1.0) + two, -4, "unexpected packed group"),
        # 300 values: the last group is short
        "short last group": (sf.render_header(1) + sf.render_descriptor(3, 100, 256, sf.Q6_K)
                             + struct.pack("<f", 1.0) + one + struct.pack("<f", 1.0) + one, -4,
                             "unexpected packed group"),
        "dense profile": (sf.dense_file([(2, 2)], 4, [np.ones(4, np.float32)]), -4, "not a block profile"),
    }
    return cases


@pytest.mark.parametrize("name", sorted(refusals()))
def test_refusals_agree(name):
    data, code, msg = refusals()[name]
    with pytest.raises(eb.SpmError, match=msg) as e:
        Q.QBlockMatrix(data)
    assert e.value.code == code
    with pytest.raises(O.SpmError, match=msg):
        O.spm_qblocks(data, np.ones(1024, np.float32), 1)


def test_writer_frames_one_block_per_group():
    blocks, rows, cols = tensor_blocks(sf.Q8_0)
    data = sf.qblock_file(rows, cols, sf.Q8_0, blocks)
    from emufpga_b200 import ternary as T

    st = T.file_stream(data, 0)
    assert (st.rows, st.cols, st.group_size, st.encoding) == (rows, cols, 32, sf.Q8_0)
    assert st.groups == len(blocks) // 34 and st.bytes == st.groups * (4 + 34)
    with pytest.raises(ValueError):
        sf.qblock_file(rows + 1, cols, sf.Q8_0, blocks)
