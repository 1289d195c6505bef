"""Host-to-HBM sweeps on the B200: every stream's result bit-identical to the
oracle, sweep after sweep, with rings from one stream wide (every copy waits
for the previous kernel) to the whole file; rewinds at the end and in
mid-sweep; the refusal past the last stream; opening by path."""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import spmfile as sf
from emufpga_b200 import sweep as S
from emufpga_b200 import ternary as T
from oracle import oracle as O
from tests.spm_cases import random_file

pytestmark = pytest.mark.gpu

# (kind, rows, cols, group)
STREAMS = [("ternary", 300, 200, 7), (sf.F32, 128, 64, 64), (sf.BF16, 257, 100, 100), ("ternary", 64, 500, 64),
           (sf.F32, 1000, 30, 333)]


def mixed_file(rng):
    descs, bodies = [], []
    for kind, rows, cols, group in STREAMS:
        if kind == "ternary":
            one, _, _ = random_file(rng, rows, cols, group)
            descs.append(sf.render_descriptor(rows, cols, group))
            bodies.append(one[64:])
        else:
            w = (rng.standard_normal(rows * cols) * rng.choice([1e-3, 1.0, 1e3], rows * cols)).astype(np.float32)
            descs.append(sf.render_descriptor(rows, cols, group, kind))
            bodies.append(sf.dense_stream_bytes(w, group, kind))
    return sf.render_header(len(STREAMS)) + b"".join(descs) + b"".join(bodies)


def oracle(data, k, x, positions):
    kind, rows, cols, _ = STREAMS[k]
    if kind == "ternary":
        st = T.file_stream(data, k)
        one = sf.render_header(1) + data[32 + 32 * k:64 + 32 * k] + data[st.offset:st.offset + st.bytes]
        return O.spm_run_gemv(one, x.reshape(positions, cols))
    return O.spm_streamed(data, x, positions, k)


def bits_equal(a, b):
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def run_sweep(sw, data, rng, cuda, positions=3, stop=None):
    import torch

    for k in range(len(STREAMS) if stop is None else stop):
        cols = STREAMS[k][2]
        x = (rng.standard_normal(positions * cols) * 10).astype(np.float32)
        index, y = sw.next(torch.from_numpy(x).to(cuda), positions)
        assert index == k
        torch.cuda.synchronize()
        assert bits_equal(y.cpu().numpy(), oracle(data, k, x, positions)), f"stream {k}"


@pytest.mark.parametrize("ring", ["largest", "default", "all"])
def test_sweeps_match_the_oracle(cuda, ring):
    import torch

    rng = np.random.default_rng(1)
    data = mixed_file(rng)
    with S.Sweep(data, device_bytes=0) as probe:
        host = probe.describe()["host_bytes"]
    device_bytes = {"largest": largest_stream(data), "default": 0, "all": host}[ring]
    with S.Sweep(data, device_bytes=device_bytes) as sw:
        assert sw.streams == len(STREAMS)
        for _ in range(3):
            run_sweep(sw, data, rng, cuda)
            with pytest.raises(eb.SpmError) as e:
                sw.next(torch.zeros(10_000, device=cuda), 1)
            assert e.value.code == -3
            sw.rewind()
        # a rewind in mid-sweep drops what was read ahead; the next sweep is whole
        run_sweep(sw, data, rng, cuda, stop=2)
        sw.rewind()
        run_sweep(sw, data, rng, cuda, positions=1)
        info = sw.describe()
        assert info["device_bytes"] == (device_bytes or 2 * largest_stream(data))
        assert info["copies"] >= 4 * len(STREAMS)


def largest_stream(data):
    """The smallest ring that opens: the refusal of a 256-byte ring names it."""
    with pytest.raises(eb.SpmError) as e:
        S.Sweep(data, device_bytes=256)
    return int(str(e.value).rsplit("(", 1)[1].split()[0])


def test_open_by_path(cuda, tmp_path):
    rng = np.random.default_rng(2)
    data = mixed_file(rng)
    path = tmp_path / "mixed.spm"
    path.write_bytes(data)
    with S.Sweep(str(path)) as sw:
        run_sweep(sw, data, rng, cuda, positions=2)


def test_sweeps_over_block_streams(cuda):
    """Block-profile streams (Q6_K, Q8_0) beside a ternary one, through a ring
    of the largest stream: each bit-identical to the oracle's q6_operation."""
    import torch

    from tests.test_qblocks import tensor_blocks

    rng = np.random.default_rng(3)
    q6, r6, c6 = tensor_blocks(sf.Q6_K)
    q8, r8, c8 = tensor_blocks(sf.Q8_0)
    tern, _, _ = random_file(rng, 40, 30, 9)
    data = (sf.render_header(3) + sf.render_descriptor(r6, c6, 256, sf.Q6_K) + sf.render_descriptor(40, 30, 9)
            + sf.render_descriptor(r8, c8, 32, sf.Q8_0) + sf.qblock_stream_bytes(q6, sf.Q6_K) + tern[64:]
            + sf.qblock_stream_bytes(q8, sf.Q8_0))
    shapes = [(r6, c6), (40, 30), (r8, c8)]
    with S.Sweep(data, device_bytes=largest_stream(data)) as sw:
        for _ in range(2):
            for k, (rows, cols) in enumerate(shapes):
                x = rng.standard_normal(2 * cols).astype(np.float32)
                index, y = sw.next(torch.from_numpy(x).to(cuda), 2)
                torch.cuda.synchronize()
                assert index == k
                if k == 1:
                    st = T.file_stream(data, 1)
                    one = sf.render_header(1) + data[64:96] + data[st.offset:st.offset + st.bytes]
                    want = O.spm_run_gemv(one, x.reshape(2, cols))
                else:
                    want = O.spm_qblocks(data, x, 2, k)
                assert bits_equal(y.cpu().numpy(), want), f"stream {k}"
            sw.rewind()
