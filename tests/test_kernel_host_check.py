"""The chain kernels' bodies, compiled for the host, against the oracle.

tests/kernel_host_check.cpp builds the ternary, dense and block kernels from
their CUDA sources for the CPU (builtins replaced by their IEEE host forms,
every thread of a launch run in turn, exact-size buffers, AddressSanitizer
when the compiler has it) so that their thread mapping, group walk, clamps
and order of operations are checked bit for bit against the oracle without a
GPU.  The GPU tests check the same kernels on the device.
"""
import shutil
import subprocess
import tempfile
from pathlib import Path

import numpy as np
import pytest

from emufpga_b200 import spmfile as sf
from oracle import oracle as O
from tests.spm_cases import random_file

ROOT = Path(__file__).resolve().parents[1]
SOURCES = [ROOT / "tests" / "kernel_host_check.cpp", ROOT / "emufpga_b200" / "csrc" / "host_spm.cpp",
           ROOT / "emufpga_b200" / "csrc" / "host_format.cpp"]


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else shutil.which("g++")
    if not cxx:
        pytest.skip("needs g++")
    exe = tmp_path_factory.mktemp("host_check") / "kernel_host_check"
    base = [cxx, "-std=c++17", "-O1", "-g", "-ffp-contract=off", "-Wno-unknown-pragmas",
            f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", *map(str, SOURCES), "-o", str(exe)]
    sanitized = subprocess.run(base[:2] + ["-fsanitize=address,undefined", "-fno-sanitize-recover=all"] + base[2:],
                               capture_output=True, text=True)
    if sanitized.returncode:
        plain = subprocess.run(base, capture_output=True, text=True)
        assert plain.returncode == 0, plain.stderr[-3000:]
    return exe


def run(checker, args):
    out = subprocess.run([str(checker), *map(str, args)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout.split()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


TERNARY = [(3, 2, 4, 1, 0, 148), (33, 17, 5, 3, 2, 148), (100, 40, 7, 8, 0, 148), (5, 100, 500, 17, 1, 148),
           (40, 300, 96, 2, 0, 148), (64, 21, 64, 8, 1, 1), (96, 18, 13, 5, 0, 2), (128, 40, 128, 16, 0, 1),
           (0, 5, 3, 2, 0, 148), (5, 0, 3, 2, 0, 148), (9, 2049, 5, 1, 0, 148)]


@pytest.mark.parametrize("rows,cols,group,lanes,extra,sms", TERNARY)
def test_ternary_kernel_body(checker, tmp_path, rows, cols, group, lanes, extra, sms):
    rng = np.random.default_rng(rows * 31 + cols + group)
    if rows * cols:
        data, codes, _ = random_file(rng, rows, cols, group)
    else:
        data, codes = sf.ternary_file(rows, cols, group, np.zeros(0, np.uint8), np.zeros(0, np.float32)), np.zeros(0)
    x = (rng.standard_normal((lanes, cols + extra)) * 10).astype(np.float32)
    (tmp_path / "a.spm").write_bytes(data)
    x.tofile(tmp_path / "x.bin")
    _, reserved = run(checker, ["ternary", tmp_path / "a.spm", tmp_path / "x.bin", lanes, cols + extra, sms,
                                tmp_path / "y.bin"])
    y = np.fromfile(tmp_path / "y.bin", np.float32).reshape(lanes, rows)
    np.testing.assert_array_equal(bits(y), bits(O.spm_run_gemv(data, x)))
    assert int(reserved) == int((codes == 2).sum())


DENSE = [(7, 5, 16, 1, sf.F32, 148), (33, 17, 5, 3, sf.BF16, 148), (40, 300, 96, 5, sf.F32, 148),
         (9, 2049, 64, 1, sf.BF16, 148), (64, 21, 64, 8, sf.F32, 1), (96, 18, 13, 5, sf.BF16, 2),
         (128, 40, 128, 16, sf.F32, 1), (0, 3, 4, 2, sf.F32, 148), (3, 0, 4, 2, sf.BF16, 148)]


@pytest.mark.parametrize("rows,cols,group,positions,enc,sms", DENSE)
def test_dense_kernel_body(checker, tmp_path, rows, cols, group, positions, enc, sms):
    rng = np.random.default_rng(rows * 37 + cols + group + enc)
    w = (rng.standard_normal(rows * cols) * rng.choice([1e-3, 1.0, 1e3], rows * cols)).astype(np.float32)
    x = (rng.standard_normal(positions * cols) * 10).astype(np.float32)
    data = sf.dense_file([(rows, cols)], group, [w], enc)
    (tmp_path / "a.spm").write_bytes(data)
    x.tofile(tmp_path / "x.bin")
    run(checker, ["dense", tmp_path / "a.spm", 0, tmp_path / "x.bin", positions, sms, tmp_path / "y.bin"])
    y = np.fromfile(tmp_path / "y.bin", np.float32).reshape(positions, rows)
    np.testing.assert_array_equal(bits(y), bits(O.spm_streamed(data, x, positions)))


@pytest.mark.parametrize("enc", [sf.Q8_0, sf.Q6_K, sf.Q5_K])
@pytest.mark.parametrize("rows_of", [1, 3, 12, "all"])
def test_block_kernel_body(checker, tmp_path, enc, rows_of):
    bv, bb = sf.BLOCK[enc]
    rng = np.random.default_rng(enc * 7 + (0 if rows_of == "all" else rows_of))
    blocks = bytearray(rng.integers(0, 256, 6 * bb, dtype=np.uint8).tobytes())
    for i in range(6):  # finite f16 scales, subnormal ones included
        for off in ((208,) if enc == sf.Q6_K else (0, 2) if enc == sf.Q5_K else (0,)):
            h = int(rng.choice([0x0001, 0x03ff, 0x2c00, 0x3c00, 0x8400 | int(rng.integers(0, 0x3ff))]))
            blocks[i * bb + off:i * bb + off + 2] = h.to_bytes(2, "little")
    rows = 6 * bv if rows_of == "all" else rows_of
    cols = 6 * bv // rows
    data = sf.qblock_file(rows, cols, enc, bytes(blocks))
    for positions, sms in ((1, 148), (3, 148), (8, 1)):
        x = (rng.standard_normal(positions * cols) * 4).astype(np.float32)
        (tmp_path / "a.spm").write_bytes(data)
        x.tofile(tmp_path / "x.bin")
        run(checker, ["qblock", tmp_path / "a.spm", tmp_path / "x.bin", positions, sms, tmp_path / "y.bin"])
        y = np.fromfile(tmp_path / "y.bin", np.float32).reshape(positions, rows)
        np.testing.assert_array_equal(bits(y), bits(O.spm_qblocks(data, x, positions)))
