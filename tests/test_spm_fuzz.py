"""Mutated and truncated .spm files: the library's host reader and the
oracle's reach the same verdict, and stream placement matches an
independent computation from the format's rules.

The reference's reader refuses a file at the first thing it cannot read
(spm-header/src/parse.rs, spm-layout/src/wire.rs, spm-file/src/read.rs);
both readers here follow the same order, so the same bytes must give the
same error kind, and a file both accept must place every stream at the
same offset.
"""
import struct

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import spmfile as sf
from emufpga_b200 import ternary as T
from oracle import oracle as O


def three_streams(rng):
    w = sf.SpmWriter([(9, 7, 5), (4, 6, 8, sf.F32), (5, 3, 4, sf.BF16)])
    for n in sf.group_lengths(9, 7, 5):
        w.write_group(float(rng.standard_normal()), rng.integers(-1, 2, n))
    for n in sf.group_lengths(4, 6, 8):
        w.write_raw_group(1.0, rng.standard_normal(n).astype("<f4").tobytes(), n)
    for n in sf.group_lengths(5, 3, 4):
        w.write_raw_group(1.0, sf.bf16_round(rng.standard_normal(n)).astype("<u2").tobytes(), n)
    return w.finish()


def placement(data):
    """(offset, bytes) of every stream from the descriptors, by the format's rules."""
    n = struct.unpack_from("<I", data, 16)[0]
    at = 32 + 32 * n
    out = []
    for i in range(n):
        rows, cols, group, enc = struct.unpack_from("<IIIB", data, 32 + 32 * i)
        full, rem = divmod(rows * cols, group)
        size = full * (4 + sf.bytes_for(enc, group)) + (4 + sf.bytes_for(enc, rem) if rem else 0)
        out.append((at, size))
        at += size
    return out


def library(fn, *args):
    try:
        return 0, fn(*args)
    except eb.SpmError as e:
        return e.code, None


def oracle_describe(data):
    try:
        return 0, O.spm_describe(data)
    except O.SpmError as e:
        return e.code, None


@pytest.mark.parametrize("seed", range(12))
def test_header_and_directory_mutations_get_the_same_verdict(seed):
    rng = np.random.default_rng(seed)
    good = three_streams(rng)
    for _ in range(40):
        b = bytearray(good)
        for _ in range(int(rng.integers(1, 4))):
            b[int(rng.integers(0, 128))] = int(rng.integers(0, 256))  # header and the three descriptors
        data = bytes(b)
        code, probe = library(T.file_probe, data)
        ocode, desc = oracle_describe(data)
        assert code == ocode, (code, ocode)
        if code == 0:
            assert probe[2] == desc["streams"]
            # every stream is placed where the (mutated) descriptors put it,
            # or refused as truncated when the file ends before it does
            for i, (off, size) in enumerate(placement(data)):
                got = library(T.file_stream, data, i)
                if off + size <= len(data):
                    assert got[0] == 0 and (got[1].offset, got[1].bytes) == (off, size)
                else:
                    assert got[0] == -3


@pytest.mark.parametrize("seed", range(4))
def test_truncations_fail_at_the_stream_they_cut(seed):
    rng = np.random.default_rng(100 + seed)
    good = three_streams(rng)
    places = placement(good)
    for cut in sorted(set(rng.integers(0, len(good), 60).tolist()) | {len(good) - 1, 96, 127, 128}):
        data = good[:cut]
        code, _ = library(T.file_probe, data)
        ocode, _ = oracle_describe(data)
        assert code == ocode
        if code:
            continue
        for i, (off, size) in enumerate(places):
            got = library(T.file_stream, data, i)
            if off + size <= cut:
                assert got[0] == 0 and (got[1].offset, got[1].bytes) == (off, size)
            else:
                assert got[0] == -3  # payload truncated in this stream or an earlier one


def test_intact_files_are_placed_as_the_format_says():
    rng = np.random.default_rng(7)
    data = three_streams(rng)
    for i, (off, size) in enumerate(placement(data)):
        st = T.file_stream(data, i)
        assert (st.offset, st.bytes) == (off, size)
