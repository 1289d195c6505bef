"""spm_dequant_rows_static, the entry point that allocates no device memory,
against spm_dequant_rows, through the C ABI.

It exists for callers that cannot allocate device memory (a hook beside a
session that holds the rest of HBM, or one that must not add the device-wide
synchronisation of cudaMalloc/cudaFree).  This file is collected last, so a
run that stops at its first failure has run every other test before it; it
also passes alone in a fresh process.  The bar is the dequantization bar:
bit-exact, on two calls in a row.
"""
import ctypes as C
import dataclasses

import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import _lib, configs

pytestmark = pytest.mark.gpu

STATIC_FLOATS = 1 << 20  # the buffer's stated limit, in floats


def _rows(fn, model, index, row0, rows, cols):
    out = np.full(rows * cols, np.nan, dtype=np.float32)
    status = getattr(_lib.lib(), fn)(model._h, index, row0, rows, out.ctypes.data_as(C.POINTER(C.c_float)))
    return status, out


@pytest.fixture(scope="module")
def model():
    # vocab 8192 x hidden 256: a 2 Mi-float embedding, larger than the buffer
    base = configs.TINY["qwen3-q6_k"]
    r = base.replace(shape=dataclasses.replace(base.shape, vocab=8192), embed_type=_lib.Q8_0)
    m = eb.Model(eb.synth_gguf(r), r.shape)
    yield m
    m.close()


def test_static_dequant_matches_the_allocating_entry_point(cuda, model):
    for index in range(model.stream_count):
        info = model.stream_info(index)
        rows, cols = info["rows"], info["cols"]
        take = min(rows, STATIC_FLOATS // cols, 1000)
        row0 = (rows - take) // 2
        st, want = _rows("spm_dequant_rows", model, index, row0, take, cols)
        assert st == 0
        for _ in range(2):
            st, got = _rows("spm_dequant_rows_static", model, index, row0, take, cols)
            assert st == 0, _lib.lib().spm_last_error()
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), index


def test_static_dequant_fills_the_buffer_and_refuses_more(cuda, model):
    index = model.stream_index("token_embd.weight")
    info = model.stream_info(index)
    cols = info["cols"]
    full = STATIC_FLOATS // cols
    assert info["rows"] > full
    st, want = _rows("spm_dequant_rows", model, index, 1, full, cols)
    assert st == 0
    for _ in range(2):
        st, got = _rows("spm_dequant_rows_static", model, index, 1, full, cols)
        assert st == 0
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    st, _ = _rows("spm_dequant_rows_static", model, index, 0, full + 1, cols)
    assert _lib.STATUS[st] == "SPM_E_ARG"
    assert b"exceeds the static buffer" in _lib.lib().spm_last_error()
