"""The synthetic model writer, through libspmsynth.so (host code only).

Benchmarks and tests make their seeded random-init GGUF models here.  The
library holds only the encoders and the GGUF writer, so a process that must
not load the GPU engine (the CPU reference arm of bench.py) can make the same
input bytes as every other process: libspmgpu.so's spm_synth_gguf writes the
same image for the same spec.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from ._lib import SPM_OK, SpmError, SynthSpec
from .configs import Recipe

SYNTH_PATH = Path(__file__).resolve().parent / "libspmsynth.so"
_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not SYNTH_PATH.exists():
            raise ImportError(f"{SYNTH_PATH} is missing: run `python -m emufpga_b200.build`")
        h = C.CDLL(str(SYNTH_PATH))
        h.spm_synth_gguf.restype = C.c_int32
        h.spm_synth_gguf.argtypes = [C.POINTER(SynthSpec), C.POINTER(C.POINTER(C.c_uint8)), C.POINTER(C.c_uint64)]
        h.spm_last_error.restype = C.c_char_p
        h.spm_last_error.argtypes = []
        h.spm_free.restype = None
        h.spm_free.argtypes = [C.c_void_p]
        _lib = h
    return _lib


def synth_gguf(recipe: Recipe, threads: int = 0) -> np.ndarray:
    """A synthetic GGUF v3 image of `recipe` (uint8 array, copied out of the library's buffer)."""
    spec = recipe.spec(threads)
    out = C.POINTER(C.c_uint8)()
    n = C.c_uint64()
    status = lib().spm_synth_gguf(C.byref(spec), C.byref(out), C.byref(n))
    if status != SPM_OK:
        raise SpmError(status, lib().spm_last_error().decode(errors="replace"))
    try:
        arr = np.ctypeslib.as_array(out, shape=(n.value,)).copy()
    finally:
        lib().spm_free(C.cast(out, C.c_void_p))
    return arr
