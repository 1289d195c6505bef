"""The synthetic model writer, through libspmsynth.so (host code only).

Benchmarks and tests make their seeded random-init GGUF models here.  The
library holds only the encoders and the GGUF writer, so the same input bytes
can be made without the GPU engine: libspmgpu.so's spm_synth_gguf writes the
same image for the same spec.  Run as a module it writes a workload's model
to a file, which is how the CPU reference arm of bench.py gets its input
without loading either library itself.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
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


def _with_image(recipe: Recipe, threads: int, use):
    """Calls use(image) on the library's buffer (a uint8 view), then frees it."""
    spec = recipe.spec(threads)
    out = C.POINTER(C.c_uint8)()
    n = C.c_uint64()
    status = lib().spm_synth_gguf(C.byref(spec), C.byref(out), C.byref(n))
    if status != SPM_OK:
        raise SpmError(status, lib().spm_last_error().decode(errors="replace"))
    try:
        return use(np.ctypeslib.as_array(out, shape=(n.value,)))
    finally:
        lib().spm_free(C.cast(out, C.c_void_p))


def synth_gguf(recipe: Recipe, threads: int = 0) -> np.ndarray:
    """A synthetic GGUF v3 image of `recipe` (uint8 array, copied out of the library's buffer)."""
    return _with_image(recipe, threads, lambda view: view.copy())


def write_gguf(recipe: Recipe, path: str, threads: int = 0) -> int:
    """Writes synth_gguf(recipe) to `path` (through `path`.part, then a
    rename); returns its size in bytes."""
    part = f"{path}.part"

    def write(view):
        view.tofile(part)
        return int(view.size)

    size = _with_image(recipe, threads, write)
    os.replace(part, path)
    return size


def main(argv: list[str]) -> int:
    """python -m emufpga_b200.synth WORKLOAD PATH: writes the workload's
    synthetic GGUF to PATH, so that a process which loads neither engine
    library can read the same bytes."""
    from .configs import RECIPES, WORKLOADS

    if len(argv) != 2 or argv[0] not in WORKLOADS:
        print("usage: python -m emufpga_b200.synth WORKLOAD PATH", file=sys.stderr)
        return 2
    write_gguf(RECIPES[WORKLOADS[argv[0]]["recipe"]], argv[1])
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
