"""Regenerates tests/golden/blocks.npz: GGML block fixtures and their decoded
values from gguf-py (the GGUF format's own Python package, 0.19.0 in this
image), the independent decoder the oracle and the device decoders are pinned
against.  Run from the repo root:

    python tests/golden/make_golden.py

Fixtures per block type:
  * the q6-pipeline transport fixture of the reference
    (components/fabric/crates/q6-pipeline/tests/pipeline.rs:11-20: byte i is
    (i % 256) * 73 + 19, wrapping), three blocks, which the reference checks
    against its own Q6_K decoder;
  * 64 blocks of seeded random bytes whose fp16 scale fields are replaced by
    finite values (normal, subnormal, zero and negative halves included).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf.quants import dequantize

OUT = Path(__file__).resolve().parent / "blocks.npz"

TYPES = {"q8_0": (T.Q8_0, 34, [0]), "q6_k": (T.Q6_K, 210, [208]), "q5_k": (T.Q5_K, 176, [0, 2]),
         "q2_k": (T.Q2_K, 84, [80, 82])}


def finite_halves(rng: np.random.Generator, n: int) -> np.ndarray:
    """fp16 bit patterns with exponent < 31: normals, subnormals, zeros, both signs."""
    exp = rng.integers(0, 31, size=n, dtype=np.uint16)
    exp[::7] = 0                      # subnormals and zeros
    frac = rng.integers(0, 1024, size=n, dtype=np.uint16)
    frac[::13] = 0
    sign = rng.integers(0, 2, size=n, dtype=np.uint16) << 15
    # keep magnitudes moderate so products stay finite: exponent in [0, 20]
    exp = np.minimum(exp, 20)
    return (sign | (exp << 10) | frac).astype(np.uint16)


def main() -> None:
    rng = np.random.default_rng(20261201)
    arrays = {}
    pipeline = np.array([((i % 256) * 73 + 19) & 0xFF for i in range(3 * 210)], dtype=np.uint8)
    arrays["q6_k_pipeline"] = pipeline
    arrays["q6_k_pipeline_out"] = dequantize(pipeline, T.Q6_K).astype(np.float32).reshape(-1)
    for name, (qt, bb, dpos) in TYPES.items():
        nblk = 64
        raw = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
        for p in dpos:
            h = finite_halves(rng, nblk)
            raw[:, p:p + 2] = h.view(np.uint8).reshape(nblk, 2)
        flat = raw.reshape(-1).copy()
        arrays[name] = flat
        arrays[name + "_out"] = dequantize(flat, qt).astype(np.float32).reshape(-1)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({', '.join(sorted(arrays))})")


if __name__ == "__main__":
    main()
