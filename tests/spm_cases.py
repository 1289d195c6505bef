"""Seeded .spm test cases, as the reference's tests draw them.

Ternary cases:

Restates spm-vectors/src/draw.rs and generate.rs: an xorshift64 state
(seed | 1; s ^= s << 13, s ^= s >> 7, s ^= s << 17), weights drawn first
(state % 3: 0 -> zero, 1 -> +1, 2 -> -1), then one scale per group
(k / 16 + 0.0625, k = state % 32), then one activation per column
(k / 16 - 2.0, k = state % 64).  Sixteenths are exact in f32, so these cases
add no rounding of their own.  Also the f64 reference of spm-numeric
(src/matmul.rs:38-48) that the reference's correctness test compares against.

Dense cases: the weights of spm-linear/tests/agreement.rs:17-31, the same
xorshift64 with values state % 64 / 16 - 2.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from emufpga_b200 import spmfile as sf

MASK = (1 << 64) - 1


def _next(s: int) -> int:
    s ^= (s << 13) & MASK
    s ^= s >> 7
    s ^= (s << 17) & MASK
    return s


@dataclasses.dataclass
class Case:
    seed: int
    rows: int
    cols: int
    group_size: int
    weights: np.ndarray      # -1/0/+1 in stream order (column-major)
    scales: np.ndarray       # f32, one per group
    activations: np.ndarray  # f32, one per column

    def spm(self) -> bytes:
        return sf.ternary_file(self.rows, self.cols, self.group_size, sf.ternary_codes(self.weights), self.scales)


def generate(seed: int, rows: int, cols: int, group_size: int) -> Case:
    total = rows * cols
    groups = -(-total // max(group_size, 1))
    state = seed | 1
    weights = np.empty(total, np.int8)
    for i in range(total):
        state = _next(state)
        weights[i] = (0, 1, -1)[state % 3]

    def fractions(count: int, span: int, offset: float) -> np.ndarray:
        nonlocal state
        out = np.empty(count, np.float32)
        for i in range(count):
            state = _next(state)
            out[i] = np.float32(state % max(span, 1)) / np.float32(16.0) + np.float32(offset)
        return out

    scales = fractions(groups, 32, 0.0625)
    activations = fractions(cols, 64, -2.0)
    return Case(seed, rows, cols, group_size, weights, scales, activations)


def reference_gemv(case: Case) -> np.ndarray:
    """f64 reference: out[row] += w * scale * x[col] over stream positions."""
    out = np.zeros(case.rows, np.float64)
    for index, w in enumerate(case.weights):
        scale = float(case.scales[index // case.group_size])
        out[index % case.rows] += float(w) * scale * float(case.activations[index // case.rows])
    return out


def random_file(rng: np.random.Generator, rows: int, cols: int, group: int, reserved: float = 0.03):
    """A ternary file with f32 scales spread over six decades (results are not
    exact in f32, so only the reference's order of additions reproduces them)
    and a share of reserved 0b10 codes."""
    total = rows * cols
    p = rng.random(total)
    codes = np.where(p < 0.3, 0, np.where(p < 0.6, 1, np.where(p < 1.0 - reserved, 3, 2))).astype(np.uint8)
    groups = -(-total // group)
    scales = (rng.standard_normal(groups) * rng.choice([1e-3, 1.0, 1e3], groups)).astype(np.float32)
    return sf.ternary_file(rows, cols, group, codes, scales), codes, scales


def sixteenths(seed: int, count: int) -> np.ndarray:
    """spm-linear/tests/agreement.rs weights(seed, count)."""
    state = seed | 1
    out = np.empty(count, np.float32)
    for i in range(count):
        state = _next(state)
        out[i] = np.float32(state % 64) / np.float32(16.0) - np.float32(2.0)
    return out
