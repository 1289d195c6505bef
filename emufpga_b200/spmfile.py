""".spm files: writing them, and the ternary code packing.

The container of spm-file/src/write.rs: a 32-byte header
(spm-header/src/lib.rs:3-25: magic, version 1.0, little-endian, stream
count), one 32-byte descriptor per stream (spm-layout/src/lib.rs:3-16: rows,
cols, group_size, encoding profile, lane_count), then every stream's scale
groups in stream order, each an f32 scale followed by its payload.  Stream
position k of a matrix holds W[k % rows][k / rows] (column-major); a group
covers `group_size` consecutive positions and the last one is short.

Ternary payloads (spm-codec/src/lib.rs:1-31) pack four weights to a byte,
least significant pair first: code 00 = 0, 01 = +1, 11 = -1 (10 is reserved);
a short group's final byte is zero-padded.  Dense payloads are little-endian
f32, or bf16 rounded to nearest even (spm-codec-bf16/src/convert.rs), behind
the inert scale 1.0.

Reading is done by the library (spm_file_probe / spm_file_stream,
spm_ternary_upload, spm_dense_upload); this module only builds files.
"""
from __future__ import annotations

import struct
from typing import Sequence

import numpy as np

MAGIC = bytes([0x89, ord("S"), ord("P"), ord("M"), 0x0D, 0x0A, 0x1A, 0x0A])
HEADER_LEN = DESCRIPTOR_LEN = 32
VERSION_MAJOR, VERSION_MINOR = 1, 0

# Encoding profile codes (spm-layout/src/model.rs Encoding::code).
TERNARY, F32, BF16, Q6_K, Q5_K, Q8_0 = 1, 2, 3, 4, 5, 6
CODE = {0: 0b00, 1: 0b01, -1: 0b11}


def bytes_for(encoding: int, count: int) -> int:
    """Wire bytes of a group of `count` weights (Encoding::bytes_for)."""
    if encoding == TERNARY:
        return (count + 3) // 4
    if encoding == F32:
        return count * 4
    if encoding == BF16:
        return count * 2
    if encoding == Q6_K:
        return (count + 255) // 256 * 210
    if encoding == Q5_K:
        return (count + 255) // 256 * 176
    if encoding == Q8_0:
        return (count + 31) // 32 * 34
    raise ValueError(f"unknown .spm encoding profile {encoding}")


def render_header(stream_count: int) -> bytes:
    return MAGIC + struct.pack("<HHB3xI12x", VERSION_MAJOR, VERSION_MINOR, 0, stream_count)


def render_descriptor(rows: int, cols: int, group_size: int, encoding: int = TERNARY, lane_count: int = 1) -> bytes:
    return struct.pack("<IIIBxH16x", rows, cols, group_size, encoding, lane_count)


def group_lengths(rows: int, cols: int, group_size: int) -> list[int]:
    """Weights in each group of one stream (spm-layout/src/tiling.rs group_len)."""
    total = rows * cols
    full, rem = divmod(total, group_size)
    return [group_size] * full + ([rem] if rem else [])


def pack_codes(codes: np.ndarray) -> bytes:
    """Pack 2-bit codes four to a byte, least significant pair first."""
    codes = np.asarray(codes, dtype=np.uint8) & 3
    pad = (-codes.size) % 4
    if pad:
        codes = np.concatenate([codes, np.zeros(pad, np.uint8)])
    q = codes.reshape(-1, 4)
    return (q[:, 0] | (q[:, 1] << 2) | (q[:, 2] << 4) | (q[:, 3] << 6)).astype(np.uint8).tobytes()


def ternary_codes(weights: Sequence[int] | np.ndarray) -> np.ndarray:
    """-1/0/+1 values -> 2-bit codes; anything else is refused (Ternary::from_value)."""
    w = np.asarray(weights)
    if w.size and not np.isin(w, (-1, 0, 1)).all():
        bad = w[~np.isin(w, (-1, 0, 1))].flat[0]
        raise ValueError(f"value {int(bad)} is not ternary (expected -1, 0 or 1)")
    return np.where(w == 0, 0, np.where(w > 0, 0b01, 0b11)).astype(np.uint8)


class SpmWriter:
    """Builds a .spm file group by group, in stream order (SpmWriter,
    spm-file/src/write.rs:15-108): the header and directory first, then each
    group's scale and payload; a group of the wrong length or past the last
    stream is refused, and finish() refuses a file with groups still owed."""

    def __init__(self, descriptors: Sequence[tuple]):
        """descriptors: (rows, cols, group_size[, encoding[, lane_count]]) per stream."""
        self.descriptors = [tuple(d) + (TERNARY, 1)[len(d) - 3:] for d in descriptors]
        for d in self.descriptors:
            if d[2] < 1:
                raise ValueError("group_size must be at least 1")
        self._out = bytearray(render_header(len(self.descriptors)))
        for d in self.descriptors:
            self._out += render_descriptor(*d)
        self._plan = [(s, n) for s, d in enumerate(self.descriptors) for n in group_lengths(d[0], d[1], d[2])]
        self._next = 0

    def _stream(self) -> int:
        return self._plan[self._next][0] if self._next < len(self._plan) else len(self.descriptors)

    def write_group(self, scale: float, weights: Sequence[int] | np.ndarray) -> None:
        """Append one ternary group (values -1/0/+1)."""
        codes = ternary_codes(weights)
        self.write_raw_group(scale, pack_codes(codes), codes.size)

    def write_raw_group(self, scale: float, payload: bytes, count: int) -> None:
        if self._next >= len(self._plan):
            raise ValueError(f"only {self._stream()} of {len(self.descriptors)} streams were written")
        stream, expected = self._plan[self._next]
        if count != expected or len(payload) != bytes_for(self.descriptors[stream][3], count):
            raise ValueError(f"group expects {expected} weights, got {count}")
        self._out += struct.pack("<f", scale) + bytes(payload)
        self._next += 1

    def finish(self) -> bytes:
        if self._next != len(self._plan):
            raise ValueError(f"only {self._stream()} of {len(self.descriptors)} streams were written")
        return bytes(self._out)


def ternary_stream_bytes(codes: np.ndarray, scales: np.ndarray, group_size: int) -> bytes:
    """The groups of one ternary stream: codes in stream order (uint8 2-bit
    codes, reserved 0b10 allowed), one f32 scale per group."""
    codes = np.asarray(codes, dtype=np.uint8).ravel()
    scales = np.asarray(scales, dtype="<f4").ravel()
    total = codes.size
    full, rem = divmod(total, group_size)
    if scales.size != full + (1 if rem else 0):
        raise ValueError("one scale per group is needed")
    parts = []
    if full:
        per = bytes_for(TERNARY, group_size)
        body = codes[: full * group_size].reshape(full, group_size)
        if group_size % 4:
            body = np.concatenate([body, np.zeros((full, per * 4 - group_size), np.uint8)], axis=1)
        q = body.reshape(full, per, 4)
        packed = (q[..., 0] | (q[..., 1] << 2) | (q[..., 2] << 4) | (q[..., 3] << 6)).astype(np.uint8)
        rec = np.empty((full, 4 + per), np.uint8)
        rec[:, :4] = scales[:full].view(np.uint8).reshape(full, 4)
        rec[:, 4:] = packed
        parts.append(rec.tobytes())
    if rem:
        parts.append(struct.pack("<f", float(scales[full])) + pack_codes(codes[full * group_size:]))
    return b"".join(parts)


def bf16_round(values) -> np.ndarray:
    """f32 -> bf16 bits, round to nearest even; NaN stays a quiet NaN
    (spm-codec-bf16/src/convert.rs round)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    out = (((bits + 0x7FFF + lsb) & 0xFFFFFFFF) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(values, dtype=np.float32))
    out[nan] = ((bits[nan] >> 16) | 0x0040).astype(np.uint16)
    return out


def dense_stream_bytes(weights: np.ndarray, group_size: int, encoding: int = F32) -> bytes:
    """The groups of one dense stream: f32 weights in stream order (column-
    major), framed with the inert scale 1.0, stored as f32 or rounded to bf16."""
    w = np.ascontiguousarray(weights, dtype=np.float32).ravel()
    if encoding == F32:
        payload = w.astype("<f4").view(np.uint8)
        es = 4
    elif encoding == BF16:
        payload = bf16_round(w).astype("<u2").view(np.uint8)
        es = 2
    else:
        raise ValueError("dense streams are F32 or BF16")
    one = struct.pack("<f", 1.0)
    parts = []
    for start in range(0, w.size, group_size):
        n = min(group_size, w.size - start)
        parts.append(one + payload[start * es:(start + n) * es].tobytes())
    return b"".join(parts)


def dense_file(shapes: Sequence[tuple[int, int]], group_size: int, matrices: Sequence[np.ndarray],
               encoding: int = F32) -> bytes:
    """A .spm file of dense streams, one per (rows, cols) shape, each matrix
    given in stream order."""
    out = render_header(len(shapes))
    for rows, cols in shapes:
        out += render_descriptor(rows, cols, group_size, encoding)
    for m in matrices:
        out += dense_stream_bytes(m, group_size, encoding)
    return out


BLOCK = {Q8_0: (32, 34), Q6_K: (256, 210), Q5_K: (256, 176)}


def qblock_stream_bytes(blocks: bytes, encoding: int) -> bytes:
    """The groups of one block-profile stream: one GGML block per group
    (source row-major order), each behind the inert scale 1.0."""
    _, bb = BLOCK[encoding]
    if len(blocks) % bb:
        raise ValueError("not a whole number of blocks")
    one = struct.pack("<f", 1.0)
    return b"".join(one + blocks[i:i + bb] for i in range(0, len(blocks), bb))


def qblock_file(rows: int, cols: int, encoding: int, blocks: bytes) -> bytes:
    """A one-stream .spm file of GGML blocks (rows x cols values, row-major)."""
    bv, bb = BLOCK[encoding]
    if rows * cols != len(blocks) // bb * bv:
        raise ValueError("rows x cols must be the blocks' value count")
    return render_header(1) + render_descriptor(rows, cols, bv, encoding) + qblock_stream_bytes(blocks, encoding)


def ternary_file(rows: int, cols: int, group_size: int, codes: np.ndarray, scales: np.ndarray,
                 lane_count: int = 1) -> bytes:
    """A one-stream ternary .spm file (codes in stream order)."""
    return (render_header(1) + render_descriptor(rows, cols, group_size, TERNARY, lane_count)
            + ternary_stream_bytes(codes, scales, group_size))
