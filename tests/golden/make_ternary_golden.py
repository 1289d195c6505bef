"""Writes tests/golden/tiny_ternary.spm from the documented .spm layout.

The bytes are assembled field by field from the format description the
reference's spm-file/tests/golden.rs:33-87 checks against (a 3x2 ternary
matrix, scale groups of 4: one group of four weights, scale 1.0, codes
+, 0, -, +; then a short group of two, scale 0.5, codes -, 0), not by the
writer under test, so the fixture and the writer are two readings of one
specification.

    python tests/golden/make_ternary_golden.py
"""
import struct
from pathlib import Path

OUT = Path(__file__).resolve().parent / "tiny_ternary.spm"


def tiny() -> bytes:
    header = bytes([0x89, 0x53, 0x50, 0x4D, 0x0D, 0x0A, 0x1A, 0x0A])  # magic
    header += struct.pack("<HH", 1, 0)                                # version 1.0
    header += bytes([0, 0, 0, 0])                                     # little-endian, reserved
    header += struct.pack("<I", 1) + bytes(12)                        # one stream, reserved
    desc = struct.pack("<III", 3, 2, 4) + bytes([1, 0]) + struct.pack("<H", 1) + bytes(16)
    g0 = struct.pack("<f", 1.0) + bytes([0b01_11_00_01])              # +, 0, -, + (LSB pair first)
    g1 = struct.pack("<f", 0.5) + bytes([0b00_11])                    # -, 0; padding bits zero
    return header + desc + g0 + g1


if __name__ == "__main__":
    OUT.write_bytes(tiny())
    print(OUT, len(tiny()), "bytes")
