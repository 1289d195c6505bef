"""The ternary GEMV of spm-gemv-ref on the device.

Mirrors the public face of spm_gemv_ref (spm-gemv-ref/src/lib.rs:45-49):
``Activations`` (spm-activations/src/activations.rs), ``run_gemv`` returning
a ``GemvOutcome`` with the accumulator ``bank`` (spm-accum/src/bank.rs: one
bank of ``rows`` accumulators per lane, ``lane(i)``) and the scan counters of
ScanMetrics (spm-stream-metrics/src/model.rs).  Errors are raised in the
reference's order: header and directory, no streams, missing activations,
then a payload that ends early.

The arithmetic runs in libspmgpu.so (spm_ternary_*): every output is
bit-identical to the reference's sequential f32 accumulation.  The whole
stream is resident in HBM, so ``resident_parameter_bytes`` is the device
footprint rather than the reference's one-group buffer, and the timing
fields of ScanMetrics are not reported.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import struct

import numpy as np

from ._lib import FileStreamInfo, SpmError, TernaryInfo, call

SPM_E_ARG, SPM_E_ACTIVATION_LEN = -1, -2


def _buf(spm) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(spm), dtype=np.uint8))


def _ptr(a: np.ndarray) -> int | None:
    return a.ctypes.data if a.size else None


@dataclasses.dataclass(frozen=True)
class FileStream:
    """One stream of a .spm file: its descriptor and where its groups lie."""
    rows: int
    cols: int
    group_size: int
    encoding: int
    lane_count: int
    groups: int
    offset: int
    bytes: int


def file_probe(spm) -> tuple[int, int, int]:
    """(version_major, version_minor, stream count); raises on a bad header or directory."""
    raw = _buf(spm)
    major, minor, n = C.c_uint32(), C.c_uint32(), C.c_int32()
    call("spm_file_probe", _ptr(raw), raw.size, C.byref(major), C.byref(minor), C.byref(n))
    return major.value, minor.value, n.value


def file_stream(spm, index: int = 0) -> FileStream:
    """Descriptor and placement of stream `index`; every group up to its end must be whole."""
    raw = _buf(spm)
    info = FileStreamInfo()
    call("spm_file_stream", _ptr(raw), raw.size, index, C.byref(info))
    return FileStream(info.rows, info.cols, info.group_size, info.encoding, info.lane_count, info.groups,
                      info.offset, info.bytes)


class Activations:
    """One activation vector per batch lane (lane-major)."""

    def __init__(self, lanes: int, cols: int, values):
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        if v.size != lanes * cols:
            raise ValueError(f"{lanes} lanes x {cols} activations needs {lanes * cols} values, got {v.size}")
        self.lanes, self.cols = lanes, cols
        self.values = v.reshape(lanes, cols)

    @classmethod
    def broadcast(cls, lanes: int, values) -> "Activations":
        """`lanes` copies of one vector (Activations::broadcast)."""
        v = np.asarray(values, dtype=np.float32).reshape(-1)
        return cls(lanes, v.size, np.tile(v, lanes))

    @classmethod
    def per_lane(cls, lanes: int, cols: int, values) -> "Activations":
        """A distinct vector per lane, lane-major (Activations::per_lane)."""
        return cls(lanes, cols, values)


@dataclasses.dataclass
class AccumulatorBank:
    """`lanes` banks of `rows` accumulators; data is lanes x rows."""
    lanes: int
    rows: int
    data: np.ndarray

    def lane(self, lane: int) -> np.ndarray:
        if not 0 <= lane < self.lanes:
            raise IndexError(f"lane {lane} out of range")
        return self.data[lane].copy()

    def __eq__(self, other) -> bool:
        return (isinstance(other, AccumulatorBank) and self.lanes == other.lanes and self.rows == other.rows
                and np.array_equal(self.data.view(np.uint32), other.data.view(np.uint32)))


@dataclasses.dataclass(frozen=True)
class ScanMetrics:
    parameter_bytes_read: int       # packed weight bytes of the stream (scales excluded)
    weights_decoded: int            # every weight, zeros included
    weight_applications: int        # weights x lanes
    resident_parameter_bytes: int   # HBM held by the packed stream
    total_parameter_bytes: int      # rows x cols / 4, rounded up

    def scan_productivity(self) -> float | None:
        return self.weight_applications / self.weights_decoded if self.weights_decoded else None

    def residency(self) -> float | None:
        return self.resident_parameter_bytes / self.total_parameter_bytes if self.total_parameter_bytes else None


@dataclasses.dataclass
class GemvOutcome:
    bank: AccumulatorBank
    metrics: ScanMetrics


class TernaryMatrix:
    """One ternary stream of a .spm file, packed in HBM (spm_ternary_upload)."""

    def __init__(self, spm, index: int = 0, device: int = 0):
        raw = _buf(spm)
        h = C.c_void_p()
        call("spm_ternary_upload", _ptr(raw), raw.size, index, device, C.byref(h))
        self._h = h
        self.device = device
        info = TernaryInfo()
        call("spm_ternary_describe", h, C.byref(info))
        self.rows, self.cols, self.group_size = info.rows, info.cols, info.group_size
        self.groups, self.payload_bytes = info.groups, info.payload_bytes
        self.reserved_codes, self.device_bytes = info.reserved_codes, info.device_bytes

    def close(self) -> None:
        if getattr(self, "_h", None):
            call("spm_ternary_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def gemv(self, x, out=None, stream=None):
        """y = W x on the device: x is a contiguous float32 CUDA tensor of
        lanes x x_cols (x_cols >= cols), the result lanes x rows."""
        import torch

        if x.dim() != 2 or x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous float32 CUDA tensor of lanes x cols")
        lanes, x_cols = x.shape
        if out is None:
            out = torch.empty((lanes, self.rows), dtype=torch.float32, device=x.device)
        elif tuple(out.shape) != (lanes, self.rows) or not out.is_contiguous() or out.dtype != torch.float32:
            raise ValueError("out must be a contiguous float32 tensor of lanes x rows")
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        call("spm_ternary_gemv", self._h, x.data_ptr() or None, lanes, x_cols, out.data_ptr() or None,
             C.c_void_p(s.cuda_stream))
        return out


def run_gemv(spm, activations: Activations, device: int = 0) -> GemvOutcome:
    """Runs the first stream of `spm` against `activations`
    (spm_gemv_ref::run_gemv, spm-gemv-ref/src/gemv.rs:39-57)."""
    import torch

    _, _, streams = file_probe(spm)
    if streams == 0:
        raise SpmError(SPM_E_ARG, "parameter stream declares no operations")
    raw = bytes(spm)
    rows, cols, group = struct.unpack_from("<III", raw, 32)
    if activations.cols < cols:
        raise SpmError(SPM_E_ACTIVATION_LEN, f"need {cols} activations per lane, got {activations.cols}")
    with TernaryMatrix(raw, 0, device) as m:
        x = torch.from_numpy(activations.values).to(f"cuda:{device}")
        y = m.gemv(x)
        bank = y.cpu().numpy()
        weights = rows * cols
        metrics = ScanMetrics(m.payload_bytes, weights, weights * activations.lanes, m.device_bytes,
                              (weights + 3) // 4)
    return GemvOutcome(AccumulatorBank(activations.lanes, rows, bank), metrics)
