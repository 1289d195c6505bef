"""Host-to-HBM streaming of a .spm file (spm_sweep_*).

The reference streams its weights from a file with a read-ahead worker
(spm-stream-file/src/prefetch.rs, PrefetchFileWeightStream) and consumes the
streams in file order with streamed()/run_gemv, rewinding between sweeps
(spm-stream-groups/src/groups.rs:88-117).  ``Sweep`` is that loop with the
device as the consumer: every stream stays packed in pinned host memory, the
device holds a ring of ``device_bytes``, and each ``next`` runs the next
stream -- dense F32/Bf16 streams as spm_linear::streamed, ternary streams as
spm_gemv_ref::run_gemv, block-profile streams as q6_operation/stream_matrix,
bit-identical to the reference -- while the streams after it are copied into
the ring.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._lib import SweepInfo, call

NEXT, REWIND = 1, 2
EVENTS, WAIT, COPY, LAUNCH, REFUSED, REWOUND = 1, 2, 3, 4, 5, 6


class Sweep:
    def __init__(self, spm, device: int = 0, device_bytes: int = 0):
        """`spm`: the file's bytes, or a path (read as PrefetchFileWeightStream::open would)."""
        h = C.c_void_p()
        if isinstance(spm, (str, os.PathLike)):
            call("spm_sweep_open_file", os.fsencode(spm), device, device_bytes, C.byref(h))
        else:
            raw = np.ascontiguousarray(np.frombuffer(bytes(spm), dtype=np.uint8))
            call("spm_sweep_open", raw.ctypes.data if raw.size else None, raw.size, device, device_bytes,
                 C.byref(h))
        self._h = h
        self.device = device
        info = self.describe()
        self.streams = info["streams"]
        self.shapes = []
        for i in range(self.streams):
            r, c, e = C.c_uint32(), C.c_uint32(), C.c_uint32()
            call("spm_sweep_stream", h, i, C.byref(r), C.byref(c), C.byref(e))
            self.shapes.append((r.value, c.value, e.value))

    def describe(self) -> dict:
        info = SweepInfo()
        call("spm_sweep_describe", self._h, C.byref(info))
        return {k: getattr(info, k) for k, _ in SweepInfo._fields_}

    def close(self) -> None:
        if getattr(self, "_h", None):
            call("spm_sweep_close", self._h)
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

    def next(self, x, positions: int, out=None, stream=None):
        """Run the next stream on `positions` activation vectors (x: a
        contiguous float32 CUDA tensor of at least positions x cols values).
        Returns (stream index, positions x rows tensor)."""
        import torch

        index = self.describe()["position"]
        if index >= self.streams:
            index = 0
        rows = self.shapes[index][0]
        if x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous float32 CUDA tensor")
        if out is None:
            out = torch.empty((positions, rows), dtype=torch.float32, device=x.device)
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        ran = C.c_int32()
        call("spm_sweep_next", self._h, x.data_ptr() or None, x.numel(), positions, out.data_ptr() or None,
             C.c_void_p(s.cuda_stream), C.byref(ran))
        return ran.value, out

    def rewind(self) -> None:
        call("spm_sweep_rewind", self._h)


def plan(region_bytes, device_bytes: int, script) -> list[tuple[int, int, int, int]]:
    """The ring schedule for `script` (NEXT / REWIND commands), computed on
    the host: (kind, stream, ring offset, event pair) records in issue order."""
    regions = (C.c_uint64 * len(region_bytes))(*region_bytes)
    cmds = (C.c_int32 * max(1, len(script)))(*script)
    n = C.c_int64()
    call("spm_sweep_plan", regions, len(region_bytes), device_bytes, cmds, len(script), None, 0, C.byref(n))
    log = (C.c_int64 * max(1, 4 * n.value))()
    call("spm_sweep_plan", regions, len(region_bytes), device_bytes, cmds, len(script), log, n.value, C.byref(n))
    flat = list(log)[: 4 * n.value]
    return [tuple(flat[i:i + 4]) for i in range(0, len(flat), 4)]
