"""The block profiles of .spm files (Q8_0, Q6K, Q5K) as the reference's block
consumers compute them, on the device.

Mirrors q6_operation (spm-granite-moe/src/layout.rs:208-242) and
stream_matrix (gemma_smoke.rs:201-236): each group is one GGML block in
source row-major order, value k is W[k / cols][k % cols], and every input
accumulates out = fma(w, x, out) over the values in order -- bit-identical
here.  The inputs are a list of activation vectors, the outputs one vector
per input, as in the reference.  This is the parity form of these profiles;
the fast GEMV over GGML blocks is the GGUF model path.
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from ._lib import DenseInfo, call


class QBlockMatrix:
    """One block-profile stream of a .spm file, in HBM (spm_qblocks_upload)."""

    def __init__(self, spm, index: int = 0, device: int = 0):
        raw = np.ascontiguousarray(np.frombuffer(bytes(spm), dtype=np.uint8))
        h = C.c_void_p()
        call("spm_qblocks_upload", raw.ctypes.data if raw.size else None, raw.size, index, device, C.byref(h))
        self._h = h
        self.device = device
        info = DenseInfo()
        call("spm_qblocks_describe", h, C.byref(info))
        self.rows, self.cols, self.group_size, self.encoding = info.rows, info.cols, info.group_size, info.encoding
        self.groups, self.payload_bytes, self.device_bytes = info.groups, info.payload_bytes, info.device_bytes

    def close(self) -> None:
        if getattr(self, "_h", None):
            call("spm_qblocks_free", self._h)
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

    def gemv(self, x, positions: int, out=None, stream=None):
        """x: contiguous float32 CUDA tensor of at least positions x cols
        values; returns positions x rows."""
        import torch

        if x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous float32 CUDA tensor")
        if out is None:
            out = torch.empty((positions, self.rows), dtype=torch.float32, device=x.device)
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        call("spm_qblocks_gemv", self._h, x.data_ptr() or None, x.numel(), positions, out.data_ptr() or None,
             C.c_void_p(s.cuda_stream))
        return out


def q_operation(spm, index: int, inputs: Sequence[np.ndarray], device: int = 0) -> list[np.ndarray]:
    """q6_operation / stream_matrix for stream `index`: one output vector per input."""
    import torch

    with QBlockMatrix(spm, index, device) as m:
        if not len(inputs):
            return []
        x = np.ascontiguousarray(np.stack([np.asarray(v, np.float32)[: m.cols] for v in inputs]))
        y = m.gemv(torch.from_numpy(x.ravel()).to(f"cuda:{device}"), len(inputs)).cpu().numpy()
        return [y[i].copy() for i in range(len(inputs))]
