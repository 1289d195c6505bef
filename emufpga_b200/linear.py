"""spm_linear's streamed GEMV for the dense .spm profiles, on the device.

Mirrors spm_linear::streamed (spm-linear/src/stream.rs:31-55): one F32 or
Bf16 stream of a .spm file times a batch of activation vectors, with
results bit-identical to the reference's (y[p][r] is the chain of fused
multiply-adds over the columns in order, from +0).  The reference pulls the
next stream off a forward-only reader; here a stream is named by its index
and its shape comes from its descriptor.  Errors keep the reference's kinds:
too few activations is ``SPM_E_ACTIVATION_LEN`` ("need N activations, got
M"), a profile without a dense decoder is ``SPM_E_STREAM`` ("parameter
stream: Q6K needs a scale-aware engine").
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import DenseInfo, call


def _buf(spm) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(spm), dtype=np.uint8))


class DenseMatrix:
    """One dense stream of a .spm file, packed in HBM (spm_dense_upload)."""

    def __init__(self, spm, index: int = 0, device: int = 0):
        raw = _buf(spm)
        h = C.c_void_p()
        call("spm_dense_upload", raw.ctypes.data if raw.size else None, raw.size, index, device, C.byref(h))
        self._h = h
        self.device = device
        info = DenseInfo()
        call("spm_dense_describe", h, C.byref(info))
        self.rows, self.cols, self.group_size, self.encoding = info.rows, info.cols, info.group_size, info.encoding
        self.groups, self.payload_bytes, self.device_bytes = info.groups, info.payload_bytes, info.device_bytes

    def close(self) -> None:
        if getattr(self, "_h", None):
            call("spm_dense_free", self._h)
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

    def streamed(self, x, positions: int, out=None, stream=None):
        """y = W x for `positions` activation vectors: x is a contiguous
        float32 CUDA tensor holding at least positions x cols values; the
        result is positions x rows."""
        import torch

        if x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous float32 CUDA tensor")
        if out is None:
            out = torch.empty((positions, self.rows), dtype=torch.float32, device=x.device)
        elif out.numel() < positions * self.rows or not out.is_contiguous() or out.dtype != torch.float32:
            raise ValueError("out must be a contiguous float32 tensor of positions x rows")
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        call("spm_dense_streamed", self._h, x.data_ptr() or None, x.numel(), positions, out.data_ptr() or None,
             C.c_void_p(s.cuda_stream))
        return out


def streamed(spm, index: int, activations, positions: int, device: int = 0) -> np.ndarray:
    """spm_linear::streamed for stream `index`: `activations` is the flat
    positions x cols buffer; returns positions x rows (host arrays)."""
    import torch

    x = np.ascontiguousarray(activations, dtype=np.float32).ravel()
    with DenseMatrix(spm, index, device) as m:
        y = m.streamed(torch.from_numpy(x).to(f"cuda:{device}"), positions)
        return y.cpu().numpy()
