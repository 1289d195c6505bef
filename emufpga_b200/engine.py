"""Python face of the token loop, mirroring the reference's interfaces.

    spm_gguf::decode_{f32,q8_0,q5_k,q6_k}  -> decode_f32/decode_q8_0/...   (host codecs)
    spm_gguf::read / read_tensor_range      -> gguf_probe / gguf_find
    spm_order::parse_order / reorder        -> order_check / default_order
    spm_linear::streamed                    -> streamed(model, index, acts, positions, out)
    spm_batch::{Client, Scratch, decode_step} -> Session.decode_step
    serve-demo's lockstep loop              -> serve()

Device work runs in libspmgpu.so; torch supplies device buffers only.
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import BLOCK, F32, Q2_K, Q5_K, Q6_K, Q8_0, SpmError, call, lib
from .configs import Recipe, Shape

__all__ = [
    "SpmError", "synth_gguf", "decode_blocks", "decode_f32", "decode_q8_0", "decode_q6_k", "decode_q5_k",
    "decode_q2_k", "gguf_probe", "gguf_find", "order_check", "default_order", "Model", "Session", "Weights",
    "streamed", "serve",
]


def _ptr(buf) -> C.c_void_p:
    if isinstance(buf, np.ndarray):
        return C.c_void_p(buf.ctypes.data)
    if isinstance(buf, (bytes, bytearray)):
        arr = np.frombuffer(buf, dtype=np.uint8)
        return C.c_void_p(arr.ctypes.data)
    raise TypeError(type(buf))


# ---------------------------------------------------------------- host ----
def synth_gguf(recipe: Recipe, threads: int = 0) -> np.ndarray:
    """A synthetic GGUF v3 image (numpy uint8 array), written by libspmsynth.so."""
    from . import synth

    return synth.synth_gguf(recipe, threads)


def decode_blocks(dtype: int, data: bytes | np.ndarray) -> np.ndarray:
    """Host decode of whole GGML blocks (spm-gguf/src/tensor.rs:69-210)."""
    raw = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data.view(np.uint8)
    raw = np.ascontiguousarray(raw)
    bv, bb = BLOCK[dtype]
    out = np.empty(max(1, raw.size // bb * bv), dtype=np.float32)
    call("spm_decode_blocks", dtype, _ptr(raw), raw.size, out.ctypes.data_as(C.POINTER(C.c_float)))
    return out[: raw.size // bb * bv]


def decode_f32(data) -> np.ndarray:
    return decode_blocks(F32, data)


def decode_q8_0(data) -> np.ndarray:
    return decode_blocks(Q8_0, data)


def decode_q6_k(data) -> np.ndarray:
    return decode_blocks(Q6_K, data)


def decode_q5_k(data) -> np.ndarray:
    return decode_blocks(Q5_K, data)


def decode_q2_k(data) -> np.ndarray:
    return decode_blocks(Q2_K, data)


def gguf_probe(image: np.ndarray) -> tuple[int, int]:
    """(tensor count, data offset) after the bounded parse."""
    t, o = C.c_uint64(), C.c_uint64()
    call("spm_gguf_probe", _ptr(image), len(image), C.byref(t), C.byref(o))
    return t.value, o.value


def gguf_find(image: np.ndarray, name: str) -> dict:
    dt, off, nb = C.c_uint32(), C.c_uint64(), C.c_uint64()
    dims = (C.c_uint64 * 4)()
    call("spm_gguf_find", _ptr(image), len(image), name.encode(), C.byref(dt), dims, C.byref(off), C.byref(nb))
    return {"dtype": dt.value, "dims": list(dims), "offset": off.value, "nbytes": nb.value}


def order_check(text: str, image: np.ndarray) -> None:
    call("spm_order_check", text.encode(), _ptr(image), len(image))


def default_order(shape: Shape, image: np.ndarray | None = None) -> str:
    """Consumption order of a model shape as .order text (router biases listed if `image` holds them)."""
    cfg = shape.cfg()
    out = C.c_void_p()
    call("spm_order_default", C.byref(cfg), _ptr(image) if image is not None else None,
         len(image) if image is not None else 0, C.byref(out))
    try:
        return C.string_at(out).decode()
    finally:
        lib().spm_free(out)


# -------------------------------------------------------------- device ----
def _dev_ptr(t) -> C.c_void_p:
    import torch

    if not isinstance(t, torch.Tensor) or not t.is_cuda or not t.is_contiguous():
        raise TypeError("device buffers must be contiguous CUDA tensors")
    return C.c_void_p(t.data_ptr())


def pack_image(image: np.ndarray, path: str, shape: Shape | None = None, order: str | None = None) -> None:
    """Pack a GGUF model into a device-image file (host only, no GPU)."""
    cfg = shape.cfg() if shape is not None else None
    call("spm_pack_image", _ptr(image), len(image), order.encode() if order else None,
         C.byref(cfg) if cfg is not None else None, path.encode())


def image_probe(path: str) -> tuple[int, int]:
    """(image bytes, stream count) of a device-image file; raises if it is malformed."""
    b, n = C.c_uint64(), C.c_int32()
    call("spm_image_probe", path.encode(), C.byref(b), C.byref(n))
    return b.value, n.value


class Model:
    """The weight stream of one model, packed in HBM in consumption order."""

    def __init__(self, image: np.ndarray, shape: Shape | None = None, order: str | None = None, device: int = 0,
                 ep: tuple[int, int] | None = None):
        """`ep=(world, rank)`: expert parallel -- only experts e with
        e % world == rank are uploaded and computed on this GPU."""
        self.shape = shape
        cfg = shape.cfg() if shape is not None else None
        h = C.c_void_p()
        o = order.encode() if order else None
        cp = C.byref(cfg) if cfg is not None else None
        if ep:
            call("spm_model_open_memory_ep", _ptr(image), len(image), o, cp, device, ep[0], ep[1], C.byref(h))
        else:
            call("spm_model_open_memory", _ptr(image), len(image), o, cp, device, C.byref(h))
        self._h = h
        self.device = device
        self.ep = ep

    @classmethod
    def from_file(cls, path: str, shape: Shape | None = None, order_path: str | None = None, device: int = 0,
                  ep: tuple[int, int] | None = None):
        """Open a GGUF file (memory-mapped: ranks opening the same file share its pages)."""
        self = cls.__new__(cls)
        self.shape = shape
        cfg = shape.cfg() if shape is not None else None
        h = C.c_void_p()
        o = order_path.encode() if order_path else None
        cp = C.byref(cfg) if cfg is not None else None
        if ep:
            call("spm_model_open_ep", path.encode(), o, cp, device, ep[0], ep[1], C.byref(h))
        else:
            call("spm_model_open", path.encode(), o, cp, device, C.byref(h))
        self._h = h
        self.device = device
        self.ep = ep
        return self

    @classmethod
    def from_image(cls, path: str, shape: Shape | None = None, device: int = 0):
        """Open a packed image file (pack_image): one sequential upload."""
        self = cls.__new__(cls)
        self.shape = shape
        h = C.c_void_p()
        call("spm_model_open_image", path.encode(), device, C.byref(h))
        self._h = h
        self.device = device
        self.ep = None
        return self

    def close(self) -> None:
        if getattr(self, "_h", None):
            call("spm_model_close", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def weight_bytes(self) -> int:
        v = C.c_uint64()
        call("spm_model_weight_bytes", self._h, C.byref(v))
        return v.value

    @property
    def stream_count(self) -> int:
        v = C.c_int32()
        call("spm_model_stream_count", self._h, C.byref(v))
        return v.value

    def stream_index(self, name: str) -> int:
        v = C.c_int32()
        call("spm_model_stream_index", self._h, name.encode(), C.byref(v))
        return v.value

    def stream_info(self, index: int) -> dict:
        r, c, d, b = C.c_uint64(), C.c_uint64(), C.c_uint32(), C.c_uint64()
        call("spm_model_stream_info", self._h, index, C.byref(r), C.byref(c), C.byref(d), C.byref(b))
        return {"rows": r.value, "cols": c.value, "dtype": d.value, "bytes": b.value}

    def dequant_rows(self, index: int, row0: int, rows: int) -> np.ndarray:
        info = self.stream_info(index)
        out = np.empty((rows, info["cols"]), dtype=np.float32)
        call("spm_dequant_rows", self._h, index, row0, rows, out.ctypes.data_as(C.POINTER(C.c_float)))
        return out


def streamed(model: Model, index: int, acts, positions: int, out, stream=None) -> None:
    """y = W x for one stream: acts is positions x cols, out positions x rows (CUDA tensors).

    Mirrors spm_linear::streamed (spm-linear/src/stream.rs:31-55)."""
    info = model.stream_info(index)
    if acts.numel() < positions * info["cols"]:
        raise SpmError(-2, f"need {positions * info['cols']} activations, got {acts.numel()}")
    if out.numel() < positions * info["rows"]:
        raise SpmError(-1, "output buffer too small")
    call("spm_streamed", model._h, index, _dev_ptr(acts), positions, _dev_ptr(out), stream)


class Weights:
    """One quantized matrix on the device, without a model (the bare operator)."""

    def __init__(self, dtype: int, rows: int, cols: int, blocks: np.ndarray, device: int = 0):
        h = C.c_void_p()
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        call("spm_weights_upload", dtype, rows, cols, _ptr(blocks), device, C.byref(h))
        self._h, self.rows, self.cols, self.dtype = h, rows, cols, dtype

    def gemv(self, acts, positions: int, out, stream=None) -> None:
        if acts.numel() < positions * self.cols:
            raise SpmError(-2, "activation buffer too short")
        call("spm_weights_gemv", self._h, _dev_ptr(acts), positions, _dev_ptr(out), stream)

    def dequant(self, row0: int, rows: int) -> np.ndarray:
        out = np.empty((rows, self.cols), dtype=np.float32)
        call("spm_weights_dequant", self._h, row0, rows, out.ctypes.data_as(C.POINTER(C.c_float)))
        return out

    def close(self):
        if getattr(self, "_h", None):
            call("spm_weights_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """N clients sharing one weight sweep per step (spm-batch Client + Scratch)."""

    def __init__(self, model: Model, max_clients: int, context: int, graphs: bool = True):
        h = C.c_void_p()
        call("spm_session_create", model._h, max_clients, context, C.byref(h))
        self._h, self.model, self.max_clients, self.context = h, model, max_clients, context
        if not graphs:
            call("spm_session_set_graphs", h, 0)

    def close(self):
        if getattr(self, "_h", None):
            call("spm_session_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self, client: int) -> None:
        call("spm_client_reset", self._h, client)

    def length(self, client: int) -> int:
        v = C.c_int32()
        call("spm_client_len", self._h, client, C.byref(v))
        return v.value

    def decode_step(self, tokens: Sequence[int], want_logits: bool = False):
        """One step for clients 0..n-1: returns (argmax ids, logits or None)."""
        n = len(tokens)
        tok = (C.c_uint32 * n)(*tokens)
        arg = (C.c_uint32 * n)()
        vocab = self.model.shape.vocab if self.model.shape else None
        logits = np.empty((n, vocab), dtype=np.float32) if want_logits else None
        call("spm_decode_step", self._h, tok, n,
             logits.ctypes.data_as(C.POINTER(C.c_float)) if want_logits else None, arg)
        return list(arg), logits

    def set_wait_limit(self, nanoseconds: int) -> None:
        """How long device waits on other ranks spin before the step reports SPM_E_TIMEOUT."""
        call("spm_session_set_wait_limit", self._h, int(nanoseconds))

    def prefill(self, client: int, tokens: Sequence[int]) -> None:
        """Run a prompt for `client` on the tensor cores (KV appended, no logits)."""
        n = len(tokens)
        tok = (C.c_uint32 * max(1, n))(*tokens)
        call("spm_prefill", self._h, client, tok, n)

    def decode_step_device(self, tokens_dev, n: int, argmax_dev, logits_dev=None) -> None:
        call("spm_decode_step_device", self._h, _dev_ptr(tokens_dev), n,
             _dev_ptr(logits_dev) if logits_dev is not None else None, _dev_ptr(argmax_dev))

    def sync(self) -> None:
        call("spm_session_sync", self._h)

    @property
    def cuda_stream(self) -> int:
        v = C.c_void_p()
        call("spm_session_stream", self._h, C.byref(v))
        return v.value or 0

    def routes(self, n: int) -> np.ndarray:
        """Expert ids chosen in the last step: layers x clients x experts_used (route order)."""
        sh = self.model.shape
        out = np.zeros((sh.layers, n, sh.experts_used), dtype=np.int32)
        call("spm_session_routes", self._h, n, out.ctypes.data_as(C.POINTER(C.c_int32)))
        return out

    def route_gaps(self, n: int) -> np.ndarray:
        """Routing margins of the last step, layers x clients: (p_K - p_K+1) / p_K."""
        out = np.zeros((self.model.shape.layers, n), dtype=np.float32)
        call("spm_session_route_gaps", self._h, n, out.ctypes.data_as(C.POINTER(C.c_float)))
        return out

    def ep_handle(self) -> bytes:
        """This rank's exchange buffer as a 64-byte CUDA IPC handle."""
        buf = (C.c_uint8 * 64)()
        call("spm_session_ep_handle", self._h, buf)
        return bytes(buf)

    def ep_connect(self, handles: list[bytes]) -> None:
        """Map every rank's exchange buffer (handles in rank order)."""
        blob = b"".join(handles)
        if len(blob) != 64 * len(handles):
            raise SpmError(-1, "CUDA IPC handles are 64 bytes")
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        call("spm_session_ep_connect", self._h, buf)

    def launches_per_step(self, n: int) -> int:
        v = C.c_int32()
        call("spm_session_launches_per_step", self._h, n, C.byref(v))
        return v.value

    KERNEL_KINDS = ("gemv_dense", "gemv_router", "gemv_expert_gate_up", "gemv_expert_down", "gemv_head",
                    "attention", "route", "combine", "other")
    GEMV_KINDS = KERNEL_KINDS[:5]

    def set_profile(self, enable: bool) -> None:
        """Eager steps with a CUDA event pair around every kernel launch (clears the record)."""
        call("spm_session_set_profile", self._h, int(enable))

    def profile(self) -> dict:
        """The recorded launches: {'ms', 'bytes', 'kind'} arrays (kind names in KERNEL_KINDS)."""
        count = C.c_int32()
        call("spm_session_profile", self._h, 0, None, None, None, C.byref(count))
        n = count.value
        ms = np.zeros(n, np.float32)
        nbytes = np.zeros(n, np.uint64)
        kind = np.zeros(n, np.int32)
        call("spm_session_profile", self._h, n, ms.ctypes.data_as(C.POINTER(C.c_float)),
             nbytes.ctypes.data_as(C.POINTER(C.c_uint64)), kind.ctypes.data_as(C.POINTER(C.c_int32)),
             C.byref(count))
        return {"ms": ms, "bytes": nbytes, "kind": kind}


def serve(model: Model, prompts: Sequence[Sequence[int]], steps: int, max_ticks: int | None = None,
          want_logits: bool = False):
    """The lockstep loop of spm-batch/examples/serve-demo.rs:45-91.

    Every tick runs one decode step for all clients; a client feeds its next
    prompt token until its prompt is exhausted, then feeds back its greedy
    pick.  Returns (produced tokens per client, logits of the last tick)."""
    longest = max(len(p) for p in prompts)
    context = longest + steps + 1
    total = longest + steps - 1
    if max_ticks is not None:
        total = min(total, max_ticks)
    sess = Session(model, len(prompts), context)
    try:
        tokens = [p[0] for p in prompts]
        produced: list[list[int]] = [[] for _ in prompts]
        logits = None
        for tick in range(total):
            best, logits = sess.decode_step(tokens, want_logits=want_logits)
            for i, p in enumerate(prompts):
                if tick + 1 < len(p):
                    tokens[i] = p[tick + 1]
                else:
                    produced[i].append(best[i])
                    tokens[i] = best[i]
        return produced, logits
    finally:
        sess.close()
