"""ctypes face of liboracle.so -- TEST INFRASTRUCTURE ONLY.

The CPU restatement of emufpga's token loop and of its .spm stream
operators (spm_oracle.c).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as the
checker or the timed reference; the product (emufpga_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path
from typing import Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

F32, F16, Q8_0, Q2_K, Q5_K, Q6_K = 0, 1, 8, 10, 13, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q2_K: (256, 84), Q5_K: (256, 176), Q6_K: (256, 210)}


class Cfg(C.Structure):
    _fields_ = [
        ("family", C.c_uint32), ("layers", C.c_uint32), ("hidden", C.c_uint32), ("intermediate", C.c_uint32),
        ("heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("vocab", C.c_uint32),
        ("experts", C.c_uint32), ("experts_used", C.c_uint32), ("expert_ff", C.c_uint32), ("tied", C.c_uint32),
        ("rope_base", C.c_float), ("eps", C.c_float),
    ]


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        fp, u8 = C.POINTER(C.c_float), C.c_void_p
        L.or_f16_to_f32.restype, L.or_f16_to_f32.argtypes = C.c_float, [C.c_uint16]
        L.or_decode.restype, L.or_decode.argtypes = C.c_int, [C.c_uint32, u8, C.c_uint64, fp]
        for name in ("or_gemv_fma", "or_gemv_dot"):
            f = getattr(L, name)
            f.restype, f.argtypes = C.c_int, [C.c_uint32, u8, C.c_uint64, C.c_uint64, fp, C.c_int, fp, C.c_int]
        L.or_scaled_rms_norm.argtypes = [fp, fp, C.c_float, C.c_int, C.c_int]
        L.or_rms_norm_slice.argtypes = [fp, fp, C.c_int, C.c_float, fp]
        L.or_rope_smol.argtypes = [fp, C.c_int, C.c_int, C.c_float]
        L.or_rope_slice.argtypes = [fp, C.c_int, C.c_int, C.c_float]
        L.or_silu.restype, L.or_silu.argtypes = C.c_float, [C.c_float]
        for name in ("or_attend_cached", "or_attend_slice"):
            getattr(L, name).argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_int, C.c_int, fp]
        L.or_softmax_route.argtypes = [fp, C.c_int, fp]
        L.or_top_k.argtypes = [fp, C.c_int, C.c_int, C.POINTER(C.c_int), fp]
        L.or_argmax_last.restype, L.or_argmax_last.argtypes = C.c_uint32, [fp, C.c_uint64]
        L.or_gguf_parse.restype = C.c_int
        L.or_gguf_parse.argtypes = [u8, C.c_uint64, C.POINTER(C.c_void_p), C.c_char_p, C.c_int]
        L.or_gguf_free.argtypes = [C.c_void_p]
        L.or_model_new.restype = C.c_void_p
        L.or_model_new.argtypes = [u8, C.c_uint64, C.POINTER(Cfg), C.c_char_p, C.c_int]
        L.or_model_free.argtypes = [C.c_void_p]
        L.or_session_new.restype = C.c_void_p
        L.or_session_new.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.or_session_free.argtypes = [C.c_void_p]
        L.or_decode_step.restype = C.c_int
        L.or_decode_step.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), fp, C.c_int, C.POINTER(C.c_int32)]
        L.or_session_route_margins.restype = C.c_int
        L.or_session_route_margins.argtypes = [C.c_void_p, fp]
        L.or_serve.restype = C.c_int
        L.or_serve.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_int), C.c_int, C.c_int,
                               C.POINTER(C.c_uint32), C.POINTER(C.c_int), fp, C.c_int, C.c_int]
        u32p = C.POINTER(C.c_uint32)
        L.or_spm_describe.restype = C.c_int
        L.or_spm_describe.argtypes = [u8, C.c_uint64, C.c_int32, u32p, u32p, u32p, u32p, u32p, C.c_char_p, C.c_int]
        L.or_spm_run_gemv.restype = C.c_int
        L.or_spm_run_gemv.argtypes = [u8, C.c_uint64, fp, C.c_int, C.c_uint64, fp, C.c_uint64, C.c_char_p, C.c_int]
        L.or_spm_streamed.restype = C.c_int
        L.or_spm_streamed.argtypes = [u8, C.c_uint64, C.c_int32, C.c_uint32, C.c_uint32, fp, C.c_uint64, C.c_int,
                                      fp, C.c_char_p, C.c_int]
        L.or_resident.argtypes = [fp, C.c_uint32, C.c_uint32, fp, C.c_int, fp]
        L.or_spm_qblocks.restype = C.c_int
        L.or_spm_qblocks.argtypes = [u8, C.c_uint64, C.c_int32, fp, C.c_uint64, C.c_int, fp, C.c_char_p, C.c_int]
        _lib = L
    return _lib


def _f(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def f16_to_f32(bits: int) -> float:
    return lib().or_f16_to_f32(bits)


def decode(dtype: int, data) -> np.ndarray:
    raw = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8))
    bv, bb = BLOCK[dtype]
    out = np.empty(max(1, raw.size // bb * bv), dtype=np.float32)
    rc = lib().or_decode(dtype, raw.ctypes.data, raw.size, _f(out))
    if rc == -1:
        raise ValueError(f"byte length {raw.size} is not divisible by {bb}")
    if rc:
        raise ValueError(f"unsupported dtype {dtype}")
    return out[: raw.size // bb * bv]


def gemv_fma(dtype: int, blocks, rows: int, cols: int, x: np.ndarray, positions: int, threads: int = 0) -> np.ndarray:
    raw = np.ascontiguousarray(np.frombuffer(bytes(blocks), dtype=np.uint8)) if not isinstance(blocks, np.ndarray) \
        else np.ascontiguousarray(blocks.view(np.uint8))
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty((positions, rows), dtype=np.float32)
    rc = lib().or_gemv_fma(dtype, raw.ctypes.data, rows, cols, _f(x), positions, _f(y), threads)
    if rc:
        raise ValueError("bad gemv shape")
    return y


def gemv_dot(dtype: int, blocks, rows: int, cols: int, x: np.ndarray, positions: int, threads: int = 0) -> np.ndarray:
    raw = np.ascontiguousarray(blocks.view(np.uint8))
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty((positions, rows), dtype=np.float32)
    if lib().or_gemv_dot(dtype, raw.ctypes.data, rows, cols, _f(x), positions, _f(y), threads):
        raise ValueError("bad gemv shape")
    return y


def rope_smol(head: np.ndarray, position: int, base: float) -> np.ndarray:
    h = np.array(head, dtype=np.float32)
    lib().or_rope_smol(_f(h), h.size, position, base)
    return h


def rope_slice(head: np.ndarray, position: int, base: float) -> np.ndarray:
    h = np.array(head, dtype=np.float32)
    lib().or_rope_slice(_f(h), h.size, position, base)
    return h


def rms_norm_slice(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().or_rms_norm_slice(_f(x), _f(w), x.size, eps, _f(out))
    return out


def scaled_rms_norm(x: np.ndarray, w: np.ndarray, eps: float, width: int) -> np.ndarray:
    v = np.array(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    lib().or_scaled_rms_norm(_f(v), _f(w), eps, width, v.size // width)
    return v


def softmax_route(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty_like(v)
    lib().or_softmax_route(_f(v), v.size, _f(out))
    return out


def top_k(v: np.ndarray, k: int) -> list[tuple[int, float]]:
    v = np.ascontiguousarray(v, dtype=np.float32)
    ids = (C.c_int * k)()
    vals = np.empty(k, dtype=np.float32)
    lib().or_top_k(_f(v), v.size, k, ids, _f(vals))
    return [(int(ids[i]), float(vals[i])) for i in range(k)]


def attend(kind: str, q, keys, values, positions, heads, kv_heads, head_dim) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(keys, dtype=np.float32)
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(heads * head_dim, dtype=np.float32)
    fn = lib().or_attend_cached if kind == "smol" else lib().or_attend_slice
    fn(_f(q), _f(k), _f(v), positions, heads, kv_heads, head_dim, _f(out))
    return out


def argmax_last(row: np.ndarray) -> int:
    row = np.ascontiguousarray(row, dtype=np.float32)
    return int(lib().or_argmax_last(_f(row), row.size))


def silu(x: float) -> float:
    return lib().or_silu(x)


def gguf_parse_error(image: np.ndarray) -> str | None:
    """None if the bounded parse accepts the image, else its message."""
    h = C.c_void_p()
    err = C.create_string_buffer(256)
    image = np.ascontiguousarray(image, dtype=np.uint8)
    if lib().or_gguf_parse(image.ctypes.data, image.size, C.byref(h), err, 256) == 0:
        lib().or_gguf_free(h)
        return None
    return err.value.decode()


class SpmError(ValueError):
    """A .spm file or ternary GEMV the oracle refused; `code` is its OR_SPM_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def _spm_bytes(spm) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(spm), dtype=np.uint8))


def spm_describe(spm, index: int = 0) -> dict:
    """Stream count and stream `index`'s descriptor fields (header and directory only)."""
    raw = _spm_bytes(spm)
    v = [C.c_uint32() for _ in range(5)]
    err = C.create_string_buffer(256)
    rc = lib().or_spm_describe(raw.ctypes.data, raw.size, index, *[C.byref(x) for x in v], err, 256)
    if rc:
        raise SpmError(rc, err.value.decode())
    return dict(zip(("streams", "rows", "cols", "group_size", "encoding"), (x.value for x in v)))


def spm_run_gemv(spm, x: np.ndarray) -> np.ndarray:
    """spm_gemv_ref::run_gemv on the first stream: x is lanes x x_cols, the
    result lanes x rows (bank.lane(l) for every lane)."""
    raw = _spm_bytes(spm)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim != 2:
        raise ValueError("x must be lanes x cols")
    lanes, x_cols = x.shape
    err = C.create_string_buffer(256)
    head = C.c_uint32()
    rows = C.c_uint32()
    rc = lib().or_spm_describe(raw.ctypes.data, raw.size, 0, C.byref(head), C.byref(rows), None, None, None, err, 256)
    if rc:
        raise SpmError(rc, err.value.decode())
    bank = np.empty(max(1, rows.value * lanes), dtype=np.float32)
    rc = lib().or_spm_run_gemv(raw.ctypes.data, raw.size, _f(x), lanes, x_cols, _f(bank), bank.size, err, 256)
    if rc:
        raise SpmError(rc, err.value.decode())
    return bank[: rows.value * lanes].reshape(rows.value, lanes).T.copy()


def spm_streamed(spm, x: np.ndarray, positions: int, index: int = 0, shape: tuple | None = None) -> np.ndarray:
    """spm_linear::streamed on stream `index`: x is the flat activation
    buffer (positions x cols); returns positions x rows.  `shape` (rows,
    cols) defaults to the stream's descriptor."""
    raw = _spm_bytes(spm)
    rows, cols = shape if shape is not None else (lambda d: (d["rows"], d["cols"]))(spm_describe(spm, index))
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(max(1, positions * rows), dtype=np.float32)
    err = C.create_string_buffer(256)
    rc = lib().or_spm_streamed(raw.ctypes.data, raw.size, index, rows, cols, _f(x), x.size, positions, _f(out),
                               err, 256)
    if rc:
        raise SpmError(rc, err.value.decode())
    return out[: positions * rows].reshape(positions, rows)


def spm_qblocks(spm, x: np.ndarray, positions: int, index: int = 0) -> np.ndarray:
    """q6_operation / stream_matrix on the block stream `index`: x is the
    flat positions x cols buffer; returns positions x rows."""
    raw = _spm_bytes(spm)
    d = spm_describe(spm, index)
    rows = d["rows"]
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(max(1, positions * rows), dtype=np.float32)
    err = C.create_string_buffer(256)
    rc = lib().or_spm_qblocks(raw.ctypes.data, raw.size, index, _f(x), x.size, positions, _f(out), err, 256)
    if rc:
        raise SpmError(rc, err.value.decode())
    return out[: positions * rows].reshape(positions, rows)


def resident(w: np.ndarray, rows: int, cols: int, x: np.ndarray, positions: int) -> np.ndarray:
    """spm_linear::resident: w in stream order (w[k] = W[k % rows][k / rows])."""
    w = np.ascontiguousarray(w, dtype=np.float32).ravel()
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(max(1, positions * rows), dtype=np.float32)
    lib().or_resident(_f(w), rows, cols, _f(x), positions, _f(out))
    return out[: positions * rows].reshape(positions, rows)


def cfg_of(shape) -> Cfg:
    c = Cfg()
    for name, _ in Cfg._fields_:
        setattr(c, name, int(getattr(shape, name)) if name == "tied" else getattr(shape, name))
    return c


class OracleModel:
    """The CPU token loop over a GGUF image (keeps a reference to the image)."""

    def __init__(self, image: np.ndarray, shape):
        self.image = np.ascontiguousarray(image, dtype=np.uint8)
        self.shape = shape
        err = C.create_string_buffer(256)
        cfg = cfg_of(shape)
        self._h = lib().or_model_new(self.image.ctypes.data, self.image.size, C.byref(cfg), err, 256)
        if not self._h:
            raise ValueError(err.value.decode())

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_model_free(self._h)
            self._h = None

    def session(self, clients: int, context: int) -> "OracleSession":
        return OracleSession(self, clients, context)

    def serve(self, prompts: Sequence[Sequence[int]], steps: int, threads: int = 0, max_ticks: int = 0):
        """serve-demo's lockstep loop; returns (produced per client, logits of the last tick)."""
        n = len(prompts)
        longest = max(len(p) for p in prompts)
        cap = longest + steps - 1
        flat = (C.c_uint32 * sum(len(p) for p in prompts))(*[t for p in prompts for t in p])
        lens = (C.c_int * n)(*[len(p) for p in prompts])
        produced = (C.c_uint32 * (n * cap))()
        plens = (C.c_int * n)()
        last = np.zeros((n, self.shape.vocab), dtype=np.float32)
        rc = lib().or_serve(self._h, flat, lens, n, steps, produced, plens, _f(last), threads, max_ticks)
        if rc:
            raise RuntimeError(f"oracle serve failed ({rc})")
        return [[produced[i * cap + j] for j in range(plens[i])] for i in range(n)], last


class OracleSession:
    def __init__(self, model: OracleModel, clients: int, context: int):
        self.model = model
        self.clients = clients
        self._h = lib().or_session_new(model._h, clients, context)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_session_free(self._h)
            self._h = None

    def step(self, tokens: Sequence[int], threads: int = 0, routes: bool = False):
        n = self.clients
        tok = (C.c_uint32 * n)(*tokens)
        logits = np.empty((n, self.model.shape.vocab), dtype=np.float32)
        r = None
        if routes:
            r = np.zeros((self.model.shape.layers, n, max(1, self.model.shape.experts_used)), dtype=np.int32)
        rc = lib().or_decode_step(self._h, tok, _f(logits), threads,
                                  r.ctypes.data_as(C.POINTER(C.c_int32)) if r is not None else None)
        if rc:
            raise RuntimeError(f"oracle step failed ({rc})")
        return (logits, r) if routes else logits

    def route_margins(self) -> np.ndarray:
        """The last step's routing margin per layer and client, (p_K - p_K+1) / p_K
        of the routing probabilities (1 for dense layers): how close each
        client's routing came to another expert set (spm-granite-moe/src/moe.rs:17-35
        selects by these probabilities)."""
        out = np.empty((self.model.shape.layers, self.clients), dtype=np.float32)
        lib().or_session_route_margins(self._h, _f(out))
        return out
