"""ctypes binding of libspmgpu.so (include/spmgpu.h).

The library is built in-tree (``python -m emufpga_b200.build``).  Nothing here
falls back to a CPU path: if the shared library is missing, importing the
binding raises, and every compute call needs a CUDA device.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libspmgpu.so"

# status codes (spmgpu.h)
SPM_OK = 0
STATUS = {
    -1: "SPM_E_ARG", -2: "SPM_E_ACTIVATION_LEN", -3: "SPM_E_TRUNCATED", -4: "SPM_E_STREAM",
    -5: "SPM_E_ENCODING", -6: "SPM_E_CUDA", -7: "SPM_E_NCCL", -8: "SPM_E_TIMEOUT", -9: "SPM_E_CONTEXT",
    -10: "SPM_E_NO_DEVICE",
}

# GGML dtypes
F32, F16, Q8_0, Q2_K, Q5_K, Q6_K = 0, 1, 8, 10, 13, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q2_K: (256, 84), Q5_K: (256, 176), Q6_K: (256, 210)}

# families
LLAMA, QWEN3, OLMOE, QWEN3MOE = 1, 2, 3, 4


class SpmError(RuntimeError):
    """A non-zero spm_status, with the library's message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code
        self.name = STATUS.get(code, str(code))


class ModelCfg(C.Structure):
    _fields_ = [
        ("family", C.c_uint32), ("layers", C.c_uint32), ("hidden", C.c_uint32), ("intermediate", C.c_uint32),
        ("heads", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("vocab", C.c_uint32),
        ("experts", C.c_uint32), ("experts_used", C.c_uint32), ("expert_ff", C.c_uint32), ("tied", C.c_uint32),
        ("rope_base", C.c_float), ("eps", C.c_float),
    ]


class SynthSpec(C.Structure):
    _fields_ = [
        ("cfg", ModelCfg), ("layer_type", C.c_uint32), ("expert_type", C.c_uint32), ("embed_type", C.c_uint32),
        ("head_type", C.c_uint32), ("seed", C.c_uint64), ("sigma", C.c_float), ("zipf_s", C.c_float),
        ("gain_sigma", C.c_float), ("threads", C.c_int32),
    ]


_P = C.c_void_p
_U8P = C.POINTER(C.c_uint8)
_FP = C.POINTER(C.c_float)
_U32P = C.POINTER(C.c_uint32)
_U64P = C.POINTER(C.c_uint64)
_I32P = C.POINTER(C.c_int32)

# name -> (restype, argtypes); this table is also the list of exported symbols.
class FileStreamInfo(C.Structure):
    """spm_file_stream_info (spmgpu.h)."""
    _fields_ = [("rows", C.c_uint32), ("cols", C.c_uint32), ("group_size", C.c_uint32), ("encoding", C.c_uint32),
                ("lane_count", C.c_uint32), ("pad_", C.c_uint32), ("groups", C.c_uint64), ("offset", C.c_uint64),
                ("bytes", C.c_uint64)]


class TernaryInfo(C.Structure):
    """spm_ternary_info (spmgpu.h)."""
    _fields_ = [("rows", C.c_uint32), ("cols", C.c_uint32), ("group_size", C.c_uint32), ("pad_", C.c_uint32),
                ("groups", C.c_uint64), ("payload_bytes", C.c_uint64), ("reserved_codes", C.c_uint64),
                ("device_bytes", C.c_uint64)]


class DenseInfo(C.Structure):
    """spm_dense_info (spmgpu.h)."""
    _fields_ = [("rows", C.c_uint32), ("cols", C.c_uint32), ("group_size", C.c_uint32), ("encoding", C.c_uint32),
                ("groups", C.c_uint64), ("payload_bytes", C.c_uint64), ("device_bytes", C.c_uint64)]


class SweepInfo(C.Structure):
    """spm_sweep_info (spmgpu.h)."""
    _fields_ = [("streams", C.c_int32), ("position", C.c_int32), ("host_bytes", C.c_uint64),
                ("device_bytes", C.c_uint64), ("copies", C.c_uint64), ("bytes_copied", C.c_uint64)]


PROTOTYPES = {
    "spm_last_error": (C.c_char_p, []),
    "spm_version": (C.c_char_p, []),
    "spm_free": (None, [_P]),
    "spm_synth_gguf": (C.c_int32, [C.POINTER(SynthSpec), C.POINTER(_U8P), _U64P]),
    "spm_gguf_probe": (C.c_int32, [_P, C.c_uint64, _U64P, _U64P]),
    "spm_gguf_probe_file": (C.c_int32, [C.c_char_p, _U64P, _U64P]),
    "spm_gguf_find": (C.c_int32, [_P, C.c_uint64, C.c_char_p, _U32P, _U64P, _U64P, _U64P]),
    "spm_decode_blocks": (C.c_int32, [C.c_uint32, _P, C.c_uint64, _FP]),
    "spm_order_check": (C.c_int32, [C.c_char_p, _P, C.c_uint64]),
    "spm_order_default": (C.c_int32, [C.POINTER(ModelCfg), _P, C.c_uint64, C.POINTER(C.c_void_p)]),
    "spm_model_open": (C.c_int32, [C.c_char_p, C.c_char_p, C.POINTER(ModelCfg), C.c_int, C.POINTER(_P)]),
    "spm_model_open_memory": (C.c_int32, [_P, C.c_uint64, C.c_char_p, C.POINTER(ModelCfg), C.c_int, C.POINTER(_P)]),
    "spm_model_close": (C.c_int32, [_P]),
    "spm_model_weight_bytes": (C.c_int32, [_P, _U64P]),
    "spm_model_stream_count": (C.c_int32, [_P, _I32P]),
    "spm_model_stream_info": (C.c_int32, [_P, C.c_int32, _U64P, _U64P, _U32P, _U64P]),
    "spm_model_stream_index": (C.c_int32, [_P, C.c_char_p, _I32P]),
    "spm_dequant_rows": (C.c_int32, [_P, C.c_int32, C.c_uint64, C.c_uint64, _FP]),
    "spm_dequant_rows_static": (C.c_int32, [_P, C.c_int32, C.c_uint64, C.c_uint64, _FP]),
    "spm_model_open_ep": (C.c_int32, [C.c_char_p, C.c_char_p, C.POINTER(ModelCfg), C.c_int, C.c_int32, C.c_int32,
                                      C.POINTER(_P)]),
    "spm_model_open_memory_ep": (C.c_int32, [_P, C.c_uint64, C.c_char_p, C.POINTER(ModelCfg), C.c_int, C.c_int32,
                                             C.c_int32, C.POINTER(_P)]),
    "spm_pack_image": (C.c_int32, [_P, C.c_uint64, C.c_char_p, C.POINTER(ModelCfg), C.c_char_p]),
    "spm_image_probe": (C.c_int32, [C.c_char_p, _U64P, C.POINTER(C.c_int32)]),
    "spm_model_open_image": (C.c_int32, [C.c_char_p, C.c_int, C.POINTER(_P)]),
    "spm_session_ep_handle": (C.c_int32, [_P, _P]),
    "spm_session_ep_connect": (C.c_int32, [_P, _P]),
    "spm_streamed": (C.c_int32, [_P, C.c_int32, _P, C.c_int32, _P, _P]),
    "spm_weights_upload": (C.c_int32, [C.c_uint32, C.c_uint64, C.c_uint64, _P, C.c_int, C.POINTER(_P)]),
    "spm_weights_free": (C.c_int32, [_P]),
    "spm_weights_gemv": (C.c_int32, [_P, _P, C.c_int32, _P, _P]),
    "spm_weights_dequant": (C.c_int32, [_P, C.c_uint64, C.c_uint64, _FP]),
    "spm_session_create": (C.c_int32, [_P, C.c_int32, C.c_int32, C.POINTER(_P)]),
    "spm_session_destroy": (C.c_int32, [_P]),
    "spm_client_reset": (C.c_int32, [_P, C.c_int32]),
    "spm_client_len": (C.c_int32, [_P, C.c_int32, _I32P]),
    "spm_decode_step": (C.c_int32, [_P, _U32P, C.c_int32, _FP, _U32P]),
    "spm_decode_step_device": (C.c_int32, [_P, _P, C.c_int32, _P, _P]),
    "spm_session_sync": (C.c_int32, [_P]),
    "spm_session_stream": (C.c_int32, [_P, C.POINTER(_P)]),
    "spm_session_set_graphs": (C.c_int32, [_P, C.c_int32]),
    "spm_session_routes": (C.c_int32, [_P, C.c_int32, _I32P]),
    "spm_session_route_gaps": (C.c_int32, [_P, C.c_int32, C.POINTER(C.c_float)]),
    "spm_session_launches_per_step": (C.c_int32, [_P, C.c_int32, _I32P]),
    "spm_session_set_profile": (C.c_int32, [_P, C.c_int32]),
    "spm_prefill": (C.c_int32, [_P, C.c_int32, _U32P, C.c_int32]),
    "spm_session_set_wait_limit": (C.c_int32, [_P, C.c_uint64]),
    "spm_session_profile": (C.c_int32, [_P, C.c_int32, _FP, _U64P, _I32P, _I32P]),
    "spm_file_probe": (C.c_int32, [_P, C.c_uint64, _U32P, _U32P, _I32P]),
    "spm_file_stream": (C.c_int32, [_P, C.c_uint64, C.c_int32, C.POINTER(FileStreamInfo)]),
    "spm_ternary_upload": (C.c_int32, [_P, C.c_uint64, C.c_int32, C.c_int, C.POINTER(_P)]),
    "spm_ternary_free": (C.c_int32, [_P]),
    "spm_ternary_describe": (C.c_int32, [_P, C.POINTER(TernaryInfo)]),
    "spm_ternary_gemv": (C.c_int32, [_P, _P, C.c_int32, C.c_uint64, _P, _P]),
    "spm_dense_upload": (C.c_int32, [_P, C.c_uint64, C.c_int32, C.c_int, C.POINTER(_P)]),
    "spm_dense_free": (C.c_int32, [_P]),
    "spm_dense_describe": (C.c_int32, [_P, C.POINTER(DenseInfo)]),
    "spm_dense_streamed": (C.c_int32, [_P, _P, C.c_uint64, C.c_int32, _P, _P]),
    "spm_qblocks_upload": (C.c_int32, [_P, C.c_uint64, C.c_int32, C.c_int, C.POINTER(_P)]),
    "spm_qblocks_free": (C.c_int32, [_P]),
    "spm_qblocks_describe": (C.c_int32, [_P, C.POINTER(DenseInfo)]),
    "spm_qblocks_gemv": (C.c_int32, [_P, _P, C.c_uint64, C.c_int32, _P, _P]),
    "spm_sweep_open": (C.c_int32, [_P, C.c_uint64, C.c_int, C.c_uint64, C.POINTER(_P)]),
    "spm_sweep_open_file": (C.c_int32, [C.c_char_p, C.c_int, C.c_uint64, C.POINTER(_P)]),
    "spm_sweep_close": (C.c_int32, [_P]),
    "spm_sweep_describe": (C.c_int32, [_P, C.POINTER(SweepInfo)]),
    "spm_sweep_stream": (C.c_int32, [_P, C.c_int32, _U32P, _U32P, _U32P]),
    "spm_sweep_next": (C.c_int32, [_P, _P, C.c_uint64, C.c_int32, _P, _P, _I32P]),
    "spm_sweep_rewind": (C.c_int32, [_P]),
    "spm_sweep_plan": (C.c_int32, [_U64P, C.c_int32, C.c_uint64, _I32P, C.c_int32, C.POINTER(C.c_int64),
                                   C.c_int64, C.POINTER(C.c_int64)]),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load libspmgpu.so (once).  Raises if the in-tree build is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m emufpga_b200.build` (no CPU fallback exists)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != SPM_OK:
        raise SpmError(status, lib().spm_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
