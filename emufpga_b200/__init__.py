"""emufpga_b200: the decode token loop of emufpga on B200 (sm_100a).

The compute lives in libspmgpu.so (built in-tree by ``emufpga_b200.build``);
this package is its Python face.  See include/spmgpu.h for the C ABI.
"""
from . import configs, linear, qblocks, spmfile, sweep, ternary
from .engine import (Model, Session, SpmError, Weights, decode_blocks, decode_f32, decode_q2_k, decode_q5_k,
                     decode_q6_k, decode_q8_0, default_order, gguf_find, gguf_probe, image_probe, order_check,
                     pack_image, serve, streamed, synth_gguf)

__all__ = [
    "configs", "linear", "qblocks", "spmfile", "sweep", "ternary", "Model", "Session", "SpmError", "Weights", "decode_blocks", "decode_f32",
    "decode_q2_k", "decode_q5_k", "decode_q6_k", "decode_q8_0", "default_order", "gguf_find", "gguf_probe",
    "image_probe", "order_check", "pack_image", "serve", "streamed", "synth_gguf",
]
