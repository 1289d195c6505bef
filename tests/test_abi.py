"""The C ABI library loads on a machine without a GPU and exports every entry
point include/spmgpu.h declares (no compute call is made here)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from emufpga_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared():
    text = (ROOT / "include" / "spmgpu.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared()
    for must in ("spm_decode_step", "spm_streamed", "spm_model_open", "spm_session_create", "spm_dequant_rows"):
        assert must in names


@pytest.mark.parametrize("name", declared())
def test_library_exports(name):
    lib = C.CDLL(str(_lib.LIB_PATH))
    assert hasattr(lib, name), name
    assert name in _lib.PROTOTYPES, f"{name} has no ctypes prototype"


def test_library_reports_no_device_cleanly():
    # Without a GPU, opening a model fails with SPM_E_NO_DEVICE, not a crash.
    import torch
    import emufpga_b200 as eb
    from emufpga_b200 import configs

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    img = eb.synth_gguf(configs.TINY["llama-q8_0"])
    with pytest.raises(eb.SpmError) as e:
        eb.Model(img, configs.TINY["llama-q8_0"].shape)
    assert e.value.name == "SPM_E_NO_DEVICE"
