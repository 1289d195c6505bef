"""Packed device-image files on the host (no GPU): the writer's layout, the
reader's validation, and refusal of damaged files."""
import numpy as np
import pytest

import emufpga_b200 as eb
from emufpga_b200 import configs


@pytest.mark.parametrize("name", ["llama-q8_0", "qwen3-q6_k", "olmoe-q2_k"])
def test_image_holds_every_stream_and_is_deterministic(tmp_path, name):
    r = configs.TINY[name]
    img = eb.synth_gguf(r)
    a, b = tmp_path / "a.spmimg", tmp_path / "b.spmimg"
    eb.pack_image(img, str(a), r.shape)
    eb.pack_image(img, str(b), r.shape)
    assert a.read_bytes() == b.read_bytes()
    nbytes, streams = eb.image_probe(str(a))
    assert streams == len([l for l in eb.default_order(r.shape, img).split("\n")
                           if l.strip().startswith("blk.") or l.strip().startswith(("token_", "output."))
                           if not l.strip().endswith(("_norm.weight", ".bias"))])
    raw = a.read_bytes()
    assert raw[:8] == b"SPMIMG01"
    data = int.from_bytes(raw[8:16], "little")
    assert data % 4096 == 0 and len(raw) == data + nbytes


def test_damaged_images_are_refused(tmp_path):
    r = configs.TINY["llama-q8_0"]
    path = tmp_path / "m.spmimg"
    eb.pack_image(eb.synth_gguf(r), str(path), r.shape)
    raw = path.read_bytes()
    bad = tmp_path / "bad.spmimg"
    bad.write_bytes(b"NOTANIMG" + raw[8:])
    with pytest.raises(eb.SpmError) as e:
        eb.image_probe(str(bad))
    assert e.value.name == "SPM_E_STREAM"
    bad.write_bytes(raw[: len(raw) // 2])
    with pytest.raises(eb.SpmError) as e:
        eb.image_probe(str(bad))
    assert e.value.name == "SPM_E_TRUNCATED"
    bad.write_bytes(raw[:100])
    with pytest.raises(eb.SpmError) as e:
        eb.image_probe(str(bad))
    assert e.value.name == "SPM_E_TRUNCATED"
