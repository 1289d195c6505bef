"""Packed device-image files on the host (no GPU): the writer's layout, the
reader's validation, and refusal of damaged files."""
import struct

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
    # a .spm container: header, one descriptor per stream, then the image's own description
    assert raw[:8] == bytes([0x89, ord("S"), ord("P"), ord("M"), 0x0D, 0x0A, 0x1A, 0x0A])
    assert struct.unpack_from("<HHB", raw, 8) == (1, 1, 0)
    assert struct.unpack_from("<I", raw, 16)[0] == streams
    block_values = {0: 1, 8: 32, 10: 256, 13: 256, 14: 256}
    for i in range(streams):
        rows, cols, group, enc, lanes = struct.unpack_from("<IIIBxH", raw, 32 + 32 * i)
        assert enc >= 0x80 and group == block_values[enc - 0x80] and lanes == 4 and rows and cols
        assert raw[32 + 32 * i + 16:32 + 32 * i + 32] == bytes(16)
    at = 32 + 32 * streams
    assert raw[at:at + 8] == b"SPMIMG02"
    data = int.from_bytes(raw[at + 8:at + 16], "little")
    assert data % 4096 == 0 and len(raw) == data + nbytes
    # a stock .spm reader refuses the tiled profiles as unknown encodings
    from emufpga_b200 import ternary as T

    with pytest.raises(eb.SpmError) as e:
        T.file_probe(raw[:at])
    assert e.value.name == "SPM_E_ENCODING"


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
    # a directory entry that disagrees with the stream table
    flipped = bytearray(raw)
    flipped[32] ^= 1
    bad.write_bytes(bytes(flipped))
    with pytest.raises(eb.SpmError, match="directory entry does not match") as e:
        eb.image_probe(str(bad))
    # a plain .spm file of streams is not an image
    from emufpga_b200 import spmfile as sf

    bad.write_bytes(sf.dense_file([(2, 2)], 4, [np.ones(4, np.float32)]) + bytes(64))
    with pytest.raises(eb.SpmError, match="not a packed image"):
        eb.image_probe(str(bad))
