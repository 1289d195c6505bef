"""Block decoders, bit for bit, against the committed gguf-py fixtures.

Both the oracle (the checker) and the product's host decoder must reproduce
tests/golden/blocks.npz exactly; the device decoder is held to the same bits
in test_gpu_kernels.py.
"""
import numpy as np
import pytest

import emufpga_b200 as eb
from oracle import oracle as O

TYPES = {"q8_0": O.Q8_0, "q6_k": O.Q6_K, "q5_k": O.Q5_K, "q2_k": O.Q2_K}


def same_bits(a, b):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("name", sorted(TYPES))
def test_oracle_matches_gguf_py(golden, name):
    assert same_bits(O.decode(TYPES[name], golden[name].tobytes()), golden[name + "_out"])


@pytest.mark.parametrize("name", sorted(TYPES))
def test_host_decoder_matches_gguf_py(golden, name):
    assert same_bits(eb.decode_blocks(TYPES[name], golden[name]), golden[name + "_out"])


def test_q6_pipeline_fixture(golden):
    # q6-pipeline/tests/pipeline.rs:22-35: the independent decoder equals the GGUF one.
    raw = golden["q6_k_pipeline"]
    assert same_bits(O.decode(O.Q6_K, raw.tobytes()), golden["q6_k_pipeline_out"])
    assert same_bits(eb.decode_q6_k(raw), golden["q6_k_pipeline_out"])


def test_partial_blocks_are_refused():
    for t, bb in ((O.Q8_0, 34), (O.Q6_K, 210), (O.Q5_K, 176), (O.Q2_K, 84)):
        with pytest.raises(eb.SpmError) as e:
            eb.decode_blocks(t, bytes(bb - 1))
        assert e.value.name == "SPM_E_TRUNCATED"


def test_golden_script_is_reproducible():
    # The committed fixture is what the committed script makes.
    import importlib.util
    from pathlib import Path

    gguf = importlib.util.find_spec("gguf")
    if gguf is None:
        pytest.skip("gguf-py is not installed here")
    import tempfile

    spec = importlib.util.spec_from_file_location("make_golden", Path(__file__).parent / "golden" / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with tempfile.TemporaryDirectory() as d:
        mod.OUT = Path(d) / "b.npz"
        mod.main()
        fresh = np.load(mod.OUT)
        ref = np.load(Path(__file__).parent / "golden" / "blocks.npz")
        assert sorted(fresh.files) == sorted(ref.files)
        for k in ref.files:
            assert np.array_equal(fresh[k].view(np.uint8), ref[k].view(np.uint8)), k


def test_golden_runs_cover_the_benchmark_workloads():
    """Every workload of the full-run parity tests has its oracle run on file,
    made from the same synthetic model recipe (tests/golden/make_runs.py)."""
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(here))
    from make_runs import RUNS

    from emufpga_b200 import configs

    for name in RUNS:
        path = here / "runs" / f"{name}.npz"
        assert path.exists(), f"no golden run for {name}: python tests/golden/make_runs.py {name}"
        g = np.load(path)
        w = configs.WORKLOADS[name]
        prompts = configs.workload_prompts(name)
        ticks = max(len(p) for p in prompts) + w["steps"] - 1
        assert g["argmax"].shape == (ticks, len(prompts))
        assert g["top_ids"].shape == (ticks, len(prompts), 8)
        # the oracle's pick is its largest logit (where there is no exact tie)
        strict = g["margin"] > 0
        assert np.array_equal(g["argmax"][strict], g["top_ids"][:, :, 0][strict])
