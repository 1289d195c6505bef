"""bench.py's reference arm runs on the CPU: one JSON line per run with the
keys the driver reads (the reference arm of a workload is the CPU oracle, so
it needs no GPU)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"metric", "value", "unit", "impl", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


@pytest.mark.parametrize("workload", ["smollm2-b5", "ternary-4096-b8", "dense-f32-4096-b8"])
def test_reference_arm_prints_one_contract_line(workload):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", workload, "--steps", "1",
                          "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert KEYS <= set(line) and line["impl"] == "reference" and line["value"] > 0
    assert line["config"]["workload"] == workload
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"


def test_reference_arm_other_ranks_exit_quietly():
    env = {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}
    import os

    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "ternary-4096-b8",
                          "--steps", "1", "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env={**os.environ, **env})
    assert out.returncode == 0 and not out.stdout.strip()


def test_cpu_baseline_reports_one_thread_and_all_cores():
    sys.path.insert(0, str(ROOT))
    import bench

    import emufpga_b200 as eb

    w, recipe, prompts = bench._workload("smollm2-b5", layers=2)
    img = eb.synth_gguf(recipe)
    one = bench.cpu_baseline(recipe, img, prompts, w["steps"], 0.3, threads=1)
    every = bench.cpu_baseline(recipe, img, prompts, w["steps"], 0.3)
    assert one["cores"] == 1 and "one thread" in one["sample"] and one["value"] > 0
    assert every["cores"] >= 1 and every["value"] > 0 and every["kind"] == one["kind"] == "port"


def test_reference_arm_loads_no_gpu_engine():
    # the reference arm's model is written by a child process; the arm's own
    # process runs the oracle and maps no other library of this repository
    code = ("import sys; sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'smollm2-b1', '--steps', '1', "
            "'--warmup', '0']; import bench; bench.main(); maps = open('/proc/self/maps').read(); "
            "print(sorted({l.split('/')[-1] for l in maps.splitlines() if l.endswith('.so') and "
            "('emufpga_b200' in l or '/oracle/' in l)}))")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip().splitlines()[-1] == "['liboracle.so']"
