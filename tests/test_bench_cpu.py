"""bench.py on the CPU: the reference arm's JSON line with the keys the
driver reads (the reference arm of a workload is the CPU oracle, so it needs
no GPU), the CPU baselines, and the host-side arithmetic of the GPU arm (its
tick plan and its roofline summary)."""
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


@pytest.mark.parametrize("workload", ["qwen3-30b-b8", "qwen3-8b-b1", "olmoe-q6_k-b8", "smollm2-b5"])
@pytest.mark.parametrize("steps,warmup", [(100, 8), (20, 3), (5000, 0)])
def test_timed_ticks_are_decode_ticks_of_the_workload(workload, steps, warmup):
    """The bench's tick plan: at least three warm-up ticks, then K timed and K
    end-to-end ticks and the profiled ones, all after every prompt is
    consumed and within the workload's decode steps."""
    sys.path.insert(0, str(ROOT))
    import bench

    w, _, prompts = bench._workload(workload)
    plan = bench._plan(w, prompts, steps, warmup)
    longest = max(len(p) for p in prompts)
    assert plan["prompt"] == longest and plan["warm"] >= 3 and plan["k"] >= 1
    assert plan["k"] <= steps
    last = plan["prompt"] + plan["warm"] + 2 * plan["k"] + bench.PROFILE_TICKS
    assert plan["ticks"] == last
    # every tick after the prompt phase is one of the workload's greedy ticks
    assert last - longest <= w["steps"] - 1
    assert plan["context"] >= longest + w["steps"]


def test_roofline_summary_from_profiled_launches():
    """roofline.achieved = streamed weight bytes of the GEMV launches over
    their summed device time; frac = achieved / peak; kinds split the tick."""
    import numpy as np

    sys.path.insert(0, str(ROOT))
    import bench
    from emufpga_b200.engine import Session

    kinds = Session.KERNEL_KINDS
    t = bench.PROFILE_TICKS
    # per tick: two dense GEMVs (1 MB in 0.5 ms each), one head GEMV (2 MB in
    # 0.25 ms), one attention launch (0.25 ms, no weight bytes)
    dense, head, attention = kinds.index("gemv_dense"), kinds.index("gemv_head"), kinds.index("attention")
    kind = np.array([dense, dense, head, attention], np.int32)
    prof = {"ms": np.tile(np.array([0.5, 0.5, 0.25, 0.25], np.float32), t),
            "bytes": np.tile(np.array([1e6, 1e6, 2e6, 0], np.float64), t),
            "kind": np.tile(kind, t)}
    r = bench._profile_summary(prof, 1000.0, "measured", "qwen3-30b-b8")
    gemv_s = t * 1.25e-3
    assert r["achieved"] == pytest.approx(t * 4e6 / gemv_s / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / 1000.0)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] == 1000.0
    assert r["by_kind"]["gemv_dense"]["launches_per_tick"] == 2
    assert r["by_kind"]["attention"]["ms_per_tick"] == pytest.approx(0.25)
    assert sum(k["share"] for k in r["by_kind"].values()) == pytest.approx(1.0)
    ratio = bench.TRAFFIC_RATIO["qwen3-30b-b8"][0]
    assert r["traffic"]["bytes_per_launch"] == pytest.approx(ratio * 4e6 / 3)
    assert bench._profile_summary(prof, 1000.0, "measured", "smollm2-b5")["traffic"] is None
