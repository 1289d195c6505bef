"""Decode-token-loop benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one lockstep tick of the workload (serve-demo schedule): every
client decodes one token off one sweep of the weights.  `value` is the
whole-job tokens/s with the weights resident in HBM, each step timed with
CUDA events on the session stream and L2 flushed (a 256 MiB write) between
steps; `e2e` runs the same ticks through spm_decode_step with host token
buffers (H2D of the tokens and D2H of the greedy picks inside the timed
region).  Dense models do not shard: N>1 runs N independent replicas
("replicas only"), and the slowest rank's time sets the job time.  Routed
(MoE) models over N>1 GPUs run expert parallel: one job serving the same
clients on every rank, experts dealt round robin over the ranks, expert
outputs exchanged over NVLink ("scaling": "strong").

`--workload ternary-4096-b8` times the ternary GEMV of spm-gemv-ref instead
(one launch over a 4096 x 4096 ternary stream with one scale per column and
8 activation lanes per step; metric: weight applications/s, the reference's
useful-weights rate), and `--workload dense-f32-4096-b8` the dense .spm
streamed GEMV of spm-linear (a 4096 x 4096 F32 stream, 8 positions), with the
same clocks, L2 flush, e2e and CPU-baseline fields; N>1 runs replicas.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DEFAULT_WORKLOAD = "smollm2-b5"
# .spm operator workloads: rows, cols, group size, lanes (positions)
TERNARY = {"ternary-4096-b8": (4096, 4096, 4096, 8)}
DENSE = {"dense-f32-4096-b8": (4096, 4096, 4096, 8)}


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=96)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--gguf-dir", default="/dev/shm",
                    help="where rank 0 writes the synthetic GGUF that expert-parallel ranks memory-map")
    ap.add_argument("--layers", type=int, default=0,
                    help="keep only the first N layers (small cases for profiler captures; not a bench number)")
    return ap.parse_args()


def _dist():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class Clocks:
    """nvidia-smi samples (200 ms) while the timed region runs."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread:
                self.thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 4 + i and r[4 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _workload(name, layers=0):
    import dataclasses

    from emufpga_b200 import configs

    w = configs.WORKLOADS[name]
    r = configs.RECIPES[w["recipe"]]
    if layers:
        r = r.replace(shape=dataclasses.replace(r.shape, layers=min(layers, r.shape.layers)))
    return w, r, configs.workload_prompts(name)


def _tick_tokens(prompts, tick, best):
    """Next tokens under serve-demo's lockstep rule."""
    return [p[tick + 1] if tick + 1 < len(p) else best[i] for i, p in enumerate(prompts)]


def cpu_baseline(recipe, img, prompts, steps, seconds: float, threads: int = 0):
    """The oracle (this repo's C restatement of the reference CPU loop) on all
    host cores (threads=0) or `threads` of them: lockstep ticks until `seconds`
    of work; tokens/s.  One thread matches the reference's single-threaded
    engine; more spread the output rows, leaving every result bit-identical."""
    from oracle import oracle as O

    n = len(prompts)
    om = O.OracleModel(img, recipe.shape)
    longest = max(len(p) for p in prompts)
    sess = om.session(n, longest + steps + 1)
    tokens = [p[0] for p in prompts]
    t0 = time.perf_counter()
    ticks = 0
    while ticks < longest + steps - 1:
        logits = sess.step(tokens, threads=threads)
        best = [O.argmax_last(logits[i]) for i in range(n)]
        tokens = _tick_tokens(prompts, ticks, best)
        ticks += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    cores = threads or os.cpu_count()
    how = "one thread" if cores == 1 else "OpenMP over rows"
    return {"value": n * ticks / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"first {ticks} lockstep ticks x {n} clients of the workload (oracle, {how})"}


def run_reference(a, rank, world):
    if rank != 0:
        return 0
    w, recipe, prompts = _workload(a.workload)
    import emufpga_b200 as eb

    img = eb.synth_gguf(recipe)
    n = len(prompts)
    from oracle import oracle as O

    om = O.OracleModel(img, recipe.shape)
    longest = max(len(p) for p in prompts)
    sess = om.session(n, longest + w["steps"] + 1)
    tokens = [p[0] for p in prompts]
    total = longest + w["steps"] - 1
    steps = min(a.steps, max(1, total - a.warmup))
    times = []
    for tick in range(min(total, a.warmup + steps)):
        t0 = time.perf_counter()
        logits = sess.step(tokens)
        best = [O.argmax_last(logits[i]) for i in range(n)]
        dt = time.perf_counter() - t0
        tokens = _tick_tokens(prompts, tick, best)
        if tick >= a.warmup:
            times.append(dt)
        if tick >= a.warmup and sum(times) > 150.0:
            break
    value = n * len(times) / sum(times)
    line = {"metric": "decode tokens/s", "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": world,
            "steps": len(times), "warmup": a.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids)",
            "config": {"workload": a.workload, "clients": n},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "kind": "port", "cores": os.cpu_count(),
                             "sample": f"{len(times)} lockstep ticks after {a.warmup} warm-up ticks"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    a = _args()
    rank, world, local = _dist()
    if a.workload in TERNARY or a.workload in DENSE:
        return run_ternary_reference(a, rank, world) if a.impl == "reference" else run_ternary(a, rank, world, local)
    if a.impl == "reference":
        return run_reference(a, rank, world)
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist
    import emufpga_b200 as eb

    w, recipe, prompts = _workload(a.workload, a.layers)
    # Routed models over several GPUs run expert parallel: every rank serves
    # all clients, and the experts are dealt round robin over the ranks (one
    # job; tokens/s is not multiplied by the ranks).  Dense models run one
    # replica per GPU.  Rank 0 writes the synthetic GGUF once; every rank
    # memory-maps it.
    ep_mode = world > 1 and recipe.shape.moe
    img = None
    if ep_mode:
        from emufpga_b200 import ep as eplib

        path = f"{a.gguf_dir}/emufpga_{a.workload}_{recipe.shape.layers}l.gguf"
        if rank == 0:
            img = eb.synth_gguf(recipe)
            if not os.path.exists(path) or os.path.getsize(path) != len(img):
                img.tofile(path + ".part")
                os.replace(path + ".part", path)
        pg.barrier()
        model = eb.Model.from_file(path, recipe.shape, device=local, ep=(world, rank))
    else:
        img = eb.synth_gguf(recipe)
        model = eb.Model(img, recipe.shape, device=local)
    n = len(prompts)
    longest = max(len(p) for p in prompts)
    total_ticks = longest + w["steps"] - 1
    warm, steps = max(a.warmup, 3), a.steps  # at least three untimed warm-up steps
    if warm + steps > total_ticks:
        steps = max(1, total_ticks - warm)
    context = longest + w["steps"] + 1
    sess = eb.Session(model, n, context)
    if ep_mode:
        eplib.connect(sess)
        pg.barrier()
    stream = torch.cuda.ExternalStream(sess.cuda_stream, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    argmax = torch.zeros(n, dtype=torch.int32, device=dev)
    prompt_dev = torch.tensor([[p[min(t + 1, len(p) - 1)] for p in prompts] for t in range(total_ticks)],
                              dtype=torch.int32, device=dev)
    in_prompt = torch.tensor([[t + 1 < len(p) for p in prompts] for t in range(total_ticks)], device=dev)
    tokens = torch.tensor([p[0] for p in prompts], dtype=torch.int32, device=dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]

    # ---- device-resident timing (value) ----
    with torch.cuda.stream(stream):
        for t in range(warm):
            sess.decode_step_device(tokens, n, argmax)
            tokens = torch.where(in_prompt[t], prompt_dev[t], argmax)
        torch.cuda.synchronize(dev)
        if pg:
            pg.barrier()
        torch.cuda.synchronize(dev)
        with Clocks(local) as clocks:
            for i in range(steps):
                t = warm + i
                flush.zero_()
                starts[i].record(stream)
                sess.decode_step_device(tokens, n, argmax)
                ends[i].record(stream)
                tokens = torch.where(in_prompt[t], prompt_dev[t], argmax)
            torch.cuda.synchronize(dev)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    local_ms = sum(step_ms)
    job_ms = local_ms
    if pg:
        tt = torch.tensor([local_ms], device=dev)
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
        job_ms = float(tt.item())
    launches = sess.launches_per_step(n)
    sess.close()

    # ---- end to end through the C ABI with host buffers (e2e) ----
    sess = eb.Session(model, n, context)
    if ep_mode:
        eplib.connect(sess)
        pg.barrier()
    toks = [p[0] for p in prompts]
    for t in range(warm):
        best, _ = sess.decode_step(toks)
        toks = _tick_tokens(prompts, t, best)
    if pg:
        pg.barrier()
    e2e_s = 0.0
    touched = []  # MoE: experts the step streamed, summed over layers
    for i in range(steps):
        t0 = time.perf_counter()
        best, _ = sess.decode_step(toks)
        e2e_s += time.perf_counter() - t0
        toks = _tick_tokens(prompts, warm + i, best)
        if recipe.shape.moe:
            r = sess.routes(n)
            touched.append(sum(len(set(r[l].ravel().tolist())) for l in range(r.shape[0])))
    if pg:
        tt = torch.tensor([e2e_s], device=dev)
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
        e2e_s = float(tt.item())
    sess.close()

    # ---- roofline of the GEMV: one sweep of every weight stream, graph-captured ----
    roof = None
    if rank == 0:
        roof = gemv_roofline(eb, model, n, dev)
    tokens_total = n * steps * (1 if ep_mode else world)
    ranks_agree = None
    if ep_mode:
        # every rank serves the same clients: their greedy tokens must agree
        got = [None] * world
        pg.all_gather_object(got, list(toks))
        ranks_agree = all(g == got[0] for g in got)
    step_bytes = model.weight_bytes
    if recipe.shape.moe:
        step_bytes += statistics.mean(touched) * expert_bytes(model)
    line = None
    if rank == 0:
        peak, how = _peaks()
        clk = clocks.summary()
        line = {
            "metric": "decode tokens/s", "value": tokens_total / (job_ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": job_ms / steps,
            "higher_is_better": True, "scaling": "strong" if ep_mode else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized by this repo's encoder, uniform prompt ids)",
            "config": {"workload": a.workload, "model": w["recipe"], "clients": n, "prompts": w["prompts"],
                       "parallelism": (f"expert parallel x{world}" if ep_mode else f"replicas x{world}")
                       if world > 1 else "single GPU",
                       "weight_bytes_per_step": round(step_bytes),
                       "l2": "flushed between timed steps (256 MiB write)"},
            "weight_stream_gbs": step_bytes * steps / (job_ms / 1e3) / 1e9,
            "e2e": {"value": tokens_total / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 4 * n,
                    "d2h_bytes_per_step": 4 * n},
            "gpu_launches": launches * steps,
            "roofline": None, "clocks": clk,
        }
        if roof:
            ach = roof["bytes"] / roof["seconds"] / 1e9
            line["roofline"] = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                                "peak_source": how, "traffic": None,
                                "kernel": "gemv_stream (one sweep of every dense stream and the LM head)",
                                "bytes_per_launch_avg": roof["bytes"] / roof["launches"],
                                "launches_per_sweep": roof["launches"]}
        if recipe.shape.moe:
            line["config"]["experts_touched_per_step"] = statistics.mean(touched)
        if ep_mode:
            line["config"]["ranks_tokens_agree"] = ranks_agree
        if a.layers:
            line["config"]["layers_kept"] = recipe.shape.layers
            line["invalid"] = "model truncated with --layers (profiling case, not a bench number)"
        if not a.no_cpu_baseline and img is not None and world == 1:  # rank 0 at N=1 only
            line["cpu_baseline"] = cpu_baseline(recipe, img, prompts, w["steps"], a.cpu_seconds)
            line["cpu_baseline_1thread"] = cpu_baseline(recipe, img, prompts, w["steps"], a.cpu_seconds / 2,
                                                        threads=1)
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def expert_streams(model):
    sh = model.shape
    if not sh.moe:
        return []
    return [model.stream_index(f"blk.{l}.ffn_{k}_exps.weight") for l in range(sh.layers)
            for k in ("gate", "up", "down")]


def expert_bytes(model):
    """Quantized bytes of one expert's gate, up and down matrices (layer 0)."""
    sh = model.shape
    return sum(model.stream_info(model.stream_index(f"blk.0.ffn_{k}_exps.weight"))["bytes"]
               for k in ("gate", "up", "down")) / sh.experts


def gemv_roofline(eb, model, n, dev):
    """Graph-capture one sweep of spm_streamed over every rotating stream plus
    the LM head (the decode step's GEMV launches, same shapes and client
    count), replay it with L2 flushed between sweeps, and time each replay
    with CUDA events: achieved = quantized bytes per sweep / sweep time."""
    import torch

    idx = list(range(model.stream_count))
    infos = [model.stream_info(i) for i in idx]
    embd = model.stream_index("token_embd.weight")
    # every matrix a step sweeps: all streams but the embedding, which is the
    # LM head itself when tied
    experts = set(expert_streams(model))
    keep = [i for i in idx if (i != embd or model.shape.tied) and i not in experts]
    maxc = max(infos[i]["cols"] for i in keep)
    maxr = max(infos[i]["rows"] for i in keep)
    x = torch.randn(n * maxc, device=dev)
    y = torch.empty(n * maxr, device=dev)
    s = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with torch.cuda.stream(s):
        for i in keep:
            eb.streamed(model, i, x, n, y, stream=s.cuda_stream)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in keep:
            eb.streamed(model, i, x, n, y, stream=s.cuda_stream)
    total = 0.0
    reps = 10
    with torch.cuda.stream(s):
        for _ in range(3):
            g.replay()
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            g.replay()
            b.record(s)
            b.synchronize()
            total += a.elapsed_time(b) / 1e3
    nbytes = sum(infos[i]["bytes"] for i in keep)
    del g
    return {"bytes": nbytes, "seconds": total / reps, "launches": len(keep)}




# ---------------------------------------------------------------------------
# .spm operators: ternary GEMV (spm-gemv-ref run_gemv), dense streamed (spm-linear)
# ---------------------------------------------------------------------------

def ternary_input(name: str, seed: int = 0):
    """A one-stream .spm file and the activations of the workload.  Ternary:
    the value distributions of the reference's golden generator
    (spm-vectors/src/draw.rs): weights uniform over {0, +1, -1}, scales
    k/16 + 1/16 (k < 32), activations k/16 - 2 (k < 64).  Dense F32: weights
    and activations k/16 - 2 (k < 64), as spm-linear/tests/agreement.rs draws
    them."""
    import numpy as np

    from emufpga_b200 import spmfile as sf

    rng = np.random.default_rng(seed)
    if name in DENSE:
        rows, cols, group, lanes = DENSE[name]
        w = (rng.integers(0, 64, rows * cols) / 16 - 2.0).astype(np.float32)
        x = (rng.integers(0, 64, (lanes, cols)) / 16 - 2.0).astype(np.float32)
        return sf.dense_file([(rows, cols)], group, [w]), x
    rows, cols, group, lanes = TERNARY[name]
    codes = np.array([0, 1, 3], np.uint8)[rng.integers(0, 3, rows * cols)]
    groups = -(-rows * cols // group)
    scales = (rng.integers(0, 32, groups) / 16 + 0.0625).astype(np.float32)
    x = (rng.integers(0, 64, (lanes, cols)) / 16 - 2.0).astype(np.float32)
    return sf.ternary_file(rows, cols, group, codes, scales), x


def _ternary_config(name):
    rows, cols, group, lanes = TERNARY.get(name) or DENSE[name]
    return {"workload": name, "rows": rows, "cols": cols, "group_size": group, "lanes": lanes}


def _oracle_run(name, data, x):
    """The oracle's form of the workload's operator: lanes x rows."""
    from oracle import oracle as O

    if name in DENSE:
        return O.spm_streamed(data, x.ravel(), x.shape[0])
    return O.spm_run_gemv(data, x)


def ternary_cpu_baseline(name, data, x, seconds: float):
    """The oracle's operator (single-threaded, like the reference's scan) on
    the whole workload, repeated until `seconds` of work."""
    from oracle import oracle as O

    lanes, cols = x.shape
    rows = O.spm_describe(data)["rows"]
    t0 = time.perf_counter()
    runs = 0
    while True:
        _oracle_run(name, data, x)
        runs += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": runs * rows * cols * lanes / dt, "unit": "weights/s", "cores": 1, "kind": "port",
            "sample": f"{runs} whole scans of the workload (oracle, one thread)"}


def run_ternary(a, rank, world, local):
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist
    from emufpga_b200 import linear as L
    from emufpga_b200 import ternary as T

    dense = a.workload in DENSE
    rows, cols, group, lanes = (DENSE if dense else TERNARY)[a.workload]
    data, x = ternary_input(a.workload)
    m = L.DenseMatrix(data, 0, local) if dense else T.TernaryMatrix(data, 0, local)
    xd = torch.from_numpy(x).to(dev)
    y = torch.empty((lanes, rows), dtype=torch.float32, device=dev)

    def gemv():
        if dense:
            m.streamed(xd, lanes, out=y)
        else:
            m.gemv(xd, out=y)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    warm, steps = max(a.warmup, 3), a.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for _ in range(warm):
        gemv()
    torch.cuda.synchronize(dev)
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    with Clocks(local) as clocks:
        for i in range(steps):
            flush.zero_()
            starts[i].record(stream)
            gemv()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    local_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    job_ms = local_ms
    if pg:
        tt = torch.tensor([local_ms], device=dev)
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
        job_ms = float(tt.item())

    # e2e: host activations in (pinned), results out, every step
    x_host = torch.from_numpy(x).pin_memory()
    y_host = torch.empty((lanes, rows), dtype=torch.float32).pin_memory()
    for _ in range(warm):
        xd.copy_(x_host, non_blocking=True)
        gemv()
        y_host.copy_(y, non_blocking=True)
    torch.cuda.synchronize(dev)
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        xd.copy_(x_host, non_blocking=True)
        gemv()
        y_host.copy_(y, non_blocking=True)
        torch.cuda.synchronize(dev)
    e2e_s = time.perf_counter() - t0
    if pg:
        tt = torch.tensor([e2e_s], device=dev)
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
        e2e_s = float(tt.item())

    if rank == 0:
        from oracle import oracle as O

        ok = bool((y_host.numpy().view("u4") == _oracle_run(a.workload, data, x).view("u4")).all())
        apps = rows * cols * lanes
        peak, how = _peaks()
        launch_s = local_ms / 1e3 / steps
        ach = m.payload_bytes / launch_s / 1e9
        line = {
            "metric": ("dense" if dense else "ternary") + " weight applications/s",
            "value": apps * steps * world / (job_ms / 1e3),
            "unit": "weights/s", "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": job_ms / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": ("synthetic (f32 weights and activations in sixteenths, as the reference's agreement test "
                     "draws them)") if dense else ("synthetic (weights uniform over {0,+1,-1}, scales and "
                                                  "activations in sixteenths, as the reference's golden generator "
                                                  "draws them)"),
            "config": dict(_ternary_config(a.workload), parallelism=f"replicas x{world}" if world > 1 else
                           "single GPU", l2="flushed between timed steps (256 MiB write)",
                           bit_identical_to_oracle=ok),
            "e2e": {"value": apps * steps * world / e2e_s, "unit": "weights/s", "h2d_bytes_per_step": x.nbytes,
                    "d2h_bytes_per_step": lanes * rows * 4},
            "gpu_launches": steps,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                         "peak_source": how, "traffic": None,
                         "kernel": "dense_streamed_kernel" if dense else "ternary_gemv_kernel",
                         "bytes_per_launch": m.payload_bytes,
                         "note": "bound by the sequential f32 chain per (row, lane) that bit-exactness "
                                 "requires, not by HBM"},
            "clocks": clocks.summary(),
        }
        if not a.no_cpu_baseline and world == 1:  # rank 0 at N=1 only
            line["cpu_baseline"] = ternary_cpu_baseline(a.workload, data, x, a.cpu_seconds)
        print(json.dumps(line), flush=True)
    m.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def run_ternary_reference(a, rank, world):
    """The reference arm for a ternary workload: the oracle's run_gemv
    (single-threaded, as the reference's scan is) timed per step."""
    if rank != 0:
        return 0
    from oracle import oracle as O

    rows, cols, group, lanes = TERNARY.get(a.workload) or DENSE[a.workload]
    data, x = ternary_input(a.workload)
    for _ in range(a.warmup):
        _oracle_run(a.workload, data, x)
    times = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        _oracle_run(a.workload, data, x)
        times.append(time.perf_counter() - t0)
        if sum(times) > 150.0:
            break
    value = rows * cols * lanes * len(times) / sum(times)
    line = {"metric": ("dense" if a.workload in DENSE else "ternary") + " weight applications/s", "value": value,
            "unit": "weights/s", "impl": "reference",
            "n_gpus": world, "steps": len(times), "warmup": a.warmup,
            "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (as the ours arm)",
            "config": _ternary_config(a.workload),
            "cpu_baseline": {"value": value, "unit": "weights/s", "kind": "port", "cores": 1,
                             "sample": f"{len(times)} whole scans after {a.warmup} warm-up scans"},
            "e2e": {"value": value, "unit": "weights/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
