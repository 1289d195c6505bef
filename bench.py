"""Decode-token-loop benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A run follows the serve-demo lockstep schedule (spm-batch/examples/
serve-demo.rs:59-91): every tick each client decodes one token off one sweep
of the weights; a client feeds its prompt one token per tick, then its greedy
picks.  The prompt ticks run untimed; then W warm-up decode ticks, then K
timed decode ticks (every client feeding back its own greedy token, contexts
past the prompts).  `value` is the whole-job tokens/s with the weights
resident in HBM, each tick timed with CUDA events on the session stream and
L2 flushed (a 256 MiB write) before each tick; `e2e` times the next K ticks
through spm_decode_step with host token buffers (H2D of the tokens and D2H of
the greedy picks inside the timed region).  `roofline` is the dominant
kernel's: every GEMV launch of a few further decode ticks run eagerly with a
CUDA event pair around each launch (spm_session_set_profile), achieved =
quantized weight bytes those launches stream / their summed duration.

The default workload is BASELINE configs[4], Qwen3-30B-A3B Q5_K with eight
clients (the largest configuration; it fits one B200), and the line carries a
`batch1` sub-record for configs[2]'s batch-1 case (Qwen3-8B Q6_K, one client)
measured the same way.  Dense models do not shard: N>1 runs N independent
replicas ("replicas only").  Routed (MoE) models over N>1 GPUs run expert
parallel: one job of n clients, rank r running the attention block of clients
r*n/N .. (r+1)*n/N - 1 and the experts dealt to it (round robin) for every
client; the attention outputs, the expert outputs and the greedy picks are
exchanged over NVLink ("scaling": "strong": the one-GPU line of a routed
workload is the same job, so it says "strong" too).

`--workload ternary-4096-b8` times the ternary GEMV of spm-gemv-ref instead
(one launch over a 4096 x 4096 ternary stream with one scale per column and
8 activation lanes per step; metric: weight applications/s, the reference's
useful-weights rate), and `--workload dense-f32-4096-b8` the dense .spm
streamed GEMV of spm-linear (a 4096 x 4096 F32 stream, 8 positions), with the
same clocks, L2 flush, e2e and CPU-baseline fields; N>1 runs replicas.

`--impl reference` times the CPU oracle (this repository's C restatement of
the reference's CPU token loop; the reference itself is Rust and cannot be
built here) on all host threads, in a process that loads no GPU code.
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

DEFAULT_WORKLOAD = "qwen3-30b-b8"
BATCH1_WORKLOAD = "qwen3-8b-b1"
PROFILE_TICKS = 3
# .spm operator workloads: rows, cols, group size, lanes (positions)
TERNARY = {"ternary-4096-b8": (4096, 4096, 4096, 8)}
DENSE = {"dense-f32-4096-b8": (4096, 4096, 4096, 8)}
# host-to-HBM sweeps of a multi-stream .spm file: kind, streams, rows, cols, lanes
SWEEP = {"sweep-ternary-32x4096-b8": ("ternary", 32, 4096, 4096, 8),
         "sweep-f32-8x4096-b8": ("f32", 8, 4096, 4096, 8)}
# DRAM bytes (read + write) per algorithmic weight byte of gemv_stream launches
# in ncu captures (gpu__... dram__bytes_read.sum + dram__bytes_write.sum over
# the launch's quantized weight bytes); the file named beside each holds the
# capture.  Used to report `roofline.traffic` per launch.
TRAFFIC_RATIO = {
    "qwen3-8b-b1": (1.003, "profiles/gemv_stream_qwen3_8b_b1.md"),
    "qwen3-30b-b8": (1.053, "profiles/gemv_stream_qwen3_30b_b8.md"),
}
STAGING = "activations staged per 32-value unit as 22-bit block fixed point (three int8 digit planes), " \
          "integer products, fp32 scales and sums"


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch1", action="store_true", help="skip the batch-1 sub-record")
    ap.add_argument("--prompt-ticks", action="store_true",
                    help="feed prompts one token per tick (serve-demo) instead of spm_prefill on the tensor cores")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--gguf-dir", default="/dev/shm",
                    help="where rank 0 writes the synthetic GGUF that expert-parallel ranks memory-map")
    ap.add_argument("--layers", type=int, default=0,
                    help="keep only the first N layers (small cases for profiler captures; not a bench number)")
    ap.add_argument("--profile-region", choices=["decode", "prefill"], default=None,
                    help="bracket the timed decode ticks or the prefill with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    return ap.parse_args()


def _init_nccl(dist, dev):
    """The NCCL process group, with anything the library prints while it sets
    up its communicator sent to stderr: stdout carries only the JSON line."""
    import datetime

    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        dist.barrier()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def _dist():
    # NCCL's version banner would land on stdout beside the JSON line
    os.environ.setdefault("NCCL_DEBUG", "WARN")
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


def _next_tokens(prompts, tick, best):
    """Tokens fed at tick+1 under serve-demo's lockstep rule."""
    return [p[tick + 1] if tick + 1 < len(p) else best[i] for i, p in enumerate(prompts)]


def _plan(w, prompts, steps, warmup):
    """Tick ranges of a run: prompt ticks [0, P), warm-up decode ticks, K timed
    decode ticks, K e2e ticks, PROFILE_TICKS profiled ticks, clamped so that
    every one is a decode tick of the workload (at most steps - 1 of them)."""
    longest = max(len(p) for p in prompts)
    decode = w["steps"] - 1
    warm = max(warmup, 3)
    k = max(1, min(steps, (decode - warm - PROFILE_TICKS) // 2))
    return {"prompt": longest, "warm": warm, "k": k, "ticks": longest + warm + 2 * k + PROFILE_TICKS,
            "context": longest + w["steps"] + 1}


def cpu_baseline(recipe, img, prompts, steps, seconds: float, threads: int = 0):
    """The oracle (this repo's C restatement of the reference CPU loop) on all
    host cores (threads=0) or `threads` of them: lockstep ticks from the first
    until `seconds` of work (at least one tick); tokens/s.  One thread matches
    the reference's single-threaded engine; more spread the output rows and the
    active experts, leaving every result bit-identical."""
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
        tokens = _next_tokens(prompts, ticks, best)
        ticks += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    cores = threads or os.cpu_count()
    how = "one thread" if cores == 1 else "OpenMP over rows and active experts"
    return {"value": n * ticks / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"first {ticks} lockstep ticks x {n} clients of the workload, contexts 1-{ticks} "
                      f"(oracle, {how})"}


def _reference_input(a) -> "np.ndarray":
    """The workload's synthetic GGUF, written by a child process
    (`python -m emufpga_b200.synth`) and read back here, so that this process
    maps no library of this repository but the oracle."""
    import numpy as np

    path = f"{a.gguf_dir}/emufpga_reference_{a.workload}_{os.getpid()}.gguf"
    try:
        subprocess.run([sys.executable, "-m", "emufpga_b200.synth", a.workload, path], cwd=ROOT, check=True)
        return np.fromfile(path, dtype=np.uint8)
    finally:
        for p in (path, path + ".part"):
            if os.path.exists(p):
                os.unlink(p)


def run_reference(a, rank, world):
    """The reference arm: the CPU oracle on all host threads, in a process
    that loads liboracle.so only (its input model is written by a child
    process; no GPU code).  It times lockstep ticks W..W+K of the run (the
    first ticks: a full run takes the oracle minutes to hours), each tick
    bounded so the whole arm ends within a few minutes."""
    if rank != 0:
        return 0
    w, recipe, prompts = _workload(a.workload)
    img = _reference_input(a)
    n = len(prompts)
    from oracle import oracle as O

    om = O.OracleModel(img, recipe.shape)
    longest = max(len(p) for p in prompts)
    sess = om.session(n, longest + w["steps"] + 1)
    tokens = [p[0] for p in prompts]
    total = longest + w["steps"] - 1
    steps = min(a.steps, max(1, total - a.warmup))
    times = []
    t_start = time.perf_counter()
    first = None
    for tick in range(min(total, a.warmup + steps)):
        t0 = time.perf_counter()
        logits = sess.step(tokens)
        best = [O.argmax_last(logits[i]) for i in range(n)]
        dt = time.perf_counter() - t0
        tokens = _next_tokens(prompts, tick, best)
        if tick >= a.warmup:
            first = tick if first is None else first
            times.append(dt)
        if time.perf_counter() - t_start > 150.0 and times:
            break
    value = n * len(times) / sum(times)
    sample = (f"lockstep ticks {first}-{first + len(times) - 1} (contexts {first + 1}-{first + len(times)}) x {n} "
              f"clients after {first} warm-up ticks; oracle on {os.cpu_count()} host threads")
    line = {"metric": "decode tokens/s", "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": world,
            "steps": len(times), "warmup": first, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "strong" if recipe.shape.moe else "weak", "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized by this repo's encoder, uniform prompt ids)",
            "config": {"workload": a.workload, "model": w["recipe"], "clients": n, "prompts": w["prompts"],
                       "timed_ticks": [first, first + len(times) - 1]},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "kind": "port", "cores": os.cpu_count(),
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def _profile_summary(prof: dict, peak: float, how: str, workload: str) -> dict:
    """Roofline of gemv_stream from the profiled launches, and every kernel
    kind's share of the profiled ticks."""
    import numpy as np

    from emufpga_b200.engine import Session

    ms = prof["ms"].astype(np.float64)
    nbytes = prof["bytes"].astype(np.float64)
    gemv = prof["kind"] < len(Session.GEMV_KINDS)
    seconds = ms[gemv].sum() / 1e3
    ach = nbytes[gemv].sum() / seconds / 1e9
    launches = int(gemv.sum())
    kinds = {}
    for k, name in enumerate(Session.KERNEL_KINDS):
        sel = prof["kind"] == k
        if sel.any():
            kinds[name] = {"launches_per_tick": int(sel.sum()) // PROFILE_TICKS,
                           "ms_per_tick": float(ms[sel].sum()) / PROFILE_TICKS,
                           "share": float(ms[sel].sum() / ms.sum())}
            if k < len(Session.GEMV_KINDS):
                kinds[name]["gbs"] = float(nbytes[sel].sum() / (ms[sel].sum() / 1e3) / 1e9)
    traffic = None
    if workload in TRAFFIC_RATIO:
        ratio, src = TRAFFIC_RATIO[workload]
        traffic = {"bytes_per_launch": ratio * nbytes[gemv].sum() / launches, "source": src,
                   "how": "ncu dram__bytes_read.sum + dram__bytes_write.sum per algorithmic byte, times the "
                          "average launch's algorithmic bytes"}
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "peak_source": how,
            "traffic": traffic, "kernel": "gemv_stream",
            "how": f"CUDA events around each of the {launches} GEMV launches of {PROFILE_TICKS} eager decode ticks "
                   f"(after the timed ticks); achieved = quantized weight bytes streamed / summed launch time",
            "bytes_per_launch_avg": nbytes[gemv].sum() / launches, "launch_us_avg": 1e3 * ms[gemv].sum() / launches,
            "gemv_share_of_eager_tick": float(ms[gemv].sum() / ms.sum()), "by_kind": kinds}


def run_decode(a, name, rank, world, local, pg, dev, ep_ok=True):
    """One decode workload; returns its JSON dict on rank 0 (None elsewhere)."""
    import torch

    import emufpga_b200 as eb

    w, recipe, prompts = _workload(name, a.layers)
    # Routed models over several GPUs run expert parallel: each rank runs the
    # attention block of its share of the clients and the experts dealt to it
    # (round robin) for all clients (one job; tokens/s is not multiplied by
    # the ranks).  Dense models run one
    # replica per GPU.  Rank 0 writes the synthetic GGUF once; every rank
    # memory-maps it.
    ep_mode = ep_ok and world > 1 and recipe.shape.moe
    img = None
    if ep_mode:
        path = f"{a.gguf_dir}/emufpga_{name}_{recipe.shape.layers}l.gguf"
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
    plan = _plan(w, prompts, a.steps, a.warmup)
    P, warm, K = plan["prompt"], plan["warm"], plan["k"]
    sess = eb.Session(model, n, plan["context"])
    if ep_mode:
        from emufpga_b200 import ep as eplib

        eplib.connect(sess)
        pg.barrier()
    stream = torch.cuda.ExternalStream(sess.cuda_stream, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    argmax = torch.zeros(n, dtype=torch.int32, device=dev)
    total_ticks = P + warm + K
    feed = torch.tensor([[p[min(t + 1, len(p) - 1)] for p in prompts] for t in range(total_ticks)],
                        dtype=torch.int32, device=dev)
    in_prompt = torch.tensor([[t + 1 < len(p) for p in prompts] for t in range(total_ticks)], device=dev)
    tokens = torch.tensor([p[0] for p in prompts], dtype=torch.int32, device=dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]

    prefill = None
    first = 0
    if not a.prompt_ticks and not ep_mode and len({len(p) for p in prompts}) == 1:
        # every prompt but its last token through spm_prefill (tensor cores),
        # timed on its own; the decode ticks then start at the prompts' last tick
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if a.profile_region == "prefill":
            torch.cuda.cudart().cudaProfilerStart()
        e0.record(stream)
        for i, p in enumerate(prompts):
            sess.prefill(i, p[:-1])
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if a.profile_region == "prefill":
            torch.cuda.cudart().cudaProfilerStop()
        pms = e0.elapsed_time(e1)
        ptoks = sum(len(p) - 1 for p in prompts)
        prefill = {"value": ptoks / (pms / 1e3), "unit": "tokens/s", "ms": pms, "tokens": ptoks,
                   "how": "spm_prefill of every client's prompt but its last token (tcgen05 products), CUDA events"}
        first = P - 1
        tokens = torch.tensor([p[-1] for p in prompts], dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        # untimed: the prompt ticks (or the prompts' last tick) and the warm-up decode ticks
        for t in range(first, P + warm):
            sess.decode_step_device(tokens, n, argmax)
            tokens = torch.where(in_prompt[t], feed[t], argmax)
        torch.cuda.synchronize(dev)
        if pg:
            pg.barrier()
        torch.cuda.synchronize(dev)
        with Clocks(local) as clocks:
            # ---- device-resident timing (value) ----
            if a.profile_region == "decode":
                torch.cuda.cudart().cudaProfilerStart()
            for i in range(K):
                flush.zero_()
                starts[i].record(stream)
                sess.decode_step_device(tokens, n, argmax)
                ends[i].record(stream)
                tokens = argmax.clone()
            torch.cuda.synchronize(dev)
            if a.profile_region == "decode":
                torch.cuda.cudart().cudaProfilerStop()
            step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
            # ---- end to end through the C ABI with host buffers (e2e) ----
            toks = tokens.cpu().tolist()
            if pg:
                pg.barrier()
            e2e_s = 0.0
            touched = []  # MoE: experts the step streamed, summed over layers
            for i in range(K):
                t0 = time.perf_counter()
                best, _ = sess.decode_step(toks)
                e2e_s += time.perf_counter() - t0
                toks = best
                if recipe.shape.moe:
                    r = sess.routes(n)
                    touched.append(sum(len(set(r[l].ravel().tolist())) for l in range(r.shape[0])))
    # ---- the GEMV launches of a few eager ticks, each between CUDA events ----
    sess.set_profile(True)
    for i in range(PROFILE_TICKS):
        best, _ = sess.decode_step(toks)
        toks = best
    prof = sess.profile()
    sess.set_profile(False)
    local_ms = sum(step_ms)
    job_ms, job_e2e = local_ms, e2e_s
    if pg:
        tt = torch.tensor([local_ms, e2e_s], device=dev, dtype=torch.float64)
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
        job_ms, job_e2e = float(tt[0].item()), float(tt[1].item())
    launches = sess.launches_per_step(n)
    ranks_agree = None
    if ep_mode:
        # the greedy picks are gathered on every rank: they must agree
        got = [None] * world
        pg.all_gather_object(got, list(toks))
        ranks_agree = all(g == got[0] for g in got)
    sess.close()
    tokens_total = n * K * (1 if ep_mode else world)
    step_bytes = model.weight_bytes
    if recipe.shape.moe:
        step_bytes += statistics.mean(touched) * expert_bytes(model)
    line = None
    if rank == 0:
        peak, how = _peaks()
        line = {
            "metric": "decode tokens/s", "value": tokens_total / (job_ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": warm, "ms_per_step": job_ms / K,
            "higher_is_better": True, "scaling": "strong" if ep_mode or (world == 1 and recipe.shape.moe and ep_ok) else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized by this repo's encoder, uniform prompt ids)",
            "config": {"workload": name, "model": w["recipe"], "clients": n, "prompts": w["prompts"],
                       "parallelism": (f"expert parallel x{world}" if ep_mode else f"replicas x{world}")
                       if world > 1 else "single GPU",
                       "prompt_ticks_untimed": P - first,
                       "prompt_phase": "spm_prefill (tensor cores), then the prompts' last tick" if prefill else
                                       "one prompt token per tick (serve-demo schedule)",
                       "timed_ticks": [P + warm, P + warm + K - 1],
                       "timed_context": [P + warm + 1, P + warm + K],
                       "e2e_ticks": [P + warm + K, P + warm + 2 * K - 1],
                       "weight_bytes_per_step": round(step_bytes),
                       "activation_staging": STAGING,
                       "l2": "flushed before every timed tick (256 MiB write)"},
            "weight_stream_gbs": step_bytes * K / (job_ms / 1e3) / 1e9,
            "e2e": {"value": tokens_total / job_e2e, "unit": "tokens/s", "h2d_bytes_per_step": 4 * n,
                    "d2h_bytes_per_step": 4 * n},
            "gpu_launches": launches * K,
            "roofline": _profile_summary(prof, peak, how, name),
        }
        line["weight_stream_frac"] = line["weight_stream_gbs"] / peak
        if prefill:
            line["prefill"] = prefill
        if recipe.shape.moe:
            line["config"]["experts_touched_per_step"] = statistics.mean(touched)
        if ep_mode:
            line["config"]["ranks_tokens_agree"] = ranks_agree
        if a.layers:
            line["config"]["layers_kept"] = recipe.shape.layers
            line["invalid"] = "model truncated with --layers (profiling case, not a bench number)"
        line["_clocks"] = clocks
        line["_img"] = img
        line["_recipe"] = recipe
        line["_prompts"] = prompts
        line["_steps"] = w["steps"]
    model.close()
    return line


def sweep_file(name, seed=0):
    """The workload's .spm file: `streams` streams of rows x cols (ternary
    weights uniform over {0,+1,-1} with one scale per column, or f32 in
    sixteenths), and the activations."""
    import numpy as np

    from emufpga_b200 import spmfile as sf

    kind, streams, rows, cols, lanes = SWEEP[name]
    rng = np.random.default_rng(seed)
    descs, bodies = [], []
    for _ in range(streams):
        if kind == "ternary":
            codes = np.array([0, 1, 3], np.uint8)[rng.integers(0, 3, rows * cols)]
            scales = (rng.integers(0, 32, -(-rows * cols // rows)) / 16 + 0.0625).astype(np.float32)
            descs.append(sf.render_descriptor(rows, cols, rows))
            bodies.append(sf.ternary_stream_bytes(codes, scales, rows))
        else:
            w = (rng.integers(0, 64, rows * cols) / 16 - 2.0).astype(np.float32)
            descs.append(sf.render_descriptor(rows, cols, rows, sf.F32))
            bodies.append(sf.dense_stream_bytes(w, rows, sf.F32))
    x = (rng.integers(0, 64, (lanes, cols)) / 16 - 2.0).astype(np.float32)
    return sf.render_header(streams) + b"".join(descs) + b"".join(bodies), x


def run_sweep(a, rank, world, local):
    """One step = one sweep of every stream of the file through the device
    ring (the streams after the running one are copied in from pinned host
    memory on a copy stream meanwhile).  Beside the streaming sweep the same
    file runs with a ring holding every stream (after the first sweep nothing
    is copied: the compute alone) and the packed bytes are copied once with a
    plain host-to-device copy (the link alone); overlap = the share of the
    shorter of the two that the streaming sweep hides."""
    import torch

    from emufpga_b200 import sweep as S

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    kind, streams, rows, cols, lanes = SWEEP[a.workload]
    data, x = sweep_file(a.workload)
    xd = torch.from_numpy(x).to(dev).reshape(-1)
    stream = torch.cuda.current_stream(dev)
    warm, steps = max(a.warmup, 3), a.steps

    def timed(sw, n):
        y = torch.empty((lanes, rows), dtype=torch.float32, device=dev)
        for _ in range(warm):
            for _ in range(streams):
                sw.next(xd, lanes, out=y)
            sw.rewind()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            for _ in range(streams):
                sw.next(xd, lanes, out=y)
            sw.rewind()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / 1e3 / n

    with S.Sweep(data, local) as sw:
        info = sw.describe()
        packed, ring = int(info["host_bytes"]), int(info["device_bytes"])
        with Clocks(local) as clocks:
            before = sw.describe()["bytes_copied"]
            t_stream = timed(sw, steps)
            copied = (sw.describe()["bytes_copied"] - before) / (warm + steps)
    with S.Sweep(data, local, device_bytes=len(data) * 2) as sw:
        t_compute = timed(sw, steps)
    nbytes = packed
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    devbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    for _ in range(3):
        devbuf.copy_(host, non_blocking=True)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        devbuf.copy_(host, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_copy = e0.elapsed_time(e1) / 1e3 / steps
    hidden = (t_compute + t_copy - t_stream) / min(t_compute, t_copy)
    apps = rows * cols * lanes * streams
    if rank == 0:
        line = {"metric": ("ternary" if kind == "ternary" else "dense") + " weight applications/s, streamed from host",
                "value": apps * world / t_stream, "unit": "weights/s", "n_gpus": world, "steps": steps, "warmup": warm,
                "ms_per_step": 1e3 * t_stream, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (weights and activations as the reference's generators draw them)",
                "config": {"workload": a.workload, "streams": streams, "rows": rows, "cols": cols, "lanes": lanes,
                           "file_bytes": len(data), "ring_bytes": ring, "packed_bytes": nbytes},
                "bytes_copied_per_sweep": copied,
                "h2d_gbs_streaming": copied / t_stream / 1e9,
                "h2d_gbs_plain_copy": nbytes / t_copy / 1e9,
                "sweep_ms_resident": 1e3 * t_compute, "copy_ms": 1e3 * t_copy,
                "overlap_hidden": hidden,
                "e2e": {"value": apps * world / t_stream, "unit": "weights/s", "h2d_bytes_per_step": nbytes,
                        "d2h_bytes_per_step": 0},
                "gpu_launches": streams * steps, "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    return 0


def main():
    a = _args()
    rank, world, local = _dist()
    if a.workload in SWEEP:
        if a.impl == "ours":
            return run_sweep(a, rank, world, local)
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "sweep workloads measure the host link; the "
                              "reference arm times the operators (ternary-4096-b8, dense-f32-4096-b8)"}), flush=True)
        return 0
    if a.workload in TERNARY or a.workload in DENSE:
        return run_ternary_reference(a, rank, world) if a.impl == "reference" else run_ternary(a, rank, world, local)
    if a.impl == "reference":
        return run_reference(a, rank, world)
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        _init_nccl(dist, dev)
        pg = dist
    line = run_decode(a, a.workload, rank, world, local, pg, dev)
    if rank == 0:
        clocks = line.pop("_clocks")
        img, recipe, prompts, wsteps = line.pop("_img"), line.pop("_recipe"), line.pop("_prompts"), line.pop("_steps")
        line["clocks"] = clocks.summary()
        if not a.no_cpu_baseline and img is not None and world == 1:  # rank 0 at N=1 only
            line["cpu_baseline"] = cpu_baseline(recipe, img, prompts, wsteps, a.cpu_seconds)
            line["cpu_baseline_1thread"] = cpu_baseline(recipe, img, prompts, wsteps, a.cpu_seconds / 2,
                                                        threads=1)
        del img
    if world == 1 and not a.no_batch1 and a.workload != BATCH1_WORKLOAD and not a.layers:
        sub = run_decode(a, BATCH1_WORKLOAD, rank, world, local, pg, dev, ep_ok=False)
        clk = sub.pop("_clocks").summary()
        for k in ("_img", "_recipe", "_prompts", "_steps"):
            sub.pop(k)
        line["batch1"] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "steps", "warmup", "weight_stream_gbs",
                                              "weight_stream_frac", "e2e", "roofline", "config", "gpu_launches",
                                              "prefill") if k in sub}
        line["batch1"]["workload"] = BATCH1_WORKLOAD
        line["batch1"]["clocks"] = clk
    if rank == 0:
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

        _init_nccl(dist, dev)
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
