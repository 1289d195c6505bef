"""Regenerates tests/golden/runs/<workload>.npz: the CPU oracle's full run of
each token-loop workload, for the full-run parity tests on the GPU.

    python tests/golden/make_runs.py [workload ...] [--threads N]

A run is the lockstep schedule of spm-batch/examples/serve-demo.rs:59-91: one
decode step per tick for every client, prompt tokens fed one per tick, and
once a client's prompt is exhausted its greedy pick (last index on ties,
serve-demo.rs:72-90) is its next token.  The model is the workload's synthetic
GGUF (this library's seeded encoder; the oracle and the device read the same
bytes).  Per tick and client the file keeps:

  argmax   the oracle's greedy pick (prompt ticks included)
  top_ids  the 8 largest logits' indices (descending value, then index)
  top_vals their values
  margin   largest minus second-largest logit
  maxabs   max |logit| (the tolerance scale: 1e-3 * maxabs)
  route_margin  routed models: the smallest over the layers of the oracle's
           routing margin (p_K - p_K+1) / p_K (1 for dense models) -- where
           it is tiny, any other order of fp32 sums may route the client
           through another expert set
  digest   a sampled SHA-256 of the GGUF image, so a test can check that it
           synthesised the same bytes

The oracle is test infrastructure (oracle/spm_oracle.c); this script only runs
it.  Full runs take from minutes (OLMoE) to about an hour (Qwen3-30B-A3B) on
eight cores; existing files are kept unless named on the command line.
"""
from __future__ import annotations

import argparse
import hashlib
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

OUT = Path(__file__).resolve().parent / "runs"
RUNS = ["olmoe-q6_k-b8", "olmoe-q2_k-b8", "qwen3-8b-b1", "qwen3-8b-b4", "qwen3-30b-b8"]
TOPK = 8


def image_digest(img: np.ndarray) -> str:
    """SHA-256 over the length and 4 KiB samples at 4096 evenly spaced offsets."""
    h = hashlib.sha256(str(img.size).encode())
    step = max(1, img.size // 4096)
    for off in range(0, img.size, step):
        h.update(img[off: off + 4096].tobytes())
    return h.hexdigest()


def top_k(logits: np.ndarray, k: int = TOPK):
    """Indices of the k largest values per row (value descending, index ascending)."""
    part = np.argpartition(-logits, k, axis=1)[:, : k + 1]
    out_ids = np.empty((logits.shape[0], k), np.int32)
    out_vals = np.empty((logits.shape[0], k), np.float32)
    for i in range(logits.shape[0]):
        ids = part[i]
        order = np.lexsort((ids, -logits[i, ids]))[:k]
        out_ids[i] = ids[order]
        out_vals[i] = logits[i, ids[order]]
    return out_ids, out_vals


def run(name: str, threads: int, out: Path = OUT) -> Path:
    import emufpga_b200 as eb
    from emufpga_b200 import configs
    from oracle import oracle as O

    w = configs.WORKLOADS[name]
    recipe = configs.RECIPES[w["recipe"]]
    prompts = configs.workload_prompts(name)
    t0 = time.time()
    img = eb.synth_gguf(recipe)
    digest = image_digest(img)
    om = O.OracleModel(img, recipe.shape)
    n = len(prompts)
    longest = max(len(p) for p in prompts)
    ticks = longest + w["steps"] - 1
    sess = om.session(n, longest + w["steps"] + 1)
    argmax = np.zeros((ticks, n), np.int32)
    top_ids = np.zeros((ticks, n, TOPK), np.int32)
    top_vals = np.zeros((ticks, n, TOPK), np.float32)
    margin = np.zeros((ticks, n), np.float32)
    route_margin = np.ones((ticks, n), np.float32)
    maxabs = np.zeros((ticks, n), np.float32)
    tokens = [p[0] for p in prompts]
    for t in range(ticks):
        logits = sess.step(tokens, threads=threads)
        best = [O.argmax_last(logits[i]) for i in range(n)]
        argmax[t] = best
        top_ids[t], top_vals[t] = top_k(logits)
        s = np.sort(logits, axis=1)
        margin[t] = s[:, -1] - s[:, -2]
        maxabs[t] = np.abs(logits).max(axis=1)
        route_margin[t] = sess.route_margins().min(axis=0)
        tokens = [p[t + 1] if t + 1 < len(p) else best[i] for i, p in enumerate(prompts)]
        if t % 64 == 0:
            print(f"{name}: tick {t}/{ticks} ({time.time() - t0:.0f} s)", flush=True)
    out.mkdir(parents=True, exist_ok=True)
    path = out / f"{name}.npz"
    np.savez_compressed(path, argmax=argmax, top_ids=top_ids, top_vals=top_vals, margin=margin, maxabs=maxabs,
                        route_margin=route_margin,
                        digest=np.array(digest), prompt_lens=np.array([len(p) for p in prompts], np.int32),
                        steps=np.array(w["steps"], np.int32))
    print(f"{name}: {ticks} ticks in {time.time() - t0:.0f} s -> {path}", flush=True)
    return path


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("workloads", nargs="*")
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--out", type=Path, default=OUT, help="directory for the .npz files")
    a = ap.parse_args()
    names = a.workloads or [n for n in RUNS if not (a.out / f"{n}.npz").exists()]
    for name in names:
        run(name, a.threads, a.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
