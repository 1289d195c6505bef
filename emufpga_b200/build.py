"""Build libspmgpu.so in-tree for sm_100a (and nothing else), and libspmsynth.so.

    python -m emufpga_b200.build          # incremental
    python -m emufpga_b200.build --clean  # from scratch

Objects go to emufpga_b200/_build/ (git-ignored); the shared libraries land
beside this file so that they travel with the source tree:

  libspmgpu.so    the engine: kernels, host orchestration, the C ABI
  libspmsynth.so  the synthetic-model writer alone (host code, no CUDA), for
                  processes that must not load the engine
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
OUT = HERE / "_build"
LIB = HERE / "libspmgpu.so"
SYNTH_LIB = HERE / "libspmsynth.so"
SYNTH_SOURCES = ("host_synth.cpp", "host_format.cpp", "synth_only.cpp")
INCLUDE = HERE.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a", "-ccbin", CXX]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
                     f"-I{INCLUDE}"]
CXX_FLAGS = ["-O2", "-fPIC", "-std=c++17", "-Wall", "-Wno-unused-function", f"-I{INCLUDE}",
             "-I/usr/local/cuda/include"]


def _headers_mtime() -> float:
    files = list(SRC.glob("*.h")) + list(SRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    obj = OUT / (src.name + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [CXX, *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return obj


def build(clean: bool = False, verbose: bool = False) -> Path:
    if clean and OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir(exist_ok=True)
    sources = sorted(SRC.glob("*.cu")) + sorted(SRC.glob("*.cpp"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = dict(zip((s.name for s in sources), pool.map(lambda s: _compile(s, verbose), sources)))
    engine = [o for n, o in objs.items() if n != "synth_only.cpp"]
    synth = [objs[n] for n in SYNTH_SOURCES]
    for lib, parts, link in ((LIB, engine, [NVCC, *ARCH, "-shared"]), (SYNTH_LIB, synth, [CXX, "-shared"])):
        newest = max(o.stat().st_mtime for o in parts)
        if not lib.exists() or lib.stat().st_mtime < newest:
            cmd = [*link, "-o", str(lib), *map(str, parts), "-lpthread"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.clean, a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
