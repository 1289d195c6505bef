"""The C ABI from C: include/spmgpu.h compiles as strict C99 and a plain C
program links libspmgpu.so and gets correct answers from its host-only entry
points (no device needed)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIBDIR = ROOT / "emufpga_b200"


@pytest.mark.skipif(shutil.which("gcc") is None and not Path("/usr/bin/gcc").exists(), reason="needs gcc")
def test_a_c99_program_links_and_runs(tmp_path):
    cc = "/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else "gcc"
    exe = tmp_path / "probe"
    build = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", f"-I{ROOT / 'include'}",
                            str(ROOT / "tests" / "c_abi_probe.c"), "-o", str(exe), f"-L{LIBDIR}", "-lspmgpu",
                            f"-Wl,-rpath,{LIBDIR}"], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    assert run.stdout.strip() == "c abi ok"
