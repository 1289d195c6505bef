import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    # Build the checker and the product once if they are missing (both are
    # in-tree .so files; a fresh checkout has neither).
    if not (ROOT / "oracle" / "liboracle.so").exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    if not (ROOT / "emufpga_b200" / "libspmgpu.so").exists():
        subprocess.run([sys.executable, "-m", "emufpga_b200.build"], cwd=ROOT, check=True)


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(ROOT / "tests" / "golden" / "blocks.npz")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a -m gpu test ran without a CUDA device")
    return torch.device("cuda:0")
