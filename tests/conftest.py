"""pytest setup: the `gpu` marker, import paths, and an up-to-date build.

Tests marked ``gpu`` need a B200 and call the sm_100a kernels through the C
ABI (``turing-sm75_b200/lib/libb200lab.so``); every other test runs on the
CPU.  The session builds the library and the CPU oracle first (``make`` is a
no-op when they are current; on a GPU box the prebuilt files are used).
"""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "turing-sm75_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a kernels)")
    if shutil.which("nvcc") and shutil.which("make"):
        subprocess.run(["make", "-s", "-C", PKG], check=True, stdout=subprocess.DEVNULL)
    if shutil.which("gcc") and shutil.which("make"):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True,
                       stdout=subprocess.DEVNULL)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
