"""Test configuration: the `gpu` marker, and the CPU oracle built before anything imports it.

`-m "not gpu"` runs the oracle against the reference's golden material, the host logic and the C-ABI surface (no GPU
calls); `-m gpu` runs the parity tests proper on a B200 through the C ABI.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _oracle_built():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all"], check=True)
    from oracle.oracle import reference_dir
    if os.path.isdir(reference_dir()) and not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libtsb_ref_cpu.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    yield


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    return torch.device("cuda:0")
