import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "nanochatllms.cpp_b200"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size model runs (minutes)")


@pytest.fixture(scope="session")
def orc():
    from oracle.oracle import Oracle
    path = os.path.join(ROOT, "oracle", "_build", "libgtenoracle.so")
    if not os.path.exists(path):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), path], check=True)
    return Oracle(path)


@pytest.fixture(scope="session")
def ref():
    """The compiled reference (oracle/_ref/libgtenref.so); skipped where it was not built."""
    from oracle.oracle import Reference
    path = os.path.join(ROOT, "oracle", "_ref", "libgtenref.so")
    if not os.path.exists(path):
        pytest.skip("reference harness not built (oracle/build_ref.sh needs the reference checkout)")
    return Reference(path)


@pytest.fixture(scope="session")
def gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    import gten_b200
    gten_b200.lib()
    return torch.device("cuda:0")
