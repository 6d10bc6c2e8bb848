"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on a
CPU-only host.  Weights are seeded stubs written by ssla_rt_b200.stub (the
reference generator's schema and draw order), so no test reads the
reference checkout at run time."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


@pytest.fixture(scope="session")
def oracle_mod():
    """The C restatement (oracle/libssla_oracle.so), built here if missing."""
    so = os.path.join(REPO, "oracle", "libssla_oracle.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", os.path.join(REPO, "oracle")], check=True,
                       stdout=subprocess.DEVNULL)
    import oracle
    return oracle


_STUBS = {}


@pytest.fixture(scope="session")
def stub_dir(tmp_path_factory):
    """stub_dir(h, w, seed, tdrop) -> directory with weights.npz + meta.json."""
    from ssla_rt_b200 import stub

    def make(h=64, w=80, seed=1, tdrop=4):
        key = (h, w, seed, tdrop)
        if key not in _STUBS:
            d = tmp_path_factory.mktemp(f"stub_{h}x{w}_s{seed}_w{tdrop}")
            _STUBS[key] = stub.write_stub(str(d), h=h, w=w, seed=seed, tdrop=tdrop)
        return _STUBS[key]
    return make


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
