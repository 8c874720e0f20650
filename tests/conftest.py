"""Shared fixtures.  Tests marked ``gpu`` need an sm_100 GPU; everything
else runs on CPU.  The oracle (oracle/) is the parity checker; the product
under test is alphazero_b200 and its native libraries."""
from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100) GPU")


@pytest.fixture(scope="session", autouse=True)
def _built_libraries():
    from alphazero_b200 import build
    import oracle

    build.build_host()
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build()
    yield


def golden_cases():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    from alphazero_b200 import weights

    sd = weights.make_state_dict(int(z["board"]), int(z["filters"]), int(z["blocks"]),
                                 seed=int(z["weight_seed"]), variant=str(z["variant"]))
    assert weights.weights_digest(sd) == str(z["weights_digest"]), "weight generator drifted"
    return z, sd


@pytest.fixture(scope="session")
def gpu_engine_factory():
    """Creates CudaEngine instances on cuda:0 (GPU tests only)."""
    from alphazero_b200 import build
    from alphazero_b200.engine import CudaEngine

    build.build_cuda()
    made = []

    def make(sd, precision="bf16", eigen_compat=False, max_batch=1024):
        e = CudaEngine(0, precision=precision, eigen_compat=eigen_compat, max_batch=max_batch)
        e.load_state_dict(sd)
        made.append(e)
        return e

    yield make
    for e in made:
        e.close()
