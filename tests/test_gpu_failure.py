"""Failure detection on the GPU without a GPU fault.

Every wait in the kernels is bounded (2 s of %globaltimer); on expiry the
waiting thread records an error code in the engine's status word, the kernel
drains its copies and MMAs, frees TMEM and ends, and the host reports the
status as MG_E_DEVICE.  The test hook MG_TEST_WITHHOLD_PROGRESS=k makes CTA k
of the persistent trunk launch never publish its finished tiles (a flag that
nothing sets): the CTAs that need those tiles, k itself included, give up
with kErrWaitDep (5).  The context stays usable: a second engine on the same
device then computes the network normally.
"""
import os
import time

import numpy as np
import pytest

import oracle
from alphazero_b200 import host_lib, weights

pytestmark = pytest.mark.gpu


def test_withheld_progress_is_reported_and_the_context_recovers(gpu_engine_factory, monkeypatch):
    sd = weights.make_state_dict(19, 128, 2, seed=3, variant="perturbed")
    # 19x19 batch 512: six tiles per CTA, so the five layers run as one
    # persistent launch whose CTAs wait on one another's progress.
    x = host_lib.random_positions(19, 512, 7, 250)
    monkeypatch.setenv("MG_TEST_WITHHOLD_PROGRESS", "3")
    stalled = gpu_engine_factory(sd, "bf16")
    for _ in range(2):  # the status is per call; the engine fails the same way again
        t0 = time.time()
        with pytest.raises(RuntimeError, match=r"gave up waiting \(device status 5\)"):
            stalled.forward(x)
        assert time.time() - t0 < 60
    monkeypatch.delenv("MG_TEST_WITHHOLD_PROGRESS")
    healthy = gpu_engine_factory(sd, "bf16")
    p, v, l = healthy.forward(x)
    assert np.isfinite(l).all() and np.abs(p.sum(1) - 1).max() < 1e-5
    rows = np.array([0, 255, 511])
    orc = oracle.EigenOracle(sd)
    _, ov, ol = orc.predict_batch(x[rows], oracle.CANONICAL, threads=min(8, os.cpu_count() or 1))
    assert np.abs(l[rows] - ol).max() < 2e-2
    assert np.abs(v[rows] - ov).max() < 2e-2


def test_withheld_progress_in_the_64_256_channel_trunk(gpu_engine_factory, monkeypatch):
    """The same failure path in the persistent trunk launch of the 64/256-
    channel kernel (conv_tc.cu, MG_TC_TRUNK=1): 19x19, 256 filters, 2 blocks,
    batch 64."""
    sd = weights.make_state_dict(19, 256, 2, seed=4, variant="perturbed")
    x = host_lib.random_positions(19, 64, 8, 250)
    monkeypatch.setenv("MG_TC_TRUNK", "1")  # the persistent launch (off by default)
    monkeypatch.setenv("MG_TEST_WITHHOLD_PROGRESS", "3")
    stalled = gpu_engine_factory(sd, "bf16", max_batch=64)
    for _ in range(2):
        t0 = time.time()
        with pytest.raises(RuntimeError, match=r"gave up waiting \(device status 5\)"):
            stalled.forward(x)
        assert time.time() - t0 < 60
    monkeypatch.delenv("MG_TEST_WITHHOLD_PROGRESS")
    healthy = gpu_engine_factory(sd, "bf16", max_batch=64)
    p, v, l = healthy.forward(x)
    rows = np.array([0, 31, 63])
    orc = oracle.EigenOracle(sd)
    _, ov, ol = orc.predict_batch(x[rows], oracle.CANONICAL, threads=min(8, os.cpu_count() or 1))
    assert np.abs(l[rows] - ol).max() < 2e-2
    assert np.abs(v[rows] - ov).max() < 2e-2
