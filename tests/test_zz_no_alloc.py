"""The forward pass that allocates nothing (mg_forward_device_noalloc).

Callers that may not call cudaMalloc or cudaFree once they are running -
both synchronise the device, and some hosts work inside a fixed GPU memory
budget - evaluate positions through this entry point, which takes every
intermediate buffer from a fixed scratch arena compiled into the library.
It runs the same kernels with the same layer wiring as the ordinary device
entry point (mg_forward_device), so its results must be bit-identical to
that entry point's, on consecutive calls that reuse the arena; one case is
also checked against the oracle.  It must refuse batches larger than the
arena holds.  This file is collected last so that a
run stopping at the first failure has run every other test first.
"""
import os

import numpy as np
import pytest

import oracle
from alphazero_b200 import host_lib, weights

pytestmark = pytest.mark.gpu

TOL = {"bf16": 2e-2, "fp32": 1e-4}


@pytest.mark.parametrize("precision,board,filters,blocks,n", [
    ("bf16", 19, 128, 10, 40),
    ("fp32", 9, 64, 3, 24),
    ("bf16", 9, 256, 2, 17),
])
def test_noalloc_forward_matches_device_forward(precision, board, filters, blocks, n):
    import torch
    from alphazero_b200.engine import CudaEngine

    sd = weights.make_state_dict(board, filters, blocks, seed=21, variant="perturbed")
    e = CudaEngine(0, precision=precision, max_batch=64)
    try:
        e.load_state_dict(sd)
        a = board * board + 1
        x = torch.from_numpy(host_lib.random_positions(board, n, 99, 250 if board == 19 else 60)).cuda()
        ref = [torch.empty((n, a), device="cuda"), torch.empty((n,), device="cuda"),
               torch.empty((n, a), device="cuda")]
        e.forward_device(x.data_ptr(), n, ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr())
        e.synchronize()
        outs = []
        for _ in range(2):  # two calls in a row share (and reuse) the arena
            got = [torch.full((n, a), float("nan"), device="cuda"),
                   torch.full((n,), float("nan"), device="cuda"),
                   torch.full((n, a), float("nan"), device="cuda")]
            e.forward_device_noalloc(x.data_ptr(), n, got[0].data_ptr(), got[1].data_ptr(),
                                     got[2].data_ptr())
            outs.append([t.cpu().numpy() for t in got])
        r = [t.cpu().numpy() for t in ref]
        for p, v, l in outs:
            assert np.isfinite(l).all() and np.isfinite(v).all()
            assert np.array_equal(l, r[2]) and np.array_equal(v, r[1]) and np.array_equal(p, r[0])
        # without the optional logits output
        p2 = torch.empty((n, a), device="cuda")
        v2 = torch.empty((n,), device="cuda")
        e.forward_device_noalloc(x.data_ptr(), n, p2.data_ptr(), v2.data_ptr(), None)
        assert np.array_equal(v2.cpu().numpy(), r[1]) and np.array_equal(p2.cpu().numpy(), r[0])
        if precision == "bf16" and filters == 128:
            # and against the oracle, at the tolerance of the parity tests
            _, ov, ol = oracle.EigenOracle(sd).predict_batch(
                x.cpu().numpy(), oracle.CANONICAL, threads=min(16, os.cpu_count() or 1))
            assert np.abs(outs[-1][2] - ol).max() < TOL[precision]
            assert np.abs(outs[-1][1] - ov).max() < TOL[precision]
    finally:
        e.close()


def test_noalloc_rejects_batches_beyond_the_arena():
    import torch
    from alphazero_b200.engine import CudaEngine

    sd = weights.make_state_dict(19, 256, 1, seed=3, variant="init")
    e = CudaEngine(0, precision="bf16", max_batch=512)
    try:
        e.load_state_dict(sd)
        n = 400  # far more 19x19 x 256-channel positions than 32 MiB holds
        x = torch.zeros((n, 17 * 361), device="cuda")
        p = torch.empty((n, 362), device="cuda")
        v = torch.empty((n,), device="cuda")
        with pytest.raises(RuntimeError, match="exceeds the no-allocation scratch arena"):
            e.forward_device_noalloc(x.data_ptr(), n, p.data_ptr(), v.data_ptr(), None)
    finally:
        e.close()
