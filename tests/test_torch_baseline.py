"""Pins the torch restatement of the reference network (oracle/torch_net.py,
the torch-CPU baseline bench.py times) against the golden fixtures, which
the reference's scripts/model.py produced in fp64.  CPU only."""
import numpy as np
import pytest

from conftest import golden_cases, load_golden
from torch_net import TorchNet


@pytest.mark.parametrize("case", golden_cases())
def test_torch_restatement_matches_reference_model(case):
    z, sd = load_golden(case)
    net = TorchNet(sd)
    logits, value = net.forward(z["positions"].astype(np.float32))
    # fp32 torch CPU against the fp64 reference
    assert np.abs(logits - z["logits"]).max() < 1e-4
    assert np.abs(value - z["value"]).max() < 1e-4
