"""Pins the oracle (the C restatement of src/eigen_engine.cpp) against the
golden fixtures produced by the reference network scripts/model.py in fp64
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest

import oracle
from conftest import golden_cases, load_golden


@pytest.mark.parametrize("case", golden_cases())
def test_oracle_canonical_matches_reference_model(case):
    z, sd = load_golden(case)
    orc = oracle.EigenOracle(sd)
    x = z["positions"].astype(np.float32)
    probs, vals, logits = orc.predict_batch(x, oracle.CANONICAL, threads=4)
    # fp32 CPU arithmetic against fp64: relative 1e-6 level; 1e-4 absolute bound.
    assert np.abs(logits - z["logits"]).max() < 1e-4
    assert np.abs(vals - z["value"]).max() < 1e-4
    ref_p = np.exp(z["logits"] - z["logits"].max(1, keepdims=True))
    ref_p /= ref_p.sum(1, keepdims=True)
    assert np.abs(probs - ref_p).max() < 1e-5


@pytest.mark.parametrize("case", golden_cases())
def test_oracle_literal_matches_eigen_semantics(case):
    z, sd = load_golden(case)
    orc = oracle.EigenOracle(sd)
    x = z["positions"].astype(np.float32)
    _, vals, logits = orc.predict_batch(x, oracle.LITERAL, threads=4)
    assert np.abs(logits - z["logits_literal"]).max() < 1e-4
    assert np.abs(vals - z["value_literal"]).max() < 1e-4


def test_literal_and_canonical_differ():
    # The column-major reading of src/eigen_engine.cpp:211,242 is a different
    # function from the NCHW network; the fixtures must show it.
    z, _ = load_golden("b9c64x6_pert")
    assert np.abs(z["logits"] - z["logits_literal"]).max() > 1e-2


def test_oracle_threads_do_not_change_results():
    z, sd = load_golden("b9c128x10_pert")
    orc = oracle.EigenOracle(sd)
    x = z["positions"].astype(np.float32)
    a = orc.predict_batch(x, oracle.CANONICAL, threads=1)
    b = orc.predict_batch(x, oracle.CANONICAL, threads=3)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)


def test_oracle_reports_missing_tensor():
    _, sd = load_golden("b5c32x3_pert")
    sd = dict(sd)
    del sd["value_fc2.bias"]
    with pytest.raises(RuntimeError, match="Missing tensor: value_fc2.bias"):
        oracle.EigenOracle(sd)
