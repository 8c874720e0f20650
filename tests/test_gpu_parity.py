"""GPU parity: the CUDA engine (through the C ABI) against the golden
fixtures of the reference network and against the oracle.

Tolerances (max |difference| of pre-softmax logits and of values):
  fp32 verification mode   1e-4
  bf16 / fp16 modes        2e-2
"""
import os

import numpy as np
import pytest

import oracle
from alphazero_b200 import host_lib, weights
from conftest import golden_cases, load_golden

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-4, "bf16": 2e-2, "fp16": 2e-2}


def softmax(l):
    e = np.exp(l - l.max(1, keepdims=True))
    return e / e.sum(1, keepdims=True)


@pytest.mark.parametrize("precision", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("case", golden_cases())
def test_engine_matches_reference_golden(gpu_engine_factory, case, precision):
    z, sd = load_golden(case)
    e = gpu_engine_factory(sd, precision)
    x = z["positions"].astype(np.float32)
    p, v, l = e.forward(x)
    tol = TOL[precision]
    assert np.isfinite(l).all() and np.isfinite(v).all()
    assert np.abs(l - z["logits"]).max() < tol
    assert np.abs(v - z["value"]).max() < tol
    assert np.abs(p - softmax(z["logits"])).max() < tol
    assert np.abs(p.sum(1) - 1).max() < 1e-5
    # the engine's probabilities are the softmax of its own logits
    assert np.abs(p - softmax(l.astype(np.float64))).max() < 1e-5


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
@pytest.mark.parametrize("case", ["b9c64x6_pert", "b19c128x10_pert", "b5c32x3_pert"])
def test_eigen_compat_matches_literal_semantics(gpu_engine_factory, case, precision):
    z, sd = load_golden(case)
    e = gpu_engine_factory(sd, precision, eigen_compat=True)
    p, v, l = e.forward(z["positions"].astype(np.float32))
    assert np.abs(l - z["logits_literal"]).max() < TOL[precision]
    assert np.abs(v - z["value_literal"]).max() < TOL[precision]


def _oracle_rows(sd, x, rows):
    orc = oracle.EigenOracle(sd)
    return orc.predict_batch(x[rows], oracle.CANONICAL, threads=min(32, os.cpu_count() or 1))


# Full-size batches of the predict_batch configurations, (board, filters,
# blocks, batch, max random moves, rows checked against the oracle).  Every
# row is checked except on the 20-block 256-filter net, where 256 of the 1024
# rows are (the oracle takes about 8x longer per position there).
FULL_CONFIGS = {
    "b9c64x6_bs16": (9, 64, 6, 16, 60, None),
    "b9c128x10_bs256": (9, 128, 10, 256, 60, None),
    "b19c128x10_bs512": (19, 128, 10, 512, 250, None),
    "b19c256x20_bs1024": (19, 256, 20, 1024, 250, 256),
}
# Weight sets: exactly the network bench.py times (seed 0, export_onnx --init
# distributions) on its rank-0 positions (seed 1000), and a perturbed-BN set
# whose logits are O(1), on other positions.
WEIGHT_SETS = {"bench": (0, "init", 1000), "perturbed": (11, "perturbed", 2024)}
_ORACLE_CACHE = {}


def _full_case(cfg, wset):
    board, filters, blocks, n, max_moves, nrows = FULL_CONFIGS[cfg]
    wseed, variant, pseed = WEIGHT_SETS[wset]
    key = (cfg, wset)
    if key not in _ORACLE_CACHE:
        sd = weights.make_state_dict(board, filters, blocks, seed=wseed, variant=variant)
        x = host_lib.random_positions(board, n, pseed, max_moves)
        rows = np.arange(n) if nrows is None else np.sort(
            np.random.default_rng(0).choice(n, nrows, replace=False))
        if nrows is not None:
            rows[0], rows[-1] = 0, n - 1
        _, ov, ol = _oracle_rows(sd, x, rows)
        _ORACLE_CACHE[key] = (sd, x, rows, ov, ol)
    return _ORACLE_CACHE[key]


def _report(entry):
    """Appends one parity record to $MGB_PARITY_REPORT (JSON lines) if set."""
    import json

    path = os.environ.get("MGB_PARITY_REPORT")
    print("parity", entry)
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(entry) + "\n")


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
@pytest.mark.parametrize("wset", sorted(WEIGHT_SETS))
@pytest.mark.parametrize("cfg", list(FULL_CONFIGS))
def test_full_size_batches(gpu_engine_factory, cfg, wset, precision):
    sd, x, rows, ov, ol = _full_case(cfg, wset)
    n = len(x)
    e = gpu_engine_factory(sd, precision, max_batch=n)
    p, v, l = e.forward(x)
    # size-independent properties over the whole batch
    assert np.isfinite(l).all() and np.isfinite(v).all()
    assert np.abs(p.sum(1) - 1).max() < 1e-5
    assert (np.abs(v) <= 1).all()
    # the checked rows against the oracle (fp32 C restatement of the reference engine)
    dl = np.abs(l[rows] - ol)
    dv = np.abs(v[rows] - ov)
    top1 = float((l[rows].argmax(1) == ol.argmax(1)).mean())
    # top-1 agreement among rows whose oracle top-2 logits are at least
    # 2x the tolerance apart (closer pairs may swap within tolerance)
    srt = np.sort(ol, axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 2 * TOL[precision]
    top1_clear = float((l[rows][clear].argmax(1) == ol[clear].argmax(1)).mean()) if clear.any() else None
    _report({"config": cfg, "weights": wset, "precision": precision, "rows": int(len(rows)),
             "batch": n, "max_dlogit": float(dl.max()), "max_dvalue": float(dv.max()),
             "logit_std": float(ol.std()), "max_dlogit_over_std": float(dl.max() / ol.std()),
             "top1_agreement": top1, "top1_agreement_clear": top1_clear,
             "clear_rows": int(clear.sum())})
    assert dl.max() < TOL[precision], float(dl.max())
    assert dv.max() < TOL[precision], float(dv.max())
    if top1_clear is not None:
        assert top1_clear == 1.0
    # positions are independent: permuting the batch permutes the results
    if cfg == "b19c128x10_bs512" and precision == "bf16":
        perm = np.random.default_rng(1).permutation(n)
        p2, v2, l2 = e.forward(x[perm])
        assert np.array_equal(l2, l[perm]) and np.array_equal(v2, v[perm])


def test_b20c256_fp32_verification_pass_on_64_positions(gpu_engine_factory):
    """The 19x19 20-block 256-filter network's fp32 verification pass: 64
    seeded random-playout positions, every row against the oracle, fp32 mode
    at 1e-4 and the bf16 default at 2e-2 on the same batch."""
    sd = weights.make_state_dict(19, 256, 20, seed=13, variant="perturbed")
    x = host_lib.random_positions(19, 64, 77, 250)
    _, ov, ol = oracle.EigenOracle(sd).predict_batch(x, oracle.CANONICAL,
                                                     threads=min(32, os.cpu_count() or 1))
    for precision in ("fp32", "bf16"):
        e = gpu_engine_factory(sd, precision, max_batch=64)
        p, v, l = e.forward(x)
        assert np.abs(p.sum(1) - 1).max() < 1e-5
        assert np.abs(l - ol).max() < TOL[precision], (precision, float(np.abs(l - ol).max()))
        assert np.abs(v - ov).max() < TOL[precision], (precision, float(np.abs(v - ov).max()))


def test_ragged_and_chunked_batches(gpu_engine_factory):
    z, sd = load_golden("b19c128x10_pert")
    e = gpu_engine_factory(sd, "bf16", max_batch=64)
    x = host_lib.random_positions(19, 150, 77, 250)
    _, v_all, l_all = e.forward(x)  # 150 > max batch 64: three chunks
    for n in (1, 3, 17, 64, 65, 129):
        _, v, l = e.forward(x[:n])
        assert np.array_equal(l, l_all[:n]) and np.array_equal(v, v_all[:n]), n
    rows = np.array([0, 63, 64, 127, 128, 149])
    _, ov, ol = _oracle_rows(sd, x, rows)
    assert np.abs(l_all[rows] - ol).max() < TOL["bf16"]


def test_duplicate_positions_identical(gpu_engine_factory):
    _, sd = load_golden("b9c64x6_pert")
    e = gpu_engine_factory(sd, "bf16")
    x = np.repeat(host_lib.random_positions(9, 1, 5, 60), 37, axis=0)
    _, v, l = e.forward(x)
    assert (l == l[0]).all() and (v == v[0]).all()


def test_interface_semantics(gpu_engine_factory, tmp_path):
    z, sd = load_golden("b9c64x6_init")
    path = weights.write_onnx(str(tmp_path / "m.onnx"), sd)
    from alphazero_b200.engine import CudaEngine

    e = CudaEngine(0, precision="fp32")
    try:
        with pytest.raises(RuntimeError, match="no model loaded"):
            e.predict(np.zeros(17 * 81, np.float32))
        e.load_model(path)
        assert (e.board_size, e.input_channels, e.num_filters, e.num_res_blocks) == (9, 17, 64, 6)
        assert e.backend_name() == "cuda"
        assert e.predict_batch([]) == []
        x = z["positions"].astype(np.float32)
        batch = e.predict_batch(list(x))
        for i in range(len(x)):
            pol, val = e.predict(x[i])
            assert np.allclose(pol, batch[i][0], atol=1e-6) and abs(val - batch[i][1]) < 1e-6
            assert abs(val - z["value"][i]) < 1e-4
        with pytest.raises(RuntimeError, match="Cannot open model file"):
            e.load_model(str(tmp_path / "missing.onnx"))
        bad = dict(sd)
        del bad["res_blocks.0.bn2.running_var"]
        with pytest.raises(RuntimeError, match="Missing tensor: res_blocks.0.bn2.running_var"):
            e.load_state_dict(bad)
    finally:
        e.close()


def test_pinned_pageable_and_device_inputs_agree(gpu_engine_factory):
    import torch

    z, sd = load_golden("b19c128x10_pert")
    e = gpu_engine_factory(sd, "bf16")
    x = host_lib.random_positions(19, 40, 9, 250)
    _, v0, l0 = e.forward(x)
    pinned = torch.from_numpy(x).pin_memory()
    _, v1, l1 = e.forward(pinned.numpy())
    assert np.array_equal(l0, l1) and np.array_equal(v0, v1)
    dx = torch.from_numpy(x).cuda()
    dp = torch.empty((40, 362), device="cuda")
    dv = torch.empty((40,), device="cuda")
    dl = torch.empty((40, 362), device="cuda")
    e.forward_device(dx.data_ptr(), 40, dp.data_ptr(), dv.data_ptr(), dl.data_ptr())
    e.synchronize()
    assert np.array_equal(dl.cpu().numpy(), l0) and np.array_equal(dv.cpu().numpy(), v0)


def test_precision_switch_round_trip(gpu_engine_factory):
    z, sd = load_golden("b9c128x10_pert")
    x = z["positions"].astype(np.float32)
    e = gpu_engine_factory(sd, "bf16")
    _, _, l_bf = e.forward(x)
    e.set_precision("fp32")
    _, _, l_32 = e.forward(x)
    e.set_precision("bf16")
    _, _, l_bf2 = e.forward(x)
    assert np.array_equal(l_bf, l_bf2)
    assert np.abs(l_32 - z["logits"]).max() < TOL["fp32"]


@pytest.mark.parametrize("eigen_compat", [False, True])
def test_packed_wire_format_matches_fp32_planes(gpu_engine_factory, eigen_compat):
    from alphazero_b200.engine import pack_states

    _, sd = load_golden("b19c128x10_pert")
    e = gpu_engine_factory(sd, "bf16", eigen_compat=eigen_compat, max_batch=64)
    x = host_lib.random_positions(19, 150, 31, 250)  # 150 > max batch: chunked
    bits = pack_states(x)
    assert bits.shape[1] == e.words_per_position()
    p1, v1, l1 = e.forward(x)
    p2, v2, l2 = e.forward_packed(bits, len(x), want_logits=True)
    assert np.array_equal(l1, l2) and np.array_equal(v1, v2) and np.array_equal(p1, p2)


@pytest.mark.parametrize("board,filters,blocks,n", [
    (19, 128, 10, 512), (19, 128, 10, 300), (9, 128, 10, 1024), (19, 128, 10, 24), (9, 128, 10, 5),
    (9, 64, 6, 16), (19, 64, 6, 200), (9, 256, 3, 17), (19, 256, 4, 64), (19, 256, 20, 1024)])
def test_persistent_trunk_matches_per_layer_launches(gpu_engine_factory, monkeypatch, board, filters,
                                                     blocks, n):
    """The all-layers persistent launch (per-CTA progress counters between
    layers) against one launch per layer: bit-identical.  128 channels: the
    same kernel (conv_pix.cu), as one launch at every batch, down to a
    single tile on a few CTAs (9x9 batch 5).  64 / 256 channels
    (conv_tc.cu): the persistent launch tiles every layer with all output
    channels, the per-layer launches may split them (small batches); the
    sums do not depend on that."""
    sd = weights.make_state_dict(board, filters, blocks, seed=5, variant="perturbed")
    x = host_lib.random_positions(board, n, 99, 250 if board == 19 else 60)
    env = "MG_PIX_TRUNK" if filters == 128 else "MG_TC_TRUNK"
    monkeypatch.setenv(env, "0")
    per_layer = gpu_engine_factory(sd, "bf16", max_batch=max(n, 64))
    monkeypatch.setenv(env, "1")
    trunk = gpu_engine_factory(sd, "bf16", max_batch=max(n, 64))
    monkeypatch.delenv(env)
    assert trunk.launches_per_forward(n) < per_layer.launches_per_forward(n)
    p0, v0, l0 = per_layer.forward(x)
    for _ in range(3):  # repeated launches reuse the progress counters
        p1, v1, l1 = trunk.forward(x)
        assert np.array_equal(l0, l1) and np.array_equal(v0, v1) and np.array_equal(p0, p1)
    rows = np.array([0, n // 2, n - 1])
    _, ov, ol = _oracle_rows(sd, x, rows)
    assert np.abs(l1[rows] - ol).max() < TOL["bf16"]
    assert np.abs(v1[rows] - ov).max() < TOL["bf16"]


def test_submitted_batches_match_synchronous_calls(gpu_engine_factory):
    """mg_submit_packed / mg_wait_submitted (the batching server's pipelined
    path): two submissions in flight on one engine, waited for in order,
    give exactly mg_forward_packed's results; pageable buffers are refused."""
    import torch
    from alphazero_b200.engine import pack_states

    _, sd = load_golden("b19c128x10_pert")
    e = gpu_engine_factory(sd, "bf16", max_batch=256)
    xs = [host_lib.random_positions(19, n, 60 + n, 250) for n in (256, 100, 7, 256)]
    ref = [e.forward_packed(pack_states(x), len(x)) for x in xs]

    def pinned(shape, dtype):
        t = torch.empty(shape, dtype=dtype).pin_memory()
        return t.numpy()

    bufs = []
    for x in xs:
        b = pinned((len(x), e.words_per_position()), torch.int32).view(np.uint32)
        b[:] = pack_states(x)
        bufs.append((b, pinned((len(x), 362), torch.float32), pinned((len(x),), torch.float32)))
    tickets = [e.submit_packed(bufs[0][0], len(xs[0]), bufs[0][1], bufs[0][2])]
    for i in range(1, len(xs)):
        tickets.append(e.submit_packed(bufs[i][0], len(xs[i]), bufs[i][1], bufs[i][2]))
        e.wait_submitted(tickets[i - 1])  # at most two outstanding
    e.wait_submitted(tickets[-1])
    for (p0, v0, _), (_, p1, v1) in zip(ref, bufs):
        assert np.array_equal(p0, p1) and np.array_equal(v0, v1)
    with pytest.raises(RuntimeError):
        e.submit_packed(pack_states(xs[2]), len(xs[2]), np.empty((7, 362), np.float32),
                        np.empty((7,), np.float32))


@pytest.mark.parametrize("board,n", [(9, 256), (9, 1024), (9, 17), (9, 5), (5, 64), (13, 100)])
def test_whole_frame_trunk_matches_the_unpadded_layout(gpu_engine_factory, monkeypatch, board, n):
    """MG_FRAME_TRUNK=1 on small boards (frame of at most 256 rows): the
    engine pads the frame stride to whole 16-row chunks and runs the
    128-channel trunk as one launch of CTAs that own whole frames and wait
    only on their own tiles.  Against the unpadded layout with the usual
    schedule: bit-identical, on repeated calls."""
    sd = weights.make_state_dict(board, 128, 10, seed=8, variant="perturbed")
    x = host_lib.random_positions(board, n, 31, 60 if board < 19 else 250)
    monkeypatch.setenv("MG_FRAME_TRUNK", "0")
    plain = gpu_engine_factory(sd, "bf16", max_batch=max(n, 64))
    monkeypatch.setenv("MG_FRAME_TRUNK", "1")  # an option, off by default
    framed = gpu_engine_factory(sd, "bf16", max_batch=max(n, 64))
    monkeypatch.delenv("MG_FRAME_TRUNK")
    assert framed.launches_per_forward(n) == 4  # staging, trunk, FC, finish
    p0, v0, l0 = plain.forward(x)
    for _ in range(3):
        p1, v1, l1 = framed.forward(x)
        assert np.array_equal(l0, l1) and np.array_equal(v0, v1) and np.array_equal(p0, p1)
    rows = np.array([0, n // 2, n - 1])
    _, ov, ol = _oracle_rows(sd, x, rows)
    assert np.abs(l1[rows] - ol).max() < TOL["bf16"]
