"""The backend plugged into the reference itself: its own `benchmark` and
`selfplay` binaries (src/main_benchmark.cpp, src/main_selfplay.cpp), built by
its own CMake with -DMINIGO_BACKEND=cuda from a copy of its tree with
alphazero_b200/integration/cuda_backend.patch applied
(alphazero_b200/build.py: build_reference_binaries).  The binaries load the
model through the reference's onnx_parser and run create_engine's CudaEngine
unchanged; the GPU tests check that they run end to end on the GPU and report
backend "cuda"."""
import os
import struct
import subprocess

import numpy as np
import pytest

from alphazero_b200 import build, weights

needs_binaries = pytest.mark.skipif(
    not (os.path.exists(build.REF_BENCHMARK_BIN) and os.path.exists(build.REF_SELFPLAY_BIN)),
    reason="reference binaries not built (no reference tree or cmake at build time)")


def _model(tmp_path, board=9, filters=64, blocks=6):
    sd = weights.make_state_dict(board, filters, blocks, seed=0, variant="init")
    return weights.write_onnx(str(tmp_path / "model.onnx"), sd)


def _run(args, timeout=600):
    return subprocess.run(args, capture_output=True, text=True, timeout=timeout)


@pytest.mark.skipif(not os.path.exists(os.path.join(build.REFERENCE_TREE, "CMakeLists.txt")),
                    reason="reference tree absent")
def test_patch_applies_to_the_reference_tree():
    r = _run(["patch", "-p1", "--dry-run", "-d", build.REFERENCE_TREE, "-i", build.PATCH])
    assert r.returncode == 0, r.stdout + r.stderr


@needs_binaries
def test_reference_benchmark_without_gpu_has_no_cpu_fallback(tmp_path):
    """On a host without a GPU the cuda backend's engine cannot be created,
    and the reference benchmark reports that it has no model (its own
    handling of a failed create_engine) instead of computing on the CPU."""
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    r = _run([build.REF_BENCHMARK_BIN, "--model", _model(tmp_path), "--games", "0"])
    assert r.returncode == 0, r.stderr
    assert "No model loaded" in r.stdout and "Backend: cuda" not in r.stdout


@pytest.mark.gpu
@needs_binaries
def test_reference_benchmark_runs_on_the_cuda_backend(tmp_path):
    r = _run([build.REF_BENCHMARK_BIN, "--model", _model(tmp_path), "--nn-iters", "200",
              "--sims", "64", "--games", "1", "--search-threads", "8"])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    out = r.stdout
    print(out)
    assert "Backend: cuda" in out
    # section 3 (predict_batch throughput, src/main_benchmark.cpp:129-157)
    rates = [int(line.split()[-2]) for line in out.splitlines()
             if line.strip().startswith("batch=") and line.strip().endswith("states/s")]
    assert len(rates) == 5 and all(v > 0 for v in rates), out
    assert "First move:" in out and "Total:" in out


@pytest.mark.gpu
@needs_binaries
def test_reference_selfplay_writes_records_on_the_cuda_backend(tmp_path):
    outdir = tmp_path / "games"
    r = _run([build.REF_SELFPLAY_BIN, "--model", _model(tmp_path), "--games", "2",
              "--threads", "2", "--search-threads", "8", "--sims", "48",
              "--output", str(outdir)])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "Backend:          cuda" in r.stdout
    for g in range(2):
        data = (outdir / f"game_{g}.bin").read_bytes()
        (n,) = struct.unpack_from("<i", data, 0)
        assert n > 0 and n % 8 == 0  # 8-fold augmented
        off = 4
        for _ in range(n):  # the record layout of src/main_selfplay.cpp:17-32
            (ss,) = struct.unpack_from("<i", data, off)
            state = np.frombuffer(data, np.float32, ss, off + 4)
            off += 4 + 4 * ss
            (ps,) = struct.unpack_from("<i", data, off)
            pol = np.frombuffer(data, np.float32, ps, off + 4)
            off += 4 + 4 * ps
            (val,) = struct.unpack_from("<f", data, off)
            off += 4
            assert ss == 17 * 81 and ps == 82
            assert set(np.unique(state)) <= {0.0, 1.0}
            assert abs(float(pol.sum()) - 1.0) < 1e-4 and val in (-1.0, 0.0, 1.0)
        assert off == len(data)
