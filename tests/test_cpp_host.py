"""C++ host code: the batching servers with a fake engine (CPU, also under
ThreadSanitizer) and CudaEngine / ShardedEvaluator on a real GPU."""
import os
import subprocess

import numpy as np
import pytest

from alphazero_b200 import build, host_lib, weights

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPP = os.path.join(ROOT, "tests", "cpp")
HOST = os.path.join(ROOT, "alphazero_b200", "host")


def _compile(src, out, extra=()):
    build.build_cuda()
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-pthread", "-I" + HOST, "-I" + os.path.join(ROOT, "include"),
           os.path.join(CPP, src), os.path.join(HOST, "cuda_engine.cpp"),
           os.path.join(HOST, "gpu_evaluator.cpp"), "-L" + build.LIB, "-lminigo_cuda",
           "-Wl,-rpath," + build.LIB, "-o", out] + list(extra)
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@pytest.mark.parametrize("sanitize", [False, True])
def test_evaluator_with_fake_engine(tmp_path, sanitize):
    exe = str(tmp_path / "test_evaluator")
    _compile("test_evaluator.cpp", exe, ["-fsanitize=thread"] if sanitize else [])
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "evaluator tests passed" in r.stdout
    if sanitize:
        assert "ThreadSanitizer" not in r.stderr


@pytest.mark.gpu
def test_cuda_engine_and_sharded_evaluator(tmp_path):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    sd = weights.make_state_dict(19, 128, 3, seed=5, variant="perturbed")
    model = weights.write_onnx(str(tmp_path / "m.onnx"), sd)
    x = host_lib.random_positions(19, 40, 8, 250)
    x.tofile(str(tmp_path / "states.f32"))
    exe = str(tmp_path / "test_cuda_engine")
    _compile("test_cuda_engine.cpp", exe)
    r = subprocess.run([exe, model, str(tmp_path / "states.f32"), "40", str(tmp_path / "out.f32")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.fromfile(str(tmp_path / "out.f32"), np.float32).reshape(40, 363)
    probs, vals = got[:, :362], got[:, 362]
    op, ov, _ = oracle.EigenOracle(sd).predict_batch(x, oracle.CANONICAL, threads=8)
    assert np.abs(vals - ov).max() < 2e-2
    assert np.abs(probs - op).max() < 2e-2
    assert "sharded ok" in r.stdout


_REF_SEARCH = [os.path.join(build.REFERENCE_TREE, s) for s in build.REFERENCE_SOURCES]


@pytest.mark.skipif(not all(os.path.exists(p) for p in _REF_SEARCH),
                    reason="the reference tree (src/mcts.cpp, src/game.cpp) is not present")
def test_selfplay_loop_with_fake_engines(tmp_path):
    """The self-play measurement loop over the reference's own MCTS (compiled
    from the reference tree) and a two-shard ShardedEvaluator of fake engines."""
    exe = str(tmp_path / "test_selfplay_loop")
    _compile("test_selfplay_loop.cpp", exe,
             ["-DMGB_USE_REFERENCE_HEADERS", "-I" + os.path.join(build.REFERENCE_TREE, "include")]
             + _REF_SEARCH)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "selfplay loop ok" in r.stdout


@pytest.mark.gpu
def test_selfplay_harness_on_gpu(tmp_path):
    """selfplay_cuda (built where the reference tree is present; it travels
    with the package) plays real games on the GPU for a short window."""
    import json

    if not os.path.exists(build.SELFPLAY_BIN):
        pytest.skip("selfplay_cuda was not built (no reference tree at build time)")
    sd = weights.make_state_dict(9, 64, 2, seed=3, variant="init")
    model = weights.write_onnx(str(tmp_path / "m.onnx"), sd)
    r = subprocess.run([build.SELFPLAY_BIN, "--model", model, "--workers", "4", "--search-threads", "4",
                        "--sims", "64", "--max-batch", "64", "--warmup-seconds", "1", "--seconds", "3"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["moves"] > 0 and out["visits_per_s"] > 0
    assert out["nn_positions_per_s"] > 0 and out["failed_batches"] == 0
    assert out["gpu_launches"] > 0


@pytest.mark.skipif(not all(os.path.exists(p) for p in _REF_SEARCH),
                    reason="the reference tree (src/mcts.cpp, src/game.cpp) is not present")
@pytest.mark.parametrize("sanitize", [False, True])
def test_fast_search_against_the_reference_mcts(tmp_path, sanitize):
    """FastSearch / GoPosition against the reference's own MCTS and GoGame:
    identical rules move by move, identical root visits for a single-threaded
    search without noise, the thread pool (also under ThreadSanitizer) and
    the failure path."""
    exe = str(tmp_path / "test_fast_search")
    cmd = ["g++", "-std=c++17", "-O1" if sanitize else "-O2", "-g", "-pthread",
           "-I" + os.path.join(build.REFERENCE_TREE, "include"), "-I" + HOST,
           os.path.join(CPP, "test_fast_search.cpp"), os.path.join(HOST, "fast_search.cpp"),
           os.path.join(HOST, "go_positions.cpp")] + _REF_SEARCH + ["-o", exe]
    if sanitize:
        cmd.append("-fsanitize=thread")
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fast search tests passed" in r.stdout
    if sanitize:
        assert "ThreadSanitizer" not in r.stderr


@pytest.mark.gpu
def test_fast_selfplay_harness_on_gpu(tmp_path):
    """selfplay_cuda --search fast: FastSearch through ShardedEvaluator's
    packed path on the GPU for a short window."""
    import json

    if not os.path.exists(build.SELFPLAY_BIN):
        pytest.skip("selfplay_cuda was not built (no reference tree at build time)")
    sd = weights.make_state_dict(9, 64, 2, seed=3, variant="init")
    model = weights.write_onnx(str(tmp_path / "m.onnx"), sd)
    r = subprocess.run([build.SELFPLAY_BIN, "--model", model, "--search", "fast", "--workers", "4",
                        "--search-threads", "4", "--sims", "64", "--max-batch", "64",
                        "--warmup-seconds", "1", "--seconds", "3"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["search"] == "fast" and out["moves"] > 0 and out["visits_per_s"] > 0
    assert out["failed_batches"] == 0 and out["gpu_launches"] > 0

    # whole games with record files in the reference selfplay's format
    rec_dir = tmp_path / "records"
    rec_dir.mkdir()
    r = subprocess.run([build.SELFPLAY_BIN, "--model", model, "--search", "fast", "--games", "2",
                        "--records", str(rec_dir), "--workers", "2", "--search-threads", "4",
                        "--sims", "32", "--max-batch", "64"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["games"] == 2 and out["records"] == 8 * out["moves"] > 0
    total = 0
    for f in sorted(rec_dir.glob("game_*.bin")):
        data = f.read_bytes()
        n = int(np.frombuffer(data[:4], np.int32)[0])
        rec = 4 + 17 * 81 * 4 + 4 + 82 * 4 + 4  # sizes, state, policy, value
        assert len(data) == 4 + n * rec
        total += n
    assert total == out["records"]


@pytest.mark.skipif(not all(os.path.exists(p) for p in _REF_SEARCH)
                    or not os.path.exists(os.path.join(build.REFERENCE_TREE, "scripts", "train.py")),
                    reason="the reference tree (src/mcts.cpp, scripts/train.py) is not present")
def test_selfplay_records_against_the_reference(tmp_path):
    """Training records: the 8-fold augmentation reproduces the reference's
    own self-play records bit for bit, and a FastSearch game's record file is
    read back by the reference trainer's reader (scripts/train.py:33-55)."""
    import importlib.util
    import sys

    exe = str(tmp_path / "test_selfplay_records")
    cmd = ["g++", "-std=c++17", "-O2", "-g", "-pthread",
           "-I" + os.path.join(build.REFERENCE_TREE, "include"), "-I" + HOST,
           os.path.join(CPP, "test_selfplay_records.cpp"), os.path.join(HOST, "selfplay_records.cpp"),
           os.path.join(HOST, "fast_search.cpp"), os.path.join(HOST, "go_positions.cpp")] + _REF_SEARCH + ["-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    path = str(tmp_path / "game_0.bin")
    r = subprocess.run([exe, path], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "records tests passed" in r.stdout
    count = int(r.stdout.split("records ")[1].split()[0])

    scripts = os.path.join(build.REFERENCE_TREE, "scripts")
    sys.path.insert(0, scripts)
    try:
        spec = importlib.util.spec_from_file_location("reference_train", os.path.join(scripts, "train.py"))
        train = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(train)
    finally:
        sys.path.remove(scripts)
    recs = train.read_selfplay_data(path)
    assert len(recs) == count and count % 8 == 0
    for state, policy, value in recs:
        assert state.shape == (17 * 25,) and policy.shape == (26,)
        assert set(np.unique(state)) <= {0.0, 1.0}
        assert abs(float(policy.sum()) - 1.0) < 1e-5 and value in (-1.0, 0.0, 1.0)
