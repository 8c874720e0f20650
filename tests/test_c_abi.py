"""The C-ABI libraries load and export every function their headers declare
(no GPU compute on this path)."""
import ctypes
import os
import re
import subprocess

import pytest

from alphazero_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mg_[a-z0-9_]+)\s*\(", text)))


def exported(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_cuda_library_exports_header():
    path = build.build_cuda()
    names = declared("minigo_cuda.h")
    assert len(names) >= 15
    missing = [n for n in names if n not in exported(path)]
    assert not missing, missing
    lib = ctypes.CDLL(path)
    for n in names:
        getattr(lib, n)


def test_host_library_exports_header():
    path = build.build_host()
    names = declared("minigo_host.h")
    missing = [n for n in names if n not in exported(path)]
    assert not missing, missing


def _gpu_visible():
    import torch
    return torch.cuda.is_available()


@pytest.mark.skipif(_gpu_visible(), reason="a GPU is visible; the gpu tests cover creation")
def test_create_without_gpu_fails_cleanly():
    from alphazero_b200.engine import CudaEngine
    with pytest.raises(RuntimeError, match="mg_create failed"):
        CudaEngine(0)


def test_pack_states_matches_numpy_and_rejects_non_binary():
    import numpy as np

    from alphazero_b200 import host_lib
    from alphazero_b200.engine import pack_states

    for board, n in ((19, 7), (9, 33), (5, 3)):
        x = host_lib.random_positions(board, n, 4, 250)
        b = pack_states(x)
        assert b.shape == (n, (17 * board * board + 31) // 32)
        ref = np.packbits(x.astype(bool), axis=1, bitorder="little")
        ref = np.pad(ref, ((0, 0), (0, b.shape[1] * 4 - ref.shape[1]))).view("<u4")
        assert np.array_equal(b, ref)
    bad = host_lib.random_positions(9, 2, 4, 60)
    bad[1, 5] = 0.5
    with pytest.raises(ValueError):
        pack_states(bad)
