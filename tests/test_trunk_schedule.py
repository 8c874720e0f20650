"""The cross-CTA schedule of the persistent trunk launches
(alphazero_b200/csrc/trunk_schedule.cuh), checked on the CPU with the
header's own index functions: over 880 launch geometries of both trunk
kernels, every tile waits for every tile of the layer before that produced
a row it reads or read a row it overwrites, never for a later one, and the
waits can always be met (tests/cpp/test_trunk_schedule.cu)."""
import os
import shutil
import subprocess

import pytest

from alphazero_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _nvcc():
    if os.path.exists(build.NVCC):
        return build.NVCC
    return shutil.which("nvcc")


@pytest.mark.skipif(_nvcc() is None, reason="nvcc not found")
def test_trunk_schedule_covers_every_dependency(tmp_path):
    exe = str(tmp_path / "test_trunk_schedule")
    r = subprocess.run([_nvcc(), build.GENCODE, "-O2", "-std=c++17", "-o", exe,
                        os.path.join(ROOT, "tests", "cpp", "test_trunk_schedule.cu")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failures" in r.stdout
