"""Builds the package's native libraries in-tree (alphazero_b200/lib/).

  libminigo_cuda.so  CUDA kernels for sm_100a + engine + C ABI
                     (include/minigo_cuda.h); nvcc, static cudart.
  libminigo_host.so  CPU-only helpers (include/minigo_host.h): position
                     generator and ONNX reader; g++.
  libminigo_evaluator.so  CudaEngine / GpuEvaluator / ShardedEvaluator
                     (the reference's C++ interfaces over the C ABI) and
                     FastSearch (the reference's MCTS at a lower host cost).
  selfplay_cuda      end-to-end self-play harness: the reference's own
                     search (src/mcts.cpp, src/game.cpp, with its model
                     loader src/onnx_loader.cpp) compiled unmodified
                     from the reference tree with this backend's evaluator;
                     built only where that tree is present (the binary then
                     travels with the package).

  ref_benchmark_cuda, ref_selfplay_cuda
                     the reference's own `benchmark` and `selfplay` binaries
                     (src/main_benchmark.cpp, src/main_selfplay.cpp) built by
                     the reference's CMake with -DMINIGO_BACKEND=cuda: a copy
                     of the reference tree in a temporary directory with
                     integration/cuda_backend.patch applied (the factory and
                     CMake changes a maintainer makes); built only where that
                     tree and cmake are present.

Run as ``python -m alphazero_b200.build``.  Rebuilds a library only when one
of its sources is newer than it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "lib")
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
INCLUDE = os.path.join(ROOT, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
GENCODE = "-gencode=arch=compute_100a,code=sm_100a"

CUDA_SOURCES = [
    os.path.join(CSRC, "conv_tc.cu"),
    os.path.join(CSRC, "conv_pix.cu"),
    os.path.join(CSRC, "conv_simt.cu"),
    os.path.join(CSRC, "stage_heads.cu"),
    os.path.join(CSRC, "engine.cu"),
    os.path.join(HOST, "net_weights.cpp"),
    os.path.join(HOST, "onnx_reader.cpp"),
]
CUDA_HEADERS = [
    os.path.join(CSRC, "kernels.cuh"),
    os.path.join(CSRC, "ptx_sm100.cuh"),
    os.path.join(CSRC, "trunk_schedule.cuh"),
    os.path.join(HOST, "net_weights.h"),
    os.path.join(HOST, "onnx_reader.h"),
    os.path.join(INCLUDE, "minigo_cuda.h"),
]
HOST_SOURCES = [
    os.path.join(HOST, "go_positions.cpp"),
    os.path.join(HOST, "onnx_reader.cpp"),
    os.path.join(HOST, "c_api_host.cpp"),
]
HOST_HEADERS = [
    os.path.join(HOST, "go_positions.h"),
    os.path.join(HOST, "onnx_reader.h"),
    os.path.join(INCLUDE, "minigo_host.h"),
]

EVAL_SOURCES = [
    os.path.join(HOST, "cuda_engine.cpp"),
    os.path.join(HOST, "gpu_evaluator.cpp"),
    os.path.join(HOST, "fast_search.cpp"),
    os.path.join(HOST, "go_positions.cpp"),
    os.path.join(HOST, "selfplay_records.cpp"),
]
EVAL_HEADERS = [
    os.path.join(HOST, "cuda_engine.h"),
    os.path.join(HOST, "gpu_evaluator.h"),
    os.path.join(HOST, "minigo_api.h"),
    os.path.join(HOST, "packed_evaluator.h"),
    os.path.join(HOST, "fast_search.h"),
    os.path.join(HOST, "go_positions.h"),
    os.path.join(HOST, "selfplay_records.h"),
    os.path.join(INCLUDE, "minigo_cuda.h"),
]

SELFPLAY_SOURCES = [
    os.path.join(HOST, "selfplay_main.cpp"),
    os.path.join(HOST, "cuda_engine.cpp"),
    os.path.join(HOST, "gpu_evaluator.cpp"),
    os.path.join(HOST, "fast_search.cpp"),
    os.path.join(HOST, "go_positions.cpp"),
    os.path.join(HOST, "selfplay_records.cpp"),
]
SELFPLAY_HEADERS = EVAL_HEADERS + [os.path.join(HOST, h) for h in (
    "selfplay_loop.h", "selfplay_window.h", "fast_selfplay.h", "fast_search.h", "go_positions.h",
    "packed_evaluator.h", "selfplay_records.h")]
# The reference tree the self-play harness compiles src/mcts.cpp and
# src/game.cpp from (read in place, never copied).  The one setting for its
# location: the MGB_REFERENCE_TREE environment variable, with this default;
# the oracle's build and the fixture generator read it from here.
REFERENCE_TREE = os.environ.get("MGB_REFERENCE_TREE", "/root/reference")
REFERENCE_SOURCES = ["src/mcts.cpp", "src/game.cpp", "src/onnx_loader.cpp"]

CUDA_LIB = os.path.join(LIB, "libminigo_cuda.so")
HOST_LIB = os.path.join(LIB, "libminigo_host.so")
EVAL_LIB = os.path.join(LIB, "libminigo_evaluator.so")
SELFPLAY_BIN = os.path.join(LIB, "selfplay_cuda")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def build_host(force: bool = False) -> str:
    os.makedirs(LIB, exist_ok=True)
    if force or _stale(HOST_LIB, HOST_SOURCES + HOST_HEADERS):
        tmp = HOST_LIB + ".tmp"
        _run(["g++", "-std=c++17", "-O3", "-fPIC", "-shared", "-Wall", "-Wextra",
              "-o", tmp] + HOST_SOURCES + ["-lpthread"])
        os.replace(tmp, HOST_LIB)
    return HOST_LIB


def build_cuda(force: bool = False) -> str:
    os.makedirs(LIB, exist_ok=True)
    if force or _stale(CUDA_LIB, CUDA_SOURCES + CUDA_HEADERS):
        if not os.path.exists(NVCC) and shutil.which("nvcc") is None:
            raise RuntimeError("nvcc not found; set CUDA_HOME")
        nvcc = NVCC if os.path.exists(NVCC) else "nvcc"
        tmp = CUDA_LIB + ".tmp"
        _run([nvcc, GENCODE, "-O3", "-lineinfo", "-std=c++17", "-shared",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "-o", tmp] + CUDA_SOURCES)
        os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_evaluator(force: bool = False) -> str:
    """C++ InferenceEngine / BatchEvaluator classes over the C ABI (host
    code only; links libminigo_cuda.so)."""
    cuda = build_cuda(force)
    if force or _stale(EVAL_LIB, EVAL_SOURCES + EVAL_HEADERS + [cuda]):
        tmp = EVAL_LIB + ".tmp"
        _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-pthread",
              "-o", tmp] + EVAL_SOURCES +
             ["-L" + LIB, "-lminigo_cuda", "-Wl,-rpath,$ORIGIN"])
        os.replace(tmp, EVAL_LIB)
    return EVAL_LIB


def build_selfplay(force: bool = False) -> str | None:
    """The self-play harness (selfplay_main.cpp).  Needs the reference
    tree's search sources; returns None (and keeps any earlier build) where
    the tree is absent."""
    ref = [os.path.join(REFERENCE_TREE, s) for s in REFERENCE_SOURCES]
    if not all(os.path.exists(r) for r in ref):
        return SELFPLAY_BIN if os.path.exists(SELFPLAY_BIN) else None
    cuda = build_cuda(force)
    if force or _stale(SELFPLAY_BIN, SELFPLAY_SOURCES + SELFPLAY_HEADERS + ref + [cuda]):
        tmp = SELFPLAY_BIN + ".tmp"
        _run(["g++", "-std=c++17", "-O2", "-pthread", "-Wall", "-DMGB_USE_REFERENCE_HEADERS",
              "-I" + os.path.join(REFERENCE_TREE, "include"), "-I" + HOST, "-o", tmp] +
             SELFPLAY_SOURCES + ref + ["-L" + LIB, "-lminigo_cuda", "-Wl,-rpath,$ORIGIN"])
        os.replace(tmp, SELFPLAY_BIN)
    return SELFPLAY_BIN


PATCH = os.path.join(PKG, "integration", "cuda_backend.patch")
REF_BENCHMARK_BIN = os.path.join(LIB, "ref_benchmark_cuda")
REF_SELFPLAY_BIN = os.path.join(LIB, "ref_selfplay_cuda")
# What the reference's minigo_core target compiles with the cuda backend.
REFERENCE_BUILD_FILES = ["CMakeLists.txt", "src/inference_engine.cpp", "src/game.cpp",
                         "src/onnx_loader.cpp", "src/nn_evaluator.cpp", "src/mcts.cpp",
                         "src/main_benchmark.cpp", "src/main_selfplay.cpp"]


def build_reference_binaries(force: bool = False) -> list[str]:
    """The reference's `benchmark` and `selfplay` targets built by its own
    CMake with -DMINIGO_BACKEND=cuda, from a temporary copy of the reference
    tree with integration/cuda_backend.patch applied.  The reference tree is
    only read.  Returns the binaries (none where the tree or cmake is absent;
    an earlier build is kept)."""
    have = [p for p in (REF_BENCHMARK_BIN, REF_SELFPLAY_BIN) if os.path.exists(p)]
    ref = [os.path.join(REFERENCE_TREE, f) for f in REFERENCE_BUILD_FILES]
    cmake = shutil.which("cmake")
    if cmake is None or shutil.which("patch") is None or not all(os.path.exists(r) for r in ref):
        return have
    cuda = build_cuda(force)
    deps = ref + [PATCH, cuda] + [os.path.join(HOST, f) for f in (
        "cuda_engine.cpp", "cuda_engine.h", "gpu_evaluator.cpp", "gpu_evaluator.h", "minigo_api.h",
        "packed_evaluator.h")] + [os.path.join(INCLUDE, "minigo_cuda.h")]
    if not force and not _stale(REF_BENCHMARK_BIN, deps) and not _stale(REF_SELFPLAY_BIN, deps):
        return have
    import tempfile

    with tempfile.TemporaryDirectory(prefix="mgb_reference_build_") as tmp:
        tree = os.path.join(tmp, "src")
        shutil.copytree(REFERENCE_TREE, tree, symlinks=True,
                        ignore=shutil.ignore_patterns(".git", "build", "third_party", "*.onnx",
                                                      "selfplay_data"))
        for root, dirs, files in os.walk(tree):  # the copy must be writable
            for n in dirs + files:
                p = os.path.join(root, n)
                if not os.path.islink(p):
                    os.chmod(p, os.stat(p).st_mode | 0o200)
        _run(["patch", "-p1", "-s", "-d", tree, "-i", PATCH])
        bld = os.path.join(tmp, "build")
        # RelWithDebInfo with portable flags: the reference's Release flags
        # are -march=native, which would tie the binaries to this host's CPU.
        _run([cmake, "-S", tree, "-B", bld, "-DMINIGO_BACKEND=cuda", "-DMGB_ROOT=" + ROOT,
              "-DCMAKE_BUILD_TYPE=RelWithDebInfo",
              "-DCMAKE_CXX_FLAGS_RELWITHDEBINFO=-O3 -march=x86-64-v3 -DNDEBUG",
              "-DCMAKE_BUILD_RPATH=$ORIGIN"])
        _run([cmake, "--build", bld, "--target", "benchmark", "selfplay", "-j",
              str(os.cpu_count() or 4)])
        for name, dst in (("benchmark", REF_BENCHMARK_BIN), ("selfplay", REF_SELFPLAY_BIN)):
            shutil.copy2(os.path.join(bld, name), dst + ".tmp")
            os.replace(dst + ".tmp", dst)
    return [REF_BENCHMARK_BIN, REF_SELFPLAY_BIN]


def build_all(force: bool = False) -> list[str]:
    out = [build_host(force), build_cuda(force), build_evaluator(force)]
    sp = build_selfplay(force)
    if sp is not None:
        out.append(sp)
    out += build_reference_binaries(force)
    return out


if __name__ == "__main__":
    for p in build_all(force="--force" in sys.argv):
        print(p)
