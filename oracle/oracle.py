"""ORACLE - test infrastructure only.

ctypes bindings of the parity checker and of the reference harness:
  * ``EigenOracle``: oracle/liboracle.so, the C restatement of
    src/eigen_engine.cpp (eigen_restated.c);
  * ``ref_random_positions`` / ``ref_read_onnx``: oracle/_ref/libref_harness.so,
    the reference's own src/game.cpp and src/onnx_loader.cpp.
Only tests, the smoke check and bench.py's CPU-baseline leg use this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_harness.so")
CANONICAL, LITERAL = 0, 1


def reference_tree() -> str:
    """The reference tree's location: alphazero_b200.build.REFERENCE_TREE
    (the MGB_REFERENCE_TREE environment variable or its default)."""
    import sys

    root = os.path.dirname(HERE)
    if root not in sys.path:
        sys.path.insert(0, root)
    from alphazero_b200 import build as native

    return native.REFERENCE_TREE


def build(ref_dir: str | None = None) -> None:
    """Runs oracle/Makefile (the _ref part only when the reference tree
    exists)."""
    if ref_dir is None:
        ref_dir = reference_tree()
    r = subprocess.run(["make", "-C", HERE, f"REF={ref_dir}"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)


_ORC = None
_REF = None


def _orc() -> ctypes.CDLL:
    global _ORC
    if _ORC is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_new.restype = ctypes.c_void_p
        L.orc_free.argtypes = [ctypes.c_void_p]
        L.orc_set.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int,
                              ctypes.c_void_p]
        L.orc_finalize.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
        L.orc_info.argtypes = [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_int)] * 5
        L.orc_predict_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p]
        _ORC = L
    return _ORC


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def _ref() -> ctypes.CDLL:
    global _REF
    if _REF is None:
        if not os.path.exists(REF_SO):
            raise RuntimeError("reference harness not built (oracle/_ref)")
        L = ctypes.CDLL(REF_SO)
        L.ref_random_positions.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint32, ctypes.c_int,
                                           ctypes.c_void_p]
        L.ref_onnx_load.argtypes = [ctypes.c_char_p]
        L.ref_onnx_name.argtypes = [ctypes.c_int]
        L.ref_onnx_name.restype = ctypes.c_char_p
        L.ref_onnx_dims.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        L.ref_onnx_floats.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
        L.ref_onnx_floats.restype = ctypes.c_int64
        _REF = L
    return _REF


class EigenOracle:
    """The restated reference CPU engine over a dict of named arrays."""

    def __init__(self, state_dict):
        L = _orc()
        self._L = L
        self._h = ctypes.c_void_p(L.orc_new())
        for name, arr in state_dict.items():
            a = np.asarray(arr)
            if a.dtype != np.float32:
                continue
            a = np.ascontiguousarray(a)
            dims = (ctypes.c_int64 * max(1, a.ndim))(*a.shape)
            L.orc_set(self._h, name.encode(), dims, a.ndim, a.ctypes.data)
        err = ctypes.create_string_buffer(512)
        if L.orc_finalize(self._h, err, 512) != 0:
            raise RuntimeError(err.value.decode())
        v = [ctypes.c_int() for _ in range(5)]
        L.orc_info(self._h, *[ctypes.byref(x) for x in v])
        self.board, self.input_channels, self.filters, self.blocks, self.actions = (x.value for x in v)

    def __del__(self):
        try:
            self._L.orc_free(self._h)
        except Exception:
            pass

    def predict_batch(self, states, mode: int = CANONICAL, threads: int = 1):
        x = np.ascontiguousarray(states, dtype=np.float32)
        n = x.shape[0]
        probs = np.empty((n, self.actions), np.float32)
        logits = np.empty((n, self.actions), np.float32)
        vals = np.empty((n,), np.float32)
        rc = self._L.orc_predict_batch(self._h, x.ctypes.data, n, mode, threads, probs.ctypes.data,
                                       logits.ctypes.data, vals.ctypes.data)
        if rc != 0:
            raise RuntimeError("oracle predict failed")
        return probs, vals, logits


def ref_random_positions(board: int, n: int, seed: int, max_moves: int) -> np.ndarray:
    out = np.empty((n, 17 * board * board), np.float32)
    if _ref().ref_random_positions(board, n, seed & 0xFFFFFFFF, max_moves, out.ctypes.data) != 0:
        raise RuntimeError("ref_random_positions failed")
    return out


def ref_read_onnx(path: str):
    """(name, dims, fp32 values) per initializer, parsed by the reference loader."""
    L = _ref()
    cnt = L.ref_onnx_load(path.encode())
    if cnt < 0:
        raise RuntimeError("reference loader rejected " + path)
    out = []
    for i in range(cnt):
        dims = (ctypes.c_int64 * 16)()
        rank = L.ref_onnx_dims(i, dims, 16)
        n = L.ref_onnx_floats(i, None, 0)
        vals = np.empty(n, np.float32)
        L.ref_onnx_floats(i, vals.ctypes.data, n)
        out.append((L.ref_onnx_name(i).decode(), tuple(dims[k] for k in range(rank)), vals))
    return out
