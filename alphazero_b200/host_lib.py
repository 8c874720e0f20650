"""ctypes binding of libminigo_host.so (include/minigo_host.h): the seeded
position generator and the ONNX initializer reader.  CPU only."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build

_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = build.HOST_LIB
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run `python -m alphazero_b200.build`")
        L = ctypes.CDLL(path)
        L.mg_random_positions.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint32, ctypes.c_int,
                                          ctypes.c_void_p]
        L.mg_random_positions.restype = ctypes.c_int
        L.mg_random_histories.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_uint32, ctypes.c_int,
                                          ctypes.c_void_p]
        L.mg_random_histories.restype = ctypes.c_int
        L.mg_history_words_for.argtypes = [ctypes.c_int]
        L.mg_history_words_for.restype = ctypes.c_int
        L.mg_onnx_open.argtypes = [ctypes.c_char_p]
        L.mg_onnx_open.restype = ctypes.c_void_p
        L.mg_onnx_error.restype = ctypes.c_char_p
        L.mg_onnx_close.argtypes = [ctypes.c_void_p]
        L.mg_onnx_count.argtypes = [ctypes.c_void_p]
        L.mg_onnx_count.restype = ctypes.c_int
        L.mg_onnx_name.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.mg_onnx_name.restype = ctypes.c_char_p
        L.mg_onnx_data_type.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.mg_onnx_data_type.restype = ctypes.c_int
        L.mg_onnx_dims.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        L.mg_onnx_dims.restype = ctypes.c_int
        L.mg_onnx_floats.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
        L.mg_onnx_floats.restype = ctypes.c_int64
        _LIB = L
    return _LIB


def random_positions(board: int, n: int, seed: int, max_moves: int) -> np.ndarray:
    """[n, 17*board*board] float32 planes of seeded random-playout positions."""
    out = np.empty((n, 17 * board * board), dtype=np.float32)
    rc = lib().mg_random_positions(board, n, seed & 0xFFFFFFFF, max_moves, out.ctypes.data)
    if rc != 0:
        raise ValueError("mg_random_positions rejected its arguments")
    return out


def random_histories(board: int, n: int, seed: int, max_moves: int) -> np.ndarray:
    """The positions of random_positions(board, n, seed, max_moves) in the
    history wire format of mg_forward_history: [n, history_words(board)]
    uint32 (a header word and the ring of the last 8 boards, 2 bits per
    point)."""
    L = lib()
    out = np.empty((n, L.mg_history_words_for(board)), dtype=np.uint32)
    rc = L.mg_random_histories(board, n, seed & 0xFFFFFFFF, max_moves, out.ctypes.data)
    if rc != 0:
        raise ValueError("mg_random_histories rejected its arguments")
    return out


def read_onnx(path: str) -> "list[tuple[str, int, tuple, np.ndarray | None]]":
    """(name, data_type, dims, fp32 values or None) per initializer."""
    L = lib()
    h = L.mg_onnx_open(path.encode())
    if not h:
        raise RuntimeError(L.mg_onnx_error().decode())
    try:
        out = []
        for i in range(L.mg_onnx_count(h)):
            dims = (ctypes.c_int64 * 16)()
            rank = L.mg_onnx_dims(h, i, dims, 16)
            shape = tuple(dims[k] for k in range(rank))
            n = L.mg_onnx_floats(h, i, None, 0)
            vals = None
            if n >= 0:
                vals = np.empty(n, np.float32)
                L.mg_onnx_floats(h, i, vals.ctypes.data, n)
            out.append((L.mg_onnx_name(h, i).decode(), L.mg_onnx_data_type(h, i), shape, vals))
        return out
    finally:
        L.mg_onnx_close(h)
