"""ORACLE - test infrastructure only.

GoGame::encode (src/game.cpp:229-256) restated over the history wire format
of mg_forward_history (include/minigo_cuda.h): it reads the board-history
ring and writes the 17 binary planes, as the reference encoder does from its
own ring (ring_buf_, include/game.h:60-66):
  * for i < min(history_length = 8, valid boards): the board i moves back is
    ring slot (top - i) mod 8 (src/game.cpp:236-238);
  * plane i marks the stones of the player to move on it, plane 8 + i the
    opponent's (src/game.cpp:239-247);
  * plane 16 is all ones when black is to move (src/game.cpp:250-254).
Used by the CPU tests to pin the format against the planes the reference's
own game.cpp and the product's generator write, and by the GPU tests as the
checker of the device-side expansion.
"""
from __future__ import annotations

import numpy as np

HISTORY = 8


def slot_words(board: int) -> int:
    return (board * board + 15) // 16


def planes_from_history(words: np.ndarray, board: int) -> np.ndarray:
    """words: [n, 1 + 8 * slot_words(board)] uint32 -> [n, 17 * board^2]
    float32 planes, plane-major."""
    w = np.asarray(words, dtype=np.uint32)
    n = w.shape[0]
    nn = board * board
    sw = slot_words(board)
    assert w.shape[1] == 1 + HISTORY * sw
    hdr = w[:, 0]
    to_move = (hdr & 3).astype(np.int64)
    valid = ((hdr >> 4) & 15).astype(np.int64)
    top = ((hdr >> 8) & 7).astype(np.int64)
    # every slot's points: [n, 8, nn] in {0, 1, 2}
    slots = w[:, 1:].reshape(n, HISTORY, sw)
    p = np.arange(nn)
    pts = (slots[:, :, p // 16] >> (2 * (p % 16)).astype(np.uint32)) & 3
    out = np.zeros((n, 2 * HISTORY + 1, nn), np.float32)
    rows = np.arange(n)
    for i in range(HISTORY):
        live = i < valid
        snap = pts[rows, (top - i) % HISTORY]  # [n, nn]
        mine = (snap == to_move[:, None]) & live[:, None]
        theirs = (snap == (3 - to_move)[:, None]) & live[:, None] & (snap != 0)
        out[:, i] = mine & (snap != 0)
        out[:, HISTORY + i] = theirs
    out[:, 2 * HISTORY] = (to_move == 1)[:, None]
    return out.reshape(n, -1)
