"""The history wire format of mg_forward_history: the product's host encoder
(GoPosition::encode_history, via mg_random_histories) against the planes of
the same positions, decoded by the oracle's restatement of GoGame::encode
(oracle/history_planes.py).  CPU only; the device-side expansion is tested
in tests/test_gpu_history.py."""
import numpy as np
import pytest

import oracle
from alphazero_b200 import host_lib
from history_planes import planes_from_history, slot_words


@pytest.mark.parametrize("board,n,seed,max_moves", [
    (19, 64, 7, 250), (9, 200, 8, 60), (5, 100, 9, 40), (19, 8, 10, 0), (13, 40, 11, 500)])
def test_history_words_decode_to_the_encoder_planes(board, n, seed, max_moves):
    hist = host_lib.random_histories(board, n, seed, max_moves)
    assert hist.shape == (n, 1 + 8 * slot_words(board))
    planes = host_lib.random_positions(board, n, seed, max_moves)
    assert np.array_equal(planes_from_history(hist, board), planes)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference harness not built")
def test_history_words_decode_to_the_reference_planes():
    # the reference's own src/game.cpp playing and encoding the same positions
    hist = host_lib.random_histories(19, 48, 12, 250)
    assert np.array_equal(planes_from_history(hist, 19), oracle.ref_random_positions(19, 48, 12, 250))


def test_history_header_fields():
    hist = host_lib.random_histories(9, 300, 13, 60)
    to_move = hist[:, 0] & 3
    valid = (hist[:, 0] >> 4) & 15
    assert set(np.unique(to_move)) <= {1, 2}
    assert valid.min() >= 1 and valid.max() <= 8
    assert (hist[:, 0] >> 11 == 0).all()
    # 2-bit points hold 0, 1 or 2 only
    pts = np.stack([(hist[:, 1:] >> (2 * k)) & 3 for k in range(16)])
    assert pts.max() <= 2
