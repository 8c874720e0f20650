"""The product's seeded position generator (alphazero_b200/host/go_positions)
against the reference rules and encoder (src/game.cpp), bit for bit."""
import numpy as np
import pytest

import oracle
from alphazero_b200 import host_lib

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference harness not built")


@needs_ref
@pytest.mark.parametrize("board,n,seed,max_moves", [
    (9, 64, 0, 60), (9, 64, 99, 200), (19, 24, 1, 250), (19, 8, 7, 700), (13, 32, 5, 170),
    (5, 300, 11, 120), (2, 50, 3, 30), (3, 80, 4, 60),
])
def test_positions_identical_to_reference_game(board, n, seed, max_moves):
    mine = host_lib.random_positions(board, n, seed, max_moves)
    ref = oracle.ref_random_positions(board, n, seed, max_moves)
    assert np.array_equal(mine, ref)


def test_empty_board_encoding():
    # k = 0 moves is drawn with probability 1/(max_moves+1); max_moves = 0 forces it.
    x = host_lib.random_positions(9, 3, 0, 0).reshape(3, 17, 81)
    assert not x[:, :16].any()          # no stones in any history plane
    assert (x[:, 16] == 1).all()        # black to move


def test_planes_are_binary_and_consistent():
    x = host_lib.random_positions(19, 32, 42, 250).reshape(32, 17, 361)
    assert set(np.unique(x)).issubset({0.0, 1.0})
    # a point holds at most one stone in each history step
    assert ((x[:, 0:8] + x[:, 8:16]) <= 1).all()
    # colour plane is constant per position
    assert (x[:, 16].min(1) == x[:, 16].max(1)).all()


def test_zero_positions_and_bad_args():
    assert host_lib.random_positions(9, 0, 1, 10).shape == (0, 17 * 81)
    with pytest.raises(ValueError):
        host_lib.random_positions(20, 1, 1, 10)
    with pytest.raises(ValueError):
        host_lib.random_positions(1, 1, 1, 10)


def test_deterministic():
    a = host_lib.random_positions(19, 8, 5, 250)
    b = host_lib.random_positions(19, 8, 5, 250)
    c = host_lib.random_positions(19, 8, 6, 250)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
