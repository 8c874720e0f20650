"""GPU: the history wire format (mg_forward_history), whose 17 input planes
are expanded on the device from the board-history ring, against the same
positions shipped as fp32 planes (mg_forward) and as the oracle's decoding
of the words; results must be bit-identical, since the staged rows are."""
import numpy as np
import pytest

from alphazero_b200 import host_lib, weights
from conftest import load_golden
from history_planes import planes_from_history

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision", ["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("eigen_compat", [False, True])
def test_history_matches_planes(gpu_engine_factory, precision, eigen_compat):
    _, sd = load_golden("b19c128x10_pert")
    e = gpu_engine_factory(sd, precision, eigen_compat=eigen_compat, max_batch=64)
    hist = host_lib.random_histories(19, 150, 41, 250)  # 150 > max batch: chunked
    planes = host_lib.random_positions(19, 150, 41, 250)
    assert np.array_equal(planes_from_history(hist, 19), planes)
    assert hist.shape[1] == e.history_words()
    p1, v1, l1 = e.forward(planes)
    p2, v2, l2 = e.forward_history(hist, len(hist), want_logits=True)
    assert np.array_equal(l1, l2) and np.array_equal(v1, v2) and np.array_equal(p1, p2)


@pytest.mark.parametrize("board,filters,blocks,n,max_moves", [(9, 64, 6, 16, 60), (9, 128, 10, 256, 60),
                                                              (19, 256, 2, 100, 250)])
def test_history_matches_planes_across_networks(gpu_engine_factory, board, filters, blocks, n,
                                                max_moves):
    sd = weights.make_state_dict(board, filters, blocks, seed=3, variant="perturbed")
    e = gpu_engine_factory(sd, "bf16", max_batch=n)
    hist = host_lib.random_histories(board, n, 5, max_moves)
    p1, v1, l1 = e.forward(planes_from_history(hist, board))
    p2, v2, l2 = e.forward_history(hist, n, want_logits=True)
    assert np.array_equal(l1, l2) and np.array_equal(v1, v2)


def test_history_pinned_input(gpu_engine_factory):
    import torch

    _, sd = load_golden("b9c64x6_pert")
    e = gpu_engine_factory(sd, "bf16")
    hist = host_lib.random_histories(9, 40, 6, 60)
    pinned = torch.from_numpy(hist.view(np.int32)).pin_memory().numpy().view(np.uint32)
    _, v1, l1 = e.forward_history(hist, 40, want_logits=True)
    _, v2, l2 = e.forward_history(pinned, 40, want_logits=True)
    assert np.array_equal(l1, l2) and np.array_equal(v1, v2)
