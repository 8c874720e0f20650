"""Generates the golden fixtures in tests/golden/*.npz from the reference.

Run from the repo root in a container that has the reference tree:
    python tests/golden/make_golden.py [REFERENCE_TREE]
(default: alphazero_b200.build.REFERENCE_TREE, i.e. $MGB_REFERENCE_TREE).

For each case it
  * builds the seeded state dict (alphazero_b200.weights.make_state_dict) and
    loads it into the reference network class AlphaZeroNet imported from
    scripts/model.py, in float64;
  * generates the input positions with the reference's own src/game.cpp
    (oracle/_ref/libref_harness.so) and checks that the product's generator
    yields identical planes;
  * records the reference network's fp64 logits and tanh values
    (canonical NCHW semantics, scripts/model.py:48-62);
  * records the same network under the literal semantics of
    src/eigen_engine.cpp (column-major input Map at :211, policy flatten
    c + 2p at :242), emulated with the reference modules.
The fixtures hold positions (uint8 planes), expected outputs and a digest of
the weights, which the tests regenerate from the seed.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

# name: (board, filters, blocks, variant, weight seed, positions, position seed, max moves)
CASES = {
    "b9c64x6_init": (9, 64, 6, "init", 0, 16, 0, 60),
    "b9c64x6_pert": (9, 64, 6, "perturbed", 1, 16, 1, 60),
    "b9c128x10_pert": (9, 128, 10, "perturbed", 2, 8, 2, 60),
    "b19c128x10_init": (19, 128, 10, "init", 3, 4, 3, 250),
    "b19c128x10_pert": (19, 128, 10, "perturbed", 4, 4, 4, 250),
    "b19c256x20_pert": (19, 256, 20, "perturbed", 5, 2, 5, 250),
    "b5c32x3_pert": (5, 32, 3, "perturbed", 6, 8, 6, 40),
}


def main(ref: str) -> None:
    import torch

    sys.path.insert(0, os.path.join(ref, "scripts"))
    from model import AlphaZeroNet  # the reference network definition

    import oracle
    from alphazero_b200 import host_lib, weights

    oracle.build(ref)
    for name, (board, C, NB, variant, wseed, npos, pseed, maxm) in CASES.items():
        sd = weights.make_state_dict(board, C, NB, seed=wseed, variant=variant)
        net = AlphaZeroNet(board, 17, C, NB).double().eval()
        net.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in sd.items()})
        x = oracle.ref_random_positions(board, npos, pseed, maxm)
        mine = host_lib.random_positions(board, npos, pseed, maxm)
        assert np.array_equal(x, mine), f"{name}: position generator differs from game.cpp"
        hw = board * board
        xt = torch.from_numpy(x.astype(np.float64))
        with torch.no_grad():
            lg, v = net(xt.reshape(npos, 17, board, board))
            # literal src/eigen_engine.cpp semantics
            xl = xt.reshape(npos, hw, 17).permute(0, 2, 1).reshape(npos, 17, board, board)
            out = torch.relu(net.input_bn(net.input_conv(xl)))
            for blk in net.res_blocks:
                out = blk(out)
            p = torch.relu(net.policy_bn(net.policy_conv(out))).reshape(npos, 2, hw)
            lgl = net.policy_fc(p.permute(0, 2, 1).reshape(npos, 2 * hw))
            vv = torch.relu(net.value_bn(net.value_conv(out))).reshape(npos, hw)
            vl = torch.tanh(net.value_fc2(torch.relu(net.value_fc1(vv))))
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            board=board, filters=C, blocks=NB, variant=variant, weight_seed=wseed,
            position_seed=pseed, max_moves=maxm,
            weights_digest=weights.weights_digest(sd),
            positions=x.astype(np.uint8),
            logits=lg.numpy(), value=v.numpy()[:, 0],
            logits_literal=lgl.numpy(), value_literal=vl.numpy()[:, 0])
        print(f"{name}: logit std {lg.std().item():.3f}, |value| max {v.abs().max().item():.3f}")


if __name__ == "__main__":
    from alphazero_b200 import build as native

    main(sys.argv[1] if len(sys.argv) > 1 else native.REFERENCE_TREE)
