"""ORACLE - test infrastructure only.

A functional torch restatement of the reference network's forward pass,
``AlphaZeroNet.forward`` in eval mode (scripts/model.py:48-64, with
``ResBlock.forward`` at :19-24), over the same named state dict the engine
loads.  Each step follows the reference module it names:

  input_conv 3x3 pad 1 -> input_bn -> ReLU                      (:49)
  per block: conv1 -> bn1 -> ReLU -> conv2 -> bn2, + x, ReLU     (:19-24)
  policy: policy_conv 1x1 -> policy_bn -> ReLU -> view(n, 2*hw)
          (C-major flatten) -> policy_fc                         (:53-55)
  value: value_conv 1x1 -> value_bn -> ReLU -> view(n, hw)
         -> value_fc1 -> ReLU -> value_fc2 -> tanh               (:57-60)

BatchNorm runs with its running statistics and eps 1e-5 (the module
defaults).  It serves as the torch-CPU baseline that bench.py times on all
host cores next to the C restatement of src/eigen_engine.cpp; it is pinned
against the golden fixtures (tests/test_torch_baseline.py).  Only tests and
bench.py's CPU-baseline leg use it.
"""
from __future__ import annotations

import numpy as np


class TorchNet:
    def __init__(self, state_dict, dtype=None):
        import torch

        self.torch = torch
        self.dtype = dtype or torch.float32
        self.p = {k: torch.from_numpy(np.ascontiguousarray(v)).to(self.dtype)
                  for k, v in state_dict.items() if np.asarray(v).dtype == np.float32}
        self.blocks = sum(1 for k in self.p if k.startswith("res_blocks.") and k.endswith(".conv1.weight"))
        w = self.p["input_conv.weight"]
        self.filters, self.input_channels = int(w.shape[0]), int(w.shape[1])
        self.hw = int(self.p["value_fc1.weight"].shape[1])
        self.board = int(round(self.hw ** 0.5))

    def _bn(self, x, name):
        F = self.torch.nn.functional
        p = self.p
        return F.batch_norm(x, p[name + ".running_mean"], p[name + ".running_var"],
                            p[name + ".weight"], p[name + ".bias"], False, 0.0, 1e-5)

    def forward(self, states):
        """states: [n, 17 * hw] binary planes (plane-major, NCHW).
        Returns (logits [n, hw + 1], value [n]) as numpy arrays."""
        torch = self.torch
        F = torch.nn.functional
        p = self.p
        n = states.shape[0]
        b = self.board
        with torch.no_grad():
            x = torch.from_numpy(np.ascontiguousarray(states)).to(self.dtype)
            x = x.reshape(n, self.input_channels, b, b)
            out = F.relu(self._bn(F.conv2d(x, p["input_conv.weight"], padding=1), "input_bn"))
            for i in range(self.blocks):
                pre = f"res_blocks.{i}."
                t = F.relu(self._bn(F.conv2d(out, p[pre + "conv1.weight"], padding=1), pre + "bn1"))
                t = self._bn(F.conv2d(t, p[pre + "conv2.weight"], padding=1), pre + "bn2")
                out = F.relu(t + out)
            pol = F.relu(self._bn(F.conv2d(out, p["policy_conv.weight"]), "policy_bn"))
            logits = F.linear(pol.reshape(n, -1), p["policy_fc.weight"], p["policy_fc.bias"])
            v = F.relu(self._bn(F.conv2d(out, p["value_conv.weight"]), "value_bn"))
            v = F.relu(F.linear(v.reshape(n, -1), p["value_fc1.weight"], p["value_fc1.bias"]))
            v = torch.tanh(F.linear(v, p["value_fc2.weight"], p["value_fc2.bias"]))
        return logits.float().numpy(), v.float().numpy()[:, 0]
