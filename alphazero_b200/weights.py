"""Seeded synthetic weights for the residual policy/value network, and a
writer for the ONNX container the engine loads.

The parameter set and names are those of ``AlphaZeroNet``'s state_dict
(scripts/model.py:26-45): ``input_conv``, ``input_bn``,
``res_blocks.{i}.{conv1,bn1,conv2,bn2}``, ``policy_conv``, ``policy_bn``,
``policy_fc``, ``value_conv``, ``value_bn``, ``value_fc1``, ``value_fc2``,
plus each BatchNorm's ``num_batches_tracked`` (int64), which
scripts/export_onnx.py:26-45 also embeds.

Two variants:
  * ``"init"`` - the distributions of a freshly constructed torch module,
    i.e. what ``export_onnx.py --init`` writes: conv / linear weights and
    linear biases uniform in +-1/sqrt(fan_in); BatchNorm weight 1, bias 0,
    running mean 0, running var 1.
  * ``"perturbed"`` - larger conv weights and random BatchNorm statistics, so
    the BN fold is exercised and logits are O(1) (with "init" weights they
    are ~0.05, which makes tolerances on probabilities vacuous).

Values come from a counter-based splitmix64 stream keyed by (seed, tensor
name), so any tensor can be regenerated alone and the result does not
depend on numpy's or torch's generator versions.
"""
from __future__ import annotations

import collections
import math

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _mix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def _fnv1a64(s: str) -> int:
    h = 0xCBF29CE484222325
    for b in s.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def uniform(seed: int, name: str, shape, lo: float, hi: float) -> np.ndarray:
    """float32 array of `shape`, uniform in [lo, hi), keyed by (seed, name)."""
    count = int(np.prod(shape)) if len(shape) else 1
    key = _mix(np.array([(seed & 0xFFFFFFFFFFFFFFFF) ^ _fnv1a64(name)], dtype=np.uint64))[0]
    with np.errstate(over="ignore"):
        idx = np.arange(1, count + 1, dtype=np.uint64)
        z = _mix(key + idx * _GOLDEN)
    u = (z >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
    return (lo + (hi - lo) * u).astype(np.float32).reshape(shape)


def make_state_dict(board: int, filters: int, blocks: int, seed: int = 0,
                    variant: str = "init", input_channels: int = 17,
                    value_hidden: int = 64) -> "collections.OrderedDict[str, np.ndarray]":
    """State dict of AlphaZeroNet(board, input_channels, filters, blocks)."""
    if variant not in ("init", "perturbed"):
        raise ValueError("variant must be 'init' or 'perturbed'")
    pert = variant == "perturbed"
    hw = board * board
    actions = hw + 1
    sd: "collections.OrderedDict[str, np.ndarray]" = collections.OrderedDict()

    def conv(name, cout, cin, k, gain=1.0):
        b = gain / math.sqrt(cin * k * k)
        sd[name] = uniform(seed, name, (cout, cin, k, k), -b, b)

    def bn(prefix, ch):
        if pert:
            sd[prefix + ".weight"] = uniform(seed, prefix + ".weight", (ch,), 0.8, 1.2)
            sd[prefix + ".bias"] = uniform(seed, prefix + ".bias", (ch,), -0.1, 0.1)
            sd[prefix + ".running_mean"] = uniform(seed, prefix + ".running_mean", (ch,), -0.1, 0.1)
            sd[prefix + ".running_var"] = uniform(seed, prefix + ".running_var", (ch,), 0.8, 1.2)
        else:
            sd[prefix + ".weight"] = np.ones(ch, np.float32)
            sd[prefix + ".bias"] = np.zeros(ch, np.float32)
            sd[prefix + ".running_mean"] = np.zeros(ch, np.float32)
            sd[prefix + ".running_var"] = np.ones(ch, np.float32)
        sd[prefix + ".num_batches_tracked"] = np.zeros((), np.int64)

    def linear(prefix, out_f, in_f, gain=1.0):
        b = gain / math.sqrt(in_f)
        sd[prefix + ".weight"] = uniform(seed, prefix + ".weight", (out_f, in_f), -b, b)
        sd[prefix + ".bias"] = uniform(seed, prefix + ".bias", (out_f,), -b, b)

    # He-like gain keeps activations O(1) through the trunk in "perturbed";
    # the second conv of each block is damped by 1/sqrt(2*blocks) so the
    # residual sum stays O(1) however deep the trunk is.
    g_in = math.sqrt(6.0) if pert else 1.0
    g_c2 = math.sqrt(6.0 / (2.0 * max(blocks, 1))) if pert else 1.0
    conv("input_conv.weight", filters, input_channels, 3, g_in)
    bn("input_bn", filters)
    for i in range(blocks):
        p = f"res_blocks.{i}"
        conv(p + ".conv1.weight", filters, filters, 3, g_in)
        bn(p + ".bn1", filters)
        conv(p + ".conv2.weight", filters, filters, 3, g_c2)
        bn(p + ".bn2", filters)
    conv("policy_conv.weight", 2, filters, 1, g_in)
    bn("policy_bn", 2)
    linear("policy_fc", actions, 2 * hw, 2.0 if pert else 1.0)
    conv("value_conv.weight", 1, filters, 1, g_in)
    bn("value_bn", 1)
    linear("value_fc1", value_hidden, hw, 1.0)
    linear("value_fc2", 1, value_hidden, 1.0)
    return sd


def weights_digest(sd) -> str:
    """Short content hash of a state dict (names, shapes, bytes)."""
    import hashlib
    h = hashlib.sha256()
    for k, v in sd.items():
        h.update(k.encode())
        h.update(str(tuple(v.shape)).encode())
        h.update(np.ascontiguousarray(v).tobytes())
    return h.hexdigest()[:16]


# ---- ONNX container -------------------------------------------------------

def _varint(v: int) -> bytes:
    out = bytearray()
    v &= 0xFFFFFFFFFFFFFFFF
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _len_field(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _tensor_proto(name: str, arr: np.ndarray) -> bytes:
    if arr.dtype == np.float32:
        dtype = 1
    elif arr.dtype == np.int64:
        dtype = 7
    else:
        raise TypeError(f"{name}: unsupported dtype {arr.dtype}")
    body = b""
    if arr.ndim:
        body += _len_field(1, b"".join(_varint(int(d)) for d in arr.shape))
    body += _key(2, 0) + _varint(dtype)
    body += _len_field(8, name.encode())
    body += _len_field(9, np.ascontiguousarray(arr).astype(arr.dtype.newbyteorder("<")).tobytes())
    return body


def onnx_bytes(sd) -> bytes:
    """Serialised ModelProto holding `sd` as graph initializers.

    Layout: ModelProto {ir_version 8, producer_name, graph (7):
    GraphProto {name, initializer (5): TensorProto {dims 1, data_type 2,
    name 8, raw_data 9}...}, opset_import (8): {version 17}} - the fields
    src/onnx_loader.cpp:88-176 reads, in a file a protobuf ONNX reader also
    accepts.  The graph has no nodes: only weights are carried.
    """
    graph = _len_field(2, b"alphazero")
    for name, arr in sd.items():
        graph += _len_field(5, _tensor_proto(name, np.asarray(arr)))
    model = _key(1, 0) + _varint(8)
    model += _len_field(2, b"alphazero_b200")
    model += _len_field(7, graph)
    model += _len_field(8, _key(2, 0) + _varint(17))
    return model


def write_onnx(path: str, sd) -> str:
    with open(path, "wb") as f:
        f.write(onnx_bytes(sd))
    return path
