"""The product's ONNX initializer reader against the reference loader
(src/onnx_loader.cpp) and its error behaviour."""
import os

import numpy as np
import pytest

import oracle
from alphazero_b200 import host_lib, weights

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference harness not built")


@pytest.fixture
def model_file(tmp_path):
    sd = weights.make_state_dict(9, 64, 2, seed=3, variant="perturbed")
    return weights.write_onnx(str(tmp_path / "m.onnx"), sd), sd


@needs_ref
def test_reader_matches_reference_loader(model_file):
    path, _ = model_file
    mine = host_lib.read_onnx(path)
    ref = oracle.ref_read_onnx(path)
    assert [m[0] for m in mine] == [r[0] for r in ref]
    for m, r in zip(mine, ref):
        assert m[2] == r[1]
        if m[1] == 1:
            assert np.array_equal(m[3], r[2])


def test_reader_roundtrip_values(model_file):
    path, sd = model_file
    got = {name: (dt, dims, vals) for name, dt, dims, vals in host_lib.read_onnx(path)}
    for k, v in sd.items():
        dt, dims, vals = got[k]
        assert dims == v.shape
        if v.dtype == np.float32:
            assert dt == 1 and np.array_equal(vals.reshape(v.shape), v)
        else:
            assert dt == 7 and vals is None  # int64 num_batches_tracked is not FLOAT


def _tensor(name, dims, field4=None, raw=None):
    w = weights
    body = w._len_field(1, b"".join(w._varint(d) for d in dims))
    body += w._key(2, 0) + w._varint(1) + w._len_field(8, name.encode())
    if field4 is not None:
        body += w._len_field(4, np.asarray(field4, "<f4").tobytes())
    if raw is not None:
        body += w._len_field(9, np.asarray(raw, "<f4").tobytes())
    return w._len_field(5, body)


def test_float_data_field_and_duplicates(tmp_path):
    w = weights
    graph = _tensor("a", [3], field4=[1, 2, 3]) + _tensor("b", [2], raw=[4, 5]) + \
        _tensor("a", [2], raw=[7, 8])
    p = tmp_path / "x.onnx"
    p.write_bytes(w._len_field(7, graph))
    got = host_lib.read_onnx(str(p))
    assert [g[0] for g in got] == ["a", "b", "a"]
    assert list(got[0][3]) == [1, 2, 3] and list(got[1][3]) == [4, 5]
    if oracle.ref_available():
        ref = oracle.ref_read_onnx(str(p))
        assert [list(r[2]) for r in ref] == [list(g[3]) for g in got]


def test_missing_file_message(tmp_path):
    missing = str(tmp_path / "nope.onnx")
    with pytest.raises(RuntimeError, match="Cannot open model file: " + missing):
        host_lib.read_onnx(missing)


def test_truncated_file_is_an_error_not_a_crash(model_file, tmp_path):
    path, _ = model_file
    data = open(path, "rb").read()
    for cut in (5, 100, len(data) // 2, len(data) - 3):
        p = tmp_path / f"cut{cut}.onnx"
        p.write_bytes(data[:cut])
        with pytest.raises(RuntimeError, match="onnx: truncated"):
            host_lib.read_onnx(str(p))


def test_empty_file_has_no_tensors(tmp_path):
    p = tmp_path / "empty.onnx"
    p.write_bytes(b"")
    assert host_lib.read_onnx(str(p)) == []
    assert os.path.getsize(p) == 0
