"""The .bin model format of src/loader.js:5-77 (jstorch_b200/loader.py).

CPU: save_model writes exactly what saveModel writes (bytes checked against
the format spelled out field by field), and malformed files are rejected
before anything reaches a GPU.  GPU: load_model round trips, including files
whose tensors are not stored in key order."""
import json
import struct

import numpy as np
import pytest

from jstorch_b200 import loader


def _expected_bytes(tensors, config):
    """loader.js:46-77 by hand: header JSON with tensors in insertion order."""
    meta, blobs, off = {}, [], 0
    for k, a in tensors.items():
        meta[k] = {"shape": list(a.shape), "dtype": "float32", "offset": off, "size": a.size}
        blobs.append(a.astype("<f4").tobytes())
        off += 4 * a.size
    hdr = json.dumps({"tensors": meta, "config": config}, separators=(",", ":")).encode()
    return b"JSTORCH\0" + struct.pack("<I", 1) + struct.pack("<I", len(tensors)) + struct.pack("<Q", len(hdr)) \
        + hdr + b"".join(blobs)


def test_save_model_bytes(tmp_path):
    t = {"fc1.weight": np.arange(6, dtype=np.float32).reshape(2, 3), "fc1.bias": np.array([0.5, -2.0], np.float32),
         "empty": np.zeros((0, 4), np.float32)}
    cfg = {"hidden": 3, "name": "mlp"}
    p = tmp_path / "m.bin"
    loader.save_model(str(p), t, cfg)
    assert p.read_bytes() == _expected_bytes(t, cfg)
    # header fields (loader.js:25-31)
    version, count, header, data0 = loader.read_header(p.read_bytes())
    assert (version, count) == (1, 3) and header["config"] == cfg
    assert header["tensors"]["fc1.bias"] == {"shape": [2], "dtype": "float32", "offset": 24, "size": 2}


@pytest.mark.parametrize("mutate,msg", [
    (lambda b: b"JSTORCX\0" + b[8:], "bad magic"),
    (lambda b: b[:16] + struct.pack("<Q", 10 ** 6) + b[24:], "past the end"),
    (lambda b: b[:-4], "outside the data region"),
])
def test_malformed_files_rejected(tmp_path, mutate, msg):
    t = {"w": np.ones((3, 3), np.float32)}
    p = tmp_path / "m.bin"
    loader.save_model(str(p), t)
    p.write_bytes(mutate(p.read_bytes()))
    with pytest.raises(ValueError, match=msg):
        loader.load_model(str(p))


@pytest.mark.gpu
def test_round_trip_on_device(tmp_path):
    from jstorch_b200 import _core
    rng = np.random.default_rng(0)
    t = {"a": rng.standard_normal((17, 33)).astype(np.float32), "b": rng.standard_normal(5).astype(np.float32),
         "c": rng.standard_normal((2, 3, 4)).astype(np.float32), "z": np.zeros((0,), np.float32)}
    p = tmp_path / "m.bin"
    loader.save_model(str(p), {k: _core.Tensor.fromBuffer(v) for k, v in t.items()}, {"k": [1, 2]})
    assert p.read_bytes() == _expected_bytes(t, {"k": [1, 2]})
    state, cfg = loader.load_model(str(p))
    assert cfg == {"k": [1, 2]} and list(state) == list(t)
    for k, v in t.items():
        assert state[k].shape == list(v.shape)
        np.testing.assert_array_equal(state[k].toArray(), v)
    # loaded tensors feed the GEMM path directly (a view with an offset into the block)
    y = state["a"].matmul(_core.Tensor.fromBuffer(np.ones((33, 2), np.float32))).toArray()
    np.testing.assert_allclose(y, t["a"].astype(np.float64) @ np.ones((33, 2)), rtol=1e-5, atol=1e-4)


@pytest.mark.gpu
def test_out_of_order_offsets(tmp_path):
    """A file whose data region stores the tensors in another order than the
    header lists them (the format allows any offsets)."""
    a = np.arange(4, dtype=np.float32)
    b = -np.arange(6, dtype=np.float32)
    hdr = json.dumps({"tensors": {"a": {"shape": [4], "dtype": "float32", "offset": 24, "size": 4},
                                  "b": {"shape": [2, 3], "dtype": "float32", "offset": 0, "size": 6}},
                      "config": {}}, separators=(",", ":")).encode()
    p = tmp_path / "o.bin"
    p.write_bytes(b"JSTORCH\0" + struct.pack("<IIQ", 1, 2, len(hdr)) + hdr + b.tobytes() + a.tobytes())
    state, _ = loader.load_model(str(p))
    np.testing.assert_array_equal(state["a"].toArray(), a)
    np.testing.assert_array_equal(state["b"].toArray(), b.reshape(2, 3))
