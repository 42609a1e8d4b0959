"""safetensors read/write (CPU). The reader mirrors the reference loader's
checks (src/safetensors.ts:49-103): f32 only, integer/bool tensors skipped and
reported, other float dtypes rejected, offsets and sizes validated."""
import json
import struct

import numpy as np
import pytest

from tensorgrad_b200.safetensors import loadSafetensors, saveSafetensors


def _raw(header: dict, blob: bytes) -> bytes:
    h = json.dumps(header).encode()
    return struct.pack("<Q", len(h)) + h + blob


def test_round_trip_with_metadata():
    r = np.random.default_rng(0)
    t = {"a": r.standard_normal((3, 4)).astype(np.float32), "b/c": np.arange(5, dtype=np.float32),
         "s": np.array(2.5, np.float32)}
    buf = saveSafetensors(t, {"step": 7, "note": "x"})
    (hlen,) = struct.unpack_from("<Q", buf, 0)
    assert (8 + hlen) % 8 == 0  # data blob starts 8-byte aligned
    d = loadSafetensors(buf)
    assert set(d["tensors"]) == set(t) and d["skipped"] == {}
    for k in t:
        assert d["tensors"][k].dtype == np.float32
        np.testing.assert_array_equal(d["tensors"][k], t[k])
        assert d["shapes"][k] == list(t[k].shape)
    assert d["metadata"] == {"step": "7", "note": "x"}


def test_integer_tensors_are_skipped_and_reported():
    blob = np.ones(2, np.float32).tobytes() + np.zeros(1, np.int64).tobytes()
    buf = _raw({"w": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
                "bn.num_batches_tracked": {"dtype": "I64", "shape": [], "data_offsets": [8, 16]}}, blob)
    d = loadSafetensors(buf)
    assert list(d["tensors"]) == ["w"]
    assert d["skipped"] == {"bn.num_batches_tracked": "I64"}
    assert d["shapes"]["bn.num_batches_tracked"] == []


@pytest.mark.parametrize("header,blob,msg", [
    ({"w": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]}}, b"\0" * 4, "f32-only"),
    ({"w": {"dtype": "F32", "shape": [2], "data_offsets": [0, 16]}}, b"\0" * 8, "out of range"),
    ({"w": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8, "byte length"),
])
def test_malformed_tensors_raise(header, blob, msg):
    with pytest.raises(ValueError, match=msg):
        loadSafetensors(_raw(header, blob))


def test_malformed_containers_raise():
    with pytest.raises(ValueError, match="too small"):
        loadSafetensors(b"\0" * 4)
    with pytest.raises(ValueError, match="exceeds buffer"):
        loadSafetensors(struct.pack("<Q", 100) + b"{}")
    with pytest.raises(ValueError, match="not valid JSON"):
        loadSafetensors(struct.pack("<Q", 3) + b"{x}")
