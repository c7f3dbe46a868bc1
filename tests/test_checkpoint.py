"""The safetensors checkpoint writer: its layout, pinned by the reference's own reader
(src/libs/io/Safetensors.cpp:106-257, compiled in oracle/_ref), and (GPU) a bit-exact resume of
training from a checkpoint."""
import json
import struct

import numpy as np
import pytest

from oracle import ref as R
from oracle import veda_oracle as O


def _bf16_bits(x):
    """Round-to-nearest-even bf16 bit patterns of an fp32 array."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def test_writer_layout_and_reference_reader(tmp_path):
    from veda_b200 import train_abi as TA
    r = np.random.default_rng(5)
    a = r.standard_normal((3, 5)).astype(np.float32)
    b = r.standard_normal(7).astype(np.float32)
    c = np.arange(6, dtype=np.int64).reshape(2, 3)
    path = tmp_path / "t.safetensors"
    TA.write_safetensors(path, [("model.b", "BF16", _bf16_bits(b)), ("model.a", "F32", a),
                                ("idx", "I64", c)], {"format": "pt", "step": "3"})
    raw = path.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    header = json.loads(raw[8:8 + n])
    assert list(header) == ["__metadata__", "model.b", "model.a", "idx"]
    assert header["__metadata__"] == {"format": "pt", "step": "3"}
    assert header["model.b"] == {"dtype": "BF16", "shape": [7], "data_offsets": [0, 14]}
    assert header["model.a"] == {"dtype": "F32", "shape": [3, 5], "data_offsets": [14, 74]}
    assert header["idx"]["data_offsets"] == [74, 122] and len(raw) == 8 + n + 122
    data = raw[8 + n:]
    assert np.array_equal(np.frombuffer(data[14:74], np.float32).reshape(3, 5), a)
    assert np.array_equal(np.frombuffer(data[74:122], np.int64).reshape(2, 3), c)
    if not R.available():
        pytest.skip("reference not built")
    # the reference's reader takes BF16 and F32 (widening bf16 exactly); write a file of those
    path2 = tmp_path / "w.safetensors"
    TA.write_safetensors(path2, [("model.b", "BF16", _bf16_bits(b)), ("model.a", "F32", a)],
                         {"format": "pt"})
    got = R.read_safetensors(path2)
    assert [g[0] for g in got] == ["model.b", "model.a"]
    assert np.array_equal(got[0][1], O.bf16_round(b))
    assert np.array_equal(got[1][1], a)


def test_writer_rejects_inconsistent_tensors(tmp_path):
    from veda_b200 import train_abi as TA
    with pytest.raises(ValueError):
        TA.write_safetensors(tmp_path / "x.safetensors", [("a", "F32", np.zeros(3, np.float32)),
                                                          ("a", "F32", np.zeros(3, np.float32))])
    with pytest.raises(ValueError):
        TA.write_safetensors(tmp_path / "y.safetensors", [("a", "Q7", np.zeros(3, np.float32))])
