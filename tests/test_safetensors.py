"""Safetensors reader (nnmetal/src/safetensors.zig restated) on CPU, and a
checkpoint round trip through the library on the GPU."""
import json
import struct

import numpy as np
import pytest

from nnzap_b200 import synth
from nnzap_b200.safetensors import SafetensorsError, SafetensorsFile, save_safetensors


def _raw(header: dict, data: bytes = b"") -> bytes:
    hj = json.dumps(header).encode()
    return struct.pack("<Q", len(hj)) + hj + data


def test_roundtrip_dtypes_and_metadata(tmp_path):
    rng = np.random.default_rng(0)
    ts = [("a.u8", rng.integers(0, 256, (3, 5), dtype=np.uint8)),
          ("b.u32", rng.integers(0, 2**32, (4, 2), dtype=np.uint32)),
          ("c.f16", rng.standard_normal((7,)).astype(np.float16)),
          ("d.f32", rng.standard_normal((2, 3, 4)).astype(np.float32)),
          ("e.bf16", rng.integers(0, 2**16, (6,), dtype=np.uint16), "BF16")]
    p = tmp_path / "m.safetensors"
    save_safetensors(p, ts, metadata={"format": "mlx"})
    with SafetensorsFile(p) as f:
        assert set(f.tensors) == {t[0] for t in ts}
        for t in ts:
            d = f.get_tensor(t[0])
            assert d.shape == t[1].shape
            np.testing.assert_array_equal(d.array, t[1])
        assert f.get_tensor("e.bf16").dtype == "BF16"
        assert f.get_tensor("missing") is None


@pytest.mark.parametrize("header,data,err", [
    ({"t": {"dtype": "I64", "shape": [1], "data_offsets": [0, 8]}}, b"\0" * 8, "UnsupportedDtype"),
    ({"t": {"shape": [1], "data_offsets": [0, 4]}}, b"\0" * 4, "MissingDtype"),
    ({"t": {"dtype": "F32", "data_offsets": [0, 4]}}, b"\0" * 4, "MissingShape"),
    ({"t": {"dtype": "F32", "shape": [1, 1, 1, 1, 1], "data_offsets": [0, 4]}}, b"\0" * 4, "TooManyDimensions"),
    ({"t": {"dtype": "F32", "shape": [1]}}, b"\0" * 4, "MissingDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}, b"\0" * 4, "InvalidDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 4, "DataOffsetOutOfBounds"),
    ({"t": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8, "InvalidDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, b"\0" * 4, "InvalidShape"),
])
def test_rejects_malformed(header, data, err):
    with pytest.raises(SafetensorsError, match=err):
        SafetensorsFile(data=_raw(header, data))


def test_rejects_bad_header_length():
    with pytest.raises(SafetensorsError, match="InvalidHeader"):
        SafetensorsFile(data=struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(SafetensorsError, match="InvalidJson"):
        SafetensorsFile(data=struct.pack("<Q", 4) + b"{ab}")


def test_too_many_tensors():
    header = {f"t{i}": {"dtype": "U8", "shape": [1], "data_offsets": [i, i + 1]} for i in range(1025)}
    with pytest.raises(SafetensorsError, match="TooManyTensors"):
        SafetensorsFile(data=_raw(header, b"\0" * 1025))


def _write_shards(tmp_path, d, W, n=2):
    items = list(synth.iter_named_tensors(W))
    paths = []
    for k in range(n):
        p = tmp_path / f"model-{k:05d}-of-{n:05d}.safetensors"
        save_safetensors(p, items[k::n])
        paths.append(p)
    return paths


@pytest.mark.gpu
def test_checkpoint_load_matches_direct(tmp_path, cuda, built_lib):
    from nnzap_b200 import Model, config_from_dims
    d = synth.ModelDims(vocab=1000, hidden=256, inter=768, layers=2, n_q=4, n_kv=2, head_dim=128, gs=128,
                        quant="q1")
    W = synth.make_model(d, seed=3)
    paths = _write_shards(tmp_path, d, W)
    cfg = config_from_dims(d, max_context_length=64, max_batch=2)
    a = Model(cfg)
    a.load_weights(synth.iter_named_tensors(W))
    b = Model(cfg)
    b.load_safetensors(paths)
    toks, pos = np.array([5, 77]), np.array([0, 0])
    am_a, lg_a = a.forward_decode(toks, pos, want_logits=True)
    am_b, lg_b = b.forward_decode(toks, pos, want_logits=True)
    np.testing.assert_array_equal(am_a, am_b)
    np.testing.assert_array_equal(lg_a, lg_b)
    a.free()
    b.free()
