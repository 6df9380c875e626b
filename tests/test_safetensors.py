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


# ---- the library's C++ reader (nnz_safetensors_*) --------------------------

class Native:
    """nnz_safetensors_* through ctypes: descriptors as (name, dtype code,
    shape, bytes), or the reference error name."""

    def __init__(self, data=None, path=None):
        import ctypes as C
        from nnzap_b200 import _capi
        self.C, self.capi, self.L = C, _capi, _capi.lib()
        self.h = C.c_void_p()
        self._buf = data                      # kept alive while the reader is open
        if path is not None:
            self.rc = self.L.nnz_safetensors_open(str(path).encode(), C.byref(self.h))
        else:
            self.rc = self.L.nnz_safetensors_from_bytes(data, len(data), C.byref(self.h))
        self.err = None if self.rc == 0 else self.L.nnz_last_error().decode().split(":")[0]

    def desc(self, d):
        shape = tuple(d.dims[i] for i in range(d.rank))
        return (d.name.decode(), d.dtype, shape, self.C.string_at(d.data, d.nbytes) if d.nbytes else b"")

    def tensors(self):
        out = []
        for i in range(self.L.nnz_safetensors_count(self.h)):
            d = self.capi.NnzTensorDesc()
            assert self.L.nnz_safetensors_tensor(self.h, i, self.C.byref(d)) == 0
            out.append(self.desc(d))
        return out

    def find(self, name):
        d = self.capi.NnzTensorDesc()
        rc = self.L.nnz_safetensors_find(self.h, name.encode(), self.C.byref(d))
        return self.desc(d) if rc == 0 else rc

    def close(self):
        self.L.nnz_safetensors_close(self.h)


def _zig_file(js: str, n: int) -> bytes:
    # buildTestFile of safetensors_test.zig: length prefix, JSON, n zero bytes
    return struct.pack("<Q", len(js)) + js.encode() + b"\0" * n


def test_native_reference_cases(built_lib):
    from nnzap_b200 import _capi
    # safetensors_test.zig:33-55
    f = Native(_zig_file('{"tensor_a": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]}}', 24))
    assert f.rc == 0 and f.tensors() == [("tensor_a", _capi.NNZ_DT_F32, (2, 3), b"\0" * 24)]
    f.close()
    # :57-91
    f = Native(_zig_file('{"weight": {"dtype": "F16", "shape": [4],\n"data_offsets": [0, 8]},\n'
                         '"bias": {"dtype": "F32", "shape": [2],\n"data_offsets": [8, 16]}}', 16))
    assert f.rc == 0 and len(f.tensors()) == 2
    assert f.find("bias")[:3] == ("bias", _capi.NNZ_DT_F32, (2,))
    assert f.find("weight")[:3] == ("weight", _capi.NNZ_DT_F16, (4,))
    assert f.find("nonexistent") == _capi.NNZ_ENOTFOUND
    f.close()
    # :93-106
    f = Native(_zig_file('{"bad": {"dtype": "F32", "shape": [2], "data_offsets": [0, 999]}}', 24))
    assert f.err == "DataOffsetOutOfBounds"
    # :108-132
    f = Native(_zig_file('{"real_tensor": {"dtype": "U8", "shape": [4],\n"data_offsets": [0, 4]},\n'
                         '"__metadata__": {"format": "test",\n"version": "1.0"}}', 4))
    assert [t[:3] for t in f.tensors()] == [("real_tensor", _capi.NNZ_DT_U8, (4,))]
    assert f.find("__metadata__") == _capi.NNZ_ENOTFOUND
    f.close()
    # :134-160 (dtype strings and sizes, through the byte-count check)
    for dt, size, code in [("U8", 1, _capi.NNZ_DT_U8), ("U32", 4, _capi.NNZ_DT_U32), ("F16", 2, _capi.NNZ_DT_F16),
                           ("BF16", 2, _capi.NNZ_DT_BF16), ("F32", 4, _capi.NNZ_DT_F32)]:
        f = Native(_raw({"t": {"dtype": dt, "shape": [3], "data_offsets": [0, 3 * size]}}, b"\1" * (3 * size)))
        assert f.tensors()[0][1] == code
        f.close()
    assert Native(_raw({"t": {"dtype": "I32", "shape": [1], "data_offsets": [0, 4]}}, b"\0" * 4)).err == \
        "UnsupportedDtype"


MALFORMED = [
    ({"t": {"dtype": "I64", "shape": [1], "data_offsets": [0, 8]}}, b"\0" * 8, "UnsupportedDtype"),
    ({"t": {"shape": [1], "data_offsets": [0, 4]}}, b"\0" * 4, "MissingDtype"),
    ({"t": {"dtype": 3, "shape": [1], "data_offsets": [0, 4]}}, b"\0" * 4, "InvalidDtype"),
    ({"t": {"dtype": "F32", "data_offsets": [0, 4]}}, b"\0" * 4, "MissingShape"),
    ({"t": {"dtype": "F32", "shape": 1, "data_offsets": [0, 4]}}, b"\0" * 4, "InvalidShape"),
    ({"t": {"dtype": "F32", "shape": [True], "data_offsets": [0, 4]}}, b"\0" * 4, "InvalidShape"),
    ({"t": {"dtype": "F32", "shape": [1.0], "data_offsets": [0, 4]}}, b"\0" * 4, "InvalidShape"),
    ({"t": {"dtype": "F32", "shape": [1, 1, 1, 1, 1], "data_offsets": [0, 4]}}, b"\0" * 4, "TooManyDimensions"),
    ({"t": {"dtype": "F32", "shape": [1]}}, b"\0" * 4, "MissingDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}, b"\0" * 4, "InvalidDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [1], "data_offsets": [-4, 0]}}, b"\0" * 4, "InvalidDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [1], "data_offsets": [0]}}, b"\0" * 4, "InvalidDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [1], "data_offsets": "0,4"}}, b"\0" * 4, "InvalidDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 4, "DataOffsetOutOfBounds"),
    ({"t": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8, "InvalidDataOffsets"),
    ({"t": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, b"\0" * 4, "InvalidShape"),
    # 2^64 elements: a wrapping product would equal the 0-byte range
    ({"t": {"dtype": "U8", "shape": [65536, 65536, 65536, 65536], "data_offsets": [0, 0]}}, b"", "InvalidShape"),
    ({"t": {"dtype": "F32", "shape": [4294967295, 4294967295, 4], "data_offsets": [0, 0]}}, b"", "InvalidShape"),
    ({"t": [1, 2]}, b"", "InvalidTensorEntry"),
    ({"x" * 257: {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}}, b"\0", "InvalidTensorEntry"),
    ([1, 2], b"", "InvalidJson"),
]


@pytest.mark.parametrize("header,data,err", MALFORMED)
def test_native_and_python_reject_alike(built_lib, header, data, err):
    with pytest.raises(SafetensorsError, match=err):
        SafetensorsFile(data=_raw(header, data))
    assert Native(_raw(header, data)).err == err


def test_native_header_checks(built_lib):
    cases = [(struct.pack("<Q", 1000) + b"{}", "InvalidHeader"),
             (struct.pack("<Q", 4) + b"{ab}", "InvalidJson"),
             (struct.pack("<Q", 1 << 40) + b"{}", "InvalidHeader"),
             (b"\0" * 9, "InvalidHeader"),
             (struct.pack("<Q", 0) + b"\0\0", "InvalidJson")]
    dup = b'{"t": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}, "t": {"dtype": "U8", "shape": [1], "data_offsets": [0, 1]}}'
    cases.append((struct.pack("<Q", len(dup)) + dup + b"\0", "InvalidJson"))
    for data, err in cases:
        assert Native(data).err == err, (data[:20], err)
        with pytest.raises(SafetensorsError, match=err):
            SafetensorsFile(data=data)
    header = {f"t{i}": {"dtype": "U8", "shape": [1], "data_offsets": [i, i + 1]} for i in range(1025)}
    assert Native(_raw(header, b"\0" * 1025)).err == "TooManyTensors"


def test_native_matches_python_on_files(built_lib, tmp_path):
    d = synth.ModelDims(vocab=300, hidden=128, inter=256, layers=2, n_q=2, n_kv=1, head_dim=64, gs=32, quant="q4")
    W = synth.make_model(d, seed=1)
    items = list(synth.iter_named_tensors(W))
    p = tmp_path / "m.safetensors"
    save_safetensors(p, items, metadata={"format": "mlx"})
    code = {"U8": 0, "U32": 1, "F16": 2, "BF16": 3, "F32": 4}
    with SafetensorsFile(p) as py:
        want = [(t.name, code[t.dtype], t.shape, t.array.tobytes()) for t in py.tensors.values()]
        f = Native(path=p)
        assert f.rc == 0 and f.tensors() == want
        f.close()
    from nnzap_b200 import _capi
    assert Native(path=tmp_path / "missing.safetensors").rc == _capi.NNZ_ENOTFOUND


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
