"""Safetensors checkpoint reader (host side of the weight loader).

Restates the reference's parser (nnmetal/src/safetensors.zig:1-582) for
the Python host: an 8-byte little-endian header length, a JSON header of
tensor descriptors ({"dtype", "shape", "data_offsets"}; "__metadata__"
skipped), then the contiguous tensor data, memory-mapped.  Same limits and
checks: header <= 16 MiB and inside the file, <= 1024 tensors, names <=
256 bytes, <= 4 dimensions, dtypes U8 / U32 / F16 / F32 / BF16, offsets
ordered and inside the data region, a repeated JSON member name invalid.
One check beyond the reference (which leaves it to its loader): a tensor's
byte range equals its element count times the dtype size.  The library's
C++ reader (nnz_safetensors_*) applies the same rules.

`load_safetensors(model, paths)` is Model.loadWeights
(nnmetal/src/model.zig:196-242): every tensor of every shard file is handed
to the library (which applies the reference loader's conversions at
finalize) and the model is finalized.
"""
from __future__ import annotations

import json
import math
import mmap
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable

import numpy as np

MAX_TENSORS = 1024
MAX_DIMS = 4
MAX_HEADER_BYTES = 16 * 1024 * 1024
MAX_NAME_LENGTH = 256


def _is_uint(v, top: int) -> bool:
    """A JSON integer (not a boolean) in [0, top]."""
    return isinstance(v, int) and not isinstance(v, bool) and 0 <= v <= top

# safetensors dtype string -> (numpy dtype, bytes per element)
DTYPES = {"U8": (np.uint8, 1), "U32": (np.uint32, 4), "F16": (np.float16, 2), "F32": (np.float32, 4),
          "BF16": (np.uint16, 2)}


class SafetensorsError(ValueError):
    """A malformed file; the message names the reference error it mirrors."""


@dataclass(frozen=True)
class TensorDescriptor:
    name: str
    dtype: str
    shape: tuple
    array: np.ndarray          # view into the mapping (BF16 as raw uint16)


class SafetensorsFile:
    """Memory-mapped safetensors file (SafetensorsFile, safetensors.zig:119)."""

    def __init__(self, path: str | Path | None = None, data: bytes | None = None):
        if (path is None) == (data is None):
            raise ValueError("give exactly one of path / data")
        self._file = None
        self._map = None
        if path is not None:
            self._file = open(path, "rb")
            size = Path(path).stat().st_size
            if size < 10:
                raise SafetensorsError("InvalidHeader: file shorter than 10 bytes")
            self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
            buf = memoryview(self._map)
        else:
            if len(data) < 10:
                raise SafetensorsError("InvalidHeader: buffer shorter than 10 bytes")
            buf = memoryview(data)
        self.tensors: dict[str, TensorDescriptor] = {}
        self._parse(buf)

    def _parse(self, buf: memoryview) -> None:
        (hlen,) = struct.unpack("<Q", bytes(buf[:8]))
        if hlen > MAX_HEADER_BYTES:
            raise SafetensorsError(f"InvalidHeader: header length {hlen} exceeds {MAX_HEADER_BYTES}")
        start = 8 + hlen
        if start > len(buf):
            raise SafetensorsError(f"InvalidHeader: header length ({hlen}) exceeds file size ({len(buf)})")
        def no_duplicates(pairs):
            # a repeated member name is invalid, as in the reference's std.json
            d = {}
            for k, v in pairs:
                if k in d:
                    raise SafetensorsError(f"InvalidJson: duplicate member '{k}'")
                d[k] = v
            return d

        try:
            header = json.loads(bytes(buf[8:start]).decode("utf-8"), object_pairs_hook=no_duplicates)
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise SafetensorsError(f"InvalidJson: {e}") from None
        if not isinstance(header, dict):
            raise SafetensorsError("InvalidJson: header is not an object")
        data = buf[start:]
        for name, desc in header.items():
            if name == "__metadata__":
                continue
            if len(self.tensors) >= MAX_TENSORS:
                raise SafetensorsError(f"TooManyTensors: more than {MAX_TENSORS}")
            if not name or len(name.encode()) > MAX_NAME_LENGTH:
                raise SafetensorsError("InvalidTensorEntry: tensor name empty or longer than 256 bytes")
            if not isinstance(desc, dict):
                raise SafetensorsError(f"InvalidTensorEntry: '{name}'")
            if "dtype" not in desc:
                raise SafetensorsError(f"MissingDtype: '{name}'")
            dt = desc["dtype"]
            if not isinstance(dt, str):
                raise SafetensorsError(f"InvalidDtype: '{name}'")
            if dt not in DTYPES:
                raise SafetensorsError(f"UnsupportedDtype: '{name}' has {dt}")
            if "shape" not in desc:
                raise SafetensorsError(f"MissingShape: '{name}'")
            shape = desc["shape"]
            if not isinstance(shape, list) or not all(_is_uint(d, 0xFFFFFFFF) for d in shape):
                raise SafetensorsError(f"InvalidShape: '{name}'")
            if len(shape) > MAX_DIMS:
                raise SafetensorsError(f"TooManyDimensions: '{name}' has {len(shape)}")
            if "data_offsets" not in desc:
                raise SafetensorsError(f"MissingDataOffsets: '{name}'")
            off = desc["data_offsets"]
            if (not isinstance(off, list) or len(off) != 2 or not all(_is_uint(o, 2 ** 63 - 1) for o in off)
                    or off[0] > off[1]):
                raise SafetensorsError(f"InvalidDataOffsets: '{name}'")
            if off[1] > len(data):
                raise SafetensorsError(f"DataOffsetOutOfBounds: '{name}' ends at {off[1]} of {len(data)}")
            npdt, size = DTYPES[dt]
            count = math.prod(int(d) for d in shape)   # Python ints: no silent wrap-around
            if count * size >= 1 << 64:
                raise SafetensorsError(f"InvalidShape: '{name}' element count overflows")
            if off[1] - off[0] != count * size:
                raise SafetensorsError(f"InvalidDataOffsets: '{name}' holds {off[1] - off[0]} bytes, "
                                       f"shape needs {count * size}")
            arr = np.frombuffer(data[off[0]:off[1]], dtype=npdt).reshape(shape)
            self.tensors[name] = TensorDescriptor(name, dt, tuple(shape), arr)

    def get_tensor(self, name: str) -> TensorDescriptor | None:
        return self.tensors.get(name)

    def close(self) -> None:
        self.tensors = {}
        if self._map is not None:
            try:
                self._map.close()
            except BufferError:
                pass   # arrays handed out still view the mapping; it goes with them
            self._map = None
        if self._file is not None:
            self._file.close()
            self._file = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def save_safetensors(path: str | Path, tensors: Iterable, metadata: dict | None = None) -> None:
    """Write (name, numpy array[, dtype string]) entries as a safetensors file
    (uint16 arrays are written as F16 unless "BF16" is given)."""
    names = {np.dtype(np.uint8): "U8", np.dtype(np.uint32): "U32", np.dtype(np.float16): "F16",
             np.dtype(np.float32): "F32", np.dtype(np.uint16): "F16"}
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for item in tensors:
        name, arr = item[0], np.ascontiguousarray(item[1])
        dt = item[2] if len(item) > 2 else names[arr.dtype]
        b = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * (-len(hj) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def load_safetensors(model, paths: Iterable[str | Path]) -> None:
    """Model.loadWeights (model.zig:196-242): every tensor of every shard
    to the library, then finalize (packing, KV cache, scratch)."""
    from . import _capi as capi
    code = {"U8": capi.NNZ_DT_U8, "U32": capi.NNZ_DT_U32, "F16": capi.NNZ_DT_F16,
            "F32": capi.NNZ_DT_F32, "BF16": capi.NNZ_DT_BF16}
    files = [SafetensorsFile(p) for p in paths]
    try:
        for f in files:
            for t in f.tensors.values():
                model.load_tensor(t.name, t.array, code[t.dtype])
        model.finalize()
    finally:
        for f in files:
            f.close()
