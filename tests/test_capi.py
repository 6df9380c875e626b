"""CPU tests of the C ABI: the library loads, exports every symbol the
header declares, validates arguments, and packs weights losslessly."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_symbols():
    text = (ROOT / "include" / "nnz_b200.h").read_text()
    return sorted(set(re.findall(r"\b(nnz_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_header_symbol(built_lib):
    import ctypes
    lib = ctypes.CDLL(str(built_lib))
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    from nnzap_b200 import _capi
    bound = {n for n, _, _ in _capi.SIGNATURES}
    assert set(header_symbols()) == bound


def test_version_and_errors(built_lib):
    from nnzap_b200 import _capi
    L = _capi.lib()
    assert L.nnz_version() >= 1
    assert L.nnz_device_count() >= 0
    # invalid config is rejected before any device call
    c = _capi.NnzConfig()
    import ctypes as C
    h = C.c_void_p()
    rc = L.nnz_model_create(0, C.byref(c), C.byref(h))
    assert rc == _capi.NNZ_EINVAL
    assert L.nnz_last_error()
    assert L.nnz_packed_bytes(0, 128, 100, 128, 1) == 0      # K % gs != 0
    assert L.nnz_packed_bytes(0, 128, 256, 128, 1) == 2 * 2304
    assert L.nnz_packed_bytes(1, 129, 256, 64, 2) == 2 * 4 * 2 * 4608


def _rand_q1(rng, M, K, gs):
    return (rng.integers(0, 256, M * K // 8, dtype=np.uint8),
            rng.integers(0, 2 ** 16, M * K // gs, dtype=np.uint16), None)


def _rand_q4(rng, M, K, gs):
    return (rng.integers(0, 2 ** 32, M * K // 8, dtype=np.uint32),
            rng.integers(0, 2 ** 16, M * K // gs, dtype=np.uint16),
            rng.integers(0, 2 ** 16, M * K // gs, dtype=np.uint16))


@pytest.mark.parametrize("fmt,M,K,gs,sub", [
    (0, 128, 128, 128, 1), (0, 200, 256, 128, 1), (0, 300, 512, 64, 2), (0, 33, 96, 32, 1),
    (1, 128, 128, 64, 1), (1, 77, 256, 64, 2), (1, 256, 192, 32, 1), (1, 130, 256, 128, 1)])
def test_pack_unpack_roundtrip(built_lib, fmt, M, K, gs, sub):
    from nnzap_b200._capi import lib, check, ptr
    rng = np.random.default_rng(M * 7 + K)
    L = lib()
    nbytes = L.nnz_packed_bytes(fmt, M, K, gs, sub)
    packed = np.zeros(nbytes, dtype=np.uint8)
    mats = []
    for si in range(sub):
        w, s, b = (_rand_q1 if fmt == 0 else _rand_q4)(rng, M, K, gs)
        mats.append((w, s, b))
        check(L.nnz_pack_weights(fmt, ptr(w), ptr(s), ptr(b), M, K, gs, sub, si, ptr(packed)))
    for si, (w, s, b) in enumerate(mats):
        w2, s2 = np.zeros_like(w), np.zeros_like(s)
        b2 = None if b is None else np.zeros_like(b)
        check(L.nnz_unpack_weights(fmt, ptr(packed), M, K, gs, sub, si, ptr(w2), ptr(s2), ptr(b2)))
        np.testing.assert_array_equal(w2, w)
        np.testing.assert_array_equal(s2, s)
        if b is not None:
            np.testing.assert_array_equal(b2, b)


def test_pack_rejects_bad_shapes(built_lib):
    from nnzap_b200._capi import lib, ptr, NNZ_EINVAL
    L = lib()
    w = np.zeros(16, dtype=np.uint8)
    s = np.zeros(4, dtype=np.uint16)
    out = np.zeros(4096, dtype=np.uint8)
    assert L.nnz_pack_weights(0, ptr(w), ptr(s), None, 1, 100, 128, 1, 0, ptr(out)) == NNZ_EINVAL
    assert L.nnz_pack_weights(1, ptr(w), ptr(s), None, 1, 128, 64, 1, 0, ptr(out)) == NNZ_EINVAL
    assert L.nnz_pack_weights(0, ptr(w), ptr(s), None, 1, 128, 128, 1, 1, ptr(out)) == NNZ_EINVAL


def test_packed_layout_q1_bit_positions(built_lib):
    """One set bit lands where the packed-layout contract says it does."""
    from nnzap_b200._capi import lib, check, ptr
    L = lib()
    M, K, gs = 128, 128, 128
    for row, col in [(0, 0), (17, 5), (100, 31), (127, 127), (40, 64)]:
        bits = np.zeros(M * K // 8, dtype=np.uint8)
        f = row * K + col
        bits[f // 8] = 1 << (f % 8)
        s = np.zeros(M * K // gs, dtype=np.uint16)
        packed = np.zeros(L.nnz_packed_bytes(0, M, K, gs, 1), dtype=np.uint8)
        check(L.nnz_pack_weights(0, ptr(bits), ptr(s), None, M, K, gs, 1, 0, ptr(packed)))
        words = packed[: 4 * 512].view(np.uint32)
        j, g, rlo = row // 16, row % 8, (row // 8) % 2
        c, kk = col // 32, col % 32
        t, i, rhi = (kk % 16) // 4, kk % 4, kk // 16
        lane, r = 4 * g + t, 2 * rhi + rlo
        w = words[c * 128 + lane * 4 + r]
        assert w == (1 << (j + 8 * i)), (row, col, hex(w))
        assert np.count_nonzero(words) == 1
