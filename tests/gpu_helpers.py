"""Shared helpers for the GPU parity tests (call the CUDA path through the
C ABI, compare with the CPU oracle)."""
import numpy as np

from nnzap_b200 import _capi
from nnzap_b200._capi import check, lib, ptr
from oracle import qwen3_ref as R


def pack(fmt, t, M, K, gs, sub=1, packed=None, sub_index=0):
    """Reference-format tensor dict -> packed host bytes (via the C ABI)."""
    L = lib()
    if packed is None:
        packed = np.zeros(L.nnz_packed_bytes(fmt, M, K, gs, sub), dtype=np.uint8)
    w = np.ascontiguousarray(t["weight"])
    s = np.ascontiguousarray(t["scales"], dtype=np.uint16)
    b = None if fmt == 0 else np.ascontiguousarray(t["biases"], dtype=np.uint16)
    check(L.nnz_pack_weights(fmt, ptr(w), ptr(s), ptr(b), M, K, gs, sub, sub_index, ptr(packed)))
    return packed


def to_dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def cfg_for(fmt, gs, K, scale_dtype="f16", bf16=False):
    return R.Cfg(vocab=8, hidden=K, inter=K, layers=1, n_q=1, n_kv=1, head_dim=128, gs=gs,
                 quant="q1" if fmt == 0 else "q4", scale_dtype=scale_dtype, bf16_faithful=bf16)


def close(got, want, atol, rtol, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = np.abs(got - want)
    lim = atol + rtol * np.abs(want)
    bad = err > lim
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance; "
                           f"max err {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}")
    return float(err.max())
