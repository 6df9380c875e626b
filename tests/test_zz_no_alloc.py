"""nnz_qmv_noalloc: the matvec for callers that cannot allocate device memory.

Some hosts must not call cudaMalloc once they are running (an engine that
gave its whole device memory budget to its own pool at start-up, or work
issued while another thread captures a CUDA graph).  nnz_qmv_noalloc serves
them with split-K scratch compiled into the library.  This file checks it
against nnz_qmv on the same inputs, twice in a row (the shared scratch keeps
the previous call's contents), and that an oversized problem is refused.

It is collected last on purpose (``zz``) and passes both alone in a fresh
process and after the rest of the suite.
"""
import numpy as np
import pytest

from gpu_helpers import R, cfg_for, check, close, lib, pack, ptr, to_dev
from nnzap_b200 import _capi, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt,M,K,gs,batch,out_kind", [
    (0, 2048, 6144, 128, 1, 1),      # Q1 down-proj shape, f32 out (split-K active)
    (1, 6144, 2048, 64, 1, 0),       # Q4 config-0 shape, fp16 out
    (1, 1000, 512, 32, 13, 2),       # ragged rows, batch > 8, residual add
])
def test_noalloc_matches_qmv_twice(cuda, built_lib, fmt, M, K, gs, batch, out_kind):
    torch = cuda
    rng = np.random.default_rng(M + K + batch)
    t = synth.rand_q1(rng, M, K, gs) if fmt == 0 else synth.rand_q4(rng, M, K, gs)
    w = to_dev(torch, pack(fmt, t, M, K, gs))
    odt = torch.float16 if out_kind == 0 else torch.float32
    for call in range(2):
        x = to_dev(torch, rng.standard_normal((batch, K)).astype(np.float16))
        base = torch.randn((batch, M), device="cuda", dtype=torch.float32).to(odt)
        ref, got = base.clone(), base.clone()
        check(lib().nnz_qmv(fmt, 0, 0, ptr(w), M, K, gs, ptr(x), K, batch, ptr(ref), M, out_kind, None))
        check(lib().nnz_qmv_noalloc(fmt, 0, 0, ptr(w), M, K, gs, ptr(x), K, batch, ptr(got), M,
                                    out_kind, None))
        torch.cuda.synchronize()
        # same tolerance as the nnz_qmv parity tests (fp16 output: one rounding step)
        tol = (2e-3, 2e-3) if out_kind == 0 else (1e-3, 1e-4)
        close(got.float().cpu().numpy(), ref.float().cpu().numpy(), *tol, f"call {call}")
        # and both against the oracle
        want = R.qmv(cfg_for(fmt, gs, K), t, M, K, x.cpu().numpy().astype(np.float32))
        if out_kind == 2:
            want = want + base.float().cpu().numpy()
        close(got.float().cpu().numpy(), want, *((2e-3, 2e-3) if out_kind == 0 else (1e-3, 1e-4)),
              f"oracle call {call}")
        # no bounded wait gave up inside either call
        assert lib().nnz_stream_check(None) == _capi.NNZ_OK


def test_noalloc_rejects_oversized(cuda, built_lib):
    """Beyond the fixed scratch (here: more split-K arrival counters than the
    array holds) the call is refused before anything is launched."""
    torch = cuda
    M, K, gs, batch = 151936, 2048, 128, 1024      # 128 batch chunks x 1187 row tiles
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")   # never touched
    rc = lib().nnz_qmv_noalloc(0, 0, 0, ptr(dummy), M, K, gs, ptr(dummy), K, batch, ptr(dummy), M,
                               1, None)
    assert rc == _capi.NNZ_EINVAL
    assert b"fixed limits" in lib().nnz_last_error()


def test_noalloc_rejects_oversized_scratch(cuda, built_lib):
    """The branch that protects the fixed split-K scratch: a batch-8 matvec
    with K = 524288 (group 256) needs 16 counters but ~11 MB of split-K
    partials, more than the 8 MiB array, and is refused before any launch."""
    torch = cuda
    M, K, gs, batch = 2048, 524288, 256, 8
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")   # never touched
    rc = lib().nnz_qmv_noalloc(0, 0, 0, ptr(dummy), M, K, gs, ptr(dummy), K, batch, ptr(dummy), M,
                               1, None)
    assert rc == _capi.NNZ_EINVAL
    err = lib().nnz_last_error()
    assert b"fixed limits" in err and b"split-K scratch" in err
