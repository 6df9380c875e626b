"""Failure detection on the GPU without a GPU fault: every wait in the
library is bounded, and a wait that runs out is reported to the host as
NNZ_ETIMEDOUT while the CUDA context stays usable.

The case: the peer-memory all-reduce of tensor-parallel decode, run on one
GPU as rank 0 of a two-rank group whose peer is a local stand-in buffer that
nothing ever writes (a flag that nothing sets), with a short test limit on
the wait.  Nothing waits on another GPU or process."""
import ctypes as C
import time

import numpy as np
import pytest

from gpu_helpers import check, lib, ptr
from nnzap_b200 import _capi

pytestmark = pytest.mark.gpu


def test_bounded_peer_wait_reports_timeout(cuda, built_lib):
    torch = cuda
    flags = C.c_int(0)
    t0 = time.perf_counter()
    rc = lib().nnz_debug_tp_wait_timeout(2000, C.byref(flags))
    dt = time.perf_counter() - t0
    assert rc == _capi.NNZ_ETIMEDOUT, (rc, lib().nnz_last_error())
    assert flags.value & 8                          # ERR_SPIN_TIMEOUT
    assert b"timed out" in lib().nnz_last_error()
    assert dt < 30, dt
    # the context is still usable: ordinary device work and a clean error state
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2
    assert lib().nnz_stream_check(None) == _capi.NNZ_OK
