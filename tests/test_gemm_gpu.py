"""GPU parity of the tcgen05 prefill GEMM against the oracle.

Q1 weights (+-scale) are exact in fp16, so the only difference is the f32
accumulation order inside the tensor core: |err| <= 1e-3 + 1e-4 |ref|.  Q4
weights scale*q + bias are rounded to fp16 before the MMA (one fp16 rounding
per weight, relative error up to 2^-11, summed over K terms), so the Q4
check allows 1e-2 + 2e-3 |ref|.
"""
import numpy as np
import pytest

from gpu_helpers import R, cfg_for, check, close, lib, ptr, to_dev
from nnzap_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt,M,K,N,gs", [
    (0, 128, 128, 128, 128), (0, 512, 2048, 4096, 128), (0, 77, 2048, 300, 128),
    (0, 200, 6144, 2048, 128), (1, 512, 2048, 2048, 64), (1, 33, 512, 130, 64),
    # 4 and 2 M tiles per CTA (wide N), with a ragged last M tile
    (0, 400, 2048, 12288, 128), (1, 300, 1024, 6144, 64),
    # decode batches (<= 128 rows: weights in TMEM), split K and whole K
    (0, 64, 2048, 4096, 128), (0, 64, 6144, 2048, 128), (1, 64, 2048, 2048, 64),
    (0, 100, 2048, 12288, 128), (1, 16, 2048, 12288, 64)])
def test_prefill_gemm_vs_oracle(cuda, built_lib, fmt, M, K, N, gs):
    torch = cuda
    rng = np.random.default_rng(M + K + N)
    t = synth.rand_q1(rng, N, K, gs) if fmt == 0 else synth.rand_q4(rng, N, K, gs)
    x = rng.standard_normal((M, K)).astype(np.float16)
    keep = [to_dev(torch, np.ascontiguousarray(t["weight"]).view(np.uint8)),
            to_dev(torch, t["scales"]), to_dev(torch, t.get("biases", t["scales"])), to_dev(torch, x)]
    y16 = torch.empty((M, N), dtype=torch.float16, device="cuda")
    base = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    y32 = to_dev(torch, base)
    for out, kind in ((y16, 0), (y32, 2)):
        check(lib().nnz_prefill_gemm(fmt, 0, ptr(keep[0]), ptr(keep[1]),
                                     ptr(keep[2]) if fmt == 1 else None, M, K, N, gs, ptr(keep[3]),
                                     ptr(out), kind, None))
    torch.cuda.synchronize()
    want = R.qmv(cfg_for(fmt, gs, K), t, N, K, x.astype(np.float32))
    tol = (1e-3, 1e-4) if fmt == 0 else (1e-2, 2e-3)
    close(y32.cpu().numpy(), base + want, *tol, "f32 add")
    close(y16.cpu().numpy().astype(np.float32), want, 2e-3 + tol[0], 2e-3 + tol[1], "f16")
