"""Device sampling (sampleToken, transformer.zig:3833-3869) against the
oracle's restatement with the same uniform draws."""
import numpy as np
import pytest

from gpu_helpers import R
from nnzap_b200._capi import check, lib, ptr

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,T,k,p", [(1000, 1.0, 0, 1.0), (1000, 0.7, 50, 1.0), (1000, 1.3, 0, 0.9),
                                     (1000, 0.8, 40, 0.95), (151936, 0.6, 0, 0.92), (151936, 1.0, 64, 1.0)])
def test_sample_matches_oracle(cuda, built_lib, n, T, k, p):
    torch = cuda
    rng = np.random.default_rng(n + k)
    rows = 24
    logits = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    u = rng.random(rows, dtype=np.float32)
    d_logits = torch.from_numpy(logits.copy()).cuda()
    d_u = torch.from_numpy(u).cuda()
    d_tok = torch.zeros(rows, dtype=torch.int32, device="cuda")
    check(lib().nnz_sample(ptr(d_logits), rows, n, n, T, k, p, ptr(d_u), ptr(d_tok), None))
    torch.cuda.synchronize()
    got = d_tok.cpu().numpy()
    mism = 0
    for r in range(rows):
        want = R.sample_token(logits[r], T, k, p, float(u[r]))
        if got[r] != want:
            # only a draw within f32 rounding of a CDF boundary may land on a
            # neighbouring token (different summation order)
            mism += 1
            cum = R.sample_cdf(logits[r], T, k, p)
            lo = min(int(got[r]), want)
            assert abs(float(cum[lo]) - float(u[r])) < 1e-4, (r, got[r], want, cum[lo], u[r])
    assert mism <= 1


def test_sample_top_k1_is_argmax(cuda, built_lib):
    torch = cuda
    rng = np.random.default_rng(1)
    logits = rng.standard_normal((8, 5000)).astype(np.float32)
    d = torch.from_numpy(logits.copy()).cuda()
    u = torch.from_numpy(rng.random(8, dtype=np.float32)).cuda()
    tok = torch.zeros(8, dtype=torch.int32, device="cuda")
    check(lib().nnz_sample(ptr(d), 8, 5000, 5000, 1.0, 1, 1.0, ptr(u), ptr(tok), None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tok.cpu().numpy(), logits.argmax(axis=1))
