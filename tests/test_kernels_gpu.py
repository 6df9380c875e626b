"""GPU parity of the per-kernel entry points against the CPU oracle.

Tolerances (stated per check):
  * dequantized weights: bit-exact;
  * f32 matvec outputs: |err| <= 1e-3 + 1e-4 |ref|  (f32 summation order and
    the 15-bit fixed-point activation grid, which is exact for every element
    within 1/16 of its group maximum);
  * fp16 outputs: one fp16 rounding step on top of that, |err| <= 2e-3 + 2e-3 |ref|;
  * argmax: identical unless the oracle's top-2 gap is below 1e-3.
"""
import numpy as np
import pytest

from gpu_helpers import R, check, cfg_for, close, lib, pack, ptr, to_dev
from nnzap_b200 import _capi, synth

pytestmark = pytest.mark.gpu


def _mats(fmt, M, K, gs, seed, scale_dtype="f16"):
    rng = np.random.default_rng(seed)
    if fmt == 0:
        return synth.rand_q1(rng, M, K, gs)
    return synth.rand_q4(rng, M, K, gs, scale_dtype)


@pytest.mark.parametrize("fmt,M,K,gs,sd", [
    (0, 300, 256, 128, "f16"), (0, 128, 2048, 128, "f16"), (0, 64, 192, 64, "f16"),
    (1, 6144, 2048, 64, "f16"), (1, 200, 512, 64, "bf16"), (1, 129, 256, 128, "f16")])
def test_dequant_bit_exact(cuda, built_lib, fmt, M, K, gs, sd):
    torch = cuda
    t = _mats(fmt, M, K, gs, seed=M + K, scale_dtype=sd)
    dev = to_dev(torch, pack(fmt, t, M, K, gs))
    out = torch.empty((M, K), dtype=torch.float32, device="cuda")
    check(lib().nnz_dequant(fmt, 1 if sd == "bf16" else 0, ptr(dev), M, K, gs, 1, 0, ptr(out), None))
    torch.cuda.synchronize()
    want = R.dequant_tensor(cfg_for(fmt, gs, K, sd), t, M, K)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_dequant_sub_interleaved(cuda, built_lib):
    torch = cuda
    M, K, gs = 256, 512, 128
    ts = [_mats(0, M, K, gs, seed=s) for s in (1, 2)]
    packed = None
    for si, t in enumerate(ts):
        packed = pack(0, t, M, K, gs, sub=2, packed=packed, sub_index=si)
    dev = to_dev(torch, packed)
    for si, t in enumerate(ts):
        out = torch.empty((M, K), dtype=torch.float32, device="cuda")
        check(lib().nnz_dequant(0, 0, ptr(dev), M, K, gs, 2, si, ptr(out), None))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), R.dequant_tensor(cfg_for(0, gs, K), t, M, K))


QMV_CASES = [
    # fmt, M, K, gs, batch   (config 0 is (1, 6144, 2048, 64, 1))
    (1, 6144, 2048, 64, 1), (1, 6144, 2048, 64, 8), (0, 4096, 2048, 128, 1),
    (0, 2048, 6144, 128, 1), (0, 2048, 6144, 128, 5), (0, 300, 256, 128, 3),
    (1, 2048, 6144, 64, 1), (1, 1000, 512, 32, 13), (0, 151936, 2048, 128, 1),
    (0, 256, 2048, 128, 64), (1, 256, 2048, 64, 20)]


@pytest.mark.parametrize("fmt,M,K,gs,batch", QMV_CASES)
def test_qmv_vs_oracle(cuda, built_lib, fmt, M, K, gs, batch):
    torch = cuda
    t = _mats(fmt, M, K, gs, seed=M * 3 + batch)
    w = to_dev(torch, pack(fmt, t, M, K, gs))
    rng = np.random.default_rng(batch)
    x = rng.standard_normal((batch, K)).astype(np.float16)
    xd = to_dev(torch, x)
    want = R.qmv(cfg_for(fmt, gs, K), t, M, K, x.astype(np.float32))
    y32 = torch.empty((batch, M), dtype=torch.float32, device="cuda")
    check(lib().nnz_qmv(fmt, 0, 0, ptr(w), M, K, gs, ptr(xd), K, batch, ptr(y32), M, 1, None))
    y16 = torch.empty((batch, M), dtype=torch.float16, device="cuda")
    check(lib().nnz_qmv(fmt, 0, 0, ptr(w), M, K, gs, ptr(xd), K, batch, ptr(y16), M, 0, None))
    torch.cuda.synchronize()
    close(y32.cpu().numpy(), want, 1e-3, 1e-4, "f32 out")
    close(y16.cpu().numpy().astype(np.float32), want, 2e-3, 2e-3, "f16 out")


def test_qmv_residual_add(cuda, built_lib):
    torch = cuda
    fmt, M, K, gs = 0, 2048, 2048, 128
    t = _mats(fmt, M, K, gs, seed=5)
    w = to_dev(torch, pack(fmt, t, M, K, gs))
    x = np.random.default_rng(2).standard_normal((2, K)).astype(np.float16)
    r0 = np.random.default_rng(3).standard_normal((2, M)).astype(np.float32)
    res = to_dev(torch, r0)
    xd = to_dev(torch, x)
    check(lib().nnz_qmv(fmt, 0, 0, ptr(w), M, K, gs, ptr(xd), K, 2, ptr(res), M, 2, None))
    torch.cuda.synchronize()
    want = r0 + R.qmv(cfg_for(fmt, gs, K), t, M, K, x.astype(np.float32))
    close(res.cpu().numpy(), want, 1e-3, 1e-4, "resadd")


@pytest.mark.parametrize("fmt,bf16", [(0, False), (1, False), (1, True)])
def test_qmv_norm_prologue(cuda, built_lib, fmt, bf16):
    torch = cuda
    M, K = 1024, 2048
    gs = 128 if fmt == 0 else 64
    sd = "bf16" if bf16 else "f16"
    t = _mats(fmt, M, K, gs, seed=11, scale_dtype=sd)
    w = to_dev(torch, pack(fmt, t, M, K, gs))
    rng = np.random.default_rng(4)
    res = (rng.standard_normal((3, K)) * 3).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    out = torch.empty((3, M), dtype=torch.float16, device="cuda")
    res_d, nw_d = to_dev(torch, res), to_dev(torch, nw)   # keep alive until the sync
    check(lib().nnz_qmv_norm(fmt, int(bf16), int(bf16), ptr(w), M, K, gs, ptr(res_d),
                             ptr(nw_d), 1e-6, 3, ptr(out), M, 0, None))
    torch.cuda.synchronize()
    cfg = cfg_for(fmt, gs, K, sd, bf16)
    xn = R._to_f16(cfg, R.rmsnorm(res, nw))
    want = R._to_f16(cfg, R.qmv(cfg, t, M, K, xn))
    # bf16 mode: outputs are truncated to bf16, so allow one bf16 step (2^-8 relative)
    close(out.cpu().numpy().astype(np.float32), want, 2e-3, 8e-3 if bf16 else 2e-3, "norm+qmv")


def test_lm_head_argmax(cuda, built_lib):
    torch = cuda
    fmt, V, K, gs = 0, 151936, 2048, 128
    rng = np.random.default_rng(9)
    emb = (rng.standard_normal((V, K), dtype=np.float32) * 0.02).astype(np.float16)
    t = synth.quantize_q1_sign(emb, gs)
    w = to_dev(torch, pack(fmt, t, V, K, gs))
    res = rng.standard_normal((2, K)).astype(np.float32) * 4
    nw = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    logits = torch.empty((2, V), dtype=torch.float32, device="cuda")
    am = torch.zeros(2, dtype=torch.int32, device="cuda")
    res_d, nw_d = to_dev(torch, res), to_dev(torch, nw)
    check(lib().nnz_lm_head_argmax(fmt, 0, 0, ptr(w), V, K, gs, ptr(res_d), ptr(nw_d), 1e-6, 2,
                                   ptr(logits), ptr(am), None))
    torch.cuda.synchronize()
    cfg = cfg_for(fmt, gs, K)
    xn = R._to_f16(cfg, R.rmsnorm(res, nw))
    want = R.qmv(cfg, t, V, K, xn)
    got = logits.cpu().numpy()
    close(got, want, 1e-3, 1e-4, "logits")
    for b in range(2):
        a = int(am[b].item())
        assert a == int(np.argmax(got[b]))
        assert want[b].max() - want[b][a] <= 1e-3


@pytest.mark.parametrize("fmt,batch", [(0, 1), (0, 8), (1, 1), (1, 8)])
def test_mlp_block_config1(cuda, built_lib, fmt, batch):
    """Benchmark configuration 1 (Q1) and its 4-bit twin: down(SiLU(gate x) * up x)."""
    torch = cuda
    H, I = 2048, 6144
    gs = 128 if fmt == 0 else 64
    rng = np.random.default_rng(21)
    if fmt == 0:
        g, u, d = (synth.rand_q1(rng, I, H, gs), synth.rand_q1(rng, I, H, gs),
                   synth.rand_q1(rng, H, I, gs))
    else:
        g, u, d = (synth.rand_q4(rng, I, H, gs), synth.rand_q4(rng, I, H, gs),
                   synth.rand_q4(rng, H, I, gs))
    gu = pack(fmt, g, I, H, gs, sub=2, sub_index=0)
    gu = pack(fmt, u, I, H, gs, sub=2, packed=gu, sub_index=1)
    dn = pack(fmt, d, H, I, gs)
    x = rng.standard_normal((batch, H)).astype(np.float16)
    out = torch.empty((batch, H), dtype=torch.float32, device="cuda")
    gu_d, dn_d, x_d = to_dev(torch, gu), to_dev(torch, dn), to_dev(torch, x)
    check(lib().nnz_mlp(fmt, 0, 0, ptr(gu_d), ptr(dn_d), H, I, gs, ptr(x_d), batch, ptr(out), None))
    torch.cuda.synchronize()
    cfg = R.Cfg(vocab=8, hidden=H, inter=I, layers=1, n_q=16, n_kv=8, head_dim=128, gs=gs,
                quant="q1" if fmt == 0 else "q4")
    want = R.mlp_block(cfg, g, u, d, x.astype(np.float32))
    # the SiLU*mul intermediate is fp16 on both sides; one fp16 step there
    # moves the f32 output by at most ~|w| * 2^-11 per element
    close(out.cpu().numpy(), want, 5e-2, 2e-3, "mlp")


def _attn_oracle(qkv, qn, kn, kc, vc, pos, n_q, n_kv, hd, theta, style):
    """Oracle decode attention for one row with the cache already holding
    positions < pos; returns (out[n_q*hd], k_new fp16, v_new fp16)."""
    q = qkv[: n_q * hd].astype(np.float32).reshape(1, n_q, hd)
    k = qkv[n_q * hd: (n_q + n_kv) * hd].astype(np.float32).reshape(1, n_kv, hd)
    v = qkv[(n_q + n_kv) * hd:].astype(np.float16).reshape(n_kv, hd)
    P = np.array([pos])
    q = R.rope(R.rmsnorm(q, qn), P, theta, style)[0]
    k = R.rope(R.rmsnorm(k, kn), P, theta, style)[0].astype(np.float16)
    kcache = kc[:, : pos + 1].copy()
    vcache = vc[:, : pos + 1].copy()
    kcache[:, pos] = k
    vcache[:, pos] = v
    return R.attention_decode(q, kcache, vcache, n_kv).reshape(-1), k, v


@pytest.mark.parametrize("hd,n_q,n_kv,pos,splits,style", [
    (128, 16, 8, 0, 0, "pairwise"), (128, 16, 8, 1, 0, "pairwise"), (128, 16, 8, 33, 0, "pairwise"),
    (128, 16, 8, 2048, 0, "pairwise"), (128, 16, 8, 777, 7, "pairwise"), (128, 16, 8, 95, 1, "pairwise"),
    (128, 16, 8, 300, 0, "half_split"), (64, 2, 2, 5, 0, "pairwise"), (64, 8, 2, 130, 3, "half_split"),
    (128, 32, 8, 4095, 0, "pairwise")])
def test_attention_decode(cuda, built_lib, hd, n_q, n_kv, pos, splits, style):
    _attention_case(cuda, hd, n_q, n_kv, [pos, max(0, pos // 2)], splits, style, pos + hd)


@pytest.mark.parametrize("n_q,n_kv,positions", [
    (8, 8, [0, 15, 16, 257, 4095]), (16, 8, [255, 256, 511, 4000, 17, 1, 2048]),
    (32, 8, [3, 1000, 4094])])
def test_attention_decode_batch(cuda, built_lib, n_q, n_kv, positions):
    """Rows at chunk and block edges (16-position blocks, 256-position chunks)."""
    _attention_case(cuda, 128, n_q, n_kv, positions, 0, "pairwise", len(positions))


def _attention_case(cuda, hd, n_q, n_kv, pos_list, splits, style, seed):
    torch = cuda
    rng = np.random.default_rng(seed)
    rows, max_ctx, theta = len(pos_list), 4096, 1e6
    qkv = rng.standard_normal((rows, (n_q + 2 * n_kv) * hd)).astype(np.float16)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kc = rng.standard_normal((rows, n_kv, max_ctx, hd)).astype(np.float16)
    vc = rng.standard_normal((rows, n_kv, max_ctx, hd)).astype(np.float16)
    positions = np.array(pos_list, dtype=np.int32)
    kd, vd = to_dev(torch, kc), to_dev(torch, vc)
    out = torch.empty((rows, n_q * hd), dtype=torch.float16, device="cuda")
    keep = [to_dev(torch, a) for a in (qkv, qn, kn, positions)]   # alive until the sync
    check(lib().nnz_attn_decode(ptr(keep[0]), ptr(keep[1]), ptr(keep[2]),
                                ptr(kd), ptr(vd), max_ctx, ptr(keep[3]), rows, n_q,
                                n_kv, hd, 1e-6, theta, 0 if style == "pairwise" else 1, splits,
                                ptr(out), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float32)
    kd, vd = kd.cpu().numpy(), vd.cpu().numpy()
    for r in range(rows):
        p = int(positions[r])
        want, k, v = _attn_oracle(qkv[r], qn, kn, kc[r], vc[r], p, n_q, n_kv, hd, theta, style)
        close(got[r], want, 2e-3, 2e-3, f"attn row {r}")
        np.testing.assert_array_equal(vd[r][:, p], v)
        close(kd[r][:, p].astype(np.float32), k.astype(np.float32), 2e-3, 2e-3, "k cache")
        # untouched history
        np.testing.assert_array_equal(kd[r][:, :p], kc[r][:, :p])


def test_stream_check_reports_bad_position(cuda, built_lib):
    """A device-side error of a per-kernel entry point (here a position past
    max_context_length, which the attention kernel clamps and flags) reaches
    the host through nnz_stream_check as NNZ_EDEVICE, once: the check clears it."""
    torch = cuda
    hd, n_q, n_kv, max_ctx = 128, 2, 1, 64
    assert lib().nnz_stream_check(None) == _capi.NNZ_OK
    qkv = to_dev(torch, np.ones((1, (n_q + 2 * n_kv) * hd), np.float16))
    qn = to_dev(torch, np.ones(hd, np.float32))
    kd = torch.zeros((n_kv, max_ctx, hd), dtype=torch.float16, device="cuda")
    vd = torch.zeros_like(kd)
    pos = to_dev(torch, np.array([max_ctx + 5], np.int32))
    out = torch.empty((1, n_q * hd), dtype=torch.float16, device="cuda")
    check(lib().nnz_attn_decode(ptr(qkv), ptr(qn), ptr(qn), ptr(kd), ptr(vd), max_ctx, ptr(pos), 1, n_q,
                                n_kv, hd, 1e-6, 1e6, 0, 1, ptr(out), None))
    assert lib().nnz_stream_check(None) == _capi.NNZ_EDEVICE
    assert b"position" in lib().nnz_last_error()
    assert lib().nnz_stream_check(None) == _capi.NNZ_OK
