"""End-to-end GPU parity: engine decode / prefill / generate vs the oracle.

Bar (north star): logits within 2e-2 max-abs of the oracle; greedy tokens
identical -- checked teacher-forced: every generated token must be the
oracle's argmax at that position unless the oracle's own top-2 gap there is
below 2e-2 (a genuine near tie, where either choice is correct).
"""
import numpy as np
import pytest

from gpu_helpers import R
from nnzap_b200 import Model, GenerateOpts, config_from_dims, generate, synth

pytestmark = pytest.mark.gpu

SMALL_Q1 = synth.ModelDims(vocab=1000, hidden=256, inter=768, layers=2, n_q=4, n_kv=2,
                           head_dim=128, gs=128, quant="q1")
SMALL_Q4 = synth.ModelDims(vocab=1000, hidden=256, inter=768, layers=2, n_q=4, n_kv=2,
                           head_dim=128, gs=64, quant="q4")
SMALL_Q4_ENGINE = synth.ModelDims(vocab=1000, hidden=256, inter=768, layers=2, n_q=4, n_kv=2,
                                  head_dim=128, gs=64, quant="q4", scale_dtype="bf16",
                                  bf16_faithful=True)
SMALL_HALF = synth.ModelDims(vocab=512, hidden=256, inter=512, layers=1, n_q=8, n_kv=2,
                             head_dim=64, gs=64, quant="q1", rope_style="half_split")


def oracle_cfg(d):
    return R.Cfg(vocab=d.vocab, hidden=d.hidden, inter=d.inter, layers=d.layers, n_q=d.n_q,
                 n_kv=d.n_kv, head_dim=d.head_dim, gs=d.gs, quant=d.quant,
                 rope_theta=d.rope_theta, eps=d.eps, rope_style=d.rope_style,
                 scale_dtype=d.scale_dtype, bf16_faithful=d.bf16_faithful)


def build(d, seed=0, max_ctx=256, max_batch=4, path="persistent"):
    """path: "persistent" (the default: the single-row kernel for Q1 batch-1
    steps, else the persistent multi-row kernel), "mega" (the multi-row
    persistent kernel for every batch <= 8) or "graph" (the captured
    multi-kernel CUDA graph)."""
    import os
    W = synth.make_model(d, seed=seed)
    old = os.environ.get("NNZ_DECODE_PATH")
    os.environ["NNZ_DECODE_PATH"] = path
    try:
        m = Model(config_from_dims(d, max_context_length=max_ctx, max_batch=max_batch))
        m.load_weights(synth.iter_named_tensors(W))
    finally:
        if old is None:
            os.environ.pop("NNZ_DECODE_PATH")
        else:
            os.environ["NNZ_DECODE_PATH"] = old
    return m, W


def greedy_ok(cfg, W, prompt, toks, tol=2e-2):
    exact, worst, lg = R.greedy_check(cfg, W, prompt, toks)
    for i, t in enumerate(toks):
        row = lg[i]
        if int(np.argmax(row)) != t:
            top2 = np.sort(row)[-2:]
            assert top2[1] - top2[0] < tol and row.max() - row[t] < tol, (i, t, int(np.argmax(row)))
    return exact


@pytest.mark.parametrize("path", ["persistent", "mega", "graph"])
@pytest.mark.parametrize("d", [SMALL_Q1, SMALL_Q4, SMALL_Q4_ENGINE, SMALL_HALF],
                         ids=["q1", "q4", "q4_engine_bf16", "q1_half_split_hd64"])
def test_forward_decode_logits(cuda, built_lib, d, path):
    m, W = build(d, path=path)
    cfg = oracle_cfg(d)
    rng = np.random.default_rng(1)
    seq = rng.integers(0, d.vocab, 12)
    want = R.forward_tokens(cfg, W, seq)
    for p, tok in enumerate(seq):
        am, lg = m.forward_decode([tok], [p], want_logits=True)
        # the engine's BF16 mode truncates every projection output to BF16 (8
        # significant bits) in both the kernels and the oracle; where the two
        # f32 values straddle a truncation point they end one BF16 ulp apart,
        # 2^-7 relative, so that mode adds one ulp of the element to the bar
        tol = 2e-2 + (2.0 ** -7 * np.abs(want[p]) if d.bf16_faithful else 0.0)
        err = np.abs(lg[0] - want[p]) - tol
        assert err.max() <= 0, (p, float(np.abs(lg[0] - want[p]).max()))
        assert lg[0][am[0]] == lg[0].max()
    m.free()


@pytest.mark.parametrize("d", [SMALL_Q1, SMALL_Q4], ids=["q1", "q4"])
def test_prefill_matches_decode_and_oracle(cuda, built_lib, d):
    m, W = build(d)
    cfg = oracle_cfg(d)
    prompt = np.random.default_rng(2).integers(0, d.vocab, 100)   # two prefill chunks
    nxt, lg = m.prefill(prompt, want_logits=True)
    want = R.forward_tokens(cfg, W, prompt, logits_rows=[len(prompt) - 1])[0]
    assert np.abs(lg - want).max() <= 2e-2
    assert nxt == int(np.argmax(lg))
    # KV written by prefill == KV written by token-at-a-time decode
    k_pre, v_pre = m.read_kv(0, 0, len(prompt))
    for p, tok in enumerate(prompt):
        m.forward_decode([tok], [p])
    k_dec, v_dec = m.read_kv(0, 0, len(prompt))
    # same fp16 values up to one rounding step: prefill and the persistent decode
    # kernel sum the projection's split-K partials in different orders
    np.testing.assert_allclose(v_pre.astype(np.float32), v_dec.astype(np.float32), atol=2e-3, rtol=2e-3)
    np.testing.assert_allclose(k_pre.astype(np.float32), k_dec.astype(np.float32), atol=2e-3, rtol=2e-3)
    m.free()


@pytest.mark.parametrize("path", ["persistent", "mega", "graph"])
@pytest.mark.parametrize("d", [SMALL_Q1, SMALL_Q4], ids=["q1", "q4"])
def test_generate_greedy(cuda, built_lib, d, path):
    m, W = build(d, path=path)
    cfg = oracle_cfg(d)
    prompt = list(np.random.default_rng(3).integers(0, d.vocab, 20))
    res = generate(m, GenerateOpts(prompt_ids=prompt, max_new=24))
    assert res.tokens_generated == 24 and len(res.per_token_ns) == 24
    assert res.prefill_ns > 0 and res.decode_ns > 0
    exact = greedy_ok(cfg, W, prompt, res.tokens)
    assert exact >= 22
    # EOS stops generation like the reference (transformer.zig:3992)
    res2 = generate(m, GenerateOpts(prompt_ids=prompt, max_new=24, eos_ids=[res.tokens[5]]))
    assert res2.tokens == res.tokens[:res.tokens.index(res.tokens[5])]
    m.free()


@pytest.mark.parametrize("path", ["persistent", "graph"])
def test_batched_decode_rows_independent(cuda, built_lib, path):
    d = SMALL_Q1
    m, W = build(d, max_batch=6, path=path)
    rng = np.random.default_rng(4)
    toks = rng.integers(0, d.vocab, 6)
    pos = np.array([0, 0, 0, 0, 0, 0])
    am, lg = m.forward_decode(toks, pos, want_logits=True)
    for r in range(6):
        am1, lg1 = m.forward_decode([toks[r]], [0], want_logits=True)
        # a single row runs the single-row kernel (exact 22-bit activation
        # split) and a batch of 6 the multi-row one (15-bit split): the same
        # row agrees to the multi-row kernel's rounding, not bit for bit
        tol = 1e-4 if path != "persistent" else 2e-3
        np.testing.assert_allclose(lg1[0], lg[r], atol=tol)
    out = m.decode_steps(toks, pos + 1, steps=5)
    assert out.shape == (5, 6)
    m.free()


def test_layer_step_config2_q4(cuda, built_lib):
    """Benchmark configuration 2: one 4-bit g64 decoder layer, KV 2048 filled N(0,1)."""
    d = synth.ModelDims(vocab=256, layers=1, quant="q4", gs=64)
    m, W = build(d, max_ctx=2049, max_batch=1)
    cfg = oracle_cfg(d)
    rng = np.random.default_rng(5)
    L = 2048
    kc = rng.standard_normal((d.n_kv, L, d.head_dim)).astype(np.float16)
    vc = rng.standard_normal((d.n_kv, L, d.head_dim)).astype(np.float16)
    m.write_kv(0, 0, kc, vc)
    h = rng.standard_normal((1, d.hidden)).astype(np.float32)
    got = m.layer_step(0, h, [L])
    # oracle: the same layer at position L over the given cache
    Lw = W["layers"][0]
    xn = R._to_f16(cfg, R.rmsnorm(h, Lw["attn_norm"]))
    hd, nq, nkv = d.head_dim, d.n_q, d.n_kv
    q = R._to_f16(cfg, R.qmv(cfg, Lw["q_proj"], nq * hd, d.hidden, xn)).reshape(1, nq, hd)
    k = R._to_f16(cfg, R.qmv(cfg, Lw["k_proj"], nkv * hd, d.hidden, xn)).reshape(1, nkv, hd)
    v = R._to_f16(cfg, R.qmv(cfg, Lw["v_proj"], nkv * hd, d.hidden, xn)).reshape(nkv, hd)
    P = np.array([L])
    q = R.rope(R.rmsnorm(q, Lw["q_norm"]), P, d.rope_theta)[0]
    k = R.rope(R.rmsnorm(k, Lw["k_norm"]), P, d.rope_theta)[0].astype(np.float16)
    K_ = np.concatenate([kc, k[:, None]], axis=1)
    V_ = np.concatenate([vc, v.astype(np.float16)[:, None]], axis=1)
    att = R.attention_decode(q, K_, V_, nkv).astype(np.float16).astype(np.float32).reshape(1, -1)
    res = h + R.qmv(cfg, Lw["o_proj"], d.hidden, nq * hd, att)
    xn = R._to_f16(cfg, R.rmsnorm(res, Lw["ffn_norm"]))
    g = R.qmv(cfg, Lw["gate_proj"], d.inter, d.hidden, xn)
    u = R.qmv(cfg, Lw["up_proj"], d.inter, d.hidden, xn)
    want = res + R.qmv(cfg, Lw["down_proj"], d.hidden, d.inter, R._to_f16(cfg, R.silu_mul(g, u)))
    err = np.abs(got - want).max()
    assert err <= 2e-2 * max(1.0, np.abs(want).max() / 10), err
    m.free()


@pytest.mark.parametrize("path", ["persistent", "graph"])
def test_full_bonsai_q1_generate(cuda, built_lib, path):
    """Benchmark configuration 3 shape (28 layers, vocab 151936), short run."""
    d = synth.BONSAI_1_7B_Q1
    m, W = build(d, max_ctx=1024, max_batch=1, path=path)
    cfg = oracle_cfg(d)
    prompt = list(np.random.default_rng(0).integers(0, d.vocab, 64))
    res = generate(m, GenerateOpts(prompt_ids=prompt, max_new=8))
    assert res.tokens_generated == 8
    exact = greedy_ok(cfg, W, prompt, res.tokens)
    assert exact >= 7
    m.free()


@pytest.mark.parametrize("d", [SMALL_Q1, SMALL_Q4], ids=["q1", "q4"])
@pytest.mark.parametrize("rows", [20, 64, 100])
def test_batched_decode_gemm_rows(cuda, built_lib, d, rows):
    """Decode batches of >= 16 rows run the projections as tcgen05 GEMMs
    (weights as the TMEM operand; 64 token columns up to 64 rows, 128 above):
    every sampled row's logits match the oracle's token-at-a-time decode."""
    m, W = build(d, max_ctx=64, max_batch=rows, path="graph")
    cfg = oracle_cfg(d)
    rng = np.random.default_rng(11)
    toks = rng.integers(0, d.vocab, rows)
    am, lg = m.forward_decode(toks, np.zeros(rows, dtype=np.uint32), want_logits=True)
    for r in list(range(0, rows, 7)) + [rows - 1]:
        want = R.forward_tokens(cfg, W, [int(toks[r])])[-1]
        np.testing.assert_allclose(lg[r], want, atol=2e-2, rtol=0)
    # a second step at position 1 attends over the cache the first wrote
    nxt = am.astype(np.uint32)
    am2, lg2 = m.forward_decode(nxt, np.ones(rows, dtype=np.uint32), want_logits=True)
    for r in list(range(0, rows, 7)) + [rows - 1]:
        want = R.forward_tokens(cfg, W, [int(toks[r]), int(nxt[r])])[-1]
        np.testing.assert_allclose(lg2[r], want, atol=2e-2, rtol=0)
    m.free()


def test_generate_sampled_matches_oracle(cuda, built_lib):
    """Sampled generate(): each token is the oracle's sampleToken of the
    teacher-forced logits with the same uniform draw (a draw within rounding
    of a CDF boundary may take the neighbour)."""
    from nnzap_b200 import SamplingParams
    d = SMALL_Q1
    m, W = build(d, max_ctx=64, max_batch=1)
    prompt = [7, 300, 41, 999, 5]
    sp = SamplingParams(temperature=0.8, top_k=40, top_p=0.9, seed=11)
    res = generate(m, GenerateOpts(prompt_ids=prompt, max_new=10, params=sp))
    assert res.tokens_generated == 10
    u = np.random.default_rng(sp.seed).random(10, dtype=np.float32)
    lg = R.forward_tokens(oracle_cfg(d), W, prompt + res.tokens[:-1])[len(prompt) - 1:]
    for i, t in enumerate(res.tokens):
        want = R.sample_token(lg[i], sp.temperature, sp.top_k, sp.top_p, float(u[i]))
        if t != want:
            cum = R.sample_cdf(lg[i], sp.temperature, sp.top_k, sp.top_p)
            # logits differ from the oracle by < 2e-2, so the CDF may shift a little
            assert abs(float(cum[min(t, want)]) - float(u[i])) < 2e-2, (i, t, want)
    m.free()


@pytest.mark.parametrize("n_q,n_kv,style,plen", [(4, 4, "pairwise", 300), (4, 2, "pairwise", 700),
                                                 (8, 2, "half_split", 300), (8, 2, "pairwise", 129)],
                         ids=["G1", "G2_two_chunks", "G4_half_split", "G4_tile_edge"])
def test_prefill_attention_tiles(cuda, built_lib, n_q, n_kv, style, plen):
    """The tcgen05 prefill attention over several 128-key tiles, every GQA
    group size, both RoPE pairings, a prompt that spans two prefill chunks
    (the second chunk's queries start past the first's keys) and one that
    ends one key into a tile: last-row logits against the oracle, then the
    greedy continuation decoded from the cache the prefill wrote."""
    d = synth.ModelDims(vocab=800, hidden=256, inter=512, layers=2, n_q=n_q, n_kv=n_kv, head_dim=128,
                        gs=128, quant="q1", rope_style=style)
    m, W = build(d, max_ctx=1024)
    cfg = oracle_cfg(d)
    prompt = np.random.default_rng(plen).integers(0, d.vocab, plen)
    nxt, lg = m.prefill(prompt, want_logits=True)
    want = R.forward_tokens(cfg, W, prompt, logits_rows=[plen - 1])[0]
    assert np.abs(lg - want).max() <= 2e-2, float(np.abs(lg - want).max())
    res = generate(m, GenerateOpts(prompt_ids=list(prompt), max_new=6))
    assert greedy_ok(cfg, W, list(prompt), res.tokens) >= 0
    m.free()


def test_prefill_attention_mma_fallback(cuda, built_lib, tmp_path):
    """NNZ_PREFILL_ATTN=mma (read once per process) still selects the
    mma.sync prefill attention: run the tile test's G2 two-chunk case in a
    child process with it set."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, NNZ_PREFILL_ATTN="mma")
    here = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        os.path.join(here, "test_model_gpu.py"), "-k", "test_prefill_attention_tiles and G2_two_chunks"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
