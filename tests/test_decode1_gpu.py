"""The single-row Q1 decode kernel (csrc/decode1.cu) against the oracle.

Batch-1 decode of a Q1 / group-128 / head_dim-128 model runs this kernel by
default; these cases pin what the generic model tests do not reach:
  * that the kernel is really the one running (no silent fallback);
  * attention over long caches: splits of more than two 32-position K/V
    blocks (the in-loop refill), empty splits, position 0;
  * activations with heavy-tailed groups (norm weights with 20-60x outlier
    channels, like real Qwen3 checkpoints): the per-group fixed-point split
    must still meet the 2e-2 logits bar;
  * a multi-token launch (generate) against token-at-a-time decode.
"""
import numpy as np
import pytest

from gpu_helpers import R
from nnzap_b200 import GenerateOpts, Model, _capi, config_from_dims, generate, synth

pytestmark = pytest.mark.gpu

D = synth.ModelDims(vocab=1000, hidden=256, inter=768, layers=2, n_q=4, n_kv=2, head_dim=128, gs=128,
                    quant="q1")


def _cfg(d):
    return R.Cfg(vocab=d.vocab, hidden=d.hidden, inter=d.inter, layers=d.layers, n_q=d.n_q, n_kv=d.n_kv,
                 head_dim=d.head_dim, gs=d.gs, quant=d.quant, rope_theta=d.rope_theta, eps=d.eps,
                 rope_style=d.rope_style)


def _model(d, W, max_ctx):
    m = Model(config_from_dims(d, max_context_length=max_ctx, max_batch=1))
    m.load_weights(synth.iter_named_tensors(W))
    assert _capi.lib().nnz_debug_decode_path(m._h) == 1, "single-row decode kernel not in use"
    return m


@pytest.mark.parametrize("pos", [0, 100, 4500, 7000])
def test_long_cache_attention(cuda, built_lib, pos):
    """Random fp16 K/V history of `pos` positions in every layer; one decode
    step at `pos` vs the oracle's decode over the same cache.  At 7000 each of
    the 74 splits of a kv head holds ~95 positions (three K/V blocks)."""
    W = synth.make_model(D, seed=3)
    m = _model(D, W, 8192)
    cfg = _cfg(D)
    rng = np.random.default_rng(pos)
    kv = []
    for layer in range(D.layers):
        k = rng.standard_normal((D.n_kv, pos, D.head_dim)).astype(np.float16)
        v = rng.standard_normal((D.n_kv, pos, D.head_dim)).astype(np.float16)
        if pos:
            m.write_kv(layer, 0, k, v)
        kv.append((k, v))
    tok = int(rng.integers(0, D.vocab))
    am, lg = m.forward_decode([tok], [pos], want_logits=True)
    want = R.decode_one(cfg, W, kv, tok, pos)
    err = float(np.abs(lg[0] - want).max())
    assert err <= 2e-2, err
    assert int(am[0]) == int(np.argmax(lg[0]))
    m.free()


def test_outlier_channels(cuda, built_lib):
    """Norm weights with a few 20-60x channels make one element of a group
    dominate the others by up to ~3 orders of magnitude after RMSNorm."""
    W = synth.make_model(D, seed=5)
    rng = np.random.default_rng(9)
    for Lw in W["layers"]:
        for key in ("attn_norm", "ffn_norm"):
            idx = rng.choice(D.hidden, 6, replace=False)
            Lw[key] = Lw[key].copy()
            Lw[key][idx] *= rng.uniform(20, 60, 6).astype(np.float32)
    W["final_norm"] = W["final_norm"].copy()
    W["final_norm"][rng.choice(D.hidden, 4, replace=False)] *= 30
    m = _model(D, W, 64)
    cfg = _cfg(D)
    seq = rng.integers(0, D.vocab, 10)
    want = R.forward_tokens(cfg, W, seq)
    for p, tok in enumerate(seq):
        am, lg = m.forward_decode([int(tok)], [p], want_logits=True)
        err = float(np.abs(lg[0] - want[p]).max())
        assert err <= 2e-2, (p, err, float(np.abs(want[p]).max()))
    m.free()


def test_multi_token_launch_matches_steps(cuda, built_lib):
    """generate() decodes all tokens in one launch (the kernel loops over
    tokens on the device); token-at-a-time forward_decode of the same prompt
    gives the same greedy ids, and both pass the oracle's teacher-forced check."""
    W = synth.make_model(D, seed=7)
    m = _model(D, W, 128)
    cfg = _cfg(D)
    prompt = list(np.random.default_rng(8).integers(0, D.vocab, 16))
    res = generate(m, GenerateOpts(prompt_ids=prompt, max_new=20))
    assert res.tokens_generated == 20 and len(res.per_token_ns) == 20
    assert all(t > 0 for t in res.per_token_ns)
    exact, worst, _ = R.greedy_check(cfg, W, prompt, res.tokens)
    assert worst <= 2e-2, worst
    # the same tokens one launch per step (prompt through the same kernel)
    tok = prompt[0]
    steps = []
    for p in range(len(prompt) + len(res.tokens) - 1):
        am, _ = m.forward_decode([tok], [p])
        tok = prompt[p + 1] if p + 1 < len(prompt) else int(am[0])
        if p + 1 >= len(prompt):
            steps.append(tok)
    assert steps == res.tokens[: len(steps)]
    m.free()
