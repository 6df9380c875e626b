"""CPU oracle for the quantized Qwen3 (Bonsai) decode/prefill hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product (``nnzap_b200``) never imports it and has no CPU fallback.

What it restates (all citations are paths inside the nnzap reference tree):

* Q1 weight format, bit ``c`` of row ``r`` is bit ``(r*K+c) % 8`` of byte
  ``(r*K+c) // 8``; bit set -> +scale, clear -> -scale; one fp16 scale per
  ``gs`` consecutive elements of the flat row-major index
  (nnmetal/src/transformer_test.zig:286-321, nnmetal/src/metal.zig:235-335).
* MLX -> engine Q1 load conversion: scale / 2, bias dropped
  (nnmetal/src/model.zig:911-960, pinned by model_test.zig:251-295).
* 1-bit quantizer: bit = (w >= 0), scale = mean|w| per group
  (nnmetal/src/shaders/compute.metal:1627-1690).
* Q4 MLX affine format: 8 nibbles per little-endian u32, nibble ``c % 8`` of
  word ``(r*K+c) // 8``; W = scale*q + bias per ``gs`` group
  (nnmetal/src/metal.zig:355-469, nnmetal/src/model.zig:969-1026).
  ``scale_dtype='bf16'`` + ``bf16_faithful`` restate the engine's BF16 path
  (raw BF16 scale/bias, outputs truncated to BF16:
  nnmetal/src/shaders/q4mv_bf16_specialized.metal:44-57,165-172,288,495,806).
* RMSNorm, SiLU*mul, pairwise RoPE, softmax, GQA attention, embedding
  dequant, QMV, block composition order
  (nnmetal/src/transformer_test.zig:72-332, :364-715).
* Decode precision points: fp16 normed activations, fp16 q/k/v/attn/SiLU
  outputs, f32 residual, K cached as fp16 after norm+RoPE, Q kept in f32
  after norm+RoPE, f32 softmax, f32 logits
  (nnmetal/src/shaders/qmv_specialized.metal:1096-1279,
  nnmetal/src/shaders/transformer.metal:1467-1695, :561-608).
* Greedy argmax, first maximum wins (nnmetal/src/transformer.zig:3694-3707);
  sampling with temperature / top-k / top-p (:3709-3880) given the draw.

Parity status: UNPINNED against the reference's own outputs.  The engine
needs Zig + Apple Metal and the MLX scripts need Apple's MLX, none of which
exist here, and the reference ships no numeric golden vectors for this path.
The oracle is pinned only by the reference's known-answer unit tests that are
pure arithmetic (scale/2 table, f32->f16 table, quantizer convention), which
``tests/test_oracle.py`` replays.

The full-sequence forward (``forward_tokens``) processes every position of a
teacher-forced token sequence in one causal pass.  Each position's arithmetic
is independent except through attention over cached K/V, so this reproduces
the token-at-a-time decode of nnmetal/src/transformer.zig:4032-4123 exactly
at the precision points above.
"""
from __future__ import annotations

import dataclasses
import numpy as np

F16 = np.float16
F32 = np.float32


# --------------------------------------------------------------------------
# scalar helpers
# --------------------------------------------------------------------------

def bf16_bits_to_f32(raw: np.ndarray) -> np.ndarray:
    """Raw BF16 u16 bit pattern -> f32 (q4mv_bf16_specialized.metal:44-49)."""
    return (raw.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Zero the low 16 bits of f32 (q4mv_bf16_specialized.metal:51-57)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def f16_bits_to_f32(raw: np.ndarray) -> np.ndarray:
    return raw.astype(np.uint16).view(np.float16).astype(np.float32)


def scale_to_f32(raw_u16: np.ndarray, scale_dtype: str) -> np.ndarray:
    if scale_dtype == "f16":
        return f16_bits_to_f32(raw_u16)
    if scale_dtype == "bf16":
        return bf16_bits_to_f32(raw_u16)
    raise ValueError(scale_dtype)


# --------------------------------------------------------------------------
# weight formats
# --------------------------------------------------------------------------

def q1_unpack_signs(bits: np.ndarray, M: int, K: int) -> np.ndarray:
    """Row-major LSB-first bits -> int8 {+1,-1} [M, K]
    (transformer_test.zig:286-321: byte = flat/8, bit = flat%8)."""
    b = np.unpackbits(np.ascontiguousarray(bits).view(np.uint8)[: (M * K + 7) // 8],
                      bitorder="little")[: M * K]
    return (b.astype(np.int8) * 2 - 1).reshape(M, K)


def q1_dequant(bits: np.ndarray, scales_u16: np.ndarray, M: int, K: int,
               gs: int) -> np.ndarray:
    """Exact f32 dequant of a Q1 matrix: +-scale (scale of the flat group)."""
    sg = q1_unpack_signs(bits, M, K).astype(np.float32).reshape(-1, gs)
    s = f16_bits_to_f32(scales_u16)[: sg.shape[0]]
    return (sg * s[:, None]).reshape(M, K)


def q4_unpack(words: np.ndarray, M: int, K: int) -> np.ndarray:
    """u32 words, nibble i at bits 4i..4i+3 (metal.zig:355-469) -> u8 [M, K]."""
    w = np.ascontiguousarray(words).view(np.uint32)[: M * K // 8]
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, :]
    q = (w[:, None] >> shifts) & np.uint32(0xF)
    return q.astype(np.uint8).reshape(M, K)


def q4_dequant(words: np.ndarray, scales_u16: np.ndarray, biases_u16: np.ndarray,
               M: int, K: int, gs: int, scale_dtype: str = "f16") -> np.ndarray:
    """Exact f32 dequant W = scale*q + bias (both products exact in f32)."""
    q = q4_unpack(words, M, K).astype(np.float32).reshape(-1, gs)
    s = scale_to_f32(scales_u16, scale_dtype)[: q.shape[0]]
    b = scale_to_f32(biases_u16, scale_dtype)[: q.shape[0]]
    return (q * s[:, None] + b[:, None]).astype(np.float32).reshape(M, K)


def mlx_q1_scales_to_engine(mlx_scales_f16: np.ndarray) -> np.ndarray:
    """MLX affine Q1 scale -> symmetric engine scale: scale / 2
    (model.zig:944-959; model_test.zig:251-295)."""
    s = np.asarray(mlx_scales_f16, dtype=np.float16).astype(np.float32) / 2.0
    return s.astype(np.float16)


def quantize_q1(w: np.ndarray, gs: int):
    """f32 [M, K] -> (bits u8, scales f16-bits u16) with bit = (w >= 0) and
    scale = mean|w| over each flat group (compute.metal:1627-1690)."""
    flat = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    assert flat.size % gs == 0
    scale = np.abs(flat.reshape(-1, gs)).mean(axis=1, dtype=np.float32)
    bits = np.packbits((flat >= 0).astype(np.uint8), bitorder="little")
    return bits, scale.astype(np.float16).view(np.uint16)


# --------------------------------------------------------------------------
# kernels
# --------------------------------------------------------------------------

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """x * rsqrt(mean(x^2) + eps) * w over the last axis (transformer_test.zig:72-104)."""
    x = x.astype(np.float32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (x * (1.0 / np.sqrt(ms + np.float32(eps))) * w.astype(np.float32)).astype(np.float32)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    return (g / (1.0 + np.exp(-g)) * u.astype(np.float32)).astype(np.float32)


def rope_angles(positions: np.ndarray, head_dim: int, theta: float):
    """theta_p = theta^(-2p/hd) (transformer_test.zig:128-156)."""
    p = np.arange(head_dim // 2, dtype=np.float64)
    inv = np.power(np.float64(theta), -2.0 * p / head_dim)
    ang = positions.astype(np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope(x: np.ndarray, positions: np.ndarray, theta: float, style: str = "pairwise"):
    """x [T, H, hd].  'pairwise' rotates (2p, 2p+1) like the engine
    (transformer.metal:1535-1549); 'half_split' rotates (p, p+hd/2) like MLX/HF
    (reference/mlx_q4_layer0.py:114-136)."""
    T, H, hd = x.shape
    c, s = rope_angles(positions, hd, theta)
    c = c[:, None, :]
    s = s[:, None, :]
    out = np.empty_like(x, dtype=np.float32)
    if style == "pairwise":
        a, b = x[..., 0::2], x[..., 1::2]
        out[..., 0::2] = a * c - b * s
        out[..., 1::2] = a * s + b * c
    elif style == "half_split":
        a, b = x[..., : hd // 2], x[..., hd // 2:]
        out[..., : hd // 2] = a * c - b * s
        out[..., hd // 2:] = a * s + b * c
    else:
        raise ValueError(style)
    return out


def attention_decode(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, n_kv: int) -> np.ndarray:
    """One query position.  q [Hq, hd] f32, kc/vc [Hkv, L, hd] (fp16 values).
    Scores f32 scaled by 1/sqrt(hd), softmax f32, output f32
    (transformer_test.zig:158-255)."""
    Hq, hd = q.shape
    grp = Hq // n_kv
    out = np.empty((Hq, hd), dtype=np.float32)
    for h in range(Hq):
        k = kc[h // grp].astype(np.float32)
        v = vc[h // grp].astype(np.float32)
        s = (k @ q[h]) * np.float32(1.0 / np.sqrt(hd))
        s = np.exp(s - s.max())
        s /= s.sum()
        out[h] = s @ v
    return out


def argmax_first(logits: np.ndarray) -> int:
    """First maximum wins (transformer.zig:3694-3707)."""
    return int(np.argmax(logits))


def softmax_f32(x: np.ndarray) -> np.ndarray:
    """softmaxInPlace (transformer.zig:3724-3744), f32."""
    x = x.astype(np.float32)
    e = np.exp(x - np.max(x)).astype(np.float32)
    return (e * np.float32(1.0 / e.sum(dtype=np.float32))).astype(np.float32)


def sample_cdf(logits: np.ndarray, temperature: float, top_k: int, top_p: float) -> np.ndarray:
    """The running sum (vocabulary order) of the probabilities sampleToken
    draws from (transformer.zig:3833-3869): temperature scaling
    (applyTemperature :3709), top-k (applyTopK :3748: keep values >= the
    k-th largest), top-p (applyTopP :3779: walk the probabilities in
    descending order, keep tokens until the cumulative mass reaches p),
    softmax."""
    x = logits.astype(np.float32) * np.float32(1.0 / np.float32(temperature))
    if 0 < top_k < len(x):
        thr = np.sort(x)[::-1][top_k - 1]
        x = np.where(x < thr, np.float32(-np.inf), x)
    if top_p < 1.0:
        pr = softmax_f32(x)
        order = np.argsort(-pr, kind="stable")
        cum = np.cumsum(pr[order], dtype=np.float32)
        keep = np.searchsorted(cum, np.float32(top_p)) + 1   # through the first crossing
        x = x.copy()
        x[order[keep:]] = np.float32(-np.inf)
    return np.cumsum(softmax_f32(x), dtype=np.float32)


def sample_token(logits: np.ndarray, temperature: float, top_k: int, top_p: float, r: float) -> int:
    """sampleToken with the uniform draw r given; greedy at temperature 0.
    sampleFromDistribution (:3873): first index whose running sum exceeds r,
    else the last index."""
    if temperature == 0.0:
        return argmax_first(logits)
    cum = sample_cdf(logits, temperature, top_k, top_p)
    idx = np.nonzero(cum > np.float32(r))[0]
    return int(idx[0]) if len(idx) else len(cum) - 1


# --------------------------------------------------------------------------
# model container (reference-format tensors)
# --------------------------------------------------------------------------

@dataclasses.dataclass
class Cfg:
    vocab: int
    hidden: int
    inter: int
    layers: int
    n_q: int
    n_kv: int
    head_dim: int
    gs: int
    quant: str = "q1"            # "q1" | "q4"
    rope_theta: float = 1e6
    eps: float = 1e-6
    rope_style: str = "pairwise"
    scale_dtype: str = "f16"     # q4 only: "f16" (spec) | "bf16" (engine)
    bf16_faithful: bool = False  # q4 only: truncate outputs to bf16


PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def proj_shape(cfg: Cfg, name: str):
    qd, kvd = cfg.n_q * cfg.head_dim, cfg.n_kv * cfg.head_dim
    return {"q_proj": (qd, cfg.hidden), "k_proj": (kvd, cfg.hidden),
            "v_proj": (kvd, cfg.hidden), "o_proj": (cfg.hidden, qd),
            "gate_proj": (cfg.inter, cfg.hidden), "up_proj": (cfg.inter, cfg.hidden),
            "down_proj": (cfg.hidden, cfg.inter)}[name]


def dequant_tensor(cfg: Cfg, t: dict, M: int, K: int) -> np.ndarray:
    if cfg.quant == "q1":
        return q1_dequant(t["weight"], t["scales"], M, K, cfg.gs)
    return q4_dequant(t["weight"], t["scales"], t["biases"], M, K, cfg.gs, cfg.scale_dtype)


def _round_out(cfg: Cfg, y: np.ndarray) -> np.ndarray:
    """Kernel output rounding: engine BF16 mode truncates first."""
    return bf16_round(y) if (cfg.quant == "q4" and cfg.bf16_faithful) else y


def _to_f16(cfg: Cfg, y: np.ndarray) -> np.ndarray:
    return _round_out(cfg, y).astype(F16).astype(F32)


_DQ_CACHE = None


def set_dequant_cache(on: bool) -> None:
    """Keep every dequantized matrix (f32) after its first use, so repeated
    decode steps stop re-expanding the packed weights (the timed CPU baseline
    and the parity checks of long runs; ~7 GB for the 1.7B model)."""
    global _DQ_CACHE
    _DQ_CACHE = {} if on else None


def qmv(cfg: Cfg, t: dict, M: int, K: int, x: np.ndarray, row_chunk: int = 8192) -> np.ndarray:
    """y[T, M] = x[T, K] @ W^T with f32 accumulation; W dequantized exactly."""
    x = x.astype(np.float32)
    if _DQ_CACHE is not None:
        key = (id(t["weight"]), M, K)
        hit = _DQ_CACHE.get(key)
        if hit is None:
            hit = (t["weight"], dequant_tensor(cfg, t, M, K))   # the array ref keeps the id valid
            _DQ_CACHE[key] = hit
        return x @ hit[1].T
    if M <= row_chunk:
        return x @ dequant_tensor(cfg, t, M, K).T
    out = np.empty((x.shape[0], M), dtype=np.float32)
    for r0 in range(0, M, row_chunk):
        r1 = min(M, r0 + row_chunk)
        sub = _slice_rows(cfg, t, r0, r1, K)
        out[:, r0:r1] = x @ dequant_tensor(cfg, sub, r1 - r0, K).T
    return out


def _slice_rows(cfg: Cfg, t: dict, r0: int, r1: int, K: int) -> dict:
    g0, g1 = r0 * K // cfg.gs, r1 * K // cfg.gs
    if cfg.quant == "q1":
        return {"weight": np.ascontiguousarray(t["weight"]).view(np.uint8)[r0 * K // 8: r1 * K // 8],
                "scales": t["scales"][g0:g1]}
    return {"weight": np.ascontiguousarray(t["weight"]).view(np.uint32)[r0 * K // 8: r1 * K // 8],
            "scales": t["scales"][g0:g1], "biases": t["biases"][g0:g1]}


def embed(cfg: Cfg, emb: dict, tokens: np.ndarray) -> np.ndarray:
    """Gather + dequant rows -> f32 residual (transformer.metal:453-549)."""
    H = cfg.hidden
    rows = []
    for tok in tokens:
        sub = _slice_rows(cfg, emb, int(tok), int(tok) + 1, H)
        rows.append(dequant_tensor(cfg, sub, 1, H)[0])
    r = np.stack(rows).astype(np.float32)
    return _round_out(cfg, r)


def forward_tokens(cfg: Cfg, W: dict, tokens, logits_rows=None, return_kv=False):
    """Teacher-forced causal pass over ``tokens`` (positions 0..T-1).

    Returns f32 logits [T, vocab] (or only rows ``logits_rows``), following
    the block order of transformer_test.zig:364-715 and the decode precision
    points listed in the module docstring.
    """
    tokens = np.asarray(tokens, dtype=np.int64)
    T = len(tokens)
    hd, nq, nkv = cfg.head_dim, cfg.n_q, cfg.n_kv
    pos = np.arange(T)
    res = embed(cfg, W["embed"], tokens)                       # f32 [T, H]
    kv = []
    for li in range(cfg.layers):
        L = W["layers"][li]
        xn = _to_f16(cfg, rmsnorm(res, L["attn_norm"], cfg.eps))
        q = _to_f16(cfg, qmv(cfg, L["q_proj"], nq * hd, cfg.hidden, xn)).reshape(T, nq, hd)
        k = _to_f16(cfg, qmv(cfg, L["k_proj"], nkv * hd, cfg.hidden, xn)).reshape(T, nkv, hd)
        v = _to_f16(cfg, qmv(cfg, L["v_proj"], nkv * hd, cfg.hidden, xn)).reshape(T, nkv, hd)
        q = rope(rmsnorm(q, L["q_norm"], cfg.eps), pos, cfg.rope_theta, cfg.rope_style)
        k = rope(rmsnorm(k, L["k_norm"], cfg.eps), pos, cfg.rope_theta, cfg.rope_style)
        k = k.astype(F16).astype(F32)                         # K cache is fp16
        kt = k.transpose(1, 0, 2)
        vt = v.transpose(1, 0, 2)
        if return_kv:
            kv.append((kt.astype(F16), vt.astype(F16)))
        att = np.empty((T, nq, hd), dtype=np.float32)
        grp = nq // nkv
        inv = np.float32(1.0 / np.sqrt(hd))
        mask = np.triu(np.full((T, T), -np.inf, dtype=np.float32), 1)
        for h in range(nq):
            s = (q[:, h, :] @ kt[h // grp].T) * inv + mask
            s = np.exp(s - s.max(axis=1, keepdims=True))
            s /= s.sum(axis=1, keepdims=True)
            att[:, h, :] = s @ vt[h // grp]
        att = att.astype(F16).astype(F32).reshape(T, nq * hd)
        res = res + _round_out(cfg, qmv(cfg, L["o_proj"], cfg.hidden, nq * hd, att))
        xn = _to_f16(cfg, rmsnorm(res, L["ffn_norm"], cfg.eps))
        g = qmv(cfg, L["gate_proj"], cfg.inter, cfg.hidden, xn)    # f32, fused
        u = qmv(cfg, L["up_proj"], cfg.inter, cfg.hidden, xn)      # into SiLU*mul
        h_ = _to_f16(cfg, silu_mul(g, u))
        res = res + _round_out(cfg, qmv(cfg, L["down_proj"], cfg.hidden, cfg.inter, h_))
    rows = np.arange(T) if logits_rows is None else np.asarray(logits_rows)
    xn = _to_f16(cfg, rmsnorm(res[rows], W["final_norm"], cfg.eps))
    logits = _round_out(cfg, qmv(cfg, W["lm_head"], cfg.vocab, cfg.hidden, xn))
    if return_kv:
        return logits, kv
    return logits


def greedy_check(cfg: Cfg, W: dict, prompt, generated, tol: float = 2e-2):
    """Teacher-forced greedy check.  For each generated token, the oracle's
    logits at the preceding position must put that token within ``tol`` of
    the maximum (identical argmax unless the oracle itself has a near tie).
    Returns (n_exact_argmax_matches, worst_gap)."""
    seq = list(prompt) + list(generated)
    rows = list(range(len(prompt) - 1, len(seq) - 1))
    lg = forward_tokens(cfg, W, seq[:-1] if generated else seq, logits_rows=rows)
    exact, worst = 0, 0.0
    for i, tok in enumerate(generated):
        row = lg[i]
        gap = float(row.max() - row[tok])
        worst = max(worst, gap)
        exact += int(argmax_first(row) == tok)
    return exact, worst, lg


def mlp_block(cfg: Cfg, gate: dict, up: dict, down: dict, x: np.ndarray) -> np.ndarray:
    """Benchmark configuration 1 block: down(SiLU(gate x) * up x) with the engine's
    fp16 rounding of the SiLU*mul output (qmv_specialized.metal:1268-1276)."""
    g = qmv(cfg, gate, cfg.inter, cfg.hidden, x)
    u = qmv(cfg, up, cfg.inter, cfg.hidden, x)
    h = _to_f16(cfg, silu_mul(g, u))
    return qmv(cfg, down, cfg.hidden, cfg.inter, h)


def decode_one(cfg: Cfg, W: dict, kv: list, token: int, pos: int) -> np.ndarray:
    """One token-at-a-time decode step (transformer.zig:4072-4123) with an
    explicit KV cache: ``kv[layer] = (K [n_kv, L, hd] f16, V [...])`` grown in
    place.  Returns f32 logits [vocab].  Used as the timed CPU baseline."""
    hd, nq, nkv = cfg.head_dim, cfg.n_q, cfg.n_kv
    P = np.array([pos])
    res = embed(cfg, W["embed"], np.array([token]))
    for li in range(cfg.layers):
        L = W["layers"][li]
        xn = _to_f16(cfg, rmsnorm(res, L["attn_norm"], cfg.eps))
        q = _to_f16(cfg, qmv(cfg, L["q_proj"], nq * hd, cfg.hidden, xn)).reshape(1, nq, hd)
        k = _to_f16(cfg, qmv(cfg, L["k_proj"], nkv * hd, cfg.hidden, xn)).reshape(1, nkv, hd)
        v = _to_f16(cfg, qmv(cfg, L["v_proj"], nkv * hd, cfg.hidden, xn)).reshape(nkv, hd)
        q = rope(rmsnorm(q, L["q_norm"], cfg.eps), P, cfg.rope_theta, cfg.rope_style)[0]
        k = rope(rmsnorm(k, L["k_norm"], cfg.eps), P, cfg.rope_theta, cfg.rope_style)[0]
        if len(kv) <= li:
            kv.append((np.zeros((nkv, 0, hd), F16), np.zeros((nkv, 0, hd), F16)))
        K_, V_ = kv[li]
        K_ = np.concatenate([K_[:, :pos], k.astype(F16)[:, None]], axis=1)
        V_ = np.concatenate([V_[:, :pos], v.astype(F16)[:, None]], axis=1)
        kv[li] = (K_, V_)
        att = attention_decode(q, K_, V_, nkv).astype(F16).astype(F32).reshape(1, -1)
        res = res + _round_out(cfg, qmv(cfg, L["o_proj"], cfg.hidden, nq * hd, att))
        xn = _to_f16(cfg, rmsnorm(res, L["ffn_norm"], cfg.eps))
        g = qmv(cfg, L["gate_proj"], cfg.inter, cfg.hidden, xn)
        u = qmv(cfg, L["up_proj"], cfg.inter, cfg.hidden, xn)
        res = res + _round_out(cfg, qmv(cfg, L["down_proj"], cfg.hidden, cfg.inter,
                                        _to_f16(cfg, silu_mul(g, u))))
    xn = _to_f16(cfg, rmsnorm(res, W["final_norm"], cfg.eps))
    return _round_out(cfg, qmv(cfg, W["lm_head"], cfg.vocab, cfg.hidden, xn))[0]
