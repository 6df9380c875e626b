"""Seeded synthetic weights and inputs in the reference's on-disk formats.

There are no checkpoints on this box, so every benchmark and test runs on
random-init weights of the Qwen3-1.7B (Bonsai) architecture, generated here
in exactly the layout the nnmetal loader consumes:

* Q1: sign bits packed LSB-first over the flat row-major index, one fp16
  scale per ``gs`` flat elements (nnmetal/src/metal.zig:235-335).
* Q4: 8 nibbles per little-endian u32, fp16 (or raw BF16) scale and bias per
  ``gs`` flat elements (nnmetal/src/metal.zig:355-469).

Distributions follow the workload descriptions of the benchmark configs:
Q1 scales ~U(0.01, 0.05), Q4 scales ~U(0.005, 0.02) and biases ~U(-0.1, 0.1),
norm weights 1 + 0.1*N(0,1), tied embedding drawn fp16 ~N(0, 0.02) and then
1-bit quantized with the engine's own convention (bit = w >= 0, scale =
mean|w| per group, nnmetal/src/shaders/compute.metal:1627-1690) or 4-bit
affine quantized (min/max per group, MLX convention).
"""
from __future__ import annotations

import dataclasses
import numpy as np


@dataclasses.dataclass(frozen=True)
class ModelDims:
    vocab: int = 151936
    hidden: int = 2048
    inter: int = 6144
    layers: int = 28
    n_q: int = 16
    n_kv: int = 8
    head_dim: int = 128
    gs: int = 128
    quant: str = "q1"
    rope_theta: float = 1e6
    eps: float = 1e-6
    rope_style: str = "pairwise"
    scale_dtype: str = "f16"
    bf16_faithful: bool = False


# Bonsai-1.7B (transformer.zig:286-298 dims; vocab per the benchmark config).
BONSAI_1_7B_Q1 = ModelDims()
# Qwen3-1.7B MLX 4-bit g64 (transformer.zig:336-350).
BONSAI_1_7B_Q4 = ModelDims(quant="q4", gs=64)


def proj_shapes(d: ModelDims):
    qd, kvd = d.n_q * d.head_dim, d.n_kv * d.head_dim
    return {"q_proj": (qd, d.hidden), "k_proj": (kvd, d.hidden),
            "v_proj": (kvd, d.hidden), "o_proj": (d.hidden, qd),
            "gate_proj": (d.inter, d.hidden), "up_proj": (d.inter, d.hidden),
            "down_proj": (d.hidden, d.inter)}


def _f16_bits(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float16).view(np.uint16)


def _scale_bits(a: np.ndarray, scale_dtype: str) -> np.ndarray:
    if scale_dtype == "f16":
        return _f16_bits(a)
    # raw BF16: truncate f32 (the engine truncates f16 sources, model.zig:1191-1205)
    return (np.asarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def rand_q1(rng, M: int, K: int, gs: int, lo=0.01, hi=0.05) -> dict:
    bits = rng.integers(0, 256, size=M * K // 8, dtype=np.uint8)
    scales = rng.uniform(lo, hi, size=M * K // gs).astype(np.float32)
    return {"weight": bits, "scales": _f16_bits(scales)}


def rand_q4(rng, M: int, K: int, gs: int, scale_dtype="f16",
            s_lo=0.005, s_hi=0.02, b_lo=-0.1, b_hi=0.1) -> dict:
    words = rng.integers(0, 2**32, size=M * K // 8, dtype=np.uint32)
    s = rng.uniform(s_lo, s_hi, size=M * K // gs).astype(np.float32)
    b = rng.uniform(b_lo, b_hi, size=M * K // gs).astype(np.float32)
    return {"weight": words, "scales": _scale_bits(s, scale_dtype),
            "biases": _scale_bits(b, scale_dtype)}


def quantize_q1_sign(w: np.ndarray, gs: int) -> dict:
    """bit = (w >= 0), scale = mean|w| of the flat group (fp16)."""
    flat = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    scale = np.abs(flat.reshape(-1, gs)).mean(axis=1, dtype=np.float32)
    bits = np.packbits(flat >= 0, bitorder="little")
    return {"weight": bits, "scales": _f16_bits(scale)}


def quantize_q4_affine(w: np.ndarray, gs: int, scale_dtype="f16") -> dict:
    """Per-group min/max affine 4-bit: scale = (max-min)/15, bias = min,
    q = round((w - bias)/scale) clamped to 0..15, packed 8 per u32."""
    flat = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, gs)
    mn, mx = flat.min(axis=1), flat.max(axis=1)
    scale = np.maximum((mx - mn) / 15.0, 1e-8).astype(np.float32)
    sb = _scale_bits(scale, scale_dtype)
    bb = _scale_bits(mn, scale_dtype)
    q = np.clip(np.rint((flat - mn[:, None]) / scale[:, None]), 0, 15).astype(np.uint32)
    q = q.reshape(-1, 8)
    words = np.zeros(q.shape[0], dtype=np.uint32)
    for i in range(8):
        words |= q[:, i] << np.uint32(4 * i)
    return {"weight": words, "scales": sb, "biases": bb}


def make_model(d: ModelDims, seed: int = 0, layers: int | None = None) -> dict:
    """Random-init model in reference tensor formats.  ``layers`` overrides
    the layer count (used by small parity cases)."""
    rng = np.random.default_rng(seed)
    nl = d.layers if layers is None else layers
    shapes = proj_shapes(d)
    W = {"layers": []}
    for _ in range(nl):
        L = {}
        for name, (M, K) in shapes.items():
            L[name] = (rand_q1(rng, M, K, d.gs) if d.quant == "q1"
                       else rand_q4(rng, M, K, d.gs, d.scale_dtype))
        L["attn_norm"] = (1.0 + 0.1 * rng.standard_normal(d.hidden)).astype(np.float32)
        L["ffn_norm"] = (1.0 + 0.1 * rng.standard_normal(d.hidden)).astype(np.float32)
        L["q_norm"] = (1.0 + 0.1 * rng.standard_normal(d.head_dim)).astype(np.float32)
        L["k_norm"] = (1.0 + 0.1 * rng.standard_normal(d.head_dim)).astype(np.float32)
        W["layers"].append(L)
    emb = (rng.standard_normal((d.vocab, d.hidden), dtype=np.float32) * 0.02).astype(np.float16)
    W["embed"] = (quantize_q1_sign(emb, d.gs) if d.quant == "q1"
                  else quantize_q4_affine(emb.astype(np.float32), d.gs, d.scale_dtype))
    W["lm_head"] = W["embed"]            # tied (tie_word_embeddings = true)
    W["final_norm"] = (1.0 + 0.1 * rng.standard_normal(d.hidden)).astype(np.float32)
    return W


# Reference tensor names (nnmetal/src/model.zig:571-668, :740-823).
LAYER_COMPONENTS = {
    "q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj",
    "v_proj": "self_attn.v_proj", "o_proj": "self_attn.o_proj",
    "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj",
    "down_proj": "mlp.down_proj", "attn_norm": "input_layernorm",
    "ffn_norm": "post_attention_layernorm", "q_norm": "self_attn.q_norm",
    "k_norm": "self_attn.k_norm",
}


def iter_named_tensors(W: dict):
    """Yield (reference tensor name, numpy array) for a synthetic model."""
    for name, key in (("model.embed_tokens", "embed"),):
        for suf, arr in W[key].items():
            yield f"{name}.{suf}", arr
    yield "model.norm.weight", W["final_norm"]
    for i, L in enumerate(W["layers"]):
        for key, comp in LAYER_COMPONENTS.items():
            t = L[key]
            if isinstance(t, dict):
                for suf, arr in t.items():
                    yield f"model.layers.{i}.{comp}.{suf}", arr
            else:
                yield f"model.layers.{i}.{comp}.weight", t
