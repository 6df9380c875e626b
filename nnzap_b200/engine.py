"""Host-side mirror of the nnmetal engine interface for the decode hot path.

The reference's Zig API (nnmetal/src/transformer.zig, model.zig):

* ``TransformerConfig(TransformerDesc)`` with the ``Bonsai1_7B`` /
  ``Bonsai1_7B_Q4`` presets (transformer.zig:62-350)
* ``Model(Config).init / loadWeights / forwardDecodeArgs`` (model.zig:123-330)
* ``forwardDecode`` (transformer.zig:2566), ``generate`` with
  ``GenerateOpts`` / ``GenerateResult`` (transformer.zig:3663-3690, :3942)

is mirrored here in Python over the C ABI of ``include/nnz_b200.h``.  All
compute runs in the CUDA library; this module only marshals arguments.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
from typing import Iterable, Sequence

import numpy as np

from . import _capi as capi
from ._capi import check, lib, ptr


@dataclasses.dataclass(frozen=True)
class TransformerConfig:
    """TransformerDesc (transformer.zig:62-81) plus the build's runtime knobs."""
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_query_heads: int
    num_kv_heads: int
    head_dim: int
    max_context_length: int
    max_prefill_length: int
    rope_theta: float
    tie_word_embeddings: bool = True
    quant_format: str = "q1_0"          # "q1_0" | "q4_mlx"
    group_size: int = 128
    eps: float = 1e-6
    max_batch: int = 1
    scale_dtype: str = "f16"            # q4: "f16" (spec) | "bf16" (engine)
    bf16_faithful: bool = False         # q4: truncate outputs to BF16
    rope_style: str = "pairwise"        # "pairwise" (engine) | "half_split" (MLX/HF)
    q1_scales_are_mlx: bool = False     # halve Q1 scales at load (model.zig:944-959)
    tp_rank: int = 0                    # tensor-parallel rank / size (batched decode)
    tp_size: int = 1

    @property
    def query_dim(self) -> int:
        return self.num_query_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def heads_per_kv_group(self) -> int:
        return self.num_query_heads // self.num_kv_heads

    def replace(self, **kw) -> "TransformerConfig":
        return dataclasses.replace(self, **kw)

    def to_c(self) -> capi.NnzConfig:
        c = capi.NnzConfig()
        for f in ("vocab_size", "hidden_size", "intermediate_size", "num_layers",
                  "num_query_heads", "num_kv_heads", "head_dim", "max_context_length",
                  "max_prefill_length", "max_batch"):
            setattr(c, f, int(getattr(self, f)))
        c.rope_theta = float(self.rope_theta)
        c.eps = float(self.eps)
        c.quant_format = {"q1_0": capi.NNZ_Q1, "q4_mlx": capi.NNZ_Q4}[self.quant_format]
        c.group_size = int(self.group_size)
        c.scale_dtype = {"f16": capi.NNZ_SCALE_F16, "bf16": capi.NNZ_SCALE_BF16}[self.scale_dtype]
        c.bf16_faithful = int(self.bf16_faithful)
        c.rope_style = {"pairwise": capi.NNZ_ROPE_PAIRWISE,
                        "half_split": capi.NNZ_ROPE_HALF_SPLIT}[self.rope_style]
        c.tie_word_embeddings = int(self.tie_word_embeddings)
        c.q1_scales_are_mlx = int(self.q1_scales_are_mlx)
        c.tp_rank, c.tp_size = int(self.tp_rank), int(self.tp_size)
        return c


# Presets (transformer.zig:286-298, :336-350).  The Q1 preset uses the
# benchmark vocabulary (151936); the reference's trimmed Bonsai vocabulary
# (151669) is one .replace(vocab_size=151669) away.
Bonsai1_7B = TransformerConfig(
    vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_layers=28,
    num_query_heads=16, num_kv_heads=8, head_dim=128, max_context_length=32768,
    max_prefill_length=512, rope_theta=1_000_000.0, tie_word_embeddings=True,
    quant_format="q1_0", group_size=128)
Bonsai1_7B_Q4 = Bonsai1_7B.replace(quant_format="q4_mlx", group_size=64)
# TinyBlock of the reference unit tests (transformer_test.zig:53-65).
TinyBlock = TransformerConfig(
    vocab_size=32, hidden_size=128, intermediate_size=256, num_layers=1, num_query_heads=2,
    num_kv_heads=2, head_dim=64, max_context_length=8, max_prefill_length=4,
    rope_theta=10000.0, tie_word_embeddings=True)


@dataclasses.dataclass
class SamplingParams:
    """transformer.zig:3655-3660; only greedy decoding runs on this path."""
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int = 42


@dataclasses.dataclass
class GenerateOpts:
    """transformer.zig:3672-3690 (scratch/indices are not needed on GPU)."""
    prompt_ids: Sequence[int]
    max_new: int
    eos_ids: Sequence[int] = ()
    params: SamplingParams = dataclasses.field(default_factory=SamplingParams)
    per_token_ns: bool = True


@dataclasses.dataclass
class GenerateResult:
    """transformer.zig:3663-3667 plus the tokens and per-token times."""
    tokens_generated: int
    prefill_ns: int
    decode_ns: int
    tokens: list
    per_token_ns: list


def _dtype_code(a: np.ndarray) -> int:
    return {np.dtype(np.uint8): capi.NNZ_DT_U8, np.dtype(np.uint32): capi.NNZ_DT_U32,
            np.dtype(np.float16): capi.NNZ_DT_F16, np.dtype(np.float32): capi.NNZ_DT_F32,
            np.dtype(np.uint16): capi.NNZ_DT_F16}[a.dtype]


class Model:
    """Model(Config) of model.zig: owns every device buffer of one model."""

    def __init__(self, config: TransformerConfig, device: int = 0, tp_unique_id: bytes | None = None):
        """With config.tp_size > 1 this process holds rank config.tp_rank's
        shard; every rank passes the same ``tp_unique_id`` (from
        :func:`tp_unique_id` on one rank, shared by the caller) and the
        constructor joins the NCCL group."""
        self.config = config
        self.device = device
        self._h = C.c_void_p()
        check(lib().nnz_model_create(device, C.byref(config.to_c()), C.byref(self._h)))
        self._finalized = False
        if config.tp_size > 1:
            if tp_unique_id is None:
                raise ValueError("tensor-parallel model needs tp_unique_id")
            uid = (C.c_uint8 * len(tp_unique_id)).from_buffer_copy(tp_unique_id)
            check(lib().nnz_tp_init(self._h, uid, len(tp_unique_id)))

    @property
    def vocab_shard(self) -> int:
        """LM-head rows this rank computes (vocab_size without TP)."""
        return int(lib().nnz_model_vocab_shard(self._h))

    # -- model.zig:196 loadWeights ---------------------------------------
    def load_tensor(self, name: str, arr: np.ndarray, dtype: int | None = None) -> None:
        arr = np.ascontiguousarray(arr)
        code = _dtype_code(arr) if dtype is None else dtype
        if name.endswith((".scales", ".biases")) and arr.dtype == np.uint16 and dtype is None:
            code = (capi.NNZ_DT_BF16 if self.config.scale_dtype == "bf16"
                    and self.config.quant_format == "q4_mlx" else capi.NNZ_DT_F16)
        check(lib().nnz_model_load_tensor(self._h, name.encode(), code, ptr(arr), arr.nbytes))

    def load_weights(self, tensors: Iterable) -> None:
        for name, arr in tensors:
            self.load_tensor(name, arr)
        self.finalize()

    def load_safetensors(self, paths) -> None:
        """loadWeights from safetensors shard files (model.zig:196-242)."""
        from .safetensors import load_safetensors
        load_safetensors(self, [paths] if isinstance(paths, (str, bytes)) or hasattr(paths, "open") else paths)

    def finalize(self) -> None:
        check(lib().nnz_model_finalize(self._h))
        self._finalized = True

    def device_bytes(self) -> int:
        return int(lib().nnz_model_device_bytes(self._h))

    # -- transformer.zig:2566 forwardDecode + :3694 argmax ------------------
    def forward_decode(self, tokens, positions, want_logits: bool = False):
        t = np.ascontiguousarray(np.atleast_1d(tokens), dtype=np.uint32)
        p = np.ascontiguousarray(np.atleast_1d(positions), dtype=np.uint32)
        b = len(t)
        am = np.zeros(b, dtype=np.uint32)
        lg = np.empty((b, self.vocab_shard), dtype=np.float32) if want_logits else None
        check(lib().nnz_forward_decode(self._h, ptr(t), ptr(p), b, ptr(lg), ptr(am)))
        return am, lg

    def prefill(self, tokens, want_logits: bool = False):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        nxt = np.zeros(1, dtype=np.uint32)
        lg = np.empty(self.vocab_shard, dtype=np.float32) if want_logits else None
        check(lib().nnz_prefill(self._h, ptr(t), len(t), ptr(nxt), ptr(lg)))
        return int(nxt[0]), lg

    def decode_steps(self, tokens, positions, steps: int, timings: bool = False):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint32)
        out = np.zeros((steps, len(t)), dtype=np.uint32)
        ns = np.zeros(steps, dtype=np.uint64) if timings else None
        check(lib().nnz_decode_steps(self._h, ptr(t), ptr(p), len(t), steps, ptr(out), ptr(ns)))
        return (out, ns) if timings else out

    def write_kv(self, layer: int, slot: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, dtype=np.float16)
        v = np.ascontiguousarray(v, dtype=np.float16)
        check(lib().nnz_model_write_kv(self._h, layer, slot, ptr(k), ptr(v), k.shape[1]))

    def read_kv(self, layer: int, slot: int, length: int):
        c = self.config
        k = np.zeros((c.num_kv_heads, length, c.head_dim), dtype=np.float16)
        v = np.zeros_like(k)
        check(lib().nnz_model_read_kv(self._h, layer, slot, ptr(k), ptr(v), length))
        return k, v

    def layer_step(self, layer: int, residual: np.ndarray, positions) -> np.ndarray:
        r = np.ascontiguousarray(residual, dtype=np.float32).copy()
        p = np.ascontiguousarray(np.atleast_1d(positions), dtype=np.uint32)
        check(lib().nnz_model_layer_step(self._h, layer, ptr(r), ptr(p), r.shape[0]))
        return r

    def bench_decode_graph(self, batch: int, iters: int) -> float:
        us = C.c_double()
        check(lib().nnz_bench_decode_graph(self._h, batch, iters, C.byref(us)))
        return us.value

    def free(self) -> None:
        if self._h:
            lib().nnz_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def tp_unique_id() -> bytes:
    """A new NCCL group id (create on one rank, hand to all)."""
    buf = (C.c_uint8 * 256)()
    n = lib().nnz_tp_unique_id(buf, 256)
    if n < 0:
        check(n)
    return bytes(buf[:n])


def shard_weights(fmt: str, axis: int, weight: np.ndarray, scales: np.ndarray, biases, M: int, K: int,
                  gs: int, lo: int, hi: int):
    """Host-side tensor-parallel slice of a flat reference-layout matrix:
    rows [lo, hi) (axis 0) or columns [lo, hi) (axis 1)."""
    code = {"q1_0": capi.NNZ_Q1, "q4_mlx": capi.NNZ_Q4}[fmt]
    Mo, Ko = (hi - lo, K) if axis == 0 else (M, hi - lo)
    wbytes = Mo * Ko // 8 if code == capi.NNZ_Q1 else Mo * Ko // 2
    w = np.zeros(wbytes, np.uint8)
    s = np.zeros(Mo * Ko // gs, np.uint16)
    b = np.zeros_like(s) if biases is not None else None
    weight = np.ascontiguousarray(weight)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    bi = None if biases is None else np.ascontiguousarray(biases, dtype=np.uint16)
    check(lib().nnz_shard_weights(code, axis, ptr(weight), ptr(scales), ptr(bi), M, K, gs, lo, hi,
                                  ptr(w), ptr(s), ptr(b)))
    return w, s, b


def generate(model: Model, opts: GenerateOpts) -> GenerateResult:
    """generate (transformer.zig:3942-4027): device prefill, then one decode
    launch per token; greedy, or sampled on the device when
    opts.params.temperature > 0; stops at the first EOS like the reference."""
    prompt = np.ascontiguousarray(opts.prompt_ids, dtype=np.uint32)
    eos = np.ascontiguousarray(opts.eos_ids, dtype=np.uint32) if len(opts.eos_ids) else None
    out = np.zeros(opts.max_new, dtype=np.uint32)
    ns = np.zeros(opts.max_new, dtype=np.uint64)
    o = capi.NnzGenerateOpts()
    o.prompt_ids = prompt.ctypes.data_as(C.POINTER(C.c_uint32))
    o.n_prompt = len(prompt)
    o.eos_ids = eos.ctypes.data_as(C.POINTER(C.c_uint32)) if eos is not None else None
    o.n_eos = 0 if eos is None else len(eos)
    o.output_tokens = out.ctypes.data_as(C.POINTER(C.c_uint32))
    o.max_new = opts.max_new
    o.per_token_ns = ns.ctypes.data_as(C.POINTER(C.c_uint64)) if opts.per_token_ns else None
    sp = opts.params
    uni = None
    if sp.temperature > 0.0:
        # the host draws the per-token uniforms (seeded; the reference uses
        # Zig's DefaultPrng(seed), which this generator does not reproduce)
        uni = np.random.default_rng(sp.seed).random(opts.max_new, dtype=np.float32)
        o.temperature, o.top_k, o.top_p = float(sp.temperature), int(sp.top_k), float(sp.top_p)
        o.uniforms = uni.ctypes.data_as(C.POINTER(C.c_float))
    else:
        o.temperature, o.top_k, o.top_p = 0.0, 0, 1.0
    r = capi.NnzGenerateResult()
    check(lib().nnz_generate(model._h, C.byref(o), C.byref(r)))
    n = r.tokens_generated
    return GenerateResult(n, int(r.prefill_ns), int(r.decode_ns), out[:n].tolist(),
                          ns[:n].tolist())


def config_from_dims(d, max_context_length: int = 4096, max_batch: int = 1) -> TransformerConfig:
    """TransformerConfig for a ``synth.ModelDims``."""
    return TransformerConfig(
        vocab_size=d.vocab, hidden_size=d.hidden, intermediate_size=d.inter,
        num_layers=d.layers, num_query_heads=d.n_q, num_kv_heads=d.n_kv, head_dim=d.head_dim,
        max_context_length=max_context_length, max_prefill_length=512,
        rope_theta=d.rope_theta, eps=d.eps, tie_word_embeddings=True,
        quant_format="q1_0" if d.quant == "q1" else "q4_mlx", group_size=d.gs,
        max_batch=max_batch, scale_dtype=d.scale_dtype, bf16_faithful=d.bf16_faithful,
        rope_style=d.rope_style)
