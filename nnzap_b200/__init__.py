"""nnzap_b200: B200-native (sm_100a) quantized Qwen3 / Bonsai decode hot path.

The compute lives in the CUDA library ``nnzap_b200/_lib/libnnz_b200.so``
(C ABI: ``include/nnz_b200.h``); this package is its host-side mirror of the
nnmetal engine interface (``engine``), the library binding (``_capi``), the
in-tree build (``build``), seeded synthetic weights (``synth``), the
safetensors loader (``safetensors``) and the BPE tokenizer (``tokenizer``).
"""
from .engine import (Bonsai1_7B, Bonsai1_7B_Q4, GenerateOpts, GenerateResult, Model,
                     SamplingParams, TinyBlock, TransformerConfig, config_from_dims, generate,
                     shard_weights, tp_unique_id)
from .tokenizer import Tokenizer, TokenizerError

__all__ = ["Bonsai1_7B", "Bonsai1_7B_Q4", "GenerateOpts", "GenerateResult", "Model",
           "SamplingParams", "TinyBlock", "TransformerConfig", "config_from_dims", "generate",
           "shard_weights", "tp_unique_id", "Tokenizer", "TokenizerError"]
