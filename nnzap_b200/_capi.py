"""ctypes binding of the C ABI in include/nnz_b200.h.

Loads the in-tree ``nnzap_b200/_lib/libnnz_b200.so`` and fails loudly if it
is missing: there is no CPU or library fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import os

# NNZ_LIB_PATH selects another build of the same library (A/B timing of variants)
LIB_PATH = Path(os.environ.get("NNZ_LIB_PATH") or Path(__file__).resolve().parent / "_lib" / "libnnz_b200.so")

NNZ_OK, NNZ_EINVAL, NNZ_ECUDA, NNZ_ENOMEM, NNZ_ETIMEDOUT = 0, -1, -2, -3, -4
NNZ_ENOTFOUND, NNZ_ESTATE, NNZ_EDEVICE, NNZ_ENCCL, NNZ_ERANGE = -5, -6, -7, -8, -9
NNZ_Q1, NNZ_Q4 = 0, 1
NNZ_ROPE_PAIRWISE, NNZ_ROPE_HALF_SPLIT = 0, 1
NNZ_SCALE_F16, NNZ_SCALE_BF16 = 0, 1
NNZ_DT_U8, NNZ_DT_U32, NNZ_DT_F16, NNZ_DT_BF16, NNZ_DT_F32 = 0, 1, 2, 3, 4
NNZ_OUT_F16, NNZ_OUT_F32, NNZ_OUT_F32_ADD = 0, 1, 2

_ERRNAMES = {NNZ_EINVAL: "EINVAL", NNZ_ECUDA: "ECUDA", NNZ_ENOMEM: "ENOMEM",
             NNZ_ETIMEDOUT: "ETIMEDOUT", NNZ_ENOTFOUND: "ENOTFOUND", NNZ_ESTATE: "ESTATE",
             NNZ_EDEVICE: "EDEVICE", NNZ_ENCCL: "ENCCL",
             NNZ_ERANGE: "ERANGE"}


class NnzError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nnz error {_ERRNAMES.get(code, code)}: {msg}")
        self.code = code


class NnzConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "vocab_size", "hidden_size", "intermediate_size", "num_layers", "num_query_heads",
        "num_kv_heads", "head_dim", "max_context_length", "max_prefill_length", "max_batch")] + [
        ("rope_theta", C.c_float), ("eps", C.c_float)] + [(n, C.c_int32) for n in (
            "quant_format", "group_size", "scale_dtype", "bf16_faithful", "rope_style",
            "tie_word_embeddings", "q1_scales_are_mlx", "tp_rank", "tp_size")]


class NnzGenerateOpts(C.Structure):
    _fields_ = [("prompt_ids", C.POINTER(C.c_uint32)), ("n_prompt", C.c_uint32),
                ("eos_ids", C.POINTER(C.c_uint32)), ("n_eos", C.c_uint32),
                ("output_tokens", C.POINTER(C.c_uint32)), ("max_new", C.c_uint32),
                ("per_token_ns", C.POINTER(C.c_uint64)), ("temperature", C.c_float),
                ("top_k", C.c_uint32), ("top_p", C.c_float), ("uniforms", C.POINTER(C.c_float))]


class NnzTokenizerInfo(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "vocab_size", "special_token_count", "eos_token_id", "im_start_token_id",
        "im_end_token_id", "merge_count")]


class NnzTensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("rank", C.c_uint32),
                ("dims", C.c_uint32 * 4), ("data", C.c_void_p), ("nbytes", C.c_size_t)]


class NnzGenerateResult(C.Structure):
    _fields_ = [("tokens_generated", C.c_uint32), ("prefill_ns", C.c_uint64),
                ("decode_ns", C.c_uint64)]


# (name, restype, argtypes) for every exported symbol of include/nnz_b200.h
P, U32, I32, SZ, F32 = C.c_void_p, C.c_uint32, C.c_int, C.c_size_t, C.c_float
DEBUG_SIGNATURES = [("nnz_debug_gemm_profile", I32, [P]), ("nnz_debug_decode1_profile", I32, [P, P, U32]), ("nnz_debug_decode_path", I32, [P]), ("nnz_debug_tp_wait_timeout", I32, [U32, P])]
SIGNATURES = [
    ("nnz_last_error", C.c_char_p, []),
    ("nnz_version", I32, []),
    ("nnz_device_count", I32, []),
    ("nnz_model_create", I32, [I32, C.POINTER(NnzConfig), C.POINTER(P)]),
    ("nnz_model_load_tensor", I32, [P, C.c_char_p, I32, P, SZ]),
    ("nnz_model_finalize", I32, [P]),
    ("nnz_model_free", I32, [P]),
    ("nnz_model_device_bytes", SZ, [P]),
    ("nnz_model_vocab_shard", U32, [P]),
    ("nnz_shard_weights", I32, [I32, I32, P, P, P, U32, U32, U32, U32, U32, P, P, P]),
    ("nnz_tp_unique_id", I32, [P, SZ]),
    ("nnz_sample", I32, [P, U32, U32, U32, F32, U32, F32, P, P, P]),
    ("nnz_tp_init", I32, [P, P, SZ]),
    ("nnz_forward_decode", I32, [P, P, P, U32, P, P]),
    ("nnz_prefill", I32, [P, P, U32, P, P]),
    ("nnz_generate", I32, [P, C.POINTER(NnzGenerateOpts), C.POINTER(NnzGenerateResult)]),
    ("nnz_decode_steps", I32, [P, P, P, U32, U32, P, P]),
    ("nnz_model_write_kv", I32, [P, U32, U32, P, P, U32]),
    ("nnz_model_read_kv", I32, [P, U32, U32, P, P, U32]),
    ("nnz_model_layer_step", I32, [P, U32, P, P, U32]),
    ("nnz_bench_decode_graph", I32, [P, U32, U32, C.POINTER(C.c_double)]),
    ("nnz_packed_bytes", SZ, [I32, U32, U32, U32, U32]),
    ("nnz_pack_weights", I32, [I32, P, P, P, U32, U32, U32, U32, U32, P]),
    ("nnz_unpack_weights", I32, [I32, P, U32, U32, U32, U32, U32, P, P, P]),
    ("nnz_dequant", I32, [I32, I32, P, U32, U32, U32, U32, U32, P, P]),
    ("nnz_qmv", I32, [I32, I32, I32, P, U32, U32, U32, P, U32, U32, P, U32, I32, P]),
    ("nnz_stream_check", I32, [P]),
    ("nnz_qmv_noalloc", I32, [I32, I32, I32, P, U32, U32, U32, P, U32, U32, P, U32, I32, P]),
    ("nnz_qmv_norm", I32, [I32, I32, I32, P, U32, U32, U32, P, P, F32, U32, P, U32, I32, P]),
    ("nnz_lm_head_argmax", I32, [I32, I32, I32, P, U32, U32, U32, P, P, F32, U32, P, P, P]),
    ("nnz_mlp", I32, [I32, I32, I32, P, P, U32, U32, U32, P, U32, P, P]),
    ("nnz_prefill_gemm", I32, [I32, I32, P, P, P, U32, U32, U32, U32, P, P, I32, P]),
    ("nnz_attn_decode", I32, [P, P, P, P, P, U32, P, U32, U32, U32, U32, F32, F32, I32, U32, P, P]),
    ("nnz_tokenizer_from_json", I32, [C.c_char_p, SZ, P]),
    ("nnz_tokenizer_from_file", I32, [C.c_char_p, P]),
    ("nnz_tokenizer_free", I32, [P]),
    ("nnz_tokenizer_get_info", I32, [P, P]),
    ("nnz_tokenizer_encode", I32, [P, C.c_char_p, SZ, P, U32, P]),
    ("nnz_tokenizer_decode", I32, [P, P, U32, P, SZ, P]),
    ("nnz_tokenizer_chat_template", I32, [P, C.c_char_p, SZ, P, U32, P]),
    ("nnz_tokenizer_bpe_merge", I32, [P, P, U32, P]),
    ("nnz_tokenizer_token", I32, [P, U32, P, SZ, P]),
    ("nnz_token_to_bytes", I32, [C.c_char_p, SZ, P, SZ, P]),
    ("nnz_safetensors_open", I32, [C.c_char_p, P]),
    ("nnz_safetensors_from_bytes", I32, [P, SZ, P]),
    ("nnz_safetensors_close", I32, [P]),
    ("nnz_safetensors_count", U32, [P]),
    ("nnz_safetensors_tensor", I32, [P, U32, P]),
    ("nnz_safetensors_find", I32, [P, C.c_char_p, P]),
    ("nnz_pretoken_chunk", U32, [C.c_char_p, SZ]),
]

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it was never built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m nnzap_b200.build` "
                "(no CPU fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES + DEBUG_SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != NNZ_OK:
        raise NnzError(rc, lib().nnz_last_error().decode(errors="replace"))


def ptr(a) -> int | None:
    """Address of a numpy array / torch tensor / int, or None."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data
