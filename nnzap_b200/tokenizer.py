"""Byte-level BPE tokenizer: Python mirror of the reference's Tokenizer
(nnmetal/src/tokenizer.zig) over the library's C ABI (the work runs in
``csrc/tokenizer.cpp``; nothing is tokenized in Python).

    tok = Tokenizer.from_file("tokenizer.json")       # Tokenizer.init
    ids = tok.encode("Hello world")                    # Tokenizer.encode
    text = tok.decode(ids)                             # Tokenizer.decode (bytes)
    prompt = tok.apply_chat_template("Hi")             # Tokenizer.applyChatTemplate

Errors raise TokenizerError; its ``reason`` is the reference's error name
(InvalidJson, MissingField, InvalidVocabEntry, VocabTooLarge,
InvalidMergeEntry, InputTooLong, ChunkTooLong, UnknownByte, UnknownTokenId,
OutputBufferTooSmall, FileNotFound, ...).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import Iterable

import numpy as np

from . import _capi as capi
from ._capi import NnzError

MAX_INPUT_LENGTH = 1024 * 1024   # encode() input limit, bytes (tokenizer.zig:40)
MAX_TOKEN_LENGTH = 512           # pre-tokenized chunk limit, bytes (tokenizer.zig:34)


class TokenizerError(NnzError):
    """A tokenizer failure; ``reason`` names the reference's error."""

    def __init__(self, code: int, msg: str):
        super().__init__(code, msg)
        self.reason = msg.split(":", 1)[0].strip()


def _check(rc: int) -> None:
    if rc != capi.NNZ_OK:
        raise TokenizerError(rc, capi.lib().nnz_last_error().decode(errors="replace"))


def _as_bytes(text: str | bytes) -> bytes:
    return text.encode("utf-8") if isinstance(text, str) else bytes(text)


def next_pretoken_chunk(text: str | bytes) -> int:
    """Byte length of the first pre-tokenizer chunk (nextPretokenChunk,
    tokenizer.zig:936)."""
    b = _as_bytes(text)
    return int(capi.lib().nnz_pretoken_chunk(b, len(b)))


def decode_token_to_bytes(token: str | bytes) -> bytes:
    """Raw bytes of one byte-level token string (decodeTokenToBytes,
    tokenizer.zig:1066)."""
    b = _as_bytes(token)
    buf = C.create_string_buffer(max(1, len(b)))
    n = C.c_size_t()
    _check(capi.lib().nnz_token_to_bytes(b, len(b), buf, len(buf), C.byref(n)))
    return buf.raw[: n.value]


class Tokenizer:
    """A loaded tokenizer.json (immutable; safe to share between threads)."""

    def __init__(self, handle: int):
        self._h = handle
        info = capi.NnzTokenizerInfo()
        _check(capi.lib().nnz_tokenizer_get_info(self._h, C.byref(info)))
        self.vocab_size = info.vocab_size
        self.special_token_count = info.special_token_count
        self.eos_token_id = info.eos_token_id
        self.im_start_token_id = info.im_start_token_id
        self.im_end_token_id = info.im_end_token_id
        self.merge_count = info.merge_count

    @classmethod
    def from_json(cls, data: str | bytes) -> "Tokenizer":
        """Tokenizer.initFromJson (tokenizer.zig:195)."""
        b = _as_bytes(data)
        h = C.c_void_p()
        _check(capi.lib().nnz_tokenizer_from_json(b, len(b), C.byref(h)))
        return cls(h.value)

    @classmethod
    def from_file(cls, path: str | Path) -> "Tokenizer":
        """Tokenizer.init (tokenizer.zig:164)."""
        h = C.c_void_p()
        _check(capi.lib().nnz_tokenizer_from_file(str(path).encode(), C.byref(h)))
        return cls(h.value)

    def close(self) -> None:
        """Tokenizer.deinit."""
        if self._h:
            capi.lib().nnz_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def encode(self, text: str | bytes) -> list[int]:
        """Token ids of ``text`` (UTF-8 for str)."""
        return self.encode_array(text).tolist()

    def encode_array(self, text: str | bytes) -> np.ndarray:
        """Same as encode, as a uint32 array."""
        b = _as_bytes(text)
        cap = len(b) + 1          # at most one token per input byte
        out = np.empty(cap, np.uint32)
        n = C.c_uint32()
        _check(capi.lib().nnz_tokenizer_encode(self._h, b, len(b), out.ctypes.data, cap, C.byref(n)))
        return out[: n.value].copy()

    def decode(self, ids: Iterable[int]) -> bytes:
        """Raw bytes of the ids (the reference decodes to bytes, not str)."""
        arr = np.ascontiguousarray(np.fromiter(ids, dtype=np.uint32))
        cap = 16 * len(arr) + 16  # token strings are short; grow on the rare miss
        while True:
            buf = C.create_string_buffer(cap)
            n = C.c_size_t()
            rc = capi.lib().nnz_tokenizer_decode(self._h, arr.ctypes.data, len(arr), buf, cap, C.byref(n))
            if rc != capi.NNZ_ERANGE:
                _check(rc)
                return buf.raw[: n.value]
            cap *= 8

    def decode_str(self, ids: Iterable[int], errors: str = "replace") -> str:
        return self.decode(ids).decode("utf-8", errors=errors)

    def apply_chat_template(self, prompt: str | bytes) -> list[int]:
        """<|im_start|>user\\n{prompt}<|im_end|>\\n<|im_start|>assistant\\n
        (Tokenizer.applyChatTemplate, tokenizer.zig:330)."""
        b = _as_bytes(prompt)
        cap = len(b) + 32
        out = np.empty(cap, np.uint32)
        n = C.c_uint32()
        _check(capi.lib().nnz_tokenizer_chat_template(self._h, b, len(b), out.ctypes.data, cap, C.byref(n)))
        return out[: n.value].tolist()

    def bpe_merge(self, ids: Iterable[int]) -> list[int]:
        """Greedy lowest-rank merging of a token sequence (Tokenizer.bpeMerge)."""
        arr = np.ascontiguousarray(np.fromiter(ids, dtype=np.uint32))
        n = C.c_uint32()
        _check(capi.lib().nnz_tokenizer_bpe_merge(self._h, arr.ctypes.data, len(arr), C.byref(n)))
        return arr[: n.value].tolist()

    def token(self, token_id: int) -> bytes:
        """id_to_vocab[id]: the token's vocabulary string (byte-level form, UTF-8)."""
        cap = 2048
        buf = C.create_string_buffer(cap)
        n = C.c_size_t()
        rc = capi.lib().nnz_tokenizer_token(self._h, token_id, buf, cap, C.byref(n))
        if rc == capi.NNZ_ERANGE:
            cap = 1 << 20
            buf = C.create_string_buffer(cap)
            rc = capi.lib().nnz_tokenizer_token(self._h, token_id, buf, cap, C.byref(n))
        _check(rc)
        return buf.raw[: n.value]
