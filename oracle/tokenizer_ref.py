"""CPU oracle for the BPE tokenizer (pure Python).

TEST INFRASTRUCTURE ONLY.  This module is the checker that the library's C++
tokenizer (``nnzap_b200/csrc/tokenizer.cpp``) is compared against.  Only
``tests/`` and ``bench.py``'s baseline legs may import it; the product never
does.

It restates nnmetal/src/tokenizer.zig literally, with the reference's own
data structures where they decide behaviour (paths inside the nnzap
reference tree):

* GPT-2 byte <-> unicode table: bytes 33-126, 161-172, 174-255 map to
  themselves, the other 68 to 256.. in byte order (tokenizer.zig:76-108).
* tokenizer.json reading (a repeated member name is invalid JSON, the
  default of the reference's std.json parser): model.vocab (ids must be
  integers in u32 and < 200000), model.merges as "a b" strings or
  ["a", "b"] pairs keyed by the joined string, rank = array index, a
  repeated key keeps the later rank;
  added_tokens go into the vocabulary (id_to_vocab only where unused) and,
  when "special", into the special list (at most 256); eos / im_start /
  im_end resolved by content (tokenizer.zig:375-656); the byte -> base token
  table (tokenizer.zig:659-686).
* encode: longest special token at each position (first listed among equal
  lengths), otherwise the segment up to the next special-token start is
  pre-tokenized and each chunk BPE-merged (tokenizer.zig:247-289, 691-758,
  832-878).
* bpeMerge / findBestPair: repeatedly merge the adjacent pair whose joined
  "a b" key has the lowest rank (leftmost on ties); stop when none is left or
  the joined token string is not in the vocabulary (tokenizer.zig:761-930).
* nextPretokenChunk and the byte classes (tokenizer.zig:936-1060).
* decode and decodeTokenToBytes (tokenizer.zig:293-324, 1066-1140).
* applyChatTemplate (tokenizer.zig:330-370).

Errors raise ``TokError(name)`` with the reference's error name.
"""
from __future__ import annotations

import json

MAX_VOCAB_SIZE = 200_000
MAX_MERGES = 200_000
MAX_TOKEN_LENGTH = 512
MAX_SPECIAL_TOKENS = 256
MAX_INPUT_LENGTH = 1024 * 1024


class TokError(Exception):
    def __init__(self, name: str):
        super().__init__(name)
        self.name = name


def _direct(b: int) -> bool:
    return 33 <= b <= 126 or 161 <= b <= 172 or b >= 174


def _build_byte_map():
    fwd, rev, extra = [0] * 256, {}, 0
    for b in range(256):
        if _direct(b):
            cp = b
        else:
            cp = 256 + extra
            extra += 1
        fwd[b] = cp
        rev[cp] = b
    assert extra == 68
    return fwd, rev


BYTE_FWD, BYTE_REV = _build_byte_map()


# ---- pre-tokenizer (tokenizer.zig:936-1060) ------------------------------
def is_letter(b: int) -> bool:
    return 97 <= b <= 122 or 65 <= b <= 90 or b >= 0x80


def is_digit(b: int) -> bool:
    return 48 <= b <= 57


def is_whitespace(b: int) -> bool:
    return b in (32, 9, 10, 13, 0x0B, 0x0C)


def is_newline(b: int) -> bool:
    return b in (10, 13)


def is_symbol(b: int) -> bool:
    return not is_letter(b) and not is_digit(b) and not is_whitespace(b)


def _contraction(t: bytes, n: int) -> int:
    if n < 2:
        return 0
    c1 = t[1] | 0x20
    if c1 in (ord("s"), ord("t"), ord("m"), ord("d")):
        return 2
    if n < 3:
        return 0
    c2 = t[2] | 0x20
    if (c1, c2) in ((ord("r"), ord("e")), (ord("v"), ord("e")), (ord("l"), ord("l"))):
        return 3
    return 0


def next_pretoken_chunk(t: bytes) -> int:
    n = min(len(t), MAX_INPUT_LENGTH)
    assert n > 0
    if t[0] == ord("'"):
        c = _contraction(t, n)
        if c > 0:
            return c

    def letters(i):
        while i < n and is_letter(t[i]):
            i += 1
        return i

    if is_letter(t[0]):
        return letters(0)
    if n > 1 and not (is_letter(t[0]) or is_digit(t[0])) and not is_newline(t[0]) and is_letter(t[1]):
        return letters(1)
    if is_digit(t[0]):
        e = 1
        while e < n and e < 3 and is_digit(t[e]):
            e += 1
        return e
    if is_symbol(t[0]):
        e = 1
        while e < n and is_symbol(t[e]):
            e += 1
        return e
    if t[0] == 32 and n > 1 and is_symbol(t[1]):
        e = 2
        while e < n and is_symbol(t[e]):
            e += 1
        return e
    if is_newline(t[0]):
        e = 1
        while e < n and is_newline(t[e]):
            e += 1
        return e
    if is_whitespace(t[0]):
        e = 1
        while e < n and is_whitespace(t[e]) and not is_newline(t[e]):
            e += 1
        return e
    return 1


# ---- decode helpers (tokenizer.zig:1066-1140) ----------------------------
def utf8_sequence_length(first: int) -> int:
    if first < 0x80:
        return 1
    if first < 0xC0:
        return 1
    if first < 0xE0:
        return 2
    if first < 0xF0:
        return 3
    return 4


def decode_utf8_codepoint(b: bytes) -> int:
    if len(b) == 1:
        return b[0]
    if len(b) == 2:
        return (b[0] & 0x1F) << 6 | (b[1] & 0x3F)
    if len(b) == 3:
        return (b[0] & 0x0F) << 12 | (b[1] & 0x3F) << 6 | (b[2] & 0x3F)
    return (b[0] & 0x07) << 18 | (b[1] & 0x3F) << 12 | (b[2] & 0x3F) << 6 | (b[3] & 0x3F)


def decode_token_to_bytes(s: bytes) -> bytes:
    out = bytearray()
    i = 0
    while i < len(s):
        L = utf8_sequence_length(s[i])
        if i + L > len(s):
            out.append(s[i])
            i += 1
            continue
        cp = decode_utf8_codepoint(s[i:i + L])
        if cp in BYTE_REV:
            out.append(BYTE_REV[cp])
        else:
            out += s[i:i + L]
        i += L
    return bytes(out)


class Tokenizer:
    """tokenizer.zig's Tokenizer, state for state (byte strings throughout)."""

    def __init__(self, json_bytes: bytes | str):
        if isinstance(json_bytes, str):
            json_bytes = json_bytes.encode()
        def no_duplicates(pairs):
            # the reference's std.json rejects a repeated member name
            d = {}
            for k, v in pairs:
                if k in d:
                    raise TokError("InvalidJson")
                d[k] = v
            return d

        try:
            root = json.loads(json_bytes.decode("utf-8"), object_pairs_hook=no_duplicates)
        except (UnicodeDecodeError, json.JSONDecodeError):
            raise TokError("InvalidJson") from None
        if not isinstance(root, dict):
            raise TokError("InvalidJson")
        self.vocab_to_id: dict[bytes, int] = {}
        self.id_to_vocab: dict[int, bytes] = {}
        self.merge_ranks: dict[bytes, int] = {}
        self.special: list[tuple[bytes, int]] = []
        self.vocab_size = 0
        self.eos_token_id = self.im_start_token_id = self.im_end_token_id = 0
        model = root.get("model")
        if model is None:
            raise TokError("MissingField")
        if not isinstance(model, dict):
            raise TokError("InvalidJson")
        vocab = model.get("vocab")
        if vocab is None:
            raise TokError("MissingField")
        if not isinstance(vocab, dict):
            raise TokError("InvalidJson")
        for key, v in vocab.items():
            if not isinstance(v, int) or isinstance(v, bool) or v < 0 or v > 0xFFFFFFFF:
                raise TokError("InvalidVocabEntry")
            if v >= MAX_VOCAB_SIZE:
                raise TokError("VocabTooLarge")
            k = key.encode()
            self.vocab_to_id[k] = v
            self.id_to_vocab[v] = k
            self.vocab_size = max(self.vocab_size, v + 1)
        if "merges" in model:
            merges = model["merges"]
            if not isinstance(merges, list):
                raise TokError("InvalidJson")
            if len(merges) > MAX_MERGES:
                raise TokError("TooManyMerges")
            for rank, item in enumerate(merges):
                if isinstance(item, str):
                    self.merge_ranks[item.encode()] = rank
                elif isinstance(item, list):
                    if len(item) != 2 or not all(isinstance(x, str) for x in item):
                        raise TokError("InvalidMergeEntry")
                    self.merge_ranks[(item[0] + " " + item[1]).encode()] = rank
                else:
                    raise TokError("InvalidMergeEntry")
        added = root.get("added_tokens")
        if added is not None:
            if not isinstance(added, list):
                raise TokError("InvalidJson")
            for obj in added:
                if not isinstance(obj, dict):
                    continue
                tid = obj.get("id")
                if not isinstance(tid, int) or isinstance(tid, bool) or tid < 0 or tid > 0xFFFFFFFF:
                    continue
                content = obj.get("content")
                if not isinstance(content, str):
                    continue
                c = content.encode()
                special = obj.get("special") is True
                if tid < MAX_VOCAB_SIZE:
                    if not self.id_to_vocab.get(tid):
                        self.id_to_vocab[tid] = c
                    self.vocab_to_id[c] = tid
                    self.vocab_size = max(self.vocab_size, tid + 1)
                if special and len(self.special) < MAX_SPECIAL_TOKENS:
                    self.special.append((c, tid))
        if self.vocab_size == 0:
            raise TokError("InvalidJson")
        for c, tid in self.special:
            if c == b"<|endoftext|>":
                self.eos_token_id = tid
            elif c == b"<|im_start|>":
                self.im_start_token_id = tid
            elif c == b"<|im_end|>":
                self.im_end_token_id = tid
        self.byte_to_token_id = [self.vocab_to_id.get(chr(BYTE_FWD[b]).encode()) for b in range(256)]

    @property
    def special_token_count(self) -> int:
        return len(self.special)

    # ---- encoding
    def _special_at(self, text: bytes, pos: int):
        best, best_len = None, 0
        for c, tid in self.special:
            if len(c) <= best_len or len(c) > len(text) - pos:
                continue
            if text[pos:pos + len(c)] == c:
                best, best_len = (c, tid), len(c)
        return best

    def _find_best_pair(self, toks: list[int]):
        best_rank, best_i = None, None
        for i in range(len(toks) - 1):
            a, b = self.id_to_vocab.get(toks[i], b""), self.id_to_vocab.get(toks[i + 1], b"")
            key = a + b" " + b
            if len(key) > MAX_TOKEN_LENGTH * 2 + 1:
                continue
            r = self.merge_ranks.get(key)
            if r is not None and (best_rank is None or r < best_rank):
                best_rank, best_i = r, i
        return best_i

    def bpe_merge(self, toks: list[int]) -> list[int]:
        toks = list(toks)
        while len(toks) > 1:
            i = self._find_best_pair(toks)
            if i is None:
                break
            a, b = self.id_to_vocab.get(toks[i], b""), self.id_to_vocab.get(toks[i + 1], b"")
            if len(a) + len(b) > MAX_TOKEN_LENGTH * 2:
                break
            merged = self.vocab_to_id.get(a + b)
            if merged is None:
                break
            toks[i:i + 2] = [merged]
        return toks

    def _encode_chunk(self, chunk: bytes) -> list[int]:
        toks = []
        for byte in chunk:
            if len(toks) >= MAX_TOKEN_LENGTH:
                raise TokError("ChunkTooLong")
            tid = self.byte_to_token_id[byte]
            if tid is None:
                raise TokError("UnknownByte")
            toks.append(tid)
        return self.bpe_merge(toks)

    def encode(self, text: bytes | str) -> list[int]:
        if isinstance(text, str):
            text = text.encode()
        if not text:
            return []
        if len(text) > MAX_INPUT_LENGTH:
            raise TokError("InputTooLong")
        out, cur = [], 0
        while cur < len(text):
            st = self._special_at(text, cur)
            if st is not None:
                out.append(st[1])
                cur += len(st[0])
                continue
            end = cur + 1
            while end < len(text) and self._special_at(text, end) is None:
                end += 1
            seg, pos = text[cur:end], 0
            while pos < len(seg):
                cl = next_pretoken_chunk(seg[pos:])
                out += self._encode_chunk(seg[pos:pos + cl])
                pos += cl
            cur = end
        return out

    def decode(self, ids) -> bytes:
        out = bytearray()
        for tid in ids:
            if tid >= self.vocab_size or not self.id_to_vocab.get(tid):
                raise TokError("UnknownTokenId")
            out += decode_token_to_bytes(self.id_to_vocab[tid])
        return bytes(out)

    def apply_chat_template(self, prompt: bytes | str) -> list[int]:
        if isinstance(prompt, str):
            prompt = prompt.encode()
        return ([self.im_start_token_id] + self.encode(b"user\n") + self.encode(prompt)
                + [self.im_end_token_id] + self.encode(b"\n") + [self.im_start_token_id]
                + self.encode(b"assistant\n"))
