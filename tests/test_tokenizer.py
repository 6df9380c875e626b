"""CPU tests of the BPE tokenizer (host C++ in the library, no GPU).

* The reference's own unit tests (nnmetal/src/tokenizer_test.zig), replayed
  against both the library and the oracle (oracle/tokenizer_ref.py).
* Golden encodings of a synthetic byte-level BPE in the real tokenizer.json
  schema (tests/golden/make_tokenizer_golden.py).
* Differential tests library == oracle on seeded random text (ASCII, UTF-8,
  invalid UTF-8, special tokens inside), decode(encode(x)) == x, both merge
  formats, and the reference's error behaviour.
"""
import ctypes as C
import json
import random
import threading
from pathlib import Path

import numpy as np
import pytest

from oracle import tokenizer_ref as R

GOLDEN = Path(__file__).resolve().parent / "golden"
SYNTH = GOLDEN / "tokenizer_synth.json"


def tok_json(vocab, merges, added=()):
    return json.dumps({"model": {"type": "BPE", "vocab": vocab, "merges": list(merges)},
                       "added_tokens": list(added)})


class Lib:
    """The library through the Python mirror, with the oracle's method names."""

    def __init__(self, js):
        from nnzap_b200.tokenizer import Tokenizer
        self.t = Tokenizer.from_json(js)
        self.vocab_size = self.t.vocab_size
        self.special_token_count = self.t.special_token_count
        self.eos_token_id = self.t.eos_token_id
        self.im_start_token_id = self.t.im_start_token_id
        self.im_end_token_id = self.t.im_end_token_id

    def encode(self, text):
        return self.t.encode(text)

    def decode(self, ids):
        return self.t.decode(ids)

    def bpe_merge(self, ids):
        return self.t.bpe_merge(ids)

    def apply_chat_template(self, p):
        return self.t.apply_chat_template(p)


def make(impl, js):
    return Lib(js) if impl == "lib" else R.Tokenizer(js)


IMPLS = ["lib", "oracle"]


def err_name(impl, fn):
    from nnzap_b200.tokenizer import TokenizerError
    try:
        fn()
    except TokenizerError as e:
        return e.reason
    except R.TokError as e:
        return e.name
    return None


# ---- tokenizer_test.zig, case by case ------------------------------------

def test_byte_map_bijection_and_direct_bytes():
    # tokenizer_test.zig:10-41
    seen = set()
    for b in range(256):
        cp = R.BYTE_FWD[b]
        assert cp < 324 and cp not in seen
        seen.add(cp)
        assert R.BYTE_REV[cp] == b
    for b in range(33, 127):
        assert R.BYTE_FWD[b] == b
    assert R.BYTE_FWD[32] >= 256


def test_byte_map_through_library(built_lib):
    # every byte encodes to the vocabulary entry of its mapped code point and back
    t = Lib(SYNTH.read_bytes()).t
    for b in range(256):
        ids = t.encode(bytes([b]))
        assert len(ids) == 1
        assert t.token(ids[0]) == chr(R.BYTE_FWD[b]).encode()
        assert t.decode(ids) == bytes([b])


PRETOKEN_CASES = [  # tokenizer_test.zig:43-79
    (b"hello world", 5), (b" world", 6), (b"a", 1),
    (b"123456", 3), (b"42abc", 2), (b"7", 1),
    (b"'s great", 2), (b"'t do", 2), (b"'re done", 3), (b"'ll go", 3),
    (b"!!!", 3), (b" !!!", 4),
    (b"\n", 1), (b"\n\n", 2), (b"   abc", 3),
]


@pytest.mark.parametrize("text,n", PRETOKEN_CASES)
def test_pretoken_chunk(built_lib, text, n):
    from nnzap_b200.tokenizer import next_pretoken_chunk
    assert R.next_pretoken_chunk(text) == n
    assert next_pretoken_chunk(text) == n


def test_pretoken_chunk_random_bytes(built_lib):
    from nnzap_b200.tokenizer import next_pretoken_chunk
    rng = random.Random(5)
    alphabet = b"ab Z09'\n\r\t\x0b\x0c!?.-_ \xc3\xa9\xe4\xb8\xad\xff\x00"
    for _ in range(3000):
        t = bytes(rng.choice(alphabet) for _ in range(rng.randint(1, 12)))
        assert next_pretoken_chunk(t) == R.next_pretoken_chunk(t), t
    assert next_pretoken_chunk(b"") == 0


def test_utf8_decode_codepoint():
    # tokenizer_test.zig:81-88
    assert R.decode_utf8_codepoint(b"a") == ord("a")
    assert R.decode_utf8_codepoint(bytes([0xC4, 0xA0])) == 0x120
    assert R.decode_utf8_codepoint(bytes([0xE2, 0x82, 0xAC])) == 0x20AC


@pytest.mark.parametrize("impl", IMPLS)
def test_bpe_merge_known_sequence(built_lib, impl):
    # tokenizer_test.zig:90-131
    t = make(impl, tok_json({"a": 0, "b": 1, "c": 2, "ab": 3, "abc": 4}, ["a b", "ab c"]))
    assert t.vocab_size == 5
    assert t.bpe_merge([0, 1, 2]) == [4]


@pytest.mark.parametrize("impl", IMPLS)
def test_encode_decode_round_trip_ascii(built_lib, impl):
    # tokenizer_test.zig:133-174
    t = make(impl, tok_json({"a": 0, "b": 1, "c": 2, "d": 3, "ab": 4, "cd": 5, "abcd": 6},
                            ["a b", "c d", "ab cd"]))
    assert t.encode(b"abcd") == [6]
    assert t.decode([6]) == b"abcd"


@pytest.mark.parametrize("impl", IMPLS)
def test_encode_partial_merges(built_lib, impl):
    # tokenizer_test.zig:176-214
    t = make(impl, tok_json({"a": 0, "b": 1, "x": 2, "c": 3, "d": 4, "ab": 5, "cd": 6}, ["a b", "c d"]))
    assert t.encode(b"abxcd") == [5, 2, 6]


SPECIAL_JSON = tok_json({"a": 0, "b": 1, "ab": 2, "<s>": 10}, ["a b"],
                        [{"id": 10, "content": "<s>", "special": True}])


@pytest.mark.parametrize("impl", IMPLS)
def test_special_tokens_not_split(built_lib, impl):
    # tokenizer_test.zig:216-249
    t = make(impl, SPECIAL_JSON)
    assert t.special_token_count == 1
    assert t.encode(b"ab<s>ab") == [2, 10, 2]


@pytest.mark.parametrize("impl", IMPLS)
def test_decode_special_tokens(built_lib, impl):
    # tokenizer_test.zig:251-275
    assert make(impl, SPECIAL_JSON).decode([2, 10, 2]) == b"ab<s>ab"


@pytest.mark.parametrize("impl", IMPLS)
def test_empty_input(built_lib, impl):
    # tokenizer_test.zig:277-296
    assert make(impl, tok_json({"a": 0}, [])).encode(b"") == []


@pytest.mark.parametrize("impl", IMPLS)
def test_single_bytes_without_merges(built_lib, impl):
    # tokenizer_test.zig:298-322
    assert make(impl, tok_json({"a": 0, "b": 1, "c": 2}, [])).encode(b"abc") == [0, 1, 2]


@pytest.mark.parametrize("impl", IMPLS)
def test_well_known_special_ids(built_lib, impl):
    # tokenizer_test.zig:324-347
    t = make(impl, tok_json({"a": 0}, [], [
        {"id": 100, "content": "<|endoftext|>", "special": True},
        {"id": 101, "content": "<|im_start|>", "special": True},
        {"id": 102, "content": "<|im_end|>", "special": True}]))
    assert (t.eos_token_id, t.im_start_token_id, t.im_end_token_id) == (100, 101, 102)


@pytest.mark.parametrize("impl", IMPLS)
def test_chat_template_special_ids(built_lib, impl):
    # tokenizer_test.zig:349-390: the ids resolve; "\n" has no base token here
    vocab = {"H": 0, "i": 1, "u": 2, "s": 3, "e": 4, "r": 5, "a": 6, "t": 7, "n": 8,
             "<|im_start|>": 100, "<|im_end|>": 101}
    t = make(impl, tok_json(vocab, [], [{"id": 100, "content": "<|im_start|>", "special": True},
                                        {"id": 101, "content": "<|im_end|>", "special": True}]))
    assert (t.im_start_token_id, t.im_end_token_id) == (100, 101)
    assert err_name(impl, lambda: t.apply_chat_template(b"Hi")) == "UnknownByte"


@pytest.mark.parametrize("impl", IMPLS)
def test_decode_token_bytes(built_lib, impl):
    # tokenizer_test.zig:392-408: ASCII maps to itself, U+0120 to a space
    t = make(impl, tok_json({"hello": 0, "Ġ": 1, "Ġhello": 2}, []))
    assert t.decode([0]) == b"hello"
    assert t.decode([1]) == b" "
    assert t.decode([2, 0]) == b" hellohello"


def test_decode_token_to_bytes_function(built_lib):
    # tokenizer_test.zig:392-408, literally: "hello" -> "hello"; U+0120 -> " "
    from nnzap_b200.tokenizer import decode_token_to_bytes
    for f in (decode_token_to_bytes, R.decode_token_to_bytes):
        assert f(b"hello") == b"hello"
        assert f(bytes([0xC4, 0xA0])) == b" "
        assert f(bytes([0xE2, 0x82, 0xAC])) == "€".encode()       # not in the byte map: passes through
        assert f(bytes([0xC4])) == bytes([0xC4])                 # cut-short sequence: raw byte
    rng = random.Random(9)
    for _ in range(500):
        t = bytes(rng.randrange(256) for _ in range(rng.randint(1, 10)))
        assert decode_token_to_bytes(t) == R.decode_token_to_bytes(t)


@pytest.mark.parametrize("impl", IMPLS)
def test_merge_priority_lowest_rank(built_lib, impl):
    # tokenizer_test.zig:410-443
    t = make(impl, tok_json({"a": 0, "b": 1, "c": 2, "ab": 3, "bc": 4}, ["b c", "a b"]))
    assert t.encode(b"abc") == [0, 4]


# ---- golden fixture ----------------------------------------------------------

def golden():
    return json.loads((GOLDEN / "tokenizer_synth_golden.json").read_text(encoding="utf-8"))


@pytest.mark.parametrize("impl", IMPLS)
def test_golden_synthetic_tokenizer(built_lib, impl):
    g = golden()
    t = make(impl, SYNTH.read_bytes())
    assert (t.vocab_size, t.eos_token_id, t.im_start_token_id, t.im_end_token_id) == (
        g["vocab_size"], g["eos_token_id"], g["im_start_token_id"], g["im_end_token_id"])
    for c in g["cases"]:
        if "chat_prompt" in c:
            assert t.apply_chat_template(c["chat_prompt"]) == c["ids"]
        elif "error" in c:
            assert err_name(impl, lambda: t.encode(c["text"])) == c["error"]
        else:
            assert t.encode(c["text"]) == c["ids"], c["text"]
            assert t.decode(c["ids"]) == c["text"].encode()


# ---- differential ------------------------------------------------------------

def random_texts(seed, n):
    rng = random.Random(seed)
    pieces = ["hello", " world", "It's", " don't", "123456789", "  ", "\n\n", "\r\n", "\t",
              "é", "日本語", "😀", "—", "!?", "(x)", "<|im_start|>", "<|im_end|>", "<|endoftext|>",
              "<|im_", "bakodu", " tasefi", "'LL", "\x00", "\x7f"]
    out = []
    for _ in range(n):
        parts = []
        for _ in range(rng.randint(0, 30)):
            r = rng.random()
            if r < 0.6:
                parts.append(rng.choice(pieces).encode())
            elif r < 0.8:
                parts.append(bytes(rng.randrange(256) for _ in range(rng.randint(1, 6))))
            else:
                parts.append(bytes(rng.choice(b"abcdefghijklmnopqrstuvwxyz ") for _ in range(rng.randint(1, 20))))
        out.append(b"".join(parts))
    return out


def test_library_matches_oracle_random_text(built_lib):
    js = SYNTH.read_bytes()
    lib, ref = Lib(js), R.Tokenizer(js)
    for text in random_texts(0, 400):
        ids = lib.encode(text)
        assert ids == ref.encode(text), text
        assert lib.decode(ids) == text
    for p in [b"Hi", "How are you? 日本".encode(), b"<|im_end|>x"]:
        assert lib.apply_chat_template(p) == ref.apply_chat_template(p)


def test_string_and_pair_merge_formats_agree(built_lib):
    data = json.loads(SYNTH.read_text(encoding="utf-8"))
    assert isinstance(data["model"]["merges"][0], list)
    pair = Lib(json.dumps(data))
    data["model"]["merges"] = [" ".join(m) for m in data["model"]["merges"]]
    joined = Lib(json.dumps(data))
    for text in random_texts(1, 100):
        assert pair.encode(text) == joined.encode(text)


def test_bpe_merge_random_sequences(built_lib):
    js = SYNTH.read_bytes()
    lib, ref = Lib(js), R.Tokenizer(js)
    rng = random.Random(3)
    letters = [lib.t.encode(bytes([c]))[0] for c in b"aeioubkdtsn \xc4"]
    for _ in range(300):
        seq = [rng.choice(letters) for _ in range(rng.randint(0, 40))]
        assert lib.bpe_merge(seq) == ref.bpe_merge(seq)


def test_merge_to_missing_token_stops_merging(built_lib):
    # "a b" ranks first but "ab" is not in the vocabulary: merging stops there
    js = tok_json({"a": 0, "b": 1, "c": 2, "bc": 3}, ["a b", "b c"])
    for impl in IMPLS:
        assert make(impl, js).encode(b"abc") == [0, 1, 2]


def test_longest_special_token_wins(built_lib):
    js = tok_json({"a": 0, "<": 1, ">": 2, "b": 3}, [], [
        {"id": 10, "content": "<a>", "special": True},
        {"id": 11, "content": "<a>b", "special": True},
        {"id": 12, "content": "<a>", "special": True}])
    for impl in IMPLS:
        t = make(impl, js)
        assert t.encode(b"<a>b<a>a") == [11, 10, 0]


def test_concurrent_encode_is_consistent(built_lib):
    lib = Lib(SYNTH.read_bytes())
    texts = random_texts(2, 64)
    want = [lib.encode(t) for t in texts]
    got = [None] * len(texts)

    def work(k):
        for i in range(k, len(texts), 4):
            got[i] = lib.encode(texts[i])

    th = [threading.Thread(target=work, args=(k,)) for k in range(4)]
    for x in th:
        x.start()
    for x in th:
        x.join()
    assert got == want


# ---- errors ----------------------------------------------------------------------

@pytest.mark.parametrize("js,name", [
    ("not json", "InvalidJson"),
    ("[1, 2]", "InvalidJson"),
    ('{"added_tokens": []}', "MissingField"),
    ('{"model": 3}', "InvalidJson"),
    ('{"model": {"merges": []}}', "MissingField"),
    ('{"model": {"vocab": []}}', "InvalidJson"),
    ('{"model": {"vocab": {"a": 1.5}}}', "InvalidVocabEntry"),
    ('{"model": {"vocab": {"a": -1}}}', "InvalidVocabEntry"),
    ('{"model": {"vocab": {"a": "0"}}}', "InvalidVocabEntry"),
    ('{"model": {"vocab": {"a": 200000}}}', "VocabTooLarge"),
    ('{"model": {"vocab": {"a": 0}, "merges": "a b"}}', "InvalidJson"),
    ('{"model": {"vocab": {"a": 0}, "merges": [["a"]]}}', "InvalidMergeEntry"),
    ('{"model": {"vocab": {"a": 0}, "merges": [3]}}', "InvalidMergeEntry"),
    ('{"model": {"vocab": {"a": 0}}, "added_tokens": {}}', "InvalidJson"),
    ('{"model": {"vocab": {"a": 0, "b": 1, "a": 2}}}', "InvalidJson"),
    ('{"model": {"vocab": {"a": 0}}, "model": {"vocab": {"a": 0}}}', "InvalidJson"),
])
def test_load_errors(built_lib, js, name):
    from nnzap_b200.tokenizer import Tokenizer
    assert err_name("lib", lambda: Tokenizer.from_json(js)) == name
    assert err_name("oracle", lambda: R.Tokenizer(js)) == name


def test_skipped_added_tokens(built_lib):
    # malformed added_tokens entries are skipped, not errors (tokenizer.zig:536-585)
    js = tok_json({"a": 0}, [], [3, {"id": -1, "content": "x", "special": True},
                                 {"id": 5, "special": True}, {"id": 6, "content": 7},
                                 {"id": 7, "content": "<q>", "special": "yes"},
                                 {"id": 250000, "content": "<big>", "special": True}])
    for impl in IMPLS:
        t = make(impl, js)
        assert t.vocab_size == 8 and t.special_token_count == 1
        assert t.encode(b"<big>a") == [250000, 0]


def test_encode_errors(built_lib):
    t = Lib(tok_json({"a": 0, "b": 1, "c": 2}, []))
    ref = R.Tokenizer(tok_json({"a": 0, "b": 1, "c": 2}, []))
    assert err_name("lib", lambda: t.encode(b"abz")) == "UnknownByte"
    assert err_name("oracle", lambda: ref.encode(b"abz")) == "UnknownByte"
    assert err_name("lib", lambda: t.encode(b"a" * 513)) == "ChunkTooLong"
    assert t.encode(b"a" * 512) == [0] * 512
    assert err_name("lib", lambda: t.encode(b"a" * (1024 * 1024 + 1))) == "InputTooLong"
    assert err_name("lib", lambda: t.decode([3])) == "UnknownTokenId"
    assert err_name("oracle", lambda: ref.decode([3])) == "UnknownTokenId"


def test_output_buffer_too_small(built_lib):
    from nnzap_b200 import _capi
    t = Lib(SYNTH.read_bytes()).t
    text = b"hello world, 12345"
    n_need = len(t.encode(text))
    out = np.zeros(64, np.uint32)
    n = C.c_uint32()
    L = _capi.lib()
    assert L.nnz_tokenizer_encode(t._h, text, len(text), out.ctypes.data, n_need - 1, C.byref(n)) == _capi.NNZ_ERANGE
    assert L.nnz_last_error().startswith(b"OutputBufferTooSmall")
    assert L.nnz_tokenizer_encode(t._h, text, len(text), out.ctypes.data, n_need, C.byref(n)) == 0
    assert n.value == n_need
    buf = C.create_string_buffer(4)
    m = C.c_size_t()
    assert L.nnz_tokenizer_decode(t._h, out.ctypes.data, n_need, buf, 4, C.byref(m)) == _capi.NNZ_ERANGE
    assert L.nnz_tokenizer_chat_template(t._h, b"x", 1, out.ctypes.data, 3, C.byref(n)) == _capi.NNZ_ERANGE


def test_from_file(built_lib, tmp_path):
    from nnzap_b200 import _capi
    from nnzap_b200.tokenizer import Tokenizer, TokenizerError
    t = Tokenizer.from_file(SYNTH)
    assert t.vocab_size == golden()["vocab_size"]
    with pytest.raises(TokenizerError) as e:
        Tokenizer.from_file(tmp_path / "missing.json")
    assert e.value.code == _capi.NNZ_ENOTFOUND and e.value.reason == "FileNotFound"
    t.close()
    t.close()


def test_memo_does_not_leak_between_tokenizers(built_lib):
    # same bytes, different merges: each tokenizer keeps its own encoding when
    # they alternate on one thread, and after one is freed and another created
    a_js = tok_json({"a": 0, "b": 1, "ab": 2}, ["a b"])
    b_js = tok_json({"a": 0, "b": 1, "ab": 2}, [])
    a, b = Lib(a_js), Lib(b_js)
    for _ in range(3):
        assert a.encode(b"abab") == [2, 2]
        assert b.encode(b"abab") == [0, 1, 0, 1]
    a.t.close()
    c = Lib(b_js)
    assert c.encode(b"abab") == [0, 1, 0, 1]


def test_large_random_vocabulary_matches_oracle(built_lib):
    # ~40k random merges over the 256 byte tokens (deep merge chains, many
    # competing ranks): library == oracle on random text, and the round trip
    rng = random.Random(11)
    base = [chr(R.BYTE_FWD[b]) for b in range(256)]
    vocab = {s: i for i, s in enumerate(base)}
    merges, toks = [], list(base)
    while len(vocab) < 40000:
        a, b = rng.choice(toks), rng.choice(toks)
        if len(a) + len(b) > 12 or (a + b) in vocab:
            continue
        vocab[a + b] = len(vocab)
        toks.append(a + b)
        merges.append([a, b])
    js = tok_json(vocab, merges, [{"id": 40000, "content": "<|im_end|>", "special": True}])
    lib, ref = Lib(js), R.Tokenizer(js)
    assert lib.vocab_size == ref.vocab_size == 40001
    for text in random_texts(7, 60):
        ids = lib.encode(text)
        assert ids == ref.encode(text)
        assert lib.decode(ids) == text
