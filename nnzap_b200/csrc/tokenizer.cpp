// Byte-level BPE tokenizer behind the C ABI (host code; no device calls).
//
// Same behaviour as the reference's Tokenizer (nnmetal/src/tokenizer.zig):
// the tokenizer.json fields it reads, its limits and its errors, the GPT-2
// byte <-> unicode table, the simplified GPT-4-style pre-tokenizer, greedy
// lowest-rank merging inside each chunk, longest-first special-token
// matching, the raw-byte decode and the Qwen3 chat template.
//
// Data structures are this library's own: the merge table is keyed by the
// pair of token ids (resolved once at load from the "a b" strings) instead
// of by the joined string, special tokens are bucketed by first byte, and the
// merge loop keeps the rank of every adjacent pair so that a merge only
// re-ranks its two neighbours.  None of this changes which pair merges
// first: the lowest rank, leftmost on ties, exactly as findBestPair /
// bpeMerge (tokenizer.zig:761-930) choose it.
#include <array>
#include <atomic>
#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <new>
#include <string>
#include <string_view>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "../../include/nnz_b200.h"
#include "json_reader.h"

namespace nnz {
void set_last_error(const std::string& msg);   // nnz_last_error() text (engine.cu)
}

namespace {

using nnz_json::JsonReader;
using nnz_json::JVal;
using nnz_json::utf8_append;

// Limits of tokenizer.zig:28-46.
constexpr uint32_t kMaxVocab = 200000;
constexpr uint32_t kMaxMerges = 200000;
constexpr uint32_t kMaxTokenLength = 512;
constexpr uint32_t kMaxSpecial = 256;
constexpr size_t kMaxInput = 1024 * 1024;
constexpr size_t kMaxJsonBytes = 32u * 1024u * 1024u;
constexpr uint32_t kNone = 0xFFFFFFFFu;

int fail(int code, const std::string& msg) {
  nnz::set_last_error(msg);
  return code;
}

// No C++ exception crosses the C ABI: a failed host allocation becomes
// NNZ_ENOMEM.
template <typename F>
int host_guard(F&& f) {
  try {
    return f();
  } catch (const std::bad_alloc&) {
    return fail(NNZ_ENOMEM, "OutOfMemory: host allocation failed");
  } catch (const std::exception& e) {
    return fail(NNZ_EINVAL, std::string("host error: ") + e.what());
  }
}

// ---- GPT-2 byte <-> unicode table (tokenizer.zig:52-108) -----------------
// Bytes 33-126, 161-172 and 174-255 stand for themselves; the other 68 take
// code points 256.. in byte order.
struct ByteMap {
  uint32_t fwd[256];
  int16_t rev[324];   // code point -> byte, -1 where unmapped
  ByteMap() {
    for (int i = 0; i < 324; ++i) rev[i] = -1;
    uint32_t extra = 0;
    for (int b = 0; b < 256; ++b) {
      const bool direct = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || b >= 174;
      fwd[b] = direct ? (uint32_t)b : 256 + extra++;
      rev[fwd[b]] = (int16_t)b;
    }
  }
};
const ByteMap kByteMap;

// ---- pre-tokenizer (tokenizer.zig:936-1060) --------------------------------
inline bool is_letter(uint8_t b) { return (b >= 'a' && b <= 'z') || (b >= 'A' && b <= 'Z') || b >= 0x80; }
inline bool is_digit(uint8_t b) { return b >= '0' && b <= '9'; }
inline bool is_ws(uint8_t b) { return b == ' ' || b == '\t' || b == '\n' || b == '\r' || b == 0x0B || b == 0x0C; }
inline bool is_nl(uint8_t b) { return b == '\n' || b == '\r'; }
inline bool is_sym(uint8_t b) { return !is_letter(b) && !is_digit(b) && !is_ws(b); }

// Length of the first chunk of t[0..n), n > 0: contraction, optional
// non-letter/non-digit/non-newline byte + letters, 1-3 digits, optional
// space + symbol run, newline run, other-whitespace run, else one byte.
uint32_t pretoken_chunk(const uint8_t* t, uint32_t n) {
  if (t[0] == '\'' && n >= 2) {
    const uint8_t c1 = t[1] | 0x20;
    if (c1 == 's' || c1 == 't' || c1 == 'm' || c1 == 'd') return 2;
    if (n >= 3) {
      const uint8_t c2 = t[2] | 0x20;
      if ((c1 == 'r' && c2 == 'e') || (c1 == 'v' && c2 == 'e') || (c1 == 'l' && c2 == 'l')) return 3;
    }
  }
  auto letters_from = [&](uint32_t i) {
    while (i < n && is_letter(t[i])) ++i;
    return i;
  };
  if (is_letter(t[0])) return letters_from(0);
  if (n > 1 && !is_letter(t[0]) && !is_digit(t[0]) && !is_nl(t[0]) && is_letter(t[1])) return letters_from(1);
  if (is_digit(t[0])) {
    uint32_t e = 1;
    while (e < n && e < 3 && is_digit(t[e])) ++e;
    return e;
  }
  if (is_sym(t[0])) {
    uint32_t e = 1;
    while (e < n && is_sym(t[e])) ++e;
    return e;
  }
  if (t[0] == ' ' && n > 1 && is_sym(t[1])) {
    uint32_t e = 2;
    while (e < n && is_sym(t[e])) ++e;
    return e;
  }
  if (is_nl(t[0])) {
    uint32_t e = 1;
    while (e < n && is_nl(t[e])) ++e;
    return e;
  }
  if (is_ws(t[0])) {
    uint32_t e = 1;
    while (e < n && is_ws(t[e]) && !is_nl(t[e])) ++e;
    return e;
  }
  return 1;
}

// Token string (byte-level form) -> raw bytes (decodeTokenToBytes,
// tokenizer.zig:1066-1108): each UTF-8 sequence whose code point is in the
// byte map becomes that byte; other sequences pass through; a sequence cut
// short by the end of the string passes its first byte through.
size_t token_to_bytes(const std::string& s, char* out) {
  size_t o = 0, i = 0;
  const size_t n = s.size();
  while (i < n) {
    const uint8_t f = (uint8_t)s[i];
    const size_t len = f < 0xC0 ? 1 : f < 0xE0 ? 2 : f < 0xF0 ? 3 : 4;
    if (i + len > n) {
      out[o++] = s[i++];
      continue;
    }
    uint32_t cp;
    const uint8_t* b = reinterpret_cast<const uint8_t*>(s.data() + i);
    if (len == 1) cp = b[0];
    else if (len == 2) cp = ((uint32_t)(b[0] & 0x1F) << 6) | (b[1] & 0x3F);
    else if (len == 3) cp = ((uint32_t)(b[0] & 0x0F) << 12) | ((uint32_t)(b[1] & 0x3F) << 6) | (b[2] & 0x3F);
    else cp = ((uint32_t)(b[0] & 0x07) << 18) | ((uint32_t)(b[1] & 0x3F) << 12) | ((uint32_t)(b[2] & 0x3F) << 6) | (b[3] & 0x3F);
    if (cp < 324 && kByteMap.rev[cp] >= 0) {
      out[o++] = (char)kByteMap.rev[cp];
    } else {
      memcpy(out + o, b, len);
      o += len;
    }
    i += len;
  }
  return o;
}

struct Merge {
  uint32_t rank;
  uint32_t merged;   // id of the joined string, kNone when it is not in the vocabulary
};

inline uint64_t pair_key(uint32_t a, uint32_t b) { return ((uint64_t)a << 32) | b; }

// Open-addressing table (id pair -> Merge): power-of-two slots at most half
// full, multiplicative hash, linear probing.  Built once; read-only after.
class PairTable {
 public:
  // room for up to n entries at most half full
  void reserve(size_t n) {
    size_t cap = 16;
    while (cap < 2 * n) cap <<= 1;
    bits_ = 0;
    while ((size_t(1) << bits_) < cap) ++bits_;
    keys_.assign(cap, kEmpty);
    vals_.assign(cap, Merge{kNone, kNone});
    count_ = 0;
  }
  // insert or overwrite (a later merge entry for the same pair wins)
  void put(uint64_t key, Merge m) {
    if (2 * (count_ + 1) > keys_.size()) grow();
    const size_t mask = keys_.size() - 1;
    size_t i = slot(key);
    while (keys_[i] != kEmpty && keys_[i] != key) i = (i + 1) & mask;
    if (keys_[i] == kEmpty) ++count_;
    keys_[i] = key;
    vals_[i] = m;
  }
  const Merge* find(uint64_t key) const {
    const size_t mask = keys_.size() - 1;
    for (size_t i = slot(key);; i = (i + 1) & mask) {
      if (keys_[i] == key) return &vals_[i];
      if (keys_[i] == kEmpty) return nullptr;
    }
  }

 private:
  static constexpr uint64_t kEmpty = ~0ull;   // ids are < 2^18: never a real key
  size_t slot(uint64_t k) const { return (size_t)((k * 0x9E3779B97F4A7C15ull) >> (64 - bits_)); }
  void grow() {
    std::vector<uint64_t> k = std::move(keys_);
    std::vector<Merge> v = std::move(vals_);
    reserve(k.size());   // twice the slots
    for (size_t i = 0; i < k.size(); ++i)
      if (k[i] != kEmpty) put(k[i], v[i]);
  }
  std::vector<uint64_t> keys_{std::vector<uint64_t>(16, kEmpty)};
  std::vector<Merge> vals_{std::vector<Merge>(16, Merge{kNone, kNone})};
  size_t count_ = 0;
  unsigned bits_ = 4;
};

// Per-thread memo of merged chunks (natural text repeats its words): chunk
// bytes -> merged ids, for one tokenizer at a time (by serial number, so a
// freed and re-created handle never sees stale entries), cleared when full.
// Only successful merges are stored; the result is a pure function of the
// chunk's bytes, so the memo never changes an encoding.
struct ViewHash {
  using is_transparent = void;
  size_t operator()(std::string_view v) const { return std::hash<std::string_view>{}(v); }
};
struct ChunkMemo {
  uint64_t owner = 0;
  std::unordered_map<std::string, std::vector<uint32_t>, ViewHash, std::equal_to<>> map;
};
constexpr size_t kMemoEntries = 1 << 16;
constexpr uint32_t kMemoMaxChunk = 64;
thread_local ChunkMemo tl_memo;
std::atomic<uint64_t> g_serial{1};

}  // namespace

struct nnz_tokenizer {
  const uint64_t serial = g_serial.fetch_add(1);
  std::vector<std::string> id_to_vocab;                  // "" = unused id
  std::unordered_map<std::string, uint32_t> vocab_to_id;
  PairTable merges;
  uint32_t merge_count = 0;
  std::vector<std::pair<std::string, uint32_t>> specials;   // in added_tokens order
  std::array<std::vector<uint32_t>, 256> special_by_byte;   // indices into specials
  uint32_t byte_id[256];
  uint32_t vocab_size = 0, eos = 0, im_start = 0, im_end = 0;

  // ---- loading (parseJson / parseModel / parseVocab / parseMerges /
  // parseAddedTokens / resolveSpecialTokenIds / buildByteTokenTable,
  // tokenizer.zig:375-686)
  int load(const char* json, size_t len) {
    if (len == 0 || len > kMaxJsonBytes) return fail(NNZ_EINVAL, "InvalidJson: empty or larger than 32 MiB");
    JVal root;
    std::string err;
    if (!JsonReader(json, len).parse(root, err)) return fail(NNZ_EINVAL, "InvalidJson: " + err);
    if (root.kind != JVal::OBJ) return fail(NNZ_EINVAL, "InvalidJson: root is not an object");
    const JVal* model = root.get("model");
    if (!model) return fail(NNZ_EINVAL, "MissingField: 'model'");
    if (model->kind != JVal::OBJ) return fail(NNZ_EINVAL, "InvalidJson: 'model' is not an object");
    const JVal* vocab = model->get("vocab");
    if (!vocab) return fail(NNZ_EINVAL, "MissingField: 'model.vocab'");
    if (vocab->kind != JVal::OBJ) return fail(NNZ_EINVAL, "InvalidJson: 'model.vocab' is not an object");
    vocab_to_id.reserve(vocab->obj.size() + 64);
    for (const auto& kv : vocab->obj) {
      if (kv.second.kind != JVal::INT || kv.second.i < 0 || kv.second.i > 0xFFFFFFFFll)
        return fail(NNZ_EINVAL, "InvalidVocabEntry: '" + kv.first + "'");
      const uint32_t id = (uint32_t)kv.second.i;
      if (id >= kMaxVocab)
        return fail(NNZ_EINVAL, "VocabTooLarge: id " + std::to_string(id) + " >= 200000");
      vocab_to_id[kv.first] = id;
      if (id >= id_to_vocab.size()) id_to_vocab.resize(id + 1);
      id_to_vocab[id] = kv.first;
      if (id >= vocab_size) vocab_size = id + 1;
    }
    // merges: the joined "a b" keys by rank (a repeated key keeps its last rank)
    std::vector<std::pair<std::string, uint32_t>> keys;
    if (const JVal* m = model->get("merges")) {
      if (m->kind != JVal::ARR) return fail(NNZ_EINVAL, "InvalidJson: 'model.merges' is not an array");
      if (m->arr.size() > kMaxMerges) return fail(NNZ_EINVAL, "TooManyMerges: more than 200000");
      merge_count = (uint32_t)m->arr.size();
      for (uint32_t r = 0; r < merge_count; ++r) {
        const JVal& it = m->arr[r];
        if (it.kind == JVal::STR) {
          keys.emplace_back(it.s, r);
        } else if (it.kind == JVal::ARR) {
          if (it.arr.size() != 2 || it.arr[0].kind != JVal::STR || it.arr[1].kind != JVal::STR)
            return fail(NNZ_EINVAL, "InvalidMergeEntry: rank " + std::to_string(r));
          keys.emplace_back(it.arr[0].s + " " + it.arr[1].s, r);
        } else {
          return fail(NNZ_EINVAL, "InvalidMergeEntry: rank " + std::to_string(r));
        }
      }
    }
    // added tokens: into the vocabulary (id_to_vocab only where still unused),
    // and the special ones into the special list
    if (const JVal* added = root.get("added_tokens")) {
      if (added->kind != JVal::ARR) return fail(NNZ_EINVAL, "InvalidJson: 'added_tokens' is not an array");
      for (const JVal& it : added->arr) {
        if (it.kind != JVal::OBJ) continue;
        const JVal* idv = it.get("id");
        if (!idv || idv->kind != JVal::INT || idv->i < 0 || idv->i > 0xFFFFFFFFll) continue;
        const JVal* cv = it.get("content");
        if (!cv || cv->kind != JVal::STR) continue;
        const uint32_t id = (uint32_t)idv->i;
        const JVal* sp = it.get("special");
        const bool special = sp && sp->kind == JVal::BOOL && sp->b;
        if (id < kMaxVocab) {
          if (id >= id_to_vocab.size()) id_to_vocab.resize(id + 1);
          if (id_to_vocab[id].empty()) id_to_vocab[id] = cv->s;
          vocab_to_id[cv->s] = id;
          if (id >= vocab_size) vocab_size = id + 1;
        }
        if (special && specials.size() < kMaxSpecial) specials.emplace_back(cv->s, id);
      }
    }
    if (vocab_size == 0) return fail(NNZ_EINVAL, "InvalidJson: empty vocabulary");
    id_to_vocab.resize(vocab_size);
    for (const auto& st : specials) {
      if (st.first == "<|endoftext|>") eos = st.second;
      if (st.first == "<|im_start|>") im_start = st.second;
      if (st.first == "<|im_end|>") im_end = st.second;
    }
    for (uint32_t i = 0; i < specials.size(); ++i)
      if (!specials[i].first.empty()) special_by_byte[(uint8_t)specials[i].first[0]].push_back(i);
    for (int b = 0; b < 256; ++b) {
      std::string u;
      utf8_append(u, kByteMap.fwd[b]);
      auto it = vocab_to_id.find(u);
      byte_id[b] = it == vocab_to_id.end() ? kNone : it->second;
    }
    // A key "A B" ranks every id pair whose vocabulary strings are A and B,
    // for every split at a space (the reference compares joined strings);
    // pairs whose joined key exceeds its 1025-byte buffer never match there.
    // ids by vocabulary string: one id almost always; strings shared by
    // several ids (possible through added_tokens) keep the rest aside
    std::unordered_map<std::string_view, uint32_t> id_of;
    std::unordered_map<std::string_view, std::vector<uint32_t>> more_ids;
    id_of.reserve(vocab_size);
    for (uint32_t id = 0; id < vocab_size; ++id) {
      if (id_to_vocab[id].empty()) continue;
      auto [it, fresh] = id_of.emplace(id_to_vocab[id], id);
      if (!fresh) more_ids[it->first].push_back(id);
    }
    auto for_ids = [&](std::string_view s, auto&& f) {
      auto it = id_of.find(s);
      if (it == id_of.end()) return;
      f(it->second);
      if (!more_ids.empty()) {
        auto m = more_ids.find(s);
        if (m != more_ids.end())
          for (uint32_t id : m->second) f(id);
      }
    };
    merges.reserve(keys.size());
    std::string joined;
    for (const auto& [key, rank] : keys) {
      if (key.size() > 2 * kMaxTokenLength + 1) continue;
      for (size_t sp = key.find(' '); sp != std::string::npos; sp = key.find(' ', sp + 1)) {
        const std::string_view A(key.data(), sp), B(key.data() + sp + 1, key.size() - sp - 1);
        if (!id_of.count(A) || !id_of.count(B)) continue;
        joined.assign(A);
        joined.append(B);
        auto jm = vocab_to_id.find(joined);
        const Merge mg{rank, jm == vocab_to_id.end() ? kNone : jm->second};
        for_ids(A, [&](uint32_t a) { for_ids(B, [&](uint32_t b) { merges.put(pair_key(a, b), mg); }); });
      }
    }
    return NNZ_OK;
  }

  // ---- encoding (tokenizer.zig:247-289, 691-878)
  // Longest special token starting at t[pos] (first listed among equals).
  const std::pair<std::string, uint32_t>* special_at(const uint8_t* t, size_t n, size_t pos) const {
    const std::pair<std::string, uint32_t>* best = nullptr;
    size_t best_len = 0;
    for (uint32_t i : special_by_byte[t[pos]]) {
      const std::string& c = specials[i].first;
      if (c.size() <= best_len || c.size() > n - pos) continue;
      if (memcmp(t + pos, c.data(), c.size()) == 0) {
        best = &specials[i];
        best_len = c.size();
      }
    }
    return best;
  }

  uint32_t rank_of(uint32_t a, uint32_t b) const {
    const Merge* m = merges.find(pair_key(a, b));
    return m ? m->rank : kNone;
  }

  // Greedy merging of tok[0..n): the lowest-rank adjacent pair (leftmost on
  // ties) merges until none is left or the best pair's joined string is not
  // in the vocabulary.
  uint32_t bpe_merge(uint32_t* tok, uint32_t n) const {
    if (n < 2) return n;
    uint32_t pr[kMaxTokenLength];   // rank of each adjacent pair (n <= 512)
    for (uint32_t i = 0; i + 1 < n; ++i) pr[i] = rank_of(tok[i], tok[i + 1]);
    while (n > 1) {
      uint32_t bi = 0, br = kNone;
      for (uint32_t i = 0; i + 1 < n; ++i)
        if (pr[i] < br) { br = pr[i]; bi = i; }
      if (br == kNone) break;
      const uint32_t merged = merges.find(pair_key(tok[bi], tok[bi + 1]))->merged;
      if (merged == kNone) break;
      tok[bi] = merged;
      memmove(tok + bi + 1, tok + bi + 2, (n - bi - 2) * sizeof(uint32_t));
      // drop pr[bi] (the merged pair); pr[bi] becomes (merged, next)
      memmove(pr + bi, pr + bi + 1, (n - bi - 2) * sizeof(uint32_t));
      --n;
      if (bi + 1 < n) pr[bi] = rank_of(tok[bi], tok[bi + 1]);
      if (bi > 0) pr[bi - 1] = rank_of(tok[bi - 1], tok[bi]);
    }
    return n;
  }

  int encode(const uint8_t* t, size_t n, uint32_t* out, uint32_t cap, uint32_t* n_out) const {
    *n_out = 0;
    if (n == 0) return NNZ_OK;
    if (n > kMaxInput) return fail(NNZ_EINVAL, "InputTooLong: more than 1 MiB");
    uint32_t cnt = 0;
    uint32_t chunk[kMaxTokenLength];
    size_t cur = 0;
    while (cur < n) {
      if (const auto* st = special_at(t, n, cur)) {
        if (cnt >= cap) return fail(NNZ_ERANGE, "OutputBufferTooSmall");
        out[cnt++] = st->second;
        cur += st->first.size();
        continue;
      }
      size_t seg = cur + 1;
      while (seg < n && !special_at(t, n, seg)) ++seg;
      size_t pos = cur;
      while (pos < seg) {
        const uint32_t cl = pretoken_chunk(t + pos, (uint32_t)(seg - pos));
        const uint32_t* ids = chunk;
        uint32_t m = 0;
        const std::string_view key(reinterpret_cast<const char*>(t + pos), cl);
        const bool memoize = cl >= 2 && cl <= kMemoMaxChunk;
        ChunkMemo& memo = tl_memo;
        bool hit = false;
        if (memoize) {
          if (memo.owner != serial) {
            memo.map.clear();
            memo.owner = serial;
          }
          auto it = memo.map.find(key);   // a stored chunk's bytes all have base tokens
          if (it != memo.map.end()) {
            ids = it->second.data();
            m = (uint32_t)it->second.size();
            hit = true;
          }
        }
        if (!hit) {
          // byte by byte, as the reference checks them: an unknown byte within
          // the first 512 is reported before the chunk's length
          for (uint32_t k = 0; k < cl; ++k) {
            if (k >= kMaxTokenLength)
              return fail(NNZ_EINVAL, "ChunkTooLong: a pre-tokenized chunk exceeds 512 bytes");
            chunk[k] = byte_id[t[pos + k]];
            if (chunk[k] == kNone) {
              char msg[64];
              snprintf(msg, sizeof msg, "UnknownByte: no base token for byte 0x%02x", t[pos + k]);
              return fail(NNZ_EINVAL, msg);
            }
          }
          m = bpe_merge(chunk, cl);
          if (memoize) {
            if (memo.map.size() >= kMemoEntries) memo.map.clear();
            memo.map.emplace(std::string(key), std::vector<uint32_t>(chunk, chunk + m));
          }
        }
        if (m > cap - cnt) return fail(NNZ_ERANGE, "OutputBufferTooSmall");
        memcpy(out + cnt, ids, m * sizeof(uint32_t));
        cnt += m;
        pos += cl;
      }
      cur = seg;
    }
    *n_out = cnt;
    return NNZ_OK;
  }

  int decode(const uint32_t* ids, uint32_t n, char* out, size_t cap, size_t* n_out) const {
    *n_out = 0;
    size_t pos = 0;
    for (uint32_t k = 0; k < n; ++k) {
      const uint32_t id = ids[k];
      if (id >= vocab_size || id_to_vocab[id].empty())
        return fail(NNZ_EINVAL, "UnknownTokenId: " + std::to_string(id));
      const std::string& s = id_to_vocab[id];
      if (cap - pos < s.size()) return fail(NNZ_ERANGE, "OutputBufferTooSmall");
      pos += token_to_bytes(s, out + pos);
    }
    *n_out = pos;
    return NNZ_OK;
  }
};

extern "C" {

static int tokenizer_from_json_impl(const char* json, size_t len, nnz_tokenizer** out) {
  if (!out || (!json && len)) return fail(NNZ_EINVAL, "nnz_tokenizer_from_json: null argument");
  *out = nullptr;
  try {
    auto t = std::make_unique<nnz_tokenizer>();
    const int rc = t->load(json, len);
    if (rc != NNZ_OK) return rc;
    *out = t.release();
    return NNZ_OK;
  } catch (const std::bad_alloc&) {
    return fail(NNZ_ENOMEM, "OutOfMemory while parsing the tokenizer");
  }
}

int nnz_tokenizer_from_json(const char* json, size_t len, nnz_tokenizer** out) {
  return host_guard([&] { return tokenizer_from_json_impl(json, len, out); });
}

static int tokenizer_from_file_impl(const char* path, nnz_tokenizer** out) {
  if (!path || !out || !*path) return fail(NNZ_EINVAL, "nnz_tokenizer_from_file: null or empty path");
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) return fail(NNZ_ENOTFOUND, std::string("FileNotFound: cannot open ") + path);
  std::string buf;
  char tmp[1 << 16];
  size_t r;
  while ((r = fread(tmp, 1, sizeof tmp, f)) > 0) {
    buf.append(tmp, r);
    if (buf.size() > kMaxJsonBytes) {
      fclose(f);
      return fail(NNZ_EINVAL, "FileTooBig: tokenizer file larger than 32 MiB");
    }
  }
  fclose(f);
  return nnz_tokenizer_from_json(buf.data(), buf.size(), out);
}

int nnz_tokenizer_from_file(const char* path, nnz_tokenizer** out) {
  return host_guard([&] { return tokenizer_from_file_impl(path, out); });
}

static int tokenizer_free_impl(nnz_tokenizer* tok) {
  delete tok;
  return NNZ_OK;
}

int nnz_tokenizer_free(nnz_tokenizer* tok) {
  return host_guard([&] { return tokenizer_free_impl(tok); });
}

static int tokenizer_get_info_impl(const nnz_tokenizer* tok, nnz_tokenizer_info* info) {
  if (!tok || !info) return fail(NNZ_EINVAL, "nnz_tokenizer_get_info: null argument");
  info->vocab_size = tok->vocab_size;
  info->special_token_count = (uint32_t)tok->specials.size();
  info->eos_token_id = tok->eos;
  info->im_start_token_id = tok->im_start;
  info->im_end_token_id = tok->im_end;
  info->merge_count = tok->merge_count;
  return NNZ_OK;
}

int nnz_tokenizer_get_info(const nnz_tokenizer* tok, nnz_tokenizer_info* info) {
  return host_guard([&] { return tokenizer_get_info_impl(tok, info); });
}

static int tokenizer_encode_impl(const nnz_tokenizer* tok, const char* text, size_t len, uint32_t* ids,
                         uint32_t cap, uint32_t* n_out) {
  if (!tok || !n_out || (!text && len) || (!ids && cap)) return fail(NNZ_EINVAL, "nnz_tokenizer_encode: null argument");
  return tok->encode(reinterpret_cast<const uint8_t*>(text), len, ids, cap, n_out);
}

int nnz_tokenizer_encode(const nnz_tokenizer* tok, const char* text, size_t len, uint32_t* ids,
                         uint32_t cap, uint32_t* n_out) {
  return host_guard([&] { return tokenizer_encode_impl(tok, text, len, ids, cap, n_out); });
}

static int tokenizer_decode_impl(const nnz_tokenizer* tok, const uint32_t* ids, uint32_t n, char* out, size_t cap,
                         size_t* n_out) {
  if (!tok || !n_out || (!ids && n) || (!out && cap)) return fail(NNZ_EINVAL, "nnz_tokenizer_decode: null argument");
  return tok->decode(ids, n, out, cap, n_out);
}

int nnz_tokenizer_decode(const nnz_tokenizer* tok, const uint32_t* ids, uint32_t n, char* out, size_t cap,
                         size_t* n_out) {
  return host_guard([&] { return tokenizer_decode_impl(tok, ids, n, out, cap, n_out); });
}

static int tokenizer_chat_template_impl(const nnz_tokenizer* tok, const char* prompt, size_t len, uint32_t* ids,
                                uint32_t cap, uint32_t* n_out) {
  if (!tok || !n_out || !prompt || len == 0 || (!ids && cap))
    return fail(NNZ_EINVAL, "nnz_tokenizer_chat_template: null argument or empty prompt");
  *n_out = 0;
  uint32_t cnt = 0, m = 0;
  auto special = [&](uint32_t id) {
    if (cnt >= cap) return fail(NNZ_ERANGE, "OutputBufferTooSmall");
    ids[cnt++] = id;
    return (int)NNZ_OK;
  };
  auto text = [&](const char* s, size_t n) {
    const int rc = tok->encode(reinterpret_cast<const uint8_t*>(s), n, ids + cnt, cap - cnt, &m);
    cnt += m;
    return rc;
  };
  int rc;
  if ((rc = special(tok->im_start)) || (rc = text("user\n", 5)) || (rc = text(prompt, len)) ||
      (rc = special(tok->im_end)) || (rc = text("\n", 1)) || (rc = special(tok->im_start)) ||
      (rc = text("assistant\n", 10)))
    return rc;
  *n_out = cnt;
  return NNZ_OK;
}

int nnz_tokenizer_chat_template(const nnz_tokenizer* tok, const char* prompt, size_t len, uint32_t* ids,
                                uint32_t cap, uint32_t* n_out) {
  return host_guard([&] { return tokenizer_chat_template_impl(tok, prompt, len, ids, cap, n_out); });
}

static int tokenizer_bpe_merge_impl(const nnz_tokenizer* tok, uint32_t* ids, uint32_t n, uint32_t* n_out) {
  if (!tok || !n_out || (!ids && n)) return fail(NNZ_EINVAL, "nnz_tokenizer_bpe_merge: null argument");
  if (n > kMaxTokenLength) return fail(NNZ_EINVAL, "ChunkTooLong: more than 512 tokens");
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= tok->vocab_size) return fail(NNZ_EINVAL, "UnknownTokenId: " + std::to_string(ids[i]));
  *n_out = tok->bpe_merge(ids, n);
  return NNZ_OK;
}

int nnz_tokenizer_bpe_merge(const nnz_tokenizer* tok, uint32_t* ids, uint32_t n, uint32_t* n_out) {
  return host_guard([&] { return tokenizer_bpe_merge_impl(tok, ids, n, n_out); });
}

static int tokenizer_token_impl(const nnz_tokenizer* tok, uint32_t id, char* out, size_t cap, size_t* n_out) {
  if (!tok || !n_out || (!out && cap)) return fail(NNZ_EINVAL, "nnz_tokenizer_token: null argument");
  *n_out = 0;
  if (id >= tok->vocab_size || tok->id_to_vocab[id].empty())
    return fail(NNZ_EINVAL, "UnknownTokenId: " + std::to_string(id));
  const std::string& s = tok->id_to_vocab[id];
  if (s.size() > cap) return fail(NNZ_ERANGE, "OutputBufferTooSmall");
  memcpy(out, s.data(), s.size());
  *n_out = s.size();
  return NNZ_OK;
}

int nnz_tokenizer_token(const nnz_tokenizer* tok, uint32_t id, char* out, size_t cap, size_t* n_out) {
  return host_guard([&] { return tokenizer_token_impl(tok, id, out, cap, n_out); });
}

static int token_to_bytes_impl(const char* token, size_t len, char* out, size_t cap, size_t* n_out) {
  if (!n_out || (!token && len) || (!out && cap)) return fail(NNZ_EINVAL, "nnz_token_to_bytes: null argument");
  *n_out = 0;
  if (cap < len) return fail(NNZ_ERANGE, "OutputBufferTooSmall");
  if (len) *n_out = token_to_bytes(std::string(token, len), out);
  return NNZ_OK;
}

int nnz_token_to_bytes(const char* token, size_t len, char* out, size_t cap, size_t* n_out) {
  return host_guard([&] { return token_to_bytes_impl(token, len, out, cap, n_out); });
}

uint32_t nnz_pretoken_chunk(const char* text, size_t len) {
  if (!text || len == 0) return 0;
  const uint32_t n = len > kMaxInput ? (uint32_t)kMaxInput : (uint32_t)len;
  return pretoken_chunk(reinterpret_cast<const uint8_t*>(text), n);
}

}  // extern "C"
