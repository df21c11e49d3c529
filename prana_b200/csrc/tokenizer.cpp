// tokenizer.cpp -- the text side of prompt encoding and token decoding (host
// only): the SentencePiece-style greedy-BPE tokenizer (tokenizer.rs) and the
// GPT-2 byte-level BPE tokenizer (bpe.rs), built from piece lists or from a
// GGUF file's tokenizer metadata (gguf.rs:462-537).
//
// Text arrives as bytes.  Rust's callers hold `&str`, which is valid UTF-8 by
// construction; here invalid sequences are first replaced the way Rust's
// String::from_utf8_lossy does (one U+FFFD per maximal invalid subpart), and
// GGUF strings go through the same conversion, as the reference's loader does.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/prana_cuda.h"
#include "unicode_alpha.h"

namespace prana {
int fail(int code, const char* fmt, ...);
}
using prana::fail;

namespace {

// ------------------------------------------------------------------ UTF-8

// Length of the valid UTF-8 sequence at s[i..n), or 0 when the bytes there do
// not start one; *bad receives the length of the maximal invalid subpart.
size_t utf8_seq(const unsigned char* s, size_t i, size_t n, size_t* bad) {
  const unsigned char c = s[i];
  *bad = 1;
  if (c < 0x80) return 1;
  int need;
  unsigned char lo = 0x80, hi = 0xBF;
  if (c >= 0xC2 && c <= 0xDF) {
    need = 1;
  } else if (c >= 0xE0 && c <= 0xEF) {
    need = 2;
    if (c == 0xE0) lo = 0xA0;
    if (c == 0xED) hi = 0x9F;
  } else if (c >= 0xF0 && c <= 0xF4) {
    need = 3;
    if (c == 0xF0) lo = 0x90;
    if (c == 0xF4) hi = 0x8F;
  } else {
    return 0;  // 0x80..0xC1, 0xF5..0xFF: not a lead byte
  }
  for (int k = 1; k <= need; k++) {
    if (i + k >= n) {
      *bad = k;
      return 0;
    }
    const unsigned char b = s[i + k];
    const unsigned char l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
    if (b < l || b > h) {
      *bad = k;
      return 0;
    }
  }
  return (size_t)need + 1;
}

std::string lossy(const char* p, size_t n) {
  const unsigned char* s = reinterpret_cast<const unsigned char*>(p);
  std::string out;
  out.reserve(n);
  for (size_t i = 0; i < n;) {
    size_t bad;
    const size_t l = utf8_seq(s, i, n, &bad);
    if (l) {
      out.append(p + i, l);
      i += l;
    } else {
      out.append("\xEF\xBF\xBD");
      i += bad;
    }
  }
  return out;
}

// The code points of valid UTF-8 text, with each one's byte range.
struct Cp {
  uint32_t cp;
  size_t at, len;
};
std::vector<Cp> code_points(const std::string& t) {
  std::vector<Cp> out;
  const unsigned char* s = reinterpret_cast<const unsigned char*>(t.data());
  for (size_t i = 0; i < t.size();) {
    size_t bad;
    size_t l = utf8_seq(s, i, t.size(), &bad);
    if (!l) l = 1;  // not reached for text that went through lossy()
    uint32_t cp = s[i];
    if (l == 2) cp = ((s[i] & 0x1Fu) << 6) | (s[i + 1] & 0x3Fu);
    if (l == 3) cp = ((s[i] & 0x0Fu) << 12) | ((s[i + 1] & 0x3Fu) << 6) | (s[i + 2] & 0x3Fu);
    if (l == 4) cp = ((s[i] & 0x07u) << 18) | ((s[i + 1] & 0x3Fu) << 12) | ((s[i + 2] & 0x3Fu) << 6) | (s[i + 3] & 0x3Fu);
    out.push_back({cp, i, l});
    i += l;
  }
  return out;
}

std::string utf8_of(uint32_t cp) {
  std::string s;
  if (cp < 0x80) {
    s += (char)cp;
  } else if (cp < 0x800) {
    s += (char)(0xC0 | (cp >> 6));
    s += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    s += (char)(0xE0 | (cp >> 12));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  } else {
    s += (char)(0xF0 | (cp >> 18));
    s += (char)(0x80 | ((cp >> 12) & 0x3F));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  }
  return s;
}

bool is_letter(uint32_t cp) {
  int lo = 0, hi = prana::kAlphaRangeCount - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) / 2;
    if (cp < prana::kAlphaRanges[mid][0])
      hi = mid - 1;
    else if (cp > prana::kAlphaRanges[mid][1])
      lo = mid + 1;
    else
      return true;
  }
  return false;
}

// ------------------------------------------------------------------ SentencePiece-style (tokenizer.rs)

struct Spm {
  std::vector<std::string> vocab;  // piece bytes per id
  std::vector<float> scores;
  std::unordered_map<std::string, uint32_t> lookup;  // piece -> first id
  uint32_t bos = 1, eos = 2;
  bool add_bos = true;

  void index() {
    lookup.reserve(vocab.size());
    for (size_t i = 0; i < vocab.size(); i++) lookup.emplace(vocab[i], (uint32_t)i);
  }

  // Tokenizer::encode (tokenizer.rs:89-140): the dummy-space prefix, one seed
  // token per code point (byte fallback <0xNN> = byte + 3), then repeatedly
  // the adjacent pair whose concatenation scores highest (first on ties).
  std::vector<uint32_t> encode(const std::string& text, bool with_bos, bool with_eos) const {
    std::vector<uint32_t> t;
    if (with_bos) t.push_back(bos);
    if (!text.empty()) {
      auto it = lookup.find(" ");
      if (it != lookup.end()) t.push_back(it->second);
    }
    for (const Cp& c : code_points(text)) {
      const std::string piece = text.substr(c.at, c.len);
      auto it = lookup.find(piece);
      if (it != lookup.end()) {
        t.push_back(it->second);
      } else {
        for (unsigned char b : piece) t.push_back((uint32_t)b + 3);
      }
    }
    for (;;) {
      bool found = false;
      float best = 0.0f;
      size_t at = 0;
      uint32_t id = 0;
      for (size_t i = 0; i + 1 < t.size(); i++) {
        if (t[i] >= vocab.size() || t[i + 1] >= vocab.size()) continue;  // byte id past the vocab: never merges
        auto it = lookup.find(vocab[t[i]] + vocab[t[i + 1]]);
        if (it == lookup.end()) continue;
        const float s = scores[it->second];
        if (!found || s > best) {
          found = true;
          best = s;
          at = i;
          id = it->second;
        }
      }
      if (!found) break;
      t[at] = id;
      t.erase(t.begin() + (ptrdiff_t)at + 1);
    }
    if (with_eos) t.push_back(eos);
    return t;
  }

  // u8::from_str_radix(s, 16) on the two characters of "<0xNN>": an optional
  // '+' then hex digits, all of which must parse.
  static bool hex_byte(const char* p, uint8_t* out) {
    int i = 0, v = 0, digits = 0;
    if (p[0] == '+') i = 1;
    for (; i < 2; i++) {
      const char c = p[i];
      int d;
      if (c >= '0' && c <= '9')
        d = c - '0';
      else if (c >= 'a' && c <= 'f')
        d = c - 'a' + 10;
      else if (c >= 'A' && c <= 'F')
        d = c - 'A' + 10;
      else
        return false;
      v = v * 16 + d;
      digits++;
    }
    if (!digits) return false;
    *out = (uint8_t)v;
    return true;
  }

  // Tokenizer::decode (tokenizer.rs:144-160)
  std::string decode(uint32_t prev, uint32_t token) const {
    if (token >= vocab.size()) return std::string();
    const std::string& p = vocab[token];
    if (p.size() == 6 && p.compare(0, 3, "<0x") == 0 && p[5] == '>') {
      uint8_t b;
      if (hex_byte(p.data() + 3, &b)) return std::string(1, (char)b);
    }
    if (prev == bos && !p.empty() && p[0] == ' ') return p.substr(1);
    return p;
  }

  bool is_stop(uint32_t t) const { return t == eos || t == bos; }
};

// ------------------------------------------------------------------ byte-level BPE (bpe.rs)

struct PairHash {
  size_t operator()(const std::pair<std::string, std::string>& p) const {
    return std::hash<std::string>()(p.first) * 1000003u ^ std::hash<std::string>()(p.second);
  }
};

struct Bpe {
  std::vector<std::string> vocab;  // strings over the byte alphabet
  std::unordered_map<std::string, uint32_t> lookup;
  std::unordered_map<std::pair<std::string, std::string>, uint32_t, PairHash> ranks;
  std::string byte_enc[256];                     // byte -> its mapped character (UTF-8)
  std::unordered_map<uint32_t, uint8_t> byte_dec;  // mapped code point -> byte
  int64_t bos = -1, eos = -1;
  bool add_bos = false;
  std::vector<std::pair<std::string, uint32_t>> specials;  // longest first

  // bytes_to_unicode (bpe.rs:23-36): printable bytes map to themselves, the
  // rest to 256 + n in byte order.
  void alphabet() {
    uint32_t n = 0;
    for (uint32_t b = 0; b < 256; b++) {
      const bool printable = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
      const uint32_t cp = printable ? b : 256 + n++;
      byte_enc[b] = utf8_of(cp);
      byte_dec[cp] = (uint8_t)b;
    }
  }

  // BpeTokenizer::new (bpe.rs:57-77): first id per string; merges "left right"
  // split at the first space, a repeated pair keeping its last rank.
  void index(const std::vector<std::string>& merges) {
    lookup.reserve(vocab.size());
    for (size_t i = 0; i < vocab.size(); i++) lookup.emplace(vocab[i], (uint32_t)i);
    for (size_t r = 0; r < merges.size(); r++) {
      const size_t sp = merges[r].find(' ');
      if (sp == std::string::npos) continue;
      ranks[{merges[r].substr(0, sp), merges[r].substr(sp + 1)}] = (uint32_t)r;
    }
    alphabet();
  }

  // pre_tokenize (bpe.rs:95-132): pieces that keep one leading space, split
  // where the character class changes.
  enum Class { LETTER, DIGIT, OTHER, SPACE };
  static std::vector<std::string> pre_tokenize(const std::string& text) {
    std::vector<std::string> pieces;
    std::string cur;
    Class cur_class = SPACE;
    for (const Cp& c : code_points(text)) {
      const Class cl = is_letter(c.cp) ? LETTER : (c.cp >= '0' && c.cp <= '9') ? DIGIT : c.cp == ' ' ? SPACE : OTHER;
      bool starts_new;
      if (cur.empty())
        starts_new = false;
      else if (cur == " " && cl != SPACE)
        starts_new = false;  // a single pending space attaches to the next word
      else
        starts_new = cl != cur_class;
      if (starts_new || (cl == SPACE && !cur.empty() && cur.back() != ' ')) {
        pieces.push_back(cur);
        cur.clear();
      }
      cur.append(text, c.at, c.len);
      cur_class = cl;
    }
    if (!cur.empty()) pieces.push_back(cur);
    return pieces;
  }

  // bpe_piece (bpe.rs:135-162): one mapped symbol per byte, then the
  // lowest-ranked adjacent merge (first on ties) until none applies; symbols
  // missing from the vocab are dropped.
  void piece(const std::string& p, std::vector<uint32_t>* out) const {
    std::vector<std::string> sym;
    sym.reserve(p.size());
    for (unsigned char b : p) sym.push_back(byte_enc[b]);
    for (;;) {
      bool found = false;
      uint32_t best = 0;
      size_t at = 0;
      for (size_t i = 0; i + 1 < sym.size(); i++) {
        auto it = ranks.find({sym[i], sym[i + 1]});
        if (it != ranks.end() && (!found || it->second < best)) {
          found = true;
          best = it->second;
          at = i;
        }
      }
      if (!found) break;
      sym[at] += sym[at + 1];
      sym.erase(sym.begin() + (ptrdiff_t)at + 1);
    }
    for (const std::string& s : sym) {
      auto it = lookup.find(s);
      if (it != lookup.end()) out->push_back(it->second);
    }
  }

  // encode_prompt (bpe.rs:166-192): specials matched verbatim at their
  // earliest position (the longest one where several start there), BPE on
  // the text between them.
  std::vector<uint32_t> encode(const std::string& text) const {
    std::vector<uint32_t> out;
    if (add_bos && bos >= 0) out.push_back((uint32_t)bos);
    size_t pos = 0;
    while (pos < text.size()) {
      size_t best_at = std::string::npos, best_len = 0;
      uint32_t best_id = 0;
      for (const auto& s : specials) {
        const size_t at = text.find(s.first, pos);
        if (at != std::string::npos && (best_at == std::string::npos || at < best_at)) {
          best_at = at;
          best_len = s.first.size();
          best_id = s.second;
        }
      }
      const size_t end = best_at == std::string::npos ? text.size() : best_at;
      for (const std::string& p : pre_tokenize(text.substr(pos, end - pos))) piece(p, &out);
      if (best_at == std::string::npos) break;
      out.push_back(best_id);
      pos = best_at + best_len;
    }
    return out;
  }

  // decode (bpe.rs:194-199): the bytes behind the token's mapped characters
  std::string decode(uint32_t token) const {
    if (token >= vocab.size()) return std::string();
    std::string out;
    for (const Cp& c : code_points(vocab[token])) {
      auto it = byte_dec.find(c.cp);
      if (it != byte_dec.end()) out += (char)it->second;
    }
    return out;
  }

  bool is_stop(uint32_t t) const { return (eos >= 0 && t == (uint32_t)eos) || (bos >= 0 && t == (uint32_t)bos); }
};

// ------------------------------------------------------------------ GGUF metadata (gguf.rs value types 0..12)

struct Val {
  int type = -1;
  int64_t i = 0;
  bool neg = false;  // a signed integer below zero
  double f = 0.0;
  bool b = false;
  std::string s;
  std::vector<Val> arr;
};

struct MetaReader {
  std::vector<char> buf;
  size_t off = 0;
  bool rd(void* d, size_t n) {
    if (off + n > buf.size()) return false;
    memcpy(d, buf.data() + off, n);
    off += n;
    return true;
  }
  bool str(std::string* s) {
    uint64_t n;
    if (!rd(&n, 8) || n > buf.size() - off) return false;
    s->assign(buf.data() + off, n);
    off += n;
    return true;
  }
  bool value(uint32_t ty, Val* v) {
    v->type = (int)ty;
    switch (ty) {
      case 0: { uint8_t x; if (!rd(&x, 1)) return false; v->i = x; return true; }
      case 1: { int8_t x; if (!rd(&x, 1)) return false; v->i = x; v->neg = x < 0; return true; }
      case 2: { uint16_t x; if (!rd(&x, 2)) return false; v->i = x; return true; }
      case 3: { int16_t x; if (!rd(&x, 2)) return false; v->i = x; v->neg = x < 0; return true; }
      case 4: { uint32_t x; if (!rd(&x, 4)) return false; v->i = x; return true; }
      case 5: { int32_t x; if (!rd(&x, 4)) return false; v->i = x; v->neg = x < 0; return true; }
      case 6: { float x; if (!rd(&x, 4)) return false; v->f = x; return true; }
      case 7: { uint8_t x; if (!rd(&x, 1)) return false; v->b = x != 0; return true; }
      case 8: return str(&v->s);
      case 9: {
        uint32_t et;
        uint64_t n;
        if (!rd(&et, 4) || !rd(&n, 8) || n > buf.size()) return false;
        v->arr.resize(n);
        for (uint64_t k = 0; k < n; k++)
          if (!value(et, &v->arr[k])) return false;
        return true;
      }
      case 10: { uint64_t x; if (!rd(&x, 8)) return false; v->i = (int64_t)x; v->neg = false; return true; }
      case 11: { int64_t x; if (!rd(&x, 8)) return false; v->i = x; v->neg = x < 0; return true; }
      case 12: { double x; if (!rd(&x, 8)) return false; v->f = x; return true; }
    }
    return false;
  }
};

// Value::as_usize / as_f32 (gguf.rs:64-84)
bool as_usize(const Val& v, uint64_t* out) {
  if (v.type < 0 || v.type == 6 || v.type == 7 || v.type == 8 || v.type == 9 || v.type == 12 || v.neg) return false;
  *out = (uint64_t)v.i;
  return true;
}
float as_f32_or0(const Val& v) { return v.type == 6 || v.type == 12 ? (float)v.f : 0.0f; }

std::string replace_all(std::string s, const std::string& from, const std::string& to) {
  for (size_t at = s.find(from); at != std::string::npos; at = s.find(from, at + to.size())) s.replace(at, from.size(), to);
  return s;
}

}  // namespace

struct prana_tokenizer {
  std::unique_ptr<Spm> spm;
  std::unique_ptr<Bpe> bpe;
};

#define TOK_BEGIN try {
#define TOK_END                                                    \
  }                                                                \
  catch (const std::bad_alloc&) {                                  \
    return fail(PRANA_E_OOM, "host allocation failed");            \
  }                                                                \
  catch (...) {                                                    \
    return fail(PRANA_E_INVALID, "unexpected host exception");     \
  }

static int put_ids(const std::vector<uint32_t>& ids, uint32_t* out, size_t cap, size_t* n_out) {
  *n_out = ids.size();
  if (ids.size() > cap) return fail(PRANA_E_INVALID, "%zu token ids do not fit the output (capacity %zu)", ids.size(), cap);
  if (!ids.empty()) memcpy(out, ids.data(), ids.size() * 4);
  return PRANA_OK;
}

extern "C" {

int prana_tokenizer_spm(size_t n, const char* const* pieces, const size_t* lens, const float* scores, uint32_t bos,
                        uint32_t eos, int add_bos, prana_tokenizer** out) {
  TOK_BEGIN
  if (!out || (n && (!pieces || !lens || !scores))) return fail(PRANA_E_INVALID, "null argument");
  auto t = std::make_unique<prana_tokenizer>();
  t->spm = std::make_unique<Spm>();
  for (size_t i = 0; i < n; i++) {
    t->spm->vocab.emplace_back(pieces[i], lens[i]);
    t->spm->scores.push_back(scores[i]);
  }
  t->spm->bos = bos;
  t->spm->eos = eos;
  t->spm->add_bos = add_bos != 0;
  t->spm->index();
  *out = t.release();
  return PRANA_OK;
  TOK_END
}

int prana_tokenizer_bpe(size_t n, const char* const* pieces, const size_t* lens, size_t n_merges,
                        const char* const* merges, const size_t* merge_lens, size_t n_specials,
                        const uint32_t* special_ids, int64_t bos, int64_t eos, int add_bos, prana_tokenizer** out) {
  TOK_BEGIN
  if (!out || (n && (!pieces || !lens)) || (n_merges && (!merges || !merge_lens)) || (n_specials && !special_ids))
    return fail(PRANA_E_INVALID, "null argument");
  auto t = std::make_unique<prana_tokenizer>();
  t->bpe = std::make_unique<Bpe>();
  Bpe& b = *t->bpe;
  for (size_t i = 0; i < n; i++) b.vocab.push_back(lossy(pieces[i], lens[i]));
  std::vector<std::string> m;
  for (size_t i = 0; i < n_merges; i++) m.push_back(lossy(merges[i], merge_lens[i]));
  b.index(m);
  for (size_t i = 0; i < n_specials; i++) {  // (empty specials skipped: they would never advance)
    if (special_ids[i] >= n) return fail(PRANA_E_INVALID, "special token id %u beyond the vocabulary", special_ids[i]);
    if (!b.vocab[special_ids[i]].empty()) b.specials.emplace_back(b.vocab[special_ids[i]], special_ids[i]);
  }
  // with_specials (bpe.rs:79-84): longest first, a stable sort
  std::stable_sort(b.specials.begin(), b.specials.end(),
                   [](const auto& x, const auto& y) { return x.first.size() > y.first.size(); });
  b.bos = bos;
  b.eos = eos;
  b.add_bos = add_bos != 0;
  *out = t.release();
  return PRANA_OK;
  TOK_END
}

// load_tokenizer (gguf.rs:462-537)
int prana_tokenizer_load_gguf(const char* path, prana_tokenizer** out) {
  TOK_BEGIN
  if (!path || !out) return fail(PRANA_E_INVALID, "null argument");
  MetaReader r;
  {
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail(PRANA_E_INVALID, "cannot open '%s'", path);
    r.buf.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  }
  uint32_t magic = 0, ver = 0;
  uint64_t nt = 0, nkv = 0;
  if (!r.rd(&magic, 4) || magic != 0x46554747u) return fail(PRANA_E_FORMAT, "not a GGUF file (bad magic)");
  if (!r.rd(&ver, 4) || ver < 2 || ver > 3) return fail(PRANA_E_FORMAT, "unsupported GGUF version %u", ver);
  if (!r.rd(&nt, 8) || !r.rd(&nkv, 8)) return fail(PRANA_E_FORMAT, "gguf truncated");
  std::map<std::string, Val> meta;
  for (uint64_t i = 0; i < nkv; i++) {
    std::string key;
    uint32_t ty;
    Val v;
    if (!r.str(&key) || !r.rd(&ty, 4) || !r.value(ty, &v)) return fail(PRANA_E_FORMAT, "gguf metadata truncated");
    if (key.rfind("tokenizer.ggml.", 0) == 0) meta[key] = std::move(v);
  }
  auto get = [&](const char* k) -> const Val* {
    auto it = meta.find(k);
    return it == meta.end() ? nullptr : &it->second;
  };
  const Val* tokens = get("tokenizer.ggml.tokens");
  if (!tokens || tokens->type != 9) return fail(PRANA_E_FORMAT, "missing tokenizer.ggml.tokens");
  const Val* mv = get("tokenizer.ggml.model");
  const std::string model = mv && mv->type == 8 ? lossy(mv->s.data(), mv->s.size()) : std::string("llama");
  uint64_t bos = 0, eos = 0;
  const bool has_bos = get("tokenizer.ggml.bos_token_id") && as_usize(*get("tokenizer.ggml.bos_token_id"), &bos);
  const bool has_eos = get("tokenizer.ggml.eos_token_id") && as_usize(*get("tokenizer.ggml.eos_token_id"), &eos);
  const Val* ab = get("tokenizer.ggml.add_bos_token");
  const bool add_bos = ab && ab->type == 7 ? ab->b : model == "llama";
  auto strings = [&](const Val& arr) {
    std::vector<std::string> v;
    for (const Val& x : arr.arr) v.push_back(x.type == 8 ? lossy(x.s.data(), x.s.size()) : std::string());
    return v;
  };
  auto t = std::make_unique<prana_tokenizer>();
  if (model == "llama") {
    t->spm = std::make_unique<Spm>();
    Spm& s = *t->spm;
    for (std::string& p : strings(*tokens)) s.vocab.push_back(replace_all(p, "\xE2\x96\x81", " "));  // U+2581 -> space
    const Val* sc = get("tokenizer.ggml.scores");
    if (sc && sc->type == 9) {
      // Tokenizer::from_parts asserts one score per piece (tokenizer.rs:52)
      if (sc->arr.size() != s.vocab.size())
        return fail(PRANA_E_FORMAT, "%zu scores for %zu tokens", sc->arr.size(), s.vocab.size());
      for (const Val& x : sc->arr) s.scores.push_back(as_f32_or0(x));
    } else {
      s.scores.assign(s.vocab.size(), 0.0f);  // no scores: all 0.0
    }
    s.bos = has_bos ? (uint32_t)bos : 1u;
    s.eos = has_eos ? (uint32_t)eos : 2u;
    s.add_bos = add_bos;
    s.index();
  } else if (model == "gpt2") {
    const Val* mg = get("tokenizer.ggml.merges");
    if (!mg || mg->type != 9) return fail(PRANA_E_FORMAT, "gpt2 tokenizer requires tokenizer.ggml.merges");
    t->bpe = std::make_unique<Bpe>();
    Bpe& b = *t->bpe;
    b.vocab = strings(*tokens);
    b.index(strings(*mg));
    // token_type 3 (CONTROL) / 4 (USER_DEFINED): encoded verbatim
    // (an empty special would match everywhere and never advance: skipped)
    const Val* tt = get("tokenizer.ggml.token_type");
    if (tt && tt->type == 9 && tt->arr.size() > b.vocab.size())
      return fail(PRANA_E_FORMAT, "%zu token types for %zu tokens", tt->arr.size(), b.vocab.size());
    if (tt && tt->type == 9)
      for (size_t id = 0; id < tt->arr.size(); id++) {
        uint64_t k;
        if (as_usize(tt->arr[id], &k) && (k == 3 || k == 4) && !b.vocab[id].empty())
          b.specials.emplace_back(b.vocab[id], (uint32_t)id);
      }
    std::stable_sort(b.specials.begin(), b.specials.end(),
                     [](const auto& x, const auto& y) { return x.first.size() > y.first.size(); });
    b.bos = has_bos ? (int64_t)bos : -1;
    b.eos = has_eos ? (int64_t)eos : -1;
    b.add_bos = add_bos;
  } else {
    return fail(PRANA_E_UNSUPPORTED, "unsupported tokenizer.ggml.model '%s'", model.c_str());
  }
  *out = t.release();
  return PRANA_OK;
  TOK_END
}

int prana_tokenizer_free(prana_tokenizer* t) {
  delete t;
  return PRANA_OK;
}

int prana_tokenizer_vocab_size(const prana_tokenizer* t, size_t* out) {
  if (!t || !out) return fail(PRANA_E_INVALID, "null argument");
  *out = t->spm ? t->spm->vocab.size() : t->bpe->vocab.size();
  return PRANA_OK;
}

int prana_tokenize(const prana_tokenizer* t, const char* text, size_t len, int bos, int eos, uint32_t* ids,
                   size_t cap, size_t* n_out) {
  TOK_BEGIN
  if (!t || (len && !text) || !n_out || (cap && !ids)) return fail(PRANA_E_INVALID, "null argument");
  const std::string s = lossy(text ? text : "", len);
  if (t->spm) return put_ids(t->spm->encode(s, bos < 0 ? t->spm->add_bos : bos != 0, eos > 0), ids, cap, n_out);
  if (bos >= 0 || eos > 0) return fail(PRANA_E_INVALID, "the byte-level BPE tokenizer takes its BOS from the model (pass -1, 0)");
  return put_ids(t->bpe->encode(s), ids, cap, n_out);
  TOK_END
}

int prana_detokenize(const prana_tokenizer* t, uint32_t prev, uint32_t token, char* out, size_t cap, size_t* n_out) {
  TOK_BEGIN
  if (!t || !n_out || (cap && !out)) return fail(PRANA_E_INVALID, "null argument");
  const std::string s = t->spm ? t->spm->decode(prev, token) : t->bpe->decode(token);
  *n_out = s.size();
  if (s.size() > cap) return fail(PRANA_E_INVALID, "%zu bytes do not fit the output (capacity %zu)", s.size(), cap);
  if (!s.empty()) memcpy(out, s.data(), s.size());
  return PRANA_OK;
  TOK_END
}

int prana_tokenizer_is_stop(const prana_tokenizer* t, uint32_t token, int* out) {
  if (!t || !out) return fail(PRANA_E_INVALID, "null argument");
  *out = t->spm ? t->spm->is_stop(token) : t->bpe->is_stop(token);
  return PRANA_OK;
}

}  // extern "C"
