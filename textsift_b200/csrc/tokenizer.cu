// tokenizer.cu — host-side o200k-style byte-level BPE tokenizer (C ABI
// ts_tok_*), the native counterpart of textsift's Tokenizer
// (packages/textsift/src/browser/model/tokenizer.ts).  Same output as the
// reference's encode(): token ids and tokenToCharOffset in UTF-16 code units
// (plus UTF-8 byte offsets), for UTF-8 input.
//
// Pipeline per text (tokenizer.ts:238-291): split around special-token
// literals (the first literal, in the reference's order, that matches at the
// leftmost position); pretokenize each other slice with the reference's
// pattern (tokenizer.ts:510-525) in "isolated" mode (matches and the gaps
// between them are pieces); BPE each piece's UTF-8 bytes with the merge
// ranks (lowest rank first, all occurrences of the chosen pair merged in one
// left-to-right pass, tokenizer.ts:413-458); spread the piece's UTF-16 span
// over its tokens by their byte lengths (tokenizer.ts:467-504).
//
// The pretokenizer is a hand-written matcher, not a regex engine: for each
// alternative of the pattern it returns the match the reference's
// backtracking regex returns (leftmost start, first alternative that
// matches, greedy quantifiers backtracked in order).  Unicode classes come
// from unicode_classes.inc (gen_unicode_classes.py); \s is JavaScript's set.
// BPE runs on interned byte strings; results are cached per piece.
#include "textsift_cuda.h"
#include "ts_simt.h"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace {

// ------------------------------------------------------------------ classes
enum : uint8_t { kLu = 1, kLl = 2, kLt = 4, kLm = 8, kLo = 16, kMark = 32, kNum = 64, kSpace = 128 };
constexpr uint8_t kLetter = kLu | kLl | kLt | kLm | kLo;
constexpr uint8_t kUpperish = kLu | kLt | kLm | kLo | kMark;  // [\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}]
constexpr uint8_t kLowerish = kLl | kLm | kLo | kMark;        // [\p{Ll}\p{Lm}\p{Lo}\p{M}]

struct ClassRange {
  uint32_t lo, hi;
  uint8_t bits;
};
const ClassRange kRanges[] = {
#include "unicode_classes.inc"
};

struct ClassTable {
  uint8_t bmp[0x10000];
  ClassTable() {
    std::memset(bmp, 0, sizeof(bmp));
    for (const ClassRange& r : kRanges)
      for (uint32_t c = r.lo; c <= r.hi && c < 0x10000u; c++) bmp[c] = r.bits;
  }
  uint8_t get(uint32_t c) const {
    if (c < 0x10000u) return bmp[c];
    size_t lo = 0, hi = sizeof(kRanges) / sizeof(kRanges[0]);
    while (lo < hi) {
      const size_t mid = (lo + hi) / 2;
      if (kRanges[mid].hi < c) lo = mid + 1;
      else hi = mid;
    }
    return lo < sizeof(kRanges) / sizeof(kRanges[0]) && kRanges[lo].lo <= c ? kRanges[lo].bits : 0;
  }
};
const ClassTable& classes() {
  static const ClassTable t;
  return t;
}

// ------------------------------------------------------------------- JSON
// Enough of JSON for tokenizer.json: objects, arrays, strings (all escapes,
// surrogate pairs to UTF-8), numbers, literals.
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const char* k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonParser {
  const char* p;
  const char* end;
  std::string err;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  static void put_utf8(std::string& s, uint32_t c) {
    if (c < 0x80) s += (char)c;
    else if (c < 0x800) { s += (char)(0xC0 | (c >> 6)); s += (char)(0x80 | (c & 63)); }
    else if (c < 0x10000) { s += (char)(0xE0 | (c >> 12)); s += (char)(0x80 | ((c >> 6) & 63)); s += (char)(0x80 | (c & 63)); }
    else {
      s += (char)(0xF0 | (c >> 18)); s += (char)(0x80 | ((c >> 12) & 63));
      s += (char)(0x80 | ((c >> 6) & 63)); s += (char)(0x80 | (c & 63));
    }
  }
  bool hex4(uint32_t& v) {
    if (end - p < 4) return fail("truncated \\u escape");
    v = 0;
    for (int i = 0; i < 4; i++) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    return true;
  }
  bool string(std::string& s) {
    if (p >= end || *p != '"') return fail("expected string");
    p++;
    while (p < end && *p != '"') {
      if (*p != '\\') { s += *p++; continue; }
      if (++p >= end) return fail("truncated escape");
      const char c = *p++;
      switch (c) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t v;
          if (!hex4(v)) return false;
          if (v >= 0xD800 && v <= 0xDBFF && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            const char* save = p;
            p += 2;
            uint32_t lo;
            if (!hex4(lo)) return false;
            if (lo >= 0xDC00 && lo <= 0xDFFF) v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
            else p = save;  // lone high surrogate: keep as is
          }
          put_utf8(s, v);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p >= end) return fail("unterminated string");
    p++;
    return true;
  }
  bool value(Json& v, int depth) {
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (p >= end) return fail("unexpected end");
    const char c = *p;
    if (c == '{') {
      v.kind = Json::Obj;
      p++;
      ws();
      if (p < end && *p == '}') { p++; return true; }
      while (true) {
        ws();
        std::string k;
        if (!string(k)) return false;
        ws();
        if (p >= end || *p != ':') return fail("expected ':'");
        p++;
        v.obj.emplace_back(std::move(k), Json());
        if (!value(v.obj.back().second, depth + 1)) return false;
        ws();
        if (p < end && *p == ',') { p++; continue; }
        if (p < end && *p == '}') { p++; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::Arr;
      p++;
      ws();
      if (p < end && *p == ']') { p++; return true; }
      while (true) {
        v.arr.emplace_back();
        if (!value(v.arr.back(), depth + 1)) return false;
        ws();
        if (p < end && *p == ',') { p++; continue; }
        if (p < end && *p == ']') { p++; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::Str;
      return string(v.str);
    }
    if (c == 't' || c == 'f' || c == 'n') {
      const char* w = c == 't' ? "true" : (c == 'f' ? "false" : "null");
      const size_t n = std::strlen(w);
      if ((size_t)(end - p) < n || std::strncmp(p, w, n) != 0) return fail("bad literal");
      p += n;
      v.kind = c == 'n' ? Json::Null : Json::Bool;
      v.b = c == 't';
      return true;
    }
    char* q = nullptr;
    std::string num;
    while (p < end && (std::strchr("+-0123456789.eE", *p) != nullptr)) num += *p++;
    if (num.empty()) return fail("unexpected character");
    v.kind = Json::Num;
    v.num = std::strtod(num.c_str(), &q);
    return true;
  }
};

// ------------------------------------------------------------------ UTF-8
// Decodes valid UTF-8 into code points with their byte offsets; false on
// malformed input (overlong forms, surrogates, values above U+10FFFF).
bool decode_utf8(const uint8_t* s, size_t n, std::vector<uint32_t>& cps, std::vector<uint32_t>& boff) {
  cps.clear();
  boff.clear();
  size_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    uint32_t cp, len;
    if (c < 0x80) { cp = c; len = 1; }
    else if ((c & 0xE0) == 0xC0) { cp = c & 0x1F; len = 2; }
    else if ((c & 0xF0) == 0xE0) { cp = c & 0x0F; len = 3; }
    else if ((c & 0xF8) == 0xF0) { cp = c & 0x07; len = 4; }
    else return false;
    if (i + len > n) return false;
    for (uint32_t k = 1; k < len; k++) {
      if ((s[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (s[i + k] & 0x3F);
    }
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) || cp > 0x10FFFF ||
        (cp >= 0xD800 && cp <= 0xDFFF))
      return false;
    cps.push_back(cp);
    boff.push_back((uint32_t)i);
    i += len;
  }
  boff.push_back((uint32_t)n);
  return true;
}

// GPT-2's bytes_to_unicode (tokenizer.ts:488-507): byte -> printable code point.
void byte_map(uint32_t (&b2c)[256]) {
  bool direct[256] = {};
  for (uint32_t b = '!'; b <= '~'; b++) direct[b] = true;
  for (uint32_t b = 0xA1; b <= 0xAC; b++) direct[b] = true;
  for (uint32_t b = 0xAE; b <= 0xFF; b++) direct[b] = true;
  uint32_t n = 0;
  for (uint32_t b = 0; b < 256; b++) b2c[b] = direct[b] ? b : 256 + n++;
}

// ------------------------------------------------------------------- model
struct Model {
  uint32_t b2c[256];
  std::unordered_map<uint32_t, uint8_t> c2b;
  std::unordered_map<std::string, int32_t> sym_index;  // byte string -> symbol
  std::vector<std::string> sym_bytes;
  std::vector<int32_t> sym_vocab;                      // symbol -> vocab id, -1 if none
  int32_t byte_sym[256];
  std::unordered_map<uint64_t, uint64_t> merges;       // (a << 32 | b) -> (rank << 32 | merged symbol)
  std::vector<std::string> id_bytes;                   // vocab id -> bytes it decodes to
  std::vector<uint32_t> id_u16;                        // vocab id -> UTF-16 length of its vocab string
  std::vector<uint8_t> id_special, id_known;
  std::vector<std::pair<std::string, int32_t>> specials;  // in the reference's matching order

  int32_t intern(const std::string& b) {
    auto it = sym_index.find(b);
    if (it != sym_index.end()) return it->second;
    const int32_t s = (int32_t)sym_bytes.size();
    sym_index.emplace(b, s);
    sym_bytes.push_back(b);
    return s;
  }
  // a vocab string of byte-mapped characters -> the bytes (false if a
  // character is outside the byte map)
  bool unmap(const std::string& utf8, std::string& out) const {
    std::vector<uint32_t> cps, bo;
    if (!decode_utf8(reinterpret_cast<const uint8_t*>(utf8.data()), utf8.size(), cps, bo)) return false;
    out.clear();
    for (uint32_t c : cps) {
      auto it = c2b.find(c);
      if (it == c2b.end()) return false;
      out += (char)it->second;
    }
    return true;
  }
  std::string map_bytes(const std::string& b) const {
    std::string s;
    for (unsigned char c : b) JsonParser::put_utf8(s, b2c[c]);
    return s;
  }
};

uint32_t u16_length(const std::string& utf8) {
  std::vector<uint32_t> cps, bo;
  if (!decode_utf8(reinterpret_cast<const uint8_t*>(utf8.data()), utf8.size(), cps, bo)) return (uint32_t)utf8.size();
  uint32_t n = 0;
  for (uint32_t c : cps) n += c > 0xFFFF ? 2u : 1u;
  return n;
}

// Builds the model from tokenizer.json (Tokenizer.fromBundle, tokenizer.ts:134-221).
bool load_model(Model& m, const char* text, size_t len, std::string& err) {
  JsonParser jp{text, text + len, {}};
  Json root;
  if (!jp.value(root, 0)) { err = "tokenizer.json: " + jp.err; return false; }
  const Json* model = root.get("model");
  const Json* type = model ? model->get("type") : nullptr;
  if (!type || type->kind != Json::Str || type->str != "BPE") { err = "tokenizer.json: model.type must be \"BPE\""; return false; }
  const Json* vocab = model->get("vocab");
  const Json* merges = model->get("merges");
  if (!vocab || vocab->kind != Json::Obj || !merges || merges->kind != Json::Arr) {
    err = "tokenizer.json: model.vocab (object) and model.merges (array) are required";
    return false;
  }
  byte_map(m.b2c);
  for (uint32_t b = 0; b < 256; b++) m.c2b[m.b2c[b]] = (uint8_t)b;
  // vocab then added tokens, later entries overriding (a Map built in that order)
  std::unordered_map<std::string, int32_t> by_str;
  std::vector<std::pair<std::string, int32_t>> order;
  int32_t max_id = -1;
  auto add = [&](const std::string& s, double idd) -> bool {
    if (idd < 0 || idd > 0x7fffffff || idd != (double)(int64_t)idd) return false;
    const int32_t id = (int32_t)idd;
    by_str[s] = id;
    order.emplace_back(s, id);
    max_id = std::max(max_id, id);
    return true;
  };
  for (const auto& kv : vocab->obj)
    if (kv.second.kind != Json::Num || !add(kv.first, kv.second.num)) { err = "tokenizer.json: bad vocab id for " + kv.first; return false; }
  std::vector<std::pair<std::string, int32_t>> special_list;
  if (const Json* added = root.get("added_tokens")) {
    if (added->kind != Json::Arr) { err = "tokenizer.json: added_tokens must be an array"; return false; }
    for (const Json& t : added->arr) {
      const Json* id = t.get("id");
      const Json* content = t.get("content");
      const Json* special = t.get("special");
      if (!id || id->kind != Json::Num || !content || content->kind != Json::Str || !add(content->str, id->num)) {
        err = "tokenizer.json: bad added token";
        return false;
      }
      if (special && special->kind == Json::Bool && special->b) special_list.emplace_back(content->str, (int32_t)id->num);
    }
  }
  m.id_bytes.assign((size_t)max_id + 1, std::string());
  m.id_u16.assign((size_t)max_id + 1, 0u);
  m.id_special.assign((size_t)max_id + 1, 0u);
  m.id_known.assign((size_t)max_id + 1, 0u);
  for (const auto& sp : special_list) m.id_special[sp.second] = 1;
  // id -> its string: the last string inserted with that id (idToToken)
  for (const auto& e : order) {
    const std::string& s = e.first;
    const int32_t id = e.second;
    m.id_known[id] = 1;
    m.id_u16[id] = u16_length(s);
    std::string b;
    if (m.id_special[id] || !m.unmap(s, b)) {
      if (m.id_special[id]) { m.id_bytes[id] = s; continue; }
      // characters outside the byte map decode to their own UTF-8 (tokenizer.ts:320-330)
      std::vector<uint32_t> cps, bo;
      b.clear();
      decode_utf8(reinterpret_cast<const uint8_t*>(s.data()), s.size(), cps, bo);
      for (uint32_t c : cps) {
        auto it = m.c2b.find(c);
        if (it != m.c2b.end()) b += (char)it->second;
        else JsonParser::put_utf8(b, c);
      }
    }
    m.id_bytes[id] = b;
  }
  for (uint32_t b = 0; b < 256; b++) m.byte_sym[b] = m.intern(std::string(1, (char)b));
  for (size_t i = 0; i < merges->arr.size(); i++) {
    const Json& e = merges->arr[i];
    std::string a, b;
    if (e.kind == Json::Arr && e.arr.size() == 2 && e.arr[0].kind == Json::Str && e.arr[1].kind == Json::Str) {
      a = e.arr[0].str;
      b = e.arr[1].str;
    } else if (e.kind == Json::Str && e.str.find(' ') != std::string::npos) {
      a = e.str.substr(0, e.str.find(' '));
      b = e.str.substr(e.str.find(' ') + 1);
    } else {
      err = "tokenizer.json: merges entries must be [a, b] pairs";
      return false;
    }
    std::string ab, bb;
    if (!m.unmap(a, ab) || !m.unmap(b, bb)) continue;  // never adjacent byte-level symbols
    const int32_t sa = m.intern(ab), sb = m.intern(bb), sm = m.intern(ab + bb);
    m.merges[((uint64_t)(uint32_t)sa << 32) | (uint32_t)sb] = ((uint64_t)i << 32) | (uint32_t)sm;  // last rank wins
  }
  m.sym_vocab.assign(m.sym_bytes.size(), -1);
  for (size_t s = 0; s < m.sym_bytes.size(); s++) {
    auto it = by_str.find(m.map_bytes(m.sym_bytes[s]));
    if (it != by_str.end()) m.sym_vocab[s] = it->second;
  }
  // specials: regex-escaped literals sorted (stably) by descending length (tokenizer.ts:190-204)
  auto escaped_len = [](const std::string& s) {
    uint32_t n = u16_length(s);
    for (char c : s)
      if (std::strchr(".*+?^${}()|[]\\", c) != nullptr && c != 0) n++;
    return n;
  };
  std::stable_sort(special_list.begin(), special_list.end(),
                   [&](const auto& x, const auto& y) { return escaped_len(x.first) > escaped_len(y.first); });
  m.specials = special_list;
  return true;
}

// ------------------------------------------------------------- pretokenizer
// The reference's pattern (tokenizer.ts:510-525), alternative by alternative;
// each returns the end of the match at s, or -1.
struct Pre {
  const uint32_t* cp;
  const uint8_t* cl;
  size_t n;
  bool crlf(size_t i) const { return cp[i] == '\r' || cp[i] == '\n'; }
  bool not_crlf_l_n(size_t i) const { return !crlf(i) && !(cl[i] & (kLetter | kNum)); }  // [^\r\n\p{L}\p{N}]
  bool not_s_l_n(size_t i) const { return !(cl[i] & (kSpace | kLetter | kNum)); }        // [^\s\p{L}\p{N}]
  size_t run(size_t i, uint8_t mask) const {
    size_t j = i;
    while (j < n && (cl[j] & mask)) j++;
    return j - i;
  }
  // (?i:'s|'t|'re|'ve|'m|'ll|'d)? at i (ASCII case folding only)
  size_t contraction(size_t i) const {
    if (i + 1 >= n || cp[i] != '\'') return 0;
    auto lc = [&](size_t k) { const uint32_t c = cp[k]; return (c >= 'A' && c <= 'Z') ? c + 32 : c; };
    const uint32_t a = lc(i + 1);
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
    if (i + 2 < n) {
      const uint32_t b = lc(i + 2);
      if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
    }
    return 0;
  }
  // [^\r\n\p{L}\p{N}]?[upper-ish]*[lower-ish]+(contraction)?
  long alt1(size_t s) const {
    for (int pre = 1; pre >= 0; pre--) {
      if (pre && !(s < n && not_crlf_l_n(s))) continue;
      const size_t p = s + (size_t)pre;
      const size_t umax = run(p, kUpperish);
      for (size_t u = umax + 1; u-- > 0;) {
        const size_t q = p + u;
        if (q < n && (cl[q] & kLowerish)) {
          const size_t e = q + run(q, kLowerish);
          return (long)(e + contraction(e));
        }
      }
    }
    return -1;
  }
  // [^\r\n\p{L}\p{N}]?[upper-ish]+[lower-ish]*(contraction)?
  long alt2(size_t s) const {
    for (int pre = 1; pre >= 0; pre--) {
      if (pre && !(s < n && not_crlf_l_n(s))) continue;
      const size_t p = s + (size_t)pre;
      const size_t u = run(p, kUpperish);
      if (u >= 1) {
        const size_t e = p + u + run(p + u, kLowerish);
        return (long)(e + contraction(e));
      }
    }
    return -1;
  }
  // \p{N}{1,3}
  long alt3(size_t s) const {
    const size_t r = run(s, kNum);
    return r ? (long)(s + std::min<size_t>(r, 3)) : -1;
  }
  //  ?[^\s\p{L}\p{N}]+[\r\n/]*
  long alt4(size_t s) const {
    for (int sp = 1; sp >= 0; sp--) {
      if (sp && !(s < n && cp[s] == ' ')) continue;
      const size_t p = s + (size_t)sp;
      size_t j = p;
      while (j < n && not_s_l_n(j)) j++;
      if (j > p) {
        while (j < n && (crlf(j) || cp[j] == '/')) j++;
        return (long)j;
      }
    }
    return -1;
  }
  // \s*[\r\n]+ : the whitespace run up to and including its last CR/LF
  long alt5(size_t s) const {
    const size_t w = run(s, kSpace);
    for (size_t k = w; k-- > 0;)
      if (crlf(s + k)) return (long)(s + k + 1);
    return -1;
  }
  // \s+(?!\S)
  long alt6(size_t s) const {
    const size_t w = run(s, kSpace);
    if (w == 0) return -1;
    if (s + w == n) return (long)(s + w);
    return w >= 2 ? (long)(s + w - 1) : -1;
  }
  // \s+
  long alt7(size_t s) const {
    const size_t w = run(s, kSpace);
    return w ? (long)(s + w) : -1;
  }
  long match(size_t s) const {
    long e;
    if ((e = alt1(s)) > 0) return e;
    if ((e = alt2(s)) > 0) return e;
    if ((e = alt3(s)) > 0) return e;
    if ((e = alt4(s)) > 0) return e;
    if ((e = alt5(s)) > 0) return e;
    if ((e = alt6(s)) > 0) return e;
    return alt7(s);
  }
};

// -------------------------------------------------------------------- BPE
struct Cache {
  std::unordered_map<std::string, std::vector<int32_t>> map;
};

// Token ids of one piece (its UTF-8 bytes): the reference's merge loop
// (tokenizer.ts:413-458) on interned symbols.  False if a final symbol is
// not in the vocabulary (the reference throws).
bool bpe(const Model& m, Cache& c, std::string& key, const uint8_t* p, size_t len, const std::vector<int32_t>** out) {
  key.assign(reinterpret_cast<const char*>(p), len);  // reuses the caller's buffer: no allocation on a hit
  auto it = c.map.find(key);
  if (it != c.map.end()) {
    *out = &it->second;
    return true;
  }
  std::vector<int32_t> sym(len);
  for (size_t i = 0; i < len; i++) sym[i] = m.byte_sym[p[i]];
  while (sym.size() > 1) {
    size_t best = SIZE_MAX;
    uint64_t best_rank = UINT64_MAX;
    int32_t merged = -1;
    for (size_t i = 0; i + 1 < sym.size(); i++) {
      auto mi = m.merges.find(((uint64_t)(uint32_t)sym[i] << 32) | (uint32_t)sym[i + 1]);
      if (mi != m.merges.end() && (mi->second >> 32) < best_rank) {
        best_rank = mi->second >> 32;
        best = i;
        merged = (int32_t)(uint32_t)mi->second;
      }
    }
    if (best == SIZE_MAX) break;
    const int32_t a = sym[best], b = sym[best + 1];
    size_t w = 0;
    for (size_t i = 0; i < sym.size();) {
      if (i + 1 < sym.size() && sym[i] == a && sym[i + 1] == b) {
        sym[w++] = merged;
        i += 2;
      } else {
        sym[w++] = sym[i++];
      }
    }
    sym.resize(w);
  }
  std::vector<int32_t> ids(sym.size());
  for (size_t i = 0; i < sym.size(); i++) {
    ids[i] = m.sym_vocab[sym[i]];
    if (ids[i] < 0) return false;
  }
  if (c.map.size() > (1u << 20)) c.map.clear();
  *out = &c.map.emplace(key, std::move(ids)).first->second;
  return true;
}

// Per-text output: ids, UTF-16 start/end and byte start/end of every token.
struct Encoded {
  std::vector<int32_t> ids;
  std::vector<uint32_t> u16s, u16e, bs, be;
  void clear() { ids.clear(); u16s.clear(); u16e.clear(); bs.clear(); be.clear(); }
};

struct Scratch {
  std::string key;
  std::vector<uint32_t> cps, boff, u16, unit_byte;
  std::vector<uint8_t> cls;
  std::vector<uint32_t> bounds;
};

// A piece [a, b) of code points spread over its tokens (tokenizer.ts:467-504).
void distribute(const Model& m, Scratch& s, size_t a, size_t b, const std::vector<int32_t>& ids, Encoded& out) {
  const uint32_t b0 = s.boff[a], total = s.boff[b] - b0;
  const uint32_t u0 = s.u16[a], units = s.u16[b] - u0;
  s.unit_byte.resize(units);
  for (size_t i = a; i < b; i++) {
    const uint32_t ui = s.u16[i] - u0;
    s.unit_byte[ui] = s.boff[i] - b0;
    if (s.cps[i] > 0xFFFF) s.unit_byte[ui + 1] = s.boff[i] - b0;  // both halves of a surrogate pair
  }
  s.bounds.assign(1, 0u);
  uint32_t bc = 0;
  for (int32_t id : ids) {
    bc += m.id_u16[id];
    s.bounds.push_back(bc);
  }
  if (bc != total)
    for (uint32_t& x : s.bounds) x = std::min(x, total);
  uint32_t u = 0;
  for (size_t k = 0; k < s.bounds.size(); k++) {
    while (u < units && s.unit_byte[u] < s.bounds[k]) u++;
    if (k + 1 < s.bounds.size()) {
      out.u16s.push_back(u0 + u);
      out.bs.push_back(b0 + s.bounds[k]);
    }
    if (k > 0) {
      out.u16e.push_back(u0 + u);
      out.be.push_back(b0 + s.bounds[k]);
    }
  }
  out.ids.insert(out.ids.end(), ids.begin(), ids.end());
}

// encode() (tokenizer.ts:238-291) of one UTF-8 text.  Returns TS_OK or an
// error code with the message in err.
int encode(const Model& m, Cache& cache, Scratch& s, const uint8_t* text, size_t len, Encoded& out, std::string& err) {
  out.clear();
  if (!decode_utf8(text, len, s.cps, s.boff)) {
    err = "ts_tok_encode: input is not valid UTF-8";
    return TS_ERR_ARG;
  }
  const size_t n = s.cps.size();
  s.u16.resize(n + 1);
  s.cls.resize(n);
  uint32_t u = 0;
  const ClassTable& ct = classes();
  for (size_t i = 0; i < n; i++) {
    s.u16[i] = u;
    u += s.cps[i] > 0xFFFF ? 2u : 1u;
    s.cls[i] = ct.get(s.cps[i]);
  }
  s.u16[n] = u;
  // one non-special slice [c0, c1): pretokenize (matches and gaps) and BPE each piece
  auto slice = [&](size_t c0, size_t c1) -> bool {
    Pre sub{s.cps.data() + c0, s.cls.data() + c0, c1 - c0};
    size_t cursor = 0, pos = 0;
    auto piece = [&](size_t a, size_t b) -> bool {
      const std::vector<int32_t>* ids = nullptr;
      if (!bpe(m, cache, s.key, text + s.boff[c0 + a], s.boff[c0 + b] - s.boff[c0 + a], &ids)) return false;
      distribute(m, s, c0 + a, c0 + b, *ids, out);
      return true;
    };
    while (pos < sub.n) {
      const long e = sub.match(pos);
      if (e > (long)pos) {
        if (pos > cursor && !piece(cursor, pos)) return false;
        if (!piece(pos, (size_t)e)) return false;
        cursor = pos = (size_t)e;
      } else {
        pos++;
      }
    }
    return cursor >= sub.n || piece(cursor, sub.n);
  };
  size_t cursor = 0;
  for (size_t i = 0; i < n;) {
    const std::pair<std::string, int32_t>* hit = nullptr;
    const size_t bi = s.boff[i];
    for (const auto& sp : m.specials)
      if (sp.first.size() <= len - bi && std::memcmp(text + bi, sp.first.data(), sp.first.size()) == 0) {
        hit = &sp;
        break;
      }
    if (!hit) {
      i++;
      continue;
    }
    if (i > cursor && !slice(cursor, i)) {
      err = "ts_tok_encode: a BPE symbol is not in the vocabulary (corrupt tokenizer.json?)";
      return TS_ERR_STATE;
    }
    size_t j = i;  // first code point after the literal
    while (j < n && s.boff[j] < bi + hit->first.size()) j++;
    out.ids.push_back(hit->second);
    out.u16s.push_back(s.u16[i]);
    out.u16e.push_back(s.u16[i] + m.id_u16[hit->second]);
    out.bs.push_back((uint32_t)bi);
    out.be.push_back((uint32_t)(bi + hit->first.size()));
    cursor = i = j;
  }
  if (cursor < n && !slice(cursor, n)) {
    err = "ts_tok_encode: a BPE symbol is not in the vocabulary (corrupt tokenizer.json?)";
    return TS_ERR_STATE;
  }
  return TS_OK;
}

}  // namespace

// ------------------------------------------------------------------ C ABI
struct ts_tok {
  Model model;
  std::vector<std::unique_ptr<Cache>> caches;  // one per worker thread
  std::vector<std::unique_ptr<Scratch>> scratch;
  void ensure_workers(size_t k) {
    while (caches.size() < k) {
      caches.emplace_back(new Cache());
      scratch.emplace_back(new Scratch());
    }
  }
};

static int tok_fail(int code, const std::string& msg) {
  ts::set_last_error(msg.c_str());
  return code;
}

extern "C" {

ts_tok_t* ts_tok_create(const char* tokenizer_json, size_t len, char* err, size_t err_cap) {
  std::string e;
  if (!tokenizer_json) e = "ts_tok_create: null tokenizer.json";
  std::unique_ptr<ts_tok> t;
  if (e.empty()) {
    t.reset(new ts_tok());
    if (!load_model(t->model, tokenizer_json, len, e)) t.reset();
  }
  if (!t) {
    if (err && err_cap) {
      std::strncpy(err, e.c_str(), err_cap - 1);
      err[err_cap - 1] = 0;
    }
    ts::set_last_error(e.c_str());
    return nullptr;
  }
  t->ensure_workers(1);
  return t.release();
}

void ts_tok_destroy(ts_tok_t* t) { delete t; }

uint32_t ts_tok_vocab_size(const ts_tok_t* t) { return t ? (uint32_t)t->model.id_bytes.size() : 0u; }

int ts_tok_encode(ts_tok_t* t, const char* utf8, size_t len, int32_t* ids, uint32_t* char_offsets,
                  uint32_t* byte_offsets, size_t cap, size_t* n_tokens) {
  if (!t || (!utf8 && len) || !n_tokens) return tok_fail(TS_ERR_ARG, "ts_tok_encode: null argument");
  Encoded out;
  std::string e;
  const int rc = encode(t->model, *t->caches[0], *t->scratch[0], reinterpret_cast<const uint8_t*>(utf8), len, out, e);
  if (rc != TS_OK) return tok_fail(rc, e);
  const size_t n = out.ids.size();
  *n_tokens = n;
  if (!ids && !char_offsets && !byte_offsets) return TS_OK;  // size query
  if (n > cap) return tok_fail(TS_ERR_ARG, "ts_tok_encode: " + std::to_string(n) + " tokens > cap " + std::to_string(cap));
  if (ids) std::memcpy(ids, out.ids.data(), n * sizeof(int32_t));
  // n + 1 entries: each token's start, then the end of the last token
  if (char_offsets) {
    std::memcpy(char_offsets, out.u16s.data(), n * sizeof(uint32_t));
    char_offsets[n] = n ? out.u16e[n - 1] : 0u;
  }
  if (byte_offsets) {
    std::memcpy(byte_offsets, out.bs.data(), n * sizeof(uint32_t));
    byte_offsets[n] = n ? out.be[n - 1] : 0u;
  }
  return TS_OK;
}

int ts_tok_encode_batch(ts_tok_t* t, const char* const* texts, const size_t* lens, uint32_t n_texts, uint32_t n_threads,
                        int32_t* ids, uint32_t* starts, uint32_t* ends, size_t cap, uint64_t* token_begin) {
  if (!t || (n_texts && (!texts || !lens)) || !token_begin) return tok_fail(TS_ERR_ARG, "ts_tok_encode_batch: null argument");
  const uint32_t hw = std::max(1u, std::thread::hardware_concurrency());
  const uint32_t k = std::max(1u, std::min({n_threads ? n_threads : hw, hw * 2u, std::max(1u, n_texts)}));
  t->ensure_workers(k);
  std::vector<Encoded> res(n_texts);
  std::vector<std::string> errs(k);
  std::vector<int> rcs(k, TS_OK);
  std::atomic<uint32_t> next{0};
  auto work = [&](uint32_t w) {
    for (uint32_t i; (i = next.fetch_add(1)) < n_texts;) {
      const int rc = encode(t->model, *t->caches[w], *t->scratch[w], reinterpret_cast<const uint8_t*>(texts[i]), lens[i],
                            res[i], errs[w]);
      if (rc != TS_OK) {
        rcs[w] = rc;
        errs[w] = "text " + std::to_string(i) + ": " + errs[w];
        return;
      }
    }
  };
  std::vector<std::thread> pool;
  for (uint32_t w = 1; w < k; w++) pool.emplace_back(work, w);
  work(0);
  for (auto& th : pool) th.join();
  for (uint32_t w = 0; w < k; w++)
    if (rcs[w] != TS_OK) return tok_fail(rcs[w], "ts_tok_encode_batch: " + errs[w]);
  uint64_t total = 0;
  for (uint32_t i = 0; i < n_texts; i++) {
    token_begin[i] = total;
    total += res[i].ids.size();
  }
  token_begin[n_texts] = total;
  if (!ids && !starts && !ends) return TS_OK;  // size query
  if (total > cap) return tok_fail(TS_ERR_ARG, "ts_tok_encode_batch: " + std::to_string(total) + " tokens > cap");
  for (uint32_t i = 0; i < n_texts; i++) {
    const size_t o = token_begin[i], m = res[i].ids.size();
    if (ids) std::memcpy(ids + o, res[i].ids.data(), m * sizeof(int32_t));
    if (starts) std::memcpy(starts + o, res[i].u16s.data(), m * sizeof(uint32_t));
    if (ends) std::memcpy(ends + o, res[i].u16e.data(), m * sizeof(uint32_t));
  }
  return TS_OK;
}

int ts_tok_decode(const ts_tok_t* t, const int32_t* ids, size_t n, char* out, size_t cap, size_t* out_len) {
  if (!t || (!ids && n) || !out_len) return tok_fail(TS_ERR_ARG, "ts_tok_decode: null argument");
  const Model& m = t->model;
  size_t total = 0;
  for (size_t i = 0; i < n; i++)
    if (ids[i] >= 0 && (size_t)ids[i] < m.id_bytes.size() && m.id_known[ids[i]]) total += m.id_bytes[ids[i]].size();
  *out_len = total;
  if (!out) return TS_OK;
  if (total > cap) return tok_fail(TS_ERR_ARG, "ts_tok_decode: output larger than cap");
  size_t o = 0;
  for (size_t i = 0; i < n; i++)
    if (ids[i] >= 0 && (size_t)ids[i] < m.id_bytes.size() && m.id_known[ids[i]]) {
      std::memcpy(out + o, m.id_bytes[ids[i]].data(), m.id_bytes[ids[i]].size());
      o += m.id_bytes[ids[i]].size();
    }
  return TS_OK;
}

}  // extern "C"
