// Byte-level BPE tokenizer of the Qwen3 vocabulary, host side
// (tools/tokenizer.py:39-192).  From an HF tokenizer.json: the vocabulary
// (model.vocab), the merge ranks (model.merges, "a b" strings or [a, b]
// pairs) and the added tokens.  Encoding: added tokens are matched literally,
// leftmost-longest; the text between them is split by the GPT-2 style
// pretokenizer (contractions, letter runs with one optional leading
// non-letter, single digits, symbol runs with trailing newlines, whitespace
// runs that leave their last space to the next word), each piece's UTF-8
// bytes become byte symbols and adjacent symbols merge by lowest rank until
// none applies.  Decoding concatenates the token strings, maps each symbol
// back to its byte and decodes UTF-8 with U+FFFD for every maximal invalid
// subsequence (Python's errors="replace").  Character classes are Python's
// (str.isalpha, category N*, str.isspace), from q3_unicode_tables.inc.
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/q3_ops.h"
#include "q3_json.h"
#include "q3_unicode_tables.inc"

namespace {

template <size_t N>
bool in_ranges(const uint32_t (&r)[N][2], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid][0]) hi = mid;
    else if (cp > r[mid][1]) lo = mid + 1;
    else return true;
  }
  return false;
}

bool is_l(uint32_t c) { return in_ranges(kUniLetter, c); }
bool is_n(uint32_t c) { return in_ranges(kUniNumber, c); }
bool is_s(uint32_t c) { return in_ranges(kUniSpace, c); }
bool is_sym(uint32_t c) { return !is_s(c) && !is_l(c) && !is_n(c); }
bool is_nl(uint32_t c) { return c == '\r' || c == '\n'; }
bool is_prefix(uint32_t c) { return !is_nl(c) && !is_l(c) && !is_n(c); }

// strict UTF-8 -> code points (false on malformed input)
bool utf8_decode(const char *s, size_t n, std::vector<uint32_t> &out) {
  const unsigned char *u = reinterpret_cast<const unsigned char *>(s);
  size_t i = 0;
  while (i < n) {
    const uint32_t b = u[i];
    int len;
    uint32_t cp;
    if (b < 0x80) { len = 1; cp = b; }
    else if ((b & 0xE0) == 0xC0) { len = 2; cp = b & 0x1F; }
    else if ((b & 0xF0) == 0xE0) { len = 3; cp = b & 0x0F; }
    else if ((b & 0xF8) == 0xF0) { len = 4; cp = b & 0x07; }
    else return false;
    if (i + len > n) return false;
    for (int k = 1; k < len; ++k) {
      if ((u[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (u[i + k] & 0x3F);
    }
    static const uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
    if (cp < kMin[len] || cp > 0x10FFFF || (cp >= 0xD800 && cp < 0xE000)) return false;
    out.push_back(cp);
    i += len;
  }
  return true;
}

// bytes -> text, one U+FFFD per maximal invalid subsequence
std::string utf8_replace(const std::string &b) {
  std::string out;
  const unsigned char *u = reinterpret_cast<const unsigned char *>(b.data());
  const size_t n = b.size();
  size_t i = 0;
  while (i < n) {
    const unsigned c = u[i];
    if (c < 0x80) { out += static_cast<char>(c); ++i; continue; }
    int need;
    unsigned lo = 0x80, hi = 0xBF;
    if (c >= 0xC2 && c <= 0xDF) need = 1;
    else if (c == 0xE0) { need = 2; lo = 0xA0; }
    else if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) need = 2;
    else if (c == 0xED) { need = 2; hi = 0x9F; }
    else if (c == 0xF0) { need = 3; lo = 0x90; }
    else if (c >= 0xF1 && c <= 0xF3) need = 3;
    else if (c == 0xF4) { need = 3; hi = 0x8F; }
    else { out += "\xEF\xBF\xBD"; ++i; continue; }
    size_t j = i + 1;
    int got = 0;
    while (got < need && j < n) {
      const unsigned d = u[j];
      const unsigned a = got == 0 ? lo : 0x80, z = got == 0 ? hi : 0xBF;
      if (d < a || d > z) break;
      ++j;
      ++got;
    }
    if (got == need) out.append(b, i, j - i);
    else out += "\xEF\xBF\xBD";
    i = j;
  }
  return out;
}

}  // namespace

struct q3_tokenizer {
  std::unordered_map<std::string, int32_t> vocab;
  std::unordered_map<int32_t, std::string> id_to_token;
  std::unordered_map<std::string, int32_t> ranks;      // a + '\xff' + b -> rank
  std::string byte_sym[256];
  std::unordered_map<uint32_t, uint8_t> sym_byte;
  std::vector<std::pair<std::vector<uint32_t>, int32_t>> special;   // added tokens, file order
  int32_t eos_id = 151645;

  // tools/tokenizer.py:21-35: printable bytes keep their code point, the
  // others take 256, 257, ... in byte order
  void byte_tables() {
    uint32_t extra = 0;
    for (uint32_t b = 0; b < 256; ++b) {
      const bool keep = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE);
      const uint32_t cp = keep ? b : 256 + extra++;
      byte_sym[b].clear();
      q3json::put_utf8(byte_sym[b], cp);
      sym_byte[cp] = static_cast<uint8_t>(b);
    }
  }

  std::vector<std::vector<uint32_t>> split(const uint32_t *t, size_t n) const {
    static const char *kCon[7] = {"'s", "'t", "'re", "'ve", "'m", "'ll", "'d"};
    std::vector<std::vector<uint32_t>> chunks;
    size_t i = 0;
    auto emit = [&](size_t a, size_t b) { chunks.emplace_back(t + a, t + b); };
    while (i < n) {
      const uint32_t c = t[i];
      bool done = false;
      for (const char *con : kCon) {
        const size_t len = strlen(con);
        if (i + len > n) continue;
        bool eq = true;
        for (size_t k = 0; k < len && eq; ++k) {
          uint32_t x = t[i + k];
          if (x >= 'A' && x <= 'Z') x += 32;
          eq = x == static_cast<unsigned char>(con[k]);
        }
        if (eq) {
          emit(i, i + len);
          i += len;
          done = true;
          break;
        }
      }
      if (done) continue;
      if (is_l(c) || (is_prefix(c) && i + 1 < n && is_l(t[i + 1]))) {
        size_t j = is_l(c) ? i : i + 1;
        while (j < n && is_l(t[j])) ++j;
        emit(i, j);
        i = j;
      } else if (is_n(c)) {
        emit(i, i + 1);
        ++i;
      } else if (is_sym(c) || (c == ' ' && i + 1 < n && is_sym(t[i + 1]))) {
        size_t j = is_sym(c) ? i : i + 1;
        while (j < n && is_sym(t[j])) ++j;
        while (j < n && is_nl(t[j])) ++j;
        emit(i, j);
        i = j;
      } else {   // a whitespace run
        size_t j = i;
        while (j < n && is_s(t[j])) ++j;
        size_t last_nl = SIZE_MAX;
        for (size_t k = i; k < j; ++k)
          if (is_nl(t[k])) last_nl = k;
        if (last_nl != SIZE_MAX) {
          emit(i, last_nl + 1);
          i = last_nl + 1;
        } else if (j == n || j - i == 1) {
          emit(i, j);
          i = j;
        } else {
          emit(i, j - 1);
          i = j - 1;
        }
      }
    }
    return chunks;
  }

  // one piece: byte symbols merged by lowest rank (leftmost on equal rank)
  int encode_chunk(const std::vector<uint32_t> &chunk, std::vector<int32_t> &ids) const {
    std::string bytes;
    for (uint32_t cp : chunk) q3json::put_utf8(bytes, cp);
    std::vector<std::string> w;
    w.reserve(bytes.size());
    for (unsigned char b : bytes) w.push_back(byte_sym[b]);
    std::string key;
    while (w.size() > 1) {
      int32_t best_rank = -1;
      size_t best = 0;
      for (size_t k = 0; k + 1 < w.size(); ++k) {
        key.assign(w[k]);
        key += '\xff';
        key += w[k + 1];
        const auto it = ranks.find(key);
        if (it != ranks.end() && (best_rank < 0 || it->second < best_rank)) {
          best_rank = it->second;
          best = k;
        }
      }
      if (best_rank < 0) break;
      w[best] += w[best + 1];
      w.erase(w.begin() + static_cast<long>(best) + 1);
    }
    for (const std::string &s : w) {
      const auto it = vocab.find(s);
      if (it == vocab.end()) return Q3_ERR_SHAPE;
      ids.push_back(it->second);
    }
    return Q3_OK;
  }

  // length of the longest added token at t[i] (0 if none), its id in *id
  size_t special_at(const std::vector<uint32_t> &t, size_t i, int32_t *id) const {
    size_t best = 0;
    for (const auto &sp : special) {
      const size_t len = sp.first.size();
      if (len == 0 || i + len > t.size() || len <= best) continue;
      if (std::equal(sp.first.begin(), sp.first.end(), t.begin() + static_cast<long>(i))) {
        best = len;
        if (id) *id = sp.second;
      }
    }
    return best;
  }

  int encode(const std::vector<uint32_t> &t, std::vector<int32_t> &ids) const {
    size_t i = 0;
    while (i < t.size()) {
      int32_t id = 0;
      const size_t len = special_at(t, i, &id);
      if (len) {
        ids.push_back(id);
        i += len;
        continue;
      }
      size_t j = i;
      while (j < t.size() && !special_at(t, j, nullptr)) ++j;
      for (const auto &chunk : split(t.data() + i, j - i)) {
        const int rc = encode_chunk(chunk, ids);
        if (rc) return rc;
      }
      i = j;
    }
    return Q3_OK;
  }

  int decode(const int32_t *ids, uint32_t n, std::string &out) const {
    std::string text;
    for (uint32_t k = 0; k < n; ++k) {
      const auto it = id_to_token.find(ids[k]);
      if (it == id_to_token.end()) return Q3_ERR_SHAPE;
      text += it->second;
    }
    std::vector<uint32_t> cps;
    if (!utf8_decode(text.data(), text.size(), cps)) return Q3_ERR_SHAPE;
    std::string bytes;
    bytes.reserve(cps.size());
    for (uint32_t cp : cps) {
      const auto it = sym_byte.find(cp);
      if (it == sym_byte.end()) return Q3_ERR_SHAPE;
      bytes += static_cast<char>(it->second);
    }
    out = utf8_replace(bytes);
    return Q3_OK;
  }
};

extern "C" int q3_tokenizer_load(const char *path, void **tokenizer) {
  if (!path || !tokenizer) return Q3_ERR_NULL;
  *tokenizer = nullptr;
  FILE *f = fopen(path, "rb");
  if (!f) return Q3_ERR_NULL;
  std::string data;
  char buf[1 << 16];
  size_t got;
  while ((got = fread(buf, 1, sizeof buf, f)) > 0) data.append(buf, got);
  fclose(f);
  q3json::Parser jp{data.data(), data.data() + data.size()};
  const q3json::Value root = jp.value();
  if (!jp.ok || root.kind != q3json::Value::OBJ) return Q3_ERR_SHAPE;
  const q3json::Value *model = root.get("model");
  const q3json::Value *vocab = model ? model->get("vocab") : nullptr;
  const q3json::Value *merges = model ? model->get("merges") : nullptr;
  if (!vocab || vocab->kind != q3json::Value::OBJ || !merges || merges->kind != q3json::Value::ARR)
    return Q3_ERR_SHAPE;
  q3_tokenizer *t = new (std::nothrow) q3_tokenizer;
  if (!t) return Q3_ERR_CAPACITY;
  for (const auto &kv : vocab->obj) {
    if (kv.second.kind != q3json::Value::NUM) { delete t; return Q3_ERR_SHAPE; }
    const int32_t id = static_cast<int32_t>(kv.second.num);
    t->vocab[kv.first] = id;
    t->id_to_token[id] = kv.first;
  }
  int32_t rank = 0;
  for (const q3json::Value &m : merges->arr) {
    std::string a, b;
    if (m.kind == q3json::Value::STR) {
      const size_t sp = m.str.find(' ');
      if (sp == std::string::npos || m.str.find(' ', sp + 1) != std::string::npos) { delete t; return Q3_ERR_SHAPE; }
      a = m.str.substr(0, sp);
      b = m.str.substr(sp + 1);
    } else if (m.kind == q3json::Value::ARR && m.arr.size() == 2 &&
               m.arr[0].kind == q3json::Value::STR && m.arr[1].kind == q3json::Value::STR) {
      a = m.arr[0].str;
      b = m.arr[1].str;
    } else {
      delete t;
      return Q3_ERR_SHAPE;
    }
    t->ranks[a + '\xff' + b] = rank++;   // a later duplicate keeps the later rank, as a dict does
  }
  t->byte_tables();
  if (const q3json::Value *added = root.get("added_tokens")) {
    for (const q3json::Value &a : added->arr) {
      const q3json::Value *c = a.get("content"), *id = a.get("id");
      if (!c || !id || c->kind != q3json::Value::STR || id->kind != q3json::Value::NUM) continue;
      std::vector<uint32_t> cps;
      if (!utf8_decode(c->str.data(), c->str.size(), cps)) { delete t; return Q3_ERR_SHAPE; }
      const int32_t tid = static_cast<int32_t>(id->num);
      bool replaced = false;   // a repeated content keeps its first place, the latest id
      for (auto &sp : t->special)
        if (sp.first == cps) { sp.second = tid; replaced = true; }
      if (!replaced) t->special.emplace_back(std::move(cps), tid);
      t->id_to_token[tid] = c->str;
      if (c->str == "<|im_end|>") t->eos_id = tid;
    }
  }
  *tokenizer = t;
  return Q3_OK;
}

extern "C" int q3_tokenizer_encode(const void *tokenizer, const char *text, size_t text_bytes,
                                   int32_t *ids, uint32_t cap, uint32_t *n_ids) {
  if (!tokenizer || !n_ids || (!text && text_bytes)) return Q3_ERR_NULL;
  const q3_tokenizer *t = static_cast<const q3_tokenizer *>(tokenizer);
  std::vector<uint32_t> cps;
  if (!utf8_decode(text, text_bytes, cps)) return Q3_ERR_SHAPE;
  std::vector<int32_t> out;
  const int rc = t->encode(cps, out);
  if (rc) return rc;
  *n_ids = static_cast<uint32_t>(out.size());
  if (out.size() > cap) return Q3_ERR_CAPACITY;
  if (!out.empty()) {
    if (!ids) return Q3_ERR_NULL;
    memcpy(ids, out.data(), 4 * out.size());
  }
  return Q3_OK;
}

extern "C" int q3_tokenizer_decode(const void *tokenizer, const int32_t *ids, uint32_t n, char *text,
                                   size_t cap, size_t *n_bytes) {
  if (!tokenizer || !n_bytes || (!ids && n)) return Q3_ERR_NULL;
  const q3_tokenizer *t = static_cast<const q3_tokenizer *>(tokenizer);
  std::string out;
  const int rc = t->decode(ids, n, out);
  if (rc) return rc;
  *n_bytes = out.size();
  if (out.size() > cap) return Q3_ERR_CAPACITY;
  if (!out.empty()) {
    if (!text) return Q3_ERR_NULL;
    memcpy(text, out.data(), out.size());
  }
  return Q3_OK;
}

extern "C" int32_t q3_tokenizer_eos_id(const void *tokenizer) {
  return tokenizer ? static_cast<const q3_tokenizer *>(tokenizer)->eos_id : -1;
}

extern "C" int q3_tokenizer_destroy(void *tokenizer) {
  delete static_cast<q3_tokenizer *>(tokenizer);
  return Q3_OK;
}
