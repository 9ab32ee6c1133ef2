/* tokenizer.cpp — SentencePiece BPE over a GGUF vocabulary (see tokenizer.h). */
#include "tokenizer.h"

#include <algorithm>
#include <cstdio>
#include <queue>

#include "gguf.h"

namespace ulbe {

namespace {
const char kSpace[] = "\xe2\x96\x81"; /* U+2581, SentencePiece's whitespace mark */

/* the bytes of consecutive <0xXX> pieces as UTF-8: each valid character as is, every byte
   that does not start one (bad lead, short or overlong sequence, surrogate, > U+10FFFF) as
   U+FFFD */
void append_bytes_utf8(const std::string& b, std::string* s) {
  size_t i = 0;
  while (i < b.size()) {
    const unsigned char c = (unsigned char)b[i];
    size_t n = 0;
    uint32_t cp = 0, lo = 0;
    if (c < 0x80) { n = 1; cp = c; }
    else if ((c & 0xE0) == 0xC0) { n = 2; cp = c & 0x1F; lo = 0x80; }
    else if ((c & 0xF0) == 0xE0) { n = 3; cp = c & 0x0F; lo = 0x800; }
    else if ((c & 0xF8) == 0xF0) { n = 4; cp = c & 0x07; lo = 0x10000; }
    bool ok = n > 0 && i + n <= b.size();
    for (size_t k = 1; ok && k < n; ++k) {
      const unsigned char cc = (unsigned char)b[i + k];
      if ((cc & 0xC0) != 0x80) ok = false;
      else cp = (cp << 6) | (cc & 0x3F);
    }
    if (ok && n > 1 && (cp < lo || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))) ok = false;
    if (ok) {
      s->append(b, i, n);
      i += n;
    } else {
      s->append("\xef\xbf\xbd");
      i += 1;
    }
  }
}

/* byte length of the UTF-8 character starting with c (1 for a stray continuation byte) */
size_t utf8_len(unsigned char c) {
  if (c < 0x80) return 1;
  if ((c & 0xE0) == 0xC0) return 2;
  if ((c & 0xF0) == 0xE0) return 3;
  if ((c & 0xF8) == 0xF0) return 4;
  return 1;
}
}  // namespace

std::string bytes_to_utf8(const std::string& b) {
  std::string s;
  append_bytes_utf8(b, &s);
  return s;
}

bool SpmTokenizer::load(const std::vector<std::string>& pieces, const std::vector<float>& scores,
                        const std::vector<int32_t>& types, int bos, int eos, int unk, std::string* err) {
  if (pieces.empty() || scores.size() != pieces.size() || types.size() != pieces.size()) {
    if (err) *err = "tokenizer: pieces, scores and types must be non-empty and of equal length";
    return false;
  }
  pieces_ = pieces;
  scores_ = scores;
  types_ = types;
  bos_ = bos;
  eos_ = eos;
  unk_ = unk;
  mergeable_.clear();
  for (auto& v : user_) v.clear();
  for (int i = 0; i < 256; ++i) byte_id_[i] = -1;
  for (size_t i = 0; i < pieces_.size(); ++i) {
    const int t = types_[i];
    if (t == NORMAL || t == USER_DEFINED) {
      mergeable_.emplace(pieces_[i], (int32_t)i); /* the first id of a duplicated piece wins */
      if (t == USER_DEFINED && !pieces_[i].empty()) user_[(unsigned char)pieces_[i][0]].push_back((int32_t)i);
    } else if (t == BYTE) {
      unsigned v = 0;
      if (pieces_[i].size() == 6 && std::sscanf(pieces_[i].c_str(), "<0x%02X>", &v) == 1 && v < 256)
        byte_id_[v] = (int32_t)i;
    }
  }
  for (auto& v : user_)
    std::stable_sort(v.begin(), v.end(), [&](int32_t a, int32_t b) { return pieces_[a].size() > pieces_[b].size(); });
  return true;
}

bool SpmTokenizer::load(const GGUFFile& f, std::string* err) {
  const std::string model = f.str("tokenizer.ggml.model", "");
  const std::vector<std::string>* tok = f.str_array("tokenizer.ggml.tokens");
  if (model != "llama" || !tok) {
    if (err) *err = "tokenizer: no SentencePiece (tokenizer.ggml.model = llama) vocabulary";
    return false;
  }
  const std::vector<double>* sc = f.num_array("tokenizer.ggml.scores");
  const std::vector<double>* ty = f.num_array("tokenizer.ggml.token_type");
  std::vector<float> scores(tok->size(), 0.f);
  std::vector<int32_t> types(tok->size(), NORMAL);
  if (sc && sc->size() == tok->size())
    for (size_t i = 0; i < sc->size(); ++i) scores[i] = (float)(*sc)[i];
  if (ty && ty->size() == tok->size())
    for (size_t i = 0; i < ty->size(); ++i) types[i] = (int32_t)(*ty)[i];
  if (!load(*tok, scores, types, (int)f.num("tokenizer.ggml.bos_token_id", 1),
            (int)f.num("tokenizer.ggml.eos_token_id", 2), (int)f.num("tokenizer.ggml.unknown_token_id", 0), err))
    return false;
  set_flags(f.num("tokenizer.ggml.add_bos_token", 1) != 0, f.num("tokenizer.ggml.add_space_prefix", 1) != 0);
  return true;
}

std::vector<int32_t> SpmTokenizer::encode(const std::string& text, bool add_bos) const {
  std::vector<int32_t> out;
  if (add_bos && bos_ >= 0) out.push_back(bos_);
  if (text.empty()) return out;
  std::string norm = add_space_prefix_ ? kSpace : "";
  for (char ch : text) {
    if (ch == ' ') norm += kSpace;
    else norm.push_back(ch);
  }
  /* symbols: byte ranges of norm in a doubly linked list */
  struct Sym {
    size_t off, len;
    int prev, next;
    bool frozen; /* a user-defined piece: never merged */
  };
  std::vector<Sym> sym;
  for (size_t o = 0; o < norm.size();) {
    size_t l = 0;
    for (int32_t id : user_[(unsigned char)norm[o]])
      if (norm.compare(o, pieces_[id].size(), pieces_[id]) == 0) {
        l = pieces_[id].size();
        break;
      }
    const bool frozen = l > 0;
    if (!frozen) {
      l = utf8_len((unsigned char)norm[o]);
      if (o + l > norm.size()) l = norm.size() - o;
    }
    sym.push_back({o, l, (int)sym.size() - 1, (int)sym.size() + 1, frozen});
    o += l;
  }
  sym.back().next = -1;
  /* candidate merges, best score first, then leftmost; stale entries skipped by length */
  struct Cand {
    float score;
    int left, right;
    size_t len;
  };
  auto worse = [](const Cand& a, const Cand& b) {
    return a.score < b.score || (a.score == b.score && a.left > b.left);
  };
  std::priority_queue<Cand, std::vector<Cand>, decltype(worse)> q(worse);
  auto propose = [&](int l, int r) {
    if (l < 0 || r < 0 || sym[l].frozen || sym[r].frozen) return;
    const std::string s = norm.substr(sym[l].off, sym[l].len + sym[r].len);
    auto it = mergeable_.find(s);
    if (it != mergeable_.end()) q.push({scores_[it->second], l, r, s.size()});
  };
  for (int i = 0; i + 1 < (int)sym.size(); ++i) propose(i, i + 1);
  while (!q.empty()) {
    const Cand c = q.top();
    q.pop();
    Sym &L = sym[c.left], &R = sym[c.right];
    if (L.len == 0 || R.len == 0 || L.next != c.right || L.len + R.len != c.len) continue; /* stale */
    L.len += R.len;
    R.len = 0;
    L.next = R.next;
    if (R.next >= 0) sym[R.next].prev = c.left;
    propose(L.prev, c.left);
    propose(c.left, L.next);
  }
  for (int i = 0; i >= 0; i = sym[i].next) {
    const std::string s = norm.substr(sym[i].off, sym[i].len);
    auto it = mergeable_.find(s);
    if (it != mergeable_.end()) {
      out.push_back(it->second);
      continue;
    }
    for (unsigned char b : s) out.push_back(byte_id_[b] >= 0 ? byte_id_[b] : unk_);
  }
  return out;
}

std::string SpmTokenizer::decode(const std::vector<int32_t>& ids) const {
  std::string s, bytes;
  for (int32_t id : ids) {
    if (id < 0 || (size_t)id >= pieces_.size()) continue;
    const int t = types_[id];
    if (t == CONTROL || t == UNUSED) continue;
    if (t == BYTE) {
      unsigned v = 0;
      if (std::sscanf(pieces_[id].c_str(), "<0x%02X>", &v) == 1) bytes.push_back((char)v);
      continue;
    }
    append_bytes_utf8(bytes, &s);
    bytes.clear();
    if (t == UNKNOWN) {
      s += " \xe2\x81\x87 ";
      continue;
    }
    const std::string& p = pieces_[id];
    for (size_t o = 0; o < p.size();) {
      if (p.compare(o, 3, kSpace) == 0) {
        s.push_back(' ');
        o += 3;
      } else {
        s.push_back(p[o++]);
      }
    }
  }
  append_bytes_utf8(bytes, &s);
  if (add_space_prefix_ && !s.empty() && s[0] == ' ') s.erase(0, 1); /* the dummy prefix */
  return s;
}

}  // namespace ulbe

/* ------------------------------------------------------------------ byte-level BPE ("gpt2") */
namespace ulbe {
namespace {
#include "unicode_ranges.h"

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
bool is_letter(uint32_t c) { return in_ranges(kLetterRanges, c); }
bool is_number(uint32_t c) { return in_ranges(kNumberRanges, c); }
/* Unicode White_Space */
bool is_space(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}
bool is_nl(uint32_t c) { return c == '\r' || c == '\n'; }
bool is_other(uint32_t c) { return !is_space(c) && !is_letter(c) && !is_number(c); }

std::string utf8_of(uint32_t cp) {
  std::string s;
  if (cp < 0x80) s.push_back((char)cp);
  else if (cp < 0x800) { s.push_back((char)(0xC0 | (cp >> 6))); s.push_back((char)(0x80 | (cp & 0x3F))); }
  else if (cp < 0x10000) {
    s.push_back((char)(0xE0 | (cp >> 12)));
    s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    s.push_back((char)(0x80 | (cp & 0x3F)));
  } else {
    s.push_back((char)(0xF0 | (cp >> 18)));
    s.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
    s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    s.push_back((char)(0x80 | (cp & 0x3F)));
  }
  return s;
}

/* code points of s with their byte offsets (offs has one extra entry, s.size()); a byte that
   starts no valid character counts as one character of its own (category: other) */
void code_points(const std::string& s, std::vector<uint32_t>* cps, std::vector<size_t>* offs) {
  for (size_t i = 0; i < s.size();) {
    const unsigned char c = (unsigned char)s[i];
    size_t n = utf8_len(c);
    uint32_t cp = n == 1 ? c : n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
    bool ok = i + n <= s.size() && !(n == 1 && c >= 0x80);
    for (size_t k = 1; ok && k < n; ++k) {
      const unsigned char cc = (unsigned char)s[i + k];
      if ((cc & 0xC0) != 0x80) ok = false;
      else cp = (cp << 6) | (cc & 0x3F);
    }
    if (!ok) { n = 1; cp = 0xFFFD; }
    cps->push_back(cp);
    offs->push_back(i);
    i += n;
  }
  offs->push_back(s.size());
}

/* end (exclusive, in code points) of the piece Llama-3's split pattern matches at i */
size_t split_piece(const std::vector<uint32_t>& c, size_t i) {
  const size_t n = c.size();
  auto lower = [](uint32_t x) { return x >= 'A' && x <= 'Z' ? x + 32 : x; };
  /* (?i:'s|'t|'re|'ve|'m|'ll|'d) */
  if (c[i] == '\'' && i + 1 < n) {
    const uint32_t a = lower(c[i + 1]), b = i + 2 < n ? lower(c[i + 2]) : 0;
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return i + 2;
    if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return i + 3;
  }
  /* [^\r\n\p{L}\p{N}]?\p{L}+ */
  {
    size_t j = i;
    if (!is_nl(c[i]) && !is_letter(c[i]) && !is_number(c[i]) && i + 1 < n && is_letter(c[i + 1])) j = i + 1;
    if (is_letter(c[j])) {
      while (j < n && is_letter(c[j])) ++j;
      return j;
    }
  }
  /* \p{N}{1,3} */
  if (is_number(c[i])) {
    size_t j = i;
    while (j < n && j < i + 3 && is_number(c[j])) ++j;
    return j;
  }
  /*  ?[^\s\p{L}\p{N}]+[\r\n]* */
  {
    size_t j = i;
    if (c[i] == ' ' && i + 1 < n && is_other(c[i + 1])) j = i + 1;
    if (is_other(c[j])) {
      while (j < n && is_other(c[j])) ++j;
      while (j < n && is_nl(c[j])) ++j;
      return j;
    }
  }
  /* whitespace: \s*[\r\n]+ | \s+(?!\S) | \s+ */
  size_t j = i;
  while (j < n && is_space(c[j])) ++j;
  size_t last_nl = n;
  for (size_t k = i; k < j; ++k)
    if (is_nl(c[k])) last_nl = k;
  if (last_nl < n) return last_nl + 1;
  if (j == n) return j;
  if (j - i >= 2) return j - 1;
  return j > i ? j : i + 1;
}
/* end of the piece GPT-2's split pattern matches at i:
   's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+ */
size_t split_piece_gpt2(const std::vector<uint32_t>& c, size_t i) {
  const size_t n = c.size();
  if (c[i] == '\'' && i + 1 < n) {
    const uint32_t a = c[i + 1], b = i + 2 < n ? c[i + 2] : 0;
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return i + 2;
    if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return i + 3;
  }
  bool (*cls[3])(uint32_t) = {is_letter, is_number, is_other};
  for (auto f : cls) {
    size_t j = i;
    if (c[i] == ' ' && i + 1 < n && f(c[i + 1])) j = i + 1;
    if (f(c[j])) {
      while (j < n && f(c[j])) ++j;
      return j;
    }
  }
  size_t j = i;
  while (j < n && is_space(c[j])) ++j;
  if (j == n) return j;
  if (j - i >= 2) return j - 1;
  return j > i ? j : i + 1;
}
}  // namespace

bool ByteBpeTokenizer::load(const GGUFFile& f, std::string* err) {
  const std::vector<std::string>* tok = f.str_array("tokenizer.ggml.tokens");
  const std::vector<std::string>* merges = f.str_array("tokenizer.ggml.merges");
  if (f.str("tokenizer.ggml.model", "") != "gpt2" || !tok || !merges) {
    if (err) *err = "tokenizer: no byte-level BPE (tokenizer.ggml.model = gpt2) vocabulary";
    return false;
  }
  tokens_ = *tok;
  types_.assign(tokens_.size(), SpmTokenizer::NORMAL);
  if (const std::vector<double>* ty = f.num_array("tokenizer.ggml.token_type"))
    if (ty->size() == tokens_.size())
      for (size_t i = 0; i < ty->size(); ++i) types_[i] = (int32_t)(*ty)[i];
  id_.clear();
  for (size_t i = 0; i < tokens_.size(); ++i) id_.emplace(tokens_[i], (int32_t)i);
  rank_.clear();
  for (size_t i = 0; i < merges->size(); ++i) rank_.emplace((*merges)[i], (int32_t)i);
  /* GPT-2's byte <-> printable character table: bytes that are printable Latin-1 map to
     themselves, the others to U+0100 + n in byte order */
  int n = 0;
  char_byte_.clear();
  for (int b = 0; b < 256; ++b) {
    const bool keep = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
    const uint32_t cp = keep ? (uint32_t)b : 256u + (uint32_t)n++;
    byte_char_[b] = utf8_of(cp);
    char_byte_[cp] = (uint8_t)b;
  }
  for (auto& v : special_) v.clear();
  for (size_t i = 0; i < tokens_.size(); ++i)
    if ((types_[i] == SpmTokenizer::CONTROL || types_[i] == SpmTokenizer::USER_DEFINED) && !tokens_[i].empty())
      special_[(unsigned char)tokens_[i][0]].push_back((int32_t)i);
  for (auto& v : special_)
    std::stable_sort(v.begin(), v.end(), [&](int32_t a, int32_t b) { return tokens_[a].size() > tokens_[b].size(); });
  bos_ = (int)f.num("tokenizer.ggml.bos_token_id", -1);
  add_bos_ = f.num("tokenizer.ggml.add_bos_token", 1) != 0;
  /* the pre-tokenizers whose split is implemented (and pinned against HF tokenizers): GPT-2's,
     and Llama-3's (llama.cpp writes "llama-bpe"; "llama3" and an absent key mean the same);
     any other name (qwen2, deepseek-llm, starcoder, ...) splits text differently, so such a
     file is refused instead of being tokenized silently wrong */
  const std::string pre = f.str("tokenizer.ggml.pre", "");
  if (pre != "" && pre != "default" && pre != "gpt2" && pre != "llama-bpe" && pre != "llama3") {
    if (err) *err = "tokenizer: pre-tokenizer '" + pre + "' is not supported (gpt2, llama-bpe / llama3)";
    return false;
  }
  gpt2_split_ = pre == "gpt2";
  return true;
}

std::vector<int32_t> ByteBpeTokenizer::encode(const std::string& text, bool add_bos) const {
  std::vector<int32_t> out;
  if (add_bos && bos_ >= 0) out.push_back(bos_);
  /* special tokens written in the text, longest first at each position */
  size_t seg = 0;
  for (size_t i = 0; i < text.size();) {
    int32_t hit = -1;
    for (int32_t id : special_[(unsigned char)text[i]])
      if (text.compare(i, tokens_[id].size(), tokens_[id]) == 0) {
        hit = id;
        break;
      }
    if (hit < 0) {
      ++i;
      continue;
    }
    encode_segment(text.substr(seg, i - seg), &out);
    out.push_back(hit);
    i += tokens_[hit].size();
    seg = i;
  }
  encode_segment(text.substr(seg), &out);
  return out;
}

void ByteBpeTokenizer::encode_segment(const std::string& text, std::vector<int32_t>* outp) const {
  std::vector<int32_t>& out = *outp;
  std::vector<uint32_t> cps;
  std::vector<size_t> offs;
  code_points(text, &cps, &offs);
  for (size_t i = 0; i < cps.size();) {
    const size_t e = gpt2_split_ ? split_piece_gpt2(cps, i) : split_piece(cps, i);
    std::vector<std::string> sym;
    std::string word;
    for (size_t b = offs[i]; b < offs[e]; ++b) {
      sym.push_back(byte_char_[(unsigned char)text[b]]);
      word += sym.back();
    }
    i = e;
    auto whole = gpt2_split_ ? id_.end() : id_.find(word);
    if (whole != id_.end()) { /* a piece that is a token is not split (ignore_merges) */
      out.push_back(whole->second);
      continue;
    }
    while (sym.size() > 1) {
      int best = -1;
      int32_t best_rank = 0;
      for (size_t k = 0; k + 1 < sym.size(); ++k) {
        auto it = rank_.find(sym[k] + " " + sym[k + 1]);
        if (it != rank_.end() && (best < 0 || it->second < best_rank)) {
          best = (int)k;
          best_rank = it->second;
        }
      }
      if (best < 0) break;
      sym[best] += sym[best + 1];
      sym.erase(sym.begin() + best + 1);
    }
    for (const std::string& s : sym) {
      auto it = id_.find(s);
      if (it != id_.end()) out.push_back(it->second);
    }
  }
}

std::string ByteBpeTokenizer::decode(const std::vector<int32_t>& ids) const {
  std::string bytes;
  for (int32_t id : ids) {
    if (id < 0 || (size_t)id >= tokens_.size()) continue;
    const int t = types_[id];
    if (t == SpmTokenizer::CONTROL || t == SpmTokenizer::UNUSED) continue;
    const std::string& p = tokens_[id];
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    code_points(p, &cps, &offs);
    for (size_t k = 0; k < cps.size(); ++k) {
      auto it = char_byte_.find(cps[k]);
      if (it != char_byte_.end() && t != SpmTokenizer::USER_DEFINED) bytes.push_back((char)it->second);
      else bytes.append(p, offs[k], offs[k + 1] - offs[k]); /* added tokens keep their text */
    }
  }
  return bytes_to_utf8(bytes);
}

bool GgufTokenizer::load(const GGUFFile& f, std::string* err) {
  spm_ = SpmTokenizer();
  bpe_ = ByteBpeTokenizer();
  const std::string model = f.str("tokenizer.ggml.model", "");
  if (model == "gpt2") return bpe_.load(f, err);
  return spm_.load(f, err);
}

}  // namespace ulbe
