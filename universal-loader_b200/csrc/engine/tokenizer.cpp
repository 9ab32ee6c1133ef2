/* tokenizer.cpp — SentencePiece BPE over a GGUF vocabulary (see tokenizer.h). */
#include "tokenizer.h"

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
  for (int i = 0; i < 256; ++i) byte_id_[i] = -1;
  for (size_t i = 0; i < pieces_.size(); ++i) {
    const int t = types_[i];
    if (t == NORMAL || t == USER_DEFINED) {
      mergeable_.emplace(pieces_[i], (int32_t)i); /* the first id of a duplicated piece wins */
    } else if (t == BYTE) {
      unsigned v = 0;
      if (pieces_[i].size() == 6 && std::sscanf(pieces_[i].c_str(), "<0x%02X>", &v) == 1 && v < 256)
        byte_id_[v] = (int32_t)i;
    }
  }
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
  };
  std::vector<Sym> sym;
  for (size_t o = 0; o < norm.size();) {
    size_t l = utf8_len((unsigned char)norm[o]);
    if (o + l > norm.size()) l = norm.size() - o;
    sym.push_back({o, l, (int)sym.size() - 1, (int)sym.size() + 1});
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
    if (l < 0 || r < 0) return;
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
