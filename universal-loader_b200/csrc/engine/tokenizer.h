/*
 * tokenizer.h — the GGUF "llama" tokenizer (a SentencePiece BPE vocabulary stored as
 * tokenizer.ggml.tokens / scores / token_type) for the text surface of InferenceAPI.
 *
 * The reference's engine tokenizes with a placeholder (src/inference/tokenizer.cpp:13-64:
 * whitespace-split words looked up as decimal id strings) and never reads the GGUF vocabulary;
 * its BPETokenizer (src/inference/bpe_tokenizer.cpp:19-243) reads a private text format and is
 * not wired in.  This class is what a GGUF LLaMA checkpoint needs instead: SentencePiece BPE
 * encoding as the sentencepiece library performs it for LLaMA's model (identity normaliser,
 * a dummy-prefix space, spaces as U+2581, byte fallback).
 *
 * encode: the text (with "▁" prepended unless the file's tokenizer.ggml.add_space_prefix is
 * false, and every ' ' replaced by "▁") is split into user-defined pieces (longest match at
 * each position; these never merge further) and otherwise UTF-8
 * characters; the adjacent pair whose concatenation is a NORMAL or USER_DEFINED piece with
 * the highest score is merged (the leftmost pair on equal scores) until no pair merges; a
 * final symbol that is not a piece becomes its bytes' <0xXX> pieces (or the unknown id).
 * decode: pieces concatenated with "▁" as ' ', runs of <0xXX> pieces as UTF-8 (U+FFFD for
 * each byte that starts no valid character), control pieces dropped, the unknown piece as
 * " ⁇ ", and the leading space of the dummy prefix removed -- always valid UTF-8.
 */
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace ulbe {

class GGUFFile;

/* b as valid UTF-8: each valid character kept, every other byte as U+FFFD */
std::string bytes_to_utf8(const std::string& b);

class SpmTokenizer {
 public:
  /* GGUF token types (as tokenizer.ggml.token_type stores them) */
  enum { NORMAL = 1, UNKNOWN = 2, CONTROL = 3, USER_DEFINED = 4, UNUSED = 5, BYTE = 6 };

  /* from a GGUF file with tokenizer.ggml.model == "llama"; false (and *err) otherwise */
  bool load(const GGUFFile& f, std::string* err);
  /* from explicit pieces, scores and types (equal lengths) */
  bool load(const std::vector<std::string>& pieces, const std::vector<float>& scores,
            const std::vector<int32_t>& types, int bos, int eos, int unk, std::string* err);
  /* tokenizer.ggml.add_bos_token / add_space_prefix (both true unless the file says false):
     whether text calls prepend BOS, and whether encode prepends the dummy-prefix space (and
     decode removes it) */
  void set_flags(bool add_bos, bool add_space_prefix) {
    add_bos_ = add_bos;
    add_space_prefix_ = add_space_prefix;
  }
  bool add_bos() const { return add_bos_; }

  std::vector<int32_t> encode(const std::string& text, bool add_bos) const;
  std::string decode(const std::vector<int32_t>& ids) const;

  bool loaded() const { return !pieces_.empty(); }
  int bos() const { return bos_; }
  int eos() const { return eos_; }
  size_t size() const { return pieces_.size(); }

 private:
  std::vector<std::string> pieces_;
  std::vector<float> scores_;
  std::vector<int32_t> types_;
  std::unordered_map<std::string, int32_t> mergeable_; /* NORMAL / USER_DEFINED pieces */
  std::vector<int32_t> user_[256]; /* USER_DEFINED pieces by first byte, longest first */
  int32_t byte_id_[256];
  int bos_ = 1, eos_ = 2, unk_ = 0;
  bool add_bos_ = true, add_space_prefix_ = true;
};

/*
 * The GGUF "gpt2" tokenizer of Llama-3 files: byte-level BPE over tokenizer.ggml.tokens and
 * tokenizer.ggml.merges ("a b", rank = position), as the HF tokenizers library runs
 * Llama-3's tokenizer.json.
 * encode: the text is split by Llama-3's pattern
 *   (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|
 *   \s*[\r\n]+|\s+(?!\S)|\s+
 * (written out as a scanner; \p{L} / \p{N} from unicode_ranges.h, \s = White_Space); each
 * piece's UTF-8 bytes become GPT-2's printable byte characters; a piece that is itself a token
 * is emitted whole (ignore_merges), else the adjacent pair of lowest merge rank is merged (the
 * leftmost on equal ranks) until none merges.  Files whose tokenizer.ggml.pre is "gpt2"
 * split with GPT-2's own pattern ('s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+|
 * ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+) and always apply the merges.  Control and user-defined tokens written in the
 * text (<|eot_id|>, ...) are split out first, longest match at each position, and the text
 * between them is encoded as above.
 * decode: tokens concatenated, byte characters mapped back to bytes, the bytes as UTF-8
 * (U+FFFD for each byte that starts no valid character); control tokens dropped.
 */
class ByteBpeTokenizer {
 public:
  bool load(const GGUFFile& f, std::string* err);
  std::vector<int32_t> encode(const std::string& text, bool add_bos) const;
  std::string decode(const std::vector<int32_t>& ids) const;
  bool loaded() const { return !tokens_.empty(); }
  bool add_bos() const { return add_bos_; }

 private:
  void encode_segment(const std::string& text, std::vector<int32_t>* out) const;
  std::vector<std::string> tokens_;
  std::vector<int32_t> types_;
  std::unordered_map<std::string, int32_t> id_;
  std::unordered_map<std::string, int32_t> rank_; /* "a b" -> merge rank */
  std::vector<int32_t> special_[256];             /* control / user-defined tokens by first byte,
                                                     longest first: split out of text as is */
  std::string byte_char_[256];                     /* byte -> its printable character (UTF-8) */
  std::unordered_map<uint32_t, uint8_t> char_byte_; /* code point -> byte */
  int bos_ = -1;
  bool add_bos_ = true;
  bool gpt2_split_ = false; /* tokenizer.ggml.pre = gpt2: GPT-2's pattern, merges always applied */
};

/* the text tokenizer of a GGUF file: SentencePiece ("llama") or byte-level BPE ("gpt2") */
class GgufTokenizer {
 public:
  bool load(const GGUFFile& f, std::string* err);
  std::vector<int32_t> encode(const std::string& text, bool add_bos) const {
    return spm_.loaded() ? spm_.encode(text, add_bos) : bpe_.encode(text, add_bos);
  }
  std::string decode(const std::vector<int32_t>& ids) const {
    return spm_.loaded() ? spm_.decode(ids) : bpe_.decode(ids);
  }
  bool loaded() const { return spm_.loaded() || bpe_.loaded(); }
  bool add_bos() const { return spm_.loaded() ? spm_.add_bos() : bpe_.add_bos(); }

 private:
  SpmTokenizer spm_;
  ByteBpeTokenizer bpe_;
};

}  // namespace ulbe
