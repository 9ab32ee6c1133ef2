/*
 * gguf.h — GGUF container reader and the synthetic-model writer.
 *
 * The reader follows the reference's GGUFParser (src/core/gguf_parser.cpp:18-361: header,
 * KV metadata, tensor infos, data offset aligned to general.alignment) but sizes tensors
 * with the GGUF block table (Q4_0: 18 B per 32 weights, Q4_K: 144 B per 256) instead of
 * ggml_type_size (src/core/gguf_types.h:35-58), which returns 6 and 12 for those types and
 * makes the reference read only a prefix of every quantised tensor.  The file is mapped
 * read-only; tensor data pointers point into the mapping.
 */
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ulbe {

struct GGUFTensor {
  std::string name;
  int type = 0;
  int n_dims = 0;
  uint64_t ne[4] = {1, 1, 1, 1};
  uint64_t offset = 0;
  size_t nbytes = 0;
  const uint8_t* data = nullptr;
};

class GGUFFile {
 public:
  GGUFFile() = default;
  GGUFFile(const GGUFFile&) = delete;
  GGUFFile& operator=(const GGUFFile&) = delete;
  ~GGUFFile();

  bool open(const std::string& path, std::string* err);
  const GGUFTensor* find(const std::string& name) const;
  bool has(const std::string& key) const { return num_.count(key) || str_.count(key); }
  double num(const std::string& key, double dflt) const;
  std::string str(const std::string& key, const std::string& dflt) const;
  /* array metadata (tokenizer.ggml.tokens / scores / token_type ...); nullptr if absent */
  const std::vector<std::string>* str_array(const std::string& key) const;
  const std::vector<double>* num_array(const std::string& key) const;

  uint32_t version = 0;
  uint64_t alignment = 32;
  std::vector<GGUFTensor> tensors;
  size_t file_bytes = 0;

 private:
  void* map_ = nullptr;
  size_t map_len_ = 0;
  std::map<std::string, double> num_;
  std::map<std::string, std::string> str_;
  std::map<std::string, std::vector<std::string>> strarr_;
  std::map<std::string, std::vector<double>> numarr_;
};

/* bytes of n elements of a GGML type; 0 if unsupported or not a whole number of blocks */
size_t gguf_type_nbytes(int type, uint64_t n);

/* LLaMA-architecture synthetic model: linear weights N(0, 0.02) quantised to Q4_0 or Q4_K,
 * token_embd fp16 N(0, 0.02), norms 1.0.  Every tensor draws from its own Philox stream keyed
 * by (seed, tensor name), so two models with the same seed share identically named tensors. */
struct SynthSpec {
  std::string name = "synthetic-llama";
  int n_layer = 2, d_model = 512, n_head = 8, n_head_kv = 8, d_ff = 1408, n_vocab = 32000, ctx_len = 4096;
  float rms_eps = 1e-5f, rope_base = 10000.f;
  int wtype = 2; /* Q4_0 = 2, Q4_K = 12 */
  int embd_type = 1;  /* token_embd: F32 = 0, F16 = 1, or Q4_0 / Q8_0 = 8 / Q4_K / Q6_K = 14 */
  int out_type = -1;  /* output.weight: Q4_0 / Q8_0 / Q4_K / Q6_K; -1 = wtype */
  /* attn_v / attn_output / ffn_down of every layer: Q4_0 / Q8_0 / Q4_K / Q6_K, -1 = wtype (a
     K-quant mix such as llama.cpp's Q4_K_M puts Q6_K in attn_v and ffn_down) */
  int v_type = -1, o_type = -1, down_type = -1;
  bool tied = false;  /* no output.weight: the LM head is token_embd (tied embeddings) */
  uint64_t seed = 0;
  float stddev = 0.02f;
  /* optional SentencePiece vocabulary, written as tokenizer.ggml.{model, tokens, scores,
     token_type, bos_token_id, eos_token_id, unknown_token_id} */
  std::vector<std::string> vocab;
  std::vector<float> scores;
  std::vector<int32_t> token_types;
  std::vector<std::string> merges; /* non-empty: a byte-level BPE ("gpt2") vocabulary */
  std::string tok_pre;             /* tokenizer.ggml.pre, written when non-empty */
  int add_bos = -1, add_space_prefix = -1; /* tokenizer.ggml.add_bos_token / add_space_prefix; -1: not written */
};

bool write_synthetic_gguf(const std::string& path, const SynthSpec& spec, int threads, std::string* err);

/* quantisers (exposed for tests) */
void quantize_q4_0(const float* x, uint64_t n, uint8_t* out);
void quantize_q4_k(const float* x, uint64_t n, uint8_t* out);
void quantize_q8_0(const float* x, uint64_t n, uint8_t* out);
void quantize_q6_k(const float* x, uint64_t n, uint8_t* out);
/* the N(0,1) sample number i of the stream keyed by (seed, name) */
double synth_normal(uint64_t seed, const std::string& name, uint64_t i);

}  // namespace ulbe
