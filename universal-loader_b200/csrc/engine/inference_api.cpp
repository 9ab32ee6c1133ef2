/*
 * inference_api.cpp — the Python module `vulkangguf`, a drop-in for the reference's
 * pybind11 module of the same name (src/api/inference_api.{h,cpp}; class and method list
 * as inference_api.h:14-123 and the PYBIND11_MODULE at inference_api.cpp:389-473).
 *
 * Behaviour kept from the reference:
 *  - GenerationConfig() value-initialises every field to zero (the reference binds the
 *    aggregate with pybind11::init(), inference_api.cpp:430): a bare config asks for 0
 *    tokens and, with temperature 0, greedy decoding.
 *  - generate() returns a str; "Error: No model loaded" without a model
 *    (inference_api.cpp:59-61); methods lock one API mutex (inference_api.h:115).
 * What changes on this path:
 *  - enable_speculative_decoding(True) is wired (the reference's is a no-op,
 *    inference_api.cpp:214-216): with a draft model loaded, generation runs the device
 *    draft -> verify -> accept loop; without one it logs and decodes plainly.
 *  - temperature / top_p / top_k / do_sample reach the sampler (the reference drops them in
 *    convert_config, inference_api.cpp:380-387).  Greedy <=> do_sample False or T == 0.
 *  - get_acceptance_rate() / get_throughput() report the last generation (the reference
 *    returns 0, inference_engine.cpp:793-799).
 * Additions (the reference cannot name a draft model): load_draft_model, unload_draft_model,
 * set_speculation_length (as SpeculativeDecoder::set_speculation_length,
 * speculative_decoder.h:40), enable_tree_speculation (TreeSpeculation's beam_width /
 * max_depth, speculative_decoder.h:62-87), set_seed, GenerationConfig.seed, generate_tokens,
 * get_last_stats, and the module function write_synthetic_gguf.
 * Text: a registered custom tokenizer first; else the target GGUF's SentencePiece vocabulary
 * (tokenizer.ggml.*, tokenizer.cpp) when it has one; else byte-fallback ids (byte b -> id
 * b + 3) and back.
 */
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cctype>
#include <chrono>
#include <map>
#include <cstdio>
#include <functional>
#include <mutex>
#include <sstream>
#include <thread>

#include "gguf.h"
#include "spec_engine.h"
#include "tokenizer.h"

namespace py = pybind11;

namespace vg {

struct GenerationConfig {
  uint32_t max_tokens;
  float temperature;
  float top_p;
  uint32_t top_k;
  float frequency_penalty;
  float presence_penalty;
  bool do_sample;
  uint64_t seed;
};

struct GenerationResult {
  std::vector<uint32_t> tokens;
  std::string text;
  uint32_t num_tokens = 0;
  float time_ms = 0;
  float tokens_per_second = 0;
};

struct GenerationProgress {
  uint32_t current_step = 0;
  uint32_t total_steps = 0;
  float progress_pct = 0;
  float time_elapsed_ms = 0;
  float estimated_remaining_ms = 0;
  float tokens_per_second = 0;
  std::string last_token;
};

struct ModelMetrics {
  uint32_t vocab_size = 0;
  uint32_t num_layers = 0;
  uint32_t hidden_dim = 0;
  uint32_t context_len = 0;
  uint32_t num_heads = 0;
  size_t model_size_bytes = 0;
  std::string architecture;
};

/* as the reference's inference::QuantizationType (src/inference/quantization_manager.h) */
enum class QuantizationType { NONE = 0, FP32, FP16, INT8, FP4, NF4 };

std::string quantization_type_name(QuantizationType t) {
  switch (t) {
    case QuantizationType::NONE: return "NONE";
    case QuantizationType::FP32: return "FP32";
    case QuantizationType::FP16: return "FP16";
    case QuantizationType::INT8: return "INT8";
    case QuantizationType::FP4: return "FP4";
    case QuantizationType::NF4: return "NF4";
  }
  return "UNKNOWN";
}

class InferenceAPI {
 public:
  InferenceAPI() {
    /* the reference's internal defaults (inference_api.cpp:9-17) */
    config_.max_tokens = 100;
    config_.temperature = 1.0f;
    config_.top_p = 0.9f;
    config_.top_k = 40;
    config_.frequency_penalty = 0.f;
    config_.presence_penalty = 0.f;
    config_.do_sample = true;
    config_.seed = 0;
  }

  /* Tensor parallelism (addition; the reference's enable_multi_gpu is a flag with no effect):
     join an NCCL communicator of `world` processes, one GPU each, before load_model; the
     target is then split over the ranks and the draft replicated. */
  bool init_tensor_parallel(int rank, int world, const py::bytes& nccl_id) {
    std::lock_guard<std::mutex> lk(mu_);
    const std::string id = nccl_id;
    if (id.size() != 128) {
      std::fprintf(stderr, "[InferenceAPI] init_tensor_parallel: the NCCL id must be 128 bytes\n");
      return false;
    }
    if (!engine_) engine_.reset(new ulbe::Engine(0));
    const bool ok = engine_->ok() && engine_->init_tp(rank, world, id.data());
    if (!ok) std::fprintf(stderr, "[InferenceAPI] init_tensor_parallel: %s\n", engine_->error().c_str());
    return ok;
  }
  /* bound (seconds) on every wait for tensor-parallel work: past it the communicator is
     aborted and the generation raises instead of blocking on a peer that is gone */
  bool set_collective_timeout(double seconds) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!engine_) return false;
    const bool ok = engine_->set_tp_timeout((int)(seconds * 1000.0));
    if (!ok) std::fprintf(stderr, "[InferenceAPI] set_collective_timeout: %s\n", engine_->error().c_str());
    return ok;
  }


  bool load_model(const std::string& path) { return load(path, false); }
  bool load_draft_model(const std::string& path) { return load(path, true); }

  bool unload_model() {
    std::lock_guard<std::mutex> lk(mu_);
    if (engine_) engine_->unload(false);
    return true;
  }
  bool unload_draft_model() {
    std::lock_guard<std::mutex> lk(mu_);
    if (engine_) engine_->unload(true);
    return true;
  }

  std::string generate(const std::string& prompt, const GenerationConfig& cfg) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!engine_ || !engine_->has_model(false)) return "Error: No model loaded";
    std::vector<std::vector<int32_t>> out;
    if (!run({encode(prompt)}, cfg, &out)) return "Error: " + engine_->error();
    return decode(out[0]);
  }

  GenerationResult generate_default(const std::string& prompt) {
    std::lock_guard<std::mutex> lk(mu_);
    GenerationResult r;
    if (!engine_ || !engine_->has_model(false)) {
      r.text = "Error: No model loaded";
      return r;
    }
    std::vector<std::vector<int32_t>> out;
    if (!run({encode(prompt)}, config_, &out)) {
      r.text = "Error: " + engine_->error();
      return r;
    }
    r.tokens.assign(out[0].begin(), out[0].end());
    r.text = decode(out[0]);
    r.num_tokens = (uint32_t)out[0].size();
    r.time_ms = (float)last_.total_ms;
    r.tokens_per_second = last_.total_ms > 0 ? (float)(out[0].size() * 1000.0 / last_.total_ms) : 0.f;
    return r;
  }

  std::vector<std::string> generate_batch(const std::vector<std::string>& prompts, const GenerationConfig& cfg) {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<std::string> res(prompts.size());
    if (!engine_ || !engine_->has_model(false)) {
      for (auto& s : res) s = "Error: No model loaded";
      return res;
    }
    std::vector<std::vector<int32_t>> in, out;
    for (const auto& p : prompts) in.push_back(encode(p));
    if (!run(in, cfg, &out)) {
      for (auto& s : res) s = "Error: " + engine_->error();
      return res;
    }
    for (size_t i = 0; i < res.size(); ++i) res[i] = decode(out[i]);
    return res;
  }

  std::string generate_streaming(const std::string& prompt, const GenerationConfig& cfg,
                                 std::function<void(const std::string&)> cb) {
    std::vector<std::vector<int32_t>> out;
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (!engine_ || !engine_->has_model(false)) return "Error: No model loaded";
      if (!run({encode(prompt)}, cfg, &out)) return "Error: " + engine_->error();
    }
    std::string all;
    for (int32_t t : out[0]) {
      std::string piece = decode({t});
      all += piece;
      if (cb) cb(piece);
    }
    return all;
  }

  std::string generate_with_progress(const std::string& prompt, const GenerationConfig& cfg,
                                     std::function<void(const GenerationProgress&)> cb) {
    std::vector<std::vector<int32_t>> out;
    double ms = 0;
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (!engine_ || !engine_->has_model(false)) return "Error: No model loaded";
      if (!run({encode(prompt)}, cfg, &out)) return "Error: " + engine_->error();
      ms = last_.total_ms;
    }
    std::string all;
    const size_t n = out[0].size();
    for (size_t i = 0; i < n; ++i) {
      std::string piece = decode({out[0][i]});
      all += piece;
      if (cb) {
        GenerationProgress p;
        p.current_step = (uint32_t)(i + 1);
        p.total_steps = (uint32_t)n;
        p.progress_pct = 100.f * (float)(i + 1) / (float)n;
        p.time_elapsed_ms = (float)(ms * (i + 1) / n);
        p.estimated_remaining_ms = (float)(ms - p.time_elapsed_ms);
        p.tokens_per_second = ms > 0 ? (float)(n * 1000.0 / ms) : 0.f;
        p.last_token = piece;
        cb(p);
      }
    }
    return all;
  }

  /* token ids in, token ids out: list[int] -> list[int], or list[list[int]] -> list[list[int]] */
  py::object generate_tokens(py::object prompts, const GenerationConfig& cfg) {
    std::vector<std::vector<int32_t>> in, out;
    bool single = false;
    if (py::isinstance<py::list>(prompts) && py::len(prompts) > 0 && py::isinstance<py::int_>(prompts.cast<py::list>()[0])) {
      single = true;
      in.push_back(prompts.cast<std::vector<int32_t>>());
    } else {
      in = prompts.cast<std::vector<std::vector<int32_t>>>();
    }
    bool ok;
    std::string err;
    {
      py::gil_scoped_release rel;
      std::lock_guard<std::mutex> lk(mu_);
      if (!engine_ || !engine_->has_model(false)) {
        ok = false;
        err = "no model loaded";
      } else {
        ok = run(in, cfg, &out);
        if (!ok) err = engine_->error();
      }
    }
    if (!ok) throw std::runtime_error(err);
    if (single) return py::cast(out[0]);
    return py::cast(out);
  }

  bool enable_gpu(bool enable) {
    if (!enable) std::fprintf(stderr, "[InferenceAPI] this engine has no CPU path; GPU stays enabled\n");
    return enable;
  }
  bool is_gpu_enabled() const { return true; }

  ModelMetrics get_model_info() const {
    std::lock_guard<std::mutex> lk(mu_);
    ModelMetrics m;
    if (!engine_ || !engine_->has_model(false)) return m;
    const ulbe::ModelInfo& i = engine_->info(false);
    m.vocab_size = i.n_vocab;
    m.num_layers = i.n_layer;
    m.hidden_dim = i.d_model;
    m.context_len = i.ctx_len;
    m.num_heads = i.n_head;
    m.model_size_bytes = i.file_bytes;
    m.architecture = "llama";
    return m;
  }
  std::string get_model_architecture() const { return "llama"; }

  void set_max_batch_size(uint32_t n) { std::lock_guard<std::mutex> lk(mu_); max_batch_ = n; }
  void enable_speculative_decoding(bool e) {
    std::lock_guard<std::mutex> lk(mu_);
    spec_enabled_ = e;
    if (e && (!engine_ || !engine_->has_model(true)))
      std::fprintf(stderr, "[InferenceAPI] speculative decoding enabled but no draft model is loaded: decoding plainly\n");
  }
  void enable_multi_gpu(bool e) { std::lock_guard<std::mutex> lk(mu_); multi_gpu_ = e; }
  void set_speculation_length(uint32_t k) { std::lock_guard<std::mutex> lk(mu_); spec_k_ = (int)k; }
  /* TreeSpeculation(vocab, beam_width, max_depth) (speculative_decoder.h:62-87): each round
     drafts a full tree of beam_width children per node and max_depth levels and verifies it
     in one target pass; beam_width <= 1 goes back to a chain of set_speculation_length drafts */
  void enable_tree_speculation(uint32_t beam_width, uint32_t max_depth) {
    std::lock_guard<std::mutex> lk(mu_);
    tree_width_ = beam_width >= 2 ? (int)beam_width : 0;
    if (tree_width_) spec_k_ = (int)max_depth;
  }
  void set_seed(uint64_t s) { std::lock_guard<std::mutex> lk(mu_); config_.seed = s; }

  float get_acceptance_rate() const {
    std::lock_guard<std::mutex> lk(mu_);
    return last_.drafted ? (float)last_.accepted / (float)last_.drafted : 0.f;
  }
  float get_throughput() const {
    std::lock_guard<std::mutex> lk(mu_);
    return last_.decode_ms > 0 ? (float)(last_.generated * 1000.0 / (last_.prefill_ms + last_.decode_ms)) : 0.f;
  }

  void set_temperature(float t) { std::lock_guard<std::mutex> lk(mu_); config_.temperature = t; }
  void set_top_p(float p) { std::lock_guard<std::mutex> lk(mu_); config_.top_p = p; }
  void set_top_k(uint32_t k) { std::lock_guard<std::mutex> lk(mu_); config_.top_k = k; }
  void set_cache_size_mb(size_t mb) { std::lock_guard<std::mutex> lk(mu_); cache_mb_ = mb; }
  void set_num_threads(uint32_t n) { std::lock_guard<std::mutex> lk(mu_); threads_ = n; }
  /* kernels are compiled ahead of time for sm_100a: there is no pipeline cache to persist */
  bool save_pipeline_cache(const std::string&) { return true; }
  bool load_pipeline_cache(const std::string&) { return true; }
  void enable_profiling(bool e) { std::lock_guard<std::mutex> lk(mu_); profiling_ = e; }

  std::string get_performance_report() const {
    std::lock_guard<std::mutex> lk(mu_);
    std::ostringstream o;
    o << "rounds=" << last_.rounds << " drafted=" << last_.drafted << " accepted=" << last_.accepted
      << " committed=" << last_.committed << " generated=" << last_.generated << " prefill_ms=" << last_.prefill_ms
      << " decode_ms=" << last_.decode_ms << " total_ms=" << last_.total_ms;
    return o.str();
  }

  py::dict get_last_stats() const {
    std::lock_guard<std::mutex> lk(mu_);
    py::dict d;
    d["rounds"] = last_.rounds;
    d["drafted"] = last_.drafted;
    d["accepted"] = last_.accepted;
    d["committed"] = last_.committed;
    d["generated"] = last_.generated;
    d["prefill_ms"] = last_.prefill_ms;
    d["decode_ms"] = last_.decode_ms;
    d["total_ms"] = last_.total_ms;
    d["h2d_bytes"] = last_.h2d_bytes;
    d["d2h_bytes"] = last_.d2h_bytes;
    d["launches"] = last_.launches;
    d["admitted"] = last_.admitted;
    d["speculative"] = last_spec_;
    return d;
  }

  py::dict profile_round() {
    float ms[5] = {0, 0, 0, 0, 0};
    bool ok;
    {
      std::lock_guard<std::mutex> lk(mu_);
      ok = engine_ && engine_->profile_round(ms);
    }
    if (!ok) throw std::runtime_error(engine_ ? engine_->error() : std::string("no model loaded"));
    py::dict d;
    d["draft_ms"] = ms[0];
    d["verify_ms"] = ms[1];
    d["accept_ms"] = ms[2];
    d["allreduce_ms"] = ms[3];
    d["allreduces"] = (int)ms[4];
    return d;
  }

  /* the last generation's rounds for sequence `seq`, as SpeculationResult records */
  std::vector<ulbe::SpecRound> get_speculation_results(int seq) {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<ulbe::SpecRound> out;
    if (!engine_) return out;
    if (!engine_->speculation_rounds(seq, &out)) throw std::runtime_error(engine_->error());
    return out;
  }

  std::vector<float> get_token_logits(const std::vector<uint32_t>& tokens) {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<float> out;
    if (!engine_ || !engine_->has_model(false)) return out;
    std::vector<int32_t> t(tokens.begin(), tokens.end());
    if (!engine_->last_logits(t, &out)) throw std::runtime_error(engine_->error());
    return out;
  }

  /* LoRA adapters are not on this path: the calls are accepted and have no effect */
  void set_adapter_alpha(const std::string&, float) {}
  void enable_adapter(const std::string&) {}
  void disable_adapter(const std::string&) {}
  std::vector<std::string> get_loaded_adapters() const { return {}; }

  void set_quantization_enabled(bool e) { std::lock_guard<std::mutex> lk(mu_); quant_enabled_ = e; }
  void set_weight_quantization(const std::string& t) { std::lock_guard<std::mutex> lk(mu_); wq_ = t; }
  void set_activation_quantization(const std::string& t) { std::lock_guard<std::mutex> lk(mu_); aq_ = t; }
  std::string get_quantization_config() const {
    std::lock_guard<std::mutex> lk(mu_);
    return "weights=" + wq_ + " activations=" + aq_ + (quant_enabled_ ? " (enabled)" : " (disabled)");
  }

  void register_custom_tokenizer(std::function<std::vector<uint32_t>(const std::string&)> f) {
    std::lock_guard<std::mutex> lk(mu_);
    tokenizer_ = std::move(f);
  }
  /* kernels are not compiled at run time on this path; the callback is kept but not called */
  void register_custom_kernel(std::function<void(const std::string&, const std::string&)> f) {
    std::lock_guard<std::mutex> lk(mu_);
    kernel_compiler_ = std::move(f);
  }

 private:
  bool load(const std::string& path, bool draft) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!engine_) engine_.reset(new ulbe::Engine(0));
    if (!engine_->ok()) {
      std::fprintf(stderr, "[InferenceAPI] %s\n", engine_->error().c_str());
      return false;
    }
    const bool ok = engine_->load(path, draft);
    if (!ok) std::fprintf(stderr, "[InferenceAPI] load failed: %s\n", engine_->error().c_str());
    if (ok && !draft) {
      /* the target's GGUF vocabulary, when it has one, serves the text surface */
      spm_ = ulbe::GgufTokenizer();
      ulbe::GGUFFile f;
      std::string e;
      if (f.open(path, &e)) spm_.load(f, &e);
    }
    return ok;
  }

  bool run(const std::vector<std::vector<int32_t>>& in, const GenerationConfig& cfg,
           std::vector<std::vector<int32_t>>* out) {
    ulbe::GenParams p;
    p.max_new = cfg.max_tokens;
    p.greedy = !cfg.do_sample || !(cfg.temperature > 0.f);
    p.temperature = cfg.temperature;
    p.top_k = (int)cfg.top_k;
    p.top_p = cfg.top_p;
    p.seed = cfg.seed ? cfg.seed : config_.seed;
    const bool spec = spec_enabled_ && engine_->has_model(true) && spec_k_ > 0;
    p.k = spec ? spec_k_ : 0;
    p.tree_width = spec ? tree_width_ : 0;
    p.max_batch = (int)max_batch_;
    last_spec_ = spec;
    return engine_->generate(in, p, out, &last_);
  }

  std::vector<int32_t> encode(const std::string& s) const {
    std::vector<int32_t> ids;
    if (tokenizer_) {
      py::gil_scoped_acquire g;
      for (uint32_t t : tokenizer_(s)) ids.push_back((int32_t)t);
    } else if (spm_.loaded()) {
      ids = spm_.encode(s, spm_.add_bos());
    } else {
      for (unsigned char c : s) ids.push_back((int32_t)c + 3);
    }
    if (ids.empty()) ids.push_back(1); /* BOS for an empty prompt */
    return ids;
  }

  std::string decode(const std::vector<int32_t>& ids) const {
    if (!tokenizer_ && spm_.loaded()) return spm_.decode(ids);
    /* byte-fallback ids: runs of bytes as UTF-8 (U+FFFD for invalid bytes), others as <id> */
    std::string s, run;
    for (int32_t t : ids) {
      if (t >= 3 && t < 259) {
        run.push_back((char)(t - 3));
        continue;
      }
      s += ulbe::bytes_to_utf8(run);
      run.clear();
      s += "<" + std::to_string(t) + ">";
    }
    return s + ulbe::bytes_to_utf8(run);
  }

  mutable std::mutex mu_;
  std::unique_ptr<ulbe::Engine> engine_;
  GenerationConfig config_{};
  bool spec_enabled_ = false, multi_gpu_ = false, profiling_ = false, quant_enabled_ = false, last_spec_ = false;
  int spec_k_ = 5;
  int tree_width_ = 0;
  uint32_t max_batch_ = 64, threads_ = 8;
  size_t cache_mb_ = 1024;
  std::string wq_ = "NONE", aq_ = "NONE";
  ulbe::GenStats last_;
  std::function<std::vector<uint32_t>(const std::string&)> tokenizer_;
  ulbe::GgufTokenizer spm_; /* the loaded target's GGUF vocabulary, if it has one */
  std::function<void(const std::string&, const std::string&)> kernel_compiler_;
};

bool write_synthetic(const std::string& path, py::dict spec, int threads) {
  ulbe::SynthSpec s;
  auto geti = [&](const char* k, int& v) { if (spec.contains(k)) v = spec[k].cast<int>(); };
  auto getf = [&](const char* k, float& v) { if (spec.contains(k)) v = spec[k].cast<float>(); };
  geti("n_layer", s.n_layer);
  geti("d_model", s.d_model);
  geti("n_head", s.n_head);
  s.n_head_kv = s.n_head;
  geti("n_head_kv", s.n_head_kv);
  geti("d_ff", s.d_ff);
  geti("n_vocab", s.n_vocab);
  geti("ctx_len", s.ctx_len);
  getf("rms_eps", s.rms_eps);
  getf("rope_base", s.rope_base);
  getf("stddev", s.stddev);
  if (spec.contains("wtype")) {
    py::object w = spec["wtype"];
    if (py::isinstance<py::str>(w)) {
      const std::string ws = w.cast<std::string>();
      s.wtype = (ws == "q4_k" || ws == "Q4_K") ? 12 : 2;
    } else {
      s.wtype = w.cast<int>();
    }
  }
  /* tensor types by GGML id or name */
  auto type_of = [&](const char* k, int& v) {
    if (!spec.contains(k)) return;
    py::object o = spec[k];
    if (!py::isinstance<py::str>(o)) { v = o.cast<int>(); return; }
    std::string n = o.cast<std::string>();
    for (char& ch : n) ch = (char)std::tolower((unsigned char)ch);
    const std::map<std::string, int> ids = {{"f32", 0}, {"f16", 1}, {"q4_0", 2}, {"q8_0", 8}, {"q4_k", 12}, {"q6_k", 14}};
    auto it = ids.find(n);
    if (it == ids.end()) throw std::runtime_error(std::string(k) + ": unknown tensor type " + n);
    v = it->second;
  };
  type_of("embd_type", s.embd_type);
  if (spec.contains("tied")) s.tied = spec["tied"].cast<bool>();
  type_of("out_type", s.out_type);
  type_of("v_type", s.v_type);
  type_of("o_type", s.o_type);
  type_of("down_type", s.down_type);
  if (spec.contains("vocab")) {
    s.vocab = spec["vocab"].cast<std::vector<std::string>>();
    s.scores = spec.contains("scores") ? spec["scores"].cast<std::vector<float>>() : std::vector<float>(s.vocab.size(), 0.f);
    s.token_types = spec.contains("token_types") ? spec["token_types"].cast<std::vector<int32_t>>()
                                                 : std::vector<int32_t>(s.vocab.size(), 1);
    if (spec.contains("merges")) s.merges = spec["merges"].cast<std::vector<std::string>>();
    if (spec.contains("tokenizer_pre")) s.tok_pre = spec["tokenizer_pre"].cast<std::string>();
    if (spec.contains("add_bos")) s.add_bos = spec["add_bos"].cast<bool>() ? 1 : 0;
    if (spec.contains("add_space_prefix")) s.add_space_prefix = spec["add_space_prefix"].cast<bool>() ? 1 : 0;
  }
  if (spec.contains("seed")) s.seed = spec["seed"].cast<uint64_t>();
  if (spec.contains("name")) s.name = spec["name"].cast<std::string>();
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  std::string err;
  bool ok;
  {
    py::gil_scoped_release rel;
    ok = ulbe::write_synthetic_gguf(path, s, threads, &err);
  }
  if (!ok) throw std::runtime_error(err);
  return true;
}

}  // namespace vg

/* the GGUF file's SentencePiece tokenizer, for text <-> ids without loading the model */
static ulbe::GgufTokenizer gguf_spm(const std::string& path) {
  ulbe::GGUFFile f;
  std::string err;
  if (!f.open(path, &err)) throw std::runtime_error(err);
  ulbe::GgufTokenizer t;
  if (!t.load(f, &err)) throw std::runtime_error(err);
  return t;
}

PYBIND11_MODULE(vulkangguf, m) {
  using namespace vg;
  py::class_<InferenceAPI>(m, "InferenceAPI")
      .def(py::init())
      .def("load_model", &InferenceAPI::load_model, "Load a GGUF model from disk")
      .def("unload_model", &InferenceAPI::unload_model, "Unload the current model")
      .def("generate", &InferenceAPI::generate, "Generate text from a prompt with custom config",
           py::call_guard<py::gil_scoped_release>())
      .def("generate_default", &InferenceAPI::generate_default, "Generate text with default config",
           py::call_guard<py::gil_scoped_release>())
      .def("generate_streaming", &InferenceAPI::generate_streaming, py::arg("prompt"), py::arg("config"),
           py::arg("token_callback"), "Generate text with streaming callback for each token")
      .def("generate_with_progress", &InferenceAPI::generate_with_progress, py::arg("prompt"), py::arg("config"),
           py::arg("progress_callback"), "Generate text with progress callback containing statistics")
      .def("generate_batch", &InferenceAPI::generate_batch, "Generate text for multiple prompts",
           py::call_guard<py::gil_scoped_release>())
      .def("enable_gpu", &InferenceAPI::enable_gpu, "Enable or disable GPU acceleration")
      .def("is_gpu_enabled", &InferenceAPI::is_gpu_enabled, "Check if GPU is enabled")
      .def("get_model_info", &InferenceAPI::get_model_info, "Get model metadata and metrics")
      .def("get_model_architecture", &InferenceAPI::get_model_architecture, "Get model architecture name")
      .def("set_max_batch_size", &InferenceAPI::set_max_batch_size, "Set maximum batch size")
      .def("enable_speculative_decoding", &InferenceAPI::enable_speculative_decoding,
           "Enable or disable speculative decoding")
      .def("enable_multi_gpu", &InferenceAPI::enable_multi_gpu, "Enable or disable multi-GPU")
      .def("get_acceptance_rate", &InferenceAPI::get_acceptance_rate, "Get speculative decoding acceptance rate")
      .def("get_throughput", &InferenceAPI::get_throughput, "Get current throughput in tokens/second")
      .def("set_temperature", &InferenceAPI::set_temperature, "Set sampling temperature")
      .def("set_top_p", &InferenceAPI::set_top_p, "Set nucleus sampling parameter")
      .def("set_top_k", &InferenceAPI::set_top_k, "Set top-k sampling parameter")
      .def("set_cache_size_mb", &InferenceAPI::set_cache_size_mb, "Set GPU cache size in MB")
      .def("set_num_threads", &InferenceAPI::set_num_threads, "Set number of CPU threads")
      .def("save_pipeline_cache", &InferenceAPI::save_pipeline_cache, "Save pipeline cache to disk")
      .def("load_pipeline_cache", &InferenceAPI::load_pipeline_cache, "Load pipeline cache from disk")
      .def("enable_profiling", &InferenceAPI::enable_profiling, "Enable performance profiling")
      .def("get_performance_report", &InferenceAPI::get_performance_report, "Get performance metrics report")
      .def("get_token_logits", &InferenceAPI::get_token_logits, "Get logits for generated tokens",
           py::call_guard<py::gil_scoped_release>())
      .def("set_adapter_alpha", &InferenceAPI::set_adapter_alpha, "Set LoRA adapter alpha value")
      .def("enable_adapter", &InferenceAPI::enable_adapter, "Enable a LoRA adapter")
      .def("disable_adapter", &InferenceAPI::disable_adapter, "Disable a LoRA adapter")
      .def("get_loaded_adapters", &InferenceAPI::get_loaded_adapters, "Get list of loaded adapters")
      .def("set_quantization_enabled", &InferenceAPI::set_quantization_enabled, "Enable or disable quantization")
      .def("set_weight_quantization", &InferenceAPI::set_weight_quantization, "Set weight quantization type")
      .def("set_activation_quantization", &InferenceAPI::set_activation_quantization,
           "Set activation quantization type")
      .def("get_quantization_config", &InferenceAPI::get_quantization_config, "Get quantization configuration")
      .def("register_custom_tokenizer", &InferenceAPI::register_custom_tokenizer, "Register custom tokenizer function")
      .def("register_custom_kernel", &InferenceAPI::register_custom_kernel,
           "Register custom shader compiler function")
      /* additions for the speculative path */
      .def("load_draft_model", &InferenceAPI::load_draft_model, "Load the GGUF draft model for speculative decoding")
      .def("set_collective_timeout", &InferenceAPI::set_collective_timeout, py::arg("seconds"),
           "Bound on waits for tensor-parallel work; past it the communicator is aborted and the call raises")
      .def("init_tensor_parallel", &InferenceAPI::init_tensor_parallel, py::arg("rank"), py::arg("world"),
           py::arg("nccl_id"), "Join a tensor-parallel NCCL communicator before load_model (one GPU per process)")
      .def("unload_draft_model", &InferenceAPI::unload_draft_model, "Unload the draft model")
      .def("set_speculation_length", &InferenceAPI::set_speculation_length, "Draft tokens per round (k)")
      .def("enable_tree_speculation", &InferenceAPI::enable_tree_speculation, py::arg("beam_width"),
           py::arg("max_depth"),
           "Tree speculation: beam_width candidates per node, max_depth levels per round (beam_width < 2: chain)")
      .def("set_seed", &InferenceAPI::set_seed, "Seed of the Philox sampler")
      .def("generate_tokens", &InferenceAPI::generate_tokens, py::arg("prompt_tokens"), py::arg("config"),
           "Generate from token ids; list[int] -> list[int] or list[list[int]] -> list[list[int]]")
      .def("get_last_stats", &InferenceAPI::get_last_stats, "Statistics of the last generation")
      .def("get_speculation_results", &InferenceAPI::get_speculation_results, py::arg("seq") = 0,
           "Per-round SpeculationResult records of sequence `seq` of the last generation")
      .def("profile_round", &InferenceAPI::profile_round,
           "Run one more round of the last generation's loop, timed by phase (draft / verify / accept)");

  py::class_<GenerationConfig>(m, "GenerationConfig")
      .def(py::init([]() { return GenerationConfig{}; }))
      .def_readwrite("max_tokens", &GenerationConfig::max_tokens, "Maximum number of tokens to generate")
      .def_readwrite("temperature", &GenerationConfig::temperature, "Sampling temperature (0.0 - 2.0)")
      .def_readwrite("top_p", &GenerationConfig::top_p, "Nucleus sampling parameter (0.0 - 1.0)")
      .def_readwrite("top_k", &GenerationConfig::top_k, "Top-k sampling parameter")
      .def_readwrite("frequency_penalty", &GenerationConfig::frequency_penalty, "Frequency penalty")
      .def_readwrite("presence_penalty", &GenerationConfig::presence_penalty, "Presence penalty")
      .def_readwrite("do_sample", &GenerationConfig::do_sample, "Whether to use sampling or greedy decoding")
      .def_readwrite("seed", &GenerationConfig::seed, "Philox seed (0: the API's seed)");

  py::class_<ModelMetrics>(m, "ModelMetrics")
      .def_readonly("vocab_size", &ModelMetrics::vocab_size, "Vocabulary size")
      .def_readonly("num_layers", &ModelMetrics::num_layers, "Number of layers")
      .def_readonly("hidden_dim", &ModelMetrics::hidden_dim, "Hidden dimension")
      .def_readonly("context_len", &ModelMetrics::context_len, "Context length")
      .def_readonly("num_heads", &ModelMetrics::num_heads, "Number of attention heads")
      .def_readonly("model_size_bytes", &ModelMetrics::model_size_bytes, "Model size in bytes")
      .def_readonly("architecture", &ModelMetrics::architecture, "Model architecture");

  py::class_<ulbe::SpecToken>(m, "SpeculativeToken")
      .def(py::init<>())
      .def_readwrite("token_id", &ulbe::SpecToken::token_id, "Token id")
      .def_readwrite("probability", &ulbe::SpecToken::probability,
                     "Target probability of the token under the sampling warp (1.0 when greedy)")
      .def_readwrite("position", &ulbe::SpecToken::position, "Position in the sequence");
  py::class_<ulbe::SpecRound>(m, "SpeculationResult")
      .def(py::init<>())
      .def_readwrite("accepted_tokens", &ulbe::SpecRound::accepted_tokens,
                     "Tokens committed this round: accepted drafts, then the correction or bonus token")
      .def_readwrite("rejected_tokens", &ulbe::SpecRound::rejected_tokens, "Drafts after the first rejection")
      .def_readwrite("num_accepted", &ulbe::SpecRound::num_accepted, "Tokens committed (accepted drafts + 1)")
      .def_readwrite("acceptance_rate", &ulbe::SpecRound::acceptance_rate, "Accepted drafts / drafts proposed")
      .def_readwrite("tokens", &ulbe::SpecRound::tokens, "The committed tokens as SpeculativeToken records");
  py::class_<GenerationResult>(m, "GenerationResult")
      .def_readonly("tokens", &GenerationResult::tokens, "Generated token IDs")
      .def_readonly("text", &GenerationResult::text, "Decoded text")
      .def_readonly("num_tokens", &GenerationResult::num_tokens, "Number of tokens generated")
      .def_readonly("time_ms", &GenerationResult::time_ms, "Generation time in milliseconds")
      .def_readonly("tokens_per_second", &GenerationResult::tokens_per_second, "Generation speed");

  py::class_<GenerationProgress>(m, "GenerationProgress")
      .def_readonly("current_step", &GenerationProgress::current_step, "Current step number")
      .def_readonly("total_steps", &GenerationProgress::total_steps, "Total steps to complete")
      .def_readonly("progress_pct", &GenerationProgress::progress_pct, "Progress percentage (0-100)")
      .def_readonly("time_elapsed_ms", &GenerationProgress::time_elapsed_ms, "Time elapsed in milliseconds")
      .def_readonly("estimated_remaining_ms", &GenerationProgress::estimated_remaining_ms, "Estimated time remaining")
      .def_readonly("tokens_per_second", &GenerationProgress::tokens_per_second, "Current tokens per second")
      .def_readonly("last_token", &GenerationProgress::last_token, "Last generated token");

  py::enum_<QuantizationType>(m, "QuantizationType")
      .value("NONE", QuantizationType::NONE)
      .value("FP32", QuantizationType::FP32)
      .value("FP16", QuantizationType::FP16)
      .value("INT8", QuantizationType::INT8)
      .value("FP4", QuantizationType::FP4)
      .value("NF4", QuantizationType::NF4);

  m.def("get_quantization_type_name", &quantization_type_name, "Get quantization type name");
  m.def("nccl_unique_id", []() {
    char id[128];
    if (ulb_tp_unique_id(id) != 0) throw std::runtime_error(ulb_last_error());
    return py::bytes(id, sizeof id);
  }, "A new 128-byte NCCL unique id (create on one rank, share with the others)");
  m.def(
      "gguf_tokenize",
      [](const std::string& path, const std::string& text, py::object add_bos) {
        const ulbe::GgufTokenizer t = gguf_spm(path);
        return t.encode(text, add_bos.is_none() ? t.add_bos() : add_bos.cast<bool>());
      },
      py::arg("path"), py::arg("text"), py::arg("add_bos") = py::none(),
      "Token ids of text under the GGUF file's SentencePiece vocabulary (tokenizer.ggml.*); "
      "add_bos=None follows the file's tokenizer.ggml.add_bos_token");
  m.def(
      "gguf_detokenize",
      [](const std::string& path, const std::vector<int32_t>& ids) { return py::bytes(gguf_spm(path).decode(ids)); },
      py::arg("path"), py::arg("ids"), "Text (UTF-8 bytes) of token ids under the GGUF file's vocabulary");
  m.def("write_synthetic_gguf", &write_synthetic, py::arg("path"), py::arg("spec"), py::arg("threads") = 0,
        "Write a synthetic LLaMA GGUF: Q4_0/Q4_K weights N(0, stddev), fp16 embeddings, unit norms; "
        "spec key tied=True writes no output.weight (the head is token_embd); "
        "spec keys embd_type / out_type pick other token_embd (f32, f16, q4_0, q8_0, q4_k, q6_k) and "
        "output.weight (q4_0, q8_0, q4_k, q6_k) types, v_type / o_type / down_type other attn_v / "
        "attn_output / ffn_down types (q4_0, q8_0, q4_k, q6_k); vocab / scores / token_types (+ merges, "
        "tokenizer_pre for byte-level BPE; add_bos, add_space_prefix) write a tokenizer.ggml.* vocabulary");
  m.def("synth_normal", &ulbe::synth_normal, "Sample i of the synthetic N(0,1) stream keyed by (seed, name)");
  m.attr("__version__") = "0.1";
}
