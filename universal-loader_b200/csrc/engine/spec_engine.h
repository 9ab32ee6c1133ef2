/*
 * spec_engine.h — host engine above the C ABI.
 *
 * Plays the role of the reference's InferenceEngine (src/inference/inference_engine.h) on the
 * speculative path: owns the device context, the target and draft models loaded from GGUF
 * files, and drives the device-resident draft -> verify -> accept loop (ulb_spec_*).
 */
#pragma once
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "ulb.h"

namespace ulbe {

struct ModelInfo {
  int n_layer = 0, d_model = 0, n_head = 0, n_head_kv = 0, d_ff = 0, n_vocab = 0, ctx_len = 0;
  float rms_eps = 1e-5f, rope_base = 10000.f;
  int wtype = 0;
  size_t file_bytes = 0, weight_bytes = 0;
  std::string name, path;
};

struct GenParams {
  uint32_t max_new = 0;
  float temperature = 0.f;
  int top_k = 0;
  float top_p = 1.f;
  bool greedy = true;
  uint64_t seed = 0;
  int k = 0;              /* speculation length; 0 = plain decoding */
  bool use_graphs = true;
  /* continuous batching: at most this many sequences decode at once (0 = all of them); with
     more prompts than that, a finished sequence's slot is given to the next prompt */
  int max_batch = 0;
  /* KV cache pages per model (0: every slot owns its whole capacity; otherwise on demand) */
  int kv_pages = 0;
  /* tree speculation: children per node (>= 2; 0 = a chain of k drafts); k is the depth */
  int tree_width = 0;
};

/* One round of the speculative loop for one sequence, as the reference's SpeculationResult
   (src/inference/speculative_decoder.h:17-22) with its SpeculativeToken list (:11-15). */
struct SpecToken {
  uint32_t token_id = 0;
  float probability = 0.f; /* the target's probability of the token under the warp (greedy: 1) */
  uint32_t position = 0;
};
struct SpecRound {
  std::vector<uint32_t> accepted_tokens; /* committed this round: accepted drafts, then the correction / bonus */
  std::vector<uint32_t> rejected_tokens; /* drafts after the first rejection */
  uint32_t num_accepted = 0;             /* tokens committed (accepted drafts + 1) */
  float acceptance_rate = 0.f;           /* accepted drafts / drafts proposed */
  std::vector<SpecToken> tokens;
};

struct GenStats {
  uint64_t rounds = 0, drafted = 0, accepted = 0, committed = 0, generated = 0;
  double prefill_ms = 0, decode_ms = 0, total_ms = 0;
  double h2d_bytes = 0, d2h_bytes = 0;
  uint64_t launches = 0; /* kernels launched by the library for this generation */
  uint64_t admitted = 0; /* sequences started in a freed slot (continuous batching) */
};

class Engine {
 public:
  explicit Engine(int device = 0);
  ~Engine();
  bool ok() const { return ctx_ != nullptr; }
  const std::string& error() const { return err_; }

  bool load(const std::string& path, bool draft);
  /* join a tensor-parallel communicator: later target loads keep this rank's slice (the
     draft stays replicated) */
  bool init_tp(int rank, int world, const void* nccl_id128);
  /* bound on host waits for tensor-parallel work (ulb_tp_set_timeout); 0 = unbounded */
  bool set_tp_timeout(int ms);
  void unload(bool draft);
  bool has_model(bool draft) const { return draft ? draft_ != nullptr : target_ != nullptr; }
  const ModelInfo& info(bool draft) const { return draft ? dinfo_ : tinfo_; }

  /* prompts: token ids.  Returns committed tokens per prompt (max_new each). */
  bool generate(const std::vector<std::vector<int32_t>>& prompts, const GenParams& p,
                std::vector<std::vector<int32_t>>* out, GenStats* st);
  /* logits of the last position after feeding `tokens` to the target from an empty cache */
  bool last_logits(const std::vector<int32_t>& tokens, std::vector<float>* out);
  /* time one extra round of the last generation's loop by phase: draft, verify, accept (ms),
     then the summed time of its tensor-parallel all-reduces (ms) and their count */
  bool profile_round(float ms[5]);
  /* per-round records of sequence `seq` of the last generation (empty for plain decoding) */
  bool speculation_rounds(int seq, std::vector<SpecRound>* out);

  ulb_ctx* ctx() { return ctx_; }

 private:
  bool fail(const std::string& m);
  void drop_spec();
  ulb_ctx* ctx_ = nullptr;
  int tp_rank_ = 0, tp_world_ = 1;
  ulb_model* target_ = nullptr;
  ulb_model* draft_ = nullptr;
  ModelInfo tinfo_, dinfo_;
  std::string err_;
  /* cached loop for repeated calls with the same shape */
  ulb_spec* spec_ = nullptr;
  ulb_spec_desc spec_desc_{};
  bool spec_has_draft_ = false;
  std::mutex mu_;
};

}  // namespace ulbe
