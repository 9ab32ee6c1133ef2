/*
 * spec_engine.cpp — see spec_engine.h.
 */
#include "spec_engine.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>

#include "gguf.h"

namespace ulbe {

Engine::Engine(int device) {
  if (ulb_init(device, &ctx_) != ULB_OK) {
    err_ = ulb_last_error();
    ctx_ = nullptr;
  }
}

Engine::~Engine() {
  drop_spec();
  if (draft_) ulb_model_free(draft_);
  if (target_) ulb_model_free(target_);
  if (ctx_) ulb_destroy(ctx_);
}

bool Engine::fail(const std::string& m) {
  err_ = m;
  return false;
}

void Engine::drop_spec() {
  if (spec_) ulb_spec_free(spec_);
  spec_ = nullptr;
}

void Engine::unload(bool draft) {
  std::lock_guard<std::mutex> lk(mu_);
  drop_spec();
  ulb_model*& m = draft ? draft_ : target_;
  if (m) ulb_model_free(m);
  m = nullptr;
  (draft ? dinfo_ : tinfo_) = ModelInfo();
}

bool Engine::init_tp(int rank, int world, const void* nccl_id128) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!ctx_) return fail("no CUDA device: " + err_);
  if (target_) return fail("init_tp: call before loading the target model");
  if (world > 1 && ulb_tp_init(ctx_, rank, world, nccl_id128) != ULB_OK) return fail(ulb_last_error());
  tp_rank_ = rank;
  tp_world_ = world;
  return true;
}

bool Engine::set_tp_timeout(int ms) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!ctx_) return fail("no CUDA device: " + err_);
  if (ulb_tp_set_timeout(ctx_, ms) != ULB_OK) return fail(ulb_last_error());
  return true;
}

bool Engine::load(const std::string& path, bool draft) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!ctx_) return fail("no CUDA device: " + err_);
  GGUFFile f;
  std::string e;
  if (!f.open(path, &e)) return fail(e);
  ModelInfo mi;
  mi.path = path;
  mi.file_bytes = f.file_bytes;
  mi.name = f.str("general.name", "llama");
  mi.n_layer = (int)f.num("llama.block_count", 0);
  mi.d_model = (int)f.num("llama.embedding_length", 0);
  mi.n_head = (int)f.num("llama.attention.head_count", 0);
  mi.n_head_kv = (int)f.num("llama.attention.head_count_kv", mi.n_head);
  mi.d_ff = (int)f.num("llama.feed_forward_length", 0);
  mi.ctx_len = (int)f.num("llama.context_length", 2048);
  mi.rms_eps = (float)f.num("llama.attention.layer_norm_rms_epsilon", 1e-5);
  mi.rope_base = (float)f.num("llama.rope.freq_base", 10000.0);
  const GGUFTensor* emb = f.find("token_embd.weight");
  mi.n_vocab = (int)f.num("llama.vocab_size", emb ? (double)emb->ne[1] : 0.0);
  if (mi.n_layer <= 0 || mi.d_model <= 0 || mi.n_head <= 0 || mi.d_ff <= 0 || mi.n_vocab <= 0)
    return fail(path + ": missing llama.* metadata");
  const GGUFTensor* q = f.find("blk.0.attn_q.weight");
  mi.wtype = q ? q->type : 0;
  ulb_model_desc d{};
  d.n_layer = mi.n_layer;
  d.d_model = mi.d_model;
  d.n_head = mi.n_head;
  d.n_head_kv = mi.n_head_kv;
  d.head_dim = mi.d_model / mi.n_head;
  d.d_ff = mi.d_ff;
  d.n_vocab = mi.n_vocab;
  d.rms_eps = mi.rms_eps;
  d.rope_base = mi.rope_base;
  d.max_rows = 64;
  ulb_model* m = nullptr;
  if (ulb_model_create(ctx_, &d, &m) != ULB_OK) return fail(ulb_last_error());
  if (!draft && tp_world_ > 1 && ulb_model_set_tp(m, tp_rank_, tp_world_) != ULB_OK) {
    std::string msg = ulb_last_error();
    ulb_model_free(m);
    return fail(msg);
  }
  for (const GGUFTensor& t : f.tensors) {
    if (ulb_model_set_weight(m, t.name.c_str(), t.type, t.ne, t.data, t.nbytes) != ULB_OK) {
      std::string msg = ulb_last_error();
      ulb_model_free(m);
      return fail(msg);
    }
  }
  if (ulb_model_finalize(m) != ULB_OK) {
    std::string msg = ulb_last_error();
    ulb_model_free(m);
    return fail(msg);
  }
  ulb_model_weight_bytes(m, &mi.weight_bytes);
  drop_spec();
  ulb_model*& slot = draft ? draft_ : target_;
  if (slot) ulb_model_free(slot);
  slot = m;
  (draft ? dinfo_ : tinfo_) = mi;
  return true;
}

bool Engine::generate(const std::vector<std::vector<int32_t>>& prompts, const GenParams& p,
                      std::vector<std::vector<int32_t>>* out, GenStats* st) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!target_) return fail("no model loaded");
  out->assign(prompts.size(), {});
  if (prompts.empty() || p.max_new == 0) return true;
  const auto t0 = std::chrono::steady_clock::now();
  int max_prompt = 0;
  for (const auto& pr : prompts) {
    if (pr.empty()) return fail("empty prompt");
    max_prompt = std::max(max_prompt, (int)pr.size());
  }
  const bool use_draft = draft_ != nullptr && p.k > 0;
  const int n_prompts = (int)prompts.size();
  const bool continuous = p.max_batch > 0 && n_prompts > p.max_batch;
  ulb_spec_desc sd{};
  sd.n_seq = continuous ? p.max_batch : n_prompts;
  sd.k = use_draft ? p.k : 0;
  sd.max_prompt = max_prompt;
  sd.max_new = (int)p.max_new;
  sd.warp.temperature = p.greedy ? 0.f : p.temperature;
  sd.warp.top_k = p.top_k;
  sd.warp.top_p = p.top_p;
  sd.seed = p.seed;
  sd.use_graphs = p.use_graphs ? 1 : 0;
  sd.kv_pages = p.kv_pages;
  sd.tree_width = use_draft && p.tree_width >= 2 ? p.tree_width : 0;
  if (continuous && sd.kv_pages == 0) {
    /* the slots share one pool (as much as every slot's capacity): pages follow the live
       sequences and a finished sequence's pages serve the next prompt */
    int nodes = 0;
    for (int d = 1, pw = 1; sd.tree_width >= 2 && d <= sd.k; ++d) nodes += (pw *= sd.tree_width);
    const int cap = max_prompt + (int)p.max_new + 2 * sd.k + 2 + nodes;
    sd.kv_pages = sd.n_seq * ((cap + ULB_KV_PAGE - 1) / ULB_KV_PAGE);
  }
  const bool same = spec_ && spec_has_draft_ == use_draft && !memcmp(&sd, &spec_desc_, sizeof sd);
  if (!same) {
    drop_spec();
    if (ulb_spec_create(ctx_, target_, use_draft ? draft_ : nullptr, &sd, &spec_) != ULB_OK) {
      spec_ = nullptr;
      return fail(ulb_last_error());
    }
    spec_desc_ = sd;
    spec_has_draft_ = use_draft;
  }
  std::vector<int32_t> flat((size_t)sd.n_seq * max_prompt, 0), lens(sd.n_seq);
  for (int s = 0; s < sd.n_seq; ++s) {
    lens[s] = (int32_t)prompts[s].size();
    std::copy(prompts[s].begin(), prompts[s].end(), flat.begin() + (size_t)s * max_prompt);
  }
  void *e0 = nullptr, *e1 = nullptr, *e2 = nullptr;
  ulb_event_create(ctx_, &e0);
  ulb_event_create(ctx_, &e1);
  ulb_event_create(ctx_, &e2);
  ulb_event_record(ctx_, e0);
  int rc = ulb_spec_prefill(spec_, flat.data(), lens.data());
  ulb_event_record(ctx_, e1);
  int rounds = 0;
  std::vector<int32_t> toks((size_t)sd.n_seq * sd.max_new), counts(sd.n_seq);
  uint64_t stats[4] = {0, 0, 0, 0}, launches = 0, admitted = 0;
  /* slot -> prompt it decodes (-1: idle); prompts beyond the slots wait for a finished one */
  std::vector<int> slot_of(sd.n_seq);
  for (int s = 0; s < sd.n_seq; ++s) slot_of[s] = s;
  int next = sd.n_seq;
  std::vector<std::vector<int32_t>> done_out(n_prompts);
  uint64_t run_rounds = 0;
  const int R = sd.k + 1;
  while (rc == ULB_OK) {
    if (!continuous) {
      rc = ulb_spec_run(spec_, 0, &rounds);
      break;
    }
    /* run until the first live slot can have finished, then hand its slot to the next prompt */
    rc = ulb_spec_read(spec_, toks.data(), counts.data(), stats);
    if (rc != ULB_OK) break;
    int min_rem = -1;
    bool any = false;
    for (int s = 0; s < sd.n_seq && rc == ULB_OK; ++s) {
      if (slot_of[s] < 0) continue;
      if (counts[s] >= sd.max_new) {
        done_out[slot_of[s]].assign(toks.begin() + (size_t)s * sd.max_new, toks.begin() + (size_t)(s + 1) * sd.max_new);
        slot_of[s] = -1;
        if (next < n_prompts) {
          rc = ulb_spec_admit(spec_, s, prompts[next].data(), (int)prompts[next].size());
          slot_of[s] = next++;
          ++admitted;
        }
      }
      if (slot_of[s] >= 0) {
        any = true;
        const int rem = sd.max_new - (slot_of[s] >= 0 && counts[s] < sd.max_new ? counts[s] : 1);
        if (min_rem < 0 || rem < min_rem) min_rem = rem;
      }
    }
    if (rc != ULB_OK || !any) break;
    int ran = 0;
    rc = ulb_spec_run(spec_, std::max(1, (min_rem + R - 1) / R), &ran);
    run_rounds += (uint64_t)ran;
  }
  ulb_event_record(ctx_, e2);
  if (rc == ULB_OK) rc = ulb_spec_read(spec_, toks.data(), counts.data(), stats);
  if (rc == ULB_OK) rc = ulb_spec_launch_count(spec_, &launches);
  if (rc == ULB_OK && continuous) {
    /* stats[0] is the most rounds any slot was live since its start: count every run instead */
    stats[0] = run_rounds;
    rounds = (int)run_rounds;
  }
  float pms = 0, dms = 0;
  if (rc == ULB_OK) {
    ulb_event_elapsed_ms(e0, e1, &pms);
    ulb_event_elapsed_ms(e1, e2, &dms);
  }
  ulb_event_destroy(e0);
  ulb_event_destroy(e1);
  ulb_event_destroy(e2);
  if (rc != ULB_OK) {
    std::string msg = ulb_last_error();
    drop_spec();
    return fail(msg);
  }
  uint64_t gen = 0;
  if (continuous) {
    for (int i = 0; i < n_prompts; ++i) {
      (*out)[i] = std::move(done_out[i]);
      gen += (*out)[i].size();
    }
  } else {
    for (int s = 0; s < sd.n_seq; ++s) {
      (*out)[s].assign(toks.begin() + (size_t)s * sd.max_new, toks.begin() + (size_t)s * sd.max_new + counts[s]);
      gen += (uint64_t)counts[s];
    }
  }
  if (st) {
    st->rounds = stats[0];
    st->drafted = stats[1];
    st->accepted = stats[2];
    st->committed = stats[3];
    st->generated = gen;
    st->prefill_ms = pms;
    st->decode_ms = dms;
    st->total_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    st->h2d_bytes = (double)(flat.size() + lens.size()) * 4.0;
    st->d2h_bytes = (double)(toks.size() + counts.size()) * 4.0;
    st->launches = launches;
    st->admitted = admitted;
  }
  return true;
}

bool Engine::profile_round(float ms[5]) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!spec_) return fail("no generation to profile");
  if (ulb_spec_profile_round_ex(spec_, ms) != ULB_OK) return fail(ulb_last_error());
  return true;
}

bool Engine::speculation_rounds(int seq, std::vector<SpecRound>* out) {
  std::lock_guard<std::mutex> lk(mu_);
  out->clear();
  if (!spec_) return fail("no generation");
  if (!spec_has_draft_) return true;
  int n = 0;
  if (ulb_spec_read_rounds(spec_, seq, 0, nullptr, &n) != ULB_OK) return fail(ulb_last_error());
  const int k = spec_desc_.k, words = ULB_SPEC_REC_WORDS(k);
  std::vector<int32_t> rec((size_t)n * words);
  if (n && ulb_spec_read_rounds(spec_, seq, n, rec.data(), &n) != ULB_OK) return fail(ulb_last_error());
  for (int r = 0; r < n; ++r) {
    const int32_t* w = rec.data() + (size_t)r * words;
    SpecRound sr;
    const int na = w[ULB_SPEC_REC_N_ACCEPTED];
    for (int i = 0; i < k; ++i) (i < na ? sr.accepted_tokens : sr.rejected_tokens).push_back((uint32_t)w[ULB_SPEC_REC_DRAFTS + i]);
    sr.accepted_tokens.push_back((uint32_t)w[ULB_SPEC_REC_TOKEN]);
    sr.num_accepted = (uint32_t)(na + 1);
    sr.acceptance_rate = k > 0 ? (float)na / (float)k : 0.f;
    for (int j = 0; j <= na; ++j) {
      SpecToken t;
      t.token_id = sr.accepted_tokens[j];
      float pr;
      std::memcpy(&pr, &w[ULB_SPEC_REC_DRAFTS + k + j], 4);
      t.probability = pr;
      t.position = (uint32_t)(w[ULB_SPEC_REC_POSITION] + j);
      sr.tokens.push_back(t);
    }
    out->push_back(std::move(sr));
  }
  return true;
}

bool Engine::last_logits(const std::vector<int32_t>& tokens, std::vector<float>* out) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!target_) return fail("no model loaded");
  if (tokens.empty()) return fail("empty token list");
  const int n = (int)tokens.size(), V = tinfo_.n_vocab;
  ulb_kv* kv = nullptr;
  if (ulb_kv_alloc(ctx_, target_, 1, n, &kv) != ULB_OK) return fail(ulb_last_error());
  std::vector<int32_t> seq(n, 0), pos(n);
  for (int i = 0; i < n; ++i) pos[i] = i;
  bool ok = true;
  out->assign(V, 0.f);
  /* rows are fed in chunks of 64 (the model workspace); logits of the last chunk's last row */
  const int chunk = 64;
  int32_t *dt = nullptr, *ds = nullptr, *dp = nullptr;
  float* dl = nullptr;
  if (ulb_malloc(ctx_, chunk * 4, (void**)&dt) || ulb_malloc(ctx_, chunk * 4, (void**)&ds) ||
      ulb_malloc(ctx_, chunk * 4, (void**)&dp) ||
      ulb_malloc(ctx_, (size_t)V * 4, (void**)&dl))
    ok = fail(ulb_last_error());
  for (int c0 = 0; ok && c0 < n; c0 += chunk) {
    const int m = std::min(chunk, n - c0);
    if (ulb_memcpy_h2d(ctx_, dt, tokens.data() + c0, m * 4) ||
        ulb_memcpy_h2d(ctx_, ds, seq.data() + c0, m * 4) ||
        ulb_memcpy_h2d(ctx_, dp, pos.data() + c0, m * 4) ||
        ulb_model_forward(ctx_, target_, kv, m, m, dt, ds, dp, 1, dl, V))
      ok = fail(ulb_last_error());
  }
  if (ok && ulb_memcpy_d2h(ctx_, out->data(), dl, (size_t)V * 4)) ok = fail(ulb_last_error());
  ulb_free(ctx_, dt);
  ulb_free(ctx_, ds);
  ulb_free(ctx_, dp);
  ulb_free(ctx_, dl);
  ulb_kv_free(kv);
  return ok;
}

}  // namespace ulbe
