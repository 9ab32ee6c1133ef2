/*
 * spec.cu — the device-resident speculative draft -> verify -> accept loop.
 *
 * Replaces SpeculativeDecoder::generate_with_speculation / generate_draft_tokens
 * (src/inference/speculative_decoder.cpp:25-87, k host callbacks then one verify callback)
 * and InferenceEngine::generate_streaming's decode loop
 * (src/inference/inference_engine.cpp:273-328, ~20 fenced dispatches per layer per token).
 *
 * State per sequence lives in HBM: committed tokens (prompt first), committed length L,
 * done flag, round counter.  Invariant between rounds: both KV caches hold positions
 * 0..L-2 and token L-1 is pending.  One round:
 *   draft step 0 on rows (t[L-2] @ L-2, t[L-1] @ L-1)   (refreshes L-2 after a full accept)
 *   draft step j = 1..k-1 on (d[j-1] @ L-1+j)            -> q_j logits, d_j ~ q_j
 *   verify on (t[L-1] @ L-1, d_0..d_{k-1} @ L..L+k-1)     -> p_0..p_k logits
 *   accept (rejection sampling) and commit n+1 tokens; KV rollback is the new L itself:
 *   entries past L-2 are simply overwritten by the next round.
 * The whole round is captured once into a CUDA graph (kernels chained with programmatic
 * dependent launch) and replayed; the host only reads the committed lengths between
 * batches of rounds.
 */
#include <algorithm>
#include <cstring>
#include <memory>

#include "paging.h"
#include "ulb_internal.h"

namespace ulb {
int launch_sample_seq(Ctx* c, const float* logits, int rows, int V, int ld, const ulb_warp* w, uint64_t seed,
                      const uint32_t* dev_round, uint32_t round, uint32_t slot, uint32_t tag, uint32_t seq_base,
                      int32_t* out, int out_stride);
size_t tree_accept_scratch_bytes(int B, int w, int D);
int launch_tree_children(Ctx* c, const float* logits, int rows, int V, int w, int d, const ulb_warp* wp,
                         uint64_t seed, const uint32_t* dev_round, int N, int32_t* tokens);
int launch_tree_accept_commit(Ctx* c, const float* p, const float* q, const int32_t* tokens, int B, int w, int D,
                              int V, const ulb_warp* wp, uint64_t seed, const uint32_t* dev_round, void* stats_scratch,
                              int32_t* comp, int32_t* hist, int hist_len, int32_t* L, int32_t* done,
                              const int32_t* plen, int max_new, uint32_t* round, unsigned long long* stats,
                              int32_t* active, int32_t* log, int log_rounds);
int launch_accept_commit(Ctx* c, const float* p, const float* q, const int32_t* draft, int B, int k, int V,
                         const ulb_warp* w, uint64_t seed, const uint32_t* dev_round, void* stats_scratch,
                         int32_t* hist, int hist_len, int32_t* L, int32_t* done, const int32_t* plen, int max_new,
                         uint32_t* round, unsigned long long* stats, int32_t* active_rounds, int32_t* log,
                         int log_rounds);
}  // namespace ulb

extern "C" int ulb_kv_alloc(ulb_ctx* ctx, const ulb_model* m, int n_seq, int cap, ulb_kv** out);
extern "C" int ulb_kv_alloc_paged(ulb_ctx* ctx, const ulb_model* m, int n_seq, int n_pages, int max_pages, ulb_kv** out);
extern "C" int ulb_kv_map(ulb_kv* kv, int seq, int first, int n, const int32_t* pages);
extern "C" int ulb_kv_free(ulb_kv* kv);

namespace ulb {

namespace {

__global__ void stage_draft_kernel(int S, int j, int k, const int* __restrict__ hist, int hl, const int* __restrict__ L,
                                   const int* __restrict__ draft, int* rtok, int* rseq, int* rpos) {
  ULB_TRACE_KERNEL(kTrStageDraft, j);
  pdl_wait();
  pdl_trigger();
  const int rps = j == 0 ? 2 : 1;
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= S * rps) return;
  const int s = m / rps, e = m % rps;
  int pos, tok;
  if (j == 0) {
    pos = L[s] - 2 + e;
    tok = hist[(size_t)s * hl + pos];
  } else {
    pos = L[s] - 1 + j;
    tok = draft[s * k + j - 1];
  }
  rtok[m] = tok;
  rseq[m] = s;
  rpos[m] = pos;
}

__global__ void stage_verify_kernel(int S, int k, const int* __restrict__ hist, int hl, const int* __restrict__ L,
                                    const int* __restrict__ draft, int* rtok, int* rseq, int* rpos) {
  ULB_TRACE_KERNEL(kTrStageVerify, 0);
  pdl_wait();
  pdl_trigger();
  const int R = k + 1;
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= S * R) return;
  const int s = m / R, e = m % R;
  rtok[m] = e == 0 ? hist[(size_t)s * hl + L[s] - 1] : draft[s * k + e - 1];
  rseq[m] = s;
  rpos[m] = L[s] - 1 + e;
}

__global__ void stage_prefill_kernel(int s, int c0, int n, const int* __restrict__ hist, int hl, int* rtok, int* rseq,
                                     int* rpos) {
  ULB_TRACE_KERNEL(kTrStagePrefill, 0);
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  rtok[i] = hist[(size_t)s * hl + c0 + i];
  rseq[i] = s;
  rpos[i] = c0 + i;
}

/* Tree rounds (width w, depth D = k).  Draft step 0 is the chain's (rows L - 2, L - 1, plain
   causal rows); step d >= 1 feeds the w^d nodes of depth d: node i in cache slot L + i,
   rotated as position L - 1 + d, seeing the committed keys (< L) and its ancestors. */
__global__ void stage_tree_draft_kernel(int S, int d, int w, int N, const int* __restrict__ hist, int hl,
                                        const int* __restrict__ L, const int* __restrict__ ttok, int* rtok, int* rseq,
                                        int* rpos, int* rrope, int* rpref, unsigned long long* rmask) {
  ULB_TRACE_KERNEL(kTrStageTree, d);
  pdl_wait();
  pdl_trigger();
  int per = 1;
  for (int j = 0; j < d; ++j) per *= w;
  const int rps = d == 0 ? 2 : per;
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= S * rps) return;
  const int s = m / rps, e = m % rps;
  if (d == 0) {
    const int pos = L[s] - 2 + e;
    rtok[m] = hist[(size_t)s * hl + pos];
    rpos[m] = pos;
    rrope[m] = pos;
    rpref[m] = pos + 1;
    rmask[m] = 0ull;
  } else {
    const int node = tree_first(w, d) + e;
    rtok[m] = ttok[(size_t)s * N + node];
    rpos[m] = L[s] + node;
    rrope[m] = L[s] - 1 + d;
    rpref[m] = L[s];
    rmask[m] = tree_ancestors(w, node);
  }
  rseq[m] = s;
}

/* the verify rows of a tree round: the root (the last committed token) and every node */
__global__ void stage_tree_verify_kernel(int S, int w, int N, const int* __restrict__ hist, int hl,
                                         const int* __restrict__ L, const int* __restrict__ ttok, int* rtok, int* rseq,
                                         int* rpos, int* rrope, int* rpref, unsigned long long* rmask) {
  ULB_TRACE_KERNEL(kTrStageTree + 1, 0);
  pdl_wait();
  pdl_trigger();
  const int R = N + 1;
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= S * R) return;
  const int s = m / R, e = m % R;
  if (e == 0) {
    rtok[m] = hist[(size_t)s * hl + L[s] - 1];
    rpos[m] = L[s] - 1;
    rrope[m] = L[s] - 1;
    rmask[m] = 0ull;
  } else {
    const int node = e - 1;
    rtok[m] = ttok[(size_t)s * N + node];
    rpos[m] = L[s] + node;
    rrope[m] = L[s] - 1 + tree_depth(w, node);
    rmask[m] = tree_ancestors(w, node);
  }
  rpref[m] = L[s];
  rseq[m] = s;
}

/* prompt rows per prefill forward: large enough for the tensor-core GEMM (>= 128 rows) */
constexpr int kPrefillChunk = 256;

}  // namespace

struct Spec {
  Ctx* c = nullptr;
  ulb_ctx* ctx = nullptr;
  Model* tgt = nullptr;
  Model* dft = nullptr;
  ulb_model* tgt_h = nullptr;
  ulb_model* dft_h = nullptr;
  ulb_spec_desc d{};
  int k = 0, S = 0, V = 0;
  int cap = 0, hl = 0;
  ulb_kv* kvt = nullptr;
  ulb_kv* kvd = nullptr;
  KV* kvt_i = nullptr;
  KV* kvd_i = nullptr;
  /* device */
  int32_t *hist = nullptr, *L = nullptr, *done = nullptr, *plen = nullptr, *draft = nullptr;
  int32_t *rtok = nullptr, *rseq = nullptr, *rpos = nullptr, *err = nullptr, *active = nullptr;
  int32_t* log = nullptr; /* per-round records [S][log_rounds][ULB_SPEC_REC_WORDS(k)] */
  int log_rounds = 0;
  uint32_t* round = nullptr;
  unsigned long long* stats = nullptr;
  float *plog = nullptr, *qlog = nullptr;
  void* rs = nullptr;
  size_t rs_bytes = 0, plog_bytes = 0, qlog_bytes = 0, rows_cap = 0;
  /* host */
  int32_t* h_L = nullptr;
  int32_t* h_done = nullptr;
  std::vector<int> h_plen;
  cudaGraphExec_t exec = nullptr;
  bool prefilled = false;
  /* pages of both caches on demand (desc.kv_pages > 0), else every slot owns its capacity */
  std::unique_ptr<PagePool> pool;
  /* tree speculation (tw >= 2): width, nodes, internal nodes, the drafted node tokens
     [S][tN], the last round's accepted paths for the cache compaction [S][2 + k] and the
     tree fields of the rows (RoPE position, prefix end, ancestor mask) */
  int tw = 0, tN = 0, tNI = 0;
  int32_t *ttok = nullptr, *comp = nullptr, *rrope = nullptr, *rpref = nullptr;
  unsigned long long* rmask = nullptr;
  /* launch accounting */
  uint64_t per_round = 0;   /* kernels in one round (counted while recording it) */
  uint64_t launches = 0;    /* since the last prefill */
};

static int record_round_impl(Spec* sp, void* ev_draft_done, void* ev_verify_done);

/* Enqueue one round; counts its kernels into sp->per_round the first time. */
static int record_round(Spec* sp, void* ev_draft_done = nullptr, void* ev_verify_done = nullptr) {
  const uint64_t before = sp->c->launches;
  const int rc = record_round_impl(sp, ev_draft_done, ev_verify_done);
  if (rc == ULB_OK && sp->per_round == 0) sp->per_round = sp->c->launches - before;
  return rc;
}

static int record_tree_round(Spec* sp, void* ev_draft_done, void* ev_verify_done) {
  Ctx* c = sp->c;
  const int S = sp->S, w = sp->tw, D = sp->k, V = sp->V, N = sp->tN;
  TreeRows tr;
  tr.rope = sp->rrope;
  tr.pref = sp->rpref;
  tr.mask = sp->rmask;
  size_t qbase = 0; /* q rows of the levels so far (level-major) */
  int per = 1;      /* w^d */
  for (int d = 0; d < D; ++d) {
    const int rps = d == 0 ? 2 : per, M = S * rps;
    cudaError_t e = launch_k(c, stage_tree_draft_kernel, dim3((M + 127) / 128), dim3(128), 0, S, d, w, N,
                             (const int*)sp->hist, sp->hl, (const int*)sp->L, (const int*)sp->ttok, sp->rtok, sp->rseq,
                             sp->rpos, sp->rrope, sp->rpref, sp->rmask);
    if (e != cudaSuccess) return cuda_error(e, "stage_tree_draft", __FILE__, __LINE__);
    ULB_TRY(model_forward(sp->dft, sp->kvd_i, M, rps, sp->rtok, sp->rseq, sp->rpos, d == 0 ? 1 : 0,
                          sp->qlog + qbase * V, V, sp->err, &tr));
    ULB_TRY(launch_tree_children(c, sp->qlog + qbase * V, S * per, V, w, d, &sp->d.warp, sp->d.seed, sp->round, N,
                                 sp->ttok));
    qbase += (size_t)S * per;
    per *= w;
  }
  if (ev_draft_done) ULB_CUDA(cudaEventRecord((cudaEvent_t)ev_draft_done, c->stream));
  const int M = S * (N + 1);
  cudaError_t e = launch_k(c, stage_tree_verify_kernel, dim3((M + 127) / 128), dim3(128), 0, S, w, N,
                           (const int*)sp->hist, sp->hl, (const int*)sp->L, (const int*)sp->ttok, sp->rtok, sp->rseq,
                           sp->rpos, sp->rrope, sp->rpref, sp->rmask);
  if (e != cudaSuccess) return cuda_error(e, "stage_tree_verify", __FILE__, __LINE__);
  ULB_TRY(model_forward(sp->tgt, sp->kvt_i, M, N + 1, sp->rtok, sp->rseq, sp->rpos, 0, sp->plog, V, sp->err, &tr));
  if (ev_verify_done) ULB_CUDA(cudaEventRecord((cudaEvent_t)ev_verify_done, c->stream));
  ULB_TRY(launch_tree_accept_commit(c, sp->plog, sp->qlog, sp->ttok, S, w, D, V, &sp->d.warp, sp->d.seed, sp->round,
                                    sp->rs, sp->comp, sp->hist, sp->hl, sp->L, sp->done, sp->plen, sp->d.max_new,
                                    sp->round, sp->stats, sp->active, sp->log, sp->log_rounds));
  ULB_TRY(kv_tree_compact(sp->kvt_i, sp->comp, S, D));
  return kv_tree_compact(sp->kvd_i, sp->comp, S, D);
}

static int record_round_impl(Spec* sp, void* ev_draft_done, void* ev_verify_done) {
  if (sp->tw >= 2) return record_tree_round(sp, ev_draft_done, ev_verify_done);
  Ctx* c = sp->c;
  const int S = sp->S, k = sp->k, V = sp->V;
  for (int j = 0; j < k; ++j) {
    const int rps = j == 0 ? 2 : 1, M = S * rps;
    cudaError_t e = launch_k(c, stage_draft_kernel, dim3((M + 127) / 128), dim3(128), 0, S, j, k,
                             (const int*)sp->hist, sp->hl, (const int*)sp->L, (const int*)sp->draft, sp->rtok,
                             sp->rseq, sp->rpos);
    if (e != cudaSuccess) return cuda_error(e, "stage_draft", __FILE__, __LINE__);
    ULB_TRY(model_forward(sp->dft, sp->kvd_i, M, rps, sp->rtok, sp->rseq, sp->rpos, 1, sp->qlog + (size_t)j * V,
                          k * V, sp->err));
    ULB_TRY(launch_sample_seq(c, sp->qlog + (size_t)j * V, S, V, k * V, &sp->d.warp, sp->d.seed, sp->round, 0,
                              (uint32_t)j, ULB_RNG_DRAFT, 0, sp->draft + j, k));
  }
  if (ev_draft_done) ULB_CUDA(cudaEventRecord((cudaEvent_t)ev_draft_done, c->stream));
  const int M = S * (k + 1);
  cudaError_t e = launch_k(c, stage_verify_kernel, dim3((M + 127) / 128), dim3(128), 0, S, k, (const int*)sp->hist,
                           sp->hl, (const int*)sp->L, (const int*)sp->draft, sp->rtok, sp->rseq, sp->rpos);
  if (e != cudaSuccess) return cuda_error(e, "stage_verify", __FILE__, __LINE__);
  ULB_TRY(model_forward(sp->tgt, sp->kvt_i, M, k + 1, sp->rtok, sp->rseq, sp->rpos, 0, sp->plog, V, sp->err));
  if (ev_verify_done) ULB_CUDA(cudaEventRecord((cudaEvent_t)ev_verify_done, c->stream));
  return launch_accept_commit(c, sp->plog, sp->qlog, sp->draft, S, k, V, &sp->d.warp, sp->d.seed, sp->round, sp->rs,
                              sp->hist, sp->hl, sp->L, sp->done, sp->plen, sp->d.max_new, sp->round, sp->stats,
                              sp->active, sp->log, sp->log_rounds);
}

static size_t log_bytes(const Spec* sp) {
  return (size_t)sp->S * sp->log_rounds * ULB_SPEC_REC_WORDS(sp->k) * 4;
}

static void spec_release(Spec* sp) {
  Ctx* c = sp->c;
  if (sp->exec) cudaGraphExecDestroy(sp->exec);
  dev_free(c, sp->hist, (size_t)sp->S * sp->hl * 4);
  dev_free(c, sp->L, sp->S * 4); dev_free(c, sp->done, sp->S * 4); dev_free(c, sp->plen, sp->S * 4);
  dev_free(c, sp->draft, (size_t)sp->S * std::max(sp->k, 1) * 4);
  dev_free(c, sp->rtok, sp->rows_cap * 4); dev_free(c, sp->rseq, sp->rows_cap * 4); dev_free(c, sp->rpos, sp->rows_cap * 4);
  dev_free(c, sp->err, 4); dev_free(c, sp->active, sp->S * 4);
  dev_free(c, sp->round, sp->S * 4); dev_free(c, sp->stats, 4 * 8);
  dev_free(c, sp->plog, sp->plog_bytes); dev_free(c, sp->qlog, sp->qlog_bytes); dev_free(c, sp->rs, sp->rs_bytes);
  dev_free(c, sp->log, log_bytes(sp));
  dev_free(c, sp->ttok, (size_t)sp->S * sp->tN * 4);
  dev_free(c, sp->comp, (size_t)sp->S * (2 + sp->k) * 4);
  dev_free(c, sp->rrope, sp->rows_cap * 4);
  dev_free(c, sp->rpref, sp->rows_cap * 4);
  dev_free(c, sp->rmask, sp->rows_cap * 8);
  if (sp->h_L) cudaFreeHost(sp->h_L);
  if (sp->h_done) cudaFreeHost(sp->h_done);
  ulb_kv_free(sp->kvt);
  ulb_kv_free(sp->kvd);
  cudaStreamSynchronize(c->stream);
}

/* cache positions past the committed length L that one round may write: up to L + k for a
   chain, up to L + N - 1 for a tree of N nodes (plus the pending row) */
static int round_span(const Spec* sp) { return (sp->tw >= 2 ? sp->tN : sp->k) + 1; }

/* map pages so slot s covers positions [0, positions) in both caches (paged loop only) */
static int map_slot(Spec* sp, int s, int positions) {
  if (!sp->pool) return ULB_OK;
  int first = 0;
  std::vector<int> added;
  if (!sp->pool->ensure(s, std::min(positions, sp->cap), &first, &added))
    return set_error(ULB_ENOMEM, "KV page pool exhausted: slot %d needs %d positions, %d pages free", s, positions,
                     sp->pool->free_pages());
  if (added.empty()) return ULB_OK;
  ULB_TRY(ulb_kv_map(sp->kvt, s, first, (int)added.size(), added.data()));
  if (sp->kvd) ULB_TRY(ulb_kv_map(sp->kvd, s, first, (int)added.size(), added.data()));
  return ULB_OK;
}

/* return slot s's pages to the pool (its cache rows become unmapped) */
static int unmap_slot(Spec* sp, int s) {
  if (!sp->pool || sp->pool->mapped(s) == 0) return ULB_OK;
  const int n = sp->pool->release(s);
  std::vector<int> none((size_t)n, -1);
  ULB_TRY(ulb_kv_map(sp->kvt, s, 0, n, none.data()));
  if (sp->kvd) ULB_TRY(ulb_kv_map(sp->kvd, s, 0, n, none.data()));
  return ULB_OK;
}

/* prompt rows of slot s (already in hist) through both models in chunks, then the slot's first
   token from the target's last-position logits */
static int prefill_slot(Spec* sp, int s, int n_total) {
  Ctx* c = sp->c;
  const int V = sp->V;
  for (int c0 = 0; c0 < n_total; c0 += kPrefillChunk) {
    const int n = std::min(kPrefillChunk, n_total - c0);
    cudaError_t e = launch_k(c, stage_prefill_kernel, dim3((n + 127) / 128), dim3(128), 0, s, c0, n,
                             (const int*)sp->hist, sp->hl, sp->rtok, sp->rseq, sp->rpos);
    if (e != cudaSuccess) return cuda_error(e, "stage_prefill", __FILE__, __LINE__);
    ULB_TRY(model_forward(sp->tgt, sp->kvt_i, n, n, sp->rtok, sp->rseq, sp->rpos, 1, sp->plog, V, sp->err));
    if (sp->dft) ULB_TRY(model_forward(sp->dft, sp->kvd_i, n, n, sp->rtok, sp->rseq, sp->rpos, 1, sp->qlog, V, sp->err));
  }
  return launch_sample_seq(c, sp->plog, 1, V, V, &sp->d.warp, sp->d.seed, nullptr, 0, 0, ULB_RNG_FIRST, (uint32_t)s,
                           sp->hist + (size_t)s * sp->hl + n_total, 1);
}

}  // namespace ulb

struct ulb_spec {
  ulb::Spec s;
};

using namespace ulb;

/* access to the internals of the opaque handles (defined in model.cu) */
namespace ulb {
Model* model_of(ulb_model* m);
KV* kv_of(ulb_kv* kv);
int model_vocab(const Model* m);
}  // namespace ulb

extern "C" {

int ulb_spec_create(ulb_ctx* ctx, ulb_model* target, ulb_model* draft, const ulb_spec_desc* d, ulb_spec** out) {
  ULB_CHECK(ctx && target && d && out, ULB_EINVAL, "ulb_spec_create: NULL argument");
  ULB_CHECK(d->n_seq > 0 && d->max_prompt > 0 && d->max_new > 0 && d->k >= 0, ULB_EINVAL,
            "ulb_spec_create: n_seq %d max_prompt %d max_new %d k %d", d->n_seq, d->max_prompt, d->max_new, d->k);
  ULB_CHECK(d->k <= 16, ULB_EUNSUPPORTED, "ulb_spec_create: k %d > 16", d->k);
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  std::unique_ptr<ulb_spec> h(new ulb_spec());
  Spec* sp = &h->s;
  sp->c = c;
  sp->ctx = ctx;
  sp->tgt = model_of(target);
  sp->dft = draft && d->k > 0 ? model_of(draft) : nullptr;
  sp->tgt_h = target;
  sp->dft_h = sp->dft ? draft : nullptr;
  sp->d = *d;
  sp->k = sp->dft ? d->k : 0;
  sp->S = d->n_seq;
  sp->V = model_vocab(sp->tgt);
  if (sp->dft)
    ULB_CHECK(model_vocab(sp->dft) == sp->V, ULB_EINVAL, "draft vocab %d != target vocab %d", model_vocab(sp->dft), sp->V);
  const int S = sp->S, k = sp->k, V = sp->V;
  if (sp->dft && d->tree_width >= 2) {
    ULB_CHECK(d->tree_width <= kTreeMaxWidth && k <= 8 && tree_first(d->tree_width, k + 1) <= kTreeMaxNodes,
              ULB_EUNSUPPORTED, "ulb_spec_create: a tree of width %d and depth %d (at most %d nodes, width <= %d)",
              d->tree_width, k, kTreeMaxNodes, kTreeMaxWidth);
    sp->tw = d->tree_width;
    sp->tN = tree_first(sp->tw, k + 1);
    sp->tNI = tree_first(sp->tw, k);
  }
  sp->cap = d->max_prompt + d->max_new + 2 * k + 2 + sp->tN;
  sp->hl = sp->cap;
  int rc = ULB_OK;
  auto fail = [&](int code) {
    spec_release(sp);
    return code;
  };
  if (d->kv_pages > 0) {
    /* one pool of kv_pages pages per model, mapped to slots as they grow */
    const int pps = (sp->cap + kKvPage - 1) / kKvPage;
    ULB_CHECK(pps * kKvPage <= 8192, ULB_EUNSUPPORTED, "ulb_spec_create: capacity %d > 8192 positions", sp->cap);
    sp->pool.reset(new PagePool(d->kv_pages, S, pps, kKvPage));
    if ((rc = ulb_kv_alloc_paged(ctx, target, S, d->kv_pages, pps, &sp->kvt))) return fail(rc);
    if (sp->dft && (rc = ulb_kv_alloc_paged(ctx, draft, S, d->kv_pages, pps, &sp->kvd))) return fail(rc);
  } else {
    if ((rc = ulb_kv_alloc(ctx, target, S, sp->cap, &sp->kvt))) return fail(rc);
    if (sp->dft && (rc = ulb_kv_alloc(ctx, draft, S, sp->cap, &sp->kvd))) return fail(rc);
  }
  sp->kvt_i = kv_of(sp->kvt);
  if (sp->dft) sp->kvd_i = kv_of(sp->kvd);
  sp->rows_cap = (size_t)std::max({S * (k + 1), 2 * S, kPrefillChunk, S * (sp->tN + 1)});
#define ALLOC(ptr, bytes) if ((rc = dev_alloc(c, (void**)&(ptr), (bytes)))) return fail(rc)
  ALLOC(sp->hist, (size_t)S * sp->hl * 4);
  ALLOC(sp->L, S * 4); ALLOC(sp->done, S * 4); ALLOC(sp->plen, S * 4);
  ALLOC(sp->draft, (size_t)S * std::max(k, 1) * 4);
  ALLOC(sp->rtok, sp->rows_cap * 4); ALLOC(sp->rseq, sp->rows_cap * 4); ALLOC(sp->rpos, sp->rows_cap * 4);
  ALLOC(sp->err, 4); ALLOC(sp->active, S * 4); ALLOC(sp->round, S * 4); ALLOC(sp->stats, 4 * 8);
  sp->plog_bytes = (size_t)S * (std::max(k, sp->tN) + 1) * V * 4;
  sp->qlog_bytes = (size_t)S * std::max({k, 1, sp->tNI + 1}) * V * 4;
  ALLOC(sp->plog, sp->plog_bytes);
  ALLOC(sp->qlog, sp->qlog_bytes);
  sp->rs_bytes = sp->tw >= 2 ? tree_accept_scratch_bytes(S, sp->tw, k) : accept_scratch_bytes(S, k, V);
  if (sp->tw >= 2) {
    ALLOC(sp->ttok, (size_t)S * sp->tN * 4);
    ALLOC(sp->comp, (size_t)S * (2 + k) * 4);
    ALLOC(sp->rrope, sp->rows_cap * 4);
    ALLOC(sp->rpref, sp->rows_cap * 4);
    ALLOC(sp->rmask, sp->rows_cap * 8);
  }
  ALLOC(sp->rs, sp->rs_bytes);
  /* every round commits at least one token, so max_new rounds (+1 for a profiled round) hold
     a whole generation */
  sp->log_rounds = d->max_new + 1;
  ALLOC(sp->log, log_bytes(sp));
#undef ALLOC
  if (cudaMallocHost((void**)&sp->h_L, S * 4) != cudaSuccess || cudaMallocHost((void**)&sp->h_done, S * 4) != cudaSuccess)
    return fail(set_error(ULB_ENOMEM, "pinned host allocation failed"));
  cudaMemsetAsync(sp->err, 0, 4, c->stream);
  /* workspaces for every forward shape the loop uses */
  if ((rc = model_prepare(sp->tgt, sp->kvt_i, kPrefillChunk, kPrefillChunk))) return fail(rc);
  if ((rc = model_prepare(sp->tgt, sp->kvt_i, S * (k + 1), k + 1))) return fail(rc);
  if (sp->dft) {
    if ((rc = model_prepare(sp->dft, sp->kvd_i, kPrefillChunk, kPrefillChunk))) return fail(rc);
    if ((rc = model_prepare(sp->dft, sp->kvd_i, 2 * S, 2))) return fail(rc);
    if ((rc = model_prepare(sp->dft, sp->kvd_i, S, 1))) return fail(rc);
  }
  if (sp->tw >= 2) { /* the tree round's forwards */
    if ((rc = model_prepare(sp->tgt, sp->kvt_i, S * (sp->tN + 1), sp->tN + 1, true))) return fail(rc);
    if ((rc = model_prepare(sp->dft, sp->kvd_i, 2 * S, 2, true))) return fail(rc);
    for (int dd = 1, per = sp->tw; dd < k; ++dd, per *= sp->tw)
      if ((rc = model_prepare(sp->dft, sp->kvd_i, S * per, per, true))) return fail(rc);
  }
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return fail(cuda_error(cudaGetLastError(), "create", __FILE__, __LINE__));
  *out = h.release();
  return ULB_OK;
}

int ulb_spec_prefill(ulb_spec* h, const int32_t* prompts, const int32_t* lens) {
  ULB_CHECK(h && prompts && lens, ULB_EINVAL, "ulb_spec_prefill: NULL argument");
  Spec* sp = &h->s;
  Ctx* c = sp->c;
  ULB_CUDA(cudaSetDevice(c->device));
  const int S = sp->S, V = sp->V, P = sp->d.max_prompt;
  for (int s = 0; s < S; ++s) {
    ULB_CHECK(lens[s] >= 1 && lens[s] <= P, ULB_EINVAL, "prompt %d length %d outside [1, %d]", s, lens[s], P);
    for (int i = 0; i < lens[s]; ++i)
      ULB_CHECK(prompts[(size_t)s * P + i] >= 0 && prompts[(size_t)s * P + i] < V, ULB_EINVAL,
                "prompt %d token %d = %d outside the vocabulary", s, i, prompts[(size_t)s * P + i]);
  }
  std::vector<int32_t> hist((size_t)S * sp->hl, 0);
  sp->h_plen.assign(lens, lens + S);
  for (int s = 0; s < S; ++s) memcpy(&hist[(size_t)s * sp->hl], prompts + (size_t)s * P, (size_t)lens[s] * 4);
  ULB_CUDA(cudaMemcpyAsync(sp->hist, hist.data(), hist.size() * 4, cudaMemcpyHostToDevice, c->stream));
  ULB_CUDA(cudaMemcpyAsync(sp->plen, lens, S * 4, cudaMemcpyHostToDevice, c->stream));
  ULB_CUDA(cudaMemsetAsync(sp->done, 0, S * 4, c->stream));
  ULB_CUDA(cudaMemsetAsync(sp->round, 0, S * 4, c->stream));
  ULB_CUDA(cudaMemsetAsync(sp->active, 0, S * 4, c->stream));
  ULB_CUDA(cudaMemsetAsync(sp->stats, 0, 4 * 8, c->stream));
  ULB_CUDA(cudaMemsetAsync(sp->err, 0, 4, c->stream));
  const uint64_t launches0 = c->launches;
  for (int s = 0; s < S; ++s) {
    /* pages for the prompt and the first round (it writes positions up to lens + k) */
    ULB_TRY(unmap_slot(sp, s));
    ULB_TRY(map_slot(sp, s, lens[s] + round_span(sp)));
    ULB_TRY(prefill_slot(sp, s, lens[s]));
  }
  std::vector<int32_t> L(S), done(S);
  for (int s = 0; s < S; ++s) {
    L[s] = lens[s] + 1;
    done[s] = 1 >= sp->d.max_new;
  }
  ULB_CUDA(cudaMemcpyAsync(sp->L, L.data(), S * 4, cudaMemcpyHostToDevice, c->stream));
  ULB_CUDA(cudaMemcpyAsync(sp->done, done.data(), S * 4, cudaMemcpyHostToDevice, c->stream));
  ULB_TRY(sync_stream(c));
  sp->launches = c->launches - launches0;
  sp->prefilled = true;
  return ULB_OK;
}

int ulb_spec_run(ulb_spec* h, int max_rounds, int* out_rounds) {
  ULB_CHECK(h, ULB_EINVAL, "ulb_spec_run: NULL argument");
  Spec* sp = &h->s;
  ULB_CHECK(sp->prefilled, ULB_EINVAL, "ulb_spec_run: call ulb_spec_prefill first");
  Ctx* c = sp->c;
  ULB_CUDA(cudaSetDevice(c->device));
  if (sp->d.use_graphs && !sp->exec) {
    ULB_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    int rc = record_round(sp);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return cuda_error(e, "capture round", __FILE__, __LINE__);
    e = cudaGraphInstantiate(&sp->exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { sp->exec = nullptr; return cuda_error(e, "instantiate round", __FILE__, __LINE__); }
  }
  const int S = sp->S, R = sp->k + 1;
  int ran = 0;
  while (max_rounds <= 0 || ran < max_rounds) {
    ULB_CUDA(cudaMemcpyAsync(sp->h_L, sp->L, S * 4, cudaMemcpyDeviceToHost, c->stream));
    ULB_CUDA(cudaMemcpyAsync(sp->h_done, sp->done, S * 4, cudaMemcpyDeviceToHost, c->stream));
    ULB_TRY(sync_stream(c));
    int rem_max = 0;
    for (int s = 0; s < S; ++s)
      if (!sp->h_done[s]) rem_max = std::max(rem_max, sp->d.max_new - (sp->h_L[s] - sp->h_plen[s]));
    if (rem_max <= 0) break;
    /* every sequence commits at most k+1 tokens a round: this many rounds are all needed */
    int r = std::max(1, (rem_max + R - 1) / R);
    if (max_rounds > 0) r = std::min(r, max_rounds - ran);
    if (sp->pool) {
      /* finished slots give their pages back; live ones get pages for the positions the next
         r rounds can write (each commits at most k + 1 and writes up to L + k), or for one
         round when the pool is short */
      for (int s = 0; s < S; ++s)
        if (sp->h_done[s]) ULB_TRY(unmap_slot(sp, s));
      for (int attempt = 0;; ++attempt) {
        int rc = ULB_OK;
        for (int s = 0; s < S && rc == ULB_OK; ++s)
          if (!sp->h_done[s]) rc = map_slot(sp, s, sp->h_L[s] + r * R + round_span(sp));
        if (rc == ULB_OK) break;
        if (r == 1 || attempt > 0) return rc;
        r = 1;
      }
    }
    for (int i = 0; i < r; ++i) {
      if (sp->exec) ULB_CUDA(cudaGraphLaunch(sp->exec, c->stream));
      else ULB_TRY(record_round(sp));
      sp->launches += sp->per_round;
    }
    ran += r;
  }
  ULB_TRY(check_device_errors(c));
  int herr = 0;
  ULB_CUDA(cudaMemcpy(&herr, sp->err, 4, cudaMemcpyDeviceToHost));
  ULB_CHECK(!herr, ULB_EINVAL, "ulb_spec_run: a token id fell outside the vocabulary");
  if (out_rounds) *out_rounds = ran;
  return ULB_OK;
}

int ulb_spec_read(ulb_spec* h, int32_t* tokens, int32_t* counts, uint64_t stats[4]) {
  ULB_CHECK(h, ULB_EINVAL, "ulb_spec_read: NULL argument");
  Spec* sp = &h->s;
  ULB_CHECK(sp->prefilled, ULB_EINVAL, "ulb_spec_read: nothing generated");
  Ctx* c = sp->c;
  ULB_CUDA(cudaSetDevice(c->device));
  const int S = sp->S, N = sp->d.max_new;
  std::vector<int32_t> hist((size_t)S * sp->hl), L(S), act(S);
  unsigned long long st[4];
  ULB_CUDA(cudaMemcpyAsync(hist.data(), sp->hist, hist.size() * 4, cudaMemcpyDeviceToHost, c->stream));
  ULB_CUDA(cudaMemcpyAsync(L.data(), sp->L, S * 4, cudaMemcpyDeviceToHost, c->stream));
  ULB_CUDA(cudaMemcpyAsync(act.data(), sp->active, S * 4, cudaMemcpyDeviceToHost, c->stream));
  ULB_CUDA(cudaMemcpyAsync(st, sp->stats, sizeof st, cudaMemcpyDeviceToHost, c->stream));
  ULB_TRY(sync_stream(c));
  for (int s = 0; s < S; ++s) {
    const int P = sp->h_plen[s];
    const int cnt = std::min(L[s] - P, N);
    if (counts) counts[s] = cnt;
    if (tokens)
      for (int i = 0; i < N; ++i) tokens[(size_t)s * N + i] = i < cnt ? hist[(size_t)s * sp->hl + P + i] : -1;
  }
  if (stats) {
    stats[0] = 0;
    for (int s = 0; s < S; ++s) stats[0] = std::max<uint64_t>(stats[0], (uint64_t)act[s]);
    stats[1] = st[1];
    stats[2] = st[2];
    stats[3] = st[3];
  }
  return ULB_OK;
}

int ulb_spec_admit(ulb_spec* h, int slot, const int32_t* prompt, int len) {
  ULB_CHECK(h && prompt, ULB_EINVAL, "ulb_spec_admit: NULL argument");
  Spec* sp = &h->s;
  ULB_CHECK(sp->prefilled, ULB_EINVAL, "ulb_spec_admit: call ulb_spec_prefill first");
  ULB_CHECK(slot >= 0 && slot < sp->S, ULB_EINVAL, "ulb_spec_admit: slot %d of %d", slot, sp->S);
  ULB_CHECK(len >= 1 && len <= sp->d.max_prompt, ULB_EINVAL, "ulb_spec_admit: prompt length %d outside [1, %d]", len,
            sp->d.max_prompt);
  for (int i = 0; i < len; ++i)
    ULB_CHECK(prompt[i] >= 0 && prompt[i] < sp->V, ULB_EINVAL, "ulb_spec_admit: token %d = %d outside the vocabulary",
              i, prompt[i]);
  Ctx* c = sp->c;
  ULB_CUDA(cudaSetDevice(c->device));
  int32_t done = 0;
  ULB_CUDA(cudaMemcpyAsync(&done, sp->done + slot, 4, cudaMemcpyDeviceToHost, c->stream));
  ULB_TRY(sync_stream(c));
  ULB_CHECK(done, ULB_EINVAL, "ulb_spec_admit: slot %d is still decoding", slot);
  /* the slot starts over: its pages, prompt, lengths and counters */
  ULB_TRY(unmap_slot(sp, slot));
  ULB_TRY(map_slot(sp, slot, len + round_span(sp)));
  const int32_t zero = 0;
  ULB_CUDA(cudaMemcpyAsync(sp->hist + (size_t)slot * sp->hl, prompt, (size_t)len * 4, cudaMemcpyHostToDevice, c->stream));
  ULB_CUDA(cudaMemcpyAsync(sp->plen + slot, &len, 4, cudaMemcpyHostToDevice, c->stream));
  ULB_CUDA(cudaMemcpyAsync(sp->round + slot, &zero, 4, cudaMemcpyHostToDevice, c->stream));
  ULB_CUDA(cudaMemcpyAsync(sp->active + slot, &zero, 4, cudaMemcpyHostToDevice, c->stream));
  sp->h_plen[slot] = len;
  const uint64_t launches0 = c->launches;
  ULB_TRY(prefill_slot(sp, slot, len));
  const int32_t L = len + 1, dn = 1 >= sp->d.max_new;
  ULB_CUDA(cudaMemcpyAsync(sp->L + slot, &L, 4, cudaMemcpyHostToDevice, c->stream));
  ULB_CUDA(cudaMemcpyAsync(sp->done + slot, &dn, 4, cudaMemcpyHostToDevice, c->stream));
  ULB_TRY(sync_stream(c));
  sp->launches += c->launches - launches0;
  return ULB_OK;
}

int ulb_spec_read_rounds(ulb_spec* h, int seq, int max_records, int32_t* out, int* out_n) {
  ULB_CHECK(h && out_n, ULB_EINVAL, "ulb_spec_read_rounds: NULL argument");
  Spec* sp = &h->s;
  ULB_CHECK(sp->prefilled, ULB_EINVAL, "ulb_spec_read_rounds: nothing generated");
  ULB_CHECK(seq >= 0 && seq < sp->S, ULB_EINVAL, "ulb_spec_read_rounds: sequence %d of %d", seq, sp->S);
  Ctx* c = sp->c;
  ULB_CUDA(cudaSetDevice(c->device));
  int32_t act = 0;
  ULB_CUDA(cudaMemcpyAsync(&act, sp->active + seq, 4, cudaMemcpyDeviceToHost, c->stream));
  ULB_TRY(sync_stream(c));
  const int n = std::min(act, sp->log_rounds);
  *out_n = n;
  if (!out || max_records <= 0 || n == 0) return ULB_OK;
  const size_t words = (size_t)ULB_SPEC_REC_WORDS(sp->k);
  const size_t take = (size_t)std::min(n, max_records) * words;
  ULB_CUDA(cudaMemcpyAsync(out, sp->log + (size_t)seq * sp->log_rounds * words, take * 4, cudaMemcpyDeviceToHost,
                           c->stream));
  ULB_TRY(sync_stream(c));
  return ULB_OK;
}

int ulb_spec_profile_round(ulb_spec* h, float ms[3]) {
  ULB_CHECK(h && ms, ULB_EINVAL, "ulb_spec_profile_round: NULL argument");
  Spec* sp = &h->s;
  ULB_CHECK(sp->prefilled, ULB_EINVAL, "ulb_spec_profile_round: call ulb_spec_prefill first");
  Ctx* c = sp->c;
  ULB_CUDA(cudaSetDevice(c->device));
  cudaEvent_t ev[4];
  for (auto& e : ev) ULB_CUDA(cudaEventCreate(&e));
  int rc = ULB_OK;
  cudaError_t e = cudaEventRecord(ev[0], c->stream);
  if (e == cudaSuccess) rc = record_round(sp, ev[1], ev[2]);
  else rc = cuda_error(e, "event", __FILE__, __LINE__);
  if (rc == ULB_OK) {
    sp->launches += sp->per_round;
    e = cudaEventRecord(ev[3], c->stream);
    if (e == cudaSuccess) {
      const int src = sync_stream(c); /* bounded when the round holds tensor-parallel collectives */
      if (src != ULB_OK) {
        for (auto& x : ev) cudaEventDestroy(x);
        return src;
      }
    }
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms[0], ev[0], ev[1]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms[1], ev[1], ev[2]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms[2], ev[2], ev[3]);
    if (e != cudaSuccess) rc = cuda_error(e, "profile round", __FILE__, __LINE__);
  }
  for (auto& x : ev) cudaEventDestroy(x);
  return rc;
}

int ulb_spec_profile_round_ex(ulb_spec* h, float ms[5]) {
  ULB_CHECK(h && ms, ULB_EINVAL, "ulb_spec_profile_round_ex: NULL argument");
  Spec* sp = &h->s;
  Ctx* c = sp->c;
  ULB_CUDA(cudaSetDevice(c->device));
  /* two events per all-reduce: 2 per layer of the target's verify forward (and of the draft's
     forwards, which are replicated and do not all-reduce) */
  if (c->nccl) {
    const size_t need = (size_t)4 * 512;
    while (c->ar_events.size() < need) {
      cudaEvent_t e;
      ULB_CUDA(cudaEventCreate(&e));
      c->ar_events.push_back(e);
    }
  }
  c->ar_used = 0;
  c->ar_timing = c->nccl != nullptr;
  const int rc = ulb_spec_profile_round(h, ms);
  c->ar_timing = false;
  ms[3] = 0.f;
  ms[4] = (float)(c->ar_used / 2);
  if (rc != ULB_OK) return rc;
  for (size_t i = 0; i + 1 < c->ar_used; i += 2) {
    float t = 0.f;
    ULB_CUDA(cudaEventElapsedTime(&t, c->ar_events[i], c->ar_events[i + 1]));
    ms[3] += t;
  }
  return ULB_OK;
}

int ulb_spec_launch_count(ulb_spec* h, uint64_t* out) {
  ULB_CHECK(h && out, ULB_EINVAL, "ulb_spec_launch_count: NULL argument");
  *out = h->s.launches;
  return ULB_OK;
}

int ulb_spec_free(ulb_spec* h) {
  if (!h) return ULB_OK;
  cudaSetDevice(h->s.c->device);
  spec_release(&h->s);
  delete h;
  return ULB_OK;
}

}  // extern "C"

ULB_TRACE_UNIT(spec)
