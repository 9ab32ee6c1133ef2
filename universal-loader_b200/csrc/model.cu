/*
 * model.cu — LLaMA-family model resident in HBM, KV cache, and one forward pass.
 *
 * Replaces Model / LayerWeights / KVCache (src/inference/model.h:37-115,
 * model.cpp:11-131,154-254) and the per-layer GPU forward
 * (src/inference/inference_engine.cpp:475-692), keeping its op order
 *   norm -> Q,K,V -> RoPE -> attention -> o -> +res -> norm -> gate,up -> SiLU*mul -> down -> +res
 * with each op given its LLaMA meaning and fused as:
 *   rmsnorm(fp16 out) | QKV-GEMV (+RoPE, K/V -> cache) | attention | O-GEMV (+residual)
 *   | rmsnorm | gate/up-GEMV (+SiLU*up) | down-GEMV (+residual)
 * Tensors are named as in GGUF (the reference maps only a subset and misses the
 * blk.N.ffn_* names, model.cpp:232-245).
 */
#include <cmath>
#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "ulb_internal.h"

namespace ulb {

struct RawW {
  int type = 0;
  uint64_t ne[4] = {1, 1, 1, 1};
  void* dev = nullptr;
  size_t bytes = 0;
};

struct Layer {
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  Tensor qkv, o, gateup, down;
  /* attn_v kept as GGUF rows (Q8_0 / Q6_K / F16 / F32, as llama.cpp's K-quant mixes store it):
     qkv then holds Q and K only and v writes the V cache through the row GEMV */
  Tensor v;
};

struct Model {
  Ctx* c = nullptr;
  ulb_model_desc d{};   /* this rank's shapes (heads, d_ff divided by tp_world) */
  ulb_model_desc gd{};  /* the whole model's shapes */
  int tp_rank = 0, tp_world = 1;
  int nq = 0, nkv = 0;
  std::map<std::string, RawW> raw;
  bool finalized = false;
  int embd_type = ULB_TYPE_F16;
  void* embd = nullptr;
  size_t embd_bytes = 0;
  std::vector<Layer> layers;
  float* out_norm = nullptr;
  Tensor out;
  bool out_shared = false; /* out.dev is the token_embd buffer (tied F16 / F32 / Q8_0 / Q6_K rows) */
  size_t weight_bytes = 0;
  /* workspace */
  int ws_rows = 0;
  float* x = nullptr;
  __half* x16 = nullptr;
  float* qb = nullptr;
  __half* att = nullptr;
  __half* h16 = nullptr;
  float* tp_part = nullptr; /* [rows][d] partial attn_output / ffn_down sums (tensor parallel) */
  size_t ws_bytes = 0;
};

struct KV {
  Model* m = nullptr;
  int n_seq = 0, cap = 0;
  /* paged: per layer a pool of n_pages pages [page][n_head_kv][kKvPage][head_dim] for K and
     for V; sequence s's position p lives in page bt[s * max_pages + p / kKvPage] */
  int n_pages = 0, max_pages = 0;
  int* bt = nullptr;
  std::vector<int> h_bt;
  bool identity = false; /* bt is the identity table: kernels compute pages instead of loading them */
  __half* k = nullptr;
  __half* v = nullptr;
  size_t layer_elems = 0;
  size_t bytes = 0;
  float2* rope = nullptr;
  size_t rope_bytes = 0;
  float* attn_scratch = nullptr;
  size_t attn_floats = 0;
  int* attn_counters = nullptr;
  int n_counters = 0;
};

namespace {

/* element i of one token_embd row in fp32, by the GGUF block formulas (single roundings in
   the order of the oracle's orc_dequant):
     Q4_0 d * (q - 8); Q8_0 d * q; Q4_K (d * sc_j) * q - (dmin * m_j);
     Q6_K (d * sc_j) * (q - 32), sc_j per 16 weights (ql / qh / scales / d layout of block_q6_K) */
__device__ __forceinline__ float embd_value(const uint8_t* __restrict__ row, int type, int i) {
  auto half_at = [](const uint8_t* p) { return __half2float(*reinterpret_cast<const __half*>(p)); };
  switch (type) {
    case ULB_TYPE_F16: return __half2float(reinterpret_cast<const __half*>(row)[i]);
    case ULB_TYPE_F32: return reinterpret_cast<const float*>(row)[i];
    case ULB_TYPE_Q4_0: {
      const uint8_t* blk = row + (size_t)(i / 32) * 18;
      const int j = i % 32;
      const int q = (j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4)) - 8;
      return __fmul_rn(half_at(blk), (float)q);
    }
    case ULB_TYPE_Q8_0: {
      const uint8_t* blk = row + (size_t)(i / 32) * 34;
      return __fmul_rn(half_at(blk), (float)(int8_t)blk[2 + i % 32]);
    }
    case ULB_TYPE_Q4_K: {
      const uint8_t* blk = row + (size_t)(i / 256) * 144;
      const int ii = i % 256, j = ii / 32;
      const uint8_t* sc12 = blk + 4;
      int sc, mn;
      if (j < 4) {
        sc = sc12[j] & 63;
        mn = sc12[j + 4] & 63;
      } else {
        sc = (sc12[j + 4] & 0x0F) | ((sc12[j - 4] >> 6) << 4);
        mn = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
      }
      const uint8_t qb = blk[16 + 32 * (ii / 64) + ii % 32];
      const int q = ((ii / 32) & 1) ? (qb >> 4) : (qb & 15);
      const float s = __fmul_rn(half_at(blk), (float)sc), m = __fmul_rn(half_at(blk + 2), (float)mn);
      return __fsub_rn(__fmul_rn(s, (float)q), m);
    }
    default: { /* ULB_TYPE_Q6_K */
      const uint8_t* blk = row + (size_t)(i / 256) * 210;
      const int ii = i % 256, h = ii / 128, r = ii % 128, k = r / 32, l = r % 32;
      const int lo = (blk[64 * h + l + 32 * (k & 1)] >> (k >= 2 ? 4 : 0)) & 15;
      const int hi = (blk[128 + 32 * h + l] >> (2 * k)) & 3;
      const float step = __fmul_rn(half_at(blk + 208), (float)(int8_t)blk[192 + ii / 16]);
      return __fmul_rn(step, (float)((lo | (hi << 4)) - 32));
    }
  }
}

/* one thread per element: CTA (m, y) writes elements [256 y, 256 y + 256) of row m, so every
   load of the row is in flight at once */
__global__ void embed_kernel(const void* __restrict__ table, int table_type, size_t row_bytes, int d, int V,
                             const int* __restrict__ tokens, float* __restrict__ x, int* err) {
  ULB_TRACE_KERNEL(kTrEmbed, d);
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x, i = blockIdx.y * blockDim.x + threadIdx.x;
  int t = tokens[m];
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0 && blockIdx.y == 0) atomicOr(err, 1);
    t = t < 0 ? 0 : V - 1;
  }
  const uint8_t* row = reinterpret_cast<const uint8_t*>(table) + (size_t)t * row_bytes;
  if (i < d) x[(size_t)m * d + i] = embd_value(row, table_type, i);
}

/* out[s] = fp16((x[row] * r) * g), r = 1 / sqrt(mean(x^2) + eps); row = s*sel + sel-1 if sel.
   256 threads (rms_row_256). */
__global__ void rmsnorm_kernel(const float* __restrict__ x, int ldx, const float* __restrict__ g, int d, float eps,
                               int sel, __half* __restrict__ out, int ldo) {
  ULB_TRACE_KERNEL(kTrRmsnorm, d);
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x;
  const int row = sel > 0 ? s * sel + sel - 1 : s;
  rms_row_256(x + (size_t)row * ldx, g, d, eps, out + (size_t)s * ldo, red);
}

}  // namespace

int launch_embed_t(Ctx* c, const void* table, int type, int d, int V, const int* tokens, int M, float* x, int* err) {
  if (M == 0) return ULB_OK;
  size_t row_bytes = 0;
  switch (type) {
    case ULB_TYPE_F32: row_bytes = (size_t)d * 4; break;
    case ULB_TYPE_F16: row_bytes = (size_t)d * 2; break;
    case ULB_TYPE_Q4_0: row_bytes = d % 32 ? 0 : (size_t)d / 32 * 18; break;
    case ULB_TYPE_Q8_0: row_bytes = d % 32 ? 0 : (size_t)d / 32 * 34; break;
    case ULB_TYPE_Q4_K: row_bytes = d % 256 ? 0 : (size_t)d / 256 * 144; break;
    case ULB_TYPE_Q6_K: row_bytes = d % 256 ? 0 : (size_t)d / 256 * 210; break;
    default: break;
  }
  ULB_CHECK(row_bytes, ULB_EUNSUPPORTED, "embedding: table type %d with d=%d", type, d);
  cudaError_t e = launch_k(c, embed_kernel, dim3(M, (d + 255) / 256), dim3(256), 0, table, type, row_bytes, d, V, tokens,
                           x, err);
  if (e != cudaSuccess) return cuda_error(e, "embed launch", __FILE__, __LINE__);
  return ULB_OK;
}

int launch_rmsnorm_sel(Ctx* c, const float* x, int ldx, const float* g, int n_out, int d, float eps, int sel,
                       __half* out, int ldo) {
  if (n_out == 0) return ULB_OK;
  cudaError_t e = launch_k(c, rmsnorm_kernel, dim3(n_out), dim3(256), 0, x, ldx, g, d, eps, sel, out, ldo);
  if (e != cudaSuccess) return cuda_error(e, "rmsnorm launch", __FILE__, __LINE__);
  return ULB_OK;
}

static int ensure_ws(Model* m, int rows) {
  if (rows <= m->ws_rows) return ULB_OK;
  Ctx* c = m->c;
  dev_free(c, m->x, 0); dev_free(c, m->x16, 0); dev_free(c, m->qb, 0); dev_free(c, m->att, 0); dev_free(c, m->h16, 0);
  dev_free(c, m->tp_part, 0);
  m->tp_part = nullptr;
  c->bytes_live -= m->ws_bytes;
  m->ws_bytes = 0;
  m->ws_rows = 0;
  const ulb_model_desc& d = m->d;
  const size_t R = (size_t)rows;
  const size_t bx = R * d.d_model * 4, bx16 = R * d.d_model * 2, bq = R * m->nq * 4, ba = R * m->nq * 2,
               bh = R * d.d_ff * 2;
  ULB_TRY(dev_alloc(c, (void**)&m->x, bx));
  ULB_TRY(dev_alloc(c, (void**)&m->x16, bx16));
  ULB_TRY(dev_alloc(c, (void**)&m->qb, bq));
  ULB_TRY(dev_alloc(c, (void**)&m->att, ba));
  ULB_TRY(dev_alloc(c, (void**)&m->h16, bh));
  m->ws_bytes = bx + bx16 + bq + ba + bh;
  if (m->tp_world > 1) {
    ULB_TRY(dev_alloc(c, (void**)&m->tp_part, bx));
    m->ws_bytes += bx;
  }
  m->ws_rows = rows;
  return ULB_OK;
}

static int ensure_attn(KV* kv, int M, int rps, bool tree) {
  const ulb_model_desc& d = kv->m->d;
  ulb_attn_desc ad{d.n_head, d.n_head_kv, d.head_dim, kv->cap, kv->n_seq, 1.0f / std::sqrt((float)d.head_dim)};
  int nc = 0;
  size_t nf = 0;
  ULB_TRY(attention_scratch_need(kv->m->c, &ad, M, rps, kv->cap - 1, &nf, &nc, tree, /*bound=*/true));
  if (nf <= kv->attn_floats && nc <= kv->n_counters) return ULB_OK;
  /* grow to the largest shape seen so far: every prepared shape must keep fitting */
  const size_t f2 = nf > kv->attn_floats ? nf : kv->attn_floats;
  const int c2 = nc > kv->n_counters ? nc : kv->n_counters;
  Ctx* c = kv->m->c;
  dev_free(c, kv->attn_scratch, kv->attn_floats * 4);
  dev_free(c, kv->attn_counters, (size_t)kv->n_counters * 4);
  kv->attn_scratch = nullptr; kv->attn_counters = nullptr; kv->attn_floats = 0; kv->n_counters = 0;
  ULB_TRY(dev_alloc(c, (void**)&kv->attn_scratch, f2 * 4));
  kv->attn_floats = f2;
  ULB_TRY(dev_alloc(c, (void**)&kv->attn_counters, (size_t)c2 * 4));
  kv->n_counters = c2;
  ULB_CUDA(cudaMemsetAsync(kv->attn_counters, 0, (size_t)c2 * 4, c->stream));
  return ULB_OK;
}

/* Make workspaces large enough for a forward of M rows (rps per sequence).  Must be called
 * before a forward is captured into a CUDA graph. */
int model_prepare(Model* m, KV* kv, int M, int rps, bool tree) {
  ULB_TRY(ensure_ws(m, M));
  ULB_TRY(ensure_attn(kv, M, rps, tree));
  return ULB_OK;
}

/* x += part, elementwise (the residual add after a tensor-parallel all-reduce) */
__global__ void add_inplace_kernel(float* __restrict__ x, const float* __restrict__ part, size_t n) {
  ULB_TRACE_KERNEL(kTrAdd, 0);
  pdl_wait();
  pdl_trigger();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = x[i] + part[i];
}

static int tp_reduce_add(Model* m, int M) {
  Ctx* c = m->c;
  const size_t n = (size_t)M * m->d.d_model;
  ULB_TRY(tp_allreduce_sum(c, m->tp_part, n));
  const int grid = (int)std::min<size_t>((n + 255) / 256, (size_t)c->n_sm * 4);
  cudaError_t e = launch_k(c, add_inplace_kernel, dim3(grid), dim3(256), 0, m->x, (const float*)m->tp_part, n);
  if (e != cudaSuccess) return cuda_error(e, "residual add", __FILE__, __LINE__);
  return ULB_OK;
}

/* final RMSNorm (of every row, or of each sequence's last row) and the LM head, one kernel for
   up to 8 rows */
static int forward_head(Model* m, int M, int rps, int logits_mode, float* logits, int ld) {
  Ctx* c = m->c;
  const ulb_model_desc& d = m->d;
  const int n_out = logits_mode == 1 ? M / rps : M;
  /* the rows the logits come from: every row, or the last of each sequence's rps (a strided
     view of the residual stream) */
  const int sel = logits_mode == 1 ? rps : 1;
  EpiArgs o;
  o.y = logits;
  o.ldy = ld;
  return launch_qgemv_rms(c, &m->out, m->x + (size_t)(sel - 1) * d.d_model, sel * d.d_model, m->out_norm, d.rms_eps,
                          m->x16, n_out, EPI_STORE, o);
}

/* After a tree round: sequence s accepted n = comp[s][1] nodes; node comp[s][2 + j] sits in
   cache slot L + node (L = comp[s][0]) and moves to its sequence position L + j, in every layer,
   K and V.  Grid (layers, sequences); each thread copies the same 16-byte chunks of every row
   it moves, in path order, so a row moved into a later node's old slot was read first (the
   destinations L + j never exceed a later node's source). */
__global__ void kv_tree_compact_kernel(__half* __restrict__ kc, __half* __restrict__ vc, size_t layer_elems, int Hkv,
                                       int hd, int cap, const int* __restrict__ bt, int max_pages,
                                       const int32_t* __restrict__ comp, int D) {
  ULB_TRACE_KERNEL(kTrStageTree + 50, 0);
  pdl_wait();
  pdl_trigger();
  const int l = blockIdx.x, s = blockIdx.y;
  const int32_t* cp = comp + (size_t)s * (2 + D);
  const int L = cp[0], n = cp[1];
  __half* kl = kc + (size_t)l * layer_elems;
  __half* vl = vc + (size_t)l * layer_elems;
  /* the head-0 row of position pos, heads `hs` elements apart; false for an unmapped page */
  auto row_of = [&](int pos, size_t* base, size_t* hs) -> bool {
    if (max_pages > 0) {
      const int slot = s * max_pages + pos / kKvPage;
      const int page = bt ? bt[slot] : slot;
      if (page < 0) return false;
      *base = ((size_t)page * Hkv * kKvPage + pos % kKvPage) * hd;
      *hs = (size_t)kKvPage * hd;
    } else {
      *base = ((size_t)s * Hkv * cap + pos) * hd;
      *hs = (size_t)cap * hd;
    }
    return true;
  };
  const int cpr = hd / 8; /* 16-byte chunks per head row */
  for (int j = 0; j < n; ++j) {
    const int src = L + cp[2 + j], dst = L + j;
    size_t sb, db, hs;
    if (src == dst || src >= cap || dst < 0 || !row_of(src, &sb, &hs) || !row_of(dst, &db, &hs)) continue;
    for (int e = threadIdx.x; e < Hkv * cpr; e += blockDim.x) {
      const int h = e / cpr, c = e % cpr;
      const size_t a = sb + h * hs + c * 8, b = db + h * hs + c * 8;
      *reinterpret_cast<uint4*>(kl + b) = *reinterpret_cast<const uint4*>(kl + a);
      *reinterpret_cast<uint4*>(vl + b) = *reinterpret_cast<const uint4*>(vl + a);
    }
  }
}

int kv_tree_compact(KV* kv, const int32_t* comp, int S, int D) {
  Model* m = kv->m;
  const ulb_model_desc& d = m->d;
  cudaError_t e = launch_k(m->c, kv_tree_compact_kernel, dim3(d.n_layer, S), dim3(256), 0, kv->k, kv->v,
                           kv->layer_elems, d.n_head_kv, d.head_dim, kv->cap, (const int*)(kv->identity ? nullptr : kv->bt),
                           kv->max_pages, comp, D);
  if (e != cudaSuccess) return cuda_error(e, "tree cache compaction", __FILE__, __LINE__);
  return ULB_OK;
}

int model_forward(Model* m, KV* kv, int M, int rps, const int* tok, const int* seq, const int* pos, int logits_mode,
                  float* logits, int ld, int* err, const TreeRows* tree) {
  Ctx* c = m->c;
  const ulb_model_desc& d = m->d;
  ULB_CHECK(m->finalized, ULB_EINVAL, "forward: model not finalized");
  ULB_CHECK(kv && kv->m == m, ULB_EINVAL, "forward: KV cache belongs to another model");
  ULB_CHECK(M > 0 && rps > 0 && M % rps == 0, ULB_EINVAL, "forward: M=%d rows_per_seq=%d", M, rps);
  ULB_CHECK(M <= m->ws_rows, ULB_EINVAL, "forward: M=%d exceeds prepared workspace (%d rows)", M, m->ws_rows);
  ULB_CHECK(ld >= d.n_vocab, ULB_EINVAL, "forward: ld %d < n_vocab %d", ld, d.n_vocab);
  ulb_attn_desc ad{d.n_head, d.n_head_kv, d.head_dim, kv->cap, kv->n_seq, 1.0f / std::sqrt((float)d.head_dim)};
  ULB_TRY(launch_embed_t(c, m->embd, m->embd_type, d.d_model, d.n_vocab, tok, M, m->x, err));
  for (int l = 0; l < d.n_layer; ++l) {
    Layer& L = m->layers[l];
    __half* kc = kv->k + (size_t)l * kv->layer_elems;
    __half* vc = kv->v + (size_t)l * kv->layer_elems;
    EpiArgs a;
    a.q = m->qb; a.ldq = m->nq; a.kc = kc; a.vc = vc;
    a.nq = m->nq; a.nkv = m->nkv; a.hd = d.head_dim; a.cap = kv->cap; a.n_head_kv = d.n_head_kv; a.n_seq = kv->n_seq;
    a.row_seq = seq; a.row_pos = pos; a.rope = kv->rope;
    a.bt = kv->identity ? nullptr : kv->bt; a.max_pages = kv->max_pages;
    a.row_rope = tree ? tree->rope : nullptr;
    if (L.v.dev) { /* V as GGUF rows: the normalised rows in x16 feed the Q / K GEMV and V's row GEMV */
      ULB_TRY(launch_rmsnorm_sel(c, m->x, d.d_model, L.attn_norm, M, d.d_model, d.rms_eps, 0, m->x16, d.d_model));
      ULB_TRY(launch_qgemv(c, &L.qkv, m->x16, M, d.d_model, EPI_QKV, a));
      ULB_TRY(launch_qgemv(c, &L.v, m->x16, M, d.d_model, EPI_VCACHE, a));
    } else {
      ULB_TRY(launch_qgemv_rms(c, &L.qkv, m->x, d.d_model, L.attn_norm, d.rms_eps, m->x16, M, EPI_QKV, a));
    }
    ULB_TRY(launch_attention(c, &ad, m->qb, m->nq, kc, vc, seq, pos, M, rps, m->att, kv->attn_scratch,
                             kv->attn_counters, kv->attn_floats, kv->n_counters, kv->identity ? nullptr : kv->bt,
                             kv->max_pages, tree ? tree->pref : nullptr, tree ? tree->mask : nullptr));
    EpiArgs r;
    r.y = m->x; r.ldy = d.d_model;
    /* tensor parallel: this rank's heads / features give a partial sum of attn_output and
       ffn_down; the ranks' partials are summed (NCCL, fp32) before the residual add */
    EpiArgs pr;
    pr.y = m->tp_part; pr.ldy = d.d_model;
    const bool tp = m->tp_world > 1;
    ULB_TRY(launch_qgemv(c, &L.o, m->att, M, m->nq, tp ? EPI_STORE : EPI_RESID, tp ? pr : r));
    if (tp) ULB_TRY(tp_reduce_add(m, M));
    EpiArgs s;
    s.h = m->h16; s.ldh = d.d_ff;
    ULB_TRY(launch_qgemv_rms(c, &L.gateup, m->x, d.d_model, L.ffn_norm, d.rms_eps, m->x16, M, EPI_SWIGLU, s));
    ULB_TRY(launch_qgemv(c, &L.down, m->h16, M, d.d_ff, tp ? EPI_STORE : EPI_RESID, tp ? pr : r));
    if (tp) ULB_TRY(tp_reduce_add(m, M));
  }
  return forward_head(m, M, rps, logits_mode, logits, ld);
}

}  // namespace ulb

struct ulb_model {
  ulb::Model m;
};
struct ulb_kv {
  ulb::KV kv;
};

namespace ulb {
Model* model_of(ulb_model* m) { return &m->m; }
KV* kv_of(ulb_kv* kv) { return &kv->kv; }
int model_vocab(const Model* m) { return m->d.n_vocab; }
}  // namespace ulb

using namespace ulb;

namespace {

int upload_plain(Ctx* c, const RawW& r, void** out, size_t* bytes) {
  *bytes = r.bytes;
  ULB_TRY(dev_alloc(c, out, r.bytes));
  ULB_CUDA(cudaMemcpyAsync(*out, r.dev, r.bytes, cudaMemcpyDeviceToDevice, c->stream));
  return ULB_OK;
}

/* concatenate raw rows of several same-type matrices and repack with a row map */
int build_fused(Ctx* c, const std::vector<const RawW*>& parts, const std::vector<int>& map, Tensor* out) {
  const int type = parts[0]->type;
  const int K = (int)parts[0]->ne[0];
  size_t total = 0;
  int rows = 0;
  for (const RawW* p : parts) {
    ULB_CHECK(p->type == type, ULB_EFORMAT, "fused weights must share one quant type");
    ULB_CHECK((int)p->ne[0] == K, ULB_EFORMAT, "fused weights must share K");
    total += p->bytes;
    rows += (int)p->ne[1];
  }
  void* cat = nullptr;
  ULB_TRY(dev_alloc(c, &cat, total));
  size_t off = 0;
  for (const RawW* p : parts) {
    cudaError_t e = cudaMemcpyAsync((uint8_t*)cat + off, p->dev, p->bytes, cudaMemcpyDeviceToDevice, c->stream);
    if (e != cudaSuccess) { dev_free(c, cat, total); return cuda_error(e, "concat", __FILE__, __LINE__); }
    off += p->bytes;
  }
  int rc = repack_q4(c, type, cat, rows, K, map.data(), (int)map.size(), out);
  dev_free(c, cat, total);
  if (rc) return rc;
  out->N = (int)map.size();
  out->ne[0] = (uint64_t)K;
  out->ne[1] = (uint64_t)out->N;
  return ULB_OK;
}

int build_plain(Ctx* c, const RawW& r, Tensor* out) {
  const int N = (int)r.ne[1], K = (int)r.ne[0];
  const int rows = (N + 15) / 16 * 16;
  std::vector<int> map(rows);
  for (int i = 0; i < rows; ++i) map[i] = i < N ? i : -1;
  ULB_TRY(repack_q4(c, r.type, r.dev, N, K, map.data(), rows, out));
  out->N = N;
  out->ne[0] = (uint64_t)K;
  out->ne[1] = (uint64_t)N;
  return ULB_OK;
}

/* a matrix kept as its GGUF rows, for the row GEMV */
int build_raw(Ctx* c, const RawW& r, Tensor* out) {
  out->type = r.type;
  out->N = (int)r.ne[1];
  out->K = (int)r.ne[0];
  out->ne[0] = r.ne[0];
  out->ne[1] = r.ne[1];
  return upload_plain(c, r, &out->dev, &out->bytes);
}

void free_tensor(Ctx* c, Tensor& t) {
  dev_free(c, t.dev, t.bytes);
  t.dev = nullptr;
}

}  // namespace

namespace ulb {
namespace {
/* GGUF bytes of one row of ne0 elements */
size_t gguf_row_bytes(int type, uint64_t ne0) {
  switch (type) {
    case ULB_TYPE_F32: return ne0 * 4;
    case ULB_TYPE_F16: return ne0 * 2;
    case ULB_TYPE_Q4_0: return ne0 / 32 * 18;
    case ULB_TYPE_Q4_K: return ne0 / 256 * 144;
    case ULB_TYPE_Q8_0: return ne0 / 32 * 34;
    case ULB_TYPE_Q6_K: return ne0 / 256 * 210;
    default: return 0;
  }
}
/* this rank's part of a tensor: rows [r0, r0 + nr) or, with kslice, columns [k0, k0 + nk) of every row */
int tp_slice(Model* m, const std::string& nm, int type, const uint64_t ne[4], const uint8_t* src,
             std::vector<uint8_t>* out, uint64_t ne_out[4]) {
  const ulb_model_desc& l = m->d;
  const int hd = l.head_dim, r = m->tp_rank;
  uint64_t rows = 0, kcols = 0;
  bool ks = false;
  auto ends = [&](const char* suf) { return nm.size() > strlen(suf) && nm.compare(nm.size() - strlen(suf), strlen(suf), suf) == 0; };
  if (ends(".attn_q.weight")) rows = (uint64_t)l.n_head * hd;
  else if (ends(".attn_k.weight") || ends(".attn_v.weight")) rows = (uint64_t)l.n_head_kv * hd;
  else if (ends(".ffn_gate.weight") || ends(".ffn_up.weight")) rows = (uint64_t)l.d_ff;
  else if (ends(".attn_output.weight")) { kcols = (uint64_t)l.n_head * hd; ks = true; }
  else if (ends(".ffn_down.weight")) { kcols = (uint64_t)l.d_ff; ks = true; }
  else return 1; /* replicated */
  memcpy(ne_out, ne, 4 * sizeof(uint64_t));
  const size_t rb = gguf_row_bytes(type, ne[0]);
  ULB_CHECK(rb > 0, ULB_EUNSUPPORTED, "%s: tensor type %d cannot be sliced", nm.c_str(), type);
  if (!ks) {
    ULB_CHECK(ne[1] == rows * m->tp_world, ULB_EFORMAT, "%s: %llu rows, expected %llu", nm.c_str(),
              (unsigned long long)ne[1], (unsigned long long)(rows * m->tp_world));
    out->assign(src + (size_t)r * rows * rb, src + (size_t)(r + 1) * rows * rb);
    ne_out[1] = rows;
  } else {
    ULB_CHECK(ne[0] == kcols * m->tp_world, ULB_EFORMAT, "%s: K = %llu, expected %llu", nm.c_str(),
              (unsigned long long)ne[0], (unsigned long long)(kcols * m->tp_world));
    const size_t kb = gguf_row_bytes(type, kcols);
    /* each rank's K slice must be whole packed K-tiles (128 weights for Q4_0, 256 for Q4_K) */
    ULB_CHECK(kb > 0 && gguf_row_bytes(type, kcols) * m->tp_world == rb && kcols % (uint64_t)tile_k(type) == 0,
              ULB_EUNSUPPORTED, "%s: a K slice of %llu per rank is not a multiple of the %d-weight tile", nm.c_str(),
              (unsigned long long)kcols, tile_k(type));
    out->resize((size_t)ne[1] * kb);
    for (uint64_t i = 0; i < ne[1]; ++i) memcpy(out->data() + i * kb, src + i * rb + (size_t)r * kb, kb);
    ne_out[0] = kcols;
  }
  return ULB_OK;
}
}  // namespace

}  // namespace ulb

extern "C" {

int ulb_model_create(ulb_ctx* ctx, const ulb_model_desc* d, ulb_model** out) {
  ULB_CHECK(ctx && d && out, ULB_EINVAL, "ulb_model_create: NULL argument");
  ULB_CHECK(d->n_layer > 0 && d->d_model > 0 && d->n_head > 0 && d->n_head_kv > 0 && d->head_dim > 0 && d->d_ff > 0 &&
                d->n_vocab > 0,
            ULB_EINVAL, "ulb_model_create: non-positive dimension");
  ULB_CHECK(d->n_head % d->n_head_kv == 0, ULB_EINVAL, "n_head %d not a multiple of n_head_kv %d", d->n_head, d->n_head_kv);
  ULB_CHECK(d->head_dim % 16 == 0, ULB_EUNSUPPORTED, "head_dim %d must be a multiple of 16", d->head_dim);
  ULB_CHECK(d->d_ff % 8 == 0 && d->d_model % 8 == 0, ULB_EUNSUPPORTED, "d_model/d_ff must be multiples of 8");
  ULB_CHECK(d->d_model <= 8192, ULB_EUNSUPPORTED, "d_model %d > 8192 (rmsnorm keeps a row in registers)", d->d_model);
  std::unique_ptr<ulb_model> m(new ulb_model());
  m->m.c = &ctx->c;
  m->m.d = *d;
  m->m.gd = *d;
  m->m.nq = d->n_head * d->head_dim;
  m->m.nkv = d->n_head_kv * d->head_dim;
  m->m.layers.resize(d->n_layer);
  *out = m.release();
  return ULB_OK;
}

int ulb_model_set_tp(ulb_model* mm, int rank, int world) {
  ULB_CHECK(mm, ULB_EINVAL, "ulb_model_set_tp: NULL model");
  Model* m = &mm->m;
  ULB_CHECK(!m->finalized && m->raw.empty(), ULB_EINVAL, "ulb_model_set_tp: call before the first ulb_model_set_weight");
  ULB_CHECK(world >= 1 && rank >= 0 && rank < world, ULB_EINVAL, "ulb_model_set_tp: rank %d of %d", rank, world);
  if (world > 1)
    ULB_CHECK(m->c->nccl && m->c->tp_rank == rank && m->c->tp_world == world, ULB_EINVAL,
              "ulb_model_set_tp: the context's communicator (ulb_tp_init) is not rank %d of %d", rank, world);
  const ulb_model_desc& g = m->gd;
  ULB_CHECK(g.n_head % world == 0 && g.n_head_kv % world == 0 && g.d_ff % world == 0, ULB_EUNSUPPORTED,
            "tensor parallel: n_head %d, n_head_kv %d and d_ff %d must divide by %d", g.n_head, g.n_head_kv, g.d_ff,
            world);
  ULB_CHECK((g.d_ff / world) % 8 == 0, ULB_EUNSUPPORTED, "tensor parallel: d_ff / world = %d not a multiple of 8",
            g.d_ff / world);
  m->tp_rank = rank;
  m->tp_world = world;
  m->d = g;
  m->d.n_head = g.n_head / world;
  m->d.n_head_kv = g.n_head_kv / world;
  m->d.d_ff = g.d_ff / world;
  m->nq = m->d.n_head * m->d.head_dim;
  m->nkv = m->d.n_head_kv * m->d.head_dim;
  return ULB_OK;
}

int ulb_model_set_weight(ulb_model* mm, const char* name, int type, const uint64_t ne_in[4], const void* bytes_in,
                         size_t nbytes_in) {
  ULB_CHECK(mm && name && ne_in && bytes_in, ULB_EINVAL, "ulb_model_set_weight: NULL argument");
  Model* m = &mm->m;
  ULB_CHECK(!m->finalized, ULB_EINVAL, "ulb_model_set_weight: model already finalized");
  const uint64_t* ne = ne_in;
  const void* bytes = bytes_in;
  size_t nbytes = nbytes_in;
  std::vector<uint8_t> part;
  uint64_t ne_part[4];
  if (m->tp_world > 1) {
    const uint64_t n_in = ne_in[0] * ne_in[1] * ne_in[2] * ne_in[3];
    ULB_CHECK(gguf_row_bytes(type, ne_in[0]) * (n_in / std::max<uint64_t>(ne_in[0], 1)) == nbytes_in, ULB_EFORMAT,
              "%s: %zu bytes do not match its shape", name, nbytes_in);
    const int rc = tp_slice(m, name, type, ne_in, (const uint8_t*)bytes_in, &part, ne_part);
    if (rc < 0) return rc;
    if (rc == ULB_OK) {
      ne = ne_part;
      bytes = part.data();
      nbytes = part.size();
    }
  }
  const uint64_t n = ne[0] * ne[1] * ne[2] * ne[3];
  size_t want = 0;
  switch (type) {
    case ULB_TYPE_F32: want = n * 4; break;
    case ULB_TYPE_F16: want = n * 2; break;
    case ULB_TYPE_Q4_0: want = ne[0] % 32 ? 0 : n / 32 * 18; break;
    case ULB_TYPE_Q4_K: want = ne[0] % 256 ? 0 : n / 256 * 144; break;
    case ULB_TYPE_Q8_0: want = ne[0] % 32 ? 0 : n / 32 * 34; break;
    case ULB_TYPE_Q6_K: want = ne[0] % 256 ? 0 : n / 256 * 210; break;
    default: return set_error(ULB_EUNSUPPORTED, "%s: tensor type %d not supported", name, type);
  }
  ULB_CHECK(want && want == nbytes, ULB_EFORMAT, "%s: %zu bytes, GGUF size is %zu", name, nbytes, want);
  Ctx* c = m->c;
  ULB_CUDA(cudaSetDevice(c->device));
  auto it = m->raw.find(name);
  if (it != m->raw.end()) {
    dev_free(c, it->second.dev, it->second.bytes);
    m->raw.erase(it);
  }
  RawW r;
  r.type = type;
  memcpy(r.ne, ne, sizeof r.ne);
  r.bytes = nbytes;
  ULB_TRY(dev_alloc(c, &r.dev, nbytes));
  cudaError_t e = cudaMemcpyAsync(r.dev, bytes, nbytes, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) { dev_free(c, r.dev, nbytes); return cuda_error(e, "upload", __FILE__, __LINE__); }
  m->raw[name] = r;
  return ULB_OK;
}

int ulb_model_finalize(ulb_model* mm) {
  ULB_CHECK(mm, ULB_EINVAL, "ulb_model_finalize: NULL model");
  Model* m = &mm->m;
  if (m->finalized) return ULB_OK;
  Ctx* c = m->c;
  ULB_CUDA(cudaSetDevice(c->device));
  const ulb_model_desc& d = m->d;
  auto get = [&](const std::string& nm, const RawW** out) -> int {
    auto it = m->raw.find(nm);
    if (it == m->raw.end()) return set_error(ULB_EFORMAT, "missing tensor %s", nm.c_str());
    *out = &it->second;
    return ULB_OK;
  };
  auto expect = [&](const RawW* r, const char* nm, uint64_t ne0, uint64_t ne1) -> int {
    if (r->ne[0] != ne0 || r->ne[1] != ne1)
      return set_error(ULB_EFORMAT, "%s: shape [%llu, %llu], expected [%llu, %llu]", nm, (unsigned long long)r->ne[0],
                       (unsigned long long)r->ne[1], (unsigned long long)ne0, (unsigned long long)ne1);
    return ULB_OK;
  };
  auto is_q4 = [](int t) { return t == ULB_TYPE_Q4_0 || t == ULB_TYPE_Q4_K; };
  const RawW* r;
  ULB_TRY(get("token_embd.weight", &r));
  ULB_TRY(expect(r, "token_embd.weight", d.d_model, d.n_vocab));
  {
    const int t = r->type;
    const bool blk32 = t == ULB_TYPE_Q4_0 || t == ULB_TYPE_Q8_0, blk256 = t == ULB_TYPE_Q4_K || t == ULB_TYPE_Q6_K;
    ULB_CHECK(t == ULB_TYPE_F16 || t == ULB_TYPE_F32 || blk32 || blk256, ULB_EUNSUPPORTED,
              "token_embd must be F16, F32, Q4_0, Q8_0, Q4_K or Q6_K (type %d)", t);
    ULB_CHECK(!(blk32 && d.d_model % 32) && !(blk256 && d.d_model % 256), ULB_EFORMAT,
              "token_embd: rows of %d are not whole blocks", d.d_model);
  }
  m->embd_type = r->type;
  ULB_TRY(upload_plain(c, *r, &m->embd, &m->embd_bytes));
  const int nq = m->nq, nkv = m->nkv;
  for (int l = 0; l < d.n_layer; ++l) {
    Layer& L = m->layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    const RawW *an, *fn, *q, *k, *v, *o, *g, *u, *dn;
    ULB_TRY(get(p + "attn_norm.weight", &an));
    ULB_TRY(get(p + "ffn_norm.weight", &fn));
    ULB_TRY(get(p + "attn_q.weight", &q));
    ULB_TRY(get(p + "attn_k.weight", &k));
    ULB_TRY(get(p + "attn_v.weight", &v));
    ULB_TRY(get(p + "attn_output.weight", &o));
    ULB_TRY(get(p + "ffn_gate.weight", &g));
    ULB_TRY(get(p + "ffn_up.weight", &u));
    ULB_TRY(get(p + "ffn_down.weight", &dn));
    ULB_CHECK(an->type == ULB_TYPE_F32 && fn->type == ULB_TYPE_F32, ULB_EUNSUPPORTED, "%snorms must be F32", p.c_str());
    ULB_CHECK(an->ne[0] == (uint64_t)d.d_model && fn->ne[0] == (uint64_t)d.d_model, ULB_EFORMAT, "%snorm size", p.c_str());
    ULB_TRY(expect(q, "attn_q", d.d_model, nq));
    ULB_TRY(expect(k, "attn_k", d.d_model, nkv));
    ULB_TRY(expect(v, "attn_v", d.d_model, nkv));
    ULB_TRY(expect(o, "attn_output", nq, d.d_model));
    ULB_TRY(expect(g, "ffn_gate", d.d_model, d.d_ff));
    ULB_TRY(expect(u, "ffn_up", d.d_model, d.d_ff));
    ULB_TRY(expect(dn, "ffn_down", d.d_ff, d.d_model));
    for (const RawW* w : {q, k, g, u})
      ULB_CHECK(is_q4(w->type), ULB_EUNSUPPORTED, "%s attn_q / attn_k / ffn_gate / ffn_up must be Q4_0 or Q4_K",
                p.c_str());
    /* attn_v, attn_output and ffn_down may also be GGUF rows of another type (llama.cpp's
       Q4_K_M / Q5_K_M mixes put Q6_K there), multiplied by the row GEMV */
    auto rows_ok = [&](const RawW* w) {
      const int t = w->type;
      const bool typ = t == ULB_TYPE_Q8_0 || t == ULB_TYPE_Q6_K || t == ULB_TYPE_F16 || t == ULB_TYPE_F32;
      const uint64_t blk = t == ULB_TYPE_Q8_0 ? 32 : t == ULB_TYPE_Q6_K ? 256 : 8;
      return typ && w->ne[0] % blk == 0;
    };
    for (const RawW* w : {v, o, dn})
      ULB_CHECK(is_q4(w->type) || (rows_ok(w) && m->tp_world == 1), ULB_EUNSUPPORTED,
                "%s attn_v / attn_output / ffn_down: type %d (Q4_0, Q4_K; or Q8_0, Q6_K, F16, F32 rows of whole "
                "blocks without tensor parallelism)", p.c_str(), w->type);
    size_t b;
    ULB_TRY(upload_plain(c, *an, (void**)&L.attn_norm, &b));
    ULB_TRY(upload_plain(c, *fn, (void**)&L.ffn_norm, &b));
    /* QKV: q and k rows paired for RoPE (strip row i = feature 2i, row i+8 = 2i+1), v as is */
    std::vector<int> map(nq + 2 * nkv);
    for (int s = 0; s < (nq + 2 * nkv) / 16; ++s)
      for (int i = 0; i < 16; ++i) {
        const int f0 = s * 16;
        map[f0 + i] = f0 < nq + nkv ? (i < 8 ? f0 + 2 * i : f0 + 2 * (i - 8) + 1) : f0 + i;
      }
    if (is_q4(v->type)) {
      ULB_TRY(build_fused(c, {q, k, v}, map, &L.qkv));
    } else {
      map.resize(nq + nkv);
      ULB_TRY(build_fused(c, {q, k}, map, &L.qkv));
      ULB_TRY(build_raw(c, *v, &L.v));
    }
    ULB_TRY(is_q4(o->type) ? build_plain(c, *o, &L.o) : build_raw(c, *o, &L.o));
    /* gate/up interleaved in strips: rows 0..7 gate 8s.., rows 8..15 up 8s.. */
    std::vector<int> gm(2 * d.d_ff);
    for (int s = 0; s < d.d_ff / 8; ++s)
      for (int i = 0; i < 16; ++i) gm[s * 16 + i] = i < 8 ? s * 8 + i : d.d_ff + s * 8 + (i - 8);
    ULB_TRY(build_fused(c, {g, u}, gm, &L.gateup));
    ULB_TRY(is_q4(dn->type) ? build_plain(c, *dn, &L.down) : build_raw(c, *dn, &L.down));
    m->weight_bytes += L.qkv.bytes + L.v.bytes + L.o.bytes + L.gateup.bytes + L.down.bytes;
  }
  ULB_TRY(get("output_norm.weight", &r));
  ULB_CHECK(r->type == ULB_TYPE_F32 && r->ne[0] == (uint64_t)d.d_model, ULB_EFORMAT, "output_norm");
  size_t b;
  ULB_TRY(upload_plain(c, *r, (void**)&m->out_norm, &b));
  /* tied embeddings (no output.weight, as small LLaMA-family models store them): the LM head
     is token_embd itself */
  const bool tied = m->raw.find("output.weight") == m->raw.end();
  ULB_TRY(get(tied ? "token_embd.weight" : "output.weight", &r));
  ULB_TRY(expect(r, "output.weight", d.d_model, d.n_vocab));
  if (r->type == ULB_TYPE_Q8_0 || r->type == ULB_TYPE_Q6_K || r->type == ULB_TYPE_F16 || r->type == ULB_TYPE_F32) {
    /* kept as GGUF rows for the row GEMV (as llama.cpp's Q4_0 / Q4_K_M files store the head,
       or a tied F16 / F32 embedding) */
    ULB_CHECK(r->type == ULB_TYPE_F16 || r->type == ULB_TYPE_F32 || d.d_model % (r->type == ULB_TYPE_Q8_0 ? 32 : 256) == 0,
              ULB_EFORMAT, "output.weight: partial blocks");
    m->out.type = r->type;
    m->out.N = d.n_vocab;
    m->out.K = d.d_model;
    m->out.ne[0] = (uint64_t)d.d_model;
    m->out.ne[1] = (uint64_t)d.n_vocab;
    if (tied) {
      m->out.dev = m->embd; /* the embedding rows are the head's rows: one device copy */
      m->out.bytes = 0;
      m->out_shared = true;
    } else {
      ULB_TRY(upload_plain(c, *r, &m->out.dev, &m->out.bytes));
    }
  } else {
    ULB_CHECK(is_q4(r->type), ULB_EUNSUPPORTED, "output.weight must be Q4_0, Q4_K, Q8_0, Q6_K, F16 or F32");
    ULB_TRY(build_plain(c, *r, &m->out));
  }
  m->weight_bytes += m->out.bytes;
  for (auto& kv : m->raw) dev_free(c, kv.second.dev, kv.second.bytes);
  m->raw.clear();
  ULB_CUDA(cudaStreamSynchronize(c->stream));
  m->finalized = true;
  return ULB_OK;
}

int ulb_model_free(ulb_model* mm) {
  if (!mm) return ULB_OK;
  Model* m = &mm->m;
  Ctx* c = m->c;
  cudaSetDevice(c->device);
  for (auto& kv : m->raw) dev_free(c, kv.second.dev, kv.second.bytes);
  dev_free(c, m->embd, m->embd_bytes);
  for (Layer& L : m->layers) {
    dev_free(c, L.attn_norm, (size_t)m->d.d_model * 4);
    dev_free(c, L.ffn_norm, (size_t)m->d.d_model * 4);
    free_tensor(c, L.qkv); free_tensor(c, L.o); free_tensor(c, L.gateup); free_tensor(c, L.down);
    free_tensor(c, L.v);
  }
  dev_free(c, m->out_norm, (size_t)m->d.d_model * 4);
  if (!m->out_shared) free_tensor(c, m->out);
  dev_free(c, m->x, 0); dev_free(c, m->x16, 0); dev_free(c, m->qb, 0); dev_free(c, m->att, 0); dev_free(c, m->h16, 0);
  c->bytes_live -= m->ws_bytes;
  cudaStreamSynchronize(c->stream);
  delete mm;
  return ULB_OK;
}

int ulb_model_weight_bytes(const ulb_model* mm, size_t* out) {
  ULB_CHECK(mm && out, ULB_EINVAL, "ulb_model_weight_bytes: NULL argument");
  *out = mm->m.weight_bytes;
  return ULB_OK;
}

/* a paged cache of n_pages pages for n_seq sequences of at most max_pages pages each, with
   the block table given (host, n_seq * max_pages entries, -1 = unmapped) or identity */
static int kv_create(ulb_ctx* ctx, const ulb_model* mm, int n_seq, int cap, int n_pages, int max_pages,
                     const int* table, ulb_kv** out) {
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  std::unique_ptr<ulb_kv> kvh(new ulb_kv());
  KV* kv = &kvh->kv;
  kv->m = const_cast<Model*>(&mm->m);
  const ulb_model_desc& d = mm->m.d;
  kv->n_seq = n_seq;
  kv->cap = cap;
  kv->n_pages = n_pages;
  kv->max_pages = max_pages;
  kv->h_bt.assign(table, table + (size_t)n_seq * max_pages);
  kv->layer_elems = (size_t)n_pages * d.n_head_kv * kKvPage * d.head_dim;
  kv->bytes = kv->layer_elems * d.n_layer * 2;
  auto fail = [&](int rc) {
    dev_free(c, kv->k, kv->bytes);
    dev_free(c, kv->v, kv->bytes);
    dev_free(c, kv->bt, kv->h_bt.size() * 4);
    dev_free(c, kv->rope, kv->rope_bytes);
    return rc;
  };
  int rc;
  if ((rc = dev_alloc(c, (void**)&kv->k, kv->bytes)) || (rc = dev_alloc(c, (void**)&kv->v, kv->bytes)) ||
      (rc = dev_alloc(c, (void**)&kv->bt, kv->h_bt.size() * 4)))
    return fail(rc);
  if (cudaMemsetAsync(kv->k, 0, kv->bytes, c->stream) != cudaSuccess ||
      cudaMemsetAsync(kv->v, 0, kv->bytes, c->stream) != cudaSuccess ||
      cudaMemcpyAsync(kv->bt, kv->h_bt.data(), kv->h_bt.size() * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
    return fail(cuda_error(cudaGetLastError(), "kv init", __FILE__, __LINE__));
  /* RoPE table: theta = pos * base^(-2i/hd) in fp64, cos/sin rounded to fp32 */
  const int half = d.head_dim / 2;
  std::vector<float2> tab((size_t)cap * half);
  for (int p = 0; p < cap; ++p)
    for (int i = 0; i < half; ++i) {
      const double th = (double)p * std::pow((double)d.rope_base, -2.0 * (double)i / (double)d.head_dim);
      tab[(size_t)p * half + i] = make_float2((float)std::cos(th), (float)std::sin(th));
    }
  kv->rope_bytes = tab.size() * sizeof(float2);
  if ((rc = dev_alloc(c, (void**)&kv->rope, kv->rope_bytes))) return fail(rc);
  if (cudaMemcpyAsync(kv->rope, tab.data(), kv->rope_bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
      cudaStreamSynchronize(c->stream) != cudaSuccess)
    return fail(cuda_error(cudaGetLastError(), "kv init", __FILE__, __LINE__));
  *out = kvh.release();
  return ULB_OK;
}

int ulb_kv_alloc(ulb_ctx* ctx, const ulb_model* mm, int n_seq, int cap, ulb_kv** out) {
  ULB_CHECK(ctx && mm && out, ULB_EINVAL, "ulb_kv_alloc: NULL argument");
  ULB_CHECK(n_seq > 0 && cap > 0, ULB_EINVAL, "ulb_kv_alloc: n_seq %d cap %d", n_seq, cap);
  /* every sequence owns the pages of its whole capacity: identity block table */
  const int pps = (cap + kKvPage - 1) / kKvPage;
  ULB_CHECK((long long)n_seq * pps < (1ll << 31), ULB_EINVAL, "ulb_kv_alloc: too many pages");
  std::vector<int> table((size_t)n_seq * pps);
  for (size_t i = 0; i < table.size(); ++i) table[i] = (int)i;
  ULB_TRY(kv_create(ctx, mm, n_seq, cap, n_seq * pps, pps, table.data(), out));
  (*out)->kv.identity = true;
  return ULB_OK;
}

int ulb_kv_alloc_paged(ulb_ctx* ctx, const ulb_model* mm, int n_seq, int n_pages, int max_pages_per_seq,
                       ulb_kv** out) {
  ULB_CHECK(ctx && mm && out, ULB_EINVAL, "ulb_kv_alloc_paged: NULL argument");
  ULB_CHECK(n_seq > 0 && n_pages > 0 && max_pages_per_seq > 0, ULB_EINVAL,
            "ulb_kv_alloc_paged: n_seq %d n_pages %d max_pages %d", n_seq, n_pages, max_pages_per_seq);
  ULB_CHECK((long long)max_pages_per_seq * kKvPage <= 8192, ULB_EUNSUPPORTED,
            "ulb_kv_alloc_paged: %d pages of %d positions exceed the attention's 8192", max_pages_per_seq, kKvPage);
  std::vector<int> table((size_t)n_seq * max_pages_per_seq, -1);
  return kv_create(ctx, mm, n_seq, max_pages_per_seq * kKvPage, n_pages, max_pages_per_seq, table.data(), out);
}

int ulb_kv_map(ulb_kv* kvh, int seq, int first, int n, const int32_t* pages) {
  ULB_CHECK(kvh && (n == 0 || pages), ULB_EINVAL, "ulb_kv_map: NULL argument");
  KV* kv = &kvh->kv;
  ULB_CHECK(seq >= 0 && seq < kv->n_seq && first >= 0 && n >= 0 && first + n <= kv->max_pages, ULB_EINVAL,
            "ulb_kv_map: sequence %d pages [%d, %d) of %d", seq, first, first + n, kv->max_pages);
  for (int i = 0; i < n; ++i)
    ULB_CHECK(pages[i] >= -1 && pages[i] < kv->n_pages, ULB_EINVAL, "ulb_kv_map: page %d of %d", pages[i], kv->n_pages);
  if (n == 0) return ULB_OK;
  int* row = kv->h_bt.data() + (size_t)seq * kv->max_pages + first;
  memcpy(row, pages, (size_t)n * 4);
  kv->identity = false; /* from now on the kernels read the table */
  Ctx* c = kv->m->c;
  ULB_CUDA(cudaSetDevice(c->device));
  ULB_CUDA(cudaMemcpyAsync(kv->bt + (size_t)seq * kv->max_pages + first, row, (size_t)n * 4, cudaMemcpyHostToDevice,
                           c->stream));
  return ULB_OK;
}

int ulb_kv_free(ulb_kv* kvh) {
  if (!kvh) return ULB_OK;
  KV* kv = &kvh->kv;
  Ctx* c = kv->m->c;
  cudaSetDevice(c->device);
  dev_free(c, kv->k, kv->bytes);
  dev_free(c, kv->v, kv->bytes);
  dev_free(c, kv->bt, kv->h_bt.size() * 4);
  dev_free(c, kv->rope, kv->rope_bytes);
  dev_free(c, kv->attn_scratch, kv->attn_floats * 4);
  dev_free(c, kv->attn_counters, (size_t)kv->n_counters * 4);
  cudaStreamSynchronize(c->stream);
  delete kvh;
  return ULB_OK;
}

int ulb_model_forward(ulb_ctx* ctx, ulb_model* mm, ulb_kv* kvh, int M, int rps, const int32_t* tok,
                      const int32_t* seq, const int32_t* pos, int logits_mode, float* logits, int ld) {
  ULB_CHECK(ctx && mm && kvh && tok && seq && pos && logits, ULB_EINVAL, "ulb_model_forward: NULL argument");
  ULB_CHECK(&ctx->c == mm->m.c, ULB_EINVAL, "ulb_model_forward: model belongs to another context");
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  ULB_TRY(model_prepare(&mm->m, &kvh->kv, M, rps));
  int* err = nullptr;
  ULB_TRY(dev_alloc(c, (void**)&err, sizeof(int)));
  ULB_CUDA(cudaMemsetAsync(err, 0, sizeof(int), c->stream));
  int rc = model_forward(&mm->m, &kvh->kv, M, rps, tok, seq, pos, logits_mode, logits, ld, err);
  int herr = 0;
  if (rc == ULB_OK) {
    cudaError_t e = cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) rc = cuda_error(e, "forward", __FILE__, __LINE__);
    else rc = sync_stream(c);
  }
  dev_free(c, err, sizeof(int));
  if (rc == ULB_OK && herr) rc = set_error(ULB_EINVAL, "ulb_model_forward: token id out of range");
  if (rc == ULB_OK) rc = check_device_errors(c);
  return rc;
}

}  // extern "C"

ULB_TRACE_UNIT(model)
