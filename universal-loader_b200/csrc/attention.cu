/*
 * attention.cu — block-causal attention of the k+1 verify rows (or the draft rows) of each
 * sequence against the fp16 KV cache.
 *
 * Replaces flash_attention.glsl (src/shaders/attention/flash_attention.glsl:20-42, which
 * scores a token against itself only) and implements the feature list of
 * flash_attention_v2_fused.glsl (src/shaders/attention/flash_attention_v2_fused.glsl:13-24,
 * 42-45, 153): GQA (kv head = q head / group), causal masking, online softmax over KV
 * blocks, KV read from the cache.
 *
 * Split-KV (flash-decoding): grid = (KV chunk of 64 keys, kv head, sequence x row block).
 * All q heads of one GQA group and all rows of the block share each K/V chunk staged in
 * shared memory, so the cache is read once per verify step.  A chunk's partial
 * (max, sum, unnormalised output) goes to scratch; the CTA that arrives last for its
 * (sequence, row block, kv head) merges the chunks in chunk order, so the result is
 * deterministic and a row's arithmetic depends only on its own position.
 */
#include "ulb_internal.h"

namespace ulb {

namespace {

constexpr int ACH = 64;     /* keys per chunk */
constexpr int AQMAX = 64;   /* queries (heads x rows) per CTA */
constexpr int ATHREADS = 128;

struct AttnParams {
  int H, Hkv, hd, cap, G, rps, RB, n_rb, max_chunks, ldq, n_seq;
  float scale;
};

__global__ void __launch_bounds__(ATHREADS) attn_kernel(AttnParams p, const float* __restrict__ q,
                                                        const __half* __restrict__ kc,
                                                        const __half* __restrict__ vc,
                                                        const int* __restrict__ row_seq,
                                                        const int* __restrict__ row_pos,
                                                        __half* __restrict__ out, float* scratch,
                                                        int* counters) {
  extern __shared__ float smem[];
  const int chunk = blockIdx.x, kvh = blockIdx.y, gz = blockIdx.z;
  const int gi = gz / p.n_rb, rb = gz % p.n_rb;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hd = p.hd, hd2 = hd >> 1;
  pdl_wait();
  pdl_trigger();

  const int r0 = rb * p.RB;
  const int nr = min(p.RB, p.rps - r0);
  const int Q = p.G * nr;
  const int m0 = gi * p.rps + r0;
  int last_pos = 0;
  for (int r = 0; r < nr; ++r) last_pos = max(last_pos, row_pos[m0 + r]);
  last_pos = min(last_pos, p.cap - 1); /* positions past the cache never index it */
  const int n_valid = last_pos / ACH + 1;
  if (chunk >= n_valid) return;
  const int seq = row_seq[m0];
  if ((unsigned)seq >= (unsigned)p.n_seq) return;
  const int k0 = chunk * ACH;
  const int nk = min(ACH, last_pos + 1 - k0);

  /* shared layout */
  float* qs = smem;                                   /* [Q][hd]            */
  float* ss = qs + AQMAX * hd;                        /* [Q][ACH]           */
  int* qpos = reinterpret_cast<int*>(ss + AQMAX * ACH); /* [Q]              */
  float* ml = reinterpret_cast<float*>(qpos + AQMAX); /* [Q][2] (m, l)      */
  __half2* ks = reinterpret_cast<__half2*>(ml + 2 * AQMAX); /* [ACH][hd2 + 1] */
  __half2* vs = ks + ACH * (hd2 + 1);                  /* [ACH][hd2]         */

  for (int i = tid; i < Q * hd; i += ATHREADS) {
    const int qi = i / hd, d = i % hd;
    const int r = qi / p.G, gq = qi % p.G;
    const int h = kvh * p.G + gq;
    qs[i] = q[(size_t)(m0 + r) * p.ldq + h * hd + d];
  }
  for (int qi = tid; qi < Q; qi += ATHREADS) qpos[qi] = row_pos[m0 + qi / p.G];
  const size_t kvbase = (((size_t)seq * p.Hkv + kvh) * p.cap + k0) * hd;
  const int vec_per_row = hd / 8;
  for (int i = tid; i < nk * vec_per_row; i += ATHREADS) {
    const int j = i / vec_per_row, c = i % vec_per_row;
    const uint4 kv4 = __ldg(reinterpret_cast<const uint4*>(kc + kvbase + (size_t)j * hd) + c);
    const uint4 vv4 = __ldg(reinterpret_cast<const uint4*>(vc + kvbase + (size_t)j * hd) + c);
    const uint32_t kw[4] = {kv4.x, kv4.y, kv4.z, kv4.w};
    uint32_t* krow = reinterpret_cast<uint32_t*>(ks + j * (hd2 + 1));
#pragma unroll
    for (int e = 0; e < 4; ++e) krow[c * 4 + e] = kw[e];
    reinterpret_cast<uint4*>(vs + j * hd2)[c] = vv4;
  }
  __syncthreads();

  /* scores: warp per query, lanes over keys; sequential fma over d (same order as the CPU) */
  for (int qi = warp; qi < Q; qi += ATHREADS / 32) {
    const float2* qv = reinterpret_cast<const float2*>(qs + qi * hd);
    for (int j = lane; j < ACH; j += 32) {
      float s = -INFINITY;
      if (j < nk && k0 + j <= qpos[qi]) {
        const __half2* kr = ks + j * (hd2 + 1);
        float a = 0.f;
        for (int d2 = 0; d2 < hd2; ++d2) {
          const float2 kf = __half22float2(kr[d2]);
          const float2 qf = qv[d2];
          a = __fmaf_rn(qf.x, kf.x, a);
          a = __fmaf_rn(qf.y, kf.y, a);
        }
        s = __fmul_rn(a, p.scale);
      }
      ss[qi * ACH + j] = s;
    }
  }
  __syncthreads();
  /* per-query chunk softmax */
  for (int qi = warp; qi < Q; qi += ATHREADS / 32) {
    float m = -INFINITY;
    for (int j = lane; j < ACH; j += 32) m = fmaxf(m, ss[qi * ACH + j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int j = lane; j < ACH; j += 32) {
      const float s = ss[qi * ACH + j];
      const float e = s == -INFINITY ? 0.f : expf(s - m);
      ss[qi * ACH + j] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) { ml[2 * qi] = m; ml[2 * qi + 1] = l; }
  }
  __syncthreads();

  /* P.V: thread per (query, d pair); sequential over keys */
  float* part = nullptr;
  const int qstride = p.G * p.RB;
  if (n_valid > 1)
    part = scratch + (((size_t)gz * p.Hkv + kvh) * p.max_chunks + chunk) * (size_t)qstride * (hd + 2);
  for (int it = tid; it < Q * hd2; it += ATHREADS) {
    const int qi = it / hd2, d2 = it % hd2;
    float ox = 0.f, oy = 0.f;
    const float* pr = ss + qi * ACH;
    for (int j = 0; j < nk; ++j) {
      const float pj = pr[j];
      const float2 vf = __half22float2(vs[j * hd2 + d2]);
      ox = __fmaf_rn(pj, vf.x, ox);
      oy = __fmaf_rn(pj, vf.y, oy);
    }
    if (n_valid == 1) {
      const float l = ml[2 * qi + 1];
      const int r = qi / p.G, gq = qi % p.G;
      const int h = kvh * p.G + gq;
      __half2* op = reinterpret_cast<__half2*>(out + (size_t)(m0 + r) * p.H * hd + h * hd) + d2;
      *op = __halves2half2(__float2half_rn(ox / l), __float2half_rn(oy / l));
    } else {
      float* pq = part + (size_t)qi * (hd + 2);
      pq[2 + 2 * d2] = ox;
      pq[3 + 2 * d2] = oy;
    }
  }
  if (n_valid == 1) return;
  for (int qi = tid; qi < Q; qi += ATHREADS) {
    part[(size_t)qi * (hd + 2)] = ml[2 * qi];
    part[(size_t)qi * (hd + 2) + 1] = ml[2 * qi + 1];
  }
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (tid == 0) {
    const int prev = atomicAdd(&counters[gz * p.Hkv + kvh], 1);
    is_last = prev == n_valid - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* base = scratch + (((size_t)gz * p.Hkv + kvh) * p.max_chunks) * (size_t)qstride * (hd + 2);
  const size_t cstride = (size_t)qstride * (hd + 2);
  for (int it = tid; it < Q * hd2; it += ATHREADS) {
    const int qi = it / hd2, d2 = it % hd2;
    float M = -INFINITY;
    for (int c = 0; c < n_valid; ++c) M = fmaxf(M, __ldcg(base + c * cstride + (size_t)qi * (hd + 2)));
    float L = 0.f, ox = 0.f, oy = 0.f;
    for (int c = 0; c < n_valid; ++c) {
      const float* pc = base + c * cstride + (size_t)qi * (hd + 2);
      const float mc = __ldcg(pc);
      if (mc == -INFINITY) continue;
      const float w = expf(mc - M);
      L = __fmaf_rn(__ldcg(pc + 1), w, L);
      ox = __fmaf_rn(__ldcg(pc + 2 + 2 * d2), w, ox);
      oy = __fmaf_rn(__ldcg(pc + 3 + 2 * d2), w, oy);
    }
    const int r = qi / p.G, gq = qi % p.G;
    const int h = kvh * p.G + gq;
    __half2* op = reinterpret_cast<__half2*>(out + (size_t)(m0 + r) * p.H * hd + h * hd) + d2;
    *op = __halves2half2(__float2half_rn(ox / L), __float2half_rn(oy / L));
  }
  if (tid == 0) counters[gz * p.Hkv + kvh] = 0; /* ready for the next launch / graph replay */
}

void attn_geometry(const ulb_attn_desc* d, int M, int rps, int max_pos, AttnParams* p, int* n_groups) {
  p->H = d->n_head;
  p->Hkv = d->n_head_kv;
  p->hd = d->head_dim;
  p->cap = d->capacity;
  p->G = d->n_head / d->n_head_kv;
  p->rps = rps;
  p->RB = AQMAX / p->G < 1 ? 1 : AQMAX / p->G;
  if (p->RB > rps) p->RB = rps;
  p->n_rb = (rps + p->RB - 1) / p->RB;
  p->max_chunks = max_pos / ACH + 1;
  p->scale = d->scale;
  p->n_seq = d->n_seq;
  *n_groups = M / rps;
}

size_t attn_smem(int hd) {
  return sizeof(float) * ((size_t)AQMAX * hd + AQMAX * ACH + 2 * AQMAX) + sizeof(int) * AQMAX +
         sizeof(__half2) * ((size_t)ACH * (hd / 2 + 1) + (size_t)ACH * (hd / 2));
}

}  // namespace

size_t attention_scratch_floats(const ulb_attn_desc* d, int M, int rps, int max_pos, int* n_counters) {
  AttnParams p;
  int ng;
  attn_geometry(d, M, rps, max_pos, &p, &ng);
  *n_counters = ng * p.n_rb * p.Hkv;
  return (size_t)ng * p.n_rb * p.Hkv * p.max_chunks * (size_t)(p.G * p.RB) * (p.hd + 2);
}

int launch_attention(Ctx* c, const ulb_attn_desc* d, const float* q, int ldq, const __half* k,
                     const __half* v, const int* row_seq, const int* row_pos, int M, int rps,
                     __half* out, float* scratch, int* counters, size_t scratch_floats, int n_counters) {
  ULB_CHECK(d->n_head % d->n_head_kv == 0, ULB_EINVAL, "attention: n_head %% n_head_kv != 0");
  ULB_CHECK(d->head_dim % 8 == 0 && d->head_dim <= 256, ULB_EUNSUPPORTED, "attention: head_dim %d", d->head_dim);
  ULB_CHECK(d->n_head / d->n_head_kv <= AQMAX, ULB_EUNSUPPORTED, "attention: GQA group > %d", AQMAX);
  ULB_CHECK(rps > 0 && M % rps == 0, ULB_EINVAL, "attention: M=%d not a multiple of rows_per_seq=%d", M, rps);
  if (M == 0) return ULB_OK;
  AttnParams p;
  int ng;
  attn_geometry(d, M, rps, d->capacity - 1, &p, &ng);
  p.ldq = ldq;
  int need_c = 0;
  const size_t need = attention_scratch_floats(d, M, rps, d->capacity - 1, &need_c);
  ULB_CHECK(scratch_floats >= need && n_counters >= need_c, ULB_EINVAL,
            "attention: scratch %zu floats / %d counters, need %zu / %d", scratch_floats, n_counters, need, need_c);
  const size_t smem = attn_smem(p.hd);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem(256));
    attr_set = true;
  }
  dim3 grid(p.max_chunks, p.Hkv, ng * p.n_rb), block(ATHREADS);
  cudaError_t e = launch_k(c, attn_kernel, grid, block, smem, p, q, k, v, row_seq, row_pos, out, scratch, counters);
  if (e != cudaSuccess) return cuda_error(e, "attention launch", __FILE__, __LINE__);
  return ULB_OK;
}

}  // namespace ulb

using namespace ulb;

extern "C" int ulb_attention(ulb_ctx* ctx, const ulb_attn_desc* d, const float* q, const uint16_t* k,
                             const uint16_t* v, const int32_t* row_seq, const int32_t* row_pos, int M,
                             int rps, uint16_t* out) {
  ULB_CHECK(ctx && d && q && k && v && row_seq && row_pos && out, ULB_EINVAL, "ulb_attention: NULL argument");
  ULB_CHECK(d->capacity > 0 && d->n_seq > 0, ULB_EINVAL, "ulb_attention: capacity / n_seq");
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  int nc = 0;
  const size_t nf = attention_scratch_floats(d, M, rps, d->capacity - 1, &nc);
  float* scratch = nullptr;
  int* counters = nullptr;
  ULB_TRY(dev_alloc(c, (void**)&scratch, nf * sizeof(float)));
  int rc = dev_alloc(c, (void**)&counters, (size_t)nc * sizeof(int));
  if (rc == ULB_OK) {
    cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)nc * sizeof(int), c->stream);
    rc = e == cudaSuccess ? launch_attention(c, d, q, d->n_head * d->head_dim, (const __half*)k, (const __half*)v,
                                             row_seq, row_pos, M, rps, (__half*)out, scratch, counters, nf, nc)
                          : cuda_error(e, "memset", __FILE__, __LINE__);
  }
  dev_free(c, counters, (size_t)nc * sizeof(int));
  dev_free(c, scratch, nf * sizeof(float));
  return rc;
}
