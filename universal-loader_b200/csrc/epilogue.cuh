/*
 * epilogue.cuh — the fused epilogues of the Q4 GEMV (qgemv.cu) and the tensor-core GEMM
 * (qgemm_tc.cu), per output token.
 *
 * Both kernels produce, for one token and one 16-row strip of the packed weight layout, the
 * values of strip rows g and g + 8 (g in 0..7).  The strip layout pairs those rows:
 *   QKV (RoPE'd Q / K strips): row g = feature 2i, row g + 8 = feature 2i + 1 (one rotation
 *     pair, src/shaders/rope.glsl:50-74 adjacent-pair RoPE); V strips are identity rows;
 *   gate/up: row g = gate of feature 8s + g, row g + 8 = up of the same feature.
 * Replaces the reference's separate rope / silu / mul / add dispatches
 * (src/inference/inference_engine.cpp:602-682).
 */
#pragma once

#include "ulb_internal.h"

namespace ulb {

/* element (kv head kvh, dimension dd) of token tok's row in this layer's V cache (fp16), through
   the block table for a paged cache; nothing is written outside the cache or to an unmapped page */
__device__ __forceinline__ void store_v_cache(const EpiArgs& e, int tok, int kvh, int dd, float v) {
  const int pos = e.row_pos[tok];
  const int seq = e.row_seq[tok];
  if ((unsigned)pos >= (unsigned)e.cap || (unsigned)seq >= (unsigned)e.n_seq) return;
  size_t row;
  if (e.max_pages > 0) {
    const int slot = seq * e.max_pages + pos / kKvPage;
    const int page = e.bt ? e.bt[slot] : slot;
    if (page < 0) return;
    row = (((size_t)page * e.n_head_kv + kvh) * kKvPage + pos % kKvPage) * e.hd;
  } else {
    row = (((size_t)seq * e.n_head_kv + kvh) * e.cap + pos) * e.hd;
  }
  e.vc[row + dd] = __float2half_rn(v);
}

/* the cache coordinates of token tok's row: its position, sequence and RoPE position.  The
   row arrays are written by a stage kernel or the host at least two launches before any
   GEMV that reads them, so a GEMV may read them before its wait for the previous kernel */
struct EpiRow {
  int pos, seq, rpos;
};
__device__ __forceinline__ EpiRow epi_row(const EpiArgs& e, int tok) {
  EpiRow r;
  r.pos = e.row_pos[tok];
  r.seq = e.row_seq[tok];
  r.rpos = e.row_rope ? e.row_rope[tok] : r.pos;
  return r;
}

/* QKV epilogue of rows g (value vg) and g + 8 (vg8) of strip `strip` for the tokens of rows
   r[0 .. NTOK-1] (ok[i]: token valid): the block-table and RoPE-table loads of every token are
   issued before any result is stored.
     RoPE-permuted strip (Q / K): row g = feature f0 + 2g, row g + 8 = feature f0 + 2g + 1, one
     rotation pair (src/shaders/rope.glsl:50-74 adjacent-pair RoPE);
     V strip: identity rows.
   K / V go to the cache row of (seq, kv head, pos): contiguous [S][Hkv][cap][hd], or page pool
   [page][Hkv][kKvPage][hd] through the block table (an unmapped page is never written). */
template <int NTOK>
__device__ __forceinline__ void qkv_tokens(const EpiArgs& e, int strip, int g, const int (&tok)[NTOK],
                                           const EpiRow (&r)[NTOK], const bool (&ok_in)[NTOK],
                                           const float (&vg)[NTOK], const float (&vg8)[NTOK]) {
  const int f0 = strip * 16;
  const bool rot = f0 < e.nq + e.nkv;
  const int pair = ((f0 + 2 * g) % e.hd) >> 1;
  bool ok[NTOK];
  int page[NTOK];
  float2 cs[NTOK];
#pragma unroll
  for (int i = 0; i < NTOK; ++i) {
    /* never write outside the cache */
    ok[i] = ok_in[i] && (unsigned)r[i].pos < (unsigned)e.cap && (unsigned)r[i].seq < (unsigned)e.n_seq;
    page[i] = 0;
    if (ok[i] && e.max_pages > 0) {
      const int slot = r[i].seq * e.max_pages + r[i].pos / kKvPage;
      page[i] = e.bt ? e.bt[slot] : slot;
    }
    cs[i] = ok[i] && rot ? e.rope[(size_t)r[i].rpos * (e.hd >> 1) + pair] : make_float2(0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < NTOK; ++i) {
    if (!ok[i]) continue;
    size_t sbase, pstride;
    int prow;
    bool kv_ok = true;
    if (e.max_pages > 0) {
      kv_ok = page[i] >= 0;
      sbase = (size_t)(kv_ok ? page[i] : 0) * e.n_head_kv;
      pstride = kKvPage;
      prow = r[i].pos % kKvPage;
    } else {
      sbase = (size_t)r[i].seq * e.n_head_kv;
      pstride = (size_t)e.cap;
      prow = r[i].pos;
    }
    auto row_at = [&](int kvh) { return ((sbase + kvh) * pstride + prow) * e.hd; };
    if (rot) {
      const int f = f0 + 2 * g;
      const float y0 = __fmaf_rn(vg[i], cs[i].x, -__fmul_rn(vg8[i], cs[i].y));
      const float y1 = __fmaf_rn(vg[i], cs[i].y, __fmul_rn(vg8[i], cs[i].x));
      if (f < e.nq) {
        float* q = e.q + (size_t)tok[i] * e.ldq + f;
        q[0] = y0;
        q[1] = y1;
      } else if (kv_ok) {
        const int fk = f - e.nq, kvh = fk / e.hd, d = fk % e.hd;
        __half2* kp = reinterpret_cast<__half2*>(e.kc + row_at(kvh) + d);
        *kp = __halves2half2(__float2half_rn(y0), __float2half_rn(y1));
      }
    } else if (kv_ok) {
      const float vals[2] = {vg[i], vg8[i]};
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int fv = f0 + g + 8 * u - e.nq - e.nkv;
        const int kvh = fv / e.hd, d = fv % e.hd;
        e.vc[row_at(kvh) + d] = __float2half_rn(vals[u]);
      }
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_token(const EpiArgs& e, int strip, int g, int tok, int M, int N, float vg,
                                               float vg8) {
  if (tok >= M) return;
  if (EPI == EPI_STORE || EPI == EPI_RESID) {
    const int r0 = strip * 16 + g, r1 = r0 + 8;
    float* p0 = e.y + (size_t)tok * e.ldy + r0;
    float* p1 = p0 + 8;
    if (EPI == EPI_RESID) { /* both loads before either store */
      const float a0 = r0 < N ? __ldcg(p0) : 0.f, a1 = r1 < N ? __ldcg(p1) : 0.f;
      if (r0 < N) *p0 = a0 + vg;
      if (r1 < N) *p1 = a1 + vg8;
    } else {
      if (r0 < N) *p0 = vg;
      if (r1 < N) *p1 = vg8;
    }
  } else if (EPI == EPI_SWIGLU) {
    const int f = strip * 8 + g;
    const float sg = vg / (1.0f + expf(-vg));
    e.h[(size_t)tok * e.ldh + f] = __float2half_rn(__fmul_rn(sg, vg8));
  } else if (EPI == EPI_QKV) {
    const int tk[1] = {tok};
    const EpiRow r[1] = {epi_row(e, tok)};
    const bool ok[1] = {true};
    const float a[1] = {vg}, b[1] = {vg8};
    qkv_tokens<1>(e, strip, g, tk, r, ok, a, b);
  }
}

/* the tensor-core GEMM's epilogue of NTOK consecutive tokens tok0 .. of rows g (va) and g + 8
   (vb) of strip `strip`; rows: the tokens' cache rows (QKV), read ahead into shared memory.
   Every load of the group is issued before any store. */
template <int EPI, int NTOK>
__device__ __forceinline__ void epilogue_tokens(const EpiArgs& e, int strip, int g, int tok0, int M, int N,
                                                const float (&va)[NTOK], const float (&vb)[NTOK], const EpiRow* rows) {
  if (EPI == EPI_RESID) {
    const int r0 = strip * 16 + g, r1 = r0 + 8;
    const bool c0 = r0 < N, c1 = r1 < N;
    float a0[NTOK], a1[NTOK];
#pragma unroll
    for (int i = 0; i < NTOK; ++i) {
      const bool t = tok0 + i < M;
      const float* p = e.y + (size_t)(tok0 + i) * e.ldy + r0;
      a0[i] = t && c0 ? __ldcg(p) : 0.f;
      a1[i] = t && c1 ? __ldcg(p + 8) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < NTOK; ++i) {
      if (tok0 + i >= M) continue;
      float* p = e.y + (size_t)(tok0 + i) * e.ldy + r0;
      if (c0) p[0] = a0[i] + va[i];
      if (c1) p[8] = a1[i] + vb[i];
    }
  } else if (EPI == EPI_QKV) {
    int tk[NTOK];
    bool ok[NTOK];
    EpiRow r[NTOK];
#pragma unroll
    for (int i = 0; i < NTOK; ++i) {
      tk[i] = tok0 + i;
      ok[i] = tok0 + i < M;
      r[i] = rows[i];
    }
    qkv_tokens<NTOK>(e, strip, g, tk, r, ok, va, vb);
  } else {
#pragma unroll
    for (int i = 0; i < NTOK; ++i) epilogue_token<EPI>(e, strip, g, tok0 + i, M, N, va[i], vb[i]);
  }
}

/* the GEMV's epilogue of one lane's two tokens tok0, tok0 + 1 (v = (tok0 row g, tok0 + 1 row g,
   tok0 row g + 8, tok0 + 1 row g + 8)); pre: their rows, read before the kernel's wait (QKV),
   or NULL.  Every load of the pair is issued before any store. */
template <int EPI>
__device__ __forceinline__ void epilogue_pair(const EpiArgs& e, int strip, int g, int tok0, int M, int N,
                                              const float4& v, const EpiRow* pre) {
  if (EPI == EPI_RESID) {
    const int r0 = strip * 16 + g, r1 = r0 + 8;
    const bool t0 = tok0 < M, t1 = tok0 + 1 < M, c0 = r0 < N, c1 = r1 < N;
    float* p = e.y + (size_t)tok0 * e.ldy + r0;
    float* q = p + e.ldy;
    const float a00 = t0 && c0 ? __ldcg(p) : 0.f, a01 = t0 && c1 ? __ldcg(p + 8) : 0.f;
    const float a10 = t1 && c0 ? __ldcg(q) : 0.f, a11 = t1 && c1 ? __ldcg(q + 8) : 0.f;
    if (t0 && c0) p[0] = a00 + v.x;
    if (t0 && c1) p[8] = a01 + v.z;
    if (t1 && c0) q[0] = a10 + v.y;
    if (t1 && c1) q[8] = a11 + v.w;
  } else if (EPI == EPI_QKV) {
    const int tk[2] = {tok0, tok0 + 1};
    const bool ok[2] = {tok0 < M, tok0 + 1 < M};
    EpiRow r[2];
    if (pre) {
      r[0] = pre[0];
      r[1] = pre[1];
    } else {
      r[0] = ok[0] ? epi_row(e, tok0) : EpiRow{-1, 0, 0};
      r[1] = ok[1] ? epi_row(e, tok0 + 1) : EpiRow{-1, 0, 0};
    }
    const float a[2] = {v.x, v.y}, b[2] = {v.z, v.w};
    qkv_tokens<2>(e, strip, g, tk, r, ok, a, b);
  } else {
    epilogue_token<EPI>(e, strip, g, tok0, M, N, v.x, v.z);
    epilogue_token<EPI>(e, strip, g, tok0 + 1, M, N, v.y, v.w);
  }
}

}  // namespace ulb
