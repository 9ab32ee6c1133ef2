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

template <int EPI>
__device__ __forceinline__ void epilogue_token(const EpiArgs& e, int strip, int g, int tok, int M, int N, float vg,
                                               float vg8) {
  if (tok >= M) return;
  if (EPI == EPI_STORE || EPI == EPI_RESID) {
    const int r0 = strip * 16 + g, r1 = r0 + 8;
    if (r0 < N) {
      float* p = e.y + (size_t)tok * e.ldy + r0;
      *p = EPI == EPI_RESID ? __ldcg(p) + vg : vg;
    }
    if (r1 < N) {
      float* p = e.y + (size_t)tok * e.ldy + r1;
      *p = EPI == EPI_RESID ? __ldcg(p) + vg8 : vg8;
    }
  } else if (EPI == EPI_SWIGLU) {
    const int f = strip * 8 + g;
    const float sg = vg / (1.0f + expf(-vg));
    e.h[(size_t)tok * e.ldh + f] = __float2half_rn(__fmul_rn(sg, vg8));
  } else if (EPI == EPI_QKV) {
    const int f0 = strip * 16;
    const int pos = e.row_pos[tok];
    const int seq = e.row_seq[tok];
    if ((unsigned)pos >= (unsigned)e.cap || (unsigned)seq >= (unsigned)e.n_seq) return; /* never write outside the cache */
    /* the cache row of (seq, kv head, pos): contiguous [S][Hkv][cap][hd], or page pool
       [page][Hkv][kKvPage][hd] through the block table (an unmapped page is never written) */
    size_t sbase, pstride;
    int prow;
    bool kv_ok = true;
    if (e.max_pages > 0) {
      const int slot = seq * e.max_pages + pos / kKvPage;
      const int page = e.bt ? e.bt[slot] : slot;
      kv_ok = page >= 0;
      sbase = (size_t)(kv_ok ? page : 0) * e.n_head_kv;
      pstride = kKvPage;
      prow = pos % kKvPage;
    } else {
      sbase = (size_t)seq * e.n_head_kv;
      pstride = (size_t)e.cap;
      prow = pos;
    }
    auto row_at = [&](int kvh) { return ((sbase + kvh) * pstride + prow) * e.hd; };
    if (f0 < e.nq + e.nkv) {
      /* RoPE-permuted strip: row g = feature f0 + 2g, row g + 8 = feature f0 + 2g + 1 */
      const int f = f0 + 2 * g;
      const int pair = (f % e.hd) >> 1;
      const int rpos = e.row_rope ? e.row_rope[tok] : pos;
      const float2 cs = e.rope[(size_t)rpos * (e.hd >> 1) + pair];
      const float y0 = __fmaf_rn(vg, cs.x, -__fmul_rn(vg8, cs.y));
      const float y1 = __fmaf_rn(vg, cs.y, __fmul_rn(vg8, cs.x));
      if (f < e.nq) {
        float* q = e.q + (size_t)tok * e.ldq + f;
        q[0] = y0;
        q[1] = y1;
      } else if (kv_ok) {
        const int fk = f - e.nq, kvh = fk / e.hd, d = fk % e.hd;
        __half2* kp = reinterpret_cast<__half2*>(e.kc + row_at(kvh) + d);
        *kp = __halves2half2(__float2half_rn(y0), __float2half_rn(y1));
      }
    } else if (kv_ok) {
      /* V strip, identity rows */
      const float vals[2] = {vg, vg8};
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int fv = f0 + g + 8 * i - e.nq - e.nkv;
        const int kvh = fv / e.hd, d = fv % e.hd;
        e.vc[row_at(kvh) + d] = __float2half_rn(vals[i]);
      }
    }
  }
}

}  // namespace ulb
