/*
 * oracle.c — CPU restatement of the speculative path (see oracle.h for what it follows).
 * TEST INFRASTRUCTURE ONLY: the product never links or calls this file.
 *
 * Build: oracle/build.py (gcc -O3 -fopenmp -ffp-contract=off).  -ffp-contract=off keeps
 * every elementwise product/sum rounded exactly where the C source says; where the device
 * uses a fused multiply-add the source here calls fmaf() explicitly.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define T_F32 0
#define T_F16 1
#define T_Q4_0 2
#define T_Q4_K 12
#define T_Q8_0 8
#define T_Q6_K 14

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------ fp16 */
static float h2f(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
  if (e == 0) {
    if (m == 0) bits = s;
    else {
      /* subnormal: value = m * 2^-24 exactly */
      float f = ldexpf((float)m, -24);
      return s ? -f : f;
    }
  } else if (e == 31) bits = s | 0x7f800000u | (m << 13);
  else bits = s | ((e + 112) << 23) | (m << 13);
  float f; memcpy(&f, &bits, 4); return f;
}

/* fp32 -> fp16 round-to-nearest-even written from the arithmetic definition. */
static uint16_t f2h(float f) {
  uint32_t x; memcpy(&x, &f, 4);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  float a = fabsf(f);
  if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
  if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u);
  if (a < 6.103515625e-05f) { /* subnormal range: units of 2^-24 */
    float q = a * 16777216.0f;            /* exact scaling by a power of two */
    float r = nearbyintf(q);              /* default rounding mode: nearest-even */
    return (uint16_t)(sign | (uint16_t)r);
  }
  int e; float mant = frexpf(a, &e);      /* a = mant * 2^e, mant in [0.5, 1) */
  float q = ldexpf(mant, 11);             /* [1024, 2048) */
  float r = nearbyintf(q);
  if (r >= 2048.0f) { r = 1024.0f; e += 1; }
  int he = e - 1 + 15;                    /* half exponent field */
  if (he >= 31) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | (uint16_t)(he << 10) | (uint16_t)((int)r - 1024));
}

/* ------------------------------------------------------------------ Philox4x32-10 */
void orc_philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1,
                uint32_t out[4]) {
  uint32_t c[4] = {c0, c1, c2, c3}, k[2] = {k0, k1};
  for (int r = 0; r < 10; ++r) {
    uint64_t a = (uint64_t)0xD2511F53u * c[0], b = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n[4];
    n[0] = (uint32_t)(b >> 32) ^ c[1] ^ k[0];
    n[1] = (uint32_t)b;
    n[2] = (uint32_t)(a >> 32) ^ c[3] ^ k[1];
    n[3] = (uint32_t)a;
    memcpy(c, n, sizeof n);
    k[0] += 0x9E3779B9u; k[1] += 0xBB67AE85u;
  }
  memcpy(out, c, sizeof c);
}

float orc_uniform(uint64_t seed, uint32_t round, uint32_t seq, uint32_t slot, uint32_t tag) {
  uint32_t o[4];
  orc_philox(round, seq, slot, tag, (uint32_t)seed, (uint32_t)(seed >> 32), o);
  return (float)(o[0] >> 8) * (1.0f / 16777216.0f);
}

/* ------------------------------------------------------------------ block formats */
size_t orc_type_nbytes(int type, uint64_t n) {
  switch (type) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q4_0: return n % 32 ? 0 : n / 32 * 18;
    case T_Q4_K: return n % 256 ? 0 : n / 256 * 144;
    case T_Q8_0: return n % 32 ? 0 : n / 32 * 34;
    case T_Q6_K: return n % 256 ? 0 : n / 256 * 210;
    default: return 0;
  }
}

/* Q4_K packed 6-bit (scale, min) pair j of a super-block, GGUF get_scale_min_k4. */
static void q4k_scale_min(const uint8_t* sc12, int j, int* sc, int* mn) {
  if (j < 4) {
    *sc = sc12[j] & 63;
    *mn = sc12[j + 4] & 63;
  } else {
    *sc = (sc12[j + 4] & 0x0F) | ((sc12[j - 4] >> 6) << 4);
    *mn = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
  }
}

/* Q4_0 weight i of a block (0..31) as the integer q-8. */
static inline int q4_0_q(const uint8_t* blk, int i) {
  const uint8_t* qs = blk + 2;
  return (i < 16 ? (qs[i] & 0x0F) : (qs[i - 16] >> 4)) - 8;
}
/* Q4_K nibble of weight i (0..255) of a super-block. */
static inline int q4_k_q(const uint8_t* blk, int i) {
  const uint8_t* qs = blk + 16;
  int c = i / 64, l = i % 32, hi = (i / 32) & 1;
  uint8_t b = qs[32 * c + l];
  return hi ? (b >> 4) : (b & 0x0F);
}

/* Q8_0 weight i (0..31) of a block: int8 after the fp16 scale. */
static inline int q8_0_q(const uint8_t* blk, int i) { return (int)(int8_t)blk[2 + i]; }
/* Q6_K weight i (0..255) of a super-block as the integer q-32 (GGUF block_q6_K: ql[128],
   qh[64], int8 scales[16], fp16 d; half h = i/128, k = (i%128)/32, l = i%32: low nibble in
   ql[64h + l + 32(k&1)] (high nibble when k >= 2), top bits 2k..2k+1 of qh[32h + l]). */
static inline int q6_k_q(const uint8_t* blk, int i) {
  int h = i / 128, r = i % 128, k = r / 32, l = r % 32;
  int lo = (blk[64 * h + l + 32 * (k & 1)] >> (k >= 2 ? 4 : 0)) & 15;
  int hi = (blk[128 + 32 * h + l] >> (2 * k)) & 3;
  return (lo | (hi << 4)) - 32;
}
static inline float q6_k_step(const uint8_t* blk, int j /* 0..15 */) {
  uint16_t dh; memcpy(&dh, blk + 208, 2);
  return h2f(dh) * (float)(int8_t)blk[192 + j];
}

int orc_dequant(int type, const void* blocks, uint64_t n, float* out) {
  const uint8_t* p = (const uint8_t*)blocks;
  if (type == T_Q8_0) {
    if (n % 32) return -1;
    for (uint64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = p + b * 34;
      uint16_t dh; memcpy(&dh, blk, 2);
      float d = h2f(dh);
      for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)q8_0_q(blk, i);
    }
    return 0;
  }
  if (type == T_Q6_K) {
    if (n % 256) return -1;
    for (uint64_t b = 0; b < n / 256; ++b) {
      const uint8_t* blk = p + b * 210;
      for (int i = 0; i < 256; ++i) out[b * 256 + i] = q6_k_step(blk, i / 16) * (float)q6_k_q(blk, i);
    }
    return 0;
  }
  if (type == T_Q4_0) {
    if (n % 32) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < (int64_t)(n / 32); ++b) {
      const uint8_t* blk = p + b * 18;
      uint16_t dh; memcpy(&dh, blk, 2);
      float d = h2f(dh);
      for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)q4_0_q(blk, i);
    }
    return 0;
  }
  if (type == T_Q4_K) {
    if (n % 256) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < (int64_t)(n / 256); ++b) {
      const uint8_t* blk = p + b * 144;
      uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
      float d = h2f(dh), dmin = h2f(mh);
      for (int j = 0; j < 8; ++j) {
        int sc, mn; q4k_scale_min(blk + 4, j, &sc, &mn);
        float s = d * (float)sc, m = dmin * (float)mn;
        for (int l = 0; l < 32; ++l) {
          int i = 32 * j + l;
          out[b * 256 + i] = s * (float)q4_k_q(blk, i) - m;
        }
      }
    }
    return 0;
  }
  if (type == T_F16) {
    const uint16_t* h = (const uint16_t*)blocks;
    for (uint64_t i = 0; i < n; ++i) out[i] = h2f(h[i]);
    return 0;
  }
  if (type == T_F32) { memcpy(out, blocks, n * 4); return 0; }
  return -1;
}

/* Q4_0 quantiser: the GGUF reference algorithm (ggml quantize_row_q4_0_ref), fp32 steps. */
int orc_quantize_q4_0(const float* x, uint64_t n, void* out) {
  if (n % 32) return -1;
  uint8_t* o = (uint8_t*)out;
  for (uint64_t b = 0; b < n / 32; ++b) {
    const float* v = x + b * 32;
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < 32; ++i)
      if (fabsf(v[i]) > amax) { amax = fabsf(v[i]); mx = v[i]; }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = f2h(d);
    uint8_t* blk = o + b * 18;
    memcpy(blk, &dh, 2);
    for (int i = 0; i < 16; ++i) {
      float a = v[i] * id + 8.5f, c = v[i + 16] * id + 8.5f;
      int qa = (int)truncf(a), qc = (int)truncf(c);
      if (qa > 15) qa = 15; if (qa < 0) qa = 0;
      if (qc > 15) qc = 15; if (qc < 0) qc = 0;
      blk[2 + i] = (uint8_t)(qa | (qc << 4));
    }
  }
  return 0;
}

/*
 * Quantised GEMV with the device's arithmetic structure:
 *  Q4_0: y = sum_b d_b * (sum_{i<32} (q_i - 8) * x_i)
 *  Q4_K: y = sum_sb [ d * sum_j sc_j * S1_j  -  dmin * sum_j m_j * S0_j ],
 *        S1_j = sum_{i in j} q_i * x_i,  S0_j = sum_{i in j} x_i
 */
int orc_qgemv(int type, const void* w, int N, int K, const uint16_t* x16, int M, float* y, int ldy) {
  const uint8_t* W = (const uint8_t*)w;
  float* xf = (float*)malloc((size_t)M * K * sizeof(float));
  if (!xf) return -2;
  for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = h2f(x16[i]);
  int rc = 0;
  if (type == T_Q4_0) {
    if (K % 32) { free(xf); return -1; }
    size_t row_bytes = (size_t)K / 32 * 18;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint8_t* row = W + (size_t)n * row_bytes;
      float acc[64];
      for (int m0 = 0; m0 < M; m0 += 64) {
        int mc = M - m0 < 64 ? M - m0 : 64;
        for (int m = 0; m < mc; ++m) acc[m] = 0.0f;
        for (int b = 0; b < K / 32; ++b) {
          const uint8_t* blk = row + (size_t)b * 18;
          uint16_t dh; memcpy(&dh, blk, 2);
          float d = h2f(dh);
          float q[32];
          for (int i = 0; i < 32; ++i) q[i] = (float)q4_0_q(blk, i);
          for (int m = 0; m < mc; ++m) {
            const float* xv = xf + (size_t)(m0 + m) * K + b * 32;
            float s = 0.0f;
            for (int i = 0; i < 32; ++i) s += q[i] * xv[i];
            acc[m] = fmaf(d, s, acc[m]);
          }
        }
        for (int m = 0; m < mc; ++m) y[(size_t)(m0 + m) * ldy + n] = acc[m];
      }
    }
  } else if (type == T_Q4_K) {
    if (K % 256) { free(xf); return -1; }
    size_t row_bytes = (size_t)K / 256 * 144;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint8_t* row = W + (size_t)n * row_bytes;
      float acc[64];
      for (int m0 = 0; m0 < M; m0 += 64) {
        int mc = M - m0 < 64 ? M - m0 : 64;
        for (int m = 0; m < mc; ++m) acc[m] = 0.0f;
        for (int b = 0; b < K / 256; ++b) {
          const uint8_t* blk = row + (size_t)b * 144;
          uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
          float d = h2f(dh), dmin = h2f(mh);
          int sc[8], mn[8];
          for (int j = 0; j < 8; ++j) q4k_scale_min(blk + 4, j, &sc[j], &mn[j]);
          float q[256];
          for (int i = 0; i < 256; ++i) q[i] = (float)q4_k_q(blk, i);
          for (int m = 0; m < mc; ++m) {
            const float* xv = xf + (size_t)(m0 + m) * K + b * 256;
            float t1 = 0.0f, t0 = 0.0f;
            for (int j = 0; j < 8; ++j) {
              float s1 = 0.0f, s0 = 0.0f;
              for (int i = 0; i < 32; ++i) { s1 += q[32 * j + i] * xv[32 * j + i]; s0 += xv[32 * j + i]; }
              t1 = fmaf((float)sc[j], s1, t1);
              t0 = fmaf((float)mn[j], s0, t0);
            }
            acc[m] = fmaf(d, t1, acc[m]);
            acc[m] = fmaf(-dmin, t0, acc[m]);
          }
        }
        for (int m = 0; m < mc; ++m) y[(size_t)(m0 + m) * ldy + n] = acc[m];
      }
    }
  } else if (type == T_F16 || type == T_F32) {
    /* plain rows (a tied F16 / F32 head): y = sum_i w_i * x_i in index order */
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      for (int m = 0; m < M; ++m) {
        const float* xv = xf + (size_t)m * K;
        float acc = 0.0f;
        for (int i = 0; i < K; ++i) {
          const float wv = type == T_F16 ? h2f(((const uint16_t*)W)[(size_t)n * K + i]) : ((const float*)W)[(size_t)n * K + i];
          acc = fmaf(wv, xv[i], acc);
        }
        y[(size_t)m * ldy + n] = acc;
      }
    }
  } else if (type == T_Q8_0) {
    /* y = sum_b d_b * (sum_{i<32} q_i * x_i) */
    if (K % 32) { free(xf); return -1; }
    size_t row_bytes = (size_t)K / 32 * 34;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint8_t* row = W + (size_t)n * row_bytes;
      for (int m = 0; m < M; ++m) {
        const float* xv = xf + (size_t)m * K;
        float acc = 0.0f;
        for (int b = 0; b < K / 32; ++b) {
          const uint8_t* blk = row + (size_t)b * 34;
          uint16_t dh; memcpy(&dh, blk, 2);
          float s = 0.0f;
          for (int i = 0; i < 32; ++i) s += (float)q8_0_q(blk, i) * xv[b * 32 + i];
          acc = fmaf(h2f(dh), s, acc);
        }
        y[(size_t)m * ldy + n] = acc;
      }
    }
  } else if (type == T_Q6_K) {
    /* y = sum over 16-weight sub-blocks j of (d * sc_j) * (sum_{i in j} (q_i - 32) * x_i) */
    if (K % 256) { free(xf); return -1; }
    size_t row_bytes = (size_t)K / 256 * 210;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint8_t* row = W + (size_t)n * row_bytes;
      for (int m = 0; m < M; ++m) {
        const float* xv = xf + (size_t)m * K;
        float acc = 0.0f;
        for (int b = 0; b < K / 256; ++b) {
          const uint8_t* blk = row + (size_t)b * 210;
          for (int j = 0; j < 16; ++j) {
            float s = 0.0f;
            for (int i = 0; i < 16; ++i) s += (float)q6_k_q(blk, 16 * j + i) * xv[b * 256 + 16 * j + i];
            acc = fmaf(q6_k_step(blk, j), s, acc);
          }
        }
        y[(size_t)m * ldy + n] = acc;
      }
    }
  } else {
    rc = -1;
  }
  free(xf);
  return rc;
}

/* ------------------------------------------------------------------ RoPE / attention */
void orc_rope_table(float base, int head_dim, int n_pos, float* cos_out, float* sin_out) {
  int half = head_dim / 2;
  for (int p = 0; p < n_pos; ++p)
    for (int i = 0; i < half; ++i) {
      double theta = (double)p * pow((double)base, -2.0 * (double)i / (double)head_dim);
      cos_out[(size_t)p * half + i] = (float)cos(theta);
      sin_out[(size_t)p * half + i] = (float)sin(theta);
    }
}

int orc_attention(int H, int Hkv, int hd, int cap, float scale, const float* q, const uint16_t* k,
                  const uint16_t* v, const int32_t* row_seq, const int32_t* row_pos, int M,
                  uint16_t* out) {
  int group = H / Hkv;
#pragma omp parallel for collapse(2) schedule(static)
  for (int m = 0; m < M; ++m)
    for (int h = 0; h < H; ++h) {
      int s = row_seq[m], pos = row_pos[m], kvh = h / group;
      const float* qv = q + ((size_t)m * H + h) * hd;
      const uint16_t* kb = k + ((size_t)s * Hkv + kvh) * cap * hd;
      const uint16_t* vb = v + ((size_t)s * Hkv + kvh) * cap * hd;
      float* sc = (float*)malloc((size_t)(pos + 1) * sizeof(float));
      float mx = -INFINITY;
      for (int j = 0; j <= pos; ++j) {
        float a = 0.0f;
        for (int d = 0; d < hd; ++d) a = fmaf(qv[d], h2f(kb[(size_t)j * hd + d]), a);
        sc[j] = a * scale;
        if (sc[j] > mx) mx = sc[j];
      }
      float l = 0.0f;
      for (int j = 0; j <= pos; ++j) { sc[j] = expf(sc[j] - mx); l += sc[j]; }
      for (int d = 0; d < hd; ++d) {
        float o = 0.0f;
        for (int j = 0; j <= pos; ++j) o = fmaf(sc[j], h2f(vb[(size_t)j * hd + d]), o);
        out[((size_t)m * H + h) * hd + d] = f2h(o / l);
      }
      free(sc);
    }
  return 0;
}

/* ------------------------------------------------------------------ GGUF reader */
typedef struct {
  char name[96];
  int type;
  int n_dims;
  uint64_t ne[4];
  uint64_t offset;
  size_t nbytes;
  const uint8_t* data;
} orc_tensor;

typedef struct {
  const orc_tensor* q;
  const orc_tensor *k, *v, *o, *gate, *up, *down, *attn_norm, *ffn_norm;
} orc_layer;

struct orc_model {
  void* map;
  size_t map_len;
  orc_desc d;
  int n_tensors;
  orc_tensor* t;
  orc_layer* layers;
  const orc_tensor *embd, *out_norm, *out;
  float *rope_cos, *rope_sin;
  int rope_n;
};

struct orc_kv {
  int n_seq, cap, n_layer, Hkv, hd;
  uint16_t *k, *v; /* [L][S][Hkv][cap][hd] */
};

typedef struct { const uint8_t* p; const uint8_t* end; int bad; } rd_t;
static uint64_t rd_u(rd_t* r, int n) {
  if (r->p + n > r->end) { r->bad = 1; return 0; }
  uint64_t v = 0; memcpy(&v, r->p, n); r->p += n; return v;
}
static int rd_str(rd_t* r, char* buf, size_t cap) {
  uint64_t len = rd_u(r, 8);
  if (r->bad || r->p + len > r->end) { r->bad = 1; return -1; }
  if (buf) { size_t c = len < cap - 1 ? len : cap - 1; memcpy(buf, r->p, c); buf[c] = 0; }
  r->p += len; return 0;
}
/* GGUF value types */
enum { GV_U8, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STR, GV_ARR, GV_U64, GV_I64, GV_F64 };
static int gv_size(int t) {
  switch (t) { case GV_U8: case GV_I8: case GV_BOOL: return 1; case GV_U16: case GV_I16: return 2;
    case GV_U32: case GV_I32: case GV_F32: return 4; case GV_U64: case GV_I64: case GV_F64: return 8; }
  return -1;
}
static double rd_scalar(rd_t* r, int t) {
  uint64_t raw = rd_u(r, gv_size(t));
  switch (t) {
    case GV_I8: return (double)(int8_t)raw; case GV_I16: return (double)(int16_t)raw;
    case GV_I32: return (double)(int32_t)raw; case GV_I64: return (double)(int64_t)raw;
    case GV_F32: { float f; uint32_t u = (uint32_t)raw; memcpy(&f, &u, 4); return f; }
    case GV_F64: { double f; memcpy(&f, &raw, 8); return f; }
    default: return (double)raw;
  }
}

static const orc_tensor* find_t(const orc_model* m, const char* name) {
  for (int i = 0; i < m->n_tensors; ++i)
    if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
  return NULL;
}

orc_model* orc_model_load(const char* path, char* err, int errlen) {
#define FAIL(...) do { if (err) snprintf(err, errlen, __VA_ARGS__); goto fail; } while (0)
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  int fd = open(path, O_RDONLY);
  struct stat st;
  if (fd < 0 || fstat(fd, &st) != 0) { if (fd >= 0) close(fd); if (err) snprintf(err, errlen, "open %s", path); free(m); return NULL; }
  m->map_len = (size_t)st.st_size;
  m->map = mmap(NULL, m->map_len, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m->map == MAP_FAILED) { m->map = NULL; FAIL("mmap"); }
  {
    rd_t r = {(const uint8_t*)m->map, (const uint8_t*)m->map + m->map_len, 0};
    if (m->map_len < 24 || memcmp(r.p, "GGUF", 4) != 0) FAIL("bad magic");
    r.p += 4;
    uint32_t version = (uint32_t)rd_u(&r, 4);
    if (version < 2 || version > 3) FAIL("unsupported GGUF version %u", version);
    uint64_t n_t = rd_u(&r, 8), n_kv = rd_u(&r, 8);
    if (n_t > 100000 || n_kv > 100000) FAIL("implausible counts");
    uint64_t alignment = 32;
    double rms_eps = 1e-5, rope_base = 10000.0;
    int n_layer = -1, d_model = -1, n_head = -1, n_head_kv = -1, d_ff = -1, n_vocab = -1;
    for (uint64_t i = 0; i < n_kv; ++i) {
      char key[256];
      if (rd_str(&r, key, sizeof key)) FAIL("kv key");
      int t = (int)rd_u(&r, 4);
      if (t == GV_STR) { rd_str(&r, NULL, 0); continue; }
      if (t == GV_ARR) {
        int et = (int)rd_u(&r, 4); uint64_t cnt = rd_u(&r, 8);
        for (uint64_t j = 0; j < cnt && !r.bad; ++j) {
          if (et == GV_STR) rd_str(&r, NULL, 0);
          else if (gv_size(et) > 0) r.p += gv_size(et);
          else FAIL("nested array");
        }
        continue;
      }
      if (gv_size(t) < 0) FAIL("kv type %d", t);
      double v = rd_scalar(&r, t);
      if (!strcmp(key, "general.alignment")) alignment = (uint64_t)v;
      else if (!strcmp(key, "llama.block_count")) n_layer = (int)v;
      else if (!strcmp(key, "llama.embedding_length")) d_model = (int)v;
      else if (!strcmp(key, "llama.attention.head_count")) n_head = (int)v;
      else if (!strcmp(key, "llama.attention.head_count_kv")) n_head_kv = (int)v;
      else if (!strcmp(key, "llama.feed_forward_length")) d_ff = (int)v;
      else if (!strcmp(key, "llama.vocab_size")) n_vocab = (int)v;
      else if (!strcmp(key, "llama.attention.layer_norm_rms_epsilon")) rms_eps = v;
      else if (!strcmp(key, "llama.rope.freq_base")) rope_base = v;
    }
    if (r.bad) FAIL("truncated metadata");
    if (alignment == 0 || (alignment & (alignment - 1))) alignment = 32;
    m->n_tensors = (int)n_t;
    m->t = (orc_tensor*)calloc(n_t ? n_t : 1, sizeof(orc_tensor));
    for (uint64_t i = 0; i < n_t; ++i) {
      orc_tensor* t = &m->t[i];
      if (rd_str(&r, t->name, sizeof t->name)) FAIL("tensor name");
      t->n_dims = (int)rd_u(&r, 4);
      if (t->n_dims < 1 || t->n_dims > 4) FAIL("n_dims");
      uint64_t n = 1;
      for (int j = 0; j < 4; ++j) t->ne[j] = 1;
      for (int j = 0; j < t->n_dims; ++j) { t->ne[j] = rd_u(&r, 8); n *= t->ne[j]; }
      t->type = (int)rd_u(&r, 4);
      t->offset = rd_u(&r, 8);
      t->nbytes = orc_type_nbytes(t->type, n);
      if (!t->nbytes) FAIL("tensor %s: unsupported type %d", t->name, t->type);
    }
    if (r.bad) FAIL("truncated tensor infos");
    size_t hdr = (size_t)(r.p - (const uint8_t*)m->map);
    size_t data_off = (hdr + alignment - 1) & ~(size_t)(alignment - 1);
    for (uint64_t i = 0; i < n_t; ++i) {
      orc_tensor* t = &m->t[i];
      if (data_off + t->offset + t->nbytes > m->map_len) FAIL("tensor %s out of file", t->name);
      t->data = (const uint8_t*)m->map + data_off + t->offset;
    }
    if (n_vocab < 0) {
      const orc_tensor* e = find_t(m, "token_embd.weight");
      if (e) n_vocab = (int)e->ne[1];
    }
    if (n_head_kv < 0) n_head_kv = n_head;
    if (n_layer <= 0 || d_model <= 0 || n_head <= 0 || d_ff <= 0 || n_vocab <= 0) FAIL("missing llama.* metadata");
    orc_desc* d = &m->d;
    d->n_layer = n_layer; d->d_model = d_model; d->n_head = n_head; d->n_head_kv = n_head_kv;
    d->head_dim = d_model / n_head; d->d_ff = d_ff; d->n_vocab = n_vocab;
    d->rms_eps = (float)rms_eps; d->rope_base = (float)rope_base;
    m->layers = (orc_layer*)calloc(n_layer, sizeof(orc_layer));
    char nm[128];
    for (int l = 0; l < n_layer; ++l) {
      orc_layer* L = &m->layers[l];
#define GETT(field, suffix) snprintf(nm, sizeof nm, "blk.%d." suffix ".weight", l); L->field = find_t(m, nm); if (!L->field) FAIL("missing %s", nm);
      GETT(q, "attn_q"); GETT(k, "attn_k"); GETT(v, "attn_v"); GETT(o, "attn_output");
      GETT(gate, "ffn_gate"); GETT(up, "ffn_up"); GETT(down, "ffn_down");
      GETT(attn_norm, "attn_norm"); GETT(ffn_norm, "ffn_norm");
#undef GETT
    }
    m->embd = find_t(m, "token_embd.weight");
    m->out_norm = find_t(m, "output_norm.weight");
    m->out = find_t(m, "output.weight");
    if (!m->out) m->out = m->embd; /* tied embeddings: the LM head is token_embd */
    if (!m->embd || !m->out_norm || !m->out) FAIL("missing token_embd/output_norm/output");
    d->wtype = m->layers[0].q->type;
  }
  return m;
fail:
  orc_model_free(m);
  return NULL;
#undef FAIL
}

void orc_model_free(orc_model* m) {
  if (!m) return;
  if (m->map) munmap(m->map, m->map_len);
  free(m->t); free(m->layers); free(m->rope_cos); free(m->rope_sin);
  free(m);
}

void orc_model_get_desc(const orc_model* m, orc_desc* d) { *d = m->d; }

const void* orc_model_tensor(const orc_model* m, const char* name, int* type, uint64_t ne[4], size_t* nbytes) {
  const orc_tensor* t = find_t(m, name);
  if (!t) return NULL;
  if (type) *type = t->type;
  if (ne) memcpy(ne, t->ne, sizeof t->ne);
  if (nbytes) *nbytes = t->nbytes;
  return t->data;
}

orc_kv* orc_kv_alloc(const orc_model* m, int n_seq, int cap) {
  orc_kv* kv = (orc_kv*)calloc(1, sizeof(orc_kv));
  kv->n_seq = n_seq; kv->cap = cap; kv->n_layer = m->d.n_layer; kv->Hkv = m->d.n_head_kv; kv->hd = m->d.head_dim;
  size_t n = (size_t)kv->n_layer * n_seq * kv->Hkv * cap * kv->hd;
  kv->k = (uint16_t*)calloc(n, 2);
  kv->v = (uint16_t*)calloc(n, 2);
  if (!kv->k || !kv->v) { orc_kv_free(kv); return NULL; }
  return kv;
}
void orc_kv_free(orc_kv* kv) { if (kv) { free(kv->k); free(kv->v); free(kv); } }

static void ensure_rope(orc_model* m, int n_pos) {
  if (m->rope_n >= n_pos) return;
  int half = m->d.head_dim / 2;
  free(m->rope_cos); free(m->rope_sin);
  m->rope_cos = (float*)malloc((size_t)n_pos * half * 4);
  m->rope_sin = (float*)malloc((size_t)n_pos * half * 4);
  orc_rope_table(m->d.rope_base, m->d.head_dim, n_pos, m->rope_cos, m->rope_sin);
  m->rope_n = n_pos;
}

/* x16[m] = fp16((x[m] * r) * g) with r = 1 / sqrt(sum(x^2)/d + eps) */
static void rmsnorm16(const float* x, const float* g, int M, int d, float eps, uint16_t* out) {
  for (int m = 0; m < M; ++m) {
    const float* xv = x + (size_t)m * d;
    float ss = 0.0f;
    for (int i = 0; i < d; ++i) ss = fmaf(xv[i], xv[i], ss);
    float r = 1.0f / sqrtf(ss / (float)d + eps);
    for (int i = 0; i < d; ++i) out[(size_t)m * d + i] = f2h((xv[i] * r) * g[i]);
  }
}

int orc_forward(orc_model* mdl, orc_kv* kv, int M, int rps, const int32_t* tokens,
                const int32_t* row_seq, const int32_t* row_pos, int logits_mode, float* logits, int ld) {
  const orc_desc* D = &mdl->d;
  int d = D->d_model, H = D->n_head, Hkv = D->n_head_kv, hd = D->head_dim, F = D->d_ff, V = D->n_vocab;
  int nq = H * hd, nkv = Hkv * hd, half = hd / 2;
  int maxpos = 0;
  for (int m = 0; m < M; ++m) {
    if (row_pos[m] >= kv->cap || row_pos[m] < 0 || row_seq[m] < 0 || row_seq[m] >= kv->n_seq) return -1;
    if (tokens[m] < 0 || tokens[m] >= V) return -1;
    if (row_pos[m] > maxpos) maxpos = row_pos[m];
  }
  ensure_rope(mdl, kv->cap > maxpos + 1 ? kv->cap : maxpos + 1);
  float* x = (float*)malloc((size_t)M * d * 4);
  uint16_t* x16 = (uint16_t*)malloc((size_t)M * (F > nq ? (F > d ? F : d) : (nq > d ? nq : d)) * 2);
  float* qkv = (float*)malloc((size_t)M * (nq + 2 * nkv) * 4);
  float* tmp = (float*)malloc((size_t)M * (2 * F > d ? 2 * F : d) * 4);
  uint16_t* att = (uint16_t*)malloc((size_t)M * nq * 2);
  /* embedding rows, dequantised with the block formulas of orc_dequant */
  const size_t erow = orc_type_nbytes(mdl->embd->type, (uint64_t)d);
  for (int m = 0; m < M; ++m)
    orc_dequant(mdl->embd->type, (const uint8_t*)mdl->embd->data + (size_t)tokens[m] * erow, (uint64_t)d,
                x + (size_t)m * d);
  int wt = D->wtype;
  for (int l = 0; l < D->n_layer; ++l) {
    const orc_layer* L = &mdl->layers[l];
    size_t lay = (size_t)l * kv->n_seq * Hkv * kv->cap * hd;
    rmsnorm16(x, (const float*)L->attn_norm->data, M, d, D->rms_eps, x16);
    orc_qgemv(L->q->type, L->q->data, nq, d, x16, M, qkv, nq + 2 * nkv);
    orc_qgemv(L->k->type, L->k->data, nkv, d, x16, M, qkv + nq, nq + 2 * nkv);
    orc_qgemv(L->v->type, L->v->data, nkv, d, x16, M, qkv + nq + nkv, nq + 2 * nkv);
    for (int m = 0; m < M; ++m) {
      float* row = qkv + (size_t)m * (nq + 2 * nkv);
      const float* cs = mdl->rope_cos + (size_t)row_pos[m] * half;
      const float* sn = mdl->rope_sin + (size_t)row_pos[m] * half;
      for (int f = 0; f < nq + nkv; f += 2) {
        int i = (f % hd) / 2;
        float x0 = row[f], x1 = row[f + 1];
        row[f] = fmaf(x0, cs[i], -(x1 * sn[i]));
        row[f + 1] = fmaf(x0, sn[i], x1 * cs[i]);
      }
      int s = row_seq[m], p = row_pos[m];
      for (int h = 0; h < Hkv; ++h)
        for (int e = 0; e < hd; ++e) {
          size_t idx = lay + (((size_t)s * Hkv + h) * kv->cap + p) * hd + e;
          kv->k[idx] = f2h(row[nq + h * hd + e]);
          kv->v[idx] = f2h(row[nq + nkv + h * hd + e]);
        }
    }
    /* attention reads q from a compact [M][nq] copy */
    float* q = tmp;
    for (int m = 0; m < M; ++m) memcpy(q + (size_t)m * nq, qkv + (size_t)m * (nq + 2 * nkv), (size_t)nq * 4);
    orc_attention(H, Hkv, hd, kv->cap, 1.0f / sqrtf((float)hd), q, kv->k + lay, kv->v + lay, row_seq, row_pos, M, att);
    orc_qgemv(L->o->type, L->o->data, d, nq, att, M, tmp, d);
    for (size_t i = 0; i < (size_t)M * d; ++i) x[i] = x[i] + tmp[i];
    rmsnorm16(x, (const float*)L->ffn_norm->data, M, d, D->rms_eps, x16);
    orc_qgemv(L->gate->type, L->gate->data, F, d, x16, M, tmp, 2 * F);
    orc_qgemv(L->up->type, L->up->data, F, d, x16, M, tmp + F, 2 * F);
    for (int m = 0; m < M; ++m)
      for (int i = 0; i < F; ++i) {
        float g = tmp[(size_t)m * 2 * F + i], u = tmp[(size_t)m * 2 * F + F + i];
        float sg = g / (1.0f + expf(-g));
        x16[(size_t)m * F + i] = f2h(sg * u);
      }
    orc_qgemv(L->down->type, L->down->data, d, F, x16, M, tmp, d);
    for (size_t i = 0; i < (size_t)M * d; ++i) x[i] = x[i] + tmp[i];
  }
  (void)wt;
  /* final norm + LM head on the selected rows */
  int nsel = logits_mode == 1 ? M / rps : M;
  float* xs = (float*)malloc((size_t)nsel * d * 4);
  for (int s = 0; s < nsel; ++s) {
    int m = logits_mode == 1 ? s * rps + rps - 1 : s;
    memcpy(xs + (size_t)s * d, x + (size_t)m * d, (size_t)d * 4);
  }
  rmsnorm16(xs, (const float*)mdl->out_norm->data, nsel, d, D->rms_eps, x16);
  int rc = orc_qgemv(mdl->out->type, mdl->out->data, V, d, x16, nsel, logits, ld);
  free(xs); free(x); free(x16); free(qkv); free(tmp); free(att);
  return rc;
}

/* ------------------------------------------------------------------ sampling */
typedef struct { float z; int i; } zi_t;
static int cmp_zi_desc(const void* a, const void* b) {
  const zi_t *x = (const zi_t*)a, *y = (const zi_t*)b;
  if (x->z > y->z) return -1;
  if (x->z < y->z) return 1;
  return x->i - y->i;
}

static int argmax_f(const float* l, int V) {
  int best = 0;
  for (int i = 1; i < V; ++i) if (l[i] > l[best]) best = i;
  return best;
}

/*
 * exp(x), x = z - max z <= 0, for the warp weights: the same sequence of IEEE binary32
 * operations as ulb_warp_exp in universal-loader_b200/csrc/ulb_common.h, so the weights
 * are bit-identical (this file is built with -ffp-contract=off; fmaf is the fused op).
 * k = rint(x / ln 2); r = x - k*C1 - k*C2 with C1 = 355/512 (Cody & Waite two-part ln 2);
 * exp(r) by its degree-7 Taylor polynomial in Horner form; times 2^k.  x < -87 gives 0.
 */
float orc_warp_exp(float x) {
  if (!(x >= -87.0f)) return 0.0f;
  float kf = rintf(x * 1.44269504088896341f);
  float r = fmaf(kf, -0.693359375f, x);
  r = fmaf(kf, 2.12194440054690583e-4f, r);
  float p = 1.98412698412698413e-4f;
  p = fmaf(p, r, 1.38888888888888889e-3f);
  p = fmaf(p, r, 8.33333333333333333e-3f);
  p = fmaf(p, r, 4.16666666666666667e-2f);
  p = fmaf(p, r, 1.66666666666666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  uint32_t bits = (uint32_t)((int)kf + 127) << 23;
  float two_k;
  memcpy(&two_k, &bits, 4);
  return p * two_k;
}

/* top-p masses in 40-bit fixed point, added as integers (order-independent): floor(e * 2^40) */
static uint64_t orc_mass_fix(float e) { return (uint64_t)((double)e * 1099511627776.0); }
/* the mass the kept set reaches first: floor(top_p * total), at least 1 */
static uint64_t orc_topp_target(float top_p, uint64_t total) {
  uint64_t r = (uint64_t)((double)top_p * (double)total);
  return r < 1 ? 1 : r;
}

/*
 * Warp weights.  z = logits * (1/T), 1/T rounded once; top-k keeps z >= k-th largest z; e = orc_warp_exp(z - max)
 * as fp64; top-p keeps v iff (mass of z_u > z_v) < R, masses in fixed point (E = orc_mass_fix(e), summed as
 * integers) and R = orc_topp_target(top_p, sum of E over the top-k set); *Zout = sum of kept e (fp64).
 * Greedy (T <= 0): one-hot at the argmax, Z = 1.
 */
int orc_warp_weights(const float* logits, int V, const orc_warp* w, double* e, double* Zout) {
  if (!(w->temperature > 0.0f)) {
    for (int i = 0; i < V; ++i) e[i] = 0.0;
    e[argmax_f(logits, V)] = 1.0;
    *Zout = 1.0;
    return 0;
  }
  float iT = 1.0f / w->temperature; /* 1/T rounded once; z = logit * iT */
  float* z = (float*)malloc((size_t)V * 4);
  float mx = -INFINITY;
  for (int i = 0; i < V; ++i) { z[i] = logits[i] * iT + 0.0f; if (z[i] > mx) mx = z[i]; }
  float thr_k = -INFINITY;
  if (w->top_k > 0 && w->top_k < V) {
    zi_t* s = (zi_t*)malloc((size_t)V * sizeof(zi_t));
    for (int i = 0; i < V; ++i) { s[i].z = z[i]; s[i].i = i; }
    qsort(s, V, sizeof(zi_t), cmp_zi_desc);
    thr_k = s[w->top_k - 1].z;
    free(s);
  }
  double Z = 0.0;
  for (int i = 0; i < V; ++i) {
    e[i] = z[i] >= thr_k ? (double)orc_warp_exp(z[i] - mx) : 0.0;
    Z += e[i];
  }
  if (w->top_p > 0.0f && w->top_p < 1.0f) {
    zi_t* s = (zi_t*)malloc((size_t)V * sizeof(zi_t));
    int n = 0;
    uint64_t tot = 0;
    for (int i = 0; i < V; ++i)
      if (e[i] > 0.0) {
        s[n].z = z[i]; s[n].i = i; ++n;
        tot += orc_mass_fix((float)e[i]);
      }
    qsort(s, n, sizeof(zi_t), cmp_zi_desc);
    const uint64_t R = orc_topp_target(w->top_p, tot);
    uint64_t cum = 0;
    float thr_p = s[0].z;
    for (int j = 0; j < n; ++j) {
      cum += orc_mass_fix((float)e[s[j].i]);
      if (cum >= R) { thr_p = s[j].z; break; }
      thr_p = s[j].z;
    }
    free(s);
    Z = 0.0;
    for (int i = 0; i < V; ++i) {
      if (z[i] < thr_p) e[i] = 0.0;
      Z += e[i];
    }
  }
  free(z);
  *Zout = Z;
  return 0;
}

/* normalised warped distribution: probs = e / Z */
int orc_warp_probs(const float* logits, int V, const orc_warp* w, double* probs) {
  double Z;
  orc_warp_weights(logits, V, w, probs, &Z);
  for (int i = 0; i < V; ++i) probs[i] /= Z;
  return 0;
}

/* inverse CDF in index order over fp64 weights w: smallest i whose cumulative weight
   exceeds u * (sum of w) */
static int inv_cdf(const double* w, int V, float u) {
  double total = 0.0;
  for (int i = 0; i < V; ++i) total += w[i];
  double target = (double)u * total, cum = 0.0;
  int last = -1;
  for (int i = 0; i < V; ++i) {
    if (w[i] <= 0.0) continue;
    cum += w[i];
    last = i;
    if (cum > target) return i;
  }
  return last < 0 ? 0 : last;
}

int orc_sample(const float* logits, int V, const orc_warp* w, float u) {
  if (!(w->temperature > 0.0f)) return argmax_f(logits, V);
  double* e = (double*)malloc((size_t)V * 8);
  double Z;
  orc_warp_weights(logits, V, w, e, &Z);
  int t = inv_cdf(e, V, u);
  free(e);
  return t;
}

int orc_spec_accept(const float* pl, const float* ql, const int32_t* draft, int B, int k, int V,
                    const orc_warp* w, uint64_t seed, uint32_t round, int32_t* out_tokens, int32_t* out_n) {
  int greedy = !(w->temperature > 0.0f);
  double* p = (double*)malloc((size_t)V * 8);
  double* q = (double*)malloc((size_t)V * 8);
  for (int b = 0; b < B; ++b) {
    int n = 0, tok = -1;
    for (int i = 0; i < k; ++i) {
      const float* pi = pl + ((size_t)b * (k + 1) + i) * V;
      const float* qi = ql + ((size_t)b * k + i) * V;
      int x = draft[b * k + i];
      if (greedy) {
        int a = argmax_f(pi, V);
        if (x == a) { out_tokens[b * (k + 1) + n] = x; ++n; continue; }
        tok = a; break;
      }
      double Zp, Zq;
      orc_warp_weights(pi, V, w, p, &Zp);
      orc_warp_weights(qi, V, w, q, &Zq);
      float u = orc_uniform(seed, round, (uint32_t)b, (uint32_t)i, 2);
      double px = (unsigned)x < (unsigned)V ? p[x] / Zp : 0.0, qx = (unsigned)x < (unsigned)V ? q[x] / Zq : 0.0;
      if ((double)u * qx < px) { out_tokens[b * (k + 1) + n] = x; ++n; continue; }
      /* residual norm(max(0, p - q)) as max(0, e_p Z_q - e_q Z_p) */
      double tot = 0.0;
      for (int v = 0; v < V; ++v) { double r = p[v] * Zq - q[v] * Zp; q[v] = r > 0.0 ? r : 0.0; tot += q[v]; }
      float u2 = orc_uniform(seed, round, (uint32_t)b, (uint32_t)i, 3);
      tok = tot > 0.0 ? inv_cdf(q, V, u2) : inv_cdf(p, V, u2);
      break;
    }
    if (tok < 0) { /* all k accepted: bonus from p_k */
      const float* pk = pl + ((size_t)b * (k + 1) + k) * V;
      if (greedy) tok = argmax_f(pk, V);
      else {
        double Zp;
        orc_warp_weights(pk, V, w, p, &Zp);
        tok = inv_cdf(p, V, orc_uniform(seed, round, (uint32_t)b, (uint32_t)k, 3));
      }
    }
    out_tokens[b * (k + 1) + n] = tok;
    out_n[b] = n;
  }
  free(p); free(q);
  return 0;
}

/*
 * Tree speculation (the reference's TreeSpeculation(vocab, beam_width, max_depth),
 * src/inference/speculative_decoder.h:62-87, a stub there): a full tree of width w and depth D
 * whose nodes are numbered breadth first, depth 1 first: node i of depth d has rank
 * i - first(d) in its level (first(d) = w + w^2 + ... + w^(d-1)), and the children of the
 * root are nodes 0..w-1, those of node i (depth d < D) first(d+1) + rank * w + c.
 * p rows [B][1 + N][V]: row 0 the root (the last committed token), row 1 + i node i;
 * q rows [B][1 + first(D)][V]: row 0 the root, row 1 + i internal node i (depth < D).
 * tokens [B][N]: the drafted token of each node.
 * Walk from the root.  T = 0: move to the first child whose token is the target's argmax,
 * else commit that argmax and stop.  T > 0: multi-candidate speculative sampling (SpecInfer,
 * Miao et al. 2024): the children are w independent draws from q_u; child c_j is accepted
 * with probability min(1, P_j(x) / q(x)), where P_1 = p_u and, after each rejection,
 * P_(j+1) = norm(max(0, P_j - q_u)); when all w are rejected the correction is drawn from
 * P_(w+1).  In weights: R_1 = max(0, e_p Z_q - e_q Z_p), R_(j+1) = max(0, R_j Z_q - e_q W_j),
 * W_j = sum of R_j, P_(j+1) = R_j / W_j.  A leaf reached (depth D) draws its bonus from p.
 * Uniforms: child c's test (slot c, tag 2); the draw at p row r (slot r, tag 3).  With w = 1
 * this is orc_spec_accept.  Outputs: path[B][D] (nodes accepted, -1 after), n[B], tok[B].
 */
static int tree_first(int w, int d) { int f = 0, p = 1; for (int j = 1; j < d; ++j) { p *= w; f += p; } return f; }

int orc_tree_accept(const float* pl, const float* ql, const int32_t* tokens, int B, int width, int depth, int V,
                    const orc_warp* w, uint64_t seed, uint32_t round, int32_t* out_path, int32_t* out_n,
                    int32_t* out_tok) {
  const int N = tree_first(width, depth + 1), NI = tree_first(width, depth);
  const int greedy = !(w->temperature > 0.0f);
  double* p = (double*)malloc((size_t)V * 8);
  double* q = (double*)malloc((size_t)V * 8);
  double* r = (double*)malloc((size_t)V * 8);
  for (int b = 0; b < B; ++b) {
    int n = 0, tok = -1, u = -1, d = 0; /* u = -1: the root */
    for (int j = 0; j < depth; ++j) out_path[b * depth + j] = -1;
    while (tok < 0) {
      const int prow = u + 1;
      const float* pu = pl + ((size_t)b * (1 + N) + prow) * V;
      if (d == depth) { /* a leaf: the bonus token from p */
        if (greedy) tok = argmax_f(pu, V);
        else {
          double Zp;
          orc_warp_weights(pu, V, w, p, &Zp);
          tok = inv_cdf(p, V, orc_uniform(seed, round, (uint32_t)b, (uint32_t)prow, 3));
        }
        break;
      }
      const int c0 = u < 0 ? 0 : tree_first(width, d + 1) + (u - tree_first(width, d)) * width;
      if (greedy) {
        const int a = argmax_f(pu, V);
        int next = -1;
        for (int c = 0; c < width; ++c)
          if (tokens[b * N + c0 + c] == a) { next = c0 + c; break; }
        if (next < 0) { tok = a; break; }
        out_path[b * depth + n++] = next;
        u = next;
        ++d;
        continue;
      }
      const float* qu = ql + ((size_t)b * (1 + NI) + prow) * V;
      double Zp, Zq, W = 0.0;
      orc_warp_weights(pu, V, w, p, &Zp);
      orc_warp_weights(qu, V, w, q, &Zq);
      int next = -1, level = 0; /* level j: P_(j+1) = r / W after j rejections */
      for (int c = 0; c < width && next < 0; ++c) {
        const int x = tokens[b * N + c0 + c];
        const int ok = (unsigned)x < (unsigned)V;
        const double qx = ok ? q[x] / Zq : 0.0;
        double px;
        if (level == 0) px = ok ? p[x] / Zp : 0.0;
        else px = ok && W > 0.0 ? r[x] / W : 0.0;
        const float ua = orc_uniform(seed, round, (uint32_t)b, (uint32_t)(c0 + c), 2);
        if ((double)ua * qx < px) { next = c0 + c; break; }
        if (level > 0 && !(W > 0.0)) continue; /* nothing left to remove */
        double tot = 0.0;
        for (int v = 0; v < V; ++v) {
          const double t = level == 0 ? p[v] * Zq - q[v] * Zp : r[v] * Zq - q[v] * W;
          r[v] = t > 0.0 ? t : 0.0;
          tot += r[v];
        }
        W = tot;
        ++level;
      }
      if (next >= 0) {
        out_path[b * depth + n++] = next;
        u = next;
        ++d;
        continue;
      }
      const float u2 = orc_uniform(seed, round, (uint32_t)b, (uint32_t)prow, 3);
      tok = W > 0.0 ? inv_cdf(r, V, u2) : inv_cdf(p, V, u2);
    }
    out_n[b] = n;
    out_tok[b] = tok;
  }
  free(p); free(q); free(r);
  return 0;
}

static double top2_margin(const float* l, int V) {
  float a = -INFINITY, b = -INFINITY;
  for (int i = 0; i < V; ++i) {
    if (l[i] > a) { b = a; a = l[i]; } else if (l[i] > b) b = l[i];
  }
  return (double)a - (double)b;
}

/*
 * The device schedule (universal-loader_b200/csrc/spec.cu):
 *  prefill: target and draft over the prompt; first token from the target's last row.
 *  round r: draft step 0 on rows (t[L-2] @ L-2, t[L-1] @ L-1), steps j=1..k-1 on
 *  (d[j-1] @ L-1+j); verify rows (t[L-1] @ L-1, d[0..k-1] @ L..L+k-1); accept.
 */
int orc_spec_generate(orc_model* tg, orc_model* dr, int S, const int32_t* prompts, const int32_t* plen,
                      int max_prompt, int max_new, int k, const orc_warp* w, uint64_t seed,
                      int32_t* out_tokens, int32_t* out_counts, uint64_t stats[4], double* margin_min,
                      double* tok_margin) {
  if (!dr) k = 0;
  int V = tg->d.n_vocab;
  /* finished sequences keep being computed (not committed) until every sequence is done */
  int cap = max_prompt + max_new + 2 * k + 2;
  int hist_len = cap;
  orc_kv* kvt = orc_kv_alloc(tg, S, cap);
  orc_kv* kvd = dr ? orc_kv_alloc(dr, S, cap) : NULL;
  int32_t* hist = (int32_t*)calloc((size_t)S * hist_len, 4);
  int* L = (int*)calloc(S, sizeof(int));
  int* done = (int*)calloc(S, sizeof(int));
  int maxrows = max_prompt > (k + 1) ? max_prompt : (k + 1);
  float* lg = (float*)malloc((size_t)S * (k + 1) * V * 4);
  float* qlg = (float*)malloc((size_t)S * (k > 0 ? k : 1) * V * 4);
  int32_t* tok = (int32_t*)malloc((size_t)S * maxrows * 4 * 2);
  int32_t* seqv = (int32_t*)malloc((size_t)S * maxrows * 4 * 2);
  int32_t* posv = (int32_t*)malloc((size_t)S * maxrows * 4 * 2);
  int32_t* dtok = (int32_t*)malloc((size_t)S * (k > 0 ? k : 1) * 4);
  int32_t* otok = (int32_t*)malloc((size_t)S * (k + 1) * 4);
  int32_t* on = (int32_t*)malloc((size_t)S * 4);
  double mmin = INFINITY;
  int greedy = !(w->temperature > 0.0f);
  memset(stats, 0, 4 * sizeof(uint64_t));
  for (int s = 0; s < S; ++s) {
    int P = plen[s];
    for (int i = 0; i < P; ++i) { hist[(size_t)s * hist_len + i] = prompts[(size_t)s * max_prompt + i]; tok[i] = prompts[(size_t)s * max_prompt + i]; seqv[i] = s; posv[i] = i; }
    orc_forward(tg, kvt, P, P, tok, seqv, posv, 1, lg, V);
    if (dr) orc_forward(dr, kvd, P, P, tok, seqv, posv, 1, qlg, V);
    if (greedy) { double mg = top2_margin(lg, V); if (mg < mmin) mmin = mg; if (tok_margin) tok_margin[(size_t)s * max_new] = mg; }
    int t0 = orc_sample(lg, V, w, orc_uniform(seed, 0, (uint32_t)s, 0, 4));
    hist[(size_t)s * hist_len + P] = t0;
    L[s] = P + 1;
    if (L[s] - P >= max_new) done[s] = 1;
  }
  for (uint32_t r = 0;; ++r) {
    int active = 0;
    for (int s = 0; s < S; ++s) active += !done[s];
    if (!active) break;
    if (k > 0) {
      for (int j = 0; j < k; ++j) {
        int rps = j == 0 ? 2 : 1, M = S * rps;
        for (int s = 0; s < S; ++s)
          for (int e = 0; e < rps; ++e) {
            int m = s * rps + e;
            seqv[m] = s;
            if (j == 0) { posv[m] = L[s] - 2 + e; tok[m] = hist[(size_t)s * hist_len + L[s] - 2 + e]; }
            else { posv[m] = L[s] - 1 + j; tok[m] = dtok[s * k + j - 1]; }
          }
        /* draft logits for step j land in qlg[s][j] */
        float* stepl = (float*)malloc((size_t)S * V * 4);
        orc_forward(dr, kvd, M, rps, tok, seqv, posv, 1, stepl, V);
        for (int s = 0; s < S; ++s) {
          memcpy(qlg + ((size_t)s * k + j) * V, stepl + (size_t)s * V, (size_t)V * 4);
          dtok[s * k + j] = orc_sample(stepl + (size_t)s * V, V, w, orc_uniform(seed, r, (uint32_t)s, (uint32_t)j, 1));
        }
        free(stepl);
      }
    }
    int R = k + 1, M = S * R;
    for (int s = 0; s < S; ++s)
      for (int e = 0; e < R; ++e) {
        int m = s * R + e;
        seqv[m] = s; posv[m] = L[s] - 1 + e;
        tok[m] = e == 0 ? hist[(size_t)s * hist_len + L[s] - 1] : dtok[s * k + e - 1];
      }
    orc_forward(tg, kvt, M, R, tok, seqv, posv, 0, lg, V);
    if (greedy)
      for (int m = 0; m < M; ++m) { double mg = top2_margin(lg + (size_t)m * V, V); if (!done[m / R] && mg < mmin) mmin = mg; }
    orc_spec_accept(lg, qlg, dtok, S, k, V, w, seed, r, otok, on);
    stats[0]++;
    for (int s = 0; s < S; ++s) {
      if (done[s]) continue;
      int n = on[s];
      for (int i = 0; i <= n; ++i) hist[(size_t)s * hist_len + L[s] + i] = otok[s * (k + 1) + i];
      /* committed token i was decided by verify row i of this sequence */
      if (greedy && tok_margin)
        for (int i = 0; i <= n; ++i) {
          int idx = L[s] - plen[s] + i;
          if (idx < max_new) tok_margin[(size_t)s * max_new + idx] = top2_margin(lg + (size_t)(s * R + i) * V, V);
        }
      L[s] += n + 1;
      stats[1] += (uint64_t)k; stats[2] += (uint64_t)n; stats[3] += (uint64_t)(n + 1);
      if (L[s] - plen[s] >= max_new) done[s] = 1;
    }
  }
  for (int s = 0; s < S; ++s) {
    int c = L[s] - plen[s];
    if (c > max_new) c = max_new;
    out_counts[s] = c;
    for (int i = 0; i < max_new; ++i) out_tokens[(size_t)s * max_new + i] = i < c ? hist[(size_t)s * hist_len + plen[s] + i] : -1;
  }
  if (margin_min) *margin_min = mmin;
  orc_kv_free(kvt); orc_kv_free(kvd);
  free(hist); free(L); free(done); free(lg); free(qlg); free(tok); free(seqv); free(posv); free(dtok); free(otok); free(on);
  return 0;
}

/*
 * CPU baseline sample: `rounds` speculative rounds of one sequence (the device schedule)
 * starting at committed length ctx_len + 1, with both KV caches pre-filled with N(0,1)
 * fp16 values instead of a prefill (cache contents do not change the work done).
 * Returns tokens committed; stats as orc_spec_generate.
 */
int orc_bench_rounds(orc_model* tg, orc_model* dr, int ctx_len, int k, int rounds, const orc_warp* w,
                     uint64_t seed, uint64_t stats[4]) {
  if (!dr) k = 0;
  const int V = tg->d.n_vocab;
  const int cap = ctx_len + rounds * (k + 1) + 2 * k + 4;
  orc_kv* kvt = orc_kv_alloc(tg, 1, cap);
  orc_kv* kvd = dr ? orc_kv_alloc(dr, 1, cap) : NULL;
  if (!kvt || (dr && !kvd)) { orc_kv_free(kvt); orc_kv_free(kvd); return -2; }
  orc_kv* kvs[2] = {kvt, kvd};
  for (int c = 0; c < 2; ++c) {
    orc_kv* kv = kvs[c];
    if (!kv) continue;
    size_t n = (size_t)kv->n_layer * kv->n_seq * kv->Hkv * kv->cap * kv->hd;
    for (size_t i = 0; i < n; ++i) {
      uint32_t o[4];
      orc_philox((uint32_t)i, (uint32_t)(i >> 32), (uint32_t)c, 0xB3u, (uint32_t)seed, 7u, o);
      float u1 = ((float)(o[0] >> 8) + 1.0f) * (1.0f / 16777216.0f), u2 = (float)(o[1] >> 8) * (1.0f / 16777216.0f);
      float z = sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2);
      kv->k[i] = f2h(z);
      kv->v[i] = f2h(-z);
    }
  }
  int32_t* hist = (int32_t*)calloc((size_t)cap + 8, 4);
  for (int i = 0; i <= ctx_len; ++i) hist[i] = (int32_t)(orc_uniform(seed, 0, 0, (uint32_t)i, 9) * (float)V);
  int L = ctx_len + 1;
  float* lg = (float*)malloc((size_t)(k + 1) * V * 4);
  float* qlg = (float*)malloc((size_t)(k > 0 ? k : 1) * V * 4);
  float* stepl = (float*)malloc((size_t)V * 4);
  int32_t tok[32], seqv[32], posv[32], dtok[32], otok[32], on[1];
  memset(stats, 0, 4 * sizeof(uint64_t));
  int committed = 0;
  for (int r = 0; r < rounds; ++r) {
    for (int j = 0; j < k; ++j) {
      int rps = j == 0 ? 2 : 1;
      for (int e = 0; e < rps; ++e) {
        seqv[e] = 0;
        if (j == 0) { posv[e] = L - 2 + e; tok[e] = hist[L - 2 + e]; }
        else { posv[e] = L - 1 + j; tok[e] = dtok[j - 1]; }
      }
      orc_forward(dr, kvd, rps, rps, tok, seqv, posv, 1, stepl, V);
      memcpy(qlg + (size_t)j * V, stepl, (size_t)V * 4);
      dtok[j] = orc_sample(stepl, V, w, orc_uniform(seed, (uint32_t)r, 0, (uint32_t)j, 1));
    }
    for (int e = 0; e <= k; ++e) { seqv[e] = 0; posv[e] = L - 1 + e; tok[e] = e == 0 ? hist[L - 1] : dtok[e - 1]; }
    orc_forward(tg, kvt, k + 1, k + 1, tok, seqv, posv, 0, lg, V);
    orc_spec_accept(lg, qlg, dtok, 1, k, V, w, seed, (uint32_t)r, otok, on);
    for (int i = 0; i <= on[0]; ++i) hist[L + i] = otok[i];
    L += on[0] + 1;
    committed += on[0] + 1;
    stats[0]++; stats[1] += (uint64_t)k; stats[2] += (uint64_t)on[0]; stats[3] += (uint64_t)(on[0] + 1);
  }
  free(hist); free(lg); free(qlg); free(stepl);
  orc_kv_free(kvt); orc_kv_free(kvd);
  return committed;
}
