/*
 * ulb_common.h — definitions shared by host C++ and sm_100a device code.
 *
 *  - Philox4x32-10 counter-based RNG (Salmon, Moraes, Dror, Shaw, "Parallel Random
 *    Numbers: As Easy as 1, 2, 3", SC'11).  One definition compiled for host and device
 *    makes the speculative sampler's uniforms identical on both sides by construction.
 *  - IEEE binary16 <-> binary32 conversion (round-to-nearest-even), matching the
 *    semantics of the reference's half_to_float (src/inference/inference_engine.cpp:15-37).
 *  - The counter layout used by the speculative loop for every uniform it draws.
 *  - The exponential of the sampler's logit weights (ulb_warp_exp).
 */
#ifndef ULB_COMMON_H
#define ULB_COMMON_H

#include <stdint.h>

#if defined(__CUDACC__)
#define ULB_HD __host__ __device__ __forceinline__
#else
#define ULB_HD static inline
#endif

/* ---------------------------------------------------------------- Philox4x32-10 */
typedef struct { uint32_t v[4]; } ulb_u32x4;

ULB_HD ulb_u32x4 ulb_philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                   uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)M0 * c0;
    uint64_t p1 = (uint64_t)M1 * c2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c1 ^ k0;
    uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += W0; k1 += W1;
  }
  ulb_u32x4 o; o.v[0] = c0; o.v[1] = c1; o.v[2] = c2; o.v[3] = c3;
  return o;
}

/* Uniform in [0, 1): the top 24 bits of a 32-bit word, exactly representable in fp32. */
ULB_HD float ulb_u01(uint32_t x) { return (float)(x >> 8) * (1.0f / 16777216.0f); }

/*
 * Uniform streams of the speculative loop.  Key = 64-bit user seed.  Counter words:
 *   c0 = round index (low 32 bits), c1 = sequence id, c2 = slot, c3 = stream tag.
 * Stream tags name what the uniform decides.
 */
enum {
  ULB_RNG_DRAFT = 1,   /* draft token j of a round: slot = j                     */
  ULB_RNG_ACCEPT = 2,  /* accept test of draft slot i: slot = i                  */
  ULB_RNG_RESID = 3,   /* correction / bonus sample: slot = number accepted      */
  ULB_RNG_FIRST = 4,   /* first token after prefill: round = 0, slot = 0         */
};

ULB_HD float ulb_uniform(uint64_t seed, uint32_t round, uint32_t seq, uint32_t slot, uint32_t tag) {
  ulb_u32x4 r = ulb_philox4x32_10(round, seq, slot, tag, (uint32_t)seed, (uint32_t)(seed >> 32));
  return ulb_u01(r.v[0]);
}

/* ---------------------------------------------------------------- warp weights */
#if defined(__CUDA_ARCH__)
#define ULB_FMUL(a, b) __fmul_rn((a), (b))
#define ULB_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#define ULB_RINT(a) rintf(a)
#else
#include <math.h>
#define ULB_FMUL(a, b) ((a) * (b)) /* host builds use -ffp-contract=off */
#define ULB_FMA(a, b, c) fmaf((a), (b), (c))
#define ULB_RINT(a) rintf(a)
#endif

/*
 * exp(x) for the sampler's weights, x = z - max z <= 0, in binary32.  Every step is one
 * IEEE-rounded operation, so host and device give bit-identical weights:
 *   k = rint(x / ln 2); r = x - k ln 2 with ln 2 split in two parts (Cody & Waite, 1980:
 *   C1 = 355/512 has 9 significant bits, so k C1 is exact and x - k C1 has no rounding);
 *   exp(r), |r| <= ln(2)/2, by its Taylor series to degree 7 in Horner form (truncation
 *   below 2^-27 relative); result = exp(r) * 2^k.
 * x < -87 (a weight below 2^-125 of the largest) gives 0.
 */
ULB_HD float ulb_warp_exp(float x) {
  if (!(x >= -87.0f)) return 0.0f;
  const float kf = ULB_RINT(ULB_FMUL(x, 1.44269504088896341f));
  float r = ULB_FMA(kf, -0.693359375f, x);
  r = ULB_FMA(kf, 2.12194440054690583e-4f, r);
  float p = 1.98412698412698413e-4f;   /* 1/7! */
  p = ULB_FMA(p, r, 1.38888888888888889e-3f); /* 1/6! */
  p = ULB_FMA(p, r, 8.33333333333333333e-3f); /* 1/5! */
  p = ULB_FMA(p, r, 4.16666666666666667e-2f); /* 1/4! */
  p = ULB_FMA(p, r, 1.66666666666666667e-1f); /* 1/3! */
  p = ULB_FMA(p, r, 0.5f);
  p = ULB_FMA(p, r, 1.0f);
  p = ULB_FMA(p, r, 1.0f);
  union { uint32_t u; float f; } two_k;
  two_k.u = (uint32_t)((int)kf + 127) << 23; /* k in [-126, 0] */
  return ULB_FMUL(p, two_k.f);
}

/*
 * Top-p masses in fixed point: a warp weight e (a binary32 from ulb_warp_exp, at most 1) as
 * floor(e * 2^40) in 64 bits.  Integer sums do not depend on their order, so the host and the
 * device find the same top-p cut whatever order they add in; a vocabulary of 2^23 weights of
 * at most 2^40 each cannot overflow.  (double)e * 2^40 is exact; the conversion truncates.
 */
ULB_HD uint64_t ulb_mass_fix(float e) { return (uint64_t)((double)e * 1099511627776.0); }
/* the mass the kept set must reach: floor(top_p * total), at least 1 (the largest weight is 2^40) */
ULB_HD uint64_t ulb_topp_target(float top_p, uint64_t total) {
  const uint64_t r = (uint64_t)((double)top_p * (double)total);
  return r < 1 ? 1 : r;
}

/* ---------------------------------------------------------------- binary16 */
ULB_HD float ulb_h2f(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1f;
  uint32_t m = h & 0x3ff;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = s;
    } else { /* subnormal: renormalise */
      int ex = -1;
      do { m <<= 1; ++ex; } while ((m & 0x400) == 0);
      m &= 0x3ff;
      bits = s | ((uint32_t)(127 - 15 - ex) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = s | 0x7f800000u | (m << 13); /* inf / nan (payload kept) */
  } else {
    bits = s | ((e + 112) << 23) | (m << 13);
  }
  union { uint32_t u; float f; } cv; cv.u = bits;
  return cv.f;
}

/* fp32 -> fp16, round to nearest even, overflow to inf, NaN kept quiet. */
ULB_HD uint16_t ulb_f2h(float f) {
  union { float f; uint32_t u; } cv; cv.f = f;
  uint32_t x = cv.u;
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) { /* inf or nan */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
  if (ax < 0x38800000u) {                                   /* result subnormal or zero */
    if (ax < 0x33000000u) return (uint16_t)sign;             /* < 2^-25: rounds to 0 */
    uint32_t e = ax >> 23;
    uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126 - e; /* 14 + (112 - e) + ... : maps 2^-14 boundary */
    /* value = m * 2^(e-150); half subnormal unit = 2^-24 -> q = m * 2^(e-126) */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112;      /* rebias 127 -> 15 */
  uint32_t m = ax & 0x7fffffu;
  uint32_t h = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* carry may bump exponent: correct */
  return (uint16_t)(sign | h);
}

#endif /* ULB_COMMON_H */
