/*
 * qgemv.cu — fused Q4_0 / Q4_K dequant-GEMM for the HBM-bound regime (M <= 64 rows),
 * plus the load-time repack and the bit-exact dequant kernel.
 *
 * Replaces the reference's run_linear_q4k path (src/inference/inference_engine.cpp:532-570:
 * dequantize_q4_k_flattened.glsl materialising an fp32 [N][K] matrix, then the scalar
 * gemm_transposed_b_v2.glsl) and the unused gemm_dequant_q4_0 / gemm_coop_dequant_q4_0
 * shaders (src/shaders/gemm).
 *
 * Design (B200):
 *  - one CTA of 16 warps per SM; the matrix is one stream of 16-row x K-tile tiles in layout
 *    order, split into whole strips per CTA and equal contiguous ranges per warp, so every SM
 *    streams the same bytes to within one strip and every warp one contiguous range;
 *  - each warp loads its tiles with 128-bit L1-bypassing loads straight into a ring of D
 *    tiles of registers (~74 KB in flight per SM); the first D tiles are requested before
 *    griddepcontrol.wait, so the weight stream overlaps the previous kernel (programmatic
 *    dependent launch), and there are no shared-memory staging, mbarriers or waits;
 *  - nibbles become exact fp16 integers with one LOP3 + one HSUB2/HFMA2 per pair
 *    (0x6400 magic) and feed mma.sync.m16n8k16 (weights = A, activations = B, so M <= 8
 *    tokens fill one n-tile); each 32-weight block's scale is applied in fp32 to that
 *    block's integer dot product, so weights are never rounded;
 *  - CTAs take whole strips; a strip split between warps is summed in warp order in shared
 *    memory by the last warp to finish its part, which runs the epilogue; the split depends
 *    on (N, K, SM count) only, so a row's arithmetic never depends on M;
 *  - the fused epilogues write RoPE'd Q / K / V (K and V straight into the fp16 KV cache),
 *    SiLU(gate)*up in fp16, or the fp32 residual add;
 *  - Q8_0 / Q6_K matrices (LM heads of llama.cpp files) stay in GGUF rows and run through
 *    rowgemv_kernel, one warp per output row.
 * The tensor pipe is idle in this regime (<= 3.6 flop/B at M = 1); mma.sync is used as the
 * cheapest-to-issue dot product engine.
 */
#include "epilogue.cuh"

namespace ulb {

namespace {


__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

/* D = A(16x16 f16, row) * B(16x8 f16, col) + C (f32) */
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

/*
 * Word v holds nibbles n0..n7 at bit positions {0,16,4,20,8,24,12,28}.  Produces the four
 * fp16x2 pairs (n0,n1) (n2,n3) (n4,n5) (n6,n7) minus `bias` exactly.
 *   (v & 0x000F000F) | 0x6400_6400 = (1024 + n0, 1024 + n1)
 *   (v & 0x00F000F0) | 0x6400_6400 = (1024 + 16 n2, 1024 + 16 n3) -> x/16 - (64 + bias)
 */
/* (v & MASK) | m in one LOP3: m comes in a register (two immediates would cost two ops) */
template <uint32_t MASK>
__device__ __forceinline__ uint32_t and_or(uint32_t v, uint32_t m) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "n"(MASK), "r"(m));
  return r;
}
/* the fp16 magic 0x6400 (1024.0) twice, in a register the compiler cannot fold */
__device__ __forceinline__ uint32_t magic_1024x2() {
  uint32_t r;
  asm("mov.b32 %0, 0x64006400;" : "=r"(r));
  return r;
}

template <int BIAS>
__device__ __forceinline__ void nib_pairs(uint32_t v, uint32_t& p01, uint32_t& p23, uint32_t& p45,
                                          uint32_t& p67) {
  const uint32_t MAGIC = magic_1024x2();
  /* fp16 of 1024 + BIAS and of -(64 + BIAS), duplicated */
  constexpr uint32_t SUB = BIAS == 8 ? 0x64086408u : 0x64006400u;
  constexpr uint32_t NEG = BIAS == 8 ? 0xD480D480u : 0xD400D400u;
  constexpr uint32_t SIXTEENTH = 0x2C002C00u;
  uint32_t v8 = v >> 8;
  p01 = hsub2u(and_or<0x000F000Fu>(v, MAGIC), SUB);
  p23 = hfma2u(and_or<0x00F000F0u>(v, MAGIC), SIXTEENTH, NEG);
  p45 = hsub2u(and_or<0x000F000Fu>(v8, MAGIC), SUB);
  p67 = hfma2u(and_or<0x00F000F0u>(v8, MAGIC), SIXTEENTH, NEG);
}

/*
 * Activation rows of the lane: xr[nt] = x row (nt*8 + g) + 8t, or a zero row for padding
 * tokens >= M, so every B-fragment fetch is one unpredicated 128-bit load at an offset.
 */
template <int NT>
__device__ __forceinline__ void activation_rows(const __half* __restrict__ x, const __half* __restrict__ xzero, int ldx,
                                                int M, int g, int t, const __half* (&xr)[NT]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n = nt * 8 + g;
    xr[nt] = (n < M ? x + (size_t)n * ldx : xzero) + t * 8;
  }
}

/*
 * One 16-byte activation fragment.  XS: x is this CTA's normalised copy in shared memory
 * (padding rows still point at the global zero row), so the load is generic; otherwise x is
 * global and read-only for the kernel's lifetime.
 */
template <bool XS>
__device__ __forceinline__ uint4 xld(const __half* p) {
  if (XS) return *reinterpret_cast<const uint4*>(p);
  return __ldg(reinterpret_cast<const uint4*>(p));
}

/* column sums of one n-tile of activation fragments over a 32-weight block (an all-ones A) */
__device__ __forceinline__ void block_colsum(const uint4& bx, float (&s)[4]) {
  const uint32_t ONES = 0x3C003C00u;
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  float tmp[4];
  mma16816(tmp, ONES, ONES, ONES, ONES, bx.x, bx.y, zero);
  mma16816(s, ONES, ONES, ONES, ONES, bx.z, bx.w, tmp);
}

/* Q4_K 6-bit (scale, min) of sub-block J from the 12 packed bytes (3 little-endian words). */
template <int J>
__device__ __forceinline__ void q4k_sm(uint32_t w0, uint32_t w1, uint32_t w2, float& sc, float& mn) {
  uint32_t s, m;
  if constexpr (J < 4) {
    s = (w0 >> (8 * J)) & 63u;
    m = (w1 >> (8 * J)) & 63u;
  } else {
    s = ((w2 >> (8 * (J - 4))) & 0x0Fu) | (((w0 >> (8 * (J - 4) + 6)) & 3u) << 4);
    m = ((w2 >> (8 * (J - 4) + 4)) & 0x0Fu) | (((w1 >> (8 * (J - 4) + 6)) & 3u) << 4);
  }
  sc = (float)s;
  mn = (float)m;
}

/* ------------------------------------------------------------------ epilogues */
/* lane (g, t) holds, for n-tile nt, rows (g, g + 8) of tokens nt*8 + 2t and + 1; pre: those
   tokens' cache rows when read ahead (QKV), else NULL */
template <int EPI>
__device__ __forceinline__ void epilogue(const EpiArgs& e, int strip, int nt, int g, int t, int M,
                                         int N, const float4& v, const EpiRow* pre) {
  epilogue_pair<EPI>(e, strip, g, nt * 8 + 2 * t, M, N, v, pre);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

/* 128-bit weight load: read once, so it neither allocates in L1 (kept for the activations)
   nor waits for the previous kernel (weights are constant) */
__device__ __forceinline__ uint4 ldw(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

/*
 * A tile's weight operands in registers, straight from global memory.
 *   Q4_0: 2 x 16 B of nibble words + 16 B of scales (rows g, g + 8) per lane.
 *   Q4_K: 4 x 16 B of nibble words + the 16 B meta rows of g and g + 8.
 */
template <int QT> struct WTile;
/* load(): pw = the tile + lane * 16 (the lane's nibble words), ps = the tile + MO + g * 16 (its
   scale / meta row); both advance by TB from tile to tile */
template <> struct WTile<ULB_TYPE_Q4_0> {
  static constexpr int TB = kQ40TileBytes, TK = kQ40TileK, MO = 1024;
  uint4 w[2], sc;
  __device__ __forceinline__ void load(const uint8_t* pw, const uint8_t* ps) {
    w[0] = ldw(pw);
    w[1] = ldw(pw + 512);
    sc = ldw(ps);
  }
};
template <> struct WTile<ULB_TYPE_Q4_K> {
  static constexpr int TB = kQ4KTileBytes, TK = kQ4KTileK, MO = 2048;
  uint4 w[4], mg, mg8;
  __device__ __forceinline__ void load(const uint8_t* pw, const uint8_t* ps) {
#pragma unroll
    for (int p = 0; p < 4; ++p) w[p] = ldw(pw + p * 512);
    mg = ldw(ps);
    mg8 = ldw(ps + 8 * 16);
  }
};

/* the exact fp16 integer weights of one 32-weight block, rows g (w[0..3]) and g + 8 (w[4..7]) */
template <int BIAS>
__device__ __forceinline__ void block_weights(uint32_t vg, uint32_t vg8, uint32_t (&w)[8]) {
  nib_pairs<BIAS>(vg, w[0], w[1], w[2], w[3]);
  nib_pairs<BIAS>(vg8, w[4], w[5], w[6], w[7]);
}
/* integer dot products of one block with one n-tile of activation fragments */
__device__ __forceinline__ void block_dot(const uint32_t (&w)[8], const uint4& bx, float (&s)[4]) {
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  float tmp[4];
  mma16816(tmp, w[0], w[4], w[1], w[5], bx.x, bx.y, zero);
  mma16816(s, w[2], w[6], w[3], w[7], bx.z, bx.w, tmp);
}

constexpr int kGW = 16; /* warps per CTA (one CTA per SM) */

/* GEMV configuration per weight type and n-tile count:
     W    warps per CTA (one CTA per SM; the split of the weight stream depends on it, so it is
          the same for every NT of a weight type)
     D    weight tiles in flight per warp (the register ring) */
template <int QT, int NT> struct GemvCfg {
  static constexpr int W = kGW;
  static constexpr int D = QT == ULB_TYPE_Q4_0 ? (NT == 4 ? 2 : 4) : (NT == 4 ? 1 : 2);
};

/* one Q4_0 tile: xp[nt] points at the tile's first activation of n-tile nt (this lane's row) */
template <bool XS, int NT>
__device__ __forceinline__ void tile_compute(const WTile<ULB_TYPE_Q4_0>& r, const __half* const (&xp)[NT],
                                             float (&acc)[NT][4]) {
  const uint32_t words[8] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w, r.w[1].x, r.w[1].y, r.w[1].z, r.w[1].w};
  const uint32_t scw[4] = {r.sc.x, r.sc.y, r.sc.z, r.sc.w};
  /* block b's activation fragments are loaded one block ahead (NT <= 2) or just before use
     (NT = 4, for the registers) */
  constexpr int LA = NT <= 2 ? 1 : 0;
  uint4 xl[2][NT];
  if (LA) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) xl[0][nt] = xld<XS>(xp[nt]);
  }
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    if (b + LA < 4) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xl[(b + LA) & 1][nt] = xld<XS>(xp[nt] + (b + LA) * 32);
    }
    uint32_t wq[8];
    block_weights<8>(words[2 * b], words[2 * b + 1], wq);
    float2 dd; /* the block scales of rows g and g + 8 */
    asm("{.reg .b16 l, h; mov.b32 {l, h}, %2; cvt.f32.f16 %0, l; cvt.f32.f16 %1, h;}"
        : "=f"(dd.x), "=f"(dd.y)
        : "r"(scw[b]));
    /* one n-tile at a time: the scaled block sum goes into acc before the next n-tile's MMA */
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float s[4];
      block_dot(wq, xl[b & 1][nt], s);
      acc[nt][0] = __fmaf_rn(dd.x, s[0], acc[nt][0]);
      acc[nt][1] = __fmaf_rn(dd.x, s[1], acc[nt][1]);
      acc[nt][2] = __fmaf_rn(dd.y, s[2], acc[nt][2]);
      acc[nt][3] = __fmaf_rn(dd.y, s[3], acc[nt][3]);
    }
  }
}

template <bool XS, int NT>
__device__ __forceinline__ void tile_compute(const WTile<ULB_TYPE_Q4_K>& r, const __half* const (&xp)[NT],
                                             float (&acc)[NT][4]) {
  const uint4(&nb)[4] = r.w;
  const uint4 mg = r.mg, mg8 = r.mg8;
  const float2 dg = __half22float2(*reinterpret_cast<const __half2*>(&mg.x));   /* (d, dmin) row g */
  const float2 dg8 = __half22float2(*reinterpret_cast<const __half2*>(&mg8.x)); /* row g + 8 */
  float t1[NT][4], t0[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) t1[nt][i] = t0[nt][i] = 0.f;
#define ULB_Q4K_SUB(J)                                                                   \
  {                                                                                      \
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(&nb[(J) >> 1]);              \
    uint32_t wq[8];                                                                      \
    block_weights<0>(wp[((J) & 1) * 2], wp[((J) & 1) * 2 + 1], wq);                     \
    float scg, mng, scg8, mng8;                                                          \
    q4k_sm<J>(mg.y, mg.z, mg.w, scg, mng);                                               \
    q4k_sm<J>(mg8.y, mg8.z, mg8.w, scg8, mng8);                                          \
    _Pragma("unroll") for (int nt = 0; nt < NT; ++nt) {                                  \
      const uint4 bx = xld<XS>(xp[nt] + (J) * 32);                                       \
      float s1[4], s0[4];                                                                \
      block_dot(wq, bx, s1);                                                             \
      block_colsum(bx, s0);                                                              \
      t1[nt][0] = __fmaf_rn(scg, s1[0], t1[nt][0]);                                      \
      t1[nt][1] = __fmaf_rn(scg, s1[1], t1[nt][1]);                                      \
      t1[nt][2] = __fmaf_rn(scg8, s1[2], t1[nt][2]);                                     \
      t1[nt][3] = __fmaf_rn(scg8, s1[3], t1[nt][3]);                                     \
      t0[nt][0] = __fmaf_rn(mng, s0[0], t0[nt][0]);                                      \
      t0[nt][1] = __fmaf_rn(mng, s0[1], t0[nt][1]);                                      \
      t0[nt][2] = __fmaf_rn(mng8, s0[2], t0[nt][2]);                                     \
      t0[nt][3] = __fmaf_rn(mng8, s0[3], t0[nt][3]);                                     \
    }                                                                                    \
  }
  ULB_Q4K_SUB(0) ULB_Q4K_SUB(1) ULB_Q4K_SUB(2) ULB_Q4K_SUB(3)
  ULB_Q4K_SUB(4) ULB_Q4K_SUB(5) ULB_Q4K_SUB(6) ULB_Q4K_SUB(7)
#undef ULB_Q4K_SUB
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    acc[nt][0] = __fmaf_rn(-dg.y, t0[nt][0], __fmaf_rn(dg.x, t1[nt][0], acc[nt][0]));
    acc[nt][1] = __fmaf_rn(-dg.y, t0[nt][1], __fmaf_rn(dg.x, t1[nt][1], acc[nt][1]));
    acc[nt][2] = __fmaf_rn(-dg8.y, t0[nt][2], __fmaf_rn(dg8.x, t1[nt][2], acc[nt][2]));
    acc[nt][3] = __fmaf_rn(-dg8.y, t0[nt][3], __fmaf_rn(dg8.x, t1[nt][3], acc[nt][3]));
  }
}

/*
 * Split of the weight stream.  The matrix is one stream of n_strips * tiles tiles in layout
 * order (strip-major).  CTA c of G takes the whole strips [c*S/G, (c+1)*S/G) (S = n_strips),
 * and warp w of its Wn working warps an equal contiguous share of that CTA's tiles, so every
 * warp streams one contiguous byte range and no strip is split between CTAs: a CTA streams
 * at most one strip (16 rows x K) more than the average, less than the latency of a cross-CTA
 * reduction it saves.  A strip split between warps is summed in warp order in shared memory.
 * The split depends on (N, K, G) only, never on M, so a row's arithmetic does not depend on
 * what else is batched.  All quantities fit 32 bits.
 */
struct Split {
  uint32_t S;     /* strips in the matrix */
  uint32_t G;     /* CTAs (<= S) */
  uint32_t Wn;    /* working warps per CTA (<= W, <= the tiles of a CTA) */
  uint32_t tiles; /* tiles per strip */
};
/* first tile of CTA c (c = G gives the end of the matrix) */
__device__ __forceinline__ uint32_t cta_begin(const Split& s, uint32_t c) { return c * s.S / s.G * s.tiles; }
/* first tile of warp w of a CTA starting at c0 with tc tiles; the warp holding local tile l */
__device__ __forceinline__ uint32_t warp_begin(uint32_t c0, uint32_t tc, uint32_t Wn, uint32_t w) {
  return c0 + w * tc / Wn;
}
__device__ __forceinline__ uint32_t warp_in_cta(uint32_t tc, uint32_t Wn, uint32_t l) { return ((l + 1) * Wn - 1) / tc; }



/* RMSNorm fused into the GEMV: the fp32 rows, the norm weights and eps */
struct NormIn {
  const float* x = nullptr;
  int ldx = 0;
  const float* g = nullptr;
  float eps = 0.f;
};

/* bytes of the per-warp strip partials in shared memory: W warps x {first, last strip} */
template <int QT, int NT> constexpr size_t warp_part_bytes() {
  return (size_t)GemvCfg<QT, NT>::W * 2 * NT * 32 * sizeof(float4);
}

/* one GEMV of a launch: y (by its epilogue) = W . activations */
struct GemvStep {
  const uint8_t* w = nullptr; /* packed strips */
  Split sp{};
  int N = 0, M = 0;
  const __half* x = nullptr; /* activations [M][ldx] fp16, unless nin.x: rmsnorm(nin.x) */
  int ldx = 0;
  NormIn nin;
  EpiArgs ea;
};

/* shared-memory layout of a GEMV CTA: warp partials | normalised activations (fp16 [M][K]) */
template <int QT, int NT> __device__ __forceinline__ __half* smem_x(uint8_t* smem) {
  return reinterpret_cast<__half*>(smem + warp_part_bytes<QT, NT>());
}

/*
 * xs[m] = fp16((x[m] * r_m) * g), r_m = 1 / sqrt(sum(x[m]^2) / d + eps) for rows m < M of x
 * (fp32, row stride ldx, read through L2), by all warps of the CTA at once, with exactly the
 * arithmetic of rms_row_256 (rmsnorm_kernel): row m's sum is eight virtual 256-thread blocks'
 * per-thread fmaf chains over float4 j = i*256 + vt, a warp xor tree, and the eight virtual
 * warps in order.  Real warp w takes virtual warps w, w + NW, ... of the M * 8.
 */
constexpr int kNormMaxRows = 8; /* rows a GEMV normalises itself (one n-tile) */
template <int NW>
__device__ __forceinline__ void norm_rows(const float* __restrict__ x, int ldx, const float* __restrict__ gw, int d,
                                          float eps, int M, __half* xs, float* red /* [8 * 8 + 8] */) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n4 = d >> 2;
  for (int vwi = warp; vwi < M * 8; vwi += NW) {
    const int m = vwi >> 3, vt = (vwi & 7) * 32 + lane;
    const float4* xv = reinterpret_cast<const float4*>(x + (size_t)m * ldx);
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = i * 256 + vt;
      if (j < n4) v[i] = __ldcg(xv + j);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = i * 256 + vt;
      if (j < n4) {
        ss = __fmaf_rn(v[i].x, v[i].x, ss);
        ss = __fmaf_rn(v[i].y, v[i].y, ss);
        ss = __fmaf_rn(v[i].z, v[i].z, ss);
        ss = __fmaf_rn(v[i].w, v[i].w, ss);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[vwi] = ss;
  }
  __syncthreads();
  if (threadIdx.x < M) { /* the row scales, over red[64 + m] */
    const int m = threadIdx.x;
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[m * 8 + w];
    red[64 + m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)d), eps)));
  }
  __syncthreads();
  /* a thread takes float4 column j of every row at once (one memory round trip per column
     it owns, the norm weights loaded once for all rows) */
  const float4* gv = reinterpret_cast<const float4*>(gw);
  for (int j = threadIdx.x; j < n4; j += NW * 32) {
    const float4 gg = __ldg(gv + j);
    float4 v[kNormMaxRows];
#pragma unroll
    for (int m = 0; m < kNormMaxRows; ++m)
      if (m < M) v[m] = __ldcg(reinterpret_cast<const float4*>(x + (size_t)m * ldx) + j);
#pragma unroll
    for (int m = 0; m < kNormMaxRows; ++m)
      if (m < M) {
        const float r = red[64 + m];
        __half2* o2 = reinterpret_cast<__half2*>(xs + (size_t)m * d) + 2 * j;
        o2[0] = __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(v[m].x, r), gg.x)),
                               __float2half_rn(__fmul_rn(__fmul_rn(v[m].y, r), gg.y)));
        o2[1] = __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(v[m].z, r), gg.z)),
                               __float2half_rn(__fmul_rn(__fmul_rn(v[m].w, r), gg.w)));
      }
  }
  __syncthreads();
}

/* where a step's activation rows are: fp16 [M][ldx] */
struct XIn {
  const __half* x;
  int ldx;
};

/* the normalised activations of a step (its nin rows), in shared memory: fp16 [M][K] */
template <int QT, int NT>
__device__ __forceinline__ XIn prep_norm(const GemvStep& S, uint8_t* smem, float* red) {
  const int K = (int)S.sp.tiles * WTile<QT>::TK;
  __half* xs = smem_x<QT, NT>(smem);
  norm_rows<GemvCfg<QT, NT>::W>(S.nin.x, S.nin.ldx, S.nin.g, K, S.nin.eps, S.M, xs, red);
  return XIn{xs, K};
}

/*
 * Warp-streamed fused dequant-GEMV body, run by a CTA of 16 warps (one per SM).  Each working
 * warp streams its own contiguous range of tiles with 128-bit loads straight into a ring of D
 * tiles of registers: the first D tiles (all of a small matrix) are requested before `sync`
 * (griddepcontrol.wait, or the wait of a grid barrier), so the weight stream overlaps what
 * came before, and a tile's registers are refilled with tile j + D as soon as tile j is
 * computed.  No warp ever waits for another while streaming.
 * A strip finished inside one warp goes straight to the epilogue.  A strip split between warps
 * leaves each warp's partial in shared memory (slot 0: the warp's first strip, 1: its last);
 * the last of the CTA's warps to count itself in wcnt[first warp] sums them in warp order and
 * runs the epilogue.
 * sync(): every thread calls it once; false = abandon the step.  prep(): every thread; returns
 * the activation rows and ends with a CTA barrier.  XS: the rows are read with generic loads
 * (shared memory, or global memory written earlier in the same launch); otherwise with
 * read-only loads.
 */
template <int QT, int NT, int EPI, bool XS, class Sync, class Prep>
__device__ __forceinline__ void gemv_body(const GemvStep& S, uint8_t* smem, uint32_t* wcnt,
                                          const __half* __restrict__ xzero, Sync sync, Prep prep) {
  constexpr int TB = WTile<QT>::TB, D = GemvCfg<QT, NT>::D, W = GemvCfg<QT, NT>::W;
  const Split sp = S.sp;
  const int M = S.M, N = S.N;
  const EpiArgs& ea = S.ea;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t c = blockIdx.x;
  const uint32_t c0 = cta_begin(sp, c), c1 = cta_begin(sp, c + 1), tc = c1 - c0;
  uint32_t a = 0, b = 0;
  if ((uint32_t)warp < sp.Wn) {
    a = warp_begin(c0, tc, sp.Wn, warp);
    b = warp_begin(c0, tc, sp.Wn, warp + 1);
  }
  const int n = (int)(b - a);
  const uint8_t* src = S.w + (size_t)a * TB;
  float4* wpart = reinterpret_cast<float4*>(smem);
  /* the weights do not depend on what came before: start streaming before the wait */
  WTile<QT> ring[D];
#pragma unroll
  for (int i = 0; i < D; ++i)
    if (i < n) ring[i].load(src + (size_t)i * TB + lane * 16, src + (size_t)i * TB + WTile<QT>::MO + g * 16);
  /* QKV with one n-tile: the lane's two tokens' cache rows are read now, before the wait (see
     EpiRow), so the epilogue pays one table lookup instead of a chain of them */
  constexpr bool kPreRows = EPI == EPI_QKV && NT == 1;
  EpiRow pre[NT][2];
  if (kPreRows) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int tok = nt * 8 + 2 * t + i;
        pre[nt][i] = tok < M ? epi_row(ea, tok) : EpiRow{-1, 0, 0};
      }
  }
  if (tid < W) wcnt[tid] = 0;
  if (!sync()) return;
  const XIn xin = prep();
  ULB_TRACE_MARK(0);
  if (n == 0) return;
  const __half* xr[NT];
  /* tokens >= M only feed MMA columns the epilogue drops: in shared memory they may read row 0 */
  activation_rows<NT>(xin.x, XS ? xin.x : xzero, xin.ldx, M, g, t, xr);
  const uint32_t tiles = sp.tiles;
  const uint32_t first_strip = a / tiles;
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  /* the warp's part of strip s is in acc */
  auto flush = [&](uint32_t s) {
    const uint32_t s0 = s * tiles, s1 = s0 + tiles;
    float4 v[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) v[nt] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    if (s0 < a || s1 > b) {
      /* the warps of this CTA holding part of s, in warp order (strips never cross CTAs) */
      const uint32_t wa = warp_in_cta(tc, sp.Wn, s0 - c0), wb = warp_in_cta(tc, sp.Wn, s1 - 1 - c0);
      {
        float4* mine = wpart + ((size_t)(warp * 2 + (s == first_strip ? 0 : 1)) * NT) * 32 + lane;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mine[nt * 32] = v[nt];
        __syncwarp();
        uint32_t prev = 0;
        if (lane == 0)
          asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                       : "=r"(prev)
                       : "r"(smem_u32(&wcnt[wa]))
                       : "memory");
        if (__shfl_sync(0xffffffffu, prev, 0) != wb - wa) return;
        __syncwarp();
        if (lane == 0) wcnt[wa] = 0;
        /* warp wa holds s as its first strip iff it starts at or after s0; later warps start
           inside s */
        const int sa = warp_begin(c0, tc, sp.Wn, wa) >= s0 ? 0 : 1;
        for (uint32_t ww = wa; ww <= wb; ++ww) {
          const float4* q = wpart + ((size_t)(ww * 2 + (ww == wa ? sa : 0)) * NT) * 32 + lane;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float4 o = q[nt * 32];
            if (ww == wa) {
              v[nt] = o;
            } else {
              v[nt].x += o.x; v[nt].y += o.y; v[nt].z += o.z; v[nt].w += o.w;
            }
          }
        }
      }
    }
    ULB_TRACE_MARK_MAX(2);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) epilogue<EPI>(ea, (int)s, nt, g, t, M, N, v[nt], kPreRows ? pre[nt] : nullptr);
    ULB_TRACE_MARK_MAX(3);
  };

  uint32_t s = first_strip;
  uint32_t kt = a - first_strip * tiles;
  constexpr int TK = WTile<QT>::TK;
  const __half* xp[NT]; /* activations of the current tile */
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) xp[nt] = xr[nt] + kt * TK;
  /* the lane's addresses in the refill of the tile being computed */
  const uint8_t* wp = src + (size_t)D * TB + lane * 16;
  const uint8_t* wps = src + (size_t)D * TB + WTile<QT>::MO + g * 16;
  /* after tile j: refill its ring slot with tile j + D, step the activations, finish the strip */
#define ULB_GEMV_NEXT(u, j)                                                                  \
  {                                                                                          \
    if ((j) + D < n) ring[u].load(wp, wps);                                                  \
    wp += TB;                                                                                \
    wps += TB;                                                                               \
    if (++kt == tiles) {                                                                     \
      flush(s);                                                                              \
      _Pragma("unroll") for (int nt = 0; nt < NT; ++nt) {                                    \
        acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;                             \
        xp[nt] = xr[nt];                                                                     \
      }                                                                                      \
      ++s;                                                                                   \
      kt = 0;                                                                                \
    } else {                                                                                 \
      _Pragma("unroll") for (int nt = 0; nt < NT; ++nt) xp[nt] += TK;                        \
    }                                                                                        \
  }
  int j = 0;
  for (; j + D <= n; j += D) { /* full groups: tile j + u is in ring slot u */
#pragma unroll
    for (int u = 0; u < D; ++u) {
      tile_compute<XS, NT>(ring[u], xp, acc);
      ULB_GEMV_NEXT(u, j + u)
    }
  }
#pragma unroll
  for (int u = 0; u < D - 1; ++u) /* the last n % D tiles */
    if (j + u < n) {
      tile_compute<XS, NT>(ring[u], xp, acc);
      ULB_GEMV_NEXT(u, j + u)
    }
#undef ULB_GEMV_NEXT
  ULB_TRACE_MARK(1);
  ULB_TRACE_MARK_MAX(4);
  if (kt != 0) flush(s); /* the range ends inside strip s */
}


/* one GEMV per launch: XS, the activation rows normalised from the step's nin rows into
   shared memory; otherwise read from global memory through L1 */
template <int QT, int NT, int EPI, bool XS>
__global__ void __launch_bounds__(GemvCfg<QT, NT>::W * 32, 1)
    qgemv_kernel(GemvStep S, const __half* __restrict__ xzero) {
  ULB_TRACE_KERNEL(kTrGemv + EPI * 100 + NT * 10 + (XS ? 1 : 0), S.N);
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t wcnt[GemvCfg<QT, NT>::W];
  __shared__ float red[72];
  gemv_body<QT, NT, EPI, XS>(
      S, smem, wcnt, xzero,
      [] {
        pdl_wait();
        pdl_trigger();
        return true;
      },
      [&]() -> XIn {
        if (XS) return prep_norm<QT, NT>(S, smem, red);
        __syncthreads();
        return XIn{S.x, S.ldx};
      });
}

/* ------------------------------------------------------------------ GGUF-row GEMV (Q8_0 / Q6_K heads) */
/*
 * y[m][n] = W[n] . x16[m] for a matrix kept as GGUF rows (Q8_0: fp16 d + 32 int8 per block;
 * Q6_K: 256-weight super-blocks, weight = (d * sc_j) * (q - 32), sc_j per 16 weights), used for
 * the output.weight llama.cpp's Q4_0 / Q4_K_M files store in these types.  One warp per row,
 * M <= 8 tokens.  Q8_0: lane L takes blocks L, L + 32, ...; Q6_K: in each super-block lane L
 * takes weights 8L..8L+7 (half of sub-block L / 2: eight ql bytes, eight qh bytes).  Each
 * lane sums its integer dot products in fp32 and applies the block step with one fmaf; the
 * lanes' sums meet in a warp xor tree.
 */
template <int QT, int EPI>
__global__ void __launch_bounds__(256) rowgemv_kernel(const uint8_t* __restrict__ w, int N, int K,
                                                      const __half* __restrict__ x, int ldx, int M, EpiArgs e) {
  ULB_TRACE_KERNEL(kTrRowGemv + EPI, N);
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (n >= N) return;
  float acc[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) acc[m] = 0.f;
  auto xdot8 = [&](const int8_t (&q)[8], int k0, float step) {
#pragma unroll
    for (int m = 0; m < 8; ++m)
      if (m < M) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * ldx + k0));
        const __half* xh = reinterpret_cast<const __half*>(&raw);
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s = __fmaf_rn((float)q[e], __half2float(xh[e]), s);
        acc[m] = __fmaf_rn(step, s, acc[m]);
      }
  };
  if (QT == ULB_TYPE_F16 || QT == ULB_TYPE_F32) {
    /* plain rows: lane L takes weights 8L..8L+7 of every 256, products summed in that order */
    for (int k0 = 8 * lane; k0 < K; k0 += 256) {
      float wv[8];
      if (QT == ULB_TYPE_F16) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(w) + (size_t)n * K + k0));
        const __half* wh = reinterpret_cast<const __half*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) wv[e] = __half2float(wh[e]);
      } else {
        const float4* p4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(w) + (size_t)n * K + k0);
        const float4 a = __ldg(p4), b = __ldg(p4 + 1);
        wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w; wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
      }
#pragma unroll
      for (int m = 0; m < 8; ++m)
        if (m < M) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * ldx + k0));
          const __half* xh = reinterpret_cast<const __half*>(&raw);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[m] = __fmaf_rn(wv[e], __half2float(xh[e]), acc[m]);
        }
    }
  } else if (QT == ULB_TYPE_Q8_0) {
    const uint8_t* row = w + (size_t)n * (K / 32) * 34;
    for (int b = lane; b < K / 32; b += 32) {
      const uint8_t* blk = row + (size_t)b * 34;
      const float d = __half2float(*reinterpret_cast<const __half*>(blk));
      /* the block's integer dot product in weight order (exact products, fp32 sum) */
#pragma unroll
      for (int m = 0; m < 8; ++m)
        if (m < M) {
          float s = 0.f;
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * ldx + b * 32 + 8 * r));
            const __half* xh = reinterpret_cast<const __half*>(&raw);
#pragma unroll
            for (int e = 0; e < 8; ++e) s = __fmaf_rn((float)(int8_t)blk[2 + 8 * r + e], __half2float(xh[e]), s);
          }
          acc[m] = __fmaf_rn(d, s, acc[m]);
        }
    }
  } else {
    const uint8_t* row = w + (size_t)n * (K / 256) * 210;
    const int h = lane / 16, k = (lane % 16) / 4, l0 = (8 * lane) % 32;
    for (int b = 0; b < K / 256; ++b) {
      const uint8_t* blk = row + (size_t)b * 210;
      const uint8_t* ql = blk + 64 * h + l0 + 32 * (k & 1);
      const uint8_t* qh = blk + 128 + 32 * h + l0;
      const float step = __fmul_rn(__half2float(*reinterpret_cast<const __half*>(blk + 208)),
                                   (float)(int8_t)blk[192 + lane / 2]);
      int8_t q[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        q[e] = (int8_t)((((ql[e] >> (k >= 2 ? 4 : 0)) & 15) | (((qh[e] >> (2 * k)) & 3) << 4)) - 32);
      xdot8(q, b * 256 + 8 * lane, step);
    }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = acc[m];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && m < M) {
      if (EPI == EPI_VCACHE) {
        store_v_cache(e, m, n / e.hd, n % e.hd, v);
      } else {
        float* p = e.y + (size_t)m * e.ldy + n;
        *p = EPI == EPI_RESID ? __ldcg(p) + v : v;
      }
    }
  }
}

static bool raw_rows_type(int t) {
  return t == ULB_TYPE_Q8_0 || t == ULB_TYPE_Q6_K || t == ULB_TYPE_F16 || t == ULB_TYPE_F32;
}

template <int EPI>
static auto rowgemv_for(int type) {
  return type == ULB_TYPE_Q8_0   ? rowgemv_kernel<ULB_TYPE_Q8_0, EPI>
         : type == ULB_TYPE_Q6_K ? rowgemv_kernel<ULB_TYPE_Q6_K, EPI>
         : type == ULB_TYPE_F16  ? rowgemv_kernel<ULB_TYPE_F16, EPI>
                                 : rowgemv_kernel<ULB_TYPE_F32, EPI>;
}

/* a matrix kept as GGUF rows (Q8_0 / Q6_K / F16 / F32): LM heads, and the attn_v / attn_output /
   ffn_down projections llama.cpp's K-quant mixes store in Q6_K or Q8_0; 8 tokens per launch */
static int launch_rowgemv(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a0) {
  ULB_CHECK(((epi == EPI_STORE || epi == EPI_RESID) && a0.y) || (epi == EPI_VCACHE && a0.vc && a0.row_pos && a0.row_seq),
            ULB_EUNSUPPORTED, "qgemv: a Q8_0 / Q6_K / F16 / F32 matrix takes the store, residual or V-cache epilogue");
  ULB_CHECK(ldx % 8 == 0 && ((uintptr_t)x & 15) == 0, ULB_EINVAL, "qgemv: activations must be 16-byte aligned rows");
  ULB_CHECK(w->K % 8 == 0, ULB_EUNSUPPORTED, "row GEMV: K=%d not a multiple of 8", w->K);
  const dim3 grid((w->N + 7) / 8), block(256);
  for (int m0 = 0; m0 < M; m0 += 8) {
    const int mc = M - m0 < 8 ? M - m0 : 8;
    EpiArgs a = a0;
    if (a.y) a.y += (size_t)m0 * a.ldy;
    if (a.row_seq) a.row_seq += m0;
    if (a.row_pos) a.row_pos += m0;
    cudaError_t e;
    const uint8_t* wd = (const uint8_t*)w->dev;
    const __half* xc = x + (size_t)m0 * ldx;
    if (epi == EPI_STORE) e = launch_k(c, rowgemv_for<EPI_STORE>(w->type), grid, block, 0, wd, w->N, w->K, xc, ldx, mc, a);
    else if (epi == EPI_RESID) e = launch_k(c, rowgemv_for<EPI_RESID>(w->type), grid, block, 0, wd, w->N, w->K, xc, ldx, mc, a);
    else e = launch_k(c, rowgemv_for<EPI_VCACHE>(w->type), grid, block, 0, wd, w->N, w->K, xc, ldx, mc, a);
    if (e != cudaSuccess) return cuda_error(e, "row GEMV launch", __FILE__, __LINE__);
  }
  return ULB_OK;
}

/* ------------------------------------------------------------------ repack / dequant */
__device__ __forceinline__ uint32_t place_nibbles(const uint8_t (&n)[8]) {
  /* nibble i -> bit position {0,16,4,20,8,24,12,28}[i] */
  return (uint32_t)n[0] | ((uint32_t)n[1] << 16) | ((uint32_t)n[2] << 4) | ((uint32_t)n[3] << 20) |
         ((uint32_t)n[4] << 8) | ((uint32_t)n[5] << 24) | ((uint32_t)n[6] << 12) |
         ((uint32_t)n[7] << 28);
}
__device__ __forceinline__ int unplace(uint32_t v, int i) {
  const int pos[8] = {0, 16, 4, 20, 8, 24, 12, 28};
  return (int)((v >> pos[i]) & 15u);
}

/* grid (tiles, strips), block 32 */
__global__ void repack_q40_kernel(const uint8_t* __restrict__ raw, int K, const int* __restrict__ rmap,
                                  uint8_t* __restrict__ out, int tiles) {
  const int tile = blockIdx.x, strip = blockIdx.y, lane = threadIdx.x;
  const int g = lane >> 2, t = lane & 3;
  const size_t row_bytes = (size_t)K / 32 * 18;
  uint8_t* tp = out + ((size_t)strip * tiles + tile) * kQ40TileBytes;
  uint16_t d[2][4];
  for (int b = 0; b < 4; ++b) {
    for (int hr = 0; hr < 2; ++hr) {
      const int raw_row = rmap[strip * 16 + g + 8 * hr];
      uint32_t word = 0;
      uint16_t dd = 0;
      if (raw_row >= 0) {
        const uint8_t* blk = raw + (size_t)raw_row * row_bytes + (size_t)(tile * 4 + b) * 18;
        dd = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
        uint8_t n[8];
        for (int i = 0; i < 8; ++i) {
          const int wi = 8 * t + i;
          n[i] = wi < 16 ? (blk[2 + wi] & 15) : (blk[2 + wi - 16] >> 4);
        }
        word = place_nibbles(n);
      }
      d[hr][b] = dd;
      const int part = b >> 1;
      reinterpret_cast<uint32_t*>(tp + part * 512 + lane * 16)[(b & 1) * 2 + hr] = word;
    }
  }
  if (t == 0) {
    for (int b = 0; b < 4; ++b)
      reinterpret_cast<uint32_t*>(tp + 1024 + g * 16)[b] = (uint32_t)d[0][b] | ((uint32_t)d[1][b] << 16);
  }
}

__global__ void repack_q4k_kernel(const uint8_t* __restrict__ raw, int K, const int* __restrict__ rmap,
                                  uint8_t* __restrict__ out, int tiles) {
  const int tile = blockIdx.x, strip = blockIdx.y, lane = threadIdx.x;
  const int g = lane >> 2, t = lane & 3;
  const size_t row_bytes = (size_t)K / 256 * 144;
  uint8_t* tp = out + ((size_t)strip * tiles + tile) * kQ4KTileBytes;
  for (int j = 0; j < 8; ++j) {
    for (int hr = 0; hr < 2; ++hr) {
      const int raw_row = rmap[strip * 16 + g + 8 * hr];
      uint32_t word = 0;
      if (raw_row >= 0) {
        const uint8_t* qs = raw + (size_t)raw_row * row_bytes + (size_t)tile * 144 + 16;
        uint8_t n[8];
        for (int i = 0; i < 8; ++i) {
          const uint8_t byte = qs[32 * (j >> 1) + 8 * t + i];
          n[i] = (j & 1) ? (byte >> 4) : (byte & 15);
        }
        word = place_nibbles(n);
      }
      reinterpret_cast<uint32_t*>(tp + (j >> 1) * 512 + lane * 16)[(j & 1) * 2 + hr] = word;
    }
  }
  if (lane < 16) {
    const int raw_row = rmap[strip * 16 + lane];
    uint8_t* m = tp + 2048 + lane * 16;
    for (int i = 0; i < 16; ++i)
      m[i] = raw_row >= 0 ? raw[(size_t)raw_row * row_bytes + (size_t)tile * 144 + i] : 0;
  }
}

/* dequant: grid (tiles, strips), block 32; out[row][k] fp32, rows < N only */
__global__ void dequant_q40_kernel(const uint8_t* __restrict__ w, int tiles, int N, int K, float* __restrict__ out) {
  const int tile = blockIdx.x, strip = blockIdx.y, lane = threadIdx.x;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* tp = w + ((size_t)strip * tiles + tile) * kQ40TileBytes;
  for (int b = 0; b < 4; ++b)
    for (int hr = 0; hr < 2; ++hr) {
      const int row = strip * 16 + g + 8 * hr;
      if (row >= N) continue;
      const uint32_t word = reinterpret_cast<const uint32_t*>(tp + (b >> 1) * 512 + lane * 16)[(b & 1) * 2 + hr];
      const uint16_t dh = (uint16_t)(reinterpret_cast<const uint32_t*>(tp + 1024 + g * 16)[b] >> (16 * hr));
      const float d = __half2float(__ushort_as_half(dh));
      for (int i = 0; i < 8; ++i)
        out[(size_t)row * K + tile * 128 + b * 32 + 8 * t + i] = __fmul_rn(d, (float)(unplace(word, i) - 8));
    }
}

__global__ void dequant_q4k_kernel(const uint8_t* __restrict__ w, int tiles, int N, int K, float* __restrict__ out) {
  const int tile = blockIdx.x, strip = blockIdx.y, lane = threadIdx.x;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* tp = w + ((size_t)strip * tiles + tile) * kQ4KTileBytes;
  for (int hr = 0; hr < 2; ++hr) {
    const int row = strip * 16 + g + 8 * hr;
    if (row >= N) continue;
    const uint8_t* m = tp + 2048 + (g + 8 * hr) * 16;
    const float d = __half2float(__ushort_as_half((uint16_t)(m[0] | (m[1] << 8))));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(m[2] | (m[3] << 8))));
    const uint8_t* s12 = m + 4;
    for (int j = 0; j < 8; ++j) {
      int sc, mn;
      if (j < 4) { sc = s12[j] & 63; mn = s12[j + 4] & 63; }
      else { sc = (s12[j + 4] & 0x0F) | ((s12[j - 4] >> 6) << 4); mn = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4); }
      const float s = __fmul_rn(d, (float)sc), mm = __fmul_rn(dmin, (float)mn);
      const uint32_t word = reinterpret_cast<const uint32_t*>(tp + (j >> 1) * 512 + lane * 16)[(j & 1) * 2 + hr];
      for (int i = 0; i < 8; ++i)
        out[(size_t)row * K + tile * 256 + j * 32 + 8 * t + i] = __fsub_rn(__fmul_rn(s, (float)unplace(word, i)), mm);
    }
  }
}

/* the split of a matrix over the SMs (see Split) */
template <int QT, int NT>
static int make_split(Ctx* c, const Tensor* w, Split* sp) {
  const long long S = w->n_strips;
  ULB_CHECK(S > 0 && (long long)w->tiles * S * c->n_sm < (1ll << 31), ULB_EUNSUPPORTED, "qgemv: %lld strips of %d tiles",
            S, w->tiles);
  sp->S = (uint32_t)S;
  sp->G = (uint32_t)std::min<long long>(c->n_sm, S);
  sp->tiles = (uint32_t)w->tiles;
  sp->Wn = (uint32_t)std::min<long long>(GemvCfg<QT, NT>::W, S / sp->G * w->tiles);
  return ULB_OK;
}


/* shared memory of the normalised activation rows: M x K fp16 */
static size_t norm_bytes(int M, int K) { return ((size_t)M * K * sizeof(__half) + 15) / 16 * 16; }

template <int QT, int NT, int EPI, bool XS = false>
int launch_q(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, const EpiArgs& a, const NormIn& nin = NormIn()) {
  ULB_CHECK(w->K + 8 <= kZeroRowHalves, ULB_EUNSUPPORTED, "qgemv: K=%d too long", w->K);
  GemvStep S;
  S.w = (const uint8_t*)w->dev;
  ULB_TRY((make_split<QT, NT>(c, w, &S.sp)));
  S.N = w->N;
  S.M = M;
  S.x = x;
  S.ldx = ldx;
  S.nin = nin;
  S.ea = a;
  const size_t smem = warp_part_bytes<QT, NT>() + (XS ? norm_bytes(M, w->K) : 0);
  ULB_CHECK(smem <= kGemvSmemBytes, ULB_EUNSUPPORTED, "qgemv: %d normalised rows of %d", M, w->K);
  static bool attr_set = false;
  if (!attr_set) {
    ULB_CUDA(cudaFuncSetAttribute(qgemv_kernel<QT, NT, EPI, XS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kGemvSmemBytes));
    attr_set = true;
  }
  cudaError_t e = launch_k(c, qgemv_kernel<QT, NT, EPI, XS>, dim3(S.sp.G), dim3(GemvCfg<QT, NT>::W * 32), smem, S,
                           (const __half*)c->zero_row);
  if (e != cudaSuccess) return cuda_error(e, "qgemv launch", __FILE__, __LINE__);
  return ULB_OK;
}

template <int NT, int EPI>
int launch_nt(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, const EpiArgs& a) {
  if (w->type == ULB_TYPE_Q4_0) return launch_q<ULB_TYPE_Q4_0, NT, EPI>(c, w, x, M, ldx, a);
  return launch_q<ULB_TYPE_Q4_K, NT, EPI>(c, w, x, M, ldx, a);
}

template <int EPI>
int launch_epi(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, const EpiArgs& a) {
  if (M <= 8) return launch_nt<1, EPI>(c, w, x, M, ldx, a);
  if (M <= 16) return launch_nt<2, EPI>(c, w, x, M, ldx, a);
  return launch_nt<4, EPI>(c, w, x, M, ldx, a);
}

}  // namespace

/* Max rows per launch (larger M is chunked by the caller of launch_qgemv). */
static int max_rows_per_launch(int) { return kGemvMaxRows; }

static int launch_qgemv_impl(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a0);

int launch_qgemv(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a0) {
  return launch_qgemv_impl(c, w, x, M, ldx, epi, a0);
}

static int launch_qgemv_impl(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a0) {
  if (w && raw_rows_type(w->type)) return M == 0 ? ULB_OK : launch_rowgemv(c, w, x, M, ldx, epi, a0);
  ULB_CHECK(w && (w->type == ULB_TYPE_Q4_0 || w->type == ULB_TYPE_Q4_K), ULB_EINVAL, "qgemv: weight is not Q4_0/Q4_K");
  ULB_CHECK(M >= 0 && ldx % 8 == 0 && ldx >= w->K, ULB_EINVAL, "qgemv: bad M=%d / ldx=%d (K=%d)", M, ldx, w->K);
  ULB_CHECK(((uintptr_t)x & 15) == 0, ULB_EINVAL, "qgemv: activations must be 16-byte aligned");
  if (M == 0) return ULB_OK;
  /* dense enough for the tensor cores: one tcgen05 GEMM instead of 32-row GEMV launches */
  if (M > kGemvMaxRows && w->K % 64 == 0) return launch_qgemm_tc(c, w, x, M, ldx, epi, a0);
  const int step = max_rows_per_launch(w->type);
  for (int m0 = 0; m0 < M; m0 += step) {
    const int mc = M - m0 < step ? M - m0 : step;
    EpiArgs a = a0;
    const __half* xc = x + (size_t)m0 * ldx;
    if (a.y) a.y += (size_t)m0 * a.ldy;
    if (a.h) a.h += (size_t)m0 * a.ldh;
    if (a.q) a.q += (size_t)m0 * a.ldq;
    if (a.row_seq) a.row_seq += m0;
    if (a.row_pos) a.row_pos += m0;
    if (a.row_rope) a.row_rope += m0;
    int rc;
    switch (epi) {
      case EPI_STORE: rc = launch_epi<EPI_STORE>(c, w, xc, mc, ldx, a); break;
      case EPI_RESID: rc = launch_epi<EPI_RESID>(c, w, xc, mc, ldx, a); break;
      case EPI_SWIGLU: rc = launch_epi<EPI_SWIGLU>(c, w, xc, mc, ldx, a); break;
      case EPI_QKV: rc = launch_epi<EPI_QKV>(c, w, xc, mc, ldx, a); break;
      default: return set_error(ULB_EINVAL, "qgemv: bad epilogue %d", epi);
    }
    if (rc) return rc;
  }
  return ULB_OK;
}

int launch_qgemv_rms(Ctx* c, const Tensor* w, const float* x32, int ldx32, const float* g, float eps, __half* x16,
                     int M, int epi, const EpiArgs& a) {
  ULB_CHECK(w && (w->type == ULB_TYPE_Q4_0 || w->type == ULB_TYPE_Q4_K || raw_rows_type(w->type)), ULB_EINVAL,
            "qgemv: weight is not Q4_0/Q4_K/Q8_0/Q6_K/F16/F32");
  if (M == 0) return ULB_OK;
  const bool fuse = !raw_rows_type(w->type) && M <= 8 && (size_t)M * w->K * sizeof(__half) <= (size_t)kNormSmemBytes && w->K <= 8192 &&
                    w->K % 8 == 0 && ldx32 % 4 == 0 && ((uintptr_t)x32 & 15) == 0 && ((uintptr_t)g & 15) == 0 &&
                    (epi == EPI_QKV || epi == EPI_SWIGLU || epi == EPI_STORE);
  if (!fuse) {
    ULB_TRY(launch_rmsnorm_sel(c, x32, ldx32, g, M, w->K, eps, 0, x16, w->K));
    return launch_qgemv(c, w, x16, M, w->K, epi, a);
  }
  NormIn nin;
  nin.x = x32;
  nin.ldx = ldx32;
  nin.g = g;
  nin.eps = eps;
  const bool q40 = w->type == ULB_TYPE_Q4_0;
  int rc;
  if (epi == EPI_QKV)
    rc = q40 ? launch_q<ULB_TYPE_Q4_0, 1, EPI_QKV, true>(c, w, nullptr, M, w->K, a, nin)
             : launch_q<ULB_TYPE_Q4_K, 1, EPI_QKV, true>(c, w, nullptr, M, w->K, a, nin);
  else if (epi == EPI_SWIGLU)
    rc = q40 ? launch_q<ULB_TYPE_Q4_0, 1, EPI_SWIGLU, true>(c, w, nullptr, M, w->K, a, nin)
             : launch_q<ULB_TYPE_Q4_K, 1, EPI_SWIGLU, true>(c, w, nullptr, M, w->K, a, nin);
  else
    rc = q40 ? launch_q<ULB_TYPE_Q4_0, 1, EPI_STORE, true>(c, w, nullptr, M, w->K, a, nin)
             : launch_q<ULB_TYPE_Q4_K, 1, EPI_STORE, true>(c, w, nullptr, M, w->K, a, nin);
  return rc;
}

int launch_dequant(Ctx* c, const Tensor* w, float* out) {
  dim3 grid(w->tiles, w->n_strips), block(32);
  if (w->type == ULB_TYPE_Q4_0)
    dequant_q40_kernel<<<grid, block, 0, c->stream>>>((const uint8_t*)w->dev, w->tiles, w->N, w->K, out);
  else if (w->type == ULB_TYPE_Q4_K)
    dequant_q4k_kernel<<<grid, block, 0, c->stream>>>((const uint8_t*)w->dev, w->tiles, w->N, w->K, out);
  else
    return set_error(ULB_EINVAL, "dequant: tensor type %d is not quantised", w->type);
  ULB_CUDA(cudaGetLastError());
  return ULB_OK;
}

int repack_q4(Ctx* c, int type, const void* dev_raw, int raw_rows, int K, const int* host_row_map,
              int packed_rows, Tensor* out) {
  ULB_CHECK(type == ULB_TYPE_Q4_0 || type == ULB_TYPE_Q4_K, ULB_EINVAL, "repack: type %d", type);
  const int tk = tile_k(type);
  ULB_CHECK(K > 0 && K % tk == 0, ULB_EUNSUPPORTED, "repack: K=%d must be a multiple of %d", K, tk);
  ULB_CHECK(packed_rows > 0 && packed_rows % kStripRows == 0, ULB_EINVAL, "repack: rows %d", packed_rows);
  for (int i = 0; i < packed_rows; ++i)
    ULB_CHECK(host_row_map[i] < raw_rows, ULB_EINVAL, "repack: row map out of range");
  out->type = type;
  out->K = K;
  out->n_strips = packed_rows / kStripRows;
  out->tiles = K / tk;
  out->bytes = (size_t)out->n_strips * out->tiles * tile_bytes(type);
  ULB_TRY(dev_alloc(c, &out->dev, out->bytes));
  int* dmap = nullptr;
  ULB_TRY(dev_alloc(c, (void**)&dmap, (size_t)packed_rows * sizeof(int)));
  cudaError_t e = cudaMemcpyAsync(dmap, host_row_map, (size_t)packed_rows * sizeof(int), cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) {
    dim3 grid(out->tiles, out->n_strips), block(32);
    if (type == ULB_TYPE_Q4_0)
      repack_q40_kernel<<<grid, block, 0, c->stream>>>((const uint8_t*)dev_raw, K, dmap, (uint8_t*)out->dev, out->tiles);
    else
      repack_q4k_kernel<<<grid, block, 0, c->stream>>>((const uint8_t*)dev_raw, K, dmap, (uint8_t*)out->dev, out->tiles);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  dev_free(c, dmap, (size_t)packed_rows * sizeof(int));
  if (e != cudaSuccess) return cuda_error(e, "repack", __FILE__, __LINE__);
  return ULB_OK;
}

}  // namespace ulb

ULB_TRACE_UNIT(qgemv)
