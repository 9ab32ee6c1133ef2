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
 *  - persistent CTAs (2 per SM for M <= 8) walk 16-row strips; a strip is one contiguous
 *    range of packed tiles, streamed global -> shared in ~36 KB chunks by cp.async.bulk
 *    through a 2-slot mbarrier ring; the first chunks are issued before
 *    griddepcontrol.wait, so the weight stream overlaps the previous kernel (programmatic
 *    dependent launch), and the last warp done with a slot refills it (no producer warp,
 *    so 8 warps x 2 CTAs leave 128 registers a thread);
 *  - each warp owns tiles warp, warp + 8, ... of a chunk and loads tile j + 1 (weights
 *    from shared memory, activations from L1) into registers before computing tile j;
 *  - nibbles become exact fp16 integers with one LOP3 + one HSUB2/HFMA2 per pair
 *    (0x6400 magic) and feed mma.sync.m16n8k16 (weights = A, activations = B, so M <= 8
 *    tokens fill one n-tile); each 32-weight block's scale is applied in fp32 to that
 *    block's integer dot product, so weights are never rounded;
 *  - the fused epilogues write RoPE'd Q / K / V (K and V straight into the fp16 KV cache),
 *    SiLU(gate)*up in fp16, or the fp32 residual add.
 * The tensor pipe is idle in this regime (<= 3.6 flop/B at M = 1); mma.sync is used as the
 * cheapest-to-issue dot product engine.  The reduction order of a row never depends on M.
 */
#include "epilogue.cuh"

namespace ulb {

namespace {

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

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
template <int BIAS>
__device__ __forceinline__ void nib_pairs(uint32_t v, uint32_t& p01, uint32_t& p23, uint32_t& p45,
                                          uint32_t& p67) {
  constexpr uint32_t MAGIC = 0x64006400u;
  /* fp16 of 1024 + BIAS and of -(64 + BIAS), duplicated */
  constexpr uint32_t SUB = BIAS == 8 ? 0x64086408u : 0x64006400u;
  constexpr uint32_t NEG = BIAS == 8 ? 0xD480D480u : 0xD400D400u;
  constexpr uint32_t SIXTEENTH = 0x2C002C00u;
  uint32_t v8 = v >> 8;
  p01 = hsub2u((v & 0x000F000Fu) | MAGIC, SUB);
  p23 = hfma2u((v & 0x00F000F0u) | MAGIC, SIXTEENTH, NEG);
  p45 = hsub2u((v8 & 0x000F000Fu) | MAGIC, SUB);
  p67 = hfma2u((v8 & 0x00F000F0u) | MAGIC, SIXTEENTH, NEG);
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

/* the same column sums from activation fragments already in registers */
template <int NT>
__device__ __forceinline__ void block_colsum_r(const uint4 (&bx)[NT], float (&s)[NT][4]) {
  const uint32_t ONES = 0x3C003C00u;
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float tmp[4];
    mma16816(tmp, ONES, ONES, ONES, ONES, bx[nt].x, bx[nt].y, zero);
    mma16816(s[nt], ONES, ONES, ONES, ONES, bx[nt].z, bx[nt].w, tmp);
  }
}

/* Q4_K 6-bit (scale, min) of sub-block J from the 12 packed bytes (3 little-endian words). */
template <int J>
__device__ __forceinline__ void q4k_sm(uint32_t w0, uint32_t w1, uint32_t w2, float& sc, float& mn) {
  uint32_t s, m;
  if (J < 4) {
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
/* lane (g, t) holds, for n-tile nt, rows (g, g + 8) of tokens nt*8 + 2t and + 1 */
template <int EPI>
__device__ __forceinline__ void epilogue(const EpiArgs& e, int strip, int nt, int g, int t, int M,
                                         int N, const float4& v) {
  const int tok0 = nt * 8 + 2 * t;
  epilogue_token<EPI>(e, strip, g, tok0, M, N, v.x, v.z);
  epilogue_token<EPI>(e, strip, g, tok0 + 1, M, N, v.y, v.w);
}

constexpr int kWarps = 8;

template <int NT>
__device__ __forceinline__ void reduce_and_finish_prep(float (&acc)[NT][4], float4* red, int warp, int lane) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    red[(warp * NT + nt) * 32 + lane] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
}

/* ------------------------------------------------------------------ staged weight pipeline */
/*
 * A strip's packed bytes are copied global -> shared with cp.async.bulk in chunks of 27 KB
 * (24 Q4_0 tiles or 12 Q4_K tiles) through a ring of 3 buffers, each guarded by an
 * mbarrier.  The first three chunks are issued before griddepcontrol.wait, so the weight
 * stream of this kernel overlaps the previous kernel in the stream.
 */
constexpr int kChunkBytes = 27648;
constexpr int kNBuf = 3;
constexpr int kMaxChunks = 32;
template <int QT> struct QTraits;
template <> struct QTraits<ULB_TYPE_Q4_0> { static constexpr int TB = kQ40TileBytes, CT = 24; };
template <> struct QTraits<ULB_TYPE_Q4_K> { static constexpr int TB = kQ4KTileBytes, CT = 12; };

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
/* try_wait with a 1 ms suspend hint: a waiting thread sleeps until the phase completes
   instead of spinning on the issue slots the consumer warps need */
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
/* Wait for phase `parity`; gives up after `limit_ns` of wall time (returns false). */
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try(bar, parity))
    if (gtimer() - t0 > limit_ns) return false;
  return true;
}

/*
 * A tile's operands in registers.  The consumer loop loads tile j + 1 (shared-memory weight
 * words, and for Q4_0 at NT = 1 also the activation fragments from L1) before it computes
 * tile j, so the load latency hides behind a tile of dequant + MMA work.
 *   Q4_0: 2 x 16 B of nibble words + 16 B of scales (rows g, g + 8) per lane.
 *   Q4_K: 4 x 16 B of nibble words + the 16 B meta rows of g and g + 8.
 */
template <int QT, int NT> struct TileRegs;
template <int NT> struct TileRegs<ULB_TYPE_Q4_0, NT> {
  static constexpr bool PFX = NT == 1; /* activations prefetched with the weights */
  uint4 w[2], sc;
  uint4 x[PFX ? 4 : 1][NT];
};
template <int NT> struct TileRegs<ULB_TYPE_Q4_K, NT> {
  static constexpr bool PFX = false;
  uint4 w[4], mg, mg8;
};

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

template <bool XS, int NT>
__device__ __forceinline__ void tile_load(TileRegs<ULB_TYPE_Q4_0, NT>& r, const uint8_t* tp, int tile,
                                          const __half* const (&xr)[NT], int lane, int g) {
  r.w[0] = lds128(tp + lane * 16);
  r.w[1] = lds128(tp + 512 + lane * 16);
  r.sc = lds128(tp + 1024 + g * 16);
  if (TileRegs<ULB_TYPE_Q4_0, NT>::PFX) {
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) r.x[b][nt] = xld<XS>(xr[nt] + tile * 128 + b * 32);
  }
}

template <bool XS, int NT>
__device__ __forceinline__ void tile_load(TileRegs<ULB_TYPE_Q4_K, NT>& r, const uint8_t* tp, int, const __half* const (&)[NT],
                                          int lane, int g) {
#pragma unroll
  for (int p = 0; p < 4; ++p) r.w[p] = lds128(tp + p * 512 + lane * 16);
  r.mg = lds128(tp + 2048 + g * 16);
  r.mg8 = lds128(tp + 2048 + (g + 8) * 16);
}

/* dot products of one 32-weight block whose activation fragments are already in registers */
template <int BIAS, int NT>
__device__ __forceinline__ void block_mma_r(uint32_t vg, uint32_t vg8, const uint4 (&bx)[NT], float (&s)[NT][4]) {
  uint32_t a01, a23, a45, a67, b01, b23, b45, b67;
  nib_pairs<BIAS>(vg, a01, a23, a45, a67);
  nib_pairs<BIAS>(vg8, b01, b23, b45, b67);
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float tmp[4];
    mma16816(tmp, a01, b01, a23, b23, bx[nt].x, bx[nt].y, zero);
    mma16816(s[nt], a45, b45, a67, b67, bx[nt].z, bx[nt].w, tmp);
  }
}

template <bool XS, int NT>
__device__ __forceinline__ void tile_compute(const TileRegs<ULB_TYPE_Q4_0, NT>& r, int tile, const __half* const (&xr)[NT],
                                             float (&acc)[NT][4]) {
  const uint32_t words[8] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w, r.w[1].x, r.w[1].y, r.w[1].z, r.w[1].w};
  const uint32_t scw[4] = {r.sc.x, r.sc.y, r.sc.z, r.sc.w};
  uint4 xl[4][NT];
  if (!TileRegs<ULB_TYPE_Q4_0, NT>::PFX) { /* all of the tile's activation loads first */
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) xl[b][nt] = xld<XS>(xr[nt] + tile * 128 + b * 32);
  }
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    float s[NT][4];
    if (TileRegs<ULB_TYPE_Q4_0, NT>::PFX)
      block_mma_r<8, NT>(words[2 * b], words[2 * b + 1], r.x[TileRegs<ULB_TYPE_Q4_0, NT>::PFX ? b : 0], s);
    else
      block_mma_r<8, NT>(words[2 * b], words[2 * b + 1], xl[b], s);
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&scw[b]));
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      acc[nt][0] = __fmaf_rn(dd.x, s[nt][0], acc[nt][0]);
      acc[nt][1] = __fmaf_rn(dd.x, s[nt][1], acc[nt][1]);
      acc[nt][2] = __fmaf_rn(dd.y, s[nt][2], acc[nt][2]);
      acc[nt][3] = __fmaf_rn(dd.y, s[nt][3], acc[nt][3]);
    }
  }
}

template <bool XS, int NT>
__device__ __forceinline__ void tile_compute(const TileRegs<ULB_TYPE_Q4_K, NT>& r, int tile, const __half* const (&xr)[NT],
                                             float (&acc)[NT][4]);

/*
 * Persistent, warp-specialised form: one CTA per SM walks strips blockIdx.x, +gridDim.x, ...
 * A producer warp streams the CTA's whole sequence of weight chunks (16 tiles each)
 * through a ring of shared-memory slots with cp.async.bulk (full / empty mbarrier pairs),
 * starting before griddepcontrol.wait; CW consumer warps dequantise + MMA one tile each
 * per chunk and release the slot.  HBM never waits for compute and vice versa.
 * Every wait has a deadline (2 s after kernel start): past it the CTA stops computing,
 * raises bit 1 of *err and runs to completion without writing results.
 */
/* a chunk is ~36 KB of one strip; 2 ring slots per CTA; 2 CTAs per SM for NT <= 2 */
template <int QT> struct PQ;
template <> struct PQ<ULB_TYPE_Q4_0> { static constexpr int TB = kQ40TileBytes, CT = 32, NB = 2; };
template <> struct PQ<ULB_TYPE_Q4_K> { static constexpr int TB = kQ4KTileBytes, CT = 16, NB = 2; };
template <int NT> struct PQW {
  static constexpr int CW = 8;               /* consumer warps; fixed so reduction order is too */
  static constexpr int MINB = NT == 1 ? 2 : 1; /* resident CTAs per SM */
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_wait_deadline(uint64_t* bar, uint32_t parity, uint64_t deadline) {
  while (!mbar_try(bar, parity))
    if (gtimer() > deadline) return false;
  return true;
}

/* RMSNorm fused into the GEMV (XS): the fp32 rows, the norm weights and eps */
struct NormIn {
  const float* x = nullptr;
  int ldx = 0;
  const float* g = nullptr;
  float eps = 0.f;
};

template <int QT, int NT, int EPI, bool XS>
__global__ void __launch_bounds__(PQW<NT>::CW * 32, PQW<NT>::MINB)
    qgemv_kernel(const uint8_t* __restrict__ w, int tiles, int n_strips, int N, const __half* x, int M,
                 int ldx, EpiArgs ea, int* err, int nb, const __half* __restrict__ xzero, NormIn nin) {
  constexpr int TB = PQ<QT>::TB, CT = PQ<QT>::CT, NB = PQ<QT>::NB, CW = PQW<NT>::CW;
  constexpr int CB = CT * TB;
  /* tile i of a chunk always accumulates into slot i (of CT), and slots are summed in slot
     order, so a row's arithmetic is the same whatever NT / the number of consumer warps */
  constexpr int NSL = CT / CW;
  extern __shared__ __align__(128) uint8_t ring[]; /* nb slots of CB bytes, then the slot sums */
  float4* red = reinterpret_cast<float4*>(ring + (size_t)nb * CB);
  __shared__ uint64_t full[NB];
  __shared__ uint32_t released[NB]; /* warps done with the slot's current chunk */
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nch = (tiles + CT - 1) / CT;
  const int my_strips = (n_strips - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int total = my_strips * nch; /* chunks this CTA streams, in order */
  /* chunk q of the CTA's sequence -> ring slot q % nb */
  auto issue = [&](int q) {
    const int s = blockIdx.x + (q / nch) * gridDim.x, ch = q % nch, slot = q % nb;
    const uint32_t bytes = (uint32_t)min(CT, tiles - ch * CT) * TB;
    mbar_expect_tx(&full[slot], bytes);
    bulk_g2s(ring + (size_t)slot * CB, w + ((size_t)s * tiles + (size_t)ch * CT) * TB, bytes, &full[slot]);
  };
  if (tid == 0) {
    for (int i = 0; i < nb; ++i) {
      mbar_init(&full[i], 1);
      released[i] = 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint64_t deadline = gtimer() + 2000000000ull;
  /* the weights do not depend on the previous kernel: start streaming before the wait */
  if (tid == 0)
    for (int q = 0; q < nb && q < total; ++q) issue(q);
  pdl_wait();
  pdl_trigger();
  if (XS) {
    /* every CTA normalises the M input rows into its own shared-memory copy, with the
       arithmetic of rmsnorm_kernel (so the fused and the separate paths give the same bits) */
    __shared__ float nred[32];
    __half* xs = reinterpret_cast<__half*>(ring + (size_t)nb * CB + 2 * (size_t)CW * NT * 32 * sizeof(float4));
    const int K = tiles * (QT == ULB_TYPE_Q4_0 ? kQ40TileK : kQ4KTileK);
    for (int m = 0; m < M; ++m) rms_row_256(nin.x + (size_t)m * nin.ldx, nin.g, K, nin.eps, xs + (size_t)m * K, nred);
    __syncthreads();
    x = xs;
    ldx = K;
  }
  const int g = lane >> 2, t = lane & 3;
  const __half* xr[NT];
  activation_rows<NT>(x, xzero, ldx, M, g, t, xr);
  int seq = 0, iter = 0;
  bool ok = true;
  for (int s = blockIdx.x; s < n_strips; s += gridDim.x, ++iter) {
    float acc[NSL][NT][4];
#pragma unroll
    for (int j = 0; j < NSL; ++j)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[j][nt][0] = acc[j][nt][1] = acc[j][nt][2] = acc[j][nt][3] = 0.f;
    for (int ch = 0; ch < nch; ++ch, ++seq) {
      const int slot = seq % nb;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait_deadline(&full[slot], (uint32_t)(seq / nb) & 1u, deadline));
      if (ok) {
        const uint8_t* base = ring + (size_t)slot * CB;
        const int t0 = ch * CT, tn = min(tiles - t0, CT);
        /* software pipeline over the warp's tiles warp, warp + CW, ...: load j + 1, compute j */
        TileRegs<QT, NT> tr[2]; /* indexed by j & 1: constant after unrolling, so no copies */
        if (warp < tn) tile_load<XS, NT>(tr[0], base + warp * TB, t0 + warp, xr, lane, g);
#pragma unroll
        for (int j = 0; j < NSL; ++j) {
          const int i = warp + j * CW;
          if (j + 1 < NSL && i + CW < tn)
            tile_load<XS, NT>(tr[(j + 1) & 1], base + (i + CW) * TB, t0 + i + CW, xr, lane, g);
          if (i < tn) tile_compute<XS, NT>(tr[j & 1], t0 + i, xr, acc[j]);
        }
      }
      __syncwarp();
      if (lane == 0) {
        /* the last of the CW warps to be done with the slot refills it with chunk seq + nb:
           acq_rel makes every warp's reads of the slot happen before the refill, and the
           proxy fence orders them before the async-proxy write of the bulk copy */
        uint32_t prev;
        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "r"(smem_u32(&released[slot]))
                     : "memory");
        if (prev == CW - 1) {
          released[slot] = 0;
          if (seq + nb < total) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(seq + nb);
          }
        }
      }
    }
    /* slots w, w+CW, ... are summed in the warp, then warps in warp order: CW is the same
       for every NT, so this order is fixed.  The partials alternate between two buffers, so
       one barrier per strip suffices: a buffer is rewritten two strips later, after every
       warp (its reader included) has passed the barrier of the strip in between. */
    float4* rb = red + (size_t)(iter & 1) * CW * NT * 32;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float4 v = make_float4(acc[0][nt][0], acc[0][nt][1], acc[0][nt][2], acc[0][nt][3]);
#pragma unroll
      for (int j = 1; j < NSL; ++j) {
        v.x += acc[j][nt][0]; v.y += acc[j][nt][1]; v.z += acc[j][nt][2]; v.w += acc[j][nt][3];
      }
      rb[(warp * NT + nt) * 32 + lane] = v;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
    /* n-tile nt of this strip is finished by warp (nt + iter) % CW: the epilogue work rotates
       over the warps instead of stalling warp 0 on every strip */
    for (int nt = (warp - iter % CW + CW) % CW; nt < NT; nt += CW) {
      float4 v = rb[nt * 32 + lane];
#pragma unroll
      for (int w2 = 1; w2 < CW; ++w2) {
        const float4 o = rb[(w2 * NT + nt) * 32 + lane];
        v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
      }
      if (ok) epilogue<EPI>(ea, s, nt, g, t, M, N, v);
    }
  }
  if (!ok && lane == 0) atomicOr(err, 2);
}

/* ------------------------------------------------------------------ Q4_K tile */
template <bool XS, int NT>
__device__ __forceinline__ void tile_compute(const TileRegs<ULB_TYPE_Q4_K, NT>& r, int tile, const __half* const (&xr)[NT],
                                             float (&acc)[NT][4]) {
  {
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
    {                                                                                    \
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(&nb[(J) >> 1]);            \
      float s1[NT][4], s0[NT][4];                                                        \
      const int kofs = tile * 256 + (J) * 32;                                            \
      uint4 bx[NT];                                                                      \
      _Pragma("unroll") for (int nt = 0; nt < NT; ++nt)                                  \
        bx[nt] = xld<XS>(xr[nt] + kofs);                                                 \
      block_mma_r<0, NT>(wp[((J) & 1) * 2], wp[((J) & 1) * 2 + 1], bx, s1);              \
      block_colsum_r<NT>(bx, s0);                                                        \
      float scg, mng, scg8, mng8;                                                        \
      q4k_sm<J>(mg.y, mg.z, mg.w, scg, mng);                                             \
      q4k_sm<J>(mg8.y, mg8.z, mg8.w, scg8, mng8);                                        \
      _Pragma("unroll") for (int nt = 0; nt < NT; ++nt) {                                \
        t1[nt][0] = __fmaf_rn(scg, s1[nt][0], t1[nt][0]);                                \
        t1[nt][1] = __fmaf_rn(scg, s1[nt][1], t1[nt][1]);                                \
        t1[nt][2] = __fmaf_rn(scg8, s1[nt][2], t1[nt][2]);                               \
        t1[nt][3] = __fmaf_rn(scg8, s1[nt][3], t1[nt][3]);                               \
        t0[nt][0] = __fmaf_rn(mng, s0[nt][0], t0[nt][0]);                                \
        t0[nt][1] = __fmaf_rn(mng, s0[nt][1], t0[nt][1]);                                \
        t0[nt][2] = __fmaf_rn(mng8, s0[nt][2], t0[nt][2]);                               \
        t0[nt][3] = __fmaf_rn(mng8, s0[nt][3], t0[nt][3]);                               \
      }                                                                                  \
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

template <int QT, int NT, int EPI, bool XS = false>
int launch_q(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, const EpiArgs& a, const NormIn& nin = NormIn()) {
  constexpr int TB = PQ<QT>::TB, CT = PQ<QT>::CT, NB = PQ<QT>::NB, CW = PQW<NT>::CW;
  const int nch = (w->tiles + CT - 1) / CT;
  /* ring: as many slots as the CTA has chunks in flight, at most NB */
  ULB_CHECK(w->K + 8 <= kZeroRowHalves, ULB_EUNSUPPORTED, "qgemv: K=%d too long", w->K);
  const int ctas = c->n_sm * PQW<NT>::MINB;
  const int per_cta = (w->n_strips + ctas - 1) / ctas;
  const int grid = (w->n_strips + per_cta - 1) / per_cta; /* balanced: every CTA gets per_cta or per_cta-1 strips */
  const int slots = min(NB, per_cta * nch);
  const size_t red_bytes = 2 * (size_t)CW * NT * 32 * sizeof(float4); /* two alternating partial buffers */
  const size_t xs_bytes = XS ? (size_t)kNormSmemBytes : 0; /* normalised x (fused RMSNorm) */
  const size_t smem = (size_t)slots * CT * TB + red_bytes + xs_bytes;
  static bool attr_set = false;
  if (!attr_set) {
    ULB_CUDA(cudaFuncSetAttribute(qgemv_kernel<QT, NT, EPI, XS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)((size_t)NB * CT * TB + red_bytes + xs_bytes)));
    attr_set = true;
  }
  cudaError_t e = launch_k(c, qgemv_kernel<QT, NT, EPI, XS>, dim3(grid), dim3(CW * 32), smem,
                           (const uint8_t*)w->dev, w->tiles, w->n_strips, w->N, x, M, ldx, a, c->dev_err, slots,
                           (const __half*)c->zero_row, nin);
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

int launch_qgemv(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a0) {
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
  ULB_CHECK(w && (w->type == ULB_TYPE_Q4_0 || w->type == ULB_TYPE_Q4_K), ULB_EINVAL, "qgemv: weight is not Q4_0/Q4_K");
  if (M == 0) return ULB_OK;
  const bool fuse = M <= 8 && (size_t)M * w->K * sizeof(__half) <= (size_t)kNormSmemBytes && w->K <= 8192 &&
                    w->K % 8 == 0 && ldx32 % 4 == 0 && ((uintptr_t)x32 & 15) == 0 && ((uintptr_t)g & 15) == 0 &&
                    (epi == EPI_QKV || epi == EPI_SWIGLU);
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
  if (epi == EPI_QKV)
    return q40 ? launch_q<ULB_TYPE_Q4_0, 1, EPI_QKV, true>(c, w, nullptr, M, w->K, a, nin)
               : launch_q<ULB_TYPE_Q4_K, 1, EPI_QKV, true>(c, w, nullptr, M, w->K, a, nin);
  return q40 ? launch_q<ULB_TYPE_Q4_0, 1, EPI_SWIGLU, true>(c, w, nullptr, M, w->K, a, nin)
             : launch_q<ULB_TYPE_Q4_K, 1, EPI_SWIGLU, true>(c, w, nullptr, M, w->K, a, nin);
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
