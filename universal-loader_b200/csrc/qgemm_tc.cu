/*
 * qgemm_tc.cu — fused Q4_0 / Q4_K dequant-GEMM on the 5th-generation tensor cores, for the
 * compute-dense regime (M >= 64 rows: prefill chunks, large verify batches, the config-3
 * M = 64 / 256 sweep).  Same operator as the GEMV in qgemv.cu (packed strip layout, fused
 * epilogues), different machine.
 *
 * Replaces the reference's fp32 dequantise-then-GEMM pair (dequantize_q4_k_flattened.glsl +
 * gemm_transposed_b_v2.glsl via run_linear_q4k, src/inference/inference_engine.cpp:532-570)
 * for batched rows.
 *
 * One CTA computes a 128-weight-row x NT-token tile of y = W x^T over the whole of K, fed by
 * TMA (each copy to this CTA only): one 3-D tensor-map load per packed K-tile brings the 8 strips'
 * raw Q4 bytes, one 2-D load per 64-k stage brings the activation tile already in the
 * 128-byte-swizzled K-major layout; 8 warps dequantise each stage into fp16 weights in the
 * same layout, each weight rounded once to fp16 (a Q4_0 weight d (q - 8) is the correctly
 * rounded product of two exact fp16 values; a Q4_K weight d sc q - dmin m is formed in fp32
 * first), so a weight carries at most 2^-12 relative error here, where the GEMV regime keeps
 * weights exact; one lane issues tcgen05.mma (M = 128, N = NT, K = 16, fp16 x fp16 -> fp32 in
 * TMEM) once per k-step and commits each stage to the mbarriers that free its slots; the 8
 * warps then read TMEM and run the epilogue.
 * From kTcWideRows rows on, parallelism comes from the token tile (64 ... 256 tokens, the one
 * with the shortest estimated makespan over the SMs) and K is never split; below that (33 ... 255 rows)
 * the tile is 64 tokens and K is split S ways, S fixed per matrix (tc_splits), with the
 * partials added in split order.  Either way a row's summation order does not depend on M.
 * Every mbarrier wait has a deadline (2 s): past it the CTA raises bit 3 of the device error
 * word, stops issuing work and still waits (bounded) for its MMAs before freeing TMEM.
 */
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "epilogue.cuh"

namespace ulb {

namespace {

constexpr int BM = 128;     /* weight rows per tile = UMMA M */
constexpr int KS = 64;      /* k per stage: one 128-byte swizzle atom of fp16 */
constexpr int TCW = 11;     /* warps */

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mb_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mb_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ bool mb_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(sa(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
/* wait for the phase with this parity; false once the deadline has passed */
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t parity, uint64_t deadline) {
  while (!mb_try(b, parity))
    if (gtime() > deadline) return false;
  return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(sa(dst)),
               "l"(src), "r"(bytes), "r"(sa(bar))
               : "memory");
}
__device__ __forceinline__ void cp16z(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

/* K-major operand in the 128-byte swizzle layout: rows of 128 bytes (64 fp16 of K), 8-row
   groups 1024 bytes apart, 16-byte chunk c of row r stored at chunk c ^ (r & 7). */
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}
/* shared-memory matrix descriptor (tcgen05): start address >> 4, leading byte offset 1
   (unused by swizzled K-major layouts), stride byte offset 1024 >> 4 (next 8-row group),
   descriptor version 1, base offset 0 (atoms are 1024-byte aligned), swizzle mode 2 = 128 B */
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
/* instruction descriptor, kind::f16: D fp32 (bit 4), A = B = fp16 (formats 0), both
   K-major, N >> 3 at bit 17, M >> 4 at bit 24 */
template <int NT>
__device__ __forceinline__ uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(bar))
               : "memory");
}
/* 32 consecutive fp32 columns of this warp's 32 TMEM lanes: thread l gets lane (base + l) */
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

/* nibbles at positions {0,16,4,20,8,24,12,28} of v -> four fp16x2 pairs (q0,q1)..(q6,q7) minus bias */
template <int BIAS>
__device__ __forceinline__ void nib4(uint32_t v, uint32_t (&p)[4]) {
  constexpr uint32_t MAGIC = 0x64006400u;
  constexpr uint32_t SUB = BIAS == 8 ? 0x64086408u : 0x64006400u;
  constexpr uint32_t NEG = BIAS == 8 ? 0xD480D480u : 0xD400D400u;
  const uint32_t v8 = v >> 8;
  p[0] = h2u(__hsub2(u2h((v & 0x000F000Fu) | MAGIC), u2h(SUB)));
  p[1] = h2u(__hfma2(u2h((v & 0x00F000F0u) | MAGIC), u2h(0x2C002C00u), u2h(NEG)));
  p[2] = h2u(__hsub2(u2h((v8 & 0x000F000Fu) | MAGIC), u2h(SUB)));
  p[3] = h2u(__hfma2(u2h((v8 & 0x00F000F0u) | MAGIC), u2h(0x2C002C00u), u2h(NEG)));
}

/* Q4_K 6-bit (scale, min) of sub-block j from the 12 packed bytes */
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s12, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = s12[j] & 63;
    mn = s12[j + 4] & 63;
  } else {
    sc = (s12[j + 4] & 0x0F) | ((s12[j - 4] >> 6) << 4);
    mn = (s12[j + 4] >> 4) | ((s12[j] >> 6) << 4);
  }
}

template <int QT, int NT>
struct TcCfg {
  static constexpr int TB = QT == ULB_TYPE_Q4_0 ? kQ40TileBytes : kQ4KTileBytes;
  static constexpr int A_BYTES = BM * KS * 2;            /* 16 KB: dequantised fp16 weights      */
  static constexpr int B_BYTES = NT * KS * 2;            /* activation tile (TMA, 128 B swizzle) */
  static constexpr int RAW_BYTES = 8 * TB;               /* one packed K-tile of the 8 strips    */
  /* ring depths: A slots cover dequantise + MMA, activation slots an L2 round trip, and the
     raw-weight ring (K-tiles of 2 or 4 stages) the several-microsecond latency of weight
     tiles streamed by every SM at once */
  static constexpr int SA = NT <= 128 ? 6 : 4;
  static constexpr int SB = NT == 64 ? 8 : 3;
  static constexpr int RT = QT == ULB_TYPE_Q4_0 ? (NT == 192 ? 8 : 6) : (NT == 192 ? 4 : 3);
  static constexpr int SMEM = SA * A_BYTES + SB * B_BYTES + RT * RAW_BYTES + 1024; /* + alignment slack */
  static constexpr int TMEM_COLS = NT <= 64 ? 64 : NT <= 128 ? 128 : 256;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct TcArgs {
  int tiles, n_strips, N, M;
  int splits; /* K splits (grid z): split s covers packed K-tiles [s T / S, (s + 1) T / S) */
  int tt0;    /* first token tile of this launch */
  float* ws;  /* splits > 1: partial sums [tile of the launch][split][NT][128] */
  int* cnt;   /* splits > 1: arrivals per tile of the launch (zero between launches) */
  int* err;
};

/* TMA tile loads into this CTA: dst, tensor map, coordinates (innermost first) */
__device__ __forceinline__ void tma2(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          sa(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(sa(bar))
      : "memory");
}
__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* tm, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          sa(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(z), "r"(sa(bar))
      : "memory");
}

constexpr int kTmaBox = 144; /* u64 words per weight box: a Q4_0 tile, half a Q4_K tile */

/*
 * Warp roles (11 warps):
 *   0      activation tiles: one TMA load per stage into the B ring (the tensor map's
 *          128-byte swizzle writes the K-major layout the MMA reads; rows past M are zero)
 *   1      raw weights: one TMA load per packed K-tile (two for Q4_K) of all 8 strips into
 *          the raw ring; weights do not depend on earlier kernels, so it never waits for them
 *   2 - 9  dequantise raw -> A ring (fp16; two threads per weight row), then the epilogue
 *          from TMEM (two warps per TMEM lane quarter, each half of the token columns)
 *   10     TMEM owner; lane 0 issues tcgen05.mma and commits to the A / B free barriers
 */
template <int QT, int NT, int EPI>
__global__ void __launch_bounds__(TCW * 32, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, TcArgs a,
                    EpiArgs ea) {
  ULB_TRACE_KERNEL(kTrGemmTc + EPI, NT);
  using C = TcCfg<QT, NT>;
  constexpr int TB = C::TB;
  constexpr int TK = QT == ULB_TYPE_Q4_0 ? kQ40TileK : kQ4KTileK; /* k per packed tile */
  constexpr int SPT = TK / KS;                                     /* stages per packed tile */
  constexpr int SA = C::SA, SB = C::SB, RT = C::RT;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_raw[RT], free_raw[RT], full_a[SA], free_a[SA], full_b[SB], free_b[SB], acc_full;
  __shared__ uint32_t tmem_base_sh;
  __shared__ EpiRow srow[EPI == EPI_QKV ? NT : 1]; /* QKV: the tile's tokens' cache rows */
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* const a_ring = smem;
  uint8_t* const b_ring = smem + SA * C::A_BYTES;
  uint8_t* const raw_ring = b_ring + SB * C::B_BYTES;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wt = blockIdx.x, tt = a.tt0 + (int)blockIdx.y, split = blockIdx.z;
  const int strip0 = wt * 8;
  const int tok0 = tt * NT;
  const int kt0 = (int)((long long)split * a.tiles / a.splits);
  const int ntiles = (int)((long long)(split + 1) * a.tiles / a.splits) - kt0; /* packed K-tiles of this CTA */
  const int nk = ntiles * SPT;                                                 /* its 64-k stages */
  const int ks0 = kt0 * SPT;

  if (tid == 0) {
    for (int i = 0; i < RT; ++i) { mb_init(&full_raw[i], 1); mb_init(&free_raw[i], 8); }
    for (int i = 0; i < SA; ++i) { mb_init(&full_a[i], 8); mb_init(&free_a[i], 1); }
    for (int i = 0; i < SB; ++i) { mb_init(&full_b[i], 1); mb_init(&free_b[i], 1); }
    mb_init(&acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 10) { /* TMEM accumulator: NT fp32 columns x 128 lanes */
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&tmem_base_sh)),
                 "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint64_t deadline = gtime() + 2000000000ull;
  bool ok = true;

  if (warp == 1) {
    /* ------------------------------------------------ raw weights (TMA) */
    if (lane == 0) {
      for (int t = 0; t < ntiles; ++t) {
        const int r = t % RT;
        if (t >= RT && !mb_wait(&free_raw[r], (uint32_t)((t / RT) - 1) & 1u, deadline)) { ok = false; break; }
        uint8_t* raw = raw_ring + r * C::RAW_BYTES;
        mb_expect_tx(&full_raw[r], (uint32_t)C::RAW_BYTES);
        tma3(raw, &tw, 0, kt0 + t, strip0, &full_raw[r]);
        if (QT == ULB_TYPE_Q4_K) tma3(raw + 8 * kTmaBox * 8, &tw, kTmaBox, kt0 + t, strip0, &full_raw[r]);
      }
    }
    __syncwarp();
    pdl_wait();
    pdl_trigger();
  } else if (warp == 0) {
    /* ------------------------------------------------ activations (TMA) */
    pdl_wait();
    pdl_trigger();
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int b = i % SB;
        if (i >= SB && !mb_wait(&free_b[b], (uint32_t)((i / SB) - 1) & 1u, deadline)) { ok = false; break; }
        mb_expect_tx(&full_b[b], (uint32_t)C::B_BYTES);
        tma2(b_ring + b * C::B_BYTES, &tx, (ks0 + i) * KS, tok0, &full_b[b]);
      }
    }
    __syncwarp();
  } else if (warp >= 2 && warp <= 9) {
    /* ------------------------------------------------ dequantise: two threads per weight row,
       each one 32-weight block (4 chunks of 8) of the 64-weight stage */
    const int d = tid - 64; /* 0..255 */
    const int r = d >> 1, bb = d & 1;
    const int js = r >> 4, rr = r & 15, g = rr & 7, hr = rr >> 3;
    /* byte o of strip js's packed tile in the raw slot (a Q4_K tile arrives as two halves) */
    auto tile_byte = [&](const uint8_t* slot, int o) -> const uint8_t* {
      if (QT == ULB_TYPE_Q4_0) return slot + js * TB + o;
      constexpr int H = kTmaBox * 8;
      return o < H ? slot + js * H + o : slot + 8 * H + js * H + (o - H);
    };
    for (int i = 0; i < nk && ok; ++i) {
      const int t = i / SPT, part = i % SPT, rs = t % RT, ai = i % SA;
      if (!mb_wait(&full_raw[rs], (uint32_t)(t / RT) & 1u, deadline)) { ok = false; break; }
      if (i >= SA && !mb_wait(&free_a[ai], (uint32_t)((i / SA) - 1) & 1u, deadline)) { ok = false; break; }
      const uint8_t* slot = raw_ring + rs * C::RAW_BYTES;
      uint8_t* ahi = a_ring + ai * C::A_BYTES;
      float s = 0.f, mm = 0.f;
      __half2 d2;
      if (QT == ULB_TYPE_Q4_0) {
        const int blk = part * 2 + bb;
        const uint16_t dbits = *reinterpret_cast<const uint16_t*>(tile_byte(slot, 1024 + g * 16 + blk * 4 + hr * 2));
        d2 = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
      } else {
        const int sub = part * 2 + bb; /* 32-weight sub-block of the 256-weight super-block */
        const uint8_t* m = tile_byte(slot, 2048 + rr * 16);
        const float dd = __half2float(__ushort_as_half((uint16_t)(m[0] | (m[1] << 8))));
        const float dmin = __half2float(__ushort_as_half((uint16_t)(m[2] | (m[3] << 8))));
        int sc, mn;
        q4k_scale_min(m + 4, sub, sc, mn);
        s = __fmul_rn(dd, (float)sc);
        mm = __fmul_rn(dmin, (float)mn);
      }
#pragma unroll
      for (int t4 = 0; t4 < 4; ++t4) {
        const int c = bb * 4 + t4;
        const uint32_t word =
            *reinterpret_cast<const uint32_t*>(tile_byte(slot, part * 512 + (g * 4 + t4) * 16 + (bb * 2 + hr) * 4));
        uint32_t hi[4];
        if (QT == ULB_TYPE_Q4_0) {
          uint32_t q[4];
          nib4<8>(word, q);
#pragma unroll
          for (int e = 0; e < 4; ++e) hi[e] = h2u(__hmul2(u2h(q[e]), d2)); /* fp16(d (q - 8)), one rounding */
        } else {
          uint32_t q[4];
          nib4<0>(word, q);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 qf = __half22float2(u2h(q[e]));
            const float w0 = __fmaf_rn(s, qf.x, -mm), w1 = __fmaf_rn(s, qf.y, -mm);
            hi[e] = h2u(__floats2half2_rn(w0, w1));
          }
        }
        const uint32_t off = sw128_off(r, c);
        *reinterpret_cast<uint4*>(ahi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mb_arrive(&full_a[ai]);
        if (part == SPT - 1) mb_arrive(&free_raw[rs]);
      }
    }
    pdl_wait(); /* the epilogue reads / writes buffers of earlier kernels */
    pdl_trigger();
    if (EPI == EPI_QKV) { /* the tile's tokens' cache rows, once for all rows of the tile */
      for (int t = d; t < NT; t += 256) srow[t] = tok0 + t < a.M ? epi_row(ea, tok0 + t) : EpiRow{-1, 0, 0};
      asm volatile("bar.sync 1, 256;" ::: "memory");
    }
  } else if (warp == 10) {
    /* ------------------------------------------------ MMA issue (one lane) */
    pdl_trigger();
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<NT>();
      for (int i = 0; i < nk && ok; ++i) {
        const int ai = i % SA, bi = i % SB;
        if (!mb_wait(&full_a[ai], (uint32_t)(i / SA) & 1u, deadline) ||
            !mb_wait(&full_b[bi], (uint32_t)(i / SB) & 1u, deadline)) { ok = false; break; }
        tc_fence_after();
        uint8_t* ah = a_ring + ai * C::A_BYTES;
        const uint64_t dh = sw128_desc(sa(ah)), db = sw128_desc(sa(b_ring + bi * C::B_BYTES));
#pragma unroll
        for (int kk = 0; kk < KS / 16; ++kk) /* 32 bytes of K per step: +2 in the address field */
          umma(tmem, dh + 2 * kk, db + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&free_a[ai]);
        umma_commit(&free_b[bi]);
      }
      umma_commit(&acc_full); /* also the completion point of every MMA issued above */
    }
    __syncwarp();
  }

  /* ------------------------------------------------ epilogue (warps 2-9): TMEM -> registers ->
     the fused epilogue; lanes g and g + 8 of a strip meet through a shuffle.  With K split,
     every CTA stores its partial tile, and the CTA that arrives last for the tile adds the
     partials in split order (0, 1, ..., S - 1, whichever CTA that is) and runs the epilogue. */
  bool acc_ok = true;
  __shared__ int last_arrival;
  if (warp >= 2 && warp <= 9) {
    acc_ok = mb_wait(&acc_full, 0, deadline + 1000000000ull);
    tc_fence_after();
    const int q4 = warp & 3;                        /* TMEM lane quarter this warp may access */
    const int col0 = ((warp - 2) >> 2) * (NT / 2);  /* its half of the token columns */
    const int row = q4 * 32 + lane;                 /* row of the 128-row tile = TMEM lane */
    const int n = wt * BM + row;                    /* packed row */
    /* eight tokens at a time, every load of the eight issued before any store */
    auto finish = [&](int c0, const float (&v)[32]) {
#pragma unroll
      for (int cb = 0; cb < 32; cb += 8) {
        float va[8], vb[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          va[c] = v[cb + c];
          vb[c] = __shfl_down_sync(0xffffffffu, v[cb + c], 8);
        }
        if ((lane & 15) < 8)
          epilogue_tokens<EPI, 8>(ea, n >> 4, lane & 7, tok0 + c0 + cb, a.M, a.N, va, vb,
                                  EPI == EPI_QKV ? srow + c0 + cb : nullptr);
      }
    };
    if (a.splits == 1) {
      if (acc_ok && ok) {
#pragma unroll 1
        for (int c0 = col0; c0 < col0 + NT / 2; c0 += 32) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, v);
          finish(c0, v);
        }
      }
    } else {
      const int tile = (int)(blockIdx.y * gridDim.x + blockIdx.x);
      float* const wtile = a.ws + (size_t)tile * a.splits * NT * BM;
      if (acc_ok && ok) {
        float* const wp = wtile + (size_t)split * NT * BM;
#pragma unroll 1
        for (int c0 = col0; c0 < col0 + NT / 2; c0 += 32) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
          for (int c = 0; c < 32; ++c) __stcg(wp + (size_t)(c0 + c) * BM + row, v[c]);
        }
      }
      __threadfence();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (tid == 64) last_arrival = atomicAdd(&a.cnt[tile], 1) == a.splits - 1;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (last_arrival) {
        __threadfence();
#pragma unroll 1
        for (int c0 = col0; c0 < col0 + NT / 2; c0 += 32) {
          float v[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __ldcg(wtile + (size_t)(c0 + c) * BM + row);
#pragma unroll 1
          for (int sp = 1; sp < a.splits; ++sp) {
            const float* wp = wtile + (size_t)sp * NT * BM;
#pragma unroll
            for (int c = 0; c < 32; ++c) v[c] += __ldcg(wp + (size_t)(c0 + c) * BM + row);
          }
          finish(c0, v);
        }
        if (tid == 64) a.cnt[tile] = 0; /* ready for the next launch */
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if ((!ok || !acc_ok) && lane == 0) atomicOr(a.err, 8);
  if (warp == 10) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
  }
}

/* token tile of the wide regime: tiles of the weights x tiles of the tokens is the whole grid
   (K is never split, and the tile width does not change a row's summation order), so pick the
   width with the shortest estimated makespan: waves of CTAs x per-CTA time, a CTA's time per
   64-k stage being the larger of its dequantisation (~fixed) and its MMAs (~NT) */
inline int tc_ntile(const Ctx* c, const Tensor* w, int M) {
  const long long n_wt = (w->n_strips + 7) / 8, sm = c->n_sm > 0 ? c->n_sm : 148;
  const int cand[4] = {256, 192, 128, 64};
  int best_nt = 64;
  double best = -1.0;
  for (int i = 0; i < 4; ++i) {
    const long long ctas = n_wt * ((M + cand[i] - 1) / cand[i]);
    const double waves = (double)((ctas + sm - 1) / sm);
    const double cost = waves * std::max(320.0, 2.9 * cand[i]) + 0.02 * cand[i];
    if (best < 0 || cost < best) {
      best = cost;
      best_nt = cand[i];
    }
  }
  return best_nt;
}

/*
 * K splits for the 64-token tiles of the narrow regime (kGemvMaxRows < M < kTcWideRows): the
 * count that minimises (waves of weight tiles x splits) x (stages per split + fill), plus a
 * fixed cost for the partial-sum pass.  It depends on the matrix and the SM count only, never
 * on M, so every row of the regime is summed in the same order.
 */
inline int tc_splits(const Ctx* c, const Tensor* w) {
  const int n_wt = (w->n_strips + 7) / 8, T = w->tiles;
  const int spt = (w->type == ULB_TYPE_Q4_0 ? kQ40TileK : kQ4KTileK) / KS;
  int best_s = 1;
  long long best = -1;
  for (int s = 1; s <= std::min(16, T); ++s) {
    if ((size_t)n_wt * s * 64 * BM > c->tc_ws_floats || (s > 1 && n_wt > kTcCounters)) break;
    const long long waves = ((long long)n_wt * s + c->n_sm - 1) / c->n_sm;
    const long long cost = waves * ((long long)((T + s - 1) / s) * spt + 4) + (s > 1 ? 4 : 0);
    if (best < 0 || cost < best) {
      best = cost;
      best_s = s;
    }
  }
  return best_s;
}

/* cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link) */
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
int encode_fn(EncodeTiledFn* out) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q != cudaDriverEntryPointSuccess) err = cudaErrorNotSupported;
    fn = (EncodeTiledFn)p;
  });
  if (err != cudaSuccess || !fn) return cuda_error(err == cudaSuccess ? cudaErrorNotSupported : err,
                                                   "cuTensorMapEncodeTiled entry point", __FILE__, __LINE__);
  *out = fn;
  return ULB_OK;
}

template <int QT, int NT, int EPI>
int launch_tc3(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, const EpiArgs& ea, int splits) {
  using Cf = TcCfg<QT, NT>;
  static bool attr = false;
  if (!attr) {
    ULB_CUDA(cudaFuncSetAttribute(qgemm_tc_kernel<QT, NT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM));
    attr = true;
  }
  EncodeTiledFn enc;
  ULB_TRY(encode_fn(&enc));
  /* packed weights as u64 words [n_strips][tiles][TB / 8]; box = 144 words x 1 tile x 8 strips */
  CUtensorMap tw, tx;
  {
    const cuuint64_t dim[3] = {(cuuint64_t)(Cf::TB / 8), (cuuint64_t)w->tiles, (cuuint64_t)w->n_strips};
    const cuuint64_t str[2] = {(cuuint64_t)Cf::TB, (cuuint64_t)w->tiles * Cf::TB};
    const cuuint32_t box[3] = {(cuuint32_t)kTmaBox, 1, 8}, es[3] = {1, 1, 1};
    CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, w->dev, dim, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    ULB_CHECK(r == CUDA_SUCCESS, ULB_ECUDA, "qgemm_tc: weight tensor map (CUresult %d)", (int)r);
  }
  /* activations fp16 [M][ldx]; box = 64 k x NT tokens, 128-byte swizzle, rows >= M read as zero */
  {
    const cuuint64_t dim[2] = {(cuuint64_t)w->K, (cuuint64_t)M};
    const cuuint64_t str[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t box[2] = {(cuuint32_t)KS, (cuuint32_t)NT}, es[2] = {1, 1};
    CUresult r = enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)x, dim, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    ULB_CHECK(r == CUDA_SUCCESS, ULB_ECUDA, "qgemm_tc: activation tensor map (CUresult %d)", (int)r);
  }
  TcArgs a;
  a.tiles = w->tiles;
  a.n_strips = w->n_strips;
  a.N = w->N;
  a.M = M;
  a.splits = splits;
  a.ws = c->tc_ws;
  a.cnt = c->tc_cnt;
  a.err = c->dev_err;
  const int n_wt = (w->n_strips + 7) / 8, n_tt = (M + NT - 1) / NT;
  /* with K split, the token tiles go in launches whose partial sums fit the context's workspace */
  int per = n_tt;
  if (splits > 1) {
    per = (int)std::min<size_t>((size_t)n_tt, c->tc_ws_floats / ((size_t)n_wt * splits * NT * BM));
    per = std::min(per, kTcCounters / n_wt);
    ULB_CHECK(per >= 1, ULB_EUNSUPPORTED, "qgemm_tc: split workspace too small for %d x %d tiles", n_wt, splits);
  }
  for (int tt0 = 0; tt0 < n_tt; tt0 += per) {
    a.tt0 = tt0;
    cudaError_t e = launch_k(c, qgemm_tc_kernel<QT, NT, EPI>, dim3(n_wt, std::min(per, n_tt - tt0), splits),
                             dim3(TCW * 32), Cf::SMEM, tw, tx, a, ea);
    if (e != cudaSuccess) return cuda_error(e, "tensor-core GEMM launch", __FILE__, __LINE__);
  }
  return ULB_OK;
}

template <int QT, int EPI>
int launch_tc2(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, const EpiArgs& ea) {
  if (M < kTcWideRows) return launch_tc3<QT, 64, EPI>(c, w, x, M, ldx, ea, tc_splits(c, w));
  switch (tc_ntile(c, w, M)) {
    case 64: return launch_tc3<QT, 64, EPI>(c, w, x, M, ldx, ea, 1);
    case 128: return launch_tc3<QT, 128, EPI>(c, w, x, M, ldx, ea, 1);
    case 192: return launch_tc3<QT, 192, EPI>(c, w, x, M, ldx, ea, 1);
    default: return launch_tc3<QT, 256, EPI>(c, w, x, M, ldx, ea, 1);
  }
}

template <int EPI>
int launch_tc1(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, const EpiArgs& ea) {
  if (w->type == ULB_TYPE_Q4_0) return launch_tc2<ULB_TYPE_Q4_0, EPI>(c, w, x, M, ldx, ea);
  return launch_tc2<ULB_TYPE_Q4_K, EPI>(c, w, x, M, ldx, ea);
}

}  // namespace

int launch_qgemm_tc(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a) {
  ULB_CHECK(w && (w->type == ULB_TYPE_Q4_0 || w->type == ULB_TYPE_Q4_K), ULB_EINVAL, "qgemm_tc: weight type");
  ULB_CHECK(w->K % KS == 0, ULB_EUNSUPPORTED, "qgemm_tc: K=%d not a multiple of %d", w->K, KS);
  ULB_CHECK(ldx % 8 == 0 && ((uintptr_t)x & 15) == 0, ULB_EINVAL, "qgemm_tc: activations must be 16-byte aligned");
  if (M == 0) return ULB_OK;
  switch (epi) {
    case EPI_STORE: return launch_tc1<EPI_STORE>(c, w, x, M, ldx, a);
    case EPI_RESID: return launch_tc1<EPI_RESID>(c, w, x, M, ldx, a);
    case EPI_SWIGLU: return launch_tc1<EPI_SWIGLU>(c, w, x, M, ldx, a);
    case EPI_QKV: return launch_tc1<EPI_QKV>(c, w, x, M, ldx, a);
    default: return set_error(ULB_EINVAL, "qgemm_tc: bad epilogue %d", epi);
  }
}

}  // namespace ulb

ULB_TRACE_UNIT(qgemm_tc)
