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
 * Tensor-core flash decoding (B200, mma.sync.m16n8k16 with fp32 accumulate):
 *  - grid = (16-query tile, kv head, split of 256 keys x sequence); 4 warps per CTA, warp w
 *    owns keys [split*256 + 64w, +64): it stages that K / V block in shared memory with
 *    cp.async (XOR-swizzled 16-byte chunks, so ldmatrix reads are conflict-free), computes
 *    S = Q.K^T with Q split into hi + lo fp16 parts (two MMAs, ~22 bits of q kept), masks
 *    keys past each query's position, and accumulates O = P.V with P rounded to fp16 (the
 *    score registers are reused as A fragments);
 *  - a query tile packs the G heads of a GQA group times the rows of the sequence, so each
 *    K / V block is read once for all of them;
 *  - the 4 warp blocks merge in shared memory; with several splits each CTA writes a
 *    partial (max, sum, output) and the CTA that arrives last for its (sequence, tile, kv
 *    head) merges the splits in split order.
 * A row's key blocks and merge order depend only on its own position: blocks or splits past
 * it contribute exact zeros, so batching never changes a row's result.
 * head_dim 64 and 128; capacity <= 8192.
 */
#include <algorithm>
#include <climits>
#include <mutex>

#include "ulb_internal.h"

namespace ulb {

namespace {

constexpr int KB = 64;              /* keys per warp block */
constexpr int AW = 4;               /* warps per CTA */
constexpr int SPLITK = KB * AW;     /* keys per CTA = one split */
constexpr int MAXSPLIT = 32;        /* capacity <= 8192 */
constexpr int QT = 16;              /* queries per CTA: one m16 tile */
constexpr int kSchedMax = 256;      /* streaming form: sequences ordered longest first, up to this many */
constexpr float kLog2e = 1.44269504088896340736f;

struct AttnParams {
  int H, Hkv, hd, cap, G, rps, n_mt, max_splits, ldq, n_seq, n_groups;
  float scale2; /* softmax scale x log2(e): scores live in the base-2 domain */
  /* paged cache (max_pages > 0; one page = one key split): block table bt, NULL = identity */
  const int* bt;
  int max_pages;
  /* tree rows (speculation trees): row m sees the keys before tpref[m] and the keys
     tpref[m] + j for each set bit j of tmask[m] (its ancestors and itself); NULL = causal by
     position (key <= row_pos[m]) */
  const int* tpref;
  const unsigned long long* tmask;
};
static_assert(SPLITK == kKvPage, "a key split is one KV cache page");

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

/* 16-byte async copy; zero-fills the destination when !valid (nothing is read then) */
__device__ __forceinline__ void cp_async16z(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
/* C += A(16x16 f16, row) * B(16x8 f16, col), fp32 accumulate */
__device__ __forceinline__ void mma_acc(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
/* 16-byte chunk c of key row j is stored at chunk c ^ (j & 7): the 8 rows one ldmatrix
   phase reads fall in 8 different bank groups */
__device__ __forceinline__ int swz(int j, int c) { return c ^ (j & 7); }

/*
 * One CTA = one (sequence, kv head, 16-query tile, split of 256 keys); warp w scores the
 * tile against keys [split*256 + 64w, +64) with tensor cores and keeps that block's softmax
 * (max, sum, unnormalised output).  The 4 warp blocks merge in shared memory; with more
 * than one split, the CTA that finishes last for its (sequence, tile, kv head) merges the
 * splits in split order.  Queries: index qi = r * G + j is row r of the sequence, head
 * kv_head * G + j.
 */
/* all threads of every CTA of the cluster: the cluster's shared-memory writes are visible after */
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
/* the address in the shared memory of CTA `rank` of the cluster at this CTA's offset p */
__device__ __forceinline__ uint32_t cluster_addr(const void* p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster2(uint32_t a, float2 v) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(v.x), "f"(v.y) : "memory");
}

/*
 * The per-block arithmetic shared by both attention kernels (so a row gets the same bits from
 * either): staging of one 64-key block, Q as hi + lo fp16 fragments, the block's scores,
 * causal mask and softmax, P.V, the warp partial, the in-CTA merge of the 4 warp blocks of a
 * split and the merge of split partials in split order.
 */
/* rows [j0, j1) of a 64-key block into the swizzled buffer; rows >= nk are zero-filled */
template <int HD>
__device__ __forceinline__ void stage_rows(__half* dst, const __half* src, int nk, int j0, int j1, int lane) {
  constexpr int NCH = HD / 8;
  for (int i = lane; i < KB * NCH; i += 32) {
    const int j = i / NCH, c = i % NCH;
    if (j < j0 || j >= j1) continue;
    const bool ok = j < nk;
    const size_t off = ok ? (size_t)j * HD + c * 8 : 0;
    cp_async16z(dst + j * HD + swz(j, c) * 8, src + off, ok);
  }
}

/* Q as A fragments of rows qpa (g) / qpb (g + 8), split hi + lo into two fp16 parts so the
   scores keep ~22 bits of q */
template <int HD>
__device__ __forceinline__ void q_frags(const float* qpa, const float* qpb, bool va, bool vb, int t,
                                        uint32_t (&qh)[HD / 16][4], uint32_t (&ql)[HD / 16][4]) {
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const bool v = (r & 1) ? vb : va;
      const float* src = ((r & 1) ? qpb : qpa) + ks * 16 + 2 * t + (r >> 1) * 8;
      const float2 f = v ? *reinterpret_cast<const float2*>(src) : make_float2(0.f, 0.f);
      const __half2 h = __floats2half2_rn(f.x, f.y);
      const float2 hf = __half22float2(h);
      qh[ks][r] = *reinterpret_cast<const uint32_t*>(&h);
      ql[ks][r] = pack_h2(f.x - hf.x, f.y - hf.y);
    }
  }
}

/* scores of the tile against the 64 keys from kb0 in Ks, causal mask (key <= the query's
   position), the block softmax: s becomes exp2(s - m) (unnormalised P), l its row sums */
/* the visibility of `key` to a row: causal (key <= pos), or for a tree row the keys before
   its prefix end and the set bits of its mask after it */
template <bool TREE>
__device__ __forceinline__ bool key_visible(int key, int pos, int pref, unsigned long long mask) {
  if (!TREE) return key <= pos;
  if (key < pref) return true;
  const unsigned j = (unsigned)(key - pref);
  return j < 64u && ((mask >> j) & 1ull) != 0ull;
}

template <int HD, bool TREE = false>
__device__ __forceinline__ void score_block(const __half* Ks, const uint32_t (&qh)[HD / 16][4],
                                            const uint32_t (&ql)[HD / 16][4], int kb0, int pa, int pb, float scale2,
                                            int lane, float (&s)[8][4], float& mA, float& mB, float& lA, float& lB,
                                            int prA = 0, int prB = 0, unsigned long long mkA = 0ull,
                                            unsigned long long mkB = 0ull) {
  constexpr int KS = HD / 16;
  const int t = lane & 3;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
    const int key = nb * 8 + (lane & 7);
#pragma unroll
    for (int kp = 0; kp < KS / 2; ++kp) {
      uint32_t b0, b1, b2, b3;
      ldsm4(saddr(Ks + key * HD + swz(key, kp * 4 + (lane >> 3)) * 8), b0, b1, b2, b3);
      mma_acc(s[nb], qh[2 * kp], b0, b1);
      mma_acc(s[nb], ql[2 * kp], b0, b1);
      mma_acc(s[nb], qh[2 * kp + 1], b2, b3);
      mma_acc(s[nb], ql[2 * kp + 1], b2, b3);
    }
  }
  float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = kb0 + nb * 8 + 2 * t + e;
      s[nb][e] = key_visible<TREE>(key, pa, prA, mkA) ? s[nb][e] * scale2 : -INFINITY;
      s[nb][2 + e] = key_visible<TREE>(key, pb, prB, mkB) ? s[nb][2 + e] * scale2 : -INFINITY;
      mxA = fmaxf(mxA, s[nb][e]);
      mxB = fmaxf(mxB, s[nb][2 + e]);
    }
  mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
  mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
  mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
  mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
  float sA = 0.f, sB = 0.f;
#pragma unroll
  for (int nb = 0; nb < 8; ++nb)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      s[nb][e] = mxA == -INFINITY ? 0.f : exp2f(s[nb][e] - mxA);
      s[nb][2 + e] = mxB == -INFINITY ? 0.f : exp2f(s[nb][2 + e] - mxB);
      sA += s[nb][e];
      sB += s[nb][2 + e];
    }
  sA += __shfl_xor_sync(0xffffffffu, sA, 1);
  sA += __shfl_xor_sync(0xffffffffu, sA, 2);
  sB += __shfl_xor_sync(0xffffffffu, sB, 1);
  sB += __shfl_xor_sync(0xffffffffu, sB, 2);
  lA = sA;
  lB = sB;
  mA = mxA;
  mB = mxB;
}

/* O = P.V: P (fp16) as A fragments straight from the score registers */
template <int HD>
__device__ __forceinline__ void pv_block(const __half* Vs, const float (&s)[8][4], int lane, float (&o)[HD / 8][4]) {
  constexpr int DN = HD / 8;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint32_t pf[4] = {pack_h2(s[2 * kk][0], s[2 * kk][1]), pack_h2(s[2 * kk][2], s[2 * kk][3]),
                            pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                            pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
    const int key = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int dp = 0; dp < DN / 2; ++dp) {
      uint32_t b0, b1, b2, b3;
      ldsm4t(saddr(Vs + key * HD + swz(key, dp * 2 + (lane >> 4)) * 8), b0, b1, b2, b3);
      mma_acc(o[2 * dp], pf, b0, b1);
      mma_acc(o[2 * dp + 1], pf, b2, b3);
    }
  }
}

/* a warp block's (max, sum, output) of its 16 queries: pw[q * (HD + 2) + {0: m, 1: l, 2..: o}] */
template <int HD>
__device__ __forceinline__ void write_warp_partial(float* pw, int lane, float mA, float mB, float lA, float lB,
                                                   const float (&o)[HD / 8][4]) {
  constexpr int PST = HD + 2;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int d = 0; d < HD / 8; ++d) {
    *reinterpret_cast<float2*>(pw + g * PST + 2 + d * 8 + 2 * t) = make_float2(o[d][0], o[d][1]);
    *reinterpret_cast<float2*>(pw + (g + 8) * PST + 2 + d * 8 + 2 * t) = make_float2(o[d][2], o[d][3]);
  }
  if (t == 0) {
    pw[g * PST] = mA;
    pw[g * PST + 1] = lA;
    pw[(g + 8) * PST] = mB;
    pw[(g + 8) * PST + 1] = lB;
  }
}

/*
 * The merges, each split into a per-row step (the maxima, the sums and the factors, computed
 * once per query row) and a per-pair step (the output pairs of the row, which only apply the
 * row's factors), so no exponential is evaluated once per output element.
 *
 * In-CTA merge of a split's 4 warp partials, in warp order (warp w's partial starts at
 * part + w * wstride): row_factors gives f = {M, L, e_0 .. e_3} with M = max_w m_w,
 * e_w = exp2(m_w - M) (0 for a block without keys), L = the fmaf chain of l_w e_w;
 * merge_pair the fmaf chain of o_w e_w for output pair d2.
 */
constexpr int RF = AW + 2; /* floats of a row's factor record */
template <int HD>
__device__ __forceinline__ void row_factors(const float* part, size_t wstride, int qi, float* f) {
  constexpr int PST = HD + 2;
  float mw[AW], lw[AW];
#pragma unroll
  for (int w = 0; w < AW; ++w) {
    mw[w] = part[w * wstride + (size_t)qi * PST];
    lw[w] = part[w * wstride + (size_t)qi * PST + 1];
  }
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < AW; ++w) M = fmaxf(M, mw[w]);
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < AW; ++w) {
    const float e = mw[w] == -INFINITY ? 0.f : exp2f(mw[w] - M);
    L = __fmaf_rn(lw[w], e, L);
    f[2 + w] = e;
  }
  f[0] = M;
  f[1] = L;
}
template <int HD>
__device__ __forceinline__ float2 merge_pair(const float* part, size_t wstride, int qi, int d2, const float* f) {
  constexpr int PST = HD + 2;
  float2 o[AW];
#pragma unroll
  for (int w = 0; w < AW; ++w) o[w] = *reinterpret_cast<const float2*>(part + w * wstride + (size_t)qi * PST + 2 + 2 * d2);
  float ox = 0.f, oy = 0.f;
#pragma unroll
  for (int w = 0; w < AW; ++w) {
    ox = __fmaf_rn(o[w].x, f[2 + w], ox);
    oy = __fmaf_rn(o[w].y, f[2 + w], oy);
  }
  return make_float2(ox, oy);
}

/* Merge of split partials in split order, every form of the kernel with exactly this
   arithmetic: merge_row folds split partial (m, l) into the row's running (M, L) and returns
   the factors of the running and the new output (split 0 is taken as it is); merge_pair_next
   applies them to an output pair. */
struct MergeFac {
  float a, b;
};
__device__ __forceinline__ MergeFac merge_row(bool first, float m, float l, float& M, float& L) {
  if (first) {
    M = m;
    L = l;
    return MergeFac{0.f, 1.f};
  }
  const float Mn = fmaxf(M, m);
  const float a = M == -INFINITY ? 0.f : exp2f(M - Mn);
  const float b = m == -INFINITY ? 0.f : exp2f(m - Mn);
  L = __fmaf_rn(l, b, L * a);
  M = Mn;
  return MergeFac{a, b};
}
__device__ __forceinline__ void merge_pair_next(bool first, MergeFac f, float oxs, float oys, float& ox, float& oy) {
  if (first) {
    ox = oxs;
    oy = oys;
    return;
  }
  ox = __fmaf_rn(oxs, f.b, ox * f.a);
  oy = __fmaf_rn(oys, f.b, oy * f.a);
}

template <int HD, bool CL, bool TREE>
__global__ void __launch_bounds__(AW * 32, 1)
    attn_mma_kernel(AttnParams p, const float* __restrict__ q, const __half* __restrict__ kc,
                    const __half* __restrict__ vc, const int* __restrict__ row_seq, const int* __restrict__ row_pos,
                    __half* __restrict__ out, float* scratch, int* counters) {
  ULB_TRACE_KERNEL(kTrAttnSplit + (CL ? 1 : 0) + (TREE ? 2 : 0), HD);
  constexpr int KS = HD / 16; /* k-steps of Q.K^T */
  constexpr int DN = HD / 8;  /* n-tiles of the output */
  constexpr int PST = HD + 2; /* floats per query of a partial: m, l, o[HD] */
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  /* grid (tile, kv head, split x sequence group).  Without clusters the launch order runs
     through every head's split 0 first, so the CTAs with keys start before those past the
     sequences' ends; with clusters (CL) the max_splits CTAs of one (tile, head, group) are one
     cluster, split = the CTA's rank in it. */
  const int mt = blockIdx.x, kvh = blockIdx.y;
  const int split = CL ? blockIdx.z % p.max_splits : blockIdx.z / p.n_groups;
  const int gi = CL ? blockIdx.z / p.max_splits : blockIdx.z % p.n_groups;
  /* Rows' sequences and positions, and the cache rows before this forward's, were written
     before the previous kernel (the QKV GEMV) started: they are read, and those K / V rows
     requested, before griddepcontrol.wait; the rows this forward appended wait for it. */
  const int Q = p.G * p.rps, q0 = mt * QT, nq = min(QT, Q - q0);
  const int m0 = gi * p.rps;
  /* every index load of the CTA is issued before any is used: the tile's last position (one
     load per lane, lane < nq <= 16, then a warp max), the sequence, the lane's two query
     positions, so the CTA pays one memory latency here */
  const int qa = q0 + g, qb = q0 + g + 8; /* the lane's two query rows of the tile: g, g + 8 */
  const bool va = g < nq, vb = g + 8 < nq;
  int last_pos = lane < nq ? row_pos[m0 + (q0 + lane) / p.G] : 0;
  const int seq = row_seq[m0];
  const int pa = va ? row_pos[m0 + qa / p.G] : -1, pb = vb ? row_pos[m0 + qb / p.G] : -1;
  int prA = 0, prB = 0;
  unsigned long long mkA = 0ull, mkB = 0ull;
  if (TREE) {
    if (va) { prA = p.tpref[m0 + qa / p.G]; mkA = p.tmask[m0 + qa / p.G]; }
    if (vb) { prB = p.tpref[m0 + qb / p.G]; mkB = p.tmask[m0 + qb / p.G]; }
  }
  /* and the first position this forward wrote for the sequence (rows m0 .. m0 + rps - 1) */
  int first_new = lane < p.rps ? row_pos[m0 + lane] : INT_MAX;
  for (int r = lane + 32; r < p.rps; r += 32) first_new = min(first_new, row_pos[m0 + r]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    last_pos = max(last_pos, __shfl_xor_sync(0xffffffffu, last_pos, o));
    first_new = min(first_new, __shfl_xor_sync(0xffffffffu, first_new, o));
  }
  last_pos = max(0, min(last_pos, p.cap - 1)); /* positions past the cache never index it */
  const int n_splits = last_pos / SPLITK + 1;
  /* n_splits and seq are the same for every CTA of a cluster */
  const bool live = split < n_splits && (unsigned)seq < (unsigned)p.n_seq;
  if (!live) {
    /* a cluster's CTAs all pass its barrier (see the end of the kernel) */
    if (CL) cluster_sync();
    return;
  }

  const int kb0 = (split * AW + warp) * KB;
  /* the cache rows of this split: contiguous [S][Hkv][cap][hd], or page bt[seq][split] of the
     pool [page][Hkv][kKvPage][hd] (an unmapped page holds no keys: the split is masked out) */
  size_t kvoff;
  int page_ok = 1;
  if (p.max_pages > 0) {
    const int slot = seq * p.max_pages + split;
    const int page = p.bt ? p.bt[slot] : slot;
    page_ok = page >= 0;
    kvoff = (((size_t)max(page, 0) * p.Hkv + kvh) * kKvPage + warp * KB) * HD;
  } else {
    kvoff = (((size_t)seq * p.Hkv + kvh) * p.cap + max(kb0, 0)) * HD;
  }
  const int nk = page_ok ? min(KB, last_pos + 1 - kb0) : 0; /* keys of this warp's block (may be <= 0) */
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  float o[DN][4];
#pragma unroll
  for (int d = 0; d < DN; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  __half* Ks = reinterpret_cast<__half*>(sm) + (size_t)warp * 2 * KB * HD;
  __half* Vs = Ks + KB * HD;
  const __half* kg = kc + kvoff;
  const __half* vg = vc + kvoff;
  /* keys [0, n_old) of the block predate this forward, keys [n_old, nk) were just written */
  const int n_old = max(0, min(nk, first_new - kb0));
  if (nk > 0) {
    stage_rows<HD>(Ks, kg, nk, 0, n_old, lane);
    stage_rows<HD>(Vs, vg, nk, 0, n_old, lane);
  }
  pdl_wait();
  pdl_trigger();
  if (nk > 0) { /* the new keys, and zero fill past the last key */
    stage_rows<HD>(Ks, kg, nk, n_old, KB, lane);
    stage_rows<HD>(Vs, vg, nk, n_old, KB, lane);
    cp_commit();
  }
  const float* qpa = q + (size_t)(m0 + (va ? qa : q0) / p.G) * p.ldq + (kvh * p.G + (va ? qa : q0) % p.G) * HD;
  const float* qpb = q + (size_t)(m0 + (vb ? qb : q0) / p.G) * p.ldq + (kvh * p.G + (vb ? qb : q0) % p.G) * HD;
  uint32_t qh[KS][4], ql[KS][4];
  q_frags<HD>(qpa, qpb, va, vb, t, qh, ql);
  ULB_TRACE_MARK(0);

  if (nk > 0) {
    cp_wait_all();
    __syncwarp();
    ULB_TRACE_MARK(1);
    float s[8][4];
    score_block<HD, TREE>(Ks, qh, ql, kb0, pa, pb, p.scale2, lane, s, mA, mB, lA, lB, prA, prB, mkA, mkB);
    pv_block<HD>(Vs, s, lane, o);
  }
  ULB_TRACE_MARK(2);

  /* merge the 4 warp blocks (shared memory, warp order): each row's factors once, then its
     output pairs; rows past the tile's queries are never merged */
  float* part = reinterpret_cast<float*>(sm); /* [AW][QT][PST], over the K / V staging */
  __shared__ float rowf[QT][RF];
  __shared__ MergeFac sfac[QT][MAXSPLIT]; /* split-merge factors of each row */
  __shared__ float sinv[QT];
  __syncthreads();
  write_warp_partial<HD>(part + (size_t)warp * QT * PST, lane, mA, mB, lA, lB, o);
  __syncthreads();
  if (tid < nq) row_factors<HD>(part, (size_t)QT * PST, tid, rowf[tid]);
  __syncthreads();
  auto out_ptr = [&](int qi) {
    const int qq = q0 + qi;
    return reinterpret_cast<__half2*>(out + (size_t)(m0 + qq / p.G) * p.H * HD + (kvh * p.G + qq % p.G) * HD);
  };
  const int ti = (gi * p.n_mt + mt) * p.Hkv + kvh;
  float* gbase = scratch + (size_t)ti * p.max_splits * QT * PST;
  /* CL: the cluster's split partials [8][QT][PST] in split 0's shared memory, after its K / V
     staging and warp partials (which split 0 may still be using when the others write) */
  float* cslots = reinterpret_cast<float*>(sm + std::max((size_t)AW * 2 * KB * HD * sizeof(__half),
                                                         (size_t)AW * QT * PST * sizeof(float)));
  for (int it = tid; it < nq * (HD / 2); it += AW * 32) {
    const int qi = it / (HD / 2), d2 = it % (HD / 2);
    const float2 oo = merge_pair<HD>(part, (size_t)QT * PST, qi, d2, rowf[qi]);
    if (n_splits == 1) {
      const float L = rowf[qi][1];
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      out_ptr(qi)[d2] = __floats2half2_rn(oo.x * inv, oo.y * inv);
    } else if (CL) {
      /* into split 0's slot of this split: local, or a store to distributed shared memory */
      float* gp = cslots + ((size_t)split * QT + qi) * PST;
      if (split == 0) {
        if (d2 == 0) *reinterpret_cast<float2*>(gp) = make_float2(rowf[qi][0], rowf[qi][1]);
        *reinterpret_cast<float2*>(gp + 2 + 2 * d2) = oo;
      } else {
        if (d2 == 0) st_cluster2(cluster_addr(gp, 0), make_float2(rowf[qi][0], rowf[qi][1]));
        st_cluster2(cluster_addr(gp + 2 + 2 * d2, 0), oo);
      }
    } else {
      float* gp = gbase + (size_t)split * QT * PST + (size_t)qi * PST;
      if (d2 == 0) {
        gp[0] = rowf[qi][0];
        gp[1] = rowf[qi][1];
      }
      gp[2 + 2 * d2] = oo.x;
      gp[3 + 2 * d2] = oo.y;
    }
  }
  ULB_TRACE_MARK(3);
  if (CL) {
    /* one cluster barrier: every CTA has written its split partial into split 0's shared
       memory (release / acquire), after which no CTA's shared memory is read by another, so
       the others exit and split 0 merges the partials in split order (the arithmetic of the
       global merge below) */
    cluster_sync();
    ULB_TRACE_MARK(4);
    if (split != 0 || n_splits == 1) return;
    if (tid < nq) { /* the row's (max, sum) of every split, then the split-order merge */
      float mc[8], lc[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < n_splits) {
          const float2 ml = *reinterpret_cast<const float2*>(cslots + ((size_t)u * QT + tid) * PST);
          mc[u] = ml.x;
          lc[u] = ml.y;
        }
      float M = -INFINITY, L = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < n_splits) sfac[tid][u] = merge_row(u == 0, mc[u], lc[u], M, L);
      sinv[tid] = L > 0.f ? 1.0f / L : 0.f;
    }
    __syncthreads();
    for (int it = tid; it < nq * (HD / 2); it += AW * 32) {
      const int qi = it / (HD / 2), d2 = it % (HD / 2);
      float2 oc[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < n_splits) oc[u] = *reinterpret_cast<const float2*>(cslots + ((size_t)u * QT + qi) * PST + 2 + 2 * d2);
      float ox = 0.f, oy = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < n_splits) merge_pair_next(u == 0, sfac[qi][u], oc[u].x, oc[u].y, ox, oy);
      out_ptr(qi)[d2] = __floats2half2_rn(ox * sinv[qi], oy * sinv[qi]);
    }
    return;
  }
  if (n_splits == 1) return;
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (tid == 0) is_last = atomicAdd(&counters[ti], 1) == n_splits - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  /* merge of the splits in split order: each row's (max, sum) of every split and the factors
     first, eight splits' loads per memory round trip, then a thread per (query, output pair) */
  if (tid < nq) {
    float M = -INFINITY, L = 0.f;
    for (int c0 = 0; c0 < n_splits; c0 += 8) {
      float mc[8], lc[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u < n_splits) {
          const float* gp = gbase + (size_t)(c0 + u) * QT * PST + (size_t)tid * PST;
          mc[u] = __ldcg(gp);
          lc[u] = __ldcg(gp + 1);
        }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u < n_splits) sfac[tid][c0 + u] = merge_row(c0 + u == 0, mc[u], lc[u], M, L);
    }
    sinv[tid] = L > 0.f ? 1.0f / L : 0.f;
  }
  __syncthreads();
  for (int it = tid; it < nq * (HD / 2); it += AW * 32) {
    const int qi = it / (HD / 2), d2 = it % (HD / 2);
    float ox = 0.f, oy = 0.f;
    for (int c0 = 0; c0 < n_splits; c0 += 8) {
      float2 oc[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u < n_splits)
          oc[u] = __ldcg(reinterpret_cast<const float2*>(gbase + (size_t)(c0 + u) * QT * PST + (size_t)qi * PST + 2) + d2);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + u < n_splits) merge_pair_next(c0 + u == 0, sfac[qi][c0 + u], oc[u].x, oc[u].y, ox, oy);
    }
    out_ptr(qi)[d2] = __floats2half2_rn(ox * sinv[qi], oy * sinv[qi]);
  }
  if (tid == 0) counters[ti] = 0; /* ready for the next launch / graph replay */
}

/*
 * Streaming form for large batches (many sequences x heads, long caches): one CTA per
 * (TT 16-query tiles, kv head, sequence) walks all of its key splits in order, so a CTA never
 * exits between splits and the split partials never leave the SM.  Per split, warp (t, w)
 * scores tile t against 64-key block w exactly as attn_mma_kernel does (same staging, same
 * block arithmetic, same in-CTA merge), and each thread folds the split's partial of its
 * (query, output pair) items into a running merge in registers with merge_row /
 * merge_pair_next, the arithmetic of the other forms' split merges: a row gets the same bits
 * from either kernel.  (A split past a tile's last position adds exact zeros to its merge.)
 * The warps of tile 0 stage each 64-key block once for all TT tiles; K and V are a pipeline:
 * the next split's keys are requested as soon as this split's scores are computed, its values
 * as soon as P.V is done, so HBM keeps streaming while the SM computes.  (An L2 prefetch of
 * the split after that was measured slower: a bulk prefetch holds its warp while it issues.)
 * The warps sharing a block meet on a named barrier of their own.  Shared memory: K [4][64][HD] | V [4][64][HD] |
 * warp partials [TT][4][16][HD + 2].  No scratch, no counters.
 */
template <int HD, int TT>
__global__ void __launch_bounds__(TT * AW * 32, 1)
    attn_stream_kernel(AttnParams p, const float* __restrict__ q, const __half* __restrict__ kc,
                       const __half* __restrict__ vc, const int* __restrict__ row_seq,
                       const int* __restrict__ row_pos, __half* __restrict__ out) {
  ULB_TRACE_KERNEL(kTrAttnStream + TT, HD);
  constexpr int KS = HD / 16, DN = HD / 8, PST = HD + 2;
  constexpr int ITEMS = QT * (HD / 2) / (AW * 32); /* (query, output pair) items per thread of a tile */
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int tw = warp / AW, bw = warp % AW, ttid = tid - tw * AW * 32; /* tile of the warp, its block */
  const int mt = blockIdx.x * TT + tw, kvh = blockIdx.y;
  /* longest walks first: CTA z takes the sequence of rank z by (last position descending,
     index ascending), so the long sequences start in the first wave and the short ones fill
     the tail (for up to kSchedMax sequences; beyond that, launch order).  Only the order in
     which the work runs changes, never a result. */
  int gi = blockIdx.z;
  if (p.n_groups <= kSchedMax) {
    __shared__ int s_len[kSchedMax];
    __shared__ int s_gi;
    for (int u = tid; u < p.n_groups; u += TT * AW * 32) s_len[u] = row_pos[u * p.rps + p.rps - 1];
    __syncthreads();
    for (int u = tid; u < p.n_groups; u += TT * AW * 32) {
      const int lu = s_len[u];
      int rank = 0;
      for (int u2 = 0; u2 < p.n_groups; ++u2) {
        const int l2 = s_len[u2];
        rank += (l2 > lu || (l2 == lu && u2 < u)) ? 1 : 0;
      }
      if (rank == (int)blockIdx.z) s_gi = u;
    }
    __syncthreads();
    gi = s_gi;
  }
  const int Q = p.G * p.rps, q0 = mt * QT, nq = min(QT, Q - q0); /* nq <= 0: no such tile */
  const bool live = nq > 0;
  const int m0 = gi * p.rps;
  const int qa = q0 + g, qb = q0 + g + 8;
  const bool va = g < nq, vb = g + 8 < nq;
  /* the CTA's last position: over the TT tiles' rows (at most 32, one per lane) */
  const int cq0 = blockIdx.x * TT * QT, cnq = min(TT * QT, Q - cq0);
  int last_pos = lane < cnq ? row_pos[m0 + (cq0 + lane) / p.G] : 0;
  const int seq = row_seq[m0];
  const int pa = va ? row_pos[m0 + qa / p.G] : -1, pb = vb ? row_pos[m0 + qb / p.G] : -1;
  int first_new = lane < p.rps ? row_pos[m0 + lane] : INT_MAX;
  for (int r = lane + 32; r < p.rps; r += 32) first_new = min(first_new, row_pos[m0 + r]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    last_pos = max(last_pos, __shfl_xor_sync(0xffffffffu, last_pos, o));
    first_new = min(first_new, __shfl_xor_sync(0xffffffffu, first_new, o));
  }
  last_pos = max(0, min(last_pos, p.cap - 1));
  const int n_splits = last_pos / SPLITK + 1;
  if ((unsigned)seq >= (unsigned)p.n_seq) return;

  const bool stager = tw == 0; /* tile 0's warps stage the blocks for every tile */
  __half* const Ks = reinterpret_cast<__half*>(sm) + (size_t)bw * KB * HD;
  __half* const Vs = reinterpret_cast<__half*>(sm) + (size_t)(AW + bw) * KB * HD;
  float* const part = reinterpret_cast<float*>(sm + (size_t)2 * AW * KB * HD * sizeof(__half)) +
                      (size_t)tw * AW * QT * PST;
  /* the warps sharing block bw (one per tile): their own barrier; one warp: the warp itself */
  auto pair_sync = [&]() {
    if (TT == 1) __syncwarp();
    else asm volatile("bar.sync %0, %1;" ::"r"(1 + bw), "r"(TT * 32) : "memory");
  };
  /* block bw of split s: its first key, cache offset and key count (<= 0: none) */
  auto block_of = [&](int s, int& kb0, size_t& kvoff, int& nk) {
    kb0 = (s * AW + bw) * KB;
    int page_ok = 1;
    if (p.max_pages > 0) {
      const int slot = seq * p.max_pages + s;
      const int page = p.bt ? p.bt[slot] : slot;
      page_ok = page >= 0;
      kvoff = (((size_t)max(page, 0) * p.Hkv + kvh) * kKvPage + bw * KB) * HD;
    } else {
      kvoff = (((size_t)seq * p.Hkv + kvh) * p.cap + max(kb0, 0)) * HD;
    }
    nk = page_ok ? min(KB, last_pos + 1 - kb0) : 0;
  };
  int kb0, nk;
  size_t kvoff;
  block_of(0, kb0, kvoff, nk);
  {
    /* split 0: the rows that predate this forward before griddepcontrol.wait, the rest after */
    const int n_old = max(0, min(nk, first_new - kb0));
    if (stager && nk > 0) {
      stage_rows<HD>(Ks, kc + kvoff, nk, 0, n_old, lane);
      stage_rows<HD>(Vs, vc + kvoff, nk, 0, n_old, lane);
    }
    pdl_wait();
    pdl_trigger();
    if (stager && nk > 0) {
      stage_rows<HD>(Ks, kc + kvoff, nk, n_old, KB, lane);
      stage_rows<HD>(Vs, vc + kvoff, nk, n_old, KB, lane);
    }
    cp_commit();
  }
  const float* qpa = q + (size_t)(m0 + (va ? qa : 0) / p.G) * p.ldq + (kvh * p.G + (va ? qa : 0) % p.G) * HD;
  const float* qpb = q + (size_t)(m0 + (vb ? qb : 0) / p.G) * p.ldq + (kvh * p.G + (vb ? qb : 0) % p.G) * HD;
  uint32_t qh[KS][4], ql[KS][4];
  q_frags<HD>(qpa, qpb, va, vb, t, qh, ql);

  /* the running merge of the splits' partials: the row of thread ttid < nq keeps its (max,
     sum) and leaves the split's factors in shared memory; thread items it = ttid + 128 j of
     its tile keep their output pairs */
  __shared__ float rowf[TT][QT][RF];
  __shared__ MergeFac sfac[TT][QT];
  __shared__ float sinv[TT][QT];
  float RM = -INFINITY, RL = 0.f;
  float RX[ITEMS], RY[ITEMS];
  for (int s = 0; s < n_splits; ++s) {
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    float o[DN][4];
#pragma unroll
    for (int d = 0; d < DN; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
    float sc[8][4];
    /* keys of split s (the stager's groups pending: K_s, V_s; split 0: one group) */
    if (s == 0) asm volatile("cp.async.wait_group 0;" ::: "memory");
    else asm volatile("cp.async.wait_group 1;" ::: "memory");
    pair_sync();
    if (live && nk > 0) score_block<HD>(Ks, qh, ql, kb0, pa, pb, p.scale2, lane, sc, mA, mB, lA, lB);
    pair_sync();
    /* block bw of the next split: keys now, values once this split's are consumed */
    int kb1 = 0, nk1 = 0;
    size_t kvoff1 = 0;
    if (s + 1 < n_splits) {
      block_of(s + 1, kb1, kvoff1, nk1);
      if (stager && nk1 > 0) stage_rows<HD>(Ks, kc + kvoff1, nk1, 0, KB, lane);
    }
    cp_commit();
    asm volatile("cp.async.wait_group 1;" ::: "memory"); /* V_s */
    pair_sync();
    if (live && nk > 0) pv_block<HD>(Vs, sc, lane, o);
    pair_sync();
    if (stager && s + 1 < n_splits && nk1 > 0) stage_rows<HD>(Vs, vc + kvoff1, nk1, 0, KB, lane);
    cp_commit();
    write_warp_partial<HD>(part + (size_t)bw * QT * PST, lane, mA, mB, lA, lB, o);
    __syncthreads();
    if (ttid < nq) {
      row_factors<HD>(part, (size_t)QT * PST, ttid, rowf[tw][ttid]);
      sfac[tw][ttid] = merge_row(s == 0, rowf[tw][ttid][0], rowf[tw][ttid][1], RM, RL);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      const int it = ttid + j * AW * 32, qi = it / (HD / 2), d2 = it % (HD / 2);
      if (qi < nq) {
        const float2 oo = merge_pair<HD>(part, (size_t)QT * PST, qi, d2, rowf[tw][qi]);
        merge_pair_next(s == 0, sfac[tw][qi], oo.x, oo.y, RX[j], RY[j]);
      }
    }
    __syncthreads();
    kb0 = kb1;
    nk = nk1;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (!live) return;
  if (ttid < nq) sinv[tw][ttid] = RL > 0.f ? 1.0f / RL : 0.f;
  /* the tile's own warps: a named barrier per tile (ids 1..4 are the block pairs') */
  asm volatile("bar.sync %0, %1;" ::"r"(5 + tw), "r"(AW * 32) : "memory");
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    const int it = ttid + j * AW * 32, qi = it / (HD / 2), d2 = it % (HD / 2);
    if (qi < nq) {
      const float inv = sinv[tw][qi];
      const int qq = q0 + qi;
      reinterpret_cast<__half2*>(out + (size_t)(m0 + qq / p.G) * p.H * HD + (kvh * p.G + qq % p.G) * HD)[d2] =
          __floats2half2_rn(RX[j] * inv, RY[j] * inv);
    }
  }
}

void attn_geometry(const ulb_attn_desc* d, int M, int rps, int max_pos, AttnParams* p, int* n_groups) {
  p->H = d->n_head;
  p->Hkv = d->n_head_kv;
  p->hd = d->head_dim;
  p->cap = d->capacity;
  p->G = d->n_head / d->n_head_kv;
  p->rps = rps;
  p->n_mt = (p->G * rps + QT - 1) / QT;
  p->max_splits = max_pos / SPLITK + 1;
  p->scale2 = d->scale * kLog2e;
  p->n_seq = d->n_seq;
  *n_groups = M / rps;
  p->n_groups = *n_groups;
}

/* per-split form: K / V staging, the warp partials over it; with a cluster merge (cl) the
   cluster's split partials after both, written there by every CTA of the cluster */
size_t attn_smem(int hd, bool cl) {
  const size_t kv = (size_t)AW * 2 * KB * hd * sizeof(__half);
  const size_t part = (size_t)AW * QT * (hd + 2) * sizeof(float);
  return std::max(kv, part) + (cl ? (size_t)8 * QT * (hd + 2) * sizeof(float) : 0);
}
/* streaming form: K / V blocks of the 4 warp columns + the partials of TT tiles' warps */
size_t attn_stream_smem(int hd, int tt) {
  return (size_t)AW * 2 * KB * hd * sizeof(__half) + (size_t)tt * AW * QT * (hd + 2) * sizeof(float);
}
/* tiles per streaming CTA: two once a (kv head, sequence) has two or more query tiles */
int attn_stream_tiles(const AttnParams& p) { return p.n_mt >= 2 ? 2 : 1; }

/* Which form runs a launch: one CTA per key split (short latency for a few sequences: every
   split of every head in flight at once) or one CTA walking all splits of its (tile, head,
   sequence) (throughput for many sequences: no CTA turnover or merge traffic per split).
   Estimated from the waves each needs: a per-split CTA costs ~12 us of latency at one CTA
   per SM; a streaming CTA ~6 us plus ~2.5 us per split, two CTAs per SM at head_dim 64.
   Both forms give a row the same bits, so the choice never changes a result. */
bool attn_use_stream(const Ctx* c, const AttnParams& p, int ng, bool tree) {
  if (tree) return false; /* tree masks: the per-split form only */
  if (c && c->attn_form == ULB_ATTN_SPLIT) return false;
  if (c && c->attn_form == ULB_ATTN_STREAM) return true;
  const int n_sm = c ? c->n_sm : 0;
  if (p.max_splits < 2) return false;
  const int tt = attn_stream_tiles(p);
  const long long base = (long long)p.n_mt * p.Hkv * ng, sm = n_sm > 0 ? n_sm : 148;
  const long long sbase = (long long)((p.n_mt + tt - 1) / tt) * p.Hkv * ng, occ = p.hd == 64 && tt == 1 ? 2 : 1;
  const double t_split = (double)((base * p.max_splits + sm - 1) / sm) * 12.0;
  const double t_stream = (double)((sbase + sm * occ - 1) / (sm * occ)) * (6.0 + 2.5 * p.max_splits);
  return t_stream < 0.8 * t_split; /* a close call stays with the short-latency form */
}

}  // namespace

/*
 * With 2..8 splits (a cache of at most 2048 positions) the splits of one (tile, head, group)
 * run as one thread-block cluster and merge through distributed shared memory; the cluster
 * form is used once the device reports it can co-schedule such clusters.  Longer caches merge
 * through global memory (last CTA of the splits).
 */
template <int HD>
cudaError_t attn_setup(const bool** cl_ok_out) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  static bool cl_ok[9] = {false}; /* max_splits -> cluster form schedulable */
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(attn_mma_kernel<HD, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)attn_smem(HD, false));
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(attn_mma_kernel<HD, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)attn_smem(HD, true));
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(attn_mma_kernel<HD, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)attn_smem(HD, false));
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(attn_mma_kernel<HD, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)attn_smem(HD, true));
    for (int s = 2; s <= 8 && attr_err == cudaSuccess; ++s) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1, s);
      cfg.blockDim = dim3(AW * 32);
      cfg.dynamicSmemBytes = attn_smem(HD, true);
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension;
      a[0].val.clusterDim.x = 1;
      a[0].val.clusterDim.y = 1;
      a[0].val.clusterDim.z = s;
      cfg.attrs = a;
      cfg.numAttrs = 1;
      int n = 0;
      cl_ok[s] = cudaOccupancyMaxActiveClusters(&n, attn_mma_kernel<HD, true, false>, &cfg) == cudaSuccess && n > 0;
      cudaGetLastError();
    }
  });
  *cl_ok_out = cl_ok;
  return attr_err;
}

/* true when a launch with max_splits splits merges them in a thread-block cluster */
template <int HD>
cudaError_t attn_cluster_merge(int max_splits, bool* out) {
  const bool* cl_ok = nullptr;
  const cudaError_t e = attn_setup<HD>(&cl_ok);
  *out = e == cudaSuccess && max_splits >= 2 && max_splits <= 8 && cl_ok[max_splits];
  return e;
}

template <int HD>
cudaError_t launch_attn(Ctx* c, const AttnParams& p, int ng, const float* q, const __half* k, const __half* v,
                        const int* row_seq, const int* row_pos, __half* out, float* scratch, int* counters) {
  if (attn_use_stream(c, p, ng, p.tmask != nullptr)) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
      attr_err = cudaFuncSetAttribute(attn_stream_kernel<HD, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)attn_stream_smem(HD, 1));
      if (attr_err == cudaSuccess)
        attr_err = cudaFuncSetAttribute(attn_stream_kernel<HD, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)attn_stream_smem(HD, 2));
    });
    if (attr_err != cudaSuccess) return attr_err;
    if (attn_stream_tiles(p) == 2)
      return launch_k(c, attn_stream_kernel<HD, 2>, dim3((p.n_mt + 1) / 2, p.Hkv, ng), dim3(2 * AW * 32),
                      attn_stream_smem(HD, 2), p, q, k, v, row_seq, row_pos, out);
    return launch_k(c, attn_stream_kernel<HD, 1>, dim3(p.n_mt, p.Hkv, ng), dim3(AW * 32), attn_stream_smem(HD, 1), p,
                    q, k, v, row_seq, row_pos, out);
  }
  bool cl = false;
  const cudaError_t se = attn_cluster_merge<HD>(p.max_splits, &cl);
  if (se != cudaSuccess) return se;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_mt, p.Hkv, ng * p.max_splits);
  cfg.blockDim = dim3(AW * 32);
  cfg.dynamicSmemBytes = attn_smem(HD, cl);
  cfg.stream = c->stream;
  cudaLaunchAttribute a[2];
  a[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a[0].val.programmaticStreamSerializationAllowed = c->pdl ? 1 : 0;
  a[1].id = cudaLaunchAttributeClusterDimension;
  a[1].val.clusterDim.x = 1;
  a[1].val.clusterDim.y = 1;
  a[1].val.clusterDim.z = cl ? p.max_splits : 1;
  cfg.attrs = a;
  cfg.numAttrs = cl ? 2 : 1;
  auto kern = p.tmask ? (cl ? attn_mma_kernel<HD, true, true> : attn_mma_kernel<HD, false, true>)
                      : (cl ? attn_mma_kernel<HD, true, false> : attn_mma_kernel<HD, false, false>);
  prefer_max_shared((const void*)kern);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, q, k, v, row_seq, row_pos, out, scratch, counters);
  if (e == cudaSuccess) ++c->launches;
  return e;
}

int validate_attn_desc(const ulb_attn_desc* d, int M, int rps) {
  ULB_CHECK(d, ULB_EINVAL, "attention: NULL descriptor");
  ULB_CHECK(d->n_head > 0 && d->n_head_kv > 0 && d->n_head % d->n_head_kv == 0, ULB_EINVAL,
            "attention: n_head %d, n_head_kv %d (both > 0, n_head a multiple of n_head_kv)", d->n_head, d->n_head_kv);
  ULB_CHECK(d->head_dim == 64 || d->head_dim == 128, ULB_EUNSUPPORTED, "attention: head_dim %d (64 or 128)",
            d->head_dim);
  ULB_CHECK(d->capacity > 0 && d->n_seq > 0, ULB_EINVAL, "attention: capacity %d, n_seq %d", d->capacity, d->n_seq);
  ULB_CHECK(d->capacity <= SPLITK * MAXSPLIT, ULB_EUNSUPPORTED, "attention: capacity %d > %d", d->capacity,
            SPLITK * MAXSPLIT);
  ULB_CHECK(rps > 0 && M >= 0 && M % rps == 0, ULB_EINVAL, "attention: M=%d not a multiple of rows_per_seq=%d", M,
            rps);
  return ULB_OK;
}

int attention_scratch_need(Ctx* c, const ulb_attn_desc* d, int M, int rps, int max_pos, size_t* floats,
                           int* n_counters, bool tree, bool bound) {
  ULB_TRY(validate_attn_desc(d, M, rps));
  *floats = 0;
  *n_counters = 0;
  if (M == 0) return ULB_OK;
  AttnParams p{};
  int ng;
  attn_geometry(d, M, rps, max_pos, &p, &ng);
  /* bound: what the per-split form would need, whatever this shape's form -- a workspace sized
     by it serves every launch of up to this many rows, although the form of a smaller launch
     (a short prefill chunk, fewer sequences) may differ from this one's */
  if ((!bound && attn_use_stream(c, p, ng, tree)) || p.max_splits == 1) return ULB_OK;
  bool cl = false;
  const cudaError_t e = d->head_dim == 64 ? attn_cluster_merge<64>(p.max_splits, &cl)
                                          : attn_cluster_merge<128>(p.max_splits, &cl);
  if (e != cudaSuccess) return cuda_error(e, "attention setup", __FILE__, __LINE__);
  if (cl) return ULB_OK;
  *n_counters = ng * p.n_mt * p.Hkv;
  *floats = (size_t)ng * p.n_mt * p.Hkv * p.max_splits * QT * (size_t)(p.hd + 2);
  return ULB_OK;
}

int launch_attention(Ctx* c, const ulb_attn_desc* d, const float* q, int ldq, const __half* k,
                     const __half* v, const int* row_seq, const int* row_pos, int M, int rps,
                     __half* out, float* scratch, int* counters, size_t scratch_floats, int n_counters,
                     const int* bt, int max_pages, const int* tree_pref, const unsigned long long* tree_mask) {
  ULB_TRY(validate_attn_desc(d, M, rps));
  ULB_CHECK(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 && ldq % 4 == 0,
            ULB_EINVAL, "attention: q / k / v must be 16-byte aligned (ldq a multiple of 4)");
  if (M == 0) return ULB_OK;
  AttnParams p{};
  int ng;
  attn_geometry(d, M, rps, d->capacity - 1, &p, &ng);
  p.ldq = ldq;
  p.bt = bt;
  p.max_pages = max_pages;
  p.tpref = tree_pref;
  p.tmask = tree_mask;
  ULB_CHECK(!tree_mask == !tree_pref, ULB_EINVAL, "attention: tree rows need both prefix ends and masks");
  ULB_CHECK(max_pages == 0 || (long long)max_pages * kKvPage >= d->capacity, ULB_EINVAL,
            "attention: %d pages of %d positions per sequence cannot hold capacity %d", max_pages, kKvPage, d->capacity);
  int need_c = 0;
  size_t need = 0;
  ULB_TRY(attention_scratch_need(c, d, M, rps, d->capacity - 1, &need, &need_c, tree_mask != nullptr));
  ULB_CHECK(need == 0 || (scratch && counters && scratch_floats >= need && n_counters >= need_c), ULB_EINVAL,
            "attention: scratch %zu floats / %d counters, need %zu / %d", scratch_floats, n_counters, need, need_c);
  ULB_CHECK((long long)ng * p.max_splits <= 65535, ULB_EUNSUPPORTED, "attention: %d sequences x %d splits", ng,
            p.max_splits);
  cudaError_t e = d->head_dim == 64 ? launch_attn<64>(c, p, ng, q, k, v, row_seq, row_pos, out, scratch, counters)
                                    : launch_attn<128>(c, p, ng, q, k, v, row_seq, row_pos, out, scratch, counters);
  if (e != cudaSuccess) return cuda_error(e, "attention launch", __FILE__, __LINE__);
  return ULB_OK;
}

/* ------------------------------------------------------------------ allocation-free entry */
/*
 * Scratch of ulb_attention_noalloc lives in file-scope device arrays instead of memory the
 * call allocates: every GPU that loads this library holds them (8 MiB + 32 KiB) until the
 * process exits.  Host code cannot use the array names as device addresses; the addresses
 * are looked up once per device with cudaGetSymbolAddress.
 */
constexpr size_t kNoAllocScratchFloats = (size_t)2 << 20; /* 2 Mi floats = 8 MiB */
constexpr int kNoAllocCounters = 8192;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) int g_noalloc_counters[kNoAllocCounters];

namespace {
struct NoAllocDevice {
  bool ready = false;
  float* scratch = nullptr;
  int* counters = nullptr;
};
constexpr int kMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kMaxDevices];
std::mutex g_noalloc_mu;
}  // namespace

/* device addresses of the static scratch on the current device (set up on first use) */
static int noalloc_scratch(Ctx* c, float** scratch, int** counters) {
  ULB_CHECK(c->device >= 0 && c->device < kMaxDevices, ULB_EUNSUPPORTED, "device id %d", c->device);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[c->device];
  if (!d.ready) {
    void* s = nullptr;
    void* k = nullptr;
    ULB_CUDA(cudaGetSymbolAddress(&s, g_noalloc_scratch));
    ULB_CUDA(cudaGetSymbolAddress(&k, g_noalloc_counters));
    d.scratch = (float*)s;
    d.counters = (int*)k;
    d.ready = true;
  }
  *scratch = d.scratch;
  *counters = d.counters;
  return ULB_OK;
}

}  // namespace ulb

using namespace ulb;

extern "C" int ulb_attention_noalloc(ulb_ctx* ctx, const ulb_attn_desc* d, const float* q, const uint16_t* k,
                                     const uint16_t* v, const int32_t* row_seq, const int32_t* row_pos, int M,
                                     int rps, uint16_t* out) {
  ULB_CHECK(ctx && d && q && k && v && row_seq && row_pos && out, ULB_EINVAL, "ulb_attention_noalloc: NULL argument");
  ULB_TRY(validate_attn_desc(d, M, rps));
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  int nc = 0;
  size_t nf = 0;
  ULB_TRY(attention_scratch_need(c, d, M, rps, d->capacity - 1, &nf, &nc));
  ULB_CHECK(nf <= kNoAllocScratchFloats && nc <= kNoAllocCounters, ULB_EINVAL,
            "ulb_attention_noalloc: this shape needs %zu scratch floats and %d counters; the static scratch holds "
            "%zu floats and %d counters (use ulb_attention)",
            nf, nc, kNoAllocScratchFloats, kNoAllocCounters);
  float* scratch = nullptr;
  int* counters = nullptr;
  ULB_TRY(noalloc_scratch(c, &scratch, &counters));
  /* the arrays keep the previous call's contents: the split counters of a global merge must
     start at zero (the single-split and cluster forms read neither array) */
  if (nc > 0) ULB_CUDA(cudaMemsetAsync(counters, 0, (size_t)nc * sizeof(int), c->stream));
  return launch_attention(c, d, q, d->n_head * d->head_dim, (const __half*)k, (const __half*)v, row_seq, row_pos, M,
                          rps, (__half*)out, scratch, counters, kNoAllocScratchFloats, kNoAllocCounters);
}

extern "C" int ulb_attention_set_form(ulb_ctx* ctx, int form) {
  ULB_CHECK(ctx, ULB_EINVAL, "ulb_attention_set_form: NULL context");
  ULB_CHECK(form == ULB_ATTN_AUTO || form == ULB_ATTN_SPLIT || form == ULB_ATTN_STREAM, ULB_EINVAL,
            "ulb_attention_set_form: form %d (0 auto, 1 split, 2 stream)", form);
  ctx->c.attn_form = form;
  return ULB_OK;
}

extern "C" int ulb_attention_paged(ulb_ctx* ctx, const ulb_attn_desc* d, const float* q, const uint16_t* k_pool,
                                   const uint16_t* v_pool, const int32_t* block_table, int max_pages,
                                   const int32_t* row_seq, const int32_t* row_pos, int M, int rps, uint16_t* out) {
  ULB_CHECK(ctx && d && q && k_pool && v_pool && block_table && row_seq && row_pos && out, ULB_EINVAL,
            "ulb_attention_paged: NULL argument");
  ULB_TRY(validate_attn_desc(d, M, rps));
  ULB_CHECK(max_pages > 0 && (long long)max_pages * kKvPage >= d->capacity, ULB_EINVAL,
            "ulb_attention_paged: %d pages of %d positions per sequence, capacity %d", max_pages, kKvPage, d->capacity);
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  int nc = 0;
  size_t nf = 0;
  ULB_TRY(attention_scratch_need(c, d, M, rps, d->capacity - 1, &nf, &nc));
  float* scratch = nullptr;
  int* counters = nullptr;
  ULB_TRY(dev_alloc(c, (void**)&scratch, nf * sizeof(float)));
  int rc = dev_alloc(c, (void**)&counters, (size_t)nc * sizeof(int));
  if (rc == ULB_OK) {
    cudaError_t e = nc > 0 ? cudaMemsetAsync(counters, 0, (size_t)nc * sizeof(int), c->stream) : cudaSuccess;
    rc = e == cudaSuccess ? launch_attention(c, d, q, d->n_head * d->head_dim, (const __half*)k_pool,
                                             (const __half*)v_pool, row_seq, row_pos, M, rps, (__half*)out, scratch,
                                             counters, nf, nc, block_table, max_pages)
                          : cuda_error(e, "memset", __FILE__, __LINE__);
  }
  if (rc == ULB_OK) rc = check_device_errors(c);
  dev_free(c, counters, (size_t)nc * sizeof(int));
  dev_free(c, scratch, nf * sizeof(float));
  return rc;
}

extern "C" int ulb_attention(ulb_ctx* ctx, const ulb_attn_desc* d, const float* q, const uint16_t* k,
                             const uint16_t* v, const int32_t* row_seq, const int32_t* row_pos, int M,
                             int rps, uint16_t* out) {
  ULB_CHECK(ctx && d && q && k && v && row_seq && row_pos && out, ULB_EINVAL, "ulb_attention: NULL argument");
  ULB_TRY(validate_attn_desc(d, M, rps));
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  int nc = 0;
  size_t nf = 0;
  ULB_TRY(attention_scratch_need(c, d, M, rps, d->capacity - 1, &nf, &nc));
  float* scratch = nullptr;
  int* counters = nullptr;
  ULB_TRY(dev_alloc(c, (void**)&scratch, nf * sizeof(float)));
  int rc = dev_alloc(c, (void**)&counters, (size_t)nc * sizeof(int));
  if (rc == ULB_OK) {
    cudaError_t e = nc > 0 ? cudaMemsetAsync(counters, 0, (size_t)nc * sizeof(int), c->stream) : cudaSuccess;
    rc = e == cudaSuccess ? launch_attention(c, d, q, d->n_head * d->head_dim, (const __half*)k, (const __half*)v,
                                             row_seq, row_pos, M, rps, (__half*)out, scratch, counters, nf, nc)
                          : cuda_error(e, "memset", __FILE__, __LINE__);
  }
  if (rc == ULB_OK) rc = check_device_errors(c);
  dev_free(c, counters, (size_t)nc * sizeof(int));
  dev_free(c, scratch, nf * sizeof(float));
  return rc;
}

ULB_TRACE_UNIT(attention)
