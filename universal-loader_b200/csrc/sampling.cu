/*
 * sampling.cu — logit warping, draft-token sampling and speculative rejection sampling.
 *
 * Replaces InferenceEngine::sample_token (src/inference/inference_engine.cpp:340-367: an
 * unseeded inverse CDF over a zero logits vector), the intent of TextGenerator's
 * apply_temperature / apply_top_k / apply_top_p (src/api/gguf_loader.cpp:90-155), and
 * SpeculativeDecoder::verify_speculation (src/inference/speculative_decoder.cpp:89-110, a
 * token-match heuristic) with standard speculative rejection sampling (Leviathan et al.
 * 2023; Chen et al. 2023).
 *
 * Warp definition (identical in the CPU oracle): z = logit * iT with iT = 1/T rounded once;
 * top-k keeps z >= the k-th largest z; e = ulb_warp_exp(z - max z) (binary32, bit-identical
 * on host and device); top-p keeps tokens whose strictly-more-probable mass is below
 * R = floor(top_p * total mass), masses in 40-bit fixed point added as integers
 * (ulb_mass_fix), so the cut does not depend on the order of the additions; p = e / Z over
 * the kept set, Z summed in fp64.  Sampling is an inverse CDF over e in index order.  Keep
 * sets are decided on exact comparisons of z (the order-preserving integer key of z), so the
 * same logits give the same kept set on host and device.
 *
 * Selection of the top-k / top-p cut (B200): one pass over the row histograms it into 1024
 * bins of max z - z (the row's range spread over the bins, at least 32 bins per unit) with
 * integer atomics, which spread over many bins (no contended fp64 atomics); the bin holding
 * the cut is found by a block scan, a second pass compacts that bin's elements into shared
 * memory (one counter update per warp), and a sort of the candidates with a scan of their
 * weights finds the exact key.  Only a bin too large for the candidate buffer (a very flat
 * row) falls back to a radix select over the whole row.  The row is read from HBM once (the
 * argmax pass); the later passes find it in L2.
 *
 * Kernels: accept (one CTA per sequence, a single kernel per round: the walk over the round's
 * positions computes each p / q row's statistics -- max, keep threshold, normaliser, argmax --
 * when it reaches the row, prefetching the next rows into L2, then the accept test, residual /
 * bonus sampling and the commit; rows after the first rejection are never read); sample
 * (statistics + inverse CDF for the draft tokens); for trees, row_stats over every p / q row of
 * the trees in parallel and tree_decide (the walk of one sequence's tree).
 */
#include <algorithm>

#include "ulb_internal.h"

namespace ulb {

namespace {

constexpr int ST = 256;  /* threads per row CTA of the stats grid (many rows in flight) */
constexpr int RT = 1024; /* threads per row CTA of draft-token sampling (one row per CTA: latency-bound) */
constexpr int DT = 1024; /* threads per sequence CTA (decide: residual / bonus sampling) */

struct RowStats {
  float mx;    /* max z                                  */
  float thr;   /* keep iff z >= thr                      */
  double Z;    /* sum of exp(z - mx) over the kept set   */
  int amax;    /* argmax of the raw logits (lowest index) */
  int pad;
};

/* z = logit * iT with -0 folded to +0, so key order and float order agree; iT is 1 / T
   rounded once (a multiply per logit instead of a divide) */
__device__ __forceinline__ float zof(float x, float iT) { return __fadd_rn(__fmul_rn(x, iT), 0.0f); }

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unkey(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

/* Visit every element of a logits row as f(i, x): 128-bit loads when the row is 16-byte
   aligned and V % 4 == 0 (each thread walks float4s i = tid, tid + BT, ..., eight loads in
   flight, in that order whatever the unrolling), else scalar. */
template <int BT, typename F>
__device__ __forceinline__ void row_for_each(const float* __restrict__ l, int V, F f) {
  if ((((uintptr_t)l) & 15) == 0 && (V & 3) == 0) {
    const float4* l4 = reinterpret_cast<const float4*>(l);
    const int V4 = V >> 2;
    int i = threadIdx.x;
    for (; i + 7 * BT < V4; i += 8 * BT) { /* eight 16-byte loads in flight per thread */
      float4 a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = __ldg(l4 + i + u * BT);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int b = 4 * (i + u * BT);
        f(b, a[u].x); f(b + 1, a[u].y); f(b + 2, a[u].z); f(b + 3, a[u].w);
      }
    }
    if (i < V4) { /* the last up-to-eight float4s of the thread, all requested before any is used */
      float4 a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i + u * BT < V4) a[u] = __ldg(l4 + i + u * BT);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i + u * BT < V4) {
          const int b = 4 * (i + u * BT);
          f(b, a[u].x); f(b + 1, a[u].y); f(b + 2, a[u].z); f(b + 3, a[u].w);
        }
    }
  } else {
    int i = threadIdx.x;
    for (; i + 7 * BT < V; i += 8 * BT) {
      float a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = __ldg(l + i + u * BT);
#pragma unroll
      for (int u = 0; u < 8; ++u) f(i + u * BT, a[u]);
    }
    for (; i < V; i += BT) f(i, __ldg(l + i));
  }
}

template <int BT>
struct SmemRed {
  float f[BT / 32];
  int i[BT / 32];
  double d[BT / 32];
  unsigned long long u[BT / 32];
  unsigned long long hist_w[256]; /* radix-select weights (counts or fixed-point masses) */
  double seg[BT];
  uint32_t prefix;
  int found;
  double above;
  unsigned long long above_w;
};

/* top-k / top-p cut selection: histogram of max z - z, and the compacted cut bin */
constexpr int kSelBins = 1024;     /* bins of max z - z, width 1 / kSelBinScale */
constexpr float kSelBinScale = 32.f;
constexpr int kSelCap = 2048;      /* candidates of the cut bin held in shared memory */
struct SelSmem {
  unsigned long long bw[kSelBins]; /* weight per bin */
  uint32_t ck[kSelCap];            /* candidate keys */
  unsigned long long cw[kSelCap];  /* candidate weights */
  int n;                           /* candidates found (may exceed kSelCap) */
  int bin;                         /* the cut bin */
  unsigned long long before;       /* weight of the bins before it */
};

template <int BT>
__device__ float block_min(float v, SmemRed<BT>& s) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s.f[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = s.f[0];
#pragma unroll
  for (int w = 1; w < BT / 32; ++w) r = fminf(r, s.f[w]);
  return r;
}

template <int BT>
__device__ float block_max(float v, SmemRed<BT>& s) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s.f[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = s.f[0];
#pragma unroll
  for (int w = 1; w < BT / 32; ++w) r = fmaxf(r, s.f[w]);
  return r;
}

/* deterministic fp64 sum: per-thread partials reduced in a fixed tree */
template <int BT>
__device__ double block_sum_d(double v, SmemRed<BT>& s) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s.d[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = s.d[0];
#pragma unroll
  for (int w = 1; w < BT / 32; ++w) r += s.d[w];
  return r;
}

/* argmax, lowest index on ties; *lmin (if given): the smallest element, in the same pass */
template <int BT>
__device__ int block_argmax(const float* l, int V, SmemRed<BT>& s, float* lmin = nullptr) {
  float bv = -INFINITY, mn = INFINITY;
  int bi = 0x7fffffff;
  row_for_each<BT>(l, V, [&](int i, float x) {
    if (x > bv || (x == bv && i < bi)) { bv = x; bi = i; }
    mn = fminf(mn, x);
  });
  if (lmin) *lmin = block_min(mn, s);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) { s.f[threadIdx.x >> 5] = bv; s.i[threadIdx.x >> 5] = bi; }
  __syncthreads();
  bv = s.f[0]; bi = s.i[0];
  for (int w = 1; w < BT / 32; ++w)
    if (s.f[w] > bv || (s.f[w] == bv && s.i[w] < bi)) { bv = s.f[w]; bi = s.i[w]; }
  return bi == 0x7fffffff ? 0 : bi;
}

/* deterministic sum of unsigned 64-bit integers over the block */
template <int BT>
__device__ unsigned long long block_sum_u64(unsigned long long v, SmemRed<BT>& s) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s.u[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long r = 0;
#pragma unroll
  for (int w = 0; w < BT / 32; ++w) r += s.u[w];
  return r;
}

/*
 * Radix select over (key, weight) pairs, 8 bits a level: the key t with weight(keys > t) < R
 * <= weight(keys >= t), for 1 <= R <= the total weight.  visit(f) calls f(key, weight) for
 * every pair (the whole block calls it; each thread its share).  Weights add as integers.
 */
template <int BT, class Visit>
__device__ uint32_t radix_select(Visit visit, unsigned long long R, SmemRed<BT>& s) {
  uint32_t prefix = 0, mask = 0;
  unsigned long long above = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += BT) s.hist_w[b] = 0ull;
    __syncthreads();
    visit([&](uint32_t key, unsigned long long w) {
      if ((key & mask) == prefix) atomicAdd(&s.hist_w[(key >> shift) & 255u], w);
    });
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long a = above;
      int b = 255;
      for (; b > 0; --b) {
        if (a + s.hist_w[b] >= R) break;
        a += s.hist_w[b];
      }
      s.prefix = prefix | ((uint32_t)b << shift);
      s.above_w = a;
    }
    __syncthreads();
    prefix = s.prefix;
    above = s.above_w;
    mask |= 255u << shift;
    __syncthreads();
  }
  return prefix;
}

/* bin of z: floor((max z - z) * scale), clamped to the last bin (-inf and NaN land there).
   scale spreads the row's range over the bins (at least kSelBinScale bins per unit), so even a
   flat row puts few elements in a bin: the bins only locate the cut, whose key is then found
   exactly among the cut bin's elements */
__device__ __forceinline__ int sel_bin(float mx, float z, float scale) {
  const float d = __fmul_rn(__fsub_rn(mx, z), scale);
  return d < (float)(kSelBins - 1) ? (int)d : kSelBins - 1;
}
__device__ __forceinline__ float sel_scale(float mx, float zmin) {
  const float range = __fsub_rn(mx, zmin);
  const float sc = range > 0.f && range < INFINITY ? __fdiv_rn((float)(kSelBins - 1), range) : kSelBinScale;
  return fmaxf(sc, kSelBinScale);
}

/*
 * The key t of the cut among n (key, weight) candidates in shared memory: sorted by key,
 * largest first (a bitonic sort), the first whose cumulative weight reaches R, so that the
 * weight of the keys above t is below R and that of the keys from t up reaches it.  Weights
 * add as integers: the result does not depend on the order of equal keys.
 */
template <int BT>
__device__ uint32_t sorted_cut(uint32_t* ck, unsigned long long* cw, int n, unsigned long long R, SmemRed<BT>& s) {
  int N = 1;
  while (N < n) N <<= 1;
  for (int i = n + threadIdx.x; i < N; i += BT) { /* padding sorts last and weighs nothing */
    ck[i] = 0u;
    cw[i] = 0ull;
  }
  __syncthreads();
  for (int k = 2; k <= N; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < N; i += BT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const bool desc = (i & k) == 0; /* descending runs first: the whole array ends descending */
          const uint32_t a = ck[i], b = ck[ixj];
          if (desc ? a < b : a > b) {
            ck[i] = b;
            ck[ixj] = a;
            const unsigned long long t = cw[i];
            cw[i] = cw[ixj];
            cw[ixj] = t;
          }
        }
      }
      __syncthreads();
    }
  /* prefix sums of the weights in sorted order: thread t owns a contiguous run of per items */
  const int per = (N + BT - 1) / BT, i0 = threadIdx.x * per;
  unsigned long long mine = 0;
  for (int j = 0; j < per; ++j)
    if (i0 + j < N) mine += cw[i0 + j];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inc = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) s.u[warp] = inc;
  if (threadIdx.x == 0) s.prefix = ck[0];
  __syncthreads();
  unsigned long long cum = inc - mine;
  for (int w = 0; w < warp; ++w) cum += s.u[w];
  if (cum < R && cum + mine >= R) /* exactly one thread holds the crossing */
    for (int j = 0; j < per && i0 + j < N; ++j) {
      if (cum + cw[i0 + j] >= R) {
        s.prefix = ck[i0 + j];
        break;
      }
      cum += cw[i0 + j];
    }
  __syncthreads();
  const uint32_t t = s.prefix;
  __syncthreads();
  return t;
}

/*
 * The cut key: with weights w(key) (MASS: ulb_mass_fix of the warp weight; else 1) over the
 * elements whose key >= key_lo, the key t whose descending cumulative weight first reaches R,
 * where R = k (count) or ulb_topp_target(top_p, total mass) (MASS).
 */
template <int BT, bool MASS>
__device__ uint32_t select_cut(const float* l, int V, float iT, float mx, float scale, uint32_t key_lo, int k,
                               float top_p, SmemRed<BT>& s, SelSmem& sel) {
  auto weight = [&](float z) -> unsigned long long {
    return MASS ? (unsigned long long)ulb_mass_fix(ulb_warp_exp(__fsub_rn(z, mx))) : 1ull;
  };
  for (int b = threadIdx.x; b < kSelBins; b += BT) sel.bw[b] = 0ull;
  if (threadIdx.x == 0) sel.n = 0;
  __syncthreads();
  unsigned long long tot = 0;
  row_for_each<BT>(l, V, [&](int, float x) {
    const float z = zof(x, iT);
    if (fkey(z) >= key_lo) {
      const unsigned long long w = weight(z);
      tot += w;
      atomicAdd(&sel.bw[sel_bin(mx, z, scale)], w);
    }
  });
  tot = block_sum_u64(tot, s);
  ULB_TRACE_MARK(4);
  const unsigned long long R = MASS ? (unsigned long long)ulb_topp_target(top_p, tot) : (unsigned long long)k;
  /* the cut bin: block scan of the bins' weights (each thread a contiguous group of bins) */
  constexpr int PER = kSelBins / BT > 0 ? kSelBins / BT : 1;
  const int b0 = threadIdx.x * PER;
  unsigned long long mine = 0;
  for (int j = 0; j < PER; ++j)
    if (b0 + j < kSelBins) mine += sel.bw[b0 + j];
  unsigned long long inc = mine;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) s.u[warp] = inc;
  if (threadIdx.x == 0) s.found = kSelBins;
  __syncthreads();
  unsigned long long cum = inc - mine;
  for (int w = 0; w < warp; ++w) cum += s.u[w];
  if (b0 < kSelBins && cum < R && cum + mine >= R) { /* exactly one thread holds the crossing */
    for (int j = 0; j < PER; ++j) {
      if (cum + sel.bw[b0 + j] >= R) {
        sel.bin = b0 + j;
        sel.before = cum;
        break;
      }
      cum += sel.bw[b0 + j];
    }
  }
  __syncthreads();
  ULB_TRACE_MARK(5);
  const int cut = sel.bin;
  const unsigned long long before = sel.before;
  /* the cut bin's elements into shared memory (one slot counter update per warp and element
     step: the lanes that hold a candidate take consecutive slots) */
  row_for_each<BT>(l, V, [&](int, float x) {
    const float z = zof(x, iT);
    const uint32_t key = fkey(z);
    const bool hit = key >= key_lo && sel_bin(mx, z, scale) == cut;
    const unsigned act = __activemask();
    const unsigned m = __ballot_sync(act, hit);
    if (m) {
      const int leader = __ffs(m) - 1, lane = threadIdx.x & 31;
      int base = 0;
      if (lane == leader) base = atomicAdd(&sel.n, __popc(m));
      base = __shfl_sync(act, base, leader);
      if (hit) {
        const int slot = base + __popc(m & ((1u << lane) - 1u));
        if (slot < kSelCap) {
          sel.ck[slot] = key;
          sel.cw[slot] = weight(z);
        }
      }
    }
  });
  __syncthreads();
  ULB_TRACE_MARK(6);
  const int n = sel.n;
  if (n <= kSelCap) return sorted_cut<BT>(sel.ck, sel.cw, n, R - before, s);
  /* a very flat row: the cut bin does not fit, select over the whole row */
  return radix_select<BT>([&](auto f) {
    row_for_each<BT>(l, V, [&](int, float x) {
      const float z = zof(x, iT);
      const uint32_t key = fkey(z);
      if (key >= key_lo) f(key, weight(z));
    });
  }, R, s);
}

/* NEED_Z = false: the normaliser is not needed (draft sampling, whose inverse CDF sums the
   weights itself) and out.Z is left at 0 */
template <int BT, bool NEED_Z = true>
__device__ void compute_row_stats(const float* l, int V, const ulb_warp& w, RowStats& out, SmemRed<BT>& s,
                                  SelSmem& sel) {
  float lmin;
  const int amax = block_argmax(l, V, s, &lmin);
  ULB_TRACE_MARK(0);
  if (!(w.temperature > 0.f)) {
    if (threadIdx.x == 0) { out.mx = l[amax]; out.thr = -INFINITY; out.Z = 1.0; out.amax = amax; }
    return;
  }
  const float iT = __fdiv_rn(1.0f, w.temperature); /* inverse temperature */
  const float mx = zof(l[amax], iT); /* scaling by 1/T > 0 is monotone: max z = z of the max logit */
  const float scale = sel_scale(mx, zof(lmin, iT));
  uint32_t key_lo = 0;
  if (w.top_k > 0 && w.top_k < V) key_lo = select_cut<BT, false>(l, V, iT, mx, scale, 0u, w.top_k, 0.f, s, sel);
  if (w.top_p > 0.f && w.top_p < 1.f)
    key_lo = select_cut<BT, true>(l, V, iT, mx, scale, key_lo, 0, w.top_p, s, sel);
  ULB_TRACE_MARK(1);
  double Z = 0.0;
  if (NEED_Z) {
    double zs = 0.0;
    row_for_each<BT>(l, V, [&](int, float x) {
      const float z = zof(x, iT);
      if (fkey(z) >= key_lo) zs += (double)ulb_warp_exp(__fsub_rn(z, mx));
    });
    Z = block_sum_d(zs, s);
  }
  ULB_TRACE_MARK(2);
  if (threadIdx.x == 0) {
    out.mx = mx;
    out.thr = key_lo == 0 ? -INFINITY : unkey(key_lo);
    out.Z = Z;
    out.amax = amax;
  }
}

/* warped probability weight e (unnormalised) of token i under stats st */
__device__ __forceinline__ double warped_e(const float* l, int i, float iT, const RowStats& st) {
  const float z = zof(l[i], iT);
  if (!(z >= st.thr)) return 0.0;
  return (double)ulb_warp_exp(__fsub_rn(z, st.mx));
}

/*
 * Inverse CDF in index order over weights produced by wfun(i) (fp64, >= 0): with W the
 * total weight, returns the smallest i whose cumulative weight exceeds u * W, and W in
 * *total.  This form, for rows longer than kInvCdfMax<BT>: per-thread contiguous segments,
 * summed by a scan over the block.  One pass over the
 * weights plus a scan of the one segment that holds the target.
 */
template <int BT, typename WF>
__device__ int block_inv_cdf_seg(int V, float u, WF wfun, SmemRed<BT>& s, double* total) {
  const int seg = (V + BT - 1) / BT;
  const int b0 = threadIdx.x * seg, b1 = min(V, b0 + seg);
  double sum = 0.0;
#pragma unroll 8
  for (int i = b0; i < b1; ++i) sum += wfun(i);
  /* the segments' exclusive prefix sums: a scan inside each warp, then the warps' totals */
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double inc = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  double exc = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) exc = 0.0;
  __syncthreads();
  if (lane == 31) s.d[warp] = inc;
  if (threadIdx.x == 0) s.found = 0x7fffffff;
  __syncthreads();
  double W = 0.0, before = 0.0;
  for (int w2 = 0; w2 < BT / 32; ++w2) {
    if (w2 == warp) before = W;
    W += s.d[w2];
  }
  const double target = (double)u * W;
  const double cum = before + exc;
  /* the first lane of each warp whose segment ends past the target starts a walk of the warp,
     32 elements a step (a scan of their weights), through the rest of the warp's segments; the
     lowest crossing of all warps is the result */
  const unsigned past = __ballot_sync(0xffffffffu, b0 < b1 && cum + sum > target);
  if (past) {
    const int src = __ffs(past) - 1;
    const int w0 = __shfl_sync(0xffffffffu, b0, src), w1 = min(V, (warp * 32 + 32) * seg);
    double base = __shfl_sync(0xffffffffu, cum, src);
    for (int g0 = w0; g0 < w1; g0 += 32) {
      const int i = g0 + lane;
      const double wv = i < w1 ? wfun(i) : 0.0;
      double c = wv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, c, o);
        if (lane >= o) c += t;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, wv > 0.0 && base + c > target);
      if (hit) {
        if (lane == 0) atomicMin(&s.found, g0 + __ffs(hit) - 1);
        break;
      }
      base += __shfl_sync(0xffffffffu, c, 31);
    }
  }
  __syncthreads();
  int r = s.found;
  if (r == 0x7fffffff) { /* target at/above the total through rounding: last positive weight */
    __syncthreads();
    int last = -1;
    for (int i = threadIdx.x; i < V; i += BT)
      if (wfun(i) > 0.0) last = max(last, i);
#pragma unroll
    for (int o = 16; o; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    if ((threadIdx.x & 31) == 0) s.i[threadIdx.x >> 5] = last;
    __syncthreads();
    r = s.i[0];
    for (int w2 = 1; w2 < BT / 32; ++w2) r = max(r, s.i[w2]);
    if (r < 0) r = 0;
  }
  __syncthreads();
  if (total) *total = W;
  return r;
}

/*
 * Inverse CDF in index order, the form for rows of up to kInvCdfMax<BT> weights: each warp owns
 * a contiguous range of super-chunks (kInvCdfS chunks of 32 consecutive elements) whose
 * elements its lanes read together (coalesced, lane l the l-th of each chunk); a super-chunk's
 * weight sum (the lanes' sums, then a fixed butterfly, identical on every lane) is kept by lane
 * j of the warp for its j-th super-chunk, and the warp's total adds them in order.  A scan of
 * the warps' totals finds the warp holding the target, a scan of its super-chunk sums the
 * super-chunk, and a walk over that super-chunk's chunks (their weights computed again, a warp
 * scan each) the element.  Where the scans' roundings put the target past a range's last
 * positive weight, that weight's element is taken.
 */
constexpr int kInvCdfS = 8; /* chunks per super-chunk */
template <int BT> constexpr int kInvCdfMax = (BT / 32) * 32 * kInvCdfS * 32;
template <int BT, typename WF>
__device__ int block_inv_cdf_chunked(int V, float u, WF wfun, SmemRed<BT>& s, double* total) {
  constexpr int NW = BT / 32, SCE = kInvCdfS * 32; /* warps, elements per super-chunk */
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nsc = (V + SCE - 1) / SCE, spw = (nsc + NW - 1) / NW; /* super-chunks, per warp (<= 32) */
  const int s0 = warp * spw, s1 = min(nsc, s0 + spw);
  double mine = 0.0, wtot = 0.0;
  for (int sc = s0; sc < s1; ++sc) { /* warp-uniform */
    double v[kInvCdfS];
#pragma unroll
    for (int k = 0; k < kInvCdfS; ++k) {
      const int i = sc * SCE + k * 32 + lane;
      v[k] = i < V ? wfun(i) : 0.0;
    }
    double t = 0.0;
#pragma unroll
    for (int k = 0; k < kInvCdfS; ++k) t += v[k];
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (sc - s0 == lane) mine = t;
    wtot += t;
  }
  __syncthreads();
  if (lane == 0) s.d[warp] = wtot;
  if (threadIdx.x == 0) s.found = 0x7fffffff;
  __syncthreads();
  double W = 0.0, before = 0.0;
  for (int w2 = 0; w2 < NW; ++w2) {
    if (w2 == warp) before = W;
    W += s.d[w2];
  }
  const double target = (double)u * W;
  if (wtot > 0.0 && before <= target && target < before + wtot) { /* this warp holds the target */
    double c = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(0xffffffffu, c, o);
      if (lane >= o) c += t;
    }
    const unsigned pos = __ballot_sync(0xffffffffu, mine > 0.0);
    const unsigned hit = __ballot_sync(0xffffffffu, mine > 0.0 && before + c > target);
    int js;
    double base;
    if (hit) {
      js = __ffs(hit) - 1;
      base = before + __shfl_sync(0xffffffffu, c - mine, js); /* the super-chunks before it */
    } else { /* rounding: the last super-chunk with weight, its last positive element */
      js = pos ? 31 - __clz(pos) : 0;
      base = -INFINITY;
    }
    const int e0 = (s0 + js) * SCE;
    int found = -1, lastp = -1;
    for (int k = 0; k < kInvCdfS && found < 0; ++k) {
      const int i = e0 + k * 32 + lane;
      const double wv = i < V ? wfun(i) : 0.0;
      double cc = wv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, cc, o);
        if (lane >= o) cc += t;
      }
      const unsigned h = __ballot_sync(0xffffffffu, wv > 0.0 && base + cc > target);
      const unsigned p = __ballot_sync(0xffffffffu, wv > 0.0);
      if (p) lastp = e0 + k * 32 + 31 - __clz(p);
      if (h) found = e0 + k * 32 + __ffs(h) - 1;
      base += __shfl_sync(0xffffffffu, cc, 31);
    }
    if (lane == 0) s.found = found >= 0 ? found : (lastp >= 0 ? lastp : 0x7fffffff);
  }
  __syncthreads();
  int r = s.found;
  if (r == 0x7fffffff) { /* target at/above the total through rounding: last positive weight */
    __syncthreads();
    int last = -1;
    for (int i = threadIdx.x; i < V; i += BT)
      if (wfun(i) > 0.0) last = max(last, i);
#pragma unroll
    for (int o = 16; o; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    if ((threadIdx.x & 31) == 0) s.i[threadIdx.x >> 5] = last;
    __syncthreads();
    r = s.i[0];
    for (int w2 = 1; w2 < NW; ++w2) r = max(r, s.i[w2]);
    if (r < 0) r = 0;
  }
  __syncthreads();
  if (total) *total = W;
  return r;
}

/* the inverse CDF of a row (see the two forms) */
template <int BT, typename WF>
__device__ int block_inv_cdf(int V, float u, WF wfun, SmemRed<BT>& s, double* total) {
  if (V <= kInvCdfMax<BT>) return block_inv_cdf_chunked<BT>(V, u, wfun, s, total);
  return block_inv_cdf_seg<BT>(V, u, wfun, s, total);
}

__device__ __forceinline__ float rng_u(uint64_t seed, uint32_t round, uint32_t seq, uint32_t slot, uint32_t tag) {
  return ulb_uniform(seed, round, seq, slot, tag);
}

/* ------------------------------------------------------------------ kernels */

/* one CTA of BT threads per row: draft / first-token sampling. out[row * out_stride] = token.
   Rows run with RT = 1024 threads, so a row is requested in about one round trip and its
   passes have four times the threads of a stats row (the normaliser Z of a sampled row is
   summed in another order than stats_kernel's, which moves it by at most an fp64 ulp). */
template <int BT>
__global__ void __launch_bounds__(BT) sample_kernel(const float* __restrict__ logits, int V, int ld, ulb_warp w,
                                                    uint64_t seed, const uint32_t* dev_round, uint32_t round,
                                                    uint32_t slot, uint32_t tag, uint32_t seq_base, int32_t* out,
                                                    int out_stride) {
  ULB_TRACE_KERNEL(kTrSample, V);
  __shared__ SmemRed<BT> s;
  __shared__ SelSmem sel;
  __shared__ RowStats st;
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const float* l = logits + (size_t)row * ld;
  compute_row_stats<BT, false>(l, V, w, st, s, sel);
  __syncthreads();
  int tok;
  if (!(w.temperature > 0.f)) {
    tok = st.amax;
  } else {
    const uint32_t seq = seq_base + (uint32_t)row;
    const uint32_t r = dev_round ? dev_round[seq] : round;
    const float u = rng_u(seed, r, seq, slot, tag);
    const float iT = __fdiv_rn(1.0f, w.temperature); /* inverse temperature */
    const RowStats stc = st;
    tok = block_inv_cdf(V, u, [&](int i) { return warped_e(l, i, iT, stc); }, s, nullptr);
  }
  ULB_TRACE_MARK(3);
  if (threadIdx.x == 0) out[(size_t)row * out_stride] = tok;
}

/* stats for np p rows followed by nq q rows */
__global__ void __launch_bounds__(ST) stats_kernel(const float* __restrict__ p, const float* __restrict__ q, int np,
                                                   int nq, int V, ulb_warp w, RowStats* __restrict__ out) {
  ULB_TRACE_KERNEL(kTrStats, 0);
  __shared__ SmemRed<ST> s;
  __shared__ SelSmem sel;
  __shared__ RowStats st;
  pdl_wait();
  pdl_trigger();
  /* persistent: few rows in flight per SM, so a row read by the max pass is still in L2
     when the later passes read it again */
  const int rows = np + nq;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* l = row < np ? p + (size_t)row * V : q + (size_t)(row - np) * V;
    compute_row_stats(l, V, w, st, s, sel);
    __syncthreads();
    if (threadIdx.x == 0) out[row] = st;
    __syncthreads();
  }
}

struct SpecCommit {
  int32_t* hist;     /* [B][hist_len] committed tokens (prompt first)      */
  int hist_len;
  int32_t* L;        /* [B] committed length                                 */
  int32_t* done;     /* [B]                                                  */
  const int32_t* prompt_len; /* [B]                                          */
  int max_new;
  uint32_t* round;   /* [B] per-sequence round counter, incremented here     */
  unsigned long long* stats; /* [4] (unused), drafted, accepted, committed  */
  int32_t* active;   /* [B] rounds in which the sequence was still decoding   */
  /* per-round records [B][log_rounds][log_stride] (ULB_SPEC_REC_* layout of ulb.h), or NULL */
  int32_t* log;
  int log_rounds, log_stride;
};

/* the logits rows a walk may need next, on their way to L2 while it works on this one: the
   16-byte-aligned part of the row (the bulk prefetch takes 16-byte-aligned addresses and
   sizes; a row of a vocabulary that is not a multiple of 4 starts unaligned) */
__device__ __forceinline__ void prefetch_row_l2(const float* row, int V) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(row), a1 = a0 + (uintptr_t)V * 4u;
  const uintptr_t s0 = (a0 + 15u) & ~(uintptr_t)15u, e0 = a1 & ~(uintptr_t)15u;
  for (uintptr_t o = s0 + (uintptr_t)threadIdx.x * 32768u; o < e0; o += (uintptr_t)blockDim.x * 32768u) {
    const uint32_t len = e0 - o < 32768u ? (uint32_t)(e0 - o) : 32768u;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(o), "r"(len) : "memory");
  }
}

/*
 * Rejection sampling of one sequence's round in a single kernel (one CTA per sequence): the
 * walk computes a row's warp statistics (max, keep threshold, normaliser, argmax) only when
 * it reaches the row -- p_i, and q_i unless greedy -- and stops at the first rejection, so
 * each row is read once and rows past the first rejection are never read.  The next
 * position's rows are prefetched into L2 while this one is decided.
 */
__global__ void __launch_bounds__(DT) accept_kernel(const float* __restrict__ p, const float* __restrict__ q,
                                                    const int32_t* __restrict__ draft, int B, int k, int V,
                                                    ulb_warp w, uint64_t seed, const uint32_t* dev_round,
                                                    uint32_t round, int32_t* out_tokens, int32_t* out_n,
                                                    SpecCommit cm) {
  ULB_TRACE_KERNEL(kTrAccept, 0);
  __shared__ SmemRed<DT> s;
  __shared__ SelSmem sel;
  __shared__ RowStats st_p, st_q;
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const bool greedy = !(w.temperature > 0.f);
  const float iT = greedy ? 1.f : __fdiv_rn(1.0f, w.temperature); /* inverse temperature */
  const uint32_t rnd = dev_round ? dev_round[b] : round;
  int n = 0, tok = -1;
  /* target probability (under the warp) of each committed token, for the round record (which
     the loop keeps for k <= kMaxLoggedK; ulb_spec_accept may pass a larger k and logs nothing) */
  constexpr int kMaxLoggedK = 16;
  float pcommit[kMaxLoggedK + 1];
  auto note_p = [&](int j, float v) {
    if (j <= kMaxLoggedK) pcommit[j] = v;
  };
  auto prow = [&](int i) { return p + ((size_t)b * (k + 1) + i) * V; };
  auto qrow = [&](int i) { return q + ((size_t)b * k + i) * V; };
  for (int i = 0; i < k; ++i) {
    const int x = draft[b * k + i];
    const float* pl = prow(i);
    prefetch_row_l2(prow(i + 1), V);
    if (!greedy) {
      prefetch_row_l2(qrow(i), V);
      if (i + 1 < k) prefetch_row_l2(qrow(i + 1), V);
    }
    compute_row_stats(pl, V, w, st_p, s, sel);
    __syncthreads();
    const RowStats sp = st_p;
    if (greedy) {
      note_p(n, 1.0f);
      if (x == sp.amax) { ++n; continue; }
      tok = sp.amax;
      break;
    }
    const float* ql = qrow(i);
    compute_row_stats(ql, V, w, st_q, s, sel);
    __syncthreads();
    const RowStats sq = st_q;
    const bool in_vocab = (unsigned)x < (unsigned)V; /* a token outside the vocabulary is rejected */
    const double px = in_vocab ? warped_e(pl, x, iT, sp) / sp.Z : 0.0;
    const double qx = in_vocab ? warped_e(ql, x, iT, sq) / sq.Z : 0.0;
    const float u = rng_u(seed, rnd, (uint32_t)b, (uint32_t)i, ULB_RNG_ACCEPT);
    note_p(n, (float)px);
    if ((double)u * qx < px) { ++n; continue; }
    /* residual norm(max(0, p - q)), as max(0, e_p Z_q - e_q Z_p) = Z_p Z_q max(0, p - q) */
    auto resid = [&](int v) {
      const double r = warped_e(pl, v, iT, sp) * sq.Z - warped_e(ql, v, iT, sq) * sp.Z;
      return r > 0.0 ? r : 0.0;
    };
    const float u2 = rng_u(seed, rnd, (uint32_t)b, (uint32_t)i, ULB_RNG_RESID);
    double R = 0.0;
    tok = block_inv_cdf(V, u2, resid, s, &R);
    if (!(R > 0.0)) tok = block_inv_cdf(V, u2, [&](int v) { return warped_e(pl, v, iT, sp); }, s, nullptr);
    note_p(n, (float)(warped_e(pl, tok, iT, sp) / sp.Z));
    break;
  }
  if (tok < 0) {
    const float* pl = prow(k);
    compute_row_stats(pl, V, w, st_p, s, sel);
    __syncthreads();
    const RowStats sp = st_p;
    if (greedy) {
      tok = sp.amax;
      note_p(n, 1.0f);
    } else {
      const float u2 = rng_u(seed, rnd, (uint32_t)b, (uint32_t)k, ULB_RNG_RESID);
      tok = block_inv_cdf(V, u2, [&](int v) { return warped_e(pl, v, iT, sp); }, s, nullptr);
      note_p(n, (float)(warped_e(pl, tok, iT, sp) / sp.Z));
    }
  }
  if (threadIdx.x != 0) return;
  if (out_tokens) {
    for (int i = 0; i < n; ++i) out_tokens[b * (k + 1) + i] = draft[b * k + i];
    out_tokens[b * (k + 1) + n] = tok;
    for (int i = n + 1; i <= k; ++i) out_tokens[b * (k + 1) + i] = -1;
  }
  if (out_n) out_n[b] = n;
  if (cm.hist) {
    if (!cm.done[b]) {
      const int L = cm.L[b];
      int32_t* h = cm.hist + (size_t)b * cm.hist_len;
      for (int i = 0; i < n; ++i) h[L + i] = draft[b * k + i];
      h[L + n] = tok;
      cm.L[b] = L + n + 1;
      if (L + n + 1 - cm.prompt_len[b] >= cm.max_new) cm.done[b] = 1;
      atomicAdd(&cm.stats[1], (unsigned long long)k);
      atomicAdd(&cm.stats[2], (unsigned long long)n);
      atomicAdd(&cm.stats[3], (unsigned long long)(n + 1));
      const int a = cm.active[b];
      if (cm.log && a < cm.log_rounds && k <= kMaxLoggedK) {
        int32_t* r = cm.log + ((size_t)b * cm.log_rounds + a) * cm.log_stride;
        r[ULB_SPEC_REC_N_ACCEPTED] = n;
        r[ULB_SPEC_REC_TOKEN] = tok;
        r[ULB_SPEC_REC_POSITION] = L;
        r[ULB_SPEC_REC_K] = k;
        for (int i = 0; i < k; ++i) r[ULB_SPEC_REC_DRAFTS + i] = draft[b * k + i];
        for (int i = 0; i <= n; ++i) r[ULB_SPEC_REC_DRAFTS + k + i] = __float_as_int(pcommit[i]);
      }
      cm.active[b] = a + 1;
    }
    cm.round[b] = rnd + 1;
  }
}

/* ------------------------------------------------------------------ speculation trees */
/* argmax over the row, lowest index on ties, skipping the n indices in excl */
template <int BT>
__device__ int block_argmax_excl(const float* l, int V, const int* excl, int n, SmemRed<BT>& s) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += BT) {
    bool skip = false;
    for (int j = 0; j < n; ++j) skip |= excl[j] == i;
    const float x = l[i];
    if (!skip && (x > bv || (x == bv && i < bi))) { bv = x; bi = i; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) { s.f[threadIdx.x >> 5] = bv; s.i[threadIdx.x >> 5] = bi; }
  __syncthreads();
  bv = s.f[0]; bi = s.i[0];
  for (int w = 1; w < BT / 32; ++w)
    if (s.f[w] > bv || (s.f[w] == bv && s.i[w] < bi)) { bv = s.f[w]; bi = s.i[w]; }
  __syncthreads();
  return bi == 0x7fffffff ? 0 : bi;
}

/*
 * The children of the tree nodes of one level from the draft's logits of their parents: one
 * CTA per parent row (row m of the level: sequence m / w^d, parent rank m % w^d; level 0 is
 * the root).  Greedy: the w most probable tokens in order (lowest index on ties); sampled: w
 * independent draws from the warped q, child c with the uniform (round, sequence, slot c,
 * draft tag).  tokens [S][N] get the children's tokens.
 */
__global__ void __launch_bounds__(RT) tree_children_kernel(const float* __restrict__ logits, int V, int w, int d,
                                                           ulb_warp wp, uint64_t seed,
                                                           const uint32_t* __restrict__ dev_round, int N,
                                                           int32_t* tokens) {
  ULB_TRACE_KERNEL(kTrTreeChildren, 0);
  __shared__ SmemRed<RT> s;
  __shared__ SelSmem sel;
  __shared__ RowStats st;
  __shared__ int picked[kTreeMaxWidth];
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  int per = 1;
  for (int j = 0; j < d; ++j) per *= w;
  const int seq = m / per, r = m % per;
  const int c0 = d == 0 ? 0 : tree_first(w, d + 1) + r * w;
  const float* l = logits + (size_t)m * V;
  if (!(wp.temperature > 0.f)) {
    for (int c = 0; c < w; ++c) {
      const int t = block_argmax_excl<RT>(l, V, picked, c, s);
      if (threadIdx.x == 0) picked[c] = t;
      __syncthreads();
    }
  } else {
    compute_row_stats(l, V, wp, st, s, sel);
    __syncthreads();
    const float iT = __fdiv_rn(1.0f, wp.temperature);
    const RowStats stc = st;
    const uint32_t rnd = dev_round ? dev_round[seq] : 0u;
    for (int c = 0; c < w; ++c) {
      const float u = rng_u(seed, rnd, (uint32_t)seq, (uint32_t)(c0 + c), ULB_RNG_DRAFT);
      const int t = block_inv_cdf(V, u, [&](int i) { return warped_e(l, i, iT, stc); }, s, nullptr);
      if (threadIdx.x == 0) picked[c] = t;
      __syncthreads();
    }
  }
  if (threadIdx.x < w) tokens[(size_t)seq * N + c0 + threadIdx.x] = picked[threadIdx.x];
}

struct TreeShape {
  int w, D, N, NI;
  /* q rows: level-major (the loop: level 0 = the S roots, then level d's S * w^d rows) or
     sequence-major [S][1 + NI] (ulb_spec_tree_accept) */
  bool q_level_major;
  int S;
};
/* q row of (sequence b, node u; u < 0 = the root) */
__device__ __forceinline__ int tree_qrow(const TreeShape& t, int b, int u) {
  if (!t.q_level_major) return b * (1 + t.NI) + 1 + u;
  if (u < 0) return b;
  const int d = tree_depth(t.w, u);
  int per = 1;
  for (int j = 0; j < d; ++j) per *= t.w;
  return t.S * (1 + tree_first(t.w, d)) + b * per + (u - tree_first(t.w, d));
}

/* outputs of a tree round: the accepted nodes [B][D] (-1 after), their count, the correction /
   bonus token, and for the cache compaction [B][2 + D]: the length before the round, n, path */
struct TreeOut {
  int32_t* path;
  int32_t* n;
  int32_t* tok;
  int32_t* comp;
};

/*
 * The walk of one sequence's tree, one CTA per sequence (multi-candidate speculative sampling;
 * the arithmetic of orc_tree_accept): the root's children are tested in order against p_root
 * (and the residuals left by each rejection), the first accepted one becomes the next node,
 * and so on; the correction comes from the last residual, the bonus of a leaf from its p.
 * With a commit struct the committed tokens go to the history as in decide_kernel.
 */
__global__ void __launch_bounds__(DT) tree_decide_kernel(const float* __restrict__ p, const float* __restrict__ q,
                                                         const int32_t* __restrict__ tokens,
                                                         const RowStats* __restrict__ rs, TreeShape t, int V,
                                                         ulb_warp wp, uint64_t seed, const uint32_t* dev_round,
                                                         uint32_t round, TreeOut out, SpecCommit cm) {
  ULB_TRACE_KERNEL(kTrTreeDecide, 0);
  __shared__ SmemRed<DT> s;
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const bool greedy = !(wp.temperature > 0.f);
  const float iT = greedy ? 1.f : __fdiv_rn(1.0f, wp.temperature);
  const uint32_t rnd = dev_round ? dev_round[b] : round;
  const int np = t.S * (1 + t.N);
  int n = 0, tok = -1, u = -1, d = 0;
  int path[8]; /* depth <= 5 for width >= 2 (at most 63 nodes) */
  float pcommit[17];
  while (tok < 0) {
    const int prow = b * (1 + t.N) + u + 1;
    const RowStats sp = rs[prow];
    const float* pl = p + (size_t)prow * V;
    if (d == t.D) { /* a leaf: the bonus from p */
      if (greedy) {
        tok = sp.amax;
        pcommit[n] = 1.0f;
      } else {
        const float u2 = rng_u(seed, rnd, (uint32_t)b, (uint32_t)(u + 1), ULB_RNG_RESID);
        tok = block_inv_cdf(V, u2, [&](int v) { return warped_e(pl, v, iT, sp); }, s, nullptr);
        pcommit[n] = (float)(warped_e(pl, tok, iT, sp) / sp.Z);
      }
      break;
    }
    const int c0 = u < 0 ? 0 : tree_first(t.w, d + 1) + (u - tree_first(t.w, d)) * t.w;
    if (greedy) {
      int next = -1;
      for (int c = 0; c < t.w && next < 0; ++c)
        if (tokens[(size_t)b * t.N + c0 + c] == sp.amax) next = c0 + c;
      pcommit[n] = 1.0f;
      if (next < 0) { tok = sp.amax; break; }
      path[n++] = next;
      u = next;
      ++d;
      continue;
    }
    const int qrow = tree_qrow(t, b, u);
    const RowStats sq = rs[np + qrow];
    const float* ql = q + (size_t)qrow * V;
    /* R_1 = max(0, e_p Z_q - e_q Z_p), R_(j+1) = max(0, R_j Z_q - e_q W_j), W_j = sum of R_j */
    double W[kTreeMaxWidth + 1];
    int level = 0;
    auto resid = [&](int v) -> double {
      const double eq = warped_e(ql, v, iT, sq);
      double r = warped_e(pl, v, iT, sp) * sq.Z - eq * sp.Z;
      r = r > 0.0 ? r : 0.0;
      for (int j = 1; j < level; ++j) {
        r = r * sq.Z - eq * W[j];
        r = r > 0.0 ? r : 0.0;
      }
      return r;
    };
    int next = -1;
    bool dead = false; /* a residual summed to zero: nothing left to accept from */
    for (int c = 0; c < t.w; ++c) {
      const int x = tokens[(size_t)b * t.N + c0 + c];
      const bool ok = (unsigned)x < (unsigned)V;
      const double qx = ok ? warped_e(ql, x, iT, sq) / sq.Z : 0.0;
      double px;
      if (level == 0) px = ok ? warped_e(pl, x, iT, sp) / sp.Z : 0.0;
      else px = ok && !dead ? resid(x) / W[level] : 0.0;
      const float ua = rng_u(seed, rnd, (uint32_t)b, (uint32_t)(c0 + c), ULB_RNG_ACCEPT);
      if ((double)ua * qx < px) {
        next = c0 + c;
        pcommit[n] = (float)(warped_e(pl, x, iT, sp) / sp.Z);
        break;
      }
      if (dead) continue;
      ++level;
      double part = 0.0;
      for (int v = threadIdx.x; v < V; v += DT) part += resid(v);
      W[level] = block_sum_d<DT>(part, s);
      dead = !(W[level] > 0.0);
    }
    if (next >= 0) {
      path[n++] = next;
      u = next;
      ++d;
      continue;
    }
    const float u2 = rng_u(seed, rnd, (uint32_t)b, (uint32_t)(u + 1), ULB_RNG_RESID);
    if (!dead && level > 0) tok = block_inv_cdf(V, u2, resid, s, nullptr);
    else tok = block_inv_cdf(V, u2, [&](int v) { return warped_e(pl, v, iT, sp); }, s, nullptr);
    pcommit[n] = (float)(warped_e(pl, tok, iT, sp) / sp.Z);
  }
  if (threadIdx.x != 0) return;
  if (out.path) {
    for (int j = 0; j < t.D; ++j) out.path[b * t.D + j] = j < n ? path[j] : -1;
    out.n[b] = n;
    out.tok[b] = tok;
  }
  if (cm.hist) {
    const int L = cm.L[b];
    if (out.comp) {
      int32_t* cp = out.comp + (size_t)b * (2 + t.D);
      cp[0] = L;
      cp[1] = cm.done[b] ? 0 : n;
      for (int j = 0; j < t.D; ++j) cp[2 + j] = j < n ? path[j] : -1;
    }
    if (!cm.done[b]) {
      int32_t* h = cm.hist + (size_t)b * cm.hist_len;
      for (int i = 0; i < n; ++i) h[L + i] = tokens[(size_t)b * t.N + path[i]];
      h[L + n] = tok;
      cm.L[b] = L + n + 1;
      if (L + n + 1 - cm.prompt_len[b] >= cm.max_new) cm.done[b] = 1;
      atomicAdd(&cm.stats[1], (unsigned long long)t.D);
      atomicAdd(&cm.stats[2], (unsigned long long)n);
      atomicAdd(&cm.stats[3], (unsigned long long)(n + 1));
      const int a = cm.active[b];
      if (cm.log && a < cm.log_rounds && t.D <= 16) {
        int32_t* r = cm.log + ((size_t)b * cm.log_rounds + a) * cm.log_stride;
        r[ULB_SPEC_REC_N_ACCEPTED] = n;
        r[ULB_SPEC_REC_TOKEN] = tok;
        r[ULB_SPEC_REC_POSITION] = L;
        r[ULB_SPEC_REC_K] = t.D;
        /* the drafts of the round's record: the accepted path, then the first candidate of the
           node where the walk stopped and of its first descendants */
        int v = n > 0 ? path[n - 1] : -1;
        for (int i = 0; i < t.D; ++i) {
          if (i < n) {
            r[ULB_SPEC_REC_DRAFTS + i] = tokens[(size_t)b * t.N + path[i]];
          } else {
            v = v < 0 ? 0 : tree_first(t.w, i + 1) + (v - tree_first(t.w, i)) * t.w;
            r[ULB_SPEC_REC_DRAFTS + i] = tokens[(size_t)b * t.N + v];
          }
        }
        for (int i = 0; i <= n; ++i) r[ULB_SPEC_REC_DRAFTS + t.D + i] = __float_as_int(pcommit[i]);
      }
      cm.active[b] = a + 1;
    }
    cm.round[b] = rnd + 1;
  }
}

}  // namespace

int launch_sample_seq(Ctx* c, const float* logits, int rows, int V, int ld, const ulb_warp* w, uint64_t seed,
                      const uint32_t* dev_round, uint32_t round, uint32_t slot, uint32_t tag, uint32_t seq_base,
                      int32_t* out, int out_stride);
int launch_accept_impl(Ctx* c, const float* p, const float* q, const int32_t* draft, int B, int k, int V,
                       const ulb_warp* w, uint64_t seed, const uint32_t* dev_round, uint32_t round,
                       int32_t* out_tokens, int32_t* out_n, void* stats_scratch, const void* commit);

size_t sample_scratch_bytes(int, int) { return 0; }
size_t accept_scratch_bytes(int, int, int) { return sizeof(RowStats); }

int launch_sample(Ctx* c, const float* logits, int rows, int V, int ld, const ulb_warp* w, uint64_t seed,
                  const uint32_t* dev_round, uint32_t round, uint32_t slot, uint32_t tag, int32_t* out,
                  int out_stride, float*) {
  if (rows == 0) return ULB_OK;
  return launch_sample_seq(c, logits, rows, V, ld, w, seed, dev_round, round, slot, tag, 0, out, out_stride);
}

int launch_sample_seq(Ctx* c, const float* logits, int rows, int V, int ld, const ulb_warp* w, uint64_t seed,
                      const uint32_t* dev_round, uint32_t round, uint32_t slot, uint32_t tag, uint32_t seq_base,
                      int32_t* out, int out_stride) {
  if (rows == 0) return ULB_OK;
  cudaError_t e = launch_k(c, sample_kernel<RT>, dim3(rows), dim3(RT), 0, logits, V, ld, *w, seed, dev_round, round,
                           slot, tag, seq_base, out, out_stride);
  if (e != cudaSuccess) return cuda_error(e, "sample launch", __FILE__, __LINE__);
  return ULB_OK;
}

int launch_accept_commit(Ctx* c, const float* p, const float* q, const int32_t* draft, int B, int k, int V,
                         const ulb_warp* w, uint64_t seed, const uint32_t* dev_round, void* stats_scratch,
                         int32_t* hist, int hist_len, int32_t* L, int32_t* done, const int32_t* plen, int max_new,
                         uint32_t* round, unsigned long long* stats, int32_t* active, int32_t* log, int log_rounds) {
  SpecCommit cm;
  cm.hist = hist; cm.hist_len = hist_len; cm.L = L; cm.done = done; cm.prompt_len = plen;
  cm.max_new = max_new; cm.round = round; cm.stats = stats; cm.active = active;
  cm.log = log; cm.log_rounds = log_rounds; cm.log_stride = ULB_SPEC_REC_WORDS(k);
  return launch_accept_impl(c, p, q, draft, B, k, V, w, seed, dev_round, 0, nullptr, nullptr, stats_scratch, &cm);
}

int launch_accept_impl(Ctx* c, const float* p, const float* q, const int32_t* draft, int B, int k, int V,
                       const ulb_warp* w, uint64_t seed, const uint32_t* dev_round, uint32_t round,
                       int32_t* out_tokens, int32_t* out_n, void* stats_scratch, const void* commit) {
  if (B == 0) return ULB_OK;
  (void)stats_scratch; /* the walk keeps its row statistics in shared memory */
  SpecCommit cm = {};
  if (commit) cm = *(const SpecCommit*)commit;
  cudaError_t e = launch_k(c, accept_kernel, dim3(B), dim3(DT), 0, p, q, draft, B, k, V, *w, seed, dev_round, round,
                           out_tokens, out_n, cm);
  if (e != cudaSuccess) return cuda_error(e, "accept launch", __FILE__, __LINE__);
  return ULB_OK;
}

int launch_spec_accept(Ctx* c, const float* p, const float* q, const int32_t* draft, int B, int k, int V,
                       const ulb_warp* w, uint64_t seed, const uint32_t* dev_round, uint32_t round,
                       int32_t* out_tokens, int32_t* out_n, double* scratch) {
  return launch_accept_impl(c, p, q, draft, B, k, V, w, seed, dev_round, round, out_tokens, out_n, scratch, nullptr);
}

size_t tree_accept_scratch_bytes(int B, int w, int D) {
  return sizeof(RowStats) * (size_t)B * (2 + tree_first(w, D + 1) + tree_first(w, D));
}

int launch_tree_children(Ctx* c, const float* logits, int rows, int V, int w, int d, const ulb_warp* wp,
                         uint64_t seed, const uint32_t* dev_round, int N, int32_t* tokens) {
  if (rows == 0) return ULB_OK;
  cudaError_t e = launch_k(c, tree_children_kernel, dim3(rows), dim3(RT), 0, logits, V, w, d, *wp, seed, dev_round, N,
                           tokens);
  if (e != cudaSuccess) return cuda_error(e, "tree children launch", __FILE__, __LINE__);
  return ULB_OK;
}

/* stats of every p and q row of the trees, then the walk of each sequence's tree */
static int launch_tree_accept_impl(Ctx* c, const float* p, const float* q, const int32_t* tokens, int B, int w, int D,
                                   int V, const ulb_warp* wp, uint64_t seed, const uint32_t* dev_round, uint32_t round,
                                   bool q_level_major, void* stats_scratch, const TreeOut& out, const SpecCommit& cm) {
  if (B == 0) return ULB_OK;
  TreeShape t;
  t.w = w;
  t.D = D;
  t.N = tree_first(w, D + 1);
  t.NI = tree_first(w, D);
  t.q_level_major = q_level_major;
  t.S = B;
  RowStats* rs = (RowStats*)stats_scratch;
  const int np = B * (1 + t.N), nq = B * (1 + t.NI);
  const int fit = (int)std::min<long long>(3LL * c->n_sm, std::max<long long>(c->n_sm, 60000000LL / ((long long)V * 4)));
  const int grid = std::min(np + nq, fit);
  cudaError_t e = launch_k(c, stats_kernel, dim3(grid), dim3(ST), 0, p, q, np, nq, V, *wp, rs);
  if (e != cudaSuccess) return cuda_error(e, "stats launch", __FILE__, __LINE__);
  e = launch_k(c, tree_decide_kernel, dim3(B), dim3(DT), 0, p, q, tokens, (const RowStats*)rs, t, V, *wp, seed,
               dev_round, round, out, cm);
  if (e != cudaSuccess) return cuda_error(e, "tree decide launch", __FILE__, __LINE__);
  return ULB_OK;
}

int launch_tree_accept_commit(Ctx* c, const float* p, const float* q, const int32_t* tokens, int B, int w, int D,
                              int V, const ulb_warp* wp, uint64_t seed, const uint32_t* dev_round, void* stats_scratch,
                              int32_t* comp, int32_t* hist, int hist_len, int32_t* L, int32_t* done,
                              const int32_t* plen, int max_new, uint32_t* round, unsigned long long* stats,
                              int32_t* active, int32_t* log, int log_rounds) {
  SpecCommit cm;
  cm.hist = hist; cm.hist_len = hist_len; cm.L = L; cm.done = done; cm.prompt_len = plen;
  cm.max_new = max_new; cm.round = round; cm.stats = stats; cm.active = active;
  cm.log = log; cm.log_rounds = log_rounds; cm.log_stride = ULB_SPEC_REC_WORDS(D);
  TreeOut out = {nullptr, nullptr, nullptr, comp};
  return launch_tree_accept_impl(c, p, q, tokens, B, w, D, V, wp, seed, dev_round, 0, true, stats_scratch, out, cm);
}

}  // namespace ulb

using namespace ulb;

extern "C" int ulb_spec_tree_accept(ulb_ctx* ctx, const float* p, const float* q, const int32_t* tokens, int B,
                                    int width, int depth, int V, const ulb_warp* w, uint64_t seed, uint32_t round,
                                    int32_t* out_path, int32_t* out_n, int32_t* out_tok) {
  ULB_CHECK(ctx && p && q && tokens && w && out_path && out_n && out_tok, ULB_EINVAL,
            "ulb_spec_tree_accept: NULL argument");
  ULB_CHECK(B >= 0 && V > 0 && width >= 1 && width <= kTreeMaxWidth && depth >= 1, ULB_EINVAL,
            "ulb_spec_tree_accept: B %d, width %d, depth %d, V %d", B, width, depth, V);
  ULB_CHECK(tree_first(width, depth + 1) <= kTreeMaxNodes && depth <= 8, ULB_EUNSUPPORTED,
            "ulb_spec_tree_accept: a tree of width %d and depth %d has more than %d nodes", width, depth,
            kTreeMaxNodes);
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  void* scratch = nullptr;
  const size_t bytes = tree_accept_scratch_bytes(B, width, depth);
  ULB_TRY(dev_alloc(c, &scratch, bytes));
  TreeOut out = {out_path, out_n, out_tok, nullptr};
  int rc = launch_tree_accept_impl(c, p, q, tokens, B, width, depth, V, w, seed, nullptr, round, false, scratch, out,
                                   SpecCommit{});
  if (rc == ULB_OK) rc = check_device_errors(c);
  dev_free(c, scratch, bytes);
  return rc;
}

extern "C" int ulb_sample(ulb_ctx* ctx, const float* logits, int rows, int V, int ld, const ulb_warp* w,
                          uint64_t seed, uint32_t round, uint32_t slot, uint32_t tag, int32_t* out) {
  ULB_CHECK(ctx && logits && w && out, ULB_EINVAL, "ulb_sample: NULL argument");
  ULB_CHECK(rows >= 0 && V > 0 && ld >= V, ULB_EINVAL, "ulb_sample: bad shape");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  return launch_sample(&ctx->c, logits, rows, V, ld, w, seed, nullptr, round, slot, tag, out, 1, nullptr);
}

extern "C" int ulb_spec_accept(ulb_ctx* ctx, const float* p, const float* q, const int32_t* draft, int B, int k,
                               int V, const ulb_warp* w, uint64_t seed, uint32_t round, int32_t* out_tokens,
                               int32_t* out_n) {
  ULB_CHECK(ctx && p && w && out_tokens && out_n, ULB_EINVAL, "ulb_spec_accept: NULL argument");
  ULB_CHECK(B >= 0 && k >= 0 && V > 0, ULB_EINVAL, "ulb_spec_accept: bad shape");
  ULB_CHECK(k == 0 || (q && draft), ULB_EINVAL, "ulb_spec_accept: draft logits/tokens required for k > 0");
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  void* scratch = nullptr;
  const size_t bytes = accept_scratch_bytes(B, k, V);
  ULB_TRY(dev_alloc(c, &scratch, bytes));
  int rc = launch_spec_accept(c, p, q, draft, B, k, V, w, seed, nullptr, round, out_tokens, out_n, (double*)scratch);
  dev_free(c, scratch, bytes);
  return rc;
}

ULB_TRACE_UNIT(sampling)
