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
 * grid = (key split of 512 positions, kv head, sequence x row block).  All q heads of a GQA
 * group and all rows of the block share each 64-key K/V block, staged in shared memory with
 * cp.async and double-buffered, so the cache is read once per step.  Inside a split the CTA
 * keeps an online softmax (running max / sum, rescaled output).  Contexts up to 512 keys
 * need no merge; longer ones write one partial per split and the CTA that arrives last for
 * its (sequence, row block, kv head) merges them in split order.  The split structure depends
 * only on a row's position, so a row's arithmetic never depends on what else is batched.
 */
#include <mutex>

#include "ulb_internal.h"

namespace ulb {

namespace {

constexpr int BK = 64;      /* keys per staged block */
constexpr int SPLIT = 64;    /* keys per CTA: many CTAs per (sequence, kv head) */
constexpr int MAXSPLIT = 128; /* capacity <= 8192 */
constexpr int MERGE_UNROLL = 8;
constexpr int AQMAX = 64;    /* queries (heads x rows) per CTA */
constexpr int ATHREADS = 256;
constexpr int ANW = ATHREADS / 32;
constexpr int MAXITEMS = AQMAX * 64 / ATHREADS; /* output (query, dim pair) items per thread, hd <= 128 */

struct AttnParams {
  int H, Hkv, hd, cap, G, rps, RB, n_rb, max_splits, ldq, n_seq;
  float scale;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

struct Smem {
  float* qs;     /* [AQMAX][hd]               */
  float* ss;     /* [AQMAX][BK] scores / p    */
  int* qpos;     /* [AQMAX]                   */
  float* mrun;   /* [AQMAX] running max       */
  float* lrun;   /* [AQMAX] running sum       */
  float* scl;    /* [AQMAX] rescale of block  */
  uint4* ks;     /* [2][BK][hd/8] swizzled    */
  uint4* vs;     /* [2][BK][hd/8]             */
};

__device__ __forceinline__ Smem carve(float* base, int hd) {
  Smem s;
  s.qs = base;
  s.ss = s.qs + AQMAX * hd;
  s.qpos = reinterpret_cast<int*>(s.ss + AQMAX * BK);
  s.mrun = reinterpret_cast<float*>(s.qpos + AQMAX);
  s.lrun = s.mrun + AQMAX;
  s.scl = s.lrun + AQMAX;
  s.ks = reinterpret_cast<uint4*>(s.scl + AQMAX);
  s.vs = s.ks + 2 * BK * (hd / 8);
  return s;
}

__global__ void __launch_bounds__(ATHREADS) attn_kernel(AttnParams p, const float* __restrict__ q,
                                                        const __half* __restrict__ kc, const __half* __restrict__ vc,
                                                        const int* __restrict__ row_seq,
                                                        const int* __restrict__ row_pos, __half* __restrict__ out,
                                                        float* scratch, int* counters) {
  extern __shared__ __align__(16) float smem_raw[];
  const int split = blockIdx.x, kvh = blockIdx.y, gz = blockIdx.z;
  const int gi = gz / p.n_rb, rb = gz % p.n_rb;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hd = p.hd, hd2 = hd >> 1, vpr = hd / 8;
  const Smem S = carve(smem_raw, hd);
  pdl_wait();
  pdl_trigger();

  const int r0 = rb * p.RB;
  const int nr = min(p.RB, p.rps - r0);
  const int Q = p.G * nr;
  const int m0 = gi * p.rps + r0;
  int last_pos = 0;
  for (int r = 0; r < nr; ++r) last_pos = max(last_pos, row_pos[m0 + r]);
  last_pos = min(last_pos, p.cap - 1); /* positions past the cache never index it */
  const int n_splits = last_pos / SPLIT + 1;
  if (split >= n_splits) return;
  const int seq = row_seq[m0];
  if ((unsigned)seq >= (unsigned)p.n_seq) return;
  const int k_begin = split * SPLIT;
  const int k_end = min(k_begin + SPLIT, last_pos + 1);
  const int nblocks = (k_end - k_begin + BK - 1) / BK;
  const size_t kvbase = (((size_t)seq * p.Hkv + kvh) * p.cap) * hd;

  auto stage = [&](int b, int buf) {
    const int kb = k_begin + b * BK;
    const int nk = min(BK, k_end - kb);
    uint4* kd = S.ks + buf * BK * vpr;
    uint4* vd = S.vs + buf * BK * vpr;
    for (int i = tid; i < nk * vpr; i += ATHREADS) {
      const int j = i / vpr, c = i % vpr;
      const int cs = (c & ~7) | ((c ^ j) & 7); /* XOR swizzle inside each group of 8 chunks */
      const size_t src = kvbase + (size_t)(kb + j) * hd + c * 8;
      cp_async16(kd + j * vpr + cs, kc + src);
      cp_async16(vd + j * vpr + c, vc + src);
    }
  };

  for (int i = tid; i < Q * (hd / 4); i += ATHREADS) {
    const int qi = i / (hd / 4), c = i % (hd / 4);
    const int r = qi / p.G, gq = qi % p.G;
    cp_async16(S.qs + qi * hd + c * 4, q + (size_t)(m0 + r) * p.ldq + (kvh * p.G + gq) * hd + c * 4);
  }
  stage(0, 0);
  cp_commit();
  for (int qi = tid; qi < Q; qi += ATHREADS) {
    S.qpos[qi] = row_pos[m0 + qi / p.G];
    S.mrun[qi] = -INFINITY;
    S.lrun[qi] = 0.f;
  }
  const int n_items = Q * hd2;
  float2 o[MAXITEMS];
#pragma unroll
  for (int k = 0; k < MAXITEMS; ++k) o[k] = make_float2(0.f, 0.f);

  for (int b = 0; b < nblocks; ++b) {
    const int buf = b & 1;
    if (b + 1 < nblocks) {
      stage(b + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int kb = k_begin + b * BK;
    const int nk = min(BK, k_end - kb);
    const uint4* kbuf = S.ks + buf * BK * vpr;
    /* scores: warp per query, lanes over keys; sequential fma over d (as the CPU oracle) */
    for (int qi = warp; qi < Q; qi += ANW) {
      const float4* qv = reinterpret_cast<const float4*>(S.qs + qi * hd);
      const int qp = S.qpos[qi];
      for (int j = lane; j < BK; j += 32) {
        float s = -INFINITY;
        if (j < nk && kb + j <= qp) {
          const uint4* kr = kbuf + j * vpr;
          float a = 0.f;
          for (int c = 0; c < vpr; ++c) {
            const uint4 kk = kr[(c & ~7) | ((c ^ j) & 7)];
            const float4 qa = qv[2 * c], qb = qv[2 * c + 1];
            const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kk.x));
            const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kk.y));
            const float2 k45 = __half22float2(*reinterpret_cast<const __half2*>(&kk.z));
            const float2 k67 = __half22float2(*reinterpret_cast<const __half2*>(&kk.w));
            a = __fmaf_rn(qa.x, k01.x, a);
            a = __fmaf_rn(qa.y, k01.y, a);
            a = __fmaf_rn(qa.z, k23.x, a);
            a = __fmaf_rn(qa.w, k23.y, a);
            a = __fmaf_rn(qb.x, k45.x, a);
            a = __fmaf_rn(qb.y, k45.y, a);
            a = __fmaf_rn(qb.z, k67.x, a);
            a = __fmaf_rn(qb.w, k67.y, a);
          }
          s = __fmul_rn(a, p.scale);
        }
        S.ss[qi * BK + j] = s;
      }
      __syncwarp();
      /* online softmax update of this query (the same warp wrote its scores) */
      float mb = -INFINITY;
      for (int j = lane; j < BK; j += 32) mb = fmaxf(mb, S.ss[qi * BK + j]);
#pragma unroll
      for (int off = 16; off; off >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      const float mold = S.mrun[qi];
      const float mnew = fmaxf(mold, mb);
      float lb = 0.f;
      for (int j = lane; j < BK; j += 32) {
        const float s = S.ss[qi * BK + j];
        const float e = s == -INFINITY ? 0.f : expf(s - mnew);
        S.ss[qi * BK + j] = e;
        lb += e;
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) lb += __shfl_xor_sync(0xffffffffu, lb, off);
      __syncwarp();
      if (lane == 0) {
        const float sc = mold == -INFINITY ? 0.f : expf(mold - mnew);
        S.scl[qi] = sc;
        S.lrun[qi] = __fmaf_rn(S.lrun[qi], sc, lb);
        S.mrun[qi] = mnew;
      }
    }
    __syncthreads();
    /* P.V: thread per (query, dim pair) items; sequential over keys */
    const __half2* vbuf = reinterpret_cast<const __half2*>(S.vs + buf * BK * vpr);
#pragma unroll
    for (int k = 0; k < MAXITEMS; ++k) {
      const int it = tid + k * ATHREADS;
      if (it < n_items) {
        const int qi = it / hd2, d2 = it % hd2;
        const float sc = S.scl[qi];
        float ox = o[k].x * sc, oy = o[k].y * sc;
        const float* pr = S.ss + qi * BK;
        for (int j = 0; j < nk; ++j) {
          const float pj = pr[j];
          const float2 vf = __half22float2(vbuf[j * hd2 + d2]);
          ox = __fmaf_rn(pj, vf.x, ox);
          oy = __fmaf_rn(pj, vf.y, oy);
        }
        o[k] = make_float2(ox, oy);
      }
    }
    __syncthreads(); /* the next iteration restages this buffer */
  }

  auto out_ptr = [&](int qi) {
    const int r = qi / p.G, gq = qi % p.G;
    return reinterpret_cast<__half2*>(out + (size_t)(m0 + r) * p.H * hd + (kvh * p.G + gq) * hd);
  };
  if (n_splits == 1) {
#pragma unroll
    for (int k = 0; k < MAXITEMS; ++k) {
      const int it = tid + k * ATHREADS;
      if (it < n_items) {
        const int qi = it / hd2, d2 = it % hd2;
        const float l = S.lrun[qi];
        out_ptr(qi)[d2] = __halves2half2(__float2half_rn(o[k].x / l), __float2half_rn(o[k].y / l));
      }
    }
    return;
  }
  /* partial of this split: (m, l) then the unnormalised output */
  const int qstride = p.G * p.RB;
  const size_t pstride = (size_t)qstride * (hd + 2);
  float* base = scratch + ((size_t)gz * p.Hkv + kvh) * p.max_splits * pstride;
  float* part = base + split * pstride;
#pragma unroll
  for (int k = 0; k < MAXITEMS; ++k) {
    const int it = tid + k * ATHREADS;
    if (it < n_items) {
      const int qi = it / hd2, d2 = it % hd2;
      part[(size_t)qi * (hd + 2) + 2 + 2 * d2] = o[k].x;
      part[(size_t)qi * (hd + 2) + 3 + 2 * d2] = o[k].y;
    }
  }
  for (int qi = tid; qi < Q; qi += ATHREADS) {
    part[(size_t)qi * (hd + 2)] = S.mrun[qi];
    part[(size_t)qi * (hd + 2) + 1] = S.lrun[qi];
  }
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (tid == 0) is_last = atomicAdd(&counters[gz * p.Hkv + kvh], 1) == n_splits - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  /* merge in split order.  (1) every (query, split) max / sum is fetched in parallel into
     shared memory; (2) a thread per query turns them into weights; (3) each output item
     sums its splits with the loads of MERGE_UNROLL splits in flight at once. */
  float* msm = S.qs; /* [Q][n_splits] (max, then weight)    */
  float* lsm = S.ss; /* [Q][n_splits] sums                   */
  for (int idx = tid; idx < Q * n_splits; idx += ATHREADS) {
    const int qi = idx / n_splits, c = idx % n_splits;
    msm[idx] = __ldcg(base + c * pstride + (size_t)qi * (hd + 2));
    lsm[idx] = __ldcg(base + c * pstride + (size_t)qi * (hd + 2) + 1);
  }
  __syncthreads();
  for (int qi = tid; qi < Q; qi += ATHREADS) {
    float M = -INFINITY;
    for (int c = 0; c < n_splits; ++c) M = fmaxf(M, msm[qi * n_splits + c]);
    float L = 0.f;
    for (int c = 0; c < n_splits; ++c) {
      const float mc = msm[qi * n_splits + c];
      const float w = mc == -INFINITY ? 0.f : expf(mc - M);
      msm[qi * n_splits + c] = w;
      L = __fmaf_rn(lsm[qi * n_splits + c], w, L);
    }
    S.lrun[qi] = L;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < MAXITEMS; ++k) {
    const int it = tid + k * ATHREADS;
    if (it < n_items) {
      const int qi = it / hd2, d2 = it % hd2;
      float ox = 0.f, oy = 0.f;
      for (int c0 = 0; c0 < n_splits; c0 += MERGE_UNROLL) {
        float2 oc[MERGE_UNROLL];
#pragma unroll
        for (int u = 0; u < MERGE_UNROLL; ++u)
          if (c0 + u < n_splits)
            oc[u] = __ldcg(reinterpret_cast<const float2*>(base + (c0 + u) * pstride + (size_t)qi * (hd + 2) + 2) + d2);
#pragma unroll
        for (int u = 0; u < MERGE_UNROLL; ++u)
          if (c0 + u < n_splits) {
            const float w = msm[qi * n_splits + c0 + u];
            ox = __fmaf_rn(oc[u].x, w, ox);
            oy = __fmaf_rn(oc[u].y, w, oy);
          }
      }
      const float L = S.lrun[qi];
      out_ptr(qi)[d2] = __halves2half2(__float2half_rn(ox / L), __float2half_rn(oy / L));
    }
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
  p->max_splits = max_pos / SPLIT + 1;
  p->RB = AQMAX / p->G < 1 ? 1 : AQMAX / p->G;
  /* the merge stages (query, split) pairs in shared memory: at most AQMAX * BK of them */
  const int rb_merge = (AQMAX * BK) / (p->G * p->max_splits);
  if (p->RB > rb_merge) p->RB = rb_merge < 1 ? 1 : rb_merge;
  if (p->RB > rps) p->RB = rps;
  p->n_rb = (rps + p->RB - 1) / p->RB;
  p->scale = d->scale;
  p->n_seq = d->n_seq;
  *n_groups = M / rps;
}

size_t attn_smem(int hd) {
  return sizeof(float) * ((size_t)AQMAX * hd + AQMAX * BK + 3 * AQMAX) + sizeof(int) * AQMAX +
         sizeof(__half) * 4 * (size_t)BK * hd;
}

}  // namespace

size_t attention_scratch_floats(const ulb_attn_desc* d, int M, int rps, int max_pos, int* n_counters) {
  AttnParams p;
  int ng;
  attn_geometry(d, M, rps, max_pos, &p, &ng);
  *n_counters = ng * p.n_rb * p.Hkv;
  return (size_t)ng * p.n_rb * p.Hkv * p.max_splits * (size_t)(p.G * p.RB) * (p.hd + 2);
}

int launch_attention(Ctx* c, const ulb_attn_desc* d, const float* q, int ldq, const __half* k,
                     const __half* v, const int* row_seq, const int* row_pos, int M, int rps,
                     __half* out, float* scratch, int* counters, size_t scratch_floats, int n_counters) {
  ULB_CHECK(d->n_head % d->n_head_kv == 0, ULB_EINVAL, "attention: n_head %% n_head_kv != 0");
  ULB_CHECK(d->head_dim % 16 == 0 && d->head_dim <= 128, ULB_EUNSUPPORTED, "attention: head_dim %d", d->head_dim);
  ULB_CHECK(d->n_head / d->n_head_kv <= AQMAX, ULB_EUNSUPPORTED, "attention: GQA group > %d", AQMAX);
  ULB_CHECK(d->capacity <= SPLIT * MAXSPLIT, ULB_EUNSUPPORTED, "attention: capacity %d > %d", d->capacity,
            SPLIT * MAXSPLIT);
  ULB_CHECK(rps > 0 && M % rps == 0, ULB_EINVAL, "attention: M=%d not a multiple of rows_per_seq=%d", M, rps);
  ULB_CHECK(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 && ldq % 4 == 0,
            ULB_EINVAL, "attention: q / k / v must be 16-byte aligned (ldq a multiple of 4)");
  if (M == 0) return ULB_OK;
  AttnParams p;
  int ng;
  attn_geometry(d, M, rps, d->capacity - 1, &p, &ng);
  p.ldq = ldq;
  int need_c = 0;
  const size_t need = attention_scratch_floats(d, M, rps, d->capacity - 1, &need_c);
  ULB_CHECK(p.max_splits == 1 || (scratch_floats >= need && n_counters >= need_c), ULB_EINVAL,
            "attention: scratch %zu floats / %d counters, need %zu / %d", scratch_floats, n_counters, need, need_c);
  static bool attr_set = false;
  if (!attr_set) {
    ULB_CUDA(cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem(128)));
    attr_set = true;
  }
  dim3 grid(p.max_splits, p.Hkv, ng * p.n_rb), block(ATHREADS);
  cudaError_t e = launch_k(c, attn_kernel, grid, block, attn_smem(p.hd), p, q, k, v, row_seq, row_pos, out, scratch,
                           counters);
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
  ULB_CHECK(d->capacity > 0 && d->n_seq > 0, ULB_EINVAL, "ulb_attention_noalloc: capacity / n_seq");
  ULB_CHECK(rps > 0 && M >= 0 && M % rps == 0, ULB_EINVAL, "ulb_attention_noalloc: M=%d, rows_per_seq=%d", M, rps);
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  int nc = 0;
  const size_t nf = attention_scratch_floats(d, M, rps, d->capacity - 1, &nc);
  ULB_CHECK(nf <= kNoAllocScratchFloats && nc <= kNoAllocCounters, ULB_EINVAL,
            "ulb_attention_noalloc: this shape needs %zu scratch floats and %d counters; the static scratch holds "
            "%zu floats and %d counters (use ulb_attention)",
            nf, nc, kNoAllocScratchFloats, kNoAllocCounters);
  float* scratch = nullptr;
  int* counters = nullptr;
  ULB_TRY(noalloc_scratch(c, &scratch, &counters));
  /* the arrays keep the previous call's contents: the split counters must start at zero */
  ULB_CUDA(cudaMemsetAsync(counters, 0, (size_t)nc * sizeof(int), c->stream));
  return launch_attention(c, d, q, d->n_head * d->head_dim, (const __half*)k, (const __half*)v, row_seq, row_pos, M,
                          rps, (__half*)out, scratch, counters, kNoAllocScratchFloats, kNoAllocCounters);
}

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
  if (rc == ULB_OK) rc = check_device_errors(c);
  dev_free(c, counters, (size_t)nc * sizeof(int));
  dev_free(c, scratch, nf * sizeof(float));
  return rc;
}
