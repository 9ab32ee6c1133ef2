/*
 * ulb_internal.h — internal declarations of libulb_cuda.so (not part of the C ABI).
 */
#ifndef ULB_INTERNAL_H
#define ULB_INTERNAL_H

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/ulb.h"
#include "ulb_common.h"

namespace ulb {

/* ------------------------------------------------------------------ errors */
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what, const char* file, int line);

#define ULB_CUDA(call)                                                        \
  do {                                                                        \
    cudaError_t _e = (call);                                                  \
    if (_e != cudaSuccess) return ::ulb::cuda_error(_e, #call, __FILE__, __LINE__); \
  } while (0)
#define ULB_CHECK(cond, code, ...)                                            \
  do {                                                                        \
    if (!(cond)) return ::ulb::set_error(code, __VA_ARGS__);                  \
  } while (0)
#define ULB_TRY(call)                                                         \
  do {                                                                        \
    int _rc = (call);                                                         \
    if (_rc != ULB_OK) return _rc;                                            \
  } while (0)

/* ------------------------------------------------------------------ packed weight layout */
/*
 * Q4 weight matrices are stored as 16-row strips of K-tiles laid out for the warp-level
 * MMA of qgemv.cu.  A tile holds exactly the GGUF bytes of its 16 rows (18 B per 32
 * weights for Q4_0, 144 B per 256 for Q4_K), reordered so each lane's share is one
 * 128-bit load.
 *   Q4_0 tile = 16 rows x 128 K = 1152 B: [512 B nibbles blocks 0,1][512 B blocks 2,3]
 *                                           [128 B scales: 8 x (4 x half2(d_g, d_g+8))]
 *   Q4_K tile = 16 rows x 256 K = 2304 B: [4 x 512 B nibbles, sub-blocks 2p,2p+1]
 *                                           [256 B: per row d, dmin, 12 scale bytes]
 * In each 32-weight (sub-)block lane 4g+t holds weights 8t..8t+7 of rows g and g+8 as
 * one 32-bit word per row with nibble i at bit position {0,16,4,20,8,24,12,28}[i].
 */
constexpr int kStripRows = 16;
constexpr int kQ40TileK = 128, kQ40TileBytes = 1152;
constexpr int kQ4KTileK = 256, kQ4KTileBytes = 2304;

inline int tile_k(int type) { return type == ULB_TYPE_Q4_K ? kQ4KTileK : kQ40TileK; }
inline int tile_bytes(int type) { return type == ULB_TYPE_Q4_K ? kQ4KTileBytes : kQ40TileBytes; }

struct Tensor {
  int type = 0;
  uint64_t ne[4] = {1, 1, 1, 1};
  int N = 0, K = 0;          /* matrices: rows, inner dim                        */
  int n_strips = 0, tiles = 0;
  void* dev = nullptr;       /* packed tiles (Q4) or plain array (F32/F16)        */
  size_t bytes = 0;
};

/* ------------------------------------------------------------------ context */
struct Ctx {
  int device = 0;
  int n_sm = 0;
  cudaStream_t stream = nullptr;
  size_t bytes_live = 0;
  bool pdl = true; /* programmatic dependent launch between consecutive kernels */
  std::map<void*, size_t> user_allocs; /* buffers handed out by ulb_malloc */
  uint64_t launches = 0;               /* kernels launched through launch_k (not graph replays) */
  int* dev_err = nullptr;              /* device error word: bit 1 = a bounded wait gave up */
  void* zero_row = nullptr;            /* kZeroRowHalves fp16 zeros: padding activation rows */
  void* nccl = nullptr;                /* ncclComm_t of ulb_tp_init (tensor parallelism) */
  float* tc_ws = nullptr;              /* split-K partial sums of the tensor-core GEMM */
  size_t tc_ws_floats = 0;
  int* tc_cnt = nullptr;               /* kTcCounters arrival counters, zero between launches */
  int tp_rank = 0, tp_world = 1;
  int attn_form = 0; /* ULB_ATTN_AUTO / SPLIT / STREAM */
  /* timing of the tensor-parallel all-reduces (on while a round is profiled): a CUDA event
     pair is recorded around each ncclAllReduce, events[2i] before and events[2i+1] after */
  /* host-side bound on waits for a stream holding tensor-parallel collectives (ms, 0 = none):
     past it the communicator is aborted and the call returns ULB_ETIMEOUT */
  int tp_timeout_ms = 0;
  bool tp_aborted = false;
  bool ar_timing = false;
  std::vector<cudaEvent_t> ar_events;
  size_t ar_used = 0;
};
/* fp32 sum over the communicator's ranks, in place, on the context stream */
int tp_allreduce_sum(Ctx* c, float* buf, size_t n);
constexpr int kZeroRowHalves = 65536 + 64;

/* read and clear the device error word (synchronises the stream) */
int check_device_errors(Ctx* c);
/* wait for the context stream: cudaStreamSynchronize, or, on a context with a communicator
   and a tensor-parallel timeout, the bounded wait of watchdog.h (aborting the communicator
   when a peer never answers) */
int sync_stream(Ctx* c);

/* tracked device allocation */
int dev_alloc(Ctx* c, void** p, size_t bytes);
void dev_free(Ctx* c, void* p, size_t bytes);

/* repack raw GGUF rows into packed strips.  row_map[packed_row] = raw row or -1 (zero). */
int repack_q4(Ctx* c, int type, const void* dev_raw, int raw_rows, int K, const int* host_row_map,
              int packed_rows, Tensor* out);

/* ------------------------------------------------------------------ kernels (launchers) */
/* EPI_VCACHE: the output rows are V features (the attn_v projection kept as GGUF rows), written
   in fp16 straight into the V cache like the V strips of EPI_QKV */
enum Epi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV = 3, EPI_VCACHE = 4 };

/* KV cache pages: positions of a sequence are mapped to pages of kKvPage positions through a
   block table (bt[seq * max_pages + pos / kKvPage] = page, -1 = unmapped).  A page holds
   every kv head: [page][n_head_kv][kKvPage][head_dim] fp16, one pool per layer for K and for
   V.  One page is one attention key split, so a split never crosses pages. */
constexpr int kKvPage = 256;
static_assert(kKvPage == ULB_KV_PAGE, "the page size of the C ABI");

struct EpiArgs {
  float* y = nullptr;   int ldy = 0;   /* STORE: y[m*ldy+n] = v; RESID: y[m*ldy+n] += v     */
  __half* h = nullptr;  int ldh = 0;   /* SWIGLU: h[m*ldh + f] = fp16(silu(gate_f) * up_f)  */
  /* QKV: q[m*ldq + f] fp32 (RoPE'd); K/V cache fp16 [S][Hkv][cap][hd] of this layer     */
  float* q = nullptr;   int ldq = 0;
  __half* kc = nullptr; __half* vc = nullptr;
  int nq = 0, nkv = 0, hd = 0, cap = 0, n_head_kv = 0, n_seq = 0;
  const int* row_seq = nullptr; const int* row_pos = nullptr;
  const float2* rope = nullptr; /* [pos][hd/2] (cos, sin) */
  /* paged cache (max_pages > 0: kc / vc are the layer's page pools, sequence s's position p in
     page bt[s * max_pages + p / kKvPage], or in page s * max_pages + p / kKvPage when bt is
     NULL, the identity table); max_pages == 0: contiguous [S][Hkv][cap][hd] */
  const int* bt = nullptr; int max_pages = 0;
  /* RoPE position of each row when it differs from the cache position row_pos (tree rows:
     a node at depth d sits in cache slot L + node index but rotates as position L - 1 + d);
     NULL = row_pos */
  const int* row_rope = nullptr;
};

int launch_qgemv(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a);

/* rows of a forward that are nodes of a speculation tree: row m rotates as position rope[m]
   (its cache slot is its row position), and sees the keys before pref[m] plus pref[m] + j for
   the set bits j of mask[m] */
struct TreeRows {
  const int* rope = nullptr;
  const int* pref = nullptr;
  const unsigned long long* mask = nullptr;
};

/* the model forward of model.cu: workspaces for a shape (before any capture), then one pass
   over M rows (rps per sequence); tree != NULL for the rows of a speculation tree */
struct Model;
struct KV;
int model_prepare(Model* m, KV* kv, int M, int rps, bool tree = false);
int model_forward(Model* m, KV* kv, int M, int rps, const int* tok, const int* seq, const int* pos, int logits_mode,
                  float* logits, int ld, int* err, const TreeRows* tree = nullptr);
/* move the accepted nodes of the last tree round to their sequence positions (comp [S][2 + D]:
   length before the round, nodes accepted, their node indices) */
int kv_tree_compact(KV* kv, const int32_t* comp, int S, int D);
/* y = W . rmsnorm(x32) with the fused epilogue `epi`.  Small batches (M <= 8 rows whose fp16
   copy fits kNormSmemBytes) normalise inside the GEMV, each CTA into its own shared memory;
   otherwise rmsnorm_kernel writes x16 [M][K] first.  Both give the same bits. */
constexpr int kNormSmemBytes = 65536;
/* GEMV (M <= kGemvMaxRows): dynamic shared memory per CTA at most */
constexpr size_t kGemvSmemBytes = 230400;
/* out[s] = rmsnorm(x[row]) (row = s*sel + sel - 1 when sel > 0, else s), 256 threads a row */
int launch_rmsnorm_sel(Ctx* c, const float* x, int ldx, const float* g, int n_out, int d, float eps, int sel,
                       __half* out, int ldo);
int launch_qgemv_rms(Ctx* c, const Tensor* w, const float* x32, int ldx32, const float* g, float eps, __half* x16,
                     int M, int epi, const EpiArgs& a);
/* GEMM regimes by row count M (a row's summation order is fixed within each):
     M <= kGemvMaxRows            mma.sync GEMV (qgemv.cu), fixed lane / warp tree
     kGemvMaxRows < M < kTcWideRows  tcgen05 GEMM, 64-token tiles, K split S(matrix) ways
     M >= kTcWideRows             tcgen05 GEMM, 64..256-token tiles, K not split
   launch_qgemv routes M > kGemvMaxRows to launch_qgemm_tc. */
constexpr int kGemvMaxRows = 32;
constexpr int kTcWideRows = 256;
constexpr size_t kTcWsFloats = (size_t)8 << 20; /* 32 MiB of split partial sums per context */
constexpr int kTcCounters = 4096;
int launch_qgemm_tc(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a);

int launch_dequant(Ctx* c, const Tensor* w, float* out);

/* max_pages > 0: a paged cache (k / v are page pools [page][Hkv][kKvPage][hd]) with block
   table bt (NULL: the identity table, page = seq * max_pages + position / kKvPage);
   max_pages == 0: a contiguous cache [n_seq][Hkv][capacity][hd] */
int launch_attention(Ctx* c, const ulb_attn_desc* d, const float* q, int ldq, const __half* k,
                     const __half* v, const int* row_seq, const int* row_pos, int M, int rps,
                     __half* out, float* scratch, int* counters, size_t scratch_floats,
                     int n_counters, const int* bt = nullptr, int max_pages = 0,
                     const int* tree_pref = nullptr, const unsigned long long* tree_mask = nullptr);
/* argument checks shared by every attention entry point (no division by a zero head count) */
int validate_attn_desc(const ulb_attn_desc* d, int M, int rps);
/* split-merge scratch a launch of this shape needs: zero floats / counters when it has one key
   split, when its splits merge in a thread-block cluster, or when it runs in the streaming form
   (only a global-memory merge, over caches longer than 2048 positions, reads the scratch and
   counters); bound = true: the per-split form's need whatever the form, which covers every
   launch of up to M rows */
int attention_scratch_need(Ctx* c, const ulb_attn_desc* d, int M, int rps, int max_pos, size_t* floats,
                           int* n_counters, bool tree = false, bool bound = false);

int launch_rmsnorm(Ctx* c, const float* x, int ldx, const float* g, int M, int d, float eps,
                   const int* row_select, __half* out, int ldo);
int launch_embed(Ctx* c, const __half* table, int d, const int* tokens, int M, float* x);

int launch_sample(Ctx* c, const float* logits, int rows, int V, int ld, const ulb_warp* w,
                  uint64_t seed, const uint32_t* dev_round, uint32_t round, uint32_t slot,
                  uint32_t tag, int32_t* out, int out_stride, float* scratch);
int launch_spec_accept(Ctx* c, const float* p, const float* q, const int32_t* draft, int B, int k,
                       int V, const ulb_warp* w, uint64_t seed, const uint32_t* dev_round,
                       uint32_t round, int32_t* out_tokens, int32_t* out_n, double* scratch);
size_t sample_scratch_bytes(int rows, int V);
size_t accept_scratch_bytes(int B, int k, int V);

/* ------------------------------------------------------------------ PDL launch helper */
/*
 * Every kernel of the library asks for one shared-memory carveout: an SM whose L1 / shared
 * memory split changes between consecutive kernels first drains, which costs about a
 * microsecond per change; with one split throughout there is none.  72% of the 228 KB is the
 * 164 KB split: enough for every kernel's shared memory, and ~90 KB of L1 for the GEMV's
 * activation rows.  Set once per kernel, on its first launch.
 */
constexpr int kSharedCarveoutPct = 72;
inline void prefer_max_shared(const void* kern) {
  static std::mutex mu;
  static std::set<const void*> done;
  std::lock_guard<std::mutex> lk(mu);
  if (done.insert(kern).second)
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, kSharedCarveoutPct);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(Ctx* c, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            Args&&... args) {
  prefer_max_shared((const void*)kern);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = c->pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e == cudaSuccess) ++c->launches;
  return e;
}

}  // namespace ulb

/* opaque handles of the C ABI */
struct ulb_ctx {
  ulb::Ctx c;
};
struct ulb_tensor {
  ulb_ctx* owner = nullptr;
  ulb::Tensor t;
};

/* device-side helpers shared by the .cu files */
#ifdef __CUDACC__
namespace ulb {
/*
 * CTA timeline trace, compiled into trace builds only (-DULB_TRACE, libulb_cuda_trace.so):
 * each CTA of an instrumented kernel appends one record to a ring in device memory (one ring
 * per translation unit): the kernel's tag and argument, the CTA index and grid size, and the
 * global-timer times of the CTA's entry, of the return of its wait for the previous kernel
 * (griddepcontrol.wait), of the last exit of its warps, and of up to 8 marks of its thread
 * 0.  ulb_trace_dump_<unit> copies a ring out and clears it.  Product builds compile every
 * ULB_TRACE_* macro to nothing.
 */
enum TraceTag : unsigned {
  kTrGemv = 1000,       /* + 100 epilogue + 10 n-tiles + fused RMSNorm; argument N */
  kTrAttnSplit = 2000,  /* + cluster merge + 2 tree; argument head dim */
  kTrAttnStream = 3000, /* + tiles per CTA; argument head dim */
  kTrGemmTc = 4000,     /* + epilogue; argument token tile */
  kTrRowGemv = 5000,    /* + epilogue; argument N */
  kTrEmbed = 6000,
  kTrRmsnorm = 6100,
  kTrAdd = 6200,
  kTrSample = 7000,
  kTrStats = 7100,
  kTrAccept = 7200,
  kTrTreeChildren = 7300,
  kTrTreeDecide = 7400,
  kTrStageDraft = 8000,
  kTrStageVerify = 8100,
  kTrStagePrefill = 8200,
  kTrStageTree = 8300, /* + 1 verify rows, + 50 cache compaction */
  kTrWaitFlag = 9000,
};
#ifdef ULB_TRACE
struct TraceRec {
  unsigned tag, cta, grid, arg;
  unsigned long long t_entry, t_wait, t_exit, pad, mark[8];
};
constexpr unsigned kTraceCap = 1u << 18;
static __device__ TraceRec g_trace[kTraceCap];
static __device__ unsigned g_trace_n;
__device__ __forceinline__ unsigned long long trace_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
/* the CTA's record slot (written by thread 0 at entry, read by every warp at exit) */
__device__ __forceinline__ unsigned& trace_slot() {
  __shared__ unsigned s;
  return s;
}
struct TraceGuard {
  __device__ __forceinline__ TraceGuard(unsigned tag, unsigned arg) {
    if (threadIdx.x == 0) {
      const unsigned s = atomicAdd(&g_trace_n, 1u) & (kTraceCap - 1);
      trace_slot() = s;
      TraceRec& r = g_trace[s];
      r.tag = tag;
      r.cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
      r.grid = gridDim.x * gridDim.y * gridDim.z;
      r.arg = arg;
      r.t_wait = r.t_exit = 0;
      for (int k = 0; k < 8; ++k) r.mark[k] = 0;
      r.t_entry = trace_now();
    }
  }
  __device__ __forceinline__ ~TraceGuard() {
    /* the slot index is masked: a warp that exits before thread 0 wrote it corrupts at most
       one record, never memory outside the ring */
    if ((threadIdx.x & 31) == 0)
      atomicMax(&g_trace[*(volatile unsigned*)&trace_slot() & (kTraceCap - 1)].t_exit, trace_now());
  }
};
#define ULB_TRACE_KERNEL(tag, arg) ::ulb::TraceGuard ulb_trace_guard_((unsigned)(tag), (unsigned)(arg))
#define ULB_TRACE_MARK(k)                                                                            \
  do {                                                                                               \
    if (threadIdx.x == 0) ::ulb::g_trace[::ulb::trace_slot() & (::ulb::kTraceCap - 1)].mark[k] = ::ulb::trace_now(); \
  } while (0)
/* the latest time any warp of the CTA reaches this point (lane 0 of each warp that does) */
#define ULB_TRACE_MARK_MAX(k)                                                                        \
  do {                                                                                               \
    if ((threadIdx.x & 31) == 0)                                                                     \
      atomicMax(&::ulb::g_trace[*(volatile unsigned*)&::ulb::trace_slot() & (::ulb::kTraceCap - 1)].mark[k], ::ulb::trace_now()); \
  } while (0)
#define ULB_TRACE_UNIT(NAME)                                                                         \
  extern "C" __attribute__((visibility("default"))) int ulb_trace_dump_##NAME(void* host, unsigned* n) { \
    if (cudaDeviceSynchronize() != cudaSuccess) return ULB_ECUDA;                                    \
    if (cudaMemcpyFromSymbol(n, ::ulb::g_trace_n, sizeof(unsigned)) != cudaSuccess) return ULB_ECUDA; \
    if (cudaMemcpyFromSymbol(host, ::ulb::g_trace, sizeof(::ulb::g_trace)) != cudaSuccess) return ULB_ECUDA; \
    const unsigned zero = 0;                                                                         \
    if (cudaMemcpyToSymbol(::ulb::g_trace_n, &zero, sizeof zero) != cudaSuccess) return ULB_ECUDA;    \
    return ULB_OK;                                                                                   \
  }
#else
#define ULB_TRACE_KERNEL(tag, arg) ((void)0)
#define ULB_TRACE_MARK(k) ((void)0)
#define ULB_TRACE_MARK_MAX(k) ((void)0)
#define ULB_TRACE_UNIT(NAME)
#endif

/* Wait for the preceding kernel in the stream (programmatic dependent launch).  Every
 * kernel calls this before it touches data produced upstream, and before exiting. */
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
#ifdef ULB_TRACE
  if (threadIdx.x == 0) {
    TraceRec& r = g_trace[trace_slot() & (kTraceCap - 1)];
    if (r.t_wait == 0) r.t_wait = trace_now();
  }
#endif
}
/* Allow the next kernel in the stream to begin launching its CTAs. */
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

/* Speculation trees: full trees of width w and depth D whose nodes are numbered breadth
   first from depth 1 (the root, the last committed token, is not a node).  tree_first(w, d)
   = w + w^2 + ... + w^(d-1) is the first node of depth d, so a tree has tree_first(w, D + 1)
   nodes and tree_first(w, D) internal ones (depth < D).  The children of the root are nodes
   0..w-1; those of node i of depth d, tree_first(w, d + 1) + (i - tree_first(w, d)) * w + c. */
__host__ __device__ inline int tree_first(int w, int d) {
  int f = 0, p = 1;
  for (int j = 1; j < d; ++j) {
    p *= w;
    f += p;
  }
  return f;
}
__host__ __device__ inline int tree_depth(int w, int i) {
  int d = 1, f = 0, p = w;
  while (i >= f + p) {
    f += p;
    p *= w;
    ++d;
  }
  return d;
}
/* bit j set: node j is node i or one of its ancestors */
__host__ __device__ inline unsigned long long tree_ancestors(int w, int i) {
  unsigned long long m = 0ull;
  int d = tree_depth(w, i);
  while (true) {
    m |= 1ull << i;
    if (d == 1) break;
    i = tree_first(w, d - 1) + (i - tree_first(w, d)) / w;
    --d;
  }
  return m;
}
constexpr int kTreeMaxNodes = 63;
constexpr int kTreeMaxWidth = 8;

/* barrier of a 256-thread group: the whole block (bar == 0, a 256-thread block) or named
   barrier `bar` of 256 threads inside a larger block */
__device__ __forceinline__ void sync256(int bar) {
  if (bar == 0)
    __syncthreads();
  else
    asm volatile("bar.sync %0, 256;" ::"r"(bar) : "memory");
}

/*
 * RMSNorm of one row by a group of exactly 256 threads (all of them call it, tid = 0..255;
 * d % 4 == 0, d <= 8192): out = fp16((x * r) * g), r = 1 / sqrt(sum(x^2) / d + eps).  The
 * whole row is loaded with independent 128-bit loads before any arithmetic (one memory
 * latency), and the sum has one fixed order (per-thread fmaf chains over float4
 * j = i*256 + tid, a warp xor tree, the 8 warps in order), so every caller produces the same
 * bits.  `red` is 8 floats of shared memory private to the group; `out` may be global or
 * shared; `bar` as for sync256.
 */
__device__ __forceinline__ void rms_row_256(const float* __restrict__ x, const float* __restrict__ g, int d, float eps,
                                            __half* out, float* red, int tid = threadIdx.x, int bar = 0) {
  const float4* xv = reinterpret_cast<const float4*>(x);
  const float4* gv = reinterpret_cast<const float4*>(g);
  const int n4 = d >> 2;
  float4 v[8], gg[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int j = i * 256 + tid;
    if (j < n4) { v[i] = xv[j]; gg[i] = __ldg(gv + j); }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int j = i * 256 + tid;
    if (j < n4) {
      ss = __fmaf_rn(v[i].x, v[i].x, ss);
      ss = __fmaf_rn(v[i].y, v[i].y, ss);
      ss = __fmaf_rn(v[i].z, v[i].z, ss);
      ss = __fmaf_rn(v[i].w, v[i].w, ss);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  sync256(bar);
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  sync256(bar); /* red is free for the next row */
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)d), eps)));
  __half2* o2 = reinterpret_cast<__half2*>(out);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int j = i * 256 + tid;
    if (j < n4) {
      o2[2 * j] = __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(v[i].x, r), gg[i].x)),
                                 __float2half_rn(__fmul_rn(__fmul_rn(v[i].y, r), gg[i].y)));
      o2[2 * j + 1] = __halves2half2(__float2half_rn(__fmul_rn(__fmul_rn(v[i].z, r), gg[i].z)),
                                     __float2half_rn(__fmul_rn(__fmul_rn(v[i].w, r), gg[i].w)));
    }
  }
}
}  // namespace ulb
#endif

#endif /* ULB_INTERNAL_H */
