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
  int tp_rank = 0, tp_world = 1;
};
/* fp32 sum over the communicator's ranks, in place, on the context stream */
int tp_allreduce_sum(Ctx* c, float* buf, size_t n);
constexpr int kZeroRowHalves = 65536 + 64;

/* read and clear the device error word (synchronises the stream) */
int check_device_errors(Ctx* c);

/* tracked device allocation */
int dev_alloc(Ctx* c, void** p, size_t bytes);
void dev_free(Ctx* c, void* p, size_t bytes);

/* repack raw GGUF rows into packed strips.  row_map[packed_row] = raw row or -1 (zero). */
int repack_q4(Ctx* c, int type, const void* dev_raw, int raw_rows, int K, const int* host_row_map,
              int packed_rows, Tensor* out);

/* ------------------------------------------------------------------ kernels (launchers) */
enum Epi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

struct EpiArgs {
  float* y = nullptr;   int ldy = 0;   /* STORE: y[m*ldy+n] = v; RESID: y[m*ldy+n] += v     */
  __half* h = nullptr;  int ldh = 0;   /* SWIGLU: h[m*ldh + f] = fp16(silu(gate_f) * up_f)  */
  /* QKV: q[m*ldq + f] fp32 (RoPE'd); K/V cache fp16 [S][Hkv][cap][hd] of this layer     */
  float* q = nullptr;   int ldq = 0;
  __half* kc = nullptr; __half* vc = nullptr;
  int nq = 0, nkv = 0, hd = 0, cap = 0, n_head_kv = 0, n_seq = 0;
  const int* row_seq = nullptr; const int* row_pos = nullptr;
  const float2* rope = nullptr; /* [pos][hd/2] (cos, sin) */
};

int launch_qgemv(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a);
/* tensor-core dequant-GEMM (M >= kTcMinRows); launch_qgemv routes there */
constexpr int kTcMinRows = 128;
int launch_qgemm_tc(Ctx* c, const Tensor* w, const __half* x, int M, int ldx, int epi, const EpiArgs& a);

int launch_dequant(Ctx* c, const Tensor* w, float* out);

int launch_attention(Ctx* c, const ulb_attn_desc* d, const float* q, int ldq, const __half* k,
                     const __half* v, const int* row_seq, const int* row_pos, int M, int rps,
                     __half* out, float* scratch, int* counters, size_t scratch_floats,
                     int n_counters);
size_t attention_scratch_floats(const ulb_attn_desc* d, int M, int rps, int max_pos, int* n_counters);

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
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(Ctx* c, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            Args&&... args) {
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
/* Wait for the preceding kernel in the stream (programmatic dependent launch).  Every
 * kernel calls this before it touches data produced upstream, and before exiting. */
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
/* Allow the next kernel in the stream to begin launching its CTAs. */
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
}  // namespace ulb
#endif

#endif /* ULB_INTERNAL_H */
