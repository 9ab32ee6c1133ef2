/*
 * runtime.cu — context, errors, device memory, tensor upload and the op-level entry points
 * of the C ABI.  Replaces the reference's Vulkan plumbing: VulkanContext
 * (src/vulkan_backend/context.cpp), VulkanMemory::create_buffer / TransferEngine
 * (src/vulkan_backend/memory.cpp, transfer.cpp), and the per-dispatch descriptor / fence
 * round trip of ComputeDispatcher (src/vulkan_backend/compute.cpp:29-121), which on this
 * path becomes a kernel launch on the context's stream with no host synchronisation.
 */
#include <algorithm>
#include <cstring>
#include <memory>
#include <mutex>

#include <new>

#include <nccl.h>

#include "ulb_internal.h"
#include "watchdog.h"

namespace ulb {

static thread_local std::string g_last_error;
/* longest wait ulb_wait_flag accepts: a bounded wait must stay short enough that a missing
   writer costs seconds, not a hung device */
constexpr uint64_t kMaxFlagWaitNs = 10ull * 1000 * 1000 * 1000;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_error(cudaError_t e, const char* what, const char* file, int line) {
  const char* base = strrchr(file, '/');
  return set_error(ULB_ECUDA, "%s: %s (%s:%d)", what, cudaGetErrorString(e), base ? base + 1 : file, line);
}

int dev_alloc(Ctx* c, void** p, size_t bytes) {
  *p = nullptr;
  if (bytes == 0) return ULB_OK;
  cudaError_t e = cudaMallocAsync(p, bytes, c->stream);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return set_error(ULB_ENOMEM, "device allocation of %zu bytes failed", bytes);
  }
  if (e != cudaSuccess) return cuda_error(e, "cudaMallocAsync", __FILE__, __LINE__);
  c->bytes_live += bytes;
  return ULB_OK;
}

void dev_free(Ctx* c, void* p, size_t bytes) {
  if (!p) return;
  cudaFreeAsync(p, c->stream);
  c->bytes_live -= bytes;
}

/* one lane polls the flag with acquire loads until it reaches `value` or the timeout passes;
   on the timeout it raises bit 4 of the device error word and returns (nothing is left in
   flight: the wait is a plain load loop) */
__global__ void wait_flag_kernel(const int* flag, int value, unsigned long long timeout_ns, int* err) {
  ULB_TRACE_KERNEL(kTrWaitFlag, 0);
  pdl_wait();
  if (threadIdx.x != 0) return;
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= value) return;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > timeout_ns) {
      atomicOr(err, 16);
      return;
    }
    __nanosleep(256);
  }
}

int sync_stream(Ctx* c) {
  if (!c->nccl || c->tp_timeout_ms <= 0) {
    ULB_CUDA(cudaStreamSynchronize(c->stream));
    return ULB_OK;
  }
  ncclComm_t comm = (ncclComm_t)c->nccl;
  cudaError_t qerr = cudaSuccess;
  const int rc = bounded_wait(
      [&] {
        const cudaError_t e = cudaStreamQuery(c->stream);
        if (e == cudaSuccess) return Poll::kDone;
        if (e == cudaErrorNotReady) return Poll::kPending;
        qerr = e;
        return Poll::kError;
      },
      [&] {
        ncclResult_t a = ncclSuccess;
        return ncclCommGetAsyncError(comm, &a) == ncclSuccess && a != ncclSuccess && a != ncclInProgress;
      },
      [&] {
        /* the collective's kernel stops waiting for the missing peer; the communicator is gone */
        ncclCommAbort(comm);
        c->nccl = nullptr;
        c->tp_aborted = true;
      },
      c->tp_timeout_ms / 1000.0);
  if (rc == ULB_ECUDA) return cuda_error(qerr, "stream", __FILE__, __LINE__);
  if (rc == ULB_ETIMEOUT)
    return set_error(ULB_ETIMEOUT, "tensor parallel: the stream did not finish within %d ms (a peer rank is not "
                     "answering); the communicator was aborted", c->tp_timeout_ms);
  if (rc == ULB_ENCCL)
    return set_error(ULB_ENCCL, "tensor parallel: the communicator reported an asynchronous error; it was aborted");
  return ULB_OK;
}

int check_device_errors(Ctx* c) {
  int h = 0;
  ULB_CUDA(cudaMemcpyAsync(&h, c->dev_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  ULB_TRY(sync_stream(c));
  if (h) {
    ULB_CUDA(cudaMemsetAsync(c->dev_err, 0, sizeof(int), c->stream));

    return set_error(ULB_ETIMEOUT, "a device-side bounded wait gave up (flags 0x%x); results of that launch are invalid", h);
  }
  return ULB_OK;
}

int tp_allreduce_sum(Ctx* c, float* buf, size_t n) {
  ULB_CHECK(!c->tp_aborted, ULB_ENCCL, "tensor parallelism: the communicator was aborted after a peer stopped answering");
  ULB_CHECK(c->nccl, ULB_EINVAL, "tensor parallelism: the context has no communicator (ulb_tp_init)");
  const bool timed = c->ar_timing && c->ar_used + 2 <= c->ar_events.size();
  if (timed) ULB_CUDA(cudaEventRecord(c->ar_events[c->ar_used], c->stream));
  const ncclResult_t r = ncclAllReduce(buf, buf, n, ncclFloat, ncclSum, (ncclComm_t)c->nccl, c->stream);
  ULB_CHECK(r == ncclSuccess, ULB_ENCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
  if (timed) {
    ULB_CUDA(cudaEventRecord(c->ar_events[c->ar_used + 1], c->stream));
    c->ar_used += 2;
  }
  return ULB_OK;
}

}  // namespace ulb

using namespace ulb;

extern "C" {

const char* ulb_last_error(void) { return g_last_error.c_str(); }
const char* ulb_version(void) { return "ulb 0.1 (sm_100a)"; }

int ulb_init(int device, ulb_ctx** out) {
  ULB_CHECK(out, ULB_EINVAL, "ulb_init: out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return set_error(ULB_ECUDA, "ulb_init: no CUDA device (%s)", cudaGetErrorString(e));
  }
  ULB_CHECK(device >= 0 && device < n, ULB_EINVAL, "ulb_init: device %d of %d", device, n);
  ULB_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  ULB_CUDA(cudaGetDeviceProperties(&prop, device));
  ULB_CHECK(prop.major == 10, ULB_EUNSUPPORTED, "ulb_init: device %d is sm_%d%d; this build targets sm_100a",
            device, prop.major, prop.minor);
  std::unique_ptr<ulb_ctx> c(new ulb_ctx());
  c->c.device = device;
  c->c.n_sm = prop.multiProcessorCount;
  ULB_CUDA(cudaStreamCreateWithFlags(&c->c.stream, cudaStreamNonBlocking));
  ULB_CUDA(cudaMalloc((void**)&c->c.dev_err, sizeof(int)));
  ULB_CUDA(cudaMemset(c->c.dev_err, 0, sizeof(int)));
  ULB_CUDA(cudaMalloc(&c->c.zero_row, kZeroRowHalves * sizeof(__half)));
  ULB_CUDA(cudaMemset(c->c.zero_row, 0, kZeroRowHalves * sizeof(__half)));
  ULB_CUDA(cudaMalloc((void**)&c->c.tc_ws, kTcWsFloats * sizeof(float)));
  c->c.tc_ws_floats = kTcWsFloats;
  ULB_CUDA(cudaMalloc((void**)&c->c.tc_cnt, kTcCounters * sizeof(int)));
  ULB_CUDA(cudaMemset(c->c.tc_cnt, 0, kTcCounters * sizeof(int)));

  *out = c.release();
  return ULB_OK;
}

int ulb_tp_unique_id(void* out_id128) {
  ULB_CHECK(out_id128, ULB_EINVAL, "ulb_tp_unique_id: NULL argument");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  const ncclResult_t r = ncclGetUniqueId(&id);
  ULB_CHECK(r == ncclSuccess, ULB_ENCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  memcpy(out_id128, &id, sizeof id);
  return ULB_OK;
}

int ulb_tp_init(ulb_ctx* ctx, int rank, int world, const void* id128) {
  ULB_CHECK(ctx && id128, ULB_EINVAL, "ulb_tp_init: NULL argument");
  ULB_CHECK(world >= 1 && rank >= 0 && rank < world, ULB_EINVAL, "ulb_tp_init: rank %d of %d", rank, world);
  ULB_CHECK(!ctx->c.nccl, ULB_EINVAL, "ulb_tp_init: the context already has a communicator");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  ncclUniqueId id;
  memcpy(&id, id128, sizeof id);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = ncclCommInitRank(&comm, world, id, rank);
  ULB_CHECK(r == ncclSuccess, ULB_ENCCL, "ncclCommInitRank(rank %d of %d): %s", rank, world, ncclGetErrorString(r));
  ctx->c.nccl = comm;
  ctx->c.tp_rank = rank;
  ctx->c.tp_world = world;
  return ULB_OK;
}

int ulb_wait_flag(ulb_ctx* ctx, const int32_t* flag, int32_t value, uint64_t timeout_ns) {
  ULB_CHECK(ctx && flag, ULB_EINVAL, "ulb_wait_flag: NULL argument");
  ULB_CHECK(timeout_ns > 0 && timeout_ns <= kMaxFlagWaitNs, ULB_EINVAL, "ulb_wait_flag: timeout %llu ns outside (0, %llu]",
            (unsigned long long)timeout_ns, (unsigned long long)kMaxFlagWaitNs);
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  cudaError_t e = launch_k(c, wait_flag_kernel, dim3(1), dim3(32), 0, (const int*)flag, (int)value,
                           (unsigned long long)timeout_ns, c->dev_err);
  if (e != cudaSuccess) return cuda_error(e, "wait_flag launch", __FILE__, __LINE__);
  return ULB_OK;
}

int ulb_tp_set_timeout(ulb_ctx* ctx, int timeout_ms) {
  ULB_CHECK(ctx && timeout_ms >= 0, ULB_EINVAL, "ulb_tp_set_timeout: bad argument");
  ctx->c.tp_timeout_ms = timeout_ms;
  return ULB_OK;
}

int ulb_destroy(ulb_ctx* ctx) {
  if (!ctx) return ULB_OK;
  cudaSetDevice(ctx->c.device);
  cudaStreamSynchronize(ctx->c.stream);
  if (ctx->c.nccl) ncclCommDestroy((ncclComm_t)ctx->c.nccl);
  for (cudaEvent_t e : ctx->c.ar_events) cudaEventDestroy(e);
  cudaFree(ctx->c.dev_err);
  cudaFree(ctx->c.zero_row);
  cudaFree(ctx->c.tc_ws);
  cudaFree(ctx->c.tc_cnt);

  cudaStreamDestroy(ctx->c.stream);
  delete ctx;
  return ULB_OK;
}

void* ulb_stream(ulb_ctx* ctx) { return ctx ? (void*)ctx->c.stream : nullptr; }

int ulb_stream_sync(ulb_ctx* ctx) {
  ULB_CHECK(ctx, ULB_EINVAL, "ulb_stream_sync: NULL context");
  return check_device_errors(&ctx->c);
}

int ulb_mem_used(ulb_ctx* ctx, size_t* out) {
  ULB_CHECK(ctx && out, ULB_EINVAL, "ulb_mem_used: NULL argument");
  *out = ctx->c.bytes_live;
  return ULB_OK;
}

int ulb_malloc(ulb_ctx* ctx, size_t bytes, void** out) {
  ULB_CHECK(ctx && out, ULB_EINVAL, "ulb_malloc: NULL argument");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  *out = nullptr;
  if (bytes == 0) return ULB_OK;
  ULB_TRY(dev_alloc(&ctx->c, out, bytes));
  ULB_CUDA(cudaStreamSynchronize(ctx->c.stream));
  ctx->c.user_allocs[*out] = bytes;
  return ULB_OK;
}

int ulb_free(ulb_ctx* ctx, void* p) {
  ULB_CHECK(ctx, ULB_EINVAL, "ulb_free: NULL context");
  if (!p) return ULB_OK;
  auto it = ctx->c.user_allocs.find(p);
  ULB_CHECK(it != ctx->c.user_allocs.end(), ULB_EINVAL, "ulb_free: pointer was not returned by ulb_malloc");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  dev_free(&ctx->c, p, it->second);
  ctx->c.user_allocs.erase(it);
  ULB_CUDA(cudaStreamSynchronize(ctx->c.stream));
  return ULB_OK;
}

int ulb_memcpy_h2d(ulb_ctx* ctx, void* dst, const void* src, size_t bytes) {
  ULB_CHECK(ctx && (bytes == 0 || (dst && src)), ULB_EINVAL, "ulb_memcpy_h2d: NULL argument");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  ULB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->c.stream));
  ULB_CUDA(cudaStreamSynchronize(ctx->c.stream));
  return ULB_OK;
}

int ulb_memcpy_d2h(ulb_ctx* ctx, void* dst, const void* src, size_t bytes) {
  ULB_CHECK(ctx && (bytes == 0 || (dst && src)), ULB_EINVAL, "ulb_memcpy_d2h: NULL argument");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  ULB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->c.stream));
  ULB_CUDA(cudaStreamSynchronize(ctx->c.stream));
  return ULB_OK;
}

int ulb_event_create(ulb_ctx* ctx, void** ev) {
  ULB_CHECK(ctx && ev, ULB_EINVAL, "ulb_event_create: NULL argument");
  cudaEvent_t e;
  ULB_CUDA(cudaEventCreate(&e));
  *ev = e;
  return ULB_OK;
}
int ulb_event_record(ulb_ctx* ctx, void* ev) {
  ULB_CHECK(ctx && ev, ULB_EINVAL, "ulb_event_record: NULL argument");
  ULB_CUDA(cudaEventRecord((cudaEvent_t)ev, ctx->c.stream));
  return ULB_OK;
}
int ulb_event_elapsed_ms(void* a, void* b, float* ms) {
  ULB_CHECK(a && b && ms, ULB_EINVAL, "ulb_event_elapsed_ms: NULL argument");
  ULB_CUDA(cudaEventSynchronize((cudaEvent_t)b));
  ULB_CUDA(cudaEventElapsedTime(ms, (cudaEvent_t)a, (cudaEvent_t)b));
  return ULB_OK;
}
int ulb_event_destroy(void* ev) {
  if (ev) cudaEventDestroy((cudaEvent_t)ev);
  return ULB_OK;
}

struct ulb_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

int ulb_capture_begin(ulb_ctx* ctx) {
  ULB_CHECK(ctx, ULB_EINVAL, "ulb_capture_begin: NULL context");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  ULB_CUDA(cudaStreamBeginCapture(ctx->c.stream, cudaStreamCaptureModeThreadLocal));
  return ULB_OK;
}

int ulb_capture_end(ulb_ctx* ctx, ulb_graph** out) {
  ULB_CHECK(ctx && out, ULB_EINVAL, "ulb_capture_end: NULL argument");
  *out = nullptr;
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  cudaGraph_t g = nullptr;
  ULB_CUDA(cudaStreamEndCapture(ctx->c.stream, &g));
  cudaGraphExec_t x = nullptr;
  cudaError_t e = cudaGraphInstantiate(&x, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    return cuda_error(e, "graph instantiate", __FILE__, __LINE__);
  }
  ulb_graph* r = new (std::nothrow) ulb_graph;
  if (!r) {
    cudaGraphExecDestroy(x);
    cudaGraphDestroy(g);
    return set_error(ULB_ENOMEM, "ulb_capture_end: host allocation");
  }
  r->graph = g;
  r->exec = x;
  *out = r;
  return ULB_OK;
}

int ulb_graph_launch(ulb_ctx* ctx, const ulb_graph* g) {
  ULB_CHECK(ctx && g && g->exec, ULB_EINVAL, "ulb_graph_launch: NULL argument");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  ULB_CUDA(cudaGraphLaunch(g->exec, ctx->c.stream));
  return ULB_OK;
}

int ulb_graph_free(ulb_graph* g) {
  if (!g) return ULB_OK;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
  return ULB_OK;
}

int ulb_tensor_upload(ulb_ctx* ctx, int type, const uint64_t ne[4], const void* bytes, size_t nbytes,
                      ulb_tensor** out) {
  ULB_CHECK(ctx && ne && bytes && out, ULB_EINVAL, "ulb_tensor_upload: NULL argument");
  *out = nullptr;
  Ctx* c = &ctx->c;
  ULB_CUDA(cudaSetDevice(c->device));
  uint64_t n = ne[0] * ne[1] * ne[2] * ne[3];
  size_t want;
  switch (type) {
    case ULB_TYPE_F32: want = n * 4; break;
    case ULB_TYPE_F16: want = n * 2; break;
    case ULB_TYPE_Q4_0:
      ULB_CHECK(ne[0] % 32 == 0, ULB_EFORMAT, "Q4_0 row length %llu is not a multiple of 32", (unsigned long long)ne[0]);
      want = n / 32 * 18; break;
    case ULB_TYPE_Q4_K:
      ULB_CHECK(ne[0] % 256 == 0, ULB_EFORMAT, "Q4_K row length %llu is not a multiple of 256", (unsigned long long)ne[0]);
      want = n / 256 * 144; break;
    default: return set_error(ULB_EUNSUPPORTED, "ulb_tensor_upload: type %d not supported", type);
  }
  ULB_CHECK(nbytes == want, ULB_EFORMAT, "ulb_tensor_upload: %zu bytes given, GGUF size is %zu", nbytes, want);
  std::unique_ptr<ulb_tensor> t(new ulb_tensor());
  t->owner = ctx;
  t->t.type = type;
  memcpy(t->t.ne, ne, sizeof(t->t.ne));
  if (type == ULB_TYPE_F32 || type == ULB_TYPE_F16) {
    t->t.N = (int)(n / ne[0]);
    t->t.K = (int)ne[0];
    t->t.bytes = nbytes;
    ULB_TRY(dev_alloc(c, &t->t.dev, nbytes));
    ULB_CUDA(cudaMemcpyAsync(t->t.dev, bytes, nbytes, cudaMemcpyHostToDevice, c->stream));
    ULB_CUDA(cudaStreamSynchronize(c->stream));
  } else {
    ULB_CHECK(ne[2] == 1 && ne[3] == 1, ULB_EUNSUPPORTED, "quantised tensors must be 2-D");
    const int K = (int)ne[0], N = (int)ne[1];
    ULB_CHECK(K % tile_k(type) == 0, ULB_EUNSUPPORTED, "K=%d must be a multiple of %d for this layout", K, tile_k(type));
    void* raw = nullptr;
    ULB_TRY(dev_alloc(c, &raw, nbytes));
    cudaError_t e = cudaMemcpyAsync(raw, bytes, nbytes, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) { dev_free(c, raw, nbytes); return cuda_error(e, "upload", __FILE__, __LINE__); }
    const int rows = (N + 15) / 16 * 16;
    std::vector<int> map(rows);
    for (int i = 0; i < rows; ++i) map[i] = i < N ? i : -1;
    int rc = repack_q4(c, type, raw, N, K, map.data(), rows, &t->t);
    dev_free(c, raw, nbytes);
    if (rc) return rc;
    t->t.N = N;
  }
  *out = t.release();
  return ULB_OK;
}

int ulb_tensor_free(ulb_tensor* t) {
  if (!t) return ULB_OK;
  Ctx* c = &t->owner->c;
  cudaSetDevice(c->device);
  dev_free(c, t->t.dev, t->t.bytes);
  cudaStreamSynchronize(c->stream);
  delete t;
  return ULB_OK;
}

int ulb_tensor_info(const ulb_tensor* t, int* type, uint64_t ne[4], size_t* dev_bytes) {
  ULB_CHECK(t, ULB_EINVAL, "ulb_tensor_info: NULL tensor");
  if (type) *type = t->t.type;
  if (ne) memcpy(ne, t->t.ne, sizeof(t->t.ne));
  if (dev_bytes) *dev_bytes = t->t.bytes;
  return ULB_OK;
}

int ulb_dequant(ulb_ctx* ctx, const ulb_tensor* w, float* out) {
  ULB_CHECK(ctx && w && out, ULB_EINVAL, "ulb_dequant: NULL argument");
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  return launch_dequant(&ctx->c, &w->t, out);
}

int ulb_qgemm(ulb_ctx* ctx, const ulb_tensor* w, const uint16_t* x, int M, float* y, int ldy) {
  ULB_CHECK(ctx && w && x && y, ULB_EINVAL, "ulb_qgemm: NULL argument");
  ULB_CHECK(ldy >= w->t.N, ULB_EINVAL, "ulb_qgemm: ldy %d < N %d", ldy, w->t.N);
  ULB_CUDA(cudaSetDevice(ctx->c.device));
  EpiArgs a;
  a.y = y;
  a.ldy = ldy;
  return launch_qgemv(&ctx->c, &w->t, reinterpret_cast<const __half*>(x), M, w->t.K, EPI_STORE, a);
}

}  // extern "C"

ULB_TRACE_UNIT(runtime)
