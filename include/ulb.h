/*
 * ulb.h — C ABI of libulb_cuda.so, the sm_100a replacement for Universal-Loader's
 * Vulkan backend (src/vulkan_backend) and its dequantize / gemm / attention shaders
 * (src/shaders/{dequantize,gemm,attention}) on the speculative draft -> verify ->
 * accept path.
 *
 * Conventions
 *  - Every function returns ULB_OK (0) or a negative ULB_E* code; no C++ exception
 *    crosses this boundary.  ulb_last_error() returns the calling thread's message for
 *    the most recent failure.
 *  - Pointers named dev_* are device pointers on the context's device; host_* are host
 *    pointers borrowed for the duration of the call.  Outputs are caller-allocated unless
 *    a function says otherwise.
 *  - All work is enqueued on the context's stream (ulb_stream); calls on one context must
 *    be serialised by the caller (one context per device, one host thread at a time).
 *  - There is no CPU fallback: without a usable CUDA device ulb_init fails with ULB_ECUDA.
 */
#ifndef ULB_H
#define ULB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ULB_API __attribute__((visibility("default")))
#else
#define ULB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status codes */
#define ULB_OK 0
#define ULB_EINVAL (-1)      /* bad argument, shape or state                        */
#define ULB_ENOMEM (-2)      /* device or host allocation failed                    */
#define ULB_ECUDA (-3)       /* CUDA runtime error                                  */
#define ULB_ENCCL (-4)       /* NCCL error (tensor-parallel helpers)                */
#define ULB_ETIMEOUT (-5)    /* a bounded device-side wait gave up                   */
#define ULB_EFORMAT (-6)     /* malformed GGUF bytes / unsupported tensor layout     */
#define ULB_EUNSUPPORTED (-7)

/* GGML tensor type ids, as in the reference's ggml::GGMLType (src/core/gguf_types.h:6-33). */
#define ULB_TYPE_F32 0
#define ULB_TYPE_F16 1
#define ULB_TYPE_Q4_0 2
#define ULB_TYPE_Q4_K 12
#define ULB_TYPE_Q8_0 8  /* token_embd and output.weight only (as llama.cpp's Q4_0 files store them) */
#define ULB_TYPE_Q6_K 14 /* token_embd and output.weight only */

typedef struct ulb_ctx ulb_ctx;
typedef struct ulb_tensor ulb_tensor;
typedef struct ulb_model ulb_model;
typedef struct ulb_kv ulb_kv;
typedef struct ulb_spec ulb_spec;

/* ------------------------------------------------------------------ errors / info */
/* Replaces the reference's std::cerr + bool returns (vulkan_backend/context.cpp). */
ULB_API const char* ulb_last_error(void);
ULB_API const char* ulb_version(void);

/* ------------------------------------------------------------------ context */
/* Replaces vulkan::VulkanContext construction (src/vulkan_backend/context.cpp) and the
 * engine's initialize() GPU branch (src/inference/inference_engine.cpp:48-148). */
ULB_API int ulb_init(int device, ulb_ctx** out);
ULB_API int ulb_destroy(ulb_ctx* ctx);
/* The context's cudaStream_t (as void*). */
ULB_API void* ulb_stream(ulb_ctx* ctx);
/* Replaces ComputeDispatcher::wait_for_completion (src/vulkan_backend/compute.cpp:82-121). */
ULB_API int ulb_stream_sync(ulb_ctx* ctx);
/*
 * Bounded device-side wait: enqueue on the context stream a wait until the int32 at dev_flag
 * (device memory, or memory the device can reach: another stream's or process's flag) is
 * >= value.  Later work on the stream runs after it.  If the flag does not get there within
 * timeout_ns (at most 10 s), the wait gives up instead of hanging the device: it raises the
 * device error flag, which the next ulb_stream_sync reports as ULB_ETIMEOUT, and the context
 * stays usable.  No counterpart in the reference (its Vulkan fences wait on the host,
 * src/vulkan_backend/compute.cpp:82-121, with no bound).
 */
ULB_API int ulb_wait_flag(ulb_ctx* ctx, const int32_t* dev_flag, int32_t value, uint64_t timeout_ns);
/* Device bytes currently held by the context (weights, caches, workspaces). */
ULB_API int ulb_mem_used(ulb_ctx* ctx, size_t* out_bytes);

/* Device buffers and copies for callers of the kernels below.  Replaces VulkanMemory::
 * create_buffer / destroy_buffer and TransferEngine (src/vulkan_backend/memory.cpp,
 * transfer.cpp).  The copies are synchronous with respect to the host. */
ULB_API int ulb_malloc(ulb_ctx* ctx, size_t bytes, void** out_dev);
ULB_API int ulb_free(ulb_ctx* ctx, void* dev);
ULB_API int ulb_memcpy_h2d(ulb_ctx* ctx, void* dev_dst, const void* host_src, size_t bytes);
ULB_API int ulb_memcpy_d2h(ulb_ctx* ctx, void* host_dst, const void* dev_src, size_t bytes);

/* CUDA-event timing on the context's stream (replaces vulkan::Profiler timestamp queries,
 * src/vulkan_backend/profiler.cpp:174-230). */
ULB_API int ulb_event_create(ulb_ctx* ctx, void** out_event);
ULB_API int ulb_event_record(ulb_ctx* ctx, void* event);
ULB_API int ulb_event_elapsed_ms(void* start, void* end, float* out_ms);
ULB_API int ulb_event_destroy(void* event);

/* NCCL communicator of the context (one process per GPU; NVLink / NVSwitch inside a node).
 * ulb_tp_unique_id writes the 128-byte ncclUniqueId on one rank; share it with the others
 * (any host channel), then every rank calls ulb_tp_init on its own context. */
ULB_API int ulb_tp_unique_id(void* out_id128);
ULB_API int ulb_tp_init(ulb_ctx* ctx, int rank, int world, const void* id128);
/* Bound (ms; 0 = unbounded, the default) on every host wait of this context for work that
 * holds tensor-parallel collectives (the speculative loop, ulb_model_forward,
 * ulb_stream_sync).  Past it -- a peer rank died or stopped answering -- the communicator is
 * aborted (ncclCommAbort, so the collective's kernel stops waiting), the call returns
 * ULB_ETIMEOUT, and every later tensor-parallel call fails with ULB_ENCCL.  An asynchronous
 * communicator error is handled the same way (ULB_ENCCL).  No counterpart in the reference,
 * whose multi-GPU manager has no data path (src/vulkan_backend/multi_gpu_manager.cpp). */
ULB_API int ulb_tp_set_timeout(ulb_ctx* ctx, int timeout_ms);

/* CUDA-graph capture of a fixed sequence of per-op calls on the context's stream, replayed
 * with one launch (replaces re-recording the reference's command buffers per dispatch,
 * src/vulkan_backend/compute.cpp:27-80).  Calls between begin and end are recorded, not
 * run.  Capturable: ulb_qgemm, ulb_attention_noalloc, ulb_sample, ulb_spec_accept, once
 * each has been called on the context outside a capture; not capturable: calls that
 * synchronise with the host (ulb_attention, ulb_malloc, ulb_memcpy_*, ulb_model_forward). */
typedef struct ulb_graph ulb_graph;
ULB_API int ulb_capture_begin(ulb_ctx* ctx);
ULB_API int ulb_capture_end(ulb_ctx* ctx, ulb_graph** out);
ULB_API int ulb_graph_launch(ulb_ctx* ctx, const ulb_graph* g);
ULB_API int ulb_graph_free(ulb_graph* g);

/* ------------------------------------------------------------------ weights */
/*
 * Upload one GGUF tensor and repack it into the device layout used by the kernels.
 * Replaces the reference's repack_q4k_tensor + upload_to_gpu
 * (src/inference/inference_engine.cpp:536-548, 891-927) and VulkanMemory::create_buffer.
 *   ggml_type  ULB_TYPE_F32 / F16 / Q4_0 / Q4_K
 *   ne         GGUF dims, ne[0] = innermost (K for a weight matrix, ne[1] = rows N)
 *   gguf_bytes host pointer to the tensor's bytes exactly as stored in the GGUF file
 *   nbytes     must equal the GGUF size of the tensor (18 B / 32 weights for Q4_0,
 *              144 B / 256 weights for Q4_K) -- ULB_EFORMAT otherwise
 */
ULB_API int ulb_tensor_upload(ulb_ctx* ctx, int ggml_type, const uint64_t ne[4],
                      const void* gguf_bytes, size_t nbytes, ulb_tensor** out);
ULB_API int ulb_tensor_free(ulb_tensor* t);
ULB_API int ulb_tensor_info(const ulb_tensor* t, int* out_type, uint64_t out_ne[4], size_t* out_device_bytes);

/* ------------------------------------------------------------------ kernels */
/*
 * Bit-exact dequantisation of a whole tensor to fp32, row-major [ne1][ne0].  Parity
 * helper; replaces dequantize_q4_0.glsl / dequantize_q4_k(_flattened).glsl
 * (src/shaders/dequantize) and cpu::dequantize_q4_0_f32 / q4_k_f32
 * (src/cpu_backend/dequantize_cpu.cpp:6-74).
 */
ULB_API int ulb_dequant(ulb_ctx* ctx, const ulb_tensor* w, float* dev_out);

/*
 * Fused dequant-GEMM  y[m*ldy + n] = sum_k W[n][k] * x[m][k]   (fp32 accumulate)
 *   W      Q4_0 or Q4_K tensor from ulb_tensor_upload, N = ne[1] rows, K = ne[0]
 *   dev_x  fp16 activations, row-major [M][K]
 *   dev_y  fp32 output rows with leading dimension ldy >= N
 * Replaces run_linear_q4k = dequantize_q4_k_flattened + gemm_transposed_b_v2
 * (src/inference/inference_engine.cpp:532-570) and gemm_dequant_q4_0.glsl /
 * gemm_coop_dequant_q4_0.glsl (src/shaders/gemm).  Every output row is computed with the
 * same arithmetic whatever M is, so batching never changes a row's result.
 */
ULB_API int ulb_qgemm(ulb_ctx* ctx, const ulb_tensor* w, const uint16_t* dev_x, int M,
              float* dev_y, int ldy);

/*
 * Block-causal attention of M query rows against an fp16 KV cache.
 *   dev_q       fp32 [M][n_head][head_dim] (RoPE already applied)
 *   dev_k/v     fp16 [n_seq][n_head_kv][capacity][head_dim]
 *   dev_row_seq int32 [M] sequence of each row;  dev_row_pos int32 [M] its position
 *   Row m attends keys 0..row_pos[m] of its sequence (GQA: head h reads kv head
 *   h / (n_head / n_head_kv)).  Rows of one sequence must be consecutive, rows_per_seq each.
 *   dev_out     fp16 [M][n_head][head_dim]
 * Replaces flash_attention.glsl and the flash_attention_v2_fused/_v3 feature set
 * (src/shaders/attention, inference_engine.cpp:628-630).
 */
typedef struct ulb_attn_desc {
  int n_head, n_head_kv, head_dim, capacity, n_seq;
  float scale; /* usually 1/sqrt(head_dim) */
} ulb_attn_desc;
ULB_API int ulb_attention(ulb_ctx* ctx, const ulb_attn_desc* desc, const float* dev_q,
                  const uint16_t* dev_k, const uint16_t* dev_v, const int32_t* dev_row_seq,
                  const int32_t* dev_row_pos, int M, int rows_per_seq, uint16_t* dev_out);

/*
 * Kernel form of every attention launch on this context (ulb_attention*, ulb_model_forward,
 * the speculative loop):
 *   ULB_ATTN_AUTO    (default) chosen per launch from the shape
 *   ULB_ATTN_SPLIT   one CTA per (query tile, kv head, sequence, 256-key split): every split in
 *                    flight at once, the short-latency form for a few sequences
 *   ULB_ATTN_STREAM  one CTA per (query tile, kv head, sequence) walking its splits in order
 *                    with the K / V loads of the next split in flight: the throughput form for
 *                    many sequences and long caches
 * Both forms give every row the same bits; the setting only moves time.  No counterpart in
 * the reference (its flash_attention dispatch has one form, inference_engine.cpp:628-630).
 */
#define ULB_ATTN_AUTO 0
#define ULB_ATTN_SPLIT 1
#define ULB_ATTN_STREAM 2
ULB_API int ulb_attention_set_form(ulb_ctx* ctx, int form);

/*
 * ulb_attention over a paged KV cache, the layout the model caches use.  A sequence's
 * positions map to pages of ULB_KV_PAGE positions through its row of the block table:
 *   dev_k_pool/dev_v_pool  fp16 [n_pages][n_head_kv][ULB_KV_PAGE][head_dim]
 *   dev_block_table        int32 [n_seq][max_pages]: page of positions [j*ULB_KV_PAGE, (j+1)*ULB_KV_PAGE)
 *                          of sequence s at [s*max_pages + j], -1 = unmapped (those keys are
 *                          treated as absent; nothing is read there)
 * desc->capacity <= max_pages * ULB_KV_PAGE.  Everything else as ulb_attention.  Replaces the
 * reference's KVCache::retrieve over one flat host array per layer (src/inference/model.h:49-77).
 */
#define ULB_KV_PAGE 256
ULB_API int ulb_attention_paged(ulb_ctx* ctx, const ulb_attn_desc* desc, const float* dev_q,
                        const uint16_t* dev_k_pool, const uint16_t* dev_v_pool, const int32_t* dev_block_table,
                        int max_pages, const int32_t* dev_row_seq, const int32_t* dev_row_pos, int M,
                        int rows_per_seq, uint16_t* dev_out);

/*
 * ulb_attention without any device allocation.  This entry point has no counterpart in the
 * reference.  It is for callers that must not call cudaMalloc / cudaFree: code that runs
 * between the kernels of a latency-bound decode step (an allocation can synchronise the
 * whole device), code whose device memory is already reserved by another allocator (a
 * framework's caching allocator), and processes with no memory headroom left.
 *   - Arguments, results and errors are those of ulb_attention.  The split-KV partials and
 *     counters live in a static device array of 8 MiB + 32 KiB that every GPU loading this
 *     library holds until the process exits; a shape needing more scratch than that (at most
 *     2 Mi floats and 8192 counters, see ulb_attention's geometry) is rejected with
 *     ULB_EINVAL before anything is launched.
 *   - The first call on a device looks the array up (cudaGetSymbolAddress) on the current
 *     device; make that first call before any stream capture.
 *   - Every call shares the one array and its contents persist between calls (the counters
 *     are cleared by each call): calls that overlap on the GPU — on two streams, or from two
 *     contexts on the same device — race and give wrong results.  Calls on one context's
 *     stream are ordered and safe.
 *   - The call enqueues work and returns without synchronising; a device-side error is
 *     reported by the next ulb_stream_sync.
 */
ULB_API int ulb_attention_noalloc(ulb_ctx* ctx, const ulb_attn_desc* desc, const float* dev_q,
                          const uint16_t* dev_k, const uint16_t* dev_v, const int32_t* dev_row_seq,
                          const int32_t* dev_row_pos, int M, int rows_per_seq, uint16_t* dev_out);

/*
 * Logit warping shared by the draft sampler and the rejection sampler.  Replaces the
 * intent of TextGenerator::apply_temperature / apply_top_k / apply_top_p
 * (src/api/gguf_loader.cpp:90-155) and InferenceEngine::sample_token
 * (src/inference/inference_engine.cpp:340-367).
 *   temperature <= 0  -> greedy (argmax, lowest index on ties)
 *   top_k <= 0 or >= V -> off;  top_p <= 0 or >= 1 -> off
 * Order: logits / T -> keep logits >= k-th largest -> softmax -> keep tokens whose
 * strictly-more-probable mass is < top_p -> renormalise.
 */
typedef struct ulb_warp {
  float temperature;
  int top_k;
  float top_p;
} ulb_warp;

/* Sample one token per row: u = Philox uniform (seed; round, seq=row, slot, tag). */
ULB_API int ulb_sample(ulb_ctx* ctx, const float* dev_logits, int rows, int V, int ld,
               const ulb_warp* warp, uint64_t seed, uint32_t round, uint32_t slot,
               uint32_t tag, int32_t* dev_out_tokens);

/*
 * Single-pass speculative rejection sampling (Leviathan et al. 2023; Chen et al. 2023),
 * replacing SpeculativeDecoder::verify_speculation (src/inference/speculative_decoder.cpp:89-110).
 *   p_logits [B][k+1][V] target logits, q_logits [B][k][V] draft logits,
 *   draft_tokens [B][k].  For i = 0..k-1: accept draft i iff u_i * q_i(x_i) < p_i(x_i);
 *   at the first rejection sample from norm(max(0, p_i - q_i)); if all k are accepted
 *   sample a bonus from p_k.  Greedy warp: accept iff x_i == argmax p_i, correction /
 *   bonus = argmax.  Uniforms: tag ULB_RNG_ACCEPT slot i, tag ULB_RNG_RESID slot n.
 *   out_tokens [B][k+1]: the n accepted drafts followed by the correction/bonus token.
 *   out_n_accepted [B]: n in 0..k (tokens committed = n + 1).
 */
ULB_API int ulb_spec_accept(ulb_ctx* ctx, const float* dev_p_logits, const float* dev_q_logits,
                    const int32_t* dev_draft_tokens, int B, int k, int V, const ulb_warp* warp,
                    uint64_t seed, uint32_t round, int32_t* dev_out_tokens,
                    int32_t* dev_out_n_accepted);

/* ------------------------------------------------------------------ models */
/*
 * A LLaMA-family model resident in HBM.  Replaces Model / LayerWeights / KVCache
 * (src/inference/model.h:37-115, model.cpp:154-254) on the device side.  Tensors are
 * given by their GGUF names (token_embd.weight, blk.N.attn_q.weight, ..., output.weight).
 * Types: the linear weights Q4_0 / Q4_K; token_embd.weight F32 / F16 / Q4_0 / Q8_0 / Q4_K /
 * Q6_K (rows dequantised inside the embedding kernel); output.weight Q4_0 / Q4_K / Q8_0 / Q6_K
 * (Q8_0 / Q6_K kept as GGUF rows for a row GEMV) -- the types llama.cpp's Q4_0 files use.
 */
typedef struct ulb_model_desc {
  int n_layer, d_model, n_head, n_head_kv, head_dim, d_ff, n_vocab;
  float rms_eps, rope_base;
  int max_rows; /* largest number of query rows one forward may carry */
} ulb_model_desc;

ULB_API int ulb_model_create(ulb_ctx* ctx, const ulb_model_desc* desc, ulb_model** out);
/*
 * Tensor parallelism (config 5).  Call after ulb_model_create and before the first
 * ulb_model_set_weight, on a context that has joined a communicator (ulb_tp_init): rank r of
 * `world` keeps heads [r H/world, (r+1) H/world) of Q / K / V and their KV cache, features
 * [r F/world, ...) of gate / up, and the matching column (K) slices of attn_output and
 * ffn_down, sliced on the host while the tensors are set; embeddings, norms and output.weight
 * are replicated.  Every forward then sums the attn_output and ffn_down partial outputs
 * across the ranks with an fp32 NCCL all-reduce before the residual add, so every rank holds
 * the same residual stream and logits.  H, n_head_kv and d_ff must divide by `world`, and the
 * K slices must be whole quantisation blocks.  Replaces the reference's unimplemented
 * multi-GPU path (InferenceAPI::enable_multi_gpu, src/api/inference_api.cpp).
 */
ULB_API int ulb_model_set_tp(ulb_model* m, int rank, int world);
ULB_API int ulb_model_set_weight(ulb_model* m, const char* gguf_name, int ggml_type,
                         const uint64_t ne[4], const void* gguf_bytes, size_t nbytes);
/* Check every tensor is present and build the fused device layouts. */
ULB_API int ulb_model_finalize(ulb_model* m);
ULB_API int ulb_model_free(ulb_model* m);
ULB_API int ulb_model_weight_bytes(const ulb_model* m, size_t* out_bytes);

/* KV cache, paged: per layer a pool of pages fp16 [page][n_head_kv][ULB_KV_PAGE][head_dim] for K
 * and for V, and a block table [n_seq][max_pages] mapping each sequence's positions to pages
 * (replaces the reference's KVCache of one host array per layer, src/inference/model.h:49-77,
 * model.cpp:11-131).  ulb_kv_alloc gives every sequence the pages of its whole capacity
 * (identity table).  ulb_kv_alloc_paged makes a pool of n_pages pages shared by n_seq
 * sequences of at most max_pages_per_seq pages each, all unmapped; ulb_kv_map then maps
 * pages [first, first + n) of sequence seq (page ids, -1 = unmap) -- enqueued on the context
 * stream, so kernels after it see the new mapping.  Keys on unmapped pages are absent to the
 * attention and K / V rows for them are not written. */
ULB_API int ulb_kv_alloc(ulb_ctx* ctx, const ulb_model* m, int n_seq, int capacity, ulb_kv** out);
ULB_API int ulb_kv_alloc_paged(ulb_ctx* ctx, const ulb_model* m, int n_seq, int n_pages, int max_pages_per_seq,
                               ulb_kv** out);
ULB_API int ulb_kv_map(ulb_kv* kv, int seq, int first, int n, const int32_t* host_pages);
ULB_API int ulb_kv_free(ulb_kv* kv);

/*
 * One forward pass of M rows (rows_per_seq consecutive rows per sequence).
 *   dev_tokens/dev_row_seq/dev_row_pos int32 [M].  K/V of every row are written at
 *   (seq, pos); row m attends positions 0..pos of its sequence.
 *   logits_mode 0: logits for all M rows -> dev_logits[m*ld + v]
 *   logits_mode 1: logits only for the last row of each sequence -> dev_logits[s*ld + v]
 */
ULB_API int ulb_model_forward(ulb_ctx* ctx, ulb_model* m, ulb_kv* kv, int M, int rows_per_seq,
                      const int32_t* dev_tokens, const int32_t* dev_row_seq,
                      const int32_t* dev_row_pos, int logits_mode, float* dev_logits, int ld);

/* ------------------------------------------------------------------ speculative loop */
/*
 * Device-resident draft -> verify -> accept loop.  Replaces SpeculativeDecoder
 * (src/inference/speculative_decoder.h:24-60, .cpp:25-116) and the engine's decode loop
 * (src/inference/inference_engine.cpp:273-328).  With draft == NULL (or k == 0) each round
 * is one target step (plain decoding) through the same code.
 */
typedef struct ulb_spec_desc {
  int n_seq;        /* sequences decoded together                           */
  int k;            /* draft tokens per round (speculation length)          */
  int max_prompt;   /* longest prompt                                       */
  int max_new;      /* tokens to commit per sequence                        */
  ulb_warp warp;    /* applied identically to target and draft               */
  uint64_t seed;    /* Philox key                                           */
  int use_graphs;   /* 1: capture each round into a CUDA graph              */
  int kv_pages;     /* 0: every sequence slot owns pages for its whole capacity;
                       > 0: a pool of this many pages per model, mapped to the slots
                       as their sequences grow and returned when they finish     */
  int tree_width;   /* 0 or 1: a chain of k drafts per round; >= 2: tree speculation, a
                       full tree of this width and depth k (the reference's
                       TreeSpeculation(vocab, beam_width, max_depth),
                       src/inference/speculative_decoder.h:62-87, a stub there): k draft
                       steps over the tree's levels, one verify over all its nodes with
                       tree attention, multi-candidate acceptance (ulb_spec_tree_accept);
                       at most 63 nodes (width^1 + ... + width^k) and width <= 8 */
} ulb_spec_desc;

ULB_API int ulb_spec_create(ulb_ctx* ctx, ulb_model* target, ulb_model* draft,
                    const ulb_spec_desc* desc, ulb_spec** out);

/*
 * Acceptance of speculation trees (one per sequence), the decision of a tree round.  A tree
 * of width w and depth D has N = w + w^2 + ... + w^D nodes numbered breadth first from depth 1
 * (node i of depth d has rank r = i - first(d), first(d) = w + ... + w^(d-1); the root's
 * children are nodes 0..w-1, node i's are first(d+1) + r*w + c).  The root is the last
 * committed token.
 *   dev_p       fp32 target logits [B][1 + N][V]: row 0 the root, row 1 + i node i
 *   dev_q       fp32 draft logits [B][1 + NI][V] of the root and the NI = first(D) internal
 *               nodes (the distributions the children were drawn from)
 *   dev_tokens  int32 [B][N] the drafted token of each node
 * From the root, the children of the current node are tested in order: T = 0, the first whose
 * token is the target's argmax is accepted; T > 0, multi-candidate speculative sampling
 * (SpecInfer, Miao et al. 2024, for children drawn independently from q): child c_j is
 * accepted with probability min(1, P_j(x) / q(x)), P_1 = p and P_(j+1) = norm(max(0, P_j - q))
 * after each rejection; the first accepted child becomes the current node.  When all children
 * are rejected the correction is drawn from the last residual (T = 0: the argmax); a leaf
 * reached adds a bonus token from its p.  Uniforms: Philox (seed, round, sequence b, slot,
 * tag) with the child's node index as slot for its test (ULB_RNG_ACCEPT) and the node's p row
 * as slot for a correction / bonus draw (ULB_RNG_RESID).  A tree of width 1 is the chain of
 * ulb_spec_accept.
 *   dev_path    int32 [B][D]: the accepted nodes, -1 after;  dev_n int32 [B]: their number;
 *   dev_tok     int32 [B]: the correction / bonus token.
 * Replaces TreeSpeculation::generate_tree_speculation / verify_tree
 * (src/inference/speculative_decoder.cpp:118-176, which returns its placeholder tree).
 */
ULB_API int ulb_spec_tree_accept(ulb_ctx* ctx, const float* dev_p, const float* dev_q, const int32_t* dev_tokens,
                         int B, int width, int depth, int V, const ulb_warp* warp, uint64_t seed,
                         uint32_t round, int32_t* dev_path, int32_t* dev_n, int32_t* dev_tok);
/* Copy prompts (host int32 [n_seq][max_prompt], lengths [n_seq]) and prefill both models;
 * commits the first generated token of every sequence. */
ULB_API int ulb_spec_prefill(ulb_spec* s, const int32_t* host_prompts, const int32_t* host_prompt_lens);
/* Run rounds until every sequence has max_new tokens or max_rounds rounds ran. */
ULB_API int ulb_spec_run(ulb_spec* s, int max_rounds, int* out_rounds);
/*
 * Continuous batching: start a new sequence in slot `slot` (0..n_seq-1) once its previous one
 * is done (ULB_EINVAL while it is still decoding): the prompt (host int32, len <= max_prompt)
 * is prefilled into both caches -- on pages taken from the pool when kv_pages > 0 -- and its
 * first token committed; the next ulb_spec_run rounds decode it with the other live slots.
 * Read the finished sequence's tokens (ulb_spec_read) before admitting a new one.  The slot's
 * Philox stream restarts at round 0 (sampled decoding of successive occupants of one slot
 * draws the same uniforms).  Replaces ContinuousBatcher's queue -> padded batch stub
 * (src/inference/continuous_batcher.cpp:20-122), which never reached a model.
 */
ULB_API int ulb_spec_admit(ulb_spec* s, int slot, const int32_t* host_prompt, int len);
/* host_tokens int32 [n_seq][max_new], host_counts [n_seq];
 * stats: [0] rounds, [1] drafted tokens, [2] accepted drafts, [3] committed tokens. */
ULB_API int ulb_spec_read(ulb_spec* s, int32_t* host_tokens, int32_t* host_counts, uint64_t stats[4]);
/*
 * Per-round speculation records of sequence `seq` since its last prefill, in round order:
 * the device form of the reference's SpeculationResult / SpeculativeToken
 * (src/inference/speculative_decoder.h:11-22), one record per round in which the sequence
 * was still decoding.  Each record is ULB_SPEC_REC_WORDS(k) int32 words:
 *   [ULB_SPEC_REC_N_ACCEPTED]  n, drafts accepted (0..k); the round committed n + 1 tokens
 *   [ULB_SPEC_REC_TOKEN]       the correction (n < k) or bonus (n == k) token
 *   [ULB_SPEC_REC_POSITION]    sequence position of the first committed token
 *   [ULB_SPEC_REC_K]           k, the drafts proposed
 *   [ULB_SPEC_REC_DRAFTS + i]  draft token i, i = 0..k-1 (accepted: i < n; rejected: i >= n)
 *   [ULB_SPEC_REC_DRAFTS + k + j], j = 0..n: the float bits of the target's probability
 *       (under the warp) of committed token j (greedy decoding: 1.0)
 * *out_n = the number of records (up to max_new + 1); at most max_records are copied to
 * host_records (NULL to ask for the count only).
 */
#define ULB_SPEC_REC_N_ACCEPTED 0
#define ULB_SPEC_REC_TOKEN 1
#define ULB_SPEC_REC_POSITION 2
#define ULB_SPEC_REC_K 3
#define ULB_SPEC_REC_DRAFTS 4
#define ULB_SPEC_REC_WORDS(k) (ULB_SPEC_REC_DRAFTS + 2 * (k) + 1)
ULB_API int ulb_spec_read_rounds(ulb_spec* s, int seq, int max_records, int32_t* host_records, int* out_n);
ULB_API int ulb_spec_free(ulb_spec* s);
/* Run one round outside any CUDA graph with events between its phases:
 * ms[0] draft steps, ms[1] verify forward, ms[2] accept.  Sequences already done are computed
 * but nothing is committed for them.  Replaces the reference's never-constructed
 * vulkan::Profiler timestamps (src/vulkan_backend/profiler.cpp:174-230). */
ULB_API int ulb_spec_profile_round(ulb_spec* s, float ms[3]);
/* ulb_spec_profile_round plus the tensor-parallel exchange of the round: ms[3] the summed
 * CUDA-event time of the round's NCCL all-reduces (each measured on the context stream from
 * just before ncclAllReduce to just after, so it includes waiting for the slowest rank; 0
 * without a communicator), ms[4] how many there were.  Replaces the per-dispatch timestamps
 * the reference's multi-GPU manager never takes (src/vulkan_backend/multi_gpu_manager.cpp). */
ULB_API int ulb_spec_profile_round_ex(ulb_spec* s, float ms[5]);
/* Kernels this loop launched since its last prefill (prefill and every round included). */
ULB_API int ulb_spec_launch_count(ulb_spec* s, uint64_t* out);

#ifdef __cplusplus
}
#endif
#endif /* ULB_H */
