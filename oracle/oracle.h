/*
 * oracle.h — CPU restatement of the speculative draft -> verify -> accept path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libulb_cuda.so, the engine, the
 * vulkangguf module) links, loads or calls this code.  It is the checker that the CUDA
 * path is compared against in tests/, in __graft_entry__.smoke(), and the timed CPU
 * baseline in bench.py.
 *
 * What it follows (reference paths are relative to the Universal-Loader tree):
 *  - GGUF container parsing as src/core/gguf_parser.cpp:18-361 (header, KV metadata,
 *    tensor infos, data offset aligned to general.alignment), with tensor byte sizes from
 *    the GGUF block table (Q4_0: 18 B / 32, Q4_K: 144 B / 256) instead of the reference's
 *    ggml_type_size (src/core/gguf_types.h:35-58), which is wrong for both.
 *  - Q4_0 / Q4_K block decoding as the GGUF format defines it (the reference's decoders,
 *    src/cpu_backend/dequantize_cpu.cpp:6-74, use invented layouts and are not followed);
 *    also Q8_0 (34 B / 32) and Q6_K (210 B / 256), for the token_embd / output.weight types
 *    of llama.cpp's Q4_0 files (a widening: the reference's type set stops at Q4_K).
 *  - the reference's per-layer op order (src/inference/inference_engine.cpp:602-682:
 *    norm -> Q,K,V -> RoPE -> attention -> o -> +res -> norm -> gate,up -> SiLU*mul ->
 *    down -> +res) with each op given its standard LLaMA meaning: RMSNorm with eps,
 *    adjacent-pair RoPE as src/shaders/rope.glsl:50-74 with a configurable theta base,
 *    GQA causal attention over the KV cache (the feature list of
 *    src/shaders/attention/flash_attention_v2_fused.glsl:13-24), SwiGLU, final norm and
 *    LM head.
 *  - sampling warps as src/api/gguf_loader.cpp:90-155 intends (temperature, top-k, top-p)
 *    and speculative rejection sampling (Leviathan et al. 2023) in place of the
 *    reference's token-match heuristic (src/inference/speculative_decoder.cpp:89-110).
 *
 * Rounding points mirror the device path: fp32 residual stream, fp16 activations at
 * every linear input, fp16 K/V cache, fp32 accumulation with each quant block's scale
 * applied to the block's integer dot product, probabilities in fp64.
 */
#ifndef ULB_ORACLE_H
#define ULB_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_model orc_model;
typedef struct orc_kv orc_kv;

typedef struct orc_desc {
  int n_layer, d_model, n_head, n_head_kv, head_dim, d_ff, n_vocab;
  float rms_eps, rope_base;
  int wtype; /* weight type of the linear layers */
} orc_desc;

typedef struct orc_warp {
  float temperature;
  int top_k;
  float top_p;
} orc_warp;

/* block formats */
size_t orc_type_nbytes(int type, uint64_t n_elements);
int orc_dequant(int type, const void* blocks, uint64_t n, float* out);
/* y[m*ldy+n] = sum over blocks of scale * integer dot(block, x16[m]) */
int orc_qgemv(int type, const void* w, int N, int K, const uint16_t* x16, int M, float* y, int ldy);
/* fp16 quantisers used by the synthetic model generator's tests */
int orc_quantize_q4_0(const float* x, uint64_t n, void* out);

/* RoPE angle table, identical on host and device: [pos][i] for i < head_dim/2 */
void orc_rope_table(float base, int head_dim, int n_pos, float* cos_out, float* sin_out);

/* attention: q fp32 [M][H][hd], k/v fp16 [S][Hkv][cap][hd] -> out fp16 [M][H][hd] */
int orc_attention(int n_head, int n_head_kv, int head_dim, int cap, float scale, const float* q,
                  const uint16_t* k, const uint16_t* v, const int32_t* row_seq,
                  const int32_t* row_pos, int M, uint16_t* out);

/* GGUF model */
orc_model* orc_model_load(const char* path, char* err, int errlen);
void orc_model_free(orc_model* m);
void orc_model_get_desc(const orc_model* m, orc_desc* d);
/* raw tensor access: returns bytes pointer and fills type/ne; NULL if missing */
const void* orc_model_tensor(const orc_model* m, const char* name, int* type, uint64_t ne[4],
                             size_t* nbytes);

orc_kv* orc_kv_alloc(const orc_model* m, int n_seq, int cap);
void orc_kv_free(orc_kv* kv);
int orc_forward(orc_model* m, orc_kv* kv, int M, int rows_per_seq, const int32_t* tokens,
                const int32_t* row_seq, const int32_t* row_pos, int logits_mode, float* logits,
                int ld);

/* sampling */
float orc_uniform(uint64_t seed, uint32_t round, uint32_t seq, uint32_t slot, uint32_t tag);
void orc_philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1,
                uint32_t out[4]);
/* exp of the warp weights (binary32, the same operations as the device's ulb_warp_exp) */
float orc_warp_exp(float x);
/* unnormalised warp weights e (fp64, zero outside the kept set) and their sum *Z; returns 0 */
int orc_warp_weights(const float* logits, int V, const orc_warp* w, double* e, double* Z);
/* warped probabilities e / Z; returns 0 */
int orc_warp_probs(const float* logits, int V, const orc_warp* w, double* probs);
int orc_sample(const float* logits, int V, const orc_warp* w, float u);
/* tree speculation acceptance (see oracle.c): p rows [B][1+N][V], q rows [B][1+NI][V],
   tokens [B][N] in breadth-first node order; path [B][depth], n [B], tok [B] */
int orc_tree_accept(const float* p_logits, const float* q_logits, const int32_t* tokens, int B, int width,
                    int depth, int V, const orc_warp* w, uint64_t seed, uint32_t round, int32_t* out_path,
                    int32_t* out_n, int32_t* out_tok);
int orc_spec_accept(const float* p_logits, const float* q_logits, const int32_t* draft, int B,
                    int k, int V, const orc_warp* w, uint64_t seed, uint32_t round,
                    int32_t* out_tokens, int32_t* out_n);

/* full loop, same schedule as the device: tokens [n_seq][max_new], stats[4] */
int orc_spec_generate(orc_model* target, orc_model* draft, int n_seq, const int32_t* prompts,
                      const int32_t* prompt_lens, int max_prompt, int max_new, int k,
                      const orc_warp* w, uint64_t seed, int32_t* out_tokens, int32_t* out_counts,
                      uint64_t stats[4], double* top2_margin_min,
                      double* token_margins /* [n_seq][max_new] or NULL: top-2 margin deciding each token (greedy) */);

/* CPU-baseline sample: `rounds` rounds at context ctx_len with pre-filled caches */
int orc_bench_rounds(orc_model* target, orc_model* draft, int ctx_len, int k, int rounds,
                     const orc_warp* w, uint64_t seed, uint64_t stats[4]);

void orc_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
