/* rpg_oracle.h -- CPU restatement of the reference's token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA engine:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * it.  The engine never calls it and has no CPU fallback.
 *
 * What it restates (reference paths relative to the RPGBarEngineCUDA tree):
 *   dequant      src/quant.cc:159-167, 252-277, 321-354 (bit-exact; built
 *                with -ffp-contract=off like CMakeLists.txt:120-127)
 *   f16          src/dtypes.h:21-48 (f16 -> f32); f32 -> f16 is RNE, the
 *                rounding of __float2half_rn used by KvWriteKernel
 *                (src/kernels_gpu.cu:725), not dtypes.h:50's F32ToF16
 *   forward      src/qwen3_gpu.cu:47-180 op order; RMSNorm with a double sum
 *                (src/kernels_gpu.cu:564-591); RoPE table in double
 *                (src/gpu_model.cu:90-120), rotate-half (kernels_gpu.cu:598-621);
 *                fp16 KV (kv_cache_gpu.cu); attention with a double softmax sum
 *                (kernels_gpu.cu:737-823); SiLU (863-869); tied lm_head
 *   sampler      src/sampler_gpu.cu:42-56 (SplitMix64 counter RNG), 161-290
 *                (FilterProbsKernel: 32-step bisections), 312-336 (serial
 *                inverse transform), src/sampler.h:35-44 (options)
 *   generate     src/qwen3_gpu.cu:532-595 (sample -> append -> forward; the
 *                stop token is forwarded; counter = absolute position)
 * Arithmetic inside each op is double; values are rounded to float wherever the
 * reference stores them in a float buffer, and to fp16 where it stores fp16.
 */
#ifndef RPG_ORACLE_H
#define RPG_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);
int orc_dequant_row(uint32_t type, const uint8_t* src, int64_t n, float* dst);

/* out[t][r] = sum_c W[r][c] * x[t][c] over raw GGUF rows (double accumulation). */
int orc_matvec(uint32_t type, const uint8_t* w, int64_t rows, int64_t cols, const float* x, int64_t n_tok,
               float* out, int n_threads);

typedef struct orc_model orc_model;
orc_model* orc_model_open(const char* path, int32_t max_pos, char* err, int errlen);
void orc_model_close(orc_model* m);
/* n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, context, rope_positions, eos */
void orc_model_shape(const orc_model* m, int32_t* out10);

typedef struct orc_session orc_session;
orc_session* orc_session_create(orc_model* m, int32_t max_seq, int n_threads);
void orc_session_free(orc_session* s);
int64_t orc_session_len(const orc_session* s);
void orc_session_set_len(orc_session* s, int64_t len);
/* Appends tokens; last_logits[vocab] (nullable) receives the last position's
 * logits; hidden (nullable) receives the residual stream [n_layers+1][n][hidden]. */
int orc_prefill(orc_session* s, const int32_t* tokens, int64_t n, float* last_logits, float* hidden);
int orc_generate(orc_session* s, float temperature, int32_t top_k, float top_p, uint64_t seed, int32_t max_tokens,
                 const int32_t* stop, int32_t n_stop, int32_t* out, float* step_logits);

float orc_counter_uniform(uint64_t seed, uint64_t counter);
void orc_filter_to_probs(const float* logits, int64_t n, float temperature, int32_t top_k, float top_p,
                         float* probs);
int32_t orc_sample_token(const float* logits, int64_t n, float temperature, int32_t top_k, float top_p, float u);

#ifdef __cplusplus
}
#endif

#endif
