/* rpg_b200.h -- C ABI of the B200 token loop (model, session, prefill, generate)
 * and of its operators.  Plain pointers and sizes only; every function is
 * exported from librpg_engine_b200.so next to the ten rpg_engine_* functions.
 *
 * These are the entry points the reference's own tools bind to its internal
 * C++ API (tools/gen_check.cu, tools/graph_check.cu, tools/sample_check.cu,
 * tools/dequant_check.cu, tools/matmul_bench.cu).  The public rpg_engine_*
 * ABI (rpg_engine.h) cannot carry raw token ids or top_k / top_p
 * (src/engine.cc:459-469, 552-553), so parity and benchmarking go through
 * these, exactly as the reference's tools bypass its ABI.
 *
 * Conventions (same as the reference ABI, include/rpg_engine.h:46-48):
 * handles are >= 0 when valid; functions returning int32_t return 0 (or a
 * handle) on success and a negative value on failure with the message in
 * rpgb_last_error() (thread-local).  No C++ exception crosses this boundary.
 * Host buffers are plain host memory; "_dev" arguments are device pointers on
 * the model's device and `stream` is a cudaStream_t (NULL = legacy stream).
 */
#ifndef RPG_B200_H
#define RPG_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define RPGB_API __attribute__((visibility("default")))
#else
#define RPGB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Sampling parameters; same fields and defaults as the reference's
 * SampleOptions (src/sampler.h:35-44): temperature <= 0 is greedy, top_k is
 * active iff 1 < top_k < vocab, top_p is active iff 0 < top_p < 1. */
typedef struct rpgb_sample_options {
  float temperature;
  int32_t top_k;
  float top_p;
} rpgb_sample_options;

RPGB_API const char* rpgb_version(void);
RPGB_API const char* rpgb_last_error(void);

/* ------------------------------------------------------------------ model */

/* Loads a GGUF (qwen3, Q4_K / Q6_K matrices) onto `device` with a RoPE table
 * of min(max_pos, context_length) positions.  Replaces GpuModel::Load
 * (src/gpu_model.cu:148-246).  Returns a model handle. */
RPGB_API int32_t rpgb_model_load(const char* gguf_path, int32_t device, int32_t max_pos);
RPGB_API void rpgb_model_free(int32_t model);

/* Shape of a loaded model, written to out[0..11]: n_layers, hidden, n_heads,
 * n_kv_heads, head_dim, ffn, vocab, context_length, rope_positions, eos_id,
 * device, num_sms.  Mirrors ModelMeta (src/model_meta.h:27-62). */
RPGB_API int32_t rpgb_model_shape(int32_t model, int32_t* out, int32_t n_out);
/* Device bytes of the resident weights (GpuModel::device_bytes). */
RPGB_API int64_t rpgb_model_device_bytes(int32_t model);

/* ------------------------------------------------------------------ tensor parallel */

/* Tensor parallelism over NCCL, one process (or thread) and one GPU per rank.
 * No counterpart in the reference, which runs one GPU; the split is the one
 * planned for the 8B configuration: each rank holds 1/size of the query and
 * KV heads and of the FFN, the embedding and norms in full, 1/size of the
 * lm_head rows; the ranks sum a partial after attn_output and after ffn_down
 * and gather the logits, then all sample the same token.
 *
 * rpgb_tp_shard_plan: shape = {n_heads, n_kv_heads, head_dim, ffn, vocab};
 * out[0..4] = this rank's heads, KV heads, ffn columns, first vocabulary row
 * and vocabulary rows.  Fails when the model does not split evenly (KV heads
 * by size, attn_output and ffn_down columns into 256-column super-blocks,
 * vocabulary rows into 16-row tiles).  Host only.
 * rpgb_tp_unique_id: 128 bytes (ncclGetUniqueId) that rank 0 makes and every
 * rank passes to rpgb_tp_group_create (collective).  A model loaded with
 * rpgb_model_load_tp holds its rank's shard; prefill and generate on its
 * sessions are collective: every rank calls them with the same arguments, in
 * the same order. */
RPGB_API int32_t rpgb_tp_shard_plan(const int32_t* shape, int32_t rank, int32_t size, int32_t* out);
RPGB_API int32_t rpgb_tp_unique_id(uint8_t* id_out);
RPGB_API int32_t rpgb_tp_group_create(const uint8_t* id, int32_t rank, int32_t size, int32_t device);
RPGB_API void rpgb_tp_group_free(int32_t group);
RPGB_API int32_t rpgb_model_load_tp(const char* gguf_path, int32_t device, int32_t max_pos, int32_t group);
/* Greedy decode of a tensor-parallel session runs in the one-launch decode
 * loop with the ranks' partials exchanged directly between the GPUs' memory:
 * each rank's session exports a 64-byte CUDA IPC handle
 * (rpgb_session_tp_handle) and attaches the handles of all ranks, in rank
 * order (rpgb_session_tp_attach, collective).  Sessions not attached, and
 * sampled decode, go through the step graph with NCCL. */
RPGB_API int32_t rpgb_session_tp_handle(int32_t session, uint8_t* handle_out);
RPGB_API int32_t rpgb_session_tp_attach(int32_t session, const uint8_t* handles);

/* ------------------------------------------------------------------ session */

/* A session owns an fp16 KV cache of max_seq positions, scratch buffers and
 * a stream (GpuKvCache + GpuScratch, src/kv_cache_gpu.cu:16-36,
 * src/qwen3_gpu.h:79-98). */
RPGB_API int32_t rpgb_session_create(int32_t model, int64_t max_seq);
RPGB_API void rpgb_session_free(int32_t session);
RPGB_API int64_t rpgb_session_len(int32_t session);
/* GpuKvCache::SetLen (src/kv_cache_gpu.cu:54-58): positions >= len are
 * forgotten; the next generate needs a prefill first. */
RPGB_API int32_t rpgb_session_set_len(int32_t session, int64_t len);

/* GpuForwardFull with a KV cache (src/qwen3_gpu.cu:236-276): appends n
 * tokens at positions len .. len+n-1; the logits of the last position stay on
 * the device for rpgb_generate and are copied to last_logits[vocab] when that
 * pointer is not NULL. */
RPGB_API int32_t rpgb_prefill(int32_t session, const int32_t* tokens, int64_t n, float* last_logits);

/* GpuGenerate (src/qwen3_gpu.cu:599-640): samples from the current logits
 * with counter = absolute position, forwards every returned token (the stop
 * token included), stops after max_tokens or at the first id in stop_ids.
 * out_ids[max_tokens] receives the tokens, *n_out their count.  step_logits,
 * when not NULL, receives [max_tokens][vocab]: the distribution each token was
 * sampled from (GpuGenerateOptions::step_logits). */
RPGB_API int32_t rpgb_generate(int32_t session, const rpgb_sample_options* opt, uint64_t seed, int32_t max_tokens,
                               const int32_t* stop_ids, int32_t n_stop, int32_t* out_ids, int32_t* n_out,
                               float* step_logits);

/* Kernel launches per decode step and whether the step graph is recorded
 * (the reference's graph_check asserts graph_exec != nullptr). */
RPGB_API int32_t rpgb_session_stats(int32_t session, int32_t* kernels_per_step, int32_t* graph_ready,
                                    int64_t* graph_launches);

/* The session's CUDA stream (a cudaStream_t), so a caller can time the
 * session's work with CUDA events recorded on that stream. */
RPGB_API void* rpgb_session_stream(int32_t session);

/* Device timeline of decoding (no counterpart in the reference, which times
 * whole steps only).  In the decode loop kernel every block writes, per step
 * phase, a record {launch = step * (5 n_layers + 2) + phase, block, start =
 * end of the block's previous phase, ready = after the grid barrier where
 * there is one, end} and up to four mark records inside the phase (block
 * field | mark << 24, end = time of the mark); times are nanoseconds of the
 * SM clock anchored to %globaltimer.  In the step graph (other group sizes)
 * every block of every launch writes {launch index within the step, block,
 * start, ready = after the wait on the previous launch, end}.
 * trace_enable(cap) sets room for `cap` records (0 = off); trace_take copies
 * up to `cap` records into `out` (host memory, 32 bytes each), clears the
 * buffer and returns the count. */
typedef struct rpgb_trace_rec {
  uint32_t launch, block;
  uint64_t t_start, t_ready, t_end;
} rpgb_trace_rec;
RPGB_API int32_t rpgb_session_trace_enable(int32_t session, int32_t cap);
RPGB_API int32_t rpgb_session_trace_take(int32_t session, rpgb_trace_rec* out, int32_t cap);

/* Kernels this library has launched so far in the process (a decode loop
 * launch counts once, every node of a replayed step graph once per replay;
 * instrumentation for benchmarks). */
RPGB_API int64_t rpgb_launch_count(void);

/* ------------------------------------------------------------------ operators */

/* Uploads one GGUF matrix (Q4_K or Q6_K bytes, rows x cols) to `device` in
 * the engine's layout; returns a matrix handle (GpuModel::UploadMatrix,
 * src/gpu_model.cu:44-57). */
RPGB_API int32_t rpgb_matrix_upload(int32_t device, uint32_t ggml_type, int64_t rows, int64_t cols,
                                    const void* gguf_bytes);
RPGB_API void rpgb_matrix_free(int32_t matrix);

/* dst_dev[r][c] = dequant(row0 + r, c): bit-exact per element
 * (GpuDequantRow, src/kernels_gpu.cu:929-937). */
RPGB_API int32_t rpgb_matrix_dequant(int32_t matrix, int64_t row0, int64_t n_rows, float* dst_dev, void* stream);

/* out_dev[t][r] = sum_c W[r][c] * x_dev[t][c] (GpuMatMulQuant,
 * src/kernels_gpu.cu:939-975): n_tok == 1 uses the decode matvec, larger n
 * the prefill GEMM -- from 16 tokens (and rows a multiple of 128) the
 * tcgen05 tensor-core GEMM, which keeps fp16 operand scratch with the matrix
 * (so calls on one matrix must be ordered: one stream, or events between
 * streams).  Every path returns without waiting for the GPU and can be
 * captured in a CUDA graph once a first call with the largest n_tok has run;
 * a bounded device wait of the tensor-core GEMM that gave up is reported
 * (-1) by the next call on the same matrix. */
RPGB_API int32_t rpgb_matrix_matvec(int32_t matrix, const float* x_dev, int64_t n_tok, float* out_dev,
                                    void* stream);

/* GpuSampleToken / GpuFilterToProbs (src/sampler_gpu.cu:393-440): samples
 * one token of logits_dev[n] with u = counter_uniform(seed, counter) into
 * *out_tok_dev.  When probs_dev is not NULL it receives the filtered
 * distribution (the general path runs; otherwise the fast top-k path may). */
RPGB_API int32_t rpgb_sample(const float* logits_dev, int32_t n, const rpgb_sample_options* opt, uint64_t seed,
                             uint64_t counter, float* probs_dev, int32_t* out_tok_dev, void* stream);

/* rpgb_sample without any device-memory allocation.  No counterpart in the
 * reference: it exists for hosts that cannot allocate GPU memory when they
 * sample -- a game or UI thread that must never block (cudaMalloc and
 * cudaFree synchronise the whole device), or a process whose GPU memory is
 * already fully owned by another allocator's pool.  Same sampling as
 * rpgb_sample with probs_dev == NULL; its scratch is a fixed array inside the
 * library (about 1.1 MiB), so n must not exceed RPGB_SAMPLE_NOALLOC_MAX_VOCAB.
 * CUDA loads the library's code lazily: the array is placed on a GPU by the
 * first call on that device (or when the context starts, with
 * CUDA_MODULE_LOADING=EAGER) and held until the process exits, so make one
 * call per device at set-up, before the GPU's memory is handed to another
 * allocator and before any stream capture begins.  All calls on a device
 * share the array: calls whose GPU work overlaps race and must be
 * serialised. */
#define RPGB_SAMPLE_NOALLOC_MAX_VOCAB 262144
RPGB_API int32_t rpgb_sample_noalloc(const float* logits_dev, int32_t n, const rpgb_sample_options* opt,
                                     uint64_t seed, uint64_t counter, int32_t* out_tok_dev, void* stream);

/* u = H(seed, counter) in [0, 1) (DevCounterUniform, src/sampler_gpu.cu:364). */
RPGB_API float rpgb_counter_uniform(uint64_t seed, uint64_t counter);

/* ------------------------------------------------------------------ text layer
 *
 * The host text layer rpg_engine_generate runs, without a GPU: the same token
 * ids, prompt and parse a request turns into.  Errors return NULL / -1 with
 * the text in rpg_engine_last_error(); strings are freed with
 * rpg_engine_free(). */

/* Tokenizer of a GGUF (Tokenizer::FromGguf, src/tokenizer.cc:132-200). */
RPGB_API void* rpgb_text_open(const char* gguf_path);
RPGB_API void rpgb_text_close(void* text);

/* Token ids of len bytes of text, special tokens matched when parse_special
 * (Tokenizer::Encode, src/tokenizer.cc:314); writes up to cap ids, returns
 * the full count. */
RPGB_API int64_t rpgb_text_encode(void* text, const char* bytes, int64_t len, int32_t parse_special, int32_t* out,
                                  int64_t cap);

/* Bytes of ids, specials kept (Tokenizer::Decode, src/tokenizer.cc:353);
 * *out_len receives the length (the bytes may hold NUL). */
RPGB_API char* rpgb_text_decode(void* text, const int32_t* ids, int64_t n, int64_t* out_len);

/* The ChatML prompt of a generate request's messages / tools /
 * enable_thinking (ParseMessages + RenderChatml, src/chat_template.cc:85-206). */
RPGB_API char* rpgb_text_render(const char* request_json);

/* The parse of raw model output (ParseModelOutput, src/tool_parser.cc:125-178)
 * as JSON: {text, tool_calls: [{name, arguments}], unterminated_think,
 * unterminated_tool_call}. */
RPGB_API char* rpgb_text_parse(const char* raw, int64_t len);

#ifdef __cplusplus
}
#endif

#endif /* RPG_B200_H */
