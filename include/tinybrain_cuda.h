/*
 * tinybrain_cuda.h -- C ABI of libtinybrain_cuda, the B200 (sm_100a) backend
 * for TinyBrain's decode hot path.
 *
 * The reference (vivekptnk/tinybrain, Swift) reaches its GPU backend through a
 * type-erased plugin slot, TinyBrainBackend.metalBackend
 * (Sources/TinyBrainRuntime/Backend.swift:29), and op protocols
 * (Backend.swift:158-228) implemented by MetalBackend
 * (Sources/TinyBrainMetal/MetalBackend.swift).  This header is what a
 * `TinyBrainCUDA` Swift target binds through a module map instead; every
 * entry point names the reference interface it replaces.
 *
 * Conventions
 *  - Every function returns tb_status (0 = TB_OK).  Errors never abort; the
 *    message of the calling thread's last error is tb_last_error().
 *  - Pointers named *_host are caller-owned host memory; *_dev are device
 *    pointers on the context's GPU.  The library owns every object it creates.
 *  - Quantized tensors use the reference's own host layout: shape
 *    [in_features K, out_features N], row-major, y = x * W
 *    (Sources/TinyBrainRuntime/QuantizedTensor.swift:62-165).
 *  - One context per GPU and host thread; objects of a context are not
 *    thread-safe (the reference's ModelRunner is not either).
 */
#ifndef TINYBRAIN_CUDA_H
#define TINYBRAIN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_ABI_VERSION 1

typedef enum {
    TB_OK = 0,
    TB_ERR_INVALID_ARGUMENT = 1,
    TB_ERR_CUDA = 2,
    TB_ERR_OUT_OF_MEMORY = 3,
    TB_ERR_UNSUPPORTED = 4,
    TB_ERR_PAGE_POOL_EXHAUSTED = 5,
    TB_ERR_FORMAT = 6,
    TB_ERR_NO_DEVICE = 7,
    TB_ERR_DEVICE_TIMEOUT = 8,
    TB_ERR_STATE = 9,
    TB_ERR_DEVICE_FAULT = 10
} tb_status;

typedef struct tb_context tb_context;
typedef struct tb_qweight tb_qweight;
typedef struct tb_model tb_model;
typedef struct tb_runner tb_runner;

/* ---------------------------------------------------------------- misc -- */
int32_t tb_abi_version(void);
/* Thread-local message of the last failing call ("" if none). */
const char *tb_last_error(void);
const char *tb_status_string(tb_status s);
tb_status tb_device_count(int32_t *count);

/* Seeded synthetic weights: the reference's Tensor.random(shape:mean:std:using:)
 * over SeededGenerator (Tensor.swift:1623-1644, ModelWeights.swift:18-29).
 * *state is the LCG state (seed 0 maps to 0xdeadbeef, as SeededGenerator.init)
 * and is advanced by 2*ceil(n/2) draws.  Host-side data generation only. */
tb_status tb_rng_seed_state(uint64_t seed, uint64_t *state);
tb_status tb_rng_fill_normal(uint64_t *state, float mean, float std, int64_t n, float *out_host);

/* ------------------------------------------------------------- context -- */
/* Replaces MetalBackend.init (MetalBackend.swift:56-108) + registration in
 * TinyBrainBackend.metalBackend (Backend.swift:29). */
tb_status tb_context_create(int32_t device, tb_context **out);
tb_status tb_context_destroy(tb_context *ctx);
tb_status tb_context_synchronize(tb_context *ctx);
/* The context's CUDA stream (cudaStream_t), for callers that pass *_dev buffers. */
void *tb_context_stream(tb_context *ctx);
/* Device-side error word (bounded-wait timeouts, bad pages, bad tokens).
 * Returns TB_OK, TB_ERR_DEVICE_TIMEOUT or TB_ERR_STATE; clears the word. */
tb_status tb_context_check_device(tb_context *ctx);
/* Failure-detection probe (no reference counterpart; the reference has no
 * device-side waits): runs one kernel whose bounded wait nothing satisfies --
 * which 0: an mbarrier wait with no arrival, 1: a spin on a tagged word that
 * nothing writes (the tensor-parallel pull's wait) -- so it runs out after the
 * library's 2 s limit and records the timeout in the context's error word.
 * The next tb_context_check_device returns TB_ERR_DEVICE_TIMEOUT, and the
 * context stays usable. */
tb_status tb_debug_expire_wait(tb_context *ctx, int32_t which);

/* ---------------------------------------------------------- quantizers -- */
/* QuantizedTensor.swift:379-424 quantizePerChannel: W[K][N] fp32 ->
 * Q[K][N] int8 + scales[N].  Bit-exact with the reference's formula. */
tb_status tb_quantize_int8_per_channel(tb_context *ctx, const float *w_host, int64_t K, int64_t N,
                                       int8_t *q_host, float *scales_host);
/* QuantizedTensor.swift:502-560 quantizeINT4: flat groups of group_size,
 * packed ceil(count/2) bytes (even index -> high nibble), scales and zero
 * points ceil(count/group_size). */
tb_status tb_quantize_int4_group(tb_context *ctx, const float *x_host, int64_t count, int64_t group_size,
                                 uint8_t *packed_host, float *scales_host, int8_t *zero_points_host);
/* Device-pointer variants (enqueued on the context stream). */
tb_status tb_quantize_int8_per_channel_dev(tb_context *ctx, const float *w_dev, int64_t K, int64_t N,
                                           int8_t *q_dev, float *scales_dev);
tb_status tb_quantize_int4_group_dev(tb_context *ctx, const float *x_dev, int64_t count, int64_t group_size,
                                     uint8_t *packed_dev, float *scales_dev, int8_t *zero_points_dev);

/* ------------------------------------------------------ quantized GEMV -- */
typedef enum { TB_PREC_INT8 = 8, TB_PREC_INT4 = 4 } tb_precision;

/* A QuantizedTensor (QuantizedTensor.swift:62-165) in host memory.
 * INT8 per-channel: data = K*N int8, scales = N floats.
 * INT4 per-group:   data = ceil(K*N/2) bytes, scales = ceil(K*N/group_size).
 * zero_points may be NULL; when present they must be all zero (the
 * reference's quantizers always write 0). */
typedef struct {
    int32_t precision; /* tb_precision */
    int64_t in_features;  /* K = shape[0] */
    int64_t out_features; /* N = shape[1] */
    int64_t group_size;   /* INT4 only (reference default 32) */
    const void *data;
    int64_t data_bytes;
    const float *scales;
    int64_t num_scales;
    const int8_t *zero_points;
    int64_t num_zero_points;
} tb_qtensor_desc;

/* QuantizedTensor.dequantize (QuantizedTensor.swift:182-285) on the device:
 * out_host[K*N] = (q - zero_point) * scale, per-channel INT8 or INT4 groups
 * (zero points honoured when given). */
tb_status tb_dequantize(tb_context *ctx, const tb_qtensor_desc *desc, float *out_host);
/* PerplexityHarness.convertToINT4 (PerplexityHarness.swift:65-126) for one
 * linear weight: dequantize, then tb_quantize_int4_group's quantizer with
 * group_size, on the device; outputs as tb_quantize_int4_group. */
tb_status tb_requantize_int4(tb_context *ctx, const tb_qtensor_desc *desc, int64_t group_size, uint8_t *packed_host,
                             float *scales_host, int8_t *zero_points_host);

/* Upload a quantized weight to HBM once (replaces MetalBackend's
 * cachedQuantizedBuffers / cachedINT4Buffers, MetalBackend.swift:1282-1359). */
tb_status tb_qweight_upload(tb_context *ctx, const tb_qtensor_desc *desc, tb_qweight **out);
tb_status tb_qweight_free(tb_qweight *w);
/* QuantizedMatMulBackend.matmulQuantized (Backend.swift:173-175,
 * MetalBackend.swift:894-1048): y[M][N] = x[M][K] * dequant(W), fp32, M <= 64.
 * Synchronous, host buffers. */
tb_status tb_matmul_quantized(tb_context *ctx, const float *x_host, int64_t M, const tb_qweight *w,
                              float *y_host);
/* Same on device buffers, enqueued on the context stream (no sync). */
tb_status tb_matmul_quantized_dev(tb_context *ctx, const float *x_dev, int64_t M, const tb_qweight *w,
                                  float *y_dev);

/* A timed stream of GEMVs y = x W_i (i = 0..n-1, shared K, device x [M][K] and
 * y [M][max N]): one CUDA graph launches each weight once, replayed `reps`
 * times after one warm-up replay; *ms_out = milliseconds per replay.  pdl = 0:
 * plain stream order; 1: programmatic dependent launch, each GEMV waits for
 * the previous one to finish before reading x (a dependent chain, as inside a
 * decode step); 2: the GEMVs are treated as independent (no wait), so their
 * executions overlap the way independent projections can, and each runs with
 * whole rows per CTA (no K split: the throughput choice when launches overlap).
 * Measurement helper for the single-GEMV HBM benchmark (
 * cycle through more weight copies than fit in L2). */
tb_status tb_qgemv_stream_time(tb_context *ctx, const tb_qweight *const *ws, int32_t n, const float *x_dev,
                               int64_t M, float *y_dev, int32_t reps, int32_t pdl, float *ms_out);

/* -------------------------------------------------- decode attention -- */
/* AttentionBackend.attention (Backend.swift:205-219) for one query token over
 * a contiguous cache, with the semantics of the live CPU path
 * (ModelRunner.swift:519-579).  q[H*d], keys/values[L][Hkv*d], out[H*d].
 * The library pages the cache into HBM internally.  Synchronous, host buffers. */
tb_status tb_attention_decode(tb_context *ctx, const float *q_host, const float *keys_host,
                              const float *values_host, int64_t L, int32_t num_heads, int32_t num_kv_heads,
                              int32_t head_dim, float *out_host);
/* Paged decode attention on device buffers (the runner's layout):
 *   kv_pool_dev  [pages][num_layers][2 (K,V)][Hkv][16 tokens][d] fp32
 *   page_table_dev [batch][ptab_stride] int32 (logical page -> pool page, -1 = evicted)
 *   seq_lens_dev [batch] int32 context lengths, q_dev [batch][H*d], out_dev [batch][H*d].
 * The splits of a (sequence, KV head) combine inside their thread-block
 * cluster through distributed shared memory: no scratch memory is used. */
tb_status tb_paged_attention_dev(tb_context *ctx, const float *q_dev, int32_t batch, const float *kv_pool_dev,
                                 const int32_t *page_table_dev, int32_t ptab_stride, const int32_t *seq_lens_dev,
                                 int32_t max_len, int32_t layer, int32_t num_layers, int32_t num_heads,
                                 int32_t num_kv_heads, int32_t head_dim, float *out_dev);

/* No counterpart in the reference (its attention runs on the host).  Same
 * computation and arguments as tb_paged_attention_dev, for callers that cannot
 * allocate device memory -- a host that has given all HBM to its own pool, or
 * a latency-critical path where cudaMalloc/cudaFree would synchronise the
 * device.  It allocates nothing: the splits of each (sequence, KV head) are
 * combined inside their thread-block cluster, with no scratch memory, so any
 * batch size is accepted.  Runs on `stream` (a cudaStream_t, NULL = default
 * stream) of the current device.  The first call on a device reads its SM
 * count and the address of the error word below, and should come before any
 * stream capture.  A bounded device-side wait that runs out is recorded in one
 * error word per device (a file-scope __device__ variable shared by every call
 * on that device, including calls that overlap); read it with
 * tb_paged_attention_noalloc_status. */
tb_status tb_paged_attention_dev_noalloc(void *stream, const float *q_dev, int32_t batch, const float *kv_pool_dev,
                                         const int32_t *page_table_dev, int32_t ptab_stride,
                                         const int32_t *seq_lens_dev, int32_t max_len, int32_t layer,
                                         int32_t num_layers, int32_t num_heads, int32_t num_kv_heads,
                                         int32_t head_dim, float *out_dev);
/* Status of the allocation-free attention calls on the current device: waits
 * for `stream`, reads the shared error word (and zeroes it if `clear`), and
 * returns TB_OK, or TB_ERR_DEVICE_TIMEOUT if a bounded wait ran out since the
 * word was last cleared.  Allocates nothing. */
tb_status tb_paged_attention_noalloc_status(void *stream, int32_t clear);

/* ---------------------------------------------------------------- model -- */
typedef enum { TB_ARCH_LLAMA = 0, TB_ARCH_TOY = 1 } tb_architecture;
typedef enum {
    TB_PROJ_Q = 0, TB_PROJ_K = 1, TB_PROJ_V = 2, TB_PROJ_O = 3,
    TB_PROJ_GATE = 4, TB_PROJ_UP = 5, TB_PROJ_DOWN = 6
} tb_projection;

/* ModelConfig (ModelRunner.swift:27-121). architecture: LLaMA (RMSNorm,
 * SwiGLU, no biases) or the reference's toy model (ModelWeights.swift:171-244:
 * biases, GELU FFN, no norms). */
typedef struct {
    int32_t num_layers, hidden_dim, num_heads, num_kv_heads, vocab_size, max_seq_len, intermediate_dim;
    int32_t architecture;
    float rms_eps; /* 1e-5 in the reference (Tensor.swift:1512) */
} tb_model_config;

/* ModelWeights (ModelWeights.swift:137-168), uploaded to HBM and fused
 * (QKV concatenated, gate/up interleaved) at tb_model_finalize. */
tb_status tb_model_create(tb_context *ctx, const tb_model_config *cfg, tb_model **out);
tb_status tb_model_free(tb_model *m);
/* Tensor parallelism (new; the reference runs on one device).  Rank 0 draws
 * a 128-byte NCCL unique id, every rank receives it out of band and joins
 * the communicator on its context; the model is then told its shard before
 * any projection is set.  Projections are passed pre-sliced: q, k, v and
 * gate, up as column shards [hidden, out/world] (this rank's heads / rows),
 * o_proj and down_proj as row shards [in/world, hidden].  The step adds an
 * in-place fp32 all-reduce of the residual stream after o_proj and
 * down_proj; the LM head is replicated. */
tb_status tb_tp_unique_id(uint8_t *id /* [128] */);
tb_status tb_context_init_tp(tb_context *ctx, const uint8_t *id /* [128] */, int32_t rank, int32_t world);
tb_status tb_model_set_tensor_parallel(tb_model *m, int32_t rank, int32_t world);
/* Tensor parallel through peer memory (replaces the NCCL all-reduce of a
 * runner; LLaMA models, batch <= 16).  Every rank exports its all-reduce
 * buffer as a 64-byte CUDA IPC handle, the handles are shared out of band, and
 * each rank maps the others' buffers.  The row-parallel o_proj / down_proj
 * epilogues then write their partial rows into every rank's buffer over
 * NVLink as 64-bit (value, step tag) words; the next launch that reads the
 * residual stream spins (bounded, 2 s) until the words carry this step's tag
 * and adds the ranks' partials in rank order, so all ranks hold identical
 * bits.  No fences, counters or separate all-reduce launches. */
tb_status tb_runner_tp_handle(tb_runner *r, uint8_t *handle /* [64] */);
tb_status tb_runner_tp_connect(tb_runner *r, const uint8_t *handles /* [world][64], rank order */);
tb_status tb_model_set_embedding(tb_model *m, const float *emb_host /* [vocab][hidden] */);
tb_status tb_model_set_final_norm(tb_model *m, const float *w_host /* [hidden] */);
tb_status tb_model_set_layer_norms(tb_model *m, int32_t layer, const float *input_norm_host,
                                   const float *post_attention_norm_host);
tb_status tb_model_set_projection(tb_model *m, int32_t layer, int32_t which, const tb_qtensor_desc *w,
                                  const float *bias_host /* [N] or NULL */);
tb_status tb_model_set_output(tb_model *m, const tb_qtensor_desc *w, const float *bias_host);
tb_status tb_model_finalize(tb_model *m);
/* Bytes of weights streamed per decode step (for roofline accounting). */
tb_status tb_model_weight_bytes(const tb_model *m, int64_t *bytes);

/* --------------------------------------------------------------- runner -- */
/* ModelRunner (ModelRunner.swift:127-298) with a KVCache whose pages live in
 * HBM (KVCache.swift:108-356, PageAllocator.swift:35-152).  max_batch
 * independent sequences decode together (batch 1 = the reference).
 * max_positions bounds the RoPE table (>= max_seq_len). */
tb_status tb_runner_create(tb_model *m, int32_t max_batch, int32_t max_positions, tb_runner **out);
tb_status tb_runner_free(tb_runner *r);
/* ModelRunner.reset (ModelRunner.swift:213-217). */
tb_status tb_runner_reset(tb_runner *r);
/* ModelRunner.step(tokenId:) (ModelRunner.swift:168-208) for sequence 0 of a
 * batch-1 runner: logits_host [vocab] may be NULL; argmax_out receives the
 * greedy token (Sampler.greedy, Sampler.swift:126-138). */
tb_status tb_runner_step(tb_runner *r, int32_t token, float *logits_host, int32_t *argmax_out);
/* ModelRunner.step with the InferenceObserver hooks (InferenceObserver.swift:
 * 40-84): as tb_runner_step, plus (any may be NULL) layer_norms[num_layers] =
 * ||h||_2 at each layer's entry (didEnterLayer), attn_weights[num_layers][stride]
 * = each layer's softmax weights, num_heads x L flattened head-major with L =
 * position + 1 (didComputeAttention), final_hidden[hidden_dim] = the normalised
 * hidden state before the LM head (didComputeFinalHiddenState).  Logits are
 * didComputeLogits.  Batch-1 runners; the step runs launch by launch (no graph). */
tb_status tb_runner_step_observed(tb_runner *r, int32_t token, float *logits, int32_t *argmax_out,
                                  float *layer_norms, float *attn_weights, int64_t attn_stride,
                                  float *final_hidden);
tb_status tb_runner_position(const tb_runner *r, int32_t seq, int64_t *pos);
/* KVCache.length (KVCache.swift:138-143) and pageAllocationStatus (:352-356). */
tb_status tb_runner_kv_length(const tb_runner *r, int32_t seq, int64_t *length);
tb_status tb_runner_page_status(const tb_runner *r, int32_t seq, uint8_t *status, int64_t n);
tb_status tb_runner_max_pages(const tb_runner *r, int64_t *n);

/* Execution mode of a runner's decode step.  Default (enable = 0): one fused
 * kernel per projection and attention, the step captured as one CUDA graph.
 * enable = 1 (batch-1 INT8 LLaMA runners): the persistent single-kernel step
 * (one cooperative launch per token streams every layer's weights through a
 * shared-memory ring); measured slower than the per-projection chain, kept as
 * an option. */
tb_status tb_runner_set_persistent(tb_runner *r, int32_t enable);
tb_status tb_runner_get_persistent(const tb_runner *r, int32_t *enabled);
/* Prompt prefill of tb_runner_generate (default on): up to 64 prompt tokens
 * (of one or several sequences) per pass of the layers, each token a row with
 * its own position, so the weights stream once per chunk; the logits of prompt
 * steps are not computed (the reference discards them).  Off, or for prompts
 * that would evict KV pages, or under tensor parallelism,
 * prompts are stepped one token at a time as ModelRunner.swift:240-244 does. */
tb_status tb_runner_set_chunked_prefill(tb_runner *r, int32_t enable);
/* Copy an internal fp32 buffer of the runner to the host (diagnostics):
 * 0 h_in, 1 h_mid (persistent step), 2-5 split-K partials (qkv, o, gate/up,
 * down), 6 attention split partials, 7 logits, 8 residual stream, 9 q,
 * 10 attention context, 11 SiLU*up activations (per-op step). */
tb_status tb_runner_debug_read(tb_runner *r, int32_t which, float *out_host, int64_t n);

/* Diagnostics: run one persistent step recording, per CTA and phase,
 * out[(cta * phases + phase) * 8 + i]: %globaltimer (ns) at the phase start
 * (i = 0), its end (1) and the end of its prologue (2); ns spent waiting for
 * weight tiles (3) and in unit products (4), as seen by consumer thread 0. */
tb_status tb_runner_trace_step(tb_runner *r, uint64_t *out, int64_t n, int32_t *ctas, int32_t *phases);

/* Called once per generated token (TokenOutput, GenerationConfig.swift:149-219);
 * return nonzero to stop that sequence. */
typedef int32_t (*tb_token_callback)(void *user, int32_t seq, int32_t index, int32_t token_id);

/* ModelRunner.generateStream (ModelRunner.swift:227-298) with greedy sampling
 * (SamplerConfig(topK: 1) / Sampler.greedy) for a batch of independent
 * sequences.  prompts: concatenated token ids, prompt_offsets[n_seqs+1].
 * Each prompt is clamped to [0, vocab), all but its last token are prefilled
 * with step(), then max_new_tokens greedy steps follow; a sequence stops after
 * yielding one of stop_tokens.  out_tokens [n_seqs][max_new_tokens],
 * out_counts [n_seqs].  The whole decode loop runs on the device (one CUDA
 * graph per step); the host only reads the tokens back. */
tb_status tb_runner_generate(tb_runner *r, const int32_t *prompts, const int64_t *prompt_offsets, int32_t n_seqs,
                             int32_t max_new_tokens, const int32_t *stop_tokens, int32_t n_stop,
                             int32_t *out_tokens, int32_t *out_counts, tb_token_callback cb, void *user);

/* Sampler of tb_runner_generate (SamplerConfig, Sampler.swift:46-104;
 * Sampler.sampleDetailed, Sampler.swift:401-473).  NULL restores greedy
 * argmax decoding (the LM-head epilogue).  Otherwise every generated token is
 * drawn on the device after the LM head: repetition penalty over prompt +
 * generated tokens, top_k (> 0) else top_p (has_top_p), temperature (below
 * 0.01: unscaled), softmax, then the reference's LCG (seeded with `seed`
 * at the start of every generate call, each sequence alike; has_seed = 0
 * draws a seed from the host).  The persistent step is off while a sampler
 * is set; tb_runner_step then returns the drawn token as its argmax_out. */
typedef struct tb_sampler_config {
    float temperature;
    int32_t top_k;
    int32_t has_top_p;
    float top_p;
    float repetition_penalty;
    int32_t has_seed;
    uint64_t seed;
} tb_sampler_config;
tb_status tb_runner_set_sampler(tb_runner *r, const tb_sampler_config *cfg);
/* Sampler.sampleDetailed (Sampler.swift:401-473) on one host logits row:
 * the device sampler with `history` as the penalty history; *rng_state is the
 * LCG state, advanced by the draw (cfg->seed is not read). */
tb_status tb_sample_detailed(tb_context *ctx, const float *logits, int32_t vocab_size, const tb_sampler_config *cfg,
                             const int32_t *history, int32_t n_history, uint64_t *rng_state, int32_t *token,
                             float *prob, float *entropy);
/* Per generated token of the last tb_runner_generate with a sampler: the
 * probability of the drawn token and the entropy (nats) of the distribution
 * it was drawn from (TokenOutput.probability / .entropy), [n_seqs][max_new]. */
tb_status tb_runner_token_stats(tb_runner *r, int32_t n_seqs, int32_t max_new_tokens, float *prob, float *entropy);
/* Penalty history (prompt + generated tokens, at most position + 1 of them)
 * for the sampled draws of the following tb_runner_step / _observed calls,
 * and the probability / entropy of the last such draw. */
tb_status tb_runner_set_step_history(tb_runner *r, const int32_t *tokens, int32_t n);
tb_status tb_runner_step_stats(tb_runner *r, float *prob, float *entropy);

/* PerplexityHarness.computePerplexity (PerplexityHarness.swift:141-193) for
 * n_seqs token slices (tokens[offsets[s] .. offsets[s+1]), each >= 2 ids in
 * [0, vocab)): teacher-forced over each slice on the device, log
 * P(tokens[i+1] | tokens[..i]) in fp64 (fp32 max, fp64 log-sum-exp), summed
 * per slice in position order.  With chunked prefill on (the default) and no
 * slice long enough to evict KV pages, up to 64 positions are scored per pass
 * of the layers; otherwise one step per position.  sum_logprob[s] and
 * n_predictions[s] = length - 1; perplexity = exp(-sum / n).  No sampler may
 * be set; the runner's sequences start fresh. */
tb_status tb_runner_perplexity(tb_runner *r, const int32_t *tokens, const int64_t *offsets, int32_t n_seqs,
                               double *sum_logprob, int64_t *n_predictions);

/* Timing hooks for benchmarks: run n decode steps from the current state
 * entirely on the device (inputs already resident), returning the elapsed
 * milliseconds measured with CUDA events on the runner's stream. */
tb_status tb_runner_prefill_device(tb_runner *r, const int32_t *prompts, const int64_t *prompt_offsets,
                                   int32_t n_seqs, int32_t max_new_tokens);
tb_status tb_runner_decode_device(tb_runner *r, int32_t n_steps, float *elapsed_ms);
tb_status tb_runner_read_tokens(tb_runner *r, int32_t *out_tokens, int32_t *out_counts);
/* Host<->device bytes moved by the generate / step entry points since the
 * last reset (prompt upload, page-table updates, state pushes, token reads). */
tb_status tb_runner_io_bytes(tb_runner *r, int64_t *h2d_bytes, int64_t *d2h_bytes, int32_t reset);
/* Per-kernel timing of one step (CUDA events around each launch, no graph):
 * times_ms[n] receives the kernel durations, kinds[n] 0 = GEMV, 1 = attention;
 * *n in: capacity, out: count. */
tb_status tb_runner_profile_step(tb_runner *r, float *times_ms, int32_t *kinds, int64_t *bytes, int32_t *n);
/* Device timeline of one graph-replayed decode step: stamps[n][16] per launch:
 * globaltimer nanoseconds [0..7] (first CTA entry, last CTA entry, last
 * dependency release, last prologue done, last accumulator complete, last
 * partial-sum exchange, last exit, last first-weight arrival) and, for INT4
 * GEMVs, [8..15] SM-cycle sums of CTA 0's unit pipeline (stage waits, slot
 * waits, nibble expansion, tensor-memory store, issue waits for A and B, B
 * digit writes, units); 0 where a point does not apply.  kinds[n] as in
 * tb_runner_profile_step. */
tb_status tb_runner_trace_launches(tb_runner *r, uint64_t *stamps, int32_t *kinds, int32_t *n);

#ifdef __cplusplus
}
#endif
#endif /* TINYBRAIN_CUDA_H */
