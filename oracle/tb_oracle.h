/*
 * tb_oracle.h -- CPU restatement of TinyBrain's quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for
 * libtinybrain_cuda and the timed CPU baseline of bench.py.  Nothing in the
 * product (tinybrain_b200/, include/) links, loads or calls it; only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm do.
 *
 * Every function restates the Swift CPU path of vivekptnk/tinybrain and cites
 * the file:line it follows (paths relative to the reference project root).
 *
 * Parity pinning: the reference is a Swift package that imports Accelerate,
 * Combine and Metal, so it cannot be built or run on Linux.  The oracle is
 * pinned against the known-answer tests the reference's own test files hold
 * (pack/unpack pairs, odd element counts, all-zero groups, per-column scales,
 * greedy argmax cases, softmax/RMSNorm/SiLU numbers); numeric parity beyond
 * those KATs is "parity unpinned" at the Accelerate cblas_sgemm boundary.
 */
#ifndef TB_ORACLE_H
#define TB_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- quantization (Sources/TinyBrainRuntime/QuantizedTensor.swift) ---- */
void orc_quantize_int8_per_channel(const float *W, int64_t K, int64_t N,
                                   int8_t *Q, float *scales);
void orc_quantize_int4_group(const float *x, int64_t count, int64_t group_size,
                             uint8_t *packed, float *scales, int8_t *zero_points);
void orc_dequantize_int8_per_channel(const int8_t *Q, const float *scales,
                                     const int8_t *zp, int64_t K, int64_t N,
                                     float *W);
void orc_dequantize_int4_group(const uint8_t *packed, const float *scales,
                               const int8_t *zp, int64_t count,
                               int64_t group_size, float *W);

/* Quantized tensor in the reference's own host layout: shape [K (in), N (out)]
 * row-major, y = x * W.  precision 8 = INT8 per-channel (scale per column n),
 * precision 4 = INT4 per flat group of group_size elements, high nibble first. */
typedef struct {
    int32_t precision;
    int64_t K, N;
    int64_t group_size;
    const void *data;
    const float *scales;
    const int8_t *zero_points; /* may be NULL */
} orc_qtensor;

/* y[M,N] = x[M,K] * dequant(W).  mode 0: reference-faithful (dequantize the
 * whole weight to fp32, then an fp32 GEMV, QuantizedTensor.swift:640-642 +
 * Tensor.swift:839-861); mode 1: fp64 accumulation over fp32-dequantized
 * weights without materialising them ("truth" oracle for parity). */
void orc_qmatmul(const float *x, int64_t M, const orc_qtensor *w, float *y,
                 int mode);

/* ---- elementwise ops ---- */
void orc_rmsnorm(const float *x, const float *w, int64_t H, float eps, float *y);
float orc_silu(float x);
float orc_gelu(float x);
void orc_softmax(const float *x, int64_t n, float *y);   /* Tensor.softmax with +1e-7 */
void orc_rope(float *v, int64_t head_dim, int64_t num_heads, int64_t position,
              int64_t rotary_dims);
/* Single-query GQA attention over contiguous K/V [L, Hkv*d]. probs (may be NULL)
 * receives [H, L] softmax weights (ModelRunner.swift:519-579). */
void orc_attention(const float *q, const float *K, const float *V, int64_t L,
                   int64_t H, int64_t Hkv, int64_t d, float *ctx, float *probs);
int64_t orc_greedy(const float *logits, int64_t V);
/* Sampler.sampleDetailed (Sampler.swift:401-473) with sampleFromDistribution
 * (340-359) and the seeded LCG (369-381).  top_k <= 0: none; has_top_p = 0:
 * none; history: prompt + generated tokens.  *rng advances once per call.
 * Returns the token; *prob and *entropy as the reference reports them. */
typedef struct {
    float temperature;
    int32_t top_k;        /* <= 0: no top-k filter */
    int32_t has_top_p;
    float top_p;
    float repetition_penalty;
} orc_sampler;
uint64_t orc_lcg_next(uint64_t *state);
int64_t orc_sample_detailed(const float *logits, int64_t V, const orc_sampler *cfg, const int64_t *history,
                            int64_t n_history, uint64_t *rng, float *prob, float *entropy);

/* ---- model + runner (ModelRunner.swift, KVCache.swift, PageAllocator.swift) ---- */
typedef struct {
    int64_t num_layers, hidden, num_heads, num_kv_heads, vocab, max_seq_len,
        intermediate;
    int32_t arch;            /* 0 = llama (RMSNorm, SwiGLU), 1 = toy (bias, GELU, no norm) */
    float rms_eps;           /* 1e-5 in the reference */
} orc_config;

enum { ORC_Q = 0, ORC_K, ORC_V, ORC_O, ORC_GATE, ORC_UP, ORC_DOWN, ORC_NPROJ };

typedef struct orc_model orc_model;
typedef struct orc_runner orc_runner;

orc_model *orc_model_create(const orc_config *cfg);
void orc_model_free(orc_model *m);
/* All pointers are borrowed: the caller keeps the arrays alive. */
void orc_model_set_embedding(orc_model *m, const float *emb);
void orc_model_set_final_norm(orc_model *m, const float *w);
void orc_model_set_output(orc_model *m, const orc_qtensor *w, const float *bias);
void orc_model_set_layer_norms(orc_model *m, int64_t layer, const float *in_norm,
                               const float *post_norm);
void orc_model_set_proj(orc_model *m, int64_t layer, int32_t which,
                        const orc_qtensor *w, const float *bias);

/* mode as in orc_qmatmul. */
orc_runner *orc_runner_create(const orc_model *m, int32_t mode, int32_t nthreads);
void orc_runner_free(orc_runner *r);
void orc_runner_reset(orc_runner *r);
/* logits [vocab]. */
void orc_runner_step(orc_runner *r, int64_t token, float *logits);
/* InferenceObserver (InferenceObserver.swift:40-84) outputs of later steps, any
 * may be NULL: norms [num_layers] layer-entry ||h||_2; attn [num_layers][stride]
 * with each layer's [num_heads][L] softmax weights (L = position + 1);
 * final_hidden [hidden] post-norm, pre-projection. */
void orc_runner_set_observer(orc_runner *r, float *norms, float *attn, int64_t attn_stride, float *final_hidden);
int64_t orc_runner_position(const orc_runner *r);
int64_t orc_runner_kv_length(const orc_runner *r);
/* KVCache.pageAllocationStatus(layer:) -- status has max_pages entries. */
int64_t orc_runner_max_pages(const orc_runner *r);
void orc_runner_page_status(const orc_runner *r, int64_t layer, uint8_t *status);
/* Greedy generation (generateStream with topK=1 semantics reduced to argmax):
 * prompt ids are clamped, all but the last are prefilled, then max_tokens
 * steps each followed by argmax.  out_tokens[max_tokens]; out_gap (may be
 * NULL) receives the top-1 minus top-2 logit gap per generated token. */
/* ModelRunner.swift:227-298 with Sampler.sampleDetailed: tokens, probabilities
 * and entropies of max_tokens generated steps; *rng is the seeded state. */
int64_t orc_generate_sampled(orc_runner *r, const int64_t *prompt, int64_t n_prompt, int64_t max_tokens,
                             const orc_sampler *cfg, uint64_t *rng, int64_t *out_tokens, float *out_prob,
                             float *out_entropy);
float orc_perplexity(orc_runner *r, const int64_t *tokens, int64_t n, double *sum_logprob);
int64_t orc_generate_greedy(orc_runner *r, const int64_t *prompt, int64_t n_prompt,
                            int64_t max_tokens, int64_t *out_tokens, float *out_gap);

/* ---- thread control ---- */
/* n calls of orc_runner_step with the logits discarded, chunked (mode 1). */
void orc_runner_prefill(orc_runner *r, const int64_t *tokens, int64_t n);
/* Position L with L synthetic KV rows per layer (benchmark samples only). */
void orc_runner_fill_context(orc_runner *r, int64_t L, uint64_t seed);
/* SeededGenerator + Tensor.random (ModelWeights.swift:18-29, Tensor.swift:1623-1644). */
uint64_t orc_rng_seed(uint64_t seed);
void orc_rng_fill_normal(uint64_t *state, float mean, float stdv, int64_t n, float *out);
void orc_set_threads(int32_t n);
int32_t orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
