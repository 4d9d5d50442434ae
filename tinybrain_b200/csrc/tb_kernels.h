// tb_kernels.h -- internal kernel parameter blocks and launchers shared by the
// host runtime (tb_runtime.cu) and the kernel translation units.  Not part of
// the public C ABI (include/tinybrain_cuda.h).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace tb {

// Device error codes written into the context's error word (first writer wins).
enum DeviceError : int {
    kDevOk = 0,
    kDevWaitTimeout = 1,      // an mbarrier wait exceeded its time limit
    kDevBadPage = 2,          // KV append found no page mapped for a position
    kDevBadToken = 3,         // token id outside [0, vocab)
    kDevBadSmem = 4,          // a shared-memory buffer is not aligned as its layout requires
};

// ----------------------------------------------------------------------------
// Device weight layouts produced by the repack kernels ("GPU layout").
//
// The reference stores a quantized projection row-major as [K in][N out]
// (y = x * W).  The GPU layouts are output-row major and cut into "units" that
// are streamed with 1-D bulk copies; the units of a row block are consecutive
// (row-block major, k minor).
//
// INT8 (tensor-core path, tb_tc.cuh): row blocks ("tiles") of 128 rows, units
// of 128 k = 16 KB, values stored as signed int8, each unit in the canonical
// K-major no-swizzle operand layout of tcgen05.mma ([16 row groups][8 k-chunks
// of 16 bytes][8 rows][16 bytes]).  K is padded to a multiple of 128 and N to
// a multiple of 128 with zero weights.  The fused gate/up matrix puts 64 gate
// rows and the matching 64 up rows in each tile.
//
// INT4 (tensor-core path, tb_tc.cuh): the same 128-row tiles and 128-k units,
// 10 KB each: 8 KB of biased nibbles [4 k-chunks of 32][128 rows][16 bytes]
// (word j of a chunk: byte i = k 8j+i low, k 8j+i+4 high), then the unit's
// group scales [4 row groups of 32][128 k] fp32.  The scale buffer holds the
// largest |scale| per (32-row group, unit).
// ----------------------------------------------------------------------------
constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;  // + 1 producer warp
constexpr int kMaxGemvBatch = 64;  // batch rows of one GEMV launch (grid y splits rows beyond a CTA's)

struct QLayout {
    int precision;       // 8 or 4
    int K;               // logical reduction length
    int Kp;              // K padded to a multiple of 128
    int N;               // logical output rows
    int Np;              // N padded to a multiple of RB
    int RB;              // rows per row block (128)
    int slabs;           // units along K per row block
    int slab_k;          // k values per unit (128)
    int slab_bytes;      // bytes per row of a unit (INT8 128, INT4 64)
    int row_bytes;       // bytes per row (Kp or Kp/2)
    int fused_gu;        // 1: gate/up interleaved by half row blocks
    size_t weight_bytes; // INT8: Np * row_bytes; INT4: tiles * slabs * 10 KB (scales inline)
    size_t scale_floats; // INT8: Np row scales; INT4: (Np/32) * slabs maxima
};

// GPU row of logical row n of a matrix placed at (row_offset, interleave) in a
// fused layout (interleave 1: gate half of each row block, 2: up half).
__host__ __device__ inline int fused_row(const QLayout& L, int n, int row_offset, int interleave) {
    if (interleave == 0) return row_offset + n;
    const int half = L.RB / 2;
    return (n / half) * L.RB + (interleave == 2 ? half : 0) + n % half;
}

// RB = 64 requests the fused gate/up arrangement (INT8 tiles stay 128 rows).
QLayout make_qlayout(int precision, int K, int N, int RB);

// Prologue: how the CTA builds its activation slice x[m][k].
enum GemvPrologue : int {
    kProNone = 0,      // x = src[m][k]
    kProRmsNorm = 1,   // x = src[m][k] * inv_rms(src[m]) * norm_w[k]
    kProEmbed = 2,     // src row = embedding[token[m]]; CTA 0 copies it into resid
    kProEmbedRms = 3,  // embed, then RMSNorm
};

// Epilogue: what happens with the finished dot products.
enum GemvEpilogue : int {
    kEpiStore = 0,     // out[m][n] = v
    kEpiResidual = 1,  // out[m][n] += v
    kEpiQkv = 2,       // q with RoPE -> q_out; k with RoPE, v -> KV cache page
    kEpiSiluMul = 3,   // RB 64: out[m][n] = silu(gate) * up
    kEpiGelu = 4,      // out[m][n] = gelu(v)
    kEpiArgmax = 5,    // logits (optional) + per-sequence argmax + step bookkeeping
    kEpiPush = 6,      // tensor parallel: the partial rows go to every rank's all-reduce slot
};

// Per-sequence decode state living in device memory.
struct SeqState {
    int pos;            // position of the token processed by the current step
    int token;          // token fed to the current step
    int n_prompt;       // prompt length (prompt tokens are taken from prompt[])
    int n_out;          // tokens generated so far
    int max_out;        // capacity of out_tokens
    int active;         // 0 = finished / padding slot
    unsigned long long best;  // packed argmax key of the current step
};

// Optional device timeline of one launch (globaltimer ns; nullptr = off):
// [0] first CTA entry (min), [1] last CTA entry, [2] last dependency release,
// [3] last prologue done, [4] last accumulator complete, [5] last partial-sum
// exchange done, [6] last CTA exit, [7] last first-weight-unit arrival;
// [8..15] INT4 pipeline of CTA 0, SM cycles summed over its units: [8] stage
// waits, [9] slot waits, [10] nibble expansion, [11] tensor-memory store, [12]
// issue waits for A, [13] for B, [14] B digit writes, [15] units.
constexpr int kTracePoints = 16;

struct GemvParams {
    unsigned long long* trace;
    int independent;  // 1: reads nothing the preceding launch writes (skip the dependency wait)
    // weights (GPU layout)
    const uint8_t* w;
    const float* scales;
    const float* bias;        // [N] or null
    QLayout L;
    int P;                    // cluster size = K split factor
    int M;                    // batch rows
    // prologue
    int prologue;
    const float* src;         // [M][ld_src]
    int ld_src;
    const float* norm_w;      // [K]
    float eps;
    const float* embedding;   // [V][K]
    float* resid;             // embed prologue: copy of the embedding row
    const SeqState* seq_ro;   // token / pos source
    // epilogue
    int epilogue;
    float* out;               // [M][ld_out]
    int ld_out;
    // QKV epilogue
    int H, Hkv, head_dim, kv_dim;
    const float2* rope;       // [max_pos][head_dim/2] (cos, sin)
    int rope_max_pos;
    float* kv_pool;           // [page][layer][2][Hkv][16][d]
    const int* page_table;    // [M][ptab_stride]
    int ptab_stride;
    int layer, num_layers;
    // argmax epilogue
    SeqState* seq;            // [M]
    float* logits;            // [M][N] or null
    unsigned int* ticket;     // completion counter for step bookkeeping
    int* out_tokens;          // [M][max_out]
    const int* prompt;        // [M][prompt_stride]
    int prompt_stride;
    int vocab;
    int* err;                 // device error word
    // Tensor-parallel all-reduce through peer memory (ar_world > 1).  Buffer of
    // every rank: tagged words [slot][rank][ar_slot_words], each a 64-bit
    // (fp32 value, u32 step + 1) pair written with one store, so a reader
    // knows a value has arrived without fences or counters.  A pushing launch
    // writes its output rows into every rank's [slot][own rank] region; a
    // pulling launch reads its source as ar_hin + the ranks' partials (rank
    // order), spinning (bounded) on words whose tag is not yet this step's,
    // and its CTA (0, 0) stores that sum to ar_hout.
    int ar_world, ar_rank;
    int ar_push_slot, ar_pull_slot;  // -1: none
    unsigned long long* const* ar_peers;  // [world] buffer bases (own included)
    const unsigned long long* ar_local;   // own buffer base
    long long ar_slot_words;              // words per (slot, rank): M * H
    unsigned int* ar_step;                // step counter (the LM head's last CTA advances it)
    const float* ar_hin;
    float* ar_hout;
    // Batches over 16 rows (the "wide" INT8 path): when bimg is set, a
    // preceding wide_digits launch has written the digit operand of every unit
    // (bimg, wide_digits_bytes) and the rows' digit exponents (rowex_g [M]);
    // the GEMV then streams B beside A instead of building it per CTA.
    uint8_t* bimg;
    int* rowex_g;
};

// Launch the GEMV described by p on `stream` (PDL + cluster attributes).
cudaError_t launch_gemv(const GemvParams& p, cudaStream_t stream, bool pdl);
// The digit operand of a wide INT8 GEMV (the GEMV's prologue: embedding
// gather / RMSNorm, one exponent per row over the whole K), written once per
// launch for all of its CTAs; p is the GEMV's own parameter block.
cudaError_t launch_wide_digits(const GemvParams& p, cudaStream_t stream, bool pdl);
size_t wide_digits_bytes(const QLayout& L);  // bimg bytes for a layout
bool gemv_uses_wide(int precision, int M);
// Pick the K-split (cluster size) for a layout and batch.
int choose_ksplit(const QLayout& L, int M, int num_sms);
// The split for GEMVs whose launches overlap (independent of each other).
int choose_ksplit_stream(const QLayout& L, int M);
// CTAs of the launch launch_gemv(p) makes.
int gemv_grid_ctas(const GemvParams& p);

// Repack reference-layout quantized weights (device copies of the host
// arrays) into the GPU layout.  row_offset places the matrix at rows
// [row_offset, row_offset + N) of a fused destination; for the fused gate/up
// block, `interleave` = 1 puts this matrix in rows [0,32) of each 64-row block
// and 2 in rows [32,64).
struct RepackSrc {
    int precision;
    int K, N;
    int group_size;
    const void* data;          // INT8: [K][N] int8 ; INT4: packed nibbles of flat [K][N]
    const float* scales;       // INT8: [N] ; INT4: [K*N/gs]
    const int8_t* zero_points; // may be null; must be all zero for the fast path
};
cudaError_t launch_repack(const RepackSrc& s, const QLayout& L, uint8_t* w_out, float* scales_out,
                          int row_offset, int interleave, cudaStream_t stream);

// Device quantizers (bit-exact restatements of the reference quantizers).
cudaError_t launch_quantize_int8_per_channel(const float* W, int64_t K, int64_t N, int8_t* Q, float* scales,
                                             cudaStream_t stream);
// QuantizedTensor.dequantize on the device: prec 8 per-channel [K][N] (scales
// per column), prec 4 flat groups of gs; zps may be nullptr.
cudaError_t launch_dequantize(int prec, const uint8_t* data, const float* scales, const int8_t* zps, int64_t K,
                              int64_t N, int64_t gs, float* out, cudaStream_t stream);
cudaError_t launch_quantize_int4_group(const float* x, int64_t count, int64_t gs, uint8_t* packed,
                                       float* scales, int8_t* zp, cudaStream_t stream);

// ----------------------------------------------------------------------------
// Paged decode attention.
// ----------------------------------------------------------------------------
constexpr int kPageTokens = 16;

struct AttnParams {
    unsigned long long* trace;  // see GemvParams::trace ([0], [1], [2], [6])
    const float* q;           // [M][H*d] (post-RoPE)
    int ld_q;
    const float* kv_pool;     // [page][layer][2][Hkv][16][d]
    const int* page_table;    // [M][ptab_stride], -1 = evicted (reads as zeros)
    int ptab_stride;
    const SeqState* seq;      // L = seq.pos + 1 (if lens == null)
    const int* lens;          // optional explicit lengths [M]
    int layer, num_layers;
    int H, Hkv, d;
    int M;
    int nsplit;
    float* out;               // [M][H*d]
    int ld_out;
    int* err;
    // 0: only the last page may be written by the preceding kernel (decode:
    // earlier pages are fetched before the dependency wait); 1: any page may
    // be (chunked prefill appends a whole chunk of positions), wait first
    int wait_first;
    // Persistent chunked variant (G = 8, d = 64, set by the runner): work is
    // cut into chunks of chunk_pages pages per (sequence, KV head), spread
    // over a fixed grid; chunk partials [M * Hkv][maxch][kAttnPartFloats] go
    // to `part` and the last chunk of a (sequence, KV head) to finish (ticket
    // [M * Hkv], zero between launches) combines them.  nullptr: cluster kernel.
    float* part;
    int* ticket;
    int chunk_pages;
    int maxch;
    int probe;  // diagnostics (TB_ATTN_PROBE): consumers only release the pages
    // floats in kv_pool (the persistent variant loads its tiles through a
    // tensor map over the pool, which needs the extent)
    long long kv_floats;
};
constexpr int kAttnPartFloats = 8 * 64 + 16;  // acc [8 heads][64], m [8], l [8]
// Grid of the persistent chunked attention launch and its chunk size.
int attn_flat_grid(int num_sms);
int attn_flat_chunk_pages(int M, int Hkv, int max_pages, int num_sms);
bool attn_flat_supported(int H, int Hkv, int d, int M);
cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl);
constexpr int kMaxAttnSplits = 16;  // the splits of a (sequence, KV head) form one cluster
// balance: also split long contexts to at most ~64 pages per split
int choose_nsplit(int M, int Hkv, int max_pages, int num_sms, bool balance = true);

// ----------------------------------------------------------------------------
// Persistent decode step (batch 1): one cooperative launch per token runs all
// layers and the LM head.  See tb_step.cu.
// ----------------------------------------------------------------------------
struct StepLayer {
    const uint8_t *qkv_w, *o_w, *gu_w, *dn_w;
    const float *qkv_s, *o_s, *gu_s, *dn_s;
    const float *qkv_b, *o_b, *gu_b, *dn_b;  // GPU-row-space biases or null
    const float *in_norm, *post_norm;        // null = no norm
};

struct StepParams {
    const StepLayer* layers;  // [num_layers], device memory
    int num_layers;
    QLayout Lqkv, Lo, Lgu, Ldn, Llm;  // identical for every layer
    const uint8_t* lm_w;
    const float *lm_s, *lm_b, *final_norm;
    const float* emb;
    int H, nheads, Hkv, d, kvd, I, V;
    float eps;
    const float2* rope;
    int rope_max_pos;
    float* kv_pool;
    const int* ptab;
    SeqState* seq;
    int* out_tokens;
    const int* prompt;
    int prompt_stride;
    float* logits;
    float *hX, *hY;                               // residual stream ping-pong [H]
    float *part_qkv, *part_o, *part_gu, *part_dn;  // split-K partials [slabs][Np]
    float* attn_part;                             // [Hkv][A][G][d + 4]
    int A;                                        // attention splits per KV head
    unsigned int* bar;                            // grid barrier counter, zero at launch
    int* err;
    int nslots, slot_bytes;
    int nflight;                // producer copies in flight at most
    unsigned long long* trace;  // optional [C][phases][8] diagnostics
    // dataflow step (tb_flow.cu): 64-bit (fp32 bits, tag) words
    int flow;                            // 1: launch the dataflow kernel
    uint64_t* f_h[2];                    // residual stream h_in, h_mid [H]
    uint64_t* f_ss[2];                   // per-CTA sums of h^2 [C]
    uint64_t *f_qkv, *f_o, *f_gu, *f_dn;  // split-K partials [units][Np]
    uint64_t* f_att;                     // attention partials [Hkv][A][G][d + 2]
    uint64_t *f_dbqkv, *f_dbgu;          // segment doorbells [row blocks][units]
    unsigned int* f_epoch;               // steps completed (tag base)
    unsigned int* f_ticket;              // LM-head completion counter, zero between steps
};

constexpr int kStepConsumerWarps = 8;
constexpr int kStepThreads = (kStepConsumerWarps + 1) * 32;

// Shared memory a launch needs (and its ring geometry), or 0 if unsupported.
size_t step_smem_bytes(const StepParams& p, int grid, int* nslots, int* slot_bytes, int max_smem);
cudaError_t launch_decode_step(const StepParams& p, int grid, size_t smem, cudaStream_t stream);
// Dataflow variant (INT8 only); 0 if unsupported.
size_t flow_smem_bytes(const StepParams& p, int grid, int* nslots, int* slot_bytes, int max_smem);
cudaError_t launch_decode_flow(const StepParams& p, int grid, size_t smem, cudaStream_t stream);
// Phases per step of a launch (diagnostic trace rows).
inline int step_phases(const StepParams& p) { return p.flow ? 7 * p.num_layers + 2 : 5 * p.num_layers + 1; }

// Device sampler (Sampler.swift:401-473, sampleDetailed) after the LM head:
// one CTA per sequence draws the next token from logits[m][V] and does the
// step bookkeeping of finish_sequence_step.
struct SampleParams {
    const float* logits;      // [M][V] LM-head output
    float* work;              // [M][V] working rows when V floats exceed shared memory, else nullptr
    int V, M;
    SeqState* seq;
    const int* prompt;        // [M][prompt_stride]: penalty history, then next prompt tokens
    int prompt_stride;
    int* out_tokens;          // [M][max_out]
    float* out_prob;          // [M][max_out] probability of the drawn token
    float* out_entropy;       // [M][max_out] entropy (nats) of the final distribution
    unsigned long long* rng;  // [M] LCG state per sequence
    float temperature, top_p, repetition_penalty;
    int top_k;                // <= 0: no top-k filter
    int has_top_p;
    unsigned int* ar_step;    // tensor parallel: step counter of the peer all-reduce (or nullptr)
    double* logprob_acc;      // [M] teacher-forced scoring: prompt steps add log P(next prompt token)
    double* logprob_out;      // [M] chunked scoring: each row's log P(target) (instead of logprob_acc)
    const int* target;        // [M] chunked scoring: each row's next token (instead of prompt)
};
// Dynamic shared memory of the sampler; *in_smem says whether the working
// row fits there (else SampleParams::work is required).
size_t sample_smem_bytes(int V, bool* in_smem);
cudaError_t launch_sample(const SampleParams& p, cudaStream_t stream, bool pdl);

// Failure-detection probe: one thread runs a bounded wait that nothing will
// satisfy -- which 0: an mbarrier wait with no arrival (mbar_wait), 1: a spin
// on a tagged word that nothing writes (wait_tagged, the tensor-parallel pull)
// -- so the wait runs out and records kDevWaitTimeout in *err.  `word` is one
// zeroed 64-bit device word.
cudaError_t launch_wait_probe(int which, const unsigned long long* word, int* err, cudaStream_t stream);

// Record the calling thread's last-error message (tb_last_error); returns status.
int report_error(int status, const char* fmt, ...);

// Softmax attention weights for the observer hook: probs[M][H][L].
cudaError_t launch_attention_probs(const AttnParams& p, float* probs, int L, cudaStream_t stream);
// Observer hooks: per-row L2 norm; RMSNorm(h) * w per row (w null: copy).
cudaError_t launch_row_norm(const float* h, int H, int ld, int M, float* out, cudaStream_t stream);
cudaError_t launch_rmsnorm_rows(const float* h, const float* w, int H, int ld, int M, float eps, float* out,
                                cudaStream_t stream);

}  // namespace tb
