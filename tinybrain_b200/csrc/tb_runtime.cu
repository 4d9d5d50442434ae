// tb_runtime.cu -- host runtime and C ABI of libtinybrain_cuda.
//
// Maps the reference's runtime objects onto the device:
//   ModelWeights (Sources/TinyBrainRuntime/ModelWeights.swift:137-168)
//       -> tb_model: weights repacked once into HBM, QKV fused, gate/up fused;
//   ModelRunner (ModelRunner.swift:127-298)
//       -> tb_runner: one decode step = one CUDA graph of fused kernels;
//   KVCache + PageAllocator (KVCache.swift:108-356, PageAllocator.swift:35-152)
//       -> host page tables with the reference's length / eviction rules,
//          pages living in one HBM pool;
//   Sampler.greedy (Sampler.swift:126-138)
//       -> argmax fused into the LM-head GEMV epilogue.
// There is no CPU compute path: every numeric result comes from a kernel.
#include "../../include/tinybrain_cuda.h"
#include "tb_kernels.h"
#include "tb_nccl.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <random>
#include <vector>

using namespace tb;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
namespace {
thread_local std::string g_last_error;

tb_status fail(tb_status s, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}
tb_status ok() { return TB_OK; }
}  // namespace

int tb::report_error(int status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

namespace {

tb_status cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation) return fail(TB_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    return fail(TB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}
#define TB_CUDA(call)                                                     \
    do {                                                                  \
        cudaError_t e_ = (call);                                          \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);               \
    } while (0)
#define TB_CHECK(cond, ...)                                               \
    do {                                                                  \
        if (!(cond)) return fail(TB_ERR_INVALID_ARGUMENT, __VA_ARGS__);   \
    } while (0)

// RAII device buffer.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) {
        o.p = nullptr;
        o.bytes = 0;
    }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) {
            release();
            p = o.p;
            bytes = o.bytes;
            o.p = nullptr;
            o.bytes = 0;
        }
        return *this;
    }
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    cudaError_t alloc(size_t n) {
        release();
        if (n == 0) return cudaSuccess;
        cudaError_t e = cudaMalloc(&p, n);
        if (e == cudaSuccess) bytes = n;
        return e;
    }
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};

struct PinnedBuf {
    void* p = nullptr;
    size_t bytes = 0;
    ~PinnedBuf() {
        if (p) cudaFreeHost(p);
    }
    cudaError_t ensure(size_t n) {
        if (n <= bytes) return cudaSuccess;
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaMallocHost(&p, n);
        if (e == cudaSuccess) bytes = n;
        return e;
    }
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};
}  // namespace

// ---------------------------------------------------------------------------
// objects
// ---------------------------------------------------------------------------
struct tb_context {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    DevBuf err;          // int device error word
    DevBuf io_a, io_b, io_c, io_d;  // staging for host-pointer entry points
    DevBuf seq_tmp;
    // tensor parallelism: NCCL communicator over the ranks sharing a model
    void* comm = nullptr;
    int tp_rank = 0, tp_world = 1;
};

struct tb_qweight {
    tb_context* ctx = nullptr;
    QLayout L{};
    DevBuf w, s;
};

namespace {

struct ProjStage {
    bool set = false;
    int precision = 0;
    int K = 0, N = 0, gs = 0;
    DevBuf data, scales;
    std::vector<float> bias;
};

struct FusedWeight {
    QLayout L{};
    DevBuf w, s, bias;
    bool has_bias = false;
};

struct Layer {
    ProjStage stage[7];
    std::vector<float> in_norm, post_norm;
    FusedWeight qkv, o, up, down;  // up = fused gate/up (llama) or up (toy)
    DevBuf in_norm_d, post_norm_d;
};

}  // namespace

struct tb_model {
    tb_context* ctx = nullptr;
    tb_model_config cfg{};   // this rank's shard: heads, kv heads, intermediate are local counts
    tb_model_config full{};  // the whole model
    int head_dim = 0, kv_dim = 0, q_dim = 0;  // kv_dim, q_dim: local
    int tp_rank = 0, tp_world = 1;
    std::vector<Layer> layers;
    ProjStage out_stage;
    FusedWeight out;
    DevBuf emb, final_norm;
    bool has_final_norm = false;
    bool finalized = false;
    int64_t weight_bytes = 0;
};

namespace {

// Host mirror of the reference's per-sequence KVCache bookkeeping.
struct SeqKV {
    std::vector<int> map;   // logical page -> pool page, -1 = absent
    int64_t length = 0;
    int64_t pos = 0;        // ModelRunner.currentPosition
    int pages_held = 0;
};

struct Launch {
    int kind;  // 0 gemv, 1 attention, 3 all-reduce of the residual stream over the tensor-parallel ranks,
               // 5 sampler, 6 digit operand of the following wide GEMV (g = that GEMV's parameters)
    GemvParams g;
    AttnParams a;
    SampleParams s;
    int64_t bytes;  // algorithmic bytes (weights + activations) for roofline
};

}  // namespace

struct tb_runner {
    tb_model* m = nullptr;
    tb_context* ctx = nullptr;
    int B = 1;                 // batch slots
    int max_positions = 0;
    int ptab_stride = 0;
    int max_pages_per_seq = 0;
    int total_pages = 0;
    // device buffers
    DevBuf seq, ptab, kv, h, q, ctxv, act, logits, rope, prompt, out_tokens, ticket;
    // persistent chunked attention (GQA-8, d 64): chunk partials and per
    // (row, KV head) tickets, shared by the decode and prefill plans (they
    // never run at the same time; the tickets return to zero after each launch)
    DevBuf attn_part, attn_ticket;
    // tensor parallel through peer memory (tb_runner_tp_connect): the all-reduce
    // buffer shared over CUDA IPC, the peers' mappings, a second residual buffer
    DevBuf ar_buf, ar_peers_dev, ar_step, h2;
    std::vector<void*> ar_peer_host;  // [world]; own buffer at the own rank
    bool ar_on = false;
    // sequences and decode capacity of the last tb_runner_prefill_device, read
    // by decode_device / read_tokens / trace_launches / profile_step
    int last_n_seqs = 0, last_max_new = 0;
    // device sampler (tb_runner_set_sampler): LCG states, per-token statistics,
    // working rows for vocabularies beyond shared memory
    bool sampling = false, persistent_before = false;
    bool scoring = false;  // tb_runner_perplexity: the sampler launch scores prompt steps
    DevBuf lp_acc;         // [B] fp64 sum of log P(target)
    tb_sampler_config scfg{};
    DevBuf rng, out_prob, out_ent, swork;
    std::vector<int> step_hist;      // penalty history of tb_runner_step (sampled)
    float last_prob = 0.0f, last_ent = 0.0f;
    // chunked prefill: prompt tokens as the rows of a layers-only step plan
    bool pf_ready = false, pf_enabled = true;
    int pf_nsplit = 1;
    std::vector<Launch> pf_plan;
    cudaGraphExec_t pf_graph = nullptr;
    DevBuf pf_h, pf_q, pf_ctx, pf_act, pf_seq, pf_ptab;
    PinnedBuf pf_pin[2];
    cudaEvent_t pf_ev[2] = {nullptr, nullptr};
    // chunked scoring (tb_runner_perplexity): the prefill plan plus LM head and
    // the scoring launch, one log-probability per row
    std::vector<Launch> ps_plan;
    cudaGraphExec_t ps_graph = nullptr;
    DevBuf ps_logits, ps_lp, ps_target;
    // wide GEMVs (batches over 16 rows): the digit operand written once per
    // launch by a wide_digits launch, shared by the plan's launches in turn
    DevBuf wide_b, wide_ex;
    int64_t h2d_bytes = 0, d2h_bytes = 0;  // host<->device traffic of the generate paths
    int prompt_stride = 0, max_out = 0;
    // host mirror
    std::vector<SeqKV> kvh;
    std::vector<int> free_pages;  // LIFO
    std::vector<int> ptab_host;
    std::vector<cudaEvent_t> ptab_ev;  // last upload from each sequence's pinned staging row
    std::vector<char> ptab_dirty;
    PinnedBuf pin_ptab, pin_tokens, pin_seq;
    // step plan + graph
    std::vector<Launch> plan;
    cudaGraphExec_t graph = nullptr;
    int nsplit = 1;
    // persistent single-kernel step (batch 1, LLaMA): see tb_step.cu
    bool persistent = false;      // in use
    bool persistent_ok = false;   // supported for this model
    StepParams sp{};
    int step_grid = 0;
    size_t step_smem = 0;
    DevBuf step_layers, part_qkv, part_o, part_gu, part_dn, step_attn, hX, hY, step_bar, step_trace;
    DevBuf flow_buf;  // dataflow step: tagged words + epoch / ticket
    DevBuf obs_buf;   // observer outputs: attention weights, layer norms, final hidden
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    ~tb_runner() {
        for (size_t q = 0; q < ar_peer_host.size(); ++q)
            if (ar_peer_host[q] && ar_peer_host[q] != ar_buf.p) cudaIpcCloseMemHandle(ar_peer_host[q]);
        for (cudaEvent_t e : ptab_ev)
            if (e) cudaEventDestroy(e);
        if (graph) cudaGraphExecDestroy(graph);
        if (pf_graph) cudaGraphExecDestroy(pf_graph);
        if (ps_graph) cudaGraphExecDestroy(ps_graph);
        for (cudaEvent_t e : pf_ev)
            if (e) cudaEventDestroy(e);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
    }
};

// ---------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------
extern "C" int32_t tb_abi_version(void) { return TB_ABI_VERSION; }
extern "C" const char* tb_last_error(void) { return g_last_error.c_str(); }
extern "C" const char* tb_status_string(tb_status s) {
    switch (s) {
        case TB_OK: return "ok";
        case TB_ERR_INVALID_ARGUMENT: return "invalid argument";
        case TB_ERR_CUDA: return "CUDA error";
        case TB_ERR_OUT_OF_MEMORY: return "out of device memory";
        case TB_ERR_UNSUPPORTED: return "unsupported";
        case TB_ERR_PAGE_POOL_EXHAUSTED: return "KV page pool exhausted";
        case TB_ERR_FORMAT: return "format error";
        case TB_ERR_NO_DEVICE: return "no CUDA device";
        case TB_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case TB_ERR_STATE: return "invalid state";
        case TB_ERR_DEVICE_FAULT: return "device fault";
    }
    return "unknown";
}

extern "C" tb_status tb_device_count(int32_t* count) {
    TB_CHECK(count, "count is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count = 0;
        return fail(TB_ERR_NO_DEVICE, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    *count = n;
    return ok();
}

// ---- Tensor.random over SeededGenerator ----
namespace {
constexpr uint64_t kLcgA = 6364136223846793005ull;  // ModelWeights.swift:26
constexpr uint64_t kLcgC = 1ull;

// state after n steps of s -> a*s + c (mod 2^64)
uint64_t lcg_jump(uint64_t s, uint64_t n) {
    uint64_t A = 1, C = 0, a = kLcgA, c = kLcgC;
    while (n) {
        if (n & 1) {
            A = A * a;
            C = C * a + c;
        }
        c = (a + 1) * c;
        a = a * a;
        n >>= 1;
    }
    return A * s + C;
}

// Float.random(in: 0..<1, using:) for a 64-bit generator: the low 24 bits of
// the 32-bit truncation of next(), times 2^-24.
inline float unit_float(uint64_t v) { return (float)((uint32_t)v & 0xFFFFFFu) * 5.9604644775390625e-08f; }
}  // namespace

extern "C" tb_status tb_rng_seed_state(uint64_t seed, uint64_t* state) {
    TB_CHECK(state, "state is NULL");
    *state = seed != 0 ? seed : 0xdeadbeefull;  // ModelWeights.swift:21-23
    return ok();
}

extern "C" tb_status tb_rng_fill_normal(uint64_t* state, float mean, float stdv, int64_t n, float* out) {
    TB_CHECK(state && (out || n == 0), "NULL argument");
    TB_CHECK(n >= 0, "negative count");
    const int64_t pairs = (n + 1) / 2;
    const uint64_t s0 = *state;
    const float sd = stdv;
    unsigned nt = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
    if (pairs < 65536) nt = 1;
    auto work = [s0, sd, mean, n, out](int64_t pb, int64_t pe) {
        uint64_t s = lcg_jump(s0, (uint64_t)(2 * pb));
        const float two_pi = 2.0f * 3.14159265358979323846f;  // 2.0 * Float.pi
        for (int64_t pi = pb; pi < pe; ++pi) {
            s = kLcgA * s + kLcgC;
            float u1 = unit_float(s);
            s = kLcgA * s + kLcgC;
            const float u2 = unit_float(s);
            u1 = std::max(u1, 1.40129846e-45f);  // Float.leastNonzeroMagnitude
            const float r = sqrtf(-2.0f * logf(u1));
            const float theta = two_pi * u2;
            const int64_t i = 2 * pi;
            out[i] = mean + sd * r * cosf(theta);
            if (i + 1 < n) out[i + 1] = mean + sd * r * sinf(theta);
        }
    };
    if (nt == 1) {
        work(0, pairs);
    } else {
        std::vector<std::thread> th;
        for (unsigned t = 0; t < nt; ++t) {
            int64_t pb = pairs * t / nt, pe = pairs * (t + 1) / nt;
            th.emplace_back(work, pb, pe);
        }
        for (auto& x : th) x.join();
    }
    *state = lcg_jump(s0, (uint64_t)(2 * pairs));
    return ok();
}

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
extern "C" tb_status tb_context_create(int32_t device, tb_context** out) {
    TB_CHECK(out, "out is NULL");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(TB_ERR_NO_DEVICE, "no CUDA device visible");
    TB_CHECK(device >= 0 && device < n, "device %d out of range (%d devices)", device, n);
    TB_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop{};
    TB_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10)
        return fail(TB_ERR_UNSUPPORTED, "device %d is sm_%d%d; libtinybrain_cuda is built for sm_100a", device,
                    prop.major, prop.minor);
    auto c = std::make_unique<tb_context>();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    TB_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    TB_CUDA(c->err.alloc(sizeof(int)));
    TB_CUDA(cudaMemset(c->err.p, 0, sizeof(int)));
    *out = c.release();
    return ok();
}

extern "C" tb_status tb_context_destroy(tb_context* ctx) {
    if (!ctx) return ok();
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->comm) nccl_comm_destroy(ctx->comm);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return ok();
}

extern "C" tb_status tb_context_synchronize(tb_context* ctx) {
    TB_CHECK(ctx, "ctx is NULL");
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return ok();
}

extern "C" void* tb_context_stream(tb_context* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

extern "C" tb_status tb_context_check_device(tb_context* ctx) {
    TB_CHECK(ctx, "ctx is NULL");
    int v = 0;
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    TB_CUDA(cudaMemcpy(&v, ctx->err.p, sizeof(int), cudaMemcpyDeviceToHost));
    TB_CUDA(cudaMemset(ctx->err.p, 0, sizeof(int)));
    if (v == 0) return ok();
    if (v == kDevWaitTimeout) return fail(TB_ERR_DEVICE_TIMEOUT, "a device-side wait exceeded its time limit");
    if (v == kDevBadPage) return fail(TB_ERR_STATE, "KV append found no page mapped for the position");
    if (v == kDevBadToken) return fail(TB_ERR_STATE, "token id outside the vocabulary");
    if (v == kDevBadSmem) return fail(TB_ERR_STATE, "a kernel's shared-memory layout was misaligned (no work done)");
    return fail(TB_ERR_STATE, "device error code %d", v);
}

extern "C" tb_status tb_debug_expire_wait(tb_context* ctx, int32_t which) {
    TB_CHECK(ctx, "ctx is NULL");
    TB_CHECK(which == 0 || which == 1, "which must be 0 (mbarrier) or 1 (tagged word)");
    TB_CUDA(cudaSetDevice(ctx->device));
    DevBuf word;
    TB_CUDA(word.alloc(8));
    TB_CUDA(cudaMemsetAsync(word.p, 0, 8, ctx->stream));
    TB_CUDA(launch_wait_probe(which, word.as<unsigned long long>(), ctx->err.as<int>(), ctx->stream));
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return ok();
}

static tb_status ensure(DevBuf& b, size_t bytes) {
    if (b.bytes >= bytes) return ok();
    TB_CUDA(b.alloc(bytes));
    return ok();
}

// ---------------------------------------------------------------------------
// quantizers
// ---------------------------------------------------------------------------
extern "C" tb_status tb_quantize_int8_per_channel_dev(tb_context* ctx, const float* w, int64_t K, int64_t N,
                                                      int8_t* q, float* s) {
    TB_CHECK(ctx && w && q && s, "NULL argument");
    TB_CHECK(K > 0 && N > 0, "K and N must be positive");
    TB_CUDA(cudaSetDevice(ctx->device));
    TB_CUDA(launch_quantize_int8_per_channel(w, K, N, q, s, ctx->stream));
    return ok();
}

extern "C" tb_status tb_quantize_int4_group_dev(tb_context* ctx, const float* x, int64_t count, int64_t gs,
                                                uint8_t* packed, float* s, int8_t* zp) {
    TB_CHECK(ctx && x && packed && s, "NULL argument");
    TB_CHECK(count > 0 && gs > 0, "count and group_size must be positive");
    TB_CUDA(cudaSetDevice(ctx->device));
    TB_CUDA(launch_quantize_int4_group(x, count, gs, packed, s, zp, ctx->stream));
    return ok();
}

extern "C" tb_status tb_quantize_int8_per_channel(tb_context* ctx, const float* w, int64_t K, int64_t N, int8_t* q,
                                                  float* s) {
    TB_CHECK(ctx && w && q && s, "NULL argument");
    TB_CHECK(K > 0 && N > 0, "K and N must be positive");
    TB_CUDA(cudaSetDevice(ctx->device));
    const size_t nw = (size_t)K * N;
    DevBuf dw, dq, ds;
    TB_CUDA(dw.alloc(nw * 4));
    TB_CUDA(dq.alloc(nw));
    TB_CUDA(ds.alloc((size_t)N * 4));
    TB_CUDA(cudaMemcpyAsync(dw.p, w, nw * 4, cudaMemcpyHostToDevice, ctx->stream));
    TB_CUDA(launch_quantize_int8_per_channel(dw.as<float>(), K, N, dq.as<int8_t>(), ds.as<float>(), ctx->stream));
    TB_CUDA(cudaMemcpyAsync(q, dq.p, nw, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(s, ds.p, (size_t)N * 4, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return ok();
}

extern "C" tb_status tb_quantize_int4_group(tb_context* ctx, const float* x, int64_t count, int64_t gs,
                                            uint8_t* packed, float* s, int8_t* zp) {
    TB_CHECK(ctx && x && packed && s, "NULL argument");
    TB_CHECK(count > 0 && gs > 0, "count and group_size must be positive");
    TB_CUDA(cudaSetDevice(ctx->device));
    const size_t nb = (size_t)(count + 1) / 2, ng = (size_t)((count + gs - 1) / gs);
    DevBuf dx, dp, ds, dz;
    TB_CUDA(dx.alloc((size_t)count * 4));
    TB_CUDA(dp.alloc(nb));
    TB_CUDA(ds.alloc(ng * 4));
    TB_CUDA(dz.alloc(ng));
    TB_CUDA(cudaMemcpyAsync(dx.p, x, (size_t)count * 4, cudaMemcpyHostToDevice, ctx->stream));
    TB_CUDA(launch_quantize_int4_group(dx.as<float>(), count, gs, dp.as<uint8_t>(), ds.as<float>(),
                                       dz.as<int8_t>(), ctx->stream));
    TB_CUDA(cudaMemcpyAsync(packed, dp.p, nb, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(s, ds.p, ng * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (zp) TB_CUDA(cudaMemcpyAsync(zp, dz.p, ng, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return ok();
}

// QuantizedTensor.dequantize (QuantizedTensor.swift:182-285) of a host tensor:
// per-channel INT8 or INT4 groups, zero points honoured; staged through HBM.
static tb_status dequantize_to_device(tb_context* ctx, const tb_qtensor_desc* d, DevBuf& out) {
    TB_CHECK(d && d->data && d->scales, "NULL argument");
    TB_CHECK(d->precision == 8 || d->precision == 4, "precision must be 8 or 4 (got %d)", d->precision);
    TB_CHECK(d->in_features > 0 && d->out_features > 0, "shape must be positive");
    const int64_t cnt = d->in_features * d->out_features;
    const int64_t gs = d->precision == 4 ? (d->group_size > 0 ? d->group_size : cnt) : 0;
    const int64_t nb = d->precision == 8 ? cnt : (cnt + 1) / 2;
    const int64_t ns = d->precision == 8 ? d->out_features : (cnt + gs - 1) / gs;
    TB_CHECK(d->data_bytes == nb, "data must hold %lld bytes (got %lld)", (long long)nb, (long long)d->data_bytes);
    TB_CHECK(d->num_scales == ns, "expected %lld scales (got %lld)", (long long)ns, (long long)d->num_scales);
    TB_CHECK(!d->zero_points || d->num_zero_points == ns, "expected %lld zero points", (long long)ns);
    DevBuf dd, ds, dz;
    TB_CUDA(dd.alloc((size_t)nb));
    TB_CUDA(ds.alloc((size_t)ns * 4));
    TB_CUDA(out.alloc((size_t)cnt * 4));
    TB_CUDA(cudaMemcpyAsync(dd.p, d->data, (size_t)nb, cudaMemcpyHostToDevice, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(ds.p, d->scales, (size_t)ns * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (d->zero_points) {
        TB_CUDA(dz.alloc((size_t)ns));
        TB_CUDA(cudaMemcpyAsync(dz.p, d->zero_points, (size_t)ns, cudaMemcpyHostToDevice, ctx->stream));
    }
    TB_CUDA(launch_dequantize(d->precision, dd.as<uint8_t>(), ds.as<float>(), dz.as<int8_t>(), d->in_features,
                              d->out_features, gs, out.as<float>(), ctx->stream));
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return ok();
}

extern "C" tb_status tb_dequantize(tb_context* ctx, const tb_qtensor_desc* d, float* out_host) {
    TB_CHECK(ctx && out_host, "NULL argument");
    TB_CUDA(cudaSetDevice(ctx->device));
    DevBuf out;
    tb_status s = dequantize_to_device(ctx, d, out);
    if (s != TB_OK) return s;
    TB_CUDA(cudaMemcpy(out_host, out.p, out.bytes, cudaMemcpyDeviceToHost));
    return ok();
}

// PerplexityHarness.convertToINT4 (PerplexityHarness.swift:65-126) for one
// linear weight: dequantize, then the INT4 group quantizer, both on the device.
extern "C" tb_status tb_requantize_int4(tb_context* ctx, const tb_qtensor_desc* d, int64_t gs, uint8_t* packed,
                                        float* scales, int8_t* zps) {
    TB_CHECK(ctx && packed && scales, "NULL argument");
    TB_CHECK(gs > 0, "group_size must be positive");
    TB_CUDA(cudaSetDevice(ctx->device));
    DevBuf w;
    tb_status s = dequantize_to_device(ctx, d, w);
    if (s != TB_OK) return s;
    const int64_t cnt = d->in_features * d->out_features;
    const size_t nb = (size_t)(cnt + 1) / 2, ng = (size_t)((cnt + gs - 1) / gs);
    DevBuf dp, ds, dz;
    TB_CUDA(dp.alloc(nb));
    TB_CUDA(ds.alloc(ng * 4));
    TB_CUDA(dz.alloc(ng));
    TB_CUDA(launch_quantize_int4_group(w.as<float>(), cnt, gs, dp.as<uint8_t>(), ds.as<float>(), dz.as<int8_t>(),
                                       ctx->stream));
    TB_CUDA(cudaMemcpyAsync(packed, dp.p, nb, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(scales, ds.p, ng * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (zps) TB_CUDA(cudaMemcpyAsync(zps, dz.p, ng, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return ok();
}

// ---------------------------------------------------------------------------
// quantized weights
// ---------------------------------------------------------------------------
static tb_status validate_desc(const tb_qtensor_desc* d) {
    TB_CHECK(d, "desc is NULL");
    TB_CHECK(d->precision == 8 || d->precision == 4, "precision must be 8 or 4 (got %d)", d->precision);
    TB_CHECK(d->in_features > 0 && d->out_features > 0, "shape must be positive");
    TB_CHECK(d->in_features < (1 << 30) && d->out_features < (1 << 30), "shape too large");
    TB_CHECK(d->data && d->scales, "data and scales are required");
    const int64_t cnt = d->in_features * d->out_features;
    if (d->precision == 8) {
        TB_CHECK(d->data_bytes == cnt, "INT8 data must hold K*N = %lld bytes (got %lld)", (long long)cnt,
                 (long long)d->data_bytes);
        TB_CHECK(d->num_scales == d->out_features, "INT8 per-channel needs N = %lld scales (got %lld)",
                 (long long)d->out_features, (long long)d->num_scales);
        if (d->zero_points)
            for (int64_t i = 0; i < d->num_zero_points; ++i)
                if (d->zero_points[i] != 0)
                    return fail(TB_ERR_UNSUPPORTED, "non-zero INT8 zero points are not supported");
    } else {
        const int64_t gs = d->group_size;
        TB_CHECK(gs > 0, "INT4 group_size must be positive");
        TB_CHECK(d->data_bytes == (cnt + 1) / 2, "INT4 data must hold ceil(K*N/2) bytes");
        TB_CHECK(d->num_scales == (cnt + gs - 1) / gs, "INT4 needs ceil(K*N/group_size) scales");
        if (gs % 32 != 0 || d->out_features % gs != 0)
            return fail(TB_ERR_UNSUPPORTED,
                        "INT4 needs group_size %% 32 == 0 and out_features %% group_size == 0 (group %lld, N %lld)",
                        (long long)gs, (long long)d->out_features);
        if (d->zero_points)
            for (int64_t i = 0; i < d->num_zero_points; ++i)
                if (d->zero_points[i] != 0)
                    return fail(TB_ERR_UNSUPPORTED, "non-zero INT4 zero points are not supported");
    }
    return ok();
}

static tb_status stage_desc(tb_context* ctx, const tb_qtensor_desc* d, ProjStage& st) {
    tb_status s = validate_desc(d);
    if (s != TB_OK) return s;
    st.precision = d->precision;
    st.K = (int)d->in_features;
    st.N = (int)d->out_features;
    st.gs = (int)d->group_size;
    TB_CUDA(st.data.alloc((size_t)d->data_bytes));
    TB_CUDA(st.scales.alloc((size_t)d->num_scales * 4));
    TB_CUDA(cudaMemcpyAsync(st.data.p, d->data, (size_t)d->data_bytes, cudaMemcpyHostToDevice, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(st.scales.p, d->scales, (size_t)d->num_scales * 4, cudaMemcpyHostToDevice,
                            ctx->stream));
    st.set = true;
    return ok();
}

static tb_status alloc_fused(tb_context* ctx, FusedWeight& f, const QLayout& L) {
    f.L = L;
    TB_CUDA(f.w.alloc(L.weight_bytes));
    TB_CUDA(f.s.alloc(L.scale_floats * 4));
    // padding reads as zero weights: INT8 stores q itself, INT4 stores q + 8
    TB_CUDA(cudaMemsetAsync(f.w.p, L.precision == 8 ? 0x00 : 0x88, L.weight_bytes, ctx->stream));
    TB_CUDA(cudaMemsetAsync(f.s.p, 0, L.scale_floats * 4, ctx->stream));
    return ok();
}

static tb_status repack_into(tb_context* ctx, FusedWeight& f, const ProjStage& st, int row_offset, int interleave) {
    RepackSrc rs{};
    rs.precision = st.precision;
    rs.K = st.K;
    rs.N = st.N;
    rs.group_size = st.gs;
    rs.data = st.data.p;
    rs.scales = st.scales.as<float>();
    TB_CUDA(launch_repack(rs, f.L, f.w.as<uint8_t>(), f.s.as<float>(), row_offset, interleave, ctx->stream));
    return ok();
}

extern "C" tb_status tb_qweight_upload(tb_context* ctx, const tb_qtensor_desc* d, tb_qweight** out) {
    TB_CHECK(ctx && out, "NULL argument");
    *out = nullptr;
    TB_CUDA(cudaSetDevice(ctx->device));
    ProjStage st;
    tb_status s = stage_desc(ctx, d, st);
    if (s != TB_OK) return s;
    auto w = std::make_unique<tb_qweight>();
    w->ctx = ctx;
    FusedWeight f;
    s = alloc_fused(ctx, f, make_qlayout(st.precision, st.K, st.N, 32));
    if (s != TB_OK) return s;
    s = repack_into(ctx, f, st, 0, 0);
    if (s != TB_OK) return s;
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    w->L = f.L;
    std::swap(w->w.p, f.w.p);
    std::swap(w->w.bytes, f.w.bytes);
    std::swap(w->s.p, f.s.p);
    std::swap(w->s.bytes, f.s.bytes);
    *out = w.release();
    return ok();
}

extern "C" tb_status tb_qweight_free(tb_qweight* w) {
    if (w) {
        cudaSetDevice(w->ctx->device);
        delete w;
    }
    return ok();
}

static GemvParams plain_gemv(tb_context* ctx, const QLayout& L, const uint8_t* w, const float* s, int M) {
    GemvParams p{};
    p.w = w;
    p.scales = s;
    p.L = L;
    p.M = M;
    p.P = choose_ksplit(L, M, ctx->num_sms);
    p.prologue = kProNone;
    p.ld_src = L.K;
    p.epilogue = kEpiStore;
    p.ld_out = L.N;
    p.err = ctx->err.as<int>();
    return p;
}

// A timed stream of independent GEMVs (BASELINE config 1 measurement): one
// CUDA graph launches every weight once (in order, programmatic dependent launch
// between them so each kernel's weight stream overlaps its predecessor's tail);
// the graph is replayed `reps` times after one warm-up replay.  All weights
// share K; y must hold M x max(N).  Returns milliseconds per replay.
extern "C" tb_status tb_qgemv_stream_time(tb_context* ctx, const tb_qweight* const* ws, int32_t n, const float* x,
                                          int64_t M, float* y, int32_t reps, int32_t pdl, float* ms_out) {
    TB_CHECK(ctx && ws && x && y && ms_out && n > 0 && reps > 0, "invalid argument");
    TB_CHECK(M >= 1 && M <= kMaxGemvBatch, "M must be in [1, %d] (got %lld)", kMaxGemvBatch, (long long)M);
    TB_CUDA(cudaSetDevice(ctx->device));
    for (int i = 0; i < n; ++i) {
        TB_CHECK(ws[i], "NULL weight %d", i);
        TB_CHECK(ws[i]->L.K == ws[0]->L.K, "weights must share K");
    }
    cudaStream_t st = ctx->stream;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    TB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    cudaError_t le = cudaSuccess;
    for (int i = 0; i < n && le == cudaSuccess; ++i) {
        GemvParams p = plain_gemv(ctx, ws[i]->L, ws[i]->w.as<uint8_t>(), ws[i]->s.as<float>(), (int)M);
        p.src = x;
        p.out = y;
        p.independent = pdl == 2 ? 1 : 0;  // independent GEMVs overlap their launches
        if (pdl == 2 && !getenv("TB_GEMV_P")) p.P = choose_ksplit_stream(ws[i]->L, (int)M);
        le = launch_gemv(p, st, pdl != 0 && i > 0);
    }
    cudaError_t ce = cudaStreamEndCapture(st, &g);
    if (le != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return cuda_fail(le, "launch_gemv");
    }
    TB_CUDA(ce);
    ce = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    TB_CUDA(ce);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    ce = cudaGraphLaunch(ge, st);
    if (ce == cudaSuccess) ce = cudaEventRecord(e0, st);
    for (int r = 0; r < reps && ce == cudaSuccess; ++r) ce = cudaGraphLaunch(ge, st);
    if (ce == cudaSuccess) ce = cudaEventRecord(e1, st);
    if (ce == cudaSuccess) ce = cudaEventSynchronize(e1);
    float ms = 0.0f;
    if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(ge);
    TB_CUDA(ce);
    *ms_out = ms / (float)reps;
    return tb_context_check_device(ctx);
}

extern "C" tb_status tb_matmul_quantized_dev(tb_context* ctx, const float* x, int64_t M, const tb_qweight* w,
                                             float* y) {
    TB_CHECK(ctx && x && w && y, "NULL argument");
    TB_CHECK(M >= 1 && M <= kMaxGemvBatch, "M must be in [1, %d] for the decode GEMV (got %lld)", kMaxGemvBatch,
             (long long)M);
    TB_CUDA(cudaSetDevice(ctx->device));
    GemvParams p = plain_gemv(ctx, w->L, w->w.as<uint8_t>(), w->s.as<float>(), (int)M);
    p.src = x;
    p.out = y;
    TB_CUDA(launch_gemv(p, ctx->stream, false));
    return ok();
}

extern "C" tb_status tb_matmul_quantized(tb_context* ctx, const float* x, int64_t M, const tb_qweight* w,
                                         float* y) {
    TB_CHECK(ctx && x && w && y, "NULL argument");
    TB_CHECK(M >= 1 && M <= kMaxGemvBatch, "M must be in [1, %d] for the decode GEMV (got %lld)", kMaxGemvBatch,
             (long long)M);
    TB_CUDA(cudaSetDevice(ctx->device));
    const size_t xb = (size_t)M * w->L.K * 4, yb = (size_t)M * w->L.N * 4;
    tb_status s = ensure(ctx->io_a, xb);
    if (s != TB_OK) return s;
    s = ensure(ctx->io_b, yb);
    if (s != TB_OK) return s;
    TB_CUDA(cudaMemcpyAsync(ctx->io_a.p, x, xb, cudaMemcpyHostToDevice, ctx->stream));
    s = tb_matmul_quantized_dev(ctx, ctx->io_a.as<float>(), M, w, ctx->io_b.as<float>());
    if (s != TB_OK) return s;
    TB_CUDA(cudaMemcpyAsync(y, ctx->io_b.p, yb, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return tb_context_check_device(ctx);
}

// ---------------------------------------------------------------------------
// attention entry points
// ---------------------------------------------------------------------------
namespace {
__global__ void pack_kv_contig_kernel(const float* __restrict__ K, const float* __restrict__ V, int64_t L, int Hkv,
                                      int d, float* __restrict__ pool) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t kvdim = (int64_t)Hkv * d;
    if (i >= L * kvdim) return;
    const int64_t pos = i / kvdim, r = i % kvdim;
    const int64_t head = r / d, e = r % d;
    const int64_t page = pos / kPageTokens, slot = pos % kPageTokens;
    const size_t kb = ((((size_t)page * 1 + 0) * 2 + 0) * Hkv + head) * kPageTokens + slot;
    const size_t vb = ((((size_t)page * 1 + 0) * 2 + 1) * Hkv + head) * kPageTokens + slot;
    pool[kb * d + e] = K[i];
    pool[vb * d + e] = V[i];
}
__global__ void iota_kernel(int* p, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = i;
}
}  // namespace

static tb_status check_heads(int H, int Hkv, int d) {
    TB_CHECK(H > 0 && Hkv > 0 && d > 0 && H % Hkv == 0, "heads must divide: H %d, Hkv %d", H, Hkv);
    const int G = H / Hkv;
    bool okg = (G == 1 && (d == 16 || d == 32 || d == 64 || d == 128)) ||
               (G == 2 && (d == 16 || d == 32 || d == 64 || d == 128)) ||
               (G == 4 && (d == 16 || d == 32 || d == 64 || d == 128)) || (G == 8 && (d == 16 || d == 32 || d == 64));
    if (!okg) return fail(TB_ERR_UNSUPPORTED, "unsupported head geometry G=%d d=%d", G, d);
    return ok();
}

static tb_status run_paged_attention(tb_context* ctx, const float* q, int batch, const float* pool,
                                     const int* ptab, int ptab_stride, const int* lens, int max_len, int layer,
                                     int num_layers, int H, int Hkv, int d, float* out) {
    const int max_pages = (max_len + kPageTokens - 1) / kPageTokens;
    const int ns = choose_nsplit(batch, Hkv, std::max(1, max_pages), ctx->num_sms);
    AttnParams a{};
    a.q = q;
    a.ld_q = H * d;
    a.kv_pool = pool;
    a.page_table = ptab;
    a.ptab_stride = ptab_stride;
    a.lens = lens;
    a.seq = nullptr;
    a.layer = layer;
    a.num_layers = num_layers;
    a.H = H;
    a.Hkv = Hkv;
    a.d = d;
    a.M = batch;
    a.nsplit = ns;
    a.out = out;
    a.ld_out = H * d;
    a.err = ctx->err.as<int>();
    TB_CUDA(launch_attention(a, ctx->stream, false));
    return ok();
}

extern "C" tb_status tb_paged_attention_dev(tb_context* ctx, const float* q, int32_t batch, const float* pool,
                                            const int32_t* ptab, int32_t ptab_stride, const int32_t* lens,
                                            int32_t max_len, int32_t layer, int32_t num_layers, int32_t H,
                                            int32_t Hkv, int32_t d, float* out) {
    TB_CHECK(ctx && q && pool && ptab && lens && out, "NULL argument");
    TB_CHECK(batch >= 1 && max_len >= 1 && layer >= 0 && layer < num_layers, "bad batch/len/layer");
    tb_status s = check_heads(H, Hkv, d);
    if (s != TB_OK) return s;
    TB_CUDA(cudaSetDevice(ctx->device));
    return run_paged_attention(ctx, q, batch, pool, ptab, ptab_stride, lens, max_len, layer, num_layers, H, Hkv, d,
                               out);
}

extern "C" tb_status tb_attention_decode(tb_context* ctx, const float* q, const float* K, const float* V, int64_t L,
                                         int32_t H, int32_t Hkv, int32_t d, float* out) {
    TB_CHECK(ctx && q && K && V && out, "NULL argument");
    TB_CHECK(L >= 1 && L < (1ll << 24), "L out of range");
    tb_status s = check_heads(H, Hkv, d);
    if (s != TB_OK) return s;
    TB_CUDA(cudaSetDevice(ctx->device));
    const int64_t kvdim = (int64_t)Hkv * d;
    const int64_t pages = (L + kPageTokens - 1) / kPageTokens;
    const size_t pool_b = (size_t)pages * 2 * kvdim * kPageTokens * 4;
    DevBuf dk, dv, pool, ptab, lens, dq, dout;
    TB_CUDA(dk.alloc((size_t)L * kvdim * 4));
    TB_CUDA(dv.alloc((size_t)L * kvdim * 4));
    TB_CUDA(pool.alloc(pool_b));
    TB_CUDA(ptab.alloc((size_t)pages * 4));
    TB_CUDA(lens.alloc(4));
    TB_CUDA(dq.alloc((size_t)H * d * 4));
    TB_CUDA(dout.alloc((size_t)H * d * 4));
    TB_CUDA(cudaMemsetAsync(pool.p, 0, pool_b, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(dk.p, K, (size_t)L * kvdim * 4, cudaMemcpyHostToDevice, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(dv.p, V, (size_t)L * kvdim * 4, cudaMemcpyHostToDevice, ctx->stream));
    TB_CUDA(cudaMemcpyAsync(dq.p, q, (size_t)H * d * 4, cudaMemcpyHostToDevice, ctx->stream));
    const int l32 = (int)L;
    TB_CUDA(cudaMemcpyAsync(lens.p, &l32, 4, cudaMemcpyHostToDevice, ctx->stream));
    const int64_t tot = L * kvdim;
    pack_kv_contig_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, ctx->stream>>>(
        dk.as<float>(), dv.as<float>(), L, Hkv, d, pool.as<float>());
    iota_kernel<<<(unsigned)((pages + 255) / 256), 256, 0, ctx->stream>>>(ptab.as<int>(), (int)pages);
    TB_CUDA(cudaGetLastError());
    s = run_paged_attention(ctx, dq.as<float>(), 1, pool.as<float>(), ptab.as<int>(), (int)pages, lens.as<int>(),
                            (int)L, 0, 1, H, Hkv, d, dout.as<float>());
    if (s != TB_OK) return s;
    TB_CUDA(cudaMemcpyAsync(out, dout.p, (size_t)H * d * 4, cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    return tb_context_check_device(ctx);
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
extern "C" tb_status tb_model_create(tb_context* ctx, const tb_model_config* cfg, tb_model** out) {
    TB_CHECK(ctx && cfg && out, "NULL argument");
    *out = nullptr;
    const tb_model_config& c = *cfg;
    TB_CHECK(c.num_layers > 0 && c.hidden_dim > 0 && c.num_heads > 0 && c.num_kv_heads > 0 && c.vocab_size > 0 &&
                 c.max_seq_len > 0 && c.intermediate_dim > 0,
             "config fields must be positive");
    TB_CHECK(c.hidden_dim % c.num_heads == 0, "hidden_dim must be a multiple of num_heads");
    TB_CHECK(c.architecture == TB_ARCH_LLAMA || c.architecture == TB_ARCH_TOY, "unknown architecture %d",
             c.architecture);
    const int d = c.hidden_dim / c.num_heads;
    tb_status s = check_heads(c.num_heads, c.num_kv_heads, d);
    if (s != TB_OK) return s;
    TB_CHECK(c.hidden_dim % 32 == 0 && (d * c.num_kv_heads) % 32 == 0,
             "hidden_dim and kv_dim must be multiples of 32");
    auto m = std::make_unique<tb_model>();
    m->ctx = ctx;
    m->cfg = c;
    if (m->cfg.rms_eps == 0.0f) m->cfg.rms_eps = 1e-5f;
    m->head_dim = d;
    m->kv_dim = d * c.num_kv_heads;
    m->q_dim = c.hidden_dim;
    m->full = m->cfg;
    m->layers.resize(c.num_layers);
    *out = m.release();
    return ok();
}

extern "C" tb_status tb_tp_unique_id(uint8_t* id) {
    TB_CHECK(id, "NULL argument");
    std::string why;
    if (nccl_unique_id(id, why)) return fail(TB_ERR_UNSUPPORTED, "%s", why.c_str());
    return ok();
}

extern "C" tb_status tb_context_init_tp(tb_context* ctx, const uint8_t* id, int32_t rank, int32_t world) {
    TB_CHECK(ctx && id, "NULL argument");
    TB_CHECK(world >= 1 && rank >= 0 && rank < world, "rank %d / world %d", rank, world);
    TB_CHECK(!ctx->comm, "context already has a tensor-parallel communicator");
    TB_CUDA(cudaSetDevice(ctx->device));
    if (world > 1) {
        std::string why;
        if (nccl_comm_init(&ctx->comm, id, rank, world, why)) return fail(TB_ERR_UNSUPPORTED, "%s", why.c_str());
    }
    ctx->tp_rank = rank;
    ctx->tp_world = world;
    return ok();
}

extern "C" tb_status tb_model_set_tensor_parallel(tb_model* m, int32_t rank, int32_t world) {
    TB_CHECK(m, "NULL model");
    TB_CHECK(!m->finalized, "model already finalized");
    TB_CHECK(m->tp_world == 1, "tensor parallelism already set");
    for (const Layer& L : m->layers)
        for (const ProjStage& st : L.stage) TB_CHECK(!st.set, "set tensor parallelism before the projections");
    TB_CHECK(world >= 1 && rank >= 0 && rank < world, "rank %d / world %d", rank, world);
    TB_CHECK(m->ctx->tp_world == world && m->ctx->tp_rank == rank,
             "context is rank %d of %d (tb_context_init_tp), model asks for rank %d of %d", m->ctx->tp_rank,
             m->ctx->tp_world, rank, world);
    const tb_model_config& f = m->full;
    TB_CHECK(f.num_heads % world == 0 && f.num_kv_heads % world == 0 && f.intermediate_dim % world == 0,
             "heads %d, kv heads %d and intermediate %d must divide by %d ranks", f.num_heads, f.num_kv_heads,
             f.intermediate_dim, world);
    const int hl = f.num_heads / world, kl = f.num_kv_heads / world, il = f.intermediate_dim / world;
    TB_CHECK((hl * m->head_dim) % 32 == 0 && (kl * m->head_dim) % 32 == 0 && il % 32 == 0,
             "per-rank q, kv and intermediate widths must be multiples of 32");
    m->cfg.num_heads = hl;
    m->cfg.num_kv_heads = kl;
    m->cfg.intermediate_dim = il;
    m->q_dim = hl * m->head_dim;
    m->kv_dim = kl * m->head_dim;
    m->tp_rank = rank;
    m->tp_world = world;
    return ok();
}

extern "C" tb_status tb_model_free(tb_model* m) {
    if (m) {
        cudaSetDevice(m->ctx->device);
        delete m;
    }
    return ok();
}

extern "C" tb_status tb_model_set_embedding(tb_model* m, const float* emb) {
    TB_CHECK(m && emb, "NULL argument");
    TB_CHECK(!m->finalized, "model already finalized");
    TB_CUDA(cudaSetDevice(m->ctx->device));
    const size_t b = (size_t)m->cfg.vocab_size * m->cfg.hidden_dim * 4;
    TB_CUDA(m->emb.alloc(b));
    TB_CUDA(cudaMemcpy(m->emb.p, emb, b, cudaMemcpyHostToDevice));
    return ok();
}

extern "C" tb_status tb_model_set_final_norm(tb_model* m, const float* w) {
    TB_CHECK(m, "NULL model");
    TB_CHECK(!m->finalized, "model already finalized");
    TB_CUDA(cudaSetDevice(m->ctx->device));
    if (!w) {
        m->has_final_norm = false;
        return ok();
    }
    TB_CUDA(m->final_norm.alloc((size_t)m->cfg.hidden_dim * 4));
    TB_CUDA(cudaMemcpy(m->final_norm.p, w, (size_t)m->cfg.hidden_dim * 4, cudaMemcpyHostToDevice));
    m->has_final_norm = true;
    return ok();
}

extern "C" tb_status tb_model_set_layer_norms(tb_model* m, int32_t layer, const float* in, const float* post) {
    TB_CHECK(m && layer >= 0 && layer < m->cfg.num_layers, "bad model/layer");
    TB_CHECK(!m->finalized, "model already finalized");
    Layer& L = m->layers[layer];
    const int H = m->cfg.hidden_dim;
    L.in_norm.assign(in ? in : (const float*)nullptr, in ? in + H : (const float*)nullptr);
    L.post_norm.assign(post ? post : (const float*)nullptr, post ? post + H : (const float*)nullptr);
    return ok();
}

static tb_status expected_shape(const tb_model* m, int which, int& K, int& N) {
    const int H = m->cfg.hidden_dim, I = m->cfg.intermediate_dim, qd = m->q_dim;
    switch (which) {
        case TB_PROJ_Q: K = H; N = qd; break;
        case TB_PROJ_K:
        case TB_PROJ_V: K = H; N = m->kv_dim; break;
        case TB_PROJ_O: K = qd; N = H; break;
        case TB_PROJ_GATE:
        case TB_PROJ_UP: K = H; N = I; break;
        case TB_PROJ_DOWN: K = I; N = H; break;
        default: return fail(TB_ERR_INVALID_ARGUMENT, "unknown projection %d", which);
    }
    return ok();
}

extern "C" tb_status tb_model_set_projection(tb_model* m, int32_t layer, int32_t which, const tb_qtensor_desc* d,
                                             const float* bias) {
    TB_CHECK(m && layer >= 0 && layer < m->cfg.num_layers, "bad model/layer");
    TB_CHECK(!m->finalized, "model already finalized");
    int K = 0, N = 0;
    tb_status s = expected_shape(m, which, K, N);
    if (s != TB_OK) return s;
    TB_CHECK(d && d->in_features == K && d->out_features == N,
             "projection %d of layer %d must be [%d, %d] (got [%lld, %lld])", which, layer, K, N,
             d ? (long long)d->in_features : -1ll, d ? (long long)d->out_features : -1ll);
    TB_CUDA(cudaSetDevice(m->ctx->device));
    ProjStage& st = m->layers[layer].stage[which];
    s = stage_desc(m->ctx, d, st);
    if (s != TB_OK) return s;
    if (bias)
        st.bias.assign(bias, bias + N);
    else
        st.bias.clear();
    return ok();
}

extern "C" tb_status tb_model_set_output(tb_model* m, const tb_qtensor_desc* d, const float* bias) {
    TB_CHECK(m, "NULL model");
    TB_CHECK(!m->finalized, "model already finalized");
    TB_CHECK(d && d->in_features == m->cfg.hidden_dim && d->out_features == m->cfg.vocab_size,
             "output projection must be [%d, %d]", m->cfg.hidden_dim, m->cfg.vocab_size);
    TB_CUDA(cudaSetDevice(m->ctx->device));
    tb_status s = stage_desc(m->ctx, d, m->out_stage);
    if (s != TB_OK) return s;
    if (bias)
        m->out_stage.bias.assign(bias, bias + m->cfg.vocab_size);
    else
        m->out_stage.bias.clear();
    return ok();
}

// Scatter per-projection biases into the fused GPU row space.
static tb_status upload_bias(FusedWeight& f, const std::vector<std::pair<const ProjStage*, std::pair<int, int>>>& parts) {
    bool any = false;
    for (auto& pr : parts)
        if (!pr.first->bias.empty()) any = true;
    f.has_bias = any;
    if (!any) return ok();
    std::vector<float> hb((size_t)f.L.Np, 0.0f);
    for (auto& pr : parts) {
        const ProjStage* st = pr.first;
        const int off = pr.second.first, inter = pr.second.second;
        for (int n = 0; n < (int)st->bias.size(); ++n) {
            const int row = fused_row(f.L, n, off, inter);
            hb[row] = st->bias[n];
        }
    }
    TB_CUDA(f.bias.alloc(hb.size() * 4));
    TB_CUDA(cudaMemcpy(f.bias.p, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice));
    return ok();
}

extern "C" tb_status tb_model_finalize(tb_model* m) {
    TB_CHECK(m, "NULL model");
    if (m->finalized) return ok();
    tb_context* ctx = m->ctx;
    TB_CUDA(cudaSetDevice(ctx->device));
    const tb_model_config& c = m->cfg;
    const int H = c.hidden_dim, I = c.intermediate_dim, kvd = m->kv_dim, qd = m->q_dim;
    const bool llama = c.architecture == TB_ARCH_LLAMA;
    if (!m->emb.p) return fail(TB_ERR_STATE, "embedding not set");
    if (!m->out_stage.set) return fail(TB_ERR_STATE, "output projection not set");
    int64_t wbytes = 0;
    for (int l = 0; l < c.num_layers; ++l) {
        Layer& L = m->layers[l];
        for (int w : {TB_PROJ_Q, TB_PROJ_K, TB_PROJ_V, TB_PROJ_O, TB_PROJ_UP, TB_PROJ_DOWN})
            if (!L.stage[w].set) return fail(TB_ERR_STATE, "layer %d projection %d not set", l, w);
        if (llama && !L.stage[TB_PROJ_GATE].set) return fail(TB_ERR_STATE, "layer %d gate projection not set", l);
        const int pq = L.stage[TB_PROJ_Q].precision;
        if (L.stage[TB_PROJ_K].precision != pq || L.stage[TB_PROJ_V].precision != pq ||
            (L.stage[TB_PROJ_K].gs != L.stage[TB_PROJ_Q].gs && pq == 4))
            return fail(TB_ERR_UNSUPPORTED, "layer %d: q, k, v must share precision", l);
        tb_status s = alloc_fused(ctx, L.qkv, make_qlayout(pq, H, qd + 2 * kvd, 32));
        if (s != TB_OK) return s;
        if ((s = repack_into(ctx, L.qkv, L.stage[TB_PROJ_Q], 0, 0)) != TB_OK) return s;
        if ((s = repack_into(ctx, L.qkv, L.stage[TB_PROJ_K], qd, 0)) != TB_OK) return s;
        if ((s = repack_into(ctx, L.qkv, L.stage[TB_PROJ_V], qd + kvd, 0)) != TB_OK) return s;
        if ((s = upload_bias(L.qkv, {{&L.stage[TB_PROJ_Q], {0, 0}},
                                     {&L.stage[TB_PROJ_K], {qd, 0}},
                                     {&L.stage[TB_PROJ_V], {qd + kvd, 0}}})) != TB_OK)
            return s;
        if ((s = alloc_fused(ctx, L.o, make_qlayout(L.stage[TB_PROJ_O].precision, qd, H, 32))) != TB_OK) return s;
        if ((s = repack_into(ctx, L.o, L.stage[TB_PROJ_O], 0, 0)) != TB_OK) return s;
        if ((s = upload_bias(L.o, {{&L.stage[TB_PROJ_O], {0, 0}}})) != TB_OK) return s;
        if (llama) {
            const int pg = L.stage[TB_PROJ_GATE].precision;
            if (L.stage[TB_PROJ_UP].precision != pg)
                return fail(TB_ERR_UNSUPPORTED, "layer %d: gate and up must share precision", l);
            const int half = make_qlayout(pg, H, 64, 64).RB / 2;  // gate rows per row block
            const int Ip = (I + half - 1) / half * half;
            QLayout gl = make_qlayout(pg, H, 2 * Ip, 64);
            gl.N = I;
            if ((s = alloc_fused(ctx, L.up, gl)) != TB_OK) return s;
            if ((s = repack_into(ctx, L.up, L.stage[TB_PROJ_GATE], 0, 1)) != TB_OK) return s;
            if ((s = repack_into(ctx, L.up, L.stage[TB_PROJ_UP], 0, 2)) != TB_OK) return s;
            if ((s = upload_bias(L.up, {{&L.stage[TB_PROJ_GATE], {0, 1}}, {&L.stage[TB_PROJ_UP], {0, 2}}})) != TB_OK)
                return s;
        } else {
            if ((s = alloc_fused(ctx, L.up, make_qlayout(L.stage[TB_PROJ_UP].precision, H, I, 32))) != TB_OK)
                return s;
            if ((s = repack_into(ctx, L.up, L.stage[TB_PROJ_UP], 0, 0)) != TB_OK) return s;
            if ((s = upload_bias(L.up, {{&L.stage[TB_PROJ_UP], {0, 0}}})) != TB_OK) return s;
        }
        if ((s = alloc_fused(ctx, L.down, make_qlayout(L.stage[TB_PROJ_DOWN].precision, I, H, 32))) != TB_OK)
            return s;
        if ((s = repack_into(ctx, L.down, L.stage[TB_PROJ_DOWN], 0, 0)) != TB_OK) return s;
        if ((s = upload_bias(L.down, {{&L.stage[TB_PROJ_DOWN], {0, 0}}})) != TB_OK) return s;
        if (!L.in_norm.empty()) {
            TB_CUDA(L.in_norm_d.alloc((size_t)H * 4));
            TB_CUDA(cudaMemcpy(L.in_norm_d.p, L.in_norm.data(), (size_t)H * 4, cudaMemcpyHostToDevice));
        }
        if (!L.post_norm.empty()) {
            TB_CUDA(L.post_norm_d.alloc((size_t)H * 4));
            TB_CUDA(cudaMemcpy(L.post_norm_d.p, L.post_norm.data(), (size_t)H * 4, cudaMemcpyHostToDevice));
        }
        TB_CUDA(cudaStreamSynchronize(ctx->stream));
        for (auto& st : L.stage) {
            st.data.release();
            st.scales.release();
        }
        for (FusedWeight* f : {&L.qkv, &L.o, &L.up, &L.down})
            wbytes += (int64_t)f->L.weight_bytes + (int64_t)f->L.scale_floats * 4;
    }
    tb_status s = alloc_fused(ctx, m->out, make_qlayout(m->out_stage.precision, H, c.vocab_size, 32));
    if (s != TB_OK) return s;
    if ((s = repack_into(ctx, m->out, m->out_stage, 0, 0)) != TB_OK) return s;
    if ((s = upload_bias(m->out, {{&m->out_stage, {0, 0}}})) != TB_OK) return s;
    TB_CUDA(cudaStreamSynchronize(ctx->stream));
    m->out_stage.data.release();
    m->out_stage.scales.release();
    wbytes += (int64_t)m->out.L.weight_bytes + (int64_t)m->out.L.scale_floats * 4;
    m->weight_bytes = wbytes;
    m->finalized = true;
    return tb_context_check_device(ctx);
}

extern "C" tb_status tb_model_weight_bytes(const tb_model* m, int64_t* bytes) {
    TB_CHECK(m && bytes, "NULL argument");
    *bytes = m->weight_bytes;
    return ok();
}

// ---------------------------------------------------------------------------
// runner
// ---------------------------------------------------------------------------
// Buffers and rows of one step plan: the decode plan (the runner's batch) or
// the chunked-prefill plan (prompt tokens as rows, layers only).
struct PlanIO {
    int B;
    float *h, *h2, *q, *ctxv, *act;
    SeqState* seq;
    int* ptab;
    int nsplit;
    bool head;      // final norm + LM head (+ sampler)
    float* logits;  // [B][V] LM-head output
};

static void fill_gemv_common(tb_runner* r, GemvParams& p, const FusedWeight& f, const PlanIO& io) {
    p.w = f.w.as<uint8_t>();
    p.scales = f.s.as<float>();
    p.bias = f.has_bias ? f.bias.as<float>() : nullptr;
    p.L = f.L;
    p.M = io.B;
    p.P = choose_ksplit(f.L, io.B, r->ctx->num_sms);
    p.eps = r->m->cfg.rms_eps;
    p.vocab = r->m->cfg.vocab_size;
    p.seq_ro = io.seq;
    p.seq = io.seq;
    p.err = r->ctx->err.as<int>();
}

static int64_t gemv_bytes(const QLayout& L, int M) {
    // streamed weights + scales + activations in and out (fp32)
    int64_t w = (int64_t)L.weight_bytes + (int64_t)L.scale_floats * 4;
    return w + (int64_t)M * (L.K + L.N) * 4;
}

// Sampler launch parameters from the runner's current buffers and config.
static void fill_sample(tb_runner* r, SampleParams& s) {
    const int V = r->m->cfg.vocab_size;
    bool in_smem = false;
    sample_smem_bytes(V, &in_smem);
    s.logits = r->logits.as<float>();
    s.work = in_smem ? nullptr : r->swork.as<float>();
    s.V = V;
    s.M = r->B;
    s.seq = r->seq.as<SeqState>();
    s.prompt = r->prompt.as<int>();
    s.prompt_stride = r->prompt_stride;
    s.out_tokens = r->out_tokens.as<int>();
    s.out_prob = r->out_prob.as<float>();
    s.out_entropy = r->out_ent.as<float>();
    s.rng = r->rng.as<unsigned long long>();
    s.temperature = r->scfg.temperature;
    s.top_p = r->scfg.top_p;
    s.repetition_penalty = r->scfg.repetition_penalty;
    s.top_k = r->scfg.top_k;
    s.has_top_p = r->scfg.has_top_p;
    s.logprob_acc = r->scoring ? r->lp_acc.as<double>() : nullptr;
}

static tb_status build_plan_into(tb_runner* r, const PlanIO& io, std::vector<Launch>& plan) {
    tb_model* m = r->m;
    const tb_model_config& c = m->cfg;
    const int H = c.hidden_dim, d = m->head_dim, kvd = m->kv_dim, qd = m->q_dim, B = io.B;
    const bool llama = c.architecture == TB_ARCH_LLAMA;
    // Tensor parallel: QKV and gate/up are column shards (local heads, local
    // intermediate rows), o_proj and down row shards whose partial sums meet
    // in an all-reduce of the residual stream.  Rank 0 adds its partial to the
    // residual, the other ranks store theirs, so the sum is h + sum_r y_r.
    const bool tp = m->tp_world > 1;
    // Peer-memory all-reduce (after tb_runner_tp_connect): o_proj of layer l
    // pushes into slot 2l, down_proj into slot 2l + 1; the next launch that
    // reads the residual stream pulls the slot (residual + the ranks'
    // partials, rank order) and, in its CTA (0, 0), stores the sum to the
    // other residual buffer.  Otherwise NCCL: rank 0 adds its partial to the
    // residual, the others store theirs, then an in-place all-reduce.
    const bool ar = tp && r->ar_on;
    const int row_epi = ar ? kEpiPush : (tp && m->tp_rank != 0 ? kEpiStore : kEpiResidual);
    const int W = m->tp_world;
    float* hres[2] = {io.h, ar ? io.h2 : io.h};
    int cur = 0;  // residual buffer holding the stream
    auto ar_common = [&](GemvParams& p) {
        p.ar_world = W;
        p.ar_rank = m->tp_rank;
        p.ar_push_slot = -1;
        p.ar_pull_slot = -1;
        p.ar_peers = r->ar_peers_dev.as<unsigned long long* const>();
        p.ar_local = r->ar_buf.as<unsigned long long>();
        p.ar_slot_words = (long long)B * H;
        p.ar_step = r->ar_step.as<unsigned int>();
    };
    auto pull = [&](GemvParams& p, int slot, bool store) {
        if (!ar) return;
        ar_common(p);
        p.ar_pull_slot = slot;
        p.ar_hin = hres[cur];
        p.ar_hout = store ? hres[cur ^ 1] : nullptr;
        p.src = hres[cur];
        if (store) cur ^= 1;
    };
    auto push = [&](GemvParams& p, int slot) {
        if (!ar) return;
        ar_common(p);
        p.ar_push_slot = slot;
        p.out = nullptr;
    };
    auto push_allreduce = [&]() {
        if (!tp || ar) return;
        Launch ln{};
        ln.kind = 3;
        ln.bytes = (int64_t)B * H * 4;
        plan.push_back(ln);
    };
    plan.clear();
    for (int l = 0; l < c.num_layers; ++l) {
        Layer& Ly = m->layers[l];
        const bool has_in = Ly.in_norm_d.p != nullptr, has_post = Ly.post_norm_d.p != nullptr;
        {  // fused QKV (+ embedding gather at layer 0) + RoPE + KV append
            Launch ln{};
            ln.kind = 0;
            GemvParams& p = ln.g;
            fill_gemv_common(r, p, Ly.qkv, io);
            if (l == 0)
                p.prologue = has_in ? kProEmbedRms : kProEmbed;
            else
                p.prologue = has_in ? kProRmsNorm : kProNone;
            p.src = io.h;
            p.ld_src = H;
            p.norm_w = Ly.in_norm_d.as<float>();
            p.embedding = m->emb.as<float>();
            p.resid = io.h;
            p.epilogue = kEpiQkv;
            p.out = io.q;
            p.ld_out = qd;
            p.H = qd;
            p.Hkv = c.num_kv_heads;
            p.head_dim = d;
            p.kv_dim = kvd;
            p.rope = r->rope.as<float2>();
            p.rope_max_pos = r->max_positions;
            p.kv_pool = r->kv.as<float>();
            p.page_table = io.ptab;
            p.ptab_stride = r->ptab_stride;
            p.layer = l;
            p.num_layers = c.num_layers;
            if (l > 0) pull(p, 2 * l - 1, true);
            ln.bytes = gemv_bytes(Ly.qkv.L, B) + (int64_t)B * 2 * kvd * 4;
            plan.push_back(ln);
        }
        {  // attention
            Launch ln{};
            ln.kind = 1;
            AttnParams& a = ln.a;
            a.q = io.q;
            a.ld_q = qd;
            a.kv_pool = r->kv.as<float>();
            a.page_table = io.ptab;
            a.ptab_stride = r->ptab_stride;
            a.seq = io.seq;
            a.lens = nullptr;
            a.layer = l;
            a.num_layers = c.num_layers;
            a.H = c.num_heads;
            a.Hkv = c.num_kv_heads;
            a.d = d;
            a.M = B;
            a.nsplit = io.nsplit;
            a.out = io.ctxv;
            a.ld_out = qd;
            a.err = r->ctx->err.as<int>();
            if (r->attn_part.p && attn_flat_supported(a.H, a.Hkv, a.d, a.M) && !getenv("TB_ATTN_CLUSTER")) {
                a.part = r->attn_part.as<float>();
                a.ticket = r->attn_ticket.as<int>();
                a.chunk_pages = attn_flat_chunk_pages(a.M, a.Hkv, r->ptab_stride, r->ctx->num_sms);
                a.maxch = (r->ptab_stride + a.chunk_pages - 1) / a.chunk_pages;
                a.kv_floats = (long long)(r->kv.bytes / 4);
            }
            ln.bytes = 0;  // depends on the context length; accounted by the caller
            plan.push_back(ln);
        }
        {  // o_proj + residual
            Launch ln{};
            ln.kind = 0;
            GemvParams& p = ln.g;
            fill_gemv_common(r, p, Ly.o, io);
            p.prologue = kProNone;
            p.src = io.ctxv;
            p.ld_src = qd;
            p.epilogue = row_epi;
            p.out = io.h;
            p.ld_out = H;
            push(p, 2 * l);
            ln.bytes = gemv_bytes(Ly.o.L, B) + (int64_t)B * H * 4;
            plan.push_back(ln);
            push_allreduce();
        }
        {  // gate/up (+ post-attention RMSNorm) + SiLU*up, or toy up + GELU
            Launch ln{};
            ln.kind = 0;
            GemvParams& p = ln.g;
            fill_gemv_common(r, p, Ly.up, io);
            p.prologue = has_post ? kProRmsNorm : kProNone;
            p.src = io.h;
            p.ld_src = H;
            p.norm_w = Ly.post_norm_d.as<float>();
            p.epilogue = llama ? kEpiSiluMul : kEpiGelu;
            p.out = io.act;
            p.ld_out = c.intermediate_dim;
            pull(p, 2 * l, true);
            ln.bytes = gemv_bytes(Ly.up.L, B);
            plan.push_back(ln);
        }
        {  // down + residual
            Launch ln{};
            ln.kind = 0;
            GemvParams& p = ln.g;
            fill_gemv_common(r, p, Ly.down, io);
            p.prologue = kProNone;
            p.src = io.act;
            p.ld_src = c.intermediate_dim;
            p.epilogue = row_epi;
            p.out = io.h;
            p.ld_out = H;
            push(p, 2 * l + 1);
            ln.bytes = gemv_bytes(Ly.down.L, B) + (int64_t)B * H * 4;
            plan.push_back(ln);
            push_allreduce();
        }
    }
    if (io.head) {  // final norm + LM head + argmax + step bookkeeping
        Launch ln{};
        ln.kind = 0;
        GemvParams& p = ln.g;
        fill_gemv_common(r, p, m->out, io);
        p.prologue = m->has_final_norm ? kProRmsNorm : kProNone;
        p.src = io.h;
        p.ld_src = H;
        p.norm_w = m->final_norm.as<float>();
        if (r->sampling || r->scoring) {  // logits only; the sampler launch finishes the step
            p.epilogue = kEpiStore;
            p.out = io.logits;
            p.ld_out = c.vocab_size;
        } else {
            p.epilogue = kEpiArgmax;
            p.out = nullptr;
            p.logits = r->logits.as<float>();
            p.ticket = r->ticket.as<unsigned int>();
            p.out_tokens = r->out_tokens.as<int>();
            p.prompt = r->prompt.as<int>();
            p.prompt_stride = r->prompt_stride;
        }
        pull(p, 2 * c.num_layers - 1, false);
        ln.bytes = gemv_bytes(m->out.L, B);
        plan.push_back(ln);
    }
    if (io.head && (r->sampling || r->scoring)) {
        Launch ln{};
        ln.kind = 5;
        fill_sample(r, ln.s);
        ln.s.ar_step = ar ? r->ar_step.as<unsigned int>() : nullptr;
        ln.bytes = (int64_t)B * c.vocab_size * 4;
        plan.push_back(ln);
    }
    // Wide GEMVs (over 16 batch rows) without a tensor-parallel pull get their
    // digit operand from a wide_digits launch right before them.
    size_t need = 0;
    for (const Launch& ln : plan)
        if (ln.kind == 0 && gemv_uses_wide(ln.g.L.precision, ln.g.M) &&
            !(ln.g.ar_world > 1 && ln.g.ar_pull_slot >= 0))
            need = std::max(need, wide_digits_bytes(ln.g.L));
    if (need > 0) {
        if (r->wide_b.bytes < need) TB_CUDA(r->wide_b.alloc(need));
        if (r->wide_ex.bytes < (size_t)kMaxGemvBatch * 4) TB_CUDA(r->wide_ex.alloc((size_t)kMaxGemvBatch * 4));
        std::vector<Launch> out;
        out.reserve(plan.size() * 2);
        for (Launch ln : plan) {
            if (ln.kind == 0 && gemv_uses_wide(ln.g.L.precision, ln.g.M) &&
            !(ln.g.ar_world > 1 && ln.g.ar_pull_slot >= 0)) {
                ln.g.bimg = r->wide_b.as<uint8_t>();
                ln.g.rowex_g = r->wide_ex.as<int>();
                Launch d = ln;
                d.kind = 6;
                d.bytes = (int64_t)ln.g.M * ln.g.L.K * 4 + (int64_t)wide_digits_bytes(ln.g.L);
                out.push_back(d);
            }
            out.push_back(ln);
        }
        plan.swap(out);
    }
    return ok();
}

static tb_status build_plan(tb_runner* r) {
    PlanIO io{r->B, r->h.as<float>(), r->h2.as<float>(), r->q.as<float>(), r->ctxv.as<float>(), r->act.as<float>(),
              r->seq.as<SeqState>(), r->ptab.as<int>(), r->nsplit, true, r->logits.as<float>()};
    return build_plan_into(r, io, r->plan);
}

// One launch of the plan on `st`.
static tb_status launch_op(tb_runner* r, const Launch& ln, cudaStream_t st, bool pdl) {
    cudaError_t e;
    if (ln.kind == 3) {
        std::string why;
        e = nccl_allreduce_sum_f32(r->ctx->comm, r->h.as<float>(), (size_t)r->B * r->m->cfg.hidden_dim, st, why);
        if (e != cudaSuccess) return fail(TB_ERR_CUDA, "tensor-parallel all-reduce: %s", why.c_str());
        return ok();
    }
    if (ln.kind == 5) {
        e = launch_sample(ln.s, st, pdl);
        if (e != cudaSuccess) return cuda_fail(e, "launch_sample");
        return ok();
    }
    if (ln.kind == 6) {
        e = launch_wide_digits(ln.g, st, pdl);
        if (e != cudaSuccess) return cuda_fail(e, "launch_wide_digits");
        return ok();
    }
    e = ln.kind == 0 ? launch_gemv(ln.g, st, pdl) : launch_attention(ln.a, st, pdl);
    if (e != cudaSuccess) return cuda_fail(e, ln.kind == 0 ? "launch_gemv" : "launch_attention");
    return ok();
}

static tb_status record_plan(tb_runner* r, cudaStream_t st, bool pdl) {
    for (const Launch& ln : r->plan) {
        tb_status s = launch_op(r, ln, st, pdl);
        if (s != TB_OK) return s;
    }
    return ok();
}

// Pointers of the persistent step that change when generate() resizes buffers.
static void refresh_step_params(tb_runner* r) {
    StepParams& p = r->sp;
    p.prompt = r->prompt.as<int>();
    p.prompt_stride = r->prompt_stride;
    p.out_tokens = r->out_tokens.as<int>();
}

// Build the persistent-step parameters when the model qualifies (batch 1,
// LLaMA, one precision and shape for every layer, a supported head shape).
static tb_status build_step(tb_runner* r) {
    tb_model* m = r->m;
    const tb_model_config& c = m->cfg;
    r->persistent_ok = false;
    if (r->B != 1 || m->tp_world > 1 || c.architecture != TB_ARCH_LLAMA || c.hidden_dim > 4096 || c.intermediate_dim % 4 != 0) return ok();
    const Layer& L0 = m->layers[0];
    const int prec = L0.qkv.L.precision;
    if (prec != 8) return ok();  // INT4 decodes through the per-op tensor-core GEMVs
    auto same = [](const QLayout& a, const QLayout& b) {
        return a.precision == b.precision && a.K == b.K && a.N == b.N && a.RB == b.RB;
    };
    for (const Layer& L : m->layers)
        if (!same(L.qkv.L, L0.qkv.L) || !same(L.o.L, L0.o.L) || !same(L.up.L, L0.up.L) ||
            !same(L.down.L, L0.down.L) || L.o.L.precision != prec || L.up.L.precision != prec ||
            L.down.L.precision != prec)
            return ok();
    if (m->out.L.precision != prec) return ok();
    StepParams& p = r->sp;
    p = StepParams{};
    std::vector<StepLayer> hl(c.num_layers);
    for (int l = 0; l < c.num_layers; ++l) {
        const Layer& L = m->layers[l];
        StepLayer& s = hl[l];
        s.qkv_w = L.qkv.w.as<uint8_t>();
        s.o_w = L.o.w.as<uint8_t>();
        s.gu_w = L.up.w.as<uint8_t>();
        s.dn_w = L.down.w.as<uint8_t>();
        s.qkv_s = L.qkv.s.as<float>();
        s.o_s = L.o.s.as<float>();
        s.gu_s = L.up.s.as<float>();
        s.dn_s = L.down.s.as<float>();
        s.qkv_b = L.qkv.has_bias ? L.qkv.bias.as<float>() : nullptr;
        s.o_b = L.o.has_bias ? L.o.bias.as<float>() : nullptr;
        s.gu_b = L.up.has_bias ? L.up.bias.as<float>() : nullptr;
        s.dn_b = L.down.has_bias ? L.down.bias.as<float>() : nullptr;
        s.in_norm = L.in_norm_d.as<float>();
        s.post_norm = L.post_norm_d.as<float>();
    }
    p.num_layers = c.num_layers;
    p.Lqkv = L0.qkv.L;
    p.Lo = L0.o.L;
    p.Lgu = L0.up.L;
    p.Ldn = L0.down.L;
    p.Llm = m->out.L;
    p.lm_w = m->out.w.as<uint8_t>();
    p.lm_s = m->out.s.as<float>();
    p.lm_b = m->out.has_bias ? m->out.bias.as<float>() : nullptr;
    p.final_norm = m->has_final_norm ? m->final_norm.as<float>() : nullptr;
    p.emb = m->emb.as<float>();
    p.H = c.hidden_dim;
    p.nheads = c.num_heads;
    p.Hkv = c.num_kv_heads;
    p.d = m->head_dim;
    p.kvd = m->kv_dim;
    p.I = c.intermediate_dim;
    p.V = c.vocab_size;
    p.eps = c.rms_eps;
    p.rope = r->rope.as<float2>();
    p.rope_max_pos = r->max_positions;
    p.kv_pool = r->kv.as<float>();
    p.ptab = r->ptab.as<int>();
    p.seq = r->seq.as<SeqState>();
    p.logits = r->logits.as<float>();
    const int C = r->ctx->num_sms;
    const int G = c.num_heads / c.num_kv_heads;
    p.A = std::max(1, std::min(16, C / c.num_kv_heads));
    int max_smem = 0;
    TB_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, r->ctx->device));
    int ns = 0, sb = 0;
    size_t smem = 0;
    // INT8: the dataflow kernel (tagged words, no grid barriers) unless disabled
    const char* sel = getenv("TB_STEP_KERNEL");
    const bool try_flow = prec == 8 && !(sel && std::string(sel) == "barrier");
    if (try_flow) smem = flow_smem_bytes(p, C, &ns, &sb, max_smem - 1024);
    p.flow = smem > 0 ? 1 : 0;
    if (!p.flow) smem = step_smem_bytes(p, C, &ns, &sb, max_smem - 1024);
    if (smem == 0) return ok();
    TB_CUDA(r->step_layers.alloc(hl.size() * sizeof(StepLayer)));
    TB_CUDA(cudaMemcpy(r->step_layers.p, hl.data(), hl.size() * sizeof(StepLayer), cudaMemcpyHostToDevice));
    p.layers = r->step_layers.as<StepLayer>();
    auto part = [&](DevBuf& b, const QLayout& L) { return b.alloc((size_t)L.slabs * L.Np * 4); };
    TB_CUDA(part(r->part_qkv, p.Lqkv));
    TB_CUDA(part(r->part_o, p.Lo));
    TB_CUDA(part(r->part_gu, p.Lgu));
    TB_CUDA(part(r->part_dn, p.Ldn));
    TB_CUDA(r->step_attn.alloc((size_t)c.num_kv_heads * p.A * G * (m->head_dim + 4) * 4));
    TB_CUDA(r->hX.alloc((size_t)c.hidden_dim * 4));
    TB_CUDA(r->hY.alloc((size_t)c.hidden_dim * 4));
    TB_CUDA(r->step_bar.alloc(64));
    TB_CUDA(cudaMemset(r->step_bar.p, 0, 64));
    p.part_qkv = r->part_qkv.as<float>();
    p.part_o = r->part_o.as<float>();
    p.part_gu = r->part_gu.as<float>();
    p.part_dn = r->part_dn.as<float>();
    p.attn_part = r->step_attn.as<float>();
    p.hX = r->hX.as<float>();
    p.hY = r->hY.as<float>();
    p.bar = r->step_bar.as<unsigned int>();
    if (p.flow) {
        // tagged words start at tag 0, which no step produces
        const int H = c.hidden_dim;
        size_t off[12], total = 0;
        const size_t words[11] = {(size_t)H,
                                 (size_t)H,
                                 (size_t)C,
                                 (size_t)C,
                                 (size_t)p.Lqkv.slabs * p.Lqkv.Np,
                                 (size_t)p.Lo.slabs * p.Lo.Np,
                                 (size_t)p.Lgu.slabs * p.Lgu.Np,
                                 (size_t)p.Ldn.slabs * p.Ldn.Np,
                                 (size_t)c.num_kv_heads * p.A * G * (m->head_dim + 2),
                                 (size_t)(p.Lqkv.Np / p.Lqkv.RB) * p.Lqkv.slabs,
                                 (size_t)(p.Lgu.Np / p.Lgu.RB) * p.Lgu.slabs};
        for (int i = 0; i < 11; ++i) {
            off[i] = total;
            total += (words[i] + 1) / 2 * 2;  // 16-byte aligned sections
        }
        off[11] = total;
        TB_CUDA(r->flow_buf.alloc(total * 8 + 64));
        TB_CUDA(cudaMemset(r->flow_buf.p, 0, total * 8 + 64));
        uint64_t* b = r->flow_buf.as<uint64_t>();
        p.f_h[0] = b + off[0];
        p.f_h[1] = b + off[1];
        p.f_ss[0] = b + off[2];
        p.f_ss[1] = b + off[3];
        p.f_qkv = b + off[4];
        p.f_o = b + off[5];
        p.f_gu = b + off[6];
        p.f_dn = b + off[7];
        p.f_att = b + off[8];
        p.f_dbqkv = b + off[9];
        p.f_dbgu = b + off[10];
        p.f_epoch = reinterpret_cast<unsigned int*>(b + off[11]);
        p.f_ticket = p.f_epoch + 1;
    }
    p.err = r->ctx->err.as<int>();
    p.nslots = ns;
    p.slot_bytes = sb;
    p.nflight = std::min(ns, 4);
    if (const char* e = getenv("TB_STEP_INFLIGHT")) p.nflight = std::max(1, std::min(ns, atoi(e)));
    r->step_smem = smem;
    r->step_grid = C;
    refresh_step_params(r);
    r->persistent_ok = true;
    // The per-projection launch chain (CUDA graph + programmatic dependent
    // launch) measured faster than both persistent kernels on TinyLlama-shaped
    // batch-1 decode, so it stays the default; TB_PERSISTENT=1 flips it.
    const char* dflt = getenv("TB_PERSISTENT");
    r->persistent = dflt && std::string(dflt) == "1";
    return ok();
}

static tb_status record_step(tb_runner* r, cudaStream_t st) {
    if (r->persistent) {
        cudaError_t e = launch_decode_step(r->sp, r->step_grid, r->step_smem, st);
        if (e != cudaSuccess) return cuda_fail(e, "launch_decode_step");
        return ok();
    }
    return record_plan(r, st, true);
}

static tb_status capture_graph(tb_runner* r) {
    if (r->graph) return ok();
    cudaStream_t st = r->ctx->stream;
    cudaGraph_t g = nullptr;
    TB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    tb_status s = record_step(r, st);
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (s != TB_OK) {
        if (g) cudaGraphDestroy(g);
        return s;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&r->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    return ok();
}

extern "C" tb_status tb_runner_create(tb_model* m, int32_t max_batch, int32_t max_positions, tb_runner** out) {
    TB_CHECK(m && out, "NULL argument");
    *out = nullptr;
    TB_CHECK(m->finalized, "model not finalized");
    TB_CHECK(max_batch >= 1 && max_batch <= kMaxGemvBatch, "max_batch must be in [1, %d] (got %d)", kMaxGemvBatch,
             max_batch);
    tb_context* ctx = m->ctx;
    TB_CUDA(cudaSetDevice(ctx->device));
    const tb_model_config& c = m->cfg;
    auto r = std::make_unique<tb_runner>();
    r->m = m;
    r->ctx = ctx;
    r->B = max_batch;
    r->max_positions = std::max(max_positions, c.max_seq_len);
    r->ptab_stride = (r->max_positions + kPageTokens - 1) / kPageTokens;
    r->max_pages_per_seq = (c.max_seq_len + kPageTokens - 1) / kPageTokens;
    r->total_pages = r->max_pages_per_seq * max_batch;
    const int H = c.hidden_dim, d = m->head_dim, kvd = m->kv_dim, B = max_batch;
    const size_t page_floats = (size_t)c.num_layers * 2 * kvd * kPageTokens;
    TB_CUDA(r->seq.alloc(sizeof(SeqState) * B));
    TB_CUDA(r->ptab.alloc((size_t)B * r->ptab_stride * 4));
    TB_CUDA(r->kv.alloc((size_t)r->total_pages * page_floats * 4));
    TB_CUDA(r->h.alloc((size_t)B * H * 4));
    TB_CUDA(r->q.alloc((size_t)B * H * 4));
    TB_CUDA(r->ctxv.alloc((size_t)B * H * 4));
    TB_CUDA(r->act.alloc((size_t)B * c.intermediate_dim * 4));
    TB_CUDA(r->logits.alloc((size_t)B * c.vocab_size * 4));
    TB_CUDA(r->ticket.alloc(16));
    TB_CUDA(cudaMemset(r->ticket.p, 0, 16));
    TB_CUDA(cudaMemset(r->seq.p, 0, sizeof(SeqState) * B));
    TB_CUDA(cudaMemset(r->kv.p, 0, r->kv.bytes));
    // RoPE table with the reference's fp32 formula (ModelRunner.swift:478-486).
    {
        std::vector<float2> tab((size_t)r->max_positions * (d / 2));
        for (int pos = 0; pos < r->max_positions; ++pos)
            for (int i = 0; i < d; i += 2) {
                const float freq = (float)i / (float)d;
                const float theta = powf(10000.0f, -freq);
                const float angle = (float)pos * theta;
                tab[(size_t)pos * (d / 2) + i / 2] = make_float2(cosf(angle), sinf(angle));
            }
        TB_CUDA(r->rope.alloc(tab.size() * sizeof(float2)));
        TB_CUDA(cudaMemcpy(r->rope.p, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
    }
    // Host page bookkeeping.
    r->kvh.assign(B, SeqKV{});
    for (auto& s : r->kvh) s.map.assign(r->ptab_stride, -1);
    r->free_pages.resize(r->total_pages);
    for (int i = 0; i < r->total_pages; ++i) r->free_pages[i] = r->total_pages - 1 - i;
    r->ptab_host.assign((size_t)B * r->ptab_stride, -1);
    r->ptab_dirty.assign(B, 1);
    TB_CUDA(r->pin_ptab.ensure(r->ptab_host.size() * 4));
    TB_CUDA(r->pin_seq.ensure(sizeof(SeqState) * B));
    // Attention splits per (sequence, KV head), sized for the longest context.
    r->nsplit = choose_nsplit(B, c.num_kv_heads, r->ptab_stride, ctx->num_sms);
    {
        // chunk partials for the persistent attention: rows up to the larger
        // of the batch and the prefill chunk, chunks of at least 2 pages
        const int d = c.hidden_dim / c.num_heads;
        const int rows = std::max(B, (int)kMaxGemvBatch);  // the prefill plan has kMaxGemvBatch rows
        if (attn_flat_supported(c.num_heads, c.num_kv_heads, d, rows)) {
            const size_t pairs = (size_t)rows * c.num_kv_heads;
            const size_t maxch = (size_t)(r->ptab_stride + 1) / 2;
            TB_CUDA(r->attn_part.alloc(pairs * maxch * kAttnPartFloats * 4));
            TB_CUDA(r->attn_ticket.alloc(pairs * 4));
            TB_CUDA(cudaMemset(r->attn_ticket.p, 0, pairs * 4));
        }
    }
    tb_status s = TB_OK;
    // Prompt / output buffers start small and grow in generate.
    r->prompt_stride = 1;
    r->max_out = 1;
    TB_CUDA(r->prompt.alloc((size_t)B * 4));
    TB_CUDA(r->out_tokens.alloc((size_t)B * 4));
    TB_CUDA(r->out_prob.alloc((size_t)B * 4));
    TB_CUDA(r->out_ent.alloc((size_t)B * 4));
    TB_CUDA(r->rng.alloc((size_t)B * 8));
    TB_CUDA(cudaMemset(r->rng.p, 0, (size_t)B * 8));
    TB_CUDA(cudaEventCreate(&r->ev0));
    TB_CUDA(cudaEventCreate(&r->ev1));
    if ((s = build_plan(r.get())) != TB_OK) return s;
    if ((s = build_step(r.get())) != TB_OK) return s;
    TB_CHECK(m->tp_world == 1 || (ctx->comm && ctx->tp_world == m->tp_world), "tensor-parallel model on a context "
             "without its communicator (tb_context_init_tp)");
    if (m->tp_world > 1) {
        // One all-reduce of the step's size outside any graph capture, so the
        // communicator's connections exist before the step graph records it.
        TB_CUDA(cudaMemsetAsync(r->h.p, 0, (size_t)B * H * 4, ctx->stream));
        std::string why;
        cudaError_t e = nccl_allreduce_sum_f32(ctx->comm, r->h.as<float>(), (size_t)B * H, ctx->stream, why);
        if (e != cudaSuccess) return fail(TB_ERR_CUDA, "tensor-parallel all-reduce: %s", why.c_str());
        TB_CUDA(cudaStreamSynchronize(ctx->stream));
    }
    TB_CUDA(cudaDeviceSynchronize());
    *out = r.release();
    return ok();
}

// ---------------------------------------------------------------------------
// tensor parallel through peer memory
// ---------------------------------------------------------------------------
extern "C" tb_status tb_runner_tp_handle(tb_runner* r, uint8_t* handle) {
    TB_CHECK(r && handle, "NULL argument");
    tb_model* m = r->m;
    TB_CHECK(m->tp_world > 1, "the model is not tensor parallel");
    TB_CHECK(m->cfg.architecture == TB_ARCH_LLAMA && r->B <= 16 && m->cfg.hidden_dim % 4 == 0,
             "peer-memory all-reduce: LLaMA models, batch <= 16");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    const size_t slots = (size_t)2 * m->cfg.num_layers, W = (size_t)m->tp_world;
    const size_t bytes = slots * W * (size_t)r->B * m->cfg.hidden_dim * 8;  // tagged 64-bit words
    if (!r->ar_buf.p) {
        TB_CUDA(r->ar_buf.alloc(bytes));
        TB_CUDA(cudaMemset(r->ar_buf.p, 0, bytes));
        TB_CUDA(r->ar_step.alloc(64));
        TB_CUDA(cudaMemset(r->ar_step.p, 0, 64));
        TB_CUDA(r->h2.alloc((size_t)r->B * m->cfg.hidden_dim * 4));
    }
    cudaIpcMemHandle_t h;
    TB_CUDA(cudaIpcGetMemHandle(&h, r->ar_buf.p));
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle, &h, 64);
    return ok();
}

extern "C" tb_status tb_runner_tp_connect(tb_runner* r, const uint8_t* handles) {
    TB_CHECK(r && handles, "NULL argument");
    TB_CHECK(r->ar_buf.p, "call tb_runner_tp_handle first");
    TB_CHECK(!r->ar_on, "already connected");
    tb_model* m = r->m;
    TB_CUDA(cudaSetDevice(r->ctx->device));
    const int W = m->tp_world;
    r->ar_peer_host.assign(W, nullptr);
    for (int q = 0; q < W; ++q) {
        if (q == m->tp_rank) {
            r->ar_peer_host[q] = r->ar_buf.p;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + (size_t)q * 64, 64);
        void* ptr = nullptr;
        TB_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        r->ar_peer_host[q] = ptr;
    }
    TB_CUDA(r->ar_peers_dev.alloc((size_t)W * sizeof(void*)));
    TB_CUDA(cudaMemcpy(r->ar_peers_dev.p, r->ar_peer_host.data(), (size_t)W * sizeof(void*), cudaMemcpyHostToDevice));
    r->ar_on = true;
    tb_status s = build_plan(r);
    if (s != TB_OK) return s;
    if (r->graph) {
        cudaGraphExecDestroy(r->graph);
        r->graph = nullptr;
    }
    return ok();
}

extern "C" tb_status tb_runner_free(tb_runner* r) {
    if (r) {
        cudaSetDevice(r->ctx->device);
        cudaStreamSynchronize(r->ctx->stream);
        delete r;
    }
    return ok();
}

// KVCache.evictOldestPage (KVCache.swift:293-308): drop the lowest logical page.
static void kv_evict_oldest(tb_runner* r, int s) {
    SeqKV& k = r->kvh[s];
    for (size_t i = 0; i < k.map.size(); ++i)
        if (k.map[i] >= 0) {
            r->free_pages.push_back(k.map[i]);
            k.map[i] = -1;
            k.pages_held -= 1;
            r->ptab_host[(size_t)s * r->ptab_stride + i] = -1;
            r->ptab_dirty[s] = 1;
            return;
        }
}

// KVCache.append (KVCache.swift:157-224) bookkeeping for sequence s at its
// current position: eviction, page allocation (zero-filled), length update.
static tb_status kv_prepare(tb_runner* r, int s) {
    SeqKV& k = r->kvh[s];
    const int64_t maxTokens = r->m->cfg.max_seq_len;
    const int64_t pos = k.pos;
    if (pos >= r->max_positions)
        return fail(TB_ERR_INVALID_ARGUMENT, "position %lld exceeds the runner's max_positions %d", (long long)pos,
                    r->max_positions);
    while (k.length >= maxTokens) {
        kv_evict_oldest(r, s);
        k.length = std::max<int64_t>(0, k.length - kPageTokens);
    }
    const int64_t lp = pos / kPageTokens;
    if (k.map[lp] < 0) {
        if (k.pages_held >= r->max_pages_per_seq) kv_evict_oldest(r, s);
        if (r->free_pages.empty() || k.pages_held >= r->max_pages_per_seq)
            return fail(TB_ERR_PAGE_POOL_EXHAUSTED, "no free KV page for sequence %d", s);
        const int pg = r->free_pages.back();
        r->free_pages.pop_back();
        k.map[lp] = pg;
        k.pages_held += 1;
        r->ptab_host[(size_t)s * r->ptab_stride + lp] = pg;
        r->ptab_dirty[s] = 1;
        const tb_model_config& c = r->m->cfg;
        const size_t page_bytes = (size_t)c.num_layers * 2 * r->m->kv_dim * kPageTokens * 4;
        TB_CUDA(cudaMemsetAsync(r->kv.as<uint8_t>() + (size_t)pg * page_bytes, 0, page_bytes, r->ctx->stream));
    }
    k.length = std::max<int64_t>(k.length, pos + 1);
    if (k.length > maxTokens) k.length = maxTokens;
    return ok();
}

static tb_status flush_ptab(tb_runner* r) {
    if (r->ptab_ev.size() != (size_t)r->B) r->ptab_ev.assign(r->B, nullptr);
    for (int s = 0; s < r->B; ++s) {
        if (!r->ptab_dirty[s]) continue;
        int* pin = r->pin_ptab.as<int>() + (size_t)s * r->ptab_stride;
        // The previous upload from this staging row may still be queued behind
        // earlier steps: wait for it before overwriting the row, or an older
        // step would read a newer table (with pages evicted after it).
        if (r->ptab_ev[s]) TB_CUDA(cudaEventSynchronize(r->ptab_ev[s]));
        memcpy(pin, r->ptab_host.data() + (size_t)s * r->ptab_stride, (size_t)r->ptab_stride * 4);
        TB_CUDA(cudaMemcpyAsync(r->ptab.as<int>() + (size_t)s * r->ptab_stride, pin, (size_t)r->ptab_stride * 4,
                                cudaMemcpyHostToDevice, r->ctx->stream));
        if (!r->ptab_ev[s]) TB_CUDA(cudaEventCreateWithFlags(&r->ptab_ev[s], cudaEventDisableTiming));
        TB_CUDA(cudaEventRecord(r->ptab_ev[s], r->ctx->stream));
        r->h2d_bytes += (int64_t)r->ptab_stride * 4;
        r->ptab_dirty[s] = 0;
    }
    return ok();
}

static void kv_clear(tb_runner* r, int s) {
    SeqKV& k = r->kvh[s];
    for (size_t i = 0; i < k.map.size(); ++i)
        if (k.map[i] >= 0) {
            r->free_pages.push_back(k.map[i]);
            k.map[i] = -1;
            r->ptab_host[(size_t)s * r->ptab_stride + i] = -1;
        }
    k.pages_held = 0;
    k.length = 0;
    k.pos = 0;
    r->ptab_dirty[s] = 1;
}

extern "C" tb_status tb_runner_reset(tb_runner* r) {
    TB_CHECK(r, "NULL runner");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    for (int s = 0; s < r->B; ++s) kv_clear(r, s);
    // Restore the canonical LIFO order (PageAllocator.reset, PageAllocator.swift:131-137).
    r->free_pages.resize(r->total_pages);
    for (int i = 0; i < r->total_pages; ++i) r->free_pages[i] = r->total_pages - 1 - i;
    TB_CUDA(cudaMemsetAsync(r->seq.p, 0, sizeof(SeqState) * r->B, r->ctx->stream));
    return flush_ptab(r);
}

extern "C" tb_status tb_runner_position(const tb_runner* r, int32_t seq, int64_t* pos) {
    TB_CHECK(r && pos && seq >= 0 && seq < r->B, "bad argument");
    *pos = r->kvh[seq].pos;
    return ok();
}
extern "C" tb_status tb_runner_kv_length(const tb_runner* r, int32_t seq, int64_t* len) {
    TB_CHECK(r && len && seq >= 0 && seq < r->B, "bad argument");
    *len = r->kvh[seq].length;
    return ok();
}
extern "C" tb_status tb_runner_max_pages(const tb_runner* r, int64_t* n) {
    TB_CHECK(r && n, "bad argument");
    *n = r->max_pages_per_seq;
    return ok();
}
extern "C" tb_status tb_runner_page_status(const tb_runner* r, int32_t seq, uint8_t* status, int64_t n) {
    TB_CHECK(r && status && seq >= 0 && seq < r->B, "bad argument");
    for (int64_t i = 0; i < n; ++i)
        status[i] = (i < (int64_t)r->kvh[seq].map.size() && r->kvh[seq].map[i] >= 0) ? 1 : 0;
    return ok();
}

// Write the device SeqState array from the host values in pin_seq.
static tb_status push_seq(tb_runner* r) {
    TB_CUDA(cudaMemcpyAsync(r->seq.p, r->pin_seq.p, sizeof(SeqState) * r->B, cudaMemcpyHostToDevice,
                            r->ctx->stream));
    r->h2d_bytes += (int64_t)sizeof(SeqState) * r->B;
    return ok();
}

// Every sequence's LCG starts from the configured seed (a generate call copies
// the SamplerConfig, ModelRunner.swift:233); without one, from a host draw.
static tb_status seed_sampler(tb_runner* r) {
    uint64_t seed = r->scfg.seed;
    if (!r->scfg.has_seed) {
        std::random_device rd;
        seed = ((uint64_t)rd() << 32) ^ (uint64_t)rd();
    }
    std::vector<uint64_t> v((size_t)r->B, seed);
    TB_CUDA(cudaMemcpy(r->rng.p, v.data(), v.size() * 8, cudaMemcpyHostToDevice));
    r->h2d_bytes += (int64_t)v.size() * 8;
    return ok();
}

// Grow the prompt / output buffers to maxp prompt tokens and mo outputs per
// sequence and point the plan's (and the persistent step's) launches at them.
static tb_status ensure_io(tb_runner* r, int maxp, int mo) {
    // (Re)size prompt/output buffers.
    if (maxp > r->prompt_stride || r->B * (size_t)maxp * 4 > r->prompt.bytes) {
        r->prompt_stride = maxp;
        TB_CUDA(r->prompt.alloc((size_t)r->B * maxp * 4));
    }
    if (mo > r->max_out) {
        r->max_out = mo;
        TB_CUDA(r->out_tokens.alloc((size_t)r->B * mo * 4));
        TB_CUDA(r->out_prob.alloc((size_t)r->B * mo * 4));
        TB_CUDA(r->out_ent.alloc((size_t)r->B * mo * 4));
        for (Launch& ln : r->plan)
            if (ln.kind == 0 && ln.g.epilogue == kEpiArgmax) {
                ln.g.out_tokens = r->out_tokens.as<int>();
            }
        if (r->graph) {
            cudaGraphExecDestroy(r->graph);
            r->graph = nullptr;
        }
    }
    for (Launch& ln : r->plan)
        if (ln.kind == 0 && ln.g.epilogue == kEpiArgmax && (ln.g.prompt != r->prompt.as<int>() ||
                                                            ln.g.prompt_stride != r->prompt_stride)) {
            ln.g.prompt = r->prompt.as<int>();
            ln.g.prompt_stride = r->prompt_stride;
            if (r->graph) {
                cudaGraphExecDestroy(r->graph);
                r->graph = nullptr;
            }
        }
    for (Launch& ln : r->plan)
        if (ln.kind == 5) {
            SampleParams f = ln.s;
            fill_sample(r, f);
            if (f.prompt != ln.s.prompt || f.prompt_stride != ln.s.prompt_stride || f.out_tokens != ln.s.out_tokens ||
                f.out_prob != ln.s.out_prob || f.out_entropy != ln.s.out_entropy) {
                f.ar_step = ln.s.ar_step;
                ln.s = f;
                if (r->graph) {
                    cudaGraphExecDestroy(r->graph);
                    r->graph = nullptr;
                }
            }
        }
    if (r->persistent_ok &&
        (r->sp.prompt != r->prompt.as<int>() || r->sp.prompt_stride != r->prompt_stride ||
         r->sp.out_tokens != r->out_tokens.as<int>())) {
        refresh_step_params(r);
        if (r->persistent && r->graph) {
            cudaGraphExecDestroy(r->graph);
            r->graph = nullptr;
        }
    }
    return ok();
}

// A single step (tb_runner_step / _observed) with a sampler draws from its
// logits: the history of tb_runner_set_step_history stands in as the
// sequence's prompt (at most pos + 1 tokens, so the step is a generation
// step) and output slot 0 receives the draw.
static tb_status step_sampler_state(tb_runner* r, SeqState* st) {
    if (!r->sampling) return ok();
    const int n = (int)r->step_hist.size();
    TB_CHECK(n <= st->pos + 1, "step history holds %d tokens; at most position + 1 = %d", n, st->pos + 1);
    tb_status e = ensure_io(r, std::max(1, n), 1);
    if (e != TB_OK) return e;
    if (n > 0) {
        TB_CUDA(cudaMemcpy(r->prompt.p, r->step_hist.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
        r->h2d_bytes += (int64_t)n * 4;
    }
    st->n_prompt = n;
    st->n_out = 0;
    st->max_out = 1;
    return ok();
}

// Probability and entropy of a single step's draw (read after the step).
static tb_status step_sampler_stats(tb_runner* r) {
    if (!r->sampling) return ok();
    TB_CUDA(cudaMemcpyAsync(&r->last_prob, r->out_prob.p, 4, cudaMemcpyDeviceToHost, r->ctx->stream));
    TB_CUDA(cudaMemcpyAsync(&r->last_ent, r->out_ent.p, 4, cudaMemcpyDeviceToHost, r->ctx->stream));
    return ok();
}

static tb_status launch_step(tb_runner* r) {
    tb_status s = capture_graph(r);
    if (s != TB_OK) return s;
    TB_CUDA(cudaGraphLaunch(r->graph, r->ctx->stream));
    return ok();
}

extern "C" tb_status tb_runner_step(tb_runner* r, int32_t token, float* logits, int32_t* argmax_out) {
    TB_CHECK(r, "NULL runner");
    TB_CHECK(r->B == 1, "tb_runner_step drives batch-1 runners; use tb_runner_generate for batches");
    const int V = r->m->cfg.vocab_size;
    TB_CHECK(token >= 0 && token < V, "token %d outside [0, %d)", token, V);
    TB_CUDA(cudaSetDevice(r->ctx->device));
    tb_status s = kv_prepare(r, 0);
    if (s != TB_OK) return s;
    if ((s = flush_ptab(r)) != TB_OK) return s;
    SeqState* st = r->pin_seq.as<SeqState>();
    memset(st, 0, sizeof(SeqState));
    st->pos = (int)r->kvh[0].pos;
    st->token = token;
    st->n_prompt = 0;
    st->n_out = 0;
    st->max_out = 0;
    st->active = 1;
    st->best = 0;
    if ((s = step_sampler_state(r, st)) != TB_OK) return s;
    if ((s = push_seq(r)) != TB_OK) return s;
    if ((s = launch_step(r)) != TB_OK) return s;
    TB_CUDA(cudaMemcpyAsync(r->pin_seq.p, r->seq.p, sizeof(SeqState), cudaMemcpyDeviceToHost, r->ctx->stream));
    if (logits)
        TB_CUDA(cudaMemcpyAsync(logits, r->logits.p, (size_t)V * 4, cudaMemcpyDeviceToHost, r->ctx->stream));
    if ((s = step_sampler_stats(r)) != TB_OK) return s;
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    r->kvh[0].pos += 1;
    if (argmax_out) *argmax_out = r->pin_seq.as<SeqState>()->token;
    return tb_context_check_device(r->ctx);
}

// ModelRunner.step with the InferenceObserver hooks (InferenceObserver.swift:40-84,
// ModelRunner.swift:195-202, 395-399, 582-586): the per-projection plan runs
// launch by launch with three observer kernels in between -- the L2 norm of h
// after each layer's QKV launch (h at layer entry; layer 0's embedding row is
// gathered by that launch), the softmax weights after each attention launch,
// and RMSNorm(h) * w before the LM head.  Batch-1 runners, sequence 0.
extern "C" tb_status tb_runner_step_observed(tb_runner* r, int32_t token, float* logits, int32_t* argmax_out,
                                             float* layer_norms, float* attn_weights, int64_t attn_stride,
                                             float* final_hidden) {
    TB_CHECK(r, "NULL runner");
    if (r->m->tp_world > 1) return fail(TB_ERR_UNSUPPORTED, "observer hooks need the whole model on one GPU");
    TB_CHECK(r->B == 1, "tb_runner_step_observed drives batch-1 runners");
    tb_model* m = r->m;
    const tb_model_config& c = m->cfg;
    const int V = c.vocab_size, H = c.hidden_dim, NL = c.num_layers;
    TB_CHECK(token >= 0 && token < V, "token %d outside [0, %d)", token, V);
    const int64_t Lc = r->kvh[0].pos + 1;
    TB_CHECK(!attn_weights || attn_stride >= (int64_t)c.num_heads * Lc, "attn_stride %lld < num_heads * L = %lld",
             (long long)attn_stride, (long long)(c.num_heads * Lc));
    const size_t lm = (size_t)(5 * NL);  // the LM-head launch; the sampler (if set) follows it
    TB_CHECK(r->plan.size() == lm + (r->sampling ? 2 : 1), "observer needs the per-projection plan");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    tb_status s = kv_prepare(r, 0);
    if (s != TB_OK) return s;
    if ((s = flush_ptab(r)) != TB_OK) return s;
    SeqState* st = r->pin_seq.as<SeqState>();
    memset(st, 0, sizeof(SeqState));
    st->pos = (int)r->kvh[0].pos;
    st->token = token;
    st->active = 1;
    if ((s = step_sampler_state(r, st)) != TB_OK) return s;
    if ((s = push_seq(r)) != TB_OK) return s;
    const size_t probs_floats = (size_t)NL * c.num_heads * Lc;
    if (r->obs_buf.bytes < (probs_floats + NL + H) * 4) TB_CUDA(r->obs_buf.alloc((probs_floats + NL + H) * 4));
    float* d_probs = r->obs_buf.as<float>();
    float* d_norms = d_probs + probs_floats;
    float* d_final = d_norms + NL;
    cudaStream_t sm = r->ctx->stream;
    for (size_t i = 0; i < r->plan.size(); ++i) {
        const Launch& ln = r->plan[i];
        const int l = (int)(i / 5);
        if (i == lm) {
            cudaError_t e = launch_rmsnorm_rows(r->h.as<float>(), m->has_final_norm ? m->final_norm.as<float>() : nullptr,
                                                H, H, 1, c.rms_eps, d_final, sm);
            if (e != cudaSuccess) return cuda_fail(e, "launch_rmsnorm_rows");
        }
        tb_status ls = launch_op(r, ln, sm, false);
        if (ls != TB_OK) return ls;
        cudaError_t e = cudaSuccess;
        if (i < lm && i % 5 == 0) e = launch_row_norm(r->h.as<float>(), H, H, 1, d_norms + l, sm);
        if (i < lm && i % 5 == 1)
            e = launch_attention_probs(ln.a, d_probs + (size_t)l * c.num_heads * Lc, (int)Lc, sm);
        if (e != cudaSuccess) return cuda_fail(e, "observer kernel");
    }
    TB_CUDA(cudaMemcpyAsync(r->pin_seq.p, r->seq.p, sizeof(SeqState), cudaMemcpyDeviceToHost, sm));
    if (logits) TB_CUDA(cudaMemcpyAsync(logits, r->logits.p, (size_t)V * 4, cudaMemcpyDeviceToHost, sm));
    if (layer_norms) TB_CUDA(cudaMemcpyAsync(layer_norms, d_norms, (size_t)NL * 4, cudaMemcpyDeviceToHost, sm));
    if (final_hidden) TB_CUDA(cudaMemcpyAsync(final_hidden, d_final, (size_t)H * 4, cudaMemcpyDeviceToHost, sm));
    if (attn_weights)
        for (int l = 0; l < NL; ++l)
            TB_CUDA(cudaMemcpyAsync(attn_weights + (size_t)l * attn_stride, d_probs + (size_t)l * c.num_heads * Lc,
                                    (size_t)c.num_heads * Lc * 4, cudaMemcpyDeviceToHost, sm));
    if ((s = step_sampler_stats(r)) != TB_OK) return s;
    TB_CUDA(cudaStreamSynchronize(sm));
    r->kvh[0].pos += 1;
    if (argmax_out) *argmax_out = r->pin_seq.as<SeqState>()->token;
    return tb_context_check_device(r->ctx);
}

// Generation state kept between the split timing entry points.
namespace {
struct GenPlan {
    std::vector<int> n_prompt;
    int n_seqs = 0;
    int max_new = 0;
};
}  // namespace

static tb_status gen_setup(tb_runner* r, const int32_t* prompts, const int64_t* offs, int32_t n_seqs,
                           int32_t max_new, GenPlan& gp) {
    TB_CHECK(prompts || n_seqs == 0 || (offs && offs[n_seqs] == offs[0]), "prompts is NULL");
    TB_CHECK(offs, "prompt_offsets is NULL");
    TB_CHECK(n_seqs >= 1 && n_seqs <= r->B, "n_seqs must be in [1, %d]", r->B);
    TB_CHECK(max_new >= 0, "max_new_tokens must be >= 0");
    const int V = r->m->cfg.vocab_size;
    gp.n_seqs = n_seqs;
    gp.max_new = max_new;
    gp.n_prompt.assign(r->B, 0);
    int maxp = 1;
    for (int s = 0; s < n_seqs; ++s) {
        const int64_t n = offs[s + 1] - offs[s];
        TB_CHECK(n >= 0, "prompt offsets must be non-decreasing");
        gp.n_prompt[s] = (int)n;
        maxp = std::max<int>(maxp, (int)n);
    }
    const int mo = std::max(1, max_new);
    tb_status ie = ensure_io(r, maxp, mo);
    if (ie != TB_OK) return ie;
    if (r->sampling) {
        tb_status e = seed_sampler(r);
        if (e != TB_OK) return e;
    }
    TB_CUDA(r->pin_tokens.ensure((size_t)r->B * std::max(maxp, mo) * 4 + 64));
    int* pin = r->pin_tokens.as<int>();
    memset(pin, 0, (size_t)r->B * r->prompt_stride * 4);
    for (int s = 0; s < n_seqs; ++s)
        for (int i = 0; i < gp.n_prompt[s]; ++i) {
            int t = prompts[offs[s] + i];
            pin[(size_t)s * r->prompt_stride + i] = std::max(0, std::min(t, V - 1));  // ModelRunner.swift:236
        }
    TB_CUDA(cudaMemcpyAsync(r->prompt.p, pin, (size_t)r->B * r->prompt_stride * 4, cudaMemcpyHostToDevice,
                            r->ctx->stream));
    r->h2d_bytes += (int64_t)r->B * r->prompt_stride * 4;
    // Fresh sequences (generateStream on a reset runner).
    for (int s = 0; s < r->B; ++s) kv_clear(r, s);
    SeqState* st = r->pin_seq.as<SeqState>();
    memset(st, 0, sizeof(SeqState) * r->B);
    for (int s = 0; s < n_seqs; ++s) {
        st[s].pos = 0;
        st[s].token = gp.n_prompt[s] > 0 ? pin[(size_t)s * r->prompt_stride] : 0;
        st[s].n_prompt = gp.n_prompt[s];
        st[s].n_out = 0;
        st[s].max_out = mo;
        st[s].active = 1;
        st[s].best = 0;
    }
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    return ok();
}

// Run `steps` graph replays with host-side page bookkeeping.  `active[s]`
// says which sequences advance in every one of these steps.
static tb_status run_steps(tb_runner* r, int steps, const std::vector<char>& active) {
    for (int t = 0; t < steps; ++t) {
        for (int s = 0; s < r->B; ++s)
            if (active[s]) {
                tb_status e = kv_prepare(r, s);
                if (e != TB_OK) return e;
            }
        tb_status e = flush_ptab(r);
        if (e != TB_OK) return e;
        if ((e = launch_step(r)) != TB_OK) return e;
        for (int s = 0; s < r->B; ++s)
            if (active[s]) r->kvh[s].pos += 1;
    }
    return ok();
}

// Chunked prefill.  The reference steps every prompt token but the last one
// at a time (ModelRunner.swift:240-244); here up to kPrefillRows prompt
// tokens -- of one sequence or of several -- are the rows of one pass of the
// layers: each row carries its own position and a copy of its sequence's page
// table, so the QKV launch appends every row's K/V (RoPE at the row's
// position) and the attention launch lets row i attend over positions
// 0..pos_i, which includes the rows before it in the same chunk.  The weights
// stream once per chunk instead of once per token.  The logits of prompt
// steps are discarded by the reference, so the plan stops after the last layer.
constexpr int kPrefillRows = kMaxGemvBatch;

static tb_status pf_setup(tb_runner* r) {
    if (r->pf_ready) return ok();
    tb_model* m = r->m;
    const tb_model_config& c = m->cfg;
    const int C = kPrefillRows;
    const int wq = std::max(c.hidden_dim, m->q_dim);
    TB_CUDA(r->pf_h.alloc((size_t)C * c.hidden_dim * 4));
    TB_CUDA(r->pf_q.alloc((size_t)C * wq * 4));
    TB_CUDA(r->pf_ctx.alloc((size_t)C * wq * 4));
    TB_CUDA(r->pf_act.alloc((size_t)C * c.intermediate_dim * 4));
    TB_CUDA(r->pf_seq.alloc((size_t)C * sizeof(SeqState)));
    TB_CUDA(r->pf_ptab.alloc((size_t)C * r->ptab_stride * 4));
    // chunks of 64 rows: one split per (row, KV head) pair unless the SMs
    // would idle (rows of one chunk share their pages, and at short context
    // extra splits are empty)
    r->pf_nsplit = choose_nsplit(C, c.num_kv_heads, r->ptab_stride, r->ctx->num_sms, false);
    PlanIO io{C, r->pf_h.as<float>(), r->pf_h.as<float>(), r->pf_q.as<float>(), r->pf_ctx.as<float>(),
              r->pf_act.as<float>(), r->pf_seq.as<SeqState>(), r->pf_ptab.as<int>(), r->pf_nsplit, false, nullptr};
    tb_status e = build_plan_into(r, io, r->pf_plan);
    if (e != TB_OK) return e;
    for (Launch& ln : r->pf_plan)
        if (ln.kind == 1) ln.a.wait_first = 1;  // the chunk's QKV launch wrote any of the row's pages
    // staging slot: SeqState rows, page-table rows, scoring targets
    const size_t slot = (size_t)C * sizeof(SeqState) + (size_t)C * r->ptab_stride * 4 + (size_t)C * 4;
    for (int i = 0; i < 2; ++i) {
        TB_CUDA(r->pf_pin[i].ensure(slot));
        TB_CUDA(cudaEventCreateWithFlags(&r->pf_ev[i], cudaEventDisableTiming));
    }
    cudaStream_t st = r->ctx->stream;
    cudaGraph_t g = nullptr;
    TB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    for (const Launch& ln : r->pf_plan) {
        e = launch_op(r, ln, st, true);
        if (e != TB_OK) break;
    }
    cudaError_t ce = cudaStreamEndCapture(st, &g);
    if (e != TB_OK) {
        if (g) cudaGraphDestroy(g);
        return e;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture (prefill)");
    ce = cudaGraphInstantiate(&r->pf_graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate (prefill)");
    r->pf_ready = true;
    return ok();
}

// Chunked scoring (tb_runner_perplexity): the prefill plan with the LM head and
// the scoring launch; every row writes log P(its target) to ps_lp[row].
static tb_status ps_setup(tb_runner* r) {
    tb_status e = pf_setup(r);
    if (e != TB_OK || r->ps_graph) return e;
    const int C = kPrefillRows, V = r->m->cfg.vocab_size;
    TB_CUDA(r->ps_logits.alloc((size_t)C * V * 4));
    TB_CUDA(r->ps_lp.alloc((size_t)C * 8));
    TB_CUDA(r->ps_target.alloc((size_t)C * 4));
    PlanIO io{C, r->pf_h.as<float>(), r->pf_h.as<float>(), r->pf_q.as<float>(), r->pf_ctx.as<float>(),
              r->pf_act.as<float>(), r->pf_seq.as<SeqState>(), r->pf_ptab.as<int>(), r->pf_nsplit, true,
              r->ps_logits.as<float>()};
    const bool scoring = r->scoring;
    r->scoring = true;  // LM head stores logits; the sampler launch follows
    e = build_plan_into(r, io, r->ps_plan);
    r->scoring = scoring;
    if (e != TB_OK) return e;
    for (Launch& ln : r->ps_plan) {
        if (ln.kind == 1) ln.a.wait_first = 1;
        if (ln.kind == 5) {
            SampleParams& sp = ln.s;
            sp.logits = r->ps_logits.as<float>();
            // rows are prompt steps only: the scoring branch reads the logits
            // directly and never touches a working row, so any buffer serves
            sp.work = r->ps_logits.as<float>();
            sp.M = C;
            sp.seq = r->pf_seq.as<SeqState>();
            sp.logprob_acc = nullptr;
            sp.logprob_out = r->ps_lp.as<double>();
            sp.target = r->ps_target.as<int>();
            sp.ar_step = nullptr;
        }
    }
    cudaStream_t st = r->ctx->stream;
    cudaGraph_t g = nullptr;
    TB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    for (const Launch& ln : r->ps_plan) {
        e = launch_op(r, ln, st, true);
        if (e != TB_OK) break;
    }
    cudaError_t ce = cudaStreamEndCapture(st, &g);
    if (e != TB_OK) {
        if (g) cudaGraphDestroy(g);
        return e;
    }
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture (scoring)");
    ce = cudaGraphInstantiate(&r->ps_graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate (scoring)");
    return ok();
}

// Teacher-forced scoring of the slices in chunks of kPrefillRows positions:
// lp[i] = log P(slice token i + 1 | tokens 0..i) for every (slice, position) in
// slice order.  Slices must fit the cache without eviction.
static tb_status score_chunked(tb_runner* r, const int32_t* tokens, const int64_t* offs, int32_t n_seqs,
                               std::vector<double>& lp) {
    tb_status e = ps_setup(r);
    if (e != TB_OK) return e;
    const int C = kPrefillRows, stride = r->ptab_stride;
    for (int s = 0; s < r->B; ++s) kv_clear(r, s);
    std::vector<int> rows_s, rows_p;
    for (int s = 0; s < n_seqs; ++s)
        for (int p = 0; p + 1 < (int)(offs[s + 1] - offs[s]); ++p) {
            rows_s.push_back(s);
            rows_p.push_back(p);
        }
    const int n = (int)rows_s.size();
    lp.assign(n, 0.0);
    PinnedBuf out;
    TB_CUDA(out.ensure((size_t)std::max(1, n) * 8));
    for (int c0 = 0, slot = 0; c0 < n; c0 += C, slot ^= 1) {
        const int rows = std::min(C, n - c0);
        for (int i = 0; i < rows; ++i) {
            const int s = rows_s[c0 + i];
            if ((e = kv_prepare(r, s)) != TB_OK) return e;
            r->kvh[s].pos += 1;
        }
        TB_CUDA(cudaEventSynchronize(r->pf_ev[slot]));
        SeqState* st = r->pf_pin[slot].as<SeqState>();
        int* pt = reinterpret_cast<int*>(st + C);
        int* tg = pt + (size_t)C * stride;
        memset(st, 0, sizeof(SeqState) * C);
        for (int i = 0; i < rows; ++i) {
            const int s = rows_s[c0 + i], p = rows_p[c0 + i];
            st[i].pos = p;
            st[i].token = tokens[offs[s] + p];
            st[i].n_prompt = p + 2;  // a prompt step: scored, never sampled
            st[i].active = 1;
            tg[i] = tokens[offs[s] + p + 1];
            memcpy(pt + (size_t)i * stride, r->ptab_host.data() + (size_t)s * stride, (size_t)stride * 4);
        }
        cudaStream_t sm = r->ctx->stream;
        TB_CUDA(cudaMemcpyAsync(r->pf_seq.p, st, sizeof(SeqState) * C, cudaMemcpyHostToDevice, sm));
        TB_CUDA(cudaMemcpyAsync(r->pf_ptab.p, pt, (size_t)rows * stride * 4, cudaMemcpyHostToDevice, sm));
        TB_CUDA(cudaMemcpyAsync(r->ps_target.p, tg, (size_t)C * 4, cudaMemcpyHostToDevice, sm));
        r->h2d_bytes += (int64_t)sizeof(SeqState) * C + (int64_t)rows * stride * 4 + (int64_t)C * 4;
        TB_CUDA(cudaEventRecord(r->pf_ev[slot], sm));
        TB_CUDA(cudaGraphLaunch(r->ps_graph, sm));
        TB_CUDA(cudaMemcpyAsync(out.as<double>() + c0, r->ps_lp.p, (size_t)rows * 8, cudaMemcpyDeviceToHost, sm));
        r->d2h_bytes += (int64_t)rows * 8;
    }
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    memcpy(lp.data(), out.p, (size_t)n * 8);
    return ok();
}

// Whether every prompt's prefill fits the cache without eviction (eviction
// reorders a sequence's pages mid-prompt; such prompts prefill token by token).
static bool pf_eligible(tb_runner* r, const GenPlan& gp) {
    if (!r->pf_enabled || r->m->tp_world > 1 || r->scoring) return false;
    const int64_t cap = std::min<int64_t>(r->m->cfg.max_seq_len, (int64_t)r->max_pages_per_seq * kPageTokens);
    int total = 0;
    for (int s = 0; s < gp.n_seqs; ++s) {
        if (gp.n_prompt[s] - 1 > cap || gp.n_prompt[s] - 1 > r->max_positions) return false;
        total += std::max(0, gp.n_prompt[s] - 1);
    }
    return total >= 2;  // one token: the per-token plan is as good
}

static tb_status gen_prefill_chunked(tb_runner* r, const GenPlan& gp) {
    tb_status e = pf_setup(r);
    if (e != TB_OK) return e;
    const int C = kPrefillRows, stride = r->ptab_stride;
    const int* prompt = r->pin_tokens.as<int>();  // host copy of the clamped prompts, [B][prompt_stride]
    std::vector<int> rows_s, rows_p;               // (sequence, position) of every prefill token
    for (int s = 0; s < gp.n_seqs; ++s)
        for (int p = 0; p < gp.n_prompt[s] - 1; ++p) {
            rows_s.push_back(s);
            rows_p.push_back(p);
        }
    const int n = (int)rows_s.size();
    for (int c0 = 0, slot = 0; c0 < n; c0 += C, slot ^= 1) {
        const int rows = std::min(C, n - c0);
        // pages for every position of the chunk, in order
        for (int i = 0; i < rows; ++i) {
            const int s = rows_s[c0 + i];
            if (r->kvh[s].pos != rows_p[c0 + i]) return fail(TB_ERR_INVALID_ARGUMENT, "prefill row out of order");
            if ((e = kv_prepare(r, s)) != TB_OK) return e;
            r->kvh[s].pos += 1;
        }
        TB_CUDA(cudaEventSynchronize(r->pf_ev[slot]));  // the slot's previous upload has been consumed
        SeqState* st = r->pf_pin[slot].as<SeqState>();
        int* pt = reinterpret_cast<int*>(st + C);
        memset(st, 0, sizeof(SeqState) * C);
        for (int i = 0; i < rows; ++i) {
            const int s = rows_s[c0 + i], p = rows_p[c0 + i];
            st[i].pos = p;
            st[i].token = prompt[(size_t)s * r->prompt_stride + p];
            st[i].active = 1;
            memcpy(pt + (size_t)i * stride, r->ptab_host.data() + (size_t)s * stride, (size_t)stride * 4);
        }
        TB_CUDA(cudaMemcpyAsync(r->pf_seq.p, st, sizeof(SeqState) * C, cudaMemcpyHostToDevice, r->ctx->stream));
        TB_CUDA(cudaMemcpyAsync(r->pf_ptab.p, pt, (size_t)rows * stride * 4, cudaMemcpyHostToDevice,
                                r->ctx->stream));
        r->h2d_bytes += (int64_t)sizeof(SeqState) * C + (int64_t)rows * stride * 4;
        TB_CUDA(cudaEventRecord(r->pf_ev[slot], r->ctx->stream));
        TB_CUDA(cudaGraphLaunch(r->pf_graph, r->ctx->stream));
    }
    // the decode loop starts at the last prompt token of every sequence
    SeqState* sq = r->pin_seq.as<SeqState>();
    for (int s = 0; s < gp.n_seqs; ++s) {
        if (gp.n_prompt[s] <= 1) continue;
        sq[s].pos = gp.n_prompt[s] - 1;
        sq[s].token = prompt[(size_t)s * r->prompt_stride + gp.n_prompt[s] - 1];
    }
    return push_seq(r);
}

// Prefill: each sequence steps all but the last prompt token
// (ModelRunner.swift:240-244).  Sequences with shorter prompts wait (inactive)
// until every prompt is consumed, so the decode loop runs the whole batch.
static tb_status gen_prefill(tb_runner* r, const GenPlan& gp) {
    SeqState* st = r->pin_seq.as<SeqState>();
    int maxpre = 0;
    for (int s = 0; s < gp.n_seqs; ++s) maxpre = std::max(maxpre, gp.n_prompt[s] - 1);
    for (int t = 0; t < maxpre; ++t) {
        // Activity changes only at prompt boundaries; push the flags when they do.
        bool changed = (t == 0);
        std::vector<char> act(r->B, 0);
        for (int s = 0; s < gp.n_seqs; ++s) {
            act[s] = (t < gp.n_prompt[s] - 1) ? 1 : 0;
            if (t > 0 && (t < gp.n_prompt[s] - 1) != (t - 1 < gp.n_prompt[s] - 1)) changed = true;
        }
        if (changed) {
            // The device state of paused sequences is preserved; only `active` changes.
            TB_CUDA(cudaMemcpyAsync(r->pin_seq.p, r->seq.p, sizeof(SeqState) * r->B, cudaMemcpyDeviceToHost,
                                    r->ctx->stream));
            TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
            if (t == 0) {
                // first prefill step: the host-written initial state is authoritative
            }
            for (int s = 0; s < r->B; ++s) st[s].active = act[s];
            tb_status e = push_seq(r);
            if (e != TB_OK) return e;
        }
        tb_status e = run_steps(r, 1, act);
        if (e != TB_OK) return e;
    }
    return ok();
}

static tb_status gen_begin(tb_runner* r, const GenPlan& gp) {
    // Push the initial state, then prefill.
    tb_status e = push_seq(r);
    if (e != TB_OK) return e;
    if (pf_eligible(r, gp)) return gen_prefill_chunked(r, gp);
    return gen_prefill(r, gp);
}

static tb_status gen_activate_all(tb_runner* r, const GenPlan& gp) {
    SeqState* st = r->pin_seq.as<SeqState>();
    TB_CUDA(cudaMemcpyAsync(r->pin_seq.p, r->seq.p, sizeof(SeqState) * r->B, cudaMemcpyDeviceToHost,
                            r->ctx->stream));
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    for (int s = 0; s < r->B; ++s) st[s].active = (s < gp.n_seqs && gp.max_new > 0) ? 1 : 0;
    return push_seq(r);
}

extern "C" tb_status tb_runner_generate(tb_runner* r, const int32_t* prompts, const int64_t* offs, int32_t n_seqs,
                                        int32_t max_new, const int32_t* stop, int32_t n_stop, int32_t* out_tokens,
                                        int32_t* out_counts, tb_token_callback cb, void* user) {
    TB_CHECK(r && out_tokens && out_counts, "NULL argument");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    GenPlan gp;
    tb_status e = gen_setup(r, prompts, offs, n_seqs, max_new, gp);
    if (e != TB_OK) return e;
    if ((e = gen_begin(r, gp)) != TB_OK) return e;
    if ((e = gen_activate_all(r, gp)) != TB_OK) return e;
    std::vector<char> act(r->B, 0);
    for (int s = 0; s < n_seqs; ++s) act[s] = max_new > 0;
    std::vector<int> count(n_seqs, 0);
    const bool stepwise = (n_stop > 0 && stop) || cb;
    if (!stepwise) {
        if ((e = run_steps(r, max_new, act)) != TB_OK) return e;
        TB_CUDA(cudaMemcpyAsync(r->pin_tokens.p, r->out_tokens.p, (size_t)r->B * r->max_out * 4,
                                cudaMemcpyDeviceToHost, r->ctx->stream));
        r->d2h_bytes += (int64_t)r->B * r->max_out * 4;
        TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
        const int* pt = r->pin_tokens.as<int>();
        for (int s = 0; s < n_seqs; ++s) {
            for (int i = 0; i < max_new; ++i) out_tokens[(size_t)s * max_new + i] = pt[(size_t)s * r->max_out + i];
            out_counts[s] = max_new;
        }
        return tb_context_check_device(r->ctx);
    }
    // Step-synchronous path: yield every token, honour stop tokens
    // (ModelRunner.swift:272-292: the stop token is yielded, then the loop ends).
    SeqState* st = r->pin_seq.as<SeqState>();
    for (int t = 0; t < max_new; ++t) {
        bool any = false;
        for (int s = 0; s < n_seqs; ++s) any = any || act[s];
        if (!any) break;
        if ((e = run_steps(r, 1, act)) != TB_OK) return e;
        TB_CUDA(cudaMemcpyAsync(r->pin_seq.p, r->seq.p, sizeof(SeqState) * r->B, cudaMemcpyDeviceToHost,
                                r->ctx->stream));
        r->d2h_bytes += (int64_t)sizeof(SeqState) * r->B;
        TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
        bool changed = false;
        for (int s = 0; s < n_seqs; ++s) {
            if (!act[s]) continue;
            // After a generating step the device stored the sampled token as the next input.
            const int tok = st[s].token;
            out_tokens[(size_t)s * max_new + count[s]] = tok;
            count[s] += 1;
            bool stop_now = false;
            for (int k = 0; k < n_stop; ++k)
                if (stop[k] == tok) stop_now = true;
            if (cb && cb(user, s, count[s] - 1, tok) != 0) stop_now = true;
            if (count[s] >= max_new) stop_now = true;
            if (stop_now) {
                act[s] = 0;
                st[s].active = 0;
                changed = true;
            }
        }
        if (changed && (e = push_seq(r)) != TB_OK) return e;
    }
    for (int s = 0; s < n_seqs; ++s) out_counts[s] = count[s];
    return tb_context_check_device(r->ctx);
}

extern "C" tb_status tb_runner_prefill_device(tb_runner* r, const int32_t* prompts, const int64_t* offs,
                                              int32_t n_seqs, int32_t max_new) {
    TB_CHECK(r, "NULL runner");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    GenPlan gp;
    tb_status e = gen_setup(r, prompts, offs, n_seqs, max_new, gp);
    if (e != TB_OK) return e;
    r->last_n_seqs = gp.n_seqs;
    r->last_max_new = gp.max_new;
    if ((e = gen_begin(r, gp)) != TB_OK) return e;
    if ((e = gen_activate_all(r, gp)) != TB_OK) return e;
    if ((e = capture_graph(r)) != TB_OK) return e;
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    return tb_context_check_device(r->ctx);
}

extern "C" tb_status tb_runner_decode_device(tb_runner* r, int32_t n_steps, float* ms) {
    TB_CHECK(r && n_steps >= 0, "bad argument");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    std::vector<char> act(r->B, 0);
    for (int s = 0; s < r->last_n_seqs; ++s) act[s] = 1;
    // Pre-map the pages these steps touch so the timed loop is pure graph replays.
    TB_CUDA(cudaEventRecord(r->ev0, r->ctx->stream));
    tb_status e = run_steps(r, n_steps, act);
    if (e != TB_OK) return e;
    TB_CUDA(cudaEventRecord(r->ev1, r->ctx->stream));
    TB_CUDA(cudaEventSynchronize(r->ev1));
    float t = 0.0f;
    TB_CUDA(cudaEventElapsedTime(&t, r->ev0, r->ev1));
    if (ms) *ms = t;
    return tb_context_check_device(r->ctx);
}

// Device timeline of one graph-replayed decode step (per launch: kTracePoints
// globaltimer stamps, see GemvParams::trace) -- where the step's time goes
// between launch, dependency release, prologue, tensor-core work and exit.
extern "C" tb_status tb_runner_trace_launches(tb_runner* r, uint64_t* stamps, int32_t* kinds, int32_t* n) {
    TB_CHECK(r && stamps && kinds && n, "NULL argument");
    TB_CHECK(!r->persistent, "tracing covers the per-launch step");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    const int cnt = (int)r->plan.size();
    TB_CHECK(*n >= cnt, "capacity %d < %d launches", *n, cnt);
    DevBuf buf;
    TB_CUDA(buf.alloc((size_t)cnt * kTracePoints * 8));
    std::vector<uint64_t> init((size_t)cnt * kTracePoints, 0ull);
    for (int i = 0; i < cnt; ++i) init[(size_t)i * kTracePoints] = ~0ull;
    TB_CUDA(cudaMemcpy(buf.p, init.data(), init.size() * 8, cudaMemcpyHostToDevice));
    auto set = [&](bool on) {
        for (int i = 0; i < cnt; ++i) {
            unsigned long long* t = on ? buf.as<unsigned long long>() + (size_t)i * kTracePoints : nullptr;
            r->plan[i].g.trace = t;
            r->plan[i].a.trace = t;
        }
        if (r->graph) cudaGraphExecDestroy(r->graph);
        r->graph = nullptr;
    };
    std::vector<char> act(r->B, 0);
    for (int s = 0; s < std::max(1, r->last_n_seqs); ++s) act[s] = 1;
    set(true);
    tb_status e = run_steps(r, 1, act);
    cudaError_t ce = cudaStreamSynchronize(r->ctx->stream);
    set(false);
    if (e != TB_OK) return e;
    if (ce != cudaSuccess) return cuda_fail(ce, "trace step");
    TB_CUDA(cudaMemcpy(stamps, buf.p, (size_t)cnt * kTracePoints * 8, cudaMemcpyDeviceToHost));
    for (int i = 0; i < cnt; ++i) kinds[i] = r->plan[i].kind;
    *n = cnt;
    return tb_context_check_device(r->ctx);
}

extern "C" tb_status tb_runner_read_tokens(tb_runner* r, int32_t* out_tokens, int32_t* out_counts) {
    TB_CHECK(r && out_tokens && out_counts, "NULL argument");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    TB_CUDA(cudaMemcpyAsync(r->pin_tokens.p, r->out_tokens.p, (size_t)r->B * r->max_out * 4, cudaMemcpyDeviceToHost,
                            r->ctx->stream));
    TB_CUDA(cudaMemcpyAsync(r->pin_seq.p, r->seq.p, sizeof(SeqState) * r->B, cudaMemcpyDeviceToHost,
                            r->ctx->stream));
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    const SeqState* st = r->pin_seq.as<SeqState>();
    const int* pt = r->pin_tokens.as<int>();
    const int stride = std::max(1, r->last_max_new);
    for (int s = 0; s < r->last_n_seqs; ++s) {
        const int n = std::min(std::min(st[s].n_out, r->max_out), stride);
        out_counts[s] = n;
        for (int i = 0; i < n; ++i) out_tokens[(size_t)s * stride + i] = pt[(size_t)s * r->max_out + i];
    }
    return ok();
}

extern "C" tb_status tb_runner_profile_step(tb_runner* r, float* times_ms, int32_t* kinds, int64_t* bytes,
                                            int32_t* n) {
    TB_CHECK(r && n && times_ms && kinds && bytes, "NULL argument");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    const int cnt = (int)r->plan.size();
    TB_CHECK(*n >= cnt, "capacity %d < %d kernels", *n, cnt);
    std::vector<char> act(r->B, 0);
    for (int s = 0; s < std::max(1, r->last_n_seqs); ++s) act[s] = 1;
    for (int s = 0; s < r->B; ++s)
        if (act[s]) {
            tb_status e = kv_prepare(r, s);
            if (e != TB_OK) return e;
        }
    tb_status e = flush_ptab(r);
    if (e != TB_OK) return e;
    if (r->persistent) {
        cudaStream_t st = r->ctx->stream;
        TB_CUDA(cudaEventRecord(r->ev0, st));
        cudaError_t ce = launch_decode_step(r->sp, r->step_grid, r->step_smem, st);
        if (ce != cudaSuccess) return cuda_fail(ce, "launch_decode_step");
        TB_CUDA(cudaEventRecord(r->ev1, st));
        TB_CUDA(cudaEventSynchronize(r->ev1));
        float t = 0;
        TB_CUDA(cudaEventElapsedTime(&t, r->ev0, r->ev1));
        times_ms[0] = t;
        kinds[0] = 2;
        // algorithmic bytes: every weight + scale once, K/V of the context, the
        // embedding row and the logits
        const tb_model_config& c = r->m->cfg;
        const int64_t L = r->kvh[0].pos + 1;
        bytes[0] = r->m->weight_bytes + (int64_t)c.num_layers * 2 * L * r->m->kv_dim * 4 +
                   (int64_t)c.hidden_dim * 4 + (int64_t)c.vocab_size * 4;
        for (int s2 = 0; s2 < r->B; ++s2)
            if (act[s2]) r->kvh[s2].pos += 1;
        *n = 1;
        return tb_context_check_device(r->ctx);
    }
    std::vector<cudaEvent_t> ev(cnt + 1);
    for (auto& x : ev) TB_CUDA(cudaEventCreate(&x));
    cudaStream_t st = r->ctx->stream;
    TB_CUDA(cudaEventRecord(ev[0], st));
    for (int i = 0; i < cnt; ++i) {
        tb_status ls = launch_op(r, r->plan[i], st, false);
        if (ls != TB_OK) return ls;
        TB_CUDA(cudaEventRecord(ev[i + 1], st));
    }
    TB_CUDA(cudaEventSynchronize(ev[cnt]));
    for (int i = 0; i < cnt; ++i) {
        float t = 0;
        TB_CUDA(cudaEventElapsedTime(&t, ev[i], ev[i + 1]));
        times_ms[i] = t;
        kinds[i] = r->plan[i].kind;
        bytes[i] = r->plan[i].bytes;
    }
    for (auto& x : ev) cudaEventDestroy(x);
    for (int s = 0; s < r->B; ++s)
        if (act[s]) r->kvh[s].pos += 1;
    *n = cnt;
    return tb_context_check_device(r->ctx);
}

extern "C" tb_status tb_runner_io_bytes(tb_runner* r, int64_t* h2d, int64_t* d2h, int32_t reset) {
    TB_CHECK(r && h2d && d2h, "NULL argument");
    *h2d = r->h2d_bytes;
    *d2h = r->d2h_bytes;
    if (reset) r->h2d_bytes = r->d2h_bytes = 0;
    return ok();
}

extern "C" tb_status tb_runner_set_persistent(tb_runner* r, int32_t enable) {
    TB_CHECK(r, "NULL runner");
    const bool want = enable != 0;
    if (want && r->sampling)
        return fail(TB_ERR_UNSUPPORTED, "the persistent step decodes greedily; clear the sampler first");
    if (want && !r->persistent_ok)
        return fail(TB_ERR_UNSUPPORTED, "the persistent step needs batch 1, a LLaMA model with uniform layers "
                                        "and a supported head shape");
    if (want != r->persistent) {
        r->persistent = want;
        if (r->graph) {
            cudaGraphExecDestroy(r->graph);
            r->graph = nullptr;
        }
    }
    return ok();
}

// Sampler.sampleDetailed on one logits row from the host (the sampler kernel
// with a single sequence; history = the penalty history).
extern "C" tb_status tb_sample_detailed(tb_context* ctx, const float* logits, int32_t V, const tb_sampler_config* cfg,
                                        const int32_t* history, int32_t n_history, uint64_t* rng_state,
                                        int32_t* token, float* prob, float* entropy) {
    TB_CHECK(ctx && logits && cfg && rng_state && token && prob && entropy, "NULL argument");
    TB_CHECK(V >= 1 && n_history >= 0 && (history || n_history == 0), "bad size");
    TB_CUDA(cudaSetDevice(ctx->device));
    bool in_smem = false;
    sample_smem_bytes(V, &in_smem);
    const int nh = std::max(1, n_history);
    DevBuf dl, dseq, dhist, dout, dwork;
    TB_CUDA(dl.alloc((size_t)V * 4));
    TB_CUDA(dseq.alloc(sizeof(SeqState)));
    TB_CUDA(dhist.alloc((size_t)nh * 4));
    TB_CUDA(dout.alloc(32));
    if (!in_smem) TB_CUDA(dwork.alloc((size_t)V * 4));
    SeqState st{};
    st.pos = n_history;  // a generation step: pos >= n_prompt - 1
    st.n_prompt = n_history;
    st.max_out = 1;
    st.active = 1;
    cudaStream_t sm = ctx->stream;
    TB_CUDA(cudaMemcpyAsync(dl.p, logits, (size_t)V * 4, cudaMemcpyHostToDevice, sm));
    TB_CUDA(cudaMemcpyAsync(dseq.p, &st, sizeof st, cudaMemcpyHostToDevice, sm));
    if (n_history > 0) TB_CUDA(cudaMemcpyAsync(dhist.p, history, (size_t)n_history * 4, cudaMemcpyHostToDevice, sm));
    TB_CUDA(cudaMemcpyAsync(dout.as<char>() + 16, rng_state, 8, cudaMemcpyHostToDevice, sm));
    SampleParams p{};
    p.logits = dl.as<float>();
    p.work = dwork.as<float>();
    p.V = V;
    p.M = 1;
    p.seq = dseq.as<SeqState>();
    p.prompt = dhist.as<int>();
    p.prompt_stride = nh;
    p.out_tokens = dout.as<int>();
    p.out_prob = dout.as<float>() + 1;
    p.out_entropy = dout.as<float>() + 2;
    p.rng = reinterpret_cast<unsigned long long*>(dout.as<char>() + 16);
    p.temperature = cfg->temperature;
    p.top_p = cfg->top_p;
    p.repetition_penalty = cfg->repetition_penalty;
    p.top_k = cfg->top_k;
    p.has_top_p = cfg->has_top_p;
    cudaError_t e = launch_sample(p, sm, false);
    if (e != cudaSuccess) return cuda_fail(e, "launch_sample");
    unsigned char out[32];
    TB_CUDA(cudaMemcpyAsync(out, dout.p, 32, cudaMemcpyDeviceToHost, sm));
    TB_CUDA(cudaStreamSynchronize(sm));
    memcpy(token, out, 4);
    memcpy(prob, out + 4, 4);
    memcpy(entropy, out + 8, 4);
    memcpy(rng_state, out + 16, 8);
    return tb_context_check_device(ctx);
}

extern "C" tb_status tb_runner_set_sampler(tb_runner* r, const tb_sampler_config* cfg) {
    TB_CHECK(r, "NULL runner");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    if (cfg) {
        TB_CHECK(std::isfinite(cfg->temperature), "temperature must be finite");
        TB_CHECK(std::isfinite(cfg->repetition_penalty) && cfg->repetition_penalty > 0.0f,
                 "repetition_penalty must be finite and > 0");
        TB_CHECK(!cfg->has_top_p || std::isfinite(cfg->top_p), "top_p must be finite");
    }
    const bool want = cfg != nullptr;
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    if (want) {
        const int V = r->m->cfg.vocab_size;
        bool in_smem = false;
        sample_smem_bytes(V, &in_smem);
        if (!in_smem && r->swork.bytes < (size_t)r->B * V * 4) TB_CUDA(r->swork.alloc((size_t)r->B * V * 4));
        if (!r->sampling) {
            r->persistent_before = r->persistent;
            r->persistent = false;
        }
        r->scfg = *cfg;
        r->sampling = true;
        tb_status e = seed_sampler(r);
        if (e != TB_OK) return e;
    } else if (r->sampling) {
        r->sampling = false;
        r->persistent = r->persistent_before;
    }
    tb_status e = build_plan(r);
    if (e != TB_OK) return e;
    if (r->graph) {
        cudaGraphExecDestroy(r->graph);
        r->graph = nullptr;
    }
    return ok();
}

// PerplexityHarness.computePerplexity (PerplexityHarness.swift:141-193) for
// n_seqs token slices at once: every slice is fed teacher-forced (the slice is
// the prompt: tokens[0..n-2] are stepped, each step scores tokens[i+1]) and
// the device sums log P(target) per slice in fp64.  The runner's sequences
// start fresh, as in generate.
extern "C" tb_status tb_runner_perplexity(tb_runner* r, const int32_t* tokens, const int64_t* offs, int32_t n_seqs,
                                          double* sum_logprob, int64_t* n_predictions) {
    TB_CHECK(r && tokens && offs && sum_logprob && n_predictions, "NULL argument");
    TB_CHECK(!r->sampling, "clear the sampler before scoring");
    TB_CHECK(n_seqs >= 1 && n_seqs <= r->B, "n_seqs must be in [1, %d]", r->B);
    const int V = r->m->cfg.vocab_size;
    for (int s = 0; s < n_seqs; ++s) {
        TB_CHECK(offs[s + 1] - offs[s] >= 2, "slice %d needs at least two tokens to have a prediction target", s);
        for (int64_t i = offs[s]; i < offs[s + 1]; ++i)
            TB_CHECK(tokens[i] >= 0 && tokens[i] < V, "token %d out of vocab range [0, %d)", tokens[i], V);
    }
    TB_CUDA(cudaSetDevice(r->ctx->device));
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    // Chunked: up to 64 positions (of one or several slices) per pass, when no
    // slice would evict KV pages; the per-position log-probabilities come back
    // and are summed per slice in position order, as the reference does.
    bool chunk = r->pf_enabled && r->m->tp_world == 1;
    const int64_t cap = std::min<int64_t>(r->m->cfg.max_seq_len, (int64_t)r->max_pages_per_seq * kPageTokens);
    for (int s = 0; s < n_seqs && chunk; ++s)
        chunk = offs[s + 1] - offs[s] - 1 <= std::min<int64_t>(cap, r->max_positions);
    if (chunk) {
        std::vector<double> lp;
        tb_status e = score_chunked(r, tokens, offs, n_seqs, lp);
        if (e != TB_OK) return e;
        size_t i0 = 0;
        for (int s = 0; s < n_seqs; ++s) {
            const int64_t np = offs[s + 1] - offs[s] - 1;
            double sum = 0.0;
            for (int64_t i = 0; i < np; ++i) sum += lp[i0 + i];
            i0 += (size_t)np;
            sum_logprob[s] = sum;
            n_predictions[s] = np;
        }
        return tb_context_check_device(r->ctx);
    }
    if (r->lp_acc.bytes < (size_t)r->B * 8) TB_CUDA(r->lp_acc.alloc((size_t)r->B * 8));
    TB_CUDA(cudaMemset(r->lp_acc.p, 0, (size_t)r->B * 8));
    const bool persistent = r->persistent;
    r->persistent = false;
    r->scoring = true;
    auto restore = [&]() -> tb_status {
        r->scoring = false;
        r->persistent = persistent;
        tb_status e = build_plan(r);
        if (r->graph) {
            cudaGraphExecDestroy(r->graph);
            r->graph = nullptr;
        }
        return e;
    };
    tb_status e = build_plan(r);
    if (r->graph) {
        cudaGraphExecDestroy(r->graph);
        r->graph = nullptr;
    }
    GenPlan gp;
    if (e == TB_OK) e = gen_setup(r, tokens, offs, n_seqs, 0, gp);
    if (e == TB_OK) e = gen_begin(r, gp);
    if (e == TB_OK) {
        std::vector<double> acc((size_t)r->B);
        cudaError_t ce = cudaMemcpyAsync(acc.data(), r->lp_acc.p, (size_t)r->B * 8, cudaMemcpyDeviceToHost,
                                         r->ctx->stream);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(r->ctx->stream);
        if (ce != cudaSuccess) e = cuda_fail(ce, "perplexity read-back");
        for (int s = 0; s < n_seqs && e == TB_OK; ++s) {
            sum_logprob[s] = acc[s];
            n_predictions[s] = offs[s + 1] - offs[s] - 1;
        }
    }
    tb_status e2 = restore();
    if (e != TB_OK) return e;
    if (e2 != TB_OK) return e2;
    return tb_context_check_device(r->ctx);
}

extern "C" tb_status tb_runner_set_step_history(tb_runner* r, const int32_t* tokens, int32_t n) {
    TB_CHECK(r && (tokens || n == 0) && n >= 0, "bad argument");
    const int V = r->m->cfg.vocab_size;
    r->step_hist.resize((size_t)n);
    for (int i = 0; i < n; ++i) r->step_hist[i] = std::max(0, std::min(tokens[i], V - 1));
    return ok();
}

extern "C" tb_status tb_runner_step_stats(tb_runner* r, float* prob, float* entropy) {
    TB_CHECK(r && prob && entropy, "NULL argument");
    TB_CHECK(r->sampling, "no sampler set: greedy steps draw nothing");
    *prob = r->last_prob;
    *entropy = r->last_ent;
    return ok();
}

extern "C" tb_status tb_runner_token_stats(tb_runner* r, int32_t n_seqs, int32_t max_new, float* prob,
                                           float* entropy) {
    TB_CHECK(r && prob && entropy, "NULL argument");
    TB_CHECK(n_seqs >= 1 && n_seqs <= r->B && max_new >= 0 && max_new <= r->max_out, "bad shape");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    for (int s = 0; s < n_seqs; ++s) {
        TB_CUDA(cudaMemcpy(prob + (size_t)s * max_new, r->out_prob.as<float>() + (size_t)s * r->max_out,
                           (size_t)max_new * 4, cudaMemcpyDeviceToHost));
        TB_CUDA(cudaMemcpy(entropy + (size_t)s * max_new, r->out_ent.as<float>() + (size_t)s * r->max_out,
                           (size_t)max_new * 4, cudaMemcpyDeviceToHost));
    }
    r->d2h_bytes += (int64_t)n_seqs * max_new * 8;
    return ok();
}

extern "C" tb_status tb_runner_set_chunked_prefill(tb_runner* r, int32_t enable) {
    TB_CHECK(r, "NULL runner");
    r->pf_enabled = enable != 0;
    return ok();
}

extern "C" tb_status tb_runner_get_persistent(const tb_runner* r, int32_t* enabled) {
    TB_CHECK(r && enabled, "NULL argument");
    *enabled = r->persistent ? 1 : 0;
    return ok();
}

extern "C" tb_status tb_runner_debug_read(tb_runner* r, int32_t which, float* out, int64_t n) {
    TB_CHECK(r && out && n >= 0, "bad argument");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    const DevBuf* b = nullptr;
    switch (which) {
        case 0: b = &r->hX; break;
        case 1: b = &r->hY; break;
        case 2: b = &r->part_qkv; break;
        case 3: b = &r->part_o; break;
        case 4: b = &r->part_gu; break;
        case 5: b = &r->part_dn; break;
        case 6: b = &r->step_attn; break;
        case 7: b = &r->logits; break;
        case 8: b = &r->h; break;
        case 9: b = &r->q; break;
        case 10: b = &r->ctxv; break;
        case 11: b = &r->act; break;
        default: return fail(TB_ERR_INVALID_ARGUMENT, "unknown buffer %d", which);
    }
    TB_CHECK((size_t)n * 4 <= b->bytes, "buffer %d holds %zu bytes", which, b->bytes);
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    TB_CUDA(cudaMemcpy(out, b->p, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return ok();
}

extern "C" tb_status tb_runner_trace_step(tb_runner* r, uint64_t* out, int64_t n, int32_t* ctas, int32_t* phases) {
    TB_CHECK(r && out && ctas && phases, "NULL argument");
    TB_CHECK(r->persistent, "tracing needs the persistent step");
    TB_CUDA(cudaSetDevice(r->ctx->device));
    const int nph = step_phases(r->sp);
    const size_t cnt = (size_t)r->step_grid * nph * 8;
    TB_CHECK((size_t)n >= cnt, "need %zu entries", cnt);
    if (r->step_trace.bytes < cnt * 8) TB_CUDA(r->step_trace.alloc(cnt * 8));
    tb_status s = kv_prepare(r, 0);
    if (s != TB_OK) return s;
    if ((s = flush_ptab(r)) != TB_OK) return s;
    StepParams p = r->sp;
    p.trace = r->step_trace.as<unsigned long long>();
    TB_CUDA(cudaMemsetAsync(r->step_trace.p, 0, cnt * 8, r->ctx->stream));
    cudaError_t ce = launch_decode_step(p, r->step_grid, r->step_smem, r->ctx->stream);
    if (ce != cudaSuccess) return cuda_fail(ce, "launch_decode_step");
    TB_CUDA(cudaStreamSynchronize(r->ctx->stream));
    r->kvh[0].pos += 1;
    TB_CUDA(cudaMemcpy(out, r->step_trace.p, cnt * 8, cudaMemcpyDeviceToHost));
    *ctas = r->step_grid;
    *phases = nph;
    return tb_context_check_device(r->ctx);
}
