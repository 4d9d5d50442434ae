// tb_gemv.cu -- weight-only dequantising GEMV for decode (M <= 8), sm_100a.
//
// Replaces the reference's per-output-thread Metal kernels
// (Sources/TinyBrainMetal/Shaders/Dequant.metal:49-79 matmul_int8_dequant and
// Shaders/DequantINT4.metal:95-137 matmul_int4_dequant, dispatched from
// MetalBackend.swift:894-1048) with a streaming design for HBM3e:
//
//  * one producer warp per CTA streams 512-byte-per-row slabs of a 32/64-row
//    block with 1-D bulk async copies (cp.async.bulk, TMA) into a shared-memory
//    ring guarded by mbarriers; the first stages are issued before the
//    programmatic-dependent-launch wait, so weights of the next projection are
//    already in flight while the previous kernel finishes;
//  * eight consumer warps unpack biased int8 / int4 values to fp32 with byte
//    permutes and exponent-bias arithmetic (exact), and accumulate with packed
//    f32x2 FMAs in a fixed order;
//  * the reduction dimension is split across the CTAs of a thread-block
//    cluster; partial sums are combined through distributed shared memory in
//    rank order (deterministic, no atomics);
//  * fused prologues (embedding gather, RMSNorm: Tensor.swift:1538-1558) and
//    epilogues (per-column scale, bias, residual add, RoPE + KV-cache append:
//    ModelRunner.swift:470-517, SiLU*up: ModelRunner.swift:448-453, GELU,
//    LM-head argmax: Sampler.swift:126-138).
#include "tb_common.cuh"
#include "tb_kernels.h"
#include "tb_tc.cuh"
#include "tb_unit.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

namespace tb {

QLayout make_qlayout(int precision, int K, int N, int RB) {
    QLayout L{};
    L.precision = precision;
    L.K = K;
    L.N = N;
    L.fused_gu = RB == 64 ? 1 : 0;
    // Both precisions: 128-row tiles streamed in units of 128 k (tb_tc.cuh).
    L.Kp = (K + kTcUnitK - 1) / kTcUnitK * kTcUnitK;
    L.RB = kTcTileRows;
    L.slab_k = kTcUnitK;
    L.slab_bytes = precision == 8 ? kTcUnitK : kTcUnitK / 2;
    L.row_bytes = precision == 8 ? L.Kp : L.Kp / 2;
    L.Np = (N + L.RB - 1) / L.RB * L.RB;
    L.slabs = L.Kp / kTcUnitK;
    if (precision == 8) {
        L.weight_bytes = (size_t)L.Np * L.row_bytes;
        L.scale_floats = (size_t)L.Np;  // per-row scales
    } else {
        // units carry their group scales inline; the scale buffer holds the
        // per-(32-row group, unit) maximum |scale|
        L.weight_bytes = (size_t)(L.Np / kTcTileRows) * L.slabs * kQ4UnitBytes;
        L.scale_floats = (size_t)(L.Np / 32) * L.slabs;
    }
    return L;
}

namespace {

template <int PREC, int RB>
struct GemvCfg {
    static constexpr int kStageBytes = PREC == 8 ? kTcUnitBytes : kQ4UnitBytes;
    // 2 CTAs per SM x 4 (6) units in flight cover HBM latency many times over
    static constexpr int kStages = PREC == 8 ? 4 : 6;
};
// Digit rows of the B operand for MB batch rows: INT8 4 digits per row (N >= 8,
// 16-multiples past 8); INT4 4 digits per (row, 32-row weight group).
__host__ __device__ constexpr int tc_nb(int mb) { return mb <= 2 ? 8 : (4 * mb + 15) / 16 * 16; }
__host__ __device__ constexpr int q4_nb(int mb) { return 16 * mb; }
// INT4 pipeline slots: kQ4Slots A operands in tensor memory (32 columns each)
// and B operands in shared memory, then one accumulator of NB columns.
constexpr int kQ4Slots = 4;
constexpr int kGemvBarBytes = 512;  // mbarriers + tensor-memory address at the start of shared memory
// Row stride of the partial sums red[row][m]: one float of padding past a
// single batch row, so the epilogue warps (one tile row per lane) write
// 32 different banks.
__host__ __device__ constexpr int red_stride(int mb) { return mb == 1 ? 1 : mb + 1; }
// red [RB][red_stride], misc [16 MB], row scales and biases [2 RB], seqinfo [3 MB], rowinv / rowex [2 MB]
__host__ __device__ constexpr int gemv_head_floats(int rb, int mb) {
    return rb * red_stride(mb) + 16 * mb + 2 * rb + 5 * mb;
}
__host__ __device__ constexpr int q4_dcols(int mb) { return q4_nb(mb) < 32 ? 32 : q4_nb(mb); }
// INT4 CTAs add a tensor-core issue warp to the producer and 8 consumer warps.
// INT8 batches beyond 16 rows per CTA ("wide"): digits are built per unit
// (B slots) instead of once for the CTA's k range.
__host__ __device__ constexpr bool gemv_wide(int prec, int mb) { return prec == 8 && mb > 16; }
constexpr int kWideSlots = 2;
// wide B slots: 8-row core matrices 144 B apart (128 + 16 pad: conflict-free
// digit stores), 16-k chunks NB / 8 core matrices apart
constexpr uint32_t kWideSbo = 144;
__host__ __device__ constexpr uint32_t wide_lbo(int nb) { return (uint32_t)(nb / 8) * kWideSbo; }
__host__ __device__ constexpr int gemv_threads(int prec, int mb) {
    return (prec == 4 || gemv_wide(prec, mb)) ? kGemvThreads + 32 : kGemvThreads;
}
// At most 256 columns: two CTAs of any GEMV variant fit one SM's 512 together,
// so a CTA never waits in tcgen05.alloc for another one to finish.
__host__ __device__ constexpr int q4_tmem_cols(int mb) { return 256; }
// Batch rows handled by one CTA.
inline int gemv_mb(int prec, int M) {
    const int cap = prec == 8 ? 64 : 4;  // INT4: A slots + accumulator fit 256 TMEM columns
    const int mb = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : M <= 16 ? 16 : 64;
    return std::min(mb, cap);
}

__device__ __forceinline__ float silu_ref(float x) {
    // Tensor.swift:1135-1142: x / (1 + exp(-x))
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}
__device__ __forceinline__ float gelu_ref(float x) {
    // Tensor.swift:1107-1121 (tanh approximation, fp32)
    const float s = 0.797884583f;  // Float(sqrt(2.0 / Float.pi))
    float x3 = __fmul_rn(__fmul_rn(x, x), x);
    float inner = __fmul_rn(s, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

template <int PREC, int RB, int MB>
__global__ void __launch_bounds__(gemv_threads(PREC, MB), 2) gemv_kernel(const __grid_constant__ GemvParams p) {
    using Cfg = GemvCfg<PREC, RB>;
    static_assert(RB == kTcTileRows, "tensor-core tiles are 128 rows");
    constexpr int STAGES = Cfg::kStages;
    constexpr int NB = PREC == 8 ? tc_nb(MB) : q4_nb(MB);
    static_assert(NB <= 256, "tcgen05 N is at most 256");
    // accumulator (INT8: NB columns; INT4: A slots + two accumulators), a power of two >= 32
    static_assert(PREC != 4 || kQ4Slots * 32 + q4_dcols(MB) <= q4_tmem_cols(MB), "INT4 TMEM budget");
    constexpr uint32_t kTmemCols = PREC == 4 ? (uint32_t)q4_tmem_cols(MB)
                                             : (NB <= 32 ? 32u : NB <= 64 ? 64u : NB <= 128 ? 128u : 256u);

    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + STAGES;
    uint64_t* done = empty + STAGES;                                      // [2] accumulators complete
    uint64_t* a_ready = done + 2;                                         // INT4: [kQ4Slots] A in tensor memory
    uint64_t* b_ready = a_ready + kQ4Slots;                               // INT4: [kQ4Slots] B in shared memory
    uint64_t* s_free = b_ready + kQ4Slots;                                // INT4: [kQ4Slots] products done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_free + kQ4Slots);
    static_assert((2 * STAGES + 2 + 3 * kQ4Slots) * 8 + 4 <= kGemvBarBytes, "barrier region");
    constexpr int RS = red_stride(MB);
    float* red = reinterpret_cast<float*>(smem + kGemvBarBytes);          // [RB][RS]
    float* misc = red + RB * RS;                                          // [2][MB][8]
    float* rowsc = misc + 16 * MB;                                        // [RB] row scales (1 for INT4)
    float* rowbias = rowsc + RB;                                          // [RB] row biases (0 if none)
    int* seqinfo = reinterpret_cast<int*>(rowbias + RB);                  // [3][MB] pos, active, page
    float* rowinv = reinterpret_cast<float*>(seqinfo + 3 * MB);           // [MB] 1/rms of each batch row
    int* rowex = reinterpret_cast<int*>(rowinv + MB);                     // [MB] INT8 digit exponents
    uint8_t* stage_base = smem + (kGemvBarBytes + gemv_head_floats(RB, MB) * 4 + 1023) / 1024 * 1024;
    uint8_t* xbuf = stage_base + STAGES * Cfg::kStageBytes;
    uint8_t* xd = xbuf;  // INT8: digit operand [k/16][NB][16]

    const QLayout& L = p.L;
    const int P = p.P;
    const int rank = (P > 1) ? (int)cluster_ctarank() : 0;
    const int rb = blockIdx.x / P;
    const int s0 = rank * L.slabs / P;
    const int s1 = (rank + 1) * L.slabs / P;
    const int nunits = s1 - s0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // batch rows [m0, m0 + Mloc) of this CTA (grid y splits batches larger than MB)
    const int m0 = blockIdx.y * MB;
    const int Mloc = min(MB, p.M - m0);
    // Activation staging after the stage ring, kspan = the CTA's k range:
    //   INT8: digits [kspan/16][NB][16], x [MB][kspan] fp32, norm weights [kspan];
    //   INT4: x [MB][kspan] fp32, norm weights [kspan], B slots
    //   [kQ4Slots][NB * 128], per-unit max |x| [nunits][MB], per-unit max
    //   |scale| [4][nunits], digit exponents [MB][4].
    const int kspan = ((L.slabs + P - 1) / P) * kTcUnitK;
    constexpr bool WIDE = gemv_wide(PREC, MB);
    // wide with a precomputed digit operand (wide_digits): B streams in beside A
    const bool pre = WIDE && p.bimg != nullptr;
    // wide INT8: B slots [kWideSlots][NB * 128] at xbuf, norm weights after them, no x staging
    float* xs = reinterpret_cast<float*>(
        PREC == 8 ? xbuf + (WIDE ? (size_t)kWideSlots * wide_lbo(NB) * 8 : (size_t)kspan * NB) : xbuf);
    float* wstage = WIDE ? xs : xs + (size_t)MB * kspan;
    uint8_t* bslots = reinterpret_cast<uint8_t*>(wstage + kspan);
    float* xmax = reinterpret_cast<float*>(bslots + kQ4Slots * NB * 128);
    float* smaxs = xmax + (size_t)(kspan / kTcUnitK) * MB;
    int* ex4 = reinterpret_cast<int*>(smaxs + kQ4Groups * (kspan / kTcUnitK));

    if (threadIdx.x == 0) {
        trace_min(p.trace, 0);
        trace_max(p.trace, 1);
        if (PREC == 8 && p.trace && blockIdx.x == 0 && blockIdx.y == 0) {  // launch shape (diagnostics)
            p.trace[14] = (unsigned long long)P;
            p.trace[15] = (unsigned long long)(gridDim.x * gridDim.y);
        }
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full[i], 1);
            // INT8: released by tcgen05.commit; INT4: by the 8 consumer warps after reading it
            mbar_init(&empty[i], PREC == 8 ? 1 : kGemvConsumerWarps);
        }
        mbar_init(&done[0], 1);
        mbar_init(&done[1], 1);
        for (int i = 0; i < kQ4Slots; ++i) {
            mbar_init(&a_ready[i], 4);
            mbar_init(&b_ready[i], WIDE ? (pre ? 1 : kGemvConsumerWarps) : 4);
            mbar_init(&s_free[i], 1);
        }
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch_dependents();

    if (WIDE && warp == kGemvConsumerWarps + 1) {
        // --------------------- wide INT8: tensor-core issue ---------------------
        if (lane == 0) {
            const uint32_t tmem = *tmem_slot;
            for (int i = 0; i < nunits; ++i) {
                const int st = i % STAGES;
                const int sl = i % kWideSlots;
                if (!mbar_wait(&full[st], (i / STAGES) & 1, p.err)) break;
                if (!mbar_wait(&b_ready[sl], (uint32_t)(i / kWideSlots) & 1u, p.err)) break;
                tc_fence_after();
                const uint32_t a_s = smem_u32(stage_base + st * Cfg::kStageBytes);
                const uint32_t b_s = smem_u32(xbuf + (size_t)sl * wide_lbo(NB) * 8);
                const uint32_t idesc = tc_idesc_i8(NB);
#pragma unroll
                for (int s = 0; s < kTcUnitK / 32; ++s)
                    tc_mma_i8(tmem, tc_sdesc(a_s + s * 256, 128, 1024),
                              tc_sdesc(b_s + s * 2 * wide_lbo(NB), wide_lbo(NB), kWideSbo), idesc, i > 0 || s > 0);
                tc_commit(&empty[st]);
                tc_commit(&s_free[sl]);
            }
            tc_commit(&done[0]);
        }
        __syncwarp();
    } else if (PREC == 4 && warp == kGemvConsumerWarps + 1) {
        // ------------------------- INT4 tensor-core issue -------------------------
        if (lane == 0) {
            const uint32_t tmem = *tmem_slot;
            const uint32_t idesc = tc_idesc_i8(NB);
            int i = 0;
            unsigned long long* prb = (p.trace && blockIdx.x == 0 && blockIdx.y == 0) ? p.trace : nullptr;
            for (; i < nunits; ++i) {
                const int sl = i % kQ4Slots;
                const uint32_t par = (uint32_t)(i / kQ4Slots) & 1u;
                long long c0 = prb ? clock64() : 0;
                if (!mbar_wait(&a_ready[sl], par, p.err)) break;
                if (prb) {
                    atomicAdd(prb + 12, (unsigned long long)(clock64() - c0));
                    c0 = clock64();
                }
                if (!mbar_wait(&b_ready[sl], par, p.err)) break;
                if (prb) atomicAdd(prb + 13, (unsigned long long)(clock64() - c0));
                tc_fence_after();
                const uint32_t acol = tmem + (uint32_t)(sl * 32);
                const uint32_t bsa = smem_u32(bslots + (size_t)sl * NB * 128);
#pragma unroll
                for (int s = 0; s < kTcUnitK / 32; ++s)
                    tc_mma_i8_ts(tmem + (uint32_t)(kQ4Slots * 32), acol + 8 * s,
                                 tc_sdesc(bsa + s * 2 * NB * 16, NB * 16, 128), idesc, i > 0 || s > 0);
                tc_commit(&s_free[sl]);
            }
            tc_commit(&done[0]);
        }
        __syncwarp();
    } else if (warp == kGemvConsumerWarps) {
        // ------------------------------- producer -------------------------------
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            const uint8_t* wrb = p.w + (size_t)rb * L.slabs * Cfg::kStageBytes;
            for (int i = 0; i < nunits; ++i) {
                const int st = i % STAGES;
                if (i >= STAGES) {
                    if (!mbar_wait(&empty[st], ((i / STAGES) - 1) & 1, p.err)) break;
                }
                uint8_t* dst = stage_base + st * Cfg::kStageBytes;
                mbar_arrive_expect_tx(&full[st], Cfg::kStageBytes);
                bulk_g2s_stream(dst, wrb + (size_t)(s0 + i) * Cfg::kStageBytes, Cfg::kStageBytes, &full[st], pol);
            }
        } else if (pre && lane == 1) {
            // the digit operand of every unit, written by the preceding
            // wide_digits launch: read only after the dependency wait
            if (!p.independent) pdl_wait();
            constexpr uint32_t kBBytes = wide_lbo(NB) * 8;
            for (int i = 0; i < nunits; ++i) {
                const int sl = i % kWideSlots;
                if (i >= kWideSlots) {
                    if (!mbar_wait(&s_free[sl], (uint32_t)((i / kWideSlots) - 1) & 1u, p.err)) break;
                }
                mbar_arrive_expect_tx(&b_ready[sl], kBBytes);
                bulk_g2s(xbuf + (size_t)sl * kBBytes, p.bimg + (size_t)(s0 + i) * kBBytes, kBBytes, &b_ready[sl]);
            }
        }
    } else {
        // ------------------------------- consumers -------------------------------
        const int ctid = threadIdx.x;  // 0..255
        // weights-side epilogue constants do not depend on the previous kernel
        for (int i = ctid; i < RB; i += 256) {
            const int grow = rb * RB + i;
            rowsc[i] = PREC == 8 ? __ldg(p.scales + grow) : 1.0f;
            rowbias[i] = p.bias ? __ldg(p.bias + grow) : 0.0f;
        }
        const int kbeg = s0 * L.slab_k;
        const int kend = min(s1 * L.slab_k, L.Kp);
        const bool rms = p.prologue == kProRmsNorm || p.prologue == kProEmbedRms;
        if (rms && !pre)  // RMSNorm weights of the CTA's k range (zero past K)
            for (int k = ctid; k < kspan; k += 256) wstage[k] = kbeg + k < L.K ? __ldg(p.norm_w + kbeg + k) : 0.0f;
        if (PREC == 4)
            for (int i = ctid; i < kQ4Groups * nunits; i += 256) {
                const int g = i / nunits, u = i - g * nunits;
                smaxs[g * nunits + u] = __ldg(p.scales + ((size_t)rb * kQ4Groups + g) * L.slabs + s0 + u);
            }
        if (!p.independent) pdl_wait();
        if (ctid == 0) trace_max(p.trace, 2);
        // Tensor-parallel pull: the source is the residual stream plus the
        // ranks' partials, in rank order; a word whose tag is not this step's
        // has not arrived yet (bounded spin).
        const bool pull = p.ar_world > 1 && p.ar_pull_slot >= 0;
        const unsigned int ar_tag = (p.ar_world > 1 && p.ar_step) ? *p.ar_step + 1u : 0u;
        auto pull4 = [&](int m, int k) -> float4 {
            const size_t off = (size_t)(m0 + m) * p.ld_src + k;
            float4 a = *reinterpret_cast<const float4*>(p.ar_hin + off);
            const unsigned long long* base =
                p.ar_local + (size_t)p.ar_pull_slot * p.ar_world * p.ar_slot_words + off;
            for (int q = 0; q < p.ar_world; ++q) {
                const unsigned long long* wq = base + (size_t)q * p.ar_slot_words;
                unsigned long long w[4];
                wait_tagged<4>(wq, ar_tag, w, p.err);
                a = make_float4(__fadd_rn(a.x, __uint_as_float((uint32_t)w[0])),
                                __fadd_rn(a.y, __uint_as_float((uint32_t)w[1])),
                                __fadd_rn(a.z, __uint_as_float((uint32_t)w[2])),
                                __fadd_rn(a.w, __uint_as_float((uint32_t)w[3])));
            }
            return a;
        };
        const bool hout = pull && p.ar_hout && blockIdx.x == 0 && blockIdx.y == 0;
        if (p.epilogue == kEpiQkv && ctid < Mloc) {
            const SeqState& sq = p.seq_ro[m0 + ctid];
            const int pos = sq.pos;
            seqinfo[ctid] = pos;
            seqinfo[MB + ctid] = sq.active;
            seqinfo[2 * MB + ctid] = sq.active ? p.page_table[(size_t)(m0 + ctid) * p.ptab_stride + pos / kPageTokens] : -1;
        }
        // Source row m (embedding gather or activation buffer).
        const bool embed = p.prologue == kProEmbed || p.prologue == kProEmbedRms;
        auto srcrow = [&](int m) -> const float* {
            if (embed) {
                int tok = m < Mloc ? p.seq_ro[m0 + m].token : 0;
                if (tok < 0 || tok >= p.vocab) {
                    record_error(p.err, kDevBadToken);
                    tok = 0;
                }
                return p.embedding + (size_t)tok * p.L.K;
            }
            return p.src + (size_t)(m0 + m) * p.ld_src;
        };
        // Embedding prologue: the residual stream h of the CTA's batch rows is
        // materialised by all CTAs of its grid row, each a slice of K (one CTA
        // copying 64 rows alone took ~100 us).
        if (embed) {
            const int k0 = (int)((long long)blockIdx.x * L.K / gridDim.x);
            const int k1 = (int)((long long)(blockIdx.x + 1) * L.K / gridDim.x);
            const int w = k1 - k0;
            if (w > 0)
                for (int e = ctid; e < Mloc * w; e += 256) {  // independent elements: loads overlap
                    const int m = e / w, k = k0 + (e - m * w);
                    p.resid[(size_t)(m0 + m) * p.ld_src + k] = srcrow(m)[k];
                }
        }
        // rows are read as float4 when K and the row stride allow it
        const bool v4 = (L.K % 4 == 0) && (embed || p.ld_src % 4 == 0);
        if (pre) {
            // exponents from wide_digits (one per row over the whole K)
            if (ctid < MB) {
                rowinv[ctid] = 1.0f;
                rowex[ctid] = ctid < Mloc ? p.rowex_g[m0 + ctid] : 0;
            }
            named_bar_sync(1, 256);
        } else {
        // Tensor.swift:1538-1558: ss = sum x^2; inv = 1 / sqrt(ss/H + eps).  The
        // INT8 path also needs max |x| over this CTA's k range (digit scale).
        // One pass over the source, rows in parallel (WPR warps per row, each a
        // slice of it): the sum of squares over the whole row and the CTA's k
        // range staged into shared memory (zero past K), so the digit pass
        // reads no global memory.  Per-row 1/rms and digit exponents go to
        // shared memory (rowinv, rowex).
        const int kq = kspan / 4;  // float4 groups of the staged range
        constexpr int WPR = MB >= 8 ? 1 : 8 / MB;
        constexpr int RS = 8 / WPR;  // rows in flight
        const int sw = warp % WPR;
        __syncwarp();
        named_bar_sync(1, 256);  // norm weights staged
        for (int m = warp / WPR; m < MB; m += RS) {
            float ss = 0.0f, mx = 0.0f;
            float* xr = xs + (size_t)m * kspan;
            if (m < Mloc) {
                const float* sr = srcrow(m);
                if (rms) {
                    if (v4) {
                        for (int k = 4 * (sw * 32 + lane); k < L.K; k += 128 * WPR) {
                            const float4 a = pull ? pull4(m, k) : *reinterpret_cast<const float4*>(sr + k);
                            if (hout) *reinterpret_cast<float4*>(p.ar_hout + (size_t)(m0 + m) * p.ld_src + k) = a;
                            ss = fmaf(a.x, a.x, ss);
                            ss = fmaf(a.y, a.y, ss);
                            ss = fmaf(a.z, a.z, ss);
                            ss = fmaf(a.w, a.w, ss);
                        }
                    } else {
                        for (int k = sw * 32 + lane; k < L.K; k += 32 * WPR) ss = fmaf(sr[k], sr[k], ss);
                    }
                }
                for (int g = sw * 32 + lane; g < kq; g += 32 * WPR) {
                    const int k = kbeg + 4 * g;
                    float4 a;
                    if (v4 && k + 3 < L.K) {
                        a = pull ? pull4(m, k) : *reinterpret_cast<const float4*>(sr + k);
                    } else {
                        a.x = k < L.K ? sr[k] : 0.0f;
                        a.y = k + 1 < L.K ? sr[k + 1] : 0.0f;
                        a.z = k + 2 < L.K ? sr[k + 2] : 0.0f;
                        a.w = k + 3 < L.K ? sr[k + 3] : 0.0f;
                    }
                    if (!WIDE) *reinterpret_cast<float4*>(xr + 4 * g) = a;
                    if (PREC == 8) {
                        if (rms) {
                            const float4 w = *reinterpret_cast<const float4*>(wstage + 4 * g);
                            a = make_float4(__fmul_rn(a.x, w.x), __fmul_rn(a.y, w.y), __fmul_rn(a.z, w.z),
                                            __fmul_rn(a.w, w.w));
                        }
                        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
                    }
                }
            } else if (!WIDE) {
                for (int g = sw * 32 + lane; g < kq; g += 32 * WPR)
                    *reinterpret_cast<float4*>(xr + 4 * g) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                ss += __shfl_xor_sync(0xffffffffu, ss, o);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            if (lane == 0) {
                misc[m * 8 + sw] = ss;
                misc[(MB + m) * 8 + sw] = mx;
            }
        }
        named_bar_sync(1, 256);
        if (ctid < MB) {
            const int m = ctid;
            float ss = 0.0f, mx = 0.0f;
            for (int w = 0; w < WPR; ++w) {
                ss += misc[m * 8 + w];
                mx = fmaxf(mx, misc[(MB + m) * 8 + w]);
            }
            const float iv = rms ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)L.K), p.eps))) : 1.0f;
            rowinv[m] = iv;
            // x = src * w * inv and inv > 0: max |x| = max |src * w| * inv (one rounding above)
            rowex[m] = digit_exponent(__fmul_rn(mx, iv) * 1.0000002f);
        }
        named_bar_sync(1, 256);
        }
        // four consecutive staged k (g = (k - kbeg) / 4), normalised as the
        // reference does: (x * inv) * w
        auto xval4 = [&](int m, int g) -> float4 {
            float4 a = *reinterpret_cast<const float4*>(xs + (size_t)m * kspan + 4 * g);
            if (rms) {
                const float4 w = *reinterpret_cast<const float4*>(wstage + 4 * g);
                const float iv = rowinv[m];
                a = make_float4(__fmul_rn(__fmul_rn(a.x, iv), w.x), __fmul_rn(__fmul_rn(a.y, iv), w.y),
                                __fmul_rn(__fmul_rn(a.z, iv), w.z), __fmul_rn(__fmul_rn(a.w, iv), w.w));
            }
            return a;
        };

        if constexpr (WIDE) {
            // ---- wide INT8: digits of each unit's 128 k for all rows, per B slot ----
            // warp w: batch rows 8w + lane / 4; lane % 4 picks the 4-k word of
            // each 16-k chunk (8 chunks per unit); x read from global, the next
            // unit's values prefetched while this unit's digits are written
            static_assert(MB == 64, "wide batches are 64 rows per CTA");
            const int m = 8 * warp + (lane >> 2);
            const int kw = lane & 3;
            float4 xv[8];
            const float* sr = m < Mloc ? srcrow(m) : nullptr;
            auto load_unit = [&](int i) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const int k = kbeg + i * kTcUnitK + 16 * c + 4 * kw;
                    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (sr) {
                        if (v4 && k + 3 < L.K) {
                            a = *reinterpret_cast<const float4*>(sr + k);
                        } else {
                            a.x = k < L.K ? sr[k] : 0.0f;
                            a.y = k + 1 < L.K ? sr[k + 1] : 0.0f;
                            a.z = k + 2 < L.K ? sr[k + 2] : 0.0f;
                            a.w = k + 3 < L.K ? sr[k + 3] : 0.0f;
                        }
                    }
                    xv[c] = a;
                }
            };
            const float iv = rowinv[m];
            const float dscale = __int_as_float((127 - rowex[m]) << 23);
            if (!pre && nunits > 0) load_unit(0);
            for (int i = 0; !pre && i < nunits; ++i) {
                const int sl = i % kWideSlots;
                int ok = 1;
                if (lane == 0 && i >= kWideSlots)
                    ok = mbar_wait(&s_free[sl], (uint32_t)((i / kWideSlots) - 1) & 1u, p.err) ? 1 : 0;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                float4 cur[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) cur[c] = xv[c];
                if (i + 1 < nunits) load_unit(i + 1);
                uint8_t* bs = xbuf + (size_t)sl * wide_lbo(NB) * 8;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    float4 a = cur[c];
                    if (rms) {
                        const float4 w = *reinterpret_cast<const float4*>(wstage + i * kTcUnitK + 16 * c + 4 * kw);
                        a = make_float4(__fmul_rn(__fmul_rn(a.x, iv), w.x), __fmul_rn(__fmul_rn(a.y, iv), w.y),
                                        __fmul_rn(__fmul_rn(a.z, iv), w.z), __fmul_rn(__fmul_rn(a.w, iv), w.w));
                    }
                    put_digits4_strided(bs, wide_lbo(NB), kWideSbo, 16 * c + 4 * kw, m, a, dscale);
                }
                fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_ready[sl]);
            }
            if (ctid == 0) trace_max(p.trace, 3);
            // epilogue: all 8 warps read the accumulator, 32 columns (8 batch
            // rows) at a time; warps w and w + 4 share TMEM lanes 32 (w % 4)..
            // and take alternate column chunks
            {
                const uint32_t tmem = *tmem_slot;
                const bool okd = mbar_wait(&done[0], 0, p.err);
                if (lane == 0) trace_max(p.trace, 4);
                tc_fence_after();
                const int wq = warp & 3;
                const int row = 32 * wq + lane;
#pragma unroll 1
                for (int c = warp >> 2; c < NB / 32; c += 2) {
                    int d[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * wq) << 16) + (uint32_t)(32 * c), d);
                    tmem_ld_wait();
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int m = 8 * c + u;
                        red[row * RS + m] = okd ? combine_digits(d + kTcDigits * u, rowex[m]) : 0.0f;
                    }
                }
                tc_fence_before();
            }
        } else if constexpr (PREC == 8) {
            // Digits of x[m][kbeg:kend) into the B operand, 4 consecutive k per thread.
            const int ngroups = (kend - kbeg) / 4;
            for (int g = ctid; g < ngroups; g += 256) {
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    put_digits4(xd, NB, 4 * g, m, xval4(m, g), __int_as_float((127 - rowex[m]) << 23));
                }
                if (NB > kTcDigits * MB) {  // unused digit rows read as zero
                    uint8_t* base = xd + (size_t)(g >> 2) * NB * 16 + (4 * g & 15);
                    for (int row = kTcDigits * MB; row < NB; ++row)
                        *reinterpret_cast<uint32_t*>(base + (row >> 3) * 128 + (row & 7) * 16) = 0u;
                }
            }
            fence_proxy_async_shared();
            named_bar_sync(1, 256);
            if (ctid == 0) trace_max(p.trace, 3);
            const uint32_t tmem = *tmem_slot;
            if (warp == 0) {
                tc_fence_after();
                if (lane == 0) {
                    for (int i = 0; i < nunits; ++i) {
                        const int st = i % STAGES;
                        if (!mbar_wait(&full[st], (i / STAGES) & 1, p.err)) break;
                        if (i == 0) trace_max(p.trace, 7);
                        tc_fence_after();
                        tc_unit_mma(tmem, smem_u32(stage_base + st * Cfg::kStageBytes),
                                    smem_u32(xd + (size_t)i * (kTcUnitK / 16) * NB * 16), NB, i > 0);
                        tc_commit(&empty[st]);
                    }
                    tc_commit(&done[0]);
                }
                __syncwarp();
            } else if (warp >= 4) {
                // Epilogue warps: TMEM lanes 32 * (warp - 4) .. +31 = tile rows.
                const bool okd = mbar_wait(&done[0], 0, p.err);
                if (warp == 4 && lane == 0) trace_max(p.trace, 4);
                tc_fence_after();
                int d[NB];
#pragma unroll
                for (int c8 = 0; c8 < NB / 8; ++c8) {
                    int t[8];
                    tmem_ld8(tmem + ((uint32_t)(32 * (warp - 4)) << 16) + 8 * c8, t);
#pragma unroll
                    for (int i = 0; i < 8; ++i) d[8 * c8 + i] = t[i];
                }
                tmem_ld_wait();
                const int row = 32 * (warp - 4) + lane;
#pragma unroll
                for (int m = 0; m < MB; ++m) red[row * RS + m] = okd ? combine_digits(d + kTcDigits * m, rowex[m]) : 0.0f;
                tc_fence_before();
            }
        } else {
            // ---- INT4 on the tensor cores ----
            // (1) x[m][kbeg:kend) (normalised) into shared memory, and the
            //     largest |x| of every unit (one warp covers one unit per pass).
            const int ngroups = kspan / 4;
            for (int g = ctid; g < ngroups; g += 256) {
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    const float4 v = xval4(m, g);  // zero past K (and past this CTA's units)
                    *reinterpret_cast<float4*>(xs + (size_t)m * kspan + 4 * g) = v;
                    float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    const int u = g >> 5;  // 32 float4 per unit
                    if (lane == 0 && u < nunits) xmax[u * MB + m] = mx;
                }
            }
            named_bar_sync(1, 256);
            // (2) digit exponent of every (batch row, row group): |scale * x| is
            //     bounded by the per-unit maxima (one rounding margin).
            if (ctid < MB * kQ4Groups) {
                const int m = ctid >> 2, g = ctid & 3;
                float b = 0.0f;
                for (int u = 0; u < nunits; ++u) b = fmaxf(b, __fmul_rn(smaxs[g * nunits + u], xmax[u * MB + m]));
                ex4[ctid] = digit_exponent(b * 1.0000004f);
            }
            named_bar_sync(1, 256);
            if (ctid == 0) trace_max(p.trace, 3);
            // (3) a four-deep slot pipeline: warps 0-3 expand each unit's
            //     nibbles into an A slot in tensor memory (warp w owns TMEM
            //     lanes 32w..32w+31 = tile rows), warps 4-7 write the digits of
            //     scale * x into the matching B slot, and the issue warp runs
            //     the four K = 32 products once both are ready.  Lane 0 of each
            //     warp waits (bounded) and broadcasts the outcome, so a timed-out
            //     wait ends the warp's loop as a whole.
            const uint32_t tmem = *tmem_slot;
            const int wq = warp & 3;
            const bool arole = warp < 4;
            const uint32_t lane_base = (uint32_t)(32 * wq) << 16;
            // pipeline probes: CTA 0, lane 0 of warps 0 (A) and 4 (B)
            unsigned long long* prb =
                (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && (warp == 0 || warp == 4) && lane == 0) ? p.trace
                                                                                                      : nullptr;
            long long c0 = 0;
            uint32_t a[32];  // A role: the unit's int8 row, stored to tensor memory
            for (int i = 0; i < nunits; ++i) {
                const int st = i % STAGES;
                const int sl = i % kQ4Slots;
                int ok = 1;
                if (lane == 0) {
                    if (prb) c0 = clock64();
                    ok = mbar_wait(&full[st], (i / STAGES) & 1, p.err) ? 1 : 0;
                    if (prb && arole) atomicAdd(prb + 8, (unsigned long long)(clock64() - c0));
                    if (prb) c0 = clock64();
                    if (ok && i >= kQ4Slots) ok = mbar_wait(&s_free[sl], ((i / kQ4Slots) - 1) & 1, p.err) ? 1 : 0;
                    if (prb && arole) atomicAdd(prb + 9, (unsigned long long)(clock64() - c0));
                    if (prb) c0 = clock64();
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                const uint8_t* ust = stage_base + st * Cfg::kStageBytes;
                if (arole) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 w = *reinterpret_cast<const uint4*>(ust + (c * kTcTileRows + 32 * wq + lane) * 16);
                        q4_expand(w.x, a[8 * c + 0], a[8 * c + 1]);
                        q4_expand(w.y, a[8 * c + 2], a[8 * c + 3]);
                        q4_expand(w.z, a[8 * c + 4], a[8 * c + 5]);
                        q4_expand(w.w, a[8 * c + 6], a[8 * c + 7]);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
                    if (prb) {
                        atomicAdd(prb + 10, (unsigned long long)(clock64() - c0));
                        c0 = clock64();
                    }
                    // complete the previous unit's store (its latency overlapped
                    // this unit's waits and expansion), then issue this one's
                    if (i > 0) {
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_ready[(i - 1) % kQ4Slots]);
                    }
                    tmem_st32(tmem + lane_base + (uint32_t)(sl * 32), a);
                    if (prb) {
                        atomicAdd(prb + 11, (unsigned long long)(clock64() - c0));
                        atomicAdd(prb + 15, 1ull);
                    }
                } else {
                    // 4 consecutive k (quad q) of row group wq for every batch row
                    const int q = lane;
                    const float4 sc =
                        *reinterpret_cast<const float4*>(ust + kQ4UnitNibBytes + (wq * kTcUnitK + 4 * q) * 4);
                    uint8_t* bs = bslots + (size_t)sl * NB * 128;
#pragma unroll
                    for (int m = 0; m < MB; ++m) {
                        const float4 x = *reinterpret_cast<const float4*>(xs + (size_t)m * kspan + i * kTcUnitK + 4 * q);
                        const float4 v = make_float4(__fmul_rn(sc.x, x.x), __fmul_rn(sc.y, x.y), __fmul_rn(sc.z, x.z),
                                                     __fmul_rn(sc.w, x.w));
                        put_digits4(bs, NB, 4 * q, m * kQ4Groups + wq, v,
                                    __int_as_float((127 - ex4[m * kQ4Groups + wq]) << 23));
                    }
                    fence_proxy_async_shared();
                    __syncwarp();  // every lane has used its scales: the stage may be refilled
                    if (lane == 0) {
                        mbar_arrive(&empty[st]);
                        mbar_arrive(&b_ready[sl]);
                    }
                    if (prb) atomicAdd(prb + 14, (unsigned long long)(clock64() - c0));
                }
            }
            if (arole && nunits > 0) {  // the last unit's store
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_ready[(nunits - 1) % kQ4Slots]);
            }
            // (4) epilogue: warps 0-3 read the accumulator; lane row 32 * wq +
            //     lane belongs to row group wq.
            if (arole) {
                bool okd = true;
                if (nunits > 0) okd = mbar_wait(&done[0], 0, p.err);
                if (lane == 0) trace_max(p.trace, 4);
                tc_fence_after();
                const int row = 32 * wq + lane;
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    int d[4] = {0, 0, 0, 0};
                    if (nunits > 0)
                        tmem_ld4(tmem + lane_base + (uint32_t)(kQ4Slots * 32 + (m * kQ4Groups + wq) * kTcDigits), d);
                    tmem_ld_wait();
                    red[row * RS + m] = okd ? combine_digits(d, ex4[m * kQ4Groups + wq]) : 0.0f;
                }
                tc_fence_before();
            }
        }
    }

    // Make every CTA's partial row sums visible cluster-wide.
    __syncwarp();
    if (P > 1)
        cluster_sync();
    else
        __syncthreads();
    if (warp == 0) {  // every tcgen05.ld of the epilogue completed before the barrier
        tc_fence_after();
        tmem_dealloc(*tmem_slot, kTmemCols);
    }

    // Epilogue threads: the 8 consumer warps, and in the wide variant also the
    // producer and tensor-core issue warps, idle once the products are done.
    constexpr int ET = WIDE ? (kGemvConsumerWarps + 2) * 32 : 256;
    static_assert(!WIDE || ET == gemv_threads(PREC, MB), "wide epilogue uses every warp");
    if (warp < ET / 32) {
        const int ctid = threadIdx.x;
        if (ctid == 0) trace_max(p.trace, 5);
        unsigned long long best_mine = 0ull;
        constexpr bool RMAJ = MB >= 16;  // row-major items (below)
        // The item loops below are instantiated once per epilogue kind (EPI a
        // compile-time constant): each loop then holds only its own kind's
        // code, small enough to stay in the instruction cache.  With one
        // loop for every kind the warps stalled on instruction fetch.
        auto epilogue_items = [&](auto epi_kind) {
        constexpr int EPI = decltype(epi_kind)::value;
        // Output items handled by this rank: a contiguous chunk.
        constexpr int HALF = RB / 2;  // fused gate/up: gate rows [0, HALF), up rows [HALF, RB)
        const int nout = (EPI == kEpiQkv || EPI == kEpiSiluMul) ? HALF : RB;
        const int ob = rank * nout / P, oe = (rank + 1) * nout / P;
        const int nitems = (oe - ob) * MB;
        uint32_t rbase[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) rbase[q] = (q < P) ? dsmem_map(red, q) : 0u;
        // Partial sums of a row from every rank: all loads issued before the
        // first add (one DSMEM round trip), then summed in rank order.
        auto rowsum = [&](int row, int m) -> float {
            if (P == 1) return red[row * RS + m];
            float v[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) v[q] = q < P ? dsmem_ld_f32(rbase[q] + (uint32_t)((row * RS + m) * 4)) : 0.0f;
            float s = 0.0f;
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (q < P) s += v[q];
            return s;
        };
        auto finish = [&](int gpu_row, float s) -> float {
            const int i = gpu_row - rb * RB;
            float v = (PREC == 8) ? __fmul_rn(s, rowsc[i]) : s;
            if (p.bias) v = __fadd_rn(v, rowbias[i]);
            return v;
        };
        const unsigned int ar_tag_push = (EPI == kEpiPush) ? *p.ar_step + 1u : 0u;
        // Item order.  Up to 8 batch rows per CTA: it = ctid + ET j maps to
        // batch row it % MB = ctid % MB (MB divides ET), one argmax key per
        // thread.  From 16 rows on ("row-major" items): batch row it / nr,
        // tile row it % nr (nr = rows of this rank), so a warp's stores go to
        // consecutive outputs of one batch row; the argmax is reduced per
        // item over the lanes that share a batch row.
        static_assert(ET % MB == 0, "batch rows per CTA divide the epilogue threads");
        const int nr = oe - ob;
        // (batch row, tile-row offset) of item it = ctid + ET j, stepped by
        // ET items at a time without divisions
        const int step_m = RMAJ ? ET / nr : 0, step_o = RMAJ ? ET % nr : ET / MB;
        auto item_next = [&](int& m, int& o) {
            o += step_o;
            m += step_m;
            if (RMAJ && o >= nr) {
                o -= nr;
                ++m;
            }
        };
        // Row-major batches first gather every finished row value of this
        // rank into shared memory in batch-row-minor order (consecutive lanes
        // read consecutive partial sums of every rank: coalesced DSMEM
        // requests), then the item loop below reads them back row-major (its
        // global loads and stores coalesce).  Staging [MB][SR] reuses the
        // weight ring, idle once the accumulators are complete.
        const bool pairs = EPI == kEpiQkv || EPI == kEpiSiluMul;
        const int nloc = pairs ? 2 * nr : nr;  // tile rows of this rank
        const int SR = nloc + 1;
        float* stg = reinterpret_cast<float*>(stage_base);
        (void)SR;  // (unused by the batch-minor item order)
        (void)stg;
        auto loc_row = [&](int li) -> int {  // tile row of local index li
            if (EPI == kEpiQkv) return 2 * ob + li;
            if (EPI == kEpiSiluMul) return li < nr ? ob + li : HALF + ob + (li - nr);
            return ob + li;
        };
        if constexpr (RMAJ) {
            static_assert(!RMAJ || MB * (RB + 1) * 4 <= STAGES * Cfg::kStageBytes, "staging fits the ring");
            // (a plain loop: unrolling it was measured slower, instruction
            // fetch of a large straight-line body)
#pragma unroll 1
            for (int it = ctid; it < nloc * MB; it += ET) {
                const int m = it % MB, li = it / MB;
                const int row = loc_row(li);
                stg[m * SR + li] = finish(rb * RB + row, rowsum(row, m));
            }
            named_bar_sync(1, ET);
            if (PREC == 8 && ctid == 0) trace_max(p.trace, 8);
        }
        // finished value of tile row `row`, batch row m
        auto rowval = [&](int row, int m) -> float {
            if constexpr (RMAJ) {
                int li;
                if (EPI == kEpiQkv) li = row - 2 * ob;
                else if (EPI == kEpiSiluMul) li = row < HALF ? row - ob : nr + (row - HALF - ob);
                else li = row - ob;
                return stg[m * SR + li];
            } else {
                return finish(rb * RB + row, rowsum(row, m));
            }
        };

        // Two phases per chunk of JC items, so that every global load of a
        // chunk is in flight together: (1) reduce, scale, issue the loads the
        // stores need (RoPE table, the residual); (2) finish and store.
        constexpr int JMAX = (RB * MB + ET - 1) / ET;
        constexpr int JC = JMAX < 2 ? JMAX : 2;
        int cm = RMAJ ? ctid / nr : ctid % MB, co = RMAJ ? ctid % nr : ctid / MB;
#pragma unroll 1
        for (int jb = 0; jb < JMAX; jb += JC) {
        if ((ctid & ~31) + ET * jb >= nitems) break;  // warp-uniform: the argmax below uses whole warps
        float va[JC], vb[JC], old[JC];
        float2 cs[JC];
        unsigned long long keyj[JC];
        int keym[JC], mj[JC], oj[JC];
#pragma unroll
        for (int j = 0; j < JC; ++j) {
            keyj[j] = 0ull;
            keym[j] = -1;
            va[j] = vb[j] = old[j] = 0.0f;
            cs[j] = make_float2(1.0f, 0.0f);
            mj[j] = cm;
            oj[j] = ob + co;
            item_next(cm, co);
            const int it = ctid + ET * (jb + j);
            if (it >= nitems) continue;
            const int m = mj[j];
            const int o = oj[j];
            if (m >= Mloc) continue;
            if (EPI == kEpiQkv) {
                const int n0 = rb * RB + 2 * o;
                if (n0 >= L.N) continue;
                va[j] = rowval(2 * o, m);
                vb[j] = rowval(2 * o + 1, m);
                const int pos = seqinfo[m];
                if (seqinfo[MB + m] && n0 < p.H + p.kv_dim && pos < p.rope_max_pos) {
                    const int i = (n0 < p.H ? n0 : n0 - p.H) % p.head_dim;
                    cs[j] = p.rope[(size_t)pos * (p.head_dim / 2) + i / 2];
                }
            } else if (EPI == kEpiSiluMul) {
                if (rb * HALF + o >= L.N) continue;
                va[j] = rowval(o, m);
                vb[j] = rowval(HALF + o, m);
            } else {
                const int n = rb * RB + o;
                if (n >= L.N) continue;
                va[j] = rowval(o, m);
                if (EPI == kEpiResidual) old[j] = p.out[(size_t)(m0 + m) * p.ld_out + n];
            }
        }
#pragma unroll
        for (int j = 0; j < JC; ++j) {
            const int it = ctid + ET * (jb + j);
            if (it >= nitems) continue;
            const int m = mj[j];
            const int o = oj[j];
            if (m >= Mloc) continue;
            const int gm = m0 + m;  // batch row
            if (EPI == kEpiQkv) {
                const int n0 = rb * RB + 2 * o;
                if (n0 >= L.N || !seqinfo[MB + m]) continue;
                const int pos = seqinfo[m];
                const int d = p.head_dim;
                const float v0 = va[j], v1 = vb[j];
                if (n0 < p.H + p.kv_dim) {
                    const int i = (n0 < p.H ? n0 : n0 - p.H) % d;
                    // ModelRunner.swift:488-489
                    const float r0 = __fsub_rn(__fmul_rn(v0, cs[j].x), __fmul_rn(v1, cs[j].y));
                    const float r1 = __fadd_rn(__fmul_rn(v0, cs[j].y), __fmul_rn(v1, cs[j].x));
                    if (n0 < p.H) {
                        p.out[(size_t)gm * p.ld_out + n0] = r0;
                        p.out[(size_t)gm * p.ld_out + n0 + 1] = r1;
                        continue;
                    }
                    const int jj = n0 - p.H;
                    const int page = seqinfo[2 * MB + m];
                    if (page < 0) {
                        record_error(p.err, kDevBadPage);
                        continue;
                    }
                    const size_t base =
                        ((((size_t)page * p.num_layers + p.layer) * 2 + 0) * p.Hkv + jj / d) * kPageTokens +
                        pos % kPageTokens;
                    p.kv_pool[base * d + i] = r0;
                    p.kv_pool[base * d + i + 1] = r1;
                } else {
                    const int jj = n0 - p.H - p.kv_dim;
                    const int page = seqinfo[2 * MB + m];
                    if (page < 0) {
                        record_error(p.err, kDevBadPage);
                        continue;
                    }
                    const size_t base =
                        ((((size_t)page * p.num_layers + p.layer) * 2 + 1) * p.Hkv + jj / d) * kPageTokens +
                        pos % kPageTokens;
                    p.kv_pool[base * d + jj % d] = v0;
                    p.kv_pool[base * d + jj % d + 1] = v1;
                }
            } else if (EPI == kEpiSiluMul) {
                const int n = rb * HALF + o;
                if (n >= L.N) continue;
                p.out[(size_t)gm * p.ld_out + n] = __fmul_rn(silu_ref(va[j]), vb[j]);
            } else {
                const int n = rb * RB + o;
                if (n >= L.N) continue;
                const float v = va[j];
                if (EPI == kEpiStore) {
                    p.out[(size_t)gm * p.ld_out + n] = v;
                } else if (EPI == kEpiPush) {
                    const size_t off = ((size_t)p.ar_push_slot * p.ar_world + p.ar_rank) * p.ar_slot_words +
                                       (size_t)gm * p.ld_out + n;
                    const unsigned long long word = ((unsigned long long)ar_tag_push << 32) | __float_as_uint(v);
                    for (int q = 0; q < p.ar_world; ++q) st_relaxed_sys_u64(p.ar_peers[q] + off, word);
                } else if (EPI == kEpiResidual) {
                    p.out[(size_t)gm * p.ld_out + n] = __fadd_rn(old[j], v);
                } else if (EPI == kEpiGelu) {
                    p.out[(size_t)gm * p.ld_out + n] = gelu_ref(v);
                } else {  // kEpiArgmax
                    if (p.logits) p.logits[(size_t)gm * L.N + n] = v;
                    const unsigned long long key = argmax_key(v, n);
                    if (RMAJ) {
                        keyj[j] = key;
                        keym[j] = m;
                    } else if (key > best_mine) {
                        best_mine = key;
                    }
                }
            }
        }
        if (RMAJ && EPI == kEpiArgmax) {
            // lanes of one batch row are contiguous: per distinct row in the
            // warp, a full-warp max over its lanes' keys, one atomic
#pragma unroll
            for (int j = 0; j < JC; ++j) {
                unsigned pending = __ballot_sync(0xffffffffu, keym[j] >= 0);
                while (pending) {
                    const int leader = __ffs(pending) - 1;
                    const int target = __shfl_sync(0xffffffffu, keym[j], leader);
                    unsigned long long v = keym[j] == target ? keyj[j] : 0ull;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
                        v = t > v ? t : v;
                    }
                    if (lane == leader && v != 0ull) atomicMax(&p.seq[m0 + target].best, v);
                    pending &= ~__ballot_sync(0xffffffffu, keym[j] == target);
                }
            }
        }
        }  // item chunks
        };
        switch (p.epilogue) {
            case kEpiStore: epilogue_items(std::integral_constant<int, kEpiStore>{}); break;
            case kEpiResidual: epilogue_items(std::integral_constant<int, kEpiResidual>{}); break;
            case kEpiQkv: epilogue_items(std::integral_constant<int, kEpiQkv>{}); break;
            case kEpiSiluMul: epilogue_items(std::integral_constant<int, kEpiSiluMul>{}); break;
            case kEpiGelu: epilogue_items(std::integral_constant<int, kEpiGelu>{}); break;
            case kEpiArgmax: epilogue_items(std::integral_constant<int, kEpiArgmax>{}); break;
            case kEpiPush: epilogue_items(std::integral_constant<int, kEpiPush>{}); break;
            default: break;  // the host passes only the kinds above
        }
        if (PREC == 8 && ctid == 0) trace_max(p.trace, 9);
        if (p.epilogue == kEpiArgmax) {
            // lanes with the same batch row (lane % MB) combine, then one atomic per row and warp
            if (!RMAJ) {
                unsigned long long b = best_mine;
#pragma unroll
                for (int o = 16; o >= MB; o >>= 1) {
                    unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
                    b = t > b ? t : b;
                }
                const int m = ctid % MB;
                if (lane < MB && b != 0ull && m < Mloc) atomicMax(&p.seq[m0 + m].best, b);
            }
            named_bar_sync(1, ET);
            if (ctid == 0) {
                __threadfence();
                const unsigned int t = atomicAdd(p.ticket, 1u);
                misc[0] = __int_as_float(t == gridDim.x * gridDim.y - 1 ? 1 : 0);
            }
            named_bar_sync(1, ET);
            if (__float_as_int(misc[0]) == 1) {
                // Last CTA: finish the step for every sequence (ModelRunner.swift:251-292).
                __threadfence();
                for (int m = ctid; m < p.M; m += ET) {
                    SeqState& sq = p.seq[m];
                    if (!sq.active) {
                        sq.best = 0ull;  // paused slot: drop this step's argmax
                        continue;
                    }
                    finish_sequence_step(sq, m, p.out_tokens, p.prompt, p.prompt_stride);
                }
                if (ctid == 0) {
                    *p.ticket = 0u;
                    if (p.ar_step) *p.ar_step += 1u;  // tensor parallel: the step's pulls are done
                }
            }
        }
    }
    __syncwarp();
    if (threadIdx.x == 0) trace_max(p.trace, 6);
    if (P > 1) cluster_sync();
}

// Digit operand of a wide INT8 GEMV, once per launch: one CTA per batch row
// runs the GEMV's prologue over the whole K (embedding gather or source row,
// RMSNorm as Tensor.swift:1538-1558), takes one digit exponent for the row
// and writes the row's four digit planes into every unit's B image, laid out
// exactly as the GEMV's shared-memory B slot (so one bulk copy moves it).
__global__ void __launch_bounds__(256) wide_digits_kernel(const __grid_constant__ GemvParams p) {
    constexpr int NB = 256;  // tc_nb(64)
    __shared__ float red[2][8];
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const QLayout& L = p.L;
    // CTA (m, c) writes the digit planes of units [u0, u1); every CTA of a row
    // reduces the whole row (the same sums in the same order, so all chunks
    // agree on the row's exponent)
    const int u0 = blockIdx.y * L.slabs / gridDim.y, u1 = (blockIdx.y + 1) * L.slabs / gridDim.y;
    if (tid == 0) {
        trace_min(p.trace, 0);
        trace_max(p.trace, 1);
    }
    pdl_wait();
    pdl_launch_dependents();
    if (tid == 0) trace_max(p.trace, 2);
    const bool embed = p.prologue == kProEmbed || p.prologue == kProEmbedRms;
    const bool rms = p.prologue == kProRmsNorm || p.prologue == kProEmbedRms;
    const float* sr;
    if (embed) {
        int tok = p.seq_ro[m].token;
        if (tok < 0 || tok >= p.vocab) tok = 0;  // the GEMV records the error
        sr = p.embedding + (size_t)tok * L.K;
    } else {
        sr = p.src + (size_t)m * p.ld_src;
    }
    // one pass over the row: sum of squares and max |x * w| (the digit bound:
    // |(x * inv) * w| <= max |x * w| * inv up to two roundings, covered by the
    // margin below)
    float ss = 0.0f, mw = 0.0f;
    const bool v4 = (L.K % 4 == 0) && (embed || p.ld_src % 4 == 0);
    if (v4) {
        for (int q = tid; q < L.K / 4; q += 256) {
            const float4 a = *reinterpret_cast<const float4*>(sr + 4 * q);
            ss = fmaf(a.x, a.x, ss);
            ss = fmaf(a.y, a.y, ss);
            ss = fmaf(a.z, a.z, ss);
            ss = fmaf(a.w, a.w, ss);
            float4 b = a;
            if (rms) {
                const float4 w = *reinterpret_cast<const float4*>(p.norm_w + 4 * q);
                b = make_float4(__fmul_rn(a.x, w.x), __fmul_rn(a.y, w.y), __fmul_rn(a.z, w.z), __fmul_rn(a.w, w.w));
            }
            mw = fmaxf(mw, fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
        }
    } else {
        for (int k = tid; k < L.K; k += 256) {
            const float a = sr[k];
            ss = fmaf(a, a, ss);
            mw = fmaxf(mw, fabsf(rms ? __fmul_rn(a, p.norm_w[k]) : a));
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
        mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, o));
    }
    if (lane == 0) {
        red[0][warp] = ss;
        red[1][warp] = mw;
    }
    __syncthreads();
    float tot = 0.0f, bw = 0.0f;
    for (int w = 0; w < 8; ++w) {
        tot += red[0][w];
        bw = fmaxf(bw, red[1][w]);
    }
    const float iv = rms ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)L.K), p.eps))) : 1.0f;
    auto xval = [&](int k) -> float {
        if (k >= L.K) return 0.0f;
        float a = sr[k];
        if (rms) a = __fmul_rn(__fmul_rn(a, iv), p.norm_w[k]);
        return a;
    };
    const float bmax = rms ? __fmul_rn(bw, iv) * 1.0000004f : bw;
    const int ex = digit_exponent(bmax);
    if (tid == 0 && blockIdx.y == 0) p.rowex_g[m] = ex;
    const float dscale = __int_as_float((127 - ex) << 23);
    constexpr uint32_t kBBytes = wide_lbo(NB) * 8;
    for (int q = u0 * (kTcUnitK / 4) + tid; q < u1 * (kTcUnitK / 4); q += 256) {  // 4 consecutive k per step
        const int k = 4 * q;
        float4 a;
        if (v4 && k + 3 < L.K) {
            a = *reinterpret_cast<const float4*>(sr + k);
            if (rms) {
                const float4 w = *reinterpret_cast<const float4*>(p.norm_w + k);
                a = make_float4(__fmul_rn(__fmul_rn(a.x, iv), w.x), __fmul_rn(__fmul_rn(a.y, iv), w.y),
                                __fmul_rn(__fmul_rn(a.z, iv), w.z), __fmul_rn(__fmul_rn(a.w, iv), w.w));
            }
        } else {
            a = make_float4(xval(k), xval(k + 1), xval(k + 2), xval(k + 3));
        }
        put_digits4_strided(p.bimg + (size_t)(k / kTcUnitK) * kBBytes, wide_lbo(NB), kWideSbo, k % kTcUnitK, m, a,
                            dscale);
    }
    __syncthreads();
    if (tid == 0) trace_max(p.trace, 6);
}

// Staged activation bytes of a CTA: INT8 digits (NB per k); INT4 fp32 x,
// B slots, per-unit maxima and exponents.
inline size_t gemv_xbytes(int prec, int mb, const QLayout& L, int P) {
    const size_t units = (size_t)((L.slabs + P - 1) / P);
    const size_t xw = units * kTcUnitK * (mb + 1) * 4;  // x and norm weights, fp32
    if (gemv_wide(prec, mb)) return (size_t)kWideSlots * wide_lbo(tc_nb(mb)) * 8 + units * kTcUnitK * 4;
    if (prec == 8) return units * kTcUnitK * (size_t)tc_nb(mb) + xw;
    return xw + (size_t)kQ4Slots * q4_nb(mb) * 128 + units * (mb + kQ4Groups) * 4 + (size_t)mb * kQ4Groups * 4;
}

template <int PREC, int RB, int MB>
size_t gemv_smem_bytes(const QLayout& L, int P) {
    using Cfg = GemvCfg<PREC, RB>;
    size_t head = (kGemvBarBytes + (size_t)gemv_head_floats(RB, MB) * 4 + 1023) / 1024 * 1024;
    size_t stages = (size_t)Cfg::kStages * Cfg::kStageBytes;
    return head + stages + gemv_xbytes(PREC, MB, L, P);
}

template <int PREC, int RB, int MB>
cudaError_t launch_t(const GemvParams& p, cudaStream_t stream, bool pdl) {
    const size_t smem = gemv_smem_bytes<PREC, RB, MB>(p.L, p.P);
    auto kfn = gemv_kernel<PREC, RB, MB>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // All of the SM's unified L1/shared storage as shared memory, so that two
    // CTAs (of this launch, or of this and the next launch) fit side by side.
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(p.L.Np / RB * p.P), (unsigned)((p.M + MB - 1) / MB), 1);
    cfg.blockDim = dim3(gemv_threads(PREC, MB), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = (unsigned)p.P;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
    if (pdl) {
        attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kfn, p);
}

// Clusters of P CTAs (one launch configuration of this kernel variant) that
// can be resident at once: a cluster needs P SMs of one GPC with room, so
// large clusters of large CTAs leave SMs unused; the occupancy API counts it.
template <int PREC, int RB, int MB>
int max_clusters_t(int P, size_t smem) {
    auto kfn = gemv_kernel<PREC, RB, MB>;
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)P, 1, 1);
    cfg.blockDim = dim3(gemv_threads(PREC, MB), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute a[1];
    a[0].id = cudaLaunchAttributeClusterDimension;
    a[0].val.clusterDim.x = (unsigned)P;
    a[0].val.clusterDim.y = 1;
    a[0].val.clusterDim.z = 1;
    cfg.attrs = a;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return n;
}

int max_clusters(int prec, int mb, int P, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int, size_t>, int> cache;
    int dev = 0;
    (void)cudaGetDevice(&dev);
    const auto key = std::make_tuple(dev, prec, mb, P, smem);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (prec == 8) {
        switch (mb) {
            case 1: n = max_clusters_t<8, 128, 1>(P, smem); break;
            case 2: n = max_clusters_t<8, 128, 2>(P, smem); break;
            case 4: n = max_clusters_t<8, 128, 4>(P, smem); break;
            case 8: n = max_clusters_t<8, 128, 8>(P, smem); break;
            case 16: n = max_clusters_t<8, 128, 16>(P, smem); break;
            default: n = max_clusters_t<8, 128, 64>(P, smem); break;
        }
    } else {
        switch (mb) {
            case 1: n = max_clusters_t<4, 128, 1>(P, smem); break;
            case 2: n = max_clusters_t<4, 128, 2>(P, smem); break;
            default: n = max_clusters_t<4, 128, 4>(P, smem); break;
        }
    }
    cache[key] = n;
    return n;
}

}  // namespace

bool gemv_uses_wide(int precision, int M) { return gemv_wide(precision, gemv_mb(precision, M)); }

size_t wide_digits_bytes(const QLayout& L) { return (size_t)L.slabs * wide_lbo(tc_nb(64)) * 8; }

cudaError_t launch_wide_digits(const GemvParams& p, cudaStream_t stream, bool pdl) {
    if (!p.bimg || !p.rowex_g || !gemv_uses_wide(p.L.precision, p.M)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)p.M, (unsigned)std::min(8, p.L.slabs));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, wide_digits_kernel, p);
}

int choose_ksplit(const QLayout& L, int M, int num_sms) {
    if (const char* e = getenv("TB_GEMV_P")) {  // tuning override: a fixed cluster size
        const int f = atoi(e);
        if (f > 0) return std::max(1, std::min(std::min(8, L.slabs), f));
    }
    // Pick the cluster size P (k split) so that every CTA of the launch is
    // resident at once (no second wave: a wave boundary costs a whole CTA
    // lifetime) while each CTA streams as few units as possible.
    const int nrb = L.Np / L.RB;
    const int mb = gemv_mb(L.precision, M);
    const int splits = (M + mb - 1) / mb;  // grid y
    const size_t head = (kGemvBarBytes + (size_t)gemv_head_floats(L.RB, mb) * 4 + 1023) / 1024 * 1024;
    const size_t stages = L.precision == 8 ? (size_t)GemvCfg<8, 128>::kStages * GemvCfg<8, 128>::kStageBytes
                                           : (size_t)GemvCfg<4, 128>::kStages * GemvCfg<4, 128>::kStageBytes;
    constexpr size_t kSmPerSm = 228 * 1024;  // shared memory per SM, 1 KB reserved per CTA
    // Time model (us): a wave costs a CTA lifetime of fixed latency (launch,
    // prologue, reduction, epilogue: ~4 us measured); within it a CTA needs
    // max(its own unit pipeline: ~0.15 us per INT8 unit, ~0.42 us per INT4
    // unit, measured; the SM's share of HBM bandwidth, ~44 KB/us, for the
    // units of all CTAs on that SM).
    constexpr double kWaveUs = 4.0, kSmKBperUs = 44.0;
    const double unit_us = gemv_wide(L.precision, mb) ? 0.5 : L.precision == 8 ? 0.15 : 0.42;
    const double unit_kb = (L.precision == 8 ? kTcUnitBytes : kQ4UnitBytes) / 1024.0;
    int best = 0;
    double best_cost = 0.0;
    for (int P = 1; P <= std::min(8, L.slabs); ++P) {
        const size_t xb = gemv_xbytes(L.precision, mb, L, P);
        if (xb > 96 * 1024) continue;
        const size_t smem = head + stages + xb;
        const int occ = (int)std::min<size_t>(2, kSmPerSm / (smem + 1024));  // TMEM and registers: at most 2
        if (occ < 1) continue;
        const long long ctas = (long long)nrb * P * splits;
        // A cluster needs P free SMs of one GPC: with one CTA per SM (the wide
        // variant) or clusters beyond 4 CTAs, count the co-resident clusters;
        // small clusters at two CTAs per SM were measured to fit as counted
        const int clusters = (occ == 1 || P > 4) ? max_clusters(L.precision, mb, P, smem) : 0;
        const long long cap = clusters > 0 ? (long long)clusters * P : (long long)occ * num_sms;
        const long long waves = (ctas + cap - 1) / cap;
        const long long per_sm = (ctas + num_sms - 1) / num_sms;
        const int units = (L.slabs + P - 1) / P;
        // + the epilogue, serial in each CTA: ~0.5 ns per output item (row x batch row)
        const double epi_us = (double)L.RB * mb / P * 0.0005;
        const double cost =
            waves * (kWaveUs + epi_us + std::max(units * unit_us, (double)per_sm * units * unit_kb / kSmKBperUs));
        if (getenv("TB_GEMV_DEBUG"))
            fprintf(stderr, "ksplit K=%d N=%d M=%d P=%d smem=%zu occ=%d clusters=%d ctas=%lld cap=%lld cost=%.2f\n",
                    L.K, L.N, M, P, smem, occ, clusters, ctas, cap, cost);
        if (best == 0 || cost < best_cost) {
            best = P;
            best_cost = cost;
        }
    }
    return best > 0 ? best : std::min(8, L.slabs);
}

int choose_ksplit_stream(const QLayout& L, int M) {
    // Independent GEMVs overlap their launches, so the grid need not fill the
    // GPU by itself: whole rows per CTA (no K split, no partial-sum combine)
    // stream the most bytes per fixed CTA cost.  The smallest split whose
    // activation staging fits.
    const int mb = gemv_mb(L.precision, M);
    for (int P = 1; P <= std::min(8, L.slabs); ++P)
        if (gemv_xbytes(L.precision, mb, L, P) <= 96 * 1024) return P;
    return std::min(8, L.slabs);
}

int gemv_grid_ctas(const GemvParams& p) {
    const int mb = gemv_mb(p.L.precision, p.M);
    return (p.L.Np / p.L.RB) * p.P * ((p.M + mb - 1) / mb);
}

cudaError_t launch_gemv(const GemvParams& p, cudaStream_t stream, bool pdl) {
    const int prec = p.L.precision;
    // batches beyond one CTA's rows (INT8 16, INT4 4) are split over grid y
    const int mb = gemv_mb(prec, p.M);
    if (p.M < 1 || p.M > kMaxGemvBatch || p.L.RB != kTcTileRows) return cudaErrorInvalidValue;
    if (prec == 8) {
        switch (mb) {
            case 1: return launch_t<8, 128, 1>(p, stream, pdl);
            case 2: return launch_t<8, 128, 2>(p, stream, pdl);
            case 4: return launch_t<8, 128, 4>(p, stream, pdl);
            case 8: return launch_t<8, 128, 8>(p, stream, pdl);
            case 16: return launch_t<8, 128, 16>(p, stream, pdl);
            default: return launch_t<8, 128, 64>(p, stream, pdl);
        }
    }
    if (prec == 4) {
        switch (mb) {
            case 1: return launch_t<4, 128, 1>(p, stream, pdl);
            case 2: return launch_t<4, 128, 2>(p, stream, pdl);
            default: return launch_t<4, 128, 4>(p, stream, pdl);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace tb
