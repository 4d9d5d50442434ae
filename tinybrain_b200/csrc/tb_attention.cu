// tb_attention.cu -- single-query decode attention over the HBM paged KV cache.
//
// Semantics follow the reference's live CPU path, ModelRunner.swift:519-579:
// per query head h, kvHead = h / (H/Hkv); scores = (q.k) * 1/sqrt(d); softmax
// without epsilon; context = sum_j p_j v_j.  Rows of evicted pages read as
// zeros and are still attended (KVCache.swift:239-253).  The reference's Metal
// FlashAttention kernel (Shaders/FlashAttention.metal:55-220) is the interface
// this replaces (AttentionBackend, Backend.swift:205-219), but it works on a
// contiguous cache; this kernel reads 16-token pages through a page table.
//
// Design (sm_100a): grid = (split, kv head, sequence).  A CTA serves all
// G = H/Hkv query heads of its KV head, so each K/V byte is read once.  One
// producer warp streams the K and V tiles of each page (16 x d fp32,
// contiguous) with 1-D bulk copies into an mbarrier ring; four consumer warps
// compute scores and an online softmax.  The splits of one (sequence, KV
// head) form a thread-block cluster: each keeps its (m, l, acc) partial in
// shared memory and, after a cluster barrier, combines a slice of the outputs
// from all splits' partials through distributed shared memory, in split order
// (deterministic; no global scratch, no tickets).  Pages older than the
// current position are complete before the step starts, so their copies are
// issued before the programmatic-dependent-launch wait; only the page holding
// the row the preceding QKV kernel appends waits for it.
#include "../../include/tinybrain_cuda.h"
#include "tb_common.cuh"
#include "tb_kernels.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

namespace tb {

namespace {

constexpr int kAttnConsumerWarps = 4;
constexpr int kAttnThreads = (kAttnConsumerWarps + 1) * 32;
// K/V ring depth: 96 KB of pages in flight per CTA (12 pages at d = 64, 6 at
// d = 128), so two CTAs share an SM and one wave holds MHA models' splits.
__host__ __device__ constexpr int attn_stages(int d) { return d >= 128 ? 6 : 12; }
constexpr int kAttnHead = 512;  // mbarriers + valid flags

template <int G, int D>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnParams p) {
    constexpr int TILE = kPageTokens * D;           // floats per K (or V) tile
    constexpr int DP = 128 / (G * kPageTokens);     // threads per (head, token) score
    constexpr int CHK = D / DP;                     // dims per score thread
    constexpr int PVT = G * (D / 4);                // threads active in the PV phase
    static_assert(DP >= 1 && CHK <= 64, "unsupported head geometry");
    constexpr int kAttnStages = attn_stages(D);
    static_assert(kAttnStages * 20 <= kAttnHead, "ring barriers exceed the header");

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kAttnStages;
    int* valid = reinterpret_cast<int*>(empty + kAttnStages);            // [stages]
    float* S = reinterpret_cast<float*>(smem + kAttnHead);              // [2][G][16] scores / weights
    float* Cb = S + 2 * G * kPageTokens;                                 // [2][G] running-max corrections
    float* tiles = reinterpret_cast<float*>(smem + kAttnHead + (((2 * G * kPageTokens + 2 * G) * 4 + 127) / 128) * 128);
    float* cpart = tiles + kAttnStages * 2 * TILE;  // [G][D + 4]: acc, m, l of this split

    const int split = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kAttnStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kAttnConsumerWarps);
        }
        fence_barrier_init();
    }
    if (threadIdx.x == 0) {
        trace_min(p.trace, 0);
        trace_max(p.trace, 1);
    }
    __syncthreads();
    pdl_launch_dependents();

    // The sequence state and page table are written before the step starts
    // (the previous step's last kernel, host uploads): readable before the wait.
    const SeqState& sq = p.seq[m];
    const bool active = p.lens ? true : (sq.active != 0);
    const int Lq = p.lens ? p.lens[m] : sq.pos + 1;
    const int npages = active ? (Lq + kPageTokens - 1) / kPageTokens : 0;
    const int pps = (npages + p.nsplit - 1) / p.nsplit;
    const int pg0 = min(npages, split * pps);
    const int pg1 = min(npages, pg0 + pps);
    const int nun = pg1 - pg0;

    if (warp == kAttnConsumerWarps) {
        // The whole warp walks the pages: 32 page-table entries are loaded at
        // a time, one per lane, so the copies are not serialised behind one
        // dependent global load each; lane 0 waits and issues.
        bool waited = false;
        int pt = -1;
        for (int i = 0; i < nun; ++i) {
            const int st = i % kAttnStages;
            if ((i & 31) == 0)
                pt = i + lane < nun ? p.page_table[(size_t)m * p.ptab_stride + pg0 + i + lane] : -1;
            const int page = __shfl_sync(0xffffffffu, pt, i & 31);
            int ok = 1;
            if (lane == 0 && i >= kAttnStages) ok = mbar_wait(&empty[st], ((i / kAttnStages) - 1) & 1, p.err);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            const int lp = pg0 + i;
            if ((p.wait_first || lp == npages - 1) && !waited) {  // pages the preceding kernel appends to
                pdl_wait();
                waited = true;
            }
            if (lane == 0) {
                float* kd = tiles + st * 2 * TILE;
                if (page >= 0) {
                    valid[st] = 1;
                    const size_t kbase =
                        ((((size_t)page * p.num_layers + p.layer) * 2 + 0) * p.Hkv + kvh) * (size_t)TILE;
                    const size_t vbase =
                        ((((size_t)page * p.num_layers + p.layer) * 2 + 1) * p.Hkv + kvh) * (size_t)TILE;
                    mbar_arrive_expect_tx(&full[st], 2u * TILE * 4u);
                    bulk_g2s(kd, p.kv_pool + kbase, TILE * 4u, &full[st]);
                    bulk_g2s(kd + TILE, p.kv_pool + vbase, TILE * 4u, &full[st]);
                } else {
                    valid[st] = 0;  // evicted page: rows read as zeros
                    mbar_arrive(&full[st]);
                }
            }
        }
    } else {
        pdl_wait();
        if (threadIdx.x == 0) trace_max(p.trace, 2);
        const int t = threadIdx.x;  // 0..127
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
        // Score-phase role.
        const int pair = t / DP, dp = t % DP;
        const int gq = pair / kPageTokens, j = pair % kPageTokens;
        const int head = kvh * G + gq;
        // q slice rotated by 4j (token j's start offset) so the 16 rows of a
        // page are read as conflict-spread float4s
        constexpr bool kVec = CHK % 4 == 0;
        // softmax weights computed by the score threads (a head's 16 tokens
        // within one warp) when G >= 4; otherwise by the PV threads
        constexpr bool kSoftInScore = 16 * DP <= 32;
        const int rot = kVec ? (4 * j) % CHK : j % CHK;
        float qrot[CHK];
        {
            const float* qh = p.q + (size_t)m * p.ld_q + (size_t)head * D + dp * CHK;
#pragma unroll
            for (int e = 0; e < CHK; ++e) qrot[e] = qh[(e + rot) % CHK];
        }
        // PV-phase role.
        const bool pv = t < PVT;
        const int gv = t / (D / 4), dv = (t % (D / 4)) * 4;
        float run_m = -INFINITY, run_l = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);

        // A timed-out wait marks the CTA bad: every warp still walks the same
        // barrier sequence (no warp is left waiting on a named barrier), skips
        // shared-memory reads, and the host sees the recorded error.
        bool bad = false;
        for (int i = 0; i < nun; ++i) {
            const int st = i % kAttnStages;
            if (!bad && !mbar_wait(&full[st], (i / kAttnStages) & 1, p.err)) bad = true;
            const float* Kt = tiles + st * 2 * TILE;
            const float* Vt = Kt + TILE;
            const bool ok = !bad && valid[st] != 0;
            float* Sb = S + (i & 1) * G * kPageTokens;
            {
                float dot = 0.0f;
                if (ok) {
                    // four partial sums (independent FMA chains), added pairwise
                    const float* kr = Kt + j * D + dp * CHK;
                    if constexpr (kVec) {
                        float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;
#pragma unroll
                        for (int e = 0; e < CHK; e += 4) {
                            const float4 k4 = *reinterpret_cast<const float4*>(kr + (e + rot) % CHK);
                            d0 = fmaf(qrot[e], k4.x, d0);
                            d1 = fmaf(qrot[e + 1], k4.y, d1);
                            d2 = fmaf(qrot[e + 2], k4.z, d2);
                            d3 = fmaf(qrot[e + 3], k4.w, d3);
                        }
                        dot = (d0 + d1) + (d2 + d3);
                    } else {
#pragma unroll
                        for (int e = 0; e < CHK; ++e) dot = fmaf(qrot[e], kr[(e + rot) % CHK], dot);
                    }
                }
#pragma unroll
                for (int o = DP / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
                const int tok = (pg0 + i) * kPageTokens + j;
                const float sc = (tok < Lq) ? __fmul_rn(dot, scale) : -INFINITY;
                if constexpr (kSoftInScore) {
                    // The 16 tokens of a head sit in 16 * DP consecutive lanes:
                    // page max and the weights' sum by shuffles, the head's
                    // running (m, l) in its first lane, one exp per token.
                    float pm = sc;
#pragma unroll
                    for (int o = 8 * DP; o >= DP; o >>= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o));
                    const int leader = lane & ~(16 * DP - 1);
                    const float mold = __shfl_sync(0xffffffffu, run_m, leader);
                    const float mnew = fmaxf(mold, pm);
                    const float corr = (mold == -INFINITY) ? 0.0f : expf(mold - mnew);
                    const float e = (sc == -INFINITY) ? 0.0f : expf(sc - mnew);
                    float ps = e;
#pragma unroll
                    for (int o = 8 * DP; o >= DP; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                    if (lane == leader) {
                        run_l = __fadd_rn(__fmul_rn(run_l, corr), ps);
                        run_m = mnew;
                        Cb[(i & 1) * G + gq] = corr;
                    }
                    if (dp == 0) Sb[gq * kPageTokens + j] = e;
                } else {
                    if (dp == 0) Sb[gq * kPageTokens + j] = sc;
                }
            }
            named_bar_sync(1, 128);
            if (kSoftInScore && pv) {
                const float* Sg = Sb + gv * kPageTokens;
                const float corr = Cb[(i & 1) * G + gv];
                float4 a = make_float4(acc.x * corr, acc.y * corr, acc.z * corr, acc.w * corr);
                if (ok) {
#pragma unroll
                    for (int jj = 0; jj < kPageTokens; ++jj) {
                        const float e = Sg[jj];
                        const float4 v = *reinterpret_cast<const float4*>(Vt + jj * D + dv);
                        a.x = fmaf(e, v.x, a.x);
                        a.y = fmaf(e, v.y, a.y);
                        a.z = fmaf(e, v.z, a.z);
                        a.w = fmaf(e, v.w, a.w);
                    }
                }
                acc = a;
            } else if (pv) {
                const float* Sg = Sb + gv * kPageTokens;
                float pm = Sg[0];
#pragma unroll
                for (int jj = 1; jj < kPageTokens; ++jj) pm = fmaxf(pm, Sg[jj]);
                const float mnew = fmaxf(run_m, pm);
                const float corr = (run_m == -INFINITY) ? 0.0f : expf(run_m - mnew);
                float l = run_l * corr;
                float4 a = make_float4(acc.x * corr, acc.y * corr, acc.z * corr, acc.w * corr);
#pragma unroll
                for (int jj = 0; jj < kPageTokens; ++jj) {
                    const float s = Sg[jj];
                    const float e = (s == -INFINITY) ? 0.0f : expf(s - mnew);
                    l += e;
                    if (ok) {
                        const float4 v = *reinterpret_cast<const float4*>(Vt + jj * D + dv);
                        a.x = fmaf(e, v.x, a.x);
                        a.y = fmaf(e, v.y, a.y);
                        a.z = fmaf(e, v.z, a.z);
                        a.w = fmaf(e, v.w, a.w);
                    }
                }
                run_m = mnew;
                run_l = l;
                acc = a;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }

        if (pv) {
            float* cp = cpart + gv * (D + 4);
            *reinterpret_cast<float4*>(cp + dv) = acc;
            if (!kSoftInScore && dv == 0) {
                cp[D] = run_m;
                cp[D + 1] = run_l;
            }
        }
        if (kSoftInScore && lane == (lane & ~(16 * DP - 1))) {  // head leaders hold (m, l)
            float* cp = cpart + gq * (D + 4);
            cp[D] = run_m;
            cp[D + 1] = run_l;
        }
    }
    // Combine the splits (cluster ranks) in split order; CTA `split` produces
    // output items [split * Q / ns, (split + 1) * Q / ns), Q = G * D / 4 float4s.
    const int ns = p.nsplit;
    if (ns > 1) cluster_sync();
    else __syncthreads();
    {
        constexpr int Q = G * (D / 4);
        const int t = threadIdx.x;
        const int i0 = split * Q / ns, i1 = (split + 1) * Q / ns;
        if (t < kAttnConsumerWarps * 32 && i0 + t < i1) {
            const int item = i0 + t;
            const int g = item / (D / 4), d4 = (item % (D / 4)) * 4;
            float* out = p.out + (size_t)m * p.ld_out + (size_t)(kvh * G + g) * D + d4;
            // every split's m first (one DSMEM round trip), then (l, acc) in
            // groups of 8 splits, combined in split order
            float mq[kMaxAttnSplits];
#pragma unroll
            for (int q = 0; q < kMaxAttnSplits; ++q)
                mq[q] = q < ns ? dsmem_ld_f32(dsmem_map(cpart + g * (D + 4) + D, (uint32_t)q)) : -INFINITY;
            float M = -INFINITY;
#pragma unroll
            for (int q = 0; q < kMaxAttnSplits; ++q) M = fmaxf(M, mq[q]);
            float den = 0.0f;
            float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
            if (M != -INFINITY) {
#pragma unroll
                for (int q0 = 0; q0 < kMaxAttnSplits; q0 += 8) {
                    if (q0 >= ns) break;
                    float lq[8];
                    float4 aq[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int q = q0 + u;
                        if (q < ns) {
                            const uint32_t base = dsmem_map(cpart + g * (D + 4), (uint32_t)q);
                            lq[u] = dsmem_ld_f32(base + (D + 1) * 4);
                            aq[u] = dsmem_ld_f32x4(base + d4 * 4);
                        } else {
                            lq[u] = 0.0f;
                            aq[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int q = q0 + u;
                        if (q >= ns) continue;
                        const float w = (mq[q] == -INFINITY) ? 0.0f : expf(mq[q] - M);
                        den = fmaf(w, lq[u], den);
                        num.x = fmaf(w, aq[u].x, num.x);
                        num.y = fmaf(w, aq[u].y, num.y);
                        num.z = fmaf(w, aq[u].z, num.z);
                        num.w = fmaf(w, aq[u].w, num.w);
                    }
                }
            }
            const float il = den > 0.0f ? 1.0f / den : 0.0f;
            *reinterpret_cast<float4*>(out) = make_float4(num.x * il, num.y * il, num.z * il, num.w * il);
        }
    }
    if (ns > 1) cluster_sync();  // partials stay readable until every rank has combined
    if (threadIdx.x == 0) trace_max(p.trace, 6);
}

// ---------------------------------------------------------------------------
// Grouped-query attention with 8 query heads per KV head and d = 64 (the
// TinyLlama shape of the benchmark configurations).  Same grid, cluster
// combine and page table walk as attn_decode_kernel, but each split runs two
// passes over its pages instead of an online softmax, so no page waits on
// another page's softmax:
//   pass 1 (K tiles): thread (token j, head h) holds head h's 64 query values
//     in registers (rotated by 4j, so the four tokens of a warp read four
//     different bank groups) and forms the full dot product from 16 float4
//     reads of K row j that the 8 heads' lanes share (one broadcast each);
//     the scores go to shared memory, S[page][token][head];
//   the split's maximum per head (shuffles and four warp values), then
//     weights 2^(s - max) in place and each thread's partial sum of them;
//   pass 2 (V tiles): thread (token pair tg, dims 4dc..4dc+3) accumulates the
//     8 heads' weighted V rows of its two tokens (one float4 of V, two of
//     weights, 16 packed FFMA2 per token); the 8 token pairs' accumulators
//     are summed once, in pair order.
// The producer streams every page's K tile, then every page's V tile, through
// one ring of 4 KB tiles; each byte of K and V is read from HBM once, as in the
// one-pass kernel.  Scores are kept in base 2 (q.k / sqrt(d) * log2 e), the
// same softmax.  A split covers at most kGqaMaxPages pages (launch_attn_gqa8
// raises the split count for longer contexts; beyond 16 splits the generic
// kernel runs).
// ---------------------------------------------------------------------------
constexpr int kGqaRing = 12;      // 4 KB tiles in flight per CTA
constexpr int kGqaMaxPages = 32;  // pages per split (scores: 16 KB)
constexpr int kGqaThreads = (4 + 1) * 32;

__global__ void __launch_bounds__(kGqaThreads, 3) attn_gqa8_d64_kernel(const __grid_constant__ AttnParams p) {
    constexpr int G = 8, D = 64;
    constexpr int TILE = kPageTokens * D;  // floats per K or V tile
    static_assert(kGqaRing * 20 <= kAttnHead, "ring barriers exceed the header");
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kGqaRing;
    int* valid = reinterpret_cast<int*>(empty + kGqaRing);  // [ring]
    float* wmax = reinterpret_cast<float*>(smem + kAttnHead);    // [4 warps][G]
    float* tiles = reinterpret_cast<float*>(smem + kAttnHead + 512);
    float* S = tiles + kGqaRing * TILE;                          // [kGqaMaxPages][16][G]
    float* cpart = S + kGqaMaxPages * kPageTokens * G;           // [G][D + 4]: acc, m, l of this split
    // after pass 2: [8 token pairs][G][D] accumulators and l [16][G] reuse the ring
    float* red = tiles;
    static_assert(8 * G * D + 16 * G <= kGqaRing * TILE, "reduction area fits the ring");

    const int split = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kGqaRing; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 4);
        }
        fence_barrier_init();
        trace_min(p.trace, 0);
        trace_max(p.trace, 1);
    }
    __syncthreads();
    pdl_launch_dependents();

    const SeqState& sq = p.seq[m];
    const bool active = p.lens ? true : (sq.active != 0);
    const int Lq = p.lens ? p.lens[m] : sq.pos + 1;
    const int npages = active ? (Lq + kPageTokens - 1) / kPageTokens : 0;
    const int pps = (npages + p.nsplit - 1) / p.nsplit;
    const int pg0 = min(npages, split * pps);
    const int pg1 = min(npages, pg0 + pps);
    const int nun = min(pg1 - pg0, kGqaMaxPages);  // the launcher keeps pps <= kGqaMaxPages

    if (warp == 4) {
        // --------- producer: K tiles of the split's pages, then V tiles ---------
        // (the split's page-table entries are loaded once, one per lane, so no
        // copy waits behind a dependent global load; lane 0 waits and issues)
        bool waited = false;
        const int pt = lane < nun ? p.page_table[(size_t)m * p.ptab_stride + pg0 + lane] : -1;
        for (int i = 0; i < 2 * nun; ++i) {
            const int st = i % kGqaRing;
            const int kv = i < nun ? 0 : 1;
            const int li = i < nun ? i : i - nun;
            const int page = __shfl_sync(0xffffffffu, pt, li);
            int ok = 1;
            if (lane == 0 && i >= kGqaRing) ok = mbar_wait(&empty[st], ((i / kGqaRing) - 1) & 1, p.err);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            const int lp = pg0 + li;
            if ((p.wait_first || lp == npages - 1) && !waited) {  // pages the preceding kernel appends to
                pdl_wait();
                waited = true;
            }
            if (lane == 0) {
                if (page >= 0) {
                    valid[st] = 1;
                    const size_t base =
                        ((((size_t)page * p.num_layers + p.layer) * 2 + kv) * p.Hkv + kvh) * (size_t)TILE;
                    mbar_arrive_expect_tx(&full[st], TILE * 4u);
                    bulk_g2s(tiles + st * TILE, p.kv_pool + base, TILE * 4u, &full[st]);
                } else {
                    valid[st] = 0;  // evicted page: rows read as zeros
                    mbar_arrive(&full[st]);
                }
            }
        }
    } else {
        // ------------------------------ consumers ------------------------------
        pdl_wait();
        if (threadIdx.x == 0) trace_max(p.trace, 2);
        const int t = threadIdx.x;  // 0..127
        const float scale2 = __fmul_rn(__fdiv_rn(1.0f, __fsqrt_rn((float)D)), 1.4426950408889634f);
        // pass-1 role: lane bits [c:2][hs:1][token:2] -- token j = 4 warp +
        // (lane >> 3), dim quarter c (16 dims), heads 4 hs..4 hs+3.  The four
        // float4 of a quarter are read in the order (e + j) & 3, so the 16
        // addresses of a warp load fall in 8 bank groups (two wavefronts, the
        // minimum).  After a reduce-scatter over the 4 quarters the lane holds
        // the full dot of token j, head h = 4 hs + c.
        const int c = lane & 3, hs = (lane >> 2) & 1;
        const int j = 4 * warp + (lane >> 3), h = 4 * hs + c;
        float2 qr[4][4][2];  // [head of the half][float4 e][pair]
        {
            const float* qb = p.q + (size_t)m * p.ld_q + (size_t)(kvh * G + 4 * hs) * D + 16 * c;
#pragma unroll
            for (int hh = 0; hh < 4; ++hh)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 a = *reinterpret_cast<const float4*>(qb + hh * D + 4 * ((e + j) & 3));
                    qr[hh][e][0] = make_float2(a.x, a.y);
                    qr[hh][e][1] = make_float2(a.z, a.w);
                }
        }
        bool bad = false;
        float mt = -INFINITY;  // this thread's maximum score (head h)
        for (int i = 0; i < nun; ++i) {
            const int st = i % kGqaRing;
            if (!bad && !mbar_wait(&full[st], (i / kGqaRing) & 1, p.err)) bad = true;
            const float* Kr = tiles + st * TILE + j * D + 16 * c;
            float part[4] = {0.f, 0.f, 0.f, 0.f};
            if (!bad && valid[st]) {
                float4 kv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) kv[e] = *reinterpret_cast<const float4*>(Kr + 4 * ((e + j) & 3));
#pragma unroll
                for (int hh = 0; hh < 4; ++hh) {
                    float2 d = __fmul2_rn(qr[hh][0][0], make_float2(kv[0].x, kv[0].y));
                    d = __ffma2_rn(qr[hh][0][1], make_float2(kv[0].z, kv[0].w), d);
#pragma unroll
                    for (int e = 1; e < 4; ++e) {
                        d = __ffma2_rn(qr[hh][e][0], make_float2(kv[e].x, kv[e].y), d);
                        d = __ffma2_rn(qr[hh][e][1], make_float2(kv[e].z, kv[e].w), d);
                    }
                    part[hh] = d.x + d.y;
                }
            }
            // reduce-scatter over the quarters (lane bits 0-1): lane c keeps head c
            float r2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float mine = (c & 2) ? part[2 + u] : part[u];
                const float other = (c & 2) ? part[u] : part[2 + u];
                r2[u] = mine + __shfl_xor_sync(0xffffffffu, other, 2);
            }
            const float mine = (c & 1) ? r2[1] : r2[0];
            const float other = (c & 1) ? r2[0] : r2[1];
            const float dot = mine + __shfl_xor_sync(0xffffffffu, other, 1);
            const int tok = (pg0 + i) * kPageTokens + j;
            const float sc = (tok < Lq) ? __fmul_rn(dot, scale2) : -INFINITY;
            S[(i * kPageTokens + j) * G + h] = sc;
            mt = fmaxf(mt, sc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        // the split's maximum of head h: the 4 tokens of the warp, then the 4 warps
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
        if (lane < 8) wmax[warp * G + h] = mt;  // lanes 0-7: h = 4 hs + c covers 0..7
        named_bar_sync(1, 128);
        const float M = fmaxf(fmaxf(wmax[h], wmax[G + h]), fmaxf(wmax[2 * G + h], wmax[3 * G + h]));
        // weights of this thread's own scores (no barrier needed) and their sum
        float l_part = 0.0f;
        for (int i = 0; i < nun; ++i) {
            float* sp = S + (i * kPageTokens + j) * G + h;
            const float e = (*sp == -INFINITY) ? 0.0f : exp2f(*sp - M);
            *sp = e;
            l_part += e;
        }
        named_bar_sync(1, 128);
        // pass 2: P.V for tokens 2tg, 2tg + 1 of every page
        const int tg = t >> 4, dc = t & 15;
        float2 acc[G][2];
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = make_float2(0.0f, 0.0f);
        for (int i = 0; i < nun; ++i) {
            const int q = nun + i, st = q % kGqaRing;
            if (!bad && !mbar_wait(&full[st], (q / kGqaRing) & 1, p.err)) bad = true;
            if (!bad && valid[st]) {
                const float* Vt = tiles + st * TILE;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int jj = 2 * tg + u;
                    const float4 v = *reinterpret_cast<const float4*>(Vt + jj * D + 4 * dc);
                    const float4 pa = *reinterpret_cast<const float4*>(S + (i * kPageTokens + jj) * G);
                    const float4 pb = *reinterpret_cast<const float4*>(S + (i * kPageTokens + jj) * G + 4);
                    const float pw[G] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
                    const float2 v01 = make_float2(v.x, v.y), v23 = make_float2(v.z, v.w);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float2 w2 = make_float2(pw[g], pw[g]);
                        acc[g][0] = __ffma2_rn(w2, v01, acc[g][0]);
                        acc[g][1] = __ffma2_rn(w2, v23, acc[g][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        // ---- this split's (acc, m, l): token pairs summed in pair order ----
        named_bar_sync(1, 128);  // every warp is done with the ring
#pragma unroll
        for (int g = 0; g < G; ++g)
            *reinterpret_cast<float4*>(red + (tg * G + g) * D + 4 * dc) =
                make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
        red[8 * G * D + j * G + h] = l_part;
        named_bar_sync(1, 128);
        {
            const int g = t >> 4, d4 = 4 * (t & 15);
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = *reinterpret_cast<const float4*>(red + (q * G + g) * D + d4);
                a.x += v.x;
                a.y += v.y;
                a.z += v.z;
                a.w += v.w;
            }
            *reinterpret_cast<float4*>(cpart + g * (D + 4) + d4) = a;
        }
        if (t < G) {  // head h of lanes 0-7 of warp 0: the split's maximum and the 16 tokens' sums
            float l = 0.0f;
            for (int q = 0; q < 16; ++q) l += red[8 * G * D + q * G + h];
            cpart[h * (D + 4) + D] = M;
            cpart[h * (D + 4) + D + 1] = l;
        }
    }
    // Combine the splits (cluster ranks) in split order (maxima in base 2).
    const int ns = p.nsplit;
    if (ns > 1) cluster_sync();
    else __syncthreads();
    {
        constexpr int Q = G * (D / 4);
        const int t = threadIdx.x;
        const int i0 = split * Q / ns, i1 = (split + 1) * Q / ns;
        if (t < 128 && i0 + t < i1) {
            const int item = i0 + t;
            const int g = item / (D / 4), d4 = (item % (D / 4)) * 4;
            float* out = p.out + (size_t)m * p.ld_out + (size_t)(kvh * G + g) * D + d4;
            float mq[kMaxAttnSplits];
#pragma unroll
            for (int q = 0; q < kMaxAttnSplits; ++q)
                mq[q] = q < ns ? dsmem_ld_f32(dsmem_map(cpart + g * (D + 4) + D, (uint32_t)q)) : -INFINITY;
            float Mx = -INFINITY;
#pragma unroll
            for (int q = 0; q < kMaxAttnSplits; ++q) Mx = fmaxf(Mx, mq[q]);
            float den = 0.0f;
            float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
            if (Mx != -INFINITY) {
#pragma unroll
                for (int q0 = 0; q0 < kMaxAttnSplits; q0 += 8) {
                    if (q0 >= ns) break;
                    float lq[8];
                    float4 aq[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int q = q0 + u;
                        if (q < ns) {
                            const uint32_t base = dsmem_map(cpart + g * (D + 4), (uint32_t)q);
                            lq[u] = dsmem_ld_f32(base + (D + 1) * 4);
                            aq[u] = dsmem_ld_f32x4(base + d4 * 4);
                        } else {
                            lq[u] = 0.0f;
                            aq[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int q = q0 + u;
                        if (q >= ns) continue;
                        const float w = (mq[q] == -INFINITY) ? 0.0f : exp2f(mq[q] - Mx);
                        den = fmaf(w, lq[u], den);
                        num.x = fmaf(w, aq[u].x, num.x);
                        num.y = fmaf(w, aq[u].y, num.y);
                        num.z = fmaf(w, aq[u].z, num.z);
                        num.w = fmaf(w, aq[u].w, num.w);
                    }
                }
            }
            const float il = den > 0.0f ? 1.0f / den : 0.0f;
            *reinterpret_cast<float4*>(out) = make_float4(num.x * il, num.y * il, num.z * il, num.w * il);
        }
    }
    if (ns > 1) cluster_sync();  // partials stay readable until every rank has combined
    if (threadIdx.x == 0) trace_max(p.trace, 6);
}

// ---------------------------------------------------------------------------
// Persistent chunked GQA-8 attention (runner plans; d = 64, 8 query heads per
// KV head, up to kFlatMaxRows rows).  The cluster kernel above gives every
// (sequence, KV head) the same number of splits, so with ragged contexts its
// CTAs differ in length and run in ~5 short waves, each CTA paying its own
// start (q load, first page) and end (cluster combine).  Here the work is cut
// into chunks of chunk_pages pages per (sequence, KV head) -- equal except the
// last of each -- and a fixed grid of 3 CTAs per SM walks them round robin;
// the producer streams the next chunk's tiles while the consumers finish the
// current one, so HBM streaming does not stop between chunks.  Chunk order:
// every non-final chunk of every sequence first, then the final ones (which
// hold the page the preceding QKV kernel appends to), so a CTA fetches its
// first chunks before the programmatic-dependent-launch wait.  Each chunk runs
// the two passes of attn_gqa8_d64_kernel and writes its partial (acc, m, l) to
// `part`; the CTA that completes the last chunk of a (sequence, KV head)
// (a ticket counter) merges the partials in chunk order -- deterministic --
// writes the output and resets the ticket.  A single-chunk pair writes its
// output directly.
// ---------------------------------------------------------------------------
constexpr int kFlatCtas = 4;        // CTAs per SM
constexpr int kFlatRing = kFlatCtas == 4 ? 10 : kFlatCtas == 3 ? 12 : 20;
constexpr int kFlatSRed = 4 * 8 * 64 + 16 * 8;  // floats of the region shared by the scores and the reduction
// Ring tiles start on a 1 KB boundary (128-byte swizzle atoms of the tensor loads).
constexpr int kFlatTilesOff = (kAttnHead + 2048 + 1023) / 1024 * 1024;
constexpr int kFlatMaxPages = 16;   // pages per chunk at most
constexpr int kFlatMaxRows = 64;    // sequences (rows) per launch
constexpr int kFlatThreads = (4 + 1) * 32;

struct FlatChunk {
    int s, kvh, ci, p0, np, nch, L;
    bool tail;
};

// High tf32 part of x (the top 19 bits, low 13 cleared) as the 32-bit
// operand pattern: one logic op instead of a conversion; x - hi is exact.
__device__ __forceinline__ uint32_t tf32_hi(float x) { return __float_as_uint(x) & 0xffffe000u; }
// One 2-D tile of a tensor map -> shared memory (TMA), completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// Float offset of (token t, dimension dd) in a ring tile: two 16 x 32 halves
// (dimensions 0-31, 32-63), each row's 16-byte chunks swizzled by the row
// (chunk ^ (t % 8)), as the 128-byte-swizzle tensor load writes them.
__device__ __forceinline__ int flat_tile_off(int t, int dd) {
    return (dd >> 5) * (kPageTokens * 32) + t * 32 + ((((dd & 31) >> 2) ^ (t & 7)) << 2) + (dd & 3);
}
// d (16 x 8, fp32) += a (16 x 8, tf32, row major) x b (8 x 8, tf32, column major), one warp.
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__global__ void __launch_bounds__(kFlatThreads, kFlatCtas) attn_flat_gqa8_kernel(const __grid_constant__ AttnParams p,
                                                                                const __grid_constant__ CUtensorMap kvmap) {
    constexpr int G = 8, D = 64;
    constexpr int TILE = kPageTokens * D;
    static_assert(kFlatRing * 28 <= kAttnHead, "ring barriers exceed the header");
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    // Tile j lands in data slot j % R (R = kFlatRing) and completes full
    // barrier j % 2R.  Two full barriers per slot: a consumer warp may start
    // waiting on tile j while tile j - R (same slot) is still in flight
    // (chunks hold more pages than the ring, and the 4 warps take every 4th
    // page), and a parity wait on a single barrier would then mistake the
    // earlier tile's completed phase for tile j.  Tile j - 2R has always
    // completed by then (the waiting warp consumed tile j - 4, whose
    // production needed tile j - 4 - R released), so 2R barriers decide it.
    uint64_t* empty = full + 2 * kFlatRing;
    int* valid = reinterpret_cast<int*>(empty + kFlatRing);              // [ring]
    int* nchk = reinterpret_cast<int*>(smem + kAttnHead);                // [rows] chunks of each row
    int* pre_nt = nchk + kFlatMaxRows;                                   // [rows + 1] prefix of non-final chunks
    int* pre_t = pre_nt + kFlatMaxRows + 1;                              // [rows + 1] prefix of rows with pages
    int* lens = pre_t + kFlatMaxRows + 1;                                // [rows] context lengths
    int* misc = lens + kFlatMaxRows;                                     // [4]
    float* wmax = reinterpret_cast<float*>(misc + 4);                    // [4 warps][G]
    float* tiles = reinterpret_cast<float*>(smem + kFlatTilesOff);       // [ring][TILE], swizzled halves
    float* S = tiles + kFlatRing * TILE;                                 // [kFlatMaxPages][16][G]
    // red [4 warps][G][D] + l [16][G] shares its storage with S: it is
    // written once every warp has finished pass 2 (S is dead until the next
    // chunk's pass 1, which follows a later barrier)
    float* red = S;
    static_assert(kFlatMaxPages * kPageTokens * G <= kFlatSRed, "S fits the shared region");
    static_assert(4 * G * D + 16 * G <= kFlatSRed, "red fits the shared region");
    float* qs = S + kFlatSRed;                                           // [2][G][D] query slots
    static_assert((3 * kFlatMaxRows + 2 + 4 + 4 * G) * 4 <= 2048, "row tables");

    if (smem_u32(tiles) & 1023u) {  // the swizzled tensor loads need 1 KB-aligned tiles: do nothing
        if (threadIdx.x == 0) record_error(p.err, kDevBadSmem);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = p.M, Hkv = p.Hkv, CP = p.chunk_pages;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kFlatRing; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&full[kFlatRing + i], 1);
            mbar_init(&empty[i], 1);  // one consumer warp reads a tile
        }
        fence_barrier_init();
        trace_min(p.trace, 0);
        trace_max(p.trace, 1);
    }
    // rows: context length and chunk count (sequence state and page tables
    // are written before the step starts: readable before the dependency wait)
    for (int s = threadIdx.x; s < M; s += blockDim.x) {
        const bool act = p.lens ? true : (p.seq[s].active != 0);
        const int L = p.lens ? p.lens[s] : p.seq[s].pos + 1;
        const int np = act ? (L + kPageTokens - 1) / kPageTokens : 0;
        lens[s] = L;
        nchk[s] = (np + CP - 1) / CP;
    }
    __syncthreads();
    if (warp == 0) {  // two exclusive prefix sums over <= 64 rows (2 per lane)
        const int a0 = 2 * lane < M ? nchk[2 * lane] : 0, a1 = 2 * lane + 1 < M ? nchk[2 * lane + 1] : 0;
        const int nt0 = a0 > 0 ? a0 - 1 : 0, nt1 = a1 > 0 ? a1 - 1 : 0;
        const int t0 = a0 > 0, t1 = a1 > 0;
        int x = nt0 + nt1, y = t0 + t1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int xo = __shfl_up_sync(0xffffffffu, x, o), yo = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) {
                x += xo;
                y += yo;
            }
        }
        const int xe = x - nt0 - nt1, ye = y - t0 - t1;  // exclusive
        if (2 * lane <= M) {
            pre_nt[2 * lane] = xe;
            pre_t[2 * lane] = ye;
        }
        if (2 * lane + 1 <= M) {
            pre_nt[2 * lane + 1] = xe + nt0;
            pre_t[2 * lane + 1] = ye + t0;
        }
        if (lane == 31) {  // the totals (index M; at M = 64 no lane above reaches it)
            pre_nt[M] = x;
            pre_t[M] = y;
        }
    }
    __syncthreads();
    pdl_launch_dependents();
    const int total_nt = pre_nt[M], total_t = pre_t[M];
    const int nchunks = Hkv * (total_nt + total_t);
    // chunk c -> (row, KV head, chunk index); non-final chunks first
    auto chunk = [&](int c) -> FlatChunk {
        FlatChunk k{};
        int unit;
        bool tail = c >= Hkv * total_nt;
        if (!tail) {
            unit = c / Hkv;
            k.kvh = c - unit * Hkv;
            int lo = 0, hi = M - 1;  // last row with pre_nt[row] <= unit
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (pre_nt[mid] <= unit) lo = mid; else hi = mid - 1;
            }
            k.s = lo;
            k.ci = unit - pre_nt[lo];
        } else {
            const int c2 = c - Hkv * total_nt;
            unit = c2 / Hkv;
            k.kvh = c2 - unit * Hkv;
            int lo = 0, hi = M - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (pre_t[mid] <= unit) lo = mid; else hi = mid - 1;
            }
            k.s = lo;
            k.ci = nchk[lo] - 1;
        }
        k.tail = tail;
        k.nch = nchk[k.s];
        k.L = lens[k.s];
        const int npg = (k.L + kPageTokens - 1) / kPageTokens;
        k.p0 = k.ci * CP;
        k.np = min(CP, npg - k.p0);
        return k;
    };

    if (warp == 4) {
        // ------------- producer: every chunk's K tiles, then its V tiles -------------
        bool waited = p.wait_first == 0 ? false : (pdl_wait(), true);
        int ring = 0;
        bool stop = false;
        for (int c = blockIdx.x; c < nchunks && !stop; c += gridDim.x) {
            const FlatChunk k = chunk(c);
            const int pt = lane < k.np ? p.page_table[(size_t)k.s * p.ptab_stride + k.p0 + lane] : -1;
            if (k.tail && !waited) {  // holds the page the preceding QKV kernel appends to
                pdl_wait();
                waited = true;
            }
            for (int i = 0; i < 2 * k.np; ++i, ++ring) {
                const int st = ring % kFlatRing;
                const int kv = i < k.np ? 0 : 1;
                const int page = __shfl_sync(0xffffffffu, pt, i < k.np ? i : i - k.np);
                int ok = 1;
                if (lane == 0 && ring >= kFlatRing) ok = mbar_wait(&empty[st], ((ring / kFlatRing) - 1) & 1, p.err);
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    stop = true;
                    break;
                }
                if (page >= 0) {
                    if (lane == 0) {
                        valid[st] = 1;
                        // first pool row of the tile (a row = 64 floats)
                        const int row0 = (int)(((((size_t)page * p.num_layers + p.layer) * 2 + kv) * p.Hkv + k.kvh) *
                                               (size_t)kPageTokens);
                        uint64_t* fb = &full[ring % (2 * kFlatRing)];
                        mbar_arrive_expect_tx(fb, TILE * 4u);
                        tma_load_2d(tiles + st * TILE, &kvmap, 0, row0, fb);
                        tma_load_2d(tiles + st * TILE + kPageTokens * 32, &kvmap, 32, row0, fb);
                    }
                } else if (lane == 0) {
                    valid[st] = 0;  // evicted page: rows read as zeros
                    mbar_arrive(&full[ring % (2 * kFlatRing)]);
                }
            }
        }
    } else {
        // ------------------------------ consumers ------------------------------
        pdl_wait();
        if (threadIdx.x == 0) trace_max(p.trace, 2);
        const int t = threadIdx.x;  // 0..127
        const float scale2 = __fmul_rn(__fdiv_rn(1.0f, __fsqrt_rn((float)D)), 1.4426950408889634f);
        bool bad = false;
        int ring = 0, slot = 0;
        // diagnostics (launch tracing): SM cycles of consumer warp 0, summed
        // over CTAs: [14] chunk start, [8] pass 1, [9] between the passes,
        // [10] pass 2, [11] warp reduction, [12] partial and ticket, [13]
        // tile waits (within the passes), [15] chunks
        unsigned long long* prb = (p.trace && t == 0) ? p.trace : nullptr;
        long long cy = prb ? clock64() : 0;
        auto lap = [&](int slotid) {
            if (prb) {
                const long long n = clock64();
                atomicAdd(prb + slotid, (unsigned long long)(n - cy));
                cy = n;
            }
        };
        // query of a chunk -> shared slot (one 16-byte async copy per thread)
        auto fetch_q = [&](const FlatChunk& k, int sl) {
            const float* src = p.q + (size_t)k.s * p.ld_q + (size_t)k.kvh * G * D + 4 * t;
            const uint32_t dst = smem_u32(qs + sl * G * D + 4 * t);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        // deferred merge of the previous multi-chunk pair (thread 0 holds its ticket)
        // Two pairs in flight: A (pend_*) has its ticket increment issued,
        // its result read one chunk later; B (pb_*) has its partial stored,
        // its increment issued at the next chunk's mid-point, when the stores
        // have long completed (so the release costs no wait).
        int tk = 0, pend_pair = -1, pend_nch = 0, pend_s = 0, pend_kvh = 0;
        int pb_pair = -1, pb_nch = 0, pb_s = 0, pb_kvh = 0;
        auto merge = [&]() {  // every chunk of the pending pair is in: merge them in chunk order
            const int og = t >> 4, od = 4 * (t & 15);
            const float* pb = p.part + (size_t)pend_pair * p.maxch * kAttnPartFloats;
            float Mg = -INFINITY;
            for (int q0 = 0; q0 < pend_nch; q0 += 8) {  // 8 independent loads at a time, bypassing L1
                float mv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    mv[u] = q0 + u < pend_nch ? __ldcg(pb + (q0 + u) * kAttnPartFloats + 8 * D + og) : -INFINITY;
#pragma unroll
                for (int u = 0; u < 8; ++u) Mg = fmaxf(Mg, mv[u]);
            }
            float den = 0.0f;
            float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q0 = 0; q0 < pend_nch; q0 += 4) {  // 4 partials' loads in flight
                float mv[4], lv[4];
                float4 av[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const bool in = q0 + u < pend_nch;
                    const float* pq = pb + (q0 + u) * kAttnPartFloats;
                    mv[u] = in ? __ldcg(pq + 8 * D + og) : -INFINITY;
                    lv[u] = in ? __ldcg(pq + 8 * D + 8 + og) : 0.0f;
                    av[u] = in ? __ldcg(reinterpret_cast<const float4*>(pq + og * D + od))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float w = mv[u] == -INFINITY ? 0.0f : exp2f(mv[u] - Mg);
                    den = fmaf(w, lv[u], den);
                    num.x = fmaf(w, av[u].x, num.x);
                    num.y = fmaf(w, av[u].y, num.y);
                    num.z = fmaf(w, av[u].z, num.z);
                    num.w = fmaf(w, av[u].w, num.w);
                }
            }
            const float il = den > 0.0f ? 1.0f / den : 0.0f;
            float* out = p.out + (size_t)pend_s * p.ld_out + (size_t)(pend_kvh * G + og) * D + od;
            *reinterpret_cast<float4*>(out) = make_float4(num.x * il, num.y * il, num.z * il, num.w * il);
            if (t == 0) p.ticket[pend_pair] = 0;  // ready for the next launch
        };
        int c = blockIdx.x;
        FlatChunk k{};
        if (c < nchunks) {
            k = chunk(c);
            fetch_q(k, 0);
        }
        if (p.probe) {  // streaming alone: wait for every tile, release it
            for (; c < nchunks; c += gridDim.x) {
                const FlatChunk kk = chunk(c);
                for (int i = 0; i < 2 * kk.np; ++i, ++ring) {
                    const int st = ring % kFlatRing;
                    if (!bad && !mbar_wait(&full[ring % (2 * kFlatRing)], (ring / (2 * kFlatRing)) & 1, p.err)) bad = true;
                    __syncwarp();
                    if (lane == 0 && warp == 0) mbar_arrive(&empty[st]);
                }
            }
        }
        for (; c < nchunks; c += gridDim.x) {
            const int cn = c + (int)gridDim.x;
            FlatChunk kn{};
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            named_bar_sync(1, 128);  // this chunk's query is in its slot; the other slot is free
            if (cn < nchunks) {
                kn = chunk(cn);
                fetch_q(kn, slot ^ 1);  // the next chunk's query, behind this chunk's work
            }
            const int og = t >> 4, od = 4 * (t & 15);  // output item: head og, dims od..od+3
            float4 a;
            float lsum, mchunk;
            {
            // ---- tensor cores (mma.sync m16n8k8, tf32 split in three products
            // hi*hi + hi*lo + lo*hi ~ fp32 accuracy).  Warp w takes the
            // chunk's pages i = w, w + 4, ... in both passes.
            // lane = (g = lane / 4, t = lane % 4).  Scores: A = K tile rows
            // (tokens) g / g + 8, B = query^T (head g); block b covers 16-byte
            // chunk 2t + (b & 1) of dimension half b / 2 for lane t, and k-step
            // s uses its dims 2s (k = t) and 2s + 1 (k = t + 4): each thread
            // loads 4 consecutive dims of a row at once, and with the tile's
            // chunk swizzle (chunk ^ row % 8) the 8 lanes of a quarter warp
            // (two rows, 4 chunks of equal parity) hit 8 different chunks.
            lap(14);
            if (prb) atomicAdd(prb + 15, 1ull);
            const int gq = lane >> 2, tq = lane & 3;
            uint32_t qh[4][2][2], ql[4][2][2];  // [16-dim block][k-step][b0 / b1]
            {
                const float* qg = qs + slot * G * D + gq * D;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float4 v = *reinterpret_cast<const float4*>(qg + 32 * (b >> 1) + 4 * (2 * tq + (b & 1)));
                    const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint32_t h32 = tf32_hi(e[u]);
                        qh[b][u >> 1][u & 1] = h32;
                        ql[b][u >> 1][u & 1] = __float_as_uint(e[u] - __uint_as_float(h32));
                    }
                }
            }
            float mth[2] = {-INFINITY, -INFINITY};  // this lane's max of heads 2t, 2t + 1
            for (int i = warp; i < k.np; i += 4) {
                const int st = (ring + i) % kFlatRing;
                const long long w0 = prb ? clock64() : 0;
                if (!bad && !mbar_wait(&full[(ring + i) % (2 * kFlatRing)], ((ring + i) / (2 * kFlatRing)) & 1, p.err))
                    bad = true;
                if (prb) atomicAdd(prb + 13, (unsigned long long)(clock64() - w0));
                float c[4] = {0.f, 0.f, 0.f, 0.f};
                // two independent accumulators (block parity): dependent
                // chains of 12 products instead of 24
                float cacc[2][4];
#pragma unroll
                for (int u = 0; u < 2; ++u) cacc[u][0] = cacc[u][1] = cacc[u][2] = cacc[u][3] = 0.0f;
                if (!bad && valid[st]) {
                    const float* Kt = tiles + st * TILE;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const int dd = 32 * (b >> 1) + 4 * (2 * tq + (b & 1));
                        const float4 r0 = *reinterpret_cast<const float4*>(Kt + flat_tile_off(gq, dd));
                        const float4 r1 = *reinterpret_cast<const float4*>(Kt + flat_tile_off(gq + 8, dd));
                        const float e0[4] = {r0.x, r0.y, r0.z, r0.w}, e1[4] = {r1.x, r1.y, r1.z, r1.w};
#pragma unroll
                        for (int sstep = 0; sstep < 2; ++sstep) {
                            uint32_t ah[4], al[4];
                            const float av[4] = {e0[2 * sstep], e1[2 * sstep], e0[2 * sstep + 1], e1[2 * sstep + 1]};
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                ah[u] = tf32_hi(av[u]);
                                al[u] = __float_as_uint(av[u] - __uint_as_float(ah[u]));
                            }
                            mma_tf32(cacc[b & 1], al, qh[b][sstep]);
                            mma_tf32(cacc[b & 1], ah, ql[b][sstep]);
                            mma_tf32(cacc[b & 1], ah, qh[b][sstep]);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) c[u] = cacc[0][u] + cacc[1][u];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
                // c0 (token g, head 2t), c1 (g, 2t + 1), c2 (g + 8, 2t), c3 (g + 8, 2t + 1)
                const int tok0 = (k.p0 + i) * kPageTokens + gq;
                const float s0 = tok0 < k.L ? __fmul_rn(c[0], scale2) : -INFINITY;
                const float s1 = tok0 < k.L ? __fmul_rn(c[1], scale2) : -INFINITY;
                const float s2 = tok0 + 8 < k.L ? __fmul_rn(c[2], scale2) : -INFINITY;
                const float s3 = tok0 + 8 < k.L ? __fmul_rn(c[3], scale2) : -INFINITY;
                float* Sp = S + (i * kPageTokens) * G;
                *reinterpret_cast<float2*>(Sp + gq * G + 2 * tq) = make_float2(s0, s1);
                *reinterpret_cast<float2*>(Sp + (gq + 8) * G + 2 * tq) = make_float2(s2, s3);
                mth[0] = fmaxf(mth[0], fmaxf(s0, s2));
                mth[1] = fmaxf(mth[1], fmaxf(s1, s3));
            }
            lap(8);
            // per head: the lanes of equal t, then the 4 warps
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mth[0] = fmaxf(mth[0], __shfl_xor_sync(0xffffffffu, mth[0], o));
                mth[1] = fmaxf(mth[1], __shfl_xor_sync(0xffffffffu, mth[1], o));
            }
            if (lane < 4) {
                wmax[warp * G + 2 * tq] = mth[0];
                wmax[warp * G + 2 * tq + 1] = mth[1];
            }
            if (t == 0) {
                misc[1] = tk;  // pair A's ticket (its atomic has long completed)
                // pair B: the barrier at this chunk's start ordered every
                // thread's partial stores before this release increment
                if (pb_pair >= 0)
                    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(tk) : "l"(p.ticket + pb_pair)
                                 : "memory");
            }
            named_bar_sync(1, 128);
            float Mh[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int hh = 2 * tq + u;
                Mh[u] = fmaxf(fmaxf(wmax[hh], wmax[G + hh]), fmaxf(wmax[2 * G + hh], wmax[3 * G + hh]));
            }
            if (pend_pair >= 0 && misc[1] == pend_nch - 1) merge();
            pend_pair = pb_pair;
            pend_nch = pb_nch;
            pend_s = pb_s;
            pend_kvh = pb_kvh;
            pb_pair = -1;
            // weights of this warp's own pages, in place (no other warp reads them)
            float lh[2] = {0.f, 0.f};
            for (int i = warp; i < k.np; i += 4) {
                float* Sp = S + (i * kPageTokens) * G;
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    float2* e2 = reinterpret_cast<float2*>(Sp + (gq + 8 * r) * G + 2 * tq);
                    float2 v = *e2;
                    v.x = v.x == -INFINITY ? 0.0f : exp2f(v.x - Mh[0]);
                    v.y = v.y == -INFINITY ? 0.0f : exp2f(v.y - Mh[1]);
                    lh[0] += v.x;
                    lh[1] += v.y;
                    *e2 = v;
                }
            }
            __syncwarp();
            // pass 2: O^(rows) = A (rows 0-7: P hi of head g, rows 8-15: P lo) x V;
            // k-step s: k = t -> token 8s + 2t, k = t + 4 -> token 8s + 2t + 1
            // (row % 8 of the 4 t lanes then differs in its upper two bits, so
            // with the chunk swizzle a warp's 32 fragment loads hit 32 banks);
            // n-block v: dims 8v .. 8v + 7 (column g)
            float dacc[8][4];
#pragma unroll
            for (int v = 0; v < 8; ++v) dacc[v][0] = dacc[v][1] = dacc[v][2] = dacc[v][3] = 0.0f;
            lap(9);
            for (int i = warp; i < k.np; i += 4) {
                const int q2 = k.np + i, st = (ring + q2) % kFlatRing;
                const long long w0 = prb ? clock64() : 0;
                if (!bad && !mbar_wait(&full[(ring + q2) % (2 * kFlatRing)], ((ring + q2) / (2 * kFlatRing)) & 1, p.err))
                    bad = true;
                if (prb) atomicAdd(prb + 13, (unsigned long long)(clock64() - w0));
                if (!bad && valid[st]) {
                    const float* Vt = tiles + st * TILE;
                    const float* Sp = S + (i * kPageTokens) * G;
#pragma unroll
                    for (int sstep = 0; sstep < 2; ++sstep) {
                        const float pa = Sp[(8 * sstep + 2 * tq) * G + gq], pb = Sp[(8 * sstep + 2 * tq + 1) * G + gq];
                        uint32_t a[4];
                        a[0] = tf32_hi(pa);
                        a[2] = tf32_hi(pb);
                        a[1] = __float_as_uint(pa - __uint_as_float(a[0]));
                        a[3] = __float_as_uint(pb - __uint_as_float(a[2]));
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            const float b0 = Vt[flat_tile_off(8 * sstep + 2 * tq, 8 * v + gq)];
                            const float b1 = Vt[flat_tile_off(8 * sstep + 2 * tq + 1, 8 * v + gq)];
                            uint32_t bh[2], bl[2];
                            bh[0] = tf32_hi(b0);
                            bh[1] = tf32_hi(b1);
                            bl[0] = __float_as_uint(b0 - __uint_as_float(bh[0]));
                            bl[1] = __float_as_uint(b1 - __uint_as_float(bh[1]));
                            mma_tf32(dacc[v], a, bh);
                            mma_tf32(dacc[v], a, bl);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
            ring += 2 * k.np;
            lap(10);
            named_bar_sync(1, 128);  // every warp is past pass 2: S may be overwritten by red
            // this warp's O[head g][dims 8v + 2t, +1] = rows g + rows g + 8 -> red[warp][head][dim]
#pragma unroll
            for (int v = 0; v < 8; ++v)
                *reinterpret_cast<float2*>(red + (warp * G + gq) * D + 8 * v + 2 * tq) =
                    make_float2(dacc[v][0] + dacc[v][2], dacc[v][1] + dacc[v][3]);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                lh[0] += __shfl_xor_sync(0xffffffffu, lh[0], o);
                lh[1] += __shfl_xor_sync(0xffffffffu, lh[1], o);
            }
            if (lane < 4) {
                red[4 * G * D + warp * G + 2 * tq] = lh[0];
                red[4 * G * D + warp * G + 2 * tq + 1] = lh[1];
            }
            named_bar_sync(1, 128);
            a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = *reinterpret_cast<const float4*>(red + (q * G + og) * D + od);
                a.x += v.x;
                a.y += v.y;
                a.z += v.z;
                a.w += v.w;
            }
            lsum = 0.0f;
            for (int q = 0; q < 4; ++q) lsum += red[4 * G * D + q * G + og];
            mchunk = fmaxf(fmaxf(wmax[og], wmax[G + og]), fmaxf(wmax[2 * G + og], wmax[3 * G + og]));
            }
            lap(11);
            const int pair = k.s * Hkv + k.kvh;
            if (k.nch == 1) {
                float* out = p.out + (size_t)k.s * p.ld_out + (size_t)(k.kvh * G + og) * D + od;
                const float il = lsum > 0.0f ? 1.0f / lsum : 0.0f;
                *reinterpret_cast<float4*>(out) = make_float4(a.x * il, a.y * il, a.z * il, a.w * il);
            } else {
                float* pp = p.part + ((size_t)pair * p.maxch + k.ci) * kAttnPartFloats;
                *reinterpret_cast<float4*>(pp + og * D + od) = a;
                if ((t & 15) == 0) {
                    pp[8 * D + og] = mchunk;
                    pp[8 * D + 8 + og] = lsum;
                }
                pb_pair = pair;
                pb_nch = k.nch;
                pb_s = k.s;
                pb_kvh = k.kvh;
            }
            lap(12);
            slot ^= 1;
            k = kn;
        }
        if (pend_pair >= 0 || pb_pair >= 0) {  // drain both pending pairs
            named_bar_sync(1, 128);  // B's partial stores before thread 0's increment
            if (t == 0) {
                misc[1] = tk;
                if (pb_pair >= 0)
                    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(misc[2]) : "l"(p.ticket + pb_pair)
                                 : "memory");
            }
            named_bar_sync(1, 128);
            if (pend_pair >= 0 && misc[1] == pend_nch - 1) merge();
            if (pb_pair >= 0) {
                pend_pair = pb_pair;
                pend_nch = pb_nch;
                pend_s = pb_s;
                pend_kvh = pb_kvh;
                if (misc[2] == pend_nch - 1) merge();
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) trace_max(p.trace, 6);
}

size_t attn_flat_smem() {
    return kFlatTilesOff + (size_t)kFlatRing * kPageTokens * 64 * 4 + (size_t)kFlatSRed * 4 + (size_t)2 * 8 * 64 * 4;
}

// The driver's tensor-map encoder, fetched once through the runtime (no link
// against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

cudaError_t launch_attn_flat(const AttnParams& p, cudaStream_t stream, bool pdl, int grid) {
    const size_t smem = attn_flat_smem();
    // The KV pool as a 2-D fp32 tensor [rows][64] (a row = one token of one
    // (page, layer, K|V, KV head) tile); a box is 16 rows x 32 floats (one
    // half tile, 2 KB), landing 128-byte swizzled.
    auto encode = tensor_map_encoder();
    if (!encode || p.kv_floats < 64) return cudaErrorInvalidValue;
    CUtensorMap kvmap;
    const cuuint64_t dims[2] = {64, (cuuint64_t)(p.kv_floats / 64)};
    const cuuint64_t strides[1] = {64 * sizeof(float)};
    const cuuint32_t box[2] = {32, kPageTokens};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&kvmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p.kv_pool), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    auto kfn = attn_flat_gqa8_kernel;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3(kFlatThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kfn, p, kvmap);
}

size_t attn_gqa8_smem() {
    return kAttnHead + 512 + (size_t)kGqaRing * kPageTokens * 64 * 4 + (size_t)kGqaMaxPages * kPageTokens * 8 * 4 +
           (size_t)8 * (64 + 4) * 4;
}

cudaError_t launch_attn_gqa8(const AttnParams& p, cudaStream_t stream, bool pdl) {
    const size_t smem = attn_gqa8_smem();
    auto kfn = attn_gqa8_d64_kernel;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    if (p.nsplit > 8) {
        e = cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    if (p.nsplit < 1 || p.nsplit > kMaxAttnSplits) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)p.nsplit, (unsigned)p.Hkv, (unsigned)p.M);
    cfg.blockDim = dim3(kGqaThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kfn, p);
}

template <int G, int D>
size_t attn_smem() {
    return kAttnHead + (((2 * G * kPageTokens + 2 * G) * 4 + 127) / 128) * 128 +
           (size_t)attn_stages(D) * 2 * kPageTokens * D * 4 +
           (size_t)G * (D + 4) * 4;
}

template <int G, int D>
cudaError_t launch_attn_t(const AttnParams& p, cudaStream_t stream, bool pdl) {
    const size_t smem = attn_smem<G, D>();
    auto kfn = attn_decode_kernel<G, D>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    if (p.nsplit > 8) {  // clusters of up to 16 CTAs are a non-portable size
        e = cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)p.nsplit, (unsigned)p.Hkv, (unsigned)p.M);
    cfg.blockDim = dim3(kAttnThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    if (p.nsplit < 1 || p.nsplit > kMaxAttnSplits) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;  // the splits of a (sequence, KV head)
    attr[0].val.clusterDim.x = (unsigned)p.nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kfn, p);
}

// Observer hook: explicit softmax weights [M][H][L] (ModelRunner.swift:544-586).
__global__ void attn_probs_kernel(const AttnParams p, float* probs, int L) {
    const int h = blockIdx.x, m = blockIdx.y;
    const int G = p.H / p.Hkv, kvh = h / G, d = p.d;
    extern __shared__ float sc[];
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)d));
    const float* q = p.q + (size_t)m * p.ld_q + (size_t)h * d;
    for (int j = threadIdx.x; j < L; j += blockDim.x) {
        const int page = p.page_table[(size_t)m * p.ptab_stride + j / kPageTokens];
        float dot = 0.0f;
        if (page >= 0) {
            const float* k = p.kv_pool +
                             (((((size_t)page * p.num_layers + p.layer) * 2 + 0) * p.Hkv + kvh) * kPageTokens +
                              j % kPageTokens) * d;
            for (int t = 0; t < d; ++t) dot = fmaf(q[t], k[t], dot);
        }
        sc[j] = __fmul_rn(dot, scale);
    }
    __syncthreads();
    __shared__ float red[2];
    if (threadIdx.x == 0) {
        float mx = -INFINITY;
        for (int j = 0; j < L; ++j) mx = fmaxf(mx, sc[j]);
        float sum = 0.0f;
        for (int j = 0; j < L; ++j) sum += expf(sc[j] - mx);
        red[0] = mx;
        red[1] = sum;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < L; j += blockDim.x)
        probs[((size_t)m * p.H + h) * L + j] = __fdiv_rn(expf(sc[j] - red[0]), red[1]);
}

// Observer hook: L2 norm of each hidden row (ModelRunner.swift:395-399).
__global__ void row_norm_kernel(const float* h, int H, int ld, float* out) {
    const float* x = h + (size_t)blockIdx.x * ld;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    __shared__ float red[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        out[blockIdx.x] = __fsqrt_rn(t);
    }
}

// Observer hook: final hidden state, RMSNorm(h) * w (Tensor.swift:1538-1558),
// or h itself when the model has no final norm.
__global__ void rmsnorm_rows_kernel(const float* h, const float* w, int H, int ld, float eps, float* out) {
    const float* x = h + (size_t)blockIdx.x * ld;
    float* y = out + (size_t)blockIdx.x * H;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    __shared__ float red[32];
    __shared__ float inv_s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int q = 0; q < (int)(blockDim.x >> 5); ++q) t += red[q];
        inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)H), eps)));
    }
    __syncthreads();
    const float inv = inv_s;
    for (int i = threadIdx.x; i < H; i += blockDim.x) y[i] = w ? __fmul_rn(__fmul_rn(x[i], inv), w[i]) : x[i];
}

}  // namespace


int choose_nsplit(int M, int Hkv, int max_pages, int num_sms, bool balance_long) {
    // About one CTA per SM over the (sequence, KV head) pairs at the longest
    // context, at least 8 pages per split there, at most one cluster (16) of splits.
    int pairs = M * Hkv;
    int ns = (num_sms + pairs - 1) / pairs;
    // long contexts: at most ~64 pages per split, so that with many pairs the
    // longest sequence does not serialise a launch (work then spreads over
    // more CTAs than SMs, short sequences' splits finishing early)
    const int balance = (max_pages + 63) / 64;
    if (balance_long && ns < balance) ns = balance;
    const int by_pages = (max_pages + 7) / 8;
    if (ns > by_pages) ns = by_pages;
    if (ns > kMaxAttnSplits) ns = kMaxAttnSplits;
    return ns < 1 ? 1 : ns;
}

int attn_flat_grid(int num_sms) { return kFlatCtas * num_sms; }

bool attn_flat_supported(int H, int Hkv, int d, int M) {
    // from 64 (row, KV head) pairs on (measured: at 32 pairs the cluster
    // kernel's DSMEM combine is cheaper than chunk partials)
    return Hkv > 0 && H == 8 * Hkv && d == 64 && M <= kFlatMaxRows && M * Hkv >= 64;
}

int attn_flat_chunk_pages(int M, int Hkv, int max_pages, int num_sms) {
    // the largest chunk (fewest partials) that still gives every CTA of the
    // grid a couple of chunks at the longest context
    for (int cp = kFlatMaxPages; cp > 2; cp /= 2)
        if ((long long)M * Hkv * ((max_pages + cp - 1) / cp) >= 2LL * attn_flat_grid(num_sms)) return cp;
    return 2;
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
    const int G = p.H / p.Hkv;
    if (p.H % p.Hkv != 0) return cudaErrorInvalidValue;
    if (p.part && p.kv_floats >= 64 && p.kv_floats / 64 < (1ll << 31) && tensor_map_encoder() != nullptr &&
        attn_flat_supported(p.H, p.Hkv, p.d, p.M) && p.chunk_pages >= 1 &&
        p.chunk_pages <= kFlatMaxPages && !getenv("TB_ATTN_GENERIC")) {
        int sms = 148;
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        AttnParams q = p;
        q.probe = getenv("TB_ATTN_PROBE") != nullptr;
        return launch_attn_flat(q, stream, pdl, attn_flat_grid(sms));
    }
    if (G == 8 && p.d == 64 && !getenv("TB_ATTN_GENERIC")) {
        // at most kGqaMaxPages pages per split; the page table's width bounds
        // a sequence's pages, so raise the split count to cover it
        const int need = (p.ptab_stride + kGqaMaxPages - 1) / kGqaMaxPages;
        AttnParams q = p;
        if (need > q.nsplit) q.nsplit = need;
        if (q.nsplit <= kMaxAttnSplits) return launch_attn_gqa8(q, stream, pdl);
    }
#define TB_ATTN_CASE(g, dd) \
    if (G == g && p.d == dd) return launch_attn_t<g, dd>(p, stream, pdl);
    TB_ATTN_CASE(1, 16)
    TB_ATTN_CASE(1, 32)
    TB_ATTN_CASE(1, 64)
    TB_ATTN_CASE(1, 128)
    TB_ATTN_CASE(2, 16)
    TB_ATTN_CASE(2, 32)
    TB_ATTN_CASE(2, 64)
    TB_ATTN_CASE(2, 128)
    TB_ATTN_CASE(4, 16)
    TB_ATTN_CASE(4, 32)
    TB_ATTN_CASE(4, 64)
    TB_ATTN_CASE(4, 128)
    TB_ATTN_CASE(8, 16)
    TB_ATTN_CASE(8, 32)
    TB_ATTN_CASE(8, 64)
#undef TB_ATTN_CASE
    return cudaErrorNotSupported;
}

cudaError_t launch_row_norm(const float* h, int H, int ld, int M, float* out, cudaStream_t stream) {
    row_norm_kernel<<<M, 256, 0, stream>>>(h, H, ld, out);
    return cudaGetLastError();
}
cudaError_t launch_rmsnorm_rows(const float* h, const float* w, int H, int ld, int M, float eps, float* out,
                                cudaStream_t stream) {
    rmsnorm_rows_kernel<<<M, 256, 0, stream>>>(h, w, H, ld, eps, out);
    return cudaGetLastError();
}

cudaError_t launch_attention_probs(const AttnParams& p, float* probs, int L, cudaStream_t stream) {
    size_t smem = (size_t)L * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e =
            cudaFuncSetAttribute(attn_probs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    attn_probs_kernel<<<dim3(p.H, p.M), 128, smem, stream>>>(p, probs, L);
    return cudaGetLastError();
}

__global__ void wait_probe_kernel(int which, const unsigned long long* word, int* err) {
    __shared__ uint64_t bar;
    if (which == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_wait(&bar, 0, err);  // no thread arrives: runs out after kWaitLimitNs
    } else {
        unsigned long long w[1];
        wait_tagged<1>(word, 1u, w, err);  // the word stays zero: runs out
    }
}

cudaError_t launch_wait_probe(int which, const unsigned long long* word, int* err, cudaStream_t stream) {
    wait_probe_kernel<<<1, 1, 0, stream>>>(which, word, err);
    return cudaGetLastError();
}

}  // namespace tb

// ---------------------------------------------------------------------------
// Allocation-free variant of the paged decode attention.
//
// Some callers cannot create device allocations at all: a host that hands
// every byte of HBM to its own pool before loading this library, or code on a
// latency-critical path where cudaMalloc / cudaFree would synchronise the
// device.  tb_paged_attention_dev_noalloc serves them: the split partials are
// combined inside each CTA cluster through distributed shared memory, so the
// kernel needs no global scratch.  Its only device state is one error word
// in a file-scope __device__ variable (every GPU that loads the library holds
// it until exit): a bounded wait that runs out inside the kernel records
// kDevWaitTimeout there, and tb_paged_attention_noalloc_status reads it.  In
// host code the variable's name is only a host-side stand-in, so its device
// address is taken once per device with cudaGetSymbolAddress.
// ---------------------------------------------------------------------------
static __device__ int g_noalloc_err;

namespace tb {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
int g_noalloc_sms[kMaxDevices] = {};
int* g_noalloc_err_dev[kMaxDevices] = {};

// SM count and the error word's device address of the current device `dev`
// (called with `dev` current).
cudaError_t noalloc_setup(int dev) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_sms[dev]) return cudaSuccess;
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_err);
    if (e != cudaSuccess) return e;
    g_noalloc_err_dev[dev] = static_cast<int*>(ptr);
    g_noalloc_sms[dev] = sms;
    return cudaSuccess;
}

int noalloc_device(tb_status* st) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *st = (tb_status)report_error(TB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
        return -1;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        *st = (tb_status)report_error(TB_ERR_UNSUPPORTED, "device index %d is beyond the %d devices supported", dev,
                                      kMaxDevices);
        return -1;
    }
    e = noalloc_setup(dev);
    if (e != cudaSuccess) {
        *st = (tb_status)report_error(TB_ERR_CUDA, "allocation-free attention set-up: %s", cudaGetErrorString(e));
        return -1;
    }
    return dev;
}
}  // namespace

}  // namespace tb

extern "C" tb_status tb_paged_attention_dev_noalloc(void* stream, const float* q, int32_t batch, const float* pool,
                                                    const int32_t* ptab, int32_t ptab_stride, const int32_t* lens,
                                                    int32_t max_len, int32_t layer, int32_t num_layers, int32_t H,
                                                    int32_t Hkv, int32_t d, float* out) {
    using namespace tb;
    if (!q || !pool || !ptab || !lens || !out)
        return (tb_status)report_error(TB_ERR_INVALID_ARGUMENT, "NULL argument");
    if (batch < 1 || max_len < 1 || layer < 0 || layer >= num_layers || H <= 0 || Hkv <= 0 || d <= 0 ||
        H % Hkv != 0)
        return (tb_status)report_error(TB_ERR_INVALID_ARGUMENT, "bad batch / length / layer / head arguments");
    tb_status st = TB_OK;
    const int dev = noalloc_device(&st);
    if (dev < 0) return st;
    const int max_pages = (max_len + kPageTokens - 1) / kPageTokens;
    const int ns = choose_nsplit(batch, Hkv, max_pages, g_noalloc_sms[dev]);
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
    a.err = g_noalloc_err_dev[dev];
    cudaError_t e = launch_attention(a, static_cast<cudaStream_t>(stream), false);
    if (e != cudaSuccess)
        return (tb_status)report_error(e == cudaErrorNotSupported ? TB_ERR_UNSUPPORTED : TB_ERR_CUDA,
                                       "attention launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

extern "C" tb_status tb_paged_attention_noalloc_status(void* stream, int32_t clear) {
    using namespace tb;
    tb_status st = TB_OK;
    const int dev = noalloc_device(&st);
    if (dev < 0) return st;
    cudaStream_t sm = static_cast<cudaStream_t>(stream);
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, g_noalloc_err_dev[dev], sizeof(int), cudaMemcpyDeviceToHost, sm);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(g_noalloc_err_dev[dev], 0, sizeof(int), sm);
    if (e == cudaSuccess) e = cudaStreamSynchronize(sm);
    if (e != cudaSuccess)
        return (tb_status)report_error(TB_ERR_CUDA, "reading the device error word: %s", cudaGetErrorString(e));
    if (v == 0) return TB_OK;
    if (v == kDevWaitTimeout)
        return (tb_status)report_error(TB_ERR_DEVICE_TIMEOUT, "a device-side wait exceeded its time limit");
    return (tb_status)report_error(TB_ERR_STATE, "device error code %d", v);
}
