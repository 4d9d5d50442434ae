// tb_flow.cu -- dataflow persistent decode step for batch 1 with INT8 weights
// (sm_100a).
//
// Same work as tb_step.cu (ModelRunner.step, Sources/TinyBrainRuntime/
// ModelRunner.swift:168-208: per layer QKV -> attention -> o_proj -> gate/up ->
// down, then final norm, LM head, greedy argmax), in one cooperative launch
// with one CTA per SM, but without grid-wide barriers:
//
//  * every value that crosses CTAs is written as one 64-bit word (fp32 bits,
//    32-bit tag).  The tag names the step, layer and phase that produced it, so
//    a reader polls exactly the words it needs until their tags match -- the
//    data load and the synchronisation are the same memory round trip, and a
//    CTA starts a phase as soon as its own inputs exist instead of when the
//    slowest CTA of the grid finished the previous phase.  Every buffer is
//    rewritten only after all its readers provably consumed it (each layer has
//    two all-to-all points: the RMSNorm statistics of the two residual adds);
//  * the residual stream is reduced by row owners: CTA c owns rows
//    [c*H/C, (c+1)*H/C) of h, sums the split-K partials of those rows once,
//    adds the residual, publishes h and its share of sum(h^2).  The next
//    projection's CTAs then read only the C sums and the k range of h their own
//    weight units multiply (instead of every CTA reducing all of h);
//  * INT8 products run on the tensor cores exactly as in tb_step.cu
//    (tb_tc.cuh): a producer warp streams 16 KB weight units and KV pages into
//    a shared-memory ring ahead of the consumers, two threads issue tcgen05.mma
//    kind::i8 against the exact 4-digit split of the activations, four
//    epilogue warps read the tensor-memory accumulators back.
//
// All polls and waits are bounded (2 s of %globaltimer) and also stop as soon
// as any CTA has recorded an error, so a failure ends the step quickly with an
// error code instead of hanging the device.
#include "tb_common.cuh"
#include "tb_kernels.h"
#include "tb_tc.cuh"
#include "tb_unit.cuh"
#include "tb_persist.cuh"

namespace tb {

namespace {

using namespace persist;

constexpr int kMaxRows = 32;  // residual rows owned by one CTA (H / C)
// 8 warps: warp 3 streams (producer), the other 7 consume.  Two warps per SM
// sub-partition leave 255 registers per thread (a 9-warp CTA gets 168, too few
// for these phases without spilling).  Warps 0 and 1 issue tensor-core
// products; warps 4-7 own the four TMEM lane quadrants for the epilogues.
constexpr int kFlowWarps = 8;
constexpr int kFlowThreads = kFlowWarps * 32;
constexpr int kProducerWarp = 3;
constexpr int kFC = (kFlowWarps - 1) * 32;  // consumer threads
#ifndef TB_POLL_BACKOFF_NS
#define TB_POLL_BACKOFF_NS 64
#endif
constexpr unsigned kPollBackoffNs = TB_POLL_BACKOFF_NS;

// Tag kinds (tag = base + 8 * layer + kind).
enum : int { kTagH1 = 0, kTagQKV = 1, kTagATT = 2, kTagO = 3, kTagH2 = 4, kTagGU = 5, kTagDN = 6 };

struct FShared {
    uint64_t* full;
    uint64_t* empty;
    uint64_t* seg;          // [kMaxSegs] segment accumulators complete
    uint64_t* fin;          // [kIssuers] all tensor-core work of an issuer complete
    int* valid;             // [kMaxSlots] attention tile present (page not evicted)
    volatile int* abort;    // a wait or poll gave up
    uint32_t* tmem;         // tensor-memory base address
    float* misc;            // [kMiscFloats]
    uint8_t* ring;
    uint8_t* xd;            // digit operand
    float* att;             // attention scratch
    float* stage;           // activation staging
    float* red;             // [kMaxRows][kMaxTileSegs] partials of the owned residual rows
    float* hrow;            // [kMaxRows] owned residual rows (h_in or h_mid)
    uint8_t* seglist[4];
    uint8_t* segcnt[4];
};

__device__ __forceinline__ uint64_t tpack(float v, uint32_t tag) {
    return (uint64_t)__float_as_uint(v) | ((uint64_t)tag << 32);
}
__device__ __forceinline__ void st_tag(uint64_t* p, float v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(tpack(v, tag)) : "memory");
}
__device__ __forceinline__ uint64_t ld_tag(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Two adjacent tagged words (16-byte aligned).
__device__ __forceinline__ void ld_tag2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool tag_is(uint64_t v, uint32_t tag) { return (uint32_t)(v >> 32) == tag; }
__device__ __forceinline__ float tval(uint64_t v) { return __uint_as_float((uint32_t)v); }

// The phases are separate (non-inlined) functions: inlined into one body their
// register demands add up past the 168 registers a 9-warp CTA gets per thread.
struct Flow {
    const StepParams& p;
    FShared sh;
    Cursor rc;
    int ctid, ci, warp, lane, c, C;  // ci: consumer index 0..kFC-1 (skips the producer warp)
    int r0, r1;                      // owned residual rows
    uint32_t tmem = 0, segpar = 0;
    bool issued_mma = false;
    int xexp = 0;
    uint32_t tbase = 0;              // tag base of this step
    int nph = 0, phase = 0;          // diagnostics

    __device__ Flow(const StepParams& p_, const FShared& sh_) : p(p_), sh(sh_) {
        ctid = threadIdx.x;
        warp = ctid >> 5;
        lane = ctid & 31;
        ci = warp < kProducerWarp ? ctid : ctid - 32;
        c = blockIdx.x;
        C = gridDim.x;
        r0 = (int)((long long)c * p.H / C);
        r1 = (int)((long long)(c + 1) * p.H / C);
    }
    __device__ __forceinline__ uint32_t tag(int l, int kind) const { return tbase + (uint32_t)(8 * l + kind); }
    __device__ void bar() { named_bar_sync(1, kFC); }
    // CTA barrier + abort check (every consumer thread sees the same answer).
    __device__ bool sync_ok() {
        bar();
        return *sh.abort == 0;
    }
    __device__ bool stop() const { return *sh.abort != 0 || *reinterpret_cast<volatile int*>(p.err) != 0; }
    // Give up a poll: record the timeout once, stop this CTA.
    __device__ void give_up() {
        if (*reinterpret_cast<volatile int*>(p.err) == 0) record_error(p.err, kDevWaitTimeout);
        *sh.abort = 1;
    }

    // Diagnostics: per CTA and phase, %globaltimer at the start (0), when the
    // inputs arrived (5), at the end of the prologue (2) and at the end (1).
    __device__ void mark(int which) {
        if (p.trace && ctid == 0 && phase < nph)
            p.trace[((size_t)c * nph + phase) * 8 + which] = global_timer_ns();
    }
    __device__ void begin_phase() { mark(0); }
    __device__ void end_phase() {
        mark(1);
        ++phase;
    }

    // Poll until `fn` (which reloads its words and reports whether all tags
    // matched) succeeds; false after the time limit or once any CTA failed.
    // A failed attempt backs off briefly: hundreds of threads per CTA re-polling
    // in a tight loop would flood the L2 with requests and slow the producers.
    template <class F>
    __device__ bool poll(F&& fn) {
        if (fn()) return true;
        const uint64_t t0 = global_timer_ns();
        while (true) {
            __nanosleep(kPollBackoffNs);
            if (fn()) return true;
            if (stop() || global_timer_ns() - t0 > kWaitLimitNs) {
                give_up();
                return false;
            }
        }
    }

    // One warp polls n tagged "doorbell" words (index -> pointer by `at`) until
    // every tag matches.  Few pollers per word keep the L2 slices that hold the
    // doorbells from being flooded.  No fence is needed on either side: every
    // data word is tagged and verified by its reader, so a doorbell is only a
    // hint that the data is (about to be) there.  `use(i, value)` sees the
    // words of the successful attempt.  Every lane returns the same answer.
    template <class AT, class USE>
    __device__ bool warp_poll(int n, uint32_t tg, AT&& at, USE&& use) {
        const uint64_t t0 = global_timer_ns();
        bool first = true;
        while (true) {
            bool ok = true;
            for (int i = lane; i < n; i += 32) ok &= tag_is(ld_tag(at(i)), tg);
            if (__all_sync(0xffffffffu, ok)) break;
            if (!first && (stop() || global_timer_ns() - t0 > kWaitLimitNs)) {
                if (lane == 0) give_up();
                __syncwarp();
                return false;
            }
            first = false;
            __nanosleep(kPollBackoffNs);
        }
        for (int i = lane; i < n; i += 32) use(i, ld_tag(at(i)));
        return true;
    }
    template <class AT>
    __device__ bool warp_poll(int n, uint32_t tg, AT&& at) {
        return warp_poll(n, tg, at, [](int, uint64_t) {});
    }

    // Sums of the split-K partials of NR groups of 4 consecutive GPU rows (each
    // group within one row block), segments in unit order.  Segments are
    // loaded in polled batches of NL per group (one L2 round trip per batch).
    template <int NR, int NL>
    __device__ bool gather4(const QLayout& L, int which, const uint64_t* P, uint32_t tg, const int (&n0)[NR],
                            float4 (&out)[NR]) {
        int cnt[NR], cmax = 0;
        const uint8_t* lst[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const int rb = n0[r] / kTcTileRows;
            cnt[r] = sh.segcnt[which][rb];
            lst[r] = sh.seglist[which] + rb * kMaxTileSegs;
            cmax = max(cmax, cnt[r]);
            out[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll 1
        for (int g0 = 0; g0 < cmax; g0 += NL) {
            float4 v[NR][NL];
            const bool ok = poll([&]() -> bool {
                bool all = true;
#pragma unroll
                for (int r = 0; r < NR; ++r)
#pragma unroll
                    for (int g = 0; g < NL; ++g) {
                        if (g0 + g < cnt[r]) {
                            const uint64_t* q = P + (size_t)lst[r][g0 + g] * L.Np + n0[r];
                            uint64_t a, b, e, f;
                            ld_tag2(q, a, b);
                            ld_tag2(q + 2, e, f);
                            all &= tag_is(a, tg) & tag_is(b, tg) & tag_is(e, tg) & tag_is(f, tg);
                            v[r][g] = make_float4(tval(a), tval(b), tval(e), tval(f));
                        }
                    }
                return all;
            });
            if (!ok) return false;
#pragma unroll
            for (int r = 0; r < NR; ++r)
#pragma unroll
                for (int g = 0; g < NL; ++g)
                    if (g0 + g < cnt[r]) {
                        if (g0 + g == 0) {
                            out[r] = v[r][g];
                        } else {
                            out[r].x += v[r][g].x;
                            out[r].y += v[r][g].y;
                            out[r].z += v[r][g].z;
                            out[r].w += v[r][g].w;
                        }
                    }
        }
        return true;
    }

    // ---------------------------------------------------------------- residual
    // h[r] = src[r] + sum of the partials of row r (owned rows only); publish h
    // and this CTA's sum of h^2.  src = embedding row (emb != null) or the
    // owned rows kept from the previous residual phase.
    __device__ bool residual(const QLayout* Lp, int which, const uint64_t* P, uint32_t ptag, const float* emb,
                             uint64_t* hout, uint64_t* ssout, uint32_t otag) {
        begin_phase();
        const int nrows = r1 - r0;
        if (P) {
            // one (row, segment) pair per thread
            for (int t = ci; t < nrows * kMaxTileSegs; t += kFC) {
                const int i = t / kMaxTileSegs, g = t % kMaxTileSegs;
                const int r = r0 + i, rb = r / kTcTileRows;
                if (g >= sh.segcnt[which][rb]) continue;
                const uint64_t* q = P + (size_t)sh.seglist[which][rb * kMaxTileSegs + g] * Lp->Np + r;
                uint64_t w = 0;
                if (!poll([&]() {
                        w = ld_tag(q);
                        return tag_is(w, ptag);
                    }))
                    break;
                sh.red[t] = tval(w);
            }
            if (!sync_ok()) return false;
        }
        mark(5);
        if (warp == 0) {
            float ss = 0.0f;
            if (lane < nrows) {
                const int r = r0 + lane;
                float a = 0.0f;
                if (P) {
                    const int cnt = sh.segcnt[which][r / kTcTileRows];
                    a = sh.red[lane * kMaxTileSegs];
                    for (int g = 1; g < cnt; ++g) a += sh.red[lane * kMaxTileSegs + g];
                }
                const float src = emb ? __ldg(emb + r) : sh.hrow[lane];
                const float h = P ? __fadd_rn(src, a) : src;
                sh.hrow[lane] = h;
                st_tag(hout + r, h, otag);
                ss = __fmul_rn(h, h);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            // the share of sum(h^2) is the doorbell, issued after the rows of h
            __syncwarp();
            if (lane == 0) st_tag(ssout + c, ss, otag);
        }
        end_phase();
        return true;
    }

    // ------------------------------------------------------------- prologues
    // Block-wide max -> digit exponent (all consumer threads).
    __device__ void set_digit_exponent(float mx) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) sh.misc[32 + warp] = mx;
        bar();
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < kFlowWarps; ++w)
            if (w != kProducerWarp) t = fmaxf(t, sh.misc[32 + w]);
        xexp = digit_exponent(t * 1.0000002f);
    }
    __device__ __forceinline__ void put_group(int k, float4 v) {
        put_digits4(sh.xd, 8, k, 0, v, __int_as_float((127 - xexp) << 23));
    }
    // Units of K touched by this CTA's units of a phase: a cyclic run.
    __device__ void unit_run(const QLayout& L, int& first, int& count) {
        const int U = phase_units(L);
        const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
        first = u0 % L.slabs;
        count = min(u1 - u0, L.slabs);
    }
    __device__ __forceinline__ int kth_in_run(const QLayout& L, int first, int count, int e) {
        const int i = e / L.slab_k;
        if (i >= count) return -1;
        int s = first + i;
        if (s >= L.slabs) s -= L.slabs;
        return s * L.slab_k + (e - i * L.slab_k);
    }

    // x = RMSNorm(h) * w for the k this CTA's units need (all k: whole).
    __device__ bool normed_prologue(const QLayout& L, const uint64_t* hin, const uint64_t* ssin, uint32_t tg,
                                    const float* normw, bool whole) {
        // sum of h^2: one published share per CTA (doorbells), polled by warp 0,
        // summed in a fixed order
        if (warp == 0) {
            // each lane polls its (at most 8) shares and keeps the values of the
            // attempt in which every tag matched
            float v = 0.0f;
            const uint64_t t0 = global_timer_ns();
            bool first = true;
            while (true) {
                uint64_t w[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) w[q] = (lane + 32 * q < C) ? ld_tag(ssin + lane + 32 * q) : ((uint64_t)tg << 32);
                bool ok = true;
#pragma unroll
                for (int q = 0; q < 8; ++q) ok &= tag_is(w[q], tg);
                if (__all_sync(0xffffffffu, ok)) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) v += tval(w[q]);
                    break;
                }
                if (!first && (stop() || global_timer_ns() - t0 > kWaitLimitNs)) {
                    if (lane == 0) give_up();
                    break;
                }
                first = false;
                __nanosleep(kPollBackoffNs);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) sh.misc[0] = v;
        }
        int first = 0, count = L.slabs;
        if (!whole) unit_run(L, first, count);
        const int total = count * L.slab_k;
        if (!sync_ok()) return false;
        mark(6);
        const float ss = sh.misc[0];
        float inv = 1.0f;
        if (normw) inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.H), p.eps)));
        float mx = 0.0f;
        bool ok = true;
        for (int e = 4 * ci; e < total && ok; e += 4 * kFC) {
            const int k = kth_in_run(L, first, count, e);
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < p.H) {  // H % 4 == 0
                uint64_t a, b, d, f;
                ok = poll([&]() {
                    ld_tag2(hin + k, a, b);
                    ld_tag2(hin + k + 2, d, f);
                    return tag_is(a, tg) & tag_is(b, tg) & tag_is(d, tg) & tag_is(f, tg);
                });
                const float4 wv = normw ? __ldg(reinterpret_cast<const float4*>(normw + k))
                                        : make_float4(1.f, 1.f, 1.f, 1.f);
                x = make_float4(__fmul_rn(__fmul_rn(tval(a), inv), wv.x), __fmul_rn(__fmul_rn(tval(b), inv), wv.y),
                                __fmul_rn(__fmul_rn(tval(d), inv), wv.z), __fmul_rn(__fmul_rn(tval(f), inv), wv.w));
            }
            *reinterpret_cast<float4*>(sh.stage + e) = x;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
        mark(5);
        set_digit_exponent(mx);
        for (int e = 4 * ci; e < total; e += 4 * kFC)
            put_group(kth_in_run(L, first, count, e), *reinterpret_cast<const float4*>(sh.stage + e));
        fence_proxy_async_shared();
        return sync_ok();
    }

    // ctx[k] for the k this CTA's o_proj units need: combine the attention
    // splits (softmax rescaling of the (m, l, acc) partials, split order).
    template <int G, int D>
    __device__ bool ctx_prologue(uint32_t tg) {
        constexpr int AMAX = 16;
        const QLayout& L = p.Lo;
        const int A = p.A;
        float2* ml = reinterpret_cast<float2*>(sh.misc + 64);  // [Hkv][A][G]
        float* wts = sh.att;                                     // [Hkv][G][A]
        const uint64_t* P = p.f_att;
        int first, count;
        unit_run(L, first, count);
        const int total = count * L.slab_k;
        bool ok = true;
        // kv heads touched by this CTA's k range (a cyclic run of units)
        const int hk_lo = (first * L.slab_k) / (G * D);
        const int hk_n = count >= L.slabs ? p.Hkv : min(p.Hkv, ((count * L.slab_k + G * D - 1) / (G * D)) + 1);
        if (warp == 0) {
            ok = warp_poll(hk_n * A * G, tg, [&](int i) {
                const int hk = (hk_lo + i / (A * G)) % p.Hkv;
                return P + ((size_t)hk * A * G + i % (A * G)) * (D + 2) + D + 1;
            });
        }
        if (!sync_ok()) return false;
        const int nml = p.Hkv * A * G;
        for (int e = ci; e < nml; e += kFC) {
            const int hk = e / (A * G);
            if (((hk - hk_lo + p.Hkv) % p.Hkv) >= hk_n) continue;
            uint64_t m, l;
            ok = poll([&]() {
                ld_tag2(P + (size_t)e * (D + 2) + D, m, l);
                return tag_is(m, tg) & tag_is(l, tg);
            });
            ml[e] = make_float2(tval(m), tval(l));
            if (!ok) break;
        }
        if (!sync_ok()) return false;
        // weights of the splits: 16 lanes per (kv head, query head) pair
        for (int base = 0; base < p.Hkv * G * 16; base += kFC) {
            const int e = (base + ci) >> 4, sp = ci & 15;
            const bool live = e < p.Hkv * G && sp < A;
            const int hk = e / G, g = e % G;
            const float2 t = live ? ml[(hk * A + sp) * G + g] : make_float2(-INFINITY, 0.0f);
            float M = t.x;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            const float w = (t.x == -INFINITY || M == -INFINITY) ? 0.0f : expf(t.x - M);
            float den = w * t.y;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
            const float inv = den > 0.0f ? 1.0f / den : 0.0f;
            if (live) wts[e * A + sp] = w * inv;
        }
        bar();
        float mx = 0.0f;
        for (int e = 4 * ci; e < total && ok; e += 4 * kFC) {
            const int k = kth_in_run(L, first, count, e);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < L.K) {
                const int hq = k / D, i = k % D;
                const int hk = hq / G, g = hq % G;
                // polled batches of 8 splits (bounded registers), accumulated in split order
                const float* w = wts + (hk * G + g) * A;
                constexpr int HB = AMAX / 4;
#pragma unroll 1
                for (int hb = 0; hb < A && ok; hb += HB) {
                    float4 a[HB];
                    ok = poll([&]() {
                        bool all = true;
#pragma unroll
                        for (int s2 = 0; s2 < HB; ++s2) {
                            const int sp = hb + s2;
                            if (sp < A) {
                                const uint64_t* q = P + (((size_t)hk * A + sp) * G + g) * (D + 2) + i;
                                uint64_t x0, x1, x2, x3;
                                ld_tag2(q, x0, x1);
                                ld_tag2(q + 2, x2, x3);
                                all &= tag_is(x0, tg) & tag_is(x1, tg) & tag_is(x2, tg) & tag_is(x3, tg);
                                a[s2] = make_float4(tval(x0), tval(x1), tval(x2), tval(x3));
                            }
                        }
                        return all;
                    });
#pragma unroll
                    for (int s2 = 0; s2 < HB; ++s2)
                        if (hb + s2 < A) {
                            v.x = fmaf(w[hb + s2], a[s2].x, v.x);
                            v.y = fmaf(w[hb + s2], a[s2].y, v.y);
                            v.z = fmaf(w[hb + s2], a[s2].z, v.z);
                            v.w = fmaf(w[hb + s2], a[s2].w, v.w);
                        }
                }
            }
            *reinterpret_cast<float4*>(sh.stage + e) = v;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        mark(5);
        set_digit_exponent(mx);
        for (int e = 4 * ci; e < total; e += 4 * kFC)
            put_group(kth_in_run(L, first, count, e), *reinterpret_cast<const float4*>(sh.stage + e));
        fence_proxy_async_shared();
        return sync_ok();
    }

    // act[k] = silu(gate[k]) * up[k] for the k this CTA's down units need.
    __device__ bool act_prologue(uint32_t tg) {
        const QLayout& L = p.Ldn;
        const QLayout& GL = p.Lgu;
        int first, count;
        unit_run(L, first, count);
        const int total = count * L.slab_k;
        const int half = GL.RB / 2;
        float mx = 0.0f;
        bool ok = true;
        if (warp == 0) {
            // doorbells of the gate/up row blocks holding act[k] for this k range:
            // unit s of the down matrix covers k [128 s, 128 s + 128) = one
            // half of gate/up row blocks 2s and 2s + 1 (64 k per block)
            const int per = L.slab_k / half;  // gate/up row blocks per down unit
            int n = 0;
            for (int i = 0; i < count; ++i) {
                int su = first + i;
                if (su >= L.slabs) su -= L.slabs;
                for (int b = 0; b < per; ++b) {
                    const int T = su * per + b;
                    if (T < GL.Np / GL.RB) n += sh.segcnt[2][T];
                }
            }
            ok = warp_poll(n, tg, [&](int idx) {
                for (int i = 0; i < count; ++i) {
                    int su = first + i;
                    if (su >= L.slabs) su -= L.slabs;
                    for (int b = 0; b < per; ++b) {
                        const int T = su * per + b;
                        if (T >= GL.Np / GL.RB) continue;
                        const int cn = sh.segcnt[2][T];
                        if (idx < cn) return p.f_dbgu + (size_t)T * GL.slabs + sh.seglist[2][T * kMaxTileSegs + idx];
                        idx -= cn;
                    }
                }
                return p.f_dbgu;  // unreachable
            });
        }
        if (!sync_ok()) return false;
        for (int e = 4 * ci; e < total && ok; e += 4 * kFC) {
            const int k = kth_in_run(L, first, count, e);
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < L.K) {
                const int grow = fused_row(GL, k, 0, 1);
                const int n0[2] = {grow, grow + half};
                float4 gu[2];
                ok = gather4<2, 3>(GL, 2, p.f_gu, tg, n0, gu);
                const float4 g = gu[0], u = gu[1];
                a = make_float4(__fmul_rn(silu_ref(g.x), u.x), __fmul_rn(silu_ref(g.y), u.y),
                                __fmul_rn(silu_ref(g.z), u.z), __fmul_rn(silu_ref(g.w), u.w));
            }
            *reinterpret_cast<float4*>(sh.stage + e) = a;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
        }
        mark(5);
        set_digit_exponent(mx);
        for (int e = 4 * ci; e < total; e += 4 * kFC)
            put_group(kth_in_run(L, first, count, e), *reinterpret_cast<const float4*>(sh.stage + e));
        fence_proxy_async_shared();
        return sync_ok();
    }

    // ----------------------------------------------------------- tensor core
    // Units of this CTA's range of a GEMV phase: lane 0 of warps 0 and 1 issue
    // alternate units into their own accumulator blocks of each segment; warps
    // 4-7 combine a segment's blocks and digits, apply scale and bias, and
    // publish one tagged partial per row and segment.
    __device__ void gemv(const QLayout& L, uint64_t* part, const float* sc, const float* bias, uint32_t otag,
                         uint64_t* db) {
        mark(2);
        const int U = phase_units(L);
        const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
        if (warp < kIssuers) {
            if (lane == 0 && u1 > u0) {
                Cursor q = rc;
                int s = u0 % L.slabs, j = 0;
                bool fresh = true;
                tc_fence_after();
                for (int u = u0; u < u1; ++u) {
                    if (*sh.abort) break;
                    if (((u - u0) & (kIssuers - 1)) == warp) {
                        if (!mbar_wait(&sh.full[q.st], q.ph, p.err)) {
                            *sh.abort = 1;
                            break;
                        }
                        tc_fence_after();
                        tc_unit_mma(tmem + 8 * (kIssuers * j + warp), smem_u32(sh.ring + (size_t)q.st * p.slot_bytes),
                                    smem_u32(sh.xd + (size_t)s * (kTcUnitK / 16) * 128), 8, !fresh);
                        tc_commit(&sh.empty[q.st]);
                        issued_mma = true;
                        fresh = false;
                    }
                    q.next(p.nslots);
                    if (u + 1 == u1 || s + 1 == L.slabs) {
                        tc_commit(&sh.seg[j]);
                        ++j;
                        fresh = true;
                    }
                    if (++s == L.slabs) s = 0;
                }
            }
            __syncwarp();
        } else if (warp >= 4) {
            const int row = 32 * (warp - 4) + lane;
            const uint32_t lane_base = (uint32_t)(32 * (warp - 4)) << 16;
            int j = 0;
            for (int u = u0; u < u1; ++j) {
                const int T = u / L.slabs, sfirst = u - T * L.slabs;
                const int uend = min(u1, (T + 1) * L.slabs);
                const int n = T * kTcTileRows + row;
                const float scv = __ldg(sc + n);
                const float bv = (bias && sfirst == 0) ? __ldg(bias + n) : 0.0f;
                const uint32_t par = (segpar >> j) & 1u;
                segpar ^= 1u << j;
                const bool ok = !*sh.abort && mbar_wait(&sh.seg[j], par, p.err);
                if (!ok) *sh.abort = 1;
                tc_fence_after();
                int d[8], e[8];
                tmem_ld8(tmem + lane_base + 8 * (kIssuers * j), d);
                tmem_ld8(tmem + lane_base + 8 * (kIssuers * j + 1), e);
                tmem_ld_wait();
                const bool two = uend - u >= 2 || ((u - u0) & 1);
                const bool one = uend - u >= 2 || !((u - u0) & 1);
#pragma unroll
                for (int i = 0; i < 4; ++i) d[i] = (one ? d[i] : 0) + (two ? e[i] : 0);
                if (ok) {
                    float v = __fmul_rn(combine_digits(d, xexp), scv);
                    if (bias && sfirst == 0) v = __fadd_rn(v, bv);
                    st_tag(part + (size_t)sfirst * L.Np + n, v, otag);
                }
                u = uend;
            }
            tc_fence_before();
            if (db) {
                // doorbell per segment (row block, first unit), after all rows are stored
                named_bar_sync(2, 128);
                if (warp == 4 && lane == 0 && !*sh.abort) {
                    for (int u = u0; u < u1;) {
                        const int T = u / L.slabs;
                        st_tag(db + (size_t)T * L.slabs + (u - T * L.slabs), 0.0f, otag);
                        u = min(u1, (T + 1) * L.slabs);
                    }
                }
            }
        }
        rc.advance(u1 - u0, p.nslots);
        end_phase();
    }

    // ---------------------------------------------------------------- attention
    // q (RoPE'd), new k (RoPE'd), v of this KV head from the qkv partials, KV
    // append by the split that owns the current position, online-softmax over
    // the split's pages (ring tiles), tagged (acc, m, l) partials.
    template <int G, int D>
    __device__ bool attention(int layer, int pos, int npages, uint32_t itag, uint32_t otag) {
        // QK: G*16 (query head, row) pairs x DP lanes each (largest power of two that fits)
        constexpr int NPAIR = G * kPageTokens;
        constexpr int DP = (NPAIR * 8 <= kFC) ? 8 : (NPAIR * 4 <= kFC) ? 4 : (NPAIR * 2 <= kFC) ? 2 : 1;
        constexpr int CHK = D / DP;
        constexpr int PVT = G * (D / 4);
        static_assert(NPAIR * DP <= kFC && CHK >= 1 && CHK <= 128 && PVT <= kFC, "head geometry");
        begin_phase();
        const int A = p.A;
        const int head = c / A, split = c % A;
        const int pps = (npages + A - 1) / A;
        const int pg0 = min(npages, split * pps), pg1 = min(npages, pg0 + pps);
        float* qs = sh.att;        // [G][D]
        float* knew = qs + G * D;  // [D]
        float* vnew = knew + D;    // [D]
        float* S = vnew + D;       // [2][G][16]
        const QLayout& L = p.Lqkv;
        const float2* rope = p.rope + (size_t)min(pos, p.rope_max_pos - 1) * (D / 2);
        const bool owner = pg0 < pg1 && pg1 == npages;
        // groups of 4 rows: q (G*D/4), k (D/4), v (D/4) (ModelRunner.swift:499-515)
        const int nq = G * D / 4, nk = D / 4;
        bool ok = true;
        if (warp == 0) {
            // doorbells of the segments of the row blocks holding this head's q, k, v
            int tb[3], nt[3];
            tb[0] = (head * G * D) / kTcTileRows;
            nt[0] = (head * G * D + G * D - 1) / kTcTileRows - tb[0] + 1;
            tb[1] = (p.H + head * D) / kTcTileRows;
            nt[1] = 1;
            tb[2] = (p.H + p.kvd + head * D) / kTcTileRows;
            nt[2] = 1;
            int n = 0, base[4];
            for (int q = 0; q < 3; ++q) {
                base[q] = n;
                for (int t = 0; t < nt[q]; ++t) n += sh.segcnt[0][tb[q] + t];
            }
            base[3] = n;
            ok = warp_poll(n, itag, [&](int i) {
                int q = 0;
                while (i >= base[q + 1]) ++q;
                int t = tb[q], r = i - base[q];
                while (r >= sh.segcnt[0][t]) r -= sh.segcnt[0][t++];
                return p.f_dbqkv + (size_t)t * L.slabs + sh.seglist[0][t * kMaxTileSegs + r];
            });
        }
        if (!sync_ok()) return false;
        for (int t = ci; t < nq + 2 * nk && ok; t += kFC) {
            int n0;
            if (t < nq)
                n0 = head * G * D + 4 * t;
            else if (t < nq + nk)
                n0 = p.H + head * D + 4 * (t - nq);
            else
                n0 = p.H + p.kvd + head * D + 4 * (t - nq - nk);
            const int nn[1] = {n0};
            float4 vv[1];
            ok = gather4<1, 4>(L, 0, p.f_qkv, itag, nn, vv);
            const float4 v = vv[0];
            if (t < nq + nk) {
                const int i0 = (t < nq ? 4 * t : 4 * (t - nq)) % D;
                const float2 c0 = rope[i0 / 2], c1 = rope[i0 / 2 + 1];
                const float a0 = __fsub_rn(__fmul_rn(v.x, c0.x), __fmul_rn(v.y, c0.y));
                const float a1 = __fadd_rn(__fmul_rn(v.x, c0.y), __fmul_rn(v.y, c0.x));
                const float a2 = __fsub_rn(__fmul_rn(v.z, c1.x), __fmul_rn(v.w, c1.y));
                const float a3 = __fadd_rn(__fmul_rn(v.z, c1.y), __fmul_rn(v.w, c1.x));
                float* dst = t < nq ? qs + 4 * t : knew + 4 * (t - nq);
                dst[0] = a0;
                dst[1] = a1;
                dst[2] = a2;
                dst[3] = a3;
            } else {
                float* dst = vnew + 4 * (t - nq - nk);
                dst[0] = v.x;
                dst[1] = v.y;
                dst[2] = v.z;
                dst[3] = v.w;
            }
        }
        if (!sync_ok()) return false;
        mark(5);
        if (owner) {  // append k, v at the current position (KVCache.swift:157-224)
            const int page = p.ptab[pos / kPageTokens];
            if (page < 0) {
                if (ctid == 0) record_error(p.err, kDevBadPage);
            } else {
                const size_t kb =
                    ((((size_t)page * p.num_layers + layer) * 2 + 0) * p.Hkv + head) * kPageTokens + pos % kPageTokens;
                const size_t vb =
                    ((((size_t)page * p.num_layers + layer) * 2 + 1) * p.Hkv + head) * kPageTokens + pos % kPageTokens;
                for (int e = ci; e < D; e += kFC) {
                    p.kv_pool[kb * D + e] = knew[e];
                    p.kv_pool[vb * D + e] = vnew[e];
                }
            }
        }
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
        const bool qk = ci < NPAIR * DP;
        const int pair = qk ? ci / DP : 0, dp = ci % DP;
        const int gq = pair / kPageTokens, j = pair % kPageTokens;
        float qrot[CHK];
#pragma unroll
        for (int e = 0; e < CHK; ++e) qrot[e] = qs[gq * D + dp * CHK + (e + j) % CHK];
        const bool pv = ci < PVT;
        const int gv = ci / (D / 4), dv = (ci % (D / 4)) * 4;
        float run_m = -INFINITY, run_l = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        const int cur_row = pos % kPageTokens;
        for (int i = 0; i < pg1 - pg0; ++i) {
            // every warp walks every barrier even after a failed wait (no early exit)
            const int st = rc.st;
            bool have = !*sh.abort && mbar_wait(&sh.full[st], rc.ph, p.err);
            if (!have) *sh.abort = 1;
            const uint8_t* slot = sh.ring + (size_t)st * p.slot_bytes;
            const float* Kt = have ? reinterpret_cast<const float*>(slot) : knew;
            const float* Vt = have ? Kt + kPageTokens * D : vnew;
            const bool okp = have && sh.valid[st] != 0;
            const bool last = have && owner && (pg0 + i == npages - 1);
            float* Sb = S + (i & 1) * G * kPageTokens;
            {
                float dot = 0.0f;
                const bool cur = last && j == cur_row;
                const float* kr = cur ? knew + dp * CHK : Kt + j * D + dp * CHK;
                if (okp || cur) {
#pragma unroll
                    for (int e = 0; e < CHK; ++e) dot = fmaf(qrot[e], kr[(e + j) % CHK], dot);
                }
#pragma unroll
                for (int o = DP / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
                const int tok = (pg0 + i) * kPageTokens + j;
                if (qk && dp == 0) Sb[gq * kPageTokens + j] = (tok <= pos) ? __fmul_rn(dot, scale) : -INFINITY;
            }
            bar();
            if (pv) {
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
                    const bool cur = last && jj == cur_row;
                    if (okp || cur) {
                        const float4 v = cur ? *reinterpret_cast<const float4*>(vnew + dv)
                                             : *reinterpret_cast<const float4*>(Vt + jj * D + dv);
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
            bar();
            if (ctid == 0 && have) mbar_arrive(&sh.empty[st]);
            rc.next(p.nslots);
        }
        uint64_t* part = p.f_att + (((size_t)head * A + split) * G) * (D + 2);
        if (pv && !*sh.abort) {
            uint64_t* row = part + (size_t)gv * (D + 2);
            st_tag(row + dv + 0, acc.x, otag);
            st_tag(row + dv + 1, acc.y, otag);
            st_tag(row + dv + 2, acc.z, otag);
            st_tag(row + dv + 3, acc.w, otag);
            if (dv == 0) {
                S[2 * gv] = run_m;
                S[2 * gv + 1] = run_l;
            }
        }
        bar();
        // (m, l) of each query head is its doorbell: stored after the acc rows
        if (ci < G && !*sh.abort) {
            st_tag(part + (size_t)ci * (D + 2) + D, S[2 * ci], otag);
            st_tag(part + (size_t)ci * (D + 2) + D + 1, S[2 * ci + 1], otag);
        }
        end_phase();
        return true;
    }

    // ------------------------------------------------------------------ LM head
    // Whole tiles per CTA: logits, packed argmax (Sampler.swift:126-138).
    __device__ void lm_head(unsigned long long* best_out) {
        mark(2);
        const QLayout& L = p.Llm;
        const int nt = L.Np / kTcTileRows;
        const int t0 = (int)((long long)c * nt / C), t1 = (int)((long long)(c + 1) * nt / C);
        if (warp < kIssuers) {
            if (lane == 0 && t1 > t0) {
                Cursor q = rc;
                tc_fence_after();
                int v = 0;
                for (int t = t0; t < t1 && !*sh.abort; ++t) {
                    bool fresh = true;
                    for (int s = 0; s < L.slabs; ++s, ++v) {
                        if ((v & (kIssuers - 1)) == warp) {
                            if (!mbar_wait(&sh.full[q.st], q.ph, p.err)) {
                                *sh.abort = 1;
                                break;
                            }
                            tc_fence_after();
                            tc_unit_mma(tmem + 8 * (kIssuers * (t - t0) + warp),
                                        smem_u32(sh.ring + (size_t)q.st * p.slot_bytes),
                                        smem_u32(sh.xd + (size_t)s * (kTcUnitK / 16) * 128), 8, !fresh);
                            tc_commit(&sh.empty[q.st]);
                            issued_mma = true;
                            fresh = false;
                        }
                        q.next(p.nslots);
                    }
                    if (*sh.abort) break;
                    tc_commit(&sh.seg[t - t0]);
                }
            }
            __syncwarp();
        } else if (warp >= 4) {
            const int row = 32 * (warp - 4) + lane;
            const uint32_t lane_base = (uint32_t)(32 * (warp - 4)) << 16;
            unsigned long long best = 0ull;
            for (int t = t0; t < t1; ++t) {
                const int j = t - t0;
                const int n = t * kTcTileRows + row;
                const bool inr = n < L.N;
                const float scv = inr ? __ldg(p.lm_s + n) : 0.0f;
                const float bv = (inr && p.lm_b) ? __ldg(p.lm_b + n) : 0.0f;
                const uint32_t par = (segpar >> j) & 1u;
                segpar ^= 1u << j;
                const bool ok = !*sh.abort && mbar_wait(&sh.seg[j], par, p.err);
                if (!ok) *sh.abort = 1;
                tc_fence_after();
                int d[8], e[8];
                tmem_ld8(tmem + lane_base + 8 * (kIssuers * j), d);
                tmem_ld8(tmem + lane_base + 8 * (kIssuers * j + 1), e);
                tmem_ld_wait();
                const int v0 = j * L.slabs;
                const bool one = L.slabs >= 2 || !(v0 & 1);
                const bool two = L.slabs >= 2 || (v0 & 1);
#pragma unroll
                for (int i = 0; i < 4; ++i) d[i] = (one ? d[i] : 0) + (two ? e[i] : 0);
                if (ok && inr) {
                    float lv = __fmul_rn(combine_digits(d, xexp), scv);
                    if (p.lm_b) lv = __fadd_rn(lv, bv);
                    if (p.logits) p.logits[n] = lv;
                    const unsigned long long key = argmax_key(lv, n);
                    best = key > best ? key : best;
                }
            }
            tc_fence_before();
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
                best = t > best ? t : best;
            }
            if (lane == 0 && best != 0ull) atomicMax(best_out, best);
        }
        rc.advance((t1 - t0) * L.slabs, p.nslots);
        end_phase();
    }
};

template <int G, int D>
__device__ void run_flow(Flow& f, const StepParams& p, int pos, int npages) {
    const int A = p.A;
    const bool att_cta = f.c < A * p.Hkv;
    int tok = p.seq->token;
    if (tok < 0 || tok >= p.V) {
        if (threadIdx.x == 0) record_error(p.err, kDevBadToken);
        tok = 0;
    }
    for (int l = 0; l < p.num_layers; ++l) {
        const StepLayer& ly = p.layers[l];
        // h_in = (embedding | h_mid(l-1) + down(l-1)), owned rows
        if (!f.residual(&p.Ldn, 3, l ? p.f_dn : nullptr, f.tag(l - 1, kTagDN), l ? nullptr : p.emb + (size_t)tok * p.H,
                        p.f_h[0], p.f_ss[0], f.tag(l, kTagH1)))
            return;
        // QKV
        f.begin_phase();
        if (!f.normed_prologue(p.Lqkv, p.f_h[0], p.f_ss[0], f.tag(l, kTagH1), ly.in_norm, false)) return;
        f.gemv(p.Lqkv, p.f_qkv, ly.qkv_s, ly.qkv_b, f.tag(l, kTagQKV), p.f_dbqkv);
        if (!f.sync_ok()) return;
        // attention
        if (att_cta) {
            if (!f.attention<G, D>(l, pos, npages, f.tag(l, kTagQKV), f.tag(l, kTagATT))) return;
        } else {
            ++f.phase;
        }
        // o_proj
        f.begin_phase();
        if (!f.ctx_prologue<G, D>(f.tag(l, kTagATT))) return;
        f.gemv(p.Lo, p.f_o, ly.o_s, ly.o_b, f.tag(l, kTagO), nullptr);
        if (!f.sync_ok()) return;
        // h_mid = h_in + o, owned rows
        if (!f.residual(&p.Lo, 1, p.f_o, f.tag(l, kTagO), nullptr, p.f_h[1], p.f_ss[1], f.tag(l, kTagH2))) return;
        // gate/up
        f.begin_phase();
        if (!f.normed_prologue(p.Lgu, p.f_h[1], p.f_ss[1], f.tag(l, kTagH2), ly.post_norm, false)) return;
        f.gemv(p.Lgu, p.f_gu, ly.gu_s, ly.gu_b, f.tag(l, kTagGU), p.f_dbgu);
        if (!f.sync_ok()) return;
        // down
        f.begin_phase();
        if (!f.act_prologue(f.tag(l, kTagGU))) return;
        f.gemv(p.Ldn, p.f_dn, ly.dn_s, ly.dn_b, f.tag(l, kTagDN), nullptr);
        if (!f.sync_ok()) return;
    }
    const int L = p.num_layers;
    if (!f.residual(&p.Ldn, 3, p.f_dn, f.tag(L - 1, kTagDN), nullptr, p.f_h[0], p.f_ss[0], f.tag(L, kTagH1))) return;
    f.begin_phase();
    if (!f.normed_prologue(p.Llm, p.f_h[0], p.f_ss[0], f.tag(L, kTagH1), p.final_norm, true)) return;
    f.lm_head(&p.seq->best);
    if (!f.sync_ok()) return;
    // the last CTA to finish advances the step (ModelRunner.swift:251-292)
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int t = atomicAdd(p.f_ticket, 1u);
        if (t == (unsigned int)f.C - 1) {
            __threadfence();
            finish_sequence_step(*p.seq, 0, p.out_tokens, p.prompt, p.prompt_stride);
            *p.f_ticket = 0u;
            *p.f_epoch = *p.f_epoch + 1u;
        }
    }
}

template <int G, int D>
__global__ void __launch_bounds__(kFlowThreads, 1) decode_flow_kernel(const __grid_constant__ StepParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    FShared sh;
    sh.full = reinterpret_cast<uint64_t*>(smem);
    sh.empty = sh.full + kMaxSlots;
    sh.seg = sh.empty + kMaxSlots;
    sh.fin = sh.seg + kMaxSegs;
    sh.valid = reinterpret_cast<int*>(sh.fin + kIssuers);
    sh.abort = reinterpret_cast<volatile int*>(sh.valid + kMaxSlots);
    sh.tmem = reinterpret_cast<uint32_t*>(const_cast<int*>(sh.abort + 2));
    sh.misc = reinterpret_cast<float*>(smem + kBarRegion);
    sh.ring = smem + kBarRegion + kMiscFloats * 4;
    sh.xd = sh.ring + (size_t)p.nslots * p.slot_bytes;
    const QLayout* Ls[5] = {&p.Lqkv, &p.Lo, &p.Lgu, &p.Ldn, &p.Llm};
    int kmax = 0;
    for (int i = 0; i < 5; ++i) kmax = max(kmax, Ls[i]->slabs * Ls[i]->slab_k);
    sh.att = reinterpret_cast<float*>(sh.xd + (size_t)kmax * 8);
    sh.stage = sh.att + att_floats(G, D, p.Hkv, p.A);
    sh.red = sh.stage + kmax;
    sh.hrow = sh.red + kMaxRows * kMaxTileSegs;
    {
        uint8_t* t = reinterpret_cast<uint8_t*>(sh.hrow + kMaxRows);
        for (int i = 0; i < 4; ++i) {
            const int nrb = Ls[i]->Np / kTcTileRows;
            sh.seglist[i] = t;
            sh.segcnt[i] = t + nrb * kMaxTileSegs;
            t += seg_table_bytes(*Ls[i]);
        }
    }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = gridDim.x, c = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nslots; ++i) {
            mbar_init(&sh.full[i], 1);
            mbar_init(&sh.empty[i], 1);
        }
        for (int i = 0; i < kMaxSegs; ++i) mbar_init(&sh.seg[i], kIssuers);
        for (int i = 0; i < kIssuers; ++i) mbar_init(&sh.fin[i], 1);
        *sh.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(sh.tmem, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const int pos = p.seq->pos;
    const int npages = pos / kPageTokens + 1;
    const int A = p.A;
    const int head = c < A * p.Hkv ? c / A : -1;
    const int split = c < A * p.Hkv ? c % A : 0;
    const int pps = (npages + A - 1) / A;
    const int apg0 = min(npages, split * pps), apg1 = min(npages, apg0 + pps);

    if (warp == kProducerWarp) {
        if (lane == 0) {
            Producer<FShared> pr(p, sh);
            auto range = [&](const QLayout& L, int& u0, int& u1) {
                const int U = phase_units(L);
                u0 = (int)((long long)c * U / C);
                u1 = (int)((long long)(c + 1) * U / C);
            };
            int u0, u1;
            for (int l = 0; l < p.num_layers && !pr.dead; ++l) {
                const StepLayer& ly = p.layers[l];
                range(p.Lqkv, u0, u1);
                pr.gemv<8>(p.Lqkv, ly.qkv_w, ly.qkv_s, u0, u1);
                if (head >= 0) pr.attention(l, head, apg0, apg1);
                range(p.Lo, u0, u1);
                pr.gemv<8>(p.Lo, ly.o_w, ly.o_s, u0, u1);
                range(p.Lgu, u0, u1);
                pr.gemv<8>(p.Lgu, ly.gu_w, ly.gu_s, u0, u1);
                range(p.Ldn, u0, u1);
                pr.gemv<8>(p.Ldn, ly.dn_w, ly.dn_s, u0, u1);
            }
            if (!pr.dead) {
                const int nrb = p.Llm.Np / kTcTileRows;
                const int r0 = (int)((long long)c * nrb / C), r1 = (int)((long long)(c + 1) * nrb / C);
                pr.gemv<8>(p.Llm, p.lm_w, p.lm_s, r0 * p.Llm.slabs, r1 * p.Llm.slabs);
            }
            if (pr.dead) pr.drain();
        }
        return;
    }

    Flow f(p, sh);
    f.nph = 7 * p.num_layers + 2;
    f.tbase = (*reinterpret_cast<volatile const unsigned int*>(p.f_epoch) + 1u) * (uint32_t)(8 * (p.num_layers + 1));
    for (int i = 0; i < 4; ++i) build_seglist(sh.seglist[i], sh.segcnt[i], *Ls[i], C, f.ci, kFC);
    {
        // digit rows 4..7 of the operand stay zero for the whole step
        uint32_t* x = reinterpret_cast<uint32_t*>(sh.xd);
        for (int i = f.ci; i < kmax * 2; i += kFC) x[i] = 0u;
        f.tmem = *sh.tmem;
    }
    f.bar();
    run_flow<G, D>(f, p, pos, npages);

    // Teardown: wait (bounded) for this CTA's tensor-core work, free TMEM.
    if (warp < kIssuers) {
        if (lane == 0 && f.issued_mma) {
            tc_commit(&sh.fin[warp]);
            (void)mbar_wait(&sh.fin[warp], 0, nullptr);
        }
        __syncwarp();
    }
    tc_fence_before();
    f.bar();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(f.tmem, kTmemCols);
}

template <int G, int D>
cudaError_t launch_t(const StepParams& p, int grid, size_t smem, cudaStream_t stream) {
    auto kfn = decode_flow_kernel<G, D>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3(kFlowThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, p);
}

}  // namespace

size_t flow_smem_bytes(const StepParams& p, int grid, int* nslots, int* slot_bytes, int max_smem) {
    const int G = p.nheads / p.Hkv;
    if (p.Lqkv.precision != 8) return 0;
    if (!((G == 8 && p.d == 64) || (G == 1 && (p.d == 64 || p.d == 128)) || (G == 4 && (p.d == 32 || p.d == 64)) ||
          (G == 2 && p.d == 64) || (G == 1 && p.d == 32)))
        return 0;
    if (p.A > 16 || (size_t)p.Hkv * G * p.A * 2 + 64 > (size_t)kMiscFloats) return 0;
    if (p.H % 4 != 0 || (p.H + grid - 1) / grid > kMaxRows || grid > kFC) return 0;
    const QLayout* Ls[5] = {&p.Lqkv, &p.Lo, &p.Lgu, &p.Ldn, &p.Llm};
    for (int i = 0; i < 4; ++i) {
        if (max_segments(*Ls[i], grid, false) > kMaxSegs) return 0;
        if (max_tile_segments(*Ls[i], grid) > kMaxTileSegs) return 0;
    }
    if (max_segments(p.Llm, grid, true) > kMaxSegs) return 0;
    const int att_tile = 2 * kPageTokens * p.d * 4;
    const int sbytes = std::max(kTcUnitBytes, att_tile);
    int kmax = 0;
    for (const QLayout* L : Ls) kmax = std::max(kmax, L->slabs * L->slab_k);
    size_t tabs = 0;
    for (int i = 0; i < 4; ++i) tabs += (size_t)seg_table_bytes(*Ls[i]);
    const size_t att = (size_t)std::max(G * p.d + 2 * p.d + 2 * G * kPageTokens, p.Hkv * G * p.A) * 4;
    const size_t fixed = kBarRegion + kMiscFloats * 4 + (size_t)kmax * 8 + att + (size_t)kmax * 4 +
                         (size_t)kMaxRows * kMaxTileSegs * 4 + kMaxRows * 4 + tabs;
    if ((size_t)max_smem <= fixed + 2 * (size_t)sbytes) return 0;
    int ns = (int)((max_smem - fixed) / sbytes);
    ns = std::min(ns, kMaxSlots);
    ns = std::min(ns, 10);
    *nslots = ns;
    *slot_bytes = sbytes;
    return fixed + (size_t)ns * sbytes;
}

cudaError_t launch_decode_flow(const StepParams& p, int grid, size_t smem, cudaStream_t stream) {
    const int G = p.nheads / p.Hkv;
#define TB_FLOW_CASE(g, dd) \
    if (G == g && p.d == dd) return launch_t<g, dd>(p, grid, smem, stream);
    TB_FLOW_CASE(8, 64)
    TB_FLOW_CASE(1, 128)
    TB_FLOW_CASE(1, 64)
    TB_FLOW_CASE(4, 32)
    TB_FLOW_CASE(4, 64)
    TB_FLOW_CASE(2, 64)
    TB_FLOW_CASE(1, 32)
#undef TB_FLOW_CASE
    return cudaErrorNotSupported;
}

}  // namespace tb
