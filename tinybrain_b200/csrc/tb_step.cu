// tb_step.cu -- persistent decode step for batch 1 (sm_100a).
//
// One cooperative launch per token runs ModelRunner.step
// (Sources/TinyBrainRuntime/ModelRunner.swift:168-208) end to end: for every
// layer QKV -> attention -> o_proj -> gate/up -> down (applyLayer,
// ModelRunner.swift:392-459), then the final norm, LM head and greedy argmax.
//
// Why one kernel: a batch-1 decode step streams ~1 GB of weights through ~110
// dependent matrix products of 4-65 MB each; launched one by one, each product
// pays launch, ramp-up and drain latencies longer than its own HBM time.  Here
// one CTA per SM runs the whole step:
//
//  * a producer warp walks the CTA's static share of every phase (16 KB weight
//    units, INT4 group scales with them, and the KV-cache pages of its
//    attention split) and streams them with 1-D bulk async copies into a
//    shared-memory ring.  Weights and cached K/V do not depend on this step's
//    activations, so the stream never waits on the data dependencies between
//    phases -- only on free ring slots;
//  * eight consumer warps run the phases in order.  A phase starts after a
//    grid-wide barrier (an atomic counter in global memory, bounded spin),
//    builds its activation vector in shared memory (residual add + RMSNorm,
//    RoPE, SiLU*up, split-K / attention-split combine -- Tensor.swift:1538-1558,
//    ModelRunner.swift:470-579), multiplies it against the units in the ring,
//    and writes per-segment partial sums that the next phase reduces in a
//    fixed order (deterministic, no atomics on data);
//  * INT8 products run on the tensor cores (tb_tc.cuh): one thread issues
//    tcgen05.mma kind::i8 per unit (128 rows x 128 k) against the exact 4-digit
//    split of the activations, accumulating each segment (a run of units of one
//    128-row tile) in its own tensor-memory block; tcgen05.commit releases the
//    ring slot when the tensor core has read it and signals the segment's
//    barrier, and four epilogue warps (one tile row per thread) read the
//    accumulators back, combine the digits and apply scale and bias.  INT4
//    products run on the CUDA cores (tb_unit.cuh, 32-row units);
//  * the LM-head phase reduces whole row blocks per CTA, writes logits and
//    folds a packed (value, index) argmax into the sequence state with one
//    atomicMax per warp (Sampler.swift:126-138); CTA 0 then advances the step.
//
// All waits are bounded (2 s of %globaltimer); a timeout records an error code
// and makes the CTA leave the step early (after its tensor-core work drained and
// its tensor memory was freed) without hanging the device.
#include "tb_common.cuh"
#include "tb_kernels.h"
#include "tb_tc.cuh"
#include "tb_unit.cuh"
#include "tb_persist.cuh"

#include <algorithm>
#include <cstdlib>

namespace tb {

namespace {

using namespace persist;


struct Shared {
    uint64_t* full;
    uint64_t* empty;
    uint64_t* seg;          // [kMaxSegs] INT8 segment accumulators complete
    uint64_t* fin;          // [kIssuers] INT8: all tensor-core work of an issuer complete
    int* valid;             // [kMaxSlots] attention tile present (page not evicted)
    volatile int* abort;    // set when a wait timed out
    volatile int* go;       // thread 0's per-phase decision
    uint32_t* tmem;         // tensor-memory base address
    float* misc;            // [kMiscFloats]
    uint8_t* ring;
    float* xs;              // INT4: fp32 lane-interleaved activations; INT8: digit operand (bytes)
    float* att;             // attention scratch
    float* hs;              // staging: residual + norm weights [2][H], combined activations
    uint8_t* seglist[4];    // per row block: units where CTA segments start, ascending [rb][kMaxTileSegs]
    uint8_t* segcnt[4];     // per row block: number of segments
};

// ------------------------------------------------------------------ consumer --
struct Consumer {
    const StepParams& p;
    Shared sh;  // by value: the pointers stay in registers, not in local memory
    Cursor rc;  // next ring slot to consume
    int ctid, warp, lane, c, C;
    int nph = 0;                     // phases per step (trace stride)
    int cur_phase = 0;
    int xexp = 0;                    // INT8: digit exponent of the current activation vector
    uint32_t tmem = 0;               // INT8: tensor-memory base
    uint32_t segpar = 0;             // INT8 epilogue: next parity of each segment barrier
    bool issued_mma = false;         // INT8 issuer: tensor-core work outstanding
    unsigned long long waited = 0;   // thread 0: cycles waiting for ring slots in this phase
    unsigned long long dotted = 0;   // thread 0: cycles in unit products in this phase

    // Diagnostics (p.trace != null): per CTA and phase, %globaltimer at the
    // start (0), end (1), end of the prologue (2); cycles waiting for tiles (3)
    // and in unit products (4); the prologue's loads landed (5); SM cycles (6)
    // and ns (7) of the unit loop of a GEMV phase.
    __device__ void trace(int phase, int which) {
        if (!p.trace || ctid != 0) return;
        unsigned long long* t = p.trace + ((size_t)c * nph + phase) * 8;
        t[which] = global_timer_ns();
        if (which == 0) {
            waited = dotted = 0;
            cur_phase = phase;
        } else if (which == 1) {
            t[3] = waited;
            t[4] = dotted;
        }
    }
    __device__ __forceinline__ void mark(int which) {
        if (p.trace && ctid == 0) p.trace[((size_t)c * nph + cur_phase) * 8 + which] = global_timer_ns();
    }

    __device__ Consumer(const StepParams& p_, const Shared& sh_) : p(p_), sh(sh_) {
        ctid = threadIdx.x;
        warp = ctid >> 5;
        lane = ctid & 31;
        c = blockIdx.x;
        C = gridDim.x;
    }

    __device__ void bar() { named_bar_sync(1, kConsumers); }

    // Grid barrier: wait until every CTA finished phase (phase - 1).  Arrival
    // is one release-add on a counter, the wait an acquire poll by thread 0.
    // The go/stop decision is published through sh.go before the CTA barrier,
    // so every consumer warp takes the same branch.
    __device__ bool phase_begin(int phase) {
        if (ctid == 0) {
            if (phase > 0 && !*sh.abort) {
                const unsigned int target = (unsigned int)C * (unsigned int)phase;
                if (ld_acquire(p.bar) < target) {
                    const uint64_t t0 = global_timer_ns();
                    while (ld_acquire(p.bar) < target) {
                        if (global_timer_ns() - t0 > kWaitLimitNs) {
                            record_error(p.err, kDevWaitTimeout);
                            *sh.abort = 1;
                            break;
                        }
                    }
                }
            }
            *sh.go = *sh.abort ? 0 : 1;
            if (phase < nph) trace(phase, 0);
        }
        bar();
        return *sh.go != 0;
    }
    __device__ void phase_end(int phase) {
        bar();
        if (ctid == 0) {
            trace(phase, 1);
            red_release_add(p.bar, 1u);  // release: orders the CTA's writes (bar.sync above) before the arrival
        }
    }

    __device__ const uint8_t* wait_slot(int& st) {
        st = rc.st;
        if (*sh.abort) return nullptr;
        const bool tr = p.trace && ctid == 0;
        const long long w0 = tr ? clock64() : 0;
        const bool okw = mbar_wait(&sh.full[st], rc.ph, p.err);
        if (tr) waited += clock64() - w0;
        if (!okw) {
            *sh.abort = 1;
            return nullptr;
        }
        return sh.ring + (size_t)st * p.slot_bytes;
    }
    // Every consumer thread calls this once per slot (a CTA barrier inside).
    __device__ void release_slot(int st, bool have) {
        bar();
        if (ctid == 0 && have) mbar_arrive(&sh.empty[st]);
        rc.next(p.nslots);
    }

    // Sums of the split-K partials of NG groups of 4 consecutive GPU rows (same
    // row block).  A partial is stored (scaled; the segment starting at unit 0
    // carries the bias) at the unit where its CTA's segment of the row block
    // starts; segments are summed in unit order.  The first NL partials of
    // every group are loaded before the first add (one L2 round trip for all
    // groups); further segments, if any, follow group by group.
    template <int NG, int NL>
    __device__ void reduce4(const QLayout& L, int which, const float* part, const int (&n0)[NG],
                            const bool (&use)[NG], float4 (&out)[NG]) {
        const int ru = unit_rows(L.precision);
        float4 v[NG][NL];
        int cnt[NG];
        const uint8_t* lst[NG];
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const int rb = n0[j] / ru;
            cnt[j] = use[j] ? sh.segcnt[which][rb] : 0;
            lst[j] = sh.seglist[which] + rb * kMaxTileSegs;
#pragma unroll
            for (int g = 0; g < NL; ++g)
                v[j][g] = g < cnt[j] ? __ldcg(reinterpret_cast<const float4*>(part + (size_t)lst[j][g] * L.Np + n0[j]))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            float4 a = v[j][0];
#pragma unroll
            for (int g = 1; g < NL; ++g)
                if (g < cnt[j]) {
                    a.x += v[j][g].x;
                    a.y += v[j][g].y;
                    a.z += v[j][g].z;
                    a.w += v[j][g].w;
                }
            for (int g = NL; g < cnt[j]; ++g) {
                const float4 q = __ldcg(reinterpret_cast<const float4*>(part + (size_t)lst[j][g] * L.Np + n0[j]));
                a.x += q.x;
                a.y += q.y;
                a.z += q.z;
                a.w += q.w;
            }
            out[j] = a;
        }
    }
    // Scalar form for single rows.
    template <int NJ, int NL>
    __device__ void reduce_rows(const QLayout& L, int which, const float* part, const int (&n)[NJ],
                                float (&out)[NJ]) {
        const int ru = unit_rows(L.precision);
        float v[NJ][NL];
        int cnt[NJ];
        const uint8_t* lst[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const int rb = n[j] / ru;
            cnt[j] = sh.segcnt[which][rb];
            lst[j] = sh.seglist[which] + rb * kMaxTileSegs;
#pragma unroll
            for (int g = 0; g < NL; ++g) v[j][g] = g < cnt[j] ? __ldcg(part + (size_t)lst[j][g] * L.Np + n[j]) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            float a = v[j][0];
#pragma unroll
            for (int g = 1; g < NL; ++g)
                if (g < cnt[j]) a += v[j][g];
            for (int g = NL; g < cnt[j]; ++g) a += __ldcg(part + (size_t)lst[j][g] * L.Np + n[j]);
            out[j] = a;
        }
    }

    // Four consecutive activations (k % 4 == 0) into the phase's operand.
    template <int PREC>
    __device__ __forceinline__ void put_x_group(int k, float4 v) {
        static_assert(PREC == 8, "the persistent step runs INT8 weights");
        put_digits4(reinterpret_cast<uint8_t*>(sh.xs), 8, k, 0, v, __int_as_float((127 - xexp) << 23));
    }
    // Zero activations for k in [k0, Kp) (multiple-of-4 bounds).
    template <int PREC>
    __device__ void zero_tail(const QLayout& L, int k0) {
        for (int k = k0 + 4 * ctid; k < L.Kp; k += 4 * kConsumers) put_x_group<PREC>(k, make_float4(0.f, 0.f, 0.f, 0.f));
    }
    // Block-wide max of a per-thread value; sets xexp (all consumer threads).
    __device__ void set_digit_exponent(float mx, float factor) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) sh.misc[32 + warp] = mx;
        bar();
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < kStepConsumerWarps; ++w) t = fmaxf(t, sh.misc[32 + w]);
        xexp = digit_exponent(__fmul_rn(t, factor) * 1.0000002f);
    }
    // End of a prologue: make INT8 digits visible to the tensor core.
    template <int PREC>
    __device__ void prologue_done() {
        if (PREC == 8) fence_proxy_async_shared();
        bar();
    }

    // h = src + (reduced partials of the previous phase); optional store of
    // this CTA's slice of h; x = RMSNorm(h) * w (or h when norm == null).  The
    // source rows, norm weights and partials are loaded as float4 per group of
    // 4 rows; h is parked in shared memory (sh.hs) until the norm is known.
    template <int PREC>
    __device__ void residual_norm(const float* src, const QLayout* Lp, int which, const float* part, float* store,
                                  const float* norm, const QLayout& Lnext) {
        const int H = p.H;  // multiple of 32
        const int k0 = (int)((long long)c * H / C), k1 = (int)((long long)(c + 1) * H / C);
        float ss = 0.0f, mx = 0.0f;
        // thread t owns rows 4t..4t+3 of every 1024-row chunk
        for (int base = 0; base < H; base += 4 * 2 * kConsumers) {
            int n0[2];
            bool use[2];
            float4 add[2], sv[2], nw[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                n0[j] = base + 4 * (ctid + kConsumers * j);
                use[j] = n0[j] < H;
                if (!use[j]) n0[j] = 0;
                sv[j] = use[j] ? __ldcg(reinterpret_cast<const float4*>(src + n0[j])) : make_float4(0.f, 0.f, 0.f, 0.f);
                nw[j] = (use[j] && norm) ? __ldg(reinterpret_cast<const float4*>(norm + n0[j]))
                                         : make_float4(1.f, 1.f, 1.f, 1.f);
                add[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (Lp) reduce4<2, 10>(*Lp, which, part, n0, use, add);

#pragma unroll
            for (int j = 0; j < 2; ++j) {
                if (!use[j]) continue;
                float4 v = sv[j];
                if (Lp) {
                    v.x = __fadd_rn(v.x, add[j].x);
                    v.y = __fadd_rn(v.y, add[j].y);
                    v.z = __fadd_rn(v.z, add[j].z);
                    v.w = __fadd_rn(v.w, add[j].w);
                }
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
                if (PREC == 8) {
                    mx = fmaxf(mx, fabsf(__fmul_rn(v.x, nw[j].x)));
                    mx = fmaxf(mx, fabsf(__fmul_rn(v.y, nw[j].y)));
                    mx = fmaxf(mx, fabsf(__fmul_rn(v.z, nw[j].z)));
                    mx = fmaxf(mx, fabsf(__fmul_rn(v.w, nw[j].w)));
                }
                *reinterpret_cast<float4*>(sh.hs + n0[j]) = v;
                *reinterpret_cast<float4*>(sh.hs + H + n0[j]) = nw[j];
                if (store) {
                    const float e4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (n0[j] + e >= k0 && n0[j] + e < k1) store[n0[j] + e] = e4[e];
                }
            }
        }
        if (p.trace && ctid == 0) {
            volatile float sink = ss;
            (void)sink;
            mark(5);
        }
        float inv = 1.0f;
        if (norm) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) sh.misc[warp] = ss;
            bar();
            float t = 0.0f;
#pragma unroll
            for (int w = 0; w < kStepConsumerWarps; ++w) t += sh.misc[w];
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)H), p.eps)));
        }
        if (PREC == 8) set_digit_exponent(mx, inv);
        // each thread re-reads the rows it parked itself
        for (int n = 4 * ctid; n < H; n += 4 * kConsumers) {
            const float4 v = *reinterpret_cast<const float4*>(sh.hs + n);
            float4 x = v;
            if (norm) {
                const float4 w = *reinterpret_cast<const float4*>(sh.hs + H + n);
                x = make_float4(__fmul_rn(__fmul_rn(v.x, inv), w.x), __fmul_rn(__fmul_rn(v.y, inv), w.y),
                                __fmul_rn(__fmul_rn(v.z, inv), w.z), __fmul_rn(__fmul_rn(v.w, inv), w.w));
            }
            put_x_group<PREC>(n, x);
        }
        zero_tail<PREC>(Lnext, H);
        prologue_done<PREC>();
    }

    // ---------------------------------------------------------- GEMV phases --
    // INT8: lane 0 of warps 0 and 1 issue the tensor-core products of this
    // CTA's units (alternate units: one thread's issue latency would bound the
    // stream), each into its own accumulator block of the segment; warps 4-7
    // read each finished segment (one tile row per thread), add the blocks,
    // combine the digits, apply scale (and the bias on the segment that starts
    // at unit 0) and store one partial per row and segment at the unit where
    // the segment starts.
    __device__ void gemv_tc(const QLayout& L, float* part, const float* sc, const float* bias) {
        trace(cur_phase, 2);
        const int U = phase_units(L);
        const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
        const uint8_t* xd = reinterpret_cast<const uint8_t*>(sh.xs);
        if (warp < kIssuers) {
            if (lane == 0 && u1 > u0) {
                Cursor q = rc;
                int s = u0 % L.slabs, j = 0;
                bool fresh = true;  // next product of this issuer starts its block of the segment
                tc_fence_after();
                for (int u = u0; u < u1; ++u) {
                    if (*sh.abort) break;
                    if (((u - u0) & (kIssuers - 1)) == warp) {
                        const long long w0 = p.trace ? clock64() : 0;
                        if (!mbar_wait(&sh.full[q.st], q.ph, p.err)) {
                            *sh.abort = 1;
                            break;
                        }
                        const long long d0 = p.trace ? clock64() : 0;
                        if (p.trace) waited += d0 - w0;
                        tc_fence_after();
                        tc_unit_mma(tmem + 8 * (kIssuers * j + warp), smem_u32(sh.ring + (size_t)q.st * p.slot_bytes),
                                    smem_u32(xd + (size_t)s * (kTcUnitK / 16) * 128), 8, !fresh);
                        tc_commit(&sh.empty[q.st]);
                        issued_mma = true;
                        fresh = false;
                        if (p.trace) dotted += clock64() - d0;
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
                // block 1 holds data only if the segment has a unit at odd position
                const bool two = uend - u >= 2 || ((u - u0) & 1);
                const bool one = uend - u >= 2 || !((u - u0) & 1);
#pragma unroll
                for (int i = 0; i < 4; ++i) d[i] = (one ? d[i] : 0) + (two ? e[i] : 0);
                if (ok) {
                    float v = __fmul_rn(combine_digits(d, xexp), scv);
                    if (bias && sfirst == 0) v = __fadd_rn(v, bv);
                    part[(size_t)sfirst * L.Np + n] = v;
                }
                u = uend;
            }
            tc_fence_before();
        }
        rc.advance(u1 - u0, p.nslots);
    }

    template <int PREC>
    __device__ void gemv_units(const QLayout& L, float* part, const float* sc, const float* bias) {
        static_assert(PREC == 8, "the persistent step runs INT8 weights");
        gemv_tc(L, part, sc, bias);
    }

    // ---------------------------------------------------------------- attention
    template <int G, int D>
    __device__ void attention(int layer, int pos, int npages) {
        constexpr int DP = kConsumers / (G * kPageTokens);
        constexpr int CHK = D / DP;
        constexpr int PVT = G * (D / 4);
        static_assert(DP >= 1 && CHK >= 1 && CHK <= 64 && PVT <= kConsumers, "head geometry");
        const int A = p.A;
        if (c >= A * p.Hkv) return;  // uniform per CTA
        const int head = c / A, split = c % A;
        const int pps = (npages + A - 1) / A;
        const int pg0 = min(npages, split * pps), pg1 = min(npages, pg0 + pps);
        float* qs = sh.att;        // [G][D]
        float* knew = qs + G * D;  // [D]
        float* vnew = knew + D;    // [D]
        float* S = vnew + D;       // [2][G][16]
        const QLayout& L = p.Lqkv;
        const float2* rope = p.rope + (size_t)min(pos, p.rope_max_pos - 1) * (D / 2);
        // q (RoPE'd) for the G query heads of this KV head (ModelRunner.swift:499-515).
        for (int e = ctid; e < G * D / 2; e += kConsumers) {
            int n[2] = {head * G * D + 2 * e, head * G * D + 2 * e + 1};
            float v[2];
            reduce_rows<2, 10>(L, 0, p.part_qkv, n, v);
            const float2 cs = rope[(2 * e % D) / 2];
            qs[2 * e] = __fsub_rn(__fmul_rn(v[0], cs.x), __fmul_rn(v[1], cs.y));
            qs[2 * e + 1] = __fadd_rn(__fmul_rn(v[0], cs.y), __fmul_rn(v[1], cs.x));
        }
        const bool owner = pg0 < pg1 && pg1 == npages;
        if (owner) {  // this split holds the current position: append k, v (KVCache.swift:157-224)
            for (int e = ctid; e < D / 2; e += kConsumers) {
                const int nk = p.H + head * D + 2 * e;
                const int nv = p.H + p.kvd + head * D + 2 * e;
                int n[4] = {nk, nk + 1, nv, nv + 1};
                float v[4];
                reduce_rows<4, 10>(L, 0, p.part_qkv, n, v);
                const float2 cs = rope[e];
                const float r0 = __fsub_rn(__fmul_rn(v[0], cs.x), __fmul_rn(v[1], cs.y));
                const float r1 = __fadd_rn(__fmul_rn(v[0], cs.y), __fmul_rn(v[1], cs.x));
                knew[2 * e] = r0;
                knew[2 * e + 1] = r1;
                vnew[2 * e] = v[2];
                vnew[2 * e + 1] = v[3];
                const int page = p.ptab[pos / kPageTokens];
                if (page < 0) {
                    record_error(p.err, kDevBadPage);
                } else {
                    const size_t kb = ((((size_t)page * p.num_layers + layer) * 2 + 0) * p.Hkv + head) * kPageTokens +
                                      pos % kPageTokens;
                    const size_t vb = ((((size_t)page * p.num_layers + layer) * 2 + 1) * p.Hkv + head) * kPageTokens +
                                      pos % kPageTokens;
                    p.kv_pool[kb * D + 2 * e] = r0;
                    p.kv_pool[kb * D + 2 * e + 1] = r1;
                    p.kv_pool[vb * D + 2 * e] = v[2];
                    p.kv_pool[vb * D + 2 * e + 1] = v[3];
                }
            }
        }
        bar();
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
        const int pair = ctid / DP, dp = ctid % DP;
        const int gq = pair / kPageTokens, j = pair % kPageTokens;
        float qrot[CHK];
#pragma unroll
        for (int e = 0; e < CHK; ++e) qrot[e] = qs[gq * D + dp * CHK + (e + j) % CHK];
        const bool pv = ctid < PVT;
        const int gv = ctid / (D / 4), dv = (ctid % (D / 4)) * 4;
        float run_m = -INFINITY, run_l = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        const int cur_row = pos % kPageTokens;
        for (int i = 0; i < pg1 - pg0; ++i) {
            // Every warp walks every barrier even after a failed wait (no early exit).
            int st;
            const uint8_t* slot = wait_slot(st);
            const bool have = slot != nullptr;
            const float* Kt = have ? reinterpret_cast<const float*>(slot) : knew;
            const float* Vt = have ? Kt + kPageTokens * D : vnew;
            const bool ok = have && sh.valid[st] != 0;
            const bool last = have && owner && (pg0 + i == npages - 1);
            float* Sb = S + (i & 1) * G * kPageTokens;
            {
                float dot = 0.0f;
                const bool cur = last && j == cur_row;
                const float* kr = cur ? knew + dp * CHK : Kt + j * D + dp * CHK;
                if (ok || cur) {
#pragma unroll
                    for (int e = 0; e < CHK; ++e) dot = fmaf(qrot[e], kr[(e + j) % CHK], dot);
                }
#pragma unroll
                for (int o = DP / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
                const int tok = (pg0 + i) * kPageTokens + j;
                if (dp == 0) Sb[gq * kPageTokens + j] = (tok <= pos) ? __fmul_rn(dot, scale) : -INFINITY;
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
                    if (ok || cur) {
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
            release_slot(st, have);
        }
        if (pv && !*sh.abort) {
            float* part = p.attn_part + (((size_t)head * A + split) * G + gv) * (D + 4);
            *reinterpret_cast<float4*>(part + dv) = acc;
            if (dv == 0) {
                part[D] = run_m;
                part[D + 1] = run_l;
            }
        }
    }

    // Units of K touched by this CTA's units of a phase: a cyclic run of
    // `count` units starting at unit `first` (units are row-block major).
    __device__ void unit_run(const QLayout& L, int& first, int& count) {
        const int U = phase_units(L);
        const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
        first = u0 % L.slabs;
        count = min(u1 - u0, L.slabs);
    }
    // The e-th k of that run; -1 past the run, -2 past Kp.
    __device__ __forceinline__ int kth_in_run(const QLayout& L, int first, int count, int e) {
        const int i = e / L.slab_k;
        if (i >= count) return -1;
        int s = first + i;
        if (s >= L.slabs) s -= L.slabs;
        const int k = s * L.slab_k + (e - i * L.slab_k);
        return k < L.Kp ? k : -2;
    }

    // ctx[k] for the units this CTA's o_proj units need: combine the attention
    // splits in split order (softmax rescaling of (m, l, acc) partials).  Each
    // thread owns groups of 4 consecutive k; the acc loads of its first group
    // are issued together with the (m, l) loads, so the common case costs one
    // round trip.  INT8 stages the values (sh.hs) until their maximum is known.
    template <int PREC, int G, int D>
    __device__ void ctx_prologue() {
        constexpr int AMAX = 16;
        const QLayout& L = p.Lo;
        const int A = p.A;
        float2* ml = reinterpret_cast<float2*>(sh.misc + 64);  // [Hkv][A][G] (m, l)
        float* wts = sh.att;                                     // [Hkv][G][A]
        int first, count;
        unit_run(L, first, count);
        const int total = count * L.slab_k;  // multiple of 4
        auto group_loads = [&](int e, int& k, float4 (&a)[AMAX]) {
            k = e < total ? kth_in_run(L, first, count, e) : -1;
            const bool ok = k >= 0 && k < L.K;
            const int hq = ok ? k / D : 0, i = ok ? k % D : 0;
            const int hk = hq / G, g = hq % G;
#pragma unroll
            for (int sp = 0; sp < AMAX; ++sp)
                a[sp] = (ok && sp < A) ? __ldcg(reinterpret_cast<const float4*>(
                                             p.attn_part + (((size_t)hk * A + sp) * G + g) * (D + 4) + i))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        auto group_value = [&](int k, const float4 (&a)[AMAX]) -> float4 {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k >= 0 && k < L.K) {
                const int hq = k / D;
                const float* w = wts + ((hq / G) * G + hq % G) * A;
#pragma unroll
                for (int sp = 0; sp < AMAX; ++sp)
                    if (sp < A) {
                        v.x = fmaf(w[sp], a[sp].x, v.x);
                        v.y = fmaf(w[sp], a[sp].y, v.y);
                        v.z = fmaf(w[sp], a[sp].z, v.z);
                        v.w = fmaf(w[sp], a[sp].w, v.w);
                    }
            }
            return v;
        };
        int k0;
        float4 a0[AMAX];
        group_loads(4 * ctid, k0, a0);
        const int nml = p.Hkv * A * G;
        for (int e = ctid; e < nml; e += kConsumers) {
            const float* q = p.attn_part + (size_t)e * (D + 4) + D;
            ml[e] = make_float2(__ldcg(q), __ldcg(q + 1));
        }
        bar();
        // weights of the splits: 16 lanes per (kv head, query head) pair, one split each
        for (int base = 0; base < p.Hkv * G * 16; base += kConsumers) {
            const int e = (base + ctid) >> 4, sp = ctid & 15;
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
        mark(5);
        if (PREC == 8) {
            float mx = 0.0f;
            for (int e = 4 * ctid; e < total; e += 4 * kConsumers) {
                float4 v;
                if (e == 4 * ctid) {
                    v = group_value(k0, a0);
                } else {
                    int k;
                    float4 a[AMAX];
                    group_loads(e, k, a);
                    v = group_value(k, a);
                }
                *reinterpret_cast<float4*>(sh.hs + e) = v;
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
            set_digit_exponent(mx, 1.0f);
            for (int e = 4 * ctid; e < total; e += 4 * kConsumers) {
                const int k = kth_in_run(L, first, count, e);
                if (k >= 0) put_x_group<PREC>(k, *reinterpret_cast<const float4*>(sh.hs + e));
            }
        } else {
            if (k0 >= 0) put_x_group<PREC>(k0, group_value(k0, a0));
            for (int e = 4 * (ctid + kConsumers); e < total; e += 4 * kConsumers) {
                int k;
                float4 a[AMAX];
                group_loads(e, k, a);
                if (k >= 0) put_x_group<PREC>(k, group_value(k, a));
            }
        }
        prologue_done<PREC>();
    }

    // act[k] = silu(gate[k]) * up[k] for the units this CTA's down units need;
    // groups of 4 consecutive k, up to 2 groups per thread per batch of loads.
    template <int PREC>
    __device__ void act_prologue() {
        constexpr int NG = 2;
        const QLayout& L = p.Ldn;
        const QLayout& GL = p.Lgu;
        int first, count;
        unit_run(L, first, count);
        const int total = count * L.slab_k;  // multiple of 4
        const int half = GL.RB / 2;
        float mx = 0.0f;
        for (int e0 = 0; e0 < total; e0 += 4 * NG * kConsumers) {
            int n0[2 * NG], kk[NG];
            bool use[2 * NG];
            float4 v[2 * NG];
#pragma unroll
            for (int j = 0; j < NG; ++j) {
                const int e = e0 + 4 * (ctid + kConsumers * j);
                const int k = e < total ? kth_in_run(L, first, count, e) : -1;
                kk[j] = k;
                const bool ok = k >= 0 && k < L.K;  // K % 4 == 0
                const int grow = ok ? fused_row(GL, k, 0, 1) : 0;
                n0[2 * j] = grow;
                n0[2 * j + 1] = grow + half;
                use[2 * j] = use[2 * j + 1] = ok;
            }
            reduce4<2 * NG, 4>(GL, 2, p.part_gu, n0, use, v);
            if (e0 == 0 && p.trace && ctid == 0) {
                volatile float sink = v[0].x;
                (void)sink;
                mark(5);
            }
#pragma unroll
            for (int j = 0; j < NG; ++j) {
                if (kk[j] < 0) continue;
                const float4 g = v[2 * j], u = v[2 * j + 1];
                const bool ok = use[2 * j];
                const float4 a = ok ? make_float4(__fmul_rn(silu_ref(g.x), u.x), __fmul_rn(silu_ref(g.y), u.y),
                                                  __fmul_rn(silu_ref(g.z), u.z), __fmul_rn(silu_ref(g.w), u.w))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(sh.hs + e0 + 4 * (ctid + kConsumers * j)) = a;
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
            }
        }
        if (PREC == 8) {
            set_digit_exponent(mx, 1.0f);
            for (int e = 4 * ctid; e < total; e += 4 * kConsumers) {
                const int k = kth_in_run(L, first, count, e);
                if (k >= 0) put_x_group<PREC>(k, *reinterpret_cast<const float4*>(sh.hs + e));
            }
        }
        prologue_done<PREC>();
    }

    // LM head: whole row blocks per CTA, logits + argmax (Sampler.swift:126-138).
    __device__ void lm_head_tc(unsigned long long* best_out) {
        const QLayout& L = p.Llm;
        const int nt = L.Np / kTcTileRows;
        const int t0 = (int)((long long)c * nt / C), t1 = (int)((long long)(c + 1) * nt / C);
        const uint8_t* xd = reinterpret_cast<const uint8_t*>(sh.xs);
        if (warp < kIssuers) {
            if (lane == 0 && t1 > t0) {
                Cursor q = rc;
                tc_fence_after();
                int v = 0;  // unit position in this CTA's range
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
                                        smem_u32(xd + (size_t)s * (kTcUnitK / 16) * 128), 8, !fresh);
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
                const int v0 = j * L.slabs;  // position of the tile's first unit
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
    }

    template <int PREC>
    __device__ void lm_head(unsigned long long* best_out) {
        static_assert(PREC == 8, "the persistent step runs INT8 weights");
        lm_head_tc(best_out);
    }
};

template <int PREC, int G, int D>
__device__ void run_layers(Consumer& cs, const StepParams& p, int pos, int npages) {
    int phase = 0;
    for (int l = 0; l < p.num_layers; ++l) {
        const StepLayer& ly = p.layers[l];
        // ---- QKV: h_in = (embedding | h_mid(l-1) + down(l-1)); x = RMSNorm(h_in) ----
        if (!cs.phase_begin(phase++)) return;
        if (l == 0) {
            int tok = p.seq->token;
            if (tok < 0 || tok >= p.V) {
                if (threadIdx.x == 0) record_error(p.err, kDevBadToken);
                tok = 0;
            }
            cs.residual_norm<PREC>(p.emb + (size_t)tok * p.H, nullptr, 3, nullptr, p.hX, ly.in_norm, p.Lqkv);
        } else {
            cs.residual_norm<PREC>(p.hY, &p.Ldn, 3, p.part_dn, p.hX, ly.in_norm, p.Lqkv);
        }
        cs.gemv_units<PREC>(p.Lqkv, p.part_qkv, ly.qkv_s, ly.qkv_b);
        cs.phase_end(phase - 1);
        // ---- attention over the paged cache (+ RoPE, KV append) ----
        if (!cs.phase_begin(phase++)) return;
        cs.attention<G, D>(l, pos, npages);
        cs.phase_end(phase - 1);
        // ---- o_proj ----
        if (!cs.phase_begin(phase++)) return;
        cs.ctx_prologue<PREC, G, D>();
        cs.gemv_units<PREC>(p.Lo, p.part_o, ly.o_s, ly.o_b);
        cs.phase_end(phase - 1);
        // ---- gate/up: h_mid = h_in + o; x = RMSNorm(h_mid) ----
        if (!cs.phase_begin(phase++)) return;
        cs.residual_norm<PREC>(p.hX, &p.Lo, 1, p.part_o, p.hY, ly.post_norm, p.Lgu);
        cs.gemv_units<PREC>(p.Lgu, p.part_gu, ly.gu_s, ly.gu_b);
        cs.phase_end(phase - 1);
        // ---- down ----
        if (!cs.phase_begin(phase++)) return;
        cs.act_prologue<PREC>();
        cs.gemv_units<PREC>(p.Ldn, p.part_dn, ly.dn_s, ly.dn_b);
        cs.phase_end(phase - 1);
    }
    // ---- final norm + LM head + argmax ----
    if (!cs.phase_begin(phase++)) return;
    cs.residual_norm<PREC>(p.hY, &p.Ldn, 3, p.part_dn, nullptr, p.final_norm, p.Llm);
    cs.lm_head<PREC>(&p.seq->best);
    cs.phase_end(phase - 1);
    // ---- CTA 0 advances the step once every CTA folded its argmax ----
    if (cs.c == 0 && cs.phase_begin(phase)) {
        if (threadIdx.x == 0) {
            __threadfence();
            finish_sequence_step(*p.seq, 0, p.out_tokens, p.prompt, p.prompt_stride);
            *p.bar = 0u;  // every CTA has passed its last barrier read
        }
    }
}

template <int PREC, int G, int D>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    Shared sh;
    sh.full = reinterpret_cast<uint64_t*>(smem);
    sh.empty = sh.full + kMaxSlots;
    sh.seg = sh.empty + kMaxSlots;
    sh.fin = sh.seg + kMaxSegs;
    sh.valid = reinterpret_cast<int*>(sh.fin + kIssuers);
    sh.abort = reinterpret_cast<volatile int*>(sh.valid + kMaxSlots);
    sh.go = sh.abort + 1;
    sh.tmem = reinterpret_cast<uint32_t*>(const_cast<int*>(sh.go + 1));
    sh.misc = reinterpret_cast<float*>(smem + kBarRegion);
    sh.ring = smem + kBarRegion + kMiscFloats * 4;
    sh.xs = reinterpret_cast<float*>(sh.ring + (size_t)p.nslots * p.slot_bytes);
    const QLayout* Ls[5] = {&p.Lqkv, &p.Lo, &p.Lgu, &p.Ldn, &p.Llm};
    int kmax = 0;
    for (int i = 0; i < 5; ++i) kmax = max(kmax, Ls[i]->slabs * Ls[i]->slab_k);
    const int xbytes = PREC == 8 ? kmax * 8 : kmax * 4;
    sh.att = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sh.xs) + xbytes);
    sh.hs = sh.att + att_floats(G, D, p.Hkv, p.A);
    {
        uint8_t* t = reinterpret_cast<uint8_t*>(sh.hs + max(2 * p.H, p.Ldn.Kp));
        for (int i = 0; i < 4; ++i) {
            const int nrb = Ls[i]->Np / unit_rows(PREC);
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
        *sh.go = 1;
        fence_barrier_init();
    }
    if (PREC == 8 && warp == 0) tmem_alloc(sh.tmem, kTmemCols);
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

    if (warp == kStepConsumerWarps) {
        if (lane == 0) {
            Producer<Shared> pr(p, sh);
            auto range = [&](const QLayout& L, int& u0, int& u1) {
                const int U = phase_units(L);
                u0 = (int)((long long)c * U / C);
                u1 = (int)((long long)(c + 1) * U / C);
            };
            int u0, u1;
            for (int l = 0; l < p.num_layers && !pr.dead; ++l) {
                const StepLayer& ly = p.layers[l];
                range(p.Lqkv, u0, u1);
                pr.gemv<PREC>(p.Lqkv, ly.qkv_w, ly.qkv_s, u0, u1);
                if (head >= 0) pr.attention(l, head, apg0, apg1);
                range(p.Lo, u0, u1);
                pr.gemv<PREC>(p.Lo, ly.o_w, ly.o_s, u0, u1);
                range(p.Lgu, u0, u1);
                pr.gemv<PREC>(p.Lgu, ly.gu_w, ly.gu_s, u0, u1);
                range(p.Ldn, u0, u1);
                pr.gemv<PREC>(p.Ldn, ly.dn_w, ly.dn_s, u0, u1);
            }
            if (!pr.dead) {
                const int nrb = p.Llm.Np / unit_rows(PREC);
                const int r0 = (int)((long long)c * nrb / C), r1 = (int)((long long)(c + 1) * nrb / C);
                pr.gemv<PREC>(p.Llm, p.lm_w, p.lm_s, r0 * p.Llm.slabs, r1 * p.Llm.slabs);
            }
            if (pr.dead) pr.drain();
        }
        return;
    }

    Consumer cs(p, sh);
    cs.nph = 5 * p.num_layers + 1;
    for (int i = 0; i < 4; ++i) build_seglist(sh.seglist[i], sh.segcnt[i], *Ls[i], C, threadIdx.x, kConsumers);
    if (PREC == 8) {
        // digit rows 4..7 of the operand stay zero for the whole step
        uint32_t* x = reinterpret_cast<uint32_t*>(sh.xs);
        for (int i = threadIdx.x; i < xbytes / 4; i += kConsumers) x[i] = 0u;
        cs.tmem = *sh.tmem;
    }
    cs.bar();
    run_layers<PREC, G, D>(cs, p, pos, npages);

    // Teardown: wait (bounded) for this CTA's tensor-core work, free TMEM.
    if (PREC == 8) {
        if (warp < kIssuers) {
            if (lane == 0 && cs.issued_mma) {
                tc_commit(&sh.fin[warp]);
                (void)mbar_wait(&sh.fin[warp], 0, nullptr);
            }
            __syncwarp();
        }
        tc_fence_before();
        cs.bar();
        tc_fence_after();
        if (warp == 0) tmem_dealloc(cs.tmem, kTmemCols);
    }
}

template <int PREC, int G, int D>
cudaError_t launch_t(const StepParams& p, int grid, size_t smem, cudaStream_t stream) {
    auto kfn = decode_step_kernel<PREC, G, D>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3(kStepThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, p);
}

// INT8 weights only: INT4 projections stream through the per-op tensor-core GEMV.
bool supported(int prec, int G, int d) {
    if (prec != 8) return false;
    return (G == 8 && d == 64) || (G == 1 && (d == 64 || d == 128)) || (G == 4 && d == 32) ||
           (G == 4 && d == 64) || (G == 2 && d == 64) || (G == 1 && d == 32);
}

}  // namespace

size_t step_smem_bytes(const StepParams& p, int grid, int* nslots, int* slot_bytes, int max_smem) {
    const int G = p.nheads / p.Hkv;
    const int prec = p.Lqkv.precision;
    if (!supported(prec, G, p.d)) return 0;
    if (p.A > 16 || (size_t)p.Hkv * G * p.A * 2 + 64 > (size_t)kMiscFloats) return 0;  // (m, l) staging in misc
    const QLayout* Ls[5] = {&p.Lqkv, &p.Lo, &p.Lgu, &p.Ldn, &p.Llm};
    if (prec == 8) {
        for (int i = 0; i < 4; ++i)
            if (max_segments(*Ls[i], grid, false) > kMaxSegs) return 0;
        if (max_segments(p.Llm, grid, true) > kMaxSegs) return 0;
    }
    const int slot = kTcUnitBytes;
    const int att_tile = 2 * kPageTokens * p.d * 4;
    const int sbytes = std::max(slot, att_tile);
    int kmax = 0;
    for (const QLayout* L : Ls) kmax = std::max(kmax, L->slabs * L->slab_k);
    const size_t xbytes = (size_t)kmax * (prec == 8 ? 8 : 4);
    const size_t att = (size_t)std::max(G * p.d + 2 * p.d + 2 * G * kPageTokens, p.Hkv * G * p.A) * 4;
    size_t tabs = 0;
    for (int i = 0; i < 4; ++i) {
        tabs += (size_t)seg_table_bytes(*Ls[i]);
        if (max_tile_segments(*Ls[i], grid) > kMaxTileSegs) return 0;
    }
    // staging: [2][H] residual + norm weights; combined ctx / act values of a CTA's units
    const size_t stage = (size_t)std::max(2 * p.H, p.Ldn.Kp) * 4;
    const size_t fixed = kBarRegion + kMiscFloats * 4 + xbytes + att + stage + tabs;
    if ((size_t)max_smem <= fixed + 2 * (size_t)sbytes) return 0;
    int ns = (int)((max_smem - fixed) / sbytes);
    ns = std::min(ns, kMaxSlots);
    ns = std::min(ns, 10);
    if (const char* e = getenv("TB_STEP_SLOTS")) ns = std::max(2, std::min(ns, atoi(e)));
    *nslots = ns;
    *slot_bytes = sbytes;
    return fixed + (size_t)ns * sbytes;
}

cudaError_t launch_decode_step(const StepParams& p, int grid, size_t smem, cudaStream_t stream) {
    if (p.flow) return launch_decode_flow(p, grid, smem, stream);
    const int G = p.nheads / p.Hkv;
    const int prec = p.Lqkv.precision;
#define TB_STEP_CASE(pr, g, dd) \
    if (prec == pr && G == g && p.d == dd) return launch_t<pr, g, dd>(p, grid, smem, stream);
    TB_STEP_CASE(8, 8, 64)
    TB_STEP_CASE(8, 1, 128)
    TB_STEP_CASE(8, 1, 64)
    TB_STEP_CASE(8, 4, 32)
    TB_STEP_CASE(8, 4, 64)
    TB_STEP_CASE(8, 2, 64)
    TB_STEP_CASE(8, 1, 32)
#undef TB_STEP_CASE
    return cudaErrorNotSupported;
}

}  // namespace tb
