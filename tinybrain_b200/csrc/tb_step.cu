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
//  * a producer warp walks the CTA's static share of every phase (32-row x
//    512-byte weight units, INT4 group scales with them, and the KV-cache pages
//    of its attention split) and streams them with 1-D bulk async copies into a
//    shared-memory ring.  Weights and cached K/V do not depend on this step's
//    activations, so the stream never waits on the data dependencies between
//    phases -- only on free ring slots;
//  * eight consumer warps run the phases in order.  A phase starts after a
//    grid-wide barrier (an atomic counter in global memory, bounded spin),
//    builds its activation vector in shared memory (residual add + RMSNorm,
//    RoPE, SiLU*up, split-K / attention-split combine -- Tensor.swift:1538-1558,
//    ModelRunner.swift:470-579), multiplies it against the units already in the
//    ring, and writes per-segment partial sums that the next phase reduces in a
//    fixed order (deterministic, no atomics on data);
//  * the LM-head phase reduces whole row blocks per CTA, writes logits and
//    folds a packed (value, index) argmax into the sequence state with one
//    atomicMax per warp (Sampler.swift:126-138); CTA 0 then advances the step.
//
// All waits are bounded (2 s of %globaltimer); a timeout records an error code
// and makes the CTA leave the step early without hanging the device.
#include "tb_common.cuh"
#include "tb_kernels.h"
#include "tb_unit.cuh"

#include <algorithm>
#include <cstdlib>

namespace tb {

namespace {

constexpr int kMaxSlots = 24;
constexpr int kBarRegion = 1024;  // mbarriers + flags
constexpr int kMiscFloats = 1024;
constexpr int kConsumers = kStepConsumerWarps * 32;
constexpr int kRowBlocksCached = 16;  // per-warp scale/bias cache of a GEMV phase (row blocks)

struct Shared {
    uint64_t* full;
    uint64_t* empty;
    int* valid;             // [kMaxSlots] attention tile present (page not evicted)
    volatile int* abort;    // set when a wait timed out
    volatile int* go;       // thread 0's per-phase decision
    float* misc;            // [kMiscFloats]
    uint8_t* ring;
    float* xs;              // activation vector, lane-interleaved per slab
    float* att;             // attention scratch
    float* hs;              // [2][H] residual stream and norm weights of a prologue
    float* rows;            // [warp][kRowBlocksCached][8]: INT8 scales (4) and biases (4) of the warp's rows
    uint32_t* segmask[4];   // per 32-row block: bit s = a CTA segment starts at slab s (qkv, o, gate/up, down)
};

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// 4-byte asynchronous copy global -> shared (does not stall the issuing warp).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// The CTA whose static unit range [c*U/C, (c+1)*U/C) contains unit u.
__device__ __forceinline__ int owner_of(int u, int U, int C) { return (int)(((long long)u * C + C - 1) / U); }

__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

__device__ __forceinline__ int att_floats(int G, int d, int Hkv, int A) {
    return max(G * d + 2 * d + 2 * G * kPageTokens, Hkv * G * A);
}

// Ring position (slot, phase parity) advanced without divisions.
struct Cursor {
    int st = 0;
    uint32_t ph = 0;
    __device__ __forceinline__ void next(int n) {
        if (++st == n) {
            st = 0;
            ph ^= 1u;
        }
    }
};

// ------------------------------------------------------------------ producer --
struct Producer {
    const StepParams& p;
    Shared sh;  // by value: the pointers stay in registers, not in local memory
    int it = 0;        // copies issued
    Cursor cur;        // slot of copy `it`
    Cursor thr;        // slot of copy `it - nflight` (throttle)
    uint64_t pol;
    bool dead = false;

    __device__ Producer(const StepParams& p_, const Shared& sh_) : p(p_), sh(sh_) { pol = l2_policy_evict_first(); }

    __device__ bool spin(uint64_t* bar, uint32_t par) {
        if (mbar_try_wait(bar, par)) return true;
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(bar, par)) {
            __nanosleep(64);
            if (*sh.abort || global_timer_ns() - t0 > kWaitLimitNs) {
                if (!*sh.abort) record_error(p.err, kDevWaitTimeout);
                dead = true;
                *sh.abort = 1;
                return false;
            }
        }
        return true;
    }

    // Keep at most p.nflight copies outstanding: enough to keep HBM busy, few
    // enough not to inflate the latency of the consumers' activation loads.
    __device__ uint8_t* acquire(int& st) {
        if (it >= p.nflight) {
            if (!spin(&sh.full[thr.st], thr.ph)) return nullptr;
            thr.next(p.nslots);
        }
        st = cur.st;
        if (it >= p.nslots && !spin(&sh.empty[st], cur.ph ^ 1u)) return nullptr;
        return sh.ring + (size_t)st * p.slot_bytes;
    }
    __device__ __forceinline__ void issued() {
        ++it;
        cur.next(p.nslots);
    }

    // Units [u0, u1) of a GEMV phase (32-row block major, slab minor; a 64-row
    // block of the fused gate/up matrix is two 32-row units).
    __device__ void gemv(const QLayout& L, const uint8_t* w, const float* sc, int u0, int u1) {
        if (u1 <= u0) return;
        const int hshift = L.RB == 64 ? 1 : 0;
        int rb32 = u0 / L.slabs, s = u0 - rb32 * L.slabs;
        for (int u = u0; u < u1 && !dead; ++u) {
            const int sb = min(kSlabBytes, L.row_bytes - s * kSlabBytes);
            const int rbb = rb32 >> hshift, half = rb32 & hshift;
            const uint8_t* src =
                w + (size_t)rbb * L.RB * L.row_bytes + (size_t)s * L.RB * kSlabBytes + (size_t)half * 32 * sb;
            int st;
            uint8_t* dst = acquire(st);
            if (!dst) return;
            const uint32_t wb = 32u * sb, sbytes = (L.precision == 4) ? 4096u : 0u;
            mbar_arrive_expect_tx(&sh.full[st], wb + sbytes);
            bulk_g2s_stream(dst, src, wb, &sh.full[st], pol);
            if (L.precision == 4)
                bulk_g2s_stream(dst + 16384, sc + (((size_t)rbb * L.slabs + s) * (L.RB / 32) + half) * 1024, sbytes,
                                &sh.full[st], pol);
            issued();
            if (++s == L.slabs) {
                s = 0;
                ++rb32;
            }
        }
    }

    __device__ void attention(int layer, int head, int pg0, int pg1) {
        const int tile = kPageTokens * p.d;  // floats
        for (int pg = pg0; pg < pg1 && !dead; ++pg) {
            int st;
            uint8_t* dst = acquire(st);
            if (!dst) return;
            const int page = p.ptab[pg];
            if (page >= 0) {
                sh.valid[st] = 1;
                const size_t kb = ((((size_t)page * p.num_layers + layer) * 2 + 0) * p.Hkv + head) * (size_t)tile;
                const size_t vb = ((((size_t)page * p.num_layers + layer) * 2 + 1) * p.Hkv + head) * (size_t)tile;
                mbar_arrive_expect_tx(&sh.full[st], 2u * tile * 4u);
                bulk_g2s(dst, p.kv_pool + kb, tile * 4u, &sh.full[st]);
                bulk_g2s(dst + tile * 4, p.kv_pool + vb, tile * 4u, &sh.full[st]);
            } else {
                sh.valid[st] = 0;  // evicted page: rows read as zeros (KVCache.swift:239-253)
                mbar_arrive(&sh.full[st]);
            }
            issued();
        }
    }

    // After an abort: wait (bounded) until every copy this warp issued has landed.
    __device__ void drain() {
        const int first = it > p.nslots ? it - p.nslots : 0;
        const uint64_t t0 = global_timer_ns();
        for (int j = first; j < it; ++j) {
            const int st = j % p.nslots;
            while (!mbar_try_wait(&sh.full[st], (j / p.nslots) & 1))
                if (global_timer_ns() - t0 > kWaitLimitNs) return;
        }
    }
};

// ------------------------------------------------------------------ consumer --
struct Consumer {
    const StepParams& p;
    Shared sh;  // by value: the pointers stay in registers, not in local memory
    Cursor rc;  // next ring slot to consume
    int ctid, warp, lane, c, C;
    int nph = 0;                     // phases per step (trace stride)
    int cur_phase = 0;
    unsigned long long waited = 0;   // thread 0: cycles waiting for ring slots in this phase
    unsigned long long dotted = 0;   // thread 0: cycles in unit products in this phase

    // Diagnostics (p.trace != null): per CTA and phase, %globaltimer at the
    // start (0), end (1), end of the prologue (2); ns waiting for tiles (3) and
    // in unit products (4) (SM cycles); the prologue's loads landed (5); SM
    // cycles (6) and ns (7) of the unit loop of a GEMV phase.
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
    // is one release-add on a counter, the wait an acquire poll by thread 0
    // (measured cheaper on this part than per-CTA flags polled by a warp,
    // whose loads crowd the L2 slices holding the flags).  The go/stop
    // decision is published through sh.go before the CTA barrier, so every
    // consumer warp takes the same branch.
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

    // Issue asynchronous copies of the INT8 scales and the biases of this
    // warp's rows of every row block in the CTA's range of a GEMV phase; the
    // first flush of the phase waits for them.
    __device__ void prefetch_rows(const QLayout& L, const float* sc, const float* bias) {
        const int U = (L.Np / 32) * L.slabs;
        const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
        if (u1 <= u0) return;
        const int rb0 = u0 / L.slabs, nrb = min((u1 - 1) / L.slabs - rb0 + 1, kRowBlocksCached);
        float* rs = sh.rows + warp * kRowBlocksCached * 8;
        for (int e = lane; e < nrb * 8; e += 32) {
            const int i = e >> 3, q = e & 7;
            const int row = (rb0 + i) * 32 + warp * 4 + (q & 3);
            const float* src = q < 4 ? (L.precision == 8 ? sc : nullptr) : bias;
            if (src) cp_async4(rs + e, src + row);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
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
    __device__ void release_slot(int st) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.empty[st]);
        rc.next(p.nslots);
    }

    // Sums of the split-K partials of NJ GPU rows of a phase.  A partial is
    // stored (already scaled; the slab-0 segment carries the bias) at the slab
    // where its CTA's segment of the row block starts; segments are summed in
    // slab order.  All loads are issued before
    // the first add, so NJ rows cost one L2 round trip, not one per segment.
    template <int NJ, int SEGMAX = 4>
    __device__ void reduce_rows(const QLayout& L, const uint32_t* tab, const float* part, const int (&n)[NJ],
                                const bool (&use)[NJ], float (&out)[NJ]) {
        float v[NJ][SEGMAX];
        uint32_t m0[NJ], rest[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            uint32_t m = use[j] ? tab[n[j] >> 5] : 0u;
            m0[j] = m;
#pragma unroll
            for (int g = 0; g < SEGMAX; ++g) {
                const int sl = __ffs(m) - 1;  // -1: no segment left
                v[j][g] = sl >= 0 ? __ldcg(part + (size_t)sl * L.Np + n[j]) : 0.0f;
                m &= m - 1;
            }
            rest[j] = m;
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const int cnt = __popc(m0[j]);
            float t = 0.0f;
#pragma unroll
            for (int g = 0; g < SEGMAX; ++g)
                if (g < cnt) t += v[j][g];
            for (uint32_t m = rest[j]; m; m &= m - 1) t += __ldcg(part + (size_t)(__ffs(m) - 1) * L.Np + n[j]);
            out[j] = t;
        }
    }

    // Vector form of reduce_rows: NG groups of 4 consecutive GPU rows (same
    // 32-row block), one float4 load per segment.
    template <int NG, int SEGMAX = 4>
    __device__ void reduce4(const QLayout& L, const uint32_t* tab, const float* part, const int (&n0)[NG],
                            const bool (&use)[NG], float4 (&out)[NG]) {
        float4 v[NG][SEGMAX];
        uint32_t m0[NG], rest[NG];
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            uint32_t m = use[j] ? tab[n0[j] >> 5] : 0u;
            m0[j] = m;
#pragma unroll
            for (int g = 0; g < SEGMAX; ++g) {
                const int sl = __ffs(m) - 1;
                v[j][g] = sl >= 0 ? __ldcg(reinterpret_cast<const float4*>(part + (size_t)sl * L.Np + n0[j]))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                m &= m - 1;
            }
            rest[j] = m;
        }
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const int cnt = __popc(m0[j]);
            float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int g = 0; g < SEGMAX; ++g)
                if (g < cnt) {
                    t.x += v[j][g].x;
                    t.y += v[j][g].y;
                    t.z += v[j][g].z;
                    t.w += v[j][g].w;
                }
            for (uint32_t m = rest[j]; m; m &= m - 1) {
                const float4 q = __ldcg(reinterpret_cast<const float4*>(part + (size_t)(__ffs(m) - 1) * L.Np + n0[j]));
                t.x += q.x;
                t.y += q.y;
                t.z += q.z;
                t.w += q.w;
            }
            out[j] = t;
        }
    }

    template <int PREC>
    __device__ void put_x(const QLayout& L, int k, float v) {
        constexpr int CH = PREC == 8 ? 16 : 32;
        constexpr int SK = PREC == 8 ? kSlabBytes : 2 * kSlabBytes;  // == L.slab_k
        if (PREC == 4) v *= int4_pos_scale(k & 7);
        const int s = k / SK;
        sh.xs[s * SK + xperm<CH>(k - s * SK)] = v;
    }

    // h = src + (reduced partials of the previous phase); optional store of
    // this CTA's slice of h; x = RMSNorm(h) * w (or h when norm == null).  The
    // source rows, norm weights and partials are loaded as float4 in one batch
    // per chunk; h is parked in shared memory (sh.hs) until the norm is known.
    template <int PREC>
    __device__ void residual_norm(const float* src, const QLayout* Lp, const uint32_t* tab, const float* part,
                                  float* store, const float* norm, const QLayout& Lnext) {
        const int H = p.H;  // multiple of 32
        const int k0 = (int)((long long)c * H / C), k1 = (int)((long long)(c + 1) * H / C);
        float ss = 0.0f;
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
            if (Lp) reduce4<2>(*Lp, tab, part, n0, use, add);
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
        // each thread re-reads the rows it parked itself: no barrier needed
        for (int n = 4 * ctid; n < H; n += 4 * kConsumers) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float v = sh.hs[n + e];
                put_x<PREC>(Lnext, n + e, norm ? __fmul_rn(__fmul_rn(v, inv), sh.hs[H + n + e]) : v);
            }
        }
        for (int k = H + ctid; k < Lnext.Kp; k += kConsumers) put_x<PREC>(Lnext, k, 0.0f);
        bar();
    }

    // Multiply this CTA's units of a GEMV phase; write one partial per row and
    // segment, at the slab where the segment starts.
    template <int PREC>
    __device__ void gemv_units(const QLayout& L, float* part, const float* sc, const float* bias) {
        trace(cur_phase, 2);
        prefetch_rows(L, sc, bias);
        const int U = (L.Np / 32) * L.slabs;
        const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
        float2 acc[4][1];
        int cur = -1, s_first = 0;
        // The per-row INT8 scale is applied to each partial; the segment that
        // starts at slab 0 also carries the bias, so readers only add.  Scales
        // and biases come from the warp's prefetched row cache.
        const int rb0 = u0 / L.slabs;
        const float* rs = sh.rows + warp * kRowBlocksCached * 8;
        bool cached = false;
        auto flush = [&](int rb32, int slab) {
            const int i = rb32 - rb0;
            if (!cached) {
                cp_async_wait_all();
                __syncwarp();
                cached = true;
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                float v = acc[r][0].x + acc[r][0].y;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const int n = rb32 * 32 + warp * 4 + r;
                if (lane == r) {
                    const bool hit = i < kRowBlocksCached;
                    if (L.precision == 8) v = __fmul_rn(v, hit ? rs[i * 8 + r] : __ldg(sc + n));
                    if (bias && slab == 0) v = __fadd_rn(v, hit ? rs[i * 8 + 4 + r] : __ldg(bias + n));
                    part[(size_t)slab * L.Np + n] = v;
                }
                acc[r][0] = make_float2(0.f, 0.f);
            }
        };
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[r][0] = make_float2(0.f, 0.f);
        const long long loop_c0 = (p.trace && ctid == 0) ? clock64() : 0;
        const uint64_t loop_t0 = (p.trace && ctid == 0) ? global_timer_ns() : 0;
        int rb32 = u0 / L.slabs, s = u0 - (u0 / L.slabs) * L.slabs;
        for (int u = u0; u < u1; ++u, (++s == L.slabs ? (s = 0, ++rb32) : 0)) {
            if (rb32 != cur) {
                if (cur >= 0) flush(cur, s_first);
                cur = rb32;
                s_first = s;
            }
            int st;
            const uint8_t* slot = wait_slot(st);
            if (!slot) return;
            const int sb = min(kSlabBytes, L.row_bytes - s * kSlabBytes);
            const float* ssl = (PREC == 4) ? reinterpret_cast<const float*>(slot + 16384) : nullptr;
            const long long td = (p.trace && ctid == 0) ? clock64() : 0;
            unit_dot<PREC, 4, 1>(slot, sb, warp * 4, ssl, sh.xs + s * L.slab_k, 0, lane, acc);
            if (p.trace && ctid == 0) {
                volatile float sink = acc[0][0].x + acc[1][0].x + acc[2][0].x + acc[3][0].x;
                (void)sink;
                dotted += clock64() - td;
            }
            release_slot(st);
        }
        if (p.trace && ctid == 0) {
            unsigned long long* t = p.trace + ((size_t)c * nph + cur_phase) * 8;
            t[6] = clock64() - loop_c0;
            t[7] = global_timer_ns() - loop_t0;
        }
        if (cur >= 0) flush(cur, s_first);
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
        const StepLayer& ly = p.layers[layer];
        const float2* rope = p.rope + (size_t)min(pos, p.rope_max_pos - 1) * (D / 2);
        // q (RoPE'd) for the G query heads of this KV head (ModelRunner.swift:499-515).
        for (int e = ctid; e < G * D / 2; e += kConsumers) {
            int n[2] = {head * G * D + 2 * e, head * G * D + 2 * e + 1};
            bool use[2] = {true, true};
            float v[2];
            reduce_rows<2>(L, sh.segmask[0], p.part_qkv, n, use, v);
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
                bool use[4] = {true, true, true, true};
                float v[4];
                reduce_rows<4>(L, sh.segmask[0], p.part_qkv, n, use, v);
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
            if (have) {
                release_slot(st);
            } else {
                rc.next(p.nslots);
            }
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

    // Slabs of K touched by this CTA's units of a phase (bit per slab).
    __device__ uint32_t slab_set(const QLayout& L) {
        const int U = (L.Np / 32) * L.slabs;
        const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
        if (u1 - u0 >= L.slabs) return L.slabs >= 32 ? 0xFFFFFFFFu : ((1u << L.slabs) - 1u);
        uint32_t m = 0;
        for (int u = u0; u < u1; ++u) m |= 1u << (u % L.slabs);
        return m;
    }
    // The e-th k of the slabs in `set` (slab-major); -1 past the set, -2 past Kp.
    __device__ __forceinline__ int kth_in_set(const QLayout& L, uint32_t set, int e) {
        const int si = e / L.slab_k;
        uint32_t m = set;
        for (int i = 0; i < si && m; ++i) m &= m - 1;
        if (!m) return -1;
        const int k = (__ffs(m) - 1) * L.slab_k + e % L.slab_k;
        return k < L.Kp ? k : -2;
    }

    // ctx[k] for the slabs this CTA's o_proj units need: combine the attention
    // splits in split order (softmax rescaling of (m, l, acc) partials).  Each
    // thread owns groups of 4 consecutive k; the acc loads of its first group
    // are issued together with the (m, l) loads, so the common case costs one
    // round trip.
    template <int PREC, int G, int D>
    __device__ void ctx_prologue() {
        constexpr int AMAX = 16;
        const QLayout& L = p.Lo;
        const int A = p.A;
        float2* ml = reinterpret_cast<float2*>(sh.misc);  // [Hkv][A][G] (m, l)
        float* wts = sh.att;                              // [Hkv][G][A]
        const uint32_t set = slab_set(L);
        const int total = __popc(set) * L.slab_k;  // multiple of 4
        auto group_loads = [&](int e, int& k, float4 (&a)[AMAX]) {
            k = e < total ? kth_in_set(L, set, e) : -1;
            const bool ok = k >= 0 && k < L.K;
            const int hq = ok ? k / D : 0, i = ok ? k % D : 0;
            const int hk = hq / G, g = hq % G;
#pragma unroll
            for (int sp = 0; sp < AMAX; ++sp)
                a[sp] = (ok && sp < A) ? __ldcg(reinterpret_cast<const float4*>(
                                             p.attn_part + (((size_t)hk * A + sp) * G + g) * (D + 4) + i))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        auto group_put = [&](int k, const float4 (&a)[AMAX]) {
            if (k < 0) return;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < L.K) {
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
            put_x<PREC>(L, k + 0, v.x);
            put_x<PREC>(L, k + 1, v.y);
            put_x<PREC>(L, k + 2, v.z);
            put_x<PREC>(L, k + 3, v.w);
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
        for (int e = ctid; e < p.Hkv * G; e += kConsumers) {
            const int hk = e / G, g = e % G;
            float M = -INFINITY;
            for (int sp = 0; sp < A; ++sp) M = fmaxf(M, ml[(hk * A + sp) * G + g].x);
            float den = 0.0f;
            for (int sp = 0; sp < A; ++sp) {
                const float2 t = ml[(hk * A + sp) * G + g];
                const float w = (t.x == -INFINITY || M == -INFINITY) ? 0.0f : expf(t.x - M);
                wts[e * A + sp] = w;
                den = fmaf(w, t.y, den);
            }
            const float inv = den > 0.0f ? 1.0f / den : 0.0f;
            for (int sp = 0; sp < A; ++sp) wts[e * A + sp] *= inv;
        }
        bar();
        mark(5);
        group_put(k0, a0);
        for (int e = 4 * (ctid + kConsumers); e < total; e += 4 * kConsumers) {
            int k;
            float4 a[AMAX];
            group_loads(e, k, a);
            group_put(k, a);
        }
        bar();
    }

    // act[k] = silu(gate[k]) * up[k] for the slabs this CTA's down units need;
    // groups of 4 consecutive k, up to 4 groups per thread per batch of loads.
    template <int PREC>
    __device__ void act_prologue(const StepLayer& ly) {
        constexpr int NG = 4;
        const QLayout& L = p.Ldn;
        const QLayout& GL = p.Lgu;
        const uint32_t set = slab_set(L);
        const int total = __popc(set) * L.slab_k;  // multiple of 4
        for (int e0 = 0; e0 < total; e0 += 4 * NG * kConsumers) {
            int n0[2 * NG], kk[NG];
            bool use[2 * NG];
            float4 v[2 * NG];
#pragma unroll
            for (int j = 0; j < NG; ++j) {
                const int e = e0 + 4 * (ctid + kConsumers * j);
                const int k = e < total ? kth_in_set(L, set, e) : -1;
                kk[j] = k;
                const bool ok = k >= 0 && k < L.K;  // K % 4 == 0
                const int grow = ok ? (k / 32) * 64 + (k % 32) : 0;
                n0[2 * j] = grow;
                n0[2 * j + 1] = grow + 32;
                use[2 * j] = use[2 * j + 1] = ok;
            }
            reduce4<2 * NG, 2>(GL, sh.segmask[2], p.part_gu, n0, use, v);
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
                put_x<PREC>(L, kk[j] + 0, ok ? __fmul_rn(silu_ref(g.x), u.x) : 0.0f);
                put_x<PREC>(L, kk[j] + 1, ok ? __fmul_rn(silu_ref(g.y), u.y) : 0.0f);
                put_x<PREC>(L, kk[j] + 2, ok ? __fmul_rn(silu_ref(g.z), u.z) : 0.0f);
                put_x<PREC>(L, kk[j] + 3, ok ? __fmul_rn(silu_ref(g.w), u.w) : 0.0f);
            }
        }
        bar();
    }

    // LM head: whole row blocks per CTA, logits + argmax (Sampler.swift:126-138).
    template <int PREC>
    __device__ void lm_head(unsigned long long* best_out) {
        const QLayout& L = p.Llm;
        const int nrb = L.Np / 32;
        const int r0 = (int)((long long)c * nrb / C), r1 = (int)((long long)(c + 1) * nrb / C);
        unsigned long long best = 0ull;
        for (int rb = r0; rb < r1; ++rb) {
            float2 acc[4][1];
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][0] = make_float2(0.f, 0.f);
            for (int s = 0; s < L.slabs; ++s) {
                int st;
                const uint8_t* slot = wait_slot(st);
                if (!slot) return;
                const int sb = min(kSlabBytes, L.row_bytes - s * kSlabBytes);
                const float* ssl = (PREC == 4) ? reinterpret_cast<const float*>(slot + 16384) : nullptr;
                unit_dot<PREC, 4, 1>(slot, sb, warp * 4, ssl, sh.xs + s * L.slab_k, 0, lane, acc);
                release_slot(st);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                float v = acc[r][0].x + acc[r][0].y;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const int n = rb * 32 + warp * 4 + r;
                if (lane == r && n < L.N) {
                    float lv = (PREC == 8) ? __fmul_rn(v, p.lm_s[n]) : v;
                    if (p.lm_b) lv = __fadd_rn(lv, p.lm_b[n]);
                    if (p.logits) p.logits[n] = lv;
                    const unsigned long long key = argmax_key(lv, n);
                    best = key > best ? key : best;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
            best = t > best ? t : best;
        }
        if (lane == 0 && best != 0ull) atomicMax(best_out, best);
    }
};

template <int PREC, int G, int D>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    Shared sh;
    sh.full = reinterpret_cast<uint64_t*>(smem);
    sh.empty = sh.full + kMaxSlots;
    sh.valid = reinterpret_cast<int*>(sh.empty + kMaxSlots);
    sh.abort = reinterpret_cast<volatile int*>(sh.valid + kMaxSlots);
    sh.go = sh.abort + 1;
    sh.misc = reinterpret_cast<float*>(smem + kBarRegion);
    sh.ring = smem + kBarRegion + kMiscFloats * 4;
    sh.xs = reinterpret_cast<float*>(sh.ring + (size_t)p.nslots * p.slot_bytes);
    const int xfloats = max(max(max(p.Lqkv.slabs * p.Lqkv.slab_k, p.Lo.slabs * p.Lo.slab_k),
                                max(p.Lgu.slabs * p.Lgu.slab_k, p.Ldn.slabs * p.Ldn.slab_k)),
                            p.Llm.slabs * p.Llm.slab_k);
    sh.att = sh.xs + xfloats;
    sh.hs = sh.att + att_floats(G, D, p.Hkv, p.A);
    {
        uint32_t* t = reinterpret_cast<uint32_t*>(sh.hs + 2 * p.H);
        const QLayout* Ls[4] = {&p.Lqkv, &p.Lo, &p.Lgu, &p.Ldn};
        for (int i = 0; i < 4; ++i) {
            sh.segmask[i] = t;
            t += (Ls[i]->Np / 32 + 3) / 4 * 4;
        }
        sh.rows = reinterpret_cast<float*>(t);
    }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = gridDim.x, c = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nslots; ++i) {
            mbar_init(&sh.full[i], 1);
            mbar_init(&sh.empty[i], kStepConsumerWarps);
        }
        *sh.abort = 0;
        *sh.go = 1;
        fence_barrier_init();
    }
    __syncthreads();

    const int pos = p.seq->pos;
    const int npages = pos / kPageTokens + 1;
    const int A = p.A;
    const int head = c < A * p.Hkv ? c / A : -1;
    const int split = c < A * p.Hkv ? c % A : 0;
    const int pps = (npages + A - 1) / A;
    const int apg0 = min(npages, split * pps), apg1 = min(npages, apg0 + pps);

    if (warp == kStepConsumerWarps) {
        if (lane == 0) {
            Producer pr(p, sh);
            auto range = [&](const QLayout& L, int& u0, int& u1) {
                const int U = (L.Np / 32) * L.slabs;
                u0 = (int)((long long)c * U / C);
                u1 = (int)((long long)(c + 1) * U / C);
            };
            int u0, u1;
            for (int l = 0; l < p.num_layers && !pr.dead; ++l) {
                const StepLayer& ly = p.layers[l];
                range(p.Lqkv, u0, u1);
                pr.gemv(p.Lqkv, ly.qkv_w, ly.qkv_s, u0, u1);
                if (head >= 0) pr.attention(l, head, apg0, apg1);
                range(p.Lo, u0, u1);
                pr.gemv(p.Lo, ly.o_w, ly.o_s, u0, u1);
                range(p.Lgu, u0, u1);
                pr.gemv(p.Lgu, ly.gu_w, ly.gu_s, u0, u1);
                range(p.Ldn, u0, u1);
                pr.gemv(p.Ldn, ly.dn_w, ly.dn_s, u0, u1);
            }
            if (!pr.dead) {
                const int nrb = p.Llm.Np / 32;
                const int r0 = (int)((long long)c * nrb / C), r1 = (int)((long long)(c + 1) * nrb / C);
                pr.gemv(p.Llm, p.lm_w, p.lm_s, r0 * p.Llm.slabs, r1 * p.Llm.slabs);
            }
            if (pr.dead) pr.drain();
        }
        return;
    }

    Consumer cs(p, sh);
    cs.nph = 5 * p.num_layers + 1;
    {
        // Where the CTA segments of each 32-row block start (bit per slab).
        const QLayout* Ls[4] = {&p.Lqkv, &p.Lo, &p.Lgu, &p.Ldn};
        for (int i = 0; i < 4; ++i) {
            const QLayout& L = *Ls[i];
            const int nrb = L.Np / 32, U = nrb * L.slabs;
            for (int rb = threadIdx.x; rb < nrb; rb += kConsumers) {
                uint32_t m = 1u;
                for (int s = 1; s < L.slabs; ++s)
                    if (owner_of(rb * L.slabs + s, U, C) != owner_of(rb * L.slabs + s - 1, U, C)) m |= 1u << s;
                sh.segmask[i][rb] = m;
            }
        }
    }
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
            cs.residual_norm<PREC>(p.emb + (size_t)tok * p.H, nullptr, nullptr, nullptr, p.hX, ly.in_norm, p.Lqkv);
        } else {
            const StepLayer& pl = p.layers[l - 1];
            cs.residual_norm<PREC>(p.hY, &p.Ldn, sh.segmask[3], p.part_dn, p.hX, ly.in_norm, p.Lqkv);
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
        cs.residual_norm<PREC>(p.hX, &p.Lo, sh.segmask[1], p.part_o, p.hY, ly.post_norm, p.Lgu);
        cs.gemv_units<PREC>(p.Lgu, p.part_gu, ly.gu_s, ly.gu_b);
        cs.phase_end(phase - 1);
        // ---- down ----
        if (!cs.phase_begin(phase++)) return;
        cs.act_prologue<PREC>(ly);
        cs.gemv_units<PREC>(p.Ldn, p.part_dn, ly.dn_s, ly.dn_b);
        cs.phase_end(phase - 1);
    }
    // ---- final norm + LM head + argmax ----
    if (!cs.phase_begin(phase++)) return;
    {
        const StepLayer& pl = p.layers[p.num_layers - 1];
        cs.residual_norm<PREC>(p.hY, &p.Ldn, sh.segmask[3], p.part_dn, nullptr, p.final_norm, p.Llm);
    }
    cs.lm_head<PREC>(&p.seq->best);
    cs.phase_end(phase - 1);
    // ---- CTA 0 advances the step once every CTA folded its argmax ----
    if (c == 0 && cs.phase_begin(phase)) {
        if (threadIdx.x == 0) {
            __threadfence();
            finish_sequence_step(*p.seq, 0, p.out_tokens, p.prompt, p.prompt_stride);
            *p.bar = 0u;  // every CTA has passed its last barrier read
        }
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

bool supported(int prec, int G, int d) {
    if (prec != 8 && prec != 4) return false;
    return (G == 8 && d == 64) || (G == 1 && (d == 64 || d == 128)) || (G == 4 && d == 32) ||
           (prec == 8 && ((G == 4 && d == 64) || (G == 2 && d == 64) || (G == 1 && d == 32)));
}

}  // namespace

size_t step_smem_bytes(const StepParams& p, int* nslots, int* slot_bytes, int max_smem) {
    const int G = p.nheads / p.Hkv;
    if (!supported(p.Lqkv.precision, G, p.d)) return 0;
    if (p.A > 16 || (size_t)p.Hkv * G * p.A * 2 > (size_t)kMiscFloats) return 0;  // (m, l) staging in misc
    const int slot = p.Lqkv.precision == 4 ? 16384 + 4096 : 16384;
    const int att_tile = 2 * kPageTokens * p.d * 4;
    const int sbytes = std::max(slot, att_tile);
    const int xfloats = std::max(std::max(std::max(p.Lqkv.slabs * p.Lqkv.slab_k, p.Lo.slabs * p.Lo.slab_k),
                                          std::max(p.Lgu.slabs * p.Lgu.slab_k, p.Ldn.slabs * p.Ldn.slab_k)),
                                 p.Llm.slabs * p.Llm.slab_k);
    const size_t att = (size_t)std::max(G * p.d + 2 * p.d + 2 * G * kPageTokens, p.Hkv * G * p.A) * 4;
    size_t tabs = 0;
    for (const QLayout* L : {&p.Lqkv, &p.Lo, &p.Lgu, &p.Ldn}) {
        if (L->slabs > 32) return 0;  // segment masks are 32-bit
        tabs += (size_t)(L->Np / 32 + 3) / 4 * 4 * 4;
    }
    const size_t rows = (size_t)kStepConsumerWarps * kRowBlocksCached * 8 * 4;
    const size_t fixed =
        kBarRegion + kMiscFloats * 4 + (size_t)xfloats * 4 + att + (size_t)2 * p.H * 4 + tabs + rows;
    if ((size_t)max_smem <= fixed + 2 * (size_t)sbytes) return 0;
    int ns = (int)((max_smem - fixed) / sbytes);
    ns = std::min(ns, kMaxSlots);
    ns = std::min(ns, 10);  // leave L1 room for the few register spills
    if (const char* e = getenv("TB_STEP_SLOTS")) ns = std::max(2, std::min(ns, atoi(e)));
    *nslots = ns;
    *slot_bytes = sbytes;
    return fixed + (size_t)ns * sbytes;
}

cudaError_t launch_decode_step(const StepParams& p, int grid, size_t smem, cudaStream_t stream) {
    const int G = p.nheads / p.Hkv;
    const int prec = p.Lqkv.precision;
#define TB_STEP_CASE(pr, g, dd) \
    if (prec == pr && G == g && p.d == dd) return launch_t<pr, g, dd>(p, grid, smem, stream);
    TB_STEP_CASE(8, 8, 64)
    TB_STEP_CASE(4, 8, 64)
    TB_STEP_CASE(8, 1, 128)
    TB_STEP_CASE(4, 1, 128)
    TB_STEP_CASE(8, 1, 64)
    TB_STEP_CASE(4, 1, 64)
    TB_STEP_CASE(8, 4, 32)
    TB_STEP_CASE(4, 4, 32)
    TB_STEP_CASE(8, 4, 64)
    TB_STEP_CASE(8, 2, 64)
    TB_STEP_CASE(8, 1, 32)
#undef TB_STEP_CASE
    return cudaErrorNotSupported;
}

}  // namespace tb
