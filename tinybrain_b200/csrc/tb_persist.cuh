// tb_persist.cuh -- pieces shared by the persistent decode-step kernels
// (tb_step.cu: grid-barrier phases; tb_flow.cu: tagged dataflow phases):
// ring geometry, the weight / KV-page producer warp, split-K segment tables.
#pragma once

#include "tb_common.cuh"
#include "tb_kernels.h"
#include "tb_tc.cuh"

#include <algorithm>

namespace tb {
namespace persist {

constexpr int kMaxSlots = 24;
constexpr int kMaxSegs = 16;                 // INT8: segments per CTA and phase
constexpr int kIssuers = 2;                  // INT8: threads issuing tensor-core products (alternate units)
constexpr int kTmemCols = kMaxSegs * kIssuers * 8;  // 8 TMEM columns (4 digits + 4 zero) per block
constexpr int kBarRegion = 1024;             // mbarriers + flags
constexpr int kMiscFloats = 2048;
constexpr int kConsumers = kStepConsumerWarps * 32;
constexpr int kMaxTileSegs = 32;             // split-K segments per row block (table width)

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The CTA whose static unit range [c*U/C, (c+1)*U/C) contains unit u.
__host__ __device__ inline int owner_of(int u, int U, int C) { return (int)(((long long)u * C + C - 1) / U); }

__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

__device__ __forceinline__ int att_floats(int G, int d, int Hkv, int A) {
    return max(G * d + 2 * d + 2 * G * kPageTokens, Hkv * G * A);
}

// Rows per streamed unit (128-row tiles).
__host__ __device__ constexpr int unit_rows(int) { return kTcTileRows; }
__host__ __device__ inline int phase_units(const QLayout& L) { return (L.Np / unit_rows(L.precision)) * L.slabs; }
// Segment table bytes of a phase: [rb][kMaxTileSegs] unit indices + [rb] counts (16-byte rounded).
__host__ __device__ inline int seg_table_bytes(const QLayout& L) {
    const int nrb = L.Np / unit_rows(L.precision);
    return (nrb * kMaxTileSegs + nrb + 15) / 16 * 16;
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
    __device__ __forceinline__ void advance(int k, int n) {
        const int t = st + k;
        ph ^= (uint32_t)((t / n) & 1);
        st = t % n;
    }
};

// ------------------------------------------------------------------ producer --
template <class SH>
struct Producer {
    const StepParams& p;
    SH sh;  // by value: the pointers stay in registers, not in local memory
    int it = 0;        // copies issued
    Cursor cur;        // slot of copy `it`
    Cursor thr;        // slot of copy `it - nflight` (throttle)
    uint64_t pol;
    bool dead = false;

    __device__ Producer(const StepParams& p_, const SH& sh_) : p(p_), sh(sh_) { pol = l2_policy_evict_first(); }

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

    // Units [u0, u1) of a GEMV phase: consecutive 16 KB INT8 tiles-units in memory.
    template <int PREC>
    __device__ void gemv(const QLayout& L, const uint8_t* w, const float* sc, int u0, int u1) {
        static_assert(PREC == 8, "the persistent step streams INT8 units");
        (void)L;
        (void)sc;
        for (int u = u0; u < u1 && !dead; ++u) {
            int st;
            uint8_t* dst = acquire(st);
            if (!dst) return;
            mbar_arrive_expect_tx(&sh.full[st], kTcUnitBytes);
            bulk_g2s_stream(dst, w + (size_t)u * kTcUnitBytes, kTcUnitBytes, &sh.full[st], pol);
            issued();
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

// Segment tables: for every row block of a phase, the units (ascending) where
// a CTA's unit range starts a segment of that row block.
__device__ inline void build_seglist(uint8_t* list, uint8_t* cnt, const QLayout& L, int C, int tid, int nthreads) {
    const int ru = unit_rows(L.precision);
    const int nrb = L.Np / ru, U = nrb * L.slabs;
    for (int rb = tid; rb < nrb; rb += nthreads) {
        int n = 0;
        for (int s = 0; s < L.slabs && n < kMaxTileSegs; ++s)
            if (s == 0 || owner_of(rb * L.slabs + s, U, C) != owner_of(rb * L.slabs + s - 1, U, C))
                list[rb * kMaxTileSegs + n++] = (uint8_t)s;
        cnt[rb] = (uint8_t)n;
    }
}

// Largest number of CTA segments any row block of a phase is split into.
inline int max_tile_segments(const QLayout& L, int C) {
    const int nrb = L.Np / unit_rows(L.precision), U = nrb * L.slabs;
    int best = 0;
    for (int rb = 0; rb < nrb; ++rb) {
        int n = 0;
        for (int s = 0; s < L.slabs; ++s)
            if (s == 0 || owner_of(rb * L.slabs + s, U, C) != owner_of(rb * L.slabs + s - 1, U, C)) ++n;
        best = std::max(best, n);
    }
    return best;
}

// Largest number of row blocks any CTA's unit range of a phase touches.
inline int max_segments(const QLayout& L, int C, bool whole_blocks) {
    const int nrb = L.Np / unit_rows(L.precision);
    int best = 0;
    for (int c = 0; c < C; ++c) {
        int n;
        if (whole_blocks) {
            n = (int)((long long)(c + 1) * nrb / C) - (int)((long long)c * nrb / C);
        } else {
            const int U = nrb * L.slabs;
            const int u0 = (int)((long long)c * U / C), u1 = (int)((long long)(c + 1) * U / C);
            n = u1 > u0 ? (u1 - 1) / L.slabs - u0 / L.slabs + 1 : 0;
        }
        best = std::max(best, n);
    }
    return best;
}

}  // namespace persist
}  // namespace tb
