// tb_tc.cuh -- 5th-generation tensor-core (tcgen05) helpers for the INT8
// weight-only GEMV (sm_100a only).
//
// An INT8 projection y = W x (W: q[n][k] * scale[n]) runs on the integer
// tensor cores exactly:
//   * the activation slice x is scaled by a power of two 2^-e chosen so that
//     |x| * 2^-e < 127, and split into four signed 8-bit digits
//         u = x * 2^-e = d0 + d1 2^-7 + d2 2^-14 + d3 2^-21 (+ |r| <= 2^-22);
//     every step is exact in fp32 (power-of-two scaling, round-to-integer,
//     exact subtraction), so the digits carry x to 2^-29 of max|x|;
//   * tcgen05.mma kind::i8 multiplies a 128-row weight tile (A, K-major in
//     shared memory) by the digit matrix (B: N = 8 rows per batch row pair,
//     K-major) into int32 accumulators in tensor memory -- exact integer sums;
//   * the epilogue reads one row per thread (tcgen05.ld 32x32b), combines the
//     digit columns in int64 (D0 2^21 + D1 2^14 + D2 2^7 + D3), converts once
//     to fp32 and applies 2^(e-21), the per-row weight scale and the bias.
// The result equals the fp32 dot product of the reference
// (Sources/TinyBrainRuntime/QuantizedTensor.swift:430-460: dequantised
// weights times x, fp32 accumulation) to ~1e-7 relative, with a single
// rounding instead of K sequential ones.
//
// Shared-memory operand layouts (no swizzle, "interleaved" canonical K-major):
//   A (weights, one 16 KB unit = 128 rows x 128 k): [16 row groups][8 k-chunks of
//     16 bytes][8 rows][16 bytes]; core matrix (8 rows x 16 bytes) = 128
//     contiguous bytes; LBO (next 16-byte k-chunk) = 128 B, SBO (next 8-row
//     group) = 1024 B.  The GPU weight layout stores units in exactly this
//     form so a 1-D bulk copy lands it ready for the tensor core.
//   B (digits, NB rows): [k-chunk of 16][NB/8 row groups][8 rows][16 bytes];
//     LBO = NB * 16 B, SBO = 128 B.  Row n = 4 * m + j holds digit j of batch
//     row m.
#pragma once

#include "tb_common.cuh"

namespace tb {

constexpr int kTcTileRows = 128;    // A tile rows (M of the MMA)
constexpr int kTcUnitK = 128;       // k per weight unit
constexpr int kTcUnitBytes = kTcTileRows * kTcUnitK;  // 16 KB
constexpr int kTcDigits = 4;

// ---- tensor memory ----
// Allocate `ncols` TMEM columns (power of two >= 32); the whole warp executes.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 format: start, LBO, SBO in 16-byte
// units; version 1; no swizzle).
__device__ __forceinline__ uint64_t tc_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor: kind::i8, D s32, A s8, B s8, both K-major, M = 128.
__host__ __device__ constexpr uint32_t tc_idesc_i8(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcTileRows >> 4) << 24);
}
// D[tmem] (+)= A * B^T for one K = 32 step; issued by a single thread.
__device__ __forceinline__ void tc_mma_i8(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// Arrive once on `bar` when every tcgen05 operation issued so far by this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// Issue the four K = 32 steps of one 16 KB weight unit (A at `a_saddr`)
// against the digit columns of its k range (B at `b_saddr`).
__device__ __forceinline__ void tc_unit_mma(uint32_t dtmem, uint32_t a_saddr, uint32_t b_saddr, int nb,
                                            bool accumulate) {
    const uint32_t idesc = tc_idesc_i8(nb);
#pragma unroll
    for (int s = 0; s < kTcUnitK / 32; ++s) {
        const uint64_t ad = tc_sdesc(a_saddr + s * 256, 128, 1024);
        const uint64_t bd = tc_sdesc(b_saddr + s * 2 * nb * 16, nb * 16, 128);
        tc_mma_i8(dtmem, ad, bd, idesc, accumulate || s > 0);
    }
}

// D[tmem] (+)= A[tmem] * B^T for one K = 32 step, A read from tensor memory
// (lane = row, 32-bit column c = k 4c .. 4c+3 as bytes, low k in the low byte).
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t dtmem, uint32_t atmem, uint64_t bdesc, uint32_t idesc,
                                             bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(dtmem),
        "r"(atmem), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// Warp-collective store of 32 consecutive 32-bit columns of the warp's 32 TMEM
// lanes (lane i of the warp writes row 32 * (warp % 4) + i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---- INT4 weights on the integer tensor cores ----
// A 128-row x 128-k INT4 unit in HBM / shared memory (10 KB):
//   nibbles: [4 k-chunks of 32][128 rows][16 bytes]; in word j (k 8j .. 8j+7
//     of the chunk) byte i holds k 8j+i in its low and k 8j+i+4 in its high
//     nibble, each biased by +8 (value q in [-8, 7] stored as q + 8);
//   scales: [4 row groups of 32][128 k] fp32 (the reference's group scale of
//     those 32 rows at that k).
// Expanded to int8 in registers and stored to tensor memory as the A operand;
// the scales go into the B operand (digits of scale * x per row group).
constexpr int kQ4UnitNibBytes = kTcTileRows * kTcUnitK / 2;                 // 8 KB
constexpr int kQ4UnitBytes = kQ4UnitNibBytes + 4 * kTcUnitK * 4;            // + 2 KB of scales
constexpr int kQ4Groups = kTcTileRows / 32;                                  // row groups per tile

// One nibble word -> the int8 words of k 8j..8j+3 (lo) and 8j+4..8j+7 (hi).
// b + 0x78 stays inside its byte for b <= 15, and ^0x80 then yields b - 8 in
// two's complement.
__device__ __forceinline__ void q4_expand(uint32_t w, uint32_t& lo, uint32_t& hi) {
    lo = ((w & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
    hi = (((w >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
}

// Warp-collective load of 8 / 16 / 32 consecutive accumulator columns of the
// warp's 32 TMEM lanes (lane i of the warp gets row (32 * (warp % 4) + i)).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, int (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- activation digits ----
// Exponent e with max_abs * 2^-e < 127 (0 for max_abs == 0).
__device__ __forceinline__ int digit_exponent(float max_abs) {
    int e = 0;
    (void)frexpf(max_abs * (1.0f / 127.0f), &e);
    // max/127 = f 2^e, f in [0.5, 1): max 2^-e < 127.  The product with 1/127
    // may round up across a power of two; that only makes e larger (still safe).
    return e;
}
// Digit words of four consecutive k (k0 % 4 == 0) of batch row m, written to
// the B operand: word j = bytes (d_j(x0), d_j(x1), d_j(x2), d_j(x3)).
// Round-to-integer by the 1.5 * 2^23 magic constant (IEEE round-to-nearest-
// even, the same rounding as rintf): t = u + M holds rint(u) in its low
// mantissa bits, so the digit byte is the low byte of t's bit pattern; the
// remainder u' = 128 u - 128 (t - M) is computed exactly by two FMAs.
__device__ __forceinline__ void put_digits4(uint8_t* xd, int nb, int k0_rel, int m, float4 v, float inv_scale) {
    constexpr float kM = 12582912.0f;  // 1.5 * 2^23
    const float2 sc = make_float2(inv_scale, inv_scale);
    float2 u01 = __fmul2_rn(make_float2(v.x, v.y), sc);  // exact: power-of-two scaling
    float2 u23 = __fmul2_rn(make_float2(v.z, v.w), sc);
    uint8_t* base = xd + (size_t)(k0_rel >> 4) * nb * 16 + (k0_rel & 15);
#pragma unroll
    for (int j = 0; j < kTcDigits; ++j) {
        const float2 t01 = __fadd2_rn(u01, make_float2(kM, kM));
        const float2 t23 = __fadd2_rn(u23, make_float2(kM, kM));
        const uint32_t lo = prmt(__float_as_uint(t01.x), __float_as_uint(t01.y), 0x0040u);
        const uint32_t hi = prmt(__float_as_uint(t23.x), __float_as_uint(t23.y), 0x0040u);
        const int row = m * kTcDigits + j;
        *reinterpret_cast<uint32_t*>(base + ((row >> 3) * 128) + (row & 7) * 16) = prmt(lo, hi, 0x5410u);
        if (j + 1 < kTcDigits) {
            const float2 n01 = __ffma2_rn(t01, make_float2(-128.0f, -128.0f), make_float2(128.0f * kM, 128.0f * kM));
            const float2 n23 = __ffma2_rn(t23, make_float2(-128.0f, -128.0f), make_float2(128.0f * kM, 128.0f * kM));
            u01 = __ffma2_rn(u01, make_float2(128.0f, 128.0f), n01);
            u23 = __ffma2_rn(u23, make_float2(128.0f, 128.0f), n23);
        }
    }
}
// put_digits4 into a B operand with explicit strides: `lbo` bytes between
// 16-k chunks, `sbo` between 8-row core matrices (a padded sbo spreads the
// stores of a warp over all banks).
__device__ __forceinline__ void put_digits4_strided(uint8_t* xd, uint32_t lbo, uint32_t sbo, int k0_rel, int m,
                                                    float4 v, float inv_scale) {
    constexpr float kM = 12582912.0f;  // 1.5 * 2^23
    const float2 sc = make_float2(inv_scale, inv_scale);
    float2 u01 = __fmul2_rn(make_float2(v.x, v.y), sc);
    float2 u23 = __fmul2_rn(make_float2(v.z, v.w), sc);
    uint8_t* base = xd + (size_t)(k0_rel >> 4) * lbo + (k0_rel & 15);
#pragma unroll
    for (int j = 0; j < kTcDigits; ++j) {
        const float2 t01 = __fadd2_rn(u01, make_float2(kM, kM));
        const float2 t23 = __fadd2_rn(u23, make_float2(kM, kM));
        const uint32_t lo = prmt(__float_as_uint(t01.x), __float_as_uint(t01.y), 0x0040u);
        const uint32_t hi = prmt(__float_as_uint(t23.x), __float_as_uint(t23.y), 0x0040u);
        const int row = m * kTcDigits + j;
        *reinterpret_cast<uint32_t*>(base + (row >> 3) * sbo + (row & 7) * 16) = prmt(lo, hi, 0x5410u);
        if (j + 1 < kTcDigits) {
            const float2 n01 = __ffma2_rn(t01, make_float2(-128.0f, -128.0f), make_float2(128.0f * kM, 128.0f * kM));
            const float2 n23 = __ffma2_rn(t23, make_float2(-128.0f, -128.0f), make_float2(128.0f * kM, 128.0f * kM));
            u01 = __ffma2_rn(u01, make_float2(128.0f, 128.0f), n01);
            u23 = __ffma2_rn(u23, make_float2(128.0f, 128.0f), n23);
        }
    }
}
// Combined accumulator of one batch row: digits at columns 4m .. 4m+3.
__device__ __forceinline__ float combine_digits(const int* d, int e) {
    const long long v = ((long long)d[0] << 21) + ((long long)d[1] << 14) + ((long long)d[2] << 7) + (long long)d[3];
    const int k = e - 21;
    // one rounding (int64 -> fp32), then an exact power-of-two scaling; the
    // bit-pattern power of two covers the normal range, ldexpf the rest
    const float f = __ll2float_rn(v);
    return (k >= -126 && k <= 127) ? f * __int_as_float((k + 127) << 23) : ldexpf(f, k);
}

}  // namespace tb
