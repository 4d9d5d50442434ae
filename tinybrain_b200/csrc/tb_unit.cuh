// tb_unit.cuh -- the inner product of one streamed weight unit (32 rows x one
// 512-byte slab) against a staged activation slice, shared by the per-op GEMV
// kernel (tb_gemv.cu) and the persistent decode-step kernel (tb_step.cu).
//
// Unit layout in shared memory: 32 rows of `sb` bytes, row-major; lane l of
// warp w reads the 16 bytes at [l*16, l*16+16) of rows 4w..4w+3.  The
// activation slice of the slab is lane-interleaved (see xperm) so lane l's 16
// (INT8) or 32 (INT4) values are four or eight conflict-free float4 loads.
#pragma once

#include "tb_common.cuh"

namespace tb {

// Exponent-bias constant: a biased integer u placed in the low mantissa bits
// of 2^23 reads as 2^23 + u; subtracting (2^23 + bias * scale) is exact.
constexpr float kTwo23 = 8388608.0f;

// Position of k (relative to its slab) in the lane-interleaved x / scale layout.
template <int CH>
__device__ __forceinline__ int xperm(int k_in_slab) {
    const int lane = k_in_slab / CH;
    const int r = k_in_slab % CH;
    return ((r >> 2) * 32 + lane) * 4 + (r & 3);
}

// INT4: per-position scale factor 2^-shift folded into x so that nibble p of
// a 32-bit word can be extracted in place with a single LOP3.
__device__ __forceinline__ float int4_pos_scale(int p) {
    // nibble p sits at bit 4p (p < 5) or, after the >>12, at bit 4(p-3)
    const int shift = p < 5 ? 4 * p : 4 * (p - 3);
    return __int_as_float((127 - shift) << 23);
}

// Accumulate rows [row0, row0 + RPW) of a unit (row stride sb bytes) against
// the slab's activations xsl (lane-interleaved, MB rows xstride apart).  INT4
// units carry the group scales of these rows at ssl (lane-interleaved).
template <int PREC, int RPW, int MB>
__device__ __forceinline__ void unit_dot(const uint8_t* __restrict__ wunit, int sb, int row0,
                                         const float* __restrict__ ssl, const float* __restrict__ xsl, int xstride,
                                         int lane, float2 (&acc)[RPW][MB]) {
    if (lane * 16 >= sb) return;
    uint4 wq[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) wq[r] = lds128(wunit + (row0 + r) * sb + lane * 16);
    if (PREC == 8) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float4 xv[MB];
#pragma unroll
            for (int m = 0; m < MB; ++m) xv[m] = lds128f(xsl + m * xstride + (c * 32 + lane) * 4);
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                const uint32_t wd = c == 0 ? wq[r].x : c == 1 ? wq[r].y : c == 2 ? wq[r].z : wq[r].w;
                const float f0 = __uint_as_float(prmt(wd, 0x4B000000u, 0x7440u));
                const float f1 = __uint_as_float(prmt(wd, 0x4B000000u, 0x7441u));
                const float f2 = __uint_as_float(prmt(wd, 0x4B000000u, 0x7442u));
                const float f3 = __uint_as_float(prmt(wd, 0x4B000000u, 0x7443u));
                const float2 nb = make_float2(-(kTwo23 + 128.0f), -(kTwo23 + 128.0f));
                const float2 v01 = __fadd2_rn(make_float2(f0, f1), nb);
                const float2 v23 = __fadd2_rn(make_float2(f2, f3), nb);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    acc[r][m] = __ffma2_rn(v01, make_float2(xv[m].x, xv[m].y), acc[r][m]);
                    acc[r][m] = __ffma2_rn(v23, make_float2(xv[m].z, xv[m].w), acc[r][m]);
                }
            }
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            // word c of the lane's 16 bytes holds k = 32*lane + 8c + p, p = 0..7
            float2 xsv[MB][4];
            const float4 sa = lds128f(ssl + ((2 * c) * 32 + lane) * 4);
            const float4 sbv = lds128f(ssl + ((2 * c + 1) * 32 + lane) * 4);
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                const float4 xa = lds128f(xsl + m * xstride + ((2 * c) * 32 + lane) * 4);
                const float4 xb = lds128f(xsl + m * xstride + ((2 * c + 1) * 32 + lane) * 4);
                xsv[m][0] = __fmul2_rn(make_float2(xa.x, xa.y), make_float2(sa.x, sa.y));
                xsv[m][1] = __fmul2_rn(make_float2(xa.z, xa.w), make_float2(sa.z, sa.w));
                xsv[m][2] = __fmul2_rn(make_float2(xb.x, xb.y), make_float2(sbv.x, sbv.y));
                xsv[m][3] = __fmul2_rn(make_float2(xb.z, xb.w), make_float2(sbv.z, sbv.w));
            }
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                const uint32_t wd = c == 0 ? wq[r].x : c == 1 ? wq[r].y : c == 2 ? wq[r].z : wq[r].w;
                const uint32_t t = wd >> 12;
                const float f0 = __uint_as_float((wd & 0x0000000Fu) | 0x4B000000u);
                const float f1 = __uint_as_float((wd & 0x000000F0u) | 0x4B000000u);
                const float f2 = __uint_as_float((wd & 0x00000F00u) | 0x4B000000u);
                const float f3 = __uint_as_float((wd & 0x0000F000u) | 0x4B000000u);
                const float f4 = __uint_as_float((wd & 0x000F0000u) | 0x4B000000u);
                const float f5 = __uint_as_float((t & 0x00000F00u) | 0x4B000000u);
                const float f6 = __uint_as_float((t & 0x0000F000u) | 0x4B000000u);
                const float f7 = __uint_as_float((t & 0x000F0000u) | 0x4B000000u);
                const float2 v01 =
                    __fadd2_rn(make_float2(f0, f1), make_float2(-(kTwo23 + 8.0f), -(kTwo23 + 128.0f)));
                const float2 v23 =
                    __fadd2_rn(make_float2(f2, f3), make_float2(-(kTwo23 + 2048.0f), -(kTwo23 + 32768.0f)));
                const float2 v45 =
                    __fadd2_rn(make_float2(f4, f5), make_float2(-(kTwo23 + 524288.0f), -(kTwo23 + 2048.0f)));
                const float2 v67 =
                    __fadd2_rn(make_float2(f6, f7), make_float2(-(kTwo23 + 32768.0f), -(kTwo23 + 524288.0f)));
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    acc[r][m] = __ffma2_rn(v01, xsv[m][0], acc[r][m]);
                    acc[r][m] = __ffma2_rn(v23, xsv[m][1], acc[r][m]);
                    acc[r][m] = __ffma2_rn(v45, xsv[m][2], acc[r][m]);
                    acc[r][m] = __ffma2_rn(v67, xsv[m][3], acc[r][m]);
                }
            }
        }
    }
}

// Step bookkeeping of one sequence after its LM head (ModelRunner.swift:251-292):
// the argmax becomes the next input once the prompt is consumed (and is
// recorded as a generated token); before that the next prompt token is fed.
__device__ __forceinline__ void finish_sequence_step(SeqState& sq, int m, int* out_tokens, const int* prompt,
                                                     int prompt_stride) {
    const unsigned long long b = atomicAdd(&sq.best, 0ull);
    const int tok = (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
    int next;
    if (sq.pos >= sq.n_prompt - 1) {
        if (sq.n_out < sq.max_out) out_tokens[(size_t)m * sq.max_out + sq.n_out] = tok;
        sq.n_out += 1;
        next = tok;
    } else {
        next = prompt[(size_t)m * prompt_stride + sq.pos + 1];
    }
    sq.token = next;
    sq.pos += 1;
    sq.best = 0ull;
}

// Packed argmax key: larger value first; among equal values the lower index
// (Sampler.swift:126-138).
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
    return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

}  // namespace tb
