// tb_quant.cu -- device quantizers and the reference-layout -> GPU-layout repack.
//
// The quantizers restate Sources/TinyBrainRuntime/QuantizedTensor.swift
// bit-exactly: IEEE fp32 division (this file is compiled without fast-math),
// roundf (round half away from zero, as Swift's `round`), clamp, then the
// integer conversion.  The repack converts the reference's [K in][N out]
// row-major storage (INT8 per-column scales, INT4 flat groups packed high
// nibble first) into the streamed layouts documented in tb_kernels.h.
#include <algorithm>

#include "tb_common.cuh"
#include "tb_kernels.h"
#include "tb_tc.cuh"

namespace tb {

namespace {

constexpr float kFltTrueMin = 1.40129846e-45f;  // Float.leastNonzeroMagnitude

// QuantizedTensor.swift:388-405: per-column abs-max and scale.
__global__ void q8_scales_kernel(const float* __restrict__ W, int64_t K, int64_t N, float* __restrict__ scales) {
    const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float a = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
        const float v = fabsf(W[k * N + n]);
        if (v > a) a = v;
    }
    scales[n] = (a < kFltTrueMin) ? 1.0f : __fdiv_rn(a, 127.0f);
}

// QuantizedTensor.swift:408-416: q = clamp(round(w / scale), -127, 127).
__global__ void q8_values_kernel(const float* __restrict__ W, int64_t K, int64_t N, const float* __restrict__ scales,
                                 int8_t* __restrict__ Q) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= K * N) return;
    float q = roundf(__fdiv_rn(W[i], scales[i % N]));
    q = fmaxf(-127.0f, fminf(127.0f, q));
    Q[i] = (int8_t)q;
}

// QuantizedTensor.swift:514-535: per flat group scale (zero point 0).
__global__ void q4_scales_kernel(const float* __restrict__ x, int64_t count, int64_t gs, float* __restrict__ scales,
                                 int8_t* __restrict__ zp) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t ng = (count + gs - 1) / gs;
    if (g >= ng) return;
    const int64_t b = g * gs, e = min(b + gs, count);
    float mn = x[b], mx = x[b];
    for (int64_t i = b + 1; i < e; ++i) {
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
    }
    const float a = fmaxf(fabsf(mn), fabsf(mx));
    scales[g] = (a < kFltTrueMin) ? 1.0f : __fdiv_rn(a, 7.0f);
    if (zp) zp[g] = 0;
}

// QuantizedTensor.swift:537-551: clamp(round(x/scale), -7, 7), even index in
// the high nibble, odd index in the low nibble.
__device__ __forceinline__ int q4_of(const float* x, const float* scales, int64_t i, int64_t gs) {
    float q = roundf(__fdiv_rn(x[i], scales[i / gs]));
    q = fmaxf(-7.0f, fminf(7.0f, q));
    return (int)q;
}
__global__ void q4_pack_kernel(const float* __restrict__ x, int64_t count, int64_t gs,
                               const float* __restrict__ scales, uint8_t* __restrict__ packed) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= (count + 1) / 2) return;
    const int64_t i0 = 2 * b, i1 = i0 + 1;
    uint32_t v = ((uint32_t)(q4_of(x, scales, i0, gs) & 0x0F)) << 4;
    if (i1 < count) v |= (uint32_t)(q4_of(x, scales, i1, gs) & 0x0F);
    packed[b] = (uint8_t)v;
}

// ---- repack ----

// INT8: one thread per (destination row, 16-value k chunk): 16 signed bytes
// into the tensor-core operand layout of the row's 128-row tile.  Threads with
// consecutive n read consecutive source bytes of row k.
// QuantizedTensor.dequantize (QuantizedTensor.swift:182-285): perChannel
// [K][N] with scales (and zero points) per output column; INT4 flat groups of
// gs elements, even index = high nibble, nibbles sign-extended.
// value = (q - zero_point) * scale, in fp32.
__global__ void dequantize_kernel(int prec, const uint8_t* __restrict__ data, const float* __restrict__ scales,
                                  const int8_t* __restrict__ zps, int64_t count, int64_t N, int64_t gs,
                                  float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        int q;
        int64_t si;
        if (prec == 8) {
            q = (int)(int8_t)data[i];
            si = i % N;
        } else {
            const uint8_t b = data[i >> 1];
            const int raw = (i & 1) ? (b & 0x0F) : (b >> 4);
            q = raw > 7 ? raw - 16 : raw;
            si = i / gs;
        }
        const float zp = zps ? (float)zps[si] : 0.0f;
        out[i] = __fmul_rn(__fsub_rn((float)q, zp), scales[si]);
    }
}

__global__ void repack_q8_kernel(const int8_t* __restrict__ src, int K, int N, QLayout L, uint8_t* __restrict__ dst,
                                 int row_offset, int interleave) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int kc = blockIdx.y;  // 16-value chunk
    if (n >= N) return;
    const int drow = fused_row(L, n, row_offset, interleave);
    const int tile = drow / kTcTileRows, r = drow % kTcTileRows;
    const int k0 = kc * 16;
    const int unit = k0 / kTcUnitK, c = (k0 % kTcUnitK) / 16;
    uint8_t* out = dst + ((size_t)tile * L.slabs + unit) * kTcUnitBytes + ((r / 8) * 8 + c) * 128 + (r % 8) * 16;
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int k = k0 + q * 4 + b;
            const int v = (k < K) ? (int)src[(size_t)k * N + n] : 0;
            word |= ((uint32_t)(v & 0xFF)) << (8 * b);
        }
        w[q] = word;
    }
    *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void repack_scales_q8_kernel(const float* __restrict__ src, int N, QLayout L, float* __restrict__ dst,
                                        int row_offset, int interleave) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    dst[fused_row(L, n, row_offset, interleave)] = src[n];
}

__device__ __forceinline__ int src_nibble(const uint8_t* packed, int64_t i) {
    const uint8_t b = packed[i >> 1];
    const int raw = (i & 1) == 0 ? (b >> 4) & 0xF : b & 0xF;
    return raw > 7 ? raw - 16 : raw;
}

// INT4: one thread per (destination row n, 32-value k chunk = 16 bytes) of
// the tensor-core unit layout (tb_tc.cuh): chunk c of unit s of tile t at
// ((t * slabs + s) * kQ4UnitBytes) + (c * 128 + row) * 16; in word j, byte i =
// (q[k 8j+i] + 8) | (q[k 8j+i+4] + 8) << 4.
__global__ void repack_q4_kernel(const uint8_t* __restrict__ src, int K, int N, QLayout L, uint8_t* __restrict__ dst,
                                 int row_offset, int interleave) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int kc = blockIdx.y;  // 32-value chunk
    if (n >= N) return;
    const int drow = fused_row(L, n, row_offset, interleave);
    const int tile = drow / kTcTileRows, r = drow % kTcTileRows;
    const int s = kc >> 2, c = kc & 3;
    uint8_t* out = dst + ((size_t)tile * L.slabs + s) * kQ4UnitBytes + (size_t)(c * kTcTileRows + r) * 16;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = kc * 32 + 8 * j + i;
            const int lo = (k < K) ? src_nibble(src, (int64_t)k * N + n) : 0;
            const int hi = (k + 4 < K) ? src_nibble(src, (int64_t)(k + 4) * N + n) : 0;
            word |= ((uint32_t)((lo + 8) & 0xF) | ((uint32_t)((hi + 8) & 0xF) << 4)) << (8 * i);
        }
        w[j] = word;
    }
    *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2], w[3]);
}

// INT4 group scales into the unit's scale block [4 row groups][128 k]: one
// thread per (k, 32-row source group); the value is the scale of the
// reference group holding flat index k*N + n0 (32 | gs, gs | N: all 32 rows
// of the group share it, QuantizedTensor.swift:502-535).
__global__ void repack_scales_q4_kernel(const float* __restrict__ src, int K, int N, int gs, QLayout L,
                                        uint8_t* __restrict__ dst, int row_offset, int interleave) {
    const int g32 = blockIdx.y;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= L.slabs * kTcUnitK) return;
    const int n0 = g32 * 32;
    if (n0 >= N) return;
    const int drow = fused_row(L, n0, row_offset, interleave);
    const int tile = drow / kTcTileRows, grp = (drow % kTcTileRows) / 32;
    const int s = k / kTcUnitK, kk = k % kTcUnitK;
    float* sc = reinterpret_cast<float*>(dst + ((size_t)tile * L.slabs + s) * kQ4UnitBytes + kQ4UnitNibBytes);
    sc[grp * kTcUnitK + kk] = (k < K) ? src[((int64_t)k * N + n0) / gs] : 0.0f;
}

// Largest |scale| of every (32-row group, unit): bounds the B-operand digits.
// Table layout [tile][4 groups][slabs].
__global__ void scale_max_q4_kernel(const uint8_t* __restrict__ w, int N, QLayout L, float* __restrict__ smax,
                                    int row_offset, int interleave) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    const int g32 = blockIdx.y;
    if (s >= L.slabs || g32 * 32 >= N) return;
    const int drow = fused_row(L, g32 * 32, row_offset, interleave);
    const int tile = drow / kTcTileRows, grp = (drow % kTcTileRows) / 32;
    const float* sc =
        reinterpret_cast<const float*>(w + ((size_t)tile * L.slabs + s) * kQ4UnitBytes + kQ4UnitNibBytes) +
        grp * kTcUnitK;
    float m = 0.0f;
    for (int kk = 0; kk < kTcUnitK; ++kk) m = fmaxf(m, fabsf(sc[kk]));
    smax[((size_t)tile * kQ4Groups + grp) * L.slabs + s] = m;
}

}  // namespace

cudaError_t launch_quantize_int8_per_channel(const float* W, int64_t K, int64_t N, int8_t* Q, float* scales,
                                             cudaStream_t stream) {
    if (K <= 0 || N <= 0) return cudaSuccess;
    q8_scales_kernel<<<(unsigned)((N + 255) / 256), 256, 0, stream>>>(W, K, N, scales);
    const int64_t tot = K * N;
    q8_values_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, stream>>>(W, K, N, scales, Q);
    return cudaGetLastError();
}

cudaError_t launch_quantize_int4_group(const float* x, int64_t count, int64_t gs, uint8_t* packed, float* scales,
                                       int8_t* zp, cudaStream_t stream) {
    if (count <= 0) return cudaSuccess;
    const int64_t ng = (count + gs - 1) / gs;
    q4_scales_kernel<<<(unsigned)((ng + 255) / 256), 256, 0, stream>>>(x, count, gs, scales, zp);
    const int64_t nb = (count + 1) / 2;
    q4_pack_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, stream>>>(x, count, gs, scales, packed);
    return cudaGetLastError();
}

cudaError_t launch_dequantize(int prec, const uint8_t* data, const float* scales, const int8_t* zps, int64_t K,
                              int64_t N, int64_t gs, float* out, cudaStream_t stream) {
    const int64_t count = K * N;
    if (count <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((count + 255) / 256, 148 * 16);
    dequantize_kernel<<<(unsigned)blocks, 256, 0, stream>>>(prec, data, scales, zps, count, N, gs > 0 ? gs : count,
                                                           out);
    return cudaGetLastError();
}

cudaError_t launch_repack(const RepackSrc& s, const QLayout& L, uint8_t* w_out, float* scales_out, int row_offset,
                          int interleave, cudaStream_t stream) {
    const unsigned nb = (unsigned)((s.N + 127) / 128);
    if (s.precision == 8) {
        repack_q8_kernel<<<dim3(nb, (unsigned)(L.Kp / 16)), 128, 0, stream>>>(
            (const int8_t*)s.data, s.K, s.N, L, w_out, row_offset, interleave);
        repack_scales_q8_kernel<<<nb, 128, 0, stream>>>(s.scales, s.N, L, scales_out, row_offset, interleave);
    } else {
        repack_q4_kernel<<<dim3(nb, (unsigned)(L.Kp / 32)), 128, 0, stream>>>(
            (const uint8_t*)s.data, s.K, s.N, L, w_out, row_offset, interleave);
        const unsigned ng = (unsigned)((s.N + 31) / 32);
        const unsigned ne = (unsigned)((L.slabs * kTcUnitK + 255) / 256);
        repack_scales_q4_kernel<<<dim3(ne, ng), 256, 0, stream>>>(s.scales, s.K, s.N, s.group_size, L, w_out,
                                                                  row_offset, interleave);
        scale_max_q4_kernel<<<dim3((unsigned)((L.slabs + 127) / 128), ng), 128, 0, stream>>>(
            w_out, s.N, L, scales_out, row_offset, interleave);
    }
    return cudaGetLastError();
}

}  // namespace tb
