// tq_common.cuh — device-side definitions shared by the TurboQuant kernels.
//
// Block formats are byte-identical to LeanKV's (src/ggml-tq.h:131-141):
//   TQ4_0: 18 bytes per 32 elements = fp16 d + 16 bytes; byte j = elem j | elem (j+16) << 4
//   TQ3_0: 14 bytes per 32 elements = fp16 d + 12 bytes; each 3-byte group is a
//          little-endian 24-bit word with code i of the group at bits 3i..3i+2
//          (src/ggml-tq.c:26-55).
// The scale d is written with the standalone build's truncating fp32->fp16
// encoder and read with its decoder (src/ggml-tq.h:39-64), both restated here
// bit-for-bit, including its flush of sub-2^-14 values to zero and its
// decoding of exponent 31 as the finite value 2^16 * 1.m.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace tq {

constexpr int QK = 32;
constexpr int TQ4_BYTES = 18;
constexpr int TQ3_BYTES = 14;
constexpr int TQ2_BYTES = 10;
template <int QT> struct BlockBytes { static constexpr int value = QT == 4 ? TQ4_BYTES : QT == 3 ? TQ3_BYTES : TQ2_BYTES; };

// Lloyd-Max codebooks (src/ggml-tq.h:98-121).  Symmetric: L[n-1-i] == -L[i]
// and B[n-2-i] == -B[i] exactly in float32, which the nearest-level search
// below relies on.
__host__ __device__ constexpr float tq3_level(int i) {
    return i == 0 ? -1.0000000f : i == 1 ? -0.6245203f : i == 2 ? -0.3513239f : i == 3 ? -0.1138989f
         : i == 4 ? +0.1138989f : i == 5 ? +0.3513239f : i == 6 ? +0.6245203f : +1.0000000f;
}
__host__ __device__ constexpr float tq4_level(int i) {
    return i == 0 ? -1.0000000f : i == 1 ? -0.7573038f : i == 2 ? -0.5923403f : i == 3 ? -0.4599576f
         : i == 4 ? -0.3450764f : i == 5 ? -0.2405254f : i == 6 ? -0.1421261f : i == 7 ? -0.0470277f
         : i == 8 ? +0.0470277f : i == 9 ? +0.1421261f : i == 10 ? +0.2405254f : i == 11 ? +0.3450764f
         : i == 12 ? +0.4599576f : i == 13 ? +0.5923403f : i == 14 ? +0.7573038f : +1.0000000f;
}
__host__ __device__ constexpr float tq2_level(int i) {   // src/ggml-tq.h:89-91
    return i == 0 ? -1.0000000f : i == 1 ? -0.2997714f : i == 2 ? +0.2997714f : +1.0000000f;
}
template <int QT> __host__ __device__ constexpr float tq_level(int i) {
    return QT == 4 ? tq4_level(i) : QT == 3 ? tq3_level(i) : tq2_level(i);
}
// positive boundaries: TQ2 B[2], TQ3 B[4..6], TQ4 B[8..14]
constexpr float TQ2_P0 = 0.6498857f;
constexpr float TQ3_P0 = 0.2326114f, TQ3_P1 = 0.4879221f, TQ3_P2 = 0.8122602f;
constexpr float TQ4_P0 = 0.0945769f, TQ4_P1 = 0.1913257f, TQ4_P2 = 0.2928009f, TQ4_P3 = 0.4025170f,
                TQ4_P4 = 0.5261490f, TQ4_P5 = 0.6748221f, TQ4_P6 = 0.8786519f;

// The same levels parsed as float64 decimals, as scripts/tq3_rounding.py:18-21 does.
__host__ __device__ constexpr double tq3_level_f64(int i) {
    return i == 0 ? -1.0000000 : i == 1 ? -0.6245203 : i == 2 ? -0.3513239 : i == 3 ? -0.1138989
         : i == 4 ? +0.1138989 : i == 5 ? +0.3513239 : i == 6 ? +0.6245203 : +1.0000000;
}

// ── fp16 codec of the standalone reference build ──────────────────────────

__device__ __forceinline__ uint16_t half_trunc(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const int e = (int)((u >> 23) & 0xFFu) - 112;
    if (e <= 0) return (uint16_t)sign;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | ((u >> 13) & 0x3FFu));
}

__device__ __forceinline__ float half_decode(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 31u;
    const uint32_t m = h & 0x3FFu;
    if (e == 0) {
        const float f = __uint2float_rn(m) * 0x1p-24f;   // exact: m < 2^10
        return __uint_as_float(__float_as_uint(f) | sign);
    }
    return __uint_as_float(sign | ((e + 112u) << 23) | (m << 13));
}

// ── nearest level ─────────────────────────────────────────────────────────
// Both reference searches (src/ggml-tq.c:112-154) return #{b : B[b] < xn} for
// ordered xn (clamping to [-1, 1] never changes that count) and differ only on
// NaN: the TQ3 linear scan gives 0, the TQ4 tree gives 15.
//
// With a = |xn| and the positive boundaries P[m]:
//   xn > 0 : idx = n/2 + #{m : P[m] <  a}
//   xn < 0 : idx = n/2 - 1 - #{m : P[m] <= a}
//   xn = 0 : idx = n/2 - 1
// "<= a" is evaluated as "< nextup(a)" so that both cases share one search.

__device__ __forceinline__ float nextup_pos(float a) {  // a >= 0, finite or +inf
    return __uint_as_float(__float_as_uint(a) + 1u);
}

__device__ __forceinline__ int tq4_nearest(float xn) {
    const bool neg = xn < 0.0f;
    float a = fminf(fabsf(xn), 1.0f);          // NaN -> 1 here; fixed up below
    a = neg ? nextup_pos(a) : a;
    const bool q1 = a > TQ4_P3;
    const bool q2 = a > (q1 ? TQ4_P5 : TQ4_P1);
    const bool q3 = a > (q1 ? (q2 ? TQ4_P6 : TQ4_P4) : (q2 ? TQ4_P2 : TQ4_P0));
    const int c = (q1 ? 4 : 0) + (q2 ? 2 : 0) + (q3 ? 1 : 0);
    int idx = xn > 0.0f ? 8 + c : 7 - (neg ? c : 0);
    return (xn != xn) ? 15 : idx;
}

__device__ __forceinline__ int tq3_nearest(float xn) {
    const bool neg = xn < 0.0f;
    float a = fminf(fabsf(xn), 1.0f);
    a = neg ? nextup_pos(a) : a;
    const bool q1 = a > TQ3_P1;
    const bool q2 = a > (q1 ? TQ3_P2 : TQ3_P0);
    const int c = (q1 ? 2 : 0) + (q2 ? 1 : 0);
    int idx = xn > 0.0f ? 4 + c : 3 - (neg ? c : 0);
    return (xn != xn) ? 0 : idx;
}

__device__ __forceinline__ int tq2_nearest(float xn) {   // linear scan of src/ggml-tq.c:100-106; NaN -> 0
    const bool neg = xn < 0.0f;
    float a = fminf(fabsf(xn), 1.0f);
    a = neg ? nextup_pos(a) : a;
    const int q = a > TQ2_P0 ? 1 : 0;
    int idx = xn > 0.0f ? 2 + q : 1 - (neg ? q : 0);
    return (xn != xn) ? 0 : idx;
}

// ── LCG of randomized_hadamard_transform (src/ggml-tq.c:383-396) ──────────
// s <- s * 1664525 + 1013904223 (mod 2^32); element i of a chunk is negated when bit 31
// of the state after i + 1 steps is set.  lcg_jump(n) gives (A, C) with
// LCG^n(s) = A s + C, composed by squaring: LCG^(m+n) = (A_m A_n, A_m C_n + C_m).
constexpr uint32_t LCG_A = 1664525u, LCG_C = 1013904223u;
__host__ __device__ inline void lcg_jump(uint32_t n, uint32_t& A, uint32_t& C) {
    uint32_t ra = 1u, rc = 0u, pa = LCG_A, pc = LCG_C;   // result, and the power 2^b step
    while (n) {
        if (n & 1u) { rc = pa * rc + pc; ra = pa * ra; }
        pc = pa * pc + pc;
        pa = pa * pa;
        n >>= 1;
    }
    A = ra;
    C = rc;
}
// negate v[i] for the 32 elements starting at chunk position j0 of a chunk seeded s0
__device__ __forceinline__ void lcg_signs32(float (&v)[32], uint32_t s0, uint32_t j0) {
    uint32_t A, C;
    lcg_jump(j0, A, C);
    uint32_t s = A * s0 + C;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        s = s * LCG_A + LCG_C;
        v[i] = __uint_as_float(__float_as_uint(v[i]) ^ (s & 0x80000000u));
    }
}

// ── input element conversion ─────────────────────────────────────────────

enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

template <typename T> struct ElemBits;
template <> struct ElemBits<float> { static constexpr int bytes = 4; };
template <> struct ElemBits<__half> { static constexpr int bytes = 2; };
template <> struct ElemBits<__nv_bfloat16> { static constexpr int bytes = 2; };

// 16-bit -> float, exact
__device__ __forceinline__ float bf16_bits_to_float(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ float f16_bits_to_float(uint32_t b) {
    return __half2float(__ushort_as_half((unsigned short)b));
}

}  // namespace tq
