// tq_merge.cuh — log-sum-exp merge of one row of P partial attention results, by one warp.
//
// Part p holds a normalised output row o_p[D] and its natural-log lse_p (-inf: the part saw no
// token).  With M = max_p lse_p and w_p = exp(lse_p - M) over the parts with lse_p != -inf,
//     out = (sum_p w_p o_p) / (sum_p w_p),   lse = M + log(sum_p w_p)
// (an empty row gives out 0, lse -inf).  The sums run over p in increasing order, each
// accumulation a fused multiply-add for the output and an add for the weight sum, so every
// caller of this function produces the same bits: the NCCL all_gather + merge kernel and the
// peer-memory merge kernels of the split-sequence exchange must agree exactly.
//
// Lane p computes w_p once (parts >= 32 are handled in rounds of 32); the weights reach every
// lane by shuffles, and the row's elements are loaded lane-strided (coalesced), all parts'
// loads independent of one another.  Two dependent trips through L2 per row: the lse values,
// then the outputs.
#pragma once

#include <cmath>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace tq {

template <typename OT> __device__ __forceinline__ void merge_store(OT* p, float v);
template <> __device__ __forceinline__ void merge_store<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void merge_store<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <> __device__ __forceinline__ void merge_store<__nv_bfloat16>(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
}

// Row i: o of part p at o + p * o_stride + i * D, its lse at lse + p * lse_stride + i.  All 32
// lanes of the warp call it together.  Reads go through L2 (other GPUs may have written them).
template <typename OT>
__device__ __forceinline__ void merge_row(const float* __restrict__ o, int64_t o_stride, const float* __restrict__ lse,
                                          int64_t lse_stride, int P, int64_t i, int D, OT* __restrict__ out,
                                          float* __restrict__ lse_out, int lane) {
    // M over all parts
    float M = -INFINITY;
    for (int p0 = 0; p0 < P; p0 += 32) {
        const float l = p0 + lane < P ? __ldcg(lse + (int64_t)(p0 + lane) * lse_stride + i) : -INFINITY;
        M = fmaxf(M, l);
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    // W in part order; acc of each of this lane's elements in part order.  Rows go in chunks of
    // 128 elements (4 per lane; W is recomputed per chunk, the same value every time), parts in
    // groups of 8 whose loads are all issued before the ordered accumulation.
    constexpr int MAXE = 4, PG = 8;
    float W = 0.0f;
    for (int e0 = 0; e0 < D; e0 += 32 * MAXE) {
        float acc[MAXE];
#pragma unroll
        for (int k = 0; k < MAXE; ++k) acc[k] = 0.0f;
        W = 0.0f;
        for (int p0 = 0; p0 < P; p0 += 32) {
            const float l = p0 + lane < P ? __ldcg(lse + (int64_t)(p0 + lane) * lse_stride + i) : -INFINITY;
            const float w = l != -INFINITY ? __expf(l - M) : 0.0f;
            const int np = P - p0 < 32 ? P - p0 : 32;
            for (int g0 = 0; g0 < np; g0 += PG) {
                float v[PG][MAXE];
#pragma unroll
                for (int g = 0; g < PG; ++g) {
                    const float* op = o + (int64_t)(p0 + g0 + g) * o_stride + i * D + e0;
#pragma unroll
                    for (int k = 0; k < MAXE; ++k)
                        v[g][k] = (g0 + g < np && e0 + lane + 32 * k < D) ? __ldcg(op + lane + 32 * k) : 0.0f;
                }
#pragma unroll
                for (int g = 0; g < PG; ++g) {
                    if (g0 + g >= np) break;
                    const float wq = __shfl_sync(0xffffffffu, w, g0 + g);
                    const float lq = __shfl_sync(0xffffffffu, l, g0 + g);
                    if (lq == -INFINITY) continue;   // warp-uniform
                    W += wq;
#pragma unroll
                    for (int k = 0; k < MAXE; ++k) acc[k] = fmaf(wq, v[g][k], acc[k]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < MAXE; ++k)
            if (e0 + lane + 32 * k < D)
                merge_store<OT>(out + i * D + e0 + lane + 32 * k, M == -INFINITY ? 0.0f : acc[k] / W);
    }
    if (lse_out && lane == 0) lse_out[i] = M == -INFINITY ? -INFINITY : M + __logf(W);
}

}  // namespace tq
