// tq_proto.cu — the prototype TurboQuant vector codec (prototype/turboquant) on sm_100a.
//
// The prototype quantizes whole head vectors rather than 32-element blocks
// (prototype/turboquant/quantizer.py:103-221, kv_cache.py:150-204):
//   xr = rotate(x)                      Hadamard or randomized Hadamard (x * signs, then the
//                                       normalized butterfly), or rotated outside (dense matrix)
//   scale = ||x||_2 (per vector)        or amax |xr| per group of `group` elements
//   xn = xr / (scale + 1e-10)
//   idx = #{b : B[b] < xn}              torch.bucketize with right=False (lloyd_max.py:208-220)
//   QJL (optional): r = xn - L[idx], sign bit (r >= 0) packed 8 per byte (bit i = element 8j+i),
//                   mean_abs = mean |r| over the vector (qjl_residual.py:44-110)
// and decodes  y = (L[idx] + (2 sign - 1) * mean_abs) * scale, optionally followed by the
// inverse rotation FWHT(y) * signs.
//
// One warp per vector; element e = 32 k + lane (k < d/32), so a warp ballot packs 32 sign
// bits of consecutive elements and the butterfly stages h < 32 run across lanes by shuffle,
// h >= 32 inside each lane.
#include <cstdint>

#include "leankv_tq.h"
#include "tq_capi_internal.h"
#include "tq_common.cuh"

namespace tq {

constexpr int PROTO_WARPS = 4;
constexpr int PROTO_MAX_LEVELS = 16;

struct ProtoCodebook {
    float levels[PROTO_MAX_LEVELS];
    float bounds[PROTO_MAX_LEVELS - 1];
    int n_levels;
};

template <typename T> __device__ __forceinline__ float ld_elem(const T* p);
template <> __device__ __forceinline__ float ld_elem<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld_elem<__half>(const __half* p) { return __half2float(*p); }
template <> __device__ __forceinline__ float ld_elem<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// normalized Walsh-Hadamard transform of the warp's vector (E = d / 32 elements per lane)
template <int E>
__device__ __forceinline__ void warp_fwht(float (&v)[E], int lane, float norm) {
#pragma unroll
    for (int h = 1; h < 32; h <<= 1) {
        const bool upper = (lane & h) != 0;
#pragma unroll
        for (int k = 0; k < E; ++k) {
            const float p = __shfl_xor_sync(0xffffffffu, v[k], h);
            v[k] = upper ? p - v[k] : v[k] + p;
        }
    }
#pragma unroll
    for (int hk = 1; hk < E; hk <<= 1) {
#pragma unroll
        for (int k = 0; k < E; ++k) {
            if (k & hk) continue;
            const float a = v[k], b = v[k + hk];
            v[k] = a + b;
            v[k + hk] = a - b;
        }
    }
#pragma unroll
    for (int k = 0; k < E; ++k) v[k] *= norm;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) x += __shfl_xor_sync(0xffffffffu, x, s);
    return x;
}

// group amax over aligned groups of g consecutive elements (g a power of two, 2 .. d)
template <int E>
__device__ __forceinline__ float group_amax(const float (&v)[E], int k, int g) {
    float m = fabsf(v[k]);
    const int lanes = g < 32 ? g : 32;
    for (int s = 1; s < lanes; s <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
    if (g > 32) {   // the group also spans g / 32 consecutive k
        const int kg = g / 32, k0 = k & ~(kg - 1);
        float mm = 0.0f;
#pragma unroll
        for (int j = 0; j < E; ++j) {
            float a = fabsf(v[j]);
            for (int s = 1; s < 32; s <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, s));
            if (j >= k0 && j < k0 + kg) mm = fmaxf(mm, a);
        }
        m = mm;
    }
    return m;
}

template <typename IN, int E>
__global__ void __launch_bounds__(PROTO_WARPS * 32)
proto_encode_kernel(const IN* __restrict__ x, const float* __restrict__ xr_ext, int64_t rows, int rotate,
                    const float* __restrict__ signs, float norm, int group, const ProtoCodebook cb,
                    uint8_t* __restrict__ idx_out, float* __restrict__ scale_out, uint8_t* __restrict__ qjl_signs,
                    float* __restrict__ qjl_mean) {
    constexpr int D = 32 * E;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * PROTO_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;   // warp-uniform
    float v[E];
#pragma unroll
    for (int k = 0; k < E; ++k) v[k] = ld_elem<IN>(x + row * D + 32 * k + lane);
    float vec_norm = 0.0f;
    if (group >= D) {   // L2 norm of the unrotated vector
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < E; ++k) ss = fmaf(v[k], v[k], ss);
        vec_norm = sqrtf(warp_sum(ss));
    }
    if (xr_ext) {
#pragma unroll
        for (int k = 0; k < E; ++k) v[k] = xr_ext[row * D + 32 * k + lane];
    } else if (rotate) {
        if (signs) {
#pragma unroll
            for (int k = 0; k < E; ++k) v[k] *= signs[32 * k + lane];
        }
        warp_fwht<E>(v, lane, norm);
    }
    float xn[E];
    uint32_t code[E];
#pragma unroll
    for (int k = 0; k < E; ++k) {
        float sc = vec_norm;
        if (group < D) {
            sc = group_amax<E>(v, k, group);
            const int e = 32 * k + lane;
            if ((e & (group - 1)) == 0) scale_out[row * (D / group) + e / group] = sc;
        }
        xn[k] = __fdiv_rn(v[k], __fadd_rn(sc, 1e-10f));
        uint32_t c = 0;
        for (int b = 0; b < cb.n_levels - 1; ++b) c += cb.bounds[b] < xn[k];
        code[k] = c;
        idx_out[row * D + 32 * k + lane] = (uint8_t)c;
    }
    if (group >= D && lane == 0) scale_out[row] = vec_norm;
    if (qjl_signs) {
        float asum = 0.0f;
#pragma unroll
        for (int k = 0; k < E; ++k) {
            const float r = __fsub_rn(xn[k], cb.levels[code[k]]);
            asum += fabsf(r);
            const uint32_t bits = __ballot_sync(0xffffffffu, r >= 0.0f);
            if (lane == 0) *reinterpret_cast<uint32_t*>(qjl_signs + row * (D / 8) + 4 * k) = bits;
        }
        asum = warp_sum(asum);
        if (lane == 0) qjl_mean[row] = asum / (float)D;
    }
}

template <int E>
__global__ void __launch_bounds__(PROTO_WARPS * 32)
proto_decode_kernel(const uint8_t* __restrict__ idx, const float* __restrict__ scale, int group,
                    const uint8_t* __restrict__ qjl_signs, const float* __restrict__ qjl_mean, const ProtoCodebook cb,
                    int64_t rows, int inv_rotate, const float* __restrict__ signs, float norm, float* __restrict__ y) {
    constexpr int D = 32 * E;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * PROTO_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;   // warp-uniform
    float v[E];
    const float ma = qjl_signs ? qjl_mean[row] : 0.0f;
#pragma unroll
    for (int k = 0; k < E; ++k) {
        const int e = 32 * k + lane;
        float r = cb.levels[idx[row * D + e]];
        if (qjl_signs) {
            const bool pos = (qjl_signs[row * (D / 8) + (e >> 3)] >> (e & 7)) & 1u;
            r = __fadd_rn(r, pos ? ma : -ma);
        }
        const float sc = group < D ? scale[row * (D / group) + e / group] : scale[row];
        v[k] = __fmul_rn(r, sc);
    }
    if (inv_rotate) {
        warp_fwht<E>(v, lane, norm);
        if (signs) {
#pragma unroll
            for (int k = 0; k < E; ++k) v[k] *= signs[32 * k + lane];
        }
    }
#pragma unroll
    for (int k = 0; k < E; ++k) y[row * D + 32 * k + lane] = v[k];
}

template <typename IN>
static cudaError_t launch_enc_t(int E, const void* x, const float* xr, int64_t rows, int rotate, const float* signs,
                                float norm, int group, const ProtoCodebook& cb, uint8_t* idx, float* scale,
                                uint8_t* qs, float* qm, cudaStream_t st) {
    const unsigned grid = (unsigned)((rows + PROTO_WARPS - 1) / PROTO_WARPS);
    switch (E) {
        case 1: proto_encode_kernel<IN, 1><<<grid, PROTO_WARPS * 32, 0, st>>>((const IN*)x, xr, rows, rotate, signs, norm, group, cb, idx, scale, qs, qm); break;
        case 2: proto_encode_kernel<IN, 2><<<grid, PROTO_WARPS * 32, 0, st>>>((const IN*)x, xr, rows, rotate, signs, norm, group, cb, idx, scale, qs, qm); break;
        case 4: proto_encode_kernel<IN, 4><<<grid, PROTO_WARPS * 32, 0, st>>>((const IN*)x, xr, rows, rotate, signs, norm, group, cb, idx, scale, qs, qm); break;
        default: proto_encode_kernel<IN, 8><<<grid, PROTO_WARPS * 32, 0, st>>>((const IN*)x, xr, rows, rotate, signs, norm, group, cb, idx, scale, qs, qm); break;
    }
    return cudaGetLastError();
}

}  // namespace tq

using namespace tq;

static tq_status proto_codebook(int n_levels, const float* levels, const float* bounds, ProtoCodebook* cb) {
    if (n_levels < 2 || n_levels > PROTO_MAX_LEVELS) return set_error(TQ_ERROR_UNSUPPORTED, "n_levels=%d (2..16)", n_levels);
    if (!levels || !bounds) return set_error(TQ_ERROR_INVALID_VALUE, "null codebook");
    cb->n_levels = n_levels;
    for (int i = 0; i < n_levels; ++i) cb->levels[i] = levels[i];
    for (int i = 0; i < n_levels - 1; ++i) cb->bounds[i] = bounds[i];
    return TQ_SUCCESS;
}

static int proto_e(int d) { return d == 32 ? 1 : d == 64 ? 2 : d == 128 ? 4 : d == 256 ? 8 : 0; }

extern "C" tq_status tq_proto_encode_cuda(const void* x, tq_dtype x_dtype, const float* x_rotated, int64_t rows,
                                          int dim, int rotate, const float* signs, int group, int n_levels,
                                          const float* levels, const float* boundaries, uint8_t* indices,
                                          float* scales, uint8_t* qjl_signs, float* qjl_mean_abs, void* stream) {
    clear_error();
    const int E = proto_e(dim);
    if (!E) return set_error(TQ_ERROR_UNSUPPORTED, "dim=%d (supported: 32, 64, 128, 256)", dim);
    if (!dtype_ok(x_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad dtype");
    if (group <= 0) group = dim;
    if (group > dim || (group & (group - 1)) || dim % group) return set_error(TQ_ERROR_INVALID_VALUE, "group=%d", group);
    if (rows < 0) return set_error(TQ_ERROR_INVALID_VALUE, "rows < 0");
    ProtoCodebook cb;
    tq_status s = proto_codebook(n_levels, levels, boundaries, &cb);
    if (s) return s;
    if (rows == 0) return TQ_SUCCESS;
    if (!x || !indices || !scales || (qjl_signs && !qjl_mean_abs)) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    const float norm = fwht_norm(dim);
    cudaError_t e;
    switch (x_dtype) {
        case TQ_DTYPE_F32: e = launch_enc_t<float>(E, x, x_rotated, rows, rotate, signs, norm, group, cb, indices, scales, qjl_signs, qjl_mean_abs, (cudaStream_t)stream); break;
        case TQ_DTYPE_F16: e = launch_enc_t<__half>(E, x, x_rotated, rows, rotate, signs, norm, group, cb, indices, scales, qjl_signs, qjl_mean_abs, (cudaStream_t)stream); break;
        default: e = launch_enc_t<__nv_bfloat16>(E, x, x_rotated, rows, rotate, signs, norm, group, cb, indices, scales, qjl_signs, qjl_mean_abs, (cudaStream_t)stream); break;
    }
    return cuda_status(e, "prototype encode launch");
}

extern "C" tq_status tq_proto_decode_cuda(const uint8_t* indices, const float* scales, int64_t rows, int dim, int group,
                                          const uint8_t* qjl_signs, const float* qjl_mean_abs, int n_levels,
                                          const float* levels, int inv_rotate, const float* signs, float* y,
                                          void* stream) {
    clear_error();
    const int E = proto_e(dim);
    if (!E) return set_error(TQ_ERROR_UNSUPPORTED, "dim=%d (supported: 32, 64, 128, 256)", dim);
    if (group <= 0) group = dim;
    if (group > dim || (group & (group - 1)) || dim % group) return set_error(TQ_ERROR_INVALID_VALUE, "group=%d", group);
    if (rows < 0) return set_error(TQ_ERROR_INVALID_VALUE, "rows < 0");
    if (n_levels < 2 || n_levels > PROTO_MAX_LEVELS || !levels) return set_error(TQ_ERROR_INVALID_VALUE, "bad codebook");
    ProtoCodebook cb = {};
    cb.n_levels = n_levels;
    for (int i = 0; i < n_levels; ++i) cb.levels[i] = levels[i];
    if (rows == 0) return TQ_SUCCESS;
    if (!indices || !scales || !y || (qjl_signs && !qjl_mean_abs)) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    const unsigned grid = (unsigned)((rows + PROTO_WARPS - 1) / PROTO_WARPS);
    const float norm = fwht_norm(dim);
    cudaStream_t st = (cudaStream_t)stream;
    switch (E) {
        case 1: proto_decode_kernel<1><<<grid, PROTO_WARPS * 32, 0, st>>>(indices, scales, group, qjl_signs, qjl_mean_abs, cb, rows, inv_rotate, signs, norm, y); break;
        case 2: proto_decode_kernel<2><<<grid, PROTO_WARPS * 32, 0, st>>>(indices, scales, group, qjl_signs, qjl_mean_abs, cb, rows, inv_rotate, signs, norm, y); break;
        case 4: proto_decode_kernel<4><<<grid, PROTO_WARPS * 32, 0, st>>>(indices, scales, group, qjl_signs, qjl_mean_abs, cb, rows, inv_rotate, signs, norm, y); break;
        default: proto_decode_kernel<8><<<grid, PROTO_WARPS * 32, 0, st>>>(indices, scales, group, qjl_signs, qjl_mean_abs, cb, rows, inv_rotate, signs, norm, y); break;
    }
    return cuda_status(cudaGetLastError(), "prototype decode launch");
}
