// tq_outlier.cu — extern "C" entry points of the channel-permuted mixed-precision
// quantization (src/ggml-tq-outlier.h / .c).  The kernels live in tq_codec.cu next
// to the block encoder they share; this file checks arguments, turns a
// tq_outlier_config into a kernel plan, and wraps host pointers.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "leankv_tq.h"
#include "tq_capi_internal.h"
#include "tq_common.cuh"
#include "tq_outlier.h"

using namespace tq;

static bool tier_ok(int t) { return t == TQ_TIER_TQ2 || t == TQ_TIER_TQ3 || t == TQ_TIER_TQ4; }
static int tier_type(int t) { return t + 2; }   // TQ_TIER_TQ2 .. TQ4 -> block type 2 .. 4
static size_t tier_bytes(int t) { return t == TQ_TIER_TQ4 ? TQ4_BYTES : t == TQ_TIER_TQ3 ? TQ3_BYTES : TQ2_BYTES; }
static float tier_bits(int t) { return t == TQ_TIER_TQ4 ? 4.5f : t == TQ_TIER_TQ3 ? 3.5f : 2.5f; }

static tq_status make_plan(const tq_outlier_config* c, MixedPlan* p, bool inverse = false) {
    if (!c) return set_error(TQ_ERROR_INVALID_VALUE, "null config");
    if (c->head_dim <= 0 || c->head_dim > TQ_OUTLIER_MAX_DIM || c->head_dim % QK)
        return set_error(TQ_ERROR_UNSUPPORTED, "head_dim=%d (multiples of 32 up to %d)", c->head_dim, TQ_OUTLIER_MAX_DIM);
    if (c->n_outlier < 0 || c->n_outlier % QK || c->n_outlier + c->n_normal != c->head_dim)
        return set_error(TQ_ERROR_INVALID_VALUE, "n_outlier=%d / n_normal=%d do not split head_dim into 32-element runs",
                         c->n_outlier, c->n_normal);
    if (!tier_ok(c->outlier_tier) || !tier_ok(c->normal_tier)) return set_error(TQ_ERROR_INVALID_VALUE, "bad tier");
    p->head_dim = c->head_dim;
    p->n_outlier = c->n_outlier;
    p->otype = tier_type(c->outlier_tier);
    p->ntype = tier_type(c->normal_tier);
    for (int i = 0; i < c->head_dim; ++i) {
        const int v = inverse ? c->inv_perm[i] : c->perm[i];
        if (v < 0 || v >= c->head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "permutation entry %d out of range", i);
        p->perm[i] = v;
    }
    return TQ_SUCCESS;
}

// ── device-pointer API ───────────────────────────────────────────────────────

extern "C" tq_status tq_outlier_identify_cuda(tq_outlier_config* config, const float* calib, int n_tokens, int head_dim,
                                              float outlier_frac, tq_tier_t outlier_tier, tq_tier_t normal_tier,
                                              void* stream) {
    clear_error();
    if (!config || !calib) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (head_dim <= 0 || head_dim > TQ_OUTLIER_MAX_DIM) return set_error(TQ_ERROR_INVALID_VALUE, "head_dim=%d", head_dim);
    if (n_tokens <= 0) return set_error(TQ_ERROR_INVALID_VALUE, "n_tokens <= 0");
    if (!(outlier_frac >= 0.0f && outlier_frac <= 1.0f)) return set_error(TQ_ERROR_INVALID_VALUE, "outlier_frac outside [0, 1]");
    if (!tier_ok(outlier_tier) || !tier_ok(normal_tier)) return set_error(TQ_ERROR_INVALID_VALUE, "bad tier");
    cudaStream_t st = (cudaStream_t)stream;
    float* d_var = nullptr;
    tq_status s = cuda_status(cudaMallocAsync((void**)&d_var, 3 * sizeof(int) * TQ_OUTLIER_MAX_DIM, st), "cudaMallocAsync");
    if (s) return s;
    int* d_perm = reinterpret_cast<int*>(d_var + TQ_OUTLIER_MAX_DIM);
    int* d_inv = d_perm + TQ_OUTLIER_MAX_DIM;
    s = cuda_status(launch_outlier_calib(calib, n_tokens, head_dim, d_var, d_perm, d_inv, st), "outlier calibration launch");
    if (!s) s = cuda_status(cudaMemcpyAsync(config->channel_var, d_var, sizeof(float) * head_dim, cudaMemcpyDeviceToHost, st), "D2H");
    if (!s) s = cuda_status(cudaMemcpyAsync(config->perm, d_perm, sizeof(int) * head_dim, cudaMemcpyDeviceToHost, st), "D2H");
    if (!s) s = cuda_status(cudaMemcpyAsync(config->inv_perm, d_inv, sizeof(int) * head_dim, cudaMemcpyDeviceToHost, st), "D2H");
    cudaFreeAsync(d_var, st);
    if (!s) s = cuda_status(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (s) return s;
    config->head_dim = head_dim;
    config->outlier_frac = outlier_frac;
    config->outlier_tier = outlier_tier;
    config->normal_tier = normal_tier;
    // the top fraction, rounded up to whole 32-element blocks (ggml-tq-outlier.c:146-160)
    const int n_raw = (int)(outlier_frac * (float)head_dim + 0.5f);
    int n_outlier = n_raw == 0 ? 0 : ((n_raw + 31) / 32) * 32;
    if (n_outlier > head_dim) n_outlier = head_dim;
    config->n_outlier = n_outlier;
    config->n_normal = head_dim - n_outlier;
    return TQ_SUCCESS;
}

extern "C" tq_status tq_mixed_quantize_cuda(const tq_outlier_config* config, const void* x, tq_dtype x_dtype,
                                            int64_t n_vec, void* outlier_buf, void* normal_buf, void* stream) {
    clear_error();
    MixedPlan p;
    tq_status s = make_plan(config, &p);
    if (s) return s;
    if (!dtype_ok(x_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad dtype");
    if (n_vec < 0) return set_error(TQ_ERROR_INVALID_VALUE, "n_vec < 0");
    if (n_vec == 0) return TQ_SUCCESS;
    if (!x || (p.n_outlier && !outlier_buf) || (p.n_outlier < p.head_dim && !normal_buf))
        return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if ((((uintptr_t)outlier_buf) | ((uintptr_t)normal_buf)) & 1) return set_error(TQ_ERROR_MISALIGNED, "block buffers must be 2-byte aligned");
    if (((uintptr_t)x) % dtype_bytes(x_dtype)) return set_error(TQ_ERROR_MISALIGNED, "x not aligned to its element size");
    return cuda_status(launch_mixed_quantize((int)x_dtype, x, n_vec, p, outlier_buf, normal_buf, (cudaStream_t)stream),
                       "mixed quantize launch");
}

extern "C" tq_status tq_mixed_dequantize_cuda(const tq_outlier_config* config, const void* outlier_buf,
                                              const void* normal_buf, int64_t n_vec, float* y, void* stream) {
    clear_error();
    MixedPlan p;
    tq_status s = make_plan(config, &p);
    if (s) return s;
    if (n_vec < 0) return set_error(TQ_ERROR_INVALID_VALUE, "n_vec < 0");
    if (n_vec == 0) return TQ_SUCCESS;
    if (!y || (p.n_outlier && !outlier_buf) || (p.n_outlier < p.head_dim && !normal_buf))
        return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    return cuda_status(launch_mixed_dequantize(outlier_buf, normal_buf, n_vec, p, y, (cudaStream_t)stream),
                       "mixed dequantize launch");
}

// ── TQ2_1 (the fork's static mixed-precision block) ─────────────────────────

extern "C" tq_status tq_quantize_tq2_1_cuda(const void* x, tq_dtype x_dtype, void* y, int64_t k, void* stream) {
    clear_error();
    if (!dtype_ok(x_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown input dtype %d", (int)x_dtype);
    if (k < 0 || k % 128) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 128", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!x || !y) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (((uintptr_t)x) % dtype_bytes(x_dtype)) return set_error(TQ_ERROR_MISALIGNED, "x not aligned to its element size");
    if (((uintptr_t)y) & 1) return set_error(TQ_ERROR_MISALIGNED, "blocks must be 2-byte aligned (fp16 scales)");
    return cuda_status(launch_tq21_quantize((int)x_dtype, x, k / 128, y, (cudaStream_t)stream), "TQ2_1 quantize launch");
}

extern "C" tq_status tq_dequantize_tq2_1_cuda(const void* x, float* y, int64_t k, void* stream) {
    clear_error();
    if (k < 0 || k % 128) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 128", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!x || !y) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if ((((uintptr_t)x) & 1) || (((uintptr_t)y) & 15))
        return set_error(TQ_ERROR_MISALIGNED, "blocks must be 2-byte and y 16-byte aligned");
    return cuda_status(launch_tq21_dequantize(x, k / 128, y, (cudaStream_t)stream), "TQ2_1 dequantize launch");
}

// ── drop-in names (src/ggml-tq-outlier.h), host pointers, one head vector per call ─

[[noreturn]] static void die(const char* fn, const char* why) {
    fprintf(stderr, "leankv_tq: %s: %s\n", fn, why);
    fflush(stderr);
    abort();
}

namespace {
// device scratch for the host-pointer wrappers: synchronous, one per call
struct Scratch {
    void* p = nullptr;
    ~Scratch() { if (p) cudaFree(p); }
};
}  // namespace

extern "C" void tq_identify_outliers(tq_outlier_config* config, const float* calib_data, int n_tokens, int head_dim,
                                     float outlier_frac, tq_tier_t outlier_tier, tq_tier_t normal_tier) {
    if (!(head_dim > 0 && head_dim <= TQ_OUTLIER_MAX_DIM) || n_tokens <= 0 || !(outlier_frac >= 0.0f && outlier_frac <= 1.0f))
        die(__func__, "head_dim / n_tokens / outlier_frac out of range (the reference asserts this)");
    Scratch d;
    const size_t bytes = sizeof(float) * (size_t)n_tokens * head_dim;
    if (cudaMalloc(&d.p, bytes) != cudaSuccess) die(__func__, "cudaMalloc failed");
    if (cudaMemcpy(d.p, calib_data, bytes, cudaMemcpyHostToDevice) != cudaSuccess) die(__func__, "cudaMemcpy failed");
    if (tq_outlier_identify_cuda(config, (const float*)d.p, n_tokens, head_dim, outlier_frac, outlier_tier, normal_tier,
                                 nullptr) != TQ_SUCCESS)
        die(__func__, tq_last_error_string());
}

extern "C" void tq_outlier_config_init_uniform(tq_outlier_config* config, int head_dim, tq_tier_t tier) {
    if (!(head_dim > 0 && head_dim <= TQ_OUTLIER_MAX_DIM)) die(__func__, "head_dim out of range (the reference asserts this)");
    config->head_dim = head_dim;
    config->n_outlier = 0;
    config->n_normal = head_dim;
    config->outlier_frac = 0.0f;
    config->outlier_tier = tier;
    config->normal_tier = tier;
    for (int i = 0; i < head_dim; ++i) {
        config->perm[i] = i;
        config->inv_perm[i] = i;
        config->channel_var[i] = 0.0f;
    }
}

extern "C" void tq_mixed_buffer_sizes(const tq_outlier_config* config, size_t* outlier_size, size_t* normal_size) {
    *outlier_size = (size_t)((config->n_outlier + QK - 1) / QK) * tier_bytes(config->outlier_tier);
    *normal_size = (size_t)((config->n_normal + QK - 1) / QK) * tier_bytes(config->normal_tier);
}

extern "C" float tq_mixed_effective_bpe(const tq_outlier_config* config) {
    if (config->head_dim == 0) return 0.0f;
    const float bits = (float)config->n_outlier * tier_bits(config->outlier_tier) +
                       (float)config->n_normal * tier_bits(config->normal_tier);
    return bits / (float)config->head_dim;
}

static void host_gather(const char* fn, const float* x, float* y, const int* map, int n) {
    if (n <= 0 || n > TQ_OUTLIER_MAX_DIM) die(fn, "n out of range");
    MixedPlan p;
    p.head_dim = n;
    for (int i = 0; i < n; ++i) {
        if (map[i] < 0 || map[i] >= n) die(fn, "permutation entry out of range");
        p.perm[i] = map[i];
    }
    Scratch d;
    if (cudaMalloc(&d.p, 2 * sizeof(float) * n) != cudaSuccess) die(fn, "cudaMalloc failed");
    float* dx = (float*)d.p;
    if (cudaMemcpy(dx, x, sizeof(float) * n, cudaMemcpyHostToDevice) != cudaSuccess) die(fn, "cudaMemcpy failed");
    if (launch_gather(dx, p, 1, dx + n, nullptr) != cudaSuccess) die(fn, "gather launch failed");
    if (cudaMemcpy(y, dx + n, sizeof(float) * n, cudaMemcpyDeviceToHost) != cudaSuccess) die(fn, "cudaMemcpy failed");
}

extern "C" void tq_permute_channels(const float* x, float* y, const int* perm, int n) {
    host_gather(__func__, x, y, perm, n);
}

extern "C" void tq_unpermute_channels(const float* x, float* y, const int* inv_perm, int n) {
    host_gather(__func__, x, y, inv_perm, n);
}

extern "C" void tq_mixed_quantize(const float* x, const tq_outlier_config* config, void* outlier_buf, void* normal_buf) {
    size_t ob = 0, nb = 0;
    tq_mixed_buffer_sizes(config, &ob, &nb);
    Scratch d;
    const size_t xin = sizeof(float) * (size_t)config->head_dim;
    if (cudaMalloc(&d.p, xin + ob + nb + 16) != cudaSuccess) die(__func__, "cudaMalloc failed");
    uint8_t* base = (uint8_t*)d.p;
    if (cudaMemcpy(base, x, xin, cudaMemcpyHostToDevice) != cudaSuccess) die(__func__, "cudaMemcpy failed");
    if (tq_mixed_quantize_cuda(config, base, TQ_DTYPE_F32, 1, base + xin, base + xin + ob, nullptr) != TQ_SUCCESS)
        die(__func__, tq_last_error_string());
    if ((ob && cudaMemcpy(outlier_buf, base + xin, ob, cudaMemcpyDeviceToHost) != cudaSuccess) ||
        (nb && cudaMemcpy(normal_buf, base + xin + ob, nb, cudaMemcpyDeviceToHost) != cudaSuccess))
        die(__func__, "cudaMemcpy failed");
}

extern "C" void tq_mixed_dequantize(const void* outlier_buf, const void* normal_buf, const tq_outlier_config* config,
                                    float* y) {
    size_t ob = 0, nb = 0;
    tq_mixed_buffer_sizes(config, &ob, &nb);
    Scratch d;
    const size_t yb = sizeof(float) * (size_t)config->head_dim;
    if (cudaMalloc(&d.p, yb + ob + nb + 16) != cudaSuccess) die(__func__, "cudaMalloc failed");
    uint8_t* base = (uint8_t*)d.p;
    if ((ob && cudaMemcpy(base + yb, outlier_buf, ob, cudaMemcpyHostToDevice) != cudaSuccess) ||
        (nb && cudaMemcpy(base + yb + ob, normal_buf, nb, cudaMemcpyHostToDevice) != cudaSuccess))
        die(__func__, "cudaMemcpy failed");
    if (tq_mixed_dequantize_cuda(config, base + yb, base + yb + ob, 1, (float*)base, nullptr) != TQ_SUCCESS)
        die(__func__, tq_last_error_string());
    if (cudaMemcpy(y, base, yb, cudaMemcpyDeviceToHost) != cudaSuccess) die(__func__, "cudaMemcpy failed");
}
