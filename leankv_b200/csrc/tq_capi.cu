// tq_capi.cu — extern "C" entry points of libleankv_tq.so (include/leankv_tq.h).
//
// Argument checking turns every contract violation into a tq_status (device
// and host APIs) or, for the ggml drop-in names, into the abort the
// reference's assert() would produce.  Nothing here computes on the CPU: a
// missing device is an error, never a fallback.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "leankv_tq.h"
#include "tq_capi_internal.h"
#include "tq_common.cuh"
#include "tq_kernels.h"

namespace tq {

static thread_local char g_err[512] = "";

tq_status set_error(tq_status s, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return s;
}

tq_status cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return TQ_SUCCESS;
    cudaGetLastError();   // clear a sticky launch-configuration error
    const tq_status s = (e == cudaErrorMemoryAllocation) ? TQ_ERROR_OUT_OF_MEMORY
                      : (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) ? TQ_ERROR_NO_DEVICE
                      : TQ_ERROR_CUDA;
    return set_error(s, "%s: %s", what, cudaGetErrorString(e));
}

int log2_pow2(int64_t v) {
    if (v <= 0 || (v & (v - 1)) != 0) return -1;
    int l = 0;
    while ((int64_t(1) << l) < v) ++l;
    return l;
}

// 1/sqrt(d) with the reference's float expression (src/ggml-tq.c:377)
float fwht_norm(int d) { return 1.0f / sqrtf((float)d); }

size_t block_bytes(int type) { return type == TQ_TYPE_TQ4_0 ? TQ4_BYTES : type == TQ_TYPE_TQ3_0 ? TQ3_BYTES : TQ2_BYTES; }
size_t dtype_bytes(int dt) { return dt == TQ_DTYPE_F32 ? 4 : 2; }
bool dtype_ok(int dt) { return dt == TQ_DTYPE_F32 || dt == TQ_DTYPE_F16 || dt == TQ_DTYPE_BF16; }
bool type_ok(int t) { return t == TQ_TYPE_TQ2_0 || t == TQ_TYPE_TQ3_0 || t == TQ_TYPE_TQ4_0; }

// ── host-API contexts: two streams + two grow-only device staging buffers ───
// Host calls move their data in chunks that alternate between the two streams:
// chunk c copies in, computes and copies out on stream c % 2, so the copies of one
// chunk overlap the kernel and the copies of the other, and the host-to-device
// and device-to-host copy engines run at the same time.
struct HostCtx {
    int dev = -1;
    cudaStream_t st[2] = {nullptr, nullptr};
    void* buf[2] = {nullptr, nullptr};
    size_t cap = 0;   // bytes of each staging buffer
};

static std::mutex g_pool_mu;
static std::vector<HostCtx*> g_pool;

static tq_status ctx_acquire(HostCtx** out) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return set_error(TQ_ERROR_NO_DEVICE, "no CUDA device available");
    }
    int dev = 0;
    tq_status s = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (s) return s;
    {
        std::lock_guard<std::mutex> lk(g_pool_mu);
        for (size_t i = 0; i < g_pool.size(); ++i) {
            if (g_pool[i]->dev == dev) {
                *out = g_pool[i];
                g_pool.erase(g_pool.begin() + i);
                return TQ_SUCCESS;
            }
        }
    }
    HostCtx* c = new HostCtx;
    c->dev = dev;
    for (int i = 0; i < 2; ++i) {
        s = cuda_status(cudaStreamCreateWithFlags(&c->st[i], cudaStreamNonBlocking), "cudaStreamCreate");
        if (s) {
            if (i) cudaStreamDestroy(c->st[0]);
            delete c;
            return s;
        }
    }
    *out = c;
    return TQ_SUCCESS;
}

static void ctx_release(HostCtx* c) {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    g_pool.push_back(c);
}

static tq_status ctx_reserve(HostCtx* c, size_t bytes) {
    if (bytes <= c->cap) return TQ_SUCCESS;
    for (int i = 0; i < 2; ++i) {
        cudaStreamSynchronize(c->st[i]);
        if (c->buf[i]) cudaFree(c->buf[i]);
        c->buf[i] = nullptr;
    }
    c->cap = 0;
    const size_t cap = (bytes + ((1u << 20) - 1)) & ~size_t((1u << 20) - 1);
    for (int i = 0; i < 2; ++i) {
        tq_status s = cuda_status(cudaMalloc(&c->buf[i], cap), "cudaMalloc (host API staging)");
        if (s) return s;
    }
    c->cap = cap;
    return TQ_SUCCESS;
}

// RAII holder for a host context
struct CtxGuard {
    HostCtx* c = nullptr;
    ~CtxGuard() { if (c) ctx_release(c); }
};

// Pipelined host operation over `total` units (elements or blocks).  A chunk of n
// units reads n * in_per bytes from hin + u0 * in_per and writes n * out_per bytes to
// hout + u0 * out_per; op(dev_in, dev_out, u0, n, stream) computes it on the device
// (dev_out may equal dev_in for in-place operations).  Chunks hold about an eighth of
// the work, between 1 MiB and 64 MiB of traffic, in multiples of `align` units.
template <typename Op>
static tq_status host_pipeline(HostCtx* c, int64_t total, int64_t align, size_t in_per, size_t out_per,
                               const void* hin, void* hout, bool in_place, Op op) {
    const size_t per = in_per + out_per;
    int64_t ch = (total + 7) / 8;
    const int64_t lo = (int64_t)((size_t(1) << 20) / per), hi = (int64_t)((size_t(64) << 20) / per);
    if (ch < lo) ch = lo;
    if (ch > hi) ch = hi;
    ch = (ch + align - 1) / align * align;
    if (ch > total) ch = total;
    const size_t in_bytes = (size_t)ch * in_per, out_off = in_place ? 0 : (in_bytes + 255) & ~size_t(255);
    tq_status s = ctx_reserve(c, out_off + (in_place ? in_bytes : (size_t)ch * out_per));
    if (s) return s;
    int k = 0;
    for (int64_t u0 = 0; u0 < total && !s; u0 += ch, ++k) {
        const int64_t n = total - u0 < ch ? total - u0 : ch;
        cudaStream_t st = c->st[k & 1];
        uint8_t* d = (uint8_t*)c->buf[k & 1];
        s = cuda_status(cudaMemcpyAsync(d, (const uint8_t*)hin + u0 * in_per, n * in_per, cudaMemcpyHostToDevice, st),
                        "cudaMemcpyAsync H2D");
        if (!s) s = op(d, d + out_off, u0, n, st);
        if (!s)
            s = cuda_status(cudaMemcpyAsync((uint8_t*)hout + u0 * out_per, d + out_off, n * out_per,
                                            cudaMemcpyDeviceToHost, st),
                            "cudaMemcpyAsync D2H");
    }
    const tq_status s0 = cuda_status(cudaStreamSynchronize(c->st[0]), "cudaStreamSynchronize");
    const tq_status s1 = cuda_status(cudaStreamSynchronize(c->st[1]), "cudaStreamSynchronize");
    return s ? s : (s0 ? s0 : s1);
}

}  // namespace tq

using namespace tq;

// ── status helpers ───────────────────────────────────────────────────────────

extern "C" const char* tq_status_string(tq_status s) {
    switch (s) {
        case TQ_SUCCESS: return "success";
        case TQ_ERROR_INVALID_VALUE: return "invalid value";
        case TQ_ERROR_UNSUPPORTED: return "unsupported";
        case TQ_ERROR_MISALIGNED: return "misaligned pointer";
        case TQ_ERROR_CUDA: return "CUDA error";
        case TQ_ERROR_OUT_OF_MEMORY: return "out of device memory";
        case TQ_ERROR_NO_DEVICE: return "no CUDA device";
        case TQ_ERROR_TIMEOUT: return "device-side wait timed out";
    }
    return "unknown status";
}

extern "C" const char* tq_last_error_string(void) { return g_err; }

namespace tq {
void clear_error() { g_err[0] = 0; }
}  // namespace tq
extern "C" int tq_abi_version(void) { return LEANKV_TQ_ABI_VERSION; }

// ── device-pointer API ────────────────────────────────────────────────────────

extern "C" tq_status tq_quantize_cuda(tq_type type, const void* x, tq_dtype x_dtype, void* y, int64_t k,
                                      int fwht_head_dim, int opt_passes, void* stream) {
    g_err[0] = 0;
    if (!type_ok(type)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown block type %d", (int)type);
    if (!dtype_ok(x_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown input dtype %d", (int)x_dtype);
    if (k < 0 || k % QK != 0) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 32", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!x || !y) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (((uintptr_t)x) % dtype_bytes(x_dtype)) return set_error(TQ_ERROR_MISALIGNED, "x not aligned to its element size");
    if (opt_passes < 0 || opt_passes > 64) return set_error(TQ_ERROR_INVALID_VALUE, "opt_passes=%d out of [0, 64]", opt_passes);
    if (opt_passes > 0 && type != TQ_TYPE_TQ3_0) return set_error(TQ_ERROR_UNSUPPORTED, "optimal rounding is defined for TQ3_0 only");
    int log2_hd = -1;
    float norm = 1.0f;
    if (fwht_head_dim != 0) {
        log2_hd = log2_pow2(fwht_head_dim);
        if (log2_hd < 0) return set_error(TQ_ERROR_INVALID_VALUE, "fwht_head_dim=%d is not a power of two", fwht_head_dim);
        if (log2_hd > 10) return set_error(TQ_ERROR_UNSUPPORTED, "fused FWHT supports head_dim <= 1024 (got %d)", fwht_head_dim);
        if (k % fwht_head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "k is not a multiple of fwht_head_dim");
        norm = fwht_norm(fwht_head_dim);
    }
    return cuda_status(launch_quantize((int)type, (int)x_dtype, x, y, k / QK, log2_hd, norm, opt_passes,
                                       (cudaStream_t)stream),
                       "quantize kernel launch");
}

tq_status tq::pages_check(const tq_kv_pages* pg, int batch, int* shift) {
    if (!pg) return set_error(TQ_ERROR_INVALID_VALUE, "null page description");
    const int l2 = log2_pow2(pg->page_size);
    if (l2 < 4 || l2 > 16) return set_error(TQ_ERROR_INVALID_VALUE, "page_size=%d (a power of two, 16 .. 65536)", pg->page_size);
    if (pg->max_pages_per_seq <= 0 || pg->max_pages_per_seq > (int64_t(1) << 40))
        return set_error(TQ_ERROR_INVALID_VALUE, "max_pages_per_seq=%lld", (long long)pg->max_pages_per_seq);
    if (pg->num_pages <= 0 || pg->num_pages > INT32_MAX)
        return set_error(TQ_ERROR_INVALID_VALUE, "num_pages=%lld (1 .. 2^31 - 1)", (long long)pg->num_pages);
    if (batch > 0 && !pg->page_table) return set_error(TQ_ERROR_INVALID_VALUE, "null page table");
    if (((uintptr_t)pg->page_table) & 3) return set_error(TQ_ERROR_MISALIGNED, "page table not 4-byte aligned");
    *shift = l2;
    return TQ_SUCCESS;
}

static tq_status kv_append(tq_type type, const void* src, tq_dtype src_dtype, void* cache, int batch, int n_kv_heads,
                           int head_dim, int64_t capacity, const tq_kv_pages* pages, int page_shift, int64_t n_new,
                           const int32_t* pos, int rotate, int opt_passes, int32_t* overflow, void* stream);

extern "C" tq_status tq_kv_append_cuda(tq_type type, const void* src, tq_dtype src_dtype, void* cache, int batch,
                                       int n_kv_heads, int head_dim, int64_t capacity, int64_t n_new,
                                       const int32_t* pos, int rotate, int opt_passes, int32_t* overflow,
                                       void* stream) {
    g_err[0] = 0;
    return kv_append(type, src, src_dtype, cache, batch, n_kv_heads, head_dim, capacity, nullptr, 0, n_new, pos, rotate,
                     opt_passes, overflow, stream);
}

extern "C" tq_status tq_kv_append_paged_cuda(tq_type type, const void* src, tq_dtype src_dtype, void* pool, int batch,
                                             int n_kv_heads, int head_dim, const tq_kv_pages* pages, int64_t n_new,
                                             const int32_t* pos, int rotate, int opt_passes, int32_t* overflow,
                                             void* stream) {
    g_err[0] = 0;
    int shift = 0;
    const tq_status s = pages_check(pages, batch, &shift);
    if (s) return s;
    return kv_append(type, src, src_dtype, pool, batch, n_kv_heads, head_dim, pages->max_pages_per_seq << shift, pages,
                     shift, n_new, pos, rotate, opt_passes, overflow, stream);
}

static tq_status kv_append(tq_type type, const void* src, tq_dtype src_dtype, void* cache, int batch, int n_kv_heads,
                           int head_dim, int64_t capacity, const tq_kv_pages* pages, int page_shift, int64_t n_new,
                           const int32_t* pos, int rotate, int opt_passes, int32_t* overflow, void* stream) {
    if (!type_ok(type)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown block type %d", (int)type);
    if (!dtype_ok(src_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown input dtype %d", (int)src_dtype);
    if (batch < 0 || n_kv_heads <= 0 || capacity < 0 || n_new < 0)
        return set_error(TQ_ERROR_INVALID_VALUE, "bad batch / head / capacity / row counts");
    const int l2 = log2_pow2(head_dim);
    if (l2 < 5 || l2 > 10) return set_error(TQ_ERROR_UNSUPPORTED, "head_dim=%d (supported: powers of two 32..1024)", head_dim);
    if (opt_passes < 0 || opt_passes > 64) return set_error(TQ_ERROR_INVALID_VALUE, "opt_passes=%d out of [0, 64]", opt_passes);
    if (opt_passes > 0 && type != TQ_TYPE_TQ3_0) return set_error(TQ_ERROR_UNSUPPORTED, "optimal rounding is defined for TQ3_0 only");
    const int64_t rows = (int64_t)batch * n_kv_heads * n_new;
    if (rows == 0 || capacity == 0) return TQ_SUCCESS;
    if (!src || !cache) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (((uintptr_t)src) % dtype_bytes(src_dtype)) return set_error(TQ_ERROR_MISALIGNED, "src not aligned to its element size");
    if (((uintptr_t)cache) & 15) return set_error(TQ_ERROR_MISALIGNED, "cache must be 16-byte aligned");
    RowMap map;
    map.cap = capacity;
    map.n_new = n_new;
    map.hkv = n_kv_heads;
    map.nblk = head_dim / QK;
    map.pos = pos;
    map.overflow = overflow;
    if (pages) {
        map.pages = pages->page_table;
        map.max_pages = pages->max_pages_per_seq;
        map.num_pages = pages->num_pages;
        map.page_shift = page_shift;
    }
    return cuda_status(launch_quantize((int)type, (int)src_dtype, src, cache, rows * (head_dim / QK),
                                       rotate ? l2 : -1, rotate ? fwht_norm(head_dim) : 1.0f, opt_passes,
                                       (cudaStream_t)stream, map),
                       "kv append kernel launch");
}

extern "C" tq_status tq_dequantize_cuda(tq_type type, const void* x, void* y, tq_dtype y_dtype, int64_t k,
                                        void* stream) {
    g_err[0] = 0;
    if (!type_ok(type)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown block type %d", (int)type);
    if (!dtype_ok(y_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown output dtype %d", (int)y_dtype);
    if (k < 0 || k % QK != 0) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 32", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!x || !y) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (((uintptr_t)y) % dtype_bytes(y_dtype)) return set_error(TQ_ERROR_MISALIGNED, "y not aligned to its element size");
    if (((uintptr_t)x) & 1) return set_error(TQ_ERROR_MISALIGNED, "blocks must be 2-byte aligned (fp16 scale)");
    return cuda_status(launch_dequantize((int)type, (int)y_dtype, x, y, k / QK, (cudaStream_t)stream),
                       "dequantize kernel launch");
}

extern "C" tq_status tq_hadamard_cuda(float* x, int64_t n, int head_dim, void* stream) {
    g_err[0] = 0;
    const int l2 = log2_pow2(head_dim);
    if (l2 < 0) return set_error(TQ_ERROR_INVALID_VALUE, "head_dim=%d is not a power of two", head_dim);
    if (l2 > 15) return set_error(TQ_ERROR_UNSUPPORTED, "head_dim=%d exceeds 32768", head_dim);
    if (n < 0 || n % head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "n is not a multiple of head_dim");
    if (n == 0) return TQ_SUCCESS;
    if (!x) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (((uintptr_t)x) & 3) return set_error(TQ_ERROR_MISALIGNED, "x not 4-byte aligned");
    const float norm = fwht_norm(head_dim);
    cudaStream_t st = (cudaStream_t)stream;
    if (l2 > 10) return cuda_status(launch_fwht_large(x, n / head_dim, l2, norm, st), "fwht kernel launch");
    const int64_t bulk = n - n % QK;
    tq_status s = cuda_status(launch_fwht(x, bulk / QK, l2, norm, st), "fwht kernel launch");
    if (s) return s;
    return cuda_status(launch_fwht_tail(x + bulk, (int)(n - bulk), l2, norm, st), "fwht tail launch");
}

extern "C" tq_status tq_hadamard_randomized_cuda(float* x, int64_t n, int row_len, int head_dim, uint32_t seed,
                                                 void* stream) {
    clear_error();
    const int l2 = log2_pow2(head_dim);
    if (l2 < 0) return set_error(TQ_ERROR_INVALID_VALUE, "head_dim=%d is not a power of two", head_dim);
    if (l2 < 5 || l2 > 10) return set_error(TQ_ERROR_UNSUPPORTED, "randomized Hadamard needs head_dim in 32..1024 (got %d)", head_dim);
    if (row_len <= 0 || row_len % head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "row_len is not a multiple of head_dim");
    if (n < 0 || n % row_len) return set_error(TQ_ERROR_INVALID_VALUE, "n is not a multiple of row_len");
    if (n == 0) return TQ_SUCCESS;
    if (!x) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    return cuda_status(launch_fwht(x, n / QK, l2, fwht_norm(head_dim), (cudaStream_t)stream, seed, row_len / head_dim),
                       "randomized fwht kernel launch");
}

extern "C" tq_status tq_quantize_randomized_cuda(tq_type type, const void* x, tq_dtype x_dtype, void* y, int64_t k,
                                                 int row_len, int head_dim, uint32_t seed, int opt_passes,
                                                 void* stream) {
    clear_error();
    if (!type_ok(type)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown block type %d", (int)type);
    if (!dtype_ok(x_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown input dtype %d", (int)x_dtype);
    const int l2 = log2_pow2(head_dim);
    if (l2 < 5 || l2 > 10) return set_error(TQ_ERROR_UNSUPPORTED, "randomized Hadamard needs head_dim in 32..1024 (got %d)", head_dim);
    if (row_len <= 0 || row_len % head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "row_len is not a multiple of head_dim");
    if (k < 0 || k % row_len) return set_error(TQ_ERROR_INVALID_VALUE, "k is not a multiple of row_len");
    if (opt_passes < 0 || opt_passes > 64) return set_error(TQ_ERROR_INVALID_VALUE, "opt_passes=%d out of [0, 64]", opt_passes);
    if (opt_passes > 0 && type != TQ_TYPE_TQ3_0) return set_error(TQ_ERROR_UNSUPPORTED, "optimal rounding is defined for TQ3_0 only");
    if (k == 0) return TQ_SUCCESS;
    if (!x || !y) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (((uintptr_t)x) % dtype_bytes(x_dtype)) return set_error(TQ_ERROR_MISALIGNED, "x not aligned to its element size");
    return cuda_status(launch_quantize((int)type, (int)x_dtype, x, y, k / QK, l2, fwht_norm(head_dim), opt_passes,
                                       (cudaStream_t)stream, RowMap(), seed, row_len / head_dim),
                       "quantize kernel launch");
}

extern "C" tq_status tq_requantize_cuda(tq_type src_type, const void* src, tq_type dst_type, void* dst, int64_t k,
                                        void* stream) {
    clear_error();
    if (!type_ok(src_type) || !type_ok(dst_type)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown block type");
    if (k < 0 || k % QK != 0) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 32", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!src || !dst) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if ((((uintptr_t)src) | ((uintptr_t)dst)) & 1) return set_error(TQ_ERROR_MISALIGNED, "blocks must be 2-byte aligned (fp16 scale)");
    return cuda_status(launch_requantize((int)src_type, src, (int)dst_type, dst, k / QK, (cudaStream_t)stream),
                       "requantize kernel launch");
}

// ── host-pointer API ──────────────────────────────────────────────────────────

extern "C" tq_status tq_quantize_host(tq_type type, const void* x, tq_dtype x_dtype, void* y, int64_t k,
                                      int fwht_head_dim, int opt_passes) {
    g_err[0] = 0;
    if (!type_ok(type) || !dtype_ok(x_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad type or dtype");
    if (k < 0 || k % QK) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 32", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!x || !y) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (fwht_head_dim > 0 && k % fwht_head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "k is not a multiple of fwht_head_dim");
    CtxGuard g;
    tq_status s = ctx_acquire(&g.c);
    if (s) return s;
    // units: blocks of 32 elements, chunks aligned to whole heads
    const int64_t align = fwht_head_dim > QK ? fwht_head_dim / QK : 1;
    return host_pipeline(g.c, k / QK, align, QK * dtype_bytes(x_dtype), block_bytes(type), x, y, false,
                         [&](uint8_t* din, uint8_t* dout, int64_t, int64_t n, cudaStream_t st) {
                             return tq_quantize_cuda(type, din, x_dtype, dout, n * QK, fwht_head_dim, opt_passes, st);
                         });
}

extern "C" tq_status tq_dequantize_host(tq_type type, const void* x, void* y, tq_dtype y_dtype, int64_t k) {
    g_err[0] = 0;
    if (!type_ok(type) || !dtype_ok(y_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad type or dtype");
    if (k < 0 || k % QK) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 32", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!x || !y) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    CtxGuard g;
    tq_status s = ctx_acquire(&g.c);
    if (s) return s;
    return host_pipeline(g.c, k / QK, 8, block_bytes(type), QK * dtype_bytes(y_dtype), x, y, false,
                         [&](uint8_t* din, uint8_t* dout, int64_t, int64_t n, cudaStream_t st) {
                             return tq_dequantize_cuda(type, din, dout, y_dtype, n * QK, st);
                         });
}

extern "C" tq_status tq_hadamard_host(float* x, int64_t n, int head_dim) {
    g_err[0] = 0;
    if (log2_pow2(head_dim) < 0) return set_error(TQ_ERROR_INVALID_VALUE, "head_dim=%d is not a power of two", head_dim);
    if (n < 0 || n % head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "n is not a multiple of head_dim");
    if (n == 0) return TQ_SUCCESS;
    if (!x) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    CtxGuard g;
    tq_status s = ctx_acquire(&g.c);
    if (s) return s;
    // units: floats, chunks aligned to whole heads (and to 32-element tiles)
    const int64_t align = head_dim > QK ? head_dim : QK;
    return host_pipeline(g.c, n, n % align ? n : align, 4, 4, x, x, true,
                         [&](uint8_t* din, uint8_t*, int64_t, int64_t m, cudaStream_t st) {
                             return tq_hadamard_cuda((float*)din, m, head_dim, st);
                         });
}

extern "C" tq_status tq_hadamard_randomized_host(float* x, int64_t n, int row_len, int head_dim, uint32_t seed) {
    clear_error();
    const int l2 = log2_pow2(head_dim);
    if (l2 < 5 || l2 > 10) return set_error(TQ_ERROR_UNSUPPORTED, "randomized Hadamard needs head_dim in 32..1024 (got %d)", head_dim);
    if (row_len <= 0 || row_len % head_dim) return set_error(TQ_ERROR_INVALID_VALUE, "row_len is not a multiple of head_dim");
    if (n < 0 || n % row_len) return set_error(TQ_ERROR_INVALID_VALUE, "n is not a multiple of row_len");
    if (n == 0) return TQ_SUCCESS;
    if (!x) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    CtxGuard g;
    tq_status s = ctx_acquire(&g.c);
    if (s) return s;
    return host_pipeline(g.c, n, row_len, 4, 4, x, x, true,
                         [&](uint8_t* din, uint8_t*, int64_t, int64_t m, cudaStream_t st) {
                             return tq_hadamard_randomized_cuda((float*)din, m, row_len, head_dim, seed, st);
                         });
}

extern "C" tq_status tq_requantize_host(tq_type src_type, const void* src, tq_type dst_type, void* dst, int64_t k) {
    clear_error();
    if (!type_ok(src_type) || !type_ok(dst_type)) return set_error(TQ_ERROR_INVALID_VALUE, "unknown block type");
    if (k < 0 || k % QK) return set_error(TQ_ERROR_INVALID_VALUE, "k=%lld is not a multiple of 32", (long long)k);
    if (k == 0) return TQ_SUCCESS;
    if (!src || !dst) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    CtxGuard g;
    tq_status s = ctx_acquire(&g.c);
    if (s) return s;
    return host_pipeline(g.c, k / QK, 8, block_bytes(src_type), block_bytes(dst_type), src, dst, false,
                         [&](uint8_t* din, uint8_t* dout, int64_t, int64_t n, cudaStream_t st) {
                             return tq_requantize_cuda(src_type, din, dst_type, dout, n * QK, st);
                         });
}

// ── ggml drop-in names (src/ggml-tq.h:145-190) ───────────────────────────────

[[noreturn]] static void die(const char* fn, const char* why) {
    fprintf(stderr, "leankv_tq: %s: %s\n", fn, why);
    fflush(stderr);
    abort();
}

static void check_k(const char* fn, int64_t k) {
    if (k % QK != 0) die(fn, "k % 32 != 0 (the reference asserts k % QK == 0)");
}

extern "C" void quantize_row_tq3_0_ref(const float* TQ_RESTRICT x, block_tq3_0* TQ_RESTRICT y, int64_t k) {
    check_k(__func__, k);
    if (tq_quantize_host(TQ_TYPE_TQ3_0, x, TQ_DTYPE_F32, y, k, 0, 0) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void quantize_row_tq4_0_ref(const float* TQ_RESTRICT x, block_tq4_0* TQ_RESTRICT y, int64_t k) {
    check_k(__func__, k);
    if (tq_quantize_host(TQ_TYPE_TQ4_0, x, TQ_DTYPE_F32, y, k, 0, 0) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void quantize_row_tq3_0(const float* TQ_RESTRICT x, void* TQ_RESTRICT y, int64_t k) {
    quantize_row_tq3_0_ref(x, (block_tq3_0*)y, k);
}

extern "C" void quantize_row_tq4_0(const float* TQ_RESTRICT x, void* TQ_RESTRICT y, int64_t k) {
    quantize_row_tq4_0_ref(x, (block_tq4_0*)y, k);
}

extern "C" void quantize_row_tq3_0_opt(const float* TQ_RESTRICT x, block_tq3_0* TQ_RESTRICT y, int64_t k) {
    check_k(__func__, k);
    if (tq_quantize_host(TQ_TYPE_TQ3_0, x, TQ_DTYPE_F32, y, k, 0, 2) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void dequantize_row_tq3_0(const block_tq3_0* TQ_RESTRICT x, float* TQ_RESTRICT y, int64_t k) {
    check_k(__func__, k);
    if (tq_dequantize_host(TQ_TYPE_TQ3_0, x, y, TQ_DTYPE_F32, k) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void dequantize_row_tq4_0(const block_tq4_0* TQ_RESTRICT x, float* TQ_RESTRICT y, int64_t k) {
    check_k(__func__, k);
    if (tq_dequantize_host(TQ_TYPE_TQ4_0, x, y, TQ_DTYPE_F32, k) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void hadamard_transform(float* x, int d) {
    if (d <= 0 || (d & (d - 1)) != 0) die(__func__, "d must be a power of two (the reference asserts this)");
    if (tq_hadamard_host(x, d, d) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void hadamard_transform_row(float* x, int n, int head_dim) {
    if (head_dim <= 0 || n % head_dim != 0) die(__func__, "n % head_dim != 0 (the reference asserts this)");
    if ((head_dim & (head_dim - 1)) != 0) die(__func__, "head_dim must be a power of two (the reference asserts this)");
    if (tq_hadamard_host(x, n, head_dim) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void quantize_row_tq2_0_ref(const float* TQ_RESTRICT x, block_tq2_0* TQ_RESTRICT y, int64_t k) {
    check_k(__func__, k);
    if (tq_quantize_host(TQ_TYPE_TQ2_0, x, TQ_DTYPE_F32, y, k, 0, 0) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void quantize_row_tq2_0(const float* TQ_RESTRICT x, void* TQ_RESTRICT y, int64_t k) {
    quantize_row_tq2_0_ref(x, (block_tq2_0*)y, k);
}

extern "C" void dequantize_row_tq2_0(const block_tq2_0* TQ_RESTRICT x, float* TQ_RESTRICT y, int64_t k) {
    check_k(__func__, k);
    if (tq_dequantize_host(TQ_TYPE_TQ2_0, x, y, TQ_DTYPE_F32, k) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void requantize_tq4_to_tq3(const block_tq4_0* TQ_RESTRICT src, block_tq3_0* TQ_RESTRICT dst, int64_t k) {
    check_k(__func__, k);
    if (tq_requantize_host(TQ_TYPE_TQ4_0, src, TQ_TYPE_TQ3_0, dst, k) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void requantize_tq3_to_tq2(const block_tq3_0* TQ_RESTRICT src, block_tq2_0* TQ_RESTRICT dst, int64_t k) {
    check_k(__func__, k);
    if (tq_requantize_host(TQ_TYPE_TQ3_0, src, TQ_TYPE_TQ2_0, dst, k) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void requantize_tq4_to_tq2(const block_tq4_0* TQ_RESTRICT src, block_tq2_0* TQ_RESTRICT dst, int64_t k) {
    check_k(__func__, k);
    if (tq_requantize_host(TQ_TYPE_TQ4_0, src, TQ_TYPE_TQ2_0, dst, k) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void randomized_hadamard_transform(float* x, int d, uint32_t seed) {
    if (d <= 0 || (d & (d - 1)) != 0) die(__func__, "d must be a power of two (the reference asserts this)");
    if (tq_hadamard_randomized_host(x, d, d, d, seed) != TQ_SUCCESS) die(__func__, g_err);
}

extern "C" void randomized_hadamard_transform_row(float* x, int n, int head_dim, uint32_t seed) {
    if (head_dim <= 0 || n % head_dim != 0) die(__func__, "n % head_dim != 0 (the reference asserts this)");
    if (n == 0) return;
    if (tq_hadamard_randomized_host(x, n, n, head_dim, seed) != TQ_SUCCESS) die(__func__, g_err);
}
