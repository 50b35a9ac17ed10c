// tq_capi_attn.cu — extern "C" entry points of the decode attention.
#include <cmath>
#include <mutex>

#include "leankv_tq.h"
#include "tq_attn.h"
#include "tq_capi_internal.h"
#include "tq_common.cuh"

using namespace tq;

tq_status tq::attn_check(const tq_decode_attention_args* a, AttnRun* r, AttnPlan* p) {
    if (!a) return set_error(TQ_ERROR_INVALID_VALUE, "null argument block");
    if (a->batch < 0 || a->n_q_heads <= 0 || a->n_kv_heads <= 0)
        return set_error(TQ_ERROR_INVALID_VALUE, "bad batch / head counts");
    if (a->n_q_heads % a->n_kv_heads) return set_error(TQ_ERROR_INVALID_VALUE, "n_q_heads %% n_kv_heads != 0");
    const int grp = a->n_q_heads / a->n_kv_heads;
    if (grp > 8) return set_error(TQ_ERROR_UNSUPPORTED, "GQA group size %d (supported: 1 .. 8)", grp);
    if (a->head_dim != 128 && a->head_dim != 256)
        return set_error(TQ_ERROR_UNSUPPORTED, "head_dim %d (supported: 128, 256)", a->head_dim);
    if ((a->k_type != TQ_TYPE_TQ4_0 && a->k_type != TQ_TYPE_TQ3_0 && a->k_type != TQ_TYPE_TQ2_0) ||
        a->v_type != TQ_TYPE_TQ4_0)
        return set_error(TQ_ERROR_UNSUPPORTED, "block types K=%d V=%d (supported: K TQ4_0, TQ3_0 or TQ2_0, V TQ4_0)",
                         (int)a->k_type, (int)a->v_type);
    if (!dtype_ok(a->q_dtype) || !dtype_ok(a->out_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad dtype");
    if (a->kv_capacity < 0 || (a->kv_capacity & 1)) return set_error(TQ_ERROR_INVALID_VALUE, "kv_capacity must be even");
    if (a->max_kv_len < 0 || a->max_kv_len > a->kv_capacity)
        return set_error(TQ_ERROR_INVALID_VALUE, "max_kv_len outside [0, kv_capacity]");
    if (a->batch > 0 && (!a->q || !a->out || (a->kv_capacity > 0 && (!a->k_cache || !a->v_cache))))
        return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if ((((uintptr_t)a->k_cache) | ((uintptr_t)a->v_cache)) & 15)
        return set_error(TQ_ERROR_MISALIGNED, "cache pointers must be 16-byte aligned");
    if (((uintptr_t)a->q) % dtype_bytes(a->q_dtype) || ((uintptr_t)a->out) % dtype_bytes(a->out_dtype))
        return set_error(TQ_ERROR_MISALIGNED, "q / out not aligned to their element size");
    r->B = a->batch; r->Hq = a->n_q_heads; r->Hkv = a->n_kv_heads; r->grp = grp; r->D = a->head_dim;
    r->q = a->q; r->q_dtype = a->q_dtype; r->k = a->k_cache; r->v = a->v_cache;
    r->k_type = a->k_type; r->v_type = a->v_type; r->cap = a->kv_capacity; r->kv_len = a->kv_len;
    r->sm_scale = a->sm_scale != 0.0f ? a->sm_scale : 1.0f / sqrtf((float)a->head_dim);
    r->rotate_q = a->rotate_q != 0; r->v_rotated = a->v_rotated != 0;
    r->out = a->out; r->out_dtype = a->out_dtype; r->lse = a->lse;
    *p = attn_plan(a->batch, a->n_kv_heads, a->head_dim, a->kv_capacity, a->max_kv_len > 0 ? a->max_kv_len : a->kv_capacity);
    return TQ_SUCCESS;
}

extern "C" size_t tq_decode_attention_workspace_size(const tq_decode_attention_args* a) {
    AttnRun r;
    AttnPlan p;
    if (attn_check(a, &r, &p) != TQ_SUCCESS) return 0;
    return attn_workspace_bytes(r.B, r.Hkv, r.D, p);
}

extern "C" tq_status tq_decode_attention_cuda(const tq_decode_attention_args* a, void* stream) {
    AttnRun r;
    AttnPlan p;
    tq_status s = attn_check(a, &r, &p);
    if (s) return s;
    if (r.B == 0) return TQ_SUCCESS;
    const size_t need = attn_workspace_bytes(r.B, r.Hkv, r.D, p);
    if (!a->workspace || a->workspace_bytes < need)
        return set_error(TQ_ERROR_INVALID_VALUE, "workspace of %zu bytes needed", need);
    if (((uintptr_t)a->workspace) & 255) return set_error(TQ_ERROR_MISALIGNED, "workspace must be 256-byte aligned");
    return cuda_status(launch_decode_attention(r, p, a->workspace, (cudaStream_t)stream), "decode attention launch");
}

extern "C" tq_status tq_decode_attention_paged_cuda(const tq_decode_attention_args* a, const tq_kv_pages* pg,
                                                    void* stream) {
    AttnRun r;
    AttnPlan p;
    tq_status s = attn_check(a, &r, &p);
    if (s) return s;
    int shift = 0;
    if ((s = pages_check(pg, a->batch, &shift))) return s;
    if (a->kv_capacity != (pg->max_pages_per_seq << shift))
        return set_error(TQ_ERROR_INVALID_VALUE, "kv_capacity must equal max_pages_per_seq * page_size");
    // the kernel addresses tokens and page-table entries in 32 bits
    const int64_t page_bytes = ((int64_t)a->n_kv_heads << shift) * (a->head_dim / 32) * 18;   // the larger pool
    if (a->kv_capacity >= (int64_t(1) << 31) || (int64_t)a->batch * pg->max_pages_per_seq >= (int64_t(1) << 32) ||
        page_bytes >= (int64_t(1) << 32))
        return set_error(TQ_ERROR_UNSUPPORTED, "paged cache too large: capacity, page table and page bytes must fit 32 bits");
    if (r.B == 0) return TQ_SUCCESS;
    r.pages = pg->page_table;
    r.max_pages = pg->max_pages_per_seq;
    r.num_pages = pg->num_pages;
    r.page_shift = shift;
    const size_t need = attn_workspace_bytes(r.B, r.Hkv, r.D, p);
    if (!a->workspace || a->workspace_bytes < need)
        return set_error(TQ_ERROR_INVALID_VALUE, "workspace of %zu bytes needed", need);
    if (((uintptr_t)a->workspace) & 255) return set_error(TQ_ERROR_MISALIGNED, "workspace must be 256-byte aligned");
    return cuda_status(launch_decode_attention(r, p, a->workspace, (cudaStream_t)stream), "paged decode attention launch");
}

extern "C" tq_status tq_lse_merge_cuda(int n_parts, int64_t n_rows, int head_dim, const float* o,
                                       int64_t o_part_stride, const float* lse, int64_t lse_part_stride, void* out,
                                       tq_dtype out_dtype, float* lse_out, void* stream) {
    if (n_parts <= 0 || n_rows < 0 || head_dim <= 0) return set_error(TQ_ERROR_INVALID_VALUE, "bad sizes");
    if (!dtype_ok(out_dtype)) return set_error(TQ_ERROR_INVALID_VALUE, "bad output dtype");
    if (o_part_stride < 0 || lse_part_stride < 0) return set_error(TQ_ERROR_INVALID_VALUE, "negative part strides");
    if (n_rows == 0) return TQ_SUCCESS;
    if (!o || !lse || !out) return set_error(TQ_ERROR_INVALID_VALUE, "null pointer");
    if (((uintptr_t)out) % dtype_bytes(out_dtype)) return set_error(TQ_ERROR_MISALIGNED, "out not aligned to its element size");
    return cuda_status(launch_lse_combine(o, o_part_stride, lse, lse_part_stride, out, (int)out_dtype, lse_out, n_parts,
                                          n_rows, head_dim, (cudaStream_t)stream),
                       "lse merge launch");
}

extern "C" tq_status tq_lse_combine_cuda(int n_parts, int64_t n_rows, int head_dim, const float* o, const float* lse,
                                         float* out, float* lse_out, void* stream) {
    return tq_lse_merge_cuda(n_parts, n_rows, head_dim, o, n_rows * head_dim, lse, n_rows, out, TQ_DTYPE_F32, lse_out,
                             stream);
}

// ── fixed-scratch variant ────────────────────────────────────────────────────
//
// Some callers cannot allocate device memory at the point where they run
// decode attention: code that executes inside an allocator-free region (a
// serving loop that forbids cudaMalloc/cudaFree between steps, a plugin whose
// host framework owns every allocation, a pre-built execution plan).  This
// entry point runs the same kernels with their work memory in a static device
// array compiled into the library, so it allocates nothing.
//
// The array's host-side name is only a stand-in for the device object; its
// device address is looked up once per device with cudaGetSymbolAddress while
// that device is current.

static __device__ __align__(256) unsigned char g_attn_static_scratch[TQ_STATIC_SCRATCH_BYTES];

static std::mutex g_static_mu;
static void* g_static_ptr[64];
static bool g_static_ready[64];

static tq_status static_scratch(void** out) {
    int dev = 0;
    tq_status s = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (s) return s;
    if (dev < 0 || dev >= 64) return set_error(TQ_ERROR_UNSUPPORTED, "device ordinal %d >= 64", dev);
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ready[dev]) {
        void* p = nullptr;
        s = cuda_status(cudaGetSymbolAddress(&p, g_attn_static_scratch), "cudaGetSymbolAddress(static scratch)");
        if (s) return s;
        g_static_ptr[dev] = p;
        g_static_ready[dev] = true;
    }
    *out = g_static_ptr[dev];
    return TQ_SUCCESS;
}

extern "C" tq_status tq_decode_attention_static_cuda(const tq_decode_attention_args* a, void* stream) {
    AttnRun r;
    AttnPlan p;
    tq_status s = attn_check(a, &r, &p);
    if (s) return s;
    if (r.B == 0) return TQ_SUCCESS;
    const size_t need = attn_workspace_bytes(r.B, r.Hkv, r.D, p);
    if (need > TQ_STATIC_SCRATCH_BYTES)
        return set_error(TQ_ERROR_INVALID_VALUE,
                         "these arguments need %zu bytes of work memory; the fixed scratch holds %zu "
                         "(use tq_decode_attention_cuda with a caller workspace)",
                         need, (size_t)TQ_STATIC_SCRATCH_BYTES);
    void* ws = nullptr;
    if ((s = static_scratch(&ws))) return s;
    // the launch clears the error word and the per-pair counters, and every partial is written
    // before it is read, so the previous call's contents never leak into this one
    return cuda_status(launch_decode_attention(r, p, ws, (cudaStream_t)stream), "decode attention launch");
}
