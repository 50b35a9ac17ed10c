// tq_attn.h — internal interface of the decode-attention kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace tq {

struct AttnPlan {
    int64_t lnom = 0;            // nominal tokens per (sequence, KV head), multiple of 16
    int64_t chunk = 0;           // tokens per CTA (multiple of 16 x warps per CTA)
    int grid = 0;                // CTAs
    int slots = 0;               // partial slots per (sequence, KV head)
};

// Destination of the split-sequence exchange (world 0: the kernel writes out / lse instead).  The
// last CTA of a (sequence, KV head) pair stores the pair's rows [o (D floats) | lse] into slot
// (par, rank) of every rank's exchange buffer, then counts the pair in every rank's arrival
// counter (the buffer's first 8 bytes).  Buffer layout: counter | status | slots [2][world][slot_floats]
// from PEER_HEAD_BYTES on, each slot [o (n_rows x D) | lse (n_rows)].
constexpr size_t PEER_HEAD_BYTES = 256;
constexpr int PEER_OUT_MAX_WORLD = 64;
struct PeerOut {
    uint8_t* base[PEER_OUT_MAX_WORLD] = {};
    int world = 0, rank = 0, par = 0;
    int64_t slot_floats = 0, n_rows = 0;
};

struct AttnRun {
    int B = 0, Hq = 0, Hkv = 0, grp = 0, D = 0;
    const void* q = nullptr;
    int q_dtype = 0;
    const void* k = nullptr;
    const void* v = nullptr;
    int k_type = 4, v_type = 4;
    int64_t cap = 0;
    const int32_t* kv_len = nullptr;
    float sm_scale = 0.0f;
    int rotate_q = 1, v_rotated = 1;
    void* out = nullptr;
    int out_dtype = 0;
    float* lse = nullptr;
    PeerOut peer;
    // paged caches (pages != null): k / v are page pools [num_pages][Hkv][1 << page_shift][blocks],
    // pages[b * max_pages + i] the pool page of tokens [i << page_shift, (i + 1) << page_shift) of
    // sequence b; cap = max_pages << page_shift
    const int32_t* pages = nullptr;
    int64_t max_pages = 0, num_pages = 0;
    int page_shift = 0;
};

AttnPlan attn_plan(int B, int Hkv, int D, int64_t cap, int64_t max_len);
size_t attn_workspace_bytes(int B, int Hkv, int D, const AttnPlan& p);
cudaError_t launch_decode_attention(const AttnRun& r, const AttnPlan& p, void* workspace, cudaStream_t st);
cudaError_t launch_lse_combine(const float* o, int64_t o_stride, const float* lse, int64_t lse_stride, void* out,
                               int out_dtype, float* lse_out, int P, int64_t n, int D, cudaStream_t st);

}  // namespace tq
