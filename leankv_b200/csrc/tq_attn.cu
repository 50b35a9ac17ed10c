// tq_attn.cu — fused decode attention over packed TurboQuant K/V blocks (sm_100a).
//
// Math (restated from src/test-tq.c:532-559 and prototype/eval/cosine_sim.py:158-172,
// fused as docs/CUDA-RESULTS.md:23-52 and docs/PLAN.md:281-288 describe it):
//   q~ = FWHT(q) (K is stored rotated), s_t = sm_scale * q~ . K^_t, p = softmax(s),
//   o~ = sum_t p_t V^_t, o = FWHT(o~) when V is stored rotated.
// K^ and V^ are the reference dequantization (level[code] * d) of TQ4_0 / TQ3_0
// blocks; the kernel never materialises them in memory.
//
// Kernels
//   attn_qprep_kernel   FWHT(q) * sm_scale * log2(e) -> fp16, scattered into the
//                       register layout of the mma B operand (once per step)
//   attn_decode_kernel  persistent; CTA = 16 warps, each warp streams its own
//                       16-token K/V tiles through a 4-stage ring of 1-D bulk
//                       copies (cp.async.bulk + mbarrier), dequantizes them
//                       straight into mma.sync.m16n8k16 fragments through a
//                       shared-memory byte -> half2 codebook table, and keeps an
//                       online softmax; warps of a CTA merge in shared memory and
//                       write one (m, l, O) partial per (sequence, KV head, split)
//   attn_combine_kernel log-sum-exp merge of the split partials, inverse FWHT,
//                       output cast, optional lse
//   lse_combine_kernel  the same merge for partial results of several ranks
//
// Fragment bookkeeping (lane = 4*g + t, g = lane/4, t = lane%4):
//   S = K Q~^T: M = 16 tokens, N = 8 query heads of the GQA group (padded),
//     K-chunk kk = 2*blk + h covers qs bytes 8h .. 8h+7 of block blk; lane t
//     supplies the byte pair (8h + 2t, 8h + 2t + 1), the low byte giving the
//     elements (j, j+16) at k-cols (2t, 2t+1), the high byte at (2t+8, 2t+9).
//     q~ is permuted identically in the prep kernel.  Each block's two chunks
//     accumulate separately and are scaled by that token's block scale in fp32.
//   O^T = V^T P: M = 16 rows of one V block per m-tile (mt -> block mt/2),
//     row r of m-tile mt is element 32*(mt/2) + 2*(r%8) + (mt%2) + 16*(r/8);
//     K-chunk = the warp's 16 tokens.  The V block scales multiply P (fp16).
#include <cstdint>
#include <cstdio>

#include "leankv_tq.h"
#include "tq_attn.h"
#include "tq_capi_internal.h"
#include "tq_common.cuh"
#include "tq_kernels.h"

namespace tq {

constexpr int ATT_WARPS = 16;
constexpr int ATT_THREADS = ATT_WARPS * 32;
constexpr int ATT_TILE = 16;            // tokens per warp tile
constexpr int ATT_STAGES = 4;
constexpr int ATT_N = 8;                // query heads per mma N tile
constexpr int LUT_BYTES = 65536;        // 256 rows x 256 B: TQ4 byte table | TQ3 6-bit table
constexpr float LOG2E = 1.4426950408889634f;
constexpr uint32_t WAIT_LIMIT = 1u << 22;   // bounded mbarrier waits (about a second at most)

// ── small PTX helpers ─────────────────────────────────────────────────────────

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// bounded wait: returns false (and the caller records TQ_ERROR_TIMEOUT) instead of hanging
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < WAIT_LIMIT; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 r = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&r);
}

// Codebook table: entry for byte k (lo nibble n0, hi nibble n1) is half2(L[n0], L[n1]),
// replicated so that lane l always reads bank l: address = (k << 8) | (lane << 2).
// The TQ3 table (6-bit index, codes c0 | c1 << 3) sits at offset 128 in rows 0..63.
__device__ __forceinline__ uint32_t lut_addr(uint32_t word, uint32_t lane4, uint32_t sel) {
    return prmt(word, lane4, sel);
}
// selectors putting byte k of `word` at bits 8..15 and lane4 at bits 0..7
#define LUT_SEL0 0x5504u
#define LUT_SEL1 0x5514u
#define LUT_SEL2 0x5524u
#define LUT_SEL3 0x5534u

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// ── q preparation ─────────────────────────────────────────────────────────────
// One CTA (128 threads) per (sequence, KV head): FWHT of the grp query heads
// (same butterfly order as src/ggml-tq.c:365-374), scale, fp16, fragment layout.

template <typename QT>
__device__ __forceinline__ float load_q(const QT* p);
template <> __device__ __forceinline__ float load_q<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float load_q<__half>(const __half* p) { return __half2float(*p); }
template <> __device__ __forceinline__ float load_q<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename QT, int D>
__global__ void __launch_bounds__(128) attn_qprep_kernel(const QT* __restrict__ q, uint32_t* __restrict__ qfrag,
                                                         int Hq, int Hkv, int grp, float scale, int rotate) {
    __shared__ float sq[ATT_N][D];
    const int pair = blockIdx.x;
    const int b = pair / Hkv, g = pair % Hkv;
    for (int i = threadIdx.x; i < ATT_N * D; i += 128) {
        const int h = i / D, e = i % D;
        sq[h][e] = h < grp ? load_q<QT>(q + ((size_t)b * Hq + (size_t)g * grp + h) * D + e) : 0.0f;
    }
    __syncthreads();
    if (rotate) {
        for (int hstep = 1; hstep < D; hstep <<= 1) {
            for (int i = threadIdx.x; i < ATT_N * D / 2; i += 128) {
                const int h = i / (D / 2), p = i % (D / 2);
                const int lg = __ffs(hstep) - 1;
                const int j = ((p >> lg) << (lg + 1)) | (p & (hstep - 1));
                const float a = sq[h][j], c = sq[h][j + hstep];
                sq[h][j] = a + c;
                sq[h][j + hstep] = a - c;
            }
            __syncthreads();
        }
    }
    // scale = sm_scale * log2(e) [* 1/sqrt(D) of the FWHT folded in by the caller]
    constexpr int NCH = D / 16;
    uint32_t* out = qfrag + (size_t)pair * NCH * 64;
    for (int i = threadIdx.x; i < NCH * 32; i += 128) {
        const int kk = i / 32, lane = i % 32;
        const int gl = lane >> 2, t = lane & 3;
        const int blk = kk >> 1, h = kk & 1;
        const int e0 = 32 * blk + 8 * h + 2 * t;
        out[kk * 64 + lane * 2 + 0] = pack_h2(sq[gl][e0] * scale, sq[gl][e0 + 16] * scale);
        out[kk * 64 + lane * 2 + 1] = pack_h2(sq[gl][e0 + 1] * scale, sq[gl][e0 + 17] * scale);
    }
}

// ── decode kernel ─────────────────────────────────────────────────────────────

struct AttnKernelArgs {
    const uint32_t* qfrag;      // [pairs][D/16][32][2]
    const uint8_t* k;
    const uint8_t* v;
    const int32_t* kv_len;      // [B] or null
    float* part;                // [pairs][splits][ATT_N][D + 2]
    int* err;
    int64_t cap;                // token capacity per (sequence, KV head)
    int64_t split_tokens;       // multiple of ATT_WARPS * ATT_TILE
    int B, Hkv, grp, splits;
};

template <int D, int KT, int VT>
__global__ void __launch_bounds__(ATT_THREADS, 1) attn_decode_kernel(const AttnKernelArgs a) {
    constexpr int NBLK = D / 32;
    constexpr int KB = (KT == 4 ? TQ4_BYTES : TQ3_BYTES) * NBLK;   // bytes per token
    constexpr int VB = (VT == 4 ? TQ4_BYTES : TQ3_BYTES) * NBLK;
    constexpr int KTILE = ATT_TILE * KB, VTILE = ATT_TILE * VB;
    constexpr int NCH = D / 16;                 // QK k-chunks
    constexpr int NMT = D / 16;                 // PV m-tiles
    static_assert(KT == 4 && VT == 4, "this build covers TQ4_0 K and V");

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* lut = smem;
    uint8_t* stages = smem + LUT_BYTES;                                        // [warp][stage][K|V]
    float* dks = reinterpret_cast<float*>(stages + ATT_WARPS * ATT_STAGES * (KTILE + VTILE));   // [warp][16][NBLK]
    uint16_t* dvs = reinterpret_cast<uint16_t*>(dks + ATT_WARPS * ATT_TILE * NBLK);               // [warp][NBLK][16]
    uint64_t* bars = reinterpret_cast<uint64_t*>(dvs + ATT_WARPS * NBLK * ATT_TILE);             // [warp][stage]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const uint32_t lane4 = (uint32_t)lane << 2;

    // codebook table (TQ4 rows)
    for (int i = threadIdx.x; i < 256 * 32; i += ATT_THREADS) {
        const int k = i >> 5, l = i & 31;
        const uint32_t v = pack_h2(tq4_level(k & 15), tq4_level(k >> 4));
        *reinterpret_cast<uint32_t*>(lut + (k << 8) + (l << 2)) = v;
    }
    if (lane == 0)
        for (int s = 0; s < ATT_STAGES; ++s) mbar_init(smem_u32(&bars[warp * ATT_STAGES + s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = 0;
    const uint32_t lut_base = smem_u32(lut);
    uint8_t* my_stage = stages + warp * ATT_STAGES * (KTILE + VTILE);
    float* my_dk = dks + warp * ATT_TILE * NBLK;
    uint16_t* my_dv = dvs + warp * NBLK * ATT_TILE;
    uint32_t phase_bits = 0;   // parity per stage

    const int64_t pairs = (int64_t)a.B * a.Hkv;
    const int64_t items = pairs * a.splits;
    const int64_t per_warp = a.split_tokens / ATT_WARPS;

    for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
        const int64_t pair = item / a.splits;
        const int split = (int)(item % a.splits);
        const int bseq = (int)(pair / a.Hkv);
        int64_t len = a.kv_len ? (int64_t)a.kv_len[bseq] : a.cap;
        if (len > a.cap) len = a.cap;
        if (len < 0) len = 0;
        const int64_t t_begin = (int64_t)split * a.split_tokens + warp * per_warp;
        int64_t t_end = t_begin + per_warp;
        if (t_end > len) t_end = len;
        const int ntiles = t_end > t_begin ? (int)((t_end - t_begin + ATT_TILE - 1) / ATT_TILE) : 0;

        const uint8_t* kbase = a.k + (size_t)pair * a.cap * KB;
        const uint8_t* vbase = a.v + (size_t)pair * a.cap * VB;

        // B fragments of q~ for this pair
        uint32_t qf[NCH][2];
        {
            const uint32_t* src = a.qfrag + (size_t)pair * NCH * 64;
#pragma unroll
            for (int kk = 0; kk < NCH; ++kk) {
                qf[kk][0] = src[kk * 64 + lane * 2];
                qf[kk][1] = src[kk * 64 + lane * 2 + 1];
            }
        }

        float o[NMT][4];
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
        float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};

        // issue: one elected lane posts the bulk copies of tile i into stage i % STAGES
        auto issue = [&](int i) {
            if (lane == 0 && i < ntiles) {
                const int s = i % ATT_STAGES;
                const int64_t t0 = t_begin + (int64_t)i * ATT_TILE;
                int64_t nt = a.cap - t0;
                if (nt > ATT_TILE) nt = ATT_TILE;
                const uint32_t kbytes = (uint32_t)(nt * KB), vbytes = (uint32_t)(nt * VB);
                const uint32_t bar = smem_u32(&bars[warp * ATT_STAGES + s]);
                uint8_t* dst = my_stage + s * (KTILE + VTILE);
                mbar_expect_tx(bar, kbytes + vbytes);
                bulk_g2s(smem_u32(dst), kbase + t0 * KB, kbytes, bar);
                bulk_g2s(smem_u32(dst + KTILE), vbase + t0 * VB, vbytes, bar);
            }
        };
        for (int i = 0; i < ATT_STAGES - 1; ++i) issue(i);

        bool timed_out = false;
        for (int i = 0; i < ntiles; ++i) {
            issue(i + ATT_STAGES - 1);
            const int s = i % ATT_STAGES;
            const uint32_t bar = smem_u32(&bars[warp * ATT_STAGES + s]);
            if (!mbar_wait(bar, (phase_bits >> s) & 1u)) {
                // record the failure, then drain this warp's other copies (bounded) and leave
                if (lane == 0) {
                    atomicExch(a.err, (int)TQ_ERROR_TIMEOUT);
                    s_abort = 1;
                }
                for (int j = i + 1; j < ntiles && j < i + ATT_STAGES; ++j) {
                    const int sj = j % ATT_STAGES;
                    mbar_wait(smem_u32(&bars[warp * ATT_STAGES + sj]), (phase_bits >> sj) & 1u);
                }
                timed_out = true;
                break;
            }
            phase_bits ^= 1u << s;
            const uint8_t* kt = my_stage + s * (KTILE + VTILE);
            const uint8_t* vt = kt + KTILE;
            const int64_t t0 = t_begin + (int64_t)i * ATT_TILE;
            const int valid = (int)((t_end - t0) < ATT_TILE ? (t_end - t0) : ATT_TILE);

            // block scales of this tile: K as fp32 [tok][blk], V as fp16 bits [blk][tok]
            for (int j = lane; j < ATT_TILE * NBLK; j += 32) {
                const int tok = j / NBLK, blk = j % NBLK;
                const uint32_t hk = (uint32_t)kt[tok * KB + blk * TQ4_BYTES] |
                                    ((uint32_t)kt[tok * KB + blk * TQ4_BYTES + 1] << 8);
                const uint32_t hv = (uint32_t)vt[tok * VB + blk * TQ4_BYTES] |
                                    ((uint32_t)vt[tok * VB + blk * TQ4_BYTES + 1] << 8);
                my_dk[tok * NBLK + blk] = tok < valid ? half_decode(hk) : 0.0f;
                if (tok < valid && (hv & 0x7C00u) == 0x7C00u) atomicExch(a.err, (int)TQ_ERROR_UNSUPPORTED);
                my_dv[blk * ATT_TILE + tok] = tok < valid ? (uint16_t)hv : (uint16_t)0;
            }
            __syncwarp();

            // ---- S = K q~^T (16 tokens x 8 heads) ----
            float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const uint32_t krow0 = smem_u32(kt) + gq * KB, krow1 = krow0 + 8 * KB;
#pragma unroll
            for (int blk = 0; blk < NBLK; ++blk) {
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t off = blk * TQ4_BYTES + 2 + 8 * h + 2 * tq;
                    const uint32_t w0 = lds_u16(krow0 + off), w1 = lds_u16(krow1 + off);
                    uint32_t af[4];
                    af[0] = lds_u32(lut_base + lut_addr(w0, lane4, LUT_SEL0));
                    af[1] = lds_u32(lut_base + lut_addr(w1, lane4, LUT_SEL0));
                    af[2] = lds_u32(lut_base + lut_addr(w0, lane4, LUT_SEL1));
                    af[3] = lds_u32(lut_base + lut_addr(w1, lane4, LUT_SEL1));
                    mma16816(acc, af, qf[2 * blk + h][0], qf[2 * blk + h][1]);
                }
                const float d0 = my_dk[gq * NBLK + blk], d1 = my_dk[(gq + 8) * NBLK + blk];
                sc[0] = fmaf(d0, acc[0], sc[0]);
                sc[1] = fmaf(d0, acc[1], sc[1]);
                sc[2] = fmaf(d1, acc[2], sc[2]);
                sc[3] = fmaf(d1, acc[3], sc[3]);
            }
            // mask tokens beyond the valid range
            if (gq >= valid) { sc[0] = -INFINITY; sc[1] = -INFINITY; }
            if (gq + 8 >= valid) { sc[2] = -INFINITY; sc[3] = -INFINITY; }

            // ---- online softmax (log2 domain; heads 2tq, 2tq+1 per lane) ----
            float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
            for (int sh = 4; sh < 32; sh <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
            }
            const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
            const float al0 = mn0 == -INFINITY ? 1.0f : ex2(m_run[0] - mn0);
            const float al1 = mn1 == -INFINITY ? 1.0f : ex2(m_run[1] - mn1);
            m_run[0] = mn0;
            m_run[1] = mn1;
            if (__any_sync(0xffffffffu, al0 != 1.0f || al1 != 1.0f)) {
#pragma unroll
                for (int mt = 0; mt < NMT; ++mt) {
                    o[mt][0] *= al0; o[mt][1] *= al1; o[mt][2] *= al0; o[mt][3] *= al1;
                }
                l_run[0] *= al0;
                l_run[1] *= al1;
            }
            const float p0 = mn0 == -INFINITY ? 0.0f : ex2(sc[0] - mn0);
            const float p1 = mn1 == -INFINITY ? 0.0f : ex2(sc[1] - mn1);
            const float p2 = mn0 == -INFINITY ? 0.0f : ex2(sc[2] - mn0);
            const float p3 = mn1 == -INFINITY ? 0.0f : ex2(sc[3] - mn1);
            l_run[0] += p0 + p2;
            l_run[1] += p1 + p3;
            // P^T as the mma B operand: lane (g, t) gets head g, tokens (2t, 2t+1) and (2t+8, 2t+9)
            const uint32_t pb01 = movmatrix_t(pack_h2(p0, p1));
            const uint32_t pb23 = movmatrix_t(pack_h2(p2, p3));

            // ---- O^T += V^T P' ----
            const uint32_t vtok0 = smem_u32(vt) + (2 * tq) * VB, vtok1 = vtok0 + VB;
            const uint32_t vtok2 = vtok0 + 8 * VB, vtok3 = vtok2 + VB;
#pragma unroll
            for (int blk = 0; blk < NBLK; ++blk) {
                const uint32_t off = blk * TQ4_BYTES + 2 + 2 * gq;
                const uint32_t w0 = lds_u16(vtok0 + off), w1 = lds_u16(vtok1 + off);
                const uint32_t w2 = lds_u16(vtok2 + off), w3 = lds_u16(vtok3 + off);
                // bytes [B0(t), B0(t+1), B1(t), B1(t+1)] for the token pairs (2t,2t+1), (2t+8,2t+9)
                const uint32_t ra = prmt(w0, w1, 0x5140u), rb = prmt(w2, w3, 0x5140u);
                const uint32_t ra4 = ra >> 4, rb4 = rb >> 4;
                const uint32_t xa = (ra & 0x000F000Fu) | (ra4 & 0x00F000F0u);   // lo nibbles, byte 0 / 2
                const uint32_t ya = (ra4 & 0x000F000Fu) | ((ra >> 8) & 0x00F000F0u);   // hi nibbles
                const uint32_t xb = (rb & 0x000F000Fu) | (rb4 & 0x00F000F0u);
                const uint32_t yb = (rb4 & 0x000F000Fu) | ((rb >> 8) & 0x00F000F0u);
                // V scales of this block for the lane's token pairs, folded into P
                const uint32_t dv01 = *reinterpret_cast<const uint32_t*>(my_dv + blk * ATT_TILE + 2 * tq);
                const uint32_t dv89 = *reinterpret_cast<const uint32_t*>(my_dv + blk * ATT_TILE + 2 * tq + 8);
                const uint32_t b0 = h2_mul(pb01, dv01), b1 = h2_mul(pb23, dv89);
#pragma unroll
                for (int par = 0; par < 2; ++par) {
                    const uint32_t sel = par ? LUT_SEL2 : LUT_SEL0;
                    uint32_t af[4];
                    af[0] = lds_u32(lut_base + lut_addr(xa, lane4, sel));   // row g, tokens 2t, 2t+1
                    af[1] = lds_u32(lut_base + lut_addr(ya, lane4, sel));   // row g+8
                    af[2] = lds_u32(lut_base + lut_addr(xb, lane4, sel));   // row g, tokens 2t+8, 2t+9
                    af[3] = lds_u32(lut_base + lut_addr(yb, lane4, sel));   // row g+8
                    mma16816(o[2 * blk + par], af, b0, b1);
                }
            }
            __syncwarp();   // stage s and the scale scratch are free for reuse
        }

        // ---- merge the 16 warps of this CTA, write the split partial ----
        float l0 = l_run[0], l1 = l_run[1];
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
            l1 += __shfl_xor_sync(0xffffffffu, l1, sh);
        }
        (void)timed_out;
        __syncthreads();   // every warp is done with its stages; reuse them as scratch
        if (s_abort) return;   // uniform: every thread reads the flag after the barrier
        float* red = reinterpret_cast<float*>(stages);   // [warp][ATT_N][D + 2]
        float* mine = red + warp * ATT_N * (D + 2);
        if (gq == 0) {
            mine[(2 * tq) * (D + 2) + 0] = m_run[0];
            mine[(2 * tq + 1) * (D + 2) + 0] = m_run[1];
            mine[(2 * tq) * (D + 2) + 1] = l0;
            mine[(2 * tq + 1) * (D + 2) + 1] = l1;
        }
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt) {
            const int e0 = 32 * (mt >> 1) + 2 * gq + (mt & 1);
            mine[(2 * tq) * (D + 2) + 2 + e0] = o[mt][0];
            mine[(2 * tq + 1) * (D + 2) + 2 + e0] = o[mt][1];
            mine[(2 * tq) * (D + 2) + 2 + e0 + 16] = o[mt][2];
            mine[(2 * tq + 1) * (D + 2) + 2 + e0 + 16] = o[mt][3];
        }
        __syncthreads();
        float* dst = a.part + (size_t)item * ATT_N * (D + 2);
        for (int idx = threadIdx.x; idx < ATT_N * (D + 2); idx += ATT_THREADS) {
            const int h = idx / (D + 2), c = idx % (D + 2);
            float M = -INFINITY;
            for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, red[w * ATT_N * (D + 2) + h * (D + 2)]);
            float acc = 0.0f;
            if (c == 0) {
                acc = M;
            } else if (M != -INFINITY) {
                for (int w = 0; w < ATT_WARPS; ++w) {
                    const float mw = red[w * ATT_N * (D + 2) + h * (D + 2)];
                    if (mw != -INFINITY) acc += ex2(mw - M) * red[w * ATT_N * (D + 2) + idx];
                }
            }
            dst[idx] = acc;
        }
        __syncthreads();   // scratch (= stages) free before the next item
    }
}

// ── split combine + inverse FWHT + cast ──────────────────────────────────────

template <typename OT> __device__ __forceinline__ void store_out(OT* p, float v);
template <> __device__ __forceinline__ void store_out<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void store_out<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <> __device__ __forceinline__ void store_out<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename OT, int D>
__global__ void __launch_bounds__(128) attn_combine_kernel(const float* __restrict__ part, OT* __restrict__ out,
                                                           float* __restrict__ lse, int Hq, int Hkv, int grp,
                                                           int splits, int v_rotated, float fwht_norm) {
    __shared__ float so[D];
    __shared__ float sw[64];
    const int bh = blockIdx.x;             // sequence * Hq + head
    const int b = bh / Hq, h = bh % Hq;
    const int g = h / grp, hh = h % grp;
    const int64_t pair = (int64_t)b * Hkv + g;
    const float* p0 = part + ((size_t)pair * splits) * ATT_N * (D + 2) + hh * (D + 2);
    const size_t sstride = (size_t)ATT_N * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, p0[s * sstride]);
    float L = 0.0f;
    for (int s = 0; s < splits; ++s) {
        const float ms = p0[s * sstride];
        if (ms != -INFINITY) L += ex2(ms - M) * p0[s * sstride + 1];
    }
    for (int e = threadIdx.x; e < D; e += 128) {
        float acc = 0.0f;
        if (M != -INFINITY) {
            for (int s = 0; s < splits; ++s) {
                const float ms = p0[s * sstride];
                if (ms != -INFINITY) acc += ex2(ms - M) * p0[s * sstride + 2 + e];
            }
            acc /= L;
        }
        so[e] = acc;
    }
    __syncthreads();
    if (v_rotated) {
        for (int hs = 1; hs < D; hs <<= 1) {
            for (int p = threadIdx.x; p < D / 2; p += 128) {
                const int lg = __ffs(hs) - 1;
                const int j = ((p >> lg) << (lg + 1)) | (p & (hs - 1));
                const float x = so[j], y = so[j + hs];
                so[j] = x + y;
                so[j + hs] = x - y;
            }
            __syncthreads();
        }
    }
    for (int e = threadIdx.x; e < D; e += 128) store_out<OT>(out + (size_t)bh * D + e, v_rotated ? so[e] * fwht_norm : so[e]);
    if (lse && threadIdx.x == 0)
        lse[bh] = M == -INFINITY ? -INFINITY : (M + __log2f(L)) * 0.6931471805599453f;
    (void)sw;
}

// log-sum-exp merge of P partial results (natural-log lse), e.g. from several ranks
__global__ void __launch_bounds__(128) lse_combine_kernel(const float* __restrict__ o, const float* __restrict__ lse,
                                                          float* __restrict__ out, float* __restrict__ lse_out,
                                                          int P, int64_t n, int D) {
    const int64_t i = blockIdx.x;
    float M = -INFINITY;
    for (int p = 0; p < P; ++p) M = fmaxf(M, lse[(int64_t)p * n + i]);
    float W = 0.0f;
    for (int p = 0; p < P; ++p) {
        const float l = lse[(int64_t)p * n + i];
        if (l != -INFINITY) W += __expf(l - M);
    }
    for (int e = threadIdx.x; e < D; e += 128) {
        float acc = 0.0f;
        if (M != -INFINITY)
            for (int p = 0; p < P; ++p) {
                const float l = lse[(int64_t)p * n + i];
                if (l != -INFINITY) acc += __expf(l - M) * o[((int64_t)p * n + i) * D + e];
            }
        out[i * D + e] = M == -INFINITY ? 0.0f : acc / W;
    }
    if (lse_out && threadIdx.x == 0) lse_out[i] = M == -INFINITY ? -INFINITY : M + __logf(W);
}

// ── host side ───────────────────────────────────────────────────────────────

template <int D, int KT, int VT>
static size_t decode_smem_bytes() {
    constexpr int NBLK = D / 32;
    constexpr int KB = (KT == 4 ? TQ4_BYTES : TQ3_BYTES) * NBLK;
    constexpr int VB = (VT == 4 ? TQ4_BYTES : TQ3_BYTES) * NBLK;
    size_t s = LUT_BYTES;
    s += (size_t)ATT_WARPS * ATT_STAGES * ATT_TILE * (KB + VB);
    s += (size_t)ATT_WARPS * ATT_TILE * NBLK * 4;
    s += (size_t)ATT_WARPS * NBLK * ATT_TILE * 2;
    s += (size_t)ATT_WARPS * ATT_STAGES * 8;
    const size_t red = (size_t)ATT_WARPS * ATT_N * (D + 2) * 4;   // warp merge scratch reuses the stages
    const size_t stg = (size_t)ATT_WARPS * ATT_STAGES * ATT_TILE * (KB + VB);
    if (red > stg) s += red - stg;
    return s;
}

AttnPlan attn_plan(int B, int Hkv, int64_t cap, int64_t max_len) {
    AttnPlan p;
    const int64_t pairs = (int64_t)B * Hkv;
    const int sms = sm_count();
    const int64_t unit = ATT_WARPS * ATT_TILE;                 // 256 tokens
    const int64_t len = max_len > 0 ? max_len : cap;
    // enough (pair, split) items for a few waves over the SMs, splits of >= 1024 tokens
    int64_t want = (int64_t)sms * 4;
    int64_t splits = (want + pairs - 1) / pairs;
    int64_t max_splits = (len + 4 * unit - 1) / (4 * unit);
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    int64_t st = (len + splits - 1) / splits;
    st = (st + unit - 1) / unit * unit;
    splits = (len + st - 1) / st;
    if (splits < 1) splits = 1;
    p.splits = (int)splits;
    p.split_tokens = st;
    p.part_bytes = (size_t)pairs * splits * ATT_N * 130 * sizeof(float);   // refined by D below
    return p;
}

size_t attn_workspace_bytes(int B, int Hkv, int D, const AttnPlan& p) {
    const size_t pairs = (size_t)B * Hkv;
    size_t bytes = 256;                                           // error word (+ alignment)
    bytes += pairs * (D / 16) * 64 * sizeof(uint32_t);            // q fragments
    bytes = (bytes + 255) & ~size_t(255);
    bytes += pairs * p.splits * ATT_N * (D + 2) * sizeof(float);  // split partials
    return bytes;
}

template <typename QT, int D>
static cudaError_t launch_qprep(const void* q, uint32_t* qfrag, int B, int Hq, int Hkv, int grp, float scale,
                                int rotate, cudaStream_t st) {
    attn_qprep_kernel<QT, D><<<B * Hkv, 128, 0, st>>>((const QT*)q, qfrag, Hq, Hkv, grp, scale, rotate);
    return cudaGetLastError();
}

template <typename OT, int D>
static cudaError_t launch_combine(const float* part, void* out, float* lse, int B, int Hq, int Hkv, int grp,
                                  int splits, int v_rotated, cudaStream_t st) {
    attn_combine_kernel<OT, D><<<B * Hq, 128, 0, st>>>(part, (OT*)out, lse, Hq, Hkv, grp, splits, v_rotated,
                                                        fwht_norm(D));
    return cudaGetLastError();
}

template <int D>
static cudaError_t run_decode(const AttnRun& r, const AttnPlan& p, uint8_t* ws, cudaStream_t st) {
    int* err = reinterpret_cast<int*>(ws);
    uint32_t* qfrag = reinterpret_cast<uint32_t*>(ws + 256);
    size_t off = 256 + (size_t)r.B * r.Hkv * (D / 16) * 64 * sizeof(uint32_t);
    off = (off + 255) & ~size_t(255);
    float* part = reinterpret_cast<float*>(ws + off);
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    // q~ = FWHT(q) / sqrt(D) * sm_scale * log2(e): the FWHT normalisation folds into the scale
    const float scale = r.sm_scale * LOG2E * (r.rotate_q ? fwht_norm(D) : 1.0f);
    switch (r.q_dtype) {
        case DT_F32: e = launch_qprep<float, D>(r.q, qfrag, r.B, r.Hq, r.Hkv, r.grp, scale, r.rotate_q, st); break;
        case DT_F16: e = launch_qprep<__half, D>(r.q, qfrag, r.B, r.Hq, r.Hkv, r.grp, scale, r.rotate_q, st); break;
        default: e = launch_qprep<__nv_bfloat16, D>(r.q, qfrag, r.B, r.Hq, r.Hkv, r.grp, scale, r.rotate_q, st); break;
    }
    if (e != cudaSuccess) return e;
    AttnKernelArgs a;
    a.qfrag = qfrag;
    a.k = (const uint8_t*)r.k;
    a.v = (const uint8_t*)r.v;
    a.kv_len = r.kv_len;
    a.part = part;
    a.err = err;
    a.cap = r.cap;
    a.split_tokens = p.split_tokens;
    a.B = r.B;
    a.Hkv = r.Hkv;
    a.grp = r.grp;
    a.splits = p.splits;
    const size_t smem = decode_smem_bytes<D, 4, 4>();
    e = cudaFuncSetAttribute(attn_decode_kernel<D, 4, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int64_t items = (int64_t)r.B * r.Hkv * p.splits;
    const int grid = (int)(items < sm_count() ? items : sm_count());
    attn_decode_kernel<D, 4, 4><<<grid, ATT_THREADS, smem, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    switch (r.out_dtype) {
        case DT_F32: return launch_combine<float, D>(part, r.out, r.lse, r.B, r.Hq, r.Hkv, r.grp, p.splits, r.v_rotated, st);
        case DT_F16: return launch_combine<__half, D>(part, r.out, r.lse, r.B, r.Hq, r.Hkv, r.grp, p.splits, r.v_rotated, st);
        default: return launch_combine<__nv_bfloat16, D>(part, r.out, r.lse, r.B, r.Hq, r.Hkv, r.grp, p.splits, r.v_rotated, st);
    }
}

cudaError_t launch_decode_attention(const AttnRun& r, const AttnPlan& p, void* workspace, cudaStream_t st) {
    if (r.D == 128) return run_decode<128>(r, p, (uint8_t*)workspace, st);
    return cudaErrorInvalidValue;
}

cudaError_t launch_lse_combine(const float* o, const float* lse, float* out, float* lse_out, int P, int64_t n, int D,
                               cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    lse_combine_kernel<<<(unsigned)n, 128, 0, st>>>(o, lse, out, lse_out, P, n, D);
    return cudaGetLastError();
}

}  // namespace tq
