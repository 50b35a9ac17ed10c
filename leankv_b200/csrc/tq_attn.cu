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
//   attn_decode_kernel  persistent; CTA = 16 warps, each warp streams its own
//                       16-token K/V tiles through a 4-stage ring of 1-D bulk
//                       copies (cp.async.bulk + mbarrier), dequantizes them
//                       straight into mma.sync.m16n8k16 fragments through a
//                       shared-memory byte -> half2 codebook table, and keeps an
//                       online softmax.  Per (sequence, KV head) segment the CTA
//                       first rotates and scales the query heads of the group
//                       (FWHT(q) * sm_scale * log2(e) -> fp16 fragments) while
//                       its first tiles are in flight; at the end its warps merge
//                       in shared memory and write one (m, l, O) partial.  The
//                       last CTA to finish a pair (atomic counter) merges that
//                       pair's partials, applies the inverse FWHT, casts the
//                       output and writes the optional lse: one launch per step.
//   lse_combine_kernel  the same merge for partial results of several ranks
//
// Fragment bookkeeping (lane = 4*g + t, g = lane/4, t = lane%4):
//   S = K Q~^T: M = 16 tokens, N = 8 query heads of the GQA group (padded),
//     K-chunk kk = 2*blk + h of a TQ4 block; lane t supplies a byte pair, the
//     low byte giving the elements (j, j+16) at k-cols (2t, 2t+1), the high byte
//     at (2t+8, 2t+9): bytes (8h + 2t, 8h + 2t + 1) in even blocks (their codes
//     start 2 mod 4: two 16-bit loads per token), bytes (4t + 2h, 4t + 2h + 1)
//     in odd blocks (codes 4-byte aligned: one 32-bit load serves both chunks).
//     q~ is permuted identically when its fragments are built.  Each block's two chunks
//     accumulate separately and are scaled by that token's block scale in fp32.
//   O^T = V^T P: M = 16 rows of one V block per m-tile (mt -> block mt/2),
//     row r of m-tile mt is element 32*(mt/2) + 2*(r%8) + (mt%2) + 16*(r/8);
//     K-chunk = the warp's 16 tokens.  The V block scales multiply P (fp16).
//
// Precision: the codebook tables hold alpha * level in fp16, with alpha chosen per codebook so
// that every level rounds almost exactly (largest relative error 6.1e-5 for TQ4, 9.8e-6 for
// TQ3, against 3.1e-4 and 6.4e-5 unscaled); 1 / alpha folds into the fp32 K block scales and
// the final normalisation.  q~ is split into fp16 hi + lo parts and every score chunk runs two
// MMAs (qh and ql against the same codebook fragments), so the query is exact to about 2^-22.
#include <cstdint>
#include <cstdio>
#include <type_traits>

#include "leankv_tq.h"
#include "tq_attn.h"
#include "tq_capi_internal.h"
#include "tq_common.cuh"
#include "tq_kernels.h"
#include "tq_merge.cuh"

namespace tq {

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

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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
// prmt(word, lane4, LUT_SELk) is that address for byte k of `word`: byte k at bits 8..15,
// lane4 at bits 0..7.
#define LUT_SEL0 0x5504u
#define LUT_SEL1 0x5514u
#define LUT_SEL2 0x5524u
#define LUT_SEL3 0x5534u

// Codebook scales (fp32 constants found by search over [1, 2)): alpha * L rounds to fp16 with a
// relative error of at most 6.05e-5 (TQ4) and 9.75e-6 (TQ3).
constexpr float TQ4_ALPHA = 1.5976254940032959f;
constexpr float TQ3_ALPHA = 1.7372877597808838f;
constexpr float TQ2_ALPHA = 1.4960941076278687f;   // TQ2 levels: worst fp16 rounding 2.7e-7 relative

// hi + lo fp16 parts of two floats: hi = fp16(a), lo = fp16(a - hi)
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_h2(a - f.x, b - f.y);
}

// ── query rotation and output merge helpers ──────────────────────────────────

__device__ __forceinline__ float load_q(const void* q, int dt, size_t i) {
    if (dt == DT_F32) return static_cast<const float*>(q)[i];
    if (dt == DT_F16) return __half2float(static_cast<const __half*>(q)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(q)[i]);
}

__device__ __forceinline__ void store_out_rt(void* out, int dt, size_t i, float v) {
    if (dt == DT_F32) static_cast<float*>(out)[i] = v;
    else if (dt == DT_F16) static_cast<__half*>(out)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
}

// In-place FWHT of one row held by a warp, elements lane * EPL .. lane * EPL + EPL - 1 in v:
// stages h = 1, 2, 4, ... in the order of src/ggml-tq.c:365-374 (x[j] = a + c, x[j + h] = a - c
// for j with bit h clear), the first log2(EPL) stages in registers, the rest by shuffles.
template <int EPL>
__device__ __forceinline__ void fwht_warp_row(float (&v)[EPL], int lane) {
#pragma unroll
    for (int h = 1; h < EPL; h <<= 1) {
#pragma unroll
        for (int i = 0; i < EPL; ++i)
            if (!(i & h)) {
                const float x = v[i], y = v[i + h];
                v[i] = x + y;
                v[i + h] = x - y;
            }
    }
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const bool upper = (lane & d) != 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const float o = __shfl_xor_sync(0xffffffffu, v[i], d);
            v[i] = upper ? o - v[i] : v[i] + o;
        }
    }
}

// ── decode kernel ─────────────────────────────────────────────────────────────
//
// Work split: the (sequence, KV head, token) space, each pair padded to a
// nominal length Lnom (a multiple of 16), is cut into equal contiguous chunks,
// one per CTA, so every SM streams the same number of bytes.  A chunk covers
// one or more pair segments; within a segment warp w takes tiles w, w+16, ...
// (16 tokens each) through its private 4-stage bulk-copy ring.  At the end of a
// segment the 16 warps merge their (max, sum, O) in shared memory and the CTA
// writes one partial for (pair, slot), slot = CTA index - first CTA of the pair.
// It then counts itself in the pair's counter; the CTA that brings the count to
// the number of slots the pair spans reads all of them back from L2 (its
// predecessors fenced their partials before counting) and writes the output.
struct AttnKernelArgs {
    const void* q;              // [B][Hq][D] in q_dtype
    const uint8_t* k;
    const uint8_t* v;
    const int32_t* kv_len;      // [B] or null
    float* part;                // [pairs][slots][ATT_N][D + 2]
    int* err;
    int* cnt;                   // [pairs] CTAs finished per pair, zero at launch
    void* out;                  // [B][Hq][D] in out_dtype
    float* lse;                 // [B][Hq] or null
    int64_t cap;                // token capacity per (sequence, KV head)
    int64_t lnom;               // nominal tokens per pair (multiple of 16, >= every kv_len used)
    int64_t chunk;              // tokens per CTA (multiple of 256)
    float qscale;               // sm_scale * log2(e) [* 1/sqrt(D) of the query FWHT] / alpha of the K codebook
    float onorm;                // 1/sqrt(D) of the output FWHT
    int B, Hq, Hkv, grp, slots;
    int q_dtype, out_dtype, rotate_q, v_rotated;
    PeerOut peer;               // world 0: write out / lse; else store rows into every rank's slot
    const int32_t* pages;       // paged caches: [B][max_pages] pool pages (kernel template PG)
    int64_t max_pages, num_pages;
    int page_shift;             // log2 tokens per page, >= 4 (a 16-token tile never crosses a page)
    uint32_t page_mask;         // (1 << page_shift) - 1
    uint32_t page_kbytes, page_vbytes;   // bytes of one K / V pool page: (Hkv << page_shift) rows
};

template <int RES>
__device__ __forceinline__ uint32_t lut_ld(uint32_t word, uint32_t lane4, uint32_t sel) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(prmt(word, lane4, sel)), "n"(RES));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint32_t ld16(uint32_t base) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1+%2];" : "=h"(v) : "r"(base), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint32_t ld32(uint32_t base) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(base), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint2 ld64u(uint32_t base) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(base), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint4 ld128u(uint32_t base) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4+%5];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(base), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ float4 ld128f(uint32_t base) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4+%5];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(base), "n"(OFF));
    return v;
}

__device__ __forceinline__ void mma16816_zc(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

// bulk copy issued by lane 0 only (predicated, no branch)
__device__ __forceinline__ void bulk_issue(bool pred, uint32_t dst_k, const void* src_k, uint32_t bk,
                                           uint32_t dst_v, const void* src_v, uint32_t bv, uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %8, 0;\n\t"
        "@p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%6], %7;\n\t"
        "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%6];\n\t"
        "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%3], [%4], %5, [%6];\n\t}"
        ::"r"(dst_k), "l"(src_k), "r"(bk), "r"(dst_v), "l"(src_v), "r"(bv), "r"(bar), "r"(bk + bv),
        "r"((uint32_t)pred)
        : "memory");
}

constexpr float M_FLOOR = -1.0e30f;   // finite "minus infinity" for the running max

// a partial's value: through L2 when other CTAs wrote it, from shared memory when this CTA did
__device__ __forceinline__ float part_ld(bool in_smem, const float* p) { return in_smem ? *p : __ldcg(p); }

// compile-time loop: f(std::integral_constant<int, I>) for I in [B, E)
template <int B, int E, typename F>
__device__ __forceinline__ void static_for(F&& f) {
    if constexpr (B < E) {
        f(std::integral_constant<int, B>{});
        static_for<B + 1, E>(f);
    }
}

// Per-configuration constants.  A CTA runs 16 warps.  At head_dim 128 every warp
// streams its own tiles over all 4 blocks of a token row; at head_dim 256 the
// warps work in pairs (SPLIT = 2): both warps of a pair take the same tiles from
// one shared ring, each covers 4 of the 8 blocks (half the dimensions), and they
// add their partial scores through shared memory, so each warp's O and q
// fragments stay those of head_dim 128.  Token order inside a 16-token tile (mma row / k index r holds
// token tok_of_row(r)) is chosen per token pitch so that every fragment load is
// free of bank conflicts:
//   head_dim 128 (K pitch 72 or 56 bytes, V pitch 72): r < 8 -> 2r, r >= 8 -> 2(r-8)+1,
//     so K rows g, g+8 read tokens 2g, 2g+1 and V k-indices 2t, 2t+1, 2t+8, 2t+9
//     read tokens 4t, 4t+2, 4t+1, 4t+3;
//   head_dim 256 (K pitch 144 or 112, V pitch 144): identity.
// The softmax sum over tokens is order-free.
template <int D, int KT>
struct AttnCfg {
    static constexpr int NBLK = D / 32;                  // blocks per token row
    static constexpr int SPLIT = D / 128;                // warps per tile stream
    static constexpr int NBW = NBLK / SPLIT;             // blocks per warp (4)
    static constexpr int WARPS = 16;
    static constexpr int RINGS = WARPS / SPLIT;          // tile streams (rings) per CTA
    // stage-release barriers: the second warp of a pair frees a stage before the first refills it
    static constexpr int EBARS = SPLIT == 2 ? RINGS * ATT_STAGES : 0;
    static constexpr int THREADS = WARPS * 32;
    static constexpr int KBB = KT == 4 ? TQ4_BYTES : KT == 3 ? TQ3_BYTES : TQ2_BYTES;   // K bytes per block
    static constexpr int KB = KBB * NBLK;                          // K bytes per token
    static constexpr int VB = TQ4_BYTES * NBLK;                    // V bytes per token
    static constexpr int KTILE = ATT_TILE * KB, VTILE = ATT_TILE * VB;
    static constexpr int STAGE = KTILE + VTILE;
    static constexpr int NCH = 2 * NBW, NMT = 2 * NBW;   // mma k-chunks / m-tiles of one warp
    // scale scratch of one tile and warp: dK f32 [row][blk] | dV f16 [t][blk][rows 2t, 2t+1, 2t+8, 2t+9]
    static constexpr int SCR = ATT_TILE * NBW * 4 + NBW * ATT_TILE * 2;
    static constexpr bool INTERLEAVE = D == 128;
    __host__ __device__ static constexpr int tok_of_row(int r) {
        return INTERLEAVE ? (r < 8 ? 2 * r : 2 * (r - 8) + 1) : r;
    }
    __host__ __device__ static constexpr int row_of_tok(int t) { return INTERLEAVE ? ((t & 1) ? 8 + (t >> 1) : (t >> 1)) : t; }
    static_assert(KTILE % 16 == 0 && STAGE % 16 == 0, "bulk-copy destinations must stay 16-byte aligned");
};

__host__ __device__ constexpr int att_warps(int) { return 16; }
__host__ __device__ constexpr int att_rings(int D) { return att_warps(D) / (D / 128); }   // tile streams per CTA

// TQ3 code pairs -> byte address in the codebook table: pair i of a 24-bit group word
// (codes 2i, 2i+1) indexes row ((w >> 6i) & 63), TQ3 half of the row (byte 128 + 4 * lane).
template <int I>
__device__ __forceinline__ uint32_t tq3_lut_addr(uint32_t w, uint32_t lane4x) {
    const uint32_t f = I == 0 ? (w << 8) : I == 1 ? (w << 2) : I == 2 ? (w >> 4) : (w >> 10);
    return (f & 0x3F00u) | lane4x;
}
template <int RES>
__device__ __forceinline__ uint32_t lut_ld_addr(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(RES));
    return v;
}

// named barrier of the two warps of a pair (barrier 0 is __syncthreads)
__device__ __forceinline__ void pair_sync(int ring) {
    asm volatile("bar.sync %0, 64;" ::"r"(ring + 1) : "memory");
}

// PK (GQA group of at most 4 query heads): the score mma's 8 columns hold the group's q~ hi parts
// in columns 0-3 and its lo parts in columns 4-7, so one mma per chunk forms both products and one
// shuffle per score adds them; larger groups run a second mma per chunk with the lo parts.
// PG: paged caches; the issuing lane looks up each tile's pool page two tiles ahead of its copy.
template <int D, int KT, int RES, bool PK, bool PG>
__global__ void __launch_bounds__(att_warps(D) * 32, 1) attn_decode_kernel(const AttnKernelArgs a) {
    using Cfg = AttnCfg<D, KT>;
    constexpr int WARPS = Cfg::WARPS, THREADS = Cfg::THREADS;
    constexpr int SPLIT = Cfg::SPLIT, RINGS = Cfg::RINGS, NBLK = Cfg::NBW;   // NBLK: this warp's blocks
    static_assert(att_rings(D) == RINGS && att_warps(D) == WARPS, "host plan and kernel disagree");
    constexpr int KBB = Cfg::KBB, KB = Cfg::KB, VB = Cfg::VB;
    constexpr int KTILE = Cfg::KTILE, STAGE = Cfg::STAGE;
    constexpr int NCH = Cfg::NCH, NMT = Cfg::NMT, SCR = Cfg::SCR;
    static_assert(KT == 2 || KT == 3 || KT == 4, "TQ2_0, TQ3_0 or TQ4_0 K");
    static_assert(D == 128 || D == 256, "head_dim 128 or 256");

    extern __shared__ __align__(1024) uint8_t smem[];
    // layout: LUT | stages [ring][stage] | scale scratch [warp] | barriers [ring][stage] |
    // release barriers [ring][stage] (pairs only) | flag
    uint8_t* stages = smem + LUT_BYTES;
    uint8_t* scratch = stages + RINGS * ATT_STAGES * STAGE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(scratch + WARPS * 2 * SCR);
    uint64_t* ebars = bars + RINGS * ATT_STAGES;
    int* s_abort = reinterpret_cast<int*>(ebars + Cfg::EBARS);   // [0] abort, [1] last CTA of the pair
    // head_dim 256: the lo parts of q~'s B fragments, [half][chunk][lane], one copy per half of the
    // dimensions (every warp of a half holds the same ones), read per chunk instead of held in registers
    uint2* s_qfl = reinterpret_cast<uint2*>(s_abort + 4);
    // paged caches: the pool pages of the next tile of each stage of each ring, [ring][stage]
    int32_t* const s_pgs_all = reinterpret_cast<int32_t*>(s_qfl + (SPLIT == 2 ? 2 * NCH * 32 : 0));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ring = warp / SPLIT, half = warp % SPLIT;   // tile stream, half of the dimensions
    const int gq = lane >> 2, tq = lane & 3;
    const uint32_t lane4 = (uint32_t)lane << 2;

    if (smem_u32(smem) != (uint32_t)RES) {        // the LUT offset is an instruction immediate
        if (threadIdx.x == 0) atomicExch(a.err, (int)TQ_ERROR_UNSUPPORTED);
        return;                                    // uniform: no barrier has been used yet
    }
    for (int i = threadIdx.x; i < 256 * 32; i += THREADS) {
        const int k = i >> 5, l = i & 31;
        *reinterpret_cast<uint32_t*>(smem + (k << 8) + (l << 2)) =
            pack_h2(TQ4_ALPHA * tq4_level(k & 15), TQ4_ALPHA * tq4_level(k >> 4));
        // TQ3 pairs in the upper halves: rows 0..63 at head_dim 256 (rows 64..192 carry the pair
        // score exchange there), every row at head_dim 128, row k holding pair k mod 64 so that a
        // byte whose low 6 bits are a pair index addresses it directly
        if (KT == 3 && (SPLIT == 1 || k < 64))
            *reinterpret_cast<uint32_t*>(smem + (k << 8) + 128 + (l << 2)) =
                pack_h2(TQ3_ALPHA * tq3_level(k & 7), TQ3_ALPHA * tq3_level((k >> 3) & 7));
        // TQ2 pairs (two consecutive elements, codes c0 | c1 << 2: a nibble) in rows 0..15
        if (KT == 2 && k < 16)
            *reinterpret_cast<uint32_t*>(smem + (k << 8) + 128 + (l << 2)) =
                pack_h2(TQ2_ALPHA * tq2_level(k & 3), TQ2_ALPHA * tq2_level(k >> 2));
    }
    if (lane == 0 && half == 0)
        for (int s = 0; s < ATT_STAGES; ++s) {
            mbar_init(smem_u32(&bars[ring * ATT_STAGES + s]), 1);
            if constexpr (SPLIT == 2) mbar_init(smem_u32(&ebars[ring * ATT_STAGES + s]), 1);
        }
    if (threadIdx.x == 0) *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    const uint32_t stage0 = smem_u32(stages + ring * ATT_STAGES * STAGE);
    const uint32_t scr = smem_u32(scratch + warp * 2 * SCR);   // tile A at scr, tile B at scr + SCR
    const uint32_t bar0 = smem_u32(&bars[ring * ATT_STAGES]);
    const uint32_t ebar0 = smem_u32(ebars + ring * ATT_STAGES);   // valid when SPLIT == 2
    // this warp's blocks start hk / hv bytes into a token's K / V row
    const uint32_t hk = half * NBLK * KBB, hv = half * NBLK * TQ4_BYTES;
    // per-lane fixed offsets inside a stage
    constexpr int KROW8 = (Cfg::tok_of_row(8) - Cfg::tok_of_row(0)) * KB;   // row g+8 relative to row g
    const int ktok = Cfg::tok_of_row(gq);
    // TQ4 K, even blocks (codes start 2 mod 4): byte pair (8h + 2t, 8h + 2t + 1) for chunk h;
    // odd blocks (codes start 0 mod 4): the aligned word of bytes 4t .. 4t + 3, chunk h = bytes
    // (4t + 2h, 4t + 2h + 1)
    const uint32_t k_off = ktok * KB + hk + 2 * tq + 2;
    const uint32_t k_off_w = ktok * KB + hk + 4 * tq + 2;
    // TQ3 K: group t of each block, read as two aligned words and a funnel shift; blocks
    // start at 14 * blk bytes, which is 0 mod 4 for even and 2 mod 4 for odd blk
    const uint32_t k3_off_e = ktok * KB + hk + ((2 + 3 * tq) & ~3), k3_sh_e = 8 * ((2 + 3 * tq) & 3);
    const uint32_t k3_off_o = ktok * KB + hk + ((4 + 3 * tq) & ~3), k3_sh_o = 8 * ((4 + 3 * tq) & 3);
    const uint32_t lane4x = lane4 | 0x80u;
    // V: k-indices 2t, 2t+1, 2t+8, 2t+9 of the P fragment
    constexpr int VT0 = Cfg::tok_of_row(0);
    constexpr int VO1 = (Cfg::tok_of_row(1) - VT0) * VB, VO8 = (Cfg::tok_of_row(8) - VT0) * VB,
                  VO9 = (Cfg::tok_of_row(9) - VT0) * VB;
    const uint32_t v_off = Cfg::tok_of_row(2 * tq) * VB + hv + 2 * gq + 2;
    // scale extraction: lane handles K entries r = 0 .. NBLK/2-1 and V entries likewise; entry r
    // of this lane is token xt0 + r * TSTEP, block xb
    constexpr int TSTEP = 32 / NBLK, ROWSTEP = Cfg::INTERLEAVE ? TSTEP / 2 : TSTEP, NXH = NBLK / 2;
    const int xt0 = lane / NBLK, xb = lane % NBLK, xrow0 = Cfg::row_of_tok(xt0);
    const uint32_t xks = xt0 * KB + hk + xb * KBB, xkd = (xrow0 * NBLK + xb) * 4;
    // dV of row r, block b at (((r & 7) >> 1) * NBLK + b) * 8 + ((r & 1) + 2 * (r >> 3)) * 2: lane t then
    // finds the four P rows of every block in 2 * NBLK consecutive words.  Entry rr adds
    // rr * ROWSTEP rows to a first row whose low three bits stay below 4, hence VDELTA(rr).
    const uint32_t xvs = KTILE + xt0 * VB + hv + xb * TQ4_BYTES,
                   xvd = ATT_TILE * NBLK * 4 + ((((xrow0 & 7) >> 1) * NBLK + xb) * 8 + ((xrow0 & 1) + 2 * (xrow0 >> 3)) * 2);
    uint32_t phase_bits = 0;
    uint32_t ephase_bits = 0;   // release-barrier parities, kept by the issuing lane of a pair

    const int64_t pairs = (int64_t)a.B * a.Hkv;
    const int64_t total = pairs * a.lnom;
    int64_t gpos = (int64_t)blockIdx.x * a.chunk;
    uint32_t pairs_done = 0;   // pairs this CTA completed (thread 0), counted at the end for the exchange
    const int64_t gend = gpos + a.chunk < total ? gpos + a.chunk : total;

    while (gpos < gend) {
        const int64_t pair = gpos / a.lnom;
        const int64_t t0 = gpos - pair * a.lnom;
        int64_t t1 = a.lnom - t0 < gend - gpos ? a.lnom : t0 + (gend - gpos);
        gpos += t1 - t0;
        const int slot = (int)(blockIdx.x - (pair * a.lnom) / a.chunk);
        int64_t len = a.kv_len ? (int64_t)a.kv_len[pair / a.Hkv] : a.cap;
        if (len > a.cap) len = a.cap;
        if (t1 > len) t1 = len;
        const int ntiles_seg = t1 > t0 ? (int)((t1 - t0 + ATT_TILE - 1) / ATT_TILE) : 0;
        const int ntiles = ntiles_seg > ring ? (ntiles_seg - ring + RINGS - 1) / RINGS : 0;

        const uint8_t* kbase = a.k + (PG ? 0 : (size_t)pair * a.cap * KB);
        const uint8_t* vbase = a.v + (PG ? 0 : (size_t)pair * a.cap * VB);

        float o[NMT][4];
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;
        float m_run0 = M_FLOOR, m_run1 = M_FLOOR, l0 = 0.0f, l1 = 0.0f;

        // copy sources advance by one CTA tile row (RINGS x 16 tokens) per ring tile
        const uint8_t* ksrc = kbase + (t0 + (int64_t)ring * ATT_TILE) * KB;
        const uint8_t* vsrc = vbase + (t0 + (int64_t)ring * ATT_TILE) * VB;
        const int64_t tok_first = t0 + (int64_t)ring * ATT_TILE;      // first token of tile 0
        // tokens of the last tile that exist in memory (capacity), for the copy size
        const int64_t t_last = tok_first + (int64_t)(ntiles > 0 ? ntiles - 1 : 0) * RINGS * ATT_TILE;
        const uint32_t last_nt = PG ? (uint32_t)ATT_TILE   // pages hold whole tiles
                                    : (uint32_t)(a.cap - t_last < ATT_TILE ? a.cap - t_last : ATT_TILE);
        // tokens of the last tile below the valid length (tiles before it are full)
        const int last_valid = (int)(t1 - t_last < ATT_TILE ? t1 - t_last : ATT_TILE);
        int issued = 0;
        // paged: slot S of this ring's page slots holds the pool page of the next tile copied into
        // stage S.  The issuing lane fetches it with an asynchronous 4-byte copy (cp.async) when the
        // stage's previous tile is issued, four tiles ahead, one commit group per tile, and waits
        // for the group only when it issues the tile; a page id outside the pool is reported
        // (TQ_ERROR_INVALID_VALUE) and read as page 0.  (32-bit token offsets: the host keeps paged
        // capacities below 2^31 tokens.)
        const bool issuer = lane == 0 && half == 0;
        const int64_t pseq = PG ? pair / a.Hkv : 0;
        const uint32_t prow = PG ? (uint32_t)(pseq * a.max_pages) : 0u;                 // page-table row
        const uint32_t hrow = PG ? (uint32_t)(pair - pseq * a.Hkv) << a.page_shift : 0u;   // head's first row
        const uint32_t tok0 = (uint32_t)tok_first;
        const uint32_t s_pgs = smem_u32(s_pgs_all + ring * ATT_STAGES);
        // the page id of the tile starting at token `tok` (tile j) -> slot, then a commit; every lane
        // runs it (no divergent branch in the tile loop), the copy is predicated on the issuing lane
        auto page_fetch = [&](uint32_t tok, int j, int slot) {
            const int32_t* src = a.pages + (prow + (tok >> a.page_shift));
            asm volatile("{\n\t.reg .pred p;\n\t"
                         "setp.ne.u32 p, %2, 0;\n\t"
                         "@p cp.async.ca.shared.global [%0], [%1], 4;\n\t"
                         "cp.async.commit_group;\n\t}"
                         ::"r"(s_pgs + 4u * slot), "l"(src), "r"((uint32_t)(issuer && j < ntiles)) : "memory");
        };
        if constexpr (PG) {
#pragma unroll
            for (int j = 0; j < ATT_STAGES; ++j) page_fetch(tok0 + (uint32_t)j * (RINGS * ATT_TILE), j, j);
        }
        auto issue_next = [&](auto stage_c) {
            constexpr int S = decltype(stage_c)::value;
            const bool last = issued == ntiles - 1;
            const uint32_t nt = last ? last_nt : (uint32_t)ATT_TILE;
            if constexpr (PG) {   // tile `issued` goes into stage S = issued mod 4 (every lane runs this)
                const uint32_t tok = tok0 + (uint32_t)issued * (RINGS * ATT_TILE);
                // groups of tiles issued + 1 .. issued + 3 may still be in flight
                asm volatile("cp.async.wait_group 3;" ::: "memory");
                uint32_t pg;
                asm volatile("ld.shared.u32 %0, [%1];" : "=r"(pg) : "r"(s_pgs + 4u * S) : "memory");
                const bool bad = pg >= (uint32_t)a.num_pages;
                if (bad && issuer && issued < ntiles) atomicExch(a.err, (int)TQ_ERROR_INVALID_VALUE);
                pg = bad ? 0u : pg;
                // this tile's first token row inside its page: head * P + token in page
                const uint32_t r = hrow + (tok & a.page_mask);
                ksrc = a.k + ((uint64_t)pg * a.page_kbytes + (uint64_t)(r * (uint32_t)KB));
                vsrc = a.v + ((uint64_t)pg * a.page_vbytes + (uint64_t)(r * (uint32_t)VB));
                // after the slot's value is in use
                page_fetch(tok + ATT_STAGES * RINGS * ATT_TILE, issued + ATT_STAGES, S);
            }
            bool go = issuer && issued < ntiles;
            if (SPLIT == 2 && go && issued >= ATT_STAGES) {
                // the partner warp must be done with tile issued - ATT_STAGES in this stage; a
                // release that never comes leaves the stage unfilled and the full-barrier wait
                // of both warps then runs out and reports the timeout
                go = mbar_wait(ebar0 + 8 * S, (ephase_bits >> S) & 1u);
                ephase_bits ^= 1u << S;
            }
            bulk_issue(go, stage0 + S * STAGE, ksrc, nt * KB, stage0 + S * STAGE + KTILE, vsrc, nt * VB,
                       bar0 + 8 * S);
            if constexpr (!PG) {
                ksrc += (size_t)RINGS * ATT_TILE * KB;
                vsrc += (size_t)RINGS * ATT_TILE * VB;
            }
            ++issued;
        };
        // Tiles are processed in pairs: tiles 2p and 2p + 1 sit in stages 2p mod 4 and
        // 2p + 1 mod 4, and while a pair is computed the next pair is in flight in the
        // other two stages.  Two tiles per step give the scheduler two independent
        // dequantize / mma chains and one softmax update per 32 tokens.
        static_for<0, 2>([&](auto sc) { issue_next(sc); });

        // q~ of this pair while the first tiles are in flight: warp h < 8 loads query head h of
        // the group (zeros past grp), rotates it and scales it into the (still unused) scale
        // scratch; every warp then builds its fp16 mma B fragments from there.
        uint32_t qf[NCH][2], qfl[NCH][2];   // fp16 hi and lo parts of q~ (mma B fragments)
        {
            constexpr int SQS = D + 4;   // row pitch: the fragment reads below are at most 2-way conflicted
            static_assert(ATT_N * SQS * 4 <= WARPS * 2 * SCR, "q~ must fit the scale scratch");
            float* sq = reinterpret_cast<float*>(scratch);   // [ATT_N][SQS]
            if (warp < ATT_N) {
                constexpr int EPL = D / 32;
                float qv[EPL];
                if (warp < a.grp) {
                    const int64_t b = pair / a.Hkv, g = pair - b * a.Hkv;
                    const size_t row = ((size_t)b * a.Hq + (size_t)g * a.grp + warp) * D + (size_t)lane * EPL;
#pragma unroll
                    for (int i = 0; i < EPL; ++i) qv[i] = load_q(a.q, a.q_dtype, row + i);
                    if (a.rotate_q) fwht_warp_row<EPL>(qv, lane);
                } else {
#pragma unroll
                    for (int i = 0; i < EPL; ++i) qv[i] = 0.0f;
                }
#pragma unroll
                for (int i = 0; i < EPL; i += 4)
                    *reinterpret_cast<float4*>(sq + warp * SQS + lane * EPL + i) =
                        make_float4(qv[i] * a.qscale, qv[i + 1] * a.qscale, qv[i + 2] * a.qscale, qv[i + 3] * a.qscale);
            }
            __syncthreads();
            const float* mq = sq + (PK ? (gq & 3) : gq) * SQS;
#pragma unroll
            for (int kk = 0; kk < NCH; ++kk) {
                const int blk = half * NBLK + (kk >> 1), h = kk & 1;   // block of the token row
                if constexpr (KT == 4) {   // k-cols (2t, 2t+1) = elements (j, j+16), (2t+8, 2t+9) = (j+1, j+17)
                    const int e0 = 32 * blk + ((blk & 1) ? 4 * tq + 2 * h : 8 * h + 2 * tq);
                    split_h2(mq[e0], mq[e0 + 16], qf[kk][0], qfl[kk][0]);
                    split_h2(mq[e0 + 1], mq[e0 + 17], qf[kk][1], qfl[kk][1]);
                } else {                   // TQ3 group t: codes 4h, 4h+1 | 4h+2, 4h+3 of group t
                    const int e0 = 32 * blk + 8 * tq + 4 * h;
                    split_h2(mq[e0], mq[e0 + 1], qf[kk][0], qfl[kk][0]);
                    split_h2(mq[e0 + 2], mq[e0 + 3], qf[kk][1], qfl[kk][1]);
                }
                if constexpr (PK) {        // columns 4-7 carry the lo parts of heads 0-3
                    if (gq >= 4) {
                        qf[kk][0] = qfl[kk][0];
                        qf[kk][1] = qfl[kk][1];
                    }
                } else {
                    if (SPLIT == 2 && ring == 0) s_qfl[(half * NCH + kk) * 32 + lane] = make_uint2(qfl[kk][0], qfl[kk][1]);
                }
            }
            __syncthreads();   // q~ read by all warps before the scale scratch is reused
        }
        uint32_t bad_scale = 0;   // max |d| bits over the block scales seen

        // block-scale extraction of one tile into scratch xs: K -> f32 [row][blk], V -> f16 bits
        // [blk][row]; tokens past `valid` (stale or never-written stage bytes) get scale 0, which
        // only the last tile of a segment needs (FULL: all 16 tokens valid)
        auto extract = [&](uint32_t st, uint32_t xs, int valid, auto full_c) {
            constexpr bool FULL = decltype(full_c)::value;
            static_for<0, 2 * NXH>([&](auto r_c) {
                constexpr int r = decltype(r_c)::value;
                constexpr bool IS_V = r >= NXH;
                constexpr int rr = IS_V ? r - NXH : r;
                const uint32_t src = IS_V ? xvs + rr * TSTEP * VB : xks + rr * TSTEP * KB;
                uint16_t h;
                asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(st + src));
                if constexpr (!FULL) h = xt0 + rr * TSTEP < valid ? h : (uint16_t)0;
                // |d| >= 2^15 (|bits| >= 0x7800): exponent 31 decodes as a finite value in the reference but
                // as inf/nan in IEEE fp16, and P * d could overflow fp16: reported once per segment
                bad_scale = max(bad_scale, (uint32_t)(h & 0x7FFFu));
                if (!IS_V) {   // (the K codebook's 1/alpha is folded into the query scale)
                    const float f = __half2float(__ushort_as_half(h));
                    asm volatile("st.shared.f32 [%0], %1;" ::"r"(xs + xkd + rr * ROWSTEP * NBLK * 4), "f"(f));
                } else {
                    constexpr int VDELTA = (((rr * ROWSTEP) & 7) >> 1) * NBLK * 8 + ((rr * ROWSTEP) >> 3) * 4;
                    asm volatile("st.shared.u16 [%0], %1;" ::"r"(xs + xvd + VDELTA), "h"(h));
                }
            });
        };
        // S = K q~^T of one tile (block scales applied in fp32); tokens past `valid` -> -inf
        auto scores = [&](uint32_t st, uint32_t xs, int valid, float (&sc)[4]) {
            sc[0] = sc[1] = sc[2] = sc[3] = 0.0f;
            float dka[NBLK], dkb[NBLK];
            static_for<0, NBLK / 4>([&](auto c_c) {
                constexpr int c = decltype(c_c)::value;
                const float4 x = ld128f<c * 16>(xs + gq * NBLK * 4);
                const float4 y = ld128f<8 * NBLK * 4 + c * 16>(xs + gq * NBLK * 4);
                dka[4 * c] = x.x; dka[4 * c + 1] = x.y; dka[4 * c + 2] = x.z; dka[4 * c + 3] = x.w;
                dkb[4 * c] = y.x; dkb[4 * c + 1] = y.y; dkb[4 * c + 2] = y.z; dkb[4 * c + 3] = y.w;
            });
            // lo part of q~'s fragment for chunk kk: registers at head_dim 128, shared memory at 256
            auto qlo = [&](int kk) -> uint2 {
                if constexpr (SPLIT == 2) {
                    uint2 v;
                    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y)
                                 : "r"(smem_u32(s_qfl + (half * NCH + kk) * 32 + lane)));
                    return v;
                } else {
                    return make_uint2(qfl[kk][0], qfl[kk][1]);
                }
            };
            // the second mma of a chunk, with q~'s lo parts (groups above 4 only)
            auto lo_mma = [&](float (&acc)[4], const uint32_t (&af)[4], int kk) {
                if constexpr (!PK) {
                    const uint2 ql = qlo(kk);
                    mma16816(acc, af, ql.x, ql.y);
                }
            };
            static_for<0, NBLK>([&](auto blk_c) {
                constexpr int blk = decltype(blk_c)::value;
                float acc[4];
                uint32_t af[4];
                if constexpr (KT == 4 && (blk & 1)) {
                    const uint32_t kr = st + k_off_w;
                    const uint32_t w0 = ld32<blk * TQ4_BYTES>(kr), w1 = ld32<blk * TQ4_BYTES + KROW8>(kr);
                    af[0] = lut_ld<RES>(w0, lane4, LUT_SEL0);
                    af[1] = lut_ld<RES>(w1, lane4, LUT_SEL0);
                    af[2] = lut_ld<RES>(w0, lane4, LUT_SEL1);
                    af[3] = lut_ld<RES>(w1, lane4, LUT_SEL1);
                    mma16816_zc(acc, af, qf[2 * blk][0], qf[2 * blk][1]);
                    lo_mma(acc, af, 2 * blk);
                    af[0] = lut_ld<RES>(w0, lane4, LUT_SEL2);
                    af[1] = lut_ld<RES>(w1, lane4, LUT_SEL2);
                    af[2] = lut_ld<RES>(w0, lane4, LUT_SEL3);
                    af[3] = lut_ld<RES>(w1, lane4, LUT_SEL3);
                    mma16816(acc, af, qf[2 * blk + 1][0], qf[2 * blk + 1][1]);
                    lo_mma(acc, af, 2 * blk + 1);
                } else if constexpr (KT == 4) {
                    const uint32_t kr = st + k_off;
                    uint32_t w0 = ld16<blk * TQ4_BYTES>(kr), w1 = ld16<blk * TQ4_BYTES + KROW8>(kr);
                    af[0] = lut_ld<RES>(w0, lane4, LUT_SEL0);
                    af[1] = lut_ld<RES>(w1, lane4, LUT_SEL0);
                    af[2] = lut_ld<RES>(w0, lane4, LUT_SEL1);
                    af[3] = lut_ld<RES>(w1, lane4, LUT_SEL1);
                    mma16816_zc(acc, af, qf[2 * blk][0], qf[2 * blk][1]);
                    lo_mma(acc, af, 2 * blk);
                    w0 = ld16<blk * TQ4_BYTES + 8>(kr);
                    w1 = ld16<blk * TQ4_BYTES + 8 + KROW8>(kr);
                    af[0] = lut_ld<RES>(w0, lane4, LUT_SEL0);
                    af[1] = lut_ld<RES>(w1, lane4, LUT_SEL0);
                    af[2] = lut_ld<RES>(w0, lane4, LUT_SEL1);
                    af[3] = lut_ld<RES>(w1, lane4, LUT_SEL1);
                    mma16816(acc, af, qf[2 * blk + 1][0], qf[2 * blk + 1][1]);
                    lo_mma(acc, af, 2 * blk + 1);
                } else if constexpr (KT == 2) {
                    // TQ2 K: code bytes 2t, 2t+1 of the block hold elements 8t .. 8t+7, a nibble per
                    // element pair; the low nibbles become the bytes of nl, the high ones those of nh
                    const uint32_t kr = st + k_off;
                    const uint32_t w0 = ld16<blk * TQ2_BYTES>(kr), w1 = ld16<blk * TQ2_BYTES + KROW8>(kr);
                    const uint32_t nl0 = w0 & 0x0F0Fu, nh0 = (w0 >> 4) & 0x0F0Fu;
                    const uint32_t nl1 = w1 & 0x0F0Fu, nh1 = (w1 >> 4) & 0x0F0Fu;
                    af[0] = lut_ld<RES>(nl0, lane4x, LUT_SEL0);   // elements 8t, 8t+1 of row g
                    af[1] = lut_ld<RES>(nl1, lane4x, LUT_SEL0);   // of row g + 8
                    af[2] = lut_ld<RES>(nh0, lane4x, LUT_SEL0);   // elements 8t+2, 8t+3
                    af[3] = lut_ld<RES>(nh1, lane4x, LUT_SEL0);
                    mma16816_zc(acc, af, qf[2 * blk][0], qf[2 * blk][1]);
                    lo_mma(acc, af, 2 * blk);
                    af[0] = lut_ld<RES>(nl0, lane4x, LUT_SEL1);   // elements 8t+4, 8t+5
                    af[1] = lut_ld<RES>(nl1, lane4x, LUT_SEL1);
                    af[2] = lut_ld<RES>(nh0, lane4x, LUT_SEL1);   // elements 8t+6, 8t+7
                    af[3] = lut_ld<RES>(nh1, lane4x, LUT_SEL1);
                    mma16816(acc, af, qf[2 * blk + 1][0], qf[2 * blk + 1][1]);
                    lo_mma(acc, af, 2 * blk + 1);
                } else {
                    constexpr int IMM = blk * TQ3_BYTES - 2 * (blk & 1);
                    const uint32_t kr = st + ((blk & 1) ? k3_off_o : k3_off_e);
                    const uint32_t sh = (blk & 1) ? k3_sh_o : k3_sh_e;
                    const uint32_t wg = __funnelshift_r(ld32<IMM>(kr), ld32<IMM + 4>(kr), sh);
                    const uint32_t wh = __funnelshift_r(ld32<IMM + KROW8>(kr), ld32<IMM + KROW8 + 4>(kr), sh);
                    // head_dim 128 (table in all 256 rows): pair i read from a byte of a shifted word,
                    // pair 0 = byte 0 of w, 1 = byte 1 of w << 2, 2 = byte 1 of w >> 4, 3 = byte 2 of w >> 2
                    auto t3 = [&](auto i_c, uint32_t w) -> uint32_t {
                        constexpr int I = decltype(i_c)::value;
                        if constexpr (SPLIT == 2) return lut_ld_addr<RES>(tq3_lut_addr<I>(w, lane4x));
                        else if constexpr (I == 0) return lut_ld<RES>(w, lane4x, LUT_SEL0);
                        else if constexpr (I == 1) return lut_ld<RES>(w << 2, lane4x, LUT_SEL1);
                        else if constexpr (I == 2) return lut_ld<RES>(w >> 4, lane4x, LUT_SEL1);
                        else return lut_ld<RES>(w >> 2, lane4x, LUT_SEL2);
                    };
                    using I0 = std::integral_constant<int, 0>;
                    using I1 = std::integral_constant<int, 1>;
                    using I2 = std::integral_constant<int, 2>;
                    using I3 = std::integral_constant<int, 3>;
                    af[0] = t3(I0{}, wg);
                    af[1] = t3(I0{}, wh);
                    af[2] = t3(I1{}, wg);
                    af[3] = t3(I1{}, wh);
                    mma16816_zc(acc, af, qf[2 * blk][0], qf[2 * blk][1]);
                    lo_mma(acc, af, 2 * blk);
                    af[0] = t3(I2{}, wg);
                    af[1] = t3(I2{}, wh);
                    af[2] = t3(I3{}, wg);
                    af[3] = t3(I3{}, wh);
                    mma16816(acc, af, qf[2 * blk + 1][0], qf[2 * blk + 1][1]);
                    lo_mma(acc, af, 2 * blk + 1);
                }
                sc[0] = fmaf(dka[blk], acc[0], sc[0]);
                sc[1] = fmaf(dka[blk], acc[1], sc[1]);
                sc[2] = fmaf(dkb[blk], acc[2], sc[2]);
                sc[3] = fmaf(dkb[blk], acc[3], sc[3]);
            });
            if constexpr (PK) {   // head h's score = column h (hi) + column h + 4 (lo): lanes t and t ^ 2
#pragma unroll
                for (int i = 0; i < 4; ++i) sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 2);
            }
            if (valid < ATT_TILE) {
                if (Cfg::tok_of_row(gq) >= valid) { sc[0] = -INFINITY; sc[1] = -INFINITY; }
                if (Cfg::tok_of_row(gq + 8) >= valid) { sc[2] = -INFINITY; sc[3] = -INFINITY; }
            }
        };
        // O^T += V^T P' of one tile; pb01 / pb23 are the transposed P fragments
        auto accumulate = [&](uint32_t st, uint32_t xs, uint32_t pb01, uint32_t pb23) {
            const uint32_t vr = st + KTILE + v_off;
            const uint32_t sdv = xs + ATT_TILE * NBLK * 4 + tq * NBLK * 8;
            uint4 dvw;   // dV words of blocks blk, blk + 1: (rows 2t, 2t+1 | rows 2t+8, 2t+9) each
            static_for<0, NBLK>([&](auto blk_c) {
                constexpr int blk = decltype(blk_c)::value;
                const uint32_t w0 = ld16<blk * TQ4_BYTES>(vr), w1 = ld16<blk * TQ4_BYTES + VO1>(vr);
                const uint32_t w2 = ld16<blk * TQ4_BYTES + VO8>(vr), w3 = ld16<blk * TQ4_BYTES + VO9>(vr);
                // tokens A, B (k 2t, 2t+1) and C, D (k 2t+8, 2t+9), code bytes 0 and 1 each: the words
                // [A0 A1 C0 C1] and [B0 B1 D0 D1]; the codebook index of an element pair is (first
                // token's nibble | second token's nibble << 4), one bit-select per word gives four:
                // nlo = low nibbles (elements j, j+1 of the bytes), nhi = high nibbles (j+16, j+17)
                const uint32_t wac = prmt(w0, w2, 0x5410u), wbd = prmt(w1, w3, 0x5410u);
                const uint32_t nlo = (wac & 0x0F0F0F0Fu) | ((wbd << 4) & 0xF0F0F0F0u);
                const uint32_t nhi = ((wac >> 4) & 0x0F0F0F0Fu) | (wbd & 0xF0F0F0F0u);
                // TQ4 / TQ2 K: one 128-bit load per block pair; TQ3 K (more live offsets) one 64-bit load per block
                if constexpr (KT == 3) {
                    const uint2 d2 = ld64u<blk * 8>(sdv);
                    dvw.x = d2.x;
                    dvw.y = d2.y;
                } else if constexpr ((blk & 1) == 0) {
                    dvw = ld128u<blk * 8>(sdv);
                }
                const bool hi = KT != 3 && (blk & 1);
                const uint32_t b0 = h2_mul(pb01, hi ? dvw.z : dvw.x);
                const uint32_t b1 = h2_mul(pb23, hi ? dvw.w : dvw.y);
                uint32_t af[4];
                af[0] = lut_ld<RES>(nlo, lane4, LUT_SEL0);   // element 2g of tokens A, B
                af[1] = lut_ld<RES>(nhi, lane4, LUT_SEL0);   // element 2g + 16
                af[2] = lut_ld<RES>(nlo, lane4, LUT_SEL2);   // element 2g of tokens C, D
                af[3] = lut_ld<RES>(nhi, lane4, LUT_SEL2);
                mma16816(o[2 * blk], af, b0, b1);
                af[0] = lut_ld<RES>(nlo, lane4, LUT_SEL1);   // element 2g + 1
                af[1] = lut_ld<RES>(nhi, lane4, LUT_SEL1);   // element 2g + 17
                af[2] = lut_ld<RES>(nlo, lane4, LUT_SEL3);
                af[3] = lut_ld<RES>(nhi, lane4, LUT_SEL3);
                mma16816(o[2 * blk + 1], af, b0, b1);
            });
        };

        bool timed_out = false;
        for (int i0 = 0; i0 < ntiles && !timed_out; i0 += ATT_STAGES) {
            static_for<0, 2>([&](auto pair_c) {
                constexpr int SA = 2 * decltype(pair_c)::value, SB = SA + 1;
                const int ia = i0 + SA;
                if (ia >= ntiles || timed_out) return;
                const bool has_b = ia + 1 < ntiles;
                // the next pair goes into the stages the previous pair released
                issue_next(std::integral_constant<int, (SA + 2) % ATT_STAGES>{});
                issue_next(std::integral_constant<int, (SB + 2) % ATT_STAGES>{});
                // every lane waits; the outcome is made warp-uniform before any warp collective
                bool ok = mbar_wait(bar0 + 8 * SA, (phase_bits >> SA) & 1u);
                if (has_b) ok = ok && mbar_wait(bar0 + 8 * SB, (phase_bits >> SB) & 1u);
                ok = __all_sync(0xffffffffu, ok);
                // a pair leaves together: its partner learns the outcome at the score exchange below
                if constexpr (SPLIT == 1) {
                    if (!ok) {
                        timed_out = true;
                        return;
                    }
                    phase_bits ^= (1u << SA) | (has_b ? (1u << SB) : 0u);
                }
                const int valid_a = ia == ntiles - 1 ? last_valid : ATT_TILE;
                const int valid_b = !has_b ? 0 : (ia + 1 == ntiles - 1 ? last_valid : ATT_TILE);
                const uint32_t sta = stage0 + SA * STAGE, stb = stage0 + SB * STAGE;
                if (valid_a == ATT_TILE && valid_b == ATT_TILE) {
                    extract(sta, scr, valid_a, std::true_type{});
                    extract(stb, scr + SCR, valid_b, std::true_type{});
                } else {
                    extract(sta, scr, valid_a, std::false_type{});
                    extract(stb, scr + SCR, valid_b, std::false_type{});
                }
                __syncwarp();
                float sa[4], sb[4];
                scores(sta, scr, valid_a, sa);
                scores(stb, scr + SCR, valid_b, sb);
                if constexpr (SPLIT == 2) {
                    // add the partner warp's partial scores (the other 4 blocks of every token row),
                    // in the order half 0 + half 1 in both warps so both hold identical scores.  Slots:
                    // the upper halves of codebook-table rows 64 .. 191 (unused by both tables),
                    // 4 rows per (ring, half, tile), lanes 8k .. 8k+7 in row k.
                    auto slot = [&](int hh, int t) {
                        return smem_u32(smem) + ((64u + (uint32_t)(((ring * 2 + hh) * 2 + t) * 4) + (lane >> 3)) << 8) +
                               128u + ((uint32_t)(lane & 7) << 4);
                    };
                    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(slot(half, 0)), "f"(sa[0]), "f"(sa[1]),
                                 "f"(sa[2]), "f"(sa[3]) : "memory");
                    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(slot(half, 1)), "f"(sb[0]), "f"(sb[1]),
                                 "f"(sb[2]), "f"(sb[3]) : "memory");
                    if (lane == 0)   // this warp's wait outcome, beside the slots (row 192, upper half)
                        asm volatile("st.shared.u32 [%0], %1;" ::"r"(smem_u32(smem) + (192u << 8) + 128u +
                                                                      (uint32_t)(ring * 2 + half) * 4u),
                                     "r"((uint32_t)ok) : "memory");
                    pair_sync(ring);
                    uint32_t pok;
                    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(pok) : "r"(smem_u32(smem) + (192u << 8) + 128u +
                                                                         (uint32_t)(ring * 2 + (half ^ 1)) * 4u)
                                 : "memory");
                    float pa[4], pb[4];
                    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(pa[0]), "=f"(pa[1]), "=f"(pa[2]),
                                 "=f"(pa[3]) : "r"(slot(half ^ 1, 0)) : "memory");
                    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(pb[0]), "=f"(pb[1]), "=f"(pb[2]),
                                 "=f"(pb[3]) : "r"(slot(half ^ 1, 1)) : "memory");
                    pair_sync(ring);   // both partials read before the slots are written again
                    if (!(ok && pok != 0)) {
                        timed_out = true;
                        return;
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        sa[i] = half == 0 ? sa[i] + pa[i] : pa[i] + sa[i];
                        sb[i] = half == 0 ? sb[i] + pb[i] : pb[i] + sb[i];
                    }
                    phase_bits ^= (1u << SA) | (has_b ? (1u << SB) : 0u);
                }

                // ---- online softmax over the 32 tokens (log2 domain) ----
                float mx0 = fmaxf(fmaxf(sa[0], sa[2]), fmaxf(sb[0], sb[2]));
                float mx1 = fmaxf(fmaxf(sa[1], sa[3]), fmaxf(sb[1], sb[3]));
#pragma unroll
                for (int sh = 4; sh < 32; sh <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
                }
                // the running max moves only when a score exceeds it by more than one log2 unit,
                // so P <= 2 (scales of 2^15 and above are reported as unsupported)
                if (__any_sync(0xffffffffu, mx0 > m_run0 + 1.0f || mx1 > m_run1 + 1.0f)) {
                    const float mn0 = fmaxf(m_run0, mx0), mn1 = fmaxf(m_run1, mx1);
                    const float al0 = ex2(m_run0 - mn0), al1 = ex2(m_run1 - mn1);
                    m_run0 = mn0;
                    m_run1 = mn1;
#pragma unroll
                    for (int mt = 0; mt < NMT; ++mt) {
                        o[mt][0] *= al0; o[mt][1] *= al1; o[mt][2] *= al0; o[mt][3] *= al1;
                    }
                    l0 *= al0;
                    l1 *= al1;
                }
                const float pa0 = ex2(sa[0] - m_run0), pa1 = ex2(sa[1] - m_run1);
                const float pa2 = ex2(sa[2] - m_run0), pa3 = ex2(sa[3] - m_run1);
                const float pb0 = ex2(sb[0] - m_run0), pb1 = ex2(sb[1] - m_run1);
                const float pb2 = ex2(sb[2] - m_run0), pb3 = ex2(sb[3] - m_run1);
                l0 += (pa0 + pa2) + (pb0 + pb2);
                l1 += (pa1 + pa3) + (pb1 + pb3);
                accumulate(sta, scr, movmatrix_t(pack_h2(pa0, pa1)), movmatrix_t(pack_h2(pa2, pa3)));
                accumulate(stb, scr + SCR, movmatrix_t(pack_h2(pb0, pb1)), movmatrix_t(pack_h2(pb2, pb3)));
                __syncwarp();   // stages SA, SB and the scratch may be overwritten from here on
                if (SPLIT == 2 && half == 1 && lane == 0) {
                    mbar_arrive(ebar0 + 8 * SA);
                    if (has_b) mbar_arrive(ebar0 + 8 * SB);
                }
            });
        }
        if (timed_out) {
            // record the failure, drain this warp's copies still in flight (bounded), leave
            if (lane == 0) {
                atomicExch(a.err, (int)TQ_ERROR_TIMEOUT);
                *s_abort = 1;
            }
#pragma unroll
            for (int s2 = 0; s2 < ATT_STAGES; ++s2) mbar_wait(bar0 + 8 * s2, (phase_bits >> s2) & 1u);
            if (PG && issuer) asm volatile("cp.async.wait_all;" ::: "memory");
        }
        if (SPLIT == 2 && !timed_out && lane == 0 && half == 0) {
            // take the releases of the last tiles of the segment, which no refill waited for, so
            // that every release is waited exactly once and the parities stay in step
            for (int j = ntiles > ATT_STAGES ? ntiles - ATT_STAGES : 0; j < ntiles; ++j) {
                const int st = j % ATT_STAGES;
                if (!mbar_wait(ebar0 + 8 * st, (ephase_bits >> st) & 1u)) {
                    atomicExch(a.err, (int)TQ_ERROR_TIMEOUT);
                    *s_abort = 1;
                }
                ephase_bits ^= 1u << st;
            }
        }
        if (__any_sync(0xffffffffu, bad_scale >= 0x7800u) && lane == 0) atomicExch(a.err, (int)TQ_ERROR_UNSUPPORTED);

        // ---- merge the warps, write the (pair, slot) partial ----
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
            l1 += __shfl_xor_sync(0xffffffffu, l1, sh);
        }
        __syncthreads();   // all warps done with their stages; reuse them as merge scratch
        if (*s_abort) return;
        float* red = reinterpret_cast<float*>(stages);   // [ring][ATT_N][D + 2]
        float* mine = red + ring * ATT_N * (D + 2);
        if (gq == 0 && half == 0) {
            mine[(2 * tq) * (D + 2) + 0] = m_run0;
            mine[(2 * tq + 1) * (D + 2) + 0] = m_run1;
            mine[(2 * tq) * (D + 2) + 1] = l0;
            mine[(2 * tq + 1) * (D + 2) + 1] = l1;
        }
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt) {
            const int e0 = 128 * half + 32 * (mt >> 1) + 2 * gq + (mt & 1);
            mine[(2 * tq) * (D + 2) + 2 + e0] = o[mt][0];
            mine[(2 * tq + 1) * (D + 2) + 2 + e0] = o[mt][1];
            mine[(2 * tq) * (D + 2) + 2 + e0 + 16] = o[mt][2];
            mine[(2 * tq + 1) * (D + 2) + 2 + e0 + 16] = o[mt][3];
        }
        __syncthreads();
        // per query head: the maximum over the warps, then each warp's weight 2^(m_w - M)
        float* smax = reinterpret_cast<float*>(scratch);   // [ATT_N] (the scale scratch is free here)
        float* swt = smax + ATT_N;                          // [ATT_N][RINGS]
        if (threadIdx.x < ATT_N) {
            float M = M_FLOOR;
            for (int w = 0; w < RINGS; ++w) M = fmaxf(M, red[w * ATT_N * (D + 2) + threadIdx.x * (D + 2)]);
            smax[threadIdx.x] = M;
        }
        __syncthreads();
        if (threadIdx.x < ATT_N * RINGS) {
            const int h = threadIdx.x / RINGS, w = threadIdx.x % RINGS;
            swt[threadIdx.x] = ex2(red[w * ATT_N * (D + 2) + h * (D + 2)] - smax[h]);
        }
        __syncthreads();
        const size_t sstride = (size_t)ATT_N * (D + 2);
        const int64_t c_first = (pair * a.lnom) / a.chunk, c_last = ((pair + 1) * a.lnom - 1) / a.chunk;
        const int nslot = (int)(c_last - c_first + 1);
        // A pair inside this CTA's chunk (one slot) is finished from shared memory: no partial
        // through L2, no fence, no count.  The partial sits past the next segment's q~ staging in
        // the scale scratch, which nothing writes before the next segment's first barrier.
        // (head_dim 128: the scratch holds both; head_dim 256 pairs always go through L2.)
        constexpr int SOLO_OFF = ((ATT_N * (D + 4) * 4 + 127) / 128) * 128;
        constexpr bool SOLO_OK = SOLO_OFF + ATT_N * (D + 2) * 4 <= WARPS * 2 * SCR;
        const bool solo = SOLO_OK && nslot == 1;
        float* dst = solo ? reinterpret_cast<float*>(scratch + SOLO_OFF) : a.part + ((size_t)pair * a.slots + slot) * sstride;
        for (int idx = threadIdx.x; idx < ATT_N * (D + 2); idx += THREADS) {
            const int h = idx / (D + 2), c = idx % (D + 2);
            float acc = smax[h];
            if (c > 0) {
                acc = 0.0f;
                for (int w = 0; w < RINGS; ++w) acc += swt[h * RINGS + w] * red[w * ATT_N * (D + 2) + idx];
            }
            dst[idx] = acc;
        }
        // publish the partial, count this CTA in the pair; the stages are free for the next
        // segment's copies after this barrier
        if (!solo) __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_abort[1] = solo ? 1 : atomicAdd(a.cnt + pair, 1) == nslot - 1;
        __syncthreads();
        if (s_abort[1] && warp < a.grp) {
            // last CTA of the pair: log-sum-exp merge of the nslot partials of query head
            // hh = warp, inverse FWHT, cast; lse in natural log
            if (!solo) __threadfence();
            constexpr int EPL = D / 32;
            const float* p0 = solo ? dst + warp * (D + 2) : a.part + (size_t)pair * a.slots * sstride + warp * (D + 2);
            float M = M_FLOOR, L = 0.0f;
            float ov[EPL];
#pragma unroll
            for (int i = 0; i < EPL; ++i) ov[i] = 0.0f;
            for (int s = 0; s < nslot; ++s) M = fmaxf(M, part_ld(solo, p0 + s * sstride));
            for (int s = 0; s < nslot; ++s) L += ex2(part_ld(solo, p0 + s * sstride) - M) * part_ld(solo, p0 + s * sstride + 1);
            if (L > 0.0f)
                for (int s = 0; s < nslot; ++s) {
                    const float w = ex2(part_ld(solo, p0 + s * sstride) - M);
#pragma unroll
                    for (int i = 0; i < EPL; ++i) ov[i] += w * part_ld(solo, p0 + s * sstride + 2 + lane * EPL + i);
                }
            const bool empty = !(L > 0.0f);
            if (!empty) {
#pragma unroll
                for (int i = 0; i < EPL; ++i) ov[i] = ov[i] / L * (1.0f / TQ4_ALPHA);   // the V codebook's alpha
            }
            if (a.v_rotated) {
                fwht_warp_row<EPL>(ov, lane);
#pragma unroll
                for (int i = 0; i < EPL; ++i) ov[i] *= a.onorm;
            }
            const int64_t b = pair / a.Hkv, g = pair - b * a.Hkv;
            const size_t bh = (size_t)b * a.Hq + (size_t)g * a.grp + warp;
            const float lse_v = empty ? -INFINITY : (M + __log2f(L)) * 0.6931471805599453f;
            if (a.peer.world == 0) {
#pragma unroll
                for (int i = 0; i < EPL; ++i) store_out_rt(a.out, a.out_dtype, bh * D + lane * EPL + i, ov[i]);
                if (a.lse && lane == 0) a.lse[bh] = lse_v;
            } else {
                // split-sequence exchange: this rank's (o, lse) row goes into its slot of every rank's
                // exchange buffer (peer stores over NVLink), made visible system-wide before the count
                const int64_t slot = ((int64_t)a.peer.par * a.peer.world + a.peer.rank) * a.peer.slot_floats;
                for (int t = 0; t < a.peer.world; ++t) {
                    float* dst = reinterpret_cast<float*>(a.peer.base[t] + PEER_HEAD_BYTES) + slot;
                    static_assert(EPL % 4 == 0, "16-byte row stores");
#pragma unroll
                    for (int i = 0; i < EPL; i += 4)
                        *reinterpret_cast<float4*>(dst + bh * D + lane * EPL + i) =
                            make_float4(ov[i], ov[i + 1], ov[i + 2], ov[i + 3]);
                    if (lane == 0) dst[a.peer.n_rows * D + bh] = lse_v;
                }
            }
        }
        if (threadIdx.x == 0 && s_abort[1]) ++pairs_done;
    }
    if (a.peer.world != 0) {
        // Count this CTA's completed pairs once, at its end, in every rank's counter.  The rows of
        // early pairs have been travelling over NVLink since those pairs finished; the barrier and
        // the cumulative system-scope fence of thread 0 order every thread's row stores before the
        // counts, so a rank that sees all counts reads complete rows.
        __syncthreads();
        if (threadIdx.x == 0 && pairs_done) {
            __threadfence_system();
            for (int t = 0; t < a.peer.world; ++t)
                atomicAdd_system(reinterpret_cast<unsigned long long*>(a.peer.base[t]), (unsigned long long)pairs_done);
        }
    }
}

// ── multi-rank log-sum-exp merge ───────────────────────────────────────────────

// merge of P partial results (natural-log lse), e.g. from several ranks; part p at o + p * o_stride,
// lse + p * lse_stride; one warp per row (merge_row, shared with the peer-memory merge kernels)
constexpr int COMBINE_WARPS = 8;
template <typename OT>
__global__ void __launch_bounds__(COMBINE_WARPS * 32) lse_combine_kernel(const float* __restrict__ o, int64_t o_stride,
                                                                        const float* __restrict__ lse, int64_t lse_stride,
                                                                        OT* __restrict__ out, float* __restrict__ lse_out,
                                                                        int P, int64_t n, int D) {
    const int64_t i = (int64_t)blockIdx.x * COMBINE_WARPS + (threadIdx.x >> 5);
    if (i < n) merge_row<OT>(o, o_stride, lse, lse_stride, P, i, D, out, lse_out, threadIdx.x & 31);
}

// ── host side ───────────────────────────────────────────────────────────────

template <int D, int KT>
static size_t decode_smem_bytes() {
    using Cfg = AttnCfg<D, KT>;
    size_t s = LUT_BYTES;
    const size_t stg = (size_t)Cfg::RINGS * ATT_STAGES * Cfg::STAGE;
    const size_t red = (size_t)Cfg::RINGS * ATT_N * (D + 2) * 4;   // ring merge scratch reuses the stages
    s += stg > red ? stg : red;
    s += (size_t)Cfg::WARPS * 2 * Cfg::SCR;
    s += (size_t)Cfg::RINGS * ATT_STAGES * 8;
    s += (size_t)Cfg::EBARS * 8;
    s += 16;                                                        // s_abort
    if (Cfg::SPLIT == 2) s += (size_t)2 * Cfg::NCH * 32 * 8;        // s_qfl
    s += (size_t)Cfg::RINGS * ATT_STAGES * 4;                       // page slots (paged caches)
    return s;
}

AttnPlan attn_plan(int B, int Hkv, int D, int64_t cap, int64_t max_len) {
    AttnPlan p;
    const int64_t pairs = (int64_t)B * Hkv;
    const int64_t len = max_len > 0 ? max_len : cap;
    p.lnom = (len + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
    if (p.lnom == 0) p.lnom = ATT_TILE;
    const int64_t total = pairs * p.lnom;
    const int64_t unit = (int64_t)att_rings(D) * ATT_TILE;   // one tile per ring
    const int sms = sm_count();
    int64_t chunk = (total + sms - 1) / sms;
    chunk = (chunk + unit - 1) / unit * unit;
    if (chunk < unit) chunk = unit;
    p.chunk = chunk;
    p.grid = (int)((total + chunk - 1) / chunk);
    p.slots = (int)((p.lnom + chunk - 1) / chunk + 1);
    return p;
}

// workspace: error word | per-pair CTA counters (cleared together before each launch) | partials
static size_t attn_counters_end(size_t pairs) { return 256 + pairs * sizeof(int); }

size_t attn_workspace_bytes(int B, int Hkv, int D, const AttnPlan& p) {
    const size_t pairs = (size_t)B * Hkv;
    size_t bytes = (attn_counters_end(pairs) + 255) & ~size_t(255);
    bytes += pairs * p.slots * ATT_N * (D + 2) * sizeof(float);   // split partials
    return bytes;
}

static int reserved_smem() {
    static int cached[64];
    static bool init[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!init[dev]) {
        int v = -1;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess) v = -1;
        cached[dev] = v;
        init[dev] = true;
    }
    return cached[dev];
}

template <int D, int KT, int RES, bool PK, bool PG>
static cudaError_t launch_decode_kernel(const AttnKernelArgs& a, int grid, cudaStream_t st) {
    const size_t smem = decode_smem_bytes<D, KT>();
    // the shared-memory opt-in is set once per device, so that later calls (for example
    // inside a CUDA graph capture) issue only stream work
    static bool attr_set[64] = {};   // one per instantiation
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(attn_decode_kernel<D, KT, RES, PK, PG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    attn_decode_kernel<D, KT, RES, PK, PG><<<grid, AttnCfg<D, KT>::THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

template <int D, int RES, bool PG>
static cudaError_t launch_decode_kt(const AttnKernelArgs& a, int k_type, int grid, cudaStream_t st) {
    if (a.grp <= 4)
        return k_type == 4   ? launch_decode_kernel<D, 4, RES, true, PG>(a, grid, st)
               : k_type == 3 ? launch_decode_kernel<D, 3, RES, true, PG>(a, grid, st)
                             : launch_decode_kernel<D, 2, RES, true, PG>(a, grid, st);
    return k_type == 4   ? launch_decode_kernel<D, 4, RES, false, PG>(a, grid, st)
           : k_type == 3 ? launch_decode_kernel<D, 3, RES, false, PG>(a, grid, st)
                         : launch_decode_kernel<D, 2, RES, false, PG>(a, grid, st);
}

template <int D>
static cudaError_t run_decode(const AttnRun& r, const AttnPlan& p, uint8_t* ws, cudaStream_t st) {
    const size_t pairs = (size_t)r.B * r.Hkv;
    const size_t cnt_end = attn_counters_end(pairs);
    cudaError_t e = cudaMemsetAsync(ws, 0, cnt_end, st);
    if (e != cudaSuccess) return e;
    AttnKernelArgs a;
    a.q = r.q;
    a.k = (const uint8_t*)r.k;
    a.v = (const uint8_t*)r.v;
    a.kv_len = r.kv_len;
    a.part = reinterpret_cast<float*>(ws + ((cnt_end + 255) & ~size_t(255)));
    a.err = reinterpret_cast<int*>(ws);
    a.cnt = reinterpret_cast<int*>(ws + 256);
    a.out = r.out;
    a.lse = r.lse;
    a.cap = r.cap;
    a.lnom = p.lnom;
    a.chunk = p.chunk;
    // q~ = FWHT(q) / sqrt(D) * sm_scale * log2(e): the FWHT normalisation folds into the scale
    // K codebook tables hold alpha * level (alpha chosen for the fp16 rounding of the levels): 1/alpha
    // joins the query scale
    a.qscale = r.sm_scale * LOG2E * (r.rotate_q ? fwht_norm(D) : 1.0f) /
               (r.k_type == 4 ? TQ4_ALPHA : r.k_type == 3 ? TQ3_ALPHA : TQ2_ALPHA);
    a.onorm = fwht_norm(D);
    a.B = r.B;
    a.Hq = r.Hq;
    a.Hkv = r.Hkv;
    a.grp = r.grp;
    a.slots = p.slots;
    a.q_dtype = r.q_dtype;
    a.out_dtype = r.out_dtype;
    a.rotate_q = r.rotate_q;
    a.v_rotated = r.v_rotated;
    a.peer = r.peer;
    a.pages = r.pages;
    a.max_pages = r.max_pages;
    a.num_pages = r.num_pages;
    a.page_shift = r.page_shift;
    a.page_mask = (1u << r.page_shift) - 1u;
    {
        const uint32_t rows = (uint32_t)r.Hkv << r.page_shift;
        const uint32_t kbb = r.k_type == 4 ? TQ4_BYTES : r.k_type == 3 ? TQ3_BYTES : TQ2_BYTES;
        a.page_kbytes = rows * (uint32_t)(D / 32) * kbb;
        a.page_vbytes = rows * (uint32_t)(D / 32) * TQ4_BYTES;
    }
    // the codebook table sits at the start of the shared window, an instruction immediate: B200
    // reserves 1 KB of every CTA's shared memory below it
    if (reserved_smem() != 1024) return cudaErrorNotSupported;
    return r.pages ? launch_decode_kt<D, 1024, true>(a, r.k_type, p.grid, st)
                   : launch_decode_kt<D, 1024, false>(a, r.k_type, p.grid, st);
}

cudaError_t launch_decode_attention(const AttnRun& r, const AttnPlan& p, void* workspace, cudaStream_t st) {
    if (r.v_type != 4 || r.k_type < 2 || r.k_type > 4) return cudaErrorInvalidValue;
    if (r.D == 128) return run_decode<128>(r, p, (uint8_t*)workspace, st);
    if (r.D == 256) return run_decode<256>(r, p, (uint8_t*)workspace, st);
    return cudaErrorInvalidValue;
}

cudaError_t launch_lse_combine(const float* o, int64_t o_stride, const float* lse, int64_t lse_stride, void* out,
                               int out_dtype, float* lse_out, int P, int64_t n, int D, cudaStream_t st) {
    const int64_t rows_per_launch = (int64_t(1) << 30) * COMBINE_WARPS;   // grid.x limit
    for (int64_t r0 = 0; r0 < n; r0 += rows_per_launch) {
        const int64_t nr = n - r0 < rows_per_launch ? n - r0 : rows_per_launch;
        const unsigned grid = (unsigned)((nr + COMBINE_WARPS - 1) / COMBINE_WARPS);
        const float* oo = o + r0 * D;
        const float* ll = lse + r0;
        float* lo = lse_out ? lse_out + r0 : nullptr;
        switch (out_dtype) {
            case DT_F32:
                lse_combine_kernel<float><<<grid, COMBINE_WARPS * 32, 0, st>>>(oo, o_stride, ll, lse_stride,
                                                                               (float*)out + r0 * D, lo, P, nr, D);
                break;
            case DT_F16:
                lse_combine_kernel<__half><<<grid, COMBINE_WARPS * 32, 0, st>>>(oo, o_stride, ll, lse_stride,
                                                                                (__half*)out + r0 * D, lo, P, nr, D);
                break;
            default:
                lse_combine_kernel<__nv_bfloat16><<<grid, COMBINE_WARPS * 32, 0, st>>>(
                    oo, o_stride, ll, lse_stride, (__nv_bfloat16*)out + r0 * D, lo, P, nr, D);
                break;
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace tq
