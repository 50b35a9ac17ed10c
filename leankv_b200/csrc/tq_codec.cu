// tq_codec.cu — fused Walsh-Hadamard + TurboQuant block codecs for sm_100a.
//
// Kernels
//   quantize_kernel<QT, IN, MODE>  [FWHT per head] + TQ3_0 / TQ4_0 quantize
//                                  (src/ggml-tq.c:215-247, :273-304 after
//                                  hadamard_transform_row, :361-404), with the
//                                  TQ3 optimal-rounding refinement
//                                  (scripts/tq3_rounding.py:74-125) as MODE
//   fwht_kernel                    hadamard_transform_row in place on fp32
//   dequantize_kernel<QT, OUT>     dequantize_row_tq{3,4}_0 (:249-265, :306-321)
//
// Layout of work (quantize / FWHT): one thread owns one 32-element block, so
// a head of D elements is D/32 consecutive lanes.  A CTA of 128 threads moves
// a tile of 128 blocks: coalesced 16-byte global loads into an XOR-swizzled
// shared tile (conflict-free both for the row-major fill and for the
// per-thread row reads), FWHT stages h = 1..16 in registers, stages h >= 32 by
// warp shuffles between the lanes of a head, then amax / scale / nearest
// level / packing in registers, and a byte-exact staging of the 18- or 14-byte
// blocks in shared memory so the global stores are again 16-byte coalesced.
//
// Bit-exactness with the reference: the butterfly stages run in the
// reference's order (h ascending) with the same (a + b, a - b) operations; the
// 1/sqrt(D) factor is computed on the host with the reference's expression;
// the reciprocal is the IEEE division 1.0f / amax; the build uses no fast-math
// so every fp32 operation is correctly rounded and denormals are kept.
#include <type_traits>
#include <utility>

#include "tq_common.cuh"
#include "tq_kernels.h"
#include "tq_outlier.h"

namespace tq {

constexpr int CODEC_THREADS = 128;   // blocks per tile

// ── shared-memory tile addressing ───────────────────────────────────────────
// A tile row is one 32-element block: 128 B (fp32) or 64 B (16-bit input).
// Chunk q (16 B) of row r is stored at chunk position q ^ swz(r) so that the
// 8 lanes of a 128-bit shared-memory phase hit 8 distinct bank groups both
// when a warp fills consecutive chunks and when each lane reads its own row.
template <int ROW_BYTES>
__device__ __forceinline__ int tile_chunk_addr(int r, int q) {
    constexpr int CPR = ROW_BYTES / 16;               // chunks per row: 8 or 4
    const int swz = CPR == 8 ? (r & 7) : ((r >> 1) & 3);
    return r * ROW_BYTES + ((q ^ swz) << 4);
}

// cooperative tile load: rows [0, nrows) of 32 elements each
template <typename IN>
__device__ __forceinline__ void load_tile(uint8_t* __restrict__ smem, const IN* __restrict__ src,
                                          int nrows, bool vec_ok) {
    constexpr int EB = ElemBits<IN>::bytes;
    constexpr int ROW_BYTES = QK * EB;
    constexpr int CPR = ROW_BYTES / 16;
    if (vec_ok) {
        const int4* s4 = reinterpret_cast<const int4*>(src);
        for (int c = threadIdx.x; c < nrows * CPR; c += CODEC_THREADS) {
            const int4 v = __ldg(s4 + c);
            *reinterpret_cast<int4*>(smem + tile_chunk_addr<ROW_BYTES>(c / CPR, c % CPR)) = v;
        }
    } else {
        // element-wise fallback for inputs that are not 16-byte aligned
        const uint8_t* sb = reinterpret_cast<const uint8_t*>(src);
        for (int e = threadIdx.x; e < nrows * QK; e += CODEC_THREADS) {
            const int r = e / QK, c = e % QK;
            const int byte = c * EB;
            uint8_t* dst = smem + tile_chunk_addr<ROW_BYTES>(r, byte >> 4) + (byte & 15);
            if (EB == 4) {
                uint32_t w;
                memcpy(&w, sb + (size_t)e * 4, 4);
                *reinterpret_cast<uint32_t*>(dst) = w;
            } else {
                uint16_t w;
                memcpy(&w, sb + (size_t)e * 2, 2);
                *reinterpret_cast<uint16_t*>(dst) = w;
            }
        }
    }
}

// asynchronous tile load (16-byte aligned input): each thread issues cp.async copies of
// its chunks straight into the swizzled tile; completion is awaited with cp_async_wait
template <typename IN>
__device__ __forceinline__ void load_tile_async(uint8_t* __restrict__ smem, const IN* __restrict__ src, int nrows) {
    constexpr int ROW_BYTES = QK * ElemBits<IN>::bytes;
    constexpr int CPR = ROW_BYTES / 16;
    const char* s8 = reinterpret_cast<const char*>(src);
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
    if (nrows == CODEC_THREADS) {
#pragma unroll
        for (int i = 0; i < CPR; ++i) {
            const int c = threadIdx.x + i * CODEC_THREADS;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sbase + tile_chunk_addr<ROW_BYTES>(c / CPR, c % CPR)),
                         "l"(s8 + 16 * (size_t)c)
                         : "memory");
        }
    } else {
        for (int c = threadIdx.x; c < nrows * CPR; c += CODEC_THREADS)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sbase + tile_chunk_addr<ROW_BYTES>(c / CPR, c % CPR)),
                         "l"(s8 + 16 * (size_t)c)
                         : "memory");
    }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Programmatic dependent launch.  The quantize and dequantize kernels are launched with
// programmatic stream serialization: the next such kernel on the stream may start while this
// one runs (trigger at entry), does its setup, and waits for the whole previous grid to
// complete, with its memory visible, before its first global access (read or write).  Without
// the launch attribute both instructions are no-ops.
__device__ __forceinline__ void grid_dep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static cudaError_t launch_dependent(void (*kernel)(KArgs...), unsigned grid, unsigned block, cudaStream_t st,
                                    Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// thread-private read of row r as 32 floats (exact conversion from 16-bit)
template <typename IN>
__device__ __forceinline__ void read_row(const uint8_t* __restrict__ smem, int r, float (&v)[QK]) {
    constexpr int EB = ElemBits<IN>::bytes;
    constexpr int ROW_BYTES = QK * EB;
    constexpr int CPR = ROW_BYTES / 16;
#pragma unroll
    for (int q = 0; q < CPR; ++q) {
        const uint4 w = *reinterpret_cast<const uint4*>(smem + tile_chunk_addr<ROW_BYTES>(r, q));
        if constexpr (EB == 4) {
            v[4 * q + 0] = __uint_as_float(w.x);
            v[4 * q + 1] = __uint_as_float(w.y);
            v[4 * q + 2] = __uint_as_float(w.z);
            v[4 * q + 3] = __uint_as_float(w.w);
        } else {
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t lo = ws[i] & 0xFFFFu, hi = ws[i] >> 16;
                if constexpr (std::is_same<IN, __nv_bfloat16>::value) {
                    v[8 * q + 2 * i] = bf16_bits_to_float(lo);
                    v[8 * q + 2 * i + 1] = bf16_bits_to_float(hi);
                } else {
                    v[8 * q + 2 * i] = f16_bits_to_float(lo);
                    v[8 * q + 2 * i + 1] = f16_bits_to_float(hi);
                }
            }
        }
    }
}

// ── Walsh-Hadamard transform of one head spread over D/32 lanes ─────────────
// Stage h combines elements j and j+h as (x[j] + x[j+h], x[j] - x[j+h]),
// h = 1, 2, 4, ... (src/ggml-tq.c:365-374), then scales by norm.
// L2 >= -1 fixes log2(head_dim) at compile time (-1: no rotation), so every stage
// unrolls without branches; L2 = -2 reads it from log2_hd at run time.
template <int L2 = -2>
__device__ __forceinline__ void fwht_block(float (&v)[QK], int log2_hd_rt, float norm) {
    const int log2_hd = L2 >= -1 ? L2 : log2_hd_rt;
    // Packed fp32x2 adds: every lane of an f32x2 operation is an ordinary
    // round-to-nearest fp32 operation, and a - b is computed as fma(b, -1, a)
    // (b * -1 is exact, one rounding), so the results equal the scalar code.
    // Register pairs are (v[2i], v[2i+1]) for every packed stage, so no stage needs moves;
    // h = 1 combines the two halves of a pair and runs as scalar operations.
    const float2 m1 = make_float2(-1.0f, -1.0f);
    if (log2_hd >= 1) {
#pragma unroll
        for (int j = 0; j < QK; j += 2) {
            const float a = v[j], b = v[j + 1];
            v[j] = __fadd_rn(a, b);
            v[j + 1] = __fmaf_rn(b, -1.0f, a);
        }
    }
#pragma unroll
    for (int s = 1; s < 5; ++s) {   // h = 2 .. 16: elements j, j+1 share the stage's lower half
        if (s < log2_hd) {
            const int h = 1 << s;
#pragma unroll
            for (int j = 0; j < QK; j += 2) {
                if (j & h) continue;
                const float2 a = make_float2(v[j], v[j + 1]), b = make_float2(v[j + h], v[j + h + 1]);
                const float2 sum = __fadd2_rn(a, b), dif = __ffma2_rn(b, m1, a);
                v[j] = sum.x; v[j + 1] = sum.y; v[j + h] = dif.x; v[j + h + 1] = dif.y;
            }
        }
    }
#pragma unroll
    for (int s = 5; s < (L2 >= -1 ? (L2 > 5 ? L2 : 5) : log2_hd); ++s) {   // h >= 32: partner lane = lane ^ (h / 32)
        const int lane_bit = 1 << (s - 5);
        // lower element: self + partner = fma(self, 1, partner); upper: partner - self = fma(self, -1, partner)
        const float sg = (threadIdx.x & lane_bit) ? -1.0f : 1.0f;
        const float2 sg2 = make_float2(sg, sg);
#pragma unroll
        for (int j = 0; j < QK; j += 2) {
            const float p0 = __shfl_xor_sync(0xffffffffu, v[j], lane_bit);
            const float p1 = __shfl_xor_sync(0xffffffffu, v[j + 1], lane_bit);
            const float2 r = __ffma2_rn(make_float2(v[j], v[j + 1]), sg2, make_float2(p0, p1));
            v[j] = r.x; v[j + 1] = r.y;
        }
    }
    if (log2_hd >= 0) {
        const float2 n2 = make_float2(norm, norm);
#pragma unroll
        for (int j = 0; j < QK; j += 2) {
            const float2 r = __fmul2_rn(make_float2(v[j], v[j + 1]), n2);
            v[j] = r.x; v[j + 1] = r.y;
        }
    }
}

// ── block staging (byte-exact reference layout) ──────────────────────────────
// Write `nbytes` (18 or 14) bytes made of the fp16 scale and the packed codes
// words[] (little endian) at smem + off, where off is even.
template <int NB>
__device__ __forceinline__ void stage_block(uint8_t* __restrict__ smem, int off, uint16_t d,
                                            const uint32_t (&w)[NB]) {
    // byte stream: d_lo d_hi q0 q1 ... ; off % 4 is 0 or 2
    if ((off & 2) == 0) {
        // [d | q0 q1] [q2..q5] ...
        *reinterpret_cast<uint32_t*>(smem + off) = (uint32_t)d | (w[0] << 16);
#pragma unroll
        for (int i = 1; i < NB; ++i)
            *reinterpret_cast<uint32_t*>(smem + off + 4 * i) = (w[i - 1] >> 16) | (w[i] << 16);
        *reinterpret_cast<uint16_t*>(smem + off + 4 * NB) = (uint16_t)(w[NB - 1] >> 16);
    } else {
        *reinterpret_cast<uint16_t*>(smem + off) = d;
#pragma unroll
        for (int i = 0; i < NB; ++i) *reinterpret_cast<uint32_t*>(smem + off + 2 + 4 * i) = w[i];
    }
}

// cooperative copy of nbytes from shared staging to global by threads t0, t0 + stride, ...
// (the whole CTA by default, one warp with t0 = lane, stride = 32)
__device__ __forceinline__ void store_staged(uint8_t* __restrict__ dst, const uint8_t* __restrict__ smem,
                                             int nbytes, bool vec_ok, int t0 = threadIdx.x,
                                             int stride = CODEC_THREADS) {
    if (vec_ok && (nbytes & 15) == 0) {
        int4* d4 = reinterpret_cast<int4*>(dst);
        const int4* s4 = reinterpret_cast<const int4*>(smem);
        for (int c = t0; c < nbytes / 16; c += stride) d4[c] = s4[c];
    } else {
        for (int b = t0; b < nbytes; b += stride) dst[b] = smem[b];
    }
}

// Head rows of a tile written into a KV cache: head row R of the input (R =
// s * n_new + t, s = sequence * Hkv + head) goes to token slot pos[sequence] + t
// of s in a [s][cap][row_bytes] cache.  dst[] holds each row's byte offset
// (-1: slot outside the cache, not written).  Copies use the widest word that
// divides the row size (rows and the cache start are 16-byte aligned otherwise).
template <typename W>
__device__ __forceinline__ void copy_rows(uint8_t* __restrict__ y, const uint8_t* __restrict__ smem,
                                          const int64_t* __restrict__ dst, int nr, int row_bytes,
                                          int t0 = threadIdx.x, int stride = CODEC_THREADS) {
    const int wpr = row_bytes / (int)sizeof(W);
    for (int c = t0; c < nr * wpr; c += stride) {
        const int r = c / wpr, w = c - r * wpr;
        const int64_t off = dst[r];
        if (off >= 0)
            reinterpret_cast<W*>(y + off)[w] = reinterpret_cast<const W*>(smem + r * row_bytes)[w];
    }
}

// Destination of each head row of the tile starting at block b0 (threads < rows of the tile;
// the caller's next block-wide barrier publishes s_dst).  A head row holds nblk blocks, a power
// of two; rows and sequences are divided in 32 bits whenever every row index fits.
__device__ __forceinline__ void map_rows(int64_t* __restrict__ s_dst, int64_t b0, int nrows, int bb,
                                         const RowMap& map) {
    const int nb = map.nblk, row_bytes = nb * bb, lnb = __ffs(nb) - 1, nr = nrows >> lnb;
    if (threadIdx.x < nr) {
        const int64_t R = (b0 >> lnb) + threadIdx.x, R1 = (b0 >> lnb) + nr - 1;   // this row, the tile's last
        int64_t sh, t, seq, sh1;
        if (R1 < (int64_t(1) << 31) && map.n_new < (int64_t(1) << 31)) {
            const uint32_t r32 = (uint32_t)R, n32 = (uint32_t)map.n_new, sh32 = r32 / n32;
            sh = sh32;
            t = r32 - sh32 * n32;
            seq = sh32 / (uint32_t)map.hkv;
            sh1 = (uint32_t)R1 / n32;
        } else {
            sh = R / map.n_new;
            t = R - sh * map.n_new;
            seq = sh / map.hkv;
            sh1 = R1 / map.n_new;
        }
        const int64_t slot = (map.pos ? (int64_t)map.pos[seq] : 0) + t;
        int64_t off = -1;
        int64_t run_end = map.cap;   // the slots [slot, run_end) are consecutive in memory
        if (slot >= 0 && slot < map.cap) {
            if (map.pages) {
                const int32_t pg = map.pages[seq * map.max_pages + (slot >> map.page_shift)];
                const int64_t in_page = slot & ((int64_t(1) << map.page_shift) - 1);
                if ((uint64_t)(int64_t)pg < (uint64_t)map.num_pages)
                    off = ((((int64_t)pg * map.hkv + (sh - seq * map.hkv)) << map.page_shift) + in_page) * row_bytes;
                run_end = slot - in_page + (int64_t(1) << map.page_shift);
            } else {
                off = (sh * map.cap + slot) * row_bytes;
            }
        }
        if (off < 0 && map.overflow) atomicAdd(map.overflow, 1);
        s_dst[threadIdx.x] = off;
        if (threadIdx.x == 0) {
            // the whole tile lands in consecutive slots of one (sequence, head) when its last
            // row belongs to the same (sequence, head) and still fits (in the same page)
            s_dst[CODEC_THREADS] = (off >= 0 && sh1 == sh && slot + (nr - 1) < run_end) ? 1 : 0;
        }
    }
}

// Staged head rows stored to the rows map_rows() placed (s_dst published by an earlier barrier):
// the whole tile by all threads (t0 = threadIdx.x, stride = CODEC_THREADS, part ignored), or
// warp `part`'s 32 blocks (32 / nblk whole head rows) by its lanes (t0 = lane, stride = 32).
__device__ __forceinline__ void store_mapped_warp(uint8_t* __restrict__ y, const uint8_t* __restrict__ smem,
                                                  const int64_t* __restrict__ s_dst, int nrows, int bb,
                                                  const RowMap& map, bool y_vec, int part, int t0, int stride) {
    const int nb = map.nblk, row_bytes = nb * bb, nr = nrows / nb;
    const int rpw = stride == CODEC_THREADS ? nr : 32 / nb;
    const int r0 = stride == CODEC_THREADS ? 0 : part * rpw, r1 = nr < r0 + rpw ? nr : r0 + rpw;
    if (r0 >= r1) return;
    const uint8_t* src = smem + r0 * row_bytes;
    if (s_dst[CODEC_THREADS]) {
        uint8_t* dst = y + s_dst[0] + (int64_t)r0 * row_bytes;
        store_staged(dst, src, (r1 - r0) * row_bytes, y_vec && (((uintptr_t)dst) & 15) == 0, t0, stride);
    } else if ((row_bytes & 7) == 0) {
        copy_rows<uint2>(y, src, s_dst + r0, r1 - r0, row_bytes, t0, stride);
    } else if ((row_bytes & 3) == 0) {
        copy_rows<uint32_t>(y, src, s_dst + r0, r1 - r0, row_bytes, t0, stride);
    } else {
        copy_rows<uint16_t>(y, src, s_dst + r0, r1 - r0, row_bytes, t0, stride);
    }
}

// ── TQ3 optimal rounding (scripts/tq3_rounding.py:74-125) ───────────────────
// Coordinate descent over adjacent levels with a least-squares scale.  For an
// assignment with C = sum x*L and A = sum L^2 the least-squares block MSE is
// (sum x^2 - C^2 / A) / 32, so moving element j by (dL, dLL = L'^2 - L^2)
// improves the MSE ("new_mse < best_mse") exactly when
//     T = A * p * (p + 2C) - C^2 * dLL > 0,   p = x_j * dL
// (that is C'^2 * A > C^2 * A' with C' = C + p, A' = A + dLL).  The levels are
// the float64 decimals of the Python prototype.
//
// Per code i: {dL down, dLL down} and {dL up, dLL up} (a missing neighbour holds zeros and is
// never accepted), replicated 8 times as rep[(2 i + half) * 8 + lane % 8]: a 16-byte load is
// served a quarter warp (8 lanes) at a time, and those 8 lanes read 8 different 16-byte slots,
// so the lane-dependent lookups are free of bank conflicts.
struct Tq3OptTables {
    double2 rep[8 * 2 * 8];
    double lv[8];      // float64 levels
};

__device__ __forceinline__ uint32_t code_of(const uint32_t (&g)[4], int j) {   // code j of the group words
    return (g[j >> 3] >> (3 * (j & 7))) & 7u;
}

// Float64 coordinate descent on codes held in registers (one int per element).
// Each element-step evaluates both neighbours from one table entry (dL, dLL for
// the lower and upper level) with the incremental form of the exact test and
// accepts the first strict improvement.
__device__ __forceinline__ double tq3_opt_refine(const float (&v)[QK], uint32_t (&g)[4], int n_passes,
                                                 const Tq3OptTables* __restrict__ t) {
    const int lane8 = threadIdx.x & 7;
    int idx[QK];
#pragma unroll
    for (int j = 0; j < QK; ++j) idx[j] = (int)code_of(g, j);
    double A = 0.0, C = 0.0;
#pragma unroll
    for (int j = 0; j < QK; ++j) {
        const double l = t->lv[idx[j]];
        A = fma(l, l, A);
        C = fma((double)v[j], l, C);
    }
    double E = C * C;
    for (int pass = 0; pass < n_passes; ++pass) {
        bool improved = false;
#pragma unroll
        for (int j = 0; j < QK; ++j) {
            const int i = idx[j];
            const double2 ed = t->rep[(2 * i) * 8 + lane8], eu = t->rep[(2 * i + 1) * 8 + lane8];
            const double4 e = make_double4(ed.x, ed.y, eu.x, eu.y);   // dL down, dLL down, dL up, dLL up
            const double xd = (double)v[j];
            const double Cd = fma(xd, e.x, C), Ad = A + e.y;
            const double Cu = fma(xd, e.z, C), Au = A + e.w;
            // A missing neighbour (code 0 down, code 7 up) has dL = dLL = 0, so its test reads
            // (C * C) * A > E * A with E == C * C bit for bit, which is false: no range check.
            const bool acc_dn = Cd * Cd * A > E * Ad;          // lower neighbour first
            const bool acc_up = !acc_dn && Cu * Cu * A > E * Au;
            C = acc_dn ? Cd : (acc_up ? Cu : C);
            A = acc_dn ? Ad : (acc_up ? Au : A);
            E = C * C;   // the accepted Cd * Cd (or Cu * Cu), or the unchanged C * C
            idx[j] = i + (int)acc_up - (int)acc_dn;
            improved |= acc_dn | acc_up;
        }
        if (!improved) break;
    }
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) w |= (uint32_t)idx[8 * gi + i] << (3 * i);
        g[gi] = w;
    }
    return A == 0.0 ? 0.0 : C / A;
}

// ── nearest level by table ─────────────────────────────────────────────────
// bin(xn) = round(16 xn + 16) is the low 6 mantissa bits of fma(xn, 16, 1.5 * 2^23 + 16)
// (one ulp is 1 at that magnitude, and round-to-nearest is monotone in xn).  Each
// boundary B_k has a bin too; for every bin j the table holds
//   cnt_j = #{k : bin(B_k) < j}   and   cand_j = the boundary with bin(B_k) = j (else +inf).
// By monotonicity every xn in bin j lies above the boundaries of lower bins and below
// those of higher bins, and no bin holds two boundaries (adjacent boundaries are at
// least 0.0945 = 1.5 bins apart), so #{k : B_k < xn} = cnt_j + [cand_j < xn]: the
// reference's nearest index for finite xn (clamping xn to [-1, 1] never changes that
// count).  |xn| <= 1 + 2^-22 keeps j in 0 .. 32 whenever 1/amax is finite; blocks with
// an infinite 1/amax (amax below 2^-128) take the compare-tree search instead.  A NaN
// xn is the canonical 0x7FFFFFFF on the GPU and falls in bin 63, whose entry gives the
// reference's NaN code (TQ3 0, TQ4 15).  Rows are replicated for the 16 lanes of a half
// warp (8-byte entries: lane l reads banks 2l and 2l + 1), so lookups never conflict.
constexpr float BIN_MAGIC = 12582928.0f;   // 1.5 * 2^23 + 16
constexpr float BIN_SCALE = 16.0f;
constexpr uint32_t BIN_MASK = 0x3Fu;
constexpr int NEAR_ROWS = 64, NEAR_REP = 16;

template <int QT>
__device__ __forceinline__ float boundary(int k) {   // B_k of src/ggml-tq.h:93-121, exact fp32
    if constexpr (QT == 2) {
        return k == 0 ? -TQ2_P0 : (k == 1 ? 0.0f : TQ2_P0);
    } else if constexpr (QT == 4) {
        constexpr float P[7] = {TQ4_P0, TQ4_P1, TQ4_P2, TQ4_P3, TQ4_P4, TQ4_P5, TQ4_P6};
        return k < 7 ? -P[6 - k] : (k == 7 ? 0.0f : P[k - 8]);
    } else {
        constexpr float P[3] = {TQ3_P0, TQ3_P1, TQ3_P2};
        return k < 3 ? -P[2 - k] : (k == 3 ? 0.0f : P[k - 4]);
    }
}

template <int QT>
__device__ void near_table_init(uint2* __restrict__ t) {
    // one thread per row: count the boundaries of lower bins, find this bin's boundary,
    // then write the row's 16 replicas
    constexpr int NB = QT == 4 ? 15 : QT == 3 ? 7 : 3;
    for (int row = threadIdx.x; row < NEAR_ROWS; row += CODEC_THREADS) {
        uint32_t cnt = QT == 4 ? 15u : 0u;   // bins past 32: only a NaN reaches them
        float cand = INFINITY;
        if (row <= 32) {
            cnt = 0;
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                const float b = boundary<QT>(k);
                const int bk = (int)(__float_as_uint(__fmaf_rn(b, BIN_SCALE, BIN_MAGIC)) & BIN_MASK);
                cnt += bk < row;
                cand = bk == row ? b : cand;
            }
        }
        const uint4 e = make_uint4(__float_as_uint(cand), cnt, __float_as_uint(cand), cnt);
#pragma unroll
        for (int r = 0; r < NEAR_REP / 2; ++r) reinterpret_cast<uint4*>(t + row * NEAR_REP)[r] = e;
    }
}

// nearest indices of xn.x, xn.y; tb = shared address of the table + 8 * (lane % 16)
__device__ __forceinline__ void near_pair(float2 xn, uint32_t tb, uint32_t& i0, uint32_t& i1) {
    const float2 f = __ffma2_rn(xn, make_float2(BIN_SCALE, BIN_SCALE), make_float2(BIN_MAGIC, BIN_MAGIC));
    const uint32_t a0 = tb + ((__float_as_uint(f.x) & BIN_MASK) << 7);
    const uint32_t a1 = tb + ((__float_as_uint(f.y) & BIN_MASK) << 7);
    uint32_t c0, n0, c1, n1;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(c0), "=r"(n0) : "r"(a0));
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(c1), "=r"(n1) : "r"(a1));
    asm("{\n\t.reg .pred p;\n\tsetp.gt.f32 p, %1, %2;\n\t@p add.u32 %0, %0, 1;\n\t}" : "+r"(n0) : "f"(xn.x), "f"(__uint_as_float(c0)));
    asm("{\n\t.reg .pred p;\n\tsetp.gt.f32 p, %1, %2;\n\t@p add.u32 %0, %0, 1;\n\t}" : "+r"(n1) : "f"(xn.y), "f"(__uint_as_float(c1)));
    i0 = n0;
    i1 = n1;
}

// ── one block: amax, fp16 scale, nearest codes (or TQ3 optimal rounding), packing ──
// v holds the (rotated) float32 block; the packed block is staged at s_out + off when write.
template <int QT, int MODE>
__device__ __forceinline__ void encode_block(float (&v)[QK], uint32_t near_tb, const Tq3OptTables* tbl,
                                             int n_passes, uint8_t* __restrict__ s_out, int off, bool write) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < QK; ++j) amax = fmaxf(amax, fabsf(v[j]));   // NaN never wins
    const float inv = amax > 0.0f ? 1.0f / amax : 0.0f;
    const float2 inv2 = make_float2(inv, inv);

    // xn = x * id exactly as the reference (one fp32 multiply per element), then the table
    uint32_t code[QK];
#pragma unroll
    for (int j = 0; j < QK; j += 2)
        near_pair(__fmul2_rn(make_float2(v[j], v[j + 1]), inv2), near_tb, code[j], code[j + 1]);
    if (inv == INFINITY) {
        // amax below 2^-128: xn is +-inf (or NaN for zeros), outside the table's range
#pragma unroll
        for (int j = 0; j < QK; ++j) {
            const float xn = __fmul_rn(v[j], inv);
            code[j] = (uint32_t)(QT == 4 ? tq4_nearest(xn) : QT == 3 ? tq3_nearest(xn) : tq2_nearest(xn));
        }
    }

    uint16_t dh;
    if constexpr (QT == 4) {
        dh = half_trunc(amax);
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {   // byte j = code[j] | code[j + 16] << 4
            const int j = 4 * k;
            w[k] = code[j] + (code[j + 16] << 4) + (code[j + 1] << 8) + (code[j + 17] << 12) +
                   (code[j + 2] << 16) + (code[j + 18] << 20) + (code[j + 3] << 24) + (code[j + 19] << 28);
        }
        if (write) stage_block<4>(s_out, off, dh, w);
    } else if constexpr (QT == 2) {
        dh = half_trunc(amax);
        uint32_t w[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {   // byte i = codes 4i .. 4i+3 at bits 0, 2, 4, 6
            uint32_t acc = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) acc += code[16 * k + j] << (2 * j);
            w[k] = acc;
        }
        if (write) stage_block<2>(s_out, off, dh, w);
    } else {
        // codes as the four 24-bit group words of the TQ3 layout (code i of a group at bits 3i..3i+2)
        uint32_t g[4];
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
            const uint32_t* c = code + 8 * gi;
            g[gi] = c[0] + (c[1] << 3) + (c[2] << 6) + (c[3] << 9) + (c[4] << 12) + (c[5] << 15) + (c[6] << 18) +
                    (c[7] << 21);
        }
        if constexpr (MODE == 1) {
            if (amax > 0.0f) {
                const double d = tq3_opt_refine(v, g, n_passes, tbl);
                float df = (float)d;
                if (df != df) df = fabsf(df);
                dh = half_trunc(df);
            } else {
                g[0] = g[1] = g[2] = g[3] = 0u;
                dh = 0;
            }
        } else {
            dh = half_trunc(amax);
        }
        // 12 code bytes as 3 little-endian words
        const uint32_t w[3] = {g[0] | (g[1] << 24), (g[1] >> 8) | (g[2] << 16), (g[2] >> 16) | (g[3] << 8)};
        if (write) stage_block<3>(s_out, off, dh, w);
    }
}

// float32 values of one block of `QT` at byte pointer blk (dequantize_row_tq*_0, exact)
template <int QT>
__device__ __forceinline__ void decode_block(const uint8_t* __restrict__ blk, float (&v)[QK]) {
    const float d = half_decode((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    if constexpr (QT == 4) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t b = blk[2 + j];
            v[j] = __fmul_rn(tq4_level(b & 15u), d);
            v[j + 16] = __fmul_rn(tq4_level(b >> 4), d);
        }
    } else if constexpr (QT == 3) {
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
            const uint32_t w = (uint32_t)blk[2 + 3 * gi] | ((uint32_t)blk[3 + 3 * gi] << 8) |
                               ((uint32_t)blk[4 + 3 * gi] << 16);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[8 * gi + i] = __fmul_rn(tq3_level((w >> (3 * i)) & 7u), d);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t b = blk[2 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) v[4 * i + j] = __fmul_rn(tq2_level((b >> (2 * j)) & 3u), d);
        }
    }
}

// ── quantize ────────────────────────────────────────────────────────────────
// MODE 0: nearest level (reference).  MODE 1: TQ3 optimal rounding.
template <int QT, typename IN, int MODE, int L2>
__global__ void __launch_bounds__(CODEC_THREADS, (MODE == 0 && sizeof(IN) == 4) ? 3 : 4)
quantize_kernel(const IN* __restrict__ x, uint8_t* __restrict__ y, int64_t nblocks,
                int log2_hd, float norm, int n_passes, int x_vec, int y_vec, const RowMap map,
                uint32_t rseed, int rhpr) {
    constexpr int EB = ElemBits<IN>::bytes;
    constexpr int ROW_BYTES = QK * EB;
    constexpr int BB = BlockBytes<QT>::value;
    constexpr int NBUF = 2;   // double-buffered input tiles
    __shared__ __align__(128) uint8_t s_in2[NBUF][CODEC_THREADS * ROW_BYTES];
    __shared__ __align__(16) uint8_t s_out[CODEC_THREADS * BB];
    __shared__ Tq3OptTables s_tbl;
    // row-mapped output: byte offset of each head row | contiguous flag; two tiles' worth, since
    // tile i + 1's placement is written while tile i is still being stored
    __shared__ int64_t s_dst2[2][CODEC_THREADS + 1];
    __shared__ __align__(16) uint2 s_near[NEAR_ROWS * NEAR_REP];

    grid_dep_trigger();
    near_table_init<QT>(s_near);
    const uint32_t near_tb = (uint32_t)__cvta_generic_to_shared(s_near) + 8u * (threadIdx.x & (NEAR_REP - 1));
    if (MODE == 1) {
        for (int e = threadIdx.x; e < 8 * 2 * 8; e += CODEC_THREADS) {
            const int i = e >> 4, up = (e >> 3) & 1;
            const double L = tq3_level_f64(i);
            const double Ln = up ? (i < 7 ? tq3_level_f64(i + 1) : L) : (i > 0 ? tq3_level_f64(i - 1) : L);
            s_tbl.rep[e] = make_double2(Ln - L, Ln * Ln - L * L);
            if (e < 8) s_tbl.lv[e] = tq3_level_f64(e);
        }
    }

    const int64_t ntiles = (nblocks + CODEC_THREADS - 1) / CODEC_THREADS;
    auto rows_of = [&](int64_t t) {
        const int64_t b = t * CODEC_THREADS;
        return (int)(nblocks - b < CODEC_THREADS ? nblocks - b : CODEC_THREADS);
    };
    // Tile i is read from s_in2[i & 1]; tile i + 1 is in flight (cp.async) while tile i computes.
    // Two schedules, chosen by measurement:
    //  * bandwidth-bound modes (MODE 0): tile i + 1's copies are issued before tile i's landing
    //    wait, so they overlap the barrier too; a second barrier (staged blocks complete, tile i's
    //    input read) precedes the block-wide store;
    //  * TQ3 optimal rounding (MODE 1, compute bound): one barrier per tile; after it every thread
    //    is done with tile i - 1, so the prefetch into that buffer is issued behind it, and each
    //    warp stores its own 32 staged blocks.
    constexpr bool ONE_BARRIER = MODE == 1;
    const bool async_tiles = NBUF == 2 && x_vec;
    grid_dep_wait();
    if (async_tiles && (int64_t)blockIdx.x < ntiles)
        load_tile_async<IN>(s_in2[0], x + (int64_t)blockIdx.x * CODEC_THREADS * QK, rows_of(blockIdx.x));
    cp_async_commit();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const int64_t b0 = tile * CODEC_THREADS;
        const int nrows = rows_of(tile);
        // cache placement of this tile's rows, while its copies land (the barrier below publishes it;
        // two buffers, since a thread may still be storing the previous tile)
        int64_t* s_dst = s_dst2[it & 1];
        if (map.cap != 0) map_rows(s_dst, b0, nrows, BB, map);
        uint8_t* s_in = s_in2[it % NBUF];
        const int64_t nxt = tile + gridDim.x;
        if (async_tiles) {
            if (!ONE_BARRIER) {
                if (nxt < ntiles) load_tile_async<IN>(s_in2[(it + 1) % NBUF], x + nxt * CODEC_THREADS * QK, rows_of(nxt));
                cp_async_commit();
                cp_async_wait<1>();   // this thread's copies of the current tile have landed
            } else {
                cp_async_wait<0>();
            }
        } else {
            load_tile<IN>(s_in, x + b0 * QK, nrows, x_vec != 0);
        }
        __syncthreads();          // every thread's copies have landed; s_dst is complete
        if (ONE_BARRIER && async_tiles) {
            if (nxt < ntiles) load_tile_async<IN>(s_in2[(it + 1) % NBUF], x + nxt * CODEC_THREADS * QK, rows_of(nxt));
            cp_async_commit();
        }

        float v[QK];
        read_row<IN>(s_in, threadIdx.x < nrows ? threadIdx.x : 0, v);
        if (rhpr > 0) {
            // randomized_hadamard_transform_row: chunk h of a row is signed from seed + h
            const int64_t gb = b0 + threadIdx.x;
            const int nblk = 1 << (log2_hd - 5);
            const int64_t head = gb >> (log2_hd - 5);
            lcg_signs32(v, rseed + (uint32_t)(head % rhpr), (uint32_t)(gb & (nblk - 1)) * 32u);
        }
        fwht_block<L2>(v, log2_hd, norm);
        encode_block<QT, MODE>(v, near_tb, &s_tbl, n_passes, s_out, threadIdx.x * BB, threadIdx.x < nrows);
        if (!ONE_BARRIER) {
            __syncthreads();      // s_out complete; s_in of this tile fully read
            if (map.cap == 0) store_staged(y + b0 * BB, s_out, nrows * BB, y_vec != 0);
            else store_mapped_warp(y, s_out, s_dst, nrows, BB, map, y_vec != 0, 0, threadIdx.x, CODEC_THREADS);
        } else {
            __syncwarp();         // this warp's 32 staged blocks are complete
            if (map.cap == 0) {
                const int nw = nrows - 32 * warp;   // blocks of this warp
                if (nw > 0)
                    store_staged(y + (b0 + 32 * warp) * BB, s_out + 32 * warp * BB, (nw < 32 ? nw : 32) * BB,
                                 y_vec != 0, lane, 32);
            } else {
                store_mapped_warp(y, s_out, s_dst, nrows, BB, map, y_vec != 0, warp, lane, 32);
            }
        }
        // No barrier here: the next tile writes s_out only after its own landing barrier, which
        // every thread reaches after finishing this store; its placement goes to the other s_dst.
    }
    cp_async_wait<0>();
}

// ── in-place FWHT (hadamard_transform_row) on fp32 ──────────────────────────
__global__ void __launch_bounds__(CODEC_THREADS)
fwht_kernel(float* __restrict__ x, int64_t nblocks, int log2_hd, float norm, int x_vec, uint32_t rseed, int rhpr) {
    constexpr int ROW_BYTES = QK * 4;
    __shared__ __align__(16) uint8_t s_in[CODEC_THREADS * ROW_BYTES];
    const int64_t ntiles = (nblocks + CODEC_THREADS - 1) / CODEC_THREADS;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int64_t b0 = tile * CODEC_THREADS;
        const int nrows = (int)(nblocks - b0 < CODEC_THREADS ? nblocks - b0 : CODEC_THREADS);
        __syncthreads();
        load_tile<float>(s_in, x + b0 * QK, nrows, x_vec != 0);
        __syncthreads();
        float v[QK];
        const int r = threadIdx.x < nrows ? threadIdx.x : 0;
        read_row<float>(s_in, r, v);
        if (rhpr > 0) {   // randomized_hadamard_transform_row (heads of >= 32 elements)
            const int64_t gb = b0 + r;
            const int64_t head = gb >> (log2_hd - 5);
            lcg_signs32(v, rseed + (uint32_t)(head % rhpr), (uint32_t)(gb & ((1 << (log2_hd - 5)) - 1)) * 32u);
        }
        fwht_block(v, log2_hd, norm);
        __syncthreads();
        if (threadIdx.x < nrows) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
                *reinterpret_cast<float4*>(s_in + tile_chunk_addr<ROW_BYTES>(r, q)) =
                    make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        __syncthreads();
        float* dst = x + b0 * QK;
        if (x_vec) {
            for (int c = threadIdx.x; c < nrows * 8; c += CODEC_THREADS)
                reinterpret_cast<int4*>(dst)[c] =
                    *reinterpret_cast<const int4*>(s_in + tile_chunk_addr<ROW_BYTES>(c / 8, c % 8));
        } else {
            for (int e = threadIdx.x; e < nrows * QK; e += CODEC_THREADS) {
                const int rr = e / QK, cc = e % QK;
                dst[e] = *reinterpret_cast<const float*>(s_in + tile_chunk_addr<ROW_BYTES>(rr, cc >> 2) + 4 * (cc & 3));
            }
        }
    }
}

// ── dequantize ──────────────────────────────────────────────────────────────
// 4 lanes per block, 8 outputs each.  fp16 / bf16: lane p writes elements
// 8p .. 8p+7 (one 16-byte store, the 4 lanes of a block 64 contiguous bytes).
// fp32: lane p writes elements 4p .. 4p+3 and 16+4p .. 16+4p+3 (two 16-byte
// stores, each covering whole 32-byte sectors across the 4 lanes; for TQ4 these
// are the low and high nibbles of qs bytes 4p .. 4p+3).
constexpr int DQ_THREADS = 256;
constexpr int DQ_TILE = 256;   // blocks per tile

template <typename OUT> __device__ __forceinline__ OUT from_float(float f);
template <> __device__ __forceinline__ float from_float<float>(float f) { return f; }
template <> __device__ __forceinline__ __half from_float<__half>(float f) { return __float2half_rn(f); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float f) { return __float2bfloat16_rn(f); }

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// eight consecutive outputs at a 16-byte aligned address
template <typename OUT>
__device__ __forceinline__ void store8(OUT* dst, const float (&o)[8]) {
    if constexpr (sizeof(OUT) == 4) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(o[0], o[1], o[2], o[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(pack2(o[0], o[1], dst), pack2(o[2], o[3], dst),
                                                    pack2(o[4], o[5], dst), pack2(o[6], o[7], dst));
    }
}
__device__ __forceinline__ uint32_t lds_u16_at(const uint8_t* p) {   // 2-byte aligned shared read
    return *reinterpret_cast<const uint16_t*>(p);
}

template <int QT, typename OUT>
__global__ void __launch_bounds__(DQ_THREADS)
dequantize_kernel(const uint8_t* __restrict__ xq, OUT* __restrict__ y, int64_t nblocks, int x_vec, int y_vec) {
    constexpr int BB = BlockBytes<QT>::value;
    constexpr int NL = QT == 4 ? 16 : QT == 3 ? 8 : 4;
    __shared__ __align__(16) uint8_t s_in[DQ_TILE * BB];
    __shared__ float s_lvl[NL];
    grid_dep_trigger();
    if (threadIdx.x < NL) s_lvl[threadIdx.x] = tq_level<QT>(threadIdx.x);
    grid_dep_wait();

    const int64_t ntiles = (nblocks + DQ_TILE - 1) / DQ_TILE;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int64_t b0 = tile * DQ_TILE;
        const int nrows = (int)(nblocks - b0 < DQ_TILE ? nblocks - b0 : DQ_TILE);
        const int nbytes = nrows * BB;
        __syncthreads();
        const uint8_t* src = xq + b0 * BB;
        if (x_vec && (nbytes & 15) == 0) {
            for (int c = threadIdx.x; c < nbytes / 16; c += DQ_THREADS)
                reinterpret_cast<int4*>(s_in)[c] = __ldg(reinterpret_cast<const int4*>(src) + c);
        } else {
            for (int b = threadIdx.x; b < nbytes; b += DQ_THREADS) s_in[b] = src[b];
        }
        __syncthreads();
        const int part = threadIdx.x & 3;
        constexpr bool SPLIT = sizeof(OUT) == 4;   // outputs 4p..4p+3 | 16+4p..16+4p+3, else 8p..8p+7
        for (int r = threadIdx.x >> 2; r < nrows; r += DQ_THREADS / 4) {
            const uint8_t* blk = s_in + r * BB;
            const float d = half_decode(lds_u16_at(blk));
            uint32_t c[8];
            if constexpr (QT == 4) {
                if constexpr (SPLIT) {
                    // low and high nibbles of qs bytes 4p .. 4p+3
                    const uint8_t* q = blk + 2 + 4 * part;
                    const uint32_t w = lds_u16_at(q) | (lds_u16_at(q + 2) << 16);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        c[i] = (w >> (8 * i)) & 15u;
                        c[4 + i] = (w >> (8 * i + 4)) & 15u;
                    }
                } else {
                    // low nibbles of qs bytes 8p .. 8p+7 (p < 2), high nibbles of bytes 8(p-2) .. (p >= 2)
                    const uint8_t* q = blk + 2 + 8 * (part & 1);
                    const uint32_t sh = part < 2 ? 0u : 4u;
                    const uint32_t n0 = ((lds_u16_at(q) | (lds_u16_at(q + 2) << 16)) >> sh) & 0x0F0F0F0Fu;
                    const uint32_t n1 = ((lds_u16_at(q + 4) | (lds_u16_at(q + 6) << 16)) >> sh) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        c[i] = (n0 >> (8 * i)) & 0xFFu;
                        c[4 + i] = (n1 >> (8 * i)) & 0xFFu;
                    }
                }
            } else if constexpr (QT == 2) {
                // qs byte i holds codes 4i .. 4i+3
                const uint32_t b = SPLIT ? ((uint32_t)blk[2 + part] | ((uint32_t)blk[6 + part] << 8))
                                         : lds_u16_at(blk + 2 + 2 * part);
#pragma unroll
                for (int i = 0; i < 8; ++i) c[i] = (b >> (2 * i)) & 3u;
            } else {
                // group g (3 bytes) holds codes 8g .. 8g+7
                auto group = [&](int g) {
                    const uint8_t* q = blk + 2 + 3 * g;
                    return (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16);
                };
                if constexpr (SPLIT) {
                    const uint32_t w0 = group(part >> 1) >> (12 * (part & 1));
                    const uint32_t w1 = group(2 + (part >> 1)) >> (12 * (part & 1));
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        c[i] = (w0 >> (3 * i)) & 7u;
                        c[4 + i] = (w1 >> (3 * i)) & 7u;
                    }
                } else {
                    const uint32_t w = group(part);
#pragma unroll
                    for (int i = 0; i < 8; ++i) c[i] = (w >> (3 * i)) & 7u;
                }
            }
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(s_lvl[c[i]], d);
            OUT* row = y + (b0 + r) * QK;
            if constexpr (SPLIT) {
                float* dst0 = reinterpret_cast<float*>(row) + 4 * part;
                float* dst1 = dst0 + 16;
                if (y_vec) {
                    *reinterpret_cast<float4*>(dst0) = make_float4(o[0], o[1], o[2], o[3]);
                    *reinterpret_cast<float4*>(dst1) = make_float4(o[4], o[5], o[6], o[7]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        dst0[i] = o[i];
                        dst1[i] = o[4 + i];
                    }
                }
            } else {
                OUT* dst = row + 8 * part;
                if (y_vec) {
                    store8<OUT>(dst, o);
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) dst[i] = from_float<OUT>(o[i]);
                }
            }
        }
    }
}

// ── launchers ───────────────────────────────────────────────────────────────

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (cached[dev] == 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
        cached[dev] = sms;
    }
    return cached[dev];
}

static int codec_grid(int64_t ntiles, int per_sm) {
    const int sms = sm_count();
    const int64_t cap = (int64_t)sms * per_sm;
    return (int)(ntiles < cap ? (ntiles > 0 ? ntiles : 1) : cap);
}

struct RandRot {
    uint32_t seed = 0;
    int heads_per_row = 0;   // 0: no sign diagonal
};

template <int QT, typename IN, int MODE, int L2>
static cudaError_t launch_quant_k(const void* x, void* y, int64_t nblocks, int log2_hd, float norm, int n_passes,
                                  const RowMap& map, int grid, int xv, int yv, const RandRot& rr, cudaStream_t st) {
    return launch_dependent(quantize_kernel<QT, IN, MODE, L2>, (unsigned)grid, CODEC_THREADS, st, (const IN*)x,
                            (uint8_t*)y, nblocks, log2_hd, norm, n_passes, xv, yv, map, rr.seed, rr.heads_per_row);
}

template <int QT, typename IN, int MODE>
static cudaError_t launch_quant_l2(const void* x, void* y, int64_t nblocks, int log2_hd, float norm, int n_passes,
                                   const RowMap& map, int grid, int xv, int yv, const RandRot& rr, cudaStream_t st) {
    // head_dim 128 and 256 (and no rotation) get fully unrolled FWHT stages
    switch (log2_hd) {
        case -1: return launch_quant_k<QT, IN, MODE, -1>(x, y, nblocks, log2_hd, norm, n_passes, map, grid, xv, yv, rr, st);
        case 7: return launch_quant_k<QT, IN, MODE, 7>(x, y, nblocks, log2_hd, norm, n_passes, map, grid, xv, yv, rr, st);
        case 8: return launch_quant_k<QT, IN, MODE, 8>(x, y, nblocks, log2_hd, norm, n_passes, map, grid, xv, yv, rr, st);
        default: return launch_quant_k<QT, IN, MODE, -2>(x, y, nblocks, log2_hd, norm, n_passes, map, grid, xv, yv, rr, st);
    }
}

template <int QT, typename IN>
static cudaError_t launch_quant_t(const void* x, void* y, int64_t nblocks, int log2_hd, float norm,
                                  int n_passes, const RowMap& map, const RandRot& rr, cudaStream_t st) {
    const int64_t ntiles = (nblocks + CODEC_THREADS - 1) / CODEC_THREADS;
    // Grid, by measurement: fp32 inputs and TQ3 optimal rounding run one wave of resident CTAs
    // (3 / 4 per SM), each looping over its tiles with the next tile's copies in flight (C1 round
    // trip -10 %, fp32 without rotation +7 %); 16-bit inputs keep up to 16 CTAs per SM in flight
    // (their resident-wave grid was 2 % slower).
    const int grid = codec_grid(ntiles, n_passes > 0 ? 4 : (sizeof(IN) == 4 ? 3 : 16));
    const int xv = ((uintptr_t)x & 15) == 0, yv = ((uintptr_t)y & 15) == 0;
    if constexpr (QT == 3) {
        if (n_passes > 0) return launch_quant_l2<QT, IN, 1>(x, y, nblocks, log2_hd, norm, n_passes, map, grid, xv, yv, rr, st);
    }
    return launch_quant_l2<QT, IN, 0>(x, y, nblocks, log2_hd, norm, 0, map, grid, xv, yv, rr, st);
}

cudaError_t launch_quantize(int qtype, int in_dtype, const void* x, void* y, int64_t nblocks, int log2_hd,
                            float norm, int n_passes, cudaStream_t st, const RowMap& map, uint32_t rseed,
                            int heads_per_row) {
    if (nblocks <= 0) return cudaSuccess;
    RandRot rr;
    rr.seed = rseed;
    rr.heads_per_row = heads_per_row;
    if (qtype == 4) {
        switch (in_dtype) {
            case DT_F32: return launch_quant_t<4, float>(x, y, nblocks, log2_hd, norm, 0, map, rr, st);
            case DT_F16: return launch_quant_t<4, __half>(x, y, nblocks, log2_hd, norm, 0, map, rr, st);
            default: return launch_quant_t<4, __nv_bfloat16>(x, y, nblocks, log2_hd, norm, 0, map, rr, st);
        }
    }
    if (qtype == 2) {
        switch (in_dtype) {
            case DT_F32: return launch_quant_t<2, float>(x, y, nblocks, log2_hd, norm, 0, map, rr, st);
            case DT_F16: return launch_quant_t<2, __half>(x, y, nblocks, log2_hd, norm, 0, map, rr, st);
            default: return launch_quant_t<2, __nv_bfloat16>(x, y, nblocks, log2_hd, norm, 0, map, rr, st);
        }
    }
    switch (in_dtype) {
        case DT_F32: return launch_quant_t<3, float>(x, y, nblocks, log2_hd, norm, n_passes, map, rr, st);
        case DT_F16: return launch_quant_t<3, __half>(x, y, nblocks, log2_hd, norm, n_passes, map, rr, st);
        default: return launch_quant_t<3, __nv_bfloat16>(x, y, nblocks, log2_hd, norm, n_passes, map, rr, st);
    }
}

cudaError_t launch_fwht(float* x, int64_t nblocks, int log2_hd, float norm, cudaStream_t st, uint32_t rseed,
                        int heads_per_row) {
    if (nblocks <= 0) return cudaSuccess;
    const int64_t ntiles = (nblocks + CODEC_THREADS - 1) / CODEC_THREADS;
    fwht_kernel<<<codec_grid(ntiles, 16), CODEC_THREADS, 0, st>>>(x, nblocks, log2_hd, norm,
                                                                  ((uintptr_t)x & 15) == 0, rseed, heads_per_row);
    return cudaGetLastError();
}

// ── requantize: decode a tile of ST blocks, encode each block as DT ───────────
template <int ST, int DT>
__global__ void __launch_bounds__(CODEC_THREADS)
requant_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t nblocks, int s_vec, int d_vec) {
    constexpr int SB = BlockBytes<ST>::value, DB = BlockBytes<DT>::value;
    __shared__ __align__(16) uint8_t s_in[CODEC_THREADS * SB];
    __shared__ __align__(16) uint8_t s_out[CODEC_THREADS * DB];
    __shared__ __align__(16) uint2 s_near[NEAR_ROWS * NEAR_REP];
    near_table_init<DT>(s_near);
    const uint32_t near_tb = (uint32_t)__cvta_generic_to_shared(s_near) + 8u * (threadIdx.x & (NEAR_REP - 1));
    const int64_t ntiles = (nblocks + CODEC_THREADS - 1) / CODEC_THREADS;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int64_t b0 = tile * CODEC_THREADS;
        const int nrows = (int)(nblocks - b0 < CODEC_THREADS ? nblocks - b0 : CODEC_THREADS);
        __syncthreads();   // s_in / s_out free
        const int nbytes = nrows * SB;
        const uint8_t* sp = src + b0 * SB;
        if (s_vec && (nbytes & 15) == 0) {
            for (int c = threadIdx.x; c < nbytes / 16; c += CODEC_THREADS)
                reinterpret_cast<int4*>(s_in)[c] = __ldg(reinterpret_cast<const int4*>(sp) + c);
        } else {
            for (int b = threadIdx.x; b < nbytes; b += CODEC_THREADS) s_in[b] = sp[b];
        }
        __syncthreads();
        float v[QK];
        decode_block<ST>(s_in + (threadIdx.x < nrows ? threadIdx.x : 0) * SB, v);
        encode_block<DT, 0>(v, near_tb, nullptr, 0, s_out, threadIdx.x * DB, threadIdx.x < nrows);
        __syncthreads();
        store_staged(dst + b0 * DB, s_out, nrows * DB, d_vec != 0);
    }
}

template <int ST, int DT>
static cudaError_t launch_requant_t(const void* src, void* dst, int64_t nblocks, cudaStream_t st) {
    const int64_t ntiles = (nblocks + CODEC_THREADS - 1) / CODEC_THREADS;
    requant_kernel<ST, DT><<<codec_grid(ntiles, 16), CODEC_THREADS, 0, st>>>(
        (const uint8_t*)src, (uint8_t*)dst, nblocks, ((uintptr_t)src & 15) == 0, ((uintptr_t)dst & 15) == 0);
    return cudaGetLastError();
}

cudaError_t launch_requantize(int src_type, const void* src, int dst_type, void* dst, int64_t nblocks,
                              cudaStream_t st) {
    if (nblocks <= 0) return cudaSuccess;
#define TQ_RQ(S, D) if (src_type == S && dst_type == D) return launch_requant_t<S, D>(src, dst, nblocks, st);
    TQ_RQ(4, 3) TQ_RQ(4, 2) TQ_RQ(3, 2) TQ_RQ(3, 4) TQ_RQ(2, 4) TQ_RQ(2, 3) TQ_RQ(4, 4) TQ_RQ(3, 3) TQ_RQ(2, 2)
#undef TQ_RQ
    return cudaErrorInvalidValue;
}

template <int QT, typename OUT>
static cudaError_t launch_dq_t(const void* x, void* y, int64_t nblocks, cudaStream_t st) {
    const int64_t ntiles = (nblocks + DQ_TILE - 1) / DQ_TILE;
    return launch_dependent(dequantize_kernel<QT, OUT>, (unsigned)codec_grid(ntiles, 8), DQ_THREADS, st,
                            (const uint8_t*)x, (OUT*)y, nblocks, (int)(((uintptr_t)x & 15) == 0),
                            (int)(((uintptr_t)y & 15) == 0));
}

cudaError_t launch_dequantize(int qtype, int out_dtype, const void* x, void* y, int64_t nblocks, cudaStream_t st) {
    if (nblocks <= 0) return cudaSuccess;
    if (qtype == 2) {
        switch (out_dtype) {
            case DT_F32: return launch_dq_t<2, float>(x, y, nblocks, st);
            case DT_F16: return launch_dq_t<2, __half>(x, y, nblocks, st);
            default: return launch_dq_t<2, __nv_bfloat16>(x, y, nblocks, st);
        }
    }
    if (qtype == 4) {
        switch (out_dtype) {
            case DT_F32: return launch_dq_t<4, float>(x, y, nblocks, st);
            case DT_F16: return launch_dq_t<4, __half>(x, y, nblocks, st);
            default: return launch_dq_t<4, __nv_bfloat16>(x, y, nblocks, st);
        }
    }
    switch (out_dtype) {
        case DT_F32: return launch_dq_t<3, float>(x, y, nblocks, st);
        case DT_F16: return launch_dq_t<3, __half>(x, y, nblocks, st);
        default: return launch_dq_t<3, __nv_bfloat16>(x, y, nblocks, st);
    }
}

}  // namespace tq

namespace tq {

// ── FWHT for rows that do not fill whole 32-element tiles or exceed 1024 ────

__global__ void fwht_tail_kernel(float* __restrict__ x, int n, int log2_hd, float norm) {
    // one thread; n < 32 and heads of 2^log2_hd < 32 elements (same stage order)
    const int d = 1 << log2_hd;
    for (int base = 0; base + d <= n; base += d) {
        for (int h = 1; h < d; h <<= 1)
            for (int j = 0; j < d; ++j) {
                if (j & h) continue;
                const float a = x[base + j], b = x[base + j + h];
                x[base + j] = a + b;
                x[base + j + h] = a - b;
            }
        for (int j = 0; j < d; ++j) x[base + j] = __fmul_rn(x[base + j], norm);
    }
}

constexpr int FWHT_LARGE_THREADS = 512;

__global__ void __launch_bounds__(FWHT_LARGE_THREADS)
fwht_large_kernel(float* __restrict__ x, int log2_hd, float norm) {
    extern __shared__ float srow[];
    const int d = 1 << log2_hd;
    float* row = x + (int64_t)blockIdx.x * d;
    for (int i = threadIdx.x; i < d; i += FWHT_LARGE_THREADS) srow[i] = row[i];
    __syncthreads();
    for (int s = 0; s < log2_hd; ++s) {
        const int h = 1 << s;
        for (int p = threadIdx.x; p < d / 2; p += FWHT_LARGE_THREADS) {
            const int j = ((p >> s) << (s + 1)) | (p & (h - 1));   // p-th pair of stage h
            const float a = srow[j], b = srow[j + h];
            srow[j] = a + b;
            srow[j + h] = a - b;
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < d; i += FWHT_LARGE_THREADS) row[i] = __fmul_rn(srow[i], norm);
}

cudaError_t launch_fwht_tail(float* x, int n, int log2_hd, float norm, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    fwht_tail_kernel<<<1, 1, 0, st>>>(x, n, log2_hd, norm);
    return cudaGetLastError();
}

cudaError_t launch_fwht_large(float* x, int64_t nrows, int log2_hd, float norm, cudaStream_t st) {
    if (nrows <= 0) return cudaSuccess;
    const size_t smem = sizeof(float) << log2_hd;
    cudaError_t e = cudaFuncSetAttribute(fwht_large_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    for (int64_t r0 = 0; r0 < nrows; r0 += 65535) {
        const int64_t nr = nrows - r0 < 65535 ? nrows - r0 : 65535;
        fwht_large_kernel<<<(unsigned)nr, FWHT_LARGE_THREADS, smem, st>>>(x + (r0 << log2_hd), log2_hd, norm);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}


// ── channel-permuted mixed precision (src/ggml-tq-outlier.c:97-290) ────────────
// Calibration: per-channel mean and variance over the calibration tokens,
// accumulated in token order exactly as the reference does (one thread per
// channel, no contraction into fma); the stable descending rank of the variances
// is the permutation.  Quantize: one thread per output block gathers its 32
// permuted values and encodes them with the block encoder above (bit-identical
// to quantize_row_tq*_0_ref); the first n_outlier/32 blocks of a vector use the
// outlier tier, the rest the normal tier.  Dequantize scatters a decoded block
// back through the permutation.

// ── runtime-type dispatch of the block encoder / decoder (mixed-precision tiers) ──
__device__ __forceinline__ int block_bytes_rt(int qt) { return qt == 4 ? TQ4_BYTES : qt == 3 ? TQ3_BYTES : TQ2_BYTES; }

__device__ void near_table_init_rt(int qt, uint2* t) {
    if (qt == 4) near_table_init<4>(t);
    else if (qt == 3) near_table_init<3>(t);
    else near_table_init<2>(t);
}

// encode v as a block of type qt at global byte address dst (2-byte aligned)
__device__ void encode_block_rt(int qt, float (&v)[QK], uint32_t near_tb, uint8_t* dst) {
    uint8_t* base = reinterpret_cast<uint8_t*>((uintptr_t)dst & ~uintptr_t(3));
    const int off = (int)((uintptr_t)dst & 3u);
    if (qt == 4) encode_block<4, 0>(v, near_tb, nullptr, 0, base, off, true);
    else if (qt == 3) encode_block<3, 0>(v, near_tb, nullptr, 0, base, off, true);
    else encode_block<2, 0>(v, near_tb, nullptr, 0, base, off, true);
}

__device__ void decode_block_rt(int qt, const uint8_t* blk, float (&v)[QK]) {
    if (qt == 4) decode_block<4>(blk, v);
    else if (qt == 3) decode_block<3>(blk, v);
    else decode_block<2>(blk, v);
}


__global__ void __launch_bounds__(OUTLIER_MAX_DIM)
outlier_calib_kernel(const float* __restrict__ data, int n_tokens, int hd, float* __restrict__ var_out,
                     int* __restrict__ perm_out, int* __restrict__ inv_out) {
    __shared__ float s_var[OUTLIER_MAX_DIM];
    const int d = threadIdx.x;
    if (d < hd) {
        float m = 0.0f;
        for (int t = 0; t < n_tokens; ++t) m = __fadd_rn(m, data[(int64_t)t * hd + d]);
        m = __fdiv_rn(m, (float)n_tokens);
        float v = 0.0f;
        for (int t = 0; t < n_tokens; ++t) {
            const float diff = __fsub_rn(data[(int64_t)t * hd + d], m);
            v = __fadd_rn(v, __fmul_rn(diff, diff));
        }
        v = __fdiv_rn(v, (float)n_tokens);
        s_var[d] = v;
        var_out[d] = v;
    }
    __syncthreads();
    if (d < hd) {
        // position of channel d in a stable sort by descending variance
        int r = 0;
        for (int e = 0; e < hd; ++e) r += (s_var[e] > s_var[d]) || (s_var[e] == s_var[d] && e < d);
        perm_out[r] = d;
        inv_out[d] = r;
    }
}

template <typename IN> __device__ __forceinline__ float ld_f(const IN* p);
template <> __device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld_f<__half>(const __half* p) { return __half2float(*p); }
template <> __device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

constexpr int MIX_THREADS = 128;

template <typename IN>
__global__ void __launch_bounds__(MIX_THREADS)
mixed_quantize_kernel(const IN* __restrict__ x, int64_t n_vec, const MixedPlan plan, uint8_t* __restrict__ obuf,
                      uint8_t* __restrict__ nbuf) {
    __shared__ int s_perm[OUTLIER_MAX_DIM];
    __shared__ __align__(16) uint2 s_near[2][NEAR_ROWS * NEAR_REP];
    for (int i = threadIdx.x; i < plan.head_dim; i += MIX_THREADS) s_perm[i] = plan.perm[i];
    near_table_init_rt(plan.otype, s_near[0]);
    near_table_init_rt(plan.ntype, s_near[1]);
    __syncthreads();
    const int nblk = plan.head_dim / QK, nob = plan.n_outlier / QK, nnb = nblk - nob;
    const int64_t total = n_vec * nblk;
    const uint32_t lane_off = 8u * (threadIdx.x & (NEAR_REP - 1));
    for (int64_t gb = (int64_t)blockIdx.x * MIX_THREADS + threadIdx.x; gb < total; gb += (int64_t)gridDim.x * MIX_THREADS) {
        const int64_t v = gb / nblk;
        const int b = (int)(gb - v * nblk);
        float vals[QK];
#pragma unroll
        for (int i = 0; i < QK; ++i) vals[i] = ld_f<IN>(x + v * plan.head_dim + s_perm[QK * b + i]);
        if (b < nob) {
            const uint32_t tb = (uint32_t)__cvta_generic_to_shared(s_near[0]) + lane_off;
            encode_block_rt(plan.otype, vals, tb, obuf + (v * nob + b) * (int64_t)block_bytes_rt(plan.otype));
        } else {
            const uint32_t tb = (uint32_t)__cvta_generic_to_shared(s_near[1]) + lane_off;
            encode_block_rt(plan.ntype, vals, tb, nbuf + (v * nnb + (b - nob)) * (int64_t)block_bytes_rt(plan.ntype));
        }
    }
}

__global__ void __launch_bounds__(MIX_THREADS)
mixed_dequantize_kernel(const uint8_t* __restrict__ obuf, const uint8_t* __restrict__ nbuf, int64_t n_vec,
                        const MixedPlan plan, float* __restrict__ y) {
    __shared__ int s_perm[OUTLIER_MAX_DIM];
    for (int i = threadIdx.x; i < plan.head_dim; i += MIX_THREADS) s_perm[i] = plan.perm[i];
    __syncthreads();
    const int nblk = plan.head_dim / QK, nob = plan.n_outlier / QK, nnb = nblk - nob;
    const int64_t total = n_vec * nblk;
    for (int64_t gb = (int64_t)blockIdx.x * MIX_THREADS + threadIdx.x; gb < total; gb += (int64_t)gridDim.x * MIX_THREADS) {
        const int64_t v = gb / nblk;
        const int b = (int)(gb - v * nblk);
        float vals[QK];
        if (b < nob) decode_block_rt(plan.otype, obuf + (v * nob + b) * (int64_t)block_bytes_rt(plan.otype), vals);
        else decode_block_rt(plan.ntype, nbuf + (v * nnb + (b - nob)) * (int64_t)block_bytes_rt(plan.ntype), vals);
        // unpermute: y[perm[j]] = permuted[j]  (== y[i] = permuted[inv_perm[i]])
#pragma unroll
        for (int i = 0; i < QK; ++i) y[v * plan.head_dim + s_perm[QK * b + i]] = vals[i];
    }
}

// y[i] = x[map[i]] for n_vec vectors of n elements
__global__ void gather_kernel(const float* __restrict__ x, const MixedPlan plan, int64_t n_vec, float* __restrict__ y) {
    const int64_t total = n_vec * plan.head_dim;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t v = e / plan.head_dim;
        const int i = (int)(e - v * plan.head_dim);
        y[e] = x[v * plan.head_dim + plan.perm[i]];
    }
}

static int mix_grid(int64_t work, int threads) {
    const int64_t g = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 16;
    return (int)(g < 1 ? 1 : (g < cap ? g : cap));
}

cudaError_t launch_outlier_calib(const float* data, int n_tokens, int hd, float* var, int* perm, int* inv,
                                 cudaStream_t st) {
    outlier_calib_kernel<<<1, OUTLIER_MAX_DIM, 0, st>>>(data, n_tokens, hd, var, perm, inv);
    return cudaGetLastError();
}

cudaError_t launch_mixed_quantize(int in_dtype, const void* x, int64_t n_vec, const MixedPlan& plan, void* obuf,
                                  void* nbuf, cudaStream_t st) {
    const int grid = mix_grid(n_vec * (plan.head_dim / QK), MIX_THREADS);
    switch (in_dtype) {
        case DT_F32: mixed_quantize_kernel<float><<<grid, MIX_THREADS, 0, st>>>((const float*)x, n_vec, plan, (uint8_t*)obuf, (uint8_t*)nbuf); break;
        case DT_F16: mixed_quantize_kernel<__half><<<grid, MIX_THREADS, 0, st>>>((const __half*)x, n_vec, plan, (uint8_t*)obuf, (uint8_t*)nbuf); break;
        default: mixed_quantize_kernel<__nv_bfloat16><<<grid, MIX_THREADS, 0, st>>>((const __nv_bfloat16*)x, n_vec, plan, (uint8_t*)obuf, (uint8_t*)nbuf); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_mixed_dequantize(const void* obuf, const void* nbuf, int64_t n_vec, const MixedPlan& plan, float* y,
                                    cudaStream_t st) {
    const int grid = mix_grid(n_vec * (plan.head_dim / QK), MIX_THREADS);
    mixed_dequantize_kernel<<<grid, MIX_THREADS, 0, st>>>((const uint8_t*)obuf, (const uint8_t*)nbuf, n_vec, plan, y);
    return cudaGetLastError();
}

// ── TQ2_1: one TQ3_0 sub-block and three TQ2_0 sub-blocks per 128 elements ───
// One thread per 32-element sub-block s of block b: sub-block 0 is encoded as TQ3_0 at byte 0
// of the block, sub-blocks 1..3 as TQ2_0 at bytes 14, 24, 34 (all even: the encoder's
// 2-byte alignment holds).  The two tiers' nearest-level tables sit in shared memory.
__device__ __forceinline__ int tq21_off(int s) { return s == 0 ? 0 : TQ3_BYTES + (s - 1) * TQ2_BYTES; }

template <typename IN>
__global__ void __launch_bounds__(MIX_THREADS)
tq21_quantize_kernel(const IN* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ y) {
    __shared__ __align__(16) uint2 s_near[2][NEAR_ROWS * NEAR_REP];
    near_table_init<3>(s_near[0]);
    near_table_init<2>(s_near[1]);
    __syncthreads();
    const uint32_t lane_off = 8u * (threadIdx.x & (NEAR_REP - 1));
    const int64_t total = nblocks * 4;
    for (int64_t gs = (int64_t)blockIdx.x * MIX_THREADS + threadIdx.x; gs < total; gs += (int64_t)gridDim.x * MIX_THREADS) {
        const int64_t b = gs >> 2;
        const int s = (int)(gs & 3);
        float vals[QK];
#pragma unroll
        for (int i = 0; i < QK; ++i) vals[i] = ld_f<IN>(x + gs * QK + i);
        const uint32_t tb = (uint32_t)__cvta_generic_to_shared(s_near[s == 0 ? 0 : 1]) + lane_off;
        encode_block_rt(s == 0 ? 3 : 2, vals, tb, y + b * TQ21_BYTES + tq21_off(s));
    }
}

__global__ void __launch_bounds__(MIX_THREADS)
tq21_dequantize_kernel(const uint8_t* __restrict__ x, int64_t nblocks, float* __restrict__ y) {
    const int64_t total = nblocks * 4;
    for (int64_t gs = (int64_t)blockIdx.x * MIX_THREADS + threadIdx.x; gs < total; gs += (int64_t)gridDim.x * MIX_THREADS) {
        const int s = (int)(gs & 3);
        float vals[QK];
        decode_block_rt(s == 0 ? 3 : 2, x + (gs >> 2) * TQ21_BYTES + tq21_off(s), vals);
#pragma unroll
        for (int i = 0; i < QK; i += 4)
            *reinterpret_cast<float4*>(y + gs * QK + i) = make_float4(vals[i], vals[i + 1], vals[i + 2], vals[i + 3]);
    }
}

cudaError_t launch_tq21_quantize(int in_dtype, const void* x, int64_t nblocks, void* y, cudaStream_t st) {
    const int grid = mix_grid(nblocks * 4, MIX_THREADS);
    switch (in_dtype) {
        case DT_F32: tq21_quantize_kernel<float><<<grid, MIX_THREADS, 0, st>>>((const float*)x, nblocks, (uint8_t*)y); break;
        case DT_F16: tq21_quantize_kernel<__half><<<grid, MIX_THREADS, 0, st>>>((const __half*)x, nblocks, (uint8_t*)y); break;
        default: tq21_quantize_kernel<__nv_bfloat16><<<grid, MIX_THREADS, 0, st>>>((const __nv_bfloat16*)x, nblocks, (uint8_t*)y); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_tq21_dequantize(const void* x, int64_t nblocks, float* y, cudaStream_t st) {
    const int grid = mix_grid(nblocks * 4, MIX_THREADS);
    tq21_dequantize_kernel<<<grid, MIX_THREADS, 0, st>>>((const uint8_t*)x, nblocks, y);
    return cudaGetLastError();
}

cudaError_t launch_gather(const float* x, const MixedPlan& plan, int64_t n_vec, float* y, cudaStream_t st) {
    gather_kernel<<<mix_grid(n_vec * plan.head_dim, 256), 256, 0, st>>>(x, plan, n_vec, y);
    return cudaGetLastError();
}

}  // namespace tq
