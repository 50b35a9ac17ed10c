/*
 * tq_oracle.h — CPU restatement of LeanKV's TurboQuant KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (leankv_b200/) links,
 * loads or calls this code; tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py use it as the checker.
 *
 * Parity pins (see tests/test_oracle_cpu.py):
 *   - codec + FWHT: bit-exact against the reference C (src/ggml-tq.c compiled
 *     unchanged into oracle/_ref/ by oracle/Makefile) and against the golden
 *     fixtures in tests/golden/ that were produced by that build;
 *   - TQ3 optimal rounding: against scripts/tq3_rounding.py (float64 Python),
 *     whose outputs are committed as golden fixtures;
 *   - decode attention: no reference implementation exists in-tree; this is a
 *     float64 restatement of the math in src/test-tq.c:532-559 and
 *     prototype/eval/cosine_sim.py:158-172 built on the pinned dequantizers.
 *
 * Block byte layouts (identical to src/ggml-tq.h:131-141):
 *   TQ4_0: 18 bytes = fp16 d (little endian) + 16 bytes of nibbles,
 *          byte j holds element j (low nibble) and element j+16 (high nibble).
 *   TQ3_0: 14 bytes = fp16 d + 12 bytes = 4 groups of 8 3-bit codes in 3 bytes.
 */
#ifndef LEANKV_TQ_ORACLE_H
#define LEANKV_TQ_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 32
#define ORC_TQ4_BYTES 18
#define ORC_TQ3_BYTES 14
#define ORC_TQ2_BYTES 10

/* codebooks restated from src/ggml-tq.h:98-121 (float32, ±1 outer levels) */
extern const float ORC_TQ3_LEVELS[8];
extern const float ORC_TQ3_BOUNDS[7];
extern const float ORC_TQ4_LEVELS[16];
extern const float ORC_TQ4_BOUNDS[15];
/* TQ2 levels, src/ggml-tq.h:89-91 */
extern const float ORC_TQ2_LEVELS[4];

/* fp16 codec of the standalone build: src/ggml-tq.h:39-64 */
uint16_t orc_half_from_float(float f);
float    orc_float_from_half(uint16_t h);

/* TQ2_0 decode: dequantize_row_tq2_0, src/ggml-tq.c:191-207 (2-bit unpack :70-77) */
void orc_tq2_dequantize(const uint8_t *blocks, float *y, int64_t k);

/* Walsh-Hadamard transform: src/ggml-tq.c:361-381 and :398-404 */
void orc_fwht(float *x, int d);
void orc_fwht_rows(float *x, int64_t n, int head_dim);

/* nearest-level search: src/ggml-tq.c:112-154 */
int orc_tq3_nearest(float xn);
int orc_tq4_nearest(float xn);

/* block codecs: src/ggml-tq.c:215-265 (TQ3_0) and :273-321 (TQ4_0) */
void orc_tq3_quantize(const float *x, uint8_t *blocks, int64_t k);
void orc_tq3_dequantize(const uint8_t *blocks, float *y, int64_t k);
void orc_tq4_quantize(const float *x, uint8_t *blocks, int64_t k);
void orc_tq4_dequantize(const uint8_t *blocks, float *y, int64_t k);

/* 3-bit group packing: src/ggml-tq.c:26-68 */
void orc_tq3_pack32(const uint8_t idx[32], uint8_t qs[12]);
void orc_tq3_unpack32(const uint8_t qs[12], uint8_t idx[32]);

/*
 * TQ3_0 optimal rounding: scripts/tq3_rounding.py:51-57 (optimal_scale),
 * :74-125 (quantize_coord_descent with try_all_levels=False).
 *
 * init_f64 = 0: the starting assignment is the C nearest-level assignment of
 *               quantize_row_tq3_0_ref (float32 x * (1/amax));
 * init_f64 = 1: the starting assignment of the Python prototype
 *               (float64 clip(x / amax) against float64 boundaries).
 * All scale / MSE arithmetic is float64 with full recomputation per candidate,
 * like the Python.  The stored scale is fp16(float(d_LS)) (truncating encoder);
 * a block with amax == 0 stores d = 0 and all codes 0 (the Python's zero path).
 * Returns the number of accepted moves summed over all blocks.
 */
int64_t orc_tq3_quantize_opt(const float *x, uint8_t *blocks, int64_t k, int n_passes, int init_f64);
/* one block, exposing the float64 scale and unpacked codes (for golden checks) */
int orc_tq3_opt_block(const float x[32], uint8_t idx[32], double *scale, int n_passes, int init_f64);

/*
 * Decode attention over packed K/V blocks (float64 math).
 *   q       [B][Hq][D]  float32 queries (not rotated; rotated here when rotate_q)
 *   k, v    [B][Hkv][T][D/32 blocks] of type k_type / v_type (3 or 4)
 *   kv_len  [B] valid tokens per sequence (<= T)
 *   out     [B][Hq][D]  float32; FWHT applied to the weighted sum when v_rotated
 *   lse     [B][Hq]     natural-log sum of exp(sm_scale * q.k) (may be NULL)
 * GQA: query head h reads KV head h / (Hq / Hkv).
 * nthreads > 1 splits (b, kv head) pairs over pthreads.
 */
void orc_decode_attention(int B, int Hq, int Hkv, int D, int64_t T,
                          const float *q,
                          const uint8_t *k, int k_type,
                          const uint8_t *v, int v_type,
                          const int64_t *kv_len, float sm_scale,
                          int rotate_q, int v_rotated,
                          float *out, float *lse, int nthreads);

/* log-sum-exp merge of P partial results: o[p][n][D], lse[p][n] -> out[n][D], lse_out[n] */
void orc_lse_combine(int P, int64_t n, int D, const float *o, const float *lse,
                     float *out, float *lse_out);

/*
 * Row-parallel driver used for CPU baselines: calls fn(in + r*in_row_bytes,
 * out + r*out_row_bytes, row_elems) for every row r, rows split into
 * contiguous ranges over nthreads pthreads.  fn has the ggml from_float /
 * to_float shape (src/ggml-tq.h:154).  When fwht_head_dim > 0 each row is first
 * copied into a private float buffer and rotated with fn_fwht_row (the
 * reference's hadamard_transform_row) before fn is called.
 */
typedef void (*orc_row_fn)(const void *in, void *out, int64_t k);
typedef void (*orc_fwht_row_fn)(float *x, int n, int head_dim);
void orc_parallel_rows(orc_row_fn fn, orc_fwht_row_fn fn_fwht_row, int fwht_head_dim,
                       int in_is_bf16,
                       const void *in, int64_t in_row_bytes,
                       void *out, int64_t out_row_bytes,
                       int64_t rows, int64_t row_elems, int nthreads);

/* TQ3 optimal rounding wrapper with the orc_row_fn shape (2 passes, C init) */
void orc_tq3_quantize_opt2_row(const void *x, void *blocks, int64_t k);

#ifdef __cplusplus
}
#endif

#endif
