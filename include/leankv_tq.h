/*
 * leankv_tq.h — C ABI of the B200 (sm_100a) TurboQuant KV-cache library
 * (libleankv_tq.so).  Plain pointers and sizes only.
 *
 * Three layers:
 *
 *  1. Drop-in replacements for LeanKV's src/ggml-tq.h:145-190 (TQ3_0 / TQ4_0 /
 *     Hadamard entry points) with the same names, signatures, block layouts
 *     and results (bit-exact).  Host pointers, synchronous.  Like the
 *     reference, a k that is not a multiple of 32 (or n of head_dim) is a
 *     contract violation: the reference asserts, this library prints the
 *     reason and aborts.  A missing GPU or a CUDA failure aborts the same way.
 *
 *  2. Device-pointer API (*_cuda): asynchronous on the given stream
 *     (a cudaStream_t passed as void*; NULL = legacy default stream), returning
 *     a tq_status instead of asserting.
 *
 *  3. Host-pointer API (*_host): the device-pointer operations wrapped with
 *     host<->device copies on a library-owned stream; synchronous; thread-safe.
 *
 * Thread safety: every entry point may be called concurrently from several
 * host threads (the reference's row functions are pure and row-parallel
 * callers rely on that).
 */
#ifndef LEANKV_TQ_H
#define LEANKV_TQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
#define TQ_RESTRICT __restrict__
extern "C" {
#else
#define TQ_RESTRICT restrict
#endif

#define LEANKV_TQ_ABI_VERSION 1

/* ── block formats: byte-identical to src/ggml-tq.h:125-141 ────────────── */

#ifndef GGML_TQ_H  /* the reference header defines the same layouts */
#define QK_TQ2 32
#define QK_TQ3 32
#define QK_TQ4 32
typedef struct {
    uint16_t d;
    uint8_t  qs[8];      /* byte i = code 4i | 4i+1 << 2 | 4i+2 << 4 | 4i+3 << 6, src/ggml-tq.c:78-96 */
} block_tq2_0;           /* 10 bytes */
typedef struct {
    uint16_t d;          /* fp16 scale (truncating fp32->fp16, src/ggml-tq.h:39-48) */
    uint8_t  qs[12];     /* 4 groups x 8 codes x 3 bits, src/ggml-tq.c:26-55 */
} block_tq3_0;           /* 14 bytes */
typedef struct {
    uint16_t d;
    uint8_t  qs[16];     /* byte j = code of elem j | code of elem j+16 << 4 */
} block_tq4_0;           /* 18 bytes */
#endif

/* TQ2_1: the static mixed-precision block of the LeanKV llama.cpp fork
 * (docs/RESULTS.md:1451-1466, docs/CUDA-RESULTS.md:54-62): 128 elements in 44
 * bytes, elements 0..31 as one TQ3_0 block and 32..63, 64..95, 96..127 as three
 * TQ2_0 blocks, each with its own scale.  Byte for byte it is a block_tq3_0
 * followed by three block_tq2_0 of the reference's encoders. */
#define QK_TQ2_1 128
typedef struct {
    uint16_t d_out;      /* TQ3_0 sub-block: elements 0..31 */
    uint8_t  qs_out[12];
    uint16_t d_n0;       /* TQ2_0 sub-blocks: elements 32..63, 64..95, 96..127 */
    uint8_t  qs_n0[8];
    uint16_t d_n1;
    uint8_t  qs_n1[8];
    uint16_t d_n2;
    uint8_t  qs_n2[8];
} block_tq2_1;           /* 44 bytes */

/* ── 1. drop-in entry points (src/ggml-tq.h) ─────────────────────────────── */

/* replaces quantize_row_tq3_0_ref, src/ggml-tq.c:215-247 */
void quantize_row_tq3_0_ref(const float * TQ_RESTRICT x, block_tq3_0 * TQ_RESTRICT y, int64_t k);
/* replaces dequantize_row_tq3_0, src/ggml-tq.c:249-265 */
void dequantize_row_tq3_0(const block_tq3_0 * TQ_RESTRICT x, float * TQ_RESTRICT y, int64_t k);
/* replaces quantize_row_tq4_0_ref, src/ggml-tq.c:273-304 */
void quantize_row_tq4_0_ref(const float * TQ_RESTRICT x, block_tq4_0 * TQ_RESTRICT y, int64_t k);
/* replaces dequantize_row_tq4_0, src/ggml-tq.c:306-321 */
void dequantize_row_tq4_0(const block_tq4_0 * TQ_RESTRICT x, float * TQ_RESTRICT y, int64_t k);
/* replace the ggml from_float wrappers, src/ggml-tq.c:267-269 and :323-325 */
void quantize_row_tq3_0(const float * TQ_RESTRICT x, void * TQ_RESTRICT y, int64_t k);
void quantize_row_tq4_0(const float * TQ_RESTRICT x, void * TQ_RESTRICT y, int64_t k);
/* TQ3_0 with optimal rounding (2 coordinate-descent passes + least-squares
 * scale); restates scripts/tq3_rounding.py:74-125 (quantize_coord_descent with
 * n_passes=2), the encoder the LeanKV README.md:17,25 describes for TQ3.  Same
 * block format, so dequantize_row_tq3_0 reads it unchanged. */
void quantize_row_tq3_0_opt(const float * TQ_RESTRICT x, block_tq3_0 * TQ_RESTRICT y, int64_t k);
/* replaces hadamard_transform, src/ggml-tq.c:361-381 (d a power of two) */
void hadamard_transform(float * x, int d);
/* replaces hadamard_transform_row, src/ggml-tq.c:398-404 */
void hadamard_transform_row(float * x, int n, int head_dim);
/* replace the TQ2_0 entry points, src/ggml-tq.c:158-212 */
void quantize_row_tq2_0_ref(const float * TQ_RESTRICT x, block_tq2_0 * TQ_RESTRICT y, int64_t k);
void dequantize_row_tq2_0(const block_tq2_0 * TQ_RESTRICT x, float * TQ_RESTRICT y, int64_t k);
void quantize_row_tq2_0(const float * TQ_RESTRICT x, void * TQ_RESTRICT y, int64_t k);
/* replace the tier migrations, src/ggml-tq.c:329-357 (dequantize, then quantize_row_*_ref) */
void requantize_tq4_to_tq3(const block_tq4_0 * TQ_RESTRICT src, block_tq3_0 * TQ_RESTRICT dst, int64_t k);
void requantize_tq3_to_tq2(const block_tq3_0 * TQ_RESTRICT src, block_tq2_0 * TQ_RESTRICT dst, int64_t k);
void requantize_tq4_to_tq2(const block_tq4_0 * TQ_RESTRICT src, block_tq2_0 * TQ_RESTRICT dst, int64_t k);
/* replace randomized_hadamard_transform(_row), src/ggml-tq.c:383-396 and :406-412: signs from
 * the LCG s = s * 1664525 + 1013904223 (negate where bit 31 is set), then the Hadamard transform;
 * chunk h of a row uses seed + h.  d / head_dim: powers of two from 32 to 1024. */
void randomized_hadamard_transform(float * x, int d, uint32_t seed);
void randomized_hadamard_transform_row(float * x, int n, int head_dim, uint32_t seed);

/* ── status, types ───────────────────────────────────────────────────────── */

typedef enum {
    TQ_SUCCESS = 0,
    TQ_ERROR_INVALID_VALUE = 1,   /* bad size, null pointer, bad enum */
    TQ_ERROR_UNSUPPORTED = 2,     /* e.g. head_dim not a supported power of two */
    TQ_ERROR_MISALIGNED = 3,      /* pointer alignment below what the kernel needs */
    TQ_ERROR_CUDA = 4,            /* a CUDA call failed; see tq_last_error_string() */
    TQ_ERROR_OUT_OF_MEMORY = 5,
    TQ_ERROR_NO_DEVICE = 6,
    TQ_ERROR_TIMEOUT = 7          /* a bounded device-side wait ran out */
} tq_status;

typedef enum { TQ_DTYPE_F32 = 0, TQ_DTYPE_F16 = 1, TQ_DTYPE_BF16 = 2 } tq_dtype;
typedef enum { TQ_TYPE_TQ2_0 = 2, TQ_TYPE_TQ3_0 = 3, TQ_TYPE_TQ4_0 = 4 } tq_type;

const char *tq_status_string(tq_status s);
/* message of the last failure on the calling thread ("" if none) */
const char *tq_last_error_string(void);
int tq_abi_version(void);

/* ── 2. device-pointer API ───────────────────────────────────────────────── */

/*
 * Quantize k elements (k % 32 == 0) of x (dtype x_dtype) into k/32 blocks of
 * `type` at y.  When fwht_head_dim > 0 every consecutive run of fwht_head_dim
 * elements is first rotated with the normalized Walsh-Hadamard transform
 * exactly as hadamard_transform_row does (fused, no intermediate buffer);
 * fwht_head_dim must be a power of two <= 1024 dividing k.  opt_passes > 0
 * (TQ3_0 only) applies that many passes of optimal rounding (2 = LeanKV).
 * Results are bit-identical to running the reference functions on the
 * float32 conversion of x.  Replaces the fork's f32->TQ copy kernel
 * (docs/CUDA-RESULTS.md:75).
 */
tq_status tq_quantize_cuda(tq_type type, const void *x, tq_dtype x_dtype, void *y, int64_t k,
                           int fwht_head_dim, int opt_passes, void *stream);
/* Dequantize k elements (k/32 blocks) into y of dtype y_dtype (f32 is bit-exact
 * with dequantize_row_tq*_0; f16/bf16 round that value to nearest-even). */
tq_status tq_dequantize_cuda(tq_type type, const void *x, void *y, tq_dtype y_dtype, int64_t k, void *stream);
/* In-place hadamard_transform_row on n float32 values (head_dim a power of two <= 32768). */
tq_status tq_hadamard_cuda(float *x, int64_t n, int head_dim, void *stream);
/* In-place randomized_hadamard_transform_row(row, row_len, head_dim, seed) on every row of
 * row_len elements of x (n a multiple of row_len, row_len of head_dim; head_dim a power of two,
 * 32..1024). */
tq_status tq_hadamard_randomized_cuda(float *x, int64_t n, int row_len, int head_dim, uint32_t seed, void *stream);
/* randomized_hadamard_transform_row + quantize_row_*_ref fused: every row of row_len elements is
 * rotated with the seeded sign diagonal and Hadamard transform of each head_dim chunk, then
 * quantized (opt_passes as for tq_quantize_cuda). */
tq_status tq_quantize_randomized_cuda(tq_type type, const void *x, tq_dtype x_dtype, void *y, int64_t k, int row_len,
                                      int head_dim, uint32_t seed, int opt_passes, void *stream);
/* Requantize k elements from src_type blocks to dst_type blocks in one pass (each block is
 * dequantized to float32 and quantized again, as requantize_tq4_to_tq3 and friends do). */
tq_status tq_requantize_cuda(tq_type src_type, const void *src, tq_type dst_type, void *dst, int64_t k, void *stream);
/* TQ2_1 (the fork's mixed-precision type; block_tq2_1 above): k elements, a multiple of 128,
 * of f32 / f16 / bf16 x into k / 128 blocks (no rotation: rotate the rows first when the cache
 * holds rotated rows), and back to float32.  Codes and scales equal quantize_row_tq3_0_ref on
 * elements 0..31 and quantize_row_tq2_0_ref on the other three 32-element runs of each block. */
tq_status tq_quantize_tq2_1_cuda(const void *x, tq_dtype x_dtype, void *y, int64_t k, void *stream);
tq_status tq_dequantize_tq2_1_cuda(const void *x, float *y, int64_t k, void *stream);

/*
 * Quantize-on-write into a KV cache: [FWHT] + quantize n_new new head rows per
 * (sequence, KV head) straight into their token slots.  No counterpart in the
 * reference C; it is hadamard_transform_row + quantize_row_tq*_0 placed the way
 * the prototype's LeanKVCache.update appends tokens
 * (prototype/turboquant/kv_cache.py:109-150).
 *   src   device [batch][n_kv_heads][n_new][head_dim] of src_dtype
 *   cache device [batch][n_kv_heads][capacity][head_dim/32] blocks of `type`
 *   row t of (b, h) goes to token slot pos[b] + t; pos is a device int32 [batch]
 *   array, or NULL for slot t (a prefill from slot 0).
 * rotate != 0 applies the head_dim Hadamard rotation first (the layout the decode
 * attention reads); opt_passes as for tq_quantize_cuda.  head_dim: power of two,
 * 32..1024.  Rows whose slot is outside [0, capacity) are not written; when
 * overflow is not NULL their number is added to the device int32 *overflow.
 * The blocks written are bit-identical to tq_quantize_cuda on the same rows.
 */
tq_status tq_kv_append_cuda(tq_type type, const void *src, tq_dtype src_dtype, void *cache, int batch,
                            int n_kv_heads, int head_dim, int64_t capacity, int64_t n_new, const int32_t *pos,
                            int rotate, int opt_passes, int32_t *overflow, void *stream);

/* ── 3. host-pointer API (synchronous) ───────────────────────────────────── */

tq_status tq_quantize_host(tq_type type, const void *x, tq_dtype x_dtype, void *y, int64_t k,
                           int fwht_head_dim, int opt_passes);
tq_status tq_dequantize_host(tq_type type, const void *x, void *y, tq_dtype y_dtype, int64_t k);
tq_status tq_hadamard_host(float *x, int64_t n, int head_dim);
tq_status tq_hadamard_randomized_host(float *x, int64_t n, int row_len, int head_dim, uint32_t seed);
tq_status tq_requantize_host(tq_type src_type, const void *src, tq_type dst_type, void *dst, int64_t k);

/* ── outlier channels: channel-permuted mixed precision (src/ggml-tq-outlier.h) ─
 *
 * Same types, names and semantics as the reference (ggml-tq-outlier.h:31-169):
 * calibration ranks channels by variance (top outlier_frac, rounded up to whole
 * 32-element blocks, are the outliers); a head vector is permuted outliers-first
 * and its two runs are quantized as ordinary blocks of the two tiers.  The
 * drop-in names take host pointers and handle one head vector per call, like the
 * reference; the *_cuda variants handle n_vec vectors of device memory
 * (x: [n_vec][head_dim]; buffers: [n_vec][n_outlier/32 blocks] and
 * [n_vec][n_normal/32 blocks]).  head_dim: a multiple of 32 up to 256 for
 * quantize / dequantize. */
#ifndef GGML_TQ_OUTLIER_H
#define TQ_OUTLIER_MAX_DIM 256
typedef enum { TQ_TIER_TQ2 = 0, TQ_TIER_TQ3 = 1, TQ_TIER_TQ4 = 2 } tq_tier_t;
typedef struct {
    int head_dim, n_outlier, n_normal;
    float outlier_frac;
    tq_tier_t outlier_tier, normal_tier;
    int perm[TQ_OUTLIER_MAX_DIM];        /* position i holds original channel perm[i] */
    int inv_perm[TQ_OUTLIER_MAX_DIM];    /* original channel c sits at position inv_perm[c] */
    float channel_var[TQ_OUTLIER_MAX_DIM];
} tq_outlier_config;
#endif
void tq_identify_outliers(tq_outlier_config *config, const float *calib_data, int n_tokens, int head_dim,
                          float outlier_frac, tq_tier_t outlier_tier, tq_tier_t normal_tier);
void tq_outlier_config_init_uniform(tq_outlier_config *config, int head_dim, tq_tier_t tier);
void tq_mixed_buffer_sizes(const tq_outlier_config *config, size_t *outlier_size, size_t *normal_size);
float tq_mixed_effective_bpe(const tq_outlier_config *config);
void tq_mixed_quantize(const float *x, const tq_outlier_config *config, void *outlier_buf, void *normal_buf);
void tq_mixed_dequantize(const void *outlier_buf, const void *normal_buf, const tq_outlier_config *config, float *y);
void tq_permute_channels(const float *x, float *y, const int *perm, int n);
void tq_unpermute_channels(const float *x, float *y, const int *inv_perm, int n);
/* calibration from device data [n_tokens][head_dim]; fills the host struct (synchronous on stream) */
tq_status tq_outlier_identify_cuda(tq_outlier_config *config, const float *calib, int n_tokens, int head_dim,
                                   float outlier_frac, tq_tier_t outlier_tier, tq_tier_t normal_tier, void *stream);
tq_status tq_mixed_quantize_cuda(const tq_outlier_config *config, const void *x, tq_dtype x_dtype, int64_t n_vec,
                                 void *outlier_buf, void *normal_buf, void *stream);
tq_status tq_mixed_dequantize_cuda(const tq_outlier_config *config, const void *outlier_buf, const void *normal_buf,
                                   int64_t n_vec, float *y, void *stream);

/* ── prototype vector codec (prototype/turboquant, no C counterpart) ─────────
 *
 * The Python prototype's per-vector TurboQuant (prototype/turboquant/quantizer.py:103-221,
 * qjl_residual.py:44-110, lloyd_max.py:208-236) on the GPU, one warp per vector:
 *   xr = Hadamard(x * signs) when rotate (signs: float[dim] of +-1, or NULL), or the caller's
 *        pre-rotated x_rotated (dense rotation matrices are applied by the caller);
 *   scale = ||x||_2 per vector (group == dim or 0) or max |xr| per group of `group` elements;
 *   xn = xr / (scale + 1e-10);  indices = #{b : boundaries[b] < xn}  (torch.bucketize);
 *   with qjl_signs: r = xn - levels[idx], bit (r >= 0) packed 8 per byte (bit i of byte j =
 *   element 8j + i) and qjl_mean_abs = mean |r| per vector.
 * Decode: y = (levels[idx] + (2 bit - 1) * mean_abs) * scale, then, when inv_rotate,
 * y = Hadamard(y) * signs.  dim: 32, 64, 128 or 256; 2..16 levels; device pointers. */
tq_status tq_proto_encode_cuda(const void *x, tq_dtype x_dtype, const float *x_rotated, int64_t rows, int dim,
                               int rotate, const float *signs, int group, int n_levels, const float *levels,
                               const float *boundaries, uint8_t *indices, float *scales, uint8_t *qjl_signs,
                               float *qjl_mean_abs, void *stream);
tq_status tq_proto_decode_cuda(const uint8_t *indices, const float *scales, int64_t rows, int dim, int group,
                               const uint8_t *qjl_signs, const float *qjl_mean_abs, int n_levels,
                               const float *levels, int inv_rotate, const float *signs, float *y, void *stream);

/* ── fused decode attention over packed K/V blocks ──────────────────────────
 *
 * For each sequence b and query head h (GQA: KV head h / (n_q_heads / n_kv_heads)):
 *   q~ = FWHT(q) when rotate_q (K blocks hold Hadamard-rotated keys),
 *   s_t = sm_scale * q~ . K^_t, p = softmax(s) over the first kv_len[b] tokens,
 *   out = sum_t p_t V^_t, followed by FWHT when v_rotated (V blocks hold rotated values),
 * where K^ / V^ are dequantize_row_tq*_0 of the blocks.  This is the decode path the
 * LeanKV llama.cpp fork runs on GPU (docs/CUDA-RESULTS.md:10-52; math of
 * src/test-tq.c:532-559), fused: the dequantized cache is never written to memory.
 *
 * Cache layout: [batch][n_kv_heads][kv_capacity][head_dim/32 blocks] of block_tq4_0
 * (or block_tq3_0), i.e. every token's head row is head_dim/32 consecutive blocks.
 * q / out: [batch][n_q_heads][head_dim].  lse (optional): [batch][n_q_heads],
 * natural log of sum_t exp(s_t); -inf and a zero output for kv_len == 0.
 * Requirements: head_dim 128 or 256; n_q_heads / n_kv_heads in 1 .. 8;
 * kv_capacity even; cache pointers 16-byte aligned.  Block types: K TQ4_0,
 * TQ3_0 or TQ2_0 (the last tier of a TQ4 -> TQ3 -> TQ2 cache), V TQ4_0.  Work memory: tq_decode_attention_workspace_size() bytes of
 * device memory; its first int32 receives the kernel-side status (TQ_SUCCESS,
 * TQ_ERROR_TIMEOUT for a bulk copy that never completed, TQ_ERROR_UNSUPPORTED
 * for a block scale of magnitude >= 2^15) once the stream has run the call.
 */
typedef struct {
    int batch, n_q_heads, n_kv_heads, head_dim;
    const void *q;            tq_dtype q_dtype;
    const void *k_cache;      tq_type k_type;
    const void *v_cache;      tq_type v_type;
    int64_t kv_capacity;      /* tokens allocated per (sequence, KV head) */
    const int32_t *kv_len;    /* device [batch] valid tokens, or NULL = kv_capacity */
    int64_t max_kv_len;       /* upper bound of kv_len (sizes the split-KV plan); 0 = kv_capacity */
    float sm_scale;           /* 0 = 1/sqrt(head_dim) */
    int rotate_q;             /* apply the Hadamard rotation to q */
    int v_rotated;            /* apply the Hadamard rotation to the output */
    void *out;                tq_dtype out_dtype;
    float *lse;               /* optional */
    void *workspace;          size_t workspace_bytes;
} tq_decode_attention_args;

/* bytes of device work memory tq_decode_attention_cuda needs for these arguments */
size_t tq_decode_attention_workspace_size(const tq_decode_attention_args *a);
/* fused decode attention (new; the fork's CUDA FA vec_dot_fattn_vec_KQ_tq* path) */
tq_status tq_decode_attention_cuda(const tq_decode_attention_args *a, void *stream);
/*
 * Allocation-free variant of tq_decode_attention_cuda, for callers that cannot
 * allocate device memory when they run attention (an allocator-free serving
 * step, a plugin whose host framework owns all device allocations).  No
 * counterpart in the reference.  Same arguments and results; a->workspace and
 * a->workspace_bytes are ignored.  The work memory is a static device array of
 * TQ_STATIC_SCRATCH_BYTES compiled into the library, which every GPU that
 * loads the library holds until the process exits.  Arguments that need more
 * work memory than that (tq_decode_attention_workspace_size) are rejected with
 * TQ_ERROR_INVALID_VALUE.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress): make that first call before any
 * stream capture.  All calls share the one array, so calls that can overlap on
 * the GPU (different streams, or different host threads) race and must be
 * serialized by the caller.  This entry point calls no cudaMalloc, cudaFree or
 * other allocating routine.
 */
#define TQ_STATIC_SCRATCH_BYTES (16u << 20)
tq_status tq_decode_attention_static_cuda(const tq_decode_attention_args *a, void *stream);

/*
 * Paged KV caches (no counterpart in the reference; the page-table layout of
 * paged serving caches).  K and V each live in a pool of pages; a page holds
 * page_size consecutive token rows of every KV head of one sequence:
 *   pool [num_pages][n_kv_heads][page_size][head_dim/32 blocks]
 * and page_table[b * max_pages_per_seq + i] is the pool page holding tokens
 * [i * page_size, (i + 1) * page_size) of sequence b.  page_size is a power of
 * two, 16 .. 65536 tokens (a 16-token tile of the kernel never crosses a page).
 * A page id outside [0, num_pages) met by the attention kernel is reported as
 * TQ_ERROR_INVALID_VALUE in its status word (that tile reads page 0 instead);
 * the append kernel does not write a row whose page id is outside the pool and
 * counts it as an overflow.  The page table is device memory.
 */
typedef struct {
    const int32_t *page_table;   /* device [batch][max_pages_per_seq] */
    int64_t max_pages_per_seq;
    int64_t num_pages;           /* pages in each pool, at most 2^31 - 1 */
    int page_size;               /* tokens per page */
} tq_kv_pages;

/* Decode attention over paged K/V pools: the arguments of tq_decode_attention_cuda
 * with a->k_cache / a->v_cache pointing at the pools and a->kv_capacity equal to
 * max_pages_per_seq * page_size (tq_decode_attention_workspace_size then sizes
 * the work memory).  Results are bit-identical to tq_decode_attention_cuda on the
 * same tokens stored contiguously. */
tq_status tq_decode_attention_paged_cuda(const tq_decode_attention_args *a, const tq_kv_pages *pages, void *stream);

/* Quantize-on-write into a paged cache: tq_kv_append_cuda with the token slot
 * pos[b] + t of row t of (b, h) placed through the page table (capacity =
 * max_pages_per_seq * page_size).  Rows whose slot is outside the capacity or
 * whose page id is outside the pool are not written and are counted in
 * *overflow when overflow is not NULL. */
tq_status tq_kv_append_paged_cuda(tq_type type, const void *src, tq_dtype src_dtype, void *pool, int batch,
                                  int n_kv_heads, int head_dim, const tq_kv_pages *pages, int64_t n_new,
                                  const int32_t *pos, int rotate, int opt_passes, int32_t *overflow,
                                  void *stream);

/* log-sum-exp merge of n_parts partial results o[n_parts][n_rows][head_dim] with
 * natural-log lse[n_parts][n_rows] into out[n_rows][head_dim] (+ lse_out, optional):
 * the split-by-sequence combine of the multi-GPU path (new) */
tq_status tq_lse_combine_cuda(int n_parts, int64_t n_rows, int head_dim, const float *o, const float *lse,
                              float *out, float *lse_out, void *stream);
/* The same merge with parts at arbitrary strides (in floats) and the output in
 * out_dtype: part p's rows are o + p * o_part_stride ([n_rows][head_dim]) and
 * lse + p * lse_part_stride ([n_rows]).  This reads the partials of all ranks
 * straight out of one all-gathered buffer that packs [o | lse] per rank. */
tq_status tq_lse_merge_cuda(int n_parts, int64_t n_rows, int head_dim, const float *o, int64_t o_part_stride,
                            const float *lse, int64_t lse_part_stride, void *out, tq_dtype out_dtype,
                            float *lse_out, void *stream);

/* ── split-sequence merge over peer memory (one process per GPU, one node) ──
 *
 * The exchange step of the multi-GPU split-KV decode as one kernel, without a
 * collective library.  Every rank's kernel stores its packed partial
 * [o (n_rows x head_dim floats) | lse (n_rows floats)] into its slot of every
 * rank's exchange buffer (peer stores over NVLink), publishes it with a
 * system-scope fence and one 64-bit atomic increment per CTA on every rank's
 * arrival counter, waits (bounded) until its own counter shows the partials
 * of all ranks for this step, and merges them in rank order with the
 * arithmetic of tq_lse_merge_cuda.  No counterpart in the reference.
 *
 * Setup: every rank calls tq_peer_exchange_create with the same world,
 * n_rows and head_dim, shares the TQ_PEER_HANDLE_BYTES handle it returns with
 * all ranks (any host channel), then calls tq_peer_exchange_connect with the
 * handles of all ranks in rank order.  Steps: every rank calls
 * tq_peer_exchange_merge once per step, in the same order; the ranks run on
 * distinct GPUs of one node (the kernel of one rank waits for the kernels of
 * the others).  The exchange buffer holds two steps (alternating), so a rank
 * can run one step ahead of another.  wait_ms bounds each step's wait for the
 * other ranks (0: 2000 ms); choose it above the longest delay expected between
 * ranks (module loading, host work on one rank, SMs held by other streams).  A
 * step whose wait runs out records TQ_ERROR_TIMEOUT, read by
 * tq_peer_exchange_status, and leaves the exchange unusable: recovery is
 * teardown plus a new exchange on every rank.  The kernel's grid is capped at
 * the device's SM count, so all its CTAs are resident while they wait.
 * Callers must check tq_peer_exchange_status before trusting an output.
 * Teardown: tq_peer_exchange_disconnect on every rank, a host barrier, then
 * tq_peer_exchange_destroy.  Not for CUDA graph capture: each call passes its
 * step number to the kernel.
 */
typedef struct tq_peer_exchange tq_peer_exchange;
#define TQ_PEER_HANDLE_BYTES 64
#define TQ_PEER_MAX_WORLD 64
tq_status tq_peer_exchange_create(int world, int rank, int64_t n_rows, int head_dim, uint32_t wait_ms,
                                  tq_peer_exchange **ex, void *handle_out);
tq_status tq_peer_exchange_connect(tq_peer_exchange *ex, const void *handles);
tq_status tq_peer_exchange_merge(tq_peer_exchange *ex, const float *part, void *out, tq_dtype out_dtype,
                                 float *lse_out, void *stream);
/* One split-sequence step with the exchange fused into the attention: the decode attention of
 * `args` (this rank's token shard of every context; args->out and args->lse are not written)
 * stores each (sequence, KV head) pair's rows [o | lse] into this step's slot of every rank's
 * exchange buffer as soon as the pair is complete, and counts the pair in every rank's arrival
 * counter; a merge kernel then waits (bounded) for the pairs of all ranks and writes the merged
 * output to `out` (and lse_out).  The transfers of early pairs overlap the attention of later
 * ones.  Requires batch * n_q_heads == n_rows and head_dim of the exchange; the result equals
 * tq_decode_attention_cuda + tq_peer_exchange_merge bit for bit.  Every rank calls the same
 * sequence of tq_peer_exchange_merge / tq_peer_exchange_attention steps.  No counterpart in the
 * reference. */
tq_status tq_peer_exchange_attention(tq_peer_exchange *ex, const tq_decode_attention_args *args, void *out,
                                     tq_dtype out_dtype, float *lse_out, void *stream);
/* synchronizes the stream, then returns the kernel-side status of the steps so far */
tq_status tq_peer_exchange_status(tq_peer_exchange *ex, void *stream);
tq_status tq_peer_exchange_disconnect(tq_peer_exchange *ex);
tq_status tq_peer_exchange_destroy(tq_peer_exchange *ex);

#ifdef __cplusplus
}
#endif

#endif /* LEANKV_TQ_H */
