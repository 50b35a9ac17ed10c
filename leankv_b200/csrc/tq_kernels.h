// tq_kernels.h — internal launchers (C++ linkage, not part of the public ABI).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace tq {

int sm_count();

// Placement of quantized head rows in a KV cache (cap == 0: contiguous output).
// Input head row R = s * n_new + t (s = sequence * hkv + head) is written to token
// slot pos[sequence] + t (pos null: slot t) of s in a [s][cap][nblk blocks] cache;
// rows whose slot is outside [0, cap) are skipped and counted in *overflow.
struct RowMap {
    int64_t cap = 0;
    int64_t n_new = 1;
    int hkv = 1;
    int nblk = 1;
    const int32_t* pos = nullptr;
    int* overflow = nullptr;
    // paged cache (pages != null): slot s of (sequence q, head h) is token s & (2^page_shift - 1)
    // of pool page pages[q * max_pages + (s >> page_shift)], pool [num_pages][hkv][2^page_shift][nblk]
    const int32_t* pages = nullptr;
    int64_t max_pages = 0, num_pages = 0;
    int page_shift = 0;
};

// [FWHT over heads of 2^log2_hd elements when log2_hd >= 0] + quantize nblocks blocks.
// qtype 3 or 4; in_dtype DT_F32/DT_F16/DT_BF16; n_passes > 0 selects TQ3 optimal rounding.
// heads_per_row > 0: randomized_hadamard_transform_row signs (chunk h of a row seeded rseed + h)
// before the rotation (log2_hd >= 5)
cudaError_t launch_quantize(int qtype, int in_dtype, const void* x, void* y, int64_t nblocks, int log2_hd,
                            float norm, int n_passes, cudaStream_t st, const RowMap& map = RowMap(),
                            uint32_t rseed = 0, int heads_per_row = 0);
// in-place FWHT of nblocks 32-element rows (heads of 2^log2_hd <= 1024 elements)
cudaError_t launch_fwht(float* x, int64_t nblocks, int log2_hd, float norm, cudaStream_t st, uint32_t rseed = 0,
                        int heads_per_row = 0);
// decode src_type blocks and encode them as dst_type (types 2, 3, 4)
cudaError_t launch_requantize(int src_type, const void* src, int dst_type, void* dst, int64_t nblocks,
                              cudaStream_t st);
// FWHT of a tail shorter than 32 elements (heads smaller than 32)
cudaError_t launch_fwht_tail(float* x, int n, int log2_hd, float norm, cudaStream_t st);
// FWHT of rows longer than 1024 elements, one CTA per row
cudaError_t launch_fwht_large(float* x, int64_t nrows, int log2_hd, float norm, cudaStream_t st);
cudaError_t launch_dequantize(int qtype, int out_dtype, const void* x, void* y, int64_t nblocks, cudaStream_t st);

}  // namespace tq
