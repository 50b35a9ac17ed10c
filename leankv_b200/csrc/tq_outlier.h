// tq_outlier.h — internal interface of the mixed-precision (outlier channel) kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace tq {

constexpr int OUTLIER_MAX_DIM = 256;   // TQ_OUTLIER_MAX_DIM of src/ggml-tq-outlier.h:40

// what the kernels need from a tq_outlier_config: tiers as block types (2, 3, 4) and perm
struct MixedPlan {
    int head_dim = 0;
    int n_outlier = 0;
    int otype = 2;
    int ntype = 2;
    int perm[OUTLIER_MAX_DIM];
};

cudaError_t launch_outlier_calib(const float* data, int n_tokens, int hd, float* var, int* perm, int* inv,
                                 cudaStream_t st);
cudaError_t launch_mixed_quantize(int in_dtype, const void* x, int64_t n_vec, const MixedPlan& plan, void* obuf,
                                  void* nbuf, cudaStream_t st);
cudaError_t launch_mixed_dequantize(const void* obuf, const void* nbuf, int64_t n_vec, const MixedPlan& plan, float* y,
                                    cudaStream_t st);
// TQ2_1 blocks (44 bytes per 128 elements: a TQ3_0 block, then three TQ2_0 blocks)
constexpr int TQ21_BYTES = 44;
cudaError_t launch_tq21_quantize(int in_dtype, const void* x, int64_t nblocks, void* y, cudaStream_t st);
cudaError_t launch_tq21_dequantize(const void* x, int64_t nblocks, float* y, cudaStream_t st);
// y[v][i] = x[v][plan.perm[i]] (plan.perm may hold an inverse permutation)
cudaError_t launch_gather(const float* x, const MixedPlan& plan, int64_t n_vec, float* y, cudaStream_t st);

}  // namespace tq
