// Constants shared by the prefill kernels (list builder, CUDA-core and
// tensor-core attention).
#pragma once

#include "sd_common.cuh"

namespace sd {

constexpr int kQTile = 64;     // query rows per tile == block size the prefill kernels implement
constexpr int kHeadDim = 64;   // head_dim the prefill kernels implement
constexpr float kLog2eF = 1.4426950408889634f;

// Selection modes of sd_prefill_lists (values of the C ABI's SD_LIST_*).
constexpr int kListDense = SD_LIST_DENSE;
constexpr int kListMaskedForecast = SD_LIST_MASKED_FORECAST;
constexpr int kListMaskedStatic = SD_LIST_MASKED_STATIC;
constexpr int kListChunkedForecast = SD_LIST_CHUNKED_FORECAST;
constexpr int kListChunkedStatic = SD_LIST_CHUNKED_STATIC;

// Tensor-core (tcgen05) prefill attention for 16-bit inputs; returns
// SD_ERR_UNSUPPORTED without launching when the inputs fall outside it
// (fp32, G > 4, per-row top-k wider than 16, unaligned strides).
int launch_prefill_tc(int dtype, int G, dim3 grid, cudaStream_t s, const void *q, int64_t q_sb, int64_t q_st,
                      int64_t q_sh, const void *k, const void *v, int64_t c_sb, int64_t c_sh, int64_t c_st,
                      int64_t T_, int Hkv, int64_t B, const int32_t *lists, const int32_t *counts, int lcap,
                      const int64_t *topk, int kk, int causal, float scale_log2, void *out, int64_t o_sb,
                      int64_t o_st, int64_t o_sh);

}  // namespace sd
