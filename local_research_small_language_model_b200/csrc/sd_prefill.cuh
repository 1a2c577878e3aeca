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

}  // namespace sd
