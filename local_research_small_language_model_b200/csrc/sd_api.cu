// Library-wide entry points: error text, version, last CUDA error, length bump.
#include <math.h>

#include <atomic>

#include "sd_common.cuh"

namespace sd {

static thread_local int g_last_cuda_error = 0;
static std::atomic<int> g_pdl{0};

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

void set_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SD_ERR_CUDA;
  }
  return SD_OK;
}

float inv_sqrt(int64_t d) { return static_cast<float>(1.0 / sqrt(static_cast<double>(d))); }

int set_max_smem_raw(const void *func, size_t bytes) {
  if (bytes <= 48 * 1024) return SD_OK;
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) {
    set_cuda_error(e);
    cudaGetLastError();
    return SD_ERR_CUDA;
  }
  return SD_OK;
}

__global__ void advance_len_kernel(int32_t *lens, int n, int delta) {
  pdl_wait();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) lens[i] += delta;
}

}  // namespace sd

extern "C" {

const char *sd_strerror(int code) {
  switch (code) {
    case SD_OK: return "ok";
    case SD_ERR_INVALID: return "invalid argument (shape, stride, pointer or value)";
    case SD_ERR_UNSUPPORTED: return "unsupported configuration for the sm_100a kernels";
    case SD_ERR_CUDA: return "CUDA runtime error (see sd_last_cuda_error)";
    case SD_ERR_ALIGN: return "pointer or stride not 16-byte aligned as bulk copies require";
    default: return "unknown error";
  }
}

int sd_version(void) { return 1; }

int sd_last_cuda_error(void) { return sd::g_last_cuda_error; }

int sd_advance_len(int32_t *lens, int n, int delta, void *stream) {
  if (!lens || n <= 0) return SD_ERR_INVALID;
  return sd::launch(sd::advance_len_kernel, dim3((n + 127) / 128), dim3(128), 0, static_cast<cudaStream_t>(stream),
                    sd::pdl_enabled(), lens, n, delta);
}

int sd_set_programmatic_launch(int enable) { return sd::g_pdl.exchange(enable != 0 ? 1 : 0); }

}  // extern "C"
