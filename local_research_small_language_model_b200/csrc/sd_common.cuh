// Shared device/host helpers for the sm_100a kernels of this library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spardab200.h"

namespace sd {

// ---------------------------------------------------------------- host side
void set_cuda_error(cudaError_t e);
int check_launch();  // SD_OK or SD_ERR_CUDA after a launch

inline bool dtype_ok(int dt) { return dt == SD_DTYPE_F32 || dt == SD_DTYPE_BF16 || dt == SD_DTYPE_F16; }
inline int dtype_size(int dt) { return dt == SD_DTYPE_F32 ? 4 : 2; }
inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// 1/sqrt(D) rounded once to fp32, as a Python float scale is when it multiplies
// an fp32 tensor (model/forecast.py:115-116).
float inv_sqrt(int64_t d);
// Raises a kernel's dynamic shared-memory limit when `bytes` exceeds 48 KB.
int set_max_smem_raw(const void *func, size_t bytes);
template <typename K> int set_max_smem(K *func, size_t bytes) {
  return set_max_smem_raw(reinterpret_cast<const void *>(func), bytes);
}

// Programmatic dependent launch (sd_set_programmatic_launch): when enabled,
// the kernels that support it are launched so they may start before the
// kernel ahead of them on the stream has finished; each waits (pdl_wait) before
// it reads anything that kernel wrote.
bool pdl_enabled();

// Launches kern<<<grid, block, smem, s>>>(args...), with programmatic stream
// serialization when `pdl` is set; returns SD_OK or SD_ERR_CUDA.
template <typename... KArgs, typename... Args>
int launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args &&...args) {
  if (!pdl) {
    kern<<<grid, block, smem, s>>>(static_cast<KArgs>(args)...);
    return check_launch();
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    cudaGetLastError();
    return SD_ERR_CUDA;
  }
  return check_launch();
}

// As launch(), with thread-block clusters of `cluster` CTAs (grid dims
// multiples of it); a 1 x 1 x 1 cluster launches without the attribute.
template <typename... KArgs, typename... Args>
int launch_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, dim3 cluster, size_t smem, cudaStream_t s, bool pdl,
                   Args &&...args) {
  if (cluster.x * cluster.y * cluster.z == 1) return launch(kern, grid, block, smem, s, pdl, args...);
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = cluster.x;
  attr[na].val.clusterDim.y = cluster.y;
  attr[na].val.clusterDim.z = cluster.z;
  ++na;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    cudaGetLastError();
    return SD_ERR_CUDA;
  }
  return check_launch();
}

// ---------------------------------------------------------------- conversions
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Round a float to T's precision and back (identity for float).
template <typename T> __device__ __forceinline__ float round_to(float x) { return to_f<T>(from_f<T>(x)); }

// One rotated element with the reference's rounding sequence
// (model/rope.py:58-63): the fp32 tables cast to T, then x*cos and
// rotate_half(x)*sin and their sum each rounded to T.  rot is the element of
// rotate_half(x) at this position (-x[d + D/2] in the first half, x[d - D/2]
// in the second).
template <typename T> __device__ __forceinline__ float rope_rounded(float x, float rot, float c, float s) {
  const float a = round_to<T>(__fmul_rn(x, round_to<T>(c)));
  const float b = round_to<T>(__fmul_rn(rot, round_to<T>(s)));
  return round_to<T>(__fadd_rn(a, b));
}

// ---------------------------------------------------------------- PTX wrappers
// Waits until the kernel ahead of this one on the stream has completed and its
// writes are visible; returns at once when this kernel was not launched with
// programmatic stream serialization.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the given phase parity with a wall-clock bound (nanoseconds).
// Returns false when the bound expired; never spins forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 0; i < (1u << 30); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && global_timer_ns() - t0 > limit_ns) return false;
  }
  return false;
}

// Bulk (TMA, non-tensor) copy global -> shared, completion counted on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's earlier generic-proxy global writes before later
// async-proxy (bulk copy) reads issued after a CTA barrier.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- top-k
// Total order used everywhere for top-k: larger value first; equal values
// (including -inf) by ascending index.
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// One warp selects the k best of n entries; entry j has value get(j).
// Writes k (index, value) pairs in order.  Entries are visited without
// mutation: round r takes the best entry strictly after round r-1's winner in
// the total order.  NaN values are never selected.
template <typename Get>
__device__ __forceinline__ void warp_topk(Get get, int n, int k, int *out_idx, float *out_val) {
  const int lane = threadIdx.x & 31;
  float pv = INFINITY;
  int pi = -1;
  bool first = true;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = lane; j < n; j += 32) {
      const float v = get(j);
      // NaN marks an entry that must never be chosen, in any round
      const bool elig = (v == v) && (first || (v < pv) || (v == pv && j > pi));
      if (elig && (bi == 0x7fffffff || better(v, j, bv, bi))) {
        bv = v;
        bi = j;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || better(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_idx[r] = bi == 0x7fffffff ? -1 : bi;
      if (out_val) out_val[r] = bv;
    }
    pv = bv;
    pi = bi;
    first = false;
  }
}

// Like warp_topk, but candidate c has value val(c) and block index idx(c),
// which both orders ties and is written out.  Used to merge per-warp top-k
// lists; idx values must be distinct.
template <typename Val, typename Idx>
__device__ __forceinline__ void warp_topk_kv(Val val, Idx idx, int n, int k, int *out_idx) {
  const int lane = threadIdx.x & 31;
  float pv = INFINITY;
  int pi = -1;
  bool first = true;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < n; c += 32) {
      const float v = val(c);
      const int j = idx(c);
      // NaN marks an entry that must never be chosen, in any round
      const bool elig = (v == v) && (first || (v < pv) || (v == pv && j > pi));
      if (elig && (bi == 0x7fffffff || better(v, j, bv, bi))) {
        bv = v;
        bi = j;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || better(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) out_idx[r] = bi == 0x7fffffff ? -1 : bi;
    pv = bv;
    pi = bi;
    first = false;
  }
}

}  // namespace sd

// Expands BODY with `T` bound to the element type of SD_DTYPE_* code `dt`;
// returns SD_ERR_INVALID from the enclosing function for unknown codes.
#define SD_DISPATCH_DTYPE(dt, T, ...)                 \
  switch (dt) {                                       \
    case SD_DTYPE_F32: {                              \
      using T = float;                                \
      __VA_ARGS__;                                    \
    } break;                                          \
    case SD_DTYPE_BF16: {                             \
      using T = __nv_bfloat16;                        \
      __VA_ARGS__;                                    \
    } break;                                          \
    case SD_DTYPE_F16: {                              \
      using T = __half;                               \
      __VA_ARGS__;                                    \
    } break;                                          \
    default:                                          \
      return SD_ERR_INVALID;                          \
  }
