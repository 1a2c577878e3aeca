// Decode-time block selection shared by sd_decode_select and the fused decode
// layer kernel: the selected-set logic of model/attention/sparse.py:108-154.
#pragma once

#include "sd_common.cuh"

namespace sd {

// Scores prototypes 0..n_scored-1 of one (sequence, kv head) against the fp32
// forecast `f` (shared memory, D floats) into `scores` (shared memory).
// reps + j*r_sn is block j's prototype row (D floats); `mul` is applied to
// every dot product (1/sqrt(D), times 1/block_size when reps hold sums).
// All threads of the CTA participate; blockDim.x is a multiple of 32.
__device__ __forceinline__ void score_blocks(const float *__restrict__ reps, int64_t r_sn, int D,
                                             const float *f, int n_scored, float mul, float *scores) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int half = lane >> 4, l16 = lane & 15;
  const int nvec = D >> 2;
  if (D == 64) {
    // 16 prototype rows per warp per step: each half-warp reads 8 rows (one
    // float4 per lane per row), all loads issued before any reduction so a
    // warp keeps 8 independent DRAM requests in flight
    constexpr int U = 8;
    const float4 q = reinterpret_cast<const float4 *>(f)[l16];
    for (int j0 = 2 * U * warp; j0 < n_scored; j0 += 2 * U * nwarps) {
      float4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + 2 * u + half;
        r[u] = j < n_scored ? reinterpret_cast<const float4 *>(reps + static_cast<int64_t>(j) * r_sn)[l16]
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float acc = 0.f;
        acc = fmaf(q.x, r[u].x, acc);
        acc = fmaf(q.y, r[u].y, acc);
        acc = fmaf(q.z, r[u].z, acc);
        acc = fmaf(q.w, r[u].w, acc);
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        const int j = j0 + 2 * u + half;
        if (l16 == 0 && j < n_scored) scores[j] = acc * mul;
      }
    }
    return;
  }
  // generic D: two blocks per warp per step, each read by a half-warp as float4 chunks
  for (int j0 = 2 * warp; j0 < n_scored; j0 += 2 * nwarps) {
    const int j = j0 + half;
    float acc = 0.f;
    if (j < n_scored) {
      const float4 *row = reinterpret_cast<const float4 *>(reps + static_cast<int64_t>(j) * r_sn);
      for (int c = l16; c < nvec; c += 16) {
        const float4 r = row[c];  // plain load: rows may have been written earlier in the same kernel
        const float4 q = reinterpret_cast<const float4 *>(f)[c];
        acc = fmaf(q.x, r.x, acc);
        acc = fmaf(q.y, r.y, acc);
        acc = fmaf(q.z, r.z, acc);
        acc = fmaf(q.w, r.w, acc);
      }
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (l16 == 0 && j < n_scored) scores[j] = acc * mul;
  }
}

// The union {0, curr} U top-k (use_forecast) or {0} U the static window
// ending at curr, future blocks cleared (sparse.py:126-151), written to
// list in ascending order; returns its length.  One thread.
__device__ __forceinline__ int assemble_decode_list(bool use_forecast, const int *topk, int kk, int nb, int curr,
                                                    int top_k, int *list) {
  int n = 0;
  auto add = [&](int j) {
    if (j < 0 || j > curr) return;  // future blocks are cleared (sparse.py:150-151)
    int p = n;
    for (int i = 0; i < n; ++i) {
      if (list[i] == j) return;
      if (list[i] > j) {
        p = i;
        break;
      }
    }
    for (int i = n; i > p; --i) list[i] = list[i - 1];
    list[p] = j;
    ++n;
  };
  add(0);
  add(curr);
  if (use_forecast) {
    for (int i = 0; i < kk; ++i) add(topk[i] < nb - 1 ? topk[i] : nb - 1);
  } else {
    for (int j = curr - top_k + 1 > 0 ? curr - top_k + 1 : 0; j <= curr; ++j) add(j);
  }
  return n;
}

// Top-kk of n entries by the shared total order (value desc, index asc),
// written to out_idx; val(j) may return NaN for entries that must not be
// chosen.  Every warp takes the top-kk of a contiguous slice, then warp 0
// merges the slices' candidates.  All threads call this; it ends with a
// barrier.
template <typename Val>
__device__ __forceinline__ void cta_topk(Val val, int n, int kk, int *out_idx) {
  __shared__ int cand_i[256];
  __shared__ float cand_v[256];
  const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (nw * kk <= 256 && n >= 4 * 32) {
    const int seg = (n + nw - 1) / nw;
    const int lo = warp * seg, len = lo < n ? (n - lo < seg ? n - lo : seg) : 0;
    int *ci = cand_i + warp * kk;
    if (len >= kk) {
      warp_topk([&](int j) { return val(lo + j); }, len, kk, ci, nullptr);
      __syncwarp();
    }
    for (int r = lane; r < kk; r += 32) {
      const int li = len >= kk ? ci[r] : (r < len ? r : -1);
      if (li >= 0) {
        ci[r] = lo + li;
        cand_v[warp * kk + r] = val(lo + li);
      } else {  // exhausted slice: an entry that never wins
        ci[r] = 0x70000000 + warp * 64 + r;
        cand_v[warp * kk + r] = -INFINITY;
      }
    }
    __syncthreads();
    if (warp == 0)
      warp_topk_kv([&](int c) { return cand_v[c]; }, [&](int c) { return cand_i[c]; }, nw * kk, kk, out_idx);
  } else if (threadIdx.x < 32) {
    warp_topk(val, n, kk, out_idx, nullptr);
  }
  __syncthreads();
}

// Builds the ascending selected-block list into list[0..*count).  `scores`
// holds the scores of blocks 0..n_scored-1; blocks n_scored..nb-1 count as -inf.
// topk_tmp needs room for top_k ints.  Must be called by all threads.
__device__ __forceinline__ void build_decode_list(bool use_forecast, const float *scores, int n_scored,
                                                  int nb, int curr, int top_k, int ms, int *topk_tmp,
                                                  int *list, int *count) {
  if (nb <= ms) {  // dense fallback: every block
    for (int j = threadIdx.x; j < nb; j += blockDim.x) list[j] = j;
    if (threadIdx.x == 0) *count = nb;
    __syncthreads();
    return;
  }
  const int kk = top_k < nb ? top_k : nb;
  if (use_forecast) cta_topk([&](int j) { return j < n_scored ? scores[j] : -INFINITY; }, nb, kk, topk_tmp);
  if (threadIdx.x == 0) *count = assemble_decode_list(use_forecast, topk_tmp, kk, nb, curr, top_k, list);
  __syncthreads();
}

}  // namespace sd
