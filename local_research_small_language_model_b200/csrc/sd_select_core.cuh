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

// ------------------------------------------------------------ warp groups
// Whole warps [w0, w0 + nw) of a CTA that work together, synchronised by
// named barrier `id` (0: the whole CTA through __syncthreads).  Lets one set of
// warps score blocks while the others of the same CTA do something else.
struct WarpGroup {
  int w0, nw, id;
  __device__ __forceinline__ int warp() const { return static_cast<int>(threadIdx.x >> 5) - w0; }
  __device__ __forceinline__ void sync() const {
    if (id == 0) {
      __syncthreads();
    } else {
      asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nw * 32) : "memory");
    }
  }
};
__device__ __forceinline__ WarpGroup whole_cta() { return WarpGroup{0, static_cast<int>(blockDim.x >> 5), 0}; }

// ------------------------------------------------------------ register top-k
// Entry that is never chosen: loses every comparison, including -inf ties
// (ties are ordered by ascending index).
constexpr int kNoBlock = 0x7fffffff;

// Compare-exchange of a bitonic network step with partner lane^j: in a run
// sorted best-first (`best_first`), the lower lane keeps the better entry.
// Keys are distinct except for identical kNoBlock entries, so "self is
// better" is "other is not better"; written without branches so the warp
// never diverges inside the network.
__device__ __forceinline__ void bitonic_step(float &v, int &i, int j, bool best_first) {
  const float ov = __shfl_xor_sync(0xffffffffu, v, j);
  const int oi = __shfl_xor_sync(0xffffffffu, i, j);
  const bool lower = (threadIdx.x & j) == 0;
  const bool other_better = (ov > v) | ((ov == v) & (oi < i));
  const bool take = other_better ^ (lower != best_first);
  v = take ? ov : v;
  i = take ? oi : i;
}

// Sorts every group of K2 lanes best-first (bitonic sort network).
template <int K2> __device__ __forceinline__ void sort_groups(float &v, int &i) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= K2; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) bitonic_step(v, i, j, k == K2 || (lane & k) == 0);
}

// Sorts a bitonic sequence held by each group of K2 lanes best-first.
template <int K2> __device__ __forceinline__ void half_clean(float &v, int &i) {
#pragma unroll
  for (int j = K2 >> 1; j > 0; j >>= 1) bitonic_step(v, i, j, true);
}

// Each group of K2 lanes holds a best-first list in (av, ai) and another in
// (bv, bi); leaves the best K2 of both, best-first, in (av, ai).  best(A[l],
// B[K2-1-l]) is a bitonic sequence holding exactly that set.
template <int K2> __device__ __forceinline__ void merge_regs(float &av, int &ai, float bv, int bi) {
  const float pv = __shfl_xor_sync(0xffffffffu, bv, K2 - 1);
  const int pi = __shfl_xor_sync(0xffffffffu, bi, K2 - 1);
  const bool take = (pv > av) | ((pv == av) & (pi < ai));
  av = take ? pv : av;
  ai = take ? pi : ai;
  half_clean<K2>(av, ai);
}

// Every group of K2 lanes holds a best-first list; leaves the best K2 of all
// 32/K2 lists, best-first, in lanes 0..K2-1.  At block size s the list of
// lanes [0, K2) of an s-block meets the mirrored copy of its neighbour's list
// (lane l ^ (2s - 1)).
template <int K2> __device__ __forceinline__ void merge_lanes(float &v, int &i) {
#pragma unroll
  for (int s = K2; s < 32; s <<= 1) {
    const float pv = __shfl_xor_sync(0xffffffffu, v, 2 * s - 1);
    const int pi = __shfl_xor_sync(0xffffffffu, i, 2 * s - 1);
    const bool take = (pv > v) | ((pv == v) & (pi < i));
    v = take ? pv : v;
    i = take ? pi : i;
    half_clean<K2>(v, i);
  }
}

// Fused scoring + top-kk of one (sequence, kv head), all in registers:
// block j's score is dot(f, row(j)[0 .. 64)) * mul for j < n_scored (row(j):
// a 16-byte aligned fp32 row in global or shared memory), -inf for
// n_scored <= j < n, and block `excl` is never chosen.  Every warp takes 32
// blocks per chunk: lane (half, l16) loads float4 l16 of blocks 32c+2i+half
// for i = 0..15 (coalesced, 16 loads in flight), then a 4-step reduce-scatter
// leaves block 32c+2*l16+half's score in that lane; the dot products sum in
// the same order as score_blocks (per-lane fma chain over 4 dims, then lane
// pairs 8, 4, 2, 1 apart), so scores are bit-identical.  Each chunk's K2-lane
// groups are sorted and merged across lanes, then into the warp's running
// list; warp 0 merges the warps' lists the same way.  The order of merges
// does not change the result: entries are ordered by (value desc, index asc).  Writes
// kk <= K2 (index, value) pairs best-first to out_idx (-1 when fewer than kk
// entries exist) and out_val (nullable); NaN scores are never chosen.  All
// threads of warp group g (at most 8 warps) call it; it ends with the group's
// barrier.  sv, si: shared scratch of g.nw * K2 entries.  fv: the lane's
// float4 l16 of the fp32 forecast.  Rows are read with plain
// (coherent) loads: the fused decode kernel writes one of them earlier in the
// same launch.
template <int K2, typename Row>
__device__ __forceinline__ void cta_score_topk_k2(Row row, float4 fv, int n, int n_scored, int excl, float mul,
                                                  int kk, int *out_idx, float *out_val, float *sv, int *si,
                                                  const WarpGroup &g) {
  const int lane = threadIdx.x & 31, warp = g.warp(), nw = g.nw;
  const int half = lane >> 4, l16 = lane & 15;
  if (n_scored > n) n_scored = n;
  float rv = -INFINITY;  // running best-first list of this warp (K2-lane groups)
  int ri = kNoBlock;
  // one 32-block chunk per iteration; the loop stays rolled so its code is
  // fetched once however many chunks a warp takes (the kernels that inline
  // this run it once per launch, where instruction fetch, not issue, is what
  // an unrolled copy would cost)
#pragma unroll 1
  for (int c0 = 32 * warp; c0 < n; c0 += 32 * nw) {
    float p[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = c0 + 2 * i + half;
      float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < n_scored) r = reinterpret_cast<const float4 *>(row(j))[l16];
      float a = 0.f;
      a = fmaf(fv.x, r.x, a);
      a = fmaf(fv.y, r.y, a);
      a = fmaf(fv.z, r.z, a);
      a = fmaf(fv.w, r.w, a);
      p[i] = a;
    }
#pragma unroll
    for (int d = 8; d > 0; d >>= 1) {
      const bool hi = (lane & d) != 0;
#pragma unroll
      for (int j = 0; j < d; ++j) {
        const float send = hi ? p[j] : p[j + d];
        const float keep = hi ? p[j + d] : p[j];
        p[j] = keep + __shfl_xor_sync(0xffffffffu, send, d);
      }
    }
    const int b = c0 + 2 * l16 + half;
    const float v = b < n_scored ? p[0] * mul : -INFINITY;
    const bool ok = b < n && b != excl && v == v;
    float cv = ok ? v : -INFINITY;
    int ci = ok ? b : kNoBlock;
    sort_groups<K2>(cv, ci);
    merge_lanes<K2>(cv, ci);
    if (c0 == 32 * warp) {  // first chunk: nothing to merge with yet
      rv = cv;
      ri = ci;
    } else {
      merge_regs<K2>(rv, ri, cv, ci);  // both lists sit in lanes 0..K2-1
    }
  }
  if (lane < K2) {
    sv[warp * K2 + lane] = rv;
    si[warp * K2 + lane] = ri;
  }
  g.sync();
  if (warp == 0) {
    const int total = nw * K2;
    float v = lane < total ? sv[lane] : -INFINITY;
    int i = lane < total ? si[lane] : kNoBlock;
    for (int r = 32; r < total; r += 32) {
      const bool in = r + lane < total;
      merge_regs<K2>(v, i, in ? sv[r + lane] : -INFINITY, in ? si[r + lane] : kNoBlock);
    }
    merge_lanes<K2>(v, i);
    if (lane < kk) {
      out_idx[lane] = i == kNoBlock ? -1 : i;
      if (out_val) out_val[lane] = v;
    }
  }
  g.sync();
}

// Folding U candidates per lane into a running best-first top-8 list held in
// lanes 0..7 (rv, ri; the rest of the lanes hold (-inf, kNoBlock) pads), for
// warps that walk one row's scores chunk by chunk.  The first fold sorts the
// candidates' 8-lane groups and merges them in a tournament.  Later folds:
// only a candidate that beats the list's 8th entry can enter, which few do,
// so a ballot filters against that threshold and the survivors are inserted
// one at a time.  Both give the best 8 of everything folded so far, by
// (value desc, index asc).
template <int U>
__device__ __forceinline__ void fold_first8(float &rv, int &ri, float (&cv)[U], int (&ci)[U]) {
#pragma unroll
  for (int u = 0; u < U; ++u) sort_groups<8>(cv[u], ci[u]);
#pragma unroll
  for (int w = 1; w < U; w <<= 1)
#pragma unroll
    for (int u = 0; u + w < U; u += 2 * w) merge_regs<8>(cv[u], ci[u], cv[u + w], ci[u + w]);
  merge_lanes<8>(cv[0], ci[0]);
  merge_regs<8>(rv, ri, cv[0], ci[0]);
}

template <int U>
__device__ __forceinline__ void fold_insert8(float &rv, int &ri, const float (&cv)[U], const int (&ci)[U]) {
  const int lane = threadIdx.x & 31;
  float tv = __shfl_sync(0xffffffffu, rv, 7);
  int ti = __shfl_sync(0xffffffffu, ri, 7);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    unsigned m = __ballot_sync(0xffffffffu, ci[u] != kNoBlock && (ti == kNoBlock || better(cv[u], ci[u], tv, ti)));
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1;
      const float nv = __shfl_sync(0xffffffffu, cv[u], src);
      const int ni = __shfl_sync(0xffffffffu, ci[u], src);
      if (!(ti == kNoBlock || better(nv, ni, tv, ti))) continue;  // an earlier insertion raised the bar
      // position = entries better than the newcomer; later entries move down one lane
      const bool above = lane < 8 && ri != kNoBlock && better(rv, ri, nv, ni);
      const int pos = __popc(__ballot_sync(0xffffffffu, above));
      const float upv = __shfl_up_sync(0xffffffffu, rv, 1);
      const int upi = __shfl_up_sync(0xffffffffu, ri, 1);
      if (lane < 8 && lane > pos) {
        rv = upv;
        ri = upi;
      } else if (lane == pos) {
        rv = nv;
        ri = ni;
      }
      tv = __shfl_sync(0xffffffffu, rv, 7);
      ti = __shfl_sync(0xffffffffu, ri, 7);
    }
  }
}

// Scoring + top-kk (kk <= 32) by warp group g with caller-provided scratch
// sv, si (g.nw * 32 entries each).
template <typename Row>
__device__ __forceinline__ void group_score_topk(Row row, float4 fv, int n, int n_scored, int excl, float mul, int kk,
                                                 int *out_idx, float *out_val, float *sv, int *si,
                                                 const WarpGroup &g) {
  // two list widths keep the number of instantiations (and build time) small:
  // a top-kk list is the first kk entries of the top-8 or top-32 list
  if (kk <= 8) {
    cta_score_topk_k2<8>(row, fv, n, n_scored, excl, mul, kk, out_idx, out_val, sv, si, g);
  } else {
    cta_score_topk_k2<32>(row, fv, n, n_scored, excl, mul, kk, out_idx, out_val, sv, si, g);
  }
}

template <typename Row>
__device__ __forceinline__ void cta_score_topk_rows(Row row, float4 fv, int n, int n_scored, int excl, float mul,
                                                    int kk, int *out_idx, float *out_val) {
  __shared__ float sv[8 * 32];  // the warps' lists, one buffer for every K2
  __shared__ int si[8 * 32];
  group_score_topk(row, fv, n, n_scored, excl, mul, kk, out_idx, out_val, sv, si, whole_cta());
}

// cta_score_topk_rows over rows reps + j*r_sn (global memory).
__device__ __forceinline__ void cta_score_topk(const float *reps, int64_t r_sn, float4 fv, int n, int n_scored,
                                               int excl, float mul, int kk, int *out_idx, float *out_val) {
  cta_score_topk_rows([&](int j) { return reps + static_cast<int64_t>(j) * r_sn; }, fv, n, n_scored, excl, mul, kk,
                      out_idx, out_val);
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
