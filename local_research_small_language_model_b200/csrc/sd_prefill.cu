// Prefill side of the path: per-q-tile block lists for every selection mode of
// SparseAttention._forward_masked_sdpa (model/attention/sparse.py:185-282) and
// _forward_chunked_gather (sparse.py:284-364), and a CUDA-core block-sparse
// attention kernel over those lists (fp32 / fp16 / bf16 inputs, fp32 math).
#include "sd_prefill.cuh"

namespace sd {

// One CTA per (q-tile, h, b).  A q-tile is one 64-token query block.
__global__ void prefill_lists_kernel(int mode, int causal, int64_t T, int bs, int top_k, int H,
                                     const int64_t *__restrict__ topk, int kk, int lcap,
                                     int32_t *__restrict__ lists, int32_t *__restrict__ counts) {
  extern __shared__ int votes[];  // [nb]
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nb = static_cast<int>((T + bs - 1) / bs);
  const int nqt = gridDim.x;
  const int bq = qt;  // q-tile == q-block (bs == kQTile)
  const int64_t row0 = static_cast<int64_t>(qt) * bs;
  const int64_t row1 = row0 + bs < T ? row0 + bs : T;
  for (int j = threadIdx.x; j < nb; j += blockDim.x) votes[j] = 0;
  __syncthreads();
  const bool chunked = mode == kListChunkedForecast || mode == kListChunkedStatic;
  const int hi = (causal || chunked) ? bq : nb - 1;  // last block a row of this tile may see
  const bool use_rows = (mode == kListMaskedForecast) || (mode == kListChunkedForecast && bq > 0);
  if (use_rows) {
    const int64_t *base = topk + ((static_cast<int64_t>(b) * H + h) * T) * kk;
    const int64_t n = (row1 - row0) * kk;
    for (int64_t e = threadIdx.x; e < n; e += blockDim.x) {
      int64_t j = base[row0 * kk + e];
      j = j < 0 ? 0 : (j > nb - 1 ? nb - 1 : j);  // clamp as sparse.py:245 / :323
      if (j <= hi) atomicAdd(&votes[j], 1);
    }
  }
  __syncthreads();
  int32_t *dst = lists + ((static_cast<int64_t>(b) * H + h) * nqt + qt) * lcap;
  __shared__ int s_n;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int n = 0;
    if (mode == kListChunkedForecast && bq > 0) {  // union, cut to ms entries (warp-parallel)
      const int ms = nb < top_k + 2 ? nb : top_k + 2;
      int total = 0;
      for (int j0 = 0; j0 <= hi; j0 += 32) {
        const int j = j0 + lane;
        total += __popc(__ballot_sync(0xffffffffu, j <= hi && (votes[j] > 0 || j == 0 || j == bq)));
      }
      if (total > ms) {
        // keep the sink and the diagonal block, then the most-voted blocks
        // (ties: lower index first): a warp top-(ms-2) over blocks 1..bq-1
        __shared__ int s_pick[64];
        warp_topk([&](int i) { return votes[i + 1] > 0 ? static_cast<float>(votes[i + 1]) : NAN; }, bq - 1, ms - 2,
                  s_pick, nullptr);
        __syncwarp();
        for (int i = lane; i < ms - 2; i += 32)
          if (s_pick[i] >= 0) s_pick[i] += 1;
        __syncwarp();
        // mark the kept blocks, then the rest of the union is dropped
        for (int j0 = 0; j0 <= hi; j0 += 32) {
          const int j = j0 + lane;
          if (j <= hi) {
            bool keep = j == 0 || j == bq;
            for (int i = 0; i < ms - 2; ++i) keep = keep || s_pick[i] == j;
            votes[j] = keep ? 1 : 0;
          }
        }
        __syncwarp();
      } else {
        for (int j0 = 0; j0 <= hi; j0 += 32) {
          const int j = j0 + lane;
          if (j <= hi && (j == 0 || j == bq)) votes[j] = 1;
        }
        __syncwarp();
      }
      // emit the kept blocks in ascending order
      for (int j0 = 0; j0 <= hi; j0 += 32) {
        const int j = j0 + lane;
        const bool on = j <= hi && votes[j] > 0;
        const unsigned m = __ballot_sync(0xffffffffu, on);
        const int slot = n + __popc(m & ((1u << lane) - 1u));
        if (on && slot < lcap) dst[slot] = j;
        n += __popc(m);
      }
      n = n < lcap ? n : lcap;
    } else if (lane == 0) {
      if (mode == kListDense) {
        for (int j = 0; j <= hi && n < lcap; ++j) dst[n++] = j;
      } else if (mode == kListMaskedStatic || mode == kListChunkedStatic || mode == kListChunkedForecast) {
        // masked window: bk <= bq and bq - bk < top_k + 1 (sparse.py:250);
        // chunked window: bq - top_k + 1 .. bq (sparse.py:325-328, also the
        // forecast mode's first q-block); the sink always
        const int w = mode == kListMaskedStatic ? top_k + 1 : top_k;
        const int lo = bq - w + 1 > 0 ? bq - w + 1 : 0;
        if (lo > 0 && n < lcap) dst[n++] = 0;
        for (int j = lo; j <= bq && n < lcap; ++j) dst[n++] = j;
      } else {  // kListMaskedForecast: every row's top-k with the sink and the diagonal block
        votes[0] += 1;
        if (bq <= hi) votes[bq] += 1;
        for (int j = 0; j <= hi && n < lcap; ++j)
          if (votes[j] > 0) dst[n++] = j;
      }
    }
    if (lane == 0) s_n = n;
  }
  __syncthreads();
  const int n = s_n;
  if (threadIdx.x == 0) counts[(static_cast<int64_t>(b) * H + h) * nqt + qt] = n;
  for (int i = n + threadIdx.x; i < lcap; i += blockDim.x) dst[i] = -1;
}

// CUDA-core block-sparse prefill attention.  One CTA per (q-tile, h, b) with
// 64*G threads: thread (g, r) owns query row r of head h*G+g, keeps q and the
// fp32 accumulator in registers and streams the listed K/V blocks through
// shared memory (every thread reads the same key row: broadcast loads).
constexpr int kKeyChunk = 16;

template <typename T, int G>
__global__ void __launch_bounds__(64 * G)
    prefill_simt_kernel(const T *__restrict__ q, int64_t q_sb, int64_t q_st, int64_t q_sh, const T *__restrict__ k,
                        const T *__restrict__ v, int64_t c_sb, int64_t c_sh, int64_t c_st, int64_t T_, int Hkv,
                        const int32_t *__restrict__ lists, const int32_t *__restrict__ counts, int lcap,
                        const int64_t *__restrict__ topk, int kk, int bs, int causal, float scale_log2,
                        T *__restrict__ out, int64_t o_sb, int64_t o_st, int64_t o_sh) {
  __shared__ float ks[kQTile][kHeadDim];
  __shared__ float vs[kQTile][kHeadDim];
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nqt = gridDim.x;
  const int g = threadIdx.x / kQTile, r = threadIdx.x % kQTile;
  const int64_t t = static_cast<int64_t>(qt) * kQTile + r;
  const bool row_ok = t < T_;
  const int hq = h * G + g;
  float qr[kHeadDim], acc[kHeadDim];
  if (row_ok) {
    const T *qp = q + b * q_sb + t * q_st + hq * q_sh;
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) qr[d] = to_f(qp[d]) * scale_log2;
  } else {
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) qr[d] = 0.f;
  }
#pragma unroll
  for (int d = 0; d < kHeadDim; ++d) acc[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int64_t lrow = (static_cast<int64_t>(b) * Hkv + h) * nqt + qt;
  const int32_t *list = lists + lrow * lcap;
  int cnt = counts[lrow];
  cnt = cnt < 0 ? 0 : (cnt > lcap ? lcap : cnt);
  const int64_t *rowk = (topk && row_ok) ? topk + ((static_cast<int64_t>(b) * Hkv + h) * T_ + t) * kk : nullptr;
  const int bq = static_cast<int>(t / bs);
  const int64_t nbk = (T_ + bs - 1) / bs;
  const T *kb = k + b * c_sb + h * c_sh;
  const T *vb = v + b * c_sb + h * c_sh;
  for (int i = 0; i < cnt; ++i) {
    const int j = list[i];
    if (j < 0 || j >= nbk) continue;  // uniform: skips are the same for every thread
    const int64_t k0 = static_cast<int64_t>(j) * bs;
    __syncthreads();
    for (int e = threadIdx.x; e < kQTile * kHeadDim; e += blockDim.x) {
      const int rr = e / kHeadDim, d = e % kHeadDim;
      const int64_t kt = k0 + rr;
      const bool ok = rr < bs && kt < T_;
      ks[rr][d] = ok ? to_f(kb[kt * c_st + d]) : 0.f;
      vs[rr][d] = ok ? to_f(vb[kt * c_st + d]) : 0.f;
    }
    __syncthreads();
    if (!row_ok) continue;
    bool blk_ok = true;
    if (rowk) {  // masked forecast mode: per-row membership (sparse.py:243-247)
      blk_ok = (j == 0) || (j == bq);
      for (int e = 0; e < kk && !blk_ok; ++e) {
        int64_t jj = rowk[e];
        jj = jj < 0 ? 0 : (jj > nbk - 1 ? nbk - 1 : jj);
        blk_ok = (jj == j);
      }
    }
    if (!blk_ok) continue;
    const int nk = static_cast<int>(T_ - k0 < bs ? T_ - k0 : bs);
    // online softmax over chunks of 16 keys (keeps the unrolled body small)
    for (int c0 = 0; c0 < kQTile; c0 += kKeyChunk) {
      float s[kKeyChunk];
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kKeyChunk; ++c) {
        float a = 0.f;
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) a = fmaf(qr[d], ks[c0 + c][d], a);
        const bool ok = c0 + c < nk && (!causal || k0 + c0 + c <= t);
        s[c] = ok ? a : -INFINITY;
        mt = fmaxf(mt, s[c]);
      }
      const float mn = fmaxf(m, mt);
      if (mn == -INFINITY) continue;
      const float alpha = exp2f(m - mn);
      l *= alpha;
#pragma unroll
      for (int d = 0; d < kHeadDim; ++d) acc[d] *= alpha;
#pragma unroll
      for (int c = 0; c < kKeyChunk; ++c) {
        const float p = s[c] == -INFINITY ? 0.f : exp2f(s[c] - mn);
        l += p;
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) acc[d] = fmaf(p, vs[c0 + c][d], acc[d]);
      }
      m = mn;
    }
  }
  if (!row_ok) return;
  T *op = out + b * o_sb + t * o_st + static_cast<int64_t>(hq) * o_sh;
  const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
  for (int d = 0; d < kHeadDim; ++d) op[d] = from_f<T>(acc[d] * inv);
}

template <typename T>
int launch_prefill_simt(int G, dim3 grid, cudaStream_t s, const void *q, int64_t q_sb, int64_t q_st,
                        int64_t q_sh, const void *k, const void *v, int64_t c_sb, int64_t c_sh, int64_t c_st,
                        int64_t T_, int Hkv, const int32_t *lists, const int32_t *counts, int lcap,
                        const int64_t *topk, int kk, int bs, int causal, float sl2, void *out, int64_t o_sb,
                        int64_t o_st, int64_t o_sh) {
  const T *qq = static_cast<const T *>(q);
  const T *kp = static_cast<const T *>(k);
  const T *vp = static_cast<const T *>(v);
  T *op = static_cast<T *>(out);
  switch (G) {
    case 1:
      prefill_simt_kernel<T, 1><<<grid, 64, 0, s>>>(qq, q_sb, q_st, q_sh, kp, vp, c_sb, c_sh, c_st, T_, Hkv, lists,
                                                   counts, lcap, topk, kk, bs, causal, sl2, op, o_sb, o_st, o_sh);
      break;
    case 2:
      prefill_simt_kernel<T, 2><<<grid, 128, 0, s>>>(qq, q_sb, q_st, q_sh, kp, vp, c_sb, c_sh, c_st, T_, Hkv, lists,
                                                    counts, lcap, topk, kk, bs, causal, sl2, op, o_sb, o_st, o_sh);
      break;
    case 3:
      prefill_simt_kernel<T, 3><<<grid, 192, 0, s>>>(qq, q_sb, q_st, q_sh, kp, vp, c_sb, c_sh, c_st, T_, Hkv, lists,
                                                    counts, lcap, topk, kk, bs, causal, sl2, op, o_sb, o_st, o_sh);
      break;
    case 4:
      prefill_simt_kernel<T, 4><<<grid, 256, 0, s>>>(qq, q_sb, q_st, q_sh, kp, vp, c_sb, c_sh, c_st, T_, Hkv, lists,
                                                    counts, lcap, topk, kk, bs, causal, sl2, op, o_sb, o_st, o_sh);
      break;
    default:
      return SD_ERR_UNSUPPORTED;
  }
  return check_launch();
}

}  // namespace sd

extern "C" int sd_prefill_lists(int mode, int causal, int64_t B, int64_t H, int64_t T, int block_size, int top_k,
                                const int64_t *topk, int kk, int32_t *lists, int32_t *counts, int lcap,
                                void *stream) {
  if (!lists || !counts || B <= 0 || H <= 0 || T <= 0 || top_k <= 0 || lcap <= 0) return SD_ERR_INVALID;
  if (mode < sd::kListDense || mode > sd::kListChunkedStatic) return SD_ERR_INVALID;
  const bool rows = mode == sd::kListMaskedForecast || mode == sd::kListChunkedForecast;
  if (rows && (!topk || kk <= 0)) return SD_ERR_INVALID;
  if (block_size != sd::kQTile) return SD_ERR_UNSUPPORTED;
  if (mode == sd::kListChunkedForecast && top_k > 64) return SD_ERR_UNSUPPORTED;  // the cut keeps <= 64 voted blocks
  const int64_t nb = (T + block_size - 1) / block_size;
  if (nb > 65535 || B > 65535 || H > 65535) return SD_ERR_UNSUPPORTED;
  const size_t smem = sizeof(int) * nb;
  if (sd::set_max_smem(sd::prefill_lists_kernel, smem) != SD_OK) return SD_ERR_CUDA;
  dim3 grid(static_cast<unsigned>(nb), static_cast<unsigned>(H), static_cast<unsigned>(B));
  // 64 threads per list: most of a list's time is one warp's union / cut, so
  // small CTAs let up to 32 lists per SM overlap those serial phases
  sd::prefill_lists_kernel<<<grid, 64, smem, static_cast<cudaStream_t>(stream)>>>(
      mode, causal, T, block_size, top_k, (int)H, topk, kk, lcap, lists, counts);
  return sd::check_launch();
}

extern "C" int sd_prefill_attention(const void *q, int dtype, int64_t B, int64_t T, int64_t Hq, int64_t Hkv,
                                    int64_t D, int64_t q_sb, int64_t q_st, int64_t q_sh, const void *k,
                                    const void *v, int64_t c_sb, int64_t c_sh, int64_t c_st,
                                    const int32_t *lists, const int32_t *counts, int lcap, const int64_t *topk,
                                    int kk, int block_size, int causal, float scale, void *out, int64_t o_sb,
                                    int64_t o_st, int64_t o_sh, void *stream) {
  if (!q || !k || !v || !lists || !counts || !out || B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv ||
      lcap <= 0)
    return SD_ERR_INVALID;
  if (D != sd::kHeadDim || block_size != sd::kQTile) return SD_ERR_UNSUPPORTED;
  if (topk && kk <= 0) return SD_ERR_INVALID;
  const int64_t nqt = (T + sd::kQTile - 1) / sd::kQTile;
  if (nqt > 0x7fffffff || Hkv > 65535 || B > 65535) return SD_ERR_UNSUPPORTED;
  dim3 grid(static_cast<unsigned>(nqt), static_cast<unsigned>(Hkv), static_cast<unsigned>(B));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float sl2 = scale * sd::kLog2eF;
  const int G = static_cast<int>(Hq / Hkv);
  // 16-bit inputs run on the tensor cores; fp32 (exact parity) and shapes the
  // tensor-core kernel does not take run on CUDA cores
  const int rt = sd::launch_prefill_tc(dtype, G, grid, s, q, q_sb, q_st, q_sh, k, v, c_sb, c_sh, c_st, T, (int)Hkv,
                                       B, lists, counts, lcap, topk, kk, causal, sl2, out, o_sb, o_st, o_sh);
  if (rt != SD_ERR_UNSUPPORTED) return rt;
  SD_DISPATCH_DTYPE(dtype, E,
                    return sd::launch_prefill_simt<E>(G, grid, s, q, q_sb, q_st, q_sh, k, v, c_sb, c_sh, c_st, T,
                                                      (int)Hkv, lists, counts, lcap, topk, kk, block_size, causal,
                                                      sl2, out, o_sb, o_st, o_sh));
  return SD_OK;
}
