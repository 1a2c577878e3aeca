// K2/K3: forecast block selector (model/forecast.py:89-130), row top-k, and
// decode selected-set assembly (model/attention/sparse.py:108-154).
#include "sd_select_core.cuh"

namespace sd {

// sd_select_tc.cu: the tensor-core many-row selector (bf16 forecast, D = 64,
// k <= 8, no score tensor); SD_ERR_UNSUPPORTED where it does not apply.
int launch_select_rows_tc(const void *forecast, int f_dtype, int64_t B, int64_t Tq, int64_t H, int64_t D, int64_t f_sb,
                          int64_t f_st, int64_t f_sh, const float *reps, int64_t NB, int64_t r_sb, int64_t r_sn,
                          int64_t r_sh, int k, int block_size, int causal, int64_t q_offset, int64_t *topk_idx,
                          int32_t *err, cudaStream_t s);

constexpr int kSelThreads = 256;
constexpr int kChunk = 64;  // prototypes staged per step

// One CTA scores RT query rows of one (b, h) against all NB prototypes and
// takes each row's top-k.  Prototype chunks are staged in shared memory with a
// padded row pitch (D+1) so the 32 lanes of a warp, which read 32 different
// prototypes at the same feature, hit 32 different banks.
template <typename T>
__global__ void __launch_bounds__(kSelThreads)
    select_blocks_kernel(const T *__restrict__ fc, int64_t Tq, int H, int D, int64_t f_sb, int64_t f_st,
                         int64_t f_sh, const float *__restrict__ reps, int64_t NB, int64_t r_sb, int64_t r_sn,
                         int64_t r_sh, int k, int bs, int causal, int64_t q_offset, int RT, float scale,
                         float *__restrict__ scores_out, int64_t *__restrict__ idx_out) {
  extern __shared__ float smem[];
  const int b = blockIdx.z, h = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * RT;
  const int nrows = static_cast<int>(Tq - row0 < RT ? Tq - row0 : RT);
  float *f_s = smem;                              // [RT][D]
  float *r_s = f_s + RT * D;                      // [kChunk][D+1]
  float *sc_s = r_s + kChunk * (D + 1);           // [RT][NB]
  int *tk_s = reinterpret_cast<int *>(sc_s + static_cast<int64_t>(RT) * NB);  // [8 warps][k]

  for (int e = threadIdx.x; e < RT * D; e += blockDim.x) {
    const int r = e / D, d = e - r * D;
    f_s[e] = r < nrows ? to_f(fc[b * f_sb + (row0 + r) * f_st + h * f_sh + d]) : 0.f;
  }
  // causal: row t sees blocks j <= (t + q_offset) / bs; beyond the tile's
  // largest visible block nothing needs scoring
  int64_t jmax = NB;
  if (causal) {
    const int64_t last = (row0 + nrows - 1 + q_offset) / bs + 1;
    jmax = last < NB ? (last > 0 ? last : 0) : NB;
  }
  const int jcol = threadIdx.x & (kChunk - 1);
  const int rgrp = threadIdx.x / kChunk;          // 0..3
  const int rstep = kSelThreads / kChunk;         // 4
  for (int64_t j0 = 0; j0 < NB; j0 += kChunk) {
    __syncthreads();
    if (j0 < jmax) {
      for (int e = threadIdx.x; e < kChunk * D; e += blockDim.x) {
        const int jj = e / D, d = e - jj * D;
        r_s[jj * (D + 1) + d] = (j0 + jj < NB) ? reps[b * r_sb + (j0 + jj) * r_sn + h * r_sh + d] : 0.f;
      }
    }
    __syncthreads();
    const int64_t j = j0 + jcol;
    if (j >= NB) continue;
    for (int r = rgrp; r < RT; r += rstep) {
      float v;
      const int64_t t = row0 + r + q_offset;
      if (causal && (j > t / bs || t < 0)) {
        v = -INFINITY;
      } else if (j0 >= jmax) {
        v = -INFINITY;
      } else {
        float acc = 0.f;
        const float *fr = f_s + r * D;
        const float *rr = r_s + jcol * (D + 1);
        for (int d = 0; d < D; ++d) acc = fmaf(fr[d], rr[d], acc);
        v = acc * scale;
      }
      sc_s[static_cast<int64_t>(r) * NB + j] = v;
    }
  }
  __syncthreads();
  if (scores_out) {
    for (int r = 0; r < nrows; ++r) {
      float *dst = scores_out + ((static_cast<int64_t>(b) * H + h) * Tq + row0 + r) * NB;
      for (int64_t j = threadIdx.x; j < NB; j += blockDim.x) dst[j] = sc_s[static_cast<int64_t>(r) * NB + j];
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int *tk = tk_s + warp * k;
  for (int r = warp; r < nrows; r += kSelThreads / 32) {
    const float *row = sc_s + static_cast<int64_t>(r) * NB;
    warp_topk([&](int j) { return row[j]; }, static_cast<int>(NB), k, tk, nullptr);
    __syncwarp();
    int64_t *dst = idx_out + ((static_cast<int64_t>(b) * H + h) * Tq + row0 + r) * k;
    for (int i = lane; i < k; i += 32) dst[i] = tk[i];
    __syncwarp();
  }
}

// Many-row selector for D = 64 and top-k <= 8 (prefill): a CTA scores 64 rows
// of one (b, h) against the prototypes in chunks of 128 blocks.  Thread
// (ty, tx) accumulates a 4-row x 8-block register tile (rows 4ty.., blocks
// tx + 16c) from float4 shared-memory loads, summing d = 0..63 in order (the
// same order as select_blocks_kernel); each warp then folds its 8 rows'
// chunk scores into per-row running top-8 lists with the register tournament
// (sort_groups / merge_regs / merge_lanes).
constexpr int kTileRows = 64;
constexpr int kTileBlocks = 128;
constexpr int kPitch = 68;  // floats per staged row (16-byte aligned, conflict-free float4 reads)

template <typename T>
__global__ void __launch_bounds__(256)
    select_rows_tiled_kernel(const T *__restrict__ fc, int64_t Tq, int H, int64_t f_sb, int64_t f_st,
                             int64_t f_sh, const float *__restrict__ reps, int64_t NB, int64_t r_sb, int64_t r_sn,
                             int64_t r_sh, int k, int bs, int causal, int64_t q_offset, float scale,
                             float *__restrict__ scores_out, int64_t *__restrict__ idx_out) {
  extern __shared__ __align__(16) float tsm[];
  float *f_s = tsm;                             // [64][kPitch]
  float *r_s = f_s + kTileRows * kPitch;        // [128][kPitch]
  float *s_s = r_s + kTileBlocks * kPitch;      // [64][128 + 1]
  const int b = blockIdx.z, h = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kTileRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ty = tid >> 4, tx = tid & 15;
  for (int e = tid; e < kTileRows * 64; e += 256) {
    const int r = e >> 6, d = e & 63;
    f_s[r * kPitch + d] = row0 + r < Tq ? to_f(fc[b * f_sb + (row0 + r) * f_st + h * f_sh + d]) : 0.f;
  }
  int64_t jmax = NB;  // blocks no row of the tile can see are not scored
  if (causal) {
    const int64_t last_row = (Tq - row0 < kTileRows ? Tq - 1 : row0 + kTileRows - 1);
    const int64_t last = (last_row + q_offset) / bs + 1;
    jmax = last < NB ? (last > 0 ? last : 0) : NB;
  }
  float rv[8];
  int ri[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    rv[q] = -INFINITY;
    ri[q] = kNoBlock;
  }
  for (int64_t j0 = 0; j0 < NB; j0 += kTileBlocks) {
    __syncthreads();
    const bool scored = j0 < jmax;
    if (scored) {
      for (int e = tid; e < kTileBlocks * 16; e += 256) {
        const int jj = e >> 4, c = e & 15;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j0 + jj < NB) v = *reinterpret_cast<const float4 *>(reps + b * r_sb + (j0 + jj) * r_sn + h * r_sh + 4 * c);
        *reinterpret_cast<float4 *>(r_s + jj * kPitch + 4 * c) = v;
      }
    }
    __syncthreads();
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[i][c] = 0.f;
    if (scored) {
#pragma unroll 4
      for (int d4 = 0; d4 < 16; ++d4) {
        float4 fq[4], rr[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) fq[i] = *reinterpret_cast<const float4 *>(f_s + (4 * ty + i) * kPitch + 4 * d4);
#pragma unroll
        for (int c = 0; c < 8; ++c) rr[c] = *reinterpret_cast<const float4 *>(r_s + (tx + 16 * c) * kPitch + 4 * d4);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            acc[i][c] = fmaf(fq[i].x, rr[c].x, acc[i][c]);
            acc[i][c] = fmaf(fq[i].y, rr[c].y, acc[i][c]);
            acc[i][c] = fmaf(fq[i].z, rr[c].z, acc[i][c]);
            acc[i][c] = fmaf(fq[i].w, rr[c].w, acc[i][c]);
          }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 4 * ty + i;
      const int64_t t = row0 + r + q_offset;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int64_t j = j0 + tx + 16 * c;
        float v = acc[i][c] * scale;
        if (!scored || (causal && (t < 0 || j > t / bs))) v = -INFINITY;
        s_s[r * (kTileBlocks + 1) + tx + 16 * c] = v;
      }
    }
    __syncthreads();
    if (scores_out) {
      for (int e = tid; e < kTileRows * kTileBlocks; e += 256) {
        const int r = e / kTileBlocks, jj = e - r * kTileBlocks;
        if (row0 + r < Tq && j0 + jj < NB)
          scores_out[((static_cast<int64_t>(b) * H + h) * Tq + row0 + r) * NB + j0 + jj] =
              s_s[r * (kTileBlocks + 1) + jj];
      }
    }
    // fold the chunk into the running top-8 of each of this warp's 8 rows
    // (lanes 0..7 hold a row's list, best first).  The first chunk runs the
    // register tournament; after it a block can only enter a row's list if it
    // beats the row's 8th entry, which few do, so later chunks filter against
    // that threshold with a ballot and insert the survivors one at a time.
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int r = warp * 8 + q;
      float cv[4];
      int ci[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int jj = lane + 32 * u;
        const int64_t j = j0 + jj;
        const float v = s_s[r * (kTileBlocks + 1) + jj];
        const bool ok = j < NB && v == v;
        cv[u] = ok ? v : -INFINITY;
        ci[u] = ok ? static_cast<int>(j) : kNoBlock;
      }
      if (j0 == 0) {
        fold_first8<4>(rv[q], ri[q], cv, ci);
      } else {
        fold_insert8<4>(rv[q], ri[q], cv, ci);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int64_t row = row0 + warp * 8 + q;
    if (row < Tq && lane < k)
      idx_out[((static_cast<int64_t>(b) * H + h) * Tq + row) * k + lane] = ri[q] == kNoBlock ? -1 : ri[q];
  }
}

// One warp per row.
__global__ void topk_rows_kernel(const float *__restrict__ s, int64_t rows, int64_t n, int64_t ld, int k,
                                 int64_t *__restrict__ idx, float *__restrict__ vals) {
  __shared__ int ti[8][64];
  __shared__ float tv[8][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (r >= rows) return;
  const float *row = s + r * ld;
  warp_topk([&](int j) { return row[j]; }, static_cast<int>(n), k, ti[warp], tv[warp]);
  __syncwarp();
  for (int i = lane; i < k; i += 32) {
    idx[r * k + i] = ti[warp][i];
    if (vals) vals[r * k + i] = tv[warp][i];
  }
}

// One CTA per (b, h): scores the forecast against the prototypes, then builds
// the ascending selected list.
template <typename T>
__global__ void decode_select_kernel(const T *__restrict__ fc, int64_t f_sb, int64_t f_sh,
                                     const float *__restrict__ reps, int64_t r_sb, int64_t r_sn, int64_t r_sh,
                                     int H, int D, int64_t L, int bs, int k, int rule, float scale,
                                     int32_t *__restrict__ sel, int32_t *__restrict__ cnt, int ms_cap) {
  extern __shared__ float smem[];
  const int b = blockIdx.x / H, h = blockIdx.x - (blockIdx.x / H) * H;
  const int nb = static_cast<int>((L + bs - 1) / bs);
  const int curr = static_cast<int>((L - 1) / bs);
  const int ms = nb < k + 2 ? nb : k + 2;
  float *f_s = smem;                  // [D]
  float *sc = f_s + D;                // [nb]
  int *list = reinterpret_cast<int *>(sc + nb);  // [max(nb, k + 2)]
  int *tk = list + (nb > k + 2 ? nb : k + 2);    // [k]
  __shared__ int count;
  const bool use_f = fc != nullptr;
  int n_scored = 0;
  if (use_f && nb > ms) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) f_s[d] = to_f(fc[b * f_sb + h * f_sh + d]);
    __syncthreads();
    n_scored = rule == SD_RULE_REFERENCE ? 1 : curr + 1;
    score_blocks(reps + b * r_sb + h * r_sh, r_sn, D, f_s, n_scored, scale, sc);
    __syncthreads();
  }
  build_decode_list(use_f, sc, n_scored, nb, curr, k, ms, tk, list, &count);
  int32_t *dst = sel + static_cast<int64_t>(blockIdx.x) * ms_cap;
  for (int i = threadIdx.x; i < ms_cap; i += blockDim.x) dst[i] = i < count ? list[i] : -1;
  if (threadIdx.x == 0) cnt[blockIdx.x] = count;
}

}  // namespace sd

extern "C" int sd_select_blocks(const void *forecast, int f_dtype, int64_t B, int64_t Tq, int64_t H,
                                int64_t D, int64_t f_sb, int64_t f_st, int64_t f_sh, const float *reps,
                                int64_t NB, int64_t r_sb, int64_t r_sn, int64_t r_sh, int top_k,
                                int block_size, int causal, int64_t q_offset, float *scores,
                                int64_t *topk_idx, void *stream) {
  if (!forecast || !reps || !topk_idx || B <= 0 || Tq <= 0 || H <= 0 || NB <= 0 || top_k <= 0 ||
      block_size <= 0)
    return SD_ERR_INVALID;
  if (D < 1 || D > 256) return SD_ERR_UNSUPPORTED;
  const int k = static_cast<int>(top_k < NB ? top_k : NB);
  if (k > 64 || NB > 24576 || B > 65535 || H > 65535) return SD_ERR_UNSUPPORTED;
  if (!scores) {
    const int r = sd::launch_select_rows_tc(forecast, f_dtype, B, Tq, H, D, f_sb, f_st, f_sh, reps, NB, r_sb, r_sn,
                                            r_sh, k, block_size, causal, q_offset, topk_idx, nullptr,
                                            static_cast<cudaStream_t>(stream));
    if (r != SD_ERR_UNSUPPORTED) return r;
  }
  if (D == 64 && k <= 8 && Tq >= sd::kTileRows && (r_sn % 4) == 0 && (r_sb % 4) == 0 && (r_sh % 4) == 0 &&
      sd::aligned16(reps)) {
    // many rows: register-tiled scoring and register top-k
    const size_t tsmem = sizeof(float) * (sd::kTileRows * sd::kPitch + sd::kTileBlocks * sd::kPitch +
                                          sd::kTileRows * (sd::kTileBlocks + 1));
    const int64_t tiles = (Tq + sd::kTileRows - 1) / sd::kTileRows;
    if (tiles > 0x7fffffff) return SD_ERR_UNSUPPORTED;
    dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(H), static_cast<unsigned>(B));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float scale = sd::inv_sqrt(D);
    SD_DISPATCH_DTYPE(f_dtype, E, {
      auto kern = sd::select_rows_tiled_kernel<E>;
      if (sd::set_max_smem(kern, tsmem) != SD_OK) return SD_ERR_CUDA;
      kern<<<grid, 256, tsmem, s>>>(static_cast<const E *>(forecast), Tq, (int)H, f_sb, f_st, f_sh, reps, NB, r_sb,
                                    r_sn, r_sh, k, block_size, causal, q_offset, scale, scores, topk_idx);
    });
    return sd::check_launch();
  }
  int RT = static_cast<int>(24576 / NB);
  RT = RT > 32 ? 32 : (RT < 1 ? 1 : RT);
  if (RT > Tq) RT = static_cast<int>(Tq);
  const size_t smem = sizeof(float) * (static_cast<size_t>(RT) * D + sd::kChunk * (D + 1) +
                                       static_cast<size_t>(RT) * NB) +
                      sizeof(int) * 8 * k;
  const int64_t tiles = (Tq + RT - 1) / RT;
  if (tiles > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(H), static_cast<unsigned>(B));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float scale = sd::inv_sqrt(D);
  SD_DISPATCH_DTYPE(f_dtype, E, {
    auto kern = sd::select_blocks_kernel<E>;
    if (sd::set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
    kern<<<grid, sd::kSelThreads, smem, s>>>(static_cast<const E *>(forecast), Tq, (int)H, (int)D, f_sb, f_st,
                                             f_sh, reps, NB, r_sb, r_sn, r_sh, k, block_size, causal, q_offset,
                                             RT, scale, scores, topk_idx);
  });
  return sd::check_launch();
}

extern "C" int sd_topk_rows(const float *scores, int64_t rows, int64_t n, int64_t ld, int k, int64_t *idx,
                            float *vals, void *stream) {
  if (!scores || !idx || rows <= 0 || n <= 0 || k <= 0 || k > n || ld < n) return SD_ERR_INVALID;
  if (k > 64 || n > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  sd::topk_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      scores, rows, n, ld, k, idx, vals);
  return sd::check_launch();
}

extern "C" int sd_decode_select(const void *forecast, int f_dtype, int64_t f_sb, int64_t f_sh,
                                const float *reps, int64_t r_sb, int64_t r_sn, int64_t r_sh, int64_t B,
                                int64_t H, int64_t D, int64_t seq_len_k, int block_size, int top_k, int rule,
                                int32_t *sel, int32_t *cnt, int ms_cap, void *stream) {
  if (!sel || !cnt || B <= 0 || H <= 0 || D <= 0 || seq_len_k <= 0 || block_size <= 0 || top_k <= 0)
    return SD_ERR_INVALID;
  if (rule != SD_RULE_REFERENCE && rule != SD_RULE_ABSOLUTE) return SD_ERR_INVALID;
  const int64_t nb = (seq_len_k + block_size - 1) / block_size;
  const int64_t ms = nb < top_k + 2 ? nb : top_k + 2;
  if (ms_cap < ms) return SD_ERR_INVALID;
  if (forecast && !reps) return SD_ERR_INVALID;
  if (D % 4 != 0 || D > 256 || top_k > 64 || nb > 32768 || B * H > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  if (forecast && (!sd::aligned16(reps) || (r_sb % 4) || (r_sn % 4) || (r_sh % 4))) return SD_ERR_ALIGN;
  const int64_t lst = nb > top_k + 2 ? nb : top_k + 2;
  const size_t smem = sizeof(float) * (D + nb) + sizeof(int) * (lst + top_k);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fdt = forecast ? f_dtype : SD_DTYPE_F32;
  SD_DISPATCH_DTYPE(fdt, E, {
    auto kern = sd::decode_select_kernel<E>;
    if (sd::set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
    kern<<<static_cast<unsigned>(B * H), 128, smem, s>>>(static_cast<const E *>(forecast), f_sb, f_sh, reps,
                                                         r_sb, r_sn, r_sh, (int)H, (int)D, seq_len_k,
                                                         block_size, top_k, rule, sd::inv_sqrt(D), sel, cnt,
                                                         ms_cap);
  });
  return sd::check_launch();
}

namespace sd {

// One CTA per (b, h): top-k of every cached block except the one the next
// token lands in, from the running sums (sum / bs), for the next decode step.
template <typename F>
__global__ void decode_candidates_kernel(const F *__restrict__ fc, int64_t f_sb, const float *proto_sum, int H,
                                         int64_t NBcap, const int32_t *__restrict__ cur_len, int bs, int k,
                                         int rule, float sel_scale, int32_t *__restrict__ cand_idx,
                                         float *__restrict__ cand_val) {
  extern __shared__ float smem[];
  constexpr int D = 64;
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int64_t pos = *cur_len;
  float *f_s = smem;      // [D]
  float *sc = f_s + D;    // [NBcap]
  __shared__ int tk[64];
  int32_t *oi = cand_idx + static_cast<int64_t>(bh) * k;
  float *ov = cand_val + static_cast<int64_t>(bh) * k;
  const int64_t nb64 = pos / bs + 1;
  const int ms = nb64 < k + 2 ? static_cast<int>(nb64) : k + 2;
  if (pos < 0 || nb64 > NBcap || nb64 <= ms) {  // dense step (or nothing cached): no candidates needed
    for (int r = threadIdx.x; r < k; r += blockDim.x) {
      oi[r] = -1;
      ov[r] = -INFINITY;
    }
    return;
  }
  const int nb = static_cast<int>(nb64), curr = nb - 1;
  const int n_scored = rule == SD_RULE_REFERENCE ? 1 : curr;  // the current block is left out
  const int nsc = n_scored < curr ? n_scored : curr;
  const F *fr = fc + b * f_sb + h * D;
  if (k <= 32) {  // scoring and top-k in registers
    const int l16 = threadIdx.x & 15;
    const float4 fv = make_float4(to_f(fr[4 * l16]), to_f(fr[4 * l16 + 1]), to_f(fr[4 * l16 + 2]),
                                  to_f(fr[4 * l16 + 3]));
    cta_score_topk(proto_sum + static_cast<int64_t>(bh) * NBcap * D, D, fv, curr, nsc, -1, sel_scale, k, oi, ov);
    return;
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) f_s[d] = to_f(fr[d]);
  __syncthreads();
  score_blocks(proto_sum + static_cast<int64_t>(bh) * NBcap * D, D, D, f_s, nsc, sel_scale, sc);
  __syncthreads();
  auto val = [&](int j) { return j == curr ? __int_as_float(0x7fc00000) : (j < nsc ? sc[j] : -INFINITY); };
  cta_topk(val, nb, k, tk);
  for (int r = threadIdx.x; r < k; r += blockDim.x) {
    const int j = tk[r];
    oi[r] = j;
    ov[r] = j >= 0 ? val(j) : -INFINITY;
  }
}

}  // namespace sd

extern "C" int sd_decode_candidates(const void *forecast, int f_dtype, int64_t f_sb, const float *proto_sum,
                                    int64_t B, int64_t Hkv, int64_t D, int64_t NBcap, const int32_t *cur_len,
                                    int block_size, int top_k, int rule, float scale, int32_t *cand_idx,
                                    float *cand_val, void *stream) {
  if (!forecast || !proto_sum || !cur_len || !cand_idx || !cand_val || B <= 0 || Hkv <= 0 || NBcap <= 0 ||
      block_size <= 0 || top_k <= 0)
    return SD_ERR_INVALID;
  if (rule != SD_RULE_REFERENCE && rule != SD_RULE_ABSOLUTE) return SD_ERR_INVALID;
  if (D != 64 || top_k > 64 || NBcap > 32768 || B * Hkv > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  if (!sd::aligned16(proto_sum)) return SD_ERR_ALIGN;
  const size_t smem = top_k <= 32 ? 0 : sizeof(float) * (D + NBcap);  // register path needs none
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float sel_scale = scale / static_cast<float>(block_size);
  SD_DISPATCH_DTYPE(f_dtype, E, {
    auto kern = sd::decode_candidates_kernel<E>;
    if (sd::set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
    kern<<<static_cast<unsigned>(B * Hkv), 256, smem, s>>>(static_cast<const E *>(forecast), f_sb, proto_sum,
                                                           (int)Hkv, NBcap, cur_len, block_size, top_k, rule,
                                                           sel_scale, cand_idx, cand_val);
  });
  return sd::check_launch();
}
