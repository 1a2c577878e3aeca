// K1: block compressor (KVBlockCompressor.forward, model/forecast.py:57-78) and
// the block-major KV-cache append with the compressor's block sums fused in.
#include "sd_common.cuh"

namespace sd {

// One CTA per (block j, sequence b); threads stride over the H*D features of a
// token, so consecutive threads read consecutive elements of a token row.
template <typename T>
__global__ void compress_blocks_kernel(const T *__restrict__ k, int64_t T_, int H, int D, int64_t sb,
                                       int64_t st, int64_t sh, int bs, float *__restrict__ reps,
                                       int64_t NB) {
  const int64_t j = blockIdx.x, b = blockIdx.y;
  const int64_t t0 = j * bs;
  const int64_t t1 = t0 + bs < T_ ? t0 + bs : T_;
  const float inv = 1.0f / static_cast<float>(bs);
  for (int e = threadIdx.x; e < H * D; e += blockDim.x) {
    const int h = e / D, d = e - h * D;
    const T *p = k + b * sb + h * sh + d;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int64_t t = t0;
    for (; t + 4 <= t1; t += 4) {
      s0 += to_f(p[t * st]);
      s1 += to_f(p[(t + 1) * st]);
      s2 += to_f(p[(t + 2) * st]);
      s3 += to_f(p[(t + 3) * st]);
    }
    for (; t < t1; ++t) s0 += to_f(p[t * st]);
    // zero padding contributes nothing; divide by the full block size
    const float s = (s0 + s1) + (s2 + s3);
    reps[((b * NB + j) * H + h) * D + d] = (bs & (bs - 1)) == 0 ? s * inv : s / static_cast<float>(bs);
  }
}

// Same result through 16-byte loads, for rows whose H*D values sit in 16-byte
// aligned chunks (kV elements each).  One CTA per (block j, sequence b);
// thread (g, c) sums chunk column c of rows g, g + kGroups, ... of the block,
// all of its loads issued before any is used, then the kGroups partial sums
// of every column are added in shared memory in a fixed order.
template <typename T, int kGroups>
__global__ void __launch_bounds__(256) compress_blocks_vec_kernel(const T *__restrict__ k, int64_t T_, int H, int D,
                                                                  int64_t sb, int64_t st, int64_t sh, int bs,
                                                                  float *__restrict__ reps, int64_t NB) {
  constexpr int kV = 16 / static_cast<int>(sizeof(T));
  constexpr int kRowsPer = 64 / kGroups;  // block_size 64
  __shared__ float part[kGroups][256 / kGroups * kV];
  const int64_t j = blockIdx.x, b = blockIdx.y;
  const int cols = H * D / kV;             // chunk columns of a token row
  const int c = threadIdx.x % cols, g = threadIdx.x / cols;
  const int h = c * kV / D, d0 = c * kV - h * D;
  const int64_t t0 = j * 64;
  float acc[kV];
#pragma unroll
  for (int i = 0; i < kV; ++i) acc[i] = 0.f;
  if (g < kGroups) {
    const T *p = k + b * sb + h * sh + d0;
    uint4 u[kRowsPer];
#pragma unroll
    for (int r = 0; r < kRowsPer; ++r) {
      const int64_t t = t0 + g + r * kGroups;
      u[r] = t < T_ ? *reinterpret_cast<const uint4 *>(p + t * st) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int r = 0; r < kRowsPer; ++r) {
      const T *e = reinterpret_cast<const T *>(&u[r]);
#pragma unroll
      for (int i = 0; i < kV; ++i) acc[i] += to_f(e[i]);
    }
#pragma unroll
    for (int i = 0; i < kV; ++i) part[g][c * kV + i] = acc[i];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < H * D; e += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kGroups; ++q) s += part[q][e];
    const int hh = e / D, dd = e - hh * D;
    reps[((b * NB + j) * H + hh) * D + dd] = s * (1.0f / 64.0f);
  }
}

// Writes T new tokens of K and V into the head-major cache (any strides).
template <typename T>
__global__ void kv_copy_kernel(const T *__restrict__ xk, const T *__restrict__ xv, int H, int D, int64_t sb,
                               int64_t st, int64_t sh, int64_t vsb, int64_t vst, int64_t vsh, T *__restrict__ kc,
                               T *__restrict__ vc, int64_t Tcap, int64_t start) {
  const int64_t t = blockIdx.x, b = blockIdx.y;
  for (int e = threadIdx.x; e < H * D; e += blockDim.x) {
    const int h = e / D, d = e - h * D;
    const int64_t dst = ((b * H + h) * Tcap + start + t) * D + d;
    kc[dst] = xk[b * sb + t * st + h * sh + d];
    vc[dst] = xv[b * vsb + t * vst + h * vsh + d];
  }
}

// The append in one pass with 16-byte accesses: one CTA per (touched cache
// block j0 + blockIdx.x, sequence), 256 threads = kRowGroups row groups x
// H*D/kv column chunks (kv = 16 / sizeof(T)).  The block's new rows are read
// from xk / xv and written to the cache; its rows below `start` (a block the
// previous append left partial) are read back from the cache.  Each thread
// sums its chunk's K values over its row group's rows (rows rg, rg + RG, ...
// in order) in fp32, and the row groups' partial sums are added in row-group
// order into the block's running sum.
template <typename T, int kRowGroups>
__global__ void __launch_bounds__(256)
    kv_append_vec_kernel(const T *__restrict__ xk, const T *__restrict__ xv, int H, int D, int64_t sb, int64_t st,
                         int64_t sh, int64_t vsb, int64_t vst, int64_t vsh, T *__restrict__ kc, T *__restrict__ vc,
                         int64_t Tcap, int64_t NBcap, int64_t j0, int64_t start, int64_t end, int bs,
                         float *__restrict__ proto_sum) {
  constexpr int kv = 16 / sizeof(T);
  __shared__ float part[kRowGroups][256 / kRowGroups * kv];
  const int C = 256 / kRowGroups;  // column chunks of a token row (H * D / kv)
  const int rg = threadIdx.x / C, c = threadIdx.x - rg * C;
  const int cph = D / kv;  // chunks per head
  const int h = c / cph, d0 = (c - h * cph) * kv;
  const int64_t b = blockIdx.y, j = j0 + blockIdx.x;
  const int64_t t0 = j * bs, t1 = t0 + bs < end ? t0 + bs : end;
  T *kdst = kc + ((b * H + h) * Tcap) * D + d0;
  T *vdst = vc + ((b * H + h) * Tcap) * D + d0;
  float acc[kv];
#pragma unroll
  for (int i = 0; i < kv; ++i) acc[i] = 0.f;
  for (int64_t t = t0 + rg; t < t1; t += kRowGroups) {
    uint4 kw;
    if (t >= start) {
      const int64_t r = t - start;
      kw = *reinterpret_cast<const uint4 *>(xk + b * sb + r * st + h * sh + d0);
      const uint4 vw = *reinterpret_cast<const uint4 *>(xv + b * vsb + r * vst + h * vsh + d0);
      *reinterpret_cast<uint4 *>(kdst + t * D) = kw;
      *reinterpret_cast<uint4 *>(vdst + t * D) = vw;
    } else {
      kw = *reinterpret_cast<const uint4 *>(kdst + t * D);
    }
    const T *kx = reinterpret_cast<const T *>(&kw);
#pragma unroll
    for (int i = 0; i < kv; ++i) acc[i] += to_f(kx[i]);
  }
#pragma unroll
  for (int i = 0; i < kv; ++i) part[rg][c * kv + i] = acc[i];
  __syncthreads();
  for (int e = threadIdx.x; e < C * kv; e += 256) {
    float s = 0.f;
#pragma unroll
    for (int g = 0; g < kRowGroups; ++g) s += part[g][e];
    const int hh = e / D, dd = e - hh * D;
    proto_sum[((b * H + hh) * NBcap + j) * D + dd] = s;
  }
}

// Recomputes the running sums of cache blocks j0 .. j0+gridDim.x-1 from the
// cache rows below `end`.
template <typename T>
__global__ void block_sums_kernel(const T *__restrict__ kc, int H, int D, int64_t Tcap, int64_t NBcap,
                                  int64_t j0, int64_t end, int bs, float *__restrict__ proto_sum) {
  const int64_t j = j0 + blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t t0 = j * bs;
  const int64_t t1 = t0 + bs < end ? t0 + bs : end;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const T *p = kc + (bh * Tcap) * D + d;
    float s = 0.f;
    for (int64_t t = t0; t < t1; ++t) s += to_f(p[t * D]);
    proto_sum[(bh * NBcap + j) * D + d] = s;
  }
}

}  // namespace sd

extern "C" int sd_compress_blocks(const void *k, int dtype, int64_t B, int64_t T, int64_t H, int64_t D,
                                  int64_t sb, int64_t st, int64_t sh, int block_size, float *reps,
                                  void *stream) {
  if (!k || !reps || B <= 0 || T <= 0 || H <= 0 || D <= 0 || block_size <= 0) return SD_ERR_INVALID;
  if (H * D > (1 << 16)) return SD_ERR_UNSUPPORTED;
  const int64_t NB = (T + block_size - 1) / block_size;
  if (NB > 0x7fffffff || B > 65535) return SD_ERR_UNSUPPORTED;
  int threads = static_cast<int>(H * D < 1024 ? ((H * D + 31) / 32) * 32 : 1024);
  dim3 grid(static_cast<unsigned>(NB), static_cast<unsigned>(B));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = sd::dtype_size(dtype);
  const int64_t kv = 16 / es;
  // 16-byte path: block 64, every token row in aligned 16-byte chunks, and
  // the chunk columns of a row (H*D/kv) times 8 row groups fill 256 threads
  if (block_size == 64 && sd::aligned16(k) && D % kv == 0 && sb % kv == 0 && st % kv == 0 && sh % kv == 0 &&
      (H * D / kv) * 8 == 256) {
    SD_DISPATCH_DTYPE(dtype, E,
                      sd::compress_blocks_vec_kernel<E, 8><<<grid, 256, 0, s>>>(
                          static_cast<const E *>(k), T, (int)H, (int)D, sb, st, sh, block_size, reps, NB));
    return sd::check_launch();
  }
  SD_DISPATCH_DTYPE(dtype, E,
                    sd::compress_blocks_kernel<E><<<grid, threads, 0, s>>>(
                        static_cast<const E *>(k), T, (int)H, (int)D, sb, st, sh, block_size, reps, NB));
  return sd::check_launch();
}

extern "C" int sd_kv_append(const void *xk, const void *xv, int dtype, int64_t B, int64_t T, int64_t H,
                            int64_t D, int64_t sb, int64_t st, int64_t sh, int64_t vsb, int64_t vst, int64_t vsh,
                            void *k_cache, void *v_cache, float *proto_sum, int64_t Tcap, int64_t NBcap,
                            int64_t start, int block_size, void *stream) {
  if (!xk || !xv || !k_cache || !v_cache || !proto_sum) return SD_ERR_INVALID;
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0 || block_size <= 0 || start < 0) return SD_ERR_INVALID;
  if (start + T > Tcap || (start + T + block_size - 1) / block_size > NBcap) return SD_ERR_INVALID;
  if (H * D > (1 << 16) || B > 65535 || T > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = static_cast<int>(H * D < 1024 ? ((H * D + 31) / 32) * 32 : 1024);
  const int64_t j0 = start / block_size, j1 = (start + T - 1) / block_size;
  const int dthreads = static_cast<int>(D < 1024 ? ((D + 31) / 32) * 32 : 1024);
  // 16-byte path: aligned rows whose H*D/kv chunks divide 256 threads into
  // 4 or 8 row groups (H*D = 256 at 16 or 32 bits)
  const int es = sd::dtype_size(dtype);
  const int64_t kv = 16 / es;
  const int64_t chunks = H * D / kv;
  if (D % kv == 0 && sb % kv == 0 && st % kv == 0 && sh % kv == 0 && vsb % kv == 0 && vst % kv == 0 &&
      vsh % kv == 0 && sd::aligned16(xk) && sd::aligned16(xv) && sd::aligned16(k_cache) &&
      sd::aligned16(v_cache) && (chunks == 32 || chunks == 64) && j1 - j0 + 1 <= 0x7fffffff) {
    const dim3 grid(static_cast<unsigned>(j1 - j0 + 1), static_cast<unsigned>(B));
    SD_DISPATCH_DTYPE(dtype, E, {
      if (chunks == 32)
        sd::kv_append_vec_kernel<E, 8><<<grid, 256, 0, s>>>(
            static_cast<const E *>(xk), static_cast<const E *>(xv), (int)H, (int)D, sb, st, sh, vsb, vst, vsh,
            static_cast<E *>(k_cache), static_cast<E *>(v_cache), Tcap, NBcap, j0, start, start + T, block_size,
            proto_sum);
      else
        sd::kv_append_vec_kernel<E, 4><<<grid, 256, 0, s>>>(
            static_cast<const E *>(xk), static_cast<const E *>(xv), (int)H, (int)D, sb, st, sh, vsb, vst, vsh,
            static_cast<E *>(k_cache), static_cast<E *>(v_cache), Tcap, NBcap, j0, start, start + T, block_size,
            proto_sum);
    });
    return sd::check_launch();
  }
  SD_DISPATCH_DTYPE(dtype, E, {
    sd::kv_copy_kernel<E><<<dim3((unsigned)T, (unsigned)B), threads, 0, s>>>(
        static_cast<const E *>(xk), static_cast<const E *>(xv), (int)H, (int)D, sb, st, sh, vsb, vst, vsh,
        static_cast<E *>(k_cache), static_cast<E *>(v_cache), Tcap, start);
    sd::block_sums_kernel<E><<<dim3((unsigned)(j1 - j0 + 1), (unsigned)(B * H)), dthreads, 0, s>>>(
        static_cast<const E *>(k_cache), (int)H, (int)D, Tcap, NBcap, j0, start + T, block_size, proto_sum);
  });
  return sd::check_launch();
}
