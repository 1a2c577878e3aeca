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

// Writes T new tokens of K and V into the head-major cache.
template <typename T>
__global__ void kv_copy_kernel(const T *__restrict__ xk, const T *__restrict__ xv, int H, int D, int64_t sb,
                               int64_t st, int64_t sh, T *__restrict__ kc, T *__restrict__ vc, int64_t Tcap,
                               int64_t start) {
  const int64_t t = blockIdx.x, b = blockIdx.y;
  for (int e = threadIdx.x; e < H * D; e += blockDim.x) {
    const int h = e / D, d = e - h * D;
    const int64_t src = b * sb + t * st + h * sh + d;
    const int64_t dst = ((b * H + h) * Tcap + start + t) * D + d;
    kc[dst] = xk[src];
    vc[dst] = xv[src];
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
  SD_DISPATCH_DTYPE(dtype, E,
                    sd::compress_blocks_kernel<E><<<grid, threads, 0, s>>>(
                        static_cast<const E *>(k), T, (int)H, (int)D, sb, st, sh, block_size, reps, NB));
  return sd::check_launch();
}

extern "C" int sd_kv_append(const void *xk, const void *xv, int dtype, int64_t B, int64_t T, int64_t H,
                            int64_t D, int64_t sb, int64_t st, int64_t sh, void *k_cache, void *v_cache,
                            float *proto_sum, int64_t Tcap, int64_t NBcap, int64_t start, int block_size,
                            void *stream) {
  if (!xk || !xv || !k_cache || !v_cache || !proto_sum) return SD_ERR_INVALID;
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0 || block_size <= 0 || start < 0) return SD_ERR_INVALID;
  if (start + T > Tcap || (start + T + block_size - 1) / block_size > NBcap) return SD_ERR_INVALID;
  if (H * D > (1 << 16) || B > 65535 || T > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = static_cast<int>(H * D < 1024 ? ((H * D + 31) / 32) * 32 : 1024);
  const int64_t j0 = start / block_size, j1 = (start + T - 1) / block_size;
  const int dthreads = static_cast<int>(D < 1024 ? ((D + 31) / 32) * 32 : 1024);
  SD_DISPATCH_DTYPE(dtype, E, {
    sd::kv_copy_kernel<E><<<dim3((unsigned)T, (unsigned)B), threads, 0, s>>>(
        static_cast<const E *>(xk), static_cast<const E *>(xv), (int)H, (int)D, sb, st, sh,
        static_cast<E *>(k_cache), static_cast<E *>(v_cache), Tcap, start);
    sd::block_sums_kernel<E><<<dim3((unsigned)(j1 - j0 + 1), (unsigned)(B * H)), dthreads, 0, s>>>(
        static_cast<const E *>(k_cache), (int)H, (int)D, Tcap, NBcap, j0, start + T, block_size, proto_sum);
  });
  return sd::check_launch();
}
