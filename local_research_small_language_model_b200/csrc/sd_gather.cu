// K4: gather_kv_blocks (model/attention/sparse.py:19-62) - materialises the
// selected K/V blocks contiguously.  The attention kernels of this library do
// not need it (they read blocks in place); it backs the drop-in function of the
// same name.
#include "sd_common.cuh"

namespace sd {

// One CTA per (b, h, selected slot); threads stride over block_size*D elements.
template <typename T>
__global__ void gather_kv_kernel(const T *__restrict__ k, const T *__restrict__ v, int H, int64_t T_, int D,
                                 int64_t sb, int64_t sh, int64_t st, const int64_t *__restrict__ idx, int64_t S,
                                 int bs, T *__restrict__ ko, T *__restrict__ vo) {
  const int64_t slot = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / H, h = bh - (bh / H) * H;
  const int64_t nb = (T_ + bs - 1) / bs;
  const int64_t j = idx[bh * S + slot];
  const bool ok = j >= 0 && j < nb;
  T *kd = ko + (bh * S + slot) * bs * D;
  T *vd = vo + (bh * S + slot) * bs * D;
  for (int64_t e = threadIdx.x; e < static_cast<int64_t>(bs) * D; e += blockDim.x) {
    const int64_t r = e / D, d = e - r * D;
    const int64_t t = j * bs + r;
    if (ok && t < T_) {
      const int64_t src = b * sb + h * sh + t * st + d;
      kd[e] = k[src];
      vd[e] = v[src];
    } else {
      kd[e] = from_f<T>(0.f);
      vd[e] = from_f<T>(0.f);
    }
  }
}

}  // namespace sd

extern "C" int sd_gather_kv_blocks(const void *k, const void *v, int dtype, int64_t B, int64_t H, int64_t T,
                                   int64_t D, int64_t sb, int64_t sh, int64_t st, const int64_t *idx, int64_t S,
                                   int block_size, void *k_out, void *v_out, void *stream) {
  if (!k || !v || !idx || !k_out || !v_out || B <= 0 || H <= 0 || T <= 0 || D <= 0 || S <= 0 || block_size <= 0)
    return SD_ERR_INVALID;
  if (S > 0x7fffffff || B * H > 65535) return SD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(static_cast<unsigned>(S), static_cast<unsigned>(B * H));
  SD_DISPATCH_DTYPE(dtype, E,
                    sd::gather_kv_kernel<E><<<grid, 256, 0, s>>>(
                        static_cast<const E *>(k), static_cast<const E *>(v), (int)H, T, (int)D, sb, sh, st, idx, S,
                        block_size, static_cast<E *>(k_out), static_cast<E *>(v_out)));
  return sd::check_launch();
}
