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

// Same copy in 16-byte chunks, for rows of D elements in aligned 16-byte
// chunks: one CTA per (b, h, selected slot), each thread moves kPer chunks of
// K and of V with every load issued before the first store.
template <typename T, int kPer>
__global__ void __launch_bounds__(256) gather_kv_vec_kernel(const T *__restrict__ k, const T *__restrict__ v, int H,
                                                            int64_t T_, int D, int64_t sb, int64_t sh, int64_t st,
                                                            const int64_t *__restrict__ idx, int64_t S, int bs,
                                                            T *__restrict__ ko, T *__restrict__ vo) {
  constexpr int kV = 16 / static_cast<int>(sizeof(T));
  const int64_t slot = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / H, h = bh - (bh / H) * H;
  const int64_t nb = (T_ + bs - 1) / bs;
  const int64_t j = idx[bh * S + slot];
  const bool ok = j >= 0 && j < nb;
  const int cpr = D / kV;  // chunks per row
  const int chunks = bs * cpr;
  uint4 *kd = reinterpret_cast<uint4 *>(ko + (bh * S + slot) * bs * D);
  uint4 *vd = reinterpret_cast<uint4 *>(vo + (bh * S + slot) * bs * D);
  const T *kb = k + b * sb + h * sh, *vb = v + b * sb + h * sh;
  for (int base = 0; base < chunks; base += kPer * 256) {
    uint4 uk[kPer], uv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = base + i * 256 + threadIdx.x;
      const int r = e / cpr, c = e - r * cpr;
      const int64_t t = j * bs + r;
      uk[i] = uv[i] = make_uint4(0u, 0u, 0u, 0u);
      if (e < chunks && ok && t < T_) {
        uk[i] = *reinterpret_cast<const uint4 *>(kb + t * st + c * kV);
        uv[i] = *reinterpret_cast<const uint4 *>(vb + t * st + c * kV);
      }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = base + i * 256 + threadIdx.x;
      if (e < chunks) {
        kd[e] = uk[i];
        vd[e] = uv[i];
      }
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
  const int es = sd::dtype_size(dtype);
  const int64_t kv = 16 / es;
  if (sd::aligned16(k) && sd::aligned16(v) && sd::aligned16(k_out) && sd::aligned16(v_out) && D % kv == 0 &&
      sb % kv == 0 && sh % kv == 0 && st % kv == 0 && static_cast<int64_t>(block_size) * D <= (1 << 20)) {
    SD_DISPATCH_DTYPE(dtype, E,
                      sd::gather_kv_vec_kernel<E, 2><<<grid, 256, 0, s>>>(
                          static_cast<const E *>(k), static_cast<const E *>(v), (int)H, T, (int)D, sb, sh, st, idx,
                          S, block_size, static_cast<E *>(k_out), static_cast<E *>(v_out)));
    return sd::check_launch();
  }
  SD_DISPATCH_DTYPE(dtype, E,
                    sd::gather_kv_kernel<E><<<grid, 256, 0, s>>>(
                        static_cast<const E *>(k), static_cast<const E *>(v), (int)H, T, (int)D, sb, sh, st, idx, S,
                        block_size, static_cast<E *>(k_out), static_cast<E *>(v_out)));
  return sd::check_launch();
}
