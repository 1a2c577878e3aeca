// Row kernels of the decode step around the attention path: RMSNorm
// (model/norm.py:15-21) and the SwiGLU gate (model/transformer.py:30-31),
// each one launch instead of the several elementwise ops of the reference.
#include "sd_common.cuh"

namespace sd {

// out = T(T(x * rsqrt(mean(x^2) + eps)) * w): the reference normalises in fp32,
// casts back to the activation dtype, then multiplies by the gain in that dtype.
template <typename T>
__global__ void rmsnorm_kernel(const T *__restrict__ x, int64_t x_rs, const T *__restrict__ w, int C, float eps,
                               T *__restrict__ out, int64_t o_rs) {
  pdl_wait();  // the input rows come from the kernel ahead
  const T *xr = x + blockIdx.x * x_rs;
  T *orow = out + blockIdx.x * o_rs;
  float ss = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float v = to_f(xr[c]);
    ss = fmaf(v, v, ss);
  }
  __shared__ float red[32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / static_cast<float>(C) + eps);
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float n = round_to<T>(to_f(xr[c]) * r);
    orow[c] = from_f<T>(n * to_f(w[c]));
  }
}

// Same arithmetic for many rows (prefill): one warp per row, 16-byte vector
// loads and stores, no block-wide reductions.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const T *__restrict__ x, int64_t x_rs,
                                                           const T *__restrict__ w, int C, float eps,
                                                           T *__restrict__ out, int64_t o_rs, int64_t rows) {
  pdl_wait();  // the input rows come from the kernel ahead
  constexpr int kE = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte chunk
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * x_rs);
  const uint4 *wr = reinterpret_cast<const uint4 *>(w);
  uint4 *orow = reinterpret_cast<uint4 *>(out + row * o_rs);
  const int nv = C / kE;
  float ss = 0.f;
  for (int c = lane; c < nv; c += 32) {
    const uint4 u = xr[c];
    const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
    for (int i = 0; i < kE; ++i) {
      const float v = to_f(e[i]);
      ss = fmaf(v, v, ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float r = rsqrtf(ss / static_cast<float>(C) + eps);
  for (int c = lane; c < nv; c += 32) {
    const uint4 u = xr[c], g = wr[c];
    const T *e = reinterpret_cast<const T *>(&u);
    const T *ge = reinterpret_cast<const T *>(&g);
    uint4 o;
    T *oe = reinterpret_cast<T *>(&o);
#pragma unroll
    for (int i = 0; i < kE; ++i) oe[i] = from_f<T>(round_to<T>(to_f(e[i]) * r) * to_f(ge[i]));
    orow[c] = o;
  }
}

// Same arithmetic for few rows (decode): one CTA per row, one 16-byte chunk
// per thread, a single block-wide reduction.
// Launch contract: blockDim.x == C * sizeof(T) / 16 exactly (every thread owns
// one 16-byte chunk of the row) and blockDim.x is a multiple of 32, at most
// 1024; rows and the gain are 16-byte aligned.  sd_rmsnorm checks all of this
// before choosing this kernel; a launch that breaks it returns without writing.
template <typename T>
__global__ void rmsnorm_chunk_kernel(const T *__restrict__ x, int64_t x_rs, const T *__restrict__ w, int C,
                                     float eps, T *__restrict__ out, int64_t o_rs) {
  pdl_wait();  // the input rows come from the kernel ahead
  constexpr int kE = 16 / static_cast<int>(sizeof(T));
  __shared__ float red[32];
  if (static_cast<int>(blockDim.x) * kE != C || (blockDim.x & 31u) != 0) return;  // contract broken: no writes
  const uint4 u = reinterpret_cast<const uint4 *>(x + blockIdx.x * x_rs)[threadIdx.x];
  const uint4 g = reinterpret_cast<const uint4 *>(w)[threadIdx.x];
  const T *e = reinterpret_cast<const T *>(&u);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kE; ++i) {
    const float v = to_f(e[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(C) + eps);
  const T *ge = reinterpret_cast<const T *>(&g);
  uint4 o;
  T *oe = reinterpret_cast<T *>(&o);
#pragma unroll
  for (int i = 0; i < kE; ++i) oe[i] = from_f<T>(round_to<T>(to_f(e[i]) * r) * to_f(ge[i]));
  reinterpret_cast<uint4 *>(out + blockIdx.x * o_rs)[threadIdx.x] = o;
}

// gu rows hold [gate | up] (2F values); out = T(T(silu(gate)) * up).
template <typename T>
__global__ void silu_mul_kernel(const T *__restrict__ gu, int64_t g_rs, int F, T *__restrict__ out,
                                int64_t o_rs) {
  pdl_wait();  // the input rows come from the kernel ahead
  const T *g = gu + blockIdx.y * g_rs;
  T *o = out + blockIdx.y * o_rs;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < F; c += gridDim.x * blockDim.x) {
    const float a = to_f(g[c]);
    const float s = round_to<T>(a / (1.0f + expf(-a)));
    o[c] = from_f<T>(s * to_f(g[F + c]));
  }
}

// The same for 16-bit rows in 16-byte chunks (8 values of gate, up and out
// per load / store): one CTA per row, a block-stride loop over the row's
// chunks.  F % 8 == 0 and 16-byte aligned rows (checked on the host).
template <typename T>
__global__ void silu_mul_vec_kernel(const T *__restrict__ gu, int64_t g_rs, int F, T *__restrict__ out,
                                    int64_t o_rs) {
  pdl_wait();
  const T *g = gu + static_cast<int64_t>(blockIdx.x) * g_rs;
  T *o = out + static_cast<int64_t>(blockIdx.x) * o_rs;
  for (int c = 8 * threadIdx.x; c < F; c += 8 * blockDim.x) {
    const uint4 a = *reinterpret_cast<const uint4 *>(g + c);
    const uint4 b = *reinterpret_cast<const uint4 *>(g + F + c);
    const T *av = reinterpret_cast<const T *>(&a);
    const T *bv = reinterpret_cast<const T *>(&b);
    uint4 r;
    T *rv = reinterpret_cast<T *>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = to_f(av[i]);
      const float sg = round_to<T>(x / (1.0f + expf(-x)));
      rv[i] = from_f<T>(sg * to_f(bv[i]));
    }
    *reinterpret_cast<uint4 *>(o + c) = r;
  }
}

// Greedy next token: per row, the index of the largest value, the first one
// on ties, NaN above every number (torch.argmax's order).  One CTA of 512
// threads per row: 16-byte loads where the row allows them, a warp shuffle
// reduction, then one across the warps.
__device__ __forceinline__ bool argmax_better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na != nb) return na;
  if (na) return ia < ib;
  return a > b || (a == b && ia < ib);
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(512) argmax_rows_kernel(const T *__restrict__ x, int64_t n, int64_t ld,
                                                          int64_t *__restrict__ out, int64_t o_stride) {
  pdl_wait();
  const T *row = x + static_cast<int64_t>(blockIdx.x) * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if (kVec) {
    for (int64_t c = 8 * static_cast<int64_t>(threadIdx.x); c < n; c += 8 * blockDim.x) {
      const uint4 u = *reinterpret_cast<const uint4 *>(row + c);
      const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v = to_f(e[i]);
        const int j = static_cast<int>(c) + i;
        if (argmax_better(v, j, bv, bi)) {
          bv = v;
          bi = j;
        }
      }
    }
  } else {
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) {
      const float v = to_f(row[c]);
      if (argmax_better(v, static_cast<int>(c), bv, bi)) {
        bv = v;
        bi = static_cast<int>(c);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (argmax_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __shared__ float wv[16];
  __shared__ int wi[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    wv[warp] = bv;
    wi[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = static_cast<int>(blockDim.x >> 5);
    bv = lane < nw ? wv[lane] : -INFINITY;
    bi = lane < nw ? wi[lane] : 0x7fffffff;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (argmax_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[static_cast<int64_t>(blockIdx.x) * o_stride] = bi;
  }
}

// RoPE of q [B,T,Hq,D] and k [B,T,Hkv,D] (rows addressed through strides)
// into contiguous outputs, one CTA per token (b, t): thread i takes 8
// consecutive elements of the first half of one head and the 8 they pair
// with in the second half, in 16-byte loads.  Requires D % 16 == 0 and
// 16-byte aligned rows (checked on the host).
template <typename T>
__global__ void rope_qk_kernel(const T *__restrict__ q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                               const T *__restrict__ k, int64_t k_sb, int64_t k_st, int64_t k_sh, int64_t Tn,
                               int Hq, int Hkv, int D, const float *__restrict__ cos_t,
                               const float *__restrict__ sin_t, int64_t offset, T *__restrict__ qo,
                               T *__restrict__ ko) {
  pdl_wait();
  constexpr int kV = 8;  // elements per 16-byte chunk (16-bit types; fp32 uses two chunks)
  const int64_t row = blockIdx.x;
  const int64_t b = row / Tn, t = row - (row / Tn) * Tn;
  const int half = D / 2, per_head = half / kV;
  const float *cr = cos_t + (offset + t) * half;
  const float *sr = sin_t + (offset + t) * half;
  for (int task = threadIdx.x; task < (Hq + Hkv) * per_head; task += blockDim.x) {
    const int hh = task / per_head, d0 = (task - hh * per_head) * kV;
    const bool isq = hh < Hq;
    const int h = isq ? hh : hh - Hq;
    const T *src = isq ? q + b * q_sb + t * q_st + h * q_sh : k + b * k_sb + t * k_st + h * k_sh;
    T *dst = (isq ? qo + (row * Hq + h) * D : ko + (row * Hkv + h) * D);
    constexpr int kW = kV * static_cast<int>(sizeof(T)) / 16;  // 16-byte words per 8 elements
    uint4 ul[kW], uh[kW], ol[kW], oh[kW];
#pragma unroll
    for (int w = 0; w < kW; ++w) {
      ul[w] = reinterpret_cast<const uint4 *>(src + d0)[w];
      uh[w] = reinterpret_cast<const uint4 *>(src + half + d0)[w];
    }
    const T *lo = reinterpret_cast<const T *>(ul), *hi = reinterpret_cast<const T *>(uh);
    T *olo = reinterpret_cast<T *>(ol), *ohi = reinterpret_cast<T *>(oh);
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const float c = cr[d0 + i], sn = sr[d0 + i];
      const float xl = to_f(lo[i]), xh = to_f(hi[i]);
      olo[i] = from_f<T>(rope_rounded<T>(xl, -xh, c, sn));
      ohi[i] = from_f<T>(rope_rounded<T>(xh, xl, c, sn));
    }
#pragma unroll
    for (int w = 0; w < kW; ++w) {
      reinterpret_cast<uint4 *>(dst + d0)[w] = ol[w];
      reinterpret_cast<uint4 *>(dst + half + d0)[w] = oh[w];
    }
  }
}

}  // namespace sd

extern "C" int sd_rope_qk(const void *q, const void *k, int dtype, int64_t B, int64_t T, int64_t Hq, int64_t Hkv,
                          int64_t D, int64_t q_sb, int64_t q_st, int64_t q_sh, int64_t k_sb, int64_t k_st,
                          int64_t k_sh, const float *rope_cos, const float *rope_sin, int64_t max_pos,
                          int64_t offset, void *q_out, void *k_out, void *stream) {
  if (!q || !k || !rope_cos || !rope_sin || !q_out || !k_out || B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 ||
      offset < 0)
    return SD_ERR_INVALID;
  if (D % 16 != 0 || offset + T > max_pos) return D % 16 != 0 ? SD_ERR_UNSUPPORTED : SD_ERR_INVALID;
  const int64_t ev = 16 / sd::dtype_size(dtype);  // elements per 16 bytes
  if (!sd::aligned16(q) || !sd::aligned16(k) || !sd::aligned16(q_out) || !sd::aligned16(k_out) || q_sb % ev ||
      q_st % ev || q_sh % ev || k_sb % ev || k_st % ev || k_sh % ev)
    return SD_ERR_ALIGN;
  if (B * T > 0x7fffffff || (Hq + Hkv) * D > (1 << 16)) return SD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = static_cast<int>((Hq + Hkv) * (D / 16) < 256 ? (((Hq + Hkv) * (D / 16) + 31) / 32) * 32 : 256);
  SD_DISPATCH_DTYPE(dtype, E,
                    return sd::launch(sd::rope_qk_kernel<E>, dim3(static_cast<unsigned>(B * T)), dim3(threads), 0, s,
                                      sd::pdl_enabled(), static_cast<const E *>(q), q_sb, q_st, q_sh,
                                      static_cast<const E *>(k), k_sb, k_st, k_sh, T, (int)Hq, (int)Hkv, (int)D,
                                      rope_cos, rope_sin, offset, static_cast<E *>(q_out), static_cast<E *>(k_out)));
  return SD_OK;
}

extern "C" int sd_rmsnorm(const void *x, int dtype, int64_t rows, int64_t C, int64_t x_rs, const void *w,
                          float eps, void *out, int64_t o_rs, void *stream) {
  if (!x || !w || !out || rows <= 0 || C <= 0) return SD_ERR_INVALID;
  if (rows > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = sd::pdl_enabled();
  const int es = sd::dtype_size(dtype);
  if (rows >= 512 && (C * es) % 16 == 0 && (x_rs * es) % 16 == 0 && (o_rs * es) % 16 == 0 && sd::aligned16(x) &&
      sd::aligned16(w) && sd::aligned16(out)) {
    const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
    SD_DISPATCH_DTYPE(dtype, E,
                      return sd::launch(sd::rmsnorm_rows_kernel<E>, dim3(grid), dim3(256), 0, s, pdl,
                                        static_cast<const E *>(x), x_rs, static_cast<const E *>(w), (int)C, eps,
                                        static_cast<E *>(out), o_rs, rows));
  }
  const int64_t chunks = C * es / 16;
  if ((C * es) % 16 == 0 && chunks % 32 == 0 && chunks <= 1024 && (x_rs * es) % 16 == 0 && (o_rs * es) % 16 == 0 &&
      sd::aligned16(x) && sd::aligned16(w) && sd::aligned16(out)) {
    SD_DISPATCH_DTYPE(dtype, E,
                      return sd::launch(sd::rmsnorm_chunk_kernel<E>, dim3(static_cast<unsigned>(rows)),
                                        dim3(static_cast<unsigned>(chunks)), 0, s, pdl, static_cast<const E *>(x), x_rs,
                                        static_cast<const E *>(w), (int)C, eps, static_cast<E *>(out), o_rs));
  }
  const int threads = C >= 1024 ? 1024 : static_cast<int>(((C + 31) / 32) * 32);
  SD_DISPATCH_DTYPE(dtype, E,
                    return sd::launch(sd::rmsnorm_kernel<E>, dim3(static_cast<unsigned>(rows)), dim3(threads), 0, s,
                                      pdl, static_cast<const E *>(x), x_rs, static_cast<const E *>(w), (int)C, eps,
                                      static_cast<E *>(out), o_rs));
  return SD_OK;
}

extern "C" int sd_silu_mul(const void *gu, int dtype, int64_t rows, int64_t F, int64_t g_rs, void *out,
                           int64_t o_rs, void *stream) {
  if (!gu || !out || rows <= 0 || F <= 0) return SD_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype != SD_DTYPE_F32 && F % 8 == 0 && g_rs % 8 == 0 && o_rs % 8 == 0 && sd::aligned16(gu) &&
      sd::aligned16(out) && rows <= 0x7fffffff) {
    const int64_t chunks = F / 8;
    const unsigned threads = static_cast<unsigned>(chunks >= 256 ? 256 : ((chunks + 31) / 32) * 32);
    SD_DISPATCH_DTYPE(dtype, E,
                      return sd::launch(sd::silu_mul_vec_kernel<E>, dim3(static_cast<unsigned>(rows)), dim3(threads),
                                        0, s, sd::pdl_enabled(), static_cast<const E *>(gu), g_rs, (int)F,
                                        static_cast<E *>(out), o_rs));
  }
  if (rows > 65535) return SD_ERR_UNSUPPORTED;
  const unsigned gx = static_cast<unsigned>((F + 255) / 256 < 8 ? (F + 255) / 256 : 8);
  SD_DISPATCH_DTYPE(dtype, E,
                    return sd::launch(sd::silu_mul_kernel<E>, dim3(gx, static_cast<unsigned>(rows)), dim3(256), 0, s,
                                      sd::pdl_enabled(), static_cast<const E *>(gu), g_rs, (int)F,
                                      static_cast<E *>(out), o_rs));
  return SD_OK;
}

extern "C" int sd_argmax_rows(const void *x, int dtype, int64_t rows, int64_t n, int64_t ld, int64_t *out,
                              int64_t o_stride, void *stream) {
  if (!x || !out || rows <= 0 || n <= 0 || ld < n) return SD_ERR_INVALID;
  if (rows > 0x7fffffff || n > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = dtype != SD_DTYPE_F32 && n % 8 == 0 && ld % 8 == 0 && sd::aligned16(x);
  const dim3 grid(static_cast<unsigned>(rows));
  SD_DISPATCH_DTYPE(dtype, E, {
    if (vec)
      return sd::launch(sd::argmax_rows_kernel<E, true>, grid, dim3(512), 0, s, sd::pdl_enabled(),
                        static_cast<const E *>(x), n, ld, out, o_stride);
    return sd::launch(sd::argmax_rows_kernel<E, false>, grid, dim3(512), 0, s, sd::pdl_enabled(),
                      static_cast<const E *>(x), n, ld, out, o_stride);
  });
  return SD_OK;
}
