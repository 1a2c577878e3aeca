// Backward pass of the block-sparse GQA prefill attention: the gradients that
// autograd takes through the reference's masked and chunked SDPA paths
// (model/attention/sparse.py:185-364) when a model is trained with the sparse
// backend (tests/test_sparse_attention.py:63-77, training/trainer.py).
//
// Inputs are the forward's q, k, v, the upstream gradient dO and the same
// block lists (and per-row top-k for the masked forecast mode) as
// sd_prefill_attention, so the allowed (query, key) pairs are exactly the
// forward's.  With P the softmax of scale * q k^T over the allowed keys:
//   dV = P^T dO      dP = dO V^T      Delta = rowsum(P * dP)
//   dS = P * (dP - Delta)      dQ = scale * dS K      dK = scale * dS^T Q
// all in fp32.  One CTA per (64-token query block, query head, sequence),
// 256 threads.  Pass 1 walks the block list for each row's softmax statistics
// (running maximum, sum of exponentials and sum of exp * dP, so Delta needs no
// forward output); pass 2 walks it again for the gradients.  Every product is
// a 64 x 64 x 64 fp32 product over shared-memory tiles with rows padded to 65
// floats (column walks hit distinct banks); thread (ti, tj) owns rows ti + 16a
// and columns tj + 16b of each 64 x 64 result.  dQ rows belong to one CTA and
// are stored; dK and dV of a key block collect contributions from every query
// block and head that lists it and are added with fp32 atomics into buffers
// the entry point zeroes first.  16-bit inputs with 16-byte aligned rows take
// prefill_bwd_tc_kernel below instead (tensor-core products: all seven for
// bf16, S and dP for f16); this kernel serves fp32 inputs and other strides.
#include "sd_prefill.cuh"
#include "sd_tma.cuh"

namespace sd {
namespace bwd {

constexpr int kThreads = 256;
constexpr int kLd = kHeadDim + 1;  // padded row stride of the shared tiles, floats
constexpr int kTile = kQTile * kLd;
constexpr size_t kSmemBytes = 6 * kTile * sizeof(float) + kQTile * sizeof(int);

// acc[a][b] += sum_x A[row a][x] * B[row b][x]   (A B^T)
__device__ __forceinline__ void mm_abt(const float *A, const float *B, int ti, int tj, float (&acc)[4][4]) {
#pragma unroll 4
  for (int x = 0; x < kHeadDim; ++x) {
    float av[4], bv[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) av[a] = A[(ti + 16 * a) * kLd + x];
#pragma unroll
    for (int b = 0; b < 4; ++b) bv[b] = B[(tj + 16 * b) * kLd + x];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
  }
}

// acc[a][b] += sum_x A[row a][x] * B[x][col b]   (A B)
__device__ __forceinline__ void mm_ab(const float *A, const float *B, int ti, int tj, float (&acc)[4][4]) {
#pragma unroll 4
  for (int x = 0; x < kQTile; ++x) {
    float av[4], bv[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) av[a] = A[(ti + 16 * a) * kLd + x];
#pragma unroll
    for (int b = 0; b < 4; ++b) bv[b] = B[x * kLd + tj + 16 * b];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
  }
}

// acc[a][b] += sum_x A[x][col a] * B[x][col b]   (A^T B)
__device__ __forceinline__ void mm_atb(const float *A, const float *B, int ti, int tj, float (&acc)[4][4]) {
#pragma unroll 4
  for (int x = 0; x < kQTile; ++x) {
    float av[4], bv[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) av[a] = A[x * kLd + ti + 16 * a];
#pragma unroll
    for (int b = 0; b < 4; ++b) bv[b] = B[x * kLd + tj + 16 * b];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
  }
}

// Sum / maximum over the 16 lanes that share a row (lanes 0-15 or 16-31).
__device__ __forceinline__ float half_sum(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float half_max(float x) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    prefill_bwd_kernel(const T *__restrict__ q, int64_t q_sb, int64_t q_st, int64_t q_sh, const T *__restrict__ k,
                       const T *__restrict__ v, int64_t c_sb, int64_t c_sh, int64_t c_st,
                       const T *__restrict__ dout, int64_t g_sb, int64_t g_st, int64_t g_sh, int64_t T_, int Hq,
                       int Hkv, const int32_t *__restrict__ lists, const int32_t *__restrict__ counts, int lcap,
                       const int64_t *__restrict__ topk, int kk, int causal, float scale, float *__restrict__ dq,
                       float *__restrict__ dk, float *__restrict__ dv) {
  extern __shared__ float smf[];
  float *Qs = smf;          // q rows of the query block
  float *Gs = Qs + kTile;   // dO rows
  float *Ks = Gs + kTile;   // key block
  float *Vs = Ks + kTile;   // value block
  float *Ps = Vs + kTile;   // P of the block
  float *Ds = Ps + kTile;   // dS of the block
  int *s_ok = reinterpret_cast<int *>(Ds + kTile);  // row may see the block (valid row, member)

  const int qt = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv, h = hq / G;
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  const int64_t t0 = static_cast<int64_t>(qt) * kQTile;
  const int nqt = gridDim.x;
  const int64_t nbk = (T_ + kQTile - 1) / kQTile;

  for (int e = tid; e < kQTile * kHeadDim; e += kThreads) {
    const int r = e / kHeadDim, d = e % kHeadDim;
    const int64_t t = t0 + r;
    const bool ok = t < T_;
    Qs[r * kLd + d] = ok ? to_f(q[b * q_sb + t * q_st + hq * q_sh + d]) : 0.f;
    Gs[r * kLd + d] = ok ? to_f(dout[b * g_sb + t * g_st + hq * g_sh + d]) : 0.f;
  }
  const int64_t lrow = (static_cast<int64_t>(b) * Hkv + h) * nqt + qt;
  const int32_t *list = lists + lrow * lcap;
  int cnt = counts[lrow];
  cnt = cnt < 0 ? 0 : (cnt > lcap ? lcap : cnt);
  const T *kb = k + b * c_sb + h * c_sh;
  const T *vb = v + b * c_sb + h * c_sh;

  // stages key block j into Ks / Vs and each row's permission into s_ok
  auto stage = [&](int j) {
    const int64_t k0 = static_cast<int64_t>(j) * kQTile;
    for (int e = tid; e < kQTile * kHeadDim; e += kThreads) {
      const int rr = e / kHeadDim, d = e % kHeadDim;
      const int64_t kt = k0 + rr;
      const bool ok = kt < T_;
      Ks[rr * kLd + d] = ok ? to_f(kb[kt * c_st + d]) : 0.f;
      Vs[rr * kLd + d] = ok ? to_f(vb[kt * c_st + d]) : 0.f;
    }
    if (tid < kQTile) {
      const int64_t t = t0 + tid;
      bool ok = t < T_;
      if (ok && topk) {  // masked forecast mode: per-row membership (sparse.py:243-247)
        const int bq = static_cast<int>(t / kQTile);
        const int64_t *rowk = topk + ((static_cast<int64_t>(b) * Hkv + h) * T_ + t) * kk;
        bool in = (j == 0) || (j == bq);
        for (int e = 0; e < kk && !in; ++e) {
          int64_t jj = rowk[e];
          jj = jj < 0 ? 0 : (jj > nbk - 1 ? nbk - 1 : jj);
          in = jj == j;
        }
        ok = in;
      }
      s_ok[tid] = ok ? 1 : 0;
    }
  };
  // whether (row ti + 16a, key tj + 16b of block j) is an allowed pair
  auto allowed = [&](int a, int bb, int64_t k0) {
    const int r = ti + 16 * a;
    const int64_t kt = k0 + tj + 16 * bb;
    return s_ok[r] != 0 && kt < T_ && (!causal || kt <= t0 + r);
  };

  // ---- pass 1: per-row maximum m, sum of exponentials l, sum of exp * dP
  float m[4], l[4], pd[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    m[a] = -INFINITY;
    l[a] = 0.f;
    pd[a] = 0.f;
  }
  for (int i = 0; i < cnt; ++i) {
    const int j = list[i];
    if (j < 0 || j >= nbk) continue;  // uniform across the CTA
    __syncthreads();
    stage(j);
    __syncthreads();
    const int64_t k0 = static_cast<int64_t>(j) * kQTile;
    float s[4][4] = {}, dp[4][4] = {};
    mm_abt(Qs, Ks, ti, tj, s);
    mm_abt(Gs, Vs, ti, tj, dp);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float x[4], mx = -INFINITY;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        x[bb] = allowed(a, bb, k0) ? s[a][bb] * scale : -INFINITY;
        mx = fmaxf(mx, x[bb]);
      }
      const float mn = fmaxf(m[a], half_max(mx));
      const float alpha = m[a] == -INFINITY ? 0.f : expf(m[a] - mn);
      float ls = 0.f, lp = 0.f;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const float e = x[bb] == -INFINITY ? 0.f : expf(x[bb] - mn);
        ls += e;
        lp = fmaf(e, dp[a][bb], lp);
      }
      ls = half_sum(ls);
      lp = half_sum(lp);
      l[a] = fmaf(l[a], alpha, ls);
      pd[a] = fmaf(pd[a], alpha, lp);
      m[a] = mn;
    }
  }
  // log-sum-exp and Delta of each owned row (rows that see nothing: P = 0)
  float lse[4], delta[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    lse[a] = l[a] > 0.f ? m[a] + logf(l[a]) : INFINITY;
    delta[a] = l[a] > 0.f ? pd[a] / l[a] : 0.f;
  }

  // ---- pass 2: P, dS per block; dQ in registers, dK / dV atomically
  float gq[4][4] = {};
  for (int i = 0; i < cnt; ++i) {
    const int j = list[i];
    if (j < 0 || j >= nbk) continue;
    __syncthreads();
    stage(j);
    __syncthreads();
    const int64_t k0 = static_cast<int64_t>(j) * kQTile;
    float s[4][4] = {}, dp[4][4] = {};
    mm_abt(Qs, Ks, ti, tj, s);
    mm_abt(Gs, Vs, ti, tj, dp);
    bool any = false;
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        float p = 0.f, ds = 0.f;
        if (allowed(a, bb, k0)) {
          p = expf(s[a][bb] * scale - lse[a]);
          ds = p * (dp[a][bb] - delta[a]);
          any = true;
        }
        Ps[(ti + 16 * a) * kLd + tj + 16 * bb] = p;
        Ds[(ti + 16 * a) * kLd + tj + 16 * bb] = ds;
      }
    if (!__syncthreads_or(any)) continue;  // no allowed pair in this block: nothing to add
    mm_ab(Ds, Ks, ti, tj, gq);
    float gk[4][4] = {}, gv[4][4] = {};
    mm_atb(Ds, Qs, ti, tj, gk);
    mm_atb(Ps, Gs, ti, tj, gv);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int64_t kt = k0 + ti + 16 * a;
      if (kt >= T_) continue;
      const int64_t base = ((static_cast<int64_t>(b) * Hkv + h) * T_ + kt) * kHeadDim;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        atomicAdd(dk + base + tj + 16 * bb, scale * gk[a][bb]);
        atomicAdd(dv + base + tj + 16 * bb, gv[a][bb]);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t t = t0 + ti + 16 * a;
    if (t >= T_) continue;
    float *dst = dq + ((static_cast<int64_t>(b) * T_ + t) * Hq + hq) * kHeadDim;
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) dst[tj + 16 * bb] = scale * gq[a][bb];
  }
}

// ---------------------------------------------------------------------------
// 16-bit inputs: S = Q K^T and dP = dO V^T on the tensor cores (mma.sync
// m16n8k16, fp32 accumulators).  A product of two 16-bit values is exact in
// fp32, so these match the fp32 products above up to accumulation order.  Warp
// w computes S / dP for rows 16 (w % 4) .. +15 and keys 32 (w / 4) .. +31 of
// each block; pass 1 keeps separate running statistics per key half, merged
// once at its end.  The three products that consume P and dS:
//   * kMma (bf16): on the tensor cores too, with P and dS each split into a
//     bf16 high part and the bf16 of the remainder (16 significant bits; each
//     product runs twice and sums in fp32): dQ from dS tiles (ldmatrix) and
//     K (ldmatrix.trans), dK / dV from dS^T / P^T (ldmatrix.trans) and Q / dO;
//     warp w owns rows (dQ) or keys (dK, dV) 16 (w % 4) .. and head-dim
//     columns 32 (w / 4) ..;
//   * otherwise (f16, whose range could flush a small remainder): fp32
//     CUDA-core products reading K, Q and dO from the same 16-bit tiles.
// ---------------------------------------------------------------------------
constexpr int kLdb = 72;  // 16-bit tile row stride in elements (144 bytes: ldmatrix rows on distinct banks)
constexpr int kTileB = kQTile * kLdb;
// Q, dO, K, V tiles, then either the P / dS hi / lo tiles (kMma) or fp32 P and
// dS (the larger of the two), the row flags and the pass-1 statistics
constexpr size_t kPdBytes = 4 * kTileB * 2 > 2 * kTile * sizeof(float) ? 4 * kTileB * 2 : 2 * kTile * sizeof(float);
constexpr size_t kSmemTcBytes = 6 * kTileB * 2 + kPdBytes + 2 * kQTile * sizeof(int) + 2 * kQTile * 3 * sizeof(float);

// 16-byte asynchronous global -> shared copy; src_bytes = 0 fills zeros
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// acc[a][b] += sum_x A[row a][x] * B[x][col b], B a 16-bit tile
template <typename T>
__device__ __forceinline__ void mm_ab16(const float *A, const T *B, int ti, int tj, float (&acc)[4][4]) {
#pragma unroll 4
  for (int x = 0; x < kQTile; ++x) {
    float av[4], bv[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) av[a] = A[(ti + 16 * a) * kLd + x];
#pragma unroll
    for (int b = 0; b < 4; ++b) bv[b] = to_f(B[x * kLdb + tj + 16 * b]);
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
  }
}

// acc[a][b] += sum_x A[x][col a] * B[x][col b], B a 16-bit tile
template <typename T>
__device__ __forceinline__ void mm_atb16(const float *A, const T *B, int ti, int tj, float (&acc)[4][4]) {
#pragma unroll 4
  for (int x = 0; x < kQTile; ++x) {
    float av[4], bv[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) av[a] = A[x * kLd + ti + 16 * a];
#pragma unroll
    for (int b = 0; b < 4; ++b) bv[b] = to_f(B[x * kLdb + tj + 16 * b]);
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
  }
}

// Sum / maximum over the 4 lanes that share a row of an mma.sync C fragment.
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x + __shfl_xor_sync(0xffffffffu, x, 2);
}
__device__ __forceinline__ float quad_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
}

template <typename T, bool kMma>
__global__ void __launch_bounds__(kThreads, 2)
    prefill_bwd_tc_kernel(const T *__restrict__ q, int64_t q_sb, int64_t q_st, int64_t q_sh, const T *__restrict__ k,
                          const T *__restrict__ v, int64_t c_sb, int64_t c_sh, int64_t c_st,
                          const T *__restrict__ dout, int64_t g_sb, int64_t g_st, int64_t g_sh, int64_t T_, int Hq,
                          int Hkv, const int32_t *__restrict__ lists, const int32_t *__restrict__ counts, int lcap,
                          const int64_t *__restrict__ topk, int kk, int causal, float scale, float *__restrict__ dq,
                          float *__restrict__ dk, float *__restrict__ dv) {
  extern __shared__ __align__(16) char smraw[];
  T *Qb = reinterpret_cast<T *>(smraw);  // q  [row][d]
  T *Gb = Qb + kTileB;                   // dO [row][d]
  T *const Kbuf = Gb + kTileB;           // k, v of a block [key][d], two buffers: K0 V0 K1 V1
  T *Kb = Kbuf, *Vb = Kbuf + kTileB;     // the buffer of the block being computed
  float *Ps = reinterpret_cast<float *>(Kbuf + 4 * kTileB);  // P  [row][key] (fp32 products)
  float *Ds = Ps + kTile;                                    // dS [row][key]
  T *Ph = Kbuf + 4 * kTileB;                                 // P  high / low parts [row][key] (kMma)
  T *Pl = Ph + kTileB;
  T *Dh = Pl + kTileB;                                       // dS high / low parts
  T *Dl = Dh + kTileB;
  int *const s_okbuf = reinterpret_cast<int *>(smraw + 6 * kTileB * sizeof(T) + kPdBytes);  // [2][row]
  int *s_ok = s_okbuf;
  float *s_stat = reinterpret_cast<float *>(s_okbuf + 2 * kQTile);  // [key half][row][m, l, pd]

  const int qt = blockIdx.x, hq = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv, h = hq / G;
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  const int warp = tid >> 5, lane = tid & 31;
  const int rg = warp & 3, kh = warp >> 2;  // MMA rows 16 rg .., keys 32 kh ..
  const int r0 = 16 * rg + (lane >> 2);     // this thread's fragment rows r0 and r0 + 8
  const int kc = 32 * kh + 2 * (lane & 3);  // its fragment keys kc + 8 nt + {0, 1}
  const int64_t t0 = static_cast<int64_t>(qt) * kQTile;
  const int nqt = gridDim.x;
  const int64_t nbk = (T_ + kQTile - 1) / kQTile;
  constexpr int kCh = kHeadDim / 8;  // 16-byte chunks of a row

  for (int e = tid; e < kQTile * kCh; e += kThreads) {
    const int r = e / kCh, c8 = (e - r * kCh) * 8;
    const int64_t t = t0 + r;
    uint4 xq = make_uint4(0u, 0u, 0u, 0u), xg = xq;
    if (t < T_) {
      xq = *reinterpret_cast<const uint4 *>(q + b * q_sb + t * q_st + hq * q_sh + c8);
      xg = *reinterpret_cast<const uint4 *>(dout + b * g_sb + t * g_st + hq * g_sh + c8);
    }
    *reinterpret_cast<uint4 *>(Qb + r * kLdb + c8) = xq;
    *reinterpret_cast<uint4 *>(Gb + r * kLdb + c8) = xg;
  }
  const int64_t lrow = (static_cast<int64_t>(b) * Hkv + h) * nqt + qt;
  const int32_t *list = lists + lrow * lcap;
  int cnt = counts[lrow];
  cnt = cnt < 0 ? 0 : (cnt > lcap ? lcap : cnt);
  const T *kbase = k + b * c_sb + h * c_sh;
  const T *vbase = v + b * c_sb + h * c_sh;

  // copies block j's K / V rows into buffer `buf` (asynchronously, one
  // commit group) and writes the rows' permissions for it
  auto stage = [&](int j, int buf) {
    const int64_t k0 = static_cast<int64_t>(j) * kQTile;
    T *kd = Kbuf + 2 * buf * kTileB, *vd = kd + kTileB;
    for (int e = tid; e < kQTile * kCh; e += kThreads) {
      const int c = e / kCh, c8 = (e - c * kCh) * 8;
      const int64_t kt = k0 + c;
      const bool in = kt < T_;
      const int64_t src = in ? kt * c_st + c8 : 0;
      cp_async16(kd + c * kLdb + c8, kbase + src, in ? 16 : 0);
      cp_async16(vd + c * kLdb + c8, vbase + src, in ? 16 : 0);
    }
    cp_async_commit();
    if (tid < kQTile) {
      const int64_t t = t0 + tid;
      bool ok = t < T_;
      if (ok && topk) {  // masked forecast mode: per-row membership (sparse.py:243-247)
        const int bq = static_cast<int>(t / kQTile);
        const int64_t *rowk = topk + ((static_cast<int64_t>(b) * Hkv + h) * T_ + t) * kk;
        bool in = (j == 0) || (j == bq);
        for (int e = 0; e < kk && !in; ++e) {
          int64_t jj = rowk[e];
          jj = jj < 0 ? 0 : (jj > nbk - 1 ? nbk - 1 : jj);
          in = jj == j;
        }
        ok = in;
      }
      s_okbuf[buf * kQTile + tid] = ok ? 1 : 0;
    }
  };
  // next listed block at or after list position i (entries outside the cache are skipped)
  auto next_valid = [&](int i) {
    while (i < cnt && (list[i] < 0 || list[i] >= nbk)) ++i;
    return i;
  };
  // walks the list with block i + 1's copies in flight while block i is
  // computed; body(k0) runs with Kb / Vb / s_ok pointing at block i's buffer
  auto walk = [&](auto &&body) {
    int i = next_valid(0), buf = 0;
    if (i < cnt) stage(list[i], 0);
    while (i < cnt) {
      const int inext = next_valid(i + 1);
      __syncthreads();  // every thread is done with the other buffer (the previous block)
      if (inext < cnt) {
        stage(list[inext], buf ^ 1);
      } else {
        cp_async_commit();  // an empty group keeps the wait below uniform
      }
      cp_async_wait1();  // block i's copies (all groups but the newest) have landed
      __syncthreads();
      Kb = Kbuf + 2 * buf * kTileB;
      Vb = Kb + kTileB;
      s_ok = s_okbuf + buf * kQTile;
      body(static_cast<int64_t>(list[i]) * kQTile);
      buf ^= 1;
      i = inext;
    }
  };
  auto allowed = [&](int r, int key, int64_t k0) {
    const int64_t kt = k0 + key;
    return s_ok[r] != 0 && kt < T_ && (!causal || kt <= t0 + r);
  };
  // S (s) and dP (p) of this warp's 16 x 32 block: n-tiles nt = keys 32 kh + 8 nt ..
  auto products = [&](float (&sacc)[4][4], float (&pacc)[4][4]) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sacc[nt][i] = 0.f;
        pacc[nt][i] = 0.f;
      }
#pragma unroll
    for (int ks = 0; ks < kHeadDim / 16; ++ks) {
      uint32_t aq[4], ag[4];
      const int arow = 16 * rg + (lane & 15), acol = 16 * ks + (lane >> 4) * 8;
      ldsm_x4(smem_u32(Qb + arow * kLdb + acol), aq[0], aq[1], aq[2], aq[3]);
      ldsm_x4(smem_u32(Gb + arow * kLdb + acol), ag[0], ag[1], ag[2], ag[3]);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int brow = 32 * kh + 16 * np + (lane & 7) + ((lane >> 4) << 3);
        const int bcol = 16 * ks + ((lane >> 3) & 1) * 8;
        uint32_t bk[4], bv[4];
        ldsm_x4(smem_u32(Kb + brow * kLdb + bcol), bk[0], bk[1], bk[2], bk[3]);
        ldsm_x4(smem_u32(Vb + brow * kLdb + bcol), bv[0], bv[1], bv[2], bv[3]);
        mma16816<T>(sacc[2 * np], aq, bk[0], bk[1]);
        mma16816<T>(sacc[2 * np + 1], aq, bk[2], bk[3]);
        mma16816<T>(pacc[2 * np], ag, bv[0], bv[1]);
        mma16816<T>(pacc[2 * np + 1], ag, bv[2], bv[3]);
      }
    }
  };

  // ---- pass 1: per (row, key half) running maximum, sum of exponentials and
  // sum of exp * dP
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, pd[2] = {0.f, 0.f};
  walk([&](int64_t k0) {
    float sa[4][4], pa[4][4];
    products(sa, pa);
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = r0 + 8 * hr;
      float x[8], mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          x[2 * nt + e] = allowed(r, kc + 8 * nt + e, k0) ? sa[nt][2 * hr + e] * scale : -INFINITY;
          mx = fmaxf(mx, x[2 * nt + e]);
        }
      const float mn = fmaxf(m[hr], quad_max(mx));
      const float alpha = m[hr] == -INFINITY ? 0.f : expf(m[hr] - mn);
      float ls = 0.f, lp = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float ex = x[2 * nt + e] == -INFINITY ? 0.f : expf(x[2 * nt + e] - mn);
          ls += ex;
          lp = fmaf(ex, pa[nt][2 * hr + e], lp);
        }
      l[hr] = fmaf(l[hr], alpha, quad_sum(ls));
      pd[hr] = fmaf(pd[hr], alpha, quad_sum(lp));
      m[hr] = mn;
    }
  });
  // merge the two key halves of every row
  if ((lane & 3) == 0)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float *st = s_stat + (kh * kQTile + r0 + 8 * hr) * 3;
      st[0] = m[hr];
      st[1] = l[hr];
      st[2] = pd[hr];
    }
  __syncthreads();
  float lse[2], delta[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const float *s0 = s_stat + (r0 + 8 * hr) * 3, *s1 = s_stat + (kQTile + r0 + 8 * hr) * 3;
    const float mm = fmaxf(s0[0], s1[0]);
    const float e0 = s0[0] == -INFINITY ? 0.f : expf(s0[0] - mm), e1 = s1[0] == -INFINITY ? 0.f : expf(s1[0] - mm);
    const float ll = s0[1] * e0 + s1[1] * e1, pp = s0[2] * e0 + s1[2] * e1;
    lse[hr] = ll > 0.f ? mm + logf(ll) : INFINITY;
    delta[hr] = ll > 0.f ? pp / ll : 0.f;
  }

  // ---- pass 2: P, dS per block; dQ in registers, dK / dV atomically
  float gq[4][4] = {};  // dQ: CUDA-core 4 x 4 blocks, or (kMma) this warp's MMA fragments
  const int fg = lane >> 2, fc = lane & 3;  // fragment row group / column pair
  walk([&](int64_t k0) {
    float sa[4][4], pa[4][4];
    products(sa, pa);
    bool any = false;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = r0 + 8 * hr;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int key = kc + 8 * nt;
        float p[2] = {0.f, 0.f}, ds[2] = {0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (allowed(r, key + e, k0)) {
            p[e] = expf(sa[nt][2 * hr + e] * scale - lse[hr]);
            ds[e] = p[e] * (pa[nt][2 * hr + e] - delta[hr]);
            any = true;
          }
        if constexpr (kMma) {
          const float ph0 = to_f(from_f<T>(p[0])), ph1 = to_f(from_f<T>(p[1]));
          const float dh0 = to_f(from_f<T>(ds[0])), dh1 = to_f(from_f<T>(ds[1]));
          *reinterpret_cast<uint32_t *>(Ph + r * kLdb + key) = pack2<T>(ph0, ph1);
          *reinterpret_cast<uint32_t *>(Pl + r * kLdb + key) = pack2<T>(p[0] - ph0, p[1] - ph1);
          *reinterpret_cast<uint32_t *>(Dh + r * kLdb + key) = pack2<T>(dh0, dh1);
          *reinterpret_cast<uint32_t *>(Dl + r * kLdb + key) = pack2<T>(ds[0] - dh0, ds[1] - dh1);
        } else {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            Ps[r * kLd + key + e] = p[e];
            Ds[r * kLd + key + e] = ds[e];
          }
        }
      }
    }
    if (!__syncthreads_or(any)) return;  // no allowed pair in this block: nothing to add
    if constexpr (kMma) {
      // B fragments of a row-major [k][n] tile (K, Q or dO) for n-tiles n0, n0 + 8
      auto ldb = [&](const T *tile, int k0r, int n0, uint32_t (&bf)[4]) {
        ldsm_x4_t(smem_u32(tile + (k0r + (lane & 7) + ((lane >> 3) & 1) * 8) * kLdb + n0 + (lane >> 4) * 8), bf[0],
                  bf[1], bf[2], bf[3]);
      };
      // dQ (rows 16 rg .., columns 32 kh ..) += (dS_hi + dS_lo) K
#pragma unroll
      for (int ks = 0; ks < kQTile / 16; ++ks) {
        uint32_t ah[4], al[4];
        const int arow = 16 * rg + (lane & 15), acol = 16 * ks + (lane >> 4) * 8;
        ldsm_x4(smem_u32(Dh + arow * kLdb + acol), ah[0], ah[1], ah[2], ah[3]);
        ldsm_x4(smem_u32(Dl + arow * kLdb + acol), al[0], al[1], al[2], al[3]);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bk[4];
          ldb(Kb, 16 * ks, 32 * kh + 16 * np, bk);
          mma16816<T>(gq[2 * np], ah, bk[0], bk[1]);
          mma16816<T>(gq[2 * np], al, bk[0], bk[1]);
          mma16816<T>(gq[2 * np + 1], ah, bk[2], bk[3]);
          mma16816<T>(gq[2 * np + 1], al, bk[2], bk[3]);
        }
      }
      // dK = dS^T Q and dV = P^T dO for keys 16 rg .., columns 32 kh ..
      float gk[4][4] = {}, gv[4][4] = {};
#pragma unroll
      for (int ks = 0; ks < kQTile / 16; ++ks) {
        uint32_t dh[4], dl[4], phf[4], plf[4];
        const int trow = 16 * ks + (lane & 7) + ((lane >> 4) << 3), tcol = 16 * rg + ((lane >> 3) & 1) * 8;
        ldsm_x4_t(smem_u32(Dh + trow * kLdb + tcol), dh[0], dh[1], dh[2], dh[3]);
        ldsm_x4_t(smem_u32(Dl + trow * kLdb + tcol), dl[0], dl[1], dl[2], dl[3]);
        ldsm_x4_t(smem_u32(Ph + trow * kLdb + tcol), phf[0], phf[1], phf[2], phf[3]);
        ldsm_x4_t(smem_u32(Pl + trow * kLdb + tcol), plf[0], plf[1], plf[2], plf[3]);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bq[4], bg[4];
          ldb(Qb, 16 * ks, 32 * kh + 16 * np, bq);
          ldb(Gb, 16 * ks, 32 * kh + 16 * np, bg);
          mma16816<T>(gk[2 * np], dh, bq[0], bq[1]);
          mma16816<T>(gk[2 * np], dl, bq[0], bq[1]);
          mma16816<T>(gk[2 * np + 1], dh, bq[2], bq[3]);
          mma16816<T>(gk[2 * np + 1], dl, bq[2], bq[3]);
          mma16816<T>(gv[2 * np], phf, bg[0], bg[1]);
          mma16816<T>(gv[2 * np], plf, bg[0], bg[1]);
          mma16816<T>(gv[2 * np + 1], phf, bg[2], bg[3]);
          mma16816<T>(gv[2 * np + 1], plf, bg[2], bg[3]);
        }
      }
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int64_t kt = k0 + 16 * rg + fg + 8 * hr;
        if (kt >= T_) continue;
        const int64_t base = ((static_cast<int64_t>(b) * Hkv + h) * T_ + kt) * kHeadDim + 32 * kh + 2 * fc;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          atomicAdd(reinterpret_cast<float2 *>(dk + base + 8 * nt),
                    make_float2(scale * gk[nt][2 * hr], scale * gk[nt][2 * hr + 1]));
          atomicAdd(reinterpret_cast<float2 *>(dv + base + 8 * nt), make_float2(gv[nt][2 * hr], gv[nt][2 * hr + 1]));
        }
      }
    } else {
      mm_ab16(Ds, Kb, ti, tj, gq);  // dQ += dS K
      float gk[4][4] = {}, gv[4][4] = {};
      mm_atb16(Ds, Qb, ti, tj, gk);  // dK = dS^T Q
      mm_atb16(Ps, Gb, ti, tj, gv);  // dV = P^T dO
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int64_t kt = k0 + ti + 16 * a;
        if (kt >= T_) continue;
        const int64_t base = ((static_cast<int64_t>(b) * Hkv + h) * T_ + kt) * kHeadDim;
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
          atomicAdd(dk + base + tj + 16 * bb, scale * gk[a][bb]);
          atomicAdd(dv + base + tj + 16 * bb, gv[a][bb]);
        }
      }
    }
  });
  if constexpr (kMma) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int64_t t = t0 + 16 * rg + fg + 8 * hr;
      if (t >= T_) continue;
      float *dst = dq + ((static_cast<int64_t>(b) * T_ + t) * Hq + hq) * kHeadDim + 32 * kh + 2 * fc;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
        *reinterpret_cast<float2 *>(dst + 8 * nt) = make_float2(scale * gq[nt][2 * hr], scale * gq[nt][2 * hr + 1]);
    }
  } else {
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int64_t t = t0 + ti + 16 * a;
      if (t >= T_) continue;
      float *dst = dq + ((static_cast<int64_t>(b) * T_ + t) * Hq + hq) * kHeadDim;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) dst[tj + 16 * bb] = scale * gq[a][bb];
    }
  }
}

}  // namespace bwd
}  // namespace sd

extern "C" int sd_prefill_attention_backward(const void *q, const void *k, const void *v, const void *dout,
                                             int dtype, int64_t B, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                                             int64_t q_sb, int64_t q_st, int64_t q_sh, int64_t c_sb, int64_t c_sh,
                                             int64_t c_st, int64_t g_sb, int64_t g_st, int64_t g_sh,
                                             const int32_t *lists, const int32_t *counts, int lcap,
                                             const int64_t *topk, int kk, int block_size, int causal, float scale,
                                             float *dq, float *dk, float *dv, void *stream) {
  if (!q || !k || !v || !dout || !lists || !counts || !dq || !dk || !dv || B <= 0 || T <= 0 || Hq <= 0 ||
      Hkv <= 0 || Hq % Hkv || lcap <= 0)
    return SD_ERR_INVALID;
  if (D != sd::kHeadDim || block_size != sd::kQTile) return SD_ERR_UNSUPPORTED;
  if (topk && kk <= 0) return SD_ERR_INVALID;
  const int64_t nqt = (T + sd::kQTile - 1) / sd::kQTile;
  if (nqt > 0x7fffffff || Hq > 65535 || B > 65535) return SD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t kv_bytes = static_cast<size_t>(B * Hkv * T * D) * sizeof(float);
  cudaError_t e = cudaMemsetAsync(dk, 0, kv_bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dv, 0, kv_bytes, s);
  if (e != cudaSuccess) {
    sd::set_cuda_error(e);
    return SD_ERR_CUDA;
  }
  const dim3 grid(static_cast<unsigned>(nqt), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  // 16-bit inputs with 16-byte aligned rows: S and dP on the tensor cores
  const bool rows16 = sd::aligned16(q) && sd::aligned16(k) && sd::aligned16(v) && sd::aligned16(dout) &&
                      q_sb % 8 == 0 && q_st % 8 == 0 && q_sh % 8 == 0 && c_sb % 8 == 0 && c_sh % 8 == 0 &&
                      c_st % 8 == 0 && g_sb % 8 == 0 && g_st % 8 == 0 && g_sh % 8 == 0;
  if (dtype != SD_DTYPE_F32 && rows16) {
    auto run = [&](auto kern, auto tag) {
      using E = decltype(tag);
      if (sd::set_max_smem(kern, sd::bwd::kSmemTcBytes) != SD_OK) return SD_ERR_CUDA;
      kern<<<grid, sd::bwd::kThreads, sd::bwd::kSmemTcBytes, s>>>(
          static_cast<const E *>(q), q_sb, q_st, q_sh, static_cast<const E *>(k), static_cast<const E *>(v), c_sb,
          c_sh, c_st, static_cast<const E *>(dout), g_sb, g_st, g_sh, T, static_cast<int>(Hq), static_cast<int>(Hkv),
          lists, counts, lcap, topk, kk, causal, scale, dq, dk, dv);
      return sd::check_launch();
    };
    if (dtype == SD_DTYPE_BF16) return run(sd::bwd::prefill_bwd_tc_kernel<__nv_bfloat16, true>, __nv_bfloat16());
    if (dtype == SD_DTYPE_F16) return run(sd::bwd::prefill_bwd_tc_kernel<__half, false>, __half());
  }
  SD_DISPATCH_DTYPE(dtype, E, {
    auto kern = sd::bwd::prefill_bwd_kernel<E>;
    if (sd::set_max_smem(kern, sd::bwd::kSmemBytes) != SD_OK) return SD_ERR_CUDA;
    kern<<<grid, sd::bwd::kThreads, sd::bwd::kSmemBytes, s>>>(
        static_cast<const E *>(q), q_sb, q_st, q_sh, static_cast<const E *>(k), static_cast<const E *>(v), c_sb,
        c_sh, c_st, static_cast<const E *>(dout), g_sb, g_st, g_sh, T, static_cast<int>(Hq), static_cast<int>(Hkv),
        lists, counts, lcap, topk, kk, causal, scale, dq, dk, dv);
    return sd::check_launch();
  });
  return SD_OK;
}
