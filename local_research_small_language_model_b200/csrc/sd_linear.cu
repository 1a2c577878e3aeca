// Projections of the decode step on the 5th-generation tensor cores: the
// q|k|v|forecast projection with the attention RMSNorm in front
// (model/transformer.py:104-107, model/forecast.py:23-27, model/norm.py:15-21),
// the output projection and the FFN down projection with the residual add
// behind (transformer.py:118-129), the [w_gate; w_up] projection with the FFN
// RMSNorm in front and the SwiGLU gate behind (transformer.py:18-31), and the
// tied LM head after the final norm.
//
// out[m, n] = epilogue(sum_k X[m, k] W[n, k]) with few rows m (the decode
// batch) and many n, so the product runs transposed ("swap AB"): one CTA owns
// 128 weight rows n0..n0+127 as the MMA's M dimension and a 64-row tile of X
// as its N dimension.  Per 64-wide K chunk:
//   W tile  [128 x 64] 16-bit, TMA (128-byte swizzle) into a ring sized so
//           that, where shared memory allows, every chunk of the CTA is in
//           flight at once (the weights are the bytes that bound the call),
//   X tile  [64 x 64] by TMA: with the RMSNorm prologue every chunk of the
//           CTA stays resident and is normalised in place; otherwise one
//           chunk beside each W stage,
//   tcgen05.mma kind::f16 M=128 N=64 K=16 x 4, fp32 accumulator in TMEM.
// The weight and gain copies are issued before the wait on the preceding
// kernel (they do not depend on it).  Lane 0 of warp 0 issues the MMAs; a
// stage is refilled once the MMAs that read it have completed
// (tcgen05.commit on the stage's barrier).
//
// Small grids split K over a cluster of S = 2, 4 or 8 CTAs per output tile
// (cluster dims 1 x S x 1).  The CTAs exchange through distributed shared
// memory instead of global memory, with st.async remote stores whose bytes
// are counted on the receiver's mbarrier: the RMSNorm's per-row sums of
// squares (each CTA sums its own K chunks and sends the sums to every peer;
// each CTA adds the S partials in rank order), and the fp32 partial products
// (CTA r owns 1/S of the tile; every CTA sends it those rows of its
// accumulator, and CTA r adds the S partials in rank order and runs the
// epilogue for them).  No workspace, no atomics; the result depends only on
// the shapes.  Every mbarrier wait is bounded and reports through the error
// word.
#include <type_traits>

#include "sd_tma.cuh"

namespace sd {

namespace lin {

constexpr int kThreads = 256;
constexpr int kRowsW = 128;             // weight rows per CTA (MMA M)
constexpr int kRowsX = 64;              // batch rows per CTA (MMA N)
constexpr int kMaxStages = 8;
constexpr int kWBytes = kRowsW * 128;   // 128 rows x 64 16-bit values
constexpr int kXBytes = kRowsX * 128;   // 64 rows x 64 16-bit values
constexpr int kTmemCols = 64;
constexpr int kMaxNormK = 1024;         // the RMSNorm prologue keeps every K chunk of X in shared memory
constexpr int kMaxSplits = 8;
constexpr int kRedStride = 68;          // fp32 words per staged accumulator row (64 + 4: no bank conflicts)
constexpr int kRedBytes = kRowsW * kRedStride * 4;
constexpr int kSmemBudget = 220 * 1024;

enum Epi { kStore = 0, kResidual = 1, kSwiGLU = 2 };

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  // K-major, 128-byte swizzle: LBO 16 bytes, SBO 1024 bytes (8 rows of 128 B),
  // descriptor version 1, layout code 2
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(16 >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulator, A and B of format fmt
// (0 = f16, 1 = bf16), both K-major, N = 64, M = 128.
__host__ __device__ constexpr uint32_t idesc(uint32_t fmt) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(acc ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared memory: the W ring (nst stages), then X (norm: the CTA's cps
// chunks; else an nst-stage ring) -- once every MMA is done this tile region,
// padded to kRedBytes, holds the CTA's fp32 product staged by owner -- then
// (split) the partial products the peers send, the gain chunks, (residual)
// the residual tile and the barriers.  Tile buffers 1024-aligned.
constexpr int kResBytes = kRowsX * kRowsW * 2;
struct Smem {
  __host__ __device__ static size_t x_off(int nst) { return static_cast<size_t>(nst) * kWBytes; }
  __host__ __device__ static size_t recv_off(bool norm, int cps, int nst, int nsplit) {
    const size_t e = x_off(nst) + static_cast<size_t>(norm ? cps : nst) * kXBytes;
    (void)nsplit;
    return e < static_cast<size_t>(kRedBytes) ? static_cast<size_t>(kRedBytes) : e;
  }
  __host__ __device__ static size_t gain_off(bool norm, int cps, int nst, int nsplit) {
    return recv_off(norm, cps, nst, nsplit) + (nsplit > 1 ? kRedBytes : 0);
  }
  static constexpr int kGainBytes = kMaxNormK * 2;
  __host__ __device__ static size_t res_off(bool norm, int cps, int nst, int nsplit) {
    return gain_off(norm, cps, nst, nsplit) + kGainBytes;
  }
  __host__ __device__ static size_t bar_off(bool norm, int cps, int nst, int nsplit, bool resid) {
    return res_off(norm, cps, nst, nsplit) + (resid ? kResBytes : 0);
  }
  __host__ __device__ static size_t bytes(bool norm, int cps, int nst, int nsplit, bool resid) {
    return bar_off(norm, cps, nst, nsplit, resid) + 512;
  }
};

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(const void *p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Asynchronous remote shared-memory store that counts its bytes on the
// receiving CTA's mbarrier (`bar` is that barrier's cluster address).
__device__ __forceinline__ void st_async_f32(uint32_t a, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(a), "f"(v), "r"(bar)
               : "memory");
}

template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  using type = __nv_bfloat162;
  __device__ __forceinline__ static type pack(float a, float b) { return __floats2bfloat162_rn(a, b); }
  __device__ __forceinline__ static float2 unpack(type v) { return __bfloat1622float2(v); }
};
template <> struct Pair<__half> {
  using type = __half2;
  __device__ __forceinline__ static type pack(float a, float b) { return __floats2half2_rn(a, b); }
  __device__ __forceinline__ static float2 unpack(type v) { return __half22float2(v); }
};

// Bulk copy of `bytes` from this CTA's shared memory into a peer's (cluster
// addresses dst and bar), counted on the peer's mbarrier.
__device__ __forceinline__ void bulk_s2peer(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(bar)
               : "memory");
}

template <typename T> __device__ __forceinline__ T silu_rounded(float g) {
  return from_f<T>(g / (1.0f + expf(-g)));
}

template <typename T, int kEpi, bool kNorm>
__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const T *__restrict__ gain, float eps, const __grid_constant__ CUtensorMap tmw,
                     const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmr, int M,
                     int K, int cps, int nst, T *out, int64_t o_rs, int32_t *err) {
  extern __shared__ __align__(1024) char smem_raw[];
  char *sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int nsplit = gridDim.y;  // the cluster size
  const int rank = blockIdx.y;   // rank in the cluster (cluster dims 1 x nsplit x 1)
  constexpr bool kRes = kEpi == kResidual;
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + Smem::bar_off(kNorm, cps, nst, nsplit, kRes));  // [kMaxStages]
  uint64_t *empty = full + kMaxStages;  // [kMaxStages] MMAs done with a stage
  uint64_t *done = empty + kMaxStages;  // every MMA done
  uint64_t *xbar = done + 1;            // the X chunks and the gain landed (RMSNorm prologue)
  uint64_t *ssbar = xbar + 1;           // the peers' sums of squares landed
  uint64_t *redbar = ssbar + 1;         // the peers' partial products landed
  uint64_t *resbar = redbar + 1;        // the residual tile landed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(resbar + 1);
  __shared__ float s_ss[kMaxSplits][kRowsX];  // per-row sums of squares of each CTA of the cluster
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kRowsW;
  // this CTA's K chunks c0 .. c0 + nc - 1 (nc <= cps, the count the shared
  // memory layout is sized for)
  const int nk = K / 64;
  const int c0 = rank * nk / nsplit;
  const int nc = (rank + 1) * nk / nsplit - c0;
  const int m0 = blockIdx.z * kRowsX;
  const int mrows = M - m0 < kRowsX ? M - m0 : kRowsX;
  // Output ownership: CTA `rank` of the cluster (the only one when unsplit)
  // owns weight rows rank * R .. + R - 1 (store / residual, R = 128/S) or
  // gate rows rank * R .. + R - 1 with their up rows 64 + ... (SwiGLU,
  // R = 64/S); thread t takes row t % R and cpt = R/4 batch columns from
  // (t / R) * cpt.
  const int R = (kEpi == kSwiGLU ? 64 : kRowsW) / nsplit;
  const int cpt = R / 4;
  const int rl = tid % R;
  const int b0 = (tid / R) * cpt;
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kTxStage = kNorm ? kWBytes : kWBytes + kXBytes;
  char *xs = sm + Smem::x_off(nst);
  T *gs = reinterpret_cast<T *>(sm + Smem::gain_off(kNorm, cps, nst, nsplit));  // gain of this CTA's chunks
  T *rs = reinterpret_cast<T *>(sm + Smem::res_off(kNorm, cps, nst, nsplit));  // residual tile [64][R]
  const int rows_per = kRowsW / nsplit;  // partial-product rows each owner receives from each CTA

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(xbar, 1);
    mbar_init(ssbar, 1);
    mbar_init(redbar, 1);
    mbar_init(resbar, 1);
    if (nsplit > 1) {
      // the bytes the S - 1 peers send this CTA (st.async complete_tx)
      if (kNorm) mbar_arrive_expect_tx(ssbar, static_cast<uint32_t>(nsplit - 1) * kRowsX * 4);
      mbar_arrive_expect_tx(redbar, static_cast<uint32_t>(nsplit - 1) * rows_per * kRedStride * 4);
    }
    mbar_init_fence();
  }
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  // a CTA writes into a peer's shared memory only after the whole cluster
  // has started (and initialised its barriers): this arrive pairs with a
  // wait before the first such write
  if (nsplit > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  // Weights and gain do not depend on the kernel ahead on the stream: they
  // are requested before waiting for it; X and the residual are read after
  // the wait.  Lane 0 of warp 0 issues every copy and MMA; the other lanes of
  // warp 0 follow it in lockstep (__syncwarp).
  auto issue_w = [&](int lc) {  // W of local chunk lc into stage lc % nst
    const int s = lc % nst;
    mbar_arrive_expect_tx(&full[s], kTxStage);
    tma_load_2d(sm + s * kWBytes, &tmw, 64 * (c0 + lc), n0, &full[s]);
  };
  if (tid == 0) {
    if (kNorm) {
      mbar_arrive_expect_tx(xbar, static_cast<uint32_t>(nc) * (kXBytes + 128));
      bulk_g2s(gs, gain + 64 * c0, static_cast<uint32_t>(nc) * 128, xbar);
    }
    for (int lc = 0; lc < nc && lc < nst; ++lc) issue_w(lc);
  }
  pdl_wait();
  if (tid == 0) {
    if (kNorm) {
      for (int lc = 0; lc < nc; ++lc) tma_load_2d(xs + lc * kXBytes, &tmx, 64 * (c0 + lc), m0, xbar);
    } else {
      for (int lc = 0; lc < nc && lc < nst; ++lc) tma_load_2d(xs + lc * kXBytes, &tmx, 64 * (c0 + lc), m0, &full[lc]);
    }
    if (kRes) {
      // the residual of the rows this CTA owns, [64 batch rows][R columns]:
      // its latency hides behind the MMAs (out may alias res: the whole tile
      // is in shared memory before this CTA stores anything)
      mbar_arrive_expect_tx(resbar, static_cast<uint32_t>(R) * kRowsX * 2);
      tma_load_2d(rs, &tmr, n0 + rank * R, m0, resbar);
    }
  }
  __syncwarp();

  if (kNorm) {
    // RMSNorm of rows m0..m0+63 (model/norm.py:15-21): fp32 mean of squares
    // over the whole row, x * rsqrt(mean + eps) rounded to T, times the gain
    // rounded to T.  Thread t handles row t / 4, 16-byte groups t % 4,
    // t % 4 + 4, ... of this CTA's chunks (rows past M arrive as zeros).  Each
    // CTA sums the squares of its own chunks and sends the sums to its peers
    // (st.async into their s_ss[rank]); every CTA adds the S partials in rank
    // order.
    const bool xok = mbar_wait_bounded(xbar, 0);
    if (!xok && err && tid == 0) atomicExch(err, SD_KERR_TIMEOUT);
    const int r = tid >> 2, sub = tid & 3;
    const int ng = nc * 8;
    float ss = 0.f;
#pragma unroll 4
    for (int q = sub; q < ng; q += 4) {
      const uint4 u = *reinterpret_cast<const uint4 *>(xs + (q >> 3) * kXBytes + sw128(r, q & 7));
      const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v = to_f(e[i]);
        ss = fmaf(v, v, ss);
      }
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    if (nsplit > 1) {
      asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // the cluster has started
      if (sub == 0) s_ss[rank][r] = ss;
      for (int q = sub; q < nsplit; q += 4)
        if (q != rank) st_async_f32(peer_addr(&s_ss[rank][r], q), ss, peer_addr(ssbar, q));
      __syncthreads();
      const bool sok = mbar_wait_bounded(ssbar, 0);
      if (!sok && err && sub == 0) atomicExch(err, SD_KERR_TIMEOUT);
      float tot = 0.f;
      for (int q = 0; q < nsplit; ++q) tot += s_ss[q][r];
      ss = tot;
    }
    const float rr = rsqrtf(ss / static_cast<float>(K) + eps);
    // pairs of values: the normalised pair rounded to T by one paired
    // conversion, then times the gain pair by a paired T multiply (the exact
    // product of two T values is an fp32 number, so its single rounding
    // equals the reference's fp32 multiply rounded to T)
    using T2 = typename Pair<T>::type;
#pragma unroll 4
    for (int q = sub; q < ng; q += 4) {
      uint4 *p = reinterpret_cast<uint4 *>(xs + (q >> 3) * kXBytes + sw128(r, q & 7));
      const uint4 u = *p;
      const uint4 g = *reinterpret_cast<const uint4 *>(gs + 8 * q);
      const T2 *ev = reinterpret_cast<const T2 *>(&u);
      const T2 *ge = reinterpret_cast<const T2 *>(&g);
      uint4 o;
      T2 *oe = reinterpret_cast<T2 *>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = Pair<T>::unpack(ev[i]);
        oe[i] = __hmul2(Pair<T>::pack(f.x * rr, f.y * rr), ge[i]);
      }
      *p = o;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
  } else if (nsplit > 1) {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // the cluster has started
  }

  // ---- MMAs: local chunk lc reads stage lc % nst; when the ring is shorter
  // than the chunk count, the stage of chunk lc - 1 is refilled with chunk
  // lc - 1 + nst once its MMAs are done
  bool ok = true;
  if (warp == 0) {
    const uint32_t id = idesc(fmt);
    for (int lc = 0; lc < nc; ++lc) {
      const int s = lc % nst;
      ok = mbar_wait_bounded(&full[s], (lc / nst) & 1) && ok;
      fence_after();
      if (lane == 0) {
        const uint32_t wa = smem_u32(sm + s * kWBytes);
        const uint32_t xa = smem_u32(xs + (kNorm ? lc : s) * kXBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma(tmem, desc_sw128(wa + 32 * kk), desc_sw128(xa + 32 * kk), id, lc > 0 || kk > 0);
        commit(&empty[s]);
      }
      __syncwarp();
      const int pc = lc - 1;
      if (pc >= 0 && pc + nst < nc) {
        const int ps = pc % nst;
        ok = mbar_wait_bounded(&empty[ps], (pc / nst) & 1) && ok;
        if (lane == 0) {
          issue_w(pc + nst);
          if (!kNorm) tma_load_2d(xs + ps * kXBytes, &tmx, 64 * (c0 + pc + nst), m0, &full[ps]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) commit(done);
    __syncwarp();
  }
  ok = mbar_wait_bounded(done, 0) && ok;
  fence_after();

  // ---- this CTA's product: thread t reads TMEM lane t % 128 (weight row
  // n0 + t % 128) and batch columns 32 * (t / 128) .. +31, and stages it in
  // shared memory by owner: [S][rows_per][kRedStride] over the tile region,
  // which every finished MMA (and so every copy it read) has released
  const int row = tid & (kRowsW - 1), half = tid >> 7;
  float *stage = reinterpret_cast<float *>(sm);
  {
    int owner, j;
    if (kEpi == kSwiGLU) {
      const int g = row & 63;
      owner = g / R;
      j = g % R + (row >= 64 ? R : 0);
    } else {
      owner = row / R;
      j = row % R;
    }
    float *slot = stage + (owner * rows_per + j) * kRedStride + 32 * half;
    const uint32_t taddr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + 32 * half;
#pragma unroll 1
    for (int c = 0; c < 32; c += 16) {
      float v[16];
      tmem_ld16(taddr + c, v);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<float4 *>(slot + c + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  float *recv = reinterpret_cast<float *>(sm + Smem::recv_off(kNorm, cps, nst, nsplit));  // the peers' partials
  if (nsplit > 1) {
    // thread q sends peer q the rows it owns (one bulk copy into the peer's
    // slot for this rank, counted on its redbar); each owner adds the S
    // partials in rank order
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid < nsplit && tid != rank)
      bulk_s2peer(peer_addr(recv + rank * rows_per * kRedStride, tid), stage + tid * rows_per * kRedStride,
                  static_cast<uint32_t>(rows_per) * kRedStride * 4, peer_addr(redbar, tid));
    ok = mbar_wait_bounded(redbar, 0) && ok;
    // every CTA arrives once its peers' rows have landed; the matching wait
    // before exit keeps each CTA's staged rows (the source of its copies)
    // alive until every peer holds them.  It publishes no data: relaxed.
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  } else {
    __syncthreads();
  }
  if (kRes) ok = mbar_wait_bounded(resbar, 0) && ok;

  // ---- epilogue: row rank * R + rl, batch columns b0 .. b0 + cpt - 1, in
  // groups of 4
  const int col = kEpi == kSwiGLU ? blockIdx.x * 64 + rank * R + rl : n0 + rank * R + rl;
#pragma unroll 1
  for (int g = 0; g < cpt; g += 4) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), u = a;
#pragma unroll 1
    for (int q = 0; q < nsplit; ++q) {
      const float *src = (q == rank ? stage : recv) + (q * rows_per + rl) * kRedStride + b0 + g;
      const float4 p = *reinterpret_cast<const float4 *>(src);
      a.x += p.x;
      a.y += p.y;
      a.z += p.z;
      a.w += p.w;
      if (kEpi == kSwiGLU) {
        const float4 w = *reinterpret_cast<const float4 *>(src + R * kRedStride);
        u.x += w.x;
        u.y += w.y;
        u.z += w.z;
        u.w += w.w;
      }
    }
    const float av[4] = {a.x, a.y, a.z, a.w}, uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int b = b0 + g + i;
      if (b < mrows) {
        T o;
        if (kEpi == kSwiGLU) {
          // silu(gate) and the product each rounded to T (transformer.py:30-31)
          const float sg = to_f(silu_rounded<T>(round_to<T>(av[i])));
          o = from_f<T>(sg * round_to<T>(uv[i]));
        } else if (kEpi == kResidual) {
          // x + Linear(h): the projection rounded to T, then the sum
          o = from_f<T>(to_f(rs[b * R + rl]) + round_to<T>(av[i]));
        } else {
          o = from_f<T>(av[i]);
        }
        out[static_cast<int64_t>(m0 + b) * o_rs + col] = o;
      }
    }
  }
  if (nsplit > 1) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  if (!ok && err && tid == 0) atomicExch(err, SD_KERR_TIMEOUT);
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace lin

// K splits (cluster size) for an (M, K, N) projection: the largest of 8, 4
// and 2 (4 and 2 for SwiGLU, whose owners split 64 gate rows) that keeps the
// grid within one wave of the SMs and gives every CTA a K chunk; 1 when the
// output tiles alone fill half the SMs.
static int linear_splits(int64_t M, int64_t K, int64_t N, bool swiglu) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) ==
                                                   cudaSuccess && v > 0)
      sms = v;
    else
      sms = 148;
  }
  const int64_t tiles = (N / lin::kRowsW) * ((M + lin::kRowsX - 1) / lin::kRowsX);
  const int64_t nk = K / 64;
  if (2 * tiles >= sms) return 1;
  for (int s = swiglu ? 4 : lin::kMaxSplits; s >= 2; s /= 2)
    if (s <= nk && tiles * s <= sms) return s;
  return 1;
}

// W stages that fit beside X and the exchange buffers: every chunk of the
// CTA in flight when possible.
static int linear_stages(bool norm, int cps, int nsplit, bool resid) {
  int st = cps < lin::kMaxStages ? cps : lin::kMaxStages;
  while (st > 1 && lin::Smem::bytes(norm, cps, st, nsplit, resid) + 1024 > static_cast<size_t>(lin::kSmemBudget)) --st;
  return st;
}

template <typename T, int kEpi, bool kNorm>
static int launch_linear(const void *x, int64_t M, int64_t K, int64_t x_rs, const void *w, int64_t N,
                         const void *gain, float eps, const void *res, int64_t r_rs, void *out, int64_t o_rs,
                         int32_t *err, cudaStream_t s) {
  using namespace lin;
  const int dt = std::is_same<T, __nv_bfloat16>::value ? SD_DTYPE_BF16 : SD_DTYPE_F16;
  const int splits = linear_splits(M, K, N, kEpi == kSwiGLU);
  CUtensorMap mw, mx, mr;
  memset(&mr, 0, sizeof(mr));
  // W [N, K] in boxes of 128 rows x 64 columns; X [M, K] in boxes of 64 x 64
  // (rows past M read as zeros); the residual [M, N] in boxes of 64 rows x
  // the columns one CTA owns
  int r = encode_matrix_map(&mw, w, dt, N, K, K, kRowsW);
  if (r != SD_OK) return r;
  r = encode_matrix_map(&mx, x, dt, M, K, x_rs, kRowsX);
  if (r != SD_OK) return r;
  if (kEpi == kResidual) {
    r = encode_plain_map(&mr, res, dt, M, N, r_rs, kRowsW / splits, kRowsX);
    if (r != SD_OK) return r;
  }
  const int64_t mt = (M + kRowsX - 1) / kRowsX;
  const int cps = static_cast<int>((K / 64 + splits - 1) / splits);  // chunks of the largest CTA
  const int nst = linear_stages(kNorm, cps, splits, kEpi == kResidual);
  const size_t smem = Smem::bytes(kNorm, cps, nst, splits, kEpi == kResidual) + 1024;
  if (smem > static_cast<size_t>(kSmemBudget)) return SD_ERR_UNSUPPORTED;
  auto kern = linear_tc_kernel<T, kEpi, kNorm>;
  if (set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
  const dim3 grid(static_cast<unsigned>(N / kRowsW), static_cast<unsigned>(splits), static_cast<unsigned>(mt));
  return launch_cluster(kern, grid, dim3(kThreads), dim3(1, static_cast<unsigned>(splits), 1), smem, s,
                        pdl_enabled(), static_cast<const T *>(gain), eps, mw, mx, mr, static_cast<int>(M),
                        static_cast<int>(K), cps, nst, static_cast<T *>(out), o_rs, err);
}

}  // namespace sd

extern "C" int sd_linear(const void *x, int dtype, int64_t M, int64_t K, int64_t x_rs, const void *w, int64_t N,
                         const void *norm_w, float eps, int epilogue, const void *res, int64_t r_rs, void *out,
                         int64_t o_rs, int32_t *err, void *stream) {
  if (!x || !w || !out || M <= 0 || K <= 0 || N <= 0) return SD_ERR_INVALID;
  if (epilogue != SD_LINEAR_STORE && epilogue != SD_LINEAR_RESIDUAL && epilogue != SD_LINEAR_SWIGLU)
    return SD_ERR_INVALID;
  if (epilogue == SD_LINEAR_RESIDUAL && !res) return SD_ERR_INVALID;
  if (dtype != SD_DTYPE_BF16 && dtype != SD_DTYPE_F16) return SD_ERR_UNSUPPORTED;
  if (K % 64 || N % sd::lin::kRowsW || M > 0x7fffffff || N > 0x7fffffff || N / sd::lin::kRowsW > 0x7fffffff ||
      (M + 63) / 64 > 65535)
    return SD_ERR_UNSUPPORTED;
  if (norm_w && K > sd::lin::kMaxNormK) return SD_ERR_UNSUPPORTED;
  if (!sd::aligned16(x) || !sd::aligned16(w) || !sd::aligned16(out) || x_rs % 8 || (norm_w && !sd::aligned16(norm_w)) ||
      (res && (!sd::aligned16(res) || r_rs % 8)))
    return SD_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool norm = norm_w != nullptr;
#define SD_LIN(E, EPI)                                                                                           \
  return norm ? sd::launch_linear<E, EPI, true>(x, M, K, x_rs, w, N, norm_w, eps, res, r_rs, out, o_rs, err, s) \
              : sd::launch_linear<E, EPI, false>(x, M, K, x_rs, w, N, norm_w, eps, res, r_rs, out, o_rs, err, s)
  if (dtype == SD_DTYPE_BF16) {
    using E = __nv_bfloat16;
    if (epilogue == SD_LINEAR_STORE) SD_LIN(E, sd::lin::kStore);
    if (epilogue == SD_LINEAR_RESIDUAL) SD_LIN(E, sd::lin::kResidual);
    SD_LIN(E, sd::lin::kSwiGLU);
  } else {
    using E = __half;
    if (epilogue == SD_LINEAR_STORE) SD_LIN(E, sd::lin::kStore);
    if (epilogue == SD_LINEAR_RESIDUAL) SD_LIN(E, sd::lin::kResidual);
    SD_LIN(E, sd::lin::kSwiGLU);
  }
#undef SD_LIN
}
