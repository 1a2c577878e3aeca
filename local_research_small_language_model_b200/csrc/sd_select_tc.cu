// Many-row forecast block selector on the 5th-generation tensor cores
// (ForecastBlockSelector.forward, model/forecast.py:89-130, for prefill: one
// forecast row per query token, D = 64, top-k <= 8, bf16 forecast, no score
// tensor).
//
// Scores are fp32 dot products of a bf16 forecast row with an fp32 prototype.
// The tensor cores take 16-bit operands, so every prototype is split into
// three bf16 parts, p = hi + mid + lo (hi = bf16(p), mid = bf16(p - hi),
// lo = bf16(p - hi - mid): 24 significant bits, the whole fp32 mantissa), and
// the score is f.hi + f.mid + f.lo accumulated in fp32 by the MMA: each
// product of two bf16 values is exact in fp32, so the result differs from an
// fp32 CUDA-core dot product only by accumulation rounding.
//
// One CTA per (256 query rows, kv head, sequence), 256 threads:
//   * the forecast tile [256 rows x 64] arrives by TMA (128-byte swizzle);
//   * per chunk of 128 prototypes (blocks the tile's last row cannot see are
//     never loaded): the threads split the fp32 prototypes into the three bf16
//     planes, written in the same swizzled K-major layout;
//   * one thread issues, for each of the two 128-row halves, 3 planes x 4
//     K-steps of tcgen05.mma kind::f16 (M=128 rows, N=128 blocks, K=16) into
//     two 128-column fp32 accumulators in TMEM (the split planes serve 256
//     rows);
//   * thread t reads the 128 scores of row t (TMEM lane t % 128, columns
//     128 * (t / 128) ..) up to the warp's last visible block, with the causal
//     mask applied, maps them to ordered 32-bit keys (order-preserving score
//     bits) and keeps the row's top-8 (key, block) pairs in registers; a
//     batch's keys are staged in shared memory and the warp inserts the
//     candidates that beat the list's 8th key in rounds, one per lane per
//     round, in ascending block order, so a strict comparison leaves equal
//     scores in ascending index order;
//   * blocks past the row's last visible one follow as -inf entries in index
//     order (the reference's topk over -inf scores), and the k best indices
//     are written.
// The order is (value desc, index asc) everywhere; NaN scores are never
// chosen.  Every mbarrier wait is bounded.
#include "sd_select_core.cuh"
#include "sd_tma.cuh"

namespace sd {
namespace seltc {

constexpr int kThreads = 256;
constexpr int kRows = 256;    // forecast rows per CTA (two MMA M tiles of 128)
constexpr int kBlk = 128;     // prototypes per chunk (MMA N)
constexpr int kABytes = kRows * 128;
constexpr int kPlaneBytes = kBlk * 128;
constexpr int kTmemCols = 256;

// Shared memory: A [256][64] bf16 | hi | mid | lo planes [128][64] bf16 (once
// a chunk's MMAs are done, the planes hold the threads' staged keys) |
// barriers.  1024-aligned tiles.
constexpr int kPlaneOff = kABytes;
constexpr int kBarOff = kPlaneOff + 3 * kPlaneBytes;
constexpr int kSmemBytes = kBarOff + 64;
static_assert(16 * kThreads * 4 <= 3 * kPlaneBytes, "the staged keys fit over the planes");

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  // K-major, 128-byte swizzle: LBO 16 bytes, SBO 1024 bytes (8 rows of 128 B),
  // descriptor version 1, layout code 2
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(16 >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulator, bf16 A and B, both
// K-major, N = 128, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t a, uint64_t b, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc ? 1u : 0u)
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
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Ordered 32-bit key of a score: larger key = larger score (the float's bits
// mapped to an order-preserving unsigned integer).  0 is below every non-NaN
// score's key (an empty slot); NaN is never keyed.
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return u ^ (static_cast<uint32_t>(static_cast<int32_t>(u) >> 31) | 0x80000000u);
}
constexpr uint32_t kKeyNegInf = 0x007fffffu;  // order_key(-inf)

// Sorted insertion of (x, xi) into an 8-entry list, best first; x = 0 (or
// any key not above kv[7]) leaves the list unchanged.  A key equal to an
// entry goes after it.  Branch-free.
__device__ __forceinline__ void insert_key(uint32_t (&kv)[8], int (&ki)[8], uint32_t x, int xi) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool b = x > kv[i];
    const uint32_t tv = b ? kv[i] : x;
    const int ti = b ? ki[i] : xi;
    kv[i] = b ? x : kv[i];
    ki[i] = b ? xi : ki[i];
    x = tv;
    xi = ti;
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

__global__ void __launch_bounds__(kThreads, 2)
    select_rows_tc_kernel(const __grid_constant__ CUtensorMap tmf, int64_t Tq, int H, const float *__restrict__ reps,
                          int64_t NB, int64_t r_sb, int64_t r_sn, int64_t r_sh, int k, int bs, int causal,
                          int64_t q_offset, float scale, int64_t *__restrict__ idx_out, int32_t *err) {
  extern __shared__ __align__(1024) char smem_raw[];
  char *sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t *abar = reinterpret_cast<uint64_t *>(sm + kBarOff);  // forecast tile landed
  uint64_t *dbar = abar + 1;                                     // a chunk's MMAs done
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(dbar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.z, h = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    mbar_init(abar, 1);
    mbar_init(dbar, 1);
    mbar_init_fence();
  }
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    mbar_arrive_expect_tx(abar, kABytes);
    tma_load_4d(sm, &tmf, 0, static_cast<int>(row0), h, b, abar);
  }

  // blocks any row of the tile may see (causal: up to the last row's block)
  int64_t jmax = NB;
  if (causal) {
    const int64_t last_row = Tq - row0 < kRows ? Tq - 1 : row0 + kRows - 1;
    const int64_t t = last_row + q_offset;
    jmax = t < 0 ? 0 : (t / bs + 1 < NB ? t / bs + 1 : NB);
  }
  // this thread's row and its last visible block (inclusive; -1: none)
  const int lr = tid, half = tid >> 7;  // row; its 128-row MMA tile
  const int64_t t_abs = row0 + lr + q_offset;
  int64_t jvis = NB - 1;
  if (causal) jvis = t_abs < 0 ? -1 : (t_abs / bs < NB - 1 ? t_abs / bs : NB - 1);

  // the warp's last visible block: its scan stops there
  const int wjvis = __reduce_max_sync(0xffffffffu, static_cast<int>(jvis));

  // this thread's running top-8 of its row: ordered keys (0: empty), blocks
  uint32_t kv[8];
  int ki[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    kv[i] = 0;
    ki[i] = -1;
  }
  // per-thread staging of a batch's 16 keys, [16][256] over the planes
  // (free while the scores are read)
  uint32_t *kst = reinterpret_cast<uint32_t *>(sm + kPlaneOff);
  const float *rbase = reps + b * r_sb + h * r_sh;
  bool ok = true;
  int c = 0;
  for (int64_t j0 = 0; j0 < jmax; j0 += kBlk, ++c) {
    // ---- split prototypes j0 .. j0+127 into the hi / mid / lo planes:
    // item e = (block n, 16-byte group q of 8 values)
    for (int e = tid; e < kBlk * 8; e += kThreads) {
      const int n = e >> 3, q = e & 7;
      float x[8];
      if (j0 + n < jmax) {
        const float4 u = *reinterpret_cast<const float4 *>(rbase + (j0 + n) * r_sn + 8 * q);
        const float4 w = *reinterpret_cast<const float4 *>(rbase + (j0 + n) * r_sn + 8 * q + 4);
        x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
        x[4] = w.x; x[5] = w.y; x[6] = w.z; x[7] = w.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = 0.f;
      }
      uint4 ph, pm, pl;
      uint32_t *hw = &ph.x, *mw = &pm.x, *lw = &pl.x;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a0 = x[2 * i], a1 = x[2 * i + 1];
        const __nv_bfloat16 h0 = __float2bfloat16_rn(a0), h1 = __float2bfloat16_rn(a1);
        const float r0 = a0 - __bfloat162float(h0), r1 = a1 - __bfloat162float(h1);  // exact
        const __nv_bfloat16 m0 = __float2bfloat16_rn(r0), m1 = __float2bfloat16_rn(r1);
        const float s0 = r0 - __bfloat162float(m0), s1 = r1 - __bfloat162float(m1);  // exact
        __nv_bfloat162 hh(h0, h1), mm(m0, m1);
        hw[i] = *reinterpret_cast<uint32_t *>(&hh);
        mw[i] = *reinterpret_cast<uint32_t *>(&mm);
        lw[i] = pack_bf16(s0, s1);
      }
      const uint32_t off = sw128(n, q);
      *reinterpret_cast<uint4 *>(sm + kPlaneOff + off) = ph;
      *reinterpret_cast<uint4 *>(sm + kPlaneOff + kPlaneBytes + off) = pm;
      *reinterpret_cast<uint4 *>(sm + kPlaneOff + 2 * kPlaneBytes + off) = pl;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    fence_before();
    __syncthreads();
    fence_after();
    // warp 0 as a whole waits for the forecast tile; its lane 0 issues the
    // MMAs while the other lanes wait at __syncwarp (not on a barrier poll,
    // which would share the warp's issue slots with lane 0's work)
    if (warp == 0) {
      if (c == 0) ok = mbar_wait_bounded(abar, 0) && ok;
      if (tid == 0) {
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const uint32_t a = smem_u32(sm + m * (kABytes / 2));
          int step = 0;
#pragma unroll
          for (int p = 0; p < 3; ++p) {
            const uint32_t bp = smem_u32(sm + kPlaneOff + p * kPlaneBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk, ++step)
              mma(tmem + 128 * m, desc_sw128(a + 32 * kk), desc_sw128(bp + 32 * kk), step > 0);
          }
        }
        commit(dbar);
      }
      __syncwarp();
    }
    ok = mbar_wait_bounded(dbar, c & 1) && ok;
    fence_after();
    // ---- this thread's scores of its row (TMEM lane t % 128, columns
    // 128 * (t / 128) ..) in batches of 16, up to the warp's last visible
    // block: the batch's keys go to shared memory, the ones above the list's
    // 8th key are candidates, and the warp loops until every lane has
    // inserted its candidates (one per lane per round, lowest block first,
    // branch-free), so a rare insertion costs one round, not one per value
    const int jc = static_cast<int>(j0);  // first block of the chunk
    if (jc <= wjvis) {  // warp-uniform: tcgen05.ld is a warp-wide instruction
      const uint32_t taddr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + 128 * half;
      const int lim0 = static_cast<int>(jvis) - jc;  // scores i <= lim0 - g of a batch are visible
#pragma unroll 1
      for (int g = 0; g < 128 && jc + g <= wjvis; g += 16) {
        float v[16];
        tmem_ld16(taddr + g, v);
        const int lim = lim0 - g;
        const uint32_t thr = kv[7];
        uint32_t cand = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float sv = __fadd_rn(v[i] * scale, 0.0f);  // -0 -> +0: equal scores share one key
          const uint32_t kk = (i <= lim && sv == sv) ? order_key(sv) : 0u;
          kst[i * kThreads + tid] = kk;
          cand |= static_cast<uint32_t>(kk > thr) << i;
        }
        while (__any_sync(0xffffffffu, cand != 0)) {
          uint32_t x = 0;
          int xi = 0;
          if (cand) {
            const int i = __ffs(cand) - 1;
            cand &= cand - 1;
            x = kst[i * kThreads + tid];
            xi = jc + g + i;
          }
          insert_key(kv, ki, x, xi);
        }
      }
    }
    fence_before();
    __syncthreads();  // every TMEM read and staged key done before the next chunk
  }
  // no chunk was scored: the forecast tile's copy must still land before exit
  if (warp == 0 && c == 0) ok = mbar_wait_bounded(abar, 0) && ok;
  if (!ok && err && tid == 0) atomicExch(err, SD_KERR_TIMEOUT);

  // ---- blocks past the row's last visible one follow as -inf entries,
  // lowest index first, wherever the list has room; the k best are written
#pragma unroll 1
  for (int64_t jf = jvis + 1; jf < jvis + 9 && jf < NB; ++jf) insert_key(kv, ki, kKeyNegInf, static_cast<int>(jf));
  if (row0 + lr < Tq) {
    int64_t *dst = idx_out + ((static_cast<int64_t>(b) * H + h) * Tq + row0 + lr) * k;
#pragma unroll
    for (int i = 0; i < 8; ++i)  // constant indices keep the list in registers
      if (i < k) dst[i] = kv[i] == 0 ? -1 : static_cast<int64_t>(ki[i]);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace seltc

// Launches the tensor-core selector when it applies (bf16 forecast, D = 64,
// k <= 8, TMA-compatible strides); SD_ERR_UNSUPPORTED otherwise, so the
// caller falls back to the CUDA-core kernels.
int launch_select_rows_tc(const void *forecast, int f_dtype, int64_t B, int64_t Tq, int64_t H, int64_t D, int64_t f_sb,
                          int64_t f_st, int64_t f_sh, const float *reps, int64_t NB, int64_t r_sb, int64_t r_sn,
                          int64_t r_sh, int k, int block_size, int causal, int64_t q_offset, int64_t *topk_idx,
                          int32_t *err, cudaStream_t s) {
  using namespace seltc;
  if (f_dtype != SD_DTYPE_BF16 || D != 64 || k > 8 || Tq < kRows || NB > 0x7fffffff || Tq > 0x7fffffff ||
      B > 65535 || H > 65535)
    return SD_ERR_UNSUPPORTED;
  if (!aligned16(reps) || (r_sn % 4) || (r_sb % 4) || (r_sh % 4)) return SD_ERR_UNSUPPORTED;
  CUtensorMap mf;
  if (encode_rows_map(&mf, forecast, f_dtype, D, Tq, H, B, f_st, f_sh, f_sb, kRows) != SD_OK) return SD_ERR_UNSUPPORTED;
  const size_t smem = kSmemBytes + 1024;
  if (set_max_smem(select_rows_tc_kernel, smem) != SD_OK) return SD_ERR_CUDA;
  const dim3 grid(static_cast<unsigned>((Tq + kRows - 1) / kRows), static_cast<unsigned>(H), static_cast<unsigned>(B));
  select_rows_tc_kernel<<<grid, kThreads, smem, s>>>(mf, Tq, static_cast<int>(H), reps, NB, r_sb, r_sn, r_sh, k,
                                                     block_size, causal, q_offset, inv_sqrt(D), topk_idx, err);
  return check_launch();
}

}  // namespace sd
