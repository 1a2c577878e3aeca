// Block-sparse GQA prefill attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory) for 16-bit Q/K/V.  Replaces
// the mask construction + repeat_interleave + SDPA of
// model/attention/sparse.py:255-282 (masked path) and :334-360 (chunked path).
//
// One CTA (8 warps) per (sequence, kv head, 64-token query block).  The G <= 4
// query heads of the kv head give 64*G query rows, laid out as two 128-row
// MMA tiles (tile x holds heads 2x and 2x+1; missing heads are zero rows).
// For every listed key block (64 keys, staged by TMA with 128-byte swizzle in
// a 2-deep ring shared by the two tiles), each tile's warpgroup runs its own
// pipeline (ping-pong: one tile's softmax overlaps the other's MMAs):
//   S_x = Q_x K^T       tcgen05.mma M=128 N=64 K=64 (4 instructions), fp32 in TMEM
//   softmax             one thread per query row: tcgen05.ld of its 64 scores,
//                       masks (block membership, causality, length), online
//                       max/sum in fp32 with a lazily updated reference maximum
//                       (raised only when a block exceeds it by 2^8, the
//                       output rows in TMEM then rescaled), P row -> 16-bit
//                       pairs -> tcgen05.st over the first 32 columns of S_x
//   O_x += P_x V        tcgen05.mma M=128 N=64 K=64 with A (= P) read from
//                       tensor memory and V MN-major from shared memory,
//                       accumulated in TMEM across the blocks (no per-block
//                       read-out); the next S_x MMA, issued after it by the
//                       same thread, overwrites P only after it (tcgen05.mma
//                       operations of a thread execute in issue order)
// The first thread of each warpgroup issues its tile's MMAs and commits them
// to that tile's mbarriers; every wait is bounded.  TMEM: 256 columns (S0, S1,
// O0, O1) per CTA, 2 CTAs per SM.
#include <type_traits>

#include "sd_prefill.cuh"
#include "sd_tma.cuh"

namespace sd {

namespace tc {

constexpr int kThreads = 256;
constexpr int kStages = 2;
constexpr int kRowsTile = 128;                  // MMA M
constexpr int kTileBytes = kRowsTile * 128;     // 128 rows x 64 16-bit values
constexpr int kKvBytes = 64 * 128;              // 64 keys x 64 16-bit values
constexpr int kTmemCols = 256;
constexpr int kMaxKK = 16;                      // per-row top-k kept in registers

struct Smem {
  // all tile buffers 1024-byte aligned (128-byte swizzle atoms)
  static constexpr int kQ = 0;                          // 2 tiles
  static constexpr int kK = kQ + 2 * kTileBytes;        // kStages tiles
  static constexpr int kV = kK + kStages * kKvBytes;    // kStages tiles
  static constexpr int kBar = kV + kStages * kKvBytes;  // mbarriers
  static constexpr int kBytes = kBar + 256;
};

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  // start address >> 4 in bits [0,14), LBO >> 4 in [16,30), SBO >> 4 in
  // [32,46), descriptor version 1 in [46,48), layout 128-byte swizzle (2) in [61,64)
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(lbo_bytes >> 4) << 16) |
         (static_cast<uint64_t>(sbo_bytes >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator, A/B 16-bit format
// (0 = f16, 1 = bf16), K-major A, B K-major or MN-major, N = 64, M = 128.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t fmt, bool b_mn_major) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((64u >> 3) << 17) |
         ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc ? 1u : 0u)
      : "memory");
}

// The same MMA with A (M x K, K-major 16-bit pairs per 32-bit column) read
// from tensor memory at column address tmem_a.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane.
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

// 2^x with the SFU's approximate base-2 exponential (one instruction;
// 2^-inf = +0, so masked keys need no select).  The kernel is issue-bound,
// so the cheapest form per element wins.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 consecutive fp32 columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Lazy rescaling: a row keeps its reference maximum m (log2 units) until a
// block's maximum exceeds it by more than this; the exponentials are then at
// most 2^8, well inside bf16 and fp32, and the output rows in tensor memory
// are rescaled only on those rare increases.
constexpr float kRescaleLog2 = 8.0f;

}  // namespace tc

template <typename T>
__global__ void __launch_bounds__(tc::kThreads, 2)
    prefill_tc_kernel(const T *__restrict__ q, int64_t q_sb, int64_t q_st, int64_t q_sh,
                      const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, int64_t T_,
                      int Hkv, int G, const int32_t *__restrict__ lists, const int32_t *__restrict__ counts, int lcap,
                      const int64_t *__restrict__ topk, int kk, int causal, float scale_log2, T *__restrict__ out,
                      int64_t o_sb, int64_t o_st, int64_t o_sh) {
  using namespace tc;
  extern __shared__ __align__(1024) char smem_raw[];
  char *sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + Smem::kBar);  // [kStages]
  uint64_t *s_bar = full + kStages;  // [2]: S of tile x ready
  uint64_t *o_bar = s_bar + 2;       // [2]: PV of tile x ready
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(o_bar + 2);
  int *refill = reinterpret_cast<int *>(tmem_slot + 1);  // [kStages]: tiles done with the stage
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int nqt = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  // ---- set-up: TMEM, barriers
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      refill[s] = 0;
    }
    for (int xx = 0; xx < 2; ++xx) {
      mbar_init(&s_bar[xx], 1);
      mbar_init(&o_bar[xx], 1);
    }
    mbar_init_fence();
  }
  const int64_t lrow = (static_cast<int64_t>(b) * Hkv + h) * nqt + qt;
  const int32_t *list = lists + lrow * lcap;
  int cnt = counts[lrow];
  cnt = cnt < 0 ? 0 : (cnt > lcap ? lcap : cnt);
  const int64_t nbk = (T_ + 63) / 64;
  auto block_of = [&](int i) {
    const int j = list[i];
    return (j < 0 || j >= nbk) ? -1 : j;
  };
  auto issue = [&](int i) {  // thread 0: stage i's K and V tiles
    const int s = i % kStages;
    const int j = block_of(i);
    mbar_arrive_expect_tx(&full[s], 2u * kKvBytes);
    tma_load_4d(sm + Smem::kK + s * kKvBytes, &tmk, 0, (j < 0 ? 0 : j) * 64, h, b, &full[s]);
    tma_load_4d(sm + Smem::kV + s * kKvBytes, &tmv, 0, (j < 0 ? 0 : j) * 64, h, b, &full[s]);
  };
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0)
    for (int i = 0; i < cnt && i < kStages; ++i) issue(i);

  // ---- Q tiles: rows r of tile x = head 2x + r/64, token qt*64 + r%64
  {
    constexpr int kPer = 2 * kRowsTile * 8 / kThreads;  // 16-byte chunks per thread
    uint4 val[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {  // all loads in flight before any store
      const int e = tid + u * kThreads;
      const int x = e / (kRowsTile * 8), rem = e - x * kRowsTile * 8;
      const int r = rem >> 3, c = rem & 7;
      const int g = 2 * x + (r >> 6);
      const int64_t t = static_cast<int64_t>(qt) * 64 + (r & 63);
      val[u] = make_uint4(0u, 0u, 0u, 0u);
      if (g < G && t < T_)
        val[u] = *reinterpret_cast<const uint4 *>(q + b * q_sb + t * q_st + static_cast<int64_t>(h * G + g) * q_sh +
                                                  8 * c);
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kThreads;
      const int x = e / (kRowsTile * 8), rem = e - x * kRowsTile * 8;
      *reinterpret_cast<uint4 *>(sm + Smem::kQ + x * kTileBytes + sw128(rem >> 3, rem & 7)) = val[u];
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();

  // ---- per-thread row state
  const int x = warp >> 2;                       // MMA tile
  const int r = (warp & 3) * 32 + lane;          // row in the tile = TMEM lane
  const int g = 2 * x + (r >> 6);
  const int64_t t = static_cast<int64_t>(qt) * 64 + (r & 63);
  const bool row_ok = g < G && t < T_;
  const int bq = static_cast<int>(t / 64);
  int rk[kMaxKK];
  const bool use_rk = topk != nullptr;
#pragma unroll
  for (int e = 0; e < kMaxKK; ++e) {
    int64_t jj = -1;
    if (use_rk && row_ok && e < kk) {
      jj = topk[((static_cast<int64_t>(b) * Hkv + h) * T_ + t) * kk + e];
      jj = jj < 0 ? 0 : (jj > nbk - 1 ? nbk - 1 : jj);
    }
    rk[e] = static_cast<int>(jj);
  }
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const uint32_t t_s = tmem + lane_base + 64 * x;          // S_x columns
  const uint32_t t_o = tmem + lane_base + 128 + 64 * x;    // O_x columns: the PV MMAs accumulate into them
  float m = -INFINITY, l = 0.f;
  const uint32_t id_s = idesc_f16(fmt, false), id_pv = idesc_f16(fmt, true);
  bool ok = true;

  // a warp whose 32 rows are all padding (missing heads, rows past T) skips
  // the TMEM reads and the softmax; its P rows stay garbage and only feed
  // output rows that are never read
  const bool warp_active = __any_sync(0xffffffffu, row_ok);
  // Ping-pong: the warpgroup of tile x (warps 4x..4x+3) runs its own
  // pipeline with its own barriers and MMA-issuing thread (its first thread),
  // so one tile's softmax overlaps the other tile's tensor-core work.  The two
  // tiles share the K/V ring; the second tile to finish with a stage refills it.
  const bool leader = (tid & 127) == 0;
  const uint32_t bar_id = 1 + x;  // named barrier of this warpgroup (0 is __syncthreads)
  auto wg_sync = [&]() { asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory"); };
  auto wg_any = [&](bool pred) {
    uint32_t res;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, %2, 128, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(res)
        : "r"(pred ? 1u : 0u), "r"(bar_id)
        : "memory");
    return res != 0;
  };
  const uint32_t qaddr = smem_u32(sm + Smem::kQ + x * kTileBytes);
  auto issue_s = [&](int i) {  // leader: S_x = Q_x K^T for list entry i
    const int s = i % kStages;
    const bool got = mbar_wait_bounded(&full[s], (i / kStages) & 1);
    fence_after_sync();
    const uint32_t kaddr = smem_u32(sm + Smem::kK + s * kKvBytes);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      mma_f16(tmem + 64 * x, umma_desc_sw128(qaddr + 32 * k, 16, 1024), umma_desc_sw128(kaddr + 32 * k, 16, 1024),
              id_s, k > 0);
    mma_commit(&s_bar[x]);
    return got;
  };
  if (leader && cnt > 0) ok = issue_s(0);

  for (int i = 0; i < cnt; ++i) {
    const int s = i % kStages;
    const int j = block_of(i);
    ok = mbar_wait_bounded(&s_bar[x], i & 1) && ok;
    fence_after_sync();
    // S(i) complete implies this tile's PV(i - 1) complete (its leader issued
    // PV(i - 1) before S(i), and a commit tracks every earlier MMA of the
    // thread): both tiles done with stage (i - 1) % kStages, the second to
    // get here refills it, a softmax earlier than waiting for PV(i - 1)
    if (i > 0) {
      const int ps = (i - 1) % kStages;
      if (leader && atomicAdd(&refill[ps], 1) == 1) {
        refill[ps] = 0;
        if (i - 1 + kStages < cnt) issue(i - 1 + kStages);
      }
    }
    float sc[64];
    float mn = m, alpha = 1.f;
    if (warp_active) {
      // this row's 64 scores of block i
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        float v[16];
        tmem_ld16(t_s + 16 * c4, v);
#pragma unroll
        for (int u = 0; u < 16; ++u) sc[16 * c4 + u] = v[u];
      }
      tmem_wait_ld();
      bool blk_ok = row_ok && j >= 0;
      if (blk_ok && use_rk) {  // masked forecast rows: per-row membership (sparse.py:243-247)
        bool in = (j == 0) || (j == bq);
#pragma unroll
        for (int e = 0; e < kMaxKK; ++e) in = in || (rk[e] == j);
        blk_ok = in;
      }
      // keys k0 .. k0 + nv - 1 of this block are visible to this row
      int nv = 0;
      if (blk_ok) {
        const int k0 = j * 64;
        int lim = static_cast<int>(T_) - k0;
        if (causal) {
          const int lc = static_cast<int>(t) - k0 + 1;
          lim = lc < lim ? lc : lim;
        }
        nv = lim < 0 ? 0 : (lim > 64 ? 64 : lim);
      }
      if (nv < 64) {  // partial or masked block (rare): hide the invisible keys
#pragma unroll
        for (int c = 0; c < 64; ++c) sc[c] = c < nv ? sc[c] : -INFINITY;
      }
      // maximum over 8 interleaved partial maxima (a short dependency chain)
      float m8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = sc[e];
#pragma unroll
      for (int c = 8; c < 64; ++c) m8[c & 7] = fmaxf(m8[c & 7], sc[c]);
      const float mt = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      const float mts = mt * scale_log2;  // scale_log2 > 0: max of the scaled scores
      if (mts > m + kRescaleLog2 || (m == -INFINITY && mts > -INFINITY)) {
        mn = mts;
        alpha = m == -INFINITY ? 0.f : ex2(m - mn);
      }
    }
    // the previous block's PV MMA has finished with the P tile and with O
    if (i > 0) {
      ok = mbar_wait_bounded(&o_bar[x], (i - 1) & 1) && ok;
      fence_after_sync();
    }
    if (warp_active) {
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // a reference maximum rose: rescale the output rows so far (warp-wide
        // TMEM access; rows that keep their maximum multiply by 1)
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          float v[16];
          tmem_ld16(t_o + 16 * c4, v);
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 16; ++u) v[u] *= alpha;
          tmem_st16(t_o + 16 * c4, v);
        }
        tmem_wait_st();
      }
      const float nmn = mn == -INFINITY ? 0.f : -mn;  // rows with nothing visible yet keep p = 0
      float ps8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // 8 partial row sums
      // P row as 16-bit pairs (key 2c in the low half of column c) over the
      // first 32 columns of S_x, already read out above
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        float pw[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int kc = 32 * h2 + 2 * c;
          const float p0 = ex2(fmaf(sc[kc], scale_log2, nmn)), p1 = ex2(fmaf(sc[kc + 1], scale_log2, nmn));
          ps8[(2 * c) & 7] += p0;
          ps8[(2 * c + 1) & 7] += p1;
          pw[c] = __uint_as_float(pack2<T>(p0, p1));
        }
        tmem_st16(t_s + 16 * h2, pw);
      }
      tmem_wait_st();
      const float ps = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      l = l * alpha + ps;
      m = mn;
    }
    fence_before_sync();
    wg_sync();
    // O_x += P_x V (V tile MN-major: 64 keys of 128-byte rows; the first
    // block starts O), then the next block's S_x right behind it (S_x was
    // read out above)
    if (leader) {
      fence_after_sync();
      const uint32_t vaddr = smem_u32(sm + Smem::kV + s * kKvBytes);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_f16_ts(tmem + 128 + 64 * x, tmem + 64 * x + 8 * k, umma_desc_sw128(vaddr + 2048 * k, kKvBytes, 1024),
                   id_pv, i > 0 || k > 0);
      mma_commit(&o_bar[x]);
      if (i + 1 < cnt) ok = issue_s(i + 1) && ok;
    }
    __syncwarp();
    if (wg_any(!ok)) break;
  }
  if (cnt > 0) {  // the last PV MMA
    ok = mbar_wait_bounded(&o_bar[x], (cnt - 1) & 1) && ok;
    fence_after_sync();
  }
  const bool failed = __syncthreads_or(!ok);
  if (failed) {  // a bounded wait expired: let copies in flight land, poison the rows
    if (tid == 0)
      for (int s = 0; s < kStages; ++s) mbar_wait_bounded(&full[s], 0, 1000000ull);
    l = __int_as_float(0x7fc00000);
  }
  // ---- epilogue: O / l, from tensor memory (warp-wide loads)
  if (warp_active) {
    T *op = out + b * o_sb + t * o_st + static_cast<int64_t>(h * G + g) * o_sh;
    const float inv = l > 0.f ? 1.0f / l : (l == l ? 0.f : l);
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      float v[16];
      if (cnt > 0) {
        tmem_ld16(t_o + 16 * c4, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = 0.f;
      }
      if (row_ok) {
        uint4 w0, w1;
        w0.x = pack2<T>(v[0] * inv, v[1] * inv);
        w0.y = pack2<T>(v[2] * inv, v[3] * inv);
        w0.z = pack2<T>(v[4] * inv, v[5] * inv);
        w0.w = pack2<T>(v[6] * inv, v[7] * inv);
        w1.x = pack2<T>(v[8] * inv, v[9] * inv);
        w1.y = pack2<T>(v[10] * inv, v[11] * inv);
        w1.z = pack2<T>(v[12] * inv, v[13] * inv);
        w1.w = pack2<T>(v[14] * inv, v[15] * inv);
        *reinterpret_cast<uint4 *>(op + 16 * c4) = w0;
        *reinterpret_cast<uint4 *>(op + 16 * c4 + 8) = w1;
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Launches the tensor-core kernel when it applies; returns SD_ERR_UNSUPPORTED
// (nothing launched) otherwise, so the caller can use the CUDA-core kernel.
int launch_prefill_tc(int dtype, int G, dim3 grid, cudaStream_t s, const void *q, int64_t q_sb, int64_t q_st,
                      int64_t q_sh, const void *k, const void *v, int64_t c_sb, int64_t c_sh, int64_t c_st,
                      int64_t T_, int Hkv, int64_t B, const int32_t *lists, const int32_t *counts, int lcap,
                      const int64_t *topk, int kk, int causal, float scale_log2, void *out, int64_t o_sb,
                      int64_t o_st, int64_t o_sh) {
  if (dtype != SD_DTYPE_BF16 && dtype != SD_DTYPE_F16) return SD_ERR_UNSUPPORTED;
  if (G < 1 || G > 4 || (topk && kk > tc::kMaxKK)) return SD_ERR_UNSUPPORTED;
  // 16-byte vector access of q/out rows and TMA strides
  if (!aligned16(q) || !aligned16(out) || !aligned16(k) || !aligned16(v) || (q_sb * 2) % 16 || (q_st * 2) % 16 ||
      (q_sh * 2) % 16 || (o_sb * 2) % 16 || (o_st * 2) % 16 || (o_sh * 2) % 16 || (c_sb * 2) % 16 ||
      (c_sh * 2) % 16 || (c_st * 2) % 16)
    return SD_ERR_UNSUPPORTED;
  CUtensorMap mk, mv;
  if (encode_rows_map(&mk, k, dtype, 64, T_, Hkv, B, c_st, c_sh, c_sb, 64) != SD_OK) return SD_ERR_UNSUPPORTED;
  if (encode_rows_map(&mv, v, dtype, 64, T_, Hkv, B, c_st, c_sh, c_sb, 64) != SD_OK) return SD_ERR_UNSUPPORTED;
  const size_t smem = tc::Smem::kBytes + 1024;
  if (dtype == SD_DTYPE_BF16) {
    auto kern = prefill_tc_kernel<__nv_bfloat16>;
    if (set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
    kern<<<grid, tc::kThreads, smem, s>>>(static_cast<const __nv_bfloat16 *>(q), q_sb, q_st, q_sh, mk, mv, T_, Hkv,
                                          G, lists, counts, lcap, topk, kk, causal, scale_log2,
                                          static_cast<__nv_bfloat16 *>(out), o_sb, o_st, o_sh);
  } else {
    auto kern = prefill_tc_kernel<__half>;
    if (set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
    kern<<<grid, tc::kThreads, smem, s>>>(static_cast<const __half *>(q), q_sb, q_st, q_sh, mk, mv, T_, Hkv, G,
                                          lists, counts, lcap, topk, kk, causal, scale_log2,
                                          static_cast<__half *>(out), o_sb, o_st, o_sh);
  }
  return check_launch();
}

}  // namespace sd
