// K7 block-sparse GQA decode attention and the fused decode layer
// (RoPE + KV append + compressor update + selection + attention).
//
// Work split: one CTA (4 warps) per (sequence, kv head).  The selected KV
// blocks are cut into tiles of at most 64 cached rows of ONE block, staged into
// shared memory through a 4-stage ring completed on mbarriers, so up to 4
// tiles (K and V) are in flight per CTA while earlier ones are consumed.  (Four
// stages keep two CTAs per SM with room left for the side-stream candidate
// kernel that runs concurrently inside a decode step.)
//
// Two staging/compute paths:
//   * 16-bit caches whose rows are contiguous (the block-major cache of this
//     library): each tile is one TMA tensor copy (cp.async.bulk.tensor, 128-byte
//     swizzle) per K and V; warp w takes keys 16w..16w+15 of a tile and runs
//     QK^T and PV as mma.sync m16n8k16 with the G query heads as the rows of
//     the A operand (ldmatrix on the swizzled tile is bank-conflict free);
//   * fp32 caches (exact fp32 parity) and strided 16-bit caches: bulk copies of
//     rows and the same split of keys over warps on CUDA cores.
// Each warp keeps an online-softmax state (fp32, base-2 exponent) for all G
// heads; the four warp states are merged at the end.
// The fused kernel issues every tile it can name before any selection work -
// the sink and current blocks always, the whole list on static-window and
// dense steps - at kernel start, so the copies overlap the append and the
// scoring; the new token's K/V rows are patched into the staged tile in shared
// memory.  Selection either runs in the kernel or is merged from candidates a
// separate kernel computed earlier (sd_decode_candidates).
#include <type_traits>

#include "sd_select_core.cuh"
#include "sd_tma.cuh"

namespace sd {

constexpr int kD = 64;          // head_dim the attention kernels implement
constexpr int kRows = 64;       // rows per tile
constexpr int kStages = 5;
constexpr int kThreads = 128;  // the attention warps
constexpr int kWarps = kThreads / 32;
constexpr int kMaxTiles = 256;
constexpr float kLog2e = 1.4426950408889634f;

// The attention warps (the first kThreads threads) synchronise on named
// barrier 1, so a CTA may carry further warps (the fused kernel's next-layer
// scoring warps) that never join these barriers.  With exactly kThreads
// threads this is the same as __syncthreads().
__device__ __forceinline__ void attn_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }
__device__ __forceinline__ bool attn_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kThreads)
      : "memory");
  return r != 0;
}

template <typename T> __host__ __device__ constexpr bool is16() { return sizeof(T) == 2; }

// ---------------------------------------------------------------- CUDA-core helpers
// Per-lane feature layout of the CUDA-core QK^T product: lane l serves key
// group l>>3 and 8 features chosen so that the 8 lanes of a group read one K
// row with conflict-free 16-byte shared loads.
template <typename T> struct Feat {
  static __device__ __forceinline__ int dim(int dc, int i) { return 8 * dc + i; }
};
template <> struct Feat<float> {
  static __device__ __forceinline__ int dim(int dc, int i) { return i < 4 ? 4 * dc + i : 32 + 4 * dc + (i - 4); }
};

template <typename T> __device__ __forceinline__ void load8(const T *row, int dc, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4 *>(row + 8 * dc);
  const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f(e[i]);
}
template <> __device__ __forceinline__ void load8<float>(const float *row, int dc, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4 *>(row + 4 * dc);
  const float4 b = *reinterpret_cast<const float4 *>(row + 32 + 4 * dc);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename T> __device__ __forceinline__ float2 load2(const T *row, int lane) {
  const T *p = row + 2 * lane;
  return make_float2(to_f(p[0]), to_f(p[1]));
}
template <> __device__ __forceinline__ float2 load2<float>(const float *row, int lane) {
  return *reinterpret_cast<const float2 *>(row + 2 * lane);
}

// ---------------------------------------------------------------- shared memory
// Carve-up common to both kernels.  The stage buffers come first so that they
// sit on the 1024-byte boundary the 128-byte TMA swizzle needs; every region
// is rounded up to 128 bytes, so each one (and the tail, which holds rows read
// with 16-byte vector loads) starts 128-byte aligned.
__host__ __device__ constexpr size_t round128(size_t n) { return (n + 127) & ~static_cast<size_t>(127); }

template <typename T, int G> struct AttnSmem {
  T *k;            // [kStages][kRows][kD]
  T *v;            // [kStages][kRows][kD]
  uint64_t *full;  // [kStages]
  float *q;        // [G][kD]
  int *tile_tok;   // [kMaxTiles]
  int *tile_n;     // [kMaxTiles]
  float *red;      // [kWarps][G][kD + 2]
  T *newkv;        // [2][kD] the new token's K and V rows (fused kernel)
  char *tail;      // kernel-specific
  static constexpr size_t kKV = round128(sizeof(T) * kStages * kRows * kD);
  static constexpr size_t kFull = round128(sizeof(uint64_t) * kStages);
  static constexpr size_t kQ = round128(sizeof(float) * G * kD);
  static constexpr size_t kTiles = round128(sizeof(int) * kMaxTiles);
  static constexpr size_t kRed = round128(sizeof(float) * kWarps * G * (kD + 2));
  static constexpr size_t kNew = round128(sizeof(T) * 2 * kD);
  static constexpr size_t bytes() { return 2 * kKV + kFull + kQ + 2 * kTiles + kRed + kNew; }
  __device__ explicit AttnSmem(char *raw) {
    char *base = raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
    size_t o = 0;
    k = reinterpret_cast<T *>(base + o);
    o += kKV;
    v = reinterpret_cast<T *>(base + o);
    o += kKV;
    full = reinterpret_cast<uint64_t *>(base + o);
    o += kFull;
    q = reinterpret_cast<float *>(base + o);
    o += kQ;
    tile_tok = reinterpret_cast<int *>(base + o);
    o += kTiles;
    tile_n = reinterpret_cast<int *>(base + o);
    o += kTiles;
    red = reinterpret_cast<float *>(base + o);
    o += kRed;
    newkv = reinterpret_cast<T *>(base + o);
    o += kNew;
    tail = base + o;
  }
};
constexpr size_t kAlignSlack = 1024;

// Stage buffers 2..kStages-1 seen as fp32 prototype rows (kD floats each):
// first the K half of that region, then the V half.
template <typename T> struct ProtoStage {
  static constexpr int kRowsPerHalf = static_cast<int>((kStages - 2) * kRows * kD * sizeof(T) / (kD * sizeof(float)));
  template <int G> static __device__ float *k_half(AttnSmem<T, G> &S) {
    return reinterpret_cast<float *>(S.k + 2 * kRows * kD);
  }
  template <int G> static __device__ float *v_half(AttnSmem<T, G> &S) {
    return reinterpret_cast<float *>(S.v + 2 * kRows * kD);
  }
};

// Appends the tiles (<= kRows cached rows each) of block j to the tile table.
__device__ __forceinline__ int add_block_tiles(int64_t j, int64_t L, int bs, int *tile_tok, int *tile_n, int nt) {
  if (j < 0 || j * bs >= L) return nt;  // invalid or empty block: nothing to stage
  int64_t n = L - j * bs;
  if (n > bs) n = bs;
  for (int64_t r0 = 0; r0 < n && nt < kMaxTiles; r0 += kRows) {
    tile_tok[nt] = static_cast<int>(j * bs + r0);
    tile_n[nt] = static_cast<int>(n - r0 < kRows ? n - r0 : kRows);
    ++nt;
  }
  return nt;
}

// Appends the tiles of every listed block except skip_a / skip_b, starting at
// table index nt; returns the new tile count.  Called by one thread.
__device__ __forceinline__ int build_tiles(const int *list, int count, int64_t L, int bs, int *tile_tok,
                                           int *tile_n, int nt = 0, int skip_a = -1, int skip_b = -1) {
  for (int i = 0; i < count; ++i) {
    if (list[i] == skip_a || list[i] == skip_b) continue;
    nt = add_block_tiles(list[i], L, bs, tile_tok, tile_n, nt);
  }
  return nt;
}

// ---------------------------------------------------------------- staging
// Bulk (non-tensor TMA) copies of a tile's rows: one copy when rows are
// contiguous, one per row otherwise.  Rows land unswizzled.
template <typename T> struct BulkLoader {
  const T *kb, *vb;
  int64_t c_st;
  __device__ void operator()(T *kd, T *vd, int tok, int n, uint64_t *bar) const {
    const uint32_t row_bytes = kD * sizeof(T);
    mbar_arrive_expect_tx(bar, 2u * n * row_bytes);
    if (c_st == kD) {
      bulk_g2s(kd, kb + static_cast<int64_t>(tok) * kD, n * row_bytes, bar);
      bulk_g2s(vd, vb + static_cast<int64_t>(tok) * kD, n * row_bytes, bar);
    } else {
      for (int r = 0; r < n; ++r) {
        bulk_g2s(kd + r * kD, kb + static_cast<int64_t>(tok + r) * c_st, row_bytes, bar);
        bulk_g2s(vd + r * kD, vb + static_cast<int64_t>(tok + r) * c_st, row_bytes, bar);
      }
    }
  }
};

// TMA tensor copies of a whole 64-row box (rows past the map's extent are
// zero-filled; rows past the tile's valid count are masked by the consumer).
struct TmaLoader {
  const CUtensorMap *mk, *mv;
  int h, b;
  template <typename T> __device__ void operator()(T *kd, T *vd, int tok, int, uint64_t *bar) const {
    mbar_arrive_expect_tx(bar, 2u * kRows * kD * sizeof(T));
    tma_load_4d(kd, mk, 0, tok, h, b, bar);
    tma_load_4d(vd, mv, 0, tok, h, b, bar);
  }
};

template <typename T, int G, typename Ld>
__device__ __forceinline__ void issue_tile(AttnSmem<T, G> &S, int t, const Ld &ld) {
  const int s = t % kStages;
  ld(S.k + s * kRows * kD, S.v + s * kRows * kD, S.tile_tok[t], S.tile_n[t], &S.full[s]);
}

// Merges the per-warp states written to S.red and stores out[g*o_hs + d].
template <typename T, int G>
__device__ __forceinline__ void combine_store(AttnSmem<T, G> &S, T *out, int64_t o_hs) {
  for (int e = threadIdx.x; e < G * kD; e += kThreads) {
    const int g = e / kD, d = e - g * kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, S.red[(w * G + g) * (kD + 2)]);
    float den = 0.f, num = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float *r = S.red + (w * G + g) * (kD + 2);
        const float f = exp2f(r[0] - M);
        den = fmaf(r[1], f, den);
        num = fmaf(r[2 + d], f, num);
      }
    }
    out[g * o_hs + d] = from_f<T>(den > 0.f ? num / den : 0.f);
  }
}

// Waits for tile t; returns the uniform "all threads got it" verdict through
// the CTA barrier at the end of the tile (see the loops below).
__device__ __forceinline__ bool wait_tile(uint64_t *full, int t) {
  bool got = mbar_wait_bounded(&full[t % kStages], (t / kStages) & 1);
  return __all_sync(0xffffffffu, got);
}

// After a bounded wait expired: let the copies still in flight land before
// the CTA's shared memory is released.
template <typename T, int G>
__device__ __forceinline__ void drain(AttnSmem<T, G> &S, int t, int ntiles) {
  for (int u = t; u < ntiles && u < t + kStages; ++u) mbar_wait_bounded(&S.full[u % kStages], (u / kStages) & 1);
  attn_sync();
}

// Writes the new token's K/V rows (S.newkv) into row `row` of staged tile t,
// over whatever the copy brought for that row.  TMA tiles are 128-byte
// swizzled, bulk tiles are linear.  All threads call it (t is CTA-uniform).
template <typename T, int G>
__device__ __forceinline__ void patch_tile_rows(AttnSmem<T, G> &S, int t, int row, bool swizzled) {
  const int s = t % kStages;
  if (threadIdx.x < kD) {
    const int d = threadIdx.x;
    char *kb = reinterpret_cast<char *>(S.k + s * kRows * kD);
    char *vb = reinterpret_cast<char *>(S.v + s * kRows * kD);
    uint32_t off = swizzled ? sw128(row, d >> 3) + (d & 7) * sizeof(T) : (row * kD + d) * sizeof(T);
    *reinterpret_cast<T *>(kb + off) = S.newkv[d];
    *reinterpret_cast<T *>(vb + off) = S.newkv[kD + d];
    // the stage is refilled by the async proxy later: order these writes first
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  attn_sync();
}

// ---------------------------------------------------------------- CUDA-core path
template <typename T, int G, typename Ld>
__device__ bool attend_simt(AttnSmem<T, G> &S, int ntiles, int pre_issued, const Ld &ld, float scale_log2, T *out,
                            int64_t o_hs, int patch_t = -1, int patch_row = 0) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kg = lane >> 3, dc = lane & 7;
  if (tid == 0) {
    for (int t = pre_issued; t < ntiles && t < kStages; ++t) issue_tile(S, t, ld);
  }
  float qr[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) qr[g][i] = S.q[g * kD + Feat<T>::dim(dc, i)] * scale_log2;
  float m[G], l[G], acc[G][2];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
    acc[g][0] = acc[g][1] = 0.f;
  }
  int t = 0;
  for (; t < ntiles; ++t) {
    const int s = t % kStages;
    const bool got = wait_tile(S.full, t);
    if (t == patch_t) patch_tile_rows(S, t, patch_row, false);
    if (got) {
      const T *ks = S.k + s * kRows * kD;
      const T *vs = S.v + s * kRows * kD;
      int nv = S.tile_n[t] - 16 * warp;  // rows of this warp that hold keys
      nv = nv < 0 ? 0 : (nv > 16 ? 16 : nv);
      float sc[G][4];
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int r = 16 * warp + 4 * it + kg;
        float x[8];
        load8<T>(ks + r * kD, dc, x);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float p = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) p = fmaf(qr[g][i], x[i], p);
          p += __shfl_xor_sync(0xffffffffu, p, 1);
          p += __shfl_xor_sync(0xffffffffu, p, 2);
          p += __shfl_xor_sync(0xffffffffu, p, 4);
          sc[g][it] = (4 * it + kg < nv) ? p : -INFINITY;
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float mt = fmaxf(fmaxf(sc[g][0], sc[g][1]), fmaxf(sc[g][2], sc[g][3]));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
        const float mn = fmaxf(m[g], mt);
        if (mn == -INFINITY) continue;  // no key seen yet (uniform per warp)
        const float alpha = exp2f(m[g] - mn);
        float ps = 0.f;
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          sc[g][it] = exp2f(sc[g][it] - mn);
          ps += sc[g][it];
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 8);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        l[g] = l[g] * alpha + ps;
        acc[g][0] *= alpha;
        acc[g][1] *= alpha;
        m[g] = mn;
      }
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        if (kk < nv) {
          const float2 vv = load2<T>(vs + (16 * warp + kk) * kD, lane);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float p = __shfl_sync(0xffffffffu, sc[g][kk >> 2], (kk & 3) * 8);
            if (m[g] != -INFINITY) {
              acc[g][0] = fmaf(p, vv.x, acc[g][0]);
              acc[g][1] = fmaf(p, vv.y, acc[g][1]);
            }
          }
        }
      }
    }
    if (attn_sync_or(!got)) {
      drain(S, t, ntiles);
      return false;
    }
    if (tid == 0 && t + kStages < ntiles) issue_tile(S, t + kStages, ld);
  }
  float *rw = S.red + warp * G * (kD + 2);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      rw[g * (kD + 2)] = m[g];
      rw[g * (kD + 2) + 1] = l[g];
    }
    rw[g * (kD + 2) + 2 + 2 * lane] = acc[g][0];
    rw[g * (kD + 2) + 3 + 2 * lane] = acc[g][1];
  }
  attn_sync();
  combine_store(S, out, o_hs);
  return true;
}

// ---------------------------------------------------------------- tensor-core path
// Warp w, per tile: S[heads x 16 keys] = Q K^T as 2 n-tiles x 4 k-steps of
// m16n8k16 (A rows = the G heads, zero-padded to 16), softmax on the fp32
// accumulators (a quad of lanes holds one head's 16 scores), then
// O[heads x 64] += P V as 8 n-tiles x 1 k-step, P reused from the accumulator
// registers as the A operand.  K fragments come from ldmatrix, V fragments
// from ldmatrix.trans, both on the 128-byte-swizzled TMA tiles.
template <typename T, int G>
__device__ bool attend_mma(AttnSmem<T, G> &S, int ntiles, int pre_issued, const TmaLoader &ld, float scale_log2,
                           T *out, int64_t o_hs, int patch_t = -1, int patch_row = 0) {
  static_assert(G <= 8, "query heads per kv head must fit the 16 rows of the A operand");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 2, tig = lane & 3;
  if (tid == 0) {
    for (int t = pre_issued; t < ntiles && t < kStages; ++t) issue_tile(S, t, ld);
  }
  uint32_t qa[4][2];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const float *qr = S.q + (grp < G ? grp : 0) * kD + 16 * ks + 2 * tig;
    const float z = grp < G ? 1.f : 0.f;
    qa[ks][0] = pack2<T>(qr[0] * z, qr[1] * z);
    qa[ks][1] = pack2<T>(qr[8] * z, qr[9] * z);
  }
  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  int t = 0;
  for (; t < ntiles; ++t) {
    const int s = t % kStages;
    const bool got = wait_tile(S.full, t);
    if (t == patch_t) patch_tile_rows(S, t, patch_row, true);
    int nv = S.tile_n[t] - 16 * warp;
    nv = nv < 0 ? 0 : (nv > 16 ? 16 : nv);
    if (got && nv > 0) {
      const uint32_t kbase = smem_u32(S.k + s * kRows * kD);
      const uint32_t vbase = smem_u32(S.v + s * kRows * kD);
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        const int key = 16 * warp + 8 * nt + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + sw128(key, lane >> 3), b0, b1, b2, b3);
        mma16816<T>(sc[nt], {qa[0][0], 0u, qa[0][1], 0u}, b0, b1);
        mma16816<T>(sc[nt], {qa[1][0], 0u, qa[1][1], 0u}, b2, b3);
        ldsm_x4(kbase + sw128(key, 4 + (lane >> 3)), b0, b1, b2, b3);
        mma16816<T>(sc[nt], {qa[2][0], 0u, qa[2][1], 0u}, b0, b1);
        mma16816<T>(sc[nt], {qa[3][0], 0u, qa[3][1], 0u}, b2, b3);
      }
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kl = 8 * (i >> 1) + 2 * tig + (i & 1);  // key within the warp's 16
        v[i] = kl < nv ? sc[i >> 1][i & 1] * scale_log2 : -INFINITY;
      }
      float mt = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float mn = fmaxf(m, mt);  // finite: every warp slice with nv > 0 has a key
      const float alpha = exp2f(m - mn);
      float p[4], ps = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        p[i] = exp2f(v[i] - mn);
        ps += p[i];
      }
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      l = l * alpha + ps;
      m = mn;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        o[n][0] *= alpha;
        o[n][1] *= alpha;
      }
      const uint32_t pa[4] = {pack2<T>(p[0], p[1]), 0u, pack2<T>(p[2], p[3]), 0u};
      const int vkey = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int qd = 0; qd < 4; ++qd) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vbase + sw128(vkey, 2 * qd + (lane >> 4)), r0, r1, r2, r3);
        mma16816<T>(o[2 * qd], pa, r0, r1);
        mma16816<T>(o[2 * qd + 1], pa, r2, r3);
      }
    }
    if (attn_sync_or(!got)) {
      drain(S, t, ntiles);
      return false;
    }
    if (tid == 0 && t + kStages < ntiles) issue_tile(S, t + kStages, ld);
  }
  float *rw = S.red + warp * G * (kD + 2);
  if (grp < G) {
    float *r = rw + grp * (kD + 2);
    if (tig == 0) {
      r[0] = m;
      r[1] = l;
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      r[2 + 8 * n + 2 * tig] = o[n][0];
      r[3 + 8 * n + 2 * tig] = o[n][1];
    }
  }
  attn_sync();
  combine_store(S, out, o_hs);
  return true;
}

__device__ __forceinline__ void report(int32_t *err, int code) {
  if (err && threadIdx.x == 0) atomicExch(err, code);
}

template <typename T, int G>
__device__ __forceinline__ void init_barriers(AttnSmem<T, G> &S) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&S.full[s], 1);
    mbar_init_fence();
  }
}

// ------------------------------------------------------------ API kernel
template <typename T, int G, bool kTma>
__global__ void __launch_bounds__(kThreads)
    decode_attention_kernel(const T *__restrict__ q, int Hkv, int64_t q_sb, int64_t q_sh, const T *k_cache,
                            const T *v_cache, int64_t c_sb, int64_t c_sh, int64_t c_st,
                            const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                            const int32_t *__restrict__ sel, const int32_t *__restrict__ cnt, int ms_cap,
                            int64_t L, int bs, float scale_log2, T *__restrict__ out, int64_t o_sb,
                            int64_t o_sh, int32_t *err) {
  extern __shared__ __align__(1024) char smem_raw[];
  AttnSmem<T, G> S(smem_raw);
  int *list = reinterpret_cast<int *>(S.tail);
  __shared__ int ntiles;
  const int b = blockIdx.x / Hkv, h = blockIdx.x - (blockIdx.x / Hkv) * Hkv;
  init_barriers(S);
  for (int e = threadIdx.x; e < G * kD; e += blockDim.x) {
    const int g = e / kD, d = e - g * kD;
    S.q[e] = to_f(q[b * q_sb + static_cast<int64_t>(h * G + g) * q_sh + d]);
  }
  const int32_t *srow = sel + static_cast<int64_t>(blockIdx.x) * ms_cap;
  int c = cnt[blockIdx.x];
  c = c < 0 ? 0 : (c > ms_cap ? ms_cap : c);
  for (int i = threadIdx.x; i < c; i += blockDim.x) list[i] = srow[i];
  __syncthreads();
  if (threadIdx.x == 0) ntiles = build_tiles(list, c, L, bs, S.tile_tok, S.tile_n);
  __syncthreads();
  T *o = out + b * o_sb + static_cast<int64_t>(h * G) * o_sh;
  bool ok;
  if constexpr (kTma) {
    const TmaLoader ld{&tmk, &tmv, h, b};
    ok = attend_mma<T, G>(S, ntiles, 0, ld, scale_log2, o, o_sh);
  } else {
    const int64_t cb = b * c_sb + h * c_sh;
    const BulkLoader<T> ld{k_cache + cb, v_cache + cb, c_st};
    ok = attend_simt<T, G>(S, ntiles, 0, ld, scale_log2, o, o_sh);
  }
  if (!ok) report(err, SD_KERR_TIMEOUT);
}

// ------------------------------------------------------------ fused layer
// RoPE of one element with the reference's rounding sequence
// (model/rope.py:58-63): tables cast to the activation dtype, then
// x*cos and rotate_half(x)*sin and their sum each rounded to the dtype.
template <typename T>
__device__ __forceinline__ float rope_elem(float x, float partner, int d, float c, float s) {
  return rope_rounded<T>(x, d < kD / 2 ? -partner : partner, c, s);
}

// Tail of the fused kernel's shared memory.
struct LayerTail {
  float *f;     // [kD] forecast row (fp32)
  float *pnew;  // [kD] updated running sum of the current block
  float *pold;  // [kD] its sum before this step's token
  float *sc;    // [NBcap] prototype scores
  int *list;    // [max(NBcap, top_k + 2)] selected blocks, ascending
  int *tk;      // [top_k] merged top-k
  int *ci;      // [top_k + 1] candidate indices (precomputed ones + the current block)
  float *cv;    // [top_k + 1] candidate scores
  static size_t bytes(int64_t NBcap, int top_k) {
    const int64_t lst = NBcap > top_k + 2 ? NBcap : top_k + 2;
    return sizeof(float) * (3 * kD + NBcap) + sizeof(int) * (lst + top_k) +
           (sizeof(int) + sizeof(float)) * (top_k + 1);
  }
  __device__ LayerTail(char *p, int64_t NBcap, int top_k) {
    const int64_t lst = NBcap > top_k + 2 ? NBcap : top_k + 2;
    f = reinterpret_cast<float *>(p);
    pnew = f + kD;
    pold = pnew + kD;
    sc = pold + kD;
    list = reinterpret_cast<int *>(sc + NBcap);
    tk = list + lst;
    ci = tk + top_k;
    cv = reinterpret_cast<float *>(ci + top_k + 1);
  }
};

// Offloaded caches: the authoritative K/V rows live in pinned host memory
// (host_k/host_v, [B, Hkv, host_tcap, 64], read and written by the GPU over the
// host link), and the device holds per (sequence, kv head) a slot buffer of
// 2 + kslots blocks: slot 0 the sink block, slot 1 the block being written,
// slots 2.. the blocks a prefetch staged for this step.  host_k == nullptr
// means a plain device cache.
// The next layer's candidates, computed at the end of this layer's kernel
// (what sd_decode_candidates computes on a side stream): the next layer's
// running block sums do not change until its own step, and its forecast is
// this layer's projection.  proto == nullptr: not requested.
struct NextCand {
  const float *proto = nullptr;
  const void *fc = nullptr;  // forecast rows, activation dtype, row stride f_sb
  int64_t f_sb = 0;
  int32_t *cand_idx = nullptr;
  float *cand_val = nullptr;
};

template <typename T> struct SlotMap {
  T *host_k = nullptr, *host_v = nullptr;
  int64_t host_tcap = 0;
  const int32_t *cand_slot = nullptr;  // [B, Hkv, top_k]: slot (0..kslots-1) of candidate rank r
  int kslots = 0;
};

// kCands: the launch passes precomputed candidates (chained or side-stream
// selection).  That instantiation leaves out the in-kernel scoring code, so
// the code the common path runs is compact: the kernel runs once per layer
// between library GEMMs, its instructions are fetched cold, and a fetch that
// has to cross the unused scoring code costs microseconds while the tile
// loads keep HBM busy.
template <typename T, typename F, int G, bool kCands>
__global__ void __launch_bounds__(2 * kThreads)
    decode_layer_kernel(const T *__restrict__ qkv, int64_t qkv_sb, const F *__restrict__ fc, int64_t f_sb,
                        const float *__restrict__ rcos, const float *__restrict__ rsin,
                        const int32_t *__restrict__ cur_len, T *k_cache, T *v_cache, float *proto_sum, int Hkv,
                        int64_t Tcap, int64_t NBcap, int bs, int top_k, int rule, float sel_scale,
                        float scale_log2, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, T *__restrict__ out, int64_t o_sb,
                        const int32_t *__restrict__ cand_idx, const float *__restrict__ cand_val,
                        int32_t *sel_out, int32_t *cnt_out, int sel_cap, int32_t *err, const SlotMap<T> sm,
                        const NextCand nx) {
  extern __shared__ __align__(1024) char smem_raw[];
  const bool slots = sm.host_k != nullptr;
  // SD_SELECT_BEFORE_APPEND: score the current block with its sum before this
  // step's token, and not at all when the token opens it (the reference's
  // async prefetch selects before the append, async_offload.py:241-260)
  const bool pre_app = (rule & SD_SELECT_BEFORE_APPEND) != 0;
  rule &= ~SD_SELECT_BEFORE_APPEND;
  const int b = blockIdx.x / Hkv, h = blockIdx.x - (blockIdx.x / Hkv) * Hkv;
  const int Hq = Hkv * G;
  const int64_t bh = static_cast<int64_t>(b) * Hkv + h;
  // warp 0 requests the precomputed candidates (rank = lane) together with
  // the length, so both loads are in flight at once; phase 0 keeps the ones
  // the step uses.  The tile maps' descriptors are fetched meanwhile.
  int cj = -1, cslot = 0;
  float cv = -INFINITY;
  if (kCands && threadIdx.x < 32 && static_cast<int>(threadIdx.x) < top_k) {
    cj = cand_idx[bh * top_k + threadIdx.x];
    cv = cand_val[bh * top_k + threadIdx.x];
    if (slots) cslot = sm.cand_slot[bh * top_k + threadIdx.x];
  }
  if (threadIdx.x == 32 && is16<T>()) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
  }
  const int64_t pos = *cur_len;
  if (pos < 0 || pos >= (slots ? sm.host_tcap : Tcap)) {  // cache full (or corrupt length): write nothing
    report(err, SD_KERR_BOUNDS);
    return;
  }
  const int64_t L = pos + 1;
  const int curr = static_cast<int>(pos / bs);
  const int nb = curr + 1;
  const int ms = nb < top_k + 2 ? nb : top_k + 2;
  const int kk = top_k < nb ? top_k : nb;

  // -- next-layer scoring warps (present only when nx.proto != nullptr): the
  //    next layer's candidates for its coming step, top-k over its blocks
  //    0..curr-1 (it caches as many tokens as this layer; its sums do not
  //    change before its own step, and its forecast is this layer's
  //    projection).  They run from the kernel's start, beside the attention
  //    warps' tile ring, and share nothing with them but the CTA.
  if (threadIdx.x >= kThreads) {
    __shared__ float nsv[kWarps * 32];
    __shared__ int nsi[kWarps * 32];
    const WarpGroup g{kWarps, static_cast<int>(blockDim.x >> 5) - kWarps, 2};
    int32_t *oi = nx.cand_idx + bh * top_k;
    float *ov = nx.cand_val + bh * top_k;
    if (nb <= ms) {  // its step is dense: no candidates needed
      for (int r = threadIdx.x - kThreads; r < top_k; r += g.nw * 32) {
        oi[r] = -1;
        ov[r] = -INFINITY;
      }
      return;
    }
    pdl_wait();  // the forecast rows come from the projection kernel ahead
    const T *fr = static_cast<const T *>(nx.fc) + b * nx.f_sb + h * kD;
    const int l16 = threadIdx.x & 15;
    const float4 fv =
        make_float4(to_f(fr[4 * l16]), to_f(fr[4 * l16 + 1]), to_f(fr[4 * l16 + 2]), to_f(fr[4 * l16 + 3]));
    const int nsc = rule == SD_RULE_REFERENCE ? 1 : curr;
    const float *base = nx.proto + bh * NBcap * kD;
    group_score_topk([&](int j) { return base + static_cast<int64_t>(j) * kD; }, fv, curr, nsc, -1, sel_scale,
                     top_k, oi, ov, nsv, nsi, g);
    return;
  }

  AttnSmem<T, G> S(smem_raw);
  LayerTail X(S.tail, NBcap, top_k);
  __shared__ int count, ntiles, pre, patch_t, patch_row, disp_t;
  __shared__ __align__(8) uint64_t proto_bar;  // completion of the staged prototype rows
  const bool use_f = fc != nullptr && nb > ms;  // a forecast-driven selection is needed
  const WarpGroup ag{0, kWarps, 1};             // the attention warps
  const T *kb = k_cache + bh * Tcap * kD;
  const T *vb = v_cache + bh * Tcap * kD;
  const BulkLoader<T> bulk{kb, vb, kD};
  const TmaLoader tma{&tmk, &tmv, h, b};
  auto issue = [&](int t) {
    if constexpr (is16<T>()) {
      issue_tile(S, t, tma);
    } else {
      issue_tile(S, t, bulk);
    }
  };

  // -- 0. stage every tile that is known now (warp 0, in parallel lanes: lane
  //       s initialises stage barrier s and issues tile s).  With block_size
  //       <= 64 every block is one tile and tile t's block is known without a
  //       list: the whole window on dense and static-window steps; on forecast
  //       steps with precomputed candidates the sink, the current block and
  //       every candidate in rank order (the candidate ranked last is loaded
  //       too and dropped in phase 2 if the current block's fresh score
  //       displaces it); with in-kernel selection the sink and current block.
  const bool one_tile = bs <= kRows;
  const bool early_cands = use_f && one_tile && cand_idx != nullptr && kk <= 32;
  // In-kernel forecast selection stages the running sums of blocks
  // 0..nstage-1 (every cached block but the current one, whose sum changes
  // below) into the stage buffers 2..kStages-1, which hold no tile until the
  // selection is known: one bulk copy per K/V half of that region, issued
  // before anything else so the scoring reads shared memory.
  const int stage_cap = ProtoStage<T>::kRowsPerHalf * 2;
  const bool stage_protos = !kCands && use_f && one_tile && kk <= 32 && rule != SD_RULE_REFERENCE;
  const int nstage = stage_protos ? (curr < stage_cap ? curr : stage_cap) : 0;
  // warp 0 keeps the precomputed candidates of its lanes (rank = lane) for
  // the merge in phase 2
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    if (lane < kStages) mbar_init(&S.full[lane], 1);
    if (lane == kStages) mbar_init(&proto_bar, 1);
    mbar_init_fence();
    __syncwarp();
    if (lane == 31 && nstage > 0) {
      const float *src = proto_sum + bh * NBcap * kD;
      const int n0 = nstage < ProtoStage<T>::kRowsPerHalf ? nstage : ProtoStage<T>::kRowsPerHalf;
      mbar_arrive_expect_tx(&proto_bar, static_cast<uint32_t>(nstage) * kD * sizeof(float));
      bulk_g2s(ProtoStage<T>::k_half(S), src, n0 * kD * sizeof(float), &proto_bar);
      if (nstage > n0)
        bulk_g2s(ProtoStage<T>::v_half(S), src + static_cast<int64_t>(n0) * kD, (nstage - n0) * kD * sizeof(float),
                 &proto_bar);
    }
    int nt = 0, dt = -1, p = 0;
    if (one_tile) {
      int lo = 0;  // static window: {0} U {lo..curr}
      if (use_f) {
        nt = curr != 0 ? 2 : 1;
      } else if (nb <= ms) {
        nt = nb;
      } else {
        lo = curr - top_k + 1 > 0 ? curr - top_k + 1 : 0;
        nt = (lo > 0 ? 1 : 0) + (curr - lo + 1);
      }
      for (int t = lane; t < nt; t += 32) {
        int j;
        if (use_f) {
          j = t == 0 ? 0 : curr;
        } else if (nb <= ms) {
          j = t;
        } else {
          j = lo > 0 ? (t == 0 ? 0 : lo + t - 1) : lo + t;
        }
        const int64_t n = L - static_cast<int64_t>(j) * bs;
        // offloaded cache: the sink, current and window/dense blocks sit in
        // fixed slots (a window block j in slot 2 + j % kslots)
        const int src = !slots ? j : (j == curr ? 1 : (j == 0 ? 0 : 2 + j % sm.kslots));
        S.tile_tok[t] = src * bs;
        S.tile_n[t] = static_cast<int>(n < bs ? n : bs);
      }
      __syncwarp();
      // the tiles known without any load go out first
      p = nt < kStages ? nt : kStages;
      if (lane < p) issue(lane);
      if (early_cands) {
        // candidates are distinct blocks other than the current one; the sink
        // is already staged, so it is skipped when it is a candidate
        if (lane >= kk) {  // loaded at entry for every rank < top_k
          cj = -1;
          cv = -INFINITY;
        }
        const int cs = slots && lane < kk ? cslot : 0;
        const bool keep = cj > 0 && cj < nb && cj != curr && cs >= 0 && (!slots || cs < sm.kslots);
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        const int slot = nt + __popc(bal & ((1u << lane) - 1u));
        if (keep) {
          const int64_t n = L - static_cast<int64_t>(cj) * bs;
          S.tile_tok[slot] = (slots ? 2 + cs : cj) * bs;
          S.tile_n[slot] = static_cast<int>(n < bs ? n : bs);
        }
        dt = __shfl_sync(0xffffffffu, keep ? slot : -1, kk - 1);  // tile of the last-ranked candidate
        const int nt2 = nt + __popc(bal);
        __syncwarp();
        const int p2 = nt2 < kStages ? nt2 : kStages;
        if (lane >= p && lane < p2) issue(lane);
        nt = nt2;
        p = p2;
      }
    } else {
      if (lane == 0) {
        if (!use_f) {
          if (nb <= ms) {
            for (int j = 0; j < nb; ++j) X.list[j] = j;
            count = nb;
          } else {
            count = assemble_decode_list(false, nullptr, 0, nb, curr, top_k, X.list);
          }
          nt = build_tiles(X.list, count, L, bs, S.tile_tok, S.tile_n);
        } else {
          nt = add_block_tiles(0, L, bs, S.tile_tok, S.tile_n, 0);
          nt = add_block_tiles(curr, L, bs, S.tile_tok, S.tile_n, nt);
        }
      }
      nt = __shfl_sync(0xffffffffu, nt, 0);
      __syncwarp();
      p = nt < kStages ? nt : kStages;
      if (lane < p) issue(lane);
    }
    if (lane == 0) {
      pre = p;
      ntiles = nt;
      disp_t = dt;
    }
  }

  // -- 1. RoPE, append, compressor running sum, by warps 1..3 while warp 0
  //       stages tiles: every thread issues all of its global loads before it
  //       computes, so this phase costs one round trip.  Threads 32..95 take
  //       element d of k, v, the block sum and the forecast; warp 3 takes q.
  const T *row = qkv + b * qkv_sb;
  const float *cr = rcos + pos * (kD / 2);
  const float *sr = rsin + pos * (kD / 2);
  // q|k|v come from the projection kernel ahead on the stream; warp 0's tiles,
  // candidates and sums were written by earlier kernels and need no wait
  if (threadIdx.x >= 32) pdl_wait();
  if (threadIdx.x >= 32 && threadIdx.x < 32 + kD) {
    const int d = threadIdx.x - 32;
    const T *kr = row + static_cast<int64_t>(Hq + h) * kD;
    float *ps = proto_sum + (bh * NBcap + curr) * kD + d;
    const T kx = kr[d], kp = kr[d < kD / 2 ? d + kD / 2 : d - kD / 2];
    const T vv = row[static_cast<int64_t>(Hq + Hkv + h) * kD + d];
    const float c = cr[d & (kD / 2 - 1)], sn = sr[d & (kD / 2 - 1)];
    const float old = pos % bs == 0 ? 0.f : *ps;
    const float fx = fc != nullptr ? to_f(fc[b * f_sb + h * kD + d]) : 0.f;
    const float y = rope_elem<T>(to_f(kx), to_f(kp), d, c, sn);
    const int64_t off = (bh * Tcap + (slots ? bs + pos % bs : pos)) * kD + d;
    if (slots) {  // write-through to the host copy
      const int64_t hoff = (bh * sm.host_tcap + pos) * kD + d;
      sm.host_k[hoff] = from_f<T>(y);
      sm.host_v[hoff] = vv;
    }
    k_cache[off] = from_f<T>(y);
    v_cache[off] = vv;
    S.newkv[d] = from_f<T>(y);
    S.newkv[kD + d] = vv;
    const float pn = old + y;
    *ps = pn;
    X.pnew[d] = pn;
    X.pold[d] = old;
    if (fc != nullptr) X.f[d] = fx;
  } else if (threadIdx.x >= 32 + kD) {
    constexpr int kQT = kThreads - 32 - kD;  // threads of the q part
    constexpr int kPer = (G * kD + kQT - 1) / kQT;
    const int q0 = threadIdx.x - 32 - kD;
    T qx[kPer], qp[kPer];
    float qc[kPer], qs[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = q0 + i * kQT;
      if (e < G * kD) {
        const int g = e / kD, d = e - g * kD;
        const T *qr = row + static_cast<int64_t>(h * G + g) * kD;
        qx[i] = qr[d];
        qp[i] = qr[d < kD / 2 ? d + kD / 2 : d - kD / 2];
        qc[i] = cr[d & (kD / 2 - 1)];
        qs[i] = sr[d & (kD / 2 - 1)];
      }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = q0 + i * kQT;
      if (e < G * kD) S.q[e] = rope_elem<T>(to_f(qx[i]), to_f(qp[i]), e % kD, qc[i], qs[i]);
    }
  }
  attn_sync();

  // -- 2. selection over this layer's prototypes (sum / bs)
  if (use_f) {
    const int n_scored = rule == SD_RULE_REFERENCE ? 1 : nb;
    if constexpr (kCands) {
      // precomputed top-k (rank order) over every block but the current one,
      // whose sum changed above.  The current block is attended anyway, so
      // scoring it can only push the k-th candidate out of the top-k: one
      // comparison gives the same set as scoring every block here.
      if (threadIdx.x < 32) {
        // the current block's score, summed in the same order as the
        // in-kernel scoring (cta_score_topk) so both paths agree bit for bit
        const int lane = threadIdx.x;
        const float4 fq = reinterpret_cast<const float4 *>(X.f)[lane & 15];
        const float4 pr = reinterpret_cast<const float4 *>(pre_app ? X.pold : X.pnew)[lane & 15];
        float p = 0.f;
        p = fmaf(fq.x, pr.x, p);
        p = fmaf(fq.y, pr.y, p);
        p = fmaf(fq.z, pr.z, p);
        p = fmaf(fq.w, pr.w, p);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
        const bool cur_scored = curr < n_scored && !(pre_app && pos % bs == 0);
        const float vcur = cur_scored ? p * sel_scale : -INFINITY;
        bool displaced = false;
        for (int r = lane; r < kk; r += 32) {
          // the candidates read in phase 0 (rank r = lane; kk > 32 reads the rest)
          int j = early_cands ? cj : cand_idx[bh * top_k + r];
          float v = early_cands ? cv : cand_val[bh * top_k + r];
          if (j < 0 || j >= nb || j == curr) {
            j = -1;
            v = -INFINITY;
          }
          if (r == kk - 1 && (j < 0 || better(vcur, curr, v, j))) {  // displaced by the current block
            j = -1;
            displaced = true;
          }
          X.tk[r] = j;
        }
        // the displaced candidate's tile (staged in phase 0) is not attended
        if (__any_sync(0xffffffffu, displaced) && lane == 0 && disp_t >= 0) S.tile_n[disp_t] = 0;
      }
      attn_sync();
    } else if (kk <= 32) {  // in-kernel selection (no candidates passed)
      __shared__ float asv[kWarps * 32];
      __shared__ int asi[kWarps * 32];
      const float4 fq = reinterpret_cast<const float4 *>(X.f)[threadIdx.x & 15];
      const float *gsum = proto_sum + bh * NBcap * kD;
      const float *cur_row = pre_app ? X.pold : X.pnew;
      const int excl = pre_app && pos % bs == 0 ? curr : -1;  // a block the token opens is not scored yet
      if (nstage > 0) {
        if (!mbar_wait_bounded(&proto_bar, 0)) {
          report(err, SD_KERR_TIMEOUT);
          mbar_wait_bounded(&proto_bar, 0);  // let the copy land before the region is reused
        }
        const float *kh = ProtoStage<T>::k_half(S), *vh = ProtoStage<T>::v_half(S);
        auto prow = [&](int j) -> const float * {
          if (j < nstage)
            return j < ProtoStage<T>::kRowsPerHalf ? kh + j * kD : vh + (j - ProtoStage<T>::kRowsPerHalf) * kD;
          return j == curr ? cur_row : gsum + static_cast<int64_t>(j) * kD;
        };
        group_score_topk(prow, fq, nb, n_scored, excl, sel_scale, kk, X.tk, nullptr, asv, asi, ag);
        // the region is refilled with tiles by the async proxy next
        if (threadIdx.x == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      } else {
        group_score_topk([&](int j) { return j == curr ? cur_row : gsum + static_cast<int64_t>(j) * kD; }, fq, nb,
                         n_scored, excl, sel_scale, kk, X.tk, nullptr, asv, asi, ag);
      }
    } else {
      // top_k > 32: never launched with scoring warps, so the CTA is the
      // attention warps and CTA-wide helpers apply
      score_blocks(proto_sum + bh * NBcap * kD, kD, kD, X.f, n_scored, sel_scale, X.sc);
      __syncthreads();
      if (pre_app && curr < n_scored && threadIdx.x < 32) {  // the current block's pre-append score
        const int lane = threadIdx.x;
        const float4 fq = reinterpret_cast<const float4 *>(X.f)[lane & 15];
        const float4 pr = reinterpret_cast<const float4 *>(X.pold)[lane & 15];
        float p = 0.f;
        p = fmaf(fq.x, pr.x, p);
        p = fmaf(fq.y, pr.y, p);
        p = fmaf(fq.z, pr.z, p);
        p = fmaf(fq.w, pr.w, p);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
        if (lane == 0) X.sc[curr] = pos % bs == 0 ? -INFINITY : p * sel_scale;
      }
      __syncthreads();
      cta_topk([&](int j) { return j < n_scored ? X.sc[j] : -INFINITY; }, nb, kk, X.tk);
    }
    // in-kernel selection: tiles of the chosen blocks other than the sink and
    // the current block (already staged), in rank order, placed by one warp
    if (!early_cands && one_tile && kk <= 32) {
      if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int j = lane < kk ? X.tk[lane] : -1;
        const int cs = slots && lane < kk ? sm.cand_slot[bh * top_k + lane] : 0;
        const bool valid = j > 0 && j < nb && j != curr && cs >= 0 && (!slots || cs < sm.kslots);
        const unsigned same = __match_any_sync(0xffffffffu, valid ? j : -1 - lane);
        const bool keep = valid && (__ffs(same) - 1) == lane;
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        const int base = ntiles;
        if (keep) {
          const int slot = base + __popc(bal & ((1u << lane) - 1u));
          const int64_t n = L - static_cast<int64_t>(j) * bs;
          S.tile_tok[slot] = (slots ? 2 + cs : j) * bs;
          S.tile_n[slot] = static_cast<int>(n < bs ? n : bs);
        }
        __syncwarp();
        if (lane == 0) ntiles = base + __popc(bal);
      }
    } else if (!one_tile && threadIdx.x == 0) {
      count = assemble_decode_list(true, X.tk, kk, nb, curr, top_k, X.list);
      ntiles = build_tiles(X.list, count, L, bs, S.tile_tok, S.tile_n, ntiles, 0, curr);
    } else if (one_tile && kk > 32 && threadIdx.x == 0) {
      count = assemble_decode_list(true, X.tk, kk, nb, curr, top_k, X.list);
      ntiles = build_tiles(X.list, count, L, bs, S.tile_tok, S.tile_n, ntiles, 0, curr);
    }
  }
  if (threadIdx.x == 0) {  // the tile holding the new token gets its rows patched
    patch_t = -1;
    if (one_tile) {  // the current block's single tile
      patch_t = use_f ? (curr != 0 ? 1 : 0) : (nb <= ms ? curr : ntiles - 1);
      patch_row = static_cast<int>(pos - static_cast<int64_t>(curr) * bs);
    } else {
      for (int t = 0; t < ntiles; ++t)
        if (S.tile_tok[t] <= pos && pos < S.tile_tok[t] + S.tile_n[t]) {
          patch_t = t;
          patch_row = static_cast<int>(pos - S.tile_tok[t]);
        }
    }
  }
  attn_sync();

  // -- 3. attention over the selected blocks
  T *o = out + b * o_sb + static_cast<int64_t>(h * G) * kD;
  bool ok;
  if constexpr (is16<T>()) {
    ok = attend_mma<T, G>(S, ntiles, pre, tma, scale_log2, o, kD, patch_t, patch_row);
  } else {
    ok = attend_simt<T, G>(S, ntiles, pre, bulk, scale_log2, o, kD, patch_t, patch_row);
  }
  if (!ok) report(err, SD_KERR_TIMEOUT);

  // -- 4. optional: the selected block list, ascending (inspection only)
  if (sel_out) {
    if (threadIdx.x == 0) {
      if (use_f) {
        count = assemble_decode_list(true, X.tk, kk, nb, curr, top_k, X.list);
      } else if (nb <= ms) {
        for (int j = 0; j < nb; ++j) X.list[j] = j;
        count = nb;
      } else {
        count = assemble_decode_list(false, nullptr, 0, nb, curr, top_k, X.list);
      }
    }
    attn_sync();
    for (int i = threadIdx.x; i < sel_cap; i += kThreads) sel_out[bh * sel_cap + i] = i < count ? X.list[i] : -1;
    if (threadIdx.x == 0) cnt_out[bh] = count;
  }
}

template <typename T>
int make_maps(CUtensorMap *mk, CUtensorMap *mv, const void *kc, const void *vc, int64_t B, int64_t H, int64_t T_,
              int64_t st, int64_t sh, int64_t sb) {
  memset(mk, 0, sizeof(CUtensorMap));
  memset(mv, 0, sizeof(CUtensorMap));
  if constexpr (!is16<T>()) {
    return SD_OK;
  } else {
    const int dt = std::is_same<T, __nv_bfloat16>::value ? SD_DTYPE_BF16 : SD_DTYPE_F16;
    int r = encode_rows_map(mk, kc, dt, kD, T_, H, B, st, sh, sb, kRows);
    if (r == SD_OK) r = encode_rows_map(mv, vc, dt, kD, T_, H, B, st, sh, sb, kRows);
    return r;
  }
}

template <typename T, int G>
int launch_decode_attention(const void *q, int64_t B, int64_t Hkv, int64_t q_sb, int64_t q_sh, const void *kc,
                            const void *vc, int64_t c_sb, int64_t c_sh, int64_t c_st, int64_t Tcap,
                            const int32_t *sel, const int32_t *cnt, int ms_cap, int64_t L, int bs, float scale,
                            void *out, int64_t o_sb, int64_t o_sh, int32_t *err, cudaStream_t s) {
  const size_t smem = AttnSmem<T, G>::bytes() + sizeof(int) * ms_cap + kAlignSlack;
  // the tensor-core path needs contiguous rows laid out [B][H][T] in memory order
  const bool tma = is16<T>() && c_st == kD && c_sh >= Tcap * kD && c_sb >= Hkv * c_sh;
  CUtensorMap mk, mv;
  int r = tma ? make_maps<T>(&mk, &mv, kc, vc, B, Hkv, Tcap, c_st, c_sh, c_sb)
              : make_maps<float>(&mk, &mv, kc, vc, B, Hkv, Tcap, c_st, c_sh, c_sb);
  if (r != SD_OK) return r;
  const dim3 grid(static_cast<unsigned>(B * Hkv));
  if constexpr (is16<T>()) {
    if (tma) {
      auto kern = decode_attention_kernel<T, G, true>;
      if (set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
      kern<<<grid, kThreads, smem, s>>>(static_cast<const T *>(q), (int)Hkv, q_sb, q_sh,
                                        static_cast<const T *>(kc), static_cast<const T *>(vc), c_sb, c_sh, c_st, mk,
                                        mv, sel, cnt, ms_cap, L, bs, scale * kLog2e, static_cast<T *>(out), o_sb,
                                        o_sh, err);
      return check_launch();
    }
  }
  {
    auto kern = decode_attention_kernel<T, G, false>;
    if (set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
    kern<<<grid, kThreads, smem, s>>>(static_cast<const T *>(q), (int)Hkv, q_sb, q_sh, static_cast<const T *>(kc),
                                      static_cast<const T *>(vc), c_sb, c_sh, c_st, mk, mv, sel, cnt, ms_cap, L, bs,
                                      scale * kLog2e, static_cast<T *>(out), o_sb, o_sh, err);
  }
  return check_launch();
}

template <typename T, typename F, int G>
int launch_decode_layer(const void *qkv, int64_t qkv_sb, const void *fc, int64_t f_sb, const float *rc,
                        const float *rs, const int32_t *cur_len, void *kc, void *vc, float *ps, int64_t B,
                        int64_t Hkv, int64_t Tcap, int64_t NBcap, int bs, int top_k, int rule, float scale,
                        void *out, int64_t o_sb, const int32_t *cand_idx, const float *cand_val,
                        int32_t *sel_out, int32_t *cnt_out, int sel_cap, int32_t *err, cudaStream_t s,
                        const SlotMap<T> &sm = SlotMap<T>(), const NextCand &nx = NextCand()) {
  const size_t smem = AttnSmem<T, G>::bytes() + LayerTail::bytes(NBcap, top_k) + kAlignSlack;
  CUtensorMap mk, mv;
  const int r = make_maps<T>(&mk, &mv, kc, vc, B, Hkv, Tcap, kD, Tcap * kD, Hkv * Tcap * kD);
  if (r != SD_OK) return r;
  auto kern = cand_idx != nullptr ? decode_layer_kernel<T, F, G, true> : decode_layer_kernel<T, F, G, false>;
  if (set_max_smem(kern, smem) != SD_OK) return SD_ERR_CUDA;
  // the next layer's candidates come from a second group of kThreads threads
  const unsigned threads = nx.proto != nullptr ? 2 * kThreads : kThreads;
  // offloaded caches depend on a prefetch joined through an event: no early start
  const bool pdl = pdl_enabled() && sm.host_k == nullptr;
  return launch(kern, dim3(static_cast<unsigned>(B * Hkv)), dim3(threads), smem, s, pdl,
                static_cast<const T *>(qkv), qkv_sb, static_cast<const F *>(fc), f_sb, rc, rs, cur_len,
                static_cast<T *>(kc), static_cast<T *>(vc), ps, (int)Hkv, Tcap, NBcap, bs, top_k, rule,
                scale / static_cast<float>(bs), scale * kLog2e, mk, mv, static_cast<T *>(out), o_sb, cand_idx,
                cand_val, sel_out, cnt_out, sel_cap, err, sm, nx);
}

}  // namespace sd

#define SD_DISPATCH_G(G, ...)                             \
  switch (G) {                                            \
    case 1: { constexpr int GG = 1; __VA_ARGS__; } break; \
    case 2: { constexpr int GG = 2; __VA_ARGS__; } break; \
    case 3: { constexpr int GG = 3; __VA_ARGS__; } break; \
    case 4: { constexpr int GG = 4; __VA_ARGS__; } break; \
    case 6: { constexpr int GG = 6; __VA_ARGS__; } break; \
    case 8: { constexpr int GG = 8; __VA_ARGS__; } break; \
    default: return SD_ERR_UNSUPPORTED;                   \
  }

extern "C" int sd_decode_attention(const void *q, int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                   int64_t q_sb, int64_t q_sh, const void *k_cache, const void *v_cache,
                                   int64_t c_sb, int64_t c_sh, int64_t c_st, int64_t Tcap, const int32_t *sel,
                                   const int32_t *cnt, int ms_cap, int64_t seq_len_k, int block_size, float scale,
                                   void *out, int64_t o_sb, int64_t o_sh, int32_t *err, void *stream) {
  if (!q || !k_cache || !v_cache || !sel || !cnt || !out) return SD_ERR_INVALID;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || seq_len_k <= 0 || seq_len_k > Tcap || block_size <= 0 ||
      ms_cap <= 0)
    return SD_ERR_INVALID;
  if (D != sd::kD || B * Hkv > 0x7fffffff || B > 0x7fffffff / 2) return SD_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(ms_cap) * ((block_size + sd::kRows - 1) / sd::kRows) > sd::kMaxTiles)
    return SD_ERR_UNSUPPORTED;
  const int es = sd::dtype_size(dtype);
  if (!sd::aligned16(k_cache) || !sd::aligned16(v_cache) || (c_sb * es) % 16 || (c_sh * es) % 16 ||
      (c_st * es) % 16)
    return SD_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int G = static_cast<int>(Hq / Hkv);
  SD_DISPATCH_DTYPE(dtype, E, {
    SD_DISPATCH_G(G, return sd::launch_decode_attention<E, GG>(q, B, Hkv, q_sb, q_sh, k_cache, v_cache, c_sb, c_sh,
                                                                c_st, Tcap, sel, cnt, ms_cap, seq_len_k,
                                                                block_size, scale, out, o_sb, o_sh, err, s));
  });
  return SD_OK;
}

extern "C" int sd_decode_layer(const void *qkv, int dtype, int64_t qkv_sb, const void *forecast, int f_dtype,
                               int64_t f_sb, const float *rope_cos, const float *rope_sin, int64_t max_pos,
                               const int32_t *cur_len, void *k_cache, void *v_cache, float *proto_sum, int64_t B,
                               int64_t Hq, int64_t Hkv, int64_t D, int64_t Tcap, int64_t NBcap, int block_size,
                               int top_k, int rule, float scale, void *out, int64_t o_sb, const int32_t *cand_idx,
                               const float *cand_val, int32_t *sel_out, int32_t *cnt_out, int sel_cap,
                               int32_t *err, const float *next_proto_sum, const void *next_forecast,
                               int64_t next_f_sb, int32_t *next_cand_idx, float *next_cand_val, void *stream) {
  if (!qkv || !rope_cos || !rope_sin || !cur_len || !k_cache || !v_cache || !proto_sum || !out)
    return SD_ERR_INVALID;
  sd::NextCand nx;
  if (next_proto_sum != nullptr) {
    if (!next_forecast || !next_cand_idx || !next_cand_val) return SD_ERR_INVALID;
    if (top_k > 32) return SD_ERR_UNSUPPORTED;
    if (!sd::aligned16(next_proto_sum)) return SD_ERR_ALIGN;
    nx.proto = next_proto_sum;
    nx.fc = next_forecast;
    nx.f_sb = next_f_sb;
    nx.cand_idx = next_cand_idx;
    nx.cand_val = next_cand_val;
  }
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || block_size <= 0 || top_k <= 0 || Tcap <= 0 || NBcap <= 0 ||
      max_pos < Tcap)
    return SD_ERR_INVALID;
  const int base_rule = rule & ~SD_SELECT_BEFORE_APPEND;
  if (base_rule != SD_RULE_REFERENCE && base_rule != SD_RULE_ABSOLUTE) return SD_ERR_INVALID;
  if (NBcap * block_size < Tcap) return SD_ERR_INVALID;
  if ((sel_out == nullptr) != (cnt_out == nullptr) || (sel_out && sel_cap < top_k + 2)) return SD_ERR_INVALID;
  if ((cand_idx == nullptr) != (cand_val == nullptr)) return SD_ERR_INVALID;
  if (D != sd::kD || top_k > 64 || NBcap > 16384 || B * Hkv > 0x7fffffff) return SD_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(top_k + 2) * ((block_size + sd::kRows - 1) / sd::kRows) > sd::kMaxTiles)
    return SD_ERR_UNSUPPORTED;
  if (!sd::aligned16(k_cache) || !sd::aligned16(v_cache) || !sd::aligned16(proto_sum)) return SD_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int G = static_cast<int>(Hq / Hkv);
  const int fdt = forecast ? f_dtype : dtype;
  SD_DISPATCH_DTYPE(dtype, E, {
    if (fdt == dtype) {
      SD_DISPATCH_G(G, return sd::launch_decode_layer<E, E, GG>(qkv, qkv_sb, forecast, f_sb, rope_cos, rope_sin,
                                                                cur_len, k_cache, v_cache, proto_sum, B, Hkv,
                                                                Tcap, NBcap, block_size, top_k, rule, scale, out,
                                                                o_sb, cand_idx, cand_val, sel_out, cnt_out,
                                                                sel_cap, err, s, sd::SlotMap<E>(), nx));
    } else if (fdt == SD_DTYPE_F32) {
      SD_DISPATCH_G(G, return sd::launch_decode_layer<E, float, GG>(
                           qkv, qkv_sb, forecast, f_sb, rope_cos, rope_sin, cur_len, k_cache, v_cache, proto_sum,
                           B, Hkv, Tcap, NBcap, block_size, top_k, rule, scale, out, o_sb, cand_idx, cand_val,
                           sel_out, cnt_out, sel_cap, err, s, sd::SlotMap<E>(), nx));
    } else {
      return SD_ERR_UNSUPPORTED;
    }
  });
  return SD_OK;
}

extern "C" int sd_decode_layer_offload(const void *qkv, int dtype, int64_t qkv_sb, const void *forecast,
                                       int f_dtype, int64_t f_sb, const float *rope_cos, const float *rope_sin,
                                       int64_t max_pos, const int32_t *cur_len, void *host_k, void *host_v,
                                       int64_t host_tcap, void *slot_k, void *slot_v, int kslots, float *proto_sum,
                                       int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t NBcap, int block_size,
                                       int top_k, int rule, float scale, void *out, int64_t o_sb,
                                       const int32_t *cand_idx, const float *cand_val, const int32_t *cand_slot,
                                       int32_t *sel_out, int32_t *cnt_out, int sel_cap, int32_t *err,
                                       void *stream) {
  if (!qkv || !rope_cos || !rope_sin || !cur_len || !host_k || !host_v || !slot_k || !slot_v || !proto_sum || !out)
    return SD_ERR_INVALID;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || top_k <= 0 || host_tcap <= 0 || NBcap <= 0 ||
      max_pos < host_tcap)
    return SD_ERR_INVALID;
  const int base_rule = rule & ~SD_SELECT_BEFORE_APPEND;
  if (base_rule != SD_RULE_REFERENCE && base_rule != SD_RULE_ABSOLUTE) return SD_ERR_INVALID;
  if (NBcap * block_size < host_tcap) return SD_ERR_INVALID;
  if ((sel_out == nullptr) != (cnt_out == nullptr) || (sel_out && sel_cap < top_k + 2)) return SD_ERR_INVALID;
  // the slots only hold what a prefetch staged: forecast steps need the
  // prefetched candidates (and their slots), never in-kernel selection
  if ((cand_idx == nullptr) != (cand_val == nullptr) || (cand_idx == nullptr) != (cand_slot == nullptr))
    return SD_ERR_INVALID;
  if (forecast != nullptr && cand_idx == nullptr) return SD_ERR_INVALID;
  if (D != sd::kD || block_size != sd::kRows || kslots < top_k || kslots > 32 || top_k > 31 || NBcap > 16384 ||
      B * Hkv > 0x7fffffff)
    return SD_ERR_UNSUPPORTED;
  if (!sd::aligned16(slot_k) || !sd::aligned16(slot_v) || !sd::aligned16(proto_sum)) return SD_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int G = static_cast<int>(Hq / Hkv);
  const int fdt = forecast ? f_dtype : dtype;
  const int64_t tslot = static_cast<int64_t>(kslots + 2) * block_size;
  SD_DISPATCH_DTYPE(dtype, E, {
    sd::SlotMap<E> sm;
    sm.host_k = static_cast<E *>(host_k);
    sm.host_v = static_cast<E *>(host_v);
    sm.host_tcap = host_tcap;
    sm.cand_slot = cand_slot;
    sm.kslots = kslots;
    if (fdt == dtype) {
      SD_DISPATCH_G(G, return sd::launch_decode_layer<E, E, GG>(qkv, qkv_sb, forecast, f_sb, rope_cos, rope_sin,
                                                                cur_len, slot_k, slot_v, proto_sum, B, Hkv, tslot,
                                                                NBcap, block_size, top_k, rule, scale, out, o_sb,
                                                                cand_idx, cand_val, sel_out, cnt_out, sel_cap, err,
                                                                s, sm));
    } else if (fdt == SD_DTYPE_F32) {
      SD_DISPATCH_G(G, return sd::launch_decode_layer<E, float, GG>(
                           qkv, qkv_sb, forecast, f_sb, rope_cos, rope_sin, cur_len, slot_k, slot_v, proto_sum, B,
                           Hkv, tslot, NBcap, block_size, top_k, rule, scale, out, o_sb, cand_idx, cand_val,
                           sel_out, cnt_out, sel_cap, err, s, sm));
    } else {
      return SD_ERR_UNSUPPORTED;
    }
  });
  return SD_OK;
}
