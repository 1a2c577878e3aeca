// Forecast-guided KV prefetch for offloaded caches
// (model/attention/async_offload.py:55-112 and :170-294).
//
// The authoritative K/V rows of an offloaded layer live in pinned host memory,
// block-major [B, Hkv, Tcap, 64], which the GPU reads and writes directly over
// the host link (unified addressing; no staging copy on the host, no host
// round trip for the block indices).  Each (sequence, kv head) owns a device
// slot buffer of 2 + kslots blocks of 64 rows:
//   slot 0        the sink block 0 (loaded once it is complete),
//   slot 1        the block the next tokens are appended to,
//   slots 2..     the blocks this step attends to besides those two.
// One CTA per (sequence, kv head) decides which wanted blocks are already
// resident (hits keep their slot; in forecast mode a block can sit in any
// slot, in static/dense mode block j always uses slot 2 + j % kslots), copies
// the missing ones host -> device with 16-byte loads spread over the CTA, and
// records hit/miss/byte counts.  With more slots than candidates
// (kslots > top_k) the slots form a block cache: a block stays resident until
// its slot is needed, and a miss takes the free slot used least recently (the
// position of its last use is kept per slot).  It runs on a side stream during the previous
// layer, right after the candidate kernel that chose the blocks.
#include "sd_common.cuh"

namespace sd {

constexpr int kPfThreads = 128;
constexpr int kBlockRows = 64;
constexpr int kHd = 64;

template <typename T>
__global__ void __launch_bounds__(kPfThreads)
    offload_prefetch_kernel(const T *host_k, const T *host_v, int64_t host_tcap, T *__restrict__ slot_k,
                            T *__restrict__ slot_v, int kslots, const int32_t *__restrict__ cur_len, int top_k,
                            const int32_t *__restrict__ cand_idx, int32_t *__restrict__ slot_block,
                            int32_t *__restrict__ cand_slot, unsigned long long *__restrict__ stats) {
  __shared__ int miss_block[33], miss_slot[33], nmiss, nwant, nhit;
  const int bh = blockIdx.x;
  const int64_t pos = *cur_len;  // position the next token takes
  // per (sequence, kv head): block of each slot, the sink flag, then the
  // position each slot was last used at
  int32_t *sb = slot_block + static_cast<int64_t>(bh) * (2 * kslots + 1);
  int32_t *sage = sb + kslots + 1;
  __shared__ int slot_of_rank[32];
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int nm = 0, want = 0, hit = 0;
    if (pos >= 0 && pos < host_tcap) {
      const int curr = static_cast<int>(pos / kBlockRows);
      const int nb = curr + 1;
      const int ms = nb < top_k + 2 ? nb : top_k + 2;
      const int prev = lane < kslots ? sb[lane] : -2;
      if (cand_idx != nullptr && nb > ms) {
        // forecast mode: wanted = this step's candidates other than 0 and curr
        const int w = lane < top_k ? cand_idx[static_cast<int64_t>(bh) * top_k + lane] : -1;
        const bool valid = w > 0 && w < curr;
        int hs = -1;
        bool keep = false;
        for (int i = 0; i < kslots; ++i) {
          const int pi = __shfl_sync(0xffffffffu, prev, i);
          const int wi = __shfl_sync(0xffffffffu, w, i < top_k ? i : 0);
          if (valid && pi == w) hs = i;
          // slot `lane` keeps its block when some valid candidate wants it
          if (i < top_k && wi > 0 && wi < curr && wi == prev) keep = true;
        }
        const bool is_free = lane < kslots && !keep;
        // rank of each free slot by (last use, slot): the m-th miss takes the
        // free slot of rank m, the least recently used first (there are at
        // least as many free slots as misses: kslots >= top_k and a block
        // occupies one slot)
        const int age = lane < kslots ? sage[lane] : 0;
        int rank = 0;
        for (int i = 0; i < kslots; ++i) {
          const int ai = __shfl_sync(0xffffffffu, age, i);
          const bool fi = __shfl_sync(0xffffffffu, is_free, i);
          if (fi && (ai < age || (ai == age && i < lane))) ++rank;
        }
        if (is_free) slot_of_rank[rank] = lane;
        __syncwarp();
        const bool need = valid && hs < 0;
        const int m = __popc(__ballot_sync(0xffffffffu, need) & ((1u << lane) - 1u));
        const bool miss = need;
        const unsigned missm = __ballot_sync(0xffffffffu, miss);
        int slot = hs;
        if (miss) {
          slot = slot_of_rank[m];
          miss_block[m] = w;
          miss_slot[m] = 2 + slot;
          sb[slot] = w;
        }
        // every slot used this step (hits and fills) is stamped with the position
        if (valid && slot >= 0) sage[slot] = static_cast<int>(pos);
        if (lane < top_k) cand_slot[static_cast<int64_t>(bh) * top_k + lane] = valid ? slot : -1;
        nm = __popc(missm);
        want = __popc(__ballot_sync(0xffffffffu, valid));
        hit = __popc(__ballot_sync(0xffffffffu, valid && hs >= 0));
      } else {
        // static window or dense step: block j lives in slot 2 + j % kslots
        const int lo = nb <= ms ? 1 : (curr - top_k + 1 > 1 ? curr - top_k + 1 : 1);
        const int cnt = curr - lo > 0 ? curr - lo : 0;  // blocks lo..curr-1
        const int w = lo + lane;
        const bool valid = lane < cnt && lane < kslots;
        const int s = valid ? w % kslots : 0;
        const bool miss = valid && sb[s] != w;
        const unsigned missm = __ballot_sync(0xffffffffu, miss);
        __syncwarp();
        if (miss) {
          const int m = __popc(missm & ((1u << lane) - 1u));
          miss_block[m] = w;
          miss_slot[m] = 2 + s;
          sb[s] = w;
        }
        if (cand_slot != nullptr && lane < top_k) cand_slot[static_cast<int64_t>(bh) * top_k + lane] = -1;
        nm = __popc(missm);
        want = __popc(__ballot_sync(0xffffffffu, valid));
        hit = want - nm;
      }
      // the sink block, once complete, is loaded into slot 0 once
      if (curr >= 1 && sb[kslots] != 0) {
        __syncwarp();
        if (lane == 0) {
          miss_block[nm] = 0;
          miss_slot[nm] = 0;
          sb[kslots] = 0;
        }
        ++nm;
      }
    }
    if (lane == 0) {
      nmiss = nm;
      nwant = want;
      nhit = hit;
    }
  }
  __syncthreads();
  const int nm = nmiss;
  if (threadIdx.x == 0 && stats != nullptr) {
    atomicAdd(&stats[0], static_cast<unsigned long long>(nwant));
    atomicAdd(&stats[1], static_cast<unsigned long long>(nhit));
    atomicAdd(&stats[2], static_cast<unsigned long long>(nm) * 2ull * kBlockRows * kHd * sizeof(T));
  }
  // copy the missing blocks: 64 rows x 64 values of K and of V per block
  constexpr int kVec = kBlockRows * kHd * static_cast<int>(sizeof(T)) / 16;  // uint4 per tensor per block
  const int64_t tslot = static_cast<int64_t>(kslots + 2) * kBlockRows;
  const int total = nm * 2 * kVec;
  constexpr int kUnroll = 8;
  for (int e0 = threadIdx.x; e0 < total; e0 += kPfThreads * kUnroll) {
    uint4 buf[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int e = e0 + u * kPfThreads;
      if (e < total) {
        const int m = e / (2 * kVec), r = e - m * 2 * kVec;
        const int which = r / kVec, c = r - which * kVec;
        const T *src = (which ? host_v : host_k) +
                       (static_cast<int64_t>(bh) * host_tcap + static_cast<int64_t>(miss_block[m]) * kBlockRows) * kHd;
        buf[u] = reinterpret_cast<const uint4 *>(src)[c];
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int e = e0 + u * kPfThreads;
      if (e < total) {
        const int m = e / (2 * kVec), r = e - m * 2 * kVec;
        const int which = r / kVec, c = r - which * kVec;
        T *dst = (which ? slot_v : slot_k) + (static_cast<int64_t>(bh) * tslot + miss_slot[m] * kBlockRows) * kHd;
        reinterpret_cast<uint4 *>(dst)[c] = buf[u];
      }
    }
  }
}

}  // namespace sd

extern "C" int sd_offload_prefetch(const void *host_k, const void *host_v, int dtype, int64_t B, int64_t Hkv,
                                   int64_t D, int64_t host_tcap, void *slot_k, void *slot_v, int kslots,
                                   const int32_t *cur_len, int block_size, int top_k, const int32_t *cand_idx,
                                   int32_t *slot_block, int32_t *cand_slot, unsigned long long *stats,
                                   void *stream) {
  if (!host_k || !host_v || !slot_k || !slot_v || !cur_len || !slot_block || B <= 0 || Hkv <= 0 ||
      host_tcap <= 0 || top_k <= 0)
    return SD_ERR_INVALID;
  if (cand_idx != nullptr && cand_slot == nullptr) return SD_ERR_INVALID;
  if (D != sd::kHd || block_size != sd::kBlockRows || kslots < top_k || kslots > 32 || top_k > 31 ||
      host_tcap % block_size || B * Hkv > 0x7fffffff)
    return SD_ERR_UNSUPPORTED;
  if (!sd::aligned16(host_k) || !sd::aligned16(host_v) || !sd::aligned16(slot_k) || !sd::aligned16(slot_v))
    return SD_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(B * Hkv);
  switch (dtype) {
    case SD_DTYPE_BF16:
      sd::offload_prefetch_kernel<__nv_bfloat16><<<grid, sd::kPfThreads, 0, s>>>(
          static_cast<const __nv_bfloat16 *>(host_k), static_cast<const __nv_bfloat16 *>(host_v), host_tcap,
          static_cast<__nv_bfloat16 *>(slot_k), static_cast<__nv_bfloat16 *>(slot_v), kslots, cur_len, top_k,
          cand_idx, slot_block, cand_slot, stats);
      break;
    case SD_DTYPE_F16:
      sd::offload_prefetch_kernel<__half><<<grid, sd::kPfThreads, 0, s>>>(
          static_cast<const __half *>(host_k), static_cast<const __half *>(host_v), host_tcap,
          static_cast<__half *>(slot_k), static_cast<__half *>(slot_v), kslots, cur_len, top_k, cand_idx,
          slot_block, cand_slot, stats);
      break;
    case SD_DTYPE_F32:
      sd::offload_prefetch_kernel<float><<<grid, sd::kPfThreads, 0, s>>>(
          static_cast<const float *>(host_k), static_cast<const float *>(host_v), host_tcap,
          static_cast<float *>(slot_k), static_cast<float *>(slot_v), kslots, cur_len, top_k, cand_idx, slot_block,
          cand_slot, stats);
      break;
    default:
      return SD_ERR_INVALID;
  }
  return sd::check_launch();
}
