// Unfused block-sparse decode (sd_decode_select, then sd_decode_attention)
// with the selected-block lists kept in a fixed device array of this library
// instead of buffers the caller allocates.
//
// Who needs it: callers that must not allocate device memory per call and
// have no device allocator of their own -- a host binding through this C ABI
// alone (ctypes, cgo, JNI) with no tensor library behind it, or a runtime
// that forbids allocation on its serving path.  Those callers would otherwise
// have to manage the int32 [B,Hkv,ms] list and [B,Hkv] count buffers that
// pass between the two kernels.
//
// The scratch is two file-scope __device__ arrays of fixed size (1 MiB of
// lists for up to kMaxPairs (sequence, kv head) pairs with up to kMaxList
// entries each, plus 16 KiB of counts), one copy per device.  Their device
// addresses are looked up once per device (cudaGetSymbolAddress, with that
// device current) on the first call and cached.  Nothing in them needs to
// start at zero: the selection kernel writes every list slot and every count
// of the call before the attention kernel reads them.
//
// Calls share the scratch, so two calls whose kernels may overlap on the GPU
// (different streams without ordering between them, or different host
// threads on one device) race on it; calls on one stream are ordered.
#include <mutex>

#include "sd_common.cuh"  // declares sd_decode_select and sd_decode_attention, which this chains

namespace sd {
namespace {

constexpr int64_t kMaxPairs = 4096;  // B * Hkv
constexpr int kMaxList = 64;         // selected blocks per pair: min(N_b, top_k + 2)
constexpr int kMaxDevices = 64;

__device__ __align__(256) int32_t g_sel[kMaxPairs * kMaxList];
__device__ __align__(256) int32_t g_cnt[kMaxPairs];

struct Scratch {
  int32_t *sel = nullptr;
  int32_t *cnt = nullptr;
};
Scratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// The current device's scratch addresses; looked up on the first call per
// device (the lookup may load the module on that device, which a stream
// capture does not allow: make the first call before capturing).
int scratch_for_current_device(Scratch *out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return SD_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return SD_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  Scratch &s = g_scratch[dev];
  if (s.sel == nullptr) {
    void *ps = nullptr, *pc = nullptr;
    e = cudaGetSymbolAddress(&ps, g_sel);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&pc, g_cnt);
    if (e != cudaSuccess) {
      set_cuda_error(e);
      cudaGetLastError();
      return SD_ERR_CUDA;
    }
    s.sel = static_cast<int32_t *>(ps);
    s.cnt = static_cast<int32_t *>(pc);
  }
  *out = s;
  return SD_OK;
}

}  // namespace
}  // namespace sd

extern "C" int sd_decode_sparse_noalloc(const void *q, int dtype, int64_t q_sb, int64_t q_sh, const void *forecast,
                                        int f_dtype, int64_t f_sb, int64_t f_sh, const float *reps, int64_t r_sb,
                                        int64_t r_sn, int64_t r_sh, const void *k_cache, const void *v_cache,
                                        int64_t c_sb, int64_t c_sh, int64_t c_st, int64_t Tcap, int64_t B,
                                        int64_t Hq, int64_t Hkv, int64_t D, int64_t seq_len_k, int block_size,
                                        int top_k, int rule, float scale, void *out, int64_t o_sb, int64_t o_sh,
                                        int32_t *err, void *stream) {
  if (B <= 0 || Hkv <= 0 || seq_len_k <= 0 || block_size <= 0 || top_k <= 0) return SD_ERR_INVALID;
  const int64_t nb = (seq_len_k + block_size - 1) / block_size;
  const int64_t ms = nb < top_k + 2 ? nb : top_k + 2;
  // beyond the fixed scratch: the caller-buffer entry points have no such limit
  if (B * Hkv > sd::kMaxPairs || ms > sd::kMaxList) return SD_ERR_UNSUPPORTED;
  sd::Scratch sc;
  int r = sd::scratch_for_current_device(&sc);
  if (r != SD_OK) return r;
  r = sd_decode_select(forecast, f_dtype, f_sb, f_sh, reps, r_sb, r_sn, r_sh, B, Hkv, D, seq_len_k, block_size,
                       top_k, rule, sc.sel, sc.cnt, static_cast<int>(ms), stream);
  if (r != SD_OK) return r;
  return sd_decode_attention(q, dtype, B, Hq, Hkv, D, q_sb, q_sh, k_cache, v_cache, c_sb, c_sh, c_st, Tcap, sc.sel,
                             sc.cnt, static_cast<int>(ms), seq_len_k, block_size, scale, out, o_sb, o_sh, err,
                             stream);
}
