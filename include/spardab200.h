/*
 * spardab200.h - C ABI of the B200 (sm_100a) forecast-guided block-sparse
 * attention path.  Plain pointers and sizes only; every tensor is allocated by
 * the caller, and no entry point allocates device memory.
 *
 * Conventions
 *   - Strides are in ELEMENTS.  The innermost (head_dim) stride is always 1.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every call returns SD_OK (0) or a negative SD_ERR_* code; sd_strerror()
 *     turns it into text.  Arguments are validated on the host before launch.
 *   - Calls are asynchronous with respect to the host (stream-ordered) and
 *     re-entrant for distinct streams and devices.
 *   - `err` arguments (nullable) point to one device int32 that a kernel sets
 *     to a nonzero SD_KERR_* code when a bounded wait gives up; kernels never
 *     trap.
 *
 * Reference interfaces replaced (tyborra/local-research-Small-Language-Model):
 *   model/forecast.py            KVBlockCompressor.forward, ForecastBlockSelector.forward
 *   model/attention/sparse.py    gather_kv_blocks, SparseAttention._forward_decode_gather,
 *                                _forward_masked_sdpa, _forward_chunked_gather
 *   model/attention/base.py      KVCache.update
 *   model/attention/async_offload.py  AsyncOffloadedKVCache.async_transfer_selected_blocks,
 *                                AsyncForecastOffloadAttention.prefetch
 */
#ifndef SPARDAB200_H
#define SPARDAB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SD_API __attribute__((visibility("default")))
#else
#define SD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define SD_OK 0
#define SD_ERR_INVALID (-1)     /* bad shape, stride, pointer or value */
#define SD_ERR_UNSUPPORTED (-2) /* valid input outside what the kernels implement */
#define SD_ERR_CUDA (-3)        /* a CUDA runtime call or launch failed */
#define SD_ERR_ALIGN (-4)       /* a pointer or stride breaks the 16-byte rule of bulk copies */

/* ---- device-side error words (written to *err) ---- */
#define SD_KERR_TIMEOUT 1       /* a bounded mbarrier wait expired */
#define SD_KERR_BOUNDS 2        /* a device-side length was outside the cache capacity */

/* ---- element types ---- */
#define SD_DTYPE_F32 0
#define SD_DTYPE_BF16 1
#define SD_DTYPE_F16 2

/* ---- decode-time causal rules ----
 * SD_RULE_REFERENCE: the reference's literal rule.  The selector is called
 *   with one forecast row, so blocks j > 0 // block_size = 0 are masked to -inf
 *   (model/forecast.py:120-126 called from model/attention/sparse.py:139).
 * SD_RULE_ABSOLUTE: blocks after the block of the query's absolute position
 *   are masked (what the reference's masked prefill does for every row).
 * -inf (and other equal) scores are ordered by ascending block index. */
#define SD_RULE_REFERENCE 0
#define SD_RULE_ABSOLUTE 1

/* Selection timing, OR-ed into the `rule` of sd_decode_layer and
 * sd_decode_layer_offload.  Default (flag clear): blocks are scored after the
 * new token is appended, as SparseAttention and ForecastOffloadAttention do
 * (model/attention/sparse.py:133-139, offload.py:175-227).  With the flag: the
 * current block is scored with its sum before this step's token, and not at
 * all when the token opens it, as AsyncForecastOffloadAttention.prefetch does
 * (model/attention/async_offload.py:241-260, which selects one token ahead). */
#define SD_SELECT_BEFORE_APPEND 0x100

SD_API const char *sd_strerror(int code);
SD_API int sd_version(void);
/* cudaError_t of the last failing CUDA call made by this library on this thread. */
SD_API int sd_last_cuda_error(void);

/* K1 - block compressor.  Replaces KVBlockCompressor.forward
 * (model/forecast.py:57-78).  k: [B,T,H,D] with strides (sb, st, sh); writes
 * reps: fp32 [B,NB,H,D] contiguous, NB = ceil(T / block_size), each entry the
 * zero-padded block sum divided by block_size. */
SD_API int sd_compress_blocks(const void *k, int dtype, int64_t B, int64_t T, int64_t H, int64_t D,
                       int64_t sb, int64_t st, int64_t sh, int block_size, float *reps,
                       void *stream);

/* K2 - forecast block selector.  Replaces ForecastBlockSelector.forward
 * (model/forecast.py:89-130).  forecast: [B,Tq,H,D] (strides f_sb, f_st, f_sh),
 * reps: fp32 [B,NB,H,D] (strides r_sb, r_sn, r_sh).  scores = f.rep / sqrt(D)
 * in fp32; if causal, blocks j > (t + q_offset) // block_size are -inf
 * (q_offset = 0 is the reference).  Writes topk_idx int64 [B,H,Tq,k],
 * k = min(top_k, NB), sorted by score descending (ties: ascending index), and,
 * if scores != NULL, scores fp32 [B,H,Tq,NB].  D must be 16..256, a multiple of 4. */
SD_API int sd_select_blocks(const void *forecast, int f_dtype, int64_t B, int64_t Tq, int64_t H,
                     int64_t D, int64_t f_sb, int64_t f_st, int64_t f_sh, const float *reps,
                     int64_t NB, int64_t r_sb, int64_t r_sn, int64_t r_sh, int top_k,
                     int block_size, int causal, int64_t q_offset, float *scores,
                     int64_t *topk_idx, void *stream);

/* Top-k of fp32 rows, the ordering half of ForecastBlockSelector.forward
 * (model/forecast.py:128-129, torch.topk(largest=True, sorted=True)).
 * scores: [rows, n] with row stride ld; idx: int64 [rows, k]; vals (nullable):
 * fp32 [rows, k].  Ties (including -inf) in ascending index order. k <= 64. */
SD_API int sd_topk_rows(const float *scores, int64_t rows, int64_t n, int64_t ld, int k, int64_t *idx,
                 float *vals, void *stream);

/* K4 - block gather.  Replaces gather_kv_blocks (model/attention/sparse.py:19-62).
 * k, v: [B,H,T,D] with strides (sb, sh, st); idx: int64 [B,H,S];
 * k_out, v_out: [B,H,S*block_size,D] contiguous, rows at or past T are zero.
 * Indices outside [0, ceil(T/block_size)) produce zero rows. */
SD_API int sd_gather_kv_blocks(const void *k, const void *v, int dtype, int64_t B, int64_t H,
                        int64_t T, int64_t D, int64_t sb, int64_t sh, int64_t st,
                        const int64_t *idx, int64_t S, int block_size, void *k_out,
                        void *v_out, void *stream);

/* K3 - decode selected-set assembly.  Replaces model/attention/sparse.py:108-154
 * (and the identical blocks of offload.py:175-240): {0, curr} U top-k
 * (forecast != NULL) or the static window (forecast == NULL), future blocks
 * cleared, listed in ascending order.  When ceil(L/bs) <= min(NB, top_k+2) every
 * block is listed (the dense fallback, sparse.py:113-123).
 * forecast: [B,H,D] (strides f_sb, f_sh), reps fp32 [B,NB,H,D] (strides).
 * sel: int32 [B,H,ms_cap] (-1 padded), cnt: int32 [B,H].
 * seq_len_k = L (tokens in the cache, the new one included). */
SD_API int sd_decode_select(const void *forecast, int f_dtype, int64_t f_sb, int64_t f_sh,
                     const float *reps, int64_t r_sb, int64_t r_sn, int64_t r_sh, int64_t B,
                     int64_t H, int64_t D, int64_t seq_len_k, int block_size, int top_k,
                     int rule, int32_t *sel, int32_t *cnt, int ms_cap, void *stream);

/* K7 - block-sparse GQA decode attention.  Replaces the gather + mask +
 * repeat_interleave + SDPA of model/attention/sparse.py:156-181.
 * q: [B,Hq,D] (strides q_sb, q_sh); caches: [B,Hkv,Tcap,D] (strides c_sb, c_sh,
 * c_st, identical for K and V); sel/cnt as produced by sd_decode_select
 * (sel row stride ms_cap); keys = tokens of the listed blocks with pos < L.
 * Query head h reads kv head h / (Hq/Hkv).  out: [B,Hq,D] (strides o_sb, o_sh).
 * D = 64.  Selected K/V rows are staged into shared memory by bulk (TMA)
 * copies, which need 16-byte aligned rows. */
SD_API int sd_decode_attention(const void *q, int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                        int64_t D, int64_t q_sb, int64_t q_sh, const void *k_cache,
                        const void *v_cache, int64_t c_sb, int64_t c_sh, int64_t c_st,
                        int64_t Tcap, const int32_t *sel, const int32_t *cnt, int ms_cap,
                        int64_t seq_len_k, int block_size, float scale, void *out,
                        int64_t o_sb, int64_t o_sh, int32_t *err, void *stream);

/* sd_decode_select followed by sd_decode_attention without caller buffers:
 * the selected-block lists and counts live in a fixed device array of this
 * library (no device allocation in the call, no workspace argument).  No
 * counterpart in the reference (its decode allocates the lists as tensors,
 * model/attention/sparse.py:108-181); for callers that cannot allocate device
 * memory per call -- a host binding through this C ABI alone, or a serving
 * runtime that forbids allocation.  Arguments mean what they mean in the two
 * chained entry points (H of sd_decode_select = Hkv).  Limits of the fixed
 * scratch: B * Hkv <= 4096 and min(ceil(L / block_size), top_k + 2) <= 64,
 * else SD_ERR_UNSUPPORTED (the two chained entry points have no such limit).
 * The first call on a device looks up the scratch address with that device
 * current (make it before any stream capture); calls whose kernels may
 * overlap on one device (unordered streams, concurrent host threads) race on
 * the shared scratch. */
SD_API int sd_decode_sparse_noalloc(const void *q, int dtype, int64_t q_sb, int64_t q_sh, const void *forecast,
                                    int f_dtype, int64_t f_sb, int64_t f_sh, const float *reps, int64_t r_sb,
                                    int64_t r_sn, int64_t r_sh, const void *k_cache, const void *v_cache,
                                    int64_t c_sb, int64_t c_sh, int64_t c_st, int64_t Tcap, int64_t B, int64_t Hq,
                                    int64_t Hkv, int64_t D, int64_t seq_len_k, int block_size, int top_k, int rule,
                                    float scale, void *out, int64_t o_sb, int64_t o_sh, int32_t *err,
                                    void *stream);

/* KV-cache append with the compressor fused in.  Replaces KVCache.update
 * (model/attention/base.py:19-29) for the block-major cache of this library:
 * k_cache, v_cache [B,H,Tcap,D] contiguous, proto_sum fp32 [B,H,NBcap,D]
 * contiguous (running block sums; prototype = sum / block_size).
 * xk, xv: [B,T,H,D] with element strides (sb, st, sh) and (vsb, vst, vsh);
 * written at positions start .. start+T-1, then the sums of every touched
 * block are recomputed in fp32. */
SD_API int sd_kv_append(const void *xk, const void *xv, int dtype, int64_t B, int64_t T, int64_t H,
                 int64_t D, int64_t sb, int64_t st, int64_t sh, int64_t vsb, int64_t vst, int64_t vsh,
                 void *k_cache, void *v_cache, float *proto_sum, int64_t Tcap, int64_t NBcap, int64_t start,
                 int block_size, void *stream);

/* Fused decode layer: RoPE + KV append + compressor update + selection +
 * block-sparse attention, one CTA per (sequence, kv head).  Replaces
 * SparseAttention.forward for T == 1 (model/attention/sparse.py:366-410 with
 * _forward_decode_gather) from the point after the q/k/v projections.
 * qkv: [B, (Hq+2*Hkv)*D] rows with stride qkv_sb (q | k | v, pre-RoPE).
 * forecast (nullable): layer L-1's forecast [B,Hkv,D] with row stride f_sb.
 * rope_cos/sin: fp32 [max_pos, D/2].  cur_len: device int32, tokens cached
 * before this step (the new token is written at that position).
 * Caches as in sd_kv_append.  out: [B, Hq*D] rows with stride o_sb.
 * cand_idx/cand_val (nullable, together): candidates from
 * sd_decode_candidates for this step; without them the kernel scores every
 * prototype itself (same result).
 * sel_out/cnt_out (nullable, together): the selected block list of every
 * (sequence, kv head), int32 [B,Hkv,sel_cap] ascending and -1 padded, and its
 * length int32 [B,Hkv]; sel_cap >= top_k + 2.
 * next_* (nullable, together; top_k <= 32): the next layer's block sums, its
 * forecast rows (this layer's forecast projection, activation dtype, row
 * stride next_f_sb) and its candidate outputs [B,Hkv,top_k]: the kernel ends
 * by computing what sd_decode_candidates would for the next layer's coming
 * step, with no separate launch or stream.  The next layer's cache must have
 * this layer's geometry (B, Hkv, NBcap, head_dim, block_size): its sums are
 * indexed as [B,Hkv,NBcap,D] with this call's sizes, and nothing on the
 * device can check that. */
SD_API int sd_decode_layer(const void *qkv, int dtype, int64_t qkv_sb, const void *forecast,
                    int f_dtype, int64_t f_sb, const float *rope_cos, const float *rope_sin,
                    int64_t max_pos, const int32_t *cur_len, void *k_cache, void *v_cache,
                    float *proto_sum, int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                    int64_t Tcap, int64_t NBcap, int block_size, int top_k, int rule,
                    float scale, void *out, int64_t o_sb, const int32_t *cand_idx,
                    const float *cand_val, int32_t *sel_out, int32_t *cnt_out, int sel_cap,
                    int32_t *err, const float *next_proto_sum, const void *next_forecast,
                    int64_t next_f_sb, int32_t *next_cand_idx, float *next_cand_val, void *stream);

/* Forecast candidates for the next decode step of one layer, computed ahead
 * of time (e.g. on a side stream while the previous layer runs): the top-k
 * blocks, scored as in sd_decode_select, over every cached block except the
 * current one (the block the next token lands in, whose sum that step
 * changes).  sd_decode_layer merges them with the current block's fresh score,
 * which gives the same top-k as scoring every block in the step.
 * forecast: [B, Hkv*D] rows (stride f_sb); proto_sum as in sd_kv_append;
 * cur_len: device int32, tokens cached before the step.  cand_idx int32 /
 * cand_val fp32: [B,Hkv,top_k], -1 / -inf where no candidate exists. */
SD_API int sd_decode_candidates(const void *forecast, int f_dtype, int64_t f_sb, const float *proto_sum,
                                int64_t B, int64_t Hkv, int64_t D, int64_t NBcap, const int32_t *cur_len,
                                int block_size, int top_k, int rule, float scale, int32_t *cand_idx,
                                float *cand_val, void *stream);

/* ---- prefill block-list modes (sd_prefill_lists) ----
 * One list per (sequence, kv head, 64-token query block qb), ascending:
 *   DENSE            blocks 0..qb (sparse.py:201-224, layer 0 / no forecast / N_b <= 2)
 *   MASKED_FORECAST  {0, qb} U every row's top-k (sparse.py:226-247); the
 *                    attention kernel then applies each row's own membership
 *   MASKED_STATIC    {0} U {qb-top_k .. qb} (sparse.py:249-251)
 *   CHUNKED_FORECAST {0, qb} U union of the rows' non-causal top-k, future
 *                    blocks cleared, cut to min(N_b, top_k+2) blocks by keeping
 *                    0 and qb, then the blocks most rows picked (ties: lower
 *                    index) (sparse.py:303-333; the reference keeps an
 *                    unspecified subset of that size)
 *   CHUNKED_STATIC   {0} U {qb-top_k+1 .. qb} (sparse.py:324-328) */
#define SD_LIST_DENSE 0
#define SD_LIST_MASKED_FORECAST 1
#define SD_LIST_MASKED_STATIC 2
#define SD_LIST_CHUNKED_FORECAST 3
#define SD_LIST_CHUNKED_STATIC 4

/* Builds the prefill block lists.  topk: int64 [B,H,T,kk] selector indices
 * (needed by the *_FORECAST modes).  causal = 0 keeps future blocks for the
 * masked modes (is_causal=False); chunked modes always clear them.  lists:
 * int32 [B,H,ceil(T/64),lcap] (-1 padded), counts: int32 [B,H,ceil(T/64)].
 * block_size must be 64. */
SD_API int sd_prefill_lists(int mode, int causal, int64_t B, int64_t H, int64_t T, int block_size, int top_k,
                            const int64_t *topk, int kk, int32_t *lists, int32_t *counts, int lcap,
                            void *stream);

/* Block-sparse GQA prefill attention over the lists of sd_prefill_lists on
 * CUDA cores (fp32 math): the fp32 path, and the cross-check of the
 * tensor-core kernel.  Replaces the mask construction + repeat_interleave +
 * SDPA of model/attention/sparse.py:255-282 and :334-360.
 * q: [B,T,Hq,D] (strides q_sb, q_st, q_sh); k, v: [B,Hkv,T,D] (strides c_sb,
 * c_sh, c_st); topk (nullable): the MASKED_FORECAST rows' top-k, for per-row
 * membership; causal: key pos <= query pos.  out: [B,T,Hq,D] (strides o_sb,
 * o_st, o_sh).  D = 64, block_size = 64. */
SD_API int sd_prefill_attention(const void *q, int dtype, int64_t B, int64_t T, int64_t Hq, int64_t Hkv,
                                int64_t D, int64_t q_sb, int64_t q_st, int64_t q_sh, const void *k,
                                const void *v, int64_t c_sb, int64_t c_sh, int64_t c_st,
                                const int32_t *lists, const int32_t *counts, int lcap, const int64_t *topk,
                                int kk, int block_size, int causal, float scale, void *out, int64_t o_sb,
                                int64_t o_st, int64_t o_sh, void *stream);

/* Gradients of sd_prefill_attention: the backward that autograd takes through
 * the reference's masked / chunked SDPA prefill paths
 * (model/attention/sparse.py:185-364) when the sparse backend is trained
 * (tests/test_sparse_attention.py:63-77, training/trainer.py).  q, k, v and the
 * block lists / per-row top-k are the forward's (same layouts and strides);
 * dout [B,T,Hq,D] (element strides g_sb, g_st, g_sh) is the gradient of the
 * output, all four in `dtype`.  Writes fp32 dq [B,T,Hq,D] and dk, dv
 * [B,Hkv,T,D], all contiguous; dk and dv are zeroed on the stream first.  The
 * softmax is recomputed in fp32 (no forward statistics needed).  16-bit inputs
 * with 16-byte aligned rows run the products on the tensor cores (bf16: P and
 * dS split into high and low bf16 parts), fp32 inputs on CUDA cores; all
 * paths give fp32-level gradients.  D == 64, block_size == 64. */
SD_API int sd_prefill_attention_backward(const void *q, const void *k, const void *v, const void *dout,
                                         int dtype, int64_t B, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                                         int64_t q_sb, int64_t q_st, int64_t q_sh, int64_t c_sb, int64_t c_sh,
                                         int64_t c_st, int64_t g_sb, int64_t g_st, int64_t g_sh,
                                         const int32_t *lists, const int32_t *counts, int lcap,
                                         const int64_t *topk, int kk, int block_size, int causal, float scale,
                                         float *dq, float *dk, float *dv, void *stream);

/* RMSNorm of `rows` rows of C values (row strides x_rs, o_rs), computed as
 * model/norm.py:15-21 does: normalised in fp32, cast to the activation dtype,
 * then multiplied by the gain w [C] in that dtype. */
SD_API int sd_rmsnorm(const void *x, int dtype, int64_t rows, int64_t C, int64_t x_rs, const void *w,
                      float eps, void *out, int64_t o_rs, void *stream);

/* RoPE of a prompt's q [B,T,Hq,D] and k [B,T,Hkv,D] (element strides q_sb,
 * q_st, q_sh and k_sb, k_st, k_sh) at positions offset .. offset+T-1, written
 * to contiguous q_out [B,T,Hq,D] and k_out [B,T,Hkv,D].  Replaces
 * apply_rotary_emb (model/rope.py:34-65) with its rounding sequence: the fp32
 * tables rope_cos/rope_sin [max_pos, D/2] cast to the activation dtype, then
 * x*cos, rotate_half(x)*sin and their sum each rounded to it.  D % 16 == 0;
 * 16-byte aligned rows. */
SD_API int sd_rope_qk(const void *q, const void *k, int dtype, int64_t B, int64_t T, int64_t Hq, int64_t Hkv,
                      int64_t D, int64_t q_sb, int64_t q_st, int64_t q_sh, int64_t k_sb, int64_t k_st, int64_t k_sh,
                      const float *rope_cos, const float *rope_sin, int64_t max_pos, int64_t offset, void *q_out,
                      void *k_out, void *stream);

/* Greedy next token: out[r * o_stride] = the index of the largest of the n
 * values of row r (row stride ld), the first on ties, NaN above every number
 * -- torch.argmax(logits[:, -1, :], dim=-1) of the reference's greedy decode
 * (model/model.py:185, evaluation/latency.py:156).  int64 indices. */
SD_API int sd_argmax_rows(const void *x, int dtype, int64_t rows, int64_t n, int64_t ld, int64_t *out,
                          int64_t o_stride, void *stream);

/* SwiGLU gate of model/transformer.py:30-31 on a fused [gate | up] projection:
 * gu rows hold 2F values (row stride g_rs); out[r, c] = silu(gate) * up, each
 * op rounded to the activation dtype as the reference's separate ops are. */
SD_API int sd_silu_mul(const void *gu, int dtype, int64_t rows, int64_t F, int64_t g_rs, void *out,
                       int64_t o_rs, void *stream);

/* ---- decode-step projections (sd_linear) ---- */
#define SD_LINEAR_STORE 0    /* out = X W^T */
#define SD_LINEAR_RESIDUAL 1 /* out = res + (X W^T rounded to the dtype); out may be res */
#define SD_LINEAR_SWIGLU 2   /* W holds [gate; up] interleaved in 128-row groups (64 gate rows, then the 64 up
                                rows of the same output columns); out[m, c] = silu(gate) * up, N/2 columns */

/* One projection of the decode step on the tensor cores (tcgen05, fp32
 * accumulation), out[M, N(/2)] = epilogue(X W^T) with X [M, K] (row stride
 * x_rs) and W [N, K] contiguous, 16-bit.  norm_w (nullable, [K]): X is first
 * RMS-normalised per row with gain norm_w and eps, as model/norm.py:15-21
 * (normalised value rounded to the dtype, then times the gain).  When the
 * output tiles alone would leave SMs idle, K is split over a thread-block
 * cluster whose CTAs add their partial products through distributed shared
 * memory in a fixed order: no workspace, no allocation, and results depend
 * only on the shapes.  Replaces the nn.Linear calls around the attention
 * path: the [wq; wk; wv; wf] projection after attn_norm
 * (model/transformer.py:104-107, model/forecast.py:23-27), wo and w_down
 * with the residual add (transformer.py:118-129) and the SwiGLU FFN gate
 * (transformer.py:18-31), and the tied LM head after final_norm
 * (model/model.py:141-142).  Output row stride o_rs, residual row stride
 * r_rs.  K % 64 == 0, N % 128 == 0, K <= 1024 with norm_w; 16-byte aligned
 * X, W, norm_w, out and x_rs % 8 == 0. */
SD_API int sd_linear(const void *x, int dtype, int64_t M, int64_t K, int64_t x_rs, const void *w, int64_t N,
                     const void *norm_w, float eps, int epilogue, const void *res, int64_t r_rs, void *out,
                     int64_t o_rs, int32_t *err, void *stream);

/* lens[i] += delta for i < n (device int32 array). */
SD_API int sd_advance_len(int32_t *lens, int n, int delta, void *stream);

/* Programmatic dependent launch, process-wide, off by default; returns the
 * previous setting.  When on, sd_decode_layer, sd_rmsnorm, sd_silu_mul and
 * sd_advance_len launch with programmatic stream serialization: a kernel may
 * start while the kernel ahead of it on the stream is still running, and waits
 * for that kernel's completion (griddepcontrol.wait) before it reads anything.
 * sd_decode_layer's first warp reads the candidates, block sums, cached K/V
 * tiles and cur_len before that wait, so with the switch on those inputs must
 * have been written by kernels that finished before the kernel ahead of it
 * started (true when that kernel was launched without this attribute, as a
 * library GEMM is).  No counterpart in the reference (a launch-latency
 * optimisation of the CUDA path). */
SD_API int sd_set_programmatic_launch(int enable);

/* ---- offloaded KV caches (model/attention/offload.py, async_offload.py) ----
 * The authoritative K/V rows live in pinned host memory host_k/host_v
 * [B, Hkv, host_tcap, 64] (block-major, read and written by the GPU through
 * unified addressing).  Per (sequence, kv head) the device keeps a slot buffer
 * slot_k/slot_v [B, Hkv, (2 + kslots) * 64, 64]: slot 0 the sink block, slot 1
 * the block being appended to, slots 2.. the blocks staged for this step
 * (and, with kslots > top_k, blocks kept resident from earlier steps: a block
 * cache with least-recently-used replacement).  top_k <= kslots <= 32,
 * top_k <= 31, block_size = 64, head_dim = 64. */

/* Forecast-guided prefetch.  Replaces AsyncOffloadedKVCache.async_transfer_
 * selected_blocks (model/attention/async_offload.py:55-112) and the transfer
 * half of AsyncForecastOffloadAttention.prefetch (async_offload.py:170-294).
 * For the step whose new token takes position *cur_len: wanted blocks are
 * cand_idx [B, Hkv, top_k] (the side-stream top-k, forecast mode) or, with
 * cand_idx NULL or on dense steps, the static window / every block.  Blocks
 * already resident keep their slot; missing ones are copied from the host
 * store; a miss takes the free slot used least recently.  slot_block int32
 * [B, Hkv, 2 * kslots + 1] is the residency state (init -1): the block of
 * each slot, then the sink flag, then the position each slot was last used
 * at; cand_slot int32 [B, Hkv, top_k]
 * receives each candidate's slot (-1 = not staged).  stats (nullable) u64[3]
 * accumulates wanted blocks, hits and bytes copied. */
SD_API int sd_offload_prefetch(const void *host_k, const void *host_v, int dtype, int64_t B, int64_t Hkv,
                               int64_t D, int64_t host_tcap, void *slot_k, void *slot_v, int kslots,
                               const int32_t *cur_len, int block_size, int top_k, const int32_t *cand_idx,
                               int32_t *slot_block, int32_t *cand_slot, unsigned long long *stats, void *stream);

/* sd_decode_layer on an offloaded cache.  Replaces AsyncForecastOffloadAttention.
 * _forward_async_decode (async_offload.py:296-519): the new token's K/V go to
 * slot 1 and, written through, to the host store; attention reads the sink,
 * current and staged slots.  Forecast steps need the candidates and their
 * slots from sd_decode_candidates + sd_offload_prefetch (no in-kernel
 * selection).  Other arguments as sd_decode_layer. */
SD_API int sd_decode_layer_offload(const void *qkv, int dtype, int64_t qkv_sb, const void *forecast, int f_dtype,
                                   int64_t f_sb, const float *rope_cos, const float *rope_sin, int64_t max_pos,
                                   const int32_t *cur_len, void *host_k, void *host_v, int64_t host_tcap,
                                   void *slot_k, void *slot_v, int kslots, float *proto_sum, int64_t B, int64_t Hq,
                                   int64_t Hkv, int64_t D, int64_t NBcap, int block_size, int top_k, int rule,
                                   float scale, void *out, int64_t o_sb, const int32_t *cand_idx,
                                   const float *cand_val, const int32_t *cand_slot, int32_t *sel_out,
                                   int32_t *cnt_out, int sel_cap, int32_t *err, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* SPARDAB200_H */
