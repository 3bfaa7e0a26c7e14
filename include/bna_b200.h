/*
 * bna_b200.h — C ABI of the B200-native compressed Butterfly attention library
 * (libbna_b200.so).  Plain C: raw pointers, integer sizes/strides, a cudaStream_t
 * passed as void*.  No PyTorch types cross this boundary.
 *
 * Every entry point returns a bna_status; on failure bna_last_error() returns a
 * thread-local message.  The caller owns every buffer (inputs, outputs, cache pools);
 * the library never allocates or frees device memory.  All work is enqueued on the
 * given stream; nothing synchronises the host except the *_host selection dumps.
 *
 * Reference interfaces replaced (paths inside the Hmbown/Butterfly project):
 *   bna/torch/attention_wayfinder_permute.py  build_block_butterfly_layout      :568-682
 *   bna/torch/attention_wayfinder_permute.py  _compressed_butterfly_block_index_tensors :912-966
 *   bna/torch/attention_wayfinder_permute.py  _compressed_butterfly_active_index_tensors :969-1019
 *   bna/torch/attention_wayfinder_permute.py  _block_mean_summaries_torch       :1022-1043
 *   bna/torch/attention_wayfinder_permute.py  butterfly_compressed_attention    :1046-1122
 *   bna/torch/attention_wayfinder_permute.py  butterfly_compressed_attention_active :1125-1197
 *   bna/mlx/compressed_cache.py               CompressedKVCache.update_and_fetch :94-172
 *   bna/mlx/attention.py                      compressed_butterfly_attention_from_cache :1816-1876
 */
#ifndef BNA_B200_H
#define BNA_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define BNA_API __attribute__((visibility("default")))
#else
#define BNA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  BNA_OK = 0,
  BNA_BAD_SHAPE = 1,      /* shape/size mismatch or non-positive size  (reference: ValueError) */
  BNA_BAD_STRIDE = 2,     /* stride/alignment not usable (innermost dim must be contiguous)   */
  BNA_BAD_DTYPE = 3,      /* dtype not supported on this path                                 */
  BNA_CAPACITY = 4,       /* cache tail / summary capacity exceeded (reference: RuntimeError)  */
  BNA_UNSUPPORTED = 5,    /* configuration outside what the kernels implement                  */
  BNA_CUDA_ERROR = 6,     /* a CUDA runtime/driver call failed                                 */
  BNA_DEVICE_TIMEOUT = 7  /* a kernel gave up a bounded wait and returned early               */
} bna_status;

typedef enum { BNA_BF16 = 0, BNA_F16 = 1 } bna_dtype;

/* Partner rules of bna/topology/butterfly.py:108-141 used by the block-sparse layout. */
typedef enum {
  BNA_RULE_CAUSAL_SHIFT = 0,
  BNA_RULE_XOR = 1,
  BNA_RULE_BIT_REVERSAL = 2,
  BNA_RULE_BENES = 3
} bna_rule;

/* A strided 4-D view [d0, d1, d2, d3] with element strides; d3 (head_dim) must have
 * stride 1.  Used for q/k/v [B, H, T, dh], outputs and cache pools. */
typedef struct {
  void* data;
  int64_t size[4];
  int64_t stride[4];
} bna_tensor4;

/* Block routing of one layer (replaces BlockHamiltonianLayout, :382-405).
 * If `neighbors` is non-NULL it is a DEVICE int32 table [num_blocks, max_degree]
 * (-1 padded, head 0 rows of block_neighbors) and the rule fields are ignored;
 * otherwise rows are generated in closed form from the rule fields. */
typedef struct {
  int32_t block_size;
  int32_t num_blocks;
  int32_t max_degree;          /* summary slots per row (>= 1, <= 16) */
  int32_t rule;                /* bna_rule */
  int32_t width;               /* ceil(log2(num_blocks)), 1 if num_blocks <= 1 */
  int32_t stage_idx;
  int32_t stage_count;
  int32_t partner_count;       /* <= 8 */
  int32_t local_window_blocks;
  int32_t sink_count;
  const int32_t* neighbors;    /* optional device table */
} bna_route;

BNA_API const char* bna_last_error(void);
BNA_API const char* bna_version(void);

/* Reads and clears the device-side error word set by kernels that gave up a bounded
 * wait (0 = none).  Synchronises the given device. */
BNA_API int bna_take_device_error(int device, int32_t* code_out);

/* Tracing: when non-NULL, later prefill launches write globaltimer stamps of each work
 * unit's pipeline hand-offs to this device buffer ([grid][64 units][16] uint64, grid =
 * number of SMs).  Pass NULL to stop.  Used by the profiling tools only. */
BNA_API int bna_set_prefill_trace(void* device_buffer);

/* Profiling aid: launches an empty grid of `ctas` CTAs the way the decode step is launched
 * (programmatic dependent launch).  A graph of these gives the per-launch floor of a chain
 * of dependent decode steps. */
BNA_API int bna_launch_probe(int32_t ctas, void* stream);

/* ---- topology / selection (host) -------------------------------------------------- */

/* Fill `route` (everything but `neighbors`) for a layer; replaces
 * build_block_butterfly_layout's metadata (:568-682, butterfly.py:52-105). */
BNA_API int bna_route_init(bna_route* route, int32_t seq_len, int32_t block_size, int32_t layer_idx,
                   int32_t local_window_blocks, int32_t sink_count, int32_t partner_count,
                   int32_t rule);

/* Host dump of the block_neighbors rows [num_blocks, max_degree] (-1 padded). */
BNA_API int bna_block_neighbors_host(const bna_route* route, int32_t* out);

/* Host dump of prefill selection (:912-966): per block the raw-window start and the
 * cursor-packed valid summary blocks ([num_blocks, max_degree], -1 padded) and count.
 * Uses the same selection code the kernels run.  route->neighbors must be NULL or
 * a HOST table for this call. */
BNA_API int bna_prefill_selection_host(const bna_route* route, int32_t seq_len, int32_t window,
                               int32_t* local_start, int32_t* summary_idx, int32_t* summary_count);

/* Host dump of active-row selection (:969-1019) for `n` query positions. */
BNA_API int bna_active_selection_host(const bna_route* route, int32_t window, const int64_t* positions,
                              int32_t n, int32_t num_summary_limit, int32_t* block,
                              int32_t* local_start, int32_t* summary_idx, int32_t* summary_count);

/* Device dump of the same selections, computed by the device code path (for parity). */
BNA_API int bna_prefill_selection_device(const bna_route* route, int32_t seq_len, int32_t window,
                                 int32_t* summary_idx, int32_t* summary_count, void* stream);

/* ---- K1: mean-pool block compressor (:1022-1043; cache close :133-140) -------------- */

/* out[b,h,slot0+j,:] = mean of the valid tokens of block j (j < n_blocks) of x, where
 * block j covers positions [pos0 + j*block_size, ...) clipped to `valid_len` positions
 * counted from pos0 (partial last block averaged over its valid tokens, >= 1).
 * Token position p is read at x[b,h,idx,:] with idx = p % ring (ring > 0) or
 * idx = p - pos0 (ring == 0).  fp32 accumulation, rounded store in x's dtype. */
BNA_API int bna_compress_blocks(const bna_tensor4* x, bna_tensor4* out, int32_t dtype, int32_t block_size,
                        int64_t pos0, int32_t n_blocks, int64_t valid_len, int64_t ring,
                        int64_t slot0, void* stream);

/* The same for a K/V pair in one launch (shapes of k and v, and of k_out and v_out, equal). */
BNA_API int bna_compress_kv_blocks(const bna_tensor4* k, const bna_tensor4* v, bna_tensor4* k_out,
                                   bna_tensor4* v_out, int32_t dtype, int32_t block_size, int64_t pos0,
                                   int32_t n_blocks, int64_t valid_len, int64_t ring, int64_t slot0,
                                   void* stream);

/* ---- K2: prefill attention on tcgen05/TMEM (:1046-1122) -------------------------------
 * q [B,Hq,Tq,dh] (any strides, dh contiguous, 16-byte aligned rows), k/v [B,Hkv,Tk,dh],
 * k_sum/v_sum [B,Hkv,N,dh] block means, out [B,Hq,Tq,dh] (same dtype), lse (optional,
 * fp32, element strides lse_stride_b/h, token-contiguous).
 * Query row i has global position q_pos0+i; key row j has global position kv_pos0+j;
 * selection uses `route` over a sequence of total_len tokens.  dh must be 128,
 * Hq/Hkv in {1,2,4,8}.  scale = softmax scale (1/sqrt(dh) for SDPA's default). */
BNA_API int bna_prefill_attention(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                          const bna_tensor4* k_sum, const bna_tensor4* v_sum, bna_tensor4* out,
                          float* lse, int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype,
                          const bna_route* route, int32_t window, int64_t q_pos0, int64_t kv_pos0,
                          int64_t total_len, float scale, void* stream);

/* The same with the output gate of Qwen3.5's gated attention fused into the store:
 * out = round(round(o) * round(sigmoid(gate))) for gate [B,Hq,Tq,dh] (the q-projection's
 * gate half, same dtype and row rules as q), the rounding of the separate
 * bna_gate_sigmoid_mul after an ungated call (Qwen3_5Attention.forward,
 * transformers/models/qwen3_5/modeling_qwen3_5.py, `attn_output * torch.sigmoid(gate)`).
 * Windows too large for the ring-based kernel return BNA_UNSUPPORTED (call the ungated
 * entry point and gate separately). */
BNA_API int bna_prefill_attention_gated(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                                        const bna_tensor4* k_sum, const bna_tensor4* v_sum,
                                        const bna_tensor4* gate, bna_tensor4* out, float* lse,
                                        int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype,
                                        const bna_route* route, int32_t window, int64_t q_pos0,
                                        int64_t kv_pos0, int64_t total_len, float scale, void* stream);

/* ---- K4: active / decode attention (:1125-1197; MLX from_cache :1669-1876) -------------
 * One query row per (b, query index).  Raw keys for position p are the positions
 * [max(0,p-W+1), p]; position x is read at k[b,h,x % ring] (ring > 0) or
 * k[b,h,x - kv_pos0] (ring == 0).  Summaries are read at k_sum[b,h,n].  Query positions
 * come from `positions` (device int64, length Tq) or, if NULL, pos0 + index.
 * num_summary_limit bounds usable summary blocks (summary_count of a cache).
 * Selection block = min(p / block_size, route->num_blocks - 1). */
BNA_API int bna_active_attention(const bna_tensor4* q, const bna_tensor4* k, const bna_tensor4* v,
                         const bna_tensor4* k_sum, const bna_tensor4* v_sum, bna_tensor4* out,
                         float* lse, int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype,
                         const bna_route* route, int32_t window, const int64_t* positions,
                         int64_t pos0, int64_t kv_pos0, int64_t ring, int32_t num_summary_limit,
                         float scale, void* stream);

/* ---- K3: two-pool cache (bna/mlx/compressed_cache.py:94-172) --------------------------
 * Ring tail [B,Hkv,ring,dh] and summary pool [B,Hkv,capacity,dh].  Counter logic lives
 * in the host (it is pure integer bookkeeping); these move the data. */

/* Write src [B,Hkv,step,dh] at positions pos0..pos0+step-1 into ring slots p % ring. */
BNA_API int bna_cache_append(bna_tensor4* ring_k, bna_tensor4* ring_v, const bna_tensor4* src_k,
                     const bna_tensor4* src_v, int32_t dtype, int64_t pos0, int64_t ring, void* stream);

/* Fused decode step for one new token per sequence: append k_new/v_new [B,Hkv,1,dh] at
 * position `pos` into the ring, close block `close_block` into summary slot `close_slot`
 * when close_block >= 0 (mean of its block_size tokens read from the ring), then attend
 * q [B,Hq,1,dh] at position `pos` over the ring window and routed summaries (limit
 * num_summary_limit, counting the block closed here). */
BNA_API int bna_decode_step(const bna_tensor4* q, const bna_tensor4* k_new, const bna_tensor4* v_new,
                    bna_tensor4* ring_k, bna_tensor4* ring_v, bna_tensor4* sum_k, bna_tensor4* sum_v,
                    bna_tensor4* out, float* lse, int64_t lse_stride_b, int64_t lse_stride_h,
                    int32_t dtype, const bna_route* route, int32_t window, int64_t pos, int64_t ring,
                    int64_t close_block, int64_t close_slot, int32_t num_summary_limit, float scale,
                    void* stream);

/* ---- Decoder-layer steps around the attention (Qwen3.5) ---------------------------------
 * Fused forms of the eager ops the reference runs before and after its attention
 * (bna/integrations/qwen_torch.py:535-573 extract_qkv_from_qwen_attention: q/k RMSNorm and
 * partial rotary embedding; :1585-1591: output gate; and transformers' Qwen3_5DecoderLayer
 * norms and SwiGLU MLP around them).  16-bit storage (dtype), fp32 arithmetic inside a
 * norm, each elementwise result rounded to the storage type as the eager ops do.  Row
 * strides are in elements. */

/* y = x * rsqrt(mean(x^2) + eps) * (1 + weight) per row of `hidden` elements (Qwen3.5
 * RMSNorm).  With `res` non-NULL the normalised row is round(x + res) (the decoder layer's
 * residual add), and that sum is also written to `sum_out` when non-NULL.  hidden must be
 * 256 x {1,2,4,8,10,12,16}; pointers 16-byte aligned; strides multiples of 8. */
BNA_API int bna_rmsnorm(const void* x, int64_t x_stride, const void* res, int64_t res_stride, const void* weight,
                        void* out, int64_t out_stride, void* sum_out, int64_t sum_stride, int64_t rows,
                        int32_t hidden, float eps, int32_t dtype, void* stream);

/* q/k preparation for `tokens` tokens: per (token, head) RMSNorm over head_dim (1 + w form,
 * q_weight / k_weight [head_dim]), then the rotary embedding on the first `rot` dims in
 * rotate-half form with cos/sin [tokens, rot] (row stride cs_tok_stride), the remaining dims
 * passed through.  Source row (t, h) of q is at q + t*q_tok_stride + h*q_head_stride (so the
 * query half of a gated q_proj output is read in place); outputs are contiguous
 * [tokens, hq, head_dim] and [tokens, hkv, head_dim].  With v / v_out non-NULL the V rows
 * (strided like k) are also copied to v_out [tokens, hkv, head_dim] (so that K and V can be
 * produced straight into pre-sized buffers, e.g. after a sequence shard's halo rows).
 * head_dim must be 128. */
BNA_API int bna_qk_norm_rope(const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* k,
                             int64_t k_tok_stride, int64_t k_head_stride, const void* q_weight, const void* k_weight,
                             const void* cos, const void* sin, int64_t cs_tok_stride, int32_t rot, void* q_out,
                             void* k_out, const void* v, int64_t v_tok_stride, int64_t v_head_stride, void* v_out,
                             int64_t tokens, int32_t hq, int32_t hkv, int32_t head_dim, float eps, int32_t dtype,
                             void* stream);

/* out[t, h*head_dim + d] = o[t, h, d] * sigmoid(gate[t, h, d]); o contiguous
 * [tokens, heads, head_dim], gate strided (the gate half of a gated q_proj output). */
BNA_API int bna_gate_sigmoid_mul(const void* o, const void* gate, int64_t gate_tok_stride, int64_t gate_head_stride,
                                 void* out, int64_t tokens, int32_t heads, int32_t head_dim, int32_t dtype,
                                 void* stream);

/* out[r, i] = silu(gate_up[r, i]) * gate_up[r, up_offset + i] for i < inter; out contiguous. */
BNA_API int bna_swiglu(const void* gate_up, int64_t row_stride, int64_t up_offset, void* out, int64_t rows,
                       int32_t inter, int32_t dtype, void* stream);

/* The gate/up projection with SwiGLU in the epilogue, on tcgen05 tensor cores:
 * out[m, i] = silu(h[m,:] . w[i,:]) * (h[m,:] . w[inter + i,:]) for m < M, i < inter, with h
 * [M, K] (row stride ldh), w [2*inter, K] (gate rows, then up rows; row stride ldw) and out
 * [M, inter] (row stride ldo), all row-major.  The gate and up products, silu(gate) and the
 * product are each rounded to the 16-bit type, as the eager ops (transformers'
 * Qwen3_5MLP: act_fn(gate_proj(x)) * up_proj(x)); accumulation is fp32.  K a multiple of 64,
 * inter of 128, row strides multiples of 8 elements, pointers 16-byte aligned.
 * With row_ss non-NULL the MLP's RMSNorm is folded in: h is the un-normalised residual, w
 * carries the norm weight (1 + w_norm[k]) in column k, and row m's products are scaled by
 * rsqrt(sum(row_ss[m * row_ss_ld + 0 .. row_ss_parts)) / K + norm_eps) before rounding
 * (row_ss: fp32 partial sums of squares of the row, from bna_gemm_residual's ss_out or
 * bna_row_sumsq; row_ss_parts a multiple of 4). */
BNA_API int bna_gemm_swiglu(const void* h, int64_t ldh, const void* w, int64_t ldw, void* out, int64_t ldo,
                            int64_t M, int32_t K, int32_t inter, const float* row_ss, int64_t row_ss_ld,
                            int32_t row_ss_parts, float norm_eps, int32_t dtype, void* stream);

/* The merged q/k/v projection with the q/k RMSNorm and rotary embedding in the epilogue:
 * out[m, :] = h[m,:] . w^T for w [N, K] whose rows come in 128-row head groups
 * [q0 gate0 q1 gate1 .. q(Hq-1) gate(Hq-1) | k0 .. k(Hkv-1) | v0 .. v(Hkv-1)]
 * (N = (2 Hq + 2 Hkv) * 128, a multiple of 256); every query and key group is then
 * normalised (Qwen3.5 RMSNorm, weights q_norm_w / k_norm_w [128]) and rotated in
 * rotate-half form on its first `rot` dims with cos / sin [M, rot] (row m's tables),
 * the rounding steps of the eager ops (bna_qk_norm_rope); gate and value groups are the
 * rounded products.  K a multiple of 64, rot a multiple of 32.  row_ss / row_ss_ld /
 * row_ss_parts / norm_eps fold the layer's input RMSNorm in, as for bna_gemm_swiglu. */
BNA_API int bna_gemm_qkv_norm_rope(const void* h, int64_t ldh, const void* w, int64_t ldw, void* out, int64_t ldo,
                                   int64_t M, int32_t K, int32_t N, int32_t num_q_heads, int32_t num_kv_heads,
                                   const void* q_norm_w, const void* k_norm_w, const void* cos, const void* sin,
                                   int32_t rot, float eps, const float* row_ss, int64_t row_ss_ld,
                                   int32_t row_ss_parts, float norm_eps, int32_t dtype, void* stream);

/* A projection followed by the decoder layer's residual add, on tcgen05 tensor cores:
 * out[m, n] = round(round(h[m,:] . w[n,:]) + res[m, n]) for m < M, n < N: the projection
 * rounded, then the residual added and rounded, as the eager ops of transformers'
 * Qwen3_5DecoderLayer (residual + o_proj(attn), residual + down_proj(mlp); qwen_torch.py
 * :1585-1591 feeds o_proj).  out may be res
 * (same pointer and row stride: an in-place add); any other overlap is rejected.  K a
 * multiple of 64, N of 256, row strides multiples of 8 elements, pointers 16-byte aligned.
 * With ss_out non-NULL, ss_out[m * ss_ld + 4 t + p] receives the fp32 sum of squares of the
 * rounded outputs of row m in columns [256 t + 64 p, +64) (ss_ld >= 4 N / 256): the next
 * RMSNorm's statistics, for the row_ss argument of the SwiGLU and q/k/v GEMMs. */
BNA_API int bna_gemm_residual(const void* h, int64_t ldh, const void* w, int64_t ldw, const void* res, int64_t ldr,
                              void* out, int64_t ldo, int64_t M, int32_t K, int32_t N, float* ss_out, int64_t ss_ld,
                              int32_t dtype, void* stream);

/* out[r * ld_out + 0..3] = {sum_k x[r, k]^2, 0, 0, 0} in fp32 for r < rows, k < H: the
 * row_ss input (4 parts) of the folded-RMSNorm GEMMs for rows no residual GEMM produced. */
BNA_API int bna_row_sumsq(const void* x, int64_t x_stride, float* out, int64_t ld_out, int64_t rows, int32_t H,
                          int32_t dtype, void* stream);

/* Decode-time projections for 1..8 tokens (y = W x per token, W [out_features,
 * in_features] row-major, in_features a multiple of 256), with the layer step before the
 * projection fused in front of it and the one after it fused behind it.  Replace the
 * eager decode-step ops of the same decoder layer (q/k/v, o, gate/up and down
 * projections with their norms, gate and residual adds). */

/* y = W rmsnorm(x [+ res]) (Qwen3.5 RMSNorm with norm_weight; x + res rounded and written to
 * sum_out when non-NULL).  With swiglu != 0 the rows are [gate; up] halves and
 * out[i] = silu(gate_i) * up_i for i < out_features / 2. */
BNA_API int bna_gemv_rmsnorm(const void* x, int64_t x_stride, const void* res, int64_t res_stride,
                             const void* norm_weight, float eps, void* sum_out, int64_t sum_stride, const void* w,
                             int64_t out_features, int64_t in_features, int32_t swiglu, void* out,
                             int64_t out_stride, int32_t tokens, int32_t dtype, void* stream);

/* y = [res +] W (o * sigmoid(gate)): o [tokens, in_features] contiguous, gate[m, h, d] at
 * gate + m*gate_tok_stride + h*gate_head_stride + d (heads of head_dim columns). */
BNA_API int bna_gemv_gated(const void* o, const void* gate, int64_t gate_tok_stride, int64_t gate_head_stride,
                           int32_t head_dim, const void* w, int64_t out_features, int64_t in_features,
                           const void* res, int64_t res_stride, void* out, int64_t out_stride, int32_t tokens,
                           int32_t dtype, void* stream);

/* y = [res +] W x. */
BNA_API int bna_gemv(const void* x, int64_t x_stride, const void* w, int64_t out_features, int64_t in_features,
                     const void* res, int64_t res_stride, void* out, int64_t out_stride, int32_t tokens,
                     int32_t dtype, void* stream);

/* The fused decode step with the new token's q/k preparation fused in (replaces
 * bna_qk_norm_rope + bna_decode_step for one token): q_raw [B,Hq,1,dh] and k_raw
 * [B,Hkv,1,dh] are the raw projection rows (the query half of a gated q_proj output read in
 * place); each row gets the Qwen3.5 RMSNorm (q_norm_weight / k_norm_weight [dh], eps) and the
 * rotary embedding on its first `rot` dims with cos / sin of sequence b at
 * cos + b * cs_batch_stride, before the append (the ring stores the prepared key) and the
 * attention.  Reference: bna/integrations/qwen_torch.py:535-573 (q/k norm, RoPE, cache
 * update) followed by the decode branch :1417-1427. */
BNA_API int bna_decode_step_qk(const bna_tensor4* q_raw, const bna_tensor4* k_raw, const bna_tensor4* v_new,
                               bna_tensor4* ring_k, bna_tensor4* ring_v, bna_tensor4* sum_k, bna_tensor4* sum_v,
                               bna_tensor4* out, float* lse, int64_t lse_stride_b, int64_t lse_stride_h,
                               int32_t dtype, const bna_route* route, int32_t window, int64_t pos, int64_t ring,
                               int64_t close_block, int64_t close_slot, int32_t num_summary_limit, float scale,
                               const void* q_norm_weight, const void* k_norm_weight, const void* cos,
                               const void* sin, int64_t cs_batch_stride, int32_t rot, float eps, void* stream);

/* ---- Prefill without caller-provided scratch -------------------------------------------
 * No counterpart in the reference.  For callers that cannot allocate device memory
 * (no cudaMalloc inside their host framework's capture/allocator regions, or a fixed
 * memory plan): computes the K/V block means into an 8 MiB device array, then runs
 * bna_prefill_attention over the whole sequence (q_pos0 = kv_pos0 = 0, total_len = T).
 * The array is reserved on each device when the library's device code loads there (the
 * first call, under CUDA's default lazy loading), and that first call resolves its
 * address: make it before any stream capture, and do not call this after a
 * cudaDeviceReset of the device.  Rejects problems whose block means exceed 8 MiB
 * (BNA_CAPACITY) and bad shapes before launching anything.  The array is shared by all
 * calls: calls that overlap on the GPU race. */
BNA_API int bna_prefill_attention_static_scratch(const bna_tensor4* q, const bna_tensor4* k,
                                                 const bna_tensor4* v, bna_tensor4* out, float* lse,
                                                 int64_t lse_stride_b, int64_t lse_stride_h, int32_t dtype,
                                                 const bna_route* route, int32_t window, float scale,
                                                 void* stream);

#ifdef __cplusplus
}
#endif
#endif /* BNA_B200_H */
