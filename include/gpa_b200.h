/*
 * gpa_b200.h -- C ABI of the B200 (sm_100a) kernels for GPA-VGGT's accelerated
 * global-attention path: bipartite K/V token merging (matching, plan,
 * scatter-mean), log(count)-biased flash attention, and the frame attention
 * with a shared cross-frame K/V set of the early global blocks.
 *
 * Conventions (all entry points):
 *   - Plain device pointers, element strides (not bytes), sizes as int.
 *     The innermost dimension of every tensor is contiguous.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).
 *   - Outputs are caller-allocated; nothing here allocates device memory except
 *     where a function says so.
 *   - Return value: GPA_OK or an error code; gpa_last_error() gives the message
 *     of the last failing call on this host thread.
 *   - `status` (optional, may be NULL) is a device int that a kernel sets to a
 *     nonzero code when one of its pipeline waits gave up (lost signal); the
 *     kernel then returns early instead of hanging.  The caller reads it back.
 *
 * Reference interfaces replaced (paths inside noheat61/GPA-VGGT):
 *   merging/fused_similarity.py:81-112   fused_similarity_argmax
 *   merging/merge.py:87-176               dst/src split of token_merge_bipartite2d
 *   merging/merge.py:180-187              projected metric normalise + split
 *   merging/merge.py:189-217              edge ranking, dst_idx, merged_size
 *   merging/merge.py:234-250              merge.heads (scatter-mean)
 *   merging/fused_attention.py:130-180    attention_keybias
 *   vggt/layers/attention.py:113-140      _pool (content-adaptive summaries)
 *   vggt/layers/attention.py:164-176      two-partition log-sum-exp combine
 */
#ifndef GPA_B200_H
#define GPA_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define GPA_API __attribute__((visibility("default")))
#else
#define GPA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GPA_OK 0
#define GPA_ERR_INVALID 1     /* bad argument: shape, stride, alignment, dtype */
#define GPA_ERR_CUDA 2        /* CUDA runtime/driver error (launch, tensor map) */
#define GPA_ERR_UNSUPPORTED 3 /* shape outside what the kernels implement */

#define GPA_DTYPE_F32 0
#define GPA_DTYPE_BF16 1

/* Library version (major*10000 + minor*100 + patch). */
GPA_API int gpa_version(void);

/* Message of the last failing call on this host thread ("" if none). */
GPA_API const char* gpa_last_error(void);

/* Number of kernels this library has launched in this process so far. */
GPA_API int64_t gpa_launch_count(void);

/*
 * Self-test of the failure path shared by every pipelined kernel (no
 * counterpart in the reference, which has no device-side waits): one warp
 * waits on a shared-memory mbarrier that nothing arrives on, with the bounded
 * wait of the pipelined kernels and a limit of limit_ns (1 us .. 10 s).  The
 * wait gives up, writes 1 (timeout) to *status (device memory) and the kernel
 * returns, leaving the context usable.  Used by the tests to exercise the
 * host-side status check without faulting or hanging a GPU.
 */
GPA_API int gpa_wait_selftest(uint64_t limit_ns, int* status, void* stream);

/*
 * Similarity + row argmax (replaces merging/fused_similarity.py:81-112, kernel
 * _sim_argmax_kernel :33-78).  For each batch b and row i of a:
 *   node_max[b,i] = max_j  sum_k a[b,i,k]*b[b,j,k]   (bf16 inputs, fp32 accumulate)
 *   node_idx[b,i] = the smallest j attaining that max
 * a: [batch, m, d] bf16, b: [batch, n, d] bf16; d % 64 == 0, 64 <= d <= 256.
 * Row strides must be multiples of 8 elements, base pointers 16-byte aligned.
 * node_max: [batch, m] fp32 contiguous; node_idx: [batch, m] int32 contiguous.
 */
GPA_API int gpa_sim_argmax(const void* a, const void* b, int batch, int m, int n, int d,
                   int64_t a_stride_b, int64_t a_stride_m, int64_t b_stride_b,
                   int64_t b_stride_n, float* node_max, int32_t* node_idx, int* status,
                   void* stream);

/*
 * dst/src split of the multi-frame token sequence (replaces merging/merge.py:87-176).
 * Tokens per frame P = w*h + num_special; num_imgs frames.  dst tokens: every
 * token of frame 0, the num_special leading tokens of every frame, and one
 * token per (sy x sx) window chosen by rand_idx[f-1, wy, wx] in [0, sx*sy)
 * (rand_idx: device int64 [num_imgs-1, h/sy, w/sx], the values the reference
 * draws with torch.randint; ignored when no_rand != 0).  As in the reference,
 * the window pattern covers the first (h/sy*sy)*(w/sx*sx) patch positions of
 * a frame taken contiguously.
 * Outputs (device int32): dst_pos[num_dst], src_pos[num_src] -- absolute token
 * positions in ascending order -- and slot[N]: the dst ordinal of a dst token,
 * or -(src ordinal)-1 of a src token.  num_dst/num_src are given by
 * gpa_merge_counts().
 */
GPA_API int gpa_merge_counts(int num_imgs, int w, int h, int sx, int sy, int num_special, int no_rand,
                     int* num_dst, int* num_src);
GPA_API int gpa_merge_roles(const int64_t* rand_idx, int num_imgs, int w, int h, int sx, int sy,
                    int num_special, int no_rand, int32_t* dst_pos, int32_t* src_pos,
                    int32_t* slot, void* stream);

/*
 * Normalise the projected matching metric and split it (replaces
 * merging/merge.py:185-187 after the `metric @ proj` GEMM):
 *   a[i] = bf16(metric[src_pos[i]] / ||metric[src_pos[i]]||)  (fp32 norm)
 *   b[j] = bf16(metric[dst_pos[j]] / ||metric[dst_pos[j]]||)
 * metric: [N, d], dtype GPA_DTYPE_BF16 or GPA_DTYPE_F32, row stride metric_stride;
 * a: [num_src, d], b: [num_dst, d] contiguous bf16.  d % 8 == 0, d <= 1024.
 */
GPA_API int gpa_metric_split(const void* metric, int dtype, int64_t metric_stride, int d, const int32_t* src_pos,
                     int num_src, const int32_t* dst_pos, int num_dst, void* a, void* b,
                     void* stream);

/*
 * Matching metric in one pass (replaces merging/merge.py:180-187, the
 * `metric @ proj`, normalisation and split): for each of the `rows` rows of x
 * (bf16, row stride x_stride >= k, k % 64 == 0), m = bf16(x_row @ proj) with
 * proj_t = proj^T [128, k] bf16 contiguous (fp32 accumulation, the product
 * rounded to bf16 as the reference's autocast GEMM returns it), then
 * bf16(m / ||m||) with the norm and quotient in fp32 (the reference's
 * `metric.norm()` runs in fp32 under autocast).  The 128-wide result goes to
 * row slot[i] of b when slot[i] >= 0 (a dst token) and to row -slot[i]-1 of a
 * otherwise (a src token): the slot map of gpa_merge_roles.  a, b: [*, 128]
 * bf16 contiguous.  tcgen05 kernel; status as for the other pipelined kernels.
 */
GPA_API int gpa_proj_norm_split(const void* x, int64_t x_stride, int rows, int k, const void* proj_t,
                                const int32_t* slot, void* a, void* b, int* status, void* stream);

/*
 * Merge plan (replaces merging/merge.py:189-217).  Given node_max/node_idx of
 * the num_src src tokens, the r = min(r, num_src) src tokens with the largest
 * node_max are merged into their matched dst; ties at the cut are broken by
 * the lower src ordinal (a stable descending sort).  Outputs (device):
 *   unm_src[num_src - r]   unmerged src ordinals, ascending (output slots 0..)
 *   seg_start[num_dst + 1] CSR offsets into seg_src, per dst ordinal
 *   seg_src[r]             merged src ordinals grouped by dst, ascending in a group
 *   counts[N_m]            tokens behind each output slot (fp32):
 *                          1 for unmerged src, 1 + group size for dst
 * N_m = (num_src - r) + num_dst.  workspace: gpa_merge_plan_workspace_bytes().
 */
GPA_API int64_t gpa_merge_plan_workspace_bytes(int num_src, int num_dst);
GPA_API int gpa_merge_plan(const float* node_max, const int32_t* node_idx, int num_src, int num_dst,
                   int r, int32_t* unm_src, int32_t* seg_start, int32_t* seg_src,
                   float* counts, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Merge plan for callers that must not allocate device memory (no counterpart
 * in the reference).  Same inputs, outputs and results as gpa_merge_plan, but
 * the scratch is a fixed array of GPA_NOALLOC_SCRATCH_BYTES inside the library
 * on each GPU (held until the process exits), so the call allocates nothing.
 * Meant for hosts that give all device memory to their own arena up front, or
 * FFI callers without an allocator.  Every call resolves the array's device
 * address on the current device; the first call on a device may load the
 * library onto it, so make that first call before any stream capture.  Calls
 * that overlap on the GPU race on the shared array; sizes whose scratch exceeds
 * the array (gpa_merge_plan_workspace_bytes > GPA_NOALLOC_SCRATCH_BYTES, about
 * 630k src with 210k dst tokens) return GPA_ERR_UNSUPPORTED without launching.
 */
#define GPA_NOALLOC_SCRATCH_BYTES (16u << 20)
GPA_API int gpa_merge_plan_noalloc(const float* node_max, const int32_t* node_idx, int num_src,
                                   int num_dst, int r, int32_t* unm_src, int32_t* seg_start,
                                   int32_t* seg_src, float* counts, void* stream);

/*
 * Scatter-mean of one K or V tensor through a merge plan (replaces
 * merging/merge.py:234-250, merge.heads(t, mode), and merge() at :222-232):
 *   out[h, s]            = t[h, src_pos[unm_src[s]]]                 s < unm_len
 *   out[h, unm_len + j]  = (t[h, dst_pos[j]] + sum_{i in seg j} t[h, src_pos[i]])
 *                          / (1 + |seg j|)        (reduce_mean != 0, "mean")
 *                          or without the division (reduce_mean == 0, "sum")
 * t: [heads, n_tokens, head_dim] with strides (t_stride_h, t_stride_n), dtype
 * GPA_DTYPE_F32 or GPA_DTYPE_BF16; out has the same dtype, [heads, N_m, head_dim]
 * with strides (out_stride_h, out_stride_n).  Sums are fp32 in a fixed order
 * (dst first, then src ordinal ascending), so the result is deterministic.
 * head_dim % 8 == 0.  If log_counts != NULL, log of the tokens behind each slot
 * (fp32 [N_m]) is also written there.
 * The output slots are unm_len + num_dst > 0 (either part may be empty), so a
 * caller can merge any contiguous range of a plan's unmerged slots (offset
 * unm_src, num_dst = 0) or dst slots (offset dst_pos and seg_start, unm_len =
 * 0): the frame-sharded path merges only the slots whose tokens it owns, with
 * src_pos/dst_pos mapping ordinals to rows of its own row buffer.
 */
GPA_API int gpa_merge_kv_mean(const void* t, int dtype, int heads, int n_tokens, int head_dim,
                      int64_t t_stride_h, int64_t t_stride_n, const int32_t* src_pos,
                      const int32_t* dst_pos, const int32_t* unm_src, int unm_len,
                      const int32_t* seg_start, const int32_t* seg_src, int num_dst,
                      int reduce_mean, float* log_counts, void* out, int64_t out_stride_h,
                      int64_t out_stride_n, void* stream);

/*
 * CUDA IPC for the peer-memory exchange below (no counterpart in the
 * reference, which runs on one device).  gpa_ipc_export writes the 64-byte
 * IPC handle of the device allocation holding ptr and ptr's byte offset in it;
 * another process on the same node opens it with gpa_ipc_open, which returns
 * that process's address of the same byte (peer access enabled lazily), and
 * releases it with gpa_ipc_close(ptr, offset).  A process cannot open its own
 * handle.
 */
#define GPA_IPC_HANDLE_BYTES 64
GPA_API int gpa_ipc_export(const void* ptr, void* handle, int64_t* offset);
GPA_API int gpa_ipc_open(const void* handle, int64_t offset, void** ptr);
GPA_API int gpa_ipc_close(void* ptr, int64_t offset);

/*
 * The merged-block K/V exchange of the frame-sharded forward over NVLink peer
 * memory, fused with the scatter-mean (merging/merge.py:234-250, merge.heads,
 * whose slots the reference computes on one device; the collective itself has
 * no counterpart in the reference).  World ranks each own rows_per_rank
 * consecutive tokens; rank r's token rows (token t of the forward at row
 * t - r*rows_per_rank, row_elems elements, contiguous rows) are at
 * peer_rows[r], and every rank's merged output [unm_len + num_dst, row_elems]
 * at peer_out[r] -- both DEVICE arrays of `world` pointers as this process
 * addresses them (its own buffers and the peers' IPC mappings).  This rank
 * merges the slots whose token it owns -- unmerged slots s with
 * src_pos[unm_src[s]] in its rows, and dst slots [dst_lo, dst_hi) -- exactly as
 * gpa_merge_kv_mean does (fp32 sums, dst row first, then members in ascending
 * ordinal, divided by the count, rounded to dtype; bit-identical), reading
 * member rows from whichever rank holds them and storing each merged row into
 * every rank's output.  dtype GPA_DTYPE_BF16 or GPA_DTYPE_F32; row_elems % 8 ==
 * 0, <= 2048; buffers 16-byte aligned; world <= 8.  Every rank's row buffer
 * must be complete before any rank launches, and all launches finished before
 * an output is read or a row buffer rewritten (the caller orders them, e.g.
 * with a collective on the stream on both sides).  A token outside every
 * rank's rows is skipped and sets bit 2 of *status (when status != NULL).
 */
GPA_API int gpa_merge_exchange_p2p(const void* const* peer_rows, void* const* peer_out, int world,
                                   int rank, int dtype, int rows_per_rank, int row_elems,
                                   const int32_t* src_pos, const int32_t* dst_pos,
                                   const int32_t* unm_src, int unm_len, const int32_t* seg_start,
                                   const int32_t* seg_src, int num_dst, int dst_lo, int dst_hi,
                                   int* status, void* stream);

/*
 * Flash attention with a per-key additive bias (replaces
 * merging/fused_attention.py:130-180, kernel _attn_keybias_kernel :70-127):
 *   o[b,h,i]   = sum_j softmax_j(q.k_j * sm_scale + bias[b,h,j]) v_j
 *   lse[b,h,i] = log2 of the softmax denominator in the exp2 domain
 *                (m + log2(l) with scores scaled by log2(e)), as the reference.
 * q: [batch, heads, m, 64], k/v: [batch, heads, n, 64], o: like q; all bf16,
 * innermost dim contiguous, other strides multiples of 8 elements, 16-byte
 * aligned bases.  bias: fp32 (natural-log domain), bias[b,h,j] at
 * bias + b*bias_sb + h*bias_sh + j, or NULL for no bias.  lse may be NULL.
 */
GPA_API int gpa_attention_keybias(const void* q, const void* k, const void* v, const float* bias,
                          int batch, int heads, int m, int n, int head_dim, int64_t q_sb,
                          int64_t q_sh, int64_t q_sm, int64_t k_sb, int64_t k_sh, int64_t k_sn,
                          int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t bias_sb,
                          int64_t bias_sh, float sm_scale, void* o, int64_t o_sb, int64_t o_sh,
                          int64_t o_sm, float* lse, int64_t lse_sb, int64_t lse_sh, int* status,
                          void* stream);

/*
 * The same attention, combined in its epilogue with a second partition of the
 * same softmax over other keys (replaces the two-partition combine of
 * vggt/layers/attention.py:164-176 and the bf16 round trip before `proj`,
 * :229).  oa [batch, heads, m, 64] bf16 (strides oa_sb, oa_sh, oa_sm; multiples
 * of 8) is that partition's normalised output and lse_a [batch, heads, m] fp32
 * (strides lse_a_sb, lse_a_sh, row stride 1) its log2 row sums.  Each row
 * becomes o = (wa*oa + wb*ob) / (wa + wb), wa = 2^(lse_a - mx),
 * wb = 2^(lse_b - mx), mx = max(lse_a, lse_b), with ob and lse_b this call's
 * attention; lse, if given, receives the log2 row sums of the union.  o may be
 * the same memory as oa (every row is read before it is written), so the
 * frame blocks combine in place in the token-major layout `proj` reads.
 */
GPA_API int gpa_attention_keybias_combine(
    const void* q, const void* k, const void* v, const float* bias, int batch, int heads, int m, int n,
    int head_dim, int64_t q_sb, int64_t q_sh, int64_t q_sm, int64_t k_sb, int64_t k_sh, int64_t k_sn,
    int64_t v_sb, int64_t v_sh, int64_t v_sn, int64_t bias_sb, int64_t bias_sh, float sm_scale,
    const void* oa, int64_t oa_sb, int64_t oa_sh, int64_t oa_sm, const float* lse_a, int64_t lse_a_sb,
    int64_t lse_a_sh, void* o, int64_t o_sb, int64_t o_sh, int64_t o_sm, float* lse, int64_t lse_sb,
    int64_t lse_sh, int* status, void* stream);

/*
 * Content-adaptive pooling of each frame's patch keys/values (replaces
 * vggt/layers/attention.py:113-140, _pool).  Per head hh and frame s the patch
 * tokens t = num_special.. of k (grid ph x pw) join the seed on the stride-kp
 * lattice with the highest cosine similarity (fp32, norms clamped at 1e-6,
 * first seed on ties); a summary is the fp32 mean of its group.
 * k, v: [heads, S*P, 64] bf16 with strides (stride_h, stride_n), P = ph*pw+num_special.
 * Outputs: pk, pv [heads, S*npool, 64] bf16 with strides (out_stride_h, out_stride_n),
 * pool_size [heads, S*npool] fp32 contiguous (group sizes), npool =
 * ceil(ph/kp)*ceil(pw/kp) <= 64.
 */
GPA_API int gpa_frame_pool(const void* k, const void* v, int heads, int num_frames, int ph, int pw,
                   int num_special, int kp, int64_t stride_h, int64_t stride_n, void* pk,
                   void* pv, int64_t out_stride_h, int64_t out_stride_n, float* pool_size,
                   void* stream);

/*
 * Exact combine of two attention partitions (replaces
 * vggt/layers/attention.py:164-176): with log2 sums la, lb,
 *   wa = 2^(la-mx), wb = 2^(lb-mx), mx = max(la, lb)
 *   o  = bf16(wa/(wa+wb)) * oa + bf16(wb/(wa+wb)) * ob
 * Rows are addressed as (head, frame, row-in-frame); each *_strides array holds
 * the three element strides of that tensor in this order.  oa, ob, o: bf16
 * with head_dim contiguous elements per row; la, lb: fp32.
 */
GPA_API int gpa_lse_combine(int heads, int frames, int rows_per_frame, int head_dim, const void* oa,
                    const int64_t* oa_strides, const float* la, const int64_t* la_strides,
                    const void* ob, const int64_t* ob_strides, const float* lb,
                    const int64_t* lb_strides, void* o, const int64_t* o_strides, void* stream);

/*
 * LayerNorm of bf16 rows with fp32 statistics and a bf16 result (the norm1 /
 * norm2 of vggt/layers/block.py:85-92 as a bf16-autocast Linear consumes it).
 * out[r, c] = bf16((x[r, c] - mean_r) * rsqrt(var_r + eps) * w[c] + b[c]).
 * cols % 256 == 0 and cols <= 4096; weight/bias of dtype param_dtype (f32 or bf16).
 */
GPA_API int gpa_layernorm_bf16(const void* x, int64_t x_stride, int rows, int cols,
                               const void* weight, const void* bias, int param_dtype, float eps,
                               void* out, int64_t out_stride, void* stream);

/*
 * qk-LayerNorm + 2D rotary embedding, fused (vggt/layers/attention.py:216-220
 * with vggt/layers/rope.py:139-209).  For each token t and head h of a qkv
 * buffer (q row at qkv + t*token_stride + q_offset + h*64, k row at k_offset):
 * LayerNorm over the 64 features (fp32, eps, per-head weight/bias; NULL = none),
 * then, if positions != NULL, rotation of features 0..31 by positions[t, 0] and
 * 32..63 by positions[t, 1] with the rotate-half pairing (i, i+16) and the
 * fp32 cos/sin tables [n_pos, 32]; the bf16 results go to q_out / k_out
 * (+ t*out_token_stride + h*64), which may alias the q / k rows of qkv.
 */
GPA_API int gpa_qk_norm_rope(const void* qkv, int64_t token_stride, int64_t q_offset,
                             int64_t k_offset, int tokens, int heads, int head_dim,
                             const void* q_weight, const void* q_bias, const void* k_weight,
                             const void* k_bias, int param_dtype, float eps,
                             const int64_t* positions, const float* cos_table,
                             const float* sin_table, int n_pos, void* q_out, void* k_out,
                             int64_t out_token_stride, void* stream);

/*
 * Residual + LayerScale (vggt/layers/block.py:88,94 with
 * vggt/layers/layer_scale.py:21): out[r, c] = bf16(x[r, c] + bf16(y[r, c] * gamma[c])),
 * rounding exactly as torch's bf16 `x + y * gamma`.  All bf16; rows of `cols`
 * contiguous elements at the given row strides (elements); cols % 8 == 0;
 * 16-byte aligned rows and gamma.  out may alias x.
 */
GPA_API int gpa_residual_scale_bf16(const void* x, int64_t x_stride, const void* y,
                                    int64_t y_stride, const void* gamma, int rows, int cols,
                                    void* out, int64_t out_stride, void* stream);

/*
 * DPT head resize (heads/dpt_head.py custom_interpolate -> out_conv /
 * output_conv2, and _apply_pos_embed): bilinear, align_corners=True, in fp32,
 * of a channels-last map x [n, c, h, w] of dtype x_dtype (f32 or bf16;
 * element strides x_sn, x_sh, x_sw; channel stride 1) to out_h x out_w.
 * Optionally adds an fp32 map add[c, out_h, out_w] (strides add_sh, add_sw;
 * channel stride 1, broadcast over n), after rounding the resize to bf16 first
 * when round_first != 0; writes bf16 channels-last out: the value a
 * bf16-autocast convolution receives after the reference's resize (and add).
 * c % 8 == 0; 16-byte aligned pixels.
 */
GPA_API int gpa_upsample_bilinear_bf16(const void* x, int x_dtype, int n, int c, int h, int w,
                                       int64_t x_sn, int64_t x_sh, int64_t x_sw, const float* add,
                                       int64_t add_sh, int64_t add_sw, int round_first, int out_h,
                                       int out_w, void* out, int64_t out_sn, int64_t out_sh,
                                       int64_t out_sw, void* stream);

/*
 * Bias, ReLU and residual after a DPT-head convolution, one pass over a
 * channels-last bf16 map (replaces the bias add torch issues after each cuDNN
 * convolution, the ReLU and the skip add of heads/dpt_head.py
 * ResidualConvUnit): t = bf16(y + bias[c]); t = relu(t) if relu; out =
 * bf16(t + res) if res.  Rounds as those torch ops do (bit-exact).  y, res,
 * out: [pixels, c] bf16 contiguous (a channels-last map), c % 8 == 0, out may
 * be y; bias: [c] bf16.
 */
GPA_API int gpa_bias_act_bf16(const void* y, const void* bias, const void* res, int64_t pixels, int c,
                              int relu, void* out, void* stream);

/*
 * Exact GELU of the MLP (vggt/layers/mlp.py, nn.GELU()): out[i] =
 * bf16(0.5 * x * (1 + erf(x / sqrt(2)))) in fp32 for n bf16 values, as torch
 * evaluates it for bf16 tensors.  n % 8 == 0, 16-byte aligned; out may alias x.
 */
GPA_API int gpa_gelu_bf16(const void* x, int64_t n, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GPA_B200_H */
