/*
 * opengenie-b200 C ABI: the hot path of LTX-2.3's video self-attention block
 * on NVIDIA B200 (sm_100a).
 *
 * Every entry point:
 *   - takes device pointers the caller allocated (the library never allocates,
 *     frees or keeps tensor memory), plain sizes and element strides, and a
 *     cudaStream_t passed as `void*` (null = legacy default stream);
 *   - is stream-ordered and asynchronous: it enqueues kernels and returns;
 *   - returns OGX_OK (0) or a negative OGX_E* code; ogx_last_error() then
 *     names the failed guard with the reference's reason string (e.g.
 *     "qk_shape", "rope_shape") or the CUDA error.  There is no CPU fallback.
 * Device-side waits are bounded; a wait that gives up sets a status bit that
 * ogx_device_status() reads.
 *
 * Reference interfaces (plugyawn/opengenie) each entry point replaces are
 * cited as file:line.
 */
#ifndef OGX_H_
#define OGX_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OGX_OK 0
#define OGX_EINVAL (-1)   /* a guard rejected the arguments */
#define OGX_ECUDA (-2)    /* a CUDA runtime/driver call failed */

/* dtype codes */
#define OGX_DTYPE_BF16 0
#define OGX_DTYPE_F32 1
#define OGX_DTYPE_F16 2

/* E4M3 quantiser semantics */
#define OGX_QUANT_TORCH 0  /* ltx_serve/triton_ltx_ops.py:146-148 (bit-exact target) */
#define OGX_QUANT_SINGLE 1 /* ltx_serve/triton_ltx_ops.py:3429-3444 (one rounding)  */

int ogx_version(void);
const char* ogx_last_error(void);

/* Reads (and with clear != 0 resets) the device status word of the current
 * device: bit 1 = a bounded device-side wait gave up.  Synchronous. */
int ogx_device_status(unsigned int* status, int clear);

/* AdaZero with Ada values read from scale_shift_table + timestep:
 *   y = rmsnorm(x, eps) * (1 + scale) + shift, fp32 math, one bf16 rounding,
 *   shift/scale = bf16?(bf16?(table[idx]) + ts[b, t, idx, :]).
 * x: bf16 [batch, tokens, cols] contiguous, cols in {2048, 4096};
 * table: [P, cols] (bf16/f32), row stride table_stride_row, unit column stride;
 * timestep viewed [batch, tokens, P, cols] with strides (ts_stride_b,
 * ts_stride_t, ts_stride_p, 1) elements (ts_stride_t may be 0).
 * Replaces fused_adazero_from_ada, ltx_serve/triton_ltx_ops.py:40-91. */
int ogx_adazero_from_ada(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                         int table_dtype, int64_t table_stride_row, const void* timestep, int timestep_dtype,
                         int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int shift_index,
                         int scale_index, float eps, void* y, void* stream);

/* Optional per-head gate of the attention output: y = bf16(x * gates[row, col / dim_head]); x, y bf16
 * [rows, heads * dim_head] contiguous (dim_head a multiple of 8), gates bf16 with element strides
 * gate_stride_row, gate_stride_head.  Replaces fused_head_gate_mul_bf16,
 * ltx_serve/triton_ltx_ops.py:614-637 (kernel :3584-3609). */
int ogx_head_gate_mul_bf16(const void* x, int64_t rows, int64_t heads, int64_t dim_head, const void* gates,
                           int64_t gate_stride_row, int64_t gate_stride_head, void* y, void* stream);

/* The AdaLN affine without the norm: y = bf16(bf16(x * bf16(1 + scale)) + shift), shift/scale from
 * table + timestep as for ogx_adazero_from_ada (arguments likewise, no eps).
 * Replaces fused_adaln_affine_from_ada, ltx_serve/triton_ltx_ops.py:94-141 (kernel :3469-3534). */
int ogx_adaln_affine_from_ada(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                              int table_dtype, int64_t table_stride_row, const void* timestep, int timestep_dtype,
                              int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int shift_index,
                              int scale_index, void* y, void* stream);

/* y = bf16(x * gate), gate = the Ada value of slot gate_index (table + timestep, arguments as for
 * ogx_adazero_from_ada).  Replaces fused_mul_from_ada, ltx_serve/triton_ltx_ops.py:695-741
 * (kernel :3723-3771). */
int ogx_mul_from_ada(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table, int table_dtype,
                     int64_t table_stride_row, const void* timestep, int timestep_dtype, int64_t ts_stride_b,
                     int64_t ts_stride_t, int64_t ts_stride_p, int gate_index, void* y, void* stream);

/* Same, fused with the per-tensor E4M3 activation quantiser: q = quant(y)
 * (y itself is written only when y != NULL).  The codes equal
 * ogx_fp8_quantize_e4m3 applied to the bf16 y.
 * Replaces fused_adazero_from_ada (:40-91) followed by
 * fused_fp8_quantize_e4m3 (:144-161) inside FP8Linear.forward (:1676-1716). */
int ogx_adazero_from_ada_e4m3(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                              int table_dtype, int64_t table_stride_row, const void* timestep, int timestep_dtype,
                              int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int shift_index,
                              int scale_index, float eps, const float* input_scale, int quant_mode, void* y,
                              void* q, void* stream);

/* Same, with up to three e4m3 outputs of the one bf16 y: output i = quant_{input_scales[i]}(y) at
 * q + i * q_plane_stride (bytes, a multiple of 16).  The checkpoint path whose Q, K and V linears carry
 * different input scales: the reference quantises the bf16 AdaZero output once per linear inside
 * FP8Linear.forward (ltx_serve/triton_ltx_ops.py:1692, :1676-1716); here x is read once. */
int ogx_adazero_from_ada_e4m3_planes(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                                     int table_dtype, int64_t table_stride_row, const void* timestep,
                                     int timestep_dtype, int64_t ts_stride_b, int64_t ts_stride_t,
                                     int64_t ts_stride_p, int shift_index, int scale_index, float eps,
                                     const float* input_scales, int planes, int quant_mode, void* y, void* q,
                                     int64_t q_plane_stride, void* stream);

/* Per-tensor E4M3 quantiser: q = e4m3(clamp(x * (1/s), -448, 448)).
 * x: bf16 or f16, n elements contiguous; input_scale: device f32 scalar.
 * Replaces fused_fp8_quantize_e4m3, ltx_serve/triton_ltx_ops.py:144-161. */
int ogx_fp8_quantize_e4m3(const void* x, int x_dtype, int64_t n, const float* input_scale, int quant_mode, void* q,
                          void* stream);

/* GELU (tanh approximation) fused with the per-tensor E4M3 quantiser:
 * q = quant(round_to_x_dtype(gelu(x))); gelu_out (may be NULL) receives the rounded GELU values.
 * x: bf16 or f16, n elements contiguous; input_scale: device f32 scalar.
 * Replaces fused_gelu_tanh_fp8_quantize_e4m3, ltx_serve/triton_ltx_ops.py:164-182 (torch path
 * :166-169; Triton kernel :3535-3550). */
int ogx_gelu_tanh_fp8_quantize_e4m3(const void* x, int x_dtype, int64_t n, const float* input_scale, void* q,
                                    void* gelu_out, void* stream);

/* out = bf16(x + bf16(bias)); x bf16 [rows, cols] contiguous, bias [cols].
 * Replaces fused_bias_add_bf16, ltx_serve/triton_ltx_ops.py:185-201. */
int ogx_bias_add_bf16(const void* x, int64_t rows, int64_t cols, const void* bias, int bias_dtype, void* out,
                      void* stream);

/* out = bf16(x + bf16(bf16(y + bf16(bias)) * gate)), gate from table/timestep
 * slot gate_index (same conventions as ogx_adazero_from_ada).
 * Replaces fused_residual_gate_bias_from_ada, ltx_serve/triton_ltx_ops.py:204-262. */
int ogx_residual_gate_bias_from_ada(const void* x, const void* y, int64_t batch, int64_t tokens, int64_t cols,
                                    const void* bias, int bias_dtype, const void* table, int table_dtype,
                                    int64_t table_stride_row, const void* timestep, int timestep_dtype,
                                    int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int gate_index,
                                    void* out, void* stream);

/* Q/K RMSNorm over 4096 columns (with weight) + split RoPE per head (32 heads
 * x 128), fp32 math, one bf16 rounding.  q/k: bf16 rows of 4096 with token
 * stride in_stride_t; cos/sin: [32, tokens, 64] with strides (cs_stride_h,
 * cs_stride_t, 1) (bf16 or f32); outputs bf16 with token stride out_stride_t
 * (may alias the inputs).
 * Replaces fused_video_qk_rmsnorm_rope, ltx_serve/triton_ltx_ops.py:320-378. */
int ogx_video_qk_rmsnorm_rope(const void* q, const void* k, int64_t tokens, int64_t in_stride_t,
                              const void* q_weight, const void* k_weight, int weight_dtype, float eps,
                              const void* cos, const void* sin, int cs_dtype, int64_t cs_stride_h,
                              int64_t cs_stride_t, void* q_out, void* k_out, int64_t out_stride_t, void* stream);

/* ogx_video_qk_rmsnorm_rope with the cos/sin generated in the kernel instead of read from tables: token i
 * (global index token0 + i) sits at (t, h, w) = (g / (grid_h*grid_w), (g / grid_w) % grid_h, g % grid_w)
 * of the latent raster, and rotary slot s = 64*head + j turns by position[slot_axis[s]] * inv_freq[s]
 * radians (axis 0 = t, 1 = h, 2 = w); cos and sin are rounded to bf16 before use, as the reference's bf16
 * tables hold them.  inv_freq: float64 [2048] and slot_axis: uint8 [2048], device memory.  Saves the
 * tables' 8 KB of HBM reads per token.  The reference builds these tables in the un-vendored ltx_core
 * preprocessor and caches them (ltx_serve/triton_ltx_ops.py:2413-2497); the arithmetic on q/k is that of
 * fused_video_qk_rmsnorm_rope, :320-378. */
int ogx_video_qk_rmsnorm_rope_positions(const void* q, const void* k, int64_t tokens, int64_t in_stride_t,
                                        const void* q_weight, const void* k_weight, int weight_dtype, float eps,
                                        const double* inv_freq, const unsigned char* slot_axis, int64_t grid_h,
                                        int64_t grid_w, int64_t token0, void* q_out, void* k_out,
                                        int64_t out_stride_t, void* stream);

/* ogx_video_qkv_rmsnorm_rope_scatter with the cos/sin generated from positions as in
 * ogx_video_qk_rmsnorm_rope_positions. */
int ogx_video_qkv_rmsnorm_rope_positions_scatter(const void* q, const void* k, const void* v, int64_t tokens,
                                                 int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                                 int weight_dtype, float eps, const double* inv_freq,
                                                 const unsigned char* slot_axis, int64_t grid_h, int64_t grid_w,
                                                 int64_t token0, void* q_out, void* k_out, void* v_out,
                                                 int64_t out_stride_t, int64_t out_stride_g, int heads_per_group,
                                                 void* stream);

/* The cos/sin ogx_video_qk_rmsnorm_rope_positions generates, written as [32, tokens, 64] tables (bf16 or
 * f32) for tokens [token0, token0 + tokens): the tables the reference's interface takes
 * (ltx_serve/triton_ltx_ops.py:2413-2497 caches them), bit-equal to the generated values. */
int ogx_rope_tables_from_positions(const double* inv_freq, const unsigned char* slot_axis, int64_t grid_h,
                                   int64_t grid_w, int64_t token0, int64_t tokens, int cs_dtype, void* cos_out,
                                   void* sin_out, void* stream);

/* The same normalisation + RoPE, writing Q/K and copying V into the
 * head-grouped send layout of the sequence-to-head exchange: head h of token t
 * goes to out + t*out_stride_t + (h / heads_per_group)*out_stride_g +
 * (h % heads_per_group)*128.  No reference counterpart for the layout (the
 * reference is single-GPU); the arithmetic is that of
 * fused_video_qk_rmsnorm_rope (:320-378). */
int ogx_video_qkv_rmsnorm_rope_scatter(const void* q, const void* k, const void* v, int64_t tokens,
                                       int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                       int weight_dtype, float eps, const void* cos, const void* sin, int cs_dtype,
                                       int64_t cs_stride_h, int64_t cs_stride_t, void* q_out, void* k_out,
                                       void* v_out, int64_t out_stride_t, int64_t out_stride_g,
                                       int heads_per_group, void* stream);

/* Q/K RMSNorm over 4096 columns (with weight) and no rotary embedding, fp32 math, one bf16 rounding
 * (the arithmetic of ogx_video_qk_rmsnorm_rope with cos = 1, sin = 0): q_out = rmsnorm(q) * q_weight
 * over q_rows rows and k_out = rmsnorm(k) * k_weight over k_rows rows in one launch.  q and k may have
 * different row counts (queries from the video tokens, keys from the text context); each has its own
 * row stride (a multiple of 8) and the outputs may alias the inputs.  weight_dtype: bf16 or f32.
 * Replaces attn.q_norm(q), attn.k_norm(k) of the pre-attention when no positional embedding is given
 * (ltx_serve/triton_ltx_ops.py:1864-1865; the text cross-attention, :2880). */
int ogx_qk_rmsnorm(const void* q, int64_t q_rows, int64_t q_stride, const void* k, int64_t k_rows, int64_t k_stride,
                   const void* q_weight, const void* k_weight, int weight_dtype, float eps, void* q_out,
                   int64_t q_out_stride, void* k_out, int64_t k_out_stride, void* stream);

/* FP8 scaled matmul with bias epilogue (tcgen05, e4m3 x e4m3 -> f32 -> bf16):
 *   out[m, n] = bf16(bf16(acc * scale_a * scale_b[n / n_per_scale]) + bf16(bias[n]))
 * a: e4m3 [M, K] (row stride lda), w: e4m3 [N, K] (row stride ldw), both
 * K-major; scales are device f32 (scale_b has N / n_per_scale entries); bias
 * may be NULL; out bf16 [M, N] with row stride ldo.  K % 16 == 0, N % 32 == 0.
 * Replaces torch._scaled_mm(a, w.t(), scale_a, scale_b, out_dtype=bf16,
 * use_fast_accum=True) + bias add in FP8Linear.forward,
 * ltx_serve/triton_ltx_ops.py:1695-1707 and :742-759. */
int ogx_fp8_scaled_mm(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                      const float* scale_a, const float* scale_b, int64_t n_per_scale, const void* bias,
                      int bias_dtype, void* out, int64_t ldo, void* stream);

/* ogx_fp8_scaled_mm over `planes` activation planes: a holds planes e4m3 [M, K] planes (row stride lda,
 * plane stride M * lda); output columns [i*N/planes, (i+1)*N/planes) read plane i with scale_a[i] and
 * scale_b[i] (N / planes a multiple of 256).  One launch for the packed Q/K/V projection of a checkpoint
 * whose three linears quantise their input with different scales, where the reference runs three
 * FP8Linear.forward calls (ltx_serve/triton_ltx_ops.py:1695-1707, once per linear). */
int ogx_fp8_scaled_mm_planes(const void* a, int64_t planes, int64_t M, int64_t K, int64_t lda, const void* w,
                             int64_t N, int64_t ldw, const float* scale_a, const float* scale_b, const void* bias,
                             int bias_dtype, void* out, int64_t ldo, void* stream);

/* The FFN's first projection with GELU and the next projection's input quantiser in the epilogue:
 * out_q = quant_{q_scale}(bf16(gelu(bf16(bf16(a @ w^T * scale_a * scale_b) + bf16(bias))))), e4m3
 * [M, N] with row stride ldq (a multiple of 16).  Equals ogx_fp8_scaled_mm followed by
 * ogx_gelu_tanh_fp8_quantize_e4m3 on its bf16 output, without the bf16 hidden tensor in HBM.
 * Replaces the video FFN's FeedForward net[0] (FP8Linear.forward :1695-1707 + gelu tanh) and the
 * quantiser of net[2] (fp8_linear_without_bias :770-771; _feedforward_without_out_bias :2796-2807). */
int ogx_fp8_scaled_mm_gelu_e4m3(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N,
                                int64_t ldw, const float* scale_a, const float* scale_b, int64_t n_per_scale,
                                const void* bias, int bias_dtype, const float* q_scale, void* out_q, int64_t ldq,
                                void* stream);

/* FP8 scaled matmul fused with the block's output epilogue:
 *   y = bf16(bf16(acc * scale_a * scale_b) + bf16(bias)),
 *   out = bf16(x + bf16(y * gate)), gate from table/timestep slot gate_index
 * (rows are tokens of batch 1).
 * Replaces fp8_linear_without_bias (ltx_serve/triton_ltx_ops.py:762-781)
 * followed by fused_residual_gate_bias_from_ada (:204-262). */
int ogx_fp8_scaled_mm_residual_gate(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N,
                                    int64_t ldw, const float* scale_a, const float* scale_b, int64_t n_per_scale,
                                    const void* bias, int bias_dtype, const void* x, int64_t ldx,
                                    const void* table, int table_dtype, int64_t table_stride_row,
                                    const void* timestep, int timestep_dtype, int64_t ts_stride_t,
                                    int64_t ts_stride_p, int gate_index, void* out, int64_t ldo, void* stream);

/* The same fused out-projection with A read from the receive buffer of the
 * head-to-sequence exchange: A is K / k_block blocks of [M, k_block] e4m3
 * (block s = the columns [s*k_block, (s+1)*k_block) sent by rank s), so no
 * permute runs between the exchange and the GEMM.  k_block % 128 == 0.
 * No reference counterpart for the layout (the reference is single-GPU); the
 * arithmetic is that of ogx_fp8_scaled_mm_residual_gate. */
int ogx_fp8_scaled_mm_residual_gate_kblocked(const void* a, int64_t M, int64_t K, int64_t k_block, const void* w,
                                             int64_t N, int64_t ldw, const float* scale_a, const float* scale_b,
                                             int64_t n_per_scale, const void* bias, int bias_dtype, const void* x,
                                             int64_t ldx, const void* table, int table_dtype,
                                             int64_t table_stride_row, const void* timestep, int timestep_dtype,
                                             int64_t ts_stride_t, int64_t ts_stride_p, int gate_index, void* out,
                                             int64_t ldo, void* stream);

/* Dense bidirectional attention (tcgen05 + TMEM, online softmax), head_dim 128:
 *   out[b, t, h, :] = softmax(q[b,t,h,:] . k[b,:,h,:]^T * softmax_scale) v[b,:,h,:]
 * q/k/v: bf16, element (b, t, h, d) at ptr + b*stride_b + t*stride_t + h*128 + d
 * (all three share the strides; stride_t % 8 == 0); out bf16 with its own
 * strides.  Replaces the attention backend call attn.attention_function(q, k,
 * v, heads) (ltx_serve/triton_ltx_ops.py:2636; backend contract
 * benchmarks/official_ltx23_benchmark.py:3289-3373). */
int ogx_attention_fwd(const void* q, const void* k, const void* v, int64_t batch, int64_t tokens, int64_t heads,
                      int64_t head_dim, int64_t stride_b, int64_t stride_t, float softmax_scale, void* out,
                      int64_t out_stride_b, int64_t out_stride_t, void* stream);

/* Same attention, with the output quantised to e4m3 for the output projection
 * (bf16 rounding of O first, then the torch-path quantiser with *out_scale),
 * i.e. fused_fp8_quantize_e4m3(attention(q, k, v), to_out.input_scale) as in
 * fp8_linear_without_bias (ltx_serve/triton_ltx_ops.py:770-771). */
int ogx_attention_fwd_e4m3(const void* q, const void* k, const void* v, int64_t batch, int64_t tokens,
                           int64_t heads, int64_t head_dim, int64_t stride_b, int64_t stride_t, float softmax_scale,
                           const float* out_scale, void* out_q, int64_t out_stride_b, int64_t out_stride_t,
                           void* stream);

/* Attention whose keys and values come from a sequence of another length: q has q_tokens rows with
 * strides (q_stride_b, q_stride_t), k and v have kv_tokens rows sharing (kv_stride_b, kv_stride_t); no
 * mask.  Replaces the attention backend call of the text cross-attention (attn2: queries from the
 * video tokens, keys/values from the prompt context), which the backend serves by viewing k and v as
 * [b, -1, heads, d] (benchmarks/official_ltx23_benchmark.py:3294-3305; call ltx_serve/triton_ltx_ops.py:2880). */
int ogx_attention_fwd_kv(const void* q, const void* k, const void* v, int64_t batch, int64_t q_tokens,
                         int64_t kv_tokens, int64_t heads, int64_t head_dim, int64_t q_stride_b, int64_t q_stride_t,
                         int64_t kv_stride_b, int64_t kv_stride_t, float softmax_scale, void* out,
                         int64_t out_stride_b, int64_t out_stride_t, void* stream);

/* ogx_attention_fwd_kv with the output quantised to e4m3 as in ogx_attention_fwd_e4m3. */
int ogx_attention_fwd_kv_e4m3(const void* q, const void* k, const void* v, int64_t batch, int64_t q_tokens,
                              int64_t kv_tokens, int64_t heads, int64_t head_dim, int64_t q_stride_b,
                              int64_t q_stride_t, int64_t kv_stride_b, int64_t kv_stride_t, float softmax_scale,
                              const float* out_scale, void* out_q, int64_t out_stride_b, int64_t out_stride_t,
                              void* stream);

/* ---- Sequence-parallel exchange over NVLink (no reference counterpart: the reference is single-GPU).
 * Buffers are shared between the ranks' processes with CUDA IPC; the producing kernels store straight
 * into the destination GPU's receive buffer and a bounded-wait barrier kernel orders producer and
 * consumer.  No NVLink multicast is used. */

/* IPC handle (64 bytes) of the allocation holding ptr, and ptr's offset in it. */
int ogx_ipc_get_handle(const void* ptr, void* handle, int64_t* offset);
/* Maps a peer's allocation into this process; *base + offset addresses the peer's buffer. */
int ogx_ipc_open_handle(const void* handle, void** base);
int ogx_ipc_close_handle(void* base);

/* Cross-GPU barrier.  Each rank's signal block is 16 zero-initialised uint32 words in its own memory
 * ([0,8) arrival slots, [8] the count of barriers passed), mapped into the peers with IPC
 * (peer_signals[i] = rank i's block).  Barrier e = count + 1: stores e into slot `rank` of every peer's
 * block and waits, bounded, until every peer's slot in local_signals reaches e, then advances the count.
 * The arguments are the same on every call, so steps containing barriers can be captured in a CUDA
 * graph.  All ranks must run the same barriers in the same order.  One 32-thread launch. */
int ogx_peer_barrier(unsigned int* local_signals, void* const* peer_signals, int rank, int world, void* stream);

/* No counterpart in the reference (an addition of this library).  ogx_peer_barrier for callers that
 * cannot allocate device memory, e.g. a runtime driving all of its GPUs from one process with their
 * memory reserved up front for its own pool.  The barrier count is a 64-byte array inside the library,
 * one per GPU that loads it and held until the process exits; it is zero at load and never cleared
 * (barrier numbers only grow).  The arrivals cross between GPUs through one 4 KB page of host memory
 * inside the library, page-locked and mapped into every GPU at the first call (cudaHostRegister; it
 * stays registered until the process exits), so no GPU touches another GPU's memory and no peer access
 * is needed.  Ranks are GPUs of this process: devices[i] is rank i's device ordinal (below 64, no
 * ordinal twice) and devices[rank] must be the current device.  world is at most 8; larger values are
 * rejected.  Set-up: the first call naming a device looks up that device's array address with the
 * device made current, which creates the device's primary context if it has none (the context, not
 * this call, takes device memory) and may load the library's module there.  So every device in
 * devices[] should already have its context, and one warm-up call per rank should run before serving
 * starts and before any stream capture.  count_out (device memory, may be NULL) receives the number of
 * barriers this rank has passed.  Every call on a device shares its count and its row of arrival slots:
 * one barrier group per process, and calls that overlap on a GPU race.  Allocates no device memory. */
int ogx_peer_barrier_static(int rank, int world, const int* devices, unsigned int* count_out, void* stream);

/* ogx_video_qkv_rmsnorm_rope_scatter with one destination base per head group (groups = world size):
 * head h of token t goes to group_bases[h / (32/groups)] + t*out_stride_t + {0, 1, 2}*(32/groups)*128
 * (q, k, v) + (h % (32/groups))*128, stored over NVLink when the base is a peer's receive buffer;
 * the kernel fences its stores system-wide before it exits. */
int ogx_video_qkv_rmsnorm_rope_to_peers(const void* q, const void* k, const void* v, int64_t tokens,
                                        int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                        int weight_dtype, float eps, const void* cos, const void* sin, int cs_dtype,
                                        int64_t cs_stride_h, int64_t cs_stride_t, void* const* group_bases,
                                        int groups, int64_t out_stride_t, void* stream);

/* ogx_video_qkv_rmsnorm_rope_to_peers with the cos/sin generated from positions as in
 * ogx_video_qk_rmsnorm_rope_positions (token0 = the first token of this rank's slice). */
int ogx_video_qkv_rmsnorm_rope_positions_to_peers(const void* q, const void* k, const void* v, int64_t tokens,
                                                  int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                                  int weight_dtype, float eps, const double* inv_freq,
                                                  const unsigned char* slot_axis, int64_t grid_h, int64_t grid_w,
                                                  int64_t token0, void* const* group_bases, int groups,
                                                  int64_t out_stride_t, void* stream);

/* ogx_attention_fwd_e4m3 (batch 1) whose output row for token t goes to
 * peer_bases[t / tokens_per_peer] + (t % tokens_per_peer)*out_stride_t + head*128 (the receive buffers
 * of the head-to-sequence exchange, stored over NVLink); stores are fenced system-wide. */
int ogx_attention_fwd_e4m3_to_peers(const void* q, const void* k, const void* v, int64_t tokens, int64_t heads,
                                    int64_t stride_t, float softmax_scale, const float* out_scale,
                                    void* const* peer_bases, int peers, int64_t tokens_per_peer,
                                    int64_t out_stride_t, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OGX_H_ */
