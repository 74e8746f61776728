/*
 * mi_layers.h — C ABI of the fused row operations that feed and follow the paged attention
 * (libmi_paged.so, sm_100a).  Same conventions as mi_paged.h: plain device pointers, strides in
 * ELEMENTS, the CUDA stream as void*, no allocation or synchronization, MI_OK or MI_ERR_*.
 *
 * These replace chains of PyTorch element-wise launches of the reference model
 * (model/qwen3.py) with one launch each, keeping the chains' rounding points: in a 16-bit model
 * every intermediate the reference materialises in the model dtype is rounded to it here too;
 * statistics are fp32.  They exist to cut the launch count of a decode step (a CUDA-graph replay
 * of ~10 launches per layer instead of ~55) and to put the decode KV append where K is produced.
 */
#ifndef MI_LAYERS_H
#define MI_LAYERS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * mi_rmsnorm — out = RMSNorm(h) with h = x, or h = x + residual when `residual` is not NULL
 * (then h is also written to `residual_out` when that is not NULL; it may equal `residual`).
 * RMSNorm(h)_i = w_i * T(h_i * rsqrt(mean_j(h_j^2) + eps)), T = the element type.
 * Replaces RMSNorm.forward (model/qwen3.py:67-78) and, fused, the residual add before it
 * (Qwen3DecoderLayer.forward).  x, residual, residual_out, out: [rows, hidden] with the given row
 * strides (elements), unit stride inside a row.  hidden <= 8192 (16-bit) / 4096 (fp32) when the
 * rows are 16-byte aligned, <= 1024 otherwise.
 */
int mi_rmsnorm(const void* x, int64_t x_row_stride, const void* residual, int64_t residual_row_stride,
               void* residual_out, int64_t residual_out_row_stride, const void* weight, void* out,
               int64_t out_row_stride, int64_t rows, int hidden, float eps, int dtype, void* stream);

/*
 * mi_qk_norm_rope — per token t and head h: RMSNorm over head_dim with q_weight (query heads) or
 * k_weight (KV heads), then rotate-half RoPE with cos/sin [tokens, head_dim] in the element type:
 * out = T(T(y * cos) + T(rot(y) * sin)).  Replaces Qwen3Attention._project_qkv's q_norm, k_norm
 * and apply_rotary (model/qwen3.py:112-144, :182-217).
 *   q [tokens, hq, head_dim] at row stride q_row_stride; k, v [tokens, hkv, head_dim] likewise
 *   q_out [tokens, hq, head_dim] contiguous (required)
 *   k_out, v_out [tokens, hkv, head_dim] contiguous, each optional (NULL): roped K and a copy of V
 *   slot_mapping [tokens] int64, optional: the decode append — roped K and V also go to
 *     k_pool / v_pool [num_blocks*block_size, hkv, head_dim] at those slots (replaces
 *     Qwen3Attention._apply_paged_kv_pool's index_copy_, model/qwen3.py:282-283); an
 *     out-of-range slot is skipped and sets MI_STATUS_BAD_SLOT.
 * head_dim in {32, 64, 128, 256}.
 */
int mi_qk_norm_rope(const void* q, int64_t q_row_stride, const void* k, int64_t k_row_stride, const void* v,
                    int64_t v_row_stride, const void* q_weight, const void* k_weight, const void* cos,
                    const void* sin, int64_t cos_sin_row_stride, int64_t tokens, int hq, int hkv, int head_dim,
                    float eps, void* q_out, void* k_out, void* v_out, const int64_t* slot_mapping, void* k_pool,
                    void* v_pool, int64_t num_slots, int dtype, void* stream);

/*
 * mi_silu_mul — out = T(T(silu(gate)) * up), silu(g) = g / (1 + exp(-g)) in fp32: the MLP's
 * F.silu(gate_proj(x)) * up_proj(x) (model/qwen3.py, Qwen3MLP).  gate and up share a row stride
 * (they may be the two halves of one [rows, 2*cols] GEMM output).
 */
int mi_silu_mul(const void* gate, const void* up, int64_t in_row_stride, void* out, int64_t out_row_stride,
                int64_t rows, int64_t cols, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MI_LAYERS_H */
