// Host entry points of include/mi_layers.h: argument checks, then one launch each.
#include "../../include/mi_layers.h"

namespace {

bool all_aligned16(std::initializer_list<const void*> ptrs, std::initializer_list<int64_t> byte_values) {
  return pick_vec(ptrs, byte_values) == 16;
}

}  // namespace

int mi_rmsnorm(const void* x, int64_t x_row_stride, const void* residual, int64_t residual_row_stride,
               void* residual_out, int64_t residual_out_row_stride, const void* weight, void* out,
               int64_t out_row_stride, int64_t rows, int hidden, float eps, int dtype, void* stream) {
  const int es = elem_size(dtype);
  if (es == 0) return fail(MI_ERR_INVALID, "mi_rmsnorm: unknown dtype %d", dtype);
  if (rows < 0 || hidden <= 0) return fail(MI_ERR_INVALID, "mi_rmsnorm: bad shape rows=%lld hidden=%d",
                                           (long long)rows, hidden);
  if (rows == 0) return MI_OK;
  if (!x || !weight || !out) return fail(MI_ERR_INVALID, "mi_rmsnorm: null pointer argument");
  if (rows > INT32_MAX) return fail(MI_ERR_UNSUPPORTED, "mi_rmsnorm: more than 2^31 rows");
  mi::RmsNormArgs a{};
  a.x = static_cast<const char*>(x);
  a.x_rs = x_row_stride * es;
  a.res = static_cast<const char*>(residual);
  a.res_rs = residual_row_stride * es;
  a.res_out = residual ? static_cast<char*>(residual_out) : nullptr;
  a.res_out_rs = residual_out_row_stride * es;
  a.w = static_cast<const char*>(weight);
  a.out = static_cast<char*>(out);
  a.out_rs = out_row_stride * es;
  a.rows = rows;
  a.hidden = hidden;
  a.eps = eps;
  a.inv_hidden = 1.0f / (float)hidden;
  const bool vec16 = all_aligned16({x, residual ? residual : x, a.res_out ? a.res_out : x, weight, out},
                                   {a.x_rs, a.res_rs, a.res_out_rs, a.out_rs, (int64_t)hidden * es});
  const int per_vec = vec16 ? 16 / es : 1;
  if ((hidden + per_vec - 1) / per_vec > 128 * 8)
    return fail(MI_ERR_UNSUPPORTED, "mi_rmsnorm: hidden %d too large for one CTA per row", hidden);
  cudaError_t e = mi::launch_rmsnorm(a, vec16, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_rmsnorm launch");
}

int mi_qk_norm_rope(const void* q, int64_t q_row_stride, const void* k, int64_t k_row_stride, const void* v,
                    int64_t v_row_stride, const void* q_weight, const void* k_weight, const void* cos,
                    const void* sin, int64_t cos_sin_row_stride, int64_t tokens, int hq, int hkv, int head_dim,
                    float eps, void* q_out, void* k_out, void* v_out, const int64_t* slot_mapping, void* k_pool,
                    void* v_pool, int64_t num_slots, int dtype, void* stream) {
  const int es = elem_size(dtype);
  if (es == 0) return fail(MI_ERR_INVALID, "mi_qk_norm_rope: unknown dtype %d", dtype);
  if (tokens < 0 || hq <= 0 || hkv <= 0) return fail(MI_ERR_INVALID, "mi_qk_norm_rope: bad shape");
  if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(MI_ERR_UNSUPPORTED, "mi_qk_norm_rope: head_dim %d not in {32, 64, 128, 256}", head_dim);
  if (tokens == 0) return MI_OK;
  if (!q || !k || !v || !q_weight || !k_weight || !cos || !sin || !q_out)
    return fail(MI_ERR_INVALID, "mi_qk_norm_rope: null pointer argument");
  if (slot_mapping && (!k_pool || !v_pool || num_slots <= 0))
    return fail(MI_ERR_INVALID, "mi_qk_norm_rope: an append needs both pools and num_slots > 0");
  mi::QkNormRopeArgs a{};
  a.q = static_cast<const char*>(q);
  a.q_rs = q_row_stride * es;
  a.k = static_cast<const char*>(k);
  a.k_rs = k_row_stride * es;
  a.v = static_cast<const char*>(v);
  a.v_rs = v_row_stride * es;
  a.q_w = static_cast<const char*>(q_weight);
  a.k_w = static_cast<const char*>(k_weight);
  a.cos = static_cast<const char*>(cos);
  a.sin = static_cast<const char*>(sin);
  a.cs_rs = cos_sin_row_stride * es;
  a.tokens = tokens;
  a.hq = hq;
  a.hkv = hkv;
  a.head_dim = head_dim;
  a.eps = eps;
  a.q_out = static_cast<char*>(q_out);
  a.k_out = static_cast<char*>(k_out);
  a.v_out = static_cast<char*>(v_out);
  a.slots = slot_mapping;
  a.k_pool = static_cast<char*>(k_pool);
  a.v_pool = static_cast<char*>(v_pool);
  a.num_slots = num_slots;
  // each lane moves head_dim/32 elements: 4..32 bytes, accessed as one unit when 16 bytes
  const int lane_bytes = head_dim / 32 * es;
  const int need = lane_bytes >= 16 ? 16 : lane_bytes;
  const int got = pick_vec({q, k, v, q_weight, k_weight, cos, sin, q_out, k_out ? k_out : q_out,
                            v_out ? v_out : q_out, k_pool ? k_pool : q_out, v_pool ? v_pool : q_out},
                           {a.q_rs, a.k_rs, a.v_rs, a.cs_rs, (int64_t)lane_bytes});
  if (got < need) return fail(MI_ERR_INVALID, "mi_qk_norm_rope: operands not aligned to %d bytes", need);
  cudaError_t e = mi::launch_qk_norm_rope(a, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_qk_norm_rope launch");
}

int mi_silu_mul(const void* gate, const void* up, int64_t in_row_stride, void* out, int64_t out_row_stride,
                int64_t rows, int64_t cols, int dtype, void* stream) {
  const int es = elem_size(dtype);
  if (es == 0) return fail(MI_ERR_INVALID, "mi_silu_mul: unknown dtype %d", dtype);
  if (rows < 0 || cols < 0) return fail(MI_ERR_INVALID, "mi_silu_mul: negative size");
  if (rows == 0 || cols == 0) return MI_OK;
  if (!gate || !up || !out) return fail(MI_ERR_INVALID, "mi_silu_mul: null pointer argument");
  mi::SiluMulArgs a{};
  a.gate = static_cast<const char*>(gate);
  a.up = static_cast<const char*>(up);
  a.in_rs = in_row_stride * es;
  a.out = static_cast<char*>(out);
  a.out_rs = out_row_stride * es;
  a.rows = rows;
  a.cols = cols;
  const bool vec16 = all_aligned16({gate, up, out}, {a.in_rs, a.out_rs, cols * es});
  cudaError_t e = mi::launch_silu_mul(a, vec16, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_silu_mul launch");
}
