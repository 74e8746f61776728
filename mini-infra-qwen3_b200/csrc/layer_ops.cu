// Fused elementwise operations on either side of the paged attention, sm_100a.
//
// All three are HBM-bound row operations; each replaces a chain of PyTorch element-wise launches
// of the model (model/qwen3.py of the reference) and keeps that chain's rounding points, so a
// 16-bit model rounds exactly where the reference does:
//
// * rmsnorm_kernel — optional residual add h = T(x + r) (written back as the new residual), then
//   RMSNorm with fp32 statistics: n = T(h * rsqrt(mean(h^2) + eps)), out = T(w * n)
//   (reference model/qwen3.py:67-78 and the residual adds of the decoder layer);
// * qk_norm_rope_kernel — per (token, head): the same RMSNorm over head_dim with the q_norm /
//   k_norm weight, then rotate-half RoPE with cos/sin already in the model dtype:
//   out = T(T(y * cos) + T(rot(y) * sin)), rot(y)_i = -y_{i+D/2} (i < D/2), y_{i-D/2} otherwise
//   (reference :112-144, :182-217).  K heads also carry V: both go to contiguous [T, H, D]
//   outputs and/or straight into the pools at slot_mapping (the decode append);
// * silu_mul_kernel — out = T(T(silu(g)) * u), silu(g) = g / (1 + exp(-g)) in fp32 (the MLP).
//
// The mean is a sum times 1/n; the sum's order differs from PyTorch's reduction, which changes
// the fp32 statistic by at most a few ulp.
#include "common.cuh"
#include "kernels.cuh"

namespace mi {
namespace {

template <typename T>
__device__ __forceinline__ float round_t(float x) {
  return Elem<T>::to_f(Elem<T>::from_f(x));
}

// V consecutive elements <-> floats; 16-byte accesses when V * sizeof(T) == 16.
template <typename T, int V>
__device__ __forceinline__ void load_vec(const T* p, float (&f)[V]) {
  if constexpr (V * sizeof(T) == 16) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < V; ++i) f[i] = Elem<T>::to_f(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) f[i] = Elem<T>::to_f(p[i]);
  }
}
template <typename T, int V>
__device__ __forceinline__ void store_vec(T* p, const float (&f)[V]) {
  if constexpr (V * sizeof(T) == 16) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < V; ++i) e[i] = Elem<T>::from_f(f[i]);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = Elem<T>::from_f(f[i]);
  }
}

constexpr int kNormThreads = 128;

// One CTA per row; thread t owns vectors t, t + 128, ... (at most MAXV of V elements).
template <typename T, int V, int MAXV>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const RmsNormArgs a) {
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const T* x = reinterpret_cast<const T*>(a.x + row * a.x_rs);
  const T* r = a.res ? reinterpret_cast<const T*>(a.res + row * a.res_rs) : nullptr;
  T* r_out = a.res_out ? reinterpret_cast<T*>(a.res_out + row * a.res_out_rs) : nullptr;
  float h[MAXV][V];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int j = (tid + k * kNormThreads) * V;
    if (j < a.hidden) {
      load_vec<T, V>(x + j, h[k]);
      if (r) {
        float rv[V];
        load_vec<T, V>(r + j, rv);
#pragma unroll
        for (int i = 0; i < V; ++i) h[k][i] = round_t<T>(h[k][i] + rv[i]);
        if (r_out) store_vec<T, V>(r_out + j, h[k]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) ss = fmaf(h[k][i], h[k][i], ss);
    }
  }
  ss = warp_sum(ss);
  __shared__ float part[kNormThreads / 32];
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) total += part[w];
  const float inv = rsqrtf(total * a.inv_hidden + a.eps);
  const T* w = reinterpret_cast<const T*>(a.w);
  T* out = reinterpret_cast<T*>(a.out + row * a.out_rs);
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int j = (tid + k * kNormThreads) * V;
    if (j < a.hidden) {
      float wv[V], o[V];
      load_vec<T, V>(w + j, wv);
#pragma unroll
      for (int i = 0; i < V; ++i) o[i] = wv[i] * round_t<T>(h[k][i] * inv);
      store_vec<T, V>(out + j, o);
    }
  }
}

// One warp per (token, head); lane l owns elements [l*EPL, l*EPL + EPL) of head_dim = 32*EPL, so
// the rotate-half partner of lane l is lane l ^ 16.
template <typename T, int EPL>
__global__ void __launch_bounds__(128) qk_norm_rope_kernel(const QkNormRopeArgs a) {
  const int64_t wid = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + a.hkv;
  if (wid >= a.tokens * heads) return;  // uniform per warp
  const int64_t t = wid / heads;
  const int hd = (int)(wid - t * heads);
  const bool is_q = hd < a.hq;
  const int kh = hd - a.hq;
  constexpr int D = 32 * EPL;
  const int e0 = lane * EPL;
  const T* src = is_q ? reinterpret_cast<const T*>(a.q + t * a.q_rs) + (int64_t)hd * D
                      : reinterpret_cast<const T*>(a.k + t * a.k_rs) + (int64_t)kh * D;
  float x[EPL];
  load_vec<T, EPL>(src + e0, x);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss * (1.0f / D) + a.eps);
  float wv[EPL], c[EPL], s[EPL], y[EPL], o[EPL];
  load_vec<T, EPL>(reinterpret_cast<const T*>(is_q ? a.q_w : a.k_w) + e0, wv);
  load_vec<T, EPL>(reinterpret_cast<const T*>(a.cos + t * a.cs_rs) + e0, c);
  load_vec<T, EPL>(reinterpret_cast<const T*>(a.sin + t * a.cs_rs) + e0, s);
#pragma unroll
  for (int i = 0; i < EPL; ++i) y[i] = round_t<T>(wv[i] * round_t<T>(x[i] * inv));
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const float p = __shfl_xor_sync(0xffffffffu, y[i], 16);
    const float rot = lane < 16 ? -p : p;
    o[i] = round_t<T>(y[i] * c[i]) + round_t<T>(rot * s[i]);
  }
  if (is_q) {
    store_vec<T, EPL>(reinterpret_cast<T*>(a.q_out) + (t * a.hq + hd) * D + e0, o);
    return;
  }
  float v[EPL];
  load_vec<T, EPL>(reinterpret_cast<const T*>(a.v + t * a.v_rs) + (int64_t)kh * D + e0, v);
  if (a.k_out) store_vec<T, EPL>(reinterpret_cast<T*>(a.k_out) + (t * a.hkv + kh) * D + e0, o);
  if (a.v_out) store_vec<T, EPL>(reinterpret_cast<T*>(a.v_out) + (t * a.hkv + kh) * D + e0, v);
  if (a.slots) {
    const int64_t slot = a.slots[t];
    if (slot < 0 || slot >= a.num_slots) {
      if (lane == 0) record_status(MI_STATUS_BAD_SLOT);
      return;
    }
    const int64_t off = (slot * a.hkv + kh) * D + e0;
    store_vec<T, EPL>(reinterpret_cast<T*>(a.k_pool) + off, o);
    store_vec<T, EPL>(reinterpret_cast<T*>(a.v_pool) + off, v);
  }
}

// Grid-stride over vectors of V columns of a [rows, cols] output.
template <typename T, int V>
__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluMulArgs a) {
  const int64_t vec_per_row = a.cols / V;
  const int64_t total = a.rows * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / vec_per_row;
    const int64_t col = (i - row * vec_per_row) * V;
    float g[V], u[V], o[V];
    load_vec<T, V>(reinterpret_cast<const T*>(a.gate + row * a.in_rs) + col, g);
    load_vec<T, V>(reinterpret_cast<const T*>(a.up + row * a.in_rs) + col, u);
#pragma unroll
    for (int j = 0; j < V; ++j) o[j] = round_t<T>(g[j] / (1.0f + expf(-g[j]))) * u[j];
    store_vec<T, V>(reinterpret_cast<T*>(a.out + row * a.out_rs) + col, o);
  }
}

template <typename T, int V>
cudaError_t launch_rmsnorm_v(const RmsNormArgs& a, cudaStream_t s) {
  const int vecs = (a.hidden + V - 1) / V;
  const int per_thread = (vecs + kNormThreads - 1) / kNormThreads;
  const dim3 grid((unsigned)a.rows);
  if (per_thread <= 1) rmsnorm_kernel<T, V, 1><<<grid, kNormThreads, 0, s>>>(a);
  else if (per_thread <= 2) rmsnorm_kernel<T, V, 2><<<grid, kNormThreads, 0, s>>>(a);
  else if (per_thread <= 4) rmsnorm_kernel<T, V, 4><<<grid, kNormThreads, 0, s>>>(a);
  else if (per_thread <= 8) rmsnorm_kernel<T, V, 8><<<grid, kNormThreads, 0, s>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_rmsnorm_t(const RmsNormArgs& a, bool vec16, cudaStream_t s) {
  if (vec16) return launch_rmsnorm_v<T, 16 / sizeof(T)>(a, s);
  return launch_rmsnorm_v<T, 1>(a, s);
}

template <typename T>
cudaError_t launch_qk_norm_rope_t(const QkNormRopeArgs& a, cudaStream_t s) {
  const int64_t warps = a.tokens * (a.hq + a.hkv);
  const dim3 grid((unsigned)((warps + 3) / 4));
  switch (a.head_dim) {
    case 32: qk_norm_rope_kernel<T, 1><<<grid, 128, 0, s>>>(a); break;
    case 64: qk_norm_rope_kernel<T, 2><<<grid, 128, 0, s>>>(a); break;
    case 128: qk_norm_rope_kernel<T, 4><<<grid, 128, 0, s>>>(a); break;
    case 256: qk_norm_rope_kernel<T, 8><<<grid, 128, 0, s>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_silu_mul_t(const SiluMulArgs& a, bool vec16, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const int v = vec16 ? V : 1;
  const int64_t total = a.rows * (a.cols / v);
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
  if (vec16) silu_mul_kernel<T, V><<<blocks, 256, 0, s>>>(a);
  else silu_mul_kernel<T, 1><<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rmsnorm(const RmsNormArgs& a, bool vec16, int dtype, cudaStream_t s) {
  if (a.rows == 0) return cudaSuccess;
  if (dtype == MI_BF16) return launch_rmsnorm_t<__nv_bfloat16>(a, vec16, s);
  if (dtype == MI_F16) return launch_rmsnorm_t<__half>(a, vec16, s);
  return launch_rmsnorm_t<float>(a, vec16, s);
}

cudaError_t launch_qk_norm_rope(const QkNormRopeArgs& a, int dtype, cudaStream_t s) {
  if (a.tokens == 0) return cudaSuccess;
  if (dtype == MI_BF16) return launch_qk_norm_rope_t<__nv_bfloat16>(a, s);
  if (dtype == MI_F16) return launch_qk_norm_rope_t<__half>(a, s);
  return launch_qk_norm_rope_t<float>(a, s);
}

cudaError_t launch_silu_mul(const SiluMulArgs& a, bool vec16, int dtype, cudaStream_t s) {
  if (a.rows == 0 || a.cols == 0) return cudaSuccess;
  if (dtype == MI_BF16) return launch_silu_mul_t<__nv_bfloat16>(a, vec16, s);
  if (dtype == MI_F16) return launch_silu_mul_t<__half>(a, vec16, s);
  return launch_silu_mul_t<float>(a, vec16, s);
}

}  // namespace mi
