// Varlen chunked-prefill paged attention, sm_100a.
//
// Dispatch: bf16/fp16 with head_dim 128 run the tcgen05 kernel (paged_prefill_tc.cu).
// Generic kernel (every dtype, head_dim <= 256, any block size): one warp per (row, padded
// position, query head).  The query's keys are the first `start` positions of its history, read
// in place from the pools through the block table, followed causally by the chunk's own keys up
// to and including itself.  Single pass online softmax in fp32; padding positions get zeros.
#include "common.cuh"
#include "kernels.cuh"

namespace mi {
namespace {

template <typename T>
__global__ void __launch_bounds__(128) prefill_scalar_kernel(const PrefillArgs a) {
  constexpr int MAXD = 256 / 32;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= a.batch * a.padded_len * a.hq) return;
  const int hq = (int)(gw % a.hq);
  const int64_t bp = gw / a.hq;
  const int64_t p = bp % a.padded_len;
  const int64_t b = bp / a.padded_len;
  const int D = a.head_dim;
  T* dst = reinterpret_cast<T*>(a.out) + (bp * a.hq + hq) * (int64_t)D;
  int64_t len = a.chunk_lens[b];
  if (len > a.padded_len) {
    if (lane == 0) record_status(MI_STATUS_BAD_LENGTH);
    len = a.padded_len;
  }
  const int64_t first = a.padded_len - len;
  if (p < first) {
    for (int d = lane; d < D; d += 32) dst[d] = Elem<T>::from_f(0.f);
    return;
  }
  const int h = hq / a.groups;
  int64_t start = a.starts[b];
  if (start < 0) start = 0;
  if (start > a.table_stride * a.block_size) {
    if (lane == 0) record_status(MI_STATUS_BAD_LENGTH);
    start = a.table_stride * a.block_size;
  }
  const T* q = reinterpret_cast<const T*>(a.q + b * a.q_sb[0] + p * a.q_sb[1] + hq * a.q_sb[2]);
  float qv[MAXD], acc[MAXD];
#pragma unroll
  for (int i = 0; i < MAXD; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < D ? Elem<T>::to_f(q[d]) : 0.f;
    acc[i] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f;
  auto visit = [&](const T* k, const T* v) {
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < MAXD; ++i) {
      const int d = lane + 32 * i;
      if (d < D) part += qv[i] * Elem<T>::to_f(k[d]);
    }
    const float s = warp_sum(part) * a.scale_log2;
    const float m_new = fmaxf(m_run, s);
    const float alpha = exp2f(m_run - m_new);
    const float pr = exp2f(s - m_new);
    l_run = l_run * alpha + pr;
#pragma unroll
    for (int i = 0; i < MAXD; ++i) {
      const int d = lane + 32 * i;
      if (d < D) acc[i] = acc[i] * alpha + pr * Elem<T>::to_f(v[d]);
    }
    m_run = m_new;
  };
  const int64_t* table = a.block_tables + b * a.table_stride;
  const int64_t row_elems = (int64_t)a.hkv * D;
  const T* kp = reinterpret_cast<const T*>(a.k_pool);
  const T* vp = reinterpret_cast<const T*>(a.v_pool);
  for (int64_t t = 0; t < start; ++t) {
    const int64_t blk = table[t / a.block_size];
    if (blk < 0 || blk >= a.num_blocks) {
      if (lane == 0) record_status(MI_STATUS_BAD_BLOCK);
      continue;
    }
    const int64_t off = (blk * a.block_size + t % a.block_size) * row_elems + (int64_t)h * D;
    visit(kp + off, vp + off);
  }
  const char* kc = a.k_chunk + b * a.kv_sb[0] + h * a.kv_sb[2];
  const char* vc = a.v_chunk + b * a.kv_sb[0] + h * a.kv_sb[2];
  for (int64_t pp = first; pp <= p; ++pp) {
    visit(reinterpret_cast<const T*>(kc + pp * a.kv_sb[1]), reinterpret_cast<const T*>(vc + pp * a.kv_sb[1]));
  }
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
  for (int i = 0; i < MAXD; ++i) {
    const int d = lane + 32 * i;
    if (d < D) dst[d] = Elem<T>::from_f(acc[i] * inv);
  }
}

}  // namespace

cudaError_t launch_paged_prefill(const PrefillArgs& a, float* ws, const PrefillMaps* maps, int dtype,
                                 cudaStream_t s) {
  const int64_t warps = a.batch * a.padded_len * a.hq;
  if (warps == 0) return cudaSuccess;
  if (prefill_tc_supported(a, dtype)) return launch_paged_prefill_tc(a, ws, maps, dtype, s);
  const unsigned blocks = (unsigned)((warps + 3) / 4);
  switch (dtype) {
    case MI_BF16: prefill_scalar_kernel<__nv_bfloat16><<<blocks, 128, 0, s>>>(a); break;
    case MI_F16: prefill_scalar_kernel<__half><<<blocks, 128, 0, s>>>(a); break;
    default: prefill_scalar_kernel<float><<<blocks, 128, 0, s>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace mi
