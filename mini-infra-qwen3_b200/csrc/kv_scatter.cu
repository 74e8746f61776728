// Copy kernels of the paged KV path: token scatter / decode append (K and V in one launch),
// on-device chunk store (slot arithmetic from block tables), and whole-block gather.
//
// All three are pure data movement: bit-exact, HBM-bound, vectorised by the widest unit (16, 8, 4
// or 2 bytes) that the host proved every address and stride is aligned to.  The scatter and the
// chunk store are flat over (token, vector unit of the token's H_kv*D row): each thread loads its
// unit of K and of V, then stores both, so every thread has its two loads in flight at once and a
// warp's stores are consecutive units of one pool row (coalesced).  A token's row is contiguous in
// the pool; its source rows may be strided per head.
#include "common.cuh"
#include "kernels.cuh"

namespace mi {

namespace {

constexpr int kCopyThreads = 256;
constexpr int64_t kMaxCopyBlocks = 148 * 16;  // grid-stride beyond this

// Unit u of a token's row (head h = u / row_units) at the source / in the pool.
template <typename V>
__device__ __forceinline__ void copy_unit_kv(const char* k_src, const char* v_src, int64_t k_hstride,
                                             int64_t v_hstride, char* k_dst, char* v_dst, int u, int row_units) {
  const int h = u / row_units;
  const int w = u - h * row_units;
  const V kv = __ldg(reinterpret_cast<const V*>(k_src + h * k_hstride) + w);
  const V vv = __ldg(reinterpret_cast<const V*>(v_src + h * v_hstride) + w);
  reinterpret_cast<V*>(k_dst)[u] = kv;
  reinterpret_cast<V*>(v_dst)[u] = vv;
}

template <typename V>
__global__ void __launch_bounds__(kCopyThreads) kv_scatter_kernel(ScatterArgs a) {
  const int row_units = a.row_bytes / (int)sizeof(V);
  const int units = a.heads * row_units;  // per token (of K, and of V)
  const int64_t total = a.num_tokens * units;
  for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < total; i += (int64_t)gridDim.x * kCopyThreads) {
    const int64_t token = i / units;
    const int u = (int)(i - token * units);
    const int64_t slot = a.slots[token];
    if (slot < 0 || slot >= a.num_slots) {
      if (u == 0) record_status(MI_STATUS_BAD_SLOT);
      continue;
    }
    const int64_t row = a.rows ? a.rows[token] : token;
    const int64_t pos = a.positions ? a.positions[token] : 0;
    if (row < 0 || row >= a.src_rows || pos < 0 || pos >= a.src_positions) {
      if (u == 0) record_status(MI_STATUS_BAD_INDEX);
      continue;
    }
    const int64_t dst_off = slot * (int64_t)a.heads * a.row_bytes;
    copy_unit_kv<V>(a.k_src + row * a.k_sb[0] + pos * a.k_sb[2], a.v_src + row * a.v_sb[0] + pos * a.v_sb[2],
                    a.k_sb[1], a.v_sb[1], a.k_pool + dst_off, a.v_pool + dst_off, u, row_units);
  }
}

// Flat over (row, padded position, unit); padding positions are skipped.
template <typename V>
__global__ void __launch_bounds__(kCopyThreads) kv_store_chunks_kernel(StoreChunksArgs a) {
  const int row_units = a.row_bytes / (int)sizeof(V);
  const int units = a.heads * row_units;
  const int64_t total = a.batch * a.padded_len * units;
  for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < total; i += (int64_t)gridDim.x * kCopyThreads) {
    const int64_t item = i / units;  // row * padded_len + p
    const int u = (int)(i - item * units);
    const int64_t row = item / a.padded_len;
    const int64_t p = item - row * a.padded_len;
    const int64_t len = a.chunk_lens[row];
    const int64_t first = a.padded_len - len;
    if (p < first) continue;
    const int64_t pos = a.starts[row] + (p - first);
    const int64_t logical_block = pos / a.block_size;
    if (logical_block >= a.table_stride || pos < 0) {
      if (u == 0) record_status(MI_STATUS_BAD_LENGTH);
      continue;
    }
    const int64_t block = a.block_tables[row * a.table_stride + logical_block];
    if (block < 0 || block >= a.num_blocks) {
      if (u == 0) record_status(MI_STATUS_BAD_BLOCK);
      continue;
    }
    const int64_t slot = block * a.block_size + pos % a.block_size;
    const int64_t dst_off = slot * (int64_t)a.heads * a.row_bytes;
    copy_unit_kv<V>(a.k_src + row * a.k_sb[0] + p * a.k_sb[2], a.v_src + row * a.v_sb[0] + p * a.v_sb[2], a.k_sb[1],
                    a.v_sb[1], a.k_pool + dst_off, a.v_pool + dst_off, u, row_units);
  }
}

// One CTA (128 threads) per gathered block: bs*H*D contiguous elements.
template <typename V>
__global__ void __launch_bounds__(128) kv_gather_blocks_kernel(GatherArgs a) {
  const int64_t item = blockIdx.x;  // b * blocks_per_row + j
  const int64_t block = a.block_ids[item];
  const int units = (int)(a.block_bytes / sizeof(V));
  V* dst = reinterpret_cast<V*>(a.out + item * a.block_bytes);
  if (block < 0 || block >= a.num_blocks) {
    if (threadIdx.x == 0) record_status(MI_STATUS_BAD_BLOCK);
    for (int i = threadIdx.x; i < units; i += blockDim.x) dst[i] = V{};
    return;
  }
  const V* src = reinterpret_cast<const V*>(a.pool + block * a.block_bytes);
  for (int i = threadIdx.x; i < units; i += blockDim.x) dst[i] = __ldg(src + i);
}

int64_t copy_blocks(int64_t threads) {
  const int64_t b = (threads + kCopyThreads - 1) / kCopyThreads;
  return b < kMaxCopyBlocks ? b : kMaxCopyBlocks;
}
template <typename V>
cudaError_t launch_scatter_t(const ScatterArgs& a, cudaStream_t s) {
  const int64_t units = (int64_t)a.heads * (a.row_bytes / (int)sizeof(V));
  kv_scatter_kernel<V><<<(unsigned)copy_blocks(a.num_tokens * units), kCopyThreads, 0, s>>>(a);
  return cudaGetLastError();
}
template <typename V>
cudaError_t launch_store_t(const StoreChunksArgs& a, cudaStream_t s) {
  const int64_t units = (int64_t)a.heads * (a.row_bytes / (int)sizeof(V));
  kv_store_chunks_kernel<V><<<(unsigned)copy_blocks(a.batch * a.padded_len * units), kCopyThreads, 0, s>>>(a);
  return cudaGetLastError();
}
template <typename V>
cudaError_t launch_gather_t(const GatherArgs& a, int64_t items, cudaStream_t s) {
  kv_gather_blocks_kernel<V><<<(unsigned)items, 128, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_kv_scatter(const ScatterArgs& a, int vec_bytes, cudaStream_t s) {
  if (a.num_tokens == 0) return cudaSuccess;
  switch (vec_bytes) {
    case 16: return launch_scatter_t<uint4>(a, s);
    case 8: return launch_scatter_t<uint2>(a, s);
    case 4: return launch_scatter_t<uint32_t>(a, s);
    default: return launch_scatter_t<uint16_t>(a, s);
  }
}

cudaError_t launch_kv_store_chunks(const StoreChunksArgs& a, int vec_bytes, cudaStream_t s) {
  if (a.batch == 0 || a.padded_len == 0) return cudaSuccess;
  switch (vec_bytes) {
    case 16: return launch_store_t<uint4>(a, s);
    case 8: return launch_store_t<uint2>(a, s);
    case 4: return launch_store_t<uint32_t>(a, s);
    default: return launch_store_t<uint16_t>(a, s);
  }
}

cudaError_t launch_kv_gather_blocks(const GatherArgs& a, int64_t items, int vec_bytes, cudaStream_t s) {
  if (items == 0) return cudaSuccess;
  switch (vec_bytes) {
    case 16: return launch_gather_t<uint4>(a, items, s);
    case 8: return launch_gather_t<uint2>(a, items, s);
    case 4: return launch_gather_t<uint32_t>(a, items, s);
    default: return launch_gather_t<uint16_t>(a, items, s);
  }
}

}  // namespace mi
