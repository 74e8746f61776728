// Copy kernels of the paged KV path: token scatter / decode append (K and V in one launch),
// on-device chunk store (slot arithmetic from block tables), and whole-block gather.
//
// All three are pure data movement: bit-exact, HBM-bound, vectorised by the widest unit (16, 8, 4
// or 2 bytes) that the host proved every address and stride is aligned to.  One warp moves one
// token's H_kv*D row of K and then of V (both contiguous in the pool), so stores are fully
// coalesced 16-byte transactions.
#include "common.cuh"
#include "kernels.cuh"

namespace mi {

namespace {

constexpr int kWarpsPerBlock = 4;

// Copy `units` vector units of one head row set: source rows may be strided per head.
template <typename V>
__device__ __forceinline__ void copy_token(const char* src, int64_t src_head_stride_b, char* dst, int heads,
                                           int row_units, int lane) {
  const int total = heads * row_units;
  for (int i = lane; i < total; i += 32) {
    const int h = i / row_units;
    const int u = i - h * row_units;
    const V* s = reinterpret_cast<const V*>(src + h * src_head_stride_b) + u;
    V* d = reinterpret_cast<V*>(dst + (int64_t)h * row_units * sizeof(V)) + u;
    *d = __ldg(s);
  }
}

template <typename V>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) kv_scatter_kernel(ScatterArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t token = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (token >= a.num_tokens) return;
  const int64_t slot = a.slots[token];
  if (slot < 0 || slot >= a.num_slots) {
    if (lane == 0) record_status(MI_STATUS_BAD_SLOT);
    return;
  }
  const int64_t row = a.rows ? a.rows[token] : token;
  const int64_t pos = a.positions ? a.positions[token] : 0;
  if (row < 0 || row >= a.src_rows || pos < 0 || pos >= a.src_positions) {
    if (lane == 0) record_status(MI_STATUS_BAD_INDEX);
    return;
  }
  const int row_units = a.row_bytes / (int)sizeof(V);
  const int64_t dst_off = slot * (int64_t)a.heads * a.row_bytes;
  copy_token<V>(a.k_src + row * a.k_sb[0] + pos * a.k_sb[2], a.k_sb[1], a.k_pool + dst_off, a.heads, row_units,
                lane);
  copy_token<V>(a.v_src + row * a.v_sb[0] + pos * a.v_sb[2], a.v_sb[1], a.v_pool + dst_off, a.heads, row_units,
                lane);
}

// One warp per (row, padded position); padding positions return at once.
template <typename V>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) kv_store_chunks_kernel(StoreChunksArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (item >= a.batch * a.padded_len) return;
  const int64_t row = item / a.padded_len;
  const int64_t p = item - row * a.padded_len;
  const int64_t len = a.chunk_lens[row];
  const int64_t first = a.padded_len - len;
  if (p < first) return;
  const int64_t pos = a.starts[row] + (p - first);
  const int64_t logical_block = pos / a.block_size;
  if (logical_block >= a.table_stride || pos < 0) {
    if (lane == 0) record_status(MI_STATUS_BAD_LENGTH);
    return;
  }
  const int64_t block = a.block_tables[row * a.table_stride + logical_block];
  if (block < 0 || block >= a.num_blocks) {
    if (lane == 0) record_status(MI_STATUS_BAD_BLOCK);
    return;
  }
  const int64_t slot = block * a.block_size + pos % a.block_size;
  const int row_units = a.row_bytes / (int)sizeof(V);
  const int64_t dst_off = slot * (int64_t)a.heads * a.row_bytes;
  copy_token<V>(a.k_src + row * a.k_sb[0] + p * a.k_sb[2], a.k_sb[1], a.k_pool + dst_off, a.heads, row_units, lane);
  copy_token<V>(a.v_src + row * a.v_sb[0] + p * a.v_sb[2], a.v_sb[1], a.v_pool + dst_off, a.heads, row_units, lane);
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

template <typename V>
cudaError_t launch_scatter_t(const ScatterArgs& a, cudaStream_t s) {
  const int64_t blocks = (a.num_tokens + kWarpsPerBlock - 1) / kWarpsPerBlock;
  kv_scatter_kernel<V><<<(unsigned)blocks, 32 * kWarpsPerBlock, 0, s>>>(a);
  return cudaGetLastError();
}
template <typename V>
cudaError_t launch_store_t(const StoreChunksArgs& a, cudaStream_t s) {
  const int64_t items = a.batch * a.padded_len;
  const int64_t blocks = (items + kWarpsPerBlock - 1) / kWarpsPerBlock;
  kv_store_chunks_kernel<V><<<(unsigned)blocks, 32 * kWarpsPerBlock, 0, s>>>(a);
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
