// Decode-step metadata built on the device (mi_decode_rows).
//
// The reference packs, per decode step and on the host, one int64 row per sequence:
// [token, position, slot, context length, its block table null-padded to the longest]
// (worker/paged_runner.py:138-166), which costs O(batch x max_blocks) host work every step.  Here
// the block tables live on the device as a mirror with one row per batch slot; a step uploads only
// (batch slot, token, position) per sequence plus the table entries added since the last step
// (a sequence gains a block every block_size tokens), and two small kernels
//
//   table_delta_kernel  writes the new entries into the mirror (one thread per entry), then
//   decode_rows_kernel  writes the packed step inputs in the runner's layout
//                       ids [n] | positions [n] | slots [n] | context lens [n] | tables [n, width]:
//                       row b < batch copies its slot's mirror row (entries past its
//                       ceil((pos + 1) / bs) blocks as the null block) and computes
//                       slot = table[pos / bs] * bs + pos % bs and context = pos + 1;
//                       rows batch <= b < n are padding: token 0 at position 0 into slot 0 of the
//                       null block, context 1, a null table.
//
// Integer work only, bit-exact with the host packing.  Out-of-range slot rows, columns or
// positions set MI_STATUS_BAD_INDEX / MI_STATUS_BAD_LENGTH and are skipped (the row is written as
// padding), never a fault.
#include "common.cuh"

namespace mi {
namespace {

__global__ void table_delta_kernel(const int64_t* __restrict__ deltas, int64_t count, int64_t* __restrict__ tables,
                                   int64_t table_rows, int64_t table_stride) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const int64_t row = deltas[3 * i], col = deltas[3 * i + 1], block = deltas[3 * i + 2];
  if (row < 0 || row >= table_rows || col < 0 || col >= table_stride) {
    record_status(MI_STATUS_BAD_INDEX);
    return;
  }
  tables[row * table_stride + col] = block;
}

// grid (column chunks, n rows); one row per blockIdx.y
__global__ void decode_rows_kernel(const int64_t* __restrict__ rows, int64_t batch, const int64_t* __restrict__ tables,
                                   int64_t table_rows, int64_t table_stride, int64_t* __restrict__ out, int64_t n,
                                   int64_t width, int block_size) {
  const int64_t b = blockIdx.y;
  int64_t row = -1, token = 0, pos = 0;
  if (b < batch) {
    row = rows[3 * b];
    token = rows[3 * b + 1];
    pos = rows[3 * b + 2];
    if (row < 0 || row >= table_rows || pos < 0) {
      if (blockIdx.x == 0 && threadIdx.x == 0) record_status(MI_STATUS_BAD_INDEX);
      row = -1;
      token = 0;
      pos = 0;
    }
  }
  int64_t blocks = row >= 0 ? pos / block_size + 1 : 0;  // ceil((pos + 1) / bs)
  const int64_t cap = width < table_stride ? width : table_stride;
  if (blocks > cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_status(MI_STATUS_BAD_LENGTH);
    blocks = cap;
  }
  const int64_t* src = tables + (row >= 0 ? row : 0) * table_stride;
  int64_t* dst = out + 4 * n + b * width;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < width; c += (int64_t)gridDim.x * blockDim.x)
    dst[c] = c < blocks ? src[c] : 0;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const int64_t col = pos / block_size;
    const int64_t block = (row >= 0 && col < blocks) ? src[col] : 0;
    out[b] = token;
    out[n + b] = pos;
    out[2 * n + b] = block * block_size + pos % block_size;
    out[3 * n + b] = pos + 1;
  }
}

}  // namespace
}  // namespace mi

extern "C" {

int mi_decode_rows(const int64_t* rows, int64_t batch, const int64_t* deltas, int64_t num_deltas, int64_t* tables,
                   int64_t table_rows, int64_t table_stride, int64_t* out, int64_t n, int64_t width, int block_size,
                   void* stream) {
  if (batch < 0 || num_deltas < 0 || n < batch || width < 1 || block_size < 1 || table_rows < 1 || table_stride < 1)
    return fail(MI_ERR_INVALID,
                "mi_decode_rows: bad sizes (batch=%lld deltas=%lld n=%lld width=%lld bs=%d rows=%lld stride=%lld)",
                (long long)batch, (long long)num_deltas, (long long)n, (long long)width, block_size,
                (long long)table_rows, (long long)table_stride);
  if (n == 0) return MI_OK;
  if (!tables || !out || (batch > 0 && !rows) || (num_deltas > 0 && !deltas))
    return fail(MI_ERR_INVALID, "mi_decode_rows: null pointer argument");
  if (n > 65535) return fail(MI_ERR_UNSUPPORTED, "mi_decode_rows: %lld rows exceed 65535", (long long)n);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (num_deltas > 0) {
    const unsigned blocks = (unsigned)((num_deltas + 255) / 256);
    mi::table_delta_kernel<<<blocks, 256, 0, s>>>(deltas, num_deltas, tables, table_rows, table_stride);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "mi_decode_rows: table_delta_kernel launch");
  }
  const unsigned chunks = (unsigned)((width + 255) / 256 < 8 ? (width + 255) / 256 : 8);
  mi::decode_rows_kernel<<<dim3(chunks, (unsigned)n), 256, 0, s>>>(rows, batch, tables, table_rows, table_stride,
                                                                   out, n, width, block_size);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_decode_rows: decode_rows_kernel launch");
}

}  // extern "C"
