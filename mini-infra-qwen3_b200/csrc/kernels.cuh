// Kernel argument blocks and launcher declarations shared by the .cu files and the C-ABI layer.
// All strides here are in BYTES (the C-ABI takes element strides and converts).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mi {

struct ScatterArgs {
  const char* k_src;
  const char* v_src;
  int64_t k_sb[3];  // row, head, position
  int64_t v_sb[3];
  const int64_t* rows;       // may be null: row = token index
  const int64_t* positions;  // may be null: position 0
  const int64_t* slots;
  int64_t num_tokens;
  int64_t src_rows;       // bounds of the source: rows and positions
  int64_t src_positions;
  char* k_pool;
  char* v_pool;
  int64_t num_slots;
  int heads;
  int row_bytes;  // head_dim * element size
};

struct StoreChunksArgs {
  const char* k_src;
  const char* v_src;
  int64_t k_sb[3];
  int64_t v_sb[3];
  int64_t batch;
  int64_t padded_len;
  const int64_t* chunk_lens;
  const int64_t* starts;
  const int64_t* block_tables;
  int64_t table_stride;
  char* k_pool;
  char* v_pool;
  int64_t num_blocks;
  int block_size;
  int heads;
  int row_bytes;
};

struct GatherArgs {
  const char* pool;
  const int64_t* block_ids;
  char* out;
  int64_t num_blocks;
  int64_t block_bytes;
};

cudaError_t launch_kv_scatter(const ScatterArgs& a, int vec_bytes, cudaStream_t s);
cudaError_t launch_kv_store_chunks(const StoreChunksArgs& a, int vec_bytes, cudaStream_t s);
cudaError_t launch_kv_gather_blocks(const GatherArgs& a, int64_t items, int vec_bytes, cudaStream_t s);

// ------------------------------------------------------------------------------------------
// Paged decode
// ------------------------------------------------------------------------------------------
constexpr int kMaxPeers = 8;  // ranks of a KV-head partition reachable by peer stores

struct DecodeArgs {
  const char* q;
  int64_t q_sb, q_sh;  // bytes
  const char* k_pool;  // used by the scalar path (the TMA path reads through tensor maps)
  const char* v_pool;
  const int64_t* block_tables;
  int64_t table_stride;
  int64_t max_blocks;  // columns of block_tables that are valid to read
  const int64_t* context_lens;
  int64_t batch;
  int64_t num_blocks;
  int hq, hkv, groups;
  int head_dim;
  int block_size;
  float scale_log2;  // softmax scale * log2(e)
  int split_pages;   // pages handled by one split
  int max_splits;    // grid.x of the split kernel
  int parts_per_split;
  int max_parts;     // max_splits * parts_per_split
  float* ws_o;       // [batch, hq, max_parts, head_dim]
  float* ws_ml;      // [batch, hq, max_parts, 2]
  char* out;
  int64_t out_sb;    // bytes
  // Exchange of the output rows over a KV-head partition (mi_paged_decode_exchange): with
  // world > 0 the combine writes row b of local query head j to every rank's gathered buffer,
  // gathered[p] + b * gathered_sb + ((rank * hq + j) * head_dim) elements, instead of to `out`.
  int world;
  int rank;
  int64_t gathered_sb;  // bytes
  char* gathered[kMaxPeers];
};

// The barrier that follows an exchange: rank r stores epoch e into flags[p][r] of every peer p
// (release, system scope), then waits (acquire, bounded by timeout_ns) until flags[r][p] >= e for
// every peer; e = *epoch + 1, written back to *epoch.
struct PeerBarrierArgs {
  unsigned int* flags[kMaxPeers];
  unsigned int* epoch;
  int rank;
  int world;
  uint64_t timeout_ns;
};
cudaError_t launch_peer_barrier(const PeerBarrierArgs& a, cudaStream_t s);

struct DecodePlan {
  bool use_mma;
  int heads_per_cta;  // HB
  int parts_per_split;
  int split_pages;
  int max_splits;
  size_t ws_bytes;
};

DecodePlan plan_decode(int64_t batch, int hq, int hkv, int head_dim, int64_t max_blocks, int block_size, int dtype);

// Launches the split kernel and the combine kernel (or the scalar single-pass kernel).
cudaError_t launch_paged_decode(const DecodeArgs& a, const DecodePlan& plan, const CUtensorMap* tm_k,
                                const CUtensorMap* tm_v, int dtype, cudaStream_t s);

// ------------------------------------------------------------------------------------------
// Paged chunked prefill
// ------------------------------------------------------------------------------------------
struct PrefillArgs {
  const char* q;
  int64_t q_sb[3];  // row, position, head (bytes)
  const char* k_chunk;
  const char* v_chunk;
  int64_t kv_sb[3];
  const char* k_pool;
  const char* v_pool;
  int64_t num_blocks;
  const int64_t* block_tables;
  int64_t table_stride;
  const int64_t* starts;
  const int64_t* chunk_lens;
  int64_t batch;
  int64_t padded_len;
  int hq, hkv, groups;
  int head_dim;
  int block_size;
  float scale_log2;
  char* out;  // [batch, padded_len, hq*head_dim] contiguous
};

// TMA descriptors of the prefill operands (Q box [64, G, 128/G, 1]; chunk K/V boxes [64, 1, 64, 1];
// pool boxes [64, 1, block_size]).  With maps == nullptr the kernel stages K/V with cp.async.
struct PrefillMaps {
  CUtensorMap q, k_chunk, v_chunk, k_pool, v_pool;
};
cudaError_t launch_paged_prefill(const PrefillArgs& a, float* ws, const PrefillMaps* maps, int dtype,
                                 cudaStream_t s);
// tcgen05 variant (bf16/fp16, head_dim 128, G in {1,2,4,8}, 16-byte aligned operands); its split-KV
// partials need prefill_tc_workspace_bytes(a) bytes of workspace (0 when no row tile splits)
bool prefill_tc_supported(const PrefillArgs& a, int dtype);
size_t prefill_tc_workspace_bytes(const PrefillArgs& a);
bool prefill_tc_tma_block_size(int block_size);
cudaError_t launch_paged_prefill_tc(const PrefillArgs& a, float* ws, const PrefillMaps* maps, int dtype,
                                    cudaStream_t s);

// Model-side fused row operations around the attention (layer_ops.cu).
struct RmsNormArgs {
  const char* x;  // [rows, hidden] rows at x + row * x_rs (bytes)
  int64_t x_rs;
  const char* res;  // optional residual added first (same shape), or null
  int64_t res_rs;
  char* res_out;  // optional: receives x + res (may alias res)
  int64_t res_out_rs;
  const char* w;  // [hidden]
  char* out;
  int64_t out_rs;
  int64_t rows;
  int hidden;
  float eps;
  float inv_hidden;
};
cudaError_t launch_rmsnorm(const RmsNormArgs& a, bool vec16, int dtype, cudaStream_t s);

struct QkNormRopeArgs {
  const char* q;  // token t, head h at q + t * q_rs (bytes) + h * head_dim elements
  int64_t q_rs;
  const char* k;
  int64_t k_rs;
  const char* v;
  int64_t v_rs;
  const char* q_w;  // [head_dim] q_norm / k_norm weights
  const char* k_w;
  const char* cos;  // [tokens, head_dim] rows at cos + t * cs_rs
  const char* sin;
  int64_t cs_rs;
  int64_t tokens;
  int hq, hkv, head_dim;
  float eps;
  char* q_out;  // [tokens, hq, head_dim]
  char* k_out;  // optional [tokens, hkv, head_dim]
  char* v_out;  // optional [tokens, hkv, head_dim]
  const int64_t* slots;  // optional: append K/V to the pools at these slots
  char* k_pool;
  char* v_pool;
  int64_t num_slots;
};
cudaError_t launch_qk_norm_rope(const QkNormRopeArgs& a, int dtype, cudaStream_t s);

struct SiluMulArgs {
  const char* gate;  // [rows, cols] at gate + row * in_rs (bytes); up likewise
  const char* up;
  int64_t in_rs;
  char* out;
  int64_t out_rs;
  int64_t rows, cols;
};
cudaError_t launch_silu_mul(const SiluMulArgs& a, bool vec16, int dtype, cudaStream_t s);

}  // namespace mi
