// C-ABI entry points (include/mi_paged.h): host-side argument checks, kernel-variant selection,
// TMA descriptor encoding (cached per pool), launches on the caller's stream.  No allocation, no
// synchronisation (except mi_read_status, whose job is to synchronise).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "kernels.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MI_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int elem_size(int dtype) { return dtype == MI_F32 ? 4 : (dtype == MI_BF16 || dtype == MI_F16) ? 2 : 0; }

bool aligned(const void* p, int64_t bytes) { return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)bytes) == 0; }

// Widest copy unit (16/8/4/2 bytes) dividing every pointer, byte stride and the row size.
int pick_vec(std::initializer_list<const void*> ptrs, std::initializer_list<int64_t> byte_values) {
  for (int v : {16, 8, 4, 2}) {
    bool ok = true;
    for (const void* p : ptrs) ok = ok && aligned(p, v);
    for (int64_t x : byte_values) ok = ok && (x % v == 0);
    if (ok) return v;
  }
  return 1;
}

// ------------------------------------------------------------------------------------------
// TMA tensor maps over a pool viewed as [D (inner), H_kv, num_blocks*bs] with [64, 1, bs] boxes.
// ------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  int64_t slots;
  int hkv, d, bs, dtype;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && slots == o.slots && hkv == o.hkv && d == o.d && bs == o.bs && dtype == o.dtype;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.ptr);
    h ^= std::hash<int64_t>()(k.slots) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= (size_t)(k.hkv * 131 + k.d * 7 + k.bs * 1009 + k.dtype);
    return h;
  }
};

std::mutex g_map_mutex;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

int pool_tensor_map(const void* pool, int64_t num_blocks, int bs, int hkv, int d, int dtype, CUtensorMap* out) {
  const MapKey key{pool, num_blocks * bs, hkv, d, bs, dtype};
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return MI_OK;
    }
  }
  auto fn = encode_fn();
  if (!fn) return fail(MI_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int es = elem_size(dtype);
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)hkv, (cuuint64_t)(num_blocks * bs)};
  cuuint64_t strides[2] = {(cuuint64_t)d * es, (cuuint64_t)hkv * d * es};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)bs};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType ty =
      dtype == MI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap m;
  CUresult r = fn(&m, ty, 3, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MI_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps[key] = m;
  }
  *out = m;
  return MI_OK;
}

// Tiled, 128-byte-swizzled tensor map of a 16-bit tensor (cached by every encoding argument).
std::unordered_map<std::string, CUtensorMap> g_generic_maps;

bool encode_map(const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                int dtype, CUtensorMap* out) {
  std::string key(reinterpret_cast<const char*>(&base), sizeof(base));
  key.append(reinterpret_cast<const char*>(&rank), sizeof(rank));
  key.append(reinterpret_cast<const char*>(dims), sizeof(cuuint64_t) * rank);
  key.append(reinterpret_cast<const char*>(strides), sizeof(cuuint64_t) * (rank - 1));
  key.append(reinterpret_cast<const char*>(box), sizeof(cuuint32_t) * rank);
  key.append(reinterpret_cast<const char*>(&dtype), sizeof(dtype));
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    auto it = g_generic_maps.find(key);
    if (it != g_generic_maps.end()) {
      *out = it->second;
      return true;
    }
  }
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType ty =
      dtype == MI_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap m;
  if (fn(&m, ty, rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return false;
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    if (g_generic_maps.size() > 4096) g_generic_maps.clear();
    g_generic_maps[key] = m;
  }
  *out = m;
  return true;
}

int check_pool_geometry(int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype) {
  if (elem_size(dtype) == 0) return fail(MI_ERR_INVALID, "unknown dtype %d", dtype);
  if (num_blocks < 1 || block_size < 1 || num_kv_heads < 1 || head_dim < 1)
    return fail(MI_ERR_INVALID, "pool geometry must be positive (blocks=%lld bs=%d heads=%d dim=%d)",
                (long long)num_blocks, block_size, num_kv_heads, head_dim);
  return MI_OK;
}

}  // namespace

extern "C" {

int mi_version(void) { return 100; }

const char* mi_last_error(void) { return g_last_error.c_str(); }

int mi_read_status(unsigned int* status_out, int clear, void* stream) {
  if (!status_out) return fail(MI_ERR_INVALID, "status_out is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, mi::g_status, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "mi_read_status");
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(mi::g_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "mi_read_status(clear)");
  }
  *status_out = v;
  return MI_OK;
}

int mi_kv_scatter(const void* k_src, const void* v_src, const int64_t* k_strides, const int64_t* v_strides,
                  int64_t src_rows, int64_t src_positions, const int64_t* token_rows,
                  const int64_t* token_positions, const int64_t* slot_mapping, int64_t num_tokens, void* k_pool,
                  void* v_pool, int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype,
                  void* stream) {
  if (int rc = check_pool_geometry(num_blocks, block_size, num_kv_heads, head_dim, dtype)) return rc;
  if (num_tokens < 0) return fail(MI_ERR_INVALID, "num_tokens < 0");
  if (num_tokens == 0) return MI_OK;
  if (!k_src || !v_src || !k_strides || !v_strides || !slot_mapping || !k_pool || !v_pool)
    return fail(MI_ERR_INVALID, "mi_kv_scatter: null pointer argument");
  const int es = elem_size(dtype);
  mi::ScatterArgs a{};
  a.k_src = static_cast<const char*>(k_src);
  a.v_src = static_cast<const char*>(v_src);
  for (int i = 0; i < 3; ++i) {
    a.k_sb[i] = k_strides[i] * es;
    a.v_sb[i] = v_strides[i] * es;
  }
  a.rows = token_rows;
  a.positions = token_positions;
  a.slots = slot_mapping;
  a.num_tokens = num_tokens;
  a.src_rows = src_rows;
  a.src_positions = src_positions;
  a.k_pool = static_cast<char*>(k_pool);
  a.v_pool = static_cast<char*>(v_pool);
  a.num_slots = num_blocks * block_size;
  a.heads = num_kv_heads;
  a.row_bytes = head_dim * es;
  const int vec = pick_vec({k_src, v_src, k_pool, v_pool},
                           {a.k_sb[0], a.k_sb[1], a.k_sb[2], a.v_sb[0], a.v_sb[1], a.v_sb[2], (int64_t)a.row_bytes});
  if (vec < 2) return fail(MI_ERR_INVALID, "mi_kv_scatter: misaligned operands");
  cudaError_t e = mi::launch_kv_scatter(a, vec, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_kv_scatter launch");
}

int mi_kv_store_chunks(const void* k_src, const void* v_src, const int64_t* k_strides, const int64_t* v_strides,
                       int64_t batch, int64_t padded_len, const int64_t* chunk_lens, const int64_t* start_positions,
                       const int64_t* block_tables, int64_t table_stride, void* k_pool, void* v_pool,
                       int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype, void* stream) {
  if (int rc = check_pool_geometry(num_blocks, block_size, num_kv_heads, head_dim, dtype)) return rc;
  if (batch < 0 || padded_len < 0 || table_stride < 0) return fail(MI_ERR_INVALID, "negative size");
  if (batch == 0 || padded_len == 0) return MI_OK;
  if (!k_src || !v_src || !k_strides || !v_strides || !chunk_lens || !start_positions || !block_tables || !k_pool ||
      !v_pool)
    return fail(MI_ERR_INVALID, "mi_kv_store_chunks: null pointer argument");
  const int es = elem_size(dtype);
  mi::StoreChunksArgs a{};
  a.k_src = static_cast<const char*>(k_src);
  a.v_src = static_cast<const char*>(v_src);
  for (int i = 0; i < 3; ++i) {
    a.k_sb[i] = k_strides[i] * es;
    a.v_sb[i] = v_strides[i] * es;
  }
  a.batch = batch;
  a.padded_len = padded_len;
  a.chunk_lens = chunk_lens;
  a.starts = start_positions;
  a.block_tables = block_tables;
  a.table_stride = table_stride;
  a.k_pool = static_cast<char*>(k_pool);
  a.v_pool = static_cast<char*>(v_pool);
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.heads = num_kv_heads;
  a.row_bytes = head_dim * es;
  const int vec = pick_vec({k_src, v_src, k_pool, v_pool},
                           {a.k_sb[0], a.k_sb[1], a.k_sb[2], a.v_sb[0], a.v_sb[1], a.v_sb[2], (int64_t)a.row_bytes});
  if (vec < 2) return fail(MI_ERR_INVALID, "mi_kv_store_chunks: misaligned operands");
  cudaError_t e = mi::launch_kv_store_chunks(a, vec, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_kv_store_chunks launch");
}

int mi_kv_gather_blocks(const void* pool, const int64_t* block_ids, int64_t batch, int64_t blocks_per_row,
                        void* out, int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype,
                        void* stream) {
  if (int rc = check_pool_geometry(num_blocks, block_size, num_kv_heads, head_dim, dtype)) return rc;
  if (batch < 0 || blocks_per_row < 0) return fail(MI_ERR_INVALID, "negative size");
  if (batch * blocks_per_row == 0) return MI_OK;
  if (!pool || !block_ids || !out) return fail(MI_ERR_INVALID, "mi_kv_gather_blocks: null pointer argument");
  mi::GatherArgs a{};
  a.pool = static_cast<const char*>(pool);
  a.block_ids = block_ids;
  a.out = static_cast<char*>(out);
  a.num_blocks = num_blocks;
  a.block_bytes = (int64_t)block_size * num_kv_heads * head_dim * elem_size(dtype);
  const int vec = pick_vec({pool, out}, {a.block_bytes});
  cudaError_t e = mi::launch_kv_gather_blocks(a, batch * blocks_per_row, vec, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_kv_gather_blocks launch");
}

size_t mi_paged_decode_workspace_size(int64_t batch, int num_q_heads, int num_kv_heads, int head_dim,
                                      int64_t max_blocks_per_seq, int block_size, int dtype) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads <= 0) return 0;
  return mi::plan_decode(batch, num_q_heads, num_kv_heads, head_dim, max_blocks_per_seq, block_size, dtype).ws_bytes;
}

}  // extern "C"

namespace {

// Where the decode output goes: `out` (world == 0), or every rank's gathered buffer followed by the
// peer barrier (mi_paged_decode_exchange).
struct DecodeExchange {
  int world = 0;
  int rank = 0;
  int64_t gathered_sb = 0;  // bytes
  char* gathered[mi::kMaxPeers] = {};
  mi::PeerBarrierArgs barrier{};
};

int paged_decode_impl(const void* q, const int64_t* q_strides, const void* k_new, const void* v_new,
                      const int64_t* new_strides, const int64_t* slot_mapping, void* k_pool, void* v_pool,
                      int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                      const int64_t* block_tables, int64_t table_stride, int64_t max_blocks_per_seq,
                      const int64_t* context_lens, int64_t batch, int num_q_heads, float scale, void* out,
                      int64_t out_stride, void* workspace, size_t workspace_bytes, int dtype, void* stream,
                      const DecodeExchange& ex) {
  if (int rc = check_pool_geometry(num_blocks, block_size, num_kv_heads, head_dim, dtype)) return rc;
  if (batch < 0) return fail(MI_ERR_INVALID, "batch < 0");
  if (batch == 0) return MI_OK;
  if (batch > 65535) return fail(MI_ERR_UNSUPPORTED, "batch %lld exceeds 65535", (long long)batch);
  if (num_q_heads < 1 || num_q_heads % num_kv_heads != 0)
    return fail(MI_ERR_INVALID, "num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)", num_q_heads,
                num_kv_heads);
  if (head_dim > 256) return fail(MI_ERR_UNSUPPORTED, "head_dim %d > 256", head_dim);
  if (!q || !q_strides || !k_pool || !v_pool || !block_tables || !context_lens || (!out && ex.world == 0))
    return fail(MI_ERR_INVALID, "mi_paged_decode: null pointer argument");
  if (max_blocks_per_seq < 1 || table_stride < max_blocks_per_seq)
    return fail(MI_ERR_INVALID, "block table needs at least one column (max_blocks=%lld, stride=%lld)",
                (long long)max_blocks_per_seq, (long long)table_stride);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = elem_size(dtype);
  if (k_new || v_new || slot_mapping) {
    if (!k_new || !v_new || !slot_mapping || !new_strides)
      return fail(MI_ERR_INVALID, "k_new, v_new, new_strides and slot_mapping go together");
    const int64_t st[3] = {new_strides[0], new_strides[1], 0};
    int rc = mi_kv_scatter(k_new, v_new, st, st, batch, 1, nullptr, nullptr, slot_mapping, batch, k_pool, v_pool,
                           num_blocks, block_size, num_kv_heads, head_dim, dtype, stream);
    if (rc != MI_OK) return rc;
  }
  mi::DecodePlan plan =
      mi::plan_decode(batch, num_q_heads, num_kv_heads, head_dim, max_blocks_per_seq, block_size, dtype);
  if (plan.use_mma) {
    const bool ok = aligned(k_pool, 16) && aligned(v_pool, 16) && aligned(q, 4) && (q_strides[0] * es) % 4 == 0 &&
                    (q_strides[1] * es) % 4 == 0 && num_blocks * block_size < (int64_t(1) << 31);
    if (!ok) plan = mi::plan_decode(batch, num_q_heads, num_kv_heads, head_dim, max_blocks_per_seq, block_size, -1);
  }
  if (ex.world > 0 && !plan.use_mma)
    return fail(MI_ERR_UNSUPPORTED,
                "mi_paged_decode_exchange: needs the tensor-core decode path (bf16/fp16, head_dim 64/128, "
                "block size 16/32, at most 8 query heads per KV head, 16-byte aligned pools)");
  mi::DecodeArgs a{};
  a.q = static_cast<const char*>(q);
  a.q_sb = q_strides[0] * es;
  a.q_sh = q_strides[1] * es;
  a.k_pool = static_cast<const char*>(k_pool);
  a.v_pool = static_cast<const char*>(v_pool);
  a.block_tables = block_tables;
  a.table_stride = table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  a.batch = batch;
  a.num_blocks = num_blocks;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.groups = num_q_heads / num_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.split_pages = plan.split_pages;
  a.max_splits = plan.max_splits;
  a.parts_per_split = plan.parts_per_split;
  a.max_parts = plan.max_splits * plan.parts_per_split;
  a.out = static_cast<char*>(out);
  a.out_sb = out_stride * es;
  a.world = ex.world;
  a.rank = ex.rank;
  a.gathered_sb = ex.gathered_sb;
  for (int p = 0; p < mi::kMaxPeers; ++p) a.gathered[p] = ex.gathered[p];
  CUtensorMap tk, tv;
  if (plan.use_mma) {
    if (!workspace || workspace_bytes < plan.ws_bytes || !aligned(workspace, 256))
      return fail(MI_ERR_INVALID, "workspace must be >= %zu bytes and 256-byte aligned (got %zu)", plan.ws_bytes,
                  workspace_bytes);
    const size_t o_bytes = (size_t)batch * num_q_heads * a.max_parts * head_dim * sizeof(float);
    a.ws_o = static_cast<float*>(workspace);
    a.ws_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + ((o_bytes + 255) & ~size_t(255)));
    if (int rc = pool_tensor_map(k_pool, num_blocks, block_size, num_kv_heads, head_dim, dtype, &tk)) return rc;
    if (int rc = pool_tensor_map(v_pool, num_blocks, block_size, num_kv_heads, head_dim, dtype, &tv)) return rc;
  }
  cudaError_t e = mi::launch_paged_decode(a, plan, &tk, &tv, dtype, s);
  if (e != cudaSuccess) return cuda_fail(e, "mi_paged_decode launch");
  if (ex.world > 0) {
    e = mi::launch_peer_barrier(ex.barrier, s);
    if (e != cudaSuccess) return cuda_fail(e, "mi_paged_decode_exchange: peer barrier launch");
  }
  return MI_OK;
}

}  // namespace

extern "C" {

int mi_paged_decode(const void* q, const int64_t* q_strides, const void* k_new, const void* v_new,
                    const int64_t* new_strides, const int64_t* slot_mapping, void* k_pool, void* v_pool,
                    int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                    const int64_t* block_tables, int64_t table_stride, int64_t max_blocks_per_seq,
                    const int64_t* context_lens, int64_t batch, int num_q_heads, float scale, void* out,
                    int64_t out_stride, void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  return paged_decode_impl(q, q_strides, k_new, v_new, new_strides, slot_mapping, k_pool, v_pool, num_blocks,
                           block_size, num_kv_heads, head_dim, block_tables, table_stride, max_blocks_per_seq,
                           context_lens, batch, num_q_heads, scale, out, out_stride, workspace, workspace_bytes,
                           dtype, stream, DecodeExchange{});
}

int mi_paged_decode_exchange(const void* q, const int64_t* q_strides, const void* k_new, const void* v_new,
                             const int64_t* new_strides, const int64_t* slot_mapping, void* k_pool, void* v_pool,
                             int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                             const int64_t* block_tables, int64_t table_stride, int64_t max_blocks_per_seq,
                             const int64_t* context_lens, int64_t batch, int num_q_heads, float scale,
                             void* const* gathered, int64_t gathered_stride, unsigned int* const* flags,
                             unsigned int* epoch, int rank, int world, int64_t timeout_ns, void* workspace,
                             size_t workspace_bytes, int dtype, void* stream) {
  if (world < 2 || world > mi::kMaxPeers || rank < 0 || rank >= world)
    return fail(MI_ERR_INVALID, "mi_paged_decode_exchange: rank %d of world %d (2..%d ranks)", rank, world,
                mi::kMaxPeers);
  if (!gathered || !flags || !epoch || timeout_ns <= 0)
    return fail(MI_ERR_INVALID, "mi_paged_decode_exchange: null pointer argument or non-positive timeout");
  const int es = elem_size(dtype);
  if (es != 2) return fail(MI_ERR_INVALID, "mi_paged_decode_exchange: bf16 or fp16 only");
  if (gathered_stride < (int64_t)world * num_q_heads * head_dim)
    return fail(MI_ERR_INVALID, "mi_paged_decode_exchange: gathered rows of %lld elements hold less than %d ranks x "
                "%d heads x %d", (long long)gathered_stride, world, num_q_heads, head_dim);
  DecodeExchange ex;
  ex.world = world;
  ex.rank = rank;
  ex.gathered_sb = gathered_stride * es;
  for (int p = 0; p < world; ++p) {
    if (!gathered[p] || !flags[p] || !aligned(gathered[p], 16) || !aligned(flags[p], 4))
      return fail(MI_ERR_INVALID, "mi_paged_decode_exchange: rank %d's buffers are null or misaligned", p);
    ex.gathered[p] = static_cast<char*>(gathered[p]);
    ex.barrier.flags[p] = flags[p];
  }
  if (ex.gathered_sb % 16) return fail(MI_ERR_INVALID, "mi_paged_decode_exchange: row stride not 16-byte aligned");
  ex.barrier.epoch = epoch;
  ex.barrier.rank = rank;
  ex.barrier.world = world;
  ex.barrier.timeout_ns = (uint64_t)timeout_ns;
  return paged_decode_impl(q, q_strides, k_new, v_new, new_strides, slot_mapping, k_pool, v_pool, num_blocks,
                           block_size, num_kv_heads, head_dim, block_tables, table_stride, max_blocks_per_seq,
                           context_lens, batch, num_q_heads, scale, nullptr, 0, workspace, workspace_bytes, dtype,
                           stream, ex);
}

size_t mi_paged_prefill_workspace_size(int64_t batch, int64_t padded_len, int num_q_heads, int num_kv_heads,
                                       int head_dim, int64_t table_stride, int block_size, int dtype) {
  if (batch <= 0 || padded_len <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return 0;
  if ((dtype != MI_BF16 && dtype != MI_F16) || head_dim != 128) return 0;
  mi::PrefillArgs a{};
  a.batch = batch;
  a.padded_len = padded_len;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.groups = num_q_heads / num_kv_heads;
  a.head_dim = head_dim;
  a.table_stride = table_stride;
  a.block_size = block_size;
  return mi::prefill_tc_workspace_bytes(a);
}

int mi_paged_prefill(const void* q, const int64_t* q_strides, const void* k_chunk, const void* v_chunk,
                     const int64_t* kv_strides, const void* k_pool, const void* v_pool, int64_t num_blocks,
                     int block_size, int num_kv_heads, int head_dim, const int64_t* block_tables,
                     int64_t table_stride, const int64_t* start_positions, const int64_t* chunk_lens, int64_t batch,
                     int64_t padded_len, int num_q_heads, float scale, void* out, void* workspace,
                     size_t workspace_bytes, int dtype, void* stream) {
  if (int rc = check_pool_geometry(num_blocks, block_size, num_kv_heads, head_dim, dtype)) return rc;
  if (batch < 0 || padded_len < 0 || table_stride < 0) return fail(MI_ERR_INVALID, "negative size");
  if (batch == 0 || padded_len == 0) return MI_OK;
  if (num_q_heads < 1 || num_q_heads % num_kv_heads != 0)
    return fail(MI_ERR_INVALID, "num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)", num_q_heads,
                num_kv_heads);
  if (head_dim > 256) return fail(MI_ERR_UNSUPPORTED, "head_dim %d > 256", head_dim);
  if (!q || !q_strides || !k_chunk || !v_chunk || !kv_strides || !start_positions ||
      !chunk_lens || !out || (table_stride > 0 && !block_tables))
    return fail(MI_ERR_INVALID, "mi_paged_prefill: null pointer argument");
  if ((!k_pool || !v_pool) && table_stride > 0)
    return fail(MI_ERR_INVALID, "mi_paged_prefill: pools may be null only without history (table_stride == 0)");
  const int es = elem_size(dtype);
  mi::PrefillArgs a{};
  a.q = static_cast<const char*>(q);
  a.k_chunk = static_cast<const char*>(k_chunk);
  a.v_chunk = static_cast<const char*>(v_chunk);
  for (int i = 0; i < 3; ++i) {
    a.q_sb[i] = q_strides[i] * es;
    a.kv_sb[i] = kv_strides[i] * es;
  }
  a.k_pool = static_cast<const char*>(k_pool);
  a.v_pool = static_cast<const char*>(v_pool);
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.table_stride = table_stride;
  a.starts = start_positions;
  a.chunk_lens = chunk_lens;
  a.batch = batch;
  a.padded_len = padded_len;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.groups = num_q_heads / num_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = static_cast<char*>(out);
  float* ws = nullptr;
  mi::PrefillMaps maps{};
  bool use_maps = false;
  if (mi::prefill_tc_supported(a, dtype)) {
    const size_t need = mi::prefill_tc_workspace_bytes(a);
    if (need > 0) {
      if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
        return fail(MI_ERR_INVALID, "prefill workspace must be >= %zu bytes and 256-byte aligned (got %zu)", need,
                    workspace_bytes);
      ws = static_cast<float*>(workspace);
    }
    // TMA staging when every operand it reads has a tensor map (without history the pools are not
    // read, so any block size qualifies); otherwise the kernel uses cp.async.
    if ((table_stride == 0 || mi::prefill_tc_tma_block_size(block_size)) && padded_len < (int64_t(1) << 31)) {
      const int G = a.groups;
      const cuuint64_t qd[4] = {(cuuint64_t)head_dim, (cuuint64_t)num_q_heads, (cuuint64_t)padded_len,
                                (cuuint64_t)batch};
      const cuuint64_t qs[3] = {(cuuint64_t)a.q_sb[2], (cuuint64_t)a.q_sb[1], (cuuint64_t)a.q_sb[0]};
      const cuuint32_t qb[4] = {64, (cuuint32_t)G, (cuuint32_t)(128 / G), 1};
      const cuuint64_t kd[4] = {(cuuint64_t)head_dim, (cuuint64_t)num_kv_heads, (cuuint64_t)padded_len,
                                (cuuint64_t)batch};
      const cuuint64_t ks[3] = {(cuuint64_t)a.kv_sb[2], (cuuint64_t)a.kv_sb[1], (cuuint64_t)a.kv_sb[0]};
      const cuuint32_t kb[4] = {64, 1, 64, 1};
      use_maps = encode_map(q, 4, qd, qs, qb, dtype, &maps.q) && encode_map(k_chunk, 4, kd, ks, kb, dtype, &maps.k_chunk) &&
                 encode_map(v_chunk, 4, kd, ks, kb, dtype, &maps.v_chunk);
      if (use_maps && table_stride > 0) {
        use_maps = pool_tensor_map(k_pool, num_blocks, block_size, num_kv_heads, head_dim, dtype, &maps.k_pool) ==
                       MI_OK &&
                   pool_tensor_map(v_pool, num_blocks, block_size, num_kv_heads, head_dim, dtype, &maps.v_pool) ==
                       MI_OK;
      }
    }
  }
  cudaError_t e = mi::launch_paged_prefill(a, ws, use_maps ? &maps : nullptr, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MI_OK : cuda_fail(e, "mi_paged_prefill launch");
}

}  // extern "C"
