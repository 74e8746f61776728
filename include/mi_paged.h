/*
 * mi_paged.h — C ABI of the B200 paged KV-cache library (libmi_paged.so, sm_100a).
 *
 * The library holds the device side of mini-infra-qwen3's paged KV-cache hot path.  Every entry
 * point takes plain device pointers, element strides and sizes, plus the CUDA stream to launch on
 * (a cudaStream_t passed as void*; NULL = legacy default stream).  Nothing here allocates, frees
 * or synchronizes: callers own every buffer (pools, metadata, outputs, workspace) and calls are
 * asynchronous on the given stream.  Integer metadata (block tables, slots, lengths) is int64,
 * as the reference's PagedRunner packs it.
 *
 * Layouts (the reference's own, worker/paged_kv_cache.py:15-20):
 *   pool      [num_blocks, block_size, num_kv_heads, head_dim], contiguous; slot = block*bs + offset
 *   block 0   is the null block: it pads block tables and is never allocated
 *   tables    [batch, table_stride] int64, row b lists the physical blocks of sequence b
 *
 * Return value: MI_OK (0) or a negative MI_ERR_* code; mi_last_error() then describes it.
 * Device-side checks (out-of-range block ids or slots, bounded waits that ran out) never trap:
 * they set bits in a sticky device status word read back with mi_read_status().
 */
#ifndef MI_PAGED_H
#define MI_PAGED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define MI_F32 0
#define MI_BF16 1
#define MI_F16 2

/* return codes */
#define MI_OK 0
#define MI_ERR_INVALID (-1)     /* argument rejected on the host before any launch */
#define MI_ERR_CUDA (-2)        /* a CUDA call or launch failed */
#define MI_ERR_UNSUPPORTED (-3) /* valid arguments, but no kernel variant for them */

/* device status bits (sticky, see mi_read_status) */
#define MI_STATUS_BAD_BLOCK 1u   /* a block table entry was outside [0, num_blocks) */
#define MI_STATUS_BAD_SLOT 2u    /* a destination slot was outside [0, num_blocks*block_size) */
#define MI_STATUS_TIMEOUT 4u     /* a bounded wait inside a kernel gave up */
#define MI_STATUS_BAD_LENGTH 8u  /* a context/chunk length exceeded what the block table covers */
#define MI_STATUS_BAD_INDEX 16u  /* a scatter source row/position was outside the source tensor */

/* Library version (major*10000 + minor*100 + patch). */
int mi_version(void);

/* Text of the last host-side error of the calling thread ("" if none). */
const char* mi_last_error(void);

/* Read (and optionally clear) the device status word of the current device.  Synchronizes
 * `stream`.  *status_out receives the MI_STATUS_* bits seen since the last clear. */
int mi_read_status(unsigned int* status_out, int clear, void* stream);

/*
 * mi_kv_scatter — copy tokens into one layer's K and V pools, K and V in one launch.
 * Replaces PagedKVCachePool.write_prefill (worker/paged_kv_cache.py:74-95:
 *   pool.view(-1,H,D).index_copy_(0, slot_mapping, key[token_rows, :, token_positions, :]))
 * and the decode append of Qwen3Attention._apply_paged_kv_pool (model/qwen3.py:282-283).
 *
 * k_src/v_src element (r, h, p, d) is at  r*s[0] + h*s[1] + p*s[2] + d  (elements; d contiguous),
 * with s = k_strides / v_strides (3 entries each).  Token i copies source (token_rows[i], :,
 * token_positions[i], :) to pool slot slot_mapping[i].  token_rows == NULL means row i;
 * token_positions == NULL means position 0 (decode append: source [B, H, D]).
 * src_rows / src_positions bound the source (its B and L; L = 1 for a decode append): tokens whose
 * row/position fall outside are skipped and flagged, as are out-of-range slots.  Slots must be
 * distinct (as index_copy_ requires).
 */
int mi_kv_scatter(const void* k_src, const void* v_src, const int64_t* k_strides, const int64_t* v_strides,
                  int64_t src_rows, int64_t src_positions, const int64_t* token_rows,
                  const int64_t* token_positions, const int64_t* slot_mapping, int64_t num_tokens, void* k_pool,
                  void* v_pool, int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype,
                  void* stream);

/*
 * mi_kv_store_chunks — PagedRunner.store_prefill (worker/paged_runner.py:104-136) on the device:
 * row b's valid tokens are the last chunk_lens[b] positions of the padded length `padded_len`;
 * token j goes to logical position start_positions[b] + j, i.e. slot
 * block_tables[b, pos / bs] * bs + pos % bs.  No host-side slot list is needed.
 * Source strides as in mi_kv_scatter.  chunk_lens/start_positions are int64 [batch] on device.
 */
int mi_kv_store_chunks(const void* k_src, const void* v_src, const int64_t* k_strides, const int64_t* v_strides,
                       int64_t batch, int64_t padded_len, const int64_t* chunk_lens, const int64_t* start_positions,
                       const int64_t* block_tables, int64_t table_stride, void* k_pool, void* v_pool,
                       int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype, void* stream);

/*
 * mi_kv_gather_blocks — PagedKVCachePool.gather_blocks for one pool (worker/paged_kv_cache.py:54-72):
 * out[b, j] = pool[block_ids[b, j]], out contiguous [batch, blocks_per_row, bs, H_kv, D].
 */
int mi_kv_gather_blocks(const void* pool, const int64_t* block_ids, int64_t batch, int64_t blocks_per_row,
                        void* out, int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, int dtype,
                        void* stream);

/*
 * mi_paged_decode — one decode step of paged GQA attention for one layer (one query token per
 * sequence).  Replaces the history gather + _attend of the paged branch
 * (model/qwen3.py:285-292 and :219-255, bias of :513-527): sequence b attends to positions
 * [0, context_lens[b]) of its block table; query head hq reads KV head hq / (num_q_heads/num_kv_heads).
 * Softmax and accumulation are fp32.  The new token must already be in the pool (mi_kv_scatter),
 * unless k_new/v_new/slot_mapping are given, in which case they are appended first (same launch
 * sequence, same stream).
 *
 *   q        [batch, num_q_heads, head_dim]  element (b, h, d) at b*q_strides[0] + h*q_strides[1] + d
 *   out      [batch, num_q_heads*head_dim]   row b at b*out_stride
 *   k_new    [batch, num_kv_heads, head_dim] (optional) strides new_strides[0..1]
 *   workspace  >= mi_paged_decode_workspace_size(...) bytes, 256-byte aligned (split-K partials)
 */
size_t mi_paged_decode_workspace_size(int64_t batch, int num_q_heads, int num_kv_heads, int head_dim,
                                      int64_t max_blocks_per_seq, int block_size, int dtype);
int mi_paged_decode(const void* q, const int64_t* q_strides, const void* k_new, const void* v_new,
                    const int64_t* new_strides, const int64_t* slot_mapping, void* k_pool, void* v_pool,
                    int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                    const int64_t* block_tables, int64_t table_stride, int64_t max_blocks_per_seq,
                    const int64_t* context_lens, int64_t batch, int num_q_heads, float scale, void* out,
                    int64_t out_stride, void* workspace, size_t workspace_bytes, int dtype, void* stream);

/*
 * mi_paged_decode_static_scratch — mi_paged_decode for callers that cannot allocate device memory.
 * No counterpart in the reference: it exists for callers of this library that have no way to
 * provide the split-K workspace — hosts binding the C ABI without a device allocator of their own
 * (a C, Go or JNI program has no caching allocator to take a workspace from) and loops that cannot
 * afford cudaMalloc's implicit device synchronisation.  Same arguments and results as
 * mi_paged_decode minus the workspace: the split-K partials go to a file-scope device array of
 * MI_STATIC_SCRATCH_BYTES that every GPU loading the library holds until the process exits.
 * Nothing is allocated.  A call whose partials would exceed the array is rejected with
 * MI_ERR_UNSUPPORTED (use mi_paged_decode then).  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current) and caches it: make that first
 * call before any stream capture, and make no call after a cudaDeviceReset of that device (the
 * cached address then names a released module).  All calls share the array and it keeps the last
 * call's contents: calls that overlap on the GPU race and must be serialised by the caller.
 */
#define MI_STATIC_SCRATCH_BYTES ((size_t)32 << 20)
int mi_paged_decode_static_scratch(const void* q, const int64_t* q_strides, const void* k_new, const void* v_new,
                                   const int64_t* new_strides, const int64_t* slot_mapping, void* k_pool,
                                   void* v_pool, int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                                   const int64_t* block_tables, int64_t table_stride, int64_t max_blocks_per_seq,
                                   const int64_t* context_lens, int64_t batch, int num_q_heads, float scale,
                                   void* out, int64_t out_stride, int dtype, void* stream);

/*
 * mi_paged_decode_exchange — mi_paged_decode on a KV-head partition with the exchange of the
 * attention outputs fused in.  Replaces, for a rank of `world` that holds query heads
 * [rank*num_q_heads, (rank+1)*num_q_heads) (num_q_heads is this rank's count), the decode call
 * followed by the NCCL all-gather of the per-head outputs and the reordering into global head
 * order (the reference runs on one device and has no exchange: model/qwen3.py:219-255 produces the
 * [batch, all heads * head_dim] rows that o_proj reads).  The combine kernel stores row b of its
 * local query head j straight into every rank's gathered buffer at
 *   gathered[p] + b * gathered_stride + (rank * num_q_heads + j) * head_dim   (elements, p < world)
 * with plain stores over NVLink (no multicast), then a one-warp barrier kernel stores epoch e into
 * flags[p][rank] of every peer p (release, system scope) and waits (acquire) until every peer has
 * stored e into flags[rank][p]; e = *epoch + 1, written back to *epoch.  After the call (in stream
 * order) gathered[rank] holds all ranks' heads in global order.
 *
 *   gathered  [world] pointers valid in this process (peers' through mi_peer_open): each rank's
 *             [batch, gathered_stride >= world*num_q_heads*head_dim] buffer, 16-byte aligned rows
 *   flags     [world] pointers: each rank's [world] uint32 flag array, zero before the first call
 *   epoch     this rank's uint32 call counter (device), zero before the first call
 *   timeout_ns  bound of the barrier's wait; a peer that does not arrive in time sets
 *             MI_STATUS_TIMEOUT and the call returns (the gathered rows are then incomplete)
 * Every rank must make the same calls in the same order.  A rank may store into a peer's buffer
 * while that peer still reads the previous call's rows, so consecutive calls must alternate
 * between two buffers.  bf16/fp16 on the tensor-core decode path only (else MI_ERR_UNSUPPORTED).
 */
int mi_paged_decode_exchange(const void* q, const int64_t* q_strides, const void* k_new, const void* v_new,
                             const int64_t* new_strides, const int64_t* slot_mapping, void* k_pool, void* v_pool,
                             int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                             const int64_t* block_tables, int64_t table_stride, int64_t max_blocks_per_seq,
                             const int64_t* context_lens, int64_t batch, int num_q_heads, float scale,
                             void* const* gathered, int64_t gathered_stride, unsigned int* const* flags,
                             unsigned int* epoch, int rank, int world, int64_t timeout_ns, void* workspace,
                             size_t workspace_bytes, int dtype, void* stream);

/*
 * Peer memory for mi_paged_decode_exchange (no counterpart in the single-device reference).
 * mi_peer_handle writes the CUDA IPC handle (MI_PEER_HANDLE_BYTES) of the allocation holding `ptr`
 * and ptr's offset into it; another process of the same node opens it with mi_peer_open (a pointer
 * valid in that process, peer access enabled) and releases it with mi_peer_close.  Nothing is
 * allocated; the exporting process keeps the buffer alive until every peer has closed it.
 */
#define MI_PEER_HANDLE_BYTES 64
int mi_peer_handle(const void* ptr, void* handle_out, int64_t* offset_out);
int mi_peer_open(const void* handle, int64_t offset, void** ptr_out);
int mi_peer_close(void* ptr, int64_t offset);

/*
 * mi_paged_prefill — varlen chunked-prefill attention for one layer.  Replaces, for
 * PagedRunner.run_prefill_chunk_step (worker/paged_runner.py:32-102), the all-layer history
 * gather (gather_blocks), torch.cat(history, chunk) (model/qwen3.py:328-329), the padded causal
 * mask (:438-485) and _attend (:219-255).  Row b's chunk holds chunk_lens[b] valid tokens
 * right-aligned in padded_len (left padding); its token j is logical position
 * start_positions[b] + j and attends causally to the chunk and to the first start_positions[b]
 * positions of its history, read in place from the pools through block_tables.
 * Output rows of padding positions are written as zeros.
 *
 *   q        [batch, padded_len, num_q_heads, head_dim], element (b,p,h,d) at
 *            b*q_strides[0] + p*q_strides[1] + h*q_strides[2] + d
 *   k_chunk  [batch, padded_len, num_kv_heads, head_dim], strides kv_strides[0..2] (v_chunk same)
 *   out      [batch, padded_len, num_q_heads*head_dim] contiguous
 *   workspace  >= mi_paged_prefill_workspace_size(...) bytes, 256-byte aligned (partials of the
 *            work units that straddle two persistent CTAs, ~39 MB for the tensor-core path; the
 *            size depends only on the arguments of that function)
 */
size_t mi_paged_prefill_workspace_size(int64_t batch, int64_t padded_len, int num_q_heads, int num_kv_heads,
                                       int head_dim, int64_t table_stride, int block_size, int dtype);
int mi_paged_prefill(const void* q, const int64_t* q_strides, const void* k_chunk, const void* v_chunk,
                     const int64_t* kv_strides, const void* k_pool, const void* v_pool, int64_t num_blocks,
                     int block_size, int num_kv_heads, int head_dim, const int64_t* block_tables,
                     int64_t table_stride, const int64_t* start_positions, const int64_t* chunk_lens, int64_t batch,
                     int64_t padded_len, int num_q_heads, float scale, void* out, void* workspace,
                     size_t workspace_bytes, int dtype, void* stream);

/*
 * mi_decode_rows — the packed decode-step inputs of PagedRunner.prepare_decode_inputs
 * (worker/paged_runner.py:138-166: per sequence [token, position, slot, position + 1, block table
 * null-padded]) built on the device from a device mirror of the block tables, so a step uploads
 * O(batch) integers instead of O(batch x max_blocks).
 *
 *   tables   [table_rows, table_stride] int64 on the device: one row per batch slot, holding that
 *            slot's sequence's block table; entries are written only through `deltas`
 *   deltas   [num_deltas, 3] int64 (row, column, block id): table entries added since the last
 *            call, applied first
 *   rows     [batch, 3] int64 (table row, token, position) of the step's sequences
 *   out      int64, written as ids [n] | positions [n] | slots [n] | context lengths [n] |
 *            tables [n, width]: row b < batch gets its token and position, slot
 *            tables[row][pos / bs] * bs + pos % bs, context pos + 1 and the first
 *            ceil((pos + 1) / bs) entries of its table row (the rest 0, the null block); rows
 *            batch <= b < n are padding (token 0, position 0, slot 0, context 1, null table).
 * Bit-exact with the host packing.  Out-of-range rows, columns or lengths are skipped and set
 * MI_STATUS_BAD_INDEX / MI_STATUS_BAD_LENGTH.
 */
int mi_decode_rows(const int64_t* rows, int64_t batch, const int64_t* deltas, int64_t num_deltas, int64_t* tables,
                   int64_t table_rows, int64_t table_stride, int64_t* out, int64_t n, int64_t width, int block_size,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MI_PAGED_H */
