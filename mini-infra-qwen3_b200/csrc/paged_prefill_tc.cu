// Chunked-prefill paged attention on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Variant: bf16 / fp16, head_dim 128, any block size, G = Hq/H_kv in {1, 2, 4, 8}.
// One CTA (320 threads, one CTA per SM) = one (sequence, KV head, pair of tiles of 128 query
// rows, KV split).  A row tile packs 128/G chunk tokens x the G query heads of the KV head (row
// r = token r/G, head r%G); the CTA's two row tiles are consecutive, so every K/V tile staged in
// shared memory serves 2 x 128 query rows of the whole GQA group (half the L2 -> SM bytes per
// FLOP of one row tile per CTA).  The KV range of a row tile (history tiles, then causal chunk
// tiles) is cut into equal splits of at most kTilesPerSplit 128-position tiles so that long
// histories spread over many CTAs of equal work; the two row tiles' ranges differ only in their
// last chunk tiles, so the CTA stages the union and each row tile uses a prefix of it.  A row
// tile with one split writes its output directly, otherwise each split writes an unnormalised
// partial (O, m, l) that prefill_combine_kernel merges.  Warp roles, linked by mbarriers:
//   warp 0 (loader): both Q tiles once, then K and V tiles into a kStagesK-deep K ring and a
//      kStagesV-deep V ring (K is free once the S of both row tiles is done, V once both PVs
//      are).  With tensor maps (block size 16/32/64) the split's block ids are first resolved
//      into shared memory, then an elected lane issues TMA copies: one 3D box per pool page of a
//      history tile (a page past `start` reads rows past the pool, which TMA fills with zeros)
//      and 4D boxes of 64 tokens for a chunk tile; otherwise the warp stages rows with cp.async;
//   warp 1 (MMA, elected lane): per row tile g, S_g = Q_g K^T as 8 tcgen05.mma (M=128, N=128,
//      K=16, kind::f16, fp32 accumulate: 8 KiB of shared-memory operands per 64 cycles of math,
//      the shared-memory rate) into g's TMEM S columns, and O_g += P_g V as 8 tcgen05.mma
//      (M=128, N=128, P read from TMEM, V read MN-major) into g's TMEM O columns.  The row tiles
//      alternate: PV_0(i), S_0(i+1), PV_1(i), S_1(i+1), so the softmax of one row tile runs
//      under the MMAs of the other; tcgen05.commit signals mbarriers;
//   warps 2-5 / 6-9 (softmax of row tile 0 / 1): each thread owns one row (its TMEM lane):
//      tcgen05.ld of the row's 128 scores, causal / length mask (set to -inf) only on tiles that
//      cross a row's causal end or the history end, online softmax in the exp2 domain; the
//      running O in TMEM is rescaled (tcgen05.ld/st, warp-wide) only when a row maximum grew by
//      more than 2^8 since its last rescale (p <= 2^8 stays exact in fp32 and the final 1/l
//      absorbs it); P is written back with tcgen05.st as 16-bit pairs into the first 64 columns
//      of g's S columns (S_g(i+1) overwrites them only after PV_g(i), issued before it, has read
//      them: tcgen05.mma of one thread run in issue order).
// Epilogue: tcgen05.ld of O, divide by l (or store the partial), 16-byte stores.  Padding
// positions get zeros.
//
// Shared-memory operand layout ("SW128"): an operand of R rows x 128 two-byte columns is two
// regions of R*128 bytes (columns 0-63 and 64-127); row r of a region is 128 bytes at r*128 and
// its 16-byte unit u lives at unit u ^ (r % 8).  Every region starts 1024-byte aligned.
// Descriptors:
//   K-major (Q and K: R=128):  LBO = 16 B (unused),
//     SBO = 1024 B (8-row groups), swizzle 128B; k-step s starts at region(s/4) + (s%4)*32 B.
//   MN-major (V as the B operand of PV, N = head_dim):  LBO = 16 KiB (next 64 columns of N),
//     SBO = 1024 B (next 8 K-rows); k-step s starts at s*16 rows = s*2048 B.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace mi {
namespace {

constexpr int kTcRows = 128;                        // query rows per row tile (MMA M)
constexpr int kPair = 2;                            // row tiles per CTA, sharing every K/V tile
constexpr int kTcKv = 128;                          // KV positions per tile (MMA N of S)
constexpr int kTcDim = 128;                         // head_dim
constexpr int kSoftmaxThreads = 128;                // one warpgroup per row tile
constexpr int kTcThreads = 64 + kPair * kSoftmaxThreads;  // warp 0 loader, warp 1 MMA, then the warpgroups
constexpr int kLoaderWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kLoaderThreads = 32;
constexpr int kTilesPerSplit = 16;                  // 2048 KV positions per CTA at most
constexpr int kStagesK = 3;                         // depth of the K ring
constexpr int kStagesV = 2;                         // depth of the V ring
constexpr int kQRegion = kTcRows * 128;             // 16 KiB: one 64-column half of a Q tile
constexpr int kKvRegion = kTcKv * 128;              // 16 KiB: one 64-column half of a K or V tile
constexpr int kQBytes = 2 * kQRegion;               // 32 KiB per row tile
constexpr int kKvBytes = 2 * kKvRegion;             // 32 KiB
constexpr int kOffQ = 0;                            // kPair Q tiles
constexpr int kOffK = kOffQ + kPair * kQBytes;      // kStagesK K buffers
constexpr int kOffV = kOffK + kStagesK * kKvBytes;  // kStagesV V buffers
constexpr int kOffBar = kOffV + kStagesV * kKvBytes;
constexpr int kOffPages = kOffBar + 256;            // block ids (cp.async: kTcKv+1 int64 of one tile; TMA: 128 int32)
constexpr int kTcSmemBytes = kOffPages + (kTcKv + 1) * 8 + 1024;  // + alignment slack (~226 KiB: one CTA per SM)
static_assert(kTcSmemBytes <= 232448, "shared memory above the 227 KiB a CTA may use");
// TMEM (512 columns): S (then P) of row tile g at g*128; O of row tile g at 256 + g*128.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;
constexpr float kRescaleLog2 = 8.0f;

__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t unit16, uint32_t region) {
  // unit16 in [0, 16): 16-byte unit of a 256-byte row (128 two-byte columns)
  return (unit16 >> 3) * region + row * 128 + (((unit16 & 7) ^ (row & 7)) << 4);
}

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (uint64_t(kKvRegion >> 4) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// kind::f16 instruction descriptor: fp32 accumulate, A/B format, A K-major, B K- or MN-major, N, M.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, bool b_mn_major, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// The tcgen05 / TMA issue helpers below are executed by a whole converged warp (so their operands
// are warp-uniform and live in uniform registers); the lane chosen by elect.sync issues.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Same, with A (M=128 rows x 16 K elements, two 16-bit values per 32-bit column) read from TMEM.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                                uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_e(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_e(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                              int c3) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void mbar_expect_tx_e(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_u32(bar)), "r"(bytes)
      : "memory");
}
// Bounded wait by a whole warp; leaves the warp converged with a warp-uniform `aborted`.
__device__ __forceinline__ void mbar_wait_warp(uint64_t* bar, uint32_t parity, bool& aborted) {
  mbar_wait(bar, parity, aborted);
  aborted = __any_sync(0xffffffffu, aborted);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// tcgen05.ld of 32 columns without the wait: issue several, then one tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// tcgen05.st of 16 columns without the wait: issue several, then one tmem_wait_st().
__device__ __forceinline__ void tmem_st16_async(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t sdst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sdst), "l"(gsrc), "r"(valid ? 16u : 0u)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }


// Block-table position -> pool row: shift/mask when the block size is a power of two.
struct BlockAddr {
  int shift;  // log2(block_size), or -1
  uint32_t bs;
  __device__ __forceinline__ void split(uint32_t pos, uint32_t& blk_idx, uint32_t& off) const {
    if (shift >= 0) {
      blk_idx = pos >> shift;
      off = pos & (bs - 1);
    } else {
      blk_idx = pos / bs;
      off = pos - blk_idx * bs;
    }
  }
};

// KV tiles of a row tile: first the history tiles (positions [128k, 128k + 128) of [0, start),
// read from the pool), then the chunk tiles (chunk tokens [128k, 128k + 128) of [0, tok_end), read
// from the chunk's own K/V).  Keeping the two apart aligns every tile to its source, so each one is
// a few whole TMA boxes: pool pages [64 x 1 x block_size] or [64 x 1 x 64 x 1] chunk boxes.
struct TcGeometry {
  int64_t len, first;
  int start;
  int hist_tiles;  // ceil(start / kTcKv)
  int n_tiles;     // history tiles + chunk tiles up to the causal end of the tile's last token
};

__device__ __forceinline__ TcGeometry tc_geometry(const PrefillArgs& a, int64_t b, int64_t tok0, int tokens_per_tile,
                                                  bool report) {
  TcGeometry g;
  int64_t len = a.chunk_lens[b];
  if (len > a.padded_len) {
    if (report) record_status(MI_STATUS_BAD_LENGTH);
    len = a.padded_len;
  }
  g.len = len < 0 ? 0 : len;
  g.first = a.padded_len - g.len;
  int64_t start = a.starts[b];
  if (start < 0) start = 0;
  if (start > a.table_stride * a.block_size) {
    if (report) record_status(MI_STATUS_BAD_LENGTH);
    start = a.table_stride * a.block_size;
  }
  g.start = (int)start;
  g.hist_tiles = (int)((start + kTcKv - 1) / kTcKv);
  const int64_t tok_end = min(g.len, tok0 + tokens_per_tile);
  g.n_tiles = tok0 < g.len ? g.hist_tiles + (int)((tok_end + kTcKv - 1) / kTcKv) : 0;
  return g;
}

// Equal-size splits of a row-tile pair: the union of the pair's tile ranges (the second tile's,
// which is never shorter unless it is empty) is cut into ceil(tiles / kTilesPerSplit) parts of
// `per` tiles (the last one shorter), so a row's CTAs carry equal work and the grid's tail is
// short.  Row tile g's splits are the parts that start below its own tile count.
struct TcSplits {
  int per;         // tiles per split
  int splits[2];   // splits holding tiles of row tile 0 / 1
};
__device__ __forceinline__ TcSplits tc_splits(int n_tiles0, int n_tiles1) {
  TcSplits sp;
  const int nu = max(n_tiles0, n_tiles1);
  const int parts = max(1, (nu + kTilesPerSplit - 1) / kTilesPerSplit);
  sp.per = max(1, (nu + parts - 1) / parts);
  sp.splits[0] = (n_tiles0 + sp.per - 1) / sp.per;
  sp.splits[1] = (n_tiles1 + sp.per - 1) / sp.per;
  return sp;
}

// cp.async staging (block sizes without a TMA box) of the K or the V rows of history tile k =
// positions [128k, 128k + 128) from `pool`; rows at or past `start` zero-filled; block ids of the
// tile's pages are read once into `pages`.
template <typename T>
__device__ __forceinline__ void stage_hist_cp(const PrefillArgs& a, const BlockAddr& ba, int64_t b, int h, int start,
                                              int k, const char* pool, uint32_t dst, int lane, int64_t* pages) {
  const int unit = lane & 15;
  const int j0 = k * kTcKv;
  const int hist_rows = max(0, min(kTcKv, start - j0));
  uint32_t p0, off0, p1, off1;
  ba.split((uint32_t)j0, p0, off0);
  ba.split((uint32_t)(j0 + max(hist_rows, 1) - 1), p1, off1);
  const int64_t* table = a.block_tables + b * a.table_stride;
  for (int q = lane; q <= (int)(p1 - p0); q += 32) pages[q] = table[p0 + q];
  __syncwarp();
  const int64_t pool_row = (int64_t)a.hkv * kTcDim * sizeof(T);
  const int64_t head_off = (int64_t)h * kTcDim * sizeof(T) + unit * 16;
#pragma unroll 4
  for (int rr = lane >> 4; rr < kTcKv; rr += 2) {
    const char* src = pool;  // any valid address when zero-filling
    bool valid = rr < hist_rows;
    if (valid) {
      uint32_t bi, off;
      ba.split((uint32_t)(j0 + rr), bi, off);
      const int64_t blk = pages[bi - p0];
      if (blk < 0 || blk >= a.num_blocks) {
        if (unit == 0) record_status(MI_STATUS_BAD_BLOCK);
        valid = false;
      } else {
        src = pool + (blk * a.block_size + off) * pool_row + head_off;
      }
    }
    cp_async16(dst + sw128_offset((uint32_t)rr, (uint32_t)unit, kKvRegion), src, valid);
  }
  __syncwarp();  // `pages` is rewritten for the next tile
}

// cp.async staging of the K or V rows (`chunk` = k_chunk or v_chunk) of chunk tile k = chunk
// tokens [128k, 128k + 128); rows at or past `rows_end` zero.
__device__ __forceinline__ void stage_chunk_cp(const PrefillArgs& a, int64_t b, int h, int64_t first, int k,
                                               int rows_end, const char* chunk, uint32_t dst, int lane) {
  const int unit = lane & 15;
  const char* src = chunk + b * a.kv_sb[0] + (int64_t)h * a.kv_sb[2] + unit * 16;
#pragma unroll 4
  for (int rr = lane >> 4; rr < kTcKv; rr += 2) {
    const int jc = k * kTcKv + rr;
    const bool valid = jc < rows_end;
    cp_async16(dst + sw128_offset((uint32_t)rr, (uint32_t)unit, kKvRegion),
               valid ? src + (first + jc) * a.kv_sb[1] : chunk, valid);
  }
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T, bool kTma>
__global__ void __launch_bounds__(kTcThreads, 1) prefill_tc_kernel(const PrefillArgs a,
                                                                    const __grid_constant__ PrefillMaps maps,
                                                                    float* ws_o, float* ws_ml, int max_splits,
                                                                    int qtiles, int shift) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;                    // loader -> MMA: both Q tiles landed
  uint64_t* k_full = bars + 1;                    // [kStagesK] loader -> MMA: K stage landed
  uint64_t* k_empty = k_full + kStagesK;          // [kStagesK] MMA -> loader: the S of the stage done
  uint64_t* v_full = k_empty + kStagesK;          // [kStagesV] loader -> MMA: V stage landed
  uint64_t* v_empty = v_full + kStagesV;          // [kStagesV] MMA -> loader: the PVs of the stage done
  uint64_t* s_full = v_empty + kStagesV;          // [kPair] MMA -> softmax g: S tile ready
  uint64_t* p_full = s_full + kPair;              // [kPair] softmax g -> MMA: P written into TMEM
  uint64_t* o_done = p_full + kPair;              // [kPair] MMA -> softmax g: one phase per PV
  uint64_t* o_final = o_done + kPair;             // [kPair] MMA -> softmax g: its last PV is done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + kPair);
  int64_t* pages = reinterpret_cast<int64_t*>(smem + kOffPages);  // cp.async loader: block ids of one tile

  const int pair = blockIdx.x / max_splits;
  const int split = blockIdx.x % max_splits;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.groups;
  const int tokens_per_tile = kTcRows / G;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // row tile g of this CTA = q-tile 2*pair + g; both share the row's history and chunk geometry
  int64_t tok0[kPair], tok_end[kPair];
  int n_tiles[kPair], ng[kPair];
  TcGeometry geo{};
#pragma unroll
  for (int g = 0; g < kPair; ++g) {
    tok0[g] = (int64_t)(pair * kPair + g) * tokens_per_tile;
    geo = tc_geometry(a, b, tok0[g], tokens_per_tile, g == 0 && tid == 0 && blockIdx.x == 0 && h == 0);
    n_tiles[g] = geo.n_tiles;
    tok_end[g] = min(geo.len, tok0[g] + tokens_per_tile);
  }
  const TcSplits sp = tc_splits(n_tiles[0], n_tiles[1]);
  const int t_begin = split * sp.per;
#pragma unroll
  for (int g = 0; g < kPair; ++g) ng[g] = max(0, min(n_tiles[g], t_begin + sp.per) - t_begin);  // this split's tiles
  const int64_t first = geo.first;
  const int start = geo.start;
  const int hist_tiles = geo.hist_tiles;
  const int row_elems = a.hq * kTcDim;  // elements per output position
  T* out = reinterpret_cast<T*>(a.out);

  // Padding positions of this KV head's query heads are zeros (written by pair 0, split 0).
  if (blockIdx.x == 0) {
    const int per_pos = G * (kTcDim / 8);
    for (int64_t i = tid; i < first * per_pos; i += kTcThreads) {
      const int64_t p = i / per_pos;
      const int rem = (int)(i - p * per_pos);
      *reinterpret_cast<uint4*>(out + (b * a.padded_len + p) * row_elems + (int64_t)(h * G) * kTcDim + rem * 8) =
          make_uint4(0, 0, 0, 0);
    }
  }
  const int n = max(ng[0], ng[1]);  // tiles staged: the union (a prefix of this split's tiles for each g)
  if (n == 0) return;               // uniform for the CTA
  const int t_end = t_begin + n;

  if (tid == 0) {
    mbar_init(q_full, kTma ? 1 : kLoaderThreads);
    for (int i = 0; i < kStagesK; ++i) {
      mbar_init(&k_full[i], kTma ? 1 : kLoaderThreads);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kStagesV; ++i) {
      mbar_init(&v_full[i], kTma ? 1 : kLoaderThreads);
      mbar_init(&v_empty[i], 1);
    }
    for (int g = 0; g < kPair; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], kSoftmaxThreads);
    }
    for (int g = 0; g < kPair; ++g) {
      mbar_init(&o_done[g], 1);
      mbar_init(&o_final[g], 1);
    }
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool aborted = false;

  if (warp == kLoaderWarp) {
    // ---------------- loader: both Q tiles once, then K and V tiles into their rings --------
    // K(i) reuses the stage of tile i - kStagesK once its S is done, V(i) that of tile i - kStagesV
    // once its PVs are.  Loads go in the order K(0 .. kStagesK-1), then V(i), K(i + kStagesK) for
    // i = 0, 1, ...: the MMA warp issues PV(i - 2) before S(i), so each blocking wait ends in the
    // order the loads are issued.
    if constexpr (kTma) {
      // Block ids of the split's history pages, resolved once: the pool row of each page's first
      // slot, or a row past the pool for a page at or past `start` (TMA fills it with zeros).
      int* page_rows = reinterpret_cast<int*>(pages);
      const int pages_per_tile = kTcKv / a.block_size;
      const int num_slots = (int)(a.num_blocks * a.block_size);
      const int n_pages = max(0, min(t_end, hist_tiles) - t_begin) * pages_per_tile;
      const int64_t* table = a.block_tables + b * a.table_stride;
      for (int j = lane; j < n_pages; j += 32) {
        const int pos0 = t_begin * kTcKv + j * a.block_size;
        int row0 = num_slots;
        if (pos0 < start) {
          const int64_t blk = table[pos0 >> shift];
          if (blk < 0 || blk >= a.num_blocks) record_status(MI_STATUS_BAD_BLOCK);
          else row0 = (int)(blk * a.block_size);
        }
        page_rows[j] = row0;
      }
      __syncwarp();
      // the whole warp runs the issue loop; elected lanes issue the copies
      if (lane == 0) {
        tma_prefetch_desc(&maps.q);
        tma_prefetch_desc(&maps.k_chunk);
        tma_prefetch_desc(&maps.v_chunk);
      }
      __syncwarp();
      mbar_expect_tx_e(q_full, kPair * kQBytes);
      for (int g = 0; g < kPair; ++g)  // box [64 d, G heads, 128/G tokens]: row = token * G + head
        for (int c = 0; c < 2; ++c)
          tma_load_4d_e(smem + kOffQ + g * kQBytes + c * kQRegion, &maps.q, q_full, c * 64, h * G,
                        (int)(first + tok0[g]), (int)b);
      const int page_bytes = a.block_size * 128;
      auto load = [&](int i, bool is_v) {
        const int stages = is_v ? kStagesV : kStagesK;
        const int st = i % stages;
        if (i >= stages) mbar_wait_warp(is_v ? &v_empty[st] : &k_empty[st], ((i / stages) - 1) & 1, aborted);
        uint64_t* full = is_v ? &v_full[st] : &k_full[st];
        uint8_t* dst = smem + (is_v ? kOffV : kOffK) + st * kKvBytes;
        mbar_expect_tx_e(full, kKvBytes);
        const int t = t_begin + i;
        if (t < hist_tiles) {
          const CUtensorMap* map = is_v ? &maps.v_pool : &maps.k_pool;
          for (int pg = 0; pg < pages_per_tile; ++pg) {
            const int row0 = page_rows[i * pages_per_tile + pg];
            for (int c = 0; c < 2; ++c) tma_load_3d_e(dst + c * kKvRegion + pg * page_bytes, map, full, c * 64, h, row0);
          }
        } else {  // boxes of 64 chunk tokens (rows past the chunk read as zeros)
          const CUtensorMap* map = is_v ? &maps.v_chunk : &maps.k_chunk;
          const int pos = (int)first + (t - hist_tiles) * kTcKv;
          for (int sub = 0; sub < kTcKv / 64; ++sub)
            for (int c = 0; c < 2; ++c)
              tma_load_4d_e(dst + c * kKvRegion + sub * 64 * 128, map, full, c * 64, h, pos + sub * 64, (int)b);
        }
      };
      for (int i = 0; i < min(n, kStagesK); ++i) load(i, false);
      for (int i = 0; i < n; ++i) {
        load(i, true);
        if (i + kStagesK < n) load(i + kStagesK, false);
      }
    } else {
      const BlockAddr ba{shift, (uint32_t)a.block_size};
      const int unit = lane & 15;
      for (int g = 0; g < kPair; ++g) {
        for (int r = lane >> 4; r < kTcRows; r += kLoaderThreads / 16) {
          const int64_t tok = tok0[g] + r / G;
          const bool valid = tok < tok_end[g];
          const char* src = a.q;
          if (valid)
            src = a.q + b * a.q_sb[0] + (first + tok) * a.q_sb[1] + (int64_t)(h * G + r % G) * a.q_sb[2] + unit * 16;
          cp_async16(sbase + kOffQ + g * kQBytes + sw128_offset((uint32_t)r, (uint32_t)unit, kQRegion), src, valid);
        }
      }
      cp_async_arrive_noinc(q_full);
      const int rows_end = (int)tok_end[kPair - 1] > (int)tok_end[0] ? (int)tok_end[kPair - 1] : (int)tok_end[0];
      auto load = [&](int i, bool is_v) {
        const int stages = is_v ? kStagesV : kStagesK;
        const int st = i % stages;
        if (i >= stages) mbar_wait(is_v ? &v_empty[st] : &k_empty[st], ((i / stages) - 1) & 1, aborted);
        const int t = t_begin + i;
        const uint32_t dst = sbase + (is_v ? kOffV : kOffK) + st * kKvBytes;
        if (t < hist_tiles) stage_hist_cp<T>(a, ba, b, h, start, t, is_v ? a.v_pool : a.k_pool, dst, lane, pages);
        else stage_chunk_cp(a, b, h, first, t - hist_tiles, rows_end, is_v ? a.v_chunk : a.k_chunk, dst, lane);
        cp_async_arrive_noinc(is_v ? &v_full[st] : &k_full[st]);
      };
      for (int i = 0; i < min(n, kStagesK); ++i) load(i, false);
      for (int i = 0; i < n; ++i) {
        load(i, true);
        if (i + kStagesK < n) load(i + kStagesK, false);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer: the row tiles alternate PV_g(i), S_g(i+1) ----------------
    // The whole warp runs the loop (warp-uniform control flow); elected lanes issue.
    {
      constexpr bool kBf16 = !std::is_same<T, __half>::value;
      const uint32_t idesc_qk = idesc_f16(kBf16, false, kTcRows, kTcKv);
      const uint32_t idesc_pv = idesc_f16(kBf16, true, kTcRows, kTcDim);
      // Shared-memory descriptors: the start-address field holds address >> 4 (14 bits, every
      // address here is below 256 KiB), so the descriptor of base + off is desc(base) + off / 16.
      const uint64_t dq = desc_kmajor(sbase + kOffQ);
      const uint64_t dk = desc_kmajor(sbase + kOffK);
      const uint64_t dv = desc_mnmajor(sbase + kOffV);
      auto issue_s = [&](int g, int i) {  // S_g(i) = Q_g K(i)^T into g's S columns
        const int ks = i % kStagesK;
        fence_async_smem();
        tc_fence_after();
        const uint64_t dks = dk + (uint64_t)(ks * (kKvBytes >> 4));
#pragma unroll
        for (int s = 0; s < kTcDim / 16; ++s)
          umma_f16(tmem + g * 128, dq + (uint64_t)((g * kQBytes + (s >> 2) * kQRegion + (s & 3) * 32) >> 4),
                   dks + (uint64_t)(((s >> 2) * kKvRegion + (s & 3) * 32) >> 4), idesc_qk, s > 0 ? 1u : 0u);
        umma_commit(&s_full[g]);
        // K(i) is free once every row tile that uses tile i has issued its S (row tile 1 issues last)
        if (g == kPair - 1 || i >= ng[kPair - 1]) umma_commit(&k_empty[ks]);
      };
      auto issue_pv = [&](int g, int i) {  // O_g += P_g(i) V(i)
        const int vs = i % kStagesV;
        tc_fence_after();
        const uint64_t dvs = dv + (uint64_t)(vs * (kKvBytes >> 4));
#pragma unroll
        for (int s = 0; s < kTcKv / 16; ++s)  // P: 16-bit pairs in the first 64 of g's S columns
          umma_f16_tmem_a(tmem + kTmemO + g * 128, tmem + g * 128 + s * 8, dvs + (uint64_t)((s * 2048) >> 4),
                          idesc_pv, (i > 0 || s > 0) ? 1u : 0u);
        umma_commit(&o_done[g]);
        if (g == kPair - 1 || i >= ng[kPair - 1]) umma_commit(&v_empty[vs]);
        if (i + 1 == ng[g]) umma_commit(&o_final[g]);
      };
      // S_g(i+1) overwrites P_g(i) in g's S columns, so it follows PV_g(i); the waits suspend the
      // warp instead of spinning.
      mbar_wait_warp(q_full, 0, aborted);
      mbar_wait_warp(&k_full[0], 0, aborted);
#pragma unroll
      for (int g = 0; g < kPair; ++g)
        if (ng[g] > 0) issue_s(g, 0);
      for (int i = 0; i < n; ++i) {
#pragma unroll
        for (int g = 0; g < kPair; ++g) {
          if (i >= ng[g]) continue;
          mbar_wait_warp(&p_full[g], i & 1, aborted);
          mbar_wait_warp(&v_full[i % kStagesV], (i / kStagesV) & 1, aborted);
          issue_pv(g, i);
          if (i + 1 < ng[g]) {
            mbar_wait_warp(&k_full[(i + 1) % kStagesK], ((i + 1) / kStagesK) & 1, aborted);
            issue_s(g, i + 1);
          }
        }
      }
    }
  } else {
    // ---------------- softmax warpgroup g: thread <-> row <-> TMEM lane ----------------
    const int g = (warp - 2) / 4;
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;            // row of the tile
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int64_t my_tok0 = g == 0 ? tok0[0] : tok0[1];
    const int64_t my_tok = my_tok0 + r / G;
    const bool row_valid = my_tok < (g == 0 ? tok_end[0] : tok_end[1]);
    const int my_n = g == 0 ? ng[0] : ng[1];
    const int my_splits = g == 0 ? sp.splits[0] : sp.splits[1];
    const uint32_t s_col = (uint32_t)g * 128;
    const uint32_t o_col = kTmemO + (uint32_t)g * 128;
    const float scale = a.scale_log2;
    float m_ref = -INFINITY, l_run = 0.f;
    for (int i = 0; i < my_n; ++i) {
      const int t = t_begin + i;
      // visible columns of this tile: history keys below `start`; chunk keys up to the row's token
      bool full;
      int lim;
      if (t < hist_tiles) {
        lim = row_valid ? start - t * kTcKv : 0;
        full = (t + 1) * kTcKv <= start;
      } else {
        const int k0 = (t - hist_tiles) * kTcKv;
        lim = row_valid ? (int)my_tok + 1 - k0 : 0;
        full = k0 + kTcKv <= (int)my_tok0 + 1;
      }
      mbar_wait(&s_full[g], i & 1, aborted);
      tc_fence_after();
      const uint32_t s_addr = tmem + s_col + lane_base;
      uint32_t sr[kTcKv / 32][32];
#pragma unroll
      for (int c = 0; c < kTcKv / 32; ++c) tmem_ld32_async(s_addr + c * 32, sr[c]);
      tmem_wait_ld();
      if (!full) {  // uniform for the warpgroup: only tiles that cross a causal or history end are masked
#pragma unroll
        for (int c = 0; c < kTcKv / 32; ++c) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= lim) sr[c][e] = 0xff800000u;  // -inf: exp2 gives 0 below
        }
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kTcKv / 32; ++c) {
#pragma unroll
        for (int e = 0; e < 32; ++e) mx[e & 3] = fmaxf(mx[e & 3], __uint_as_float(sr[c][e]));
      }
      const float tile_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale;
      const float m_new = fmaxf(m_ref, tile_max);
      const bool need = i > 0 && m_ref != -INFINITY && m_new > m_ref + kRescaleLog2;
      const float alpha = need ? fast_exp2(m_ref - m_new) : 1.f;
      if (need) {
        l_run *= alpha;
        m_ref = m_new;
      } else if (m_ref == -INFINITY) {
        m_ref = m_new;
      }
      const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;  // a row with nothing visible yet: all -inf
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
      // P as the A operand of PV: 16-bit pairs over the first 64 S columns, 32 scores (16
      // columns) per store; every S value is in registers before the first store.
#pragma unroll
      for (int c = 0; c < kTcKv / 32; ++c) {
        uint32_t pw[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          // branch-free: every exponent is independent, so the ex2 issue overlaps
          const float p0 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * j]), scale, neg_m));
          const float p1 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * j + 1]), scale, neg_m));
          ps[j & 3] += p0 + p1;
          pw[j] = pack2<T>(p0, p1);
        }
        tmem_st16_async(s_addr + c * 16, pw);
      }
      l_run += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      // The running O is rescaled after P is out of registers; PV(i) waits for both.
      if (__any_sync(0xffffffffu, need)) {  // warp-collective TMEM access
        mbar_wait(&o_done[g], (i - 1) & 1, aborted);  // PV(i-1) of this row tile finished writing O
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tmem + o_col + lane_base + c * 32, ov);
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] *= alpha;
          tmem_st32(tmem + o_col + lane_base + c * 32, ov);
        }
      }
      tmem_wait_st();
      tc_fence_before();  // our tcgen05.ld of S / st of P and O before the next MMAs
      mbar_arrive(&p_full[g]);
    }
    // ---- epilogue (a row tile without tiles in this split writes nothing here) ----
    if (my_n > 0) {
      mbar_wait(&o_final[g], 0, aborted);
      tc_fence_after();
      if (my_splits == 1) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        T* dst = out + (b * a.padded_len + first + my_tok) * row_elems + (int64_t)(h * G + r % G) * kTcDim;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tmem + o_col + lane_base + c * 32, ov);
          if (row_valid) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint4 pk;
              pk.x = pack2<T>(ov[u * 8 + 0] * inv, ov[u * 8 + 1] * inv);
              pk.y = pack2<T>(ov[u * 8 + 2] * inv, ov[u * 8 + 3] * inv);
              pk.z = pack2<T>(ov[u * 8 + 4] * inv, ov[u * 8 + 5] * inv);
              pk.w = pack2<T>(ov[u * 8 + 6] * inv, ov[u * 8 + 7] * inv);
              *reinterpret_cast<uint4*>(dst + c * 32 + u * 8) = pk;
            }
          }
        }
      } else {
        const int qt = pair * kPair + g;
        const int64_t part = (b * a.hkv + h) * ((int64_t)qtiles * max_splits) + (int64_t)qt * max_splits + split;
        float* po = ws_o + (part * kTcRows + r) * kTcDim;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tmem + o_col + lane_base + c * 32, ov);
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(po + c * 32 + u * 4) =
                make_float4(ov[u * 4], ov[u * 4 + 1], ov[u * 4 + 2], ov[u * 4 + 3]);
        }
        *reinterpret_cast<float2*>(ws_ml + (part * kTcRows + r) * 2) = make_float2(m_ref, l_run);
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Merge the split partials of row tiles that needed more than one split.  A CTA takes one group
// of kCombineRows rows of a row tile; each thread merges (row, 16-byte column chunk) items in one
// online pass over the splits (running max, rescaled sums), so the loads of every split are
// independent of each other and a warp reads 512 contiguous bytes of one row per split.
constexpr int kCombineThreads = 128;
constexpr int kCombineRows = 16;

template <typename T>
__global__ void __launch_bounds__(kCombineThreads) prefill_combine_kernel(const PrefillArgs a, const float* ws_o,
                                                                          const float* ws_ml, int max_splits) {
  constexpr int kGroups = kTcRows / kCombineRows;
  const int qtile = blockIdx.x / kGroups;
  const int r0 = (blockIdx.x % kGroups) * kCombineRows;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.groups;
  const int tokens_per_tile = kTcRows / G;
  const int64_t tok0 = (int64_t)qtile * tokens_per_tile;
  const TcGeometry geo = tc_geometry(a, b, tok0, tokens_per_tile, false);
  // the split layout of this tile's pair (as the tc kernel cut it)
  const int pair_first = qtile - qtile % kPair;
  const int64_t other_tok0 = (int64_t)(pair_first + (qtile == pair_first ? 1 : 0)) * tokens_per_tile;
  const int other_tiles = tc_geometry(a, b, other_tok0, tokens_per_tile, false).n_tiles;
  const TcSplits sp = qtile == pair_first ? tc_splits(geo.n_tiles, other_tiles) : tc_splits(other_tiles, geo.n_tiles);
  const int n_splits = sp.splits[qtile == pair_first ? 0 : 1];
  if (n_splits <= 1) return;  // uniform for the CTA
  const int64_t tok_end = min(geo.len, tok0 + tokens_per_tile);
  const int rows = (int)min((int64_t)kTcRows, (tok_end - tok0) * G);  // valid rows: a prefix of the tile
  // partial (split s, row r) lives at row (part0 + s) * kTcRows + r
  const int64_t part0 = (b * a.hkv + h) * ((int64_t)(gridDim.x / kGroups) * max_splits) + (int64_t)qtile * max_splits;
  T* out = reinterpret_cast<T*>(a.out);
  constexpr int kChunks = kTcDim / 4;  // float4 chunks of a row
  for (int item = threadIdx.x; item < kCombineRows * kChunks; item += kCombineThreads) {
    const int r = r0 + item / kChunks;
    const int c = item % kChunks;
    if (r >= rows) break;  // items are row-major: the rest of this thread's items are past the end too
    float m = -INFINITY, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int sp = 0; sp < n_splits; ++sp) {
      const int64_t row = (part0 + sp) * kTcRows + r;
      const float2 ml = *reinterpret_cast<const float2*>(ws_ml + row * 2);
      const float4 o = *reinterpret_cast<const float4*>(ws_o + row * kTcDim + c * 4);
      if (ml.x == -INFINITY) continue;  // an empty split contributes nothing
      const float m_new = fmaxf(m, ml.x);
      const float alpha = exp2f(m - m_new);  // 0 on the first contribution (m = -inf)
      const float w = exp2f(ml.x - m_new);
      l = l * alpha + w * ml.y;
      acc.x = acc.x * alpha + w * o.x;
      acc.y = acc.y * alpha + w * o.y;
      acc.z = acc.z * alpha + w * o.z;
      acc.w = acc.w * alpha + w * o.w;
      m = m_new;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t tok = tok0 + r / G;
    T* dst = out + (b * a.padded_len + geo.first + tok) * (int64_t)(a.hq * kTcDim) +
             (int64_t)(h * G + r % G) * kTcDim + c * 4;
    uint2 pk;
    pk.x = pack2<T>(acc.x * inv, acc.y * inv);
    pk.y = pack2<T>(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(dst) = pk;
  }
}

struct TcPlan {
  int64_t qtiles;
  int max_splits;
  size_t ws_o_bytes, ws_ml_bytes;
};

TcPlan tc_plan(const PrefillArgs& a) {
  TcPlan p;
  const int tokens_per_tile = kTcRows / a.groups;
  p.qtiles = (a.padded_len + tokens_per_tile - 1) / tokens_per_tile;
  const int64_t max_tiles = (a.table_stride * a.block_size + kTcKv - 1) / kTcKv + (a.padded_len + kTcKv - 1) / kTcKv;
  p.max_splits = (int)std::max<int64_t>(1, (max_tiles + kTilesPerSplit - 1) / kTilesPerSplit);
  const int64_t parts = p.max_splits > 1 ? a.batch * a.hkv * p.qtiles * p.max_splits : 0;
  p.ws_o_bytes = (size_t)parts * kTcRows * kTcDim * sizeof(float);
  p.ws_ml_bytes = (size_t)parts * kTcRows * 2 * sizeof(float);
  return p;
}

int log2_if_pow2(int x) {
  if (x <= 0 || (x & (x - 1))) return -1;
  int s = 0;
  while ((1 << s) < x) ++s;
  return s;
}

template <typename T, bool kTma>
cudaError_t launch_tc(const PrefillArgs& a, float* ws, const PrefillMaps& maps, cudaStream_t s) {
  auto kern = prefill_tc_kernel<T, kTma>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes);
  if (e != cudaSuccess) return e;
  const TcPlan p = tc_plan(a);
  float* ws_o = ws;
  float* ws_ml = ws ? reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + ((p.ws_o_bytes + 255) & ~size_t(255)))
                    : nullptr;
  const int64_t pairs = (p.qtiles + kPair - 1) / kPair;
  dim3 grid((unsigned)(pairs * p.max_splits), (unsigned)a.hkv, (unsigned)a.batch);
  kern<<<grid, kTcThreads, kTcSmemBytes, s>>>(a, maps, ws_o, ws_ml, p.max_splits, (int)p.qtiles,
                                              log2_if_pow2(a.block_size));
  e = cudaGetLastError();
  if (e != cudaSuccess || p.max_splits == 1) return e;
  dim3 cgrid((unsigned)(p.qtiles * (kTcRows / kCombineRows)), (unsigned)a.hkv, (unsigned)a.batch);
  prefill_combine_kernel<T><<<cgrid, kCombineThreads, 0, s>>>(a, ws_o, ws_ml, p.max_splits);
  return cudaGetLastError();
}

}  // namespace

size_t prefill_tc_workspace_bytes(const PrefillArgs& a) {
  const TcPlan p = tc_plan(a);
  if (p.max_splits == 1) return 0;
  return ((p.ws_o_bytes + 255) & ~size_t(255)) + ((p.ws_ml_bytes + 255) & ~size_t(255));
}

bool prefill_tc_supported(const PrefillArgs& a, int dtype) {
  if (dtype != MI_BF16 && dtype != MI_F16) return false;
  if (a.head_dim != kTcDim) return false;
  if (!(a.groups == 1 || a.groups == 2 || a.groups == 4 || a.groups == 8)) return false;
  if (a.batch > 65535 || a.hkv > 65535) return false;
  if (a.table_stride * a.block_size + a.padded_len >= (int64_t(1) << 30)) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a.q) || !al16(a.k_chunk) || !al16(a.v_chunk) || !al16(a.out)) return false;
  if (a.table_stride > 0 && (!al16(a.k_pool) || !al16(a.v_pool))) return false;
  for (int i = 0; i < 3; ++i)
    if ((a.q_sb[i] & 15) || (a.kv_sb[i] & 15)) return false;
  return true;
}

bool prefill_tc_tma_block_size(int block_size) {
  return block_size == 16 || block_size == 32 || block_size == 64;
}

cudaError_t launch_paged_prefill_tc(const PrefillArgs& a, float* ws, const PrefillMaps* maps, int dtype,
                                    cudaStream_t s) {
  static const PrefillMaps kNoMaps{};
  if (maps) {
    if (dtype == MI_BF16) return launch_tc<__nv_bfloat16, true>(a, ws, *maps, s);
    return launch_tc<__half, true>(a, ws, *maps, s);
  }
  if (dtype == MI_BF16) return launch_tc<__nv_bfloat16, false>(a, ws, kNoMaps, s);
  return launch_tc<__half, false>(a, ws, kNoMaps, s);
}

}  // namespace mi
