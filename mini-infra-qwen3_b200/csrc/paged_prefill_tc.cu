// Chunked-prefill paged attention on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Variant: bf16 / fp16, head_dim 128, any block size, G = Hq/H_kv in {1, 2, 4, 8}.
// Persistent CTAs (352 threads, one per SM) share the work as equal ranges of per-KV-head streams
// of KV tiles, each unit start weighted as kUnitCost extra tiles (see TcWalker below).  A unit of a
// stream is one (sequence, pair of tiles of 128 query rows, KV head): a row tile packs 128/G chunk tokens x the G query heads of the KV head (row
// r = token r/G, head r%G); the unit's two row tiles are consecutive, so every K/V tile staged in
// shared memory serves 2 x 128 query rows of the whole GQA group (half the L2 -> SM bytes per
// FLOP of one row tile per CTA).  The KV range of a row tile is its history tiles, then its causal
// chunk tiles; the two row tiles' ranges differ only in their last chunk tiles, so the CTA stages
// the union and each row tile uses a prefix of it.  A unit inside one CTA's range writes its
// output directly; a unit cut by CTA boundaries leaves unnormalised partials (O, m, l) that
// prefill_combine_kernel merges.  Warp roles, linked by mbarriers:
//   warp 0 (loader): per unit both Q tiles, then K tiles into a kStagesK-deep ring, and warp 10
//      V tiles into a kStagesV-deep ring (K is free once the S of both row tiles is done, V once
//      both PVs are).  With tensor maps (block size 16/32/64) each loader reads the block ids of
//      its next tile's pages one tile ahead and issues the tile as one TMA box per lane: one 3D
//      box per pool page and 64-column half of a history tile (a page past `start` reads rows
//      past the pool, which TMA fills with zeros), 4D boxes of 64 tokens for a chunk tile;
//      otherwise warp 0 stages K and V rows with cp.async;
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
//      them: tcgen05.mma of one thread run in issue order).  P is released in two halves: keys
//      0-63 (p_half) once stored, so the first half of PV_g(i) runs under the softmax's second
//      half, and all 128 keys (p_full); a warp that rescales O releases its first half only
//      after the rescale.
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
constexpr int kTcThreads = 96 + kPair * kSoftmaxThreads;  // warp 0 K loader, warp 1 MMA, the warpgroups, V loader
constexpr int kVLoaderWarp = 2 + 2 * kPair * kSoftmaxThreads / 64;
constexpr int kFirstSoftmaxWarp = 2;
constexpr int kLoaderWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kLoaderThreads = 32;
constexpr int kStagesK = 2;                         // depth of the K ring (3 measured slower)
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
constexpr int kTcSmemBytes = kOffPages + (kTcKv + 1) * 8 + 1024;  // + alignment slack (~194 KiB: one CTA per SM)
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
// The tcgen05 issue helpers below are executed by a whole converged warp (so their operands
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
struct TcRow {  // one sequence: chunk placement and history length, clamped to the arguments
  int len, first;  // positions are below 2^30 (prefill_tc_supported)
  int start;
  int hist_tiles;  // ceil(start / kTcKv)
};

__device__ __forceinline__ TcRow tc_row(const PrefillArgs& a, int64_t b, bool report) {
  TcRow g;
  int64_t len = a.chunk_lens[b];
  if (len > a.padded_len) {
    if (report) record_status(MI_STATUS_BAD_LENGTH);
    len = a.padded_len;
  }
  g.len = len < 0 ? 0 : (int)len;
  g.first = (int)a.padded_len - g.len;
  int64_t start = a.starts[b];
  if (start < 0) start = 0;
  if (start > a.table_stride * a.block_size) {
    if (report) record_status(MI_STATUS_BAD_LENGTH);
    start = a.table_stride * a.block_size;
  }
  g.start = (int)start;
  g.hist_tiles = (int)((start + kTcKv - 1) / kTcKv);
  return g;
}

// Work distribution ("stream-K" per KV head).  A unit of work is (sequence b, row-tile pair p) of
// one KV head; its KV tiles are the union of the two row tiles' ranges (history tiles, then chunk
// tiles up to the causal end of the row tile's last token; the second row tile's range is never
// shorter unless it is empty), the same for every head.  The units u = b * pairs + p of a head
// laid end to end form a stream of T cost units (a unit's tiles plus kUnitCost for starting it,
// TcWalker); the grid is R CTAs per head, CTA c = r * hkv + h, and with R' = min(R, T) the CTA
// takes positions [r*T/R', (r+1)*T/R') of head h's stream, walking them
// unit after unit with its K/V rings, TMEM and barrier phases carried across unit boundaries.  The
// hkv CTAs of one r read the same pool pages at the same time (the heads of a page row are
// adjacent in memory).  A unit inside one CTA's range writes its output directly; a unit cut by
// CTA boundaries leaves one unnormalised partial (O, m, l) per piece -- the piece that opens the
// unit (CTA r0) in slot 2*c(r0) + 1, the piece in CTA r (r0 < r <= r1) in slot 2*c(r) -- and CTA
// r0 records the unit in its descriptor for prefill_combine_kernel.
struct TcPair {  // one (sequence, row-tile pair)
  int b;
  int pair;
  TcRow row;
  int tok0[kPair], tok_end[kPair];  // chunk tokens of each row tile
  int n_tiles[kPair];
  int n;  // union of the two ranges
};

__device__ __forceinline__ TcPair tc_pair(const PrefillArgs& a, int rp, int pairs) {
  TcPair u;
  u.b = rp / pairs;
  u.pair = rp - u.b * pairs;
  u.row = tc_row(a, u.b, false);
  const int tpt = kTcRows / a.groups;
#pragma unroll
  for (int g = 0; g < kPair; ++g) {
    u.tok0[g] = (u.pair * kPair + g) * tpt;
    u.tok_end[g] = min(u.row.len, u.tok0[g] + tpt);
    u.n_tiles[g] = u.tok0[g] < u.row.len ? u.row.hist_tiles + (int)((u.tok_end[g] + kTcKv - 1) / kTcKv) : 0;
  }
  u.n = max(u.n_tiles[0], u.n_tiles[1]);
  return u;
}

struct TcItem {  // one piece of a unit inside one CTA's range
  TcPair u;
  int h;
  int t_begin;     // first tile of the piece within the unit
  int n;           // tiles of the piece
  int ng[kPair];   // tiles of row tile g in the piece: [t_begin, t_begin + ng[g])
  int slot;        // partial slot, or -1 when the piece is the whole unit
};

// Positions in a head's stream are in cost units: a unit of n tiles costs kUnitCost + n, its
// first kUnitCost units standing for the work of starting a unit (the Q reload and the pipeline
// refill, ~2.5 tiles measured), so ranges holding more unit starts get fewer tiles.
constexpr int kUnitCost = 2;

struct TcWalker {  // position in a head's stream, advanced item by item
  int rp, rows;      // current row-tile pair, number of pairs in the batch (below 2^31: prefill_tc_supported)
  int h, off;        // KV head; cost offset of the position within its unit (tile off - kUnitCost)
  int left;          // cost units left in the CTA's range
  int used;          // cost units consumed so far (the next item's first tile is at range start + used)
  int pairs, cta;
  __device__ __forceinline__ bool next(const PrefillArgs& a, TcItem& it) {
    if (left <= 0) return false;
    it.u = tc_pair(a, rp, pairs);
    if (off < kUnitCost) {  // the unit's start-up cost
      const int skip = min(kUnitCost - off, left);
      off += skip;
      left -= skip;
      used += skip;
      if (left <= 0) return false;  // the range ends before the unit's first tile
    }
    const int t0 = off - kUnitCost;
    it.h = h;
    it.t_begin = t0;
    it.n = min(it.u.n - t0, left);
#pragma unroll
    for (int g = 0; g < kPair; ++g) it.ng[g] = max(0, min(it.u.n_tiles[g] - t0, it.n));
    const bool opened_before = t0 > 0, continues = t0 + it.n < it.u.n;
    it.slot = opened_before ? 2 * cta : (continues ? 2 * cta + 1 : -1);
    left -= it.n;
    off += it.n;
    used += it.n;
    if (off == kUnitCost + it.u.n) {  // on to the next unit with tiles
      off = 0;
      while (left > 0 && ++rp < rows && tc_pair(a, rp, pairs).n == 0) {
      }
    }
    return true;
  }
};

// A tile cursor: the item of the stream position and the tile's index within the item.
struct TcCursor {
  TcWalker w;
  TcItem it;
  int i;
  bool valid;
  __device__ __forceinline__ void init(const TcWalker& w0, const PrefillArgs& a) {
    w = w0;
    i = 0;
    valid = w.next(a, it);
  }
  __device__ __forceinline__ void advance(const PrefillArgs& a) {
    if (++i == it.n) {
      i = 0;
      valid = w.next(a, it);
    }
  }
  __device__ __forceinline__ bool last_of_item() const { return i + 1 == it.n; }
};

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
// 3-input maximum (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// One loader warp's stream of K (or V) tiles over the CTA's items: lanes 0..pages-1 hold the block
// ids of the next tile's pool pages, loaded one tile ahead; a tile goes out as one TMA box per lane
// (page or 64-token sub-tile x 64-column half).
struct KvTileLoader {
  TcCursor c;
  int64_t pend;
  bool pend_valid;
  int lane, shift;
  __device__ __forceinline__ void fetch(const PrefillArgs& a) {
    pend_valid = false;
    const int pages_per_tile = kTcKv / a.block_size;
    if (!c.valid || lane >= pages_per_tile) return;
    const int t = c.it.t_begin + c.i;
    const int pos0 = t * kTcKv + lane * a.block_size;
    if (t < c.it.u.row.hist_tiles && pos0 < c.it.u.row.start) {
      pend = a.block_tables[c.it.u.b * a.table_stride + (pos0 >> shift)];
      pend_valid = true;
    }
  }
  __device__ __forceinline__ void init(const TcWalker& w0, const PrefillArgs& a, int lane_, int shift_) {
    lane = lane_;
    shift = shift_;
    c.init(w0, a);
    fetch(a);
  }
  __device__ __forceinline__ void issue(const PrefillArgs& a, const CUtensorMap& pool_map, const CUtensorMap& chunk_map,
                                        uint8_t* dst, uint64_t* full) {
    const int pages_per_tile = kTcKv / a.block_size;
    int my_row = (int)(a.num_blocks * a.block_size);  // past the pool: TMA reads zeros
    if (lane < pages_per_tile && pend_valid) {
      if (pend < 0 || pend >= a.num_blocks) record_status(MI_STATUS_BAD_BLOCK);
      else my_row = (int)(pend * a.block_size);
    }
    const int t = c.it.t_begin + c.i;
    const bool hist = t < c.it.u.row.hist_tiles;
    const int h = c.it.h;
    const int pos = c.it.u.row.first + (t - c.it.u.row.hist_tiles) * kTcKv;
    const int b = c.it.u.b;
    const int boxes = hist ? 2 * pages_per_tile : 2 * (kTcKv / 64);
    const int q = lane >> 1, cc = lane & 1;
    const int row0 = __shfl_sync(0xffffffffu, my_row, q & 31);
    if (lane == 0) mbar_arrive_expect_tx(full, kKvBytes);
    __syncwarp();
    if (lane < boxes) {
      // History pages go evict-first: at config-4 shapes that keeps the chunk K/V (re-read by
      // the row's other tiles) and the split partials in L2 (111.3 against 113.5 us); the chunk
      // loads stay unhinted, since an evict-first hint there cost ~8% on compute-bound chunks.
      if (hist)
        tma_load_3d_hint(dst + cc * kKvRegion + q * a.block_size * 128, &pool_map, full, cc * 64, h, row0,
                         l2_policy_evict_first());
      else tma_load_4d(dst + cc * kKvRegion + q * 64 * 128, &chunk_map, full, cc * 64, h, pos + q * 64, b);
    }
    c.advance(a);
    fetch(a);
  }
};

// Zeros for the padding positions (left of the chunk) of rows b = blockIdx.x (mod gridDim.x), all
// query heads.
template <typename T>
__device__ __forceinline__ void zero_padding(const PrefillArgs& a, int tid) {
  const int64_t row_elems = (int64_t)a.hq * kTcDim;
  for (int64_t b = blockIdx.x; b < a.batch; b += gridDim.x) {
    const int64_t first = tc_row(a, b, tid == 0).first;
    const int64_t units = first * row_elems * (int64_t)sizeof(T) / 16;  // 16-byte stores
    uint4* dst = reinterpret_cast<uint4*>(a.out + b * a.padded_len * row_elems * (int64_t)sizeof(T));
    for (int64_t i = tid; i < units; i += kTcThreads) dst[i] = make_uint4(0, 0, 0, 0);
  }
}

// Work range of this CTA (all threads): the per-pair costs (tiles + kUnitCost) are summed in
// per-thread chunks of pairs and scanned across the block (`scratch`: 16 int64 of shared memory),
// then the thread whose chunk holds the CTA's first position locates it.  Returns the walker at
// that position, the cost of a head's stream (`total`) and the CTAs per head that share it
// (`ctas`).
__device__ __forceinline__ TcWalker tc_start(const PrefillArgs& a, int pairs, int64_t* scratch, int tid, int64_t& total,
                                             int64_t& ctas) {
  const int warp = tid >> 5, lane = tid & 31;
  const int rows = (int)(a.batch * pairs);
  const int r0 = (int)((int64_t)rows * tid / kTcThreads), r1 = (int)((int64_t)rows * (tid + 1) / kTcThreads);
  int64_t mine = 0;
  for (int rp = r0; rp < r1; ++rp) {
    const int n = tc_pair(a, rp, pairs).n;
    mine += n > 0 ? kUnitCost + n : 0;
  }
  int64_t x = mine;  // inclusive scan within the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  int64_t before = 0;
  total = 0;
  for (int w = 0; w < kTcThreads / 32; ++w) {
    const int64_t v = scratch[w];
    if (w < warp) before += v;
    total += v;
  }
  const int64_t excl = before + x - mine;  // cost units ahead of this thread's chunk
  ctas = min((int64_t)(gridDim.x / a.hkv), total);
  const int64_t c = blockIdx.x / a.hkv;  // range index within the head
  const int64_t x0 = c < ctas ? c * total / ctas : 0;
  const int64_t x1 = c < ctas ? (c + 1) * total / ctas : 0;
  __syncthreads();  // every warp total read before the start is written over them
  if (c < ctas && excl <= x0 && x0 < excl + mine) {
    int64_t pos = excl;
    for (int rp = r0; rp < r1; ++rp) {
      const int n = tc_pair(a, rp, pairs).n;
      const int cost = n > 0 ? kUnitCost + n : 0;
      if (x0 < pos + cost) {
        scratch[0] = rp;
        scratch[1] = x0 - pos;
        break;
      }
      pos += cost;
    }
  }
  __syncthreads();
  TcWalker w;
  w.rows = rows;
  w.pairs = pairs;
  w.cta = (int)blockIdx.x;
  w.left = (int)(x1 - x0);
  w.used = 0;
  w.rp = w.left > 0 ? (int)scratch[0] : 0;
  w.h = (int)(blockIdx.x % a.hkv);
  w.off = w.left > 0 ? (int)scratch[1] : 0;
  return w;
}

template <typename T, bool kTma>
__global__ void __launch_bounds__(kTcThreads, 1) prefill_tc_kernel(const PrefillArgs a,
                                                                    const __grid_constant__ PrefillMaps maps,
                                                                    float* ws_o, float* ws_ml, int64_t* ws_desc,
                                                                    int pairs, int shift) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;                    // loader -> MMA: both Q tiles of the item landed
  uint64_t* k_full = bars + 1;                    // [kStagesK] loader -> MMA: K stage landed
  uint64_t* k_empty = k_full + kStagesK;          // [kStagesK] MMA -> loader: the S of the stage done
  uint64_t* v_full = k_empty + kStagesK;          // [kStagesV] loader -> MMA: V stage landed
  uint64_t* v_empty = v_full + kStagesV;          // [kStagesV] MMA -> loader: the PVs of the stage done
  uint64_t* s_full = v_empty + kStagesV;          // [kPair] MMA -> softmax g: S tile ready
  uint64_t* p_full = s_full + kPair;              // [kPair] softmax g -> MMA: all of P written into TMEM
  uint64_t* o_done = p_full + kPair;              // [kPair] MMA -> softmax g: one phase per PV
  uint64_t* o_final = o_done + kPair;             // [kPair] MMA -> softmax g: the item's last PV is done
  uint64_t* o_free = o_final + kPair;             // [kPair] softmax g -> MMA: the item's O read out of TMEM
  uint64_t* p_half = o_free + kPair;              // [kPair] softmax g -> MMA: keys 0-63 of P in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_half + kPair);
  int64_t* pages = reinterpret_cast<int64_t*>(smem + kOffPages);  // cp.async: block ids; TMA: page-row ring

  // Launched as a programmatic dependent of the stream's previous kernel (so its CTAs are placed
  // while that kernel drains): nothing is read or written before that kernel has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = a.groups;
  const int row_elems = a.hq * kTcDim;  // elements per output position
  T* out = reinterpret_cast<T*>(a.out);

  zero_padding<T>(a, tid);
  int64_t total, ctas;
  const TcWalker walk0 = tc_start(a, pairs, reinterpret_cast<int64_t*>(smem + kOffK), tid, total, ctas);
  int64_t* const scratch = reinterpret_cast<int64_t*>(smem + kOffK);
  if (tid == 0) {  // the CTA's tiles, and the unit it opens and leaves unfinished (for the combine)
    int64_t d0 = -1, d1 = 0, d2 = 0, tiles = 0;
    TcWalker w = walk0;
    TcItem it;
    const int64_t r = blockIdx.x / a.hkv;
    const int64_t x0 = r * total / max(ctas, (int64_t)1);
    while (w.next(a, it)) {
      tiles += it.n;
      if (it.slot == 2 * (int)blockIdx.x + 1) {  // t_begin == 0: the unit's tiles follow its first one
        const int64_t first = x0 + w.used - it.n;  // cost position of the unit's first tile
        d0 = it.u.b * pairs + it.u.pair;
        d1 = it.h;
        d2 = ((first + it.u.n) * ctas - 1) / total * a.hkv + it.h;  // CTA of the unit's last tile
      }
    }
    ws_desc[blockIdx.x * 4 + 0] = d0;
    ws_desc[blockIdx.x * 4 + 1] = d1;
    ws_desc[blockIdx.x * 4 + 2] = d2;
    scratch[16] = tiles;  // clear of the words the start scan used
  }
  __syncthreads();
  const int64_t n_tiles = scratch[16];
  if (n_tiles == 0) return;  // uniform for the CTA

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
      mbar_init(&o_done[g], 1);
      mbar_init(&o_final[g], 1);
      mbar_init(&o_free[g], kSoftmaxThreads);
      mbar_init(&p_half[g], kSoftmaxThreads);
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

  auto tma_loader_prologue = [&]() {
    if (lane == 0) {
      tma_prefetch_desc(&maps.q);
      tma_prefetch_desc(&maps.k_chunk);
      tma_prefetch_desc(&maps.v_chunk);
      tma_prefetch_desc(&maps.k_pool);
      tma_prefetch_desc(&maps.v_pool);
    }
    __syncwarp();
  };
  if (warp == kVLoaderWarp) {
    if constexpr (kTma) {  // V tiles into the V ring (the cp.async loader stages both K and V)
      tma_loader_prologue();
      KvTileLoader ld;
      ld.init(walk0, a, lane, shift);
      for (int64_t j = 0; j < n_tiles; ++j) {
        if (j >= kStagesV) mbar_wait_warp(&v_empty[j % kStagesV], ((j / kStagesV) - 1) & 1, aborted);
        ld.issue(a, maps.v_pool, maps.v_chunk, smem + kOffV + (int)(j % kStagesV) * kKvBytes, &v_full[j % kStagesV]);
      }
    }
  } else if (warp == kLoaderWarp) {
    // ---------------- loader: per item both Q tiles, then K (and V) tiles into their rings ---------
    // K(j) reuses the stage of tile j - kStagesK once its S is done, V(j) that of tile j - kStagesV
    // once its PVs are (j counts the CTA's tiles across items).  With TMA this warp loads Q and K
    // and kVLoaderWarp loads V, each in tile order; the cp.async loader stages K(0 .. kStagesK-1),
    // V(0), then V(j+1), K(j + kStagesK) for j = 0, 1, ... (the MMA warp issues the PVs of tile j-1
    // before the S of tile j, so each blocking wait ends in the order the loads are issued).  The Q
    // tiles of an item are loaded once every S of the previous item is done (K(j) free, j its last
    // tile).
    if constexpr (kTma) {
      // K loader (this warp: K tiles and the Q tiles of each item); V tiles come from kVLoaderWarp.
      tma_loader_prologue();
      TcCursor cq;  // tile j of the loop below: its item's end gates the next item's Q
      cq.init(walk0, a);
      KvTileLoader ld;
      ld.init(walk0, a, lane, shift);
      auto load_q = [&](const TcItem& it) {
        if (lane == 0) mbar_arrive_expect_tx(q_full, kPair * kQBytes);
        __syncwarp();
        if (lane < 2 * kPair) {  // box [64 d, G heads, 128/G tokens]: row = token * G + head
          const int g = lane >> 1, c = lane & 1;
          const int tok0 = g ? it.u.tok0[1] : it.u.tok0[0];  // a select: no indexing by a lane value
          tma_load_4d(smem + kOffQ + g * kQBytes + c * kQRegion, &maps.q, q_full, c * 64, it.h * G,
                      it.u.row.first + tok0, it.u.b);
        }
      };
      load_q(cq.it);
      for (int64_t j = 0; j < min(n_tiles, (int64_t)kStagesK); ++j)
        ld.issue(a, maps.k_pool, maps.k_chunk, smem + kOffK + (int)(j % kStagesK) * kKvBytes, &k_full[j % kStagesK]);
      for (int64_t j = 0; j < n_tiles; ++j) {
        const bool item_end = cq.last_of_item() && j + 1 < n_tiles;
        cq.advance(a);
        if (item_end || j + kStagesK < n_tiles) mbar_wait_warp(&k_empty[j % kStagesK], (j / kStagesK) & 1, aborted);
        if (item_end) load_q(cq.it);  // every S of the finished item is done
        if (j + kStagesK < n_tiles) {
          const int64_t jk = j + kStagesK;
          ld.issue(a, maps.k_pool, maps.k_chunk, smem + kOffK + (int)(jk % kStagesK) * kKvBytes, &k_full[jk % kStagesK]);
        }
      }
    } else {
      TcCursor ck, cv;  // tiles of the next K load and of the next V load
      ck.init(walk0, a);
      cv.init(walk0, a);
      const BlockAddr ba{shift, (uint32_t)a.block_size};
      const int unit = lane & 15;
      auto load_q = [&](const TcItem& it) {
#pragma unroll
        for (int g = 0; g < kPair; ++g) {
          for (int r = lane >> 4; r < kTcRows; r += kLoaderThreads / 16) {
            const int64_t tok = it.u.tok0[g] + r / G;
            const bool valid = tok < it.u.tok_end[g];
            const char* src = a.q;
            if (valid)
              src = a.q + it.u.b * a.q_sb[0] + (it.u.row.first + tok) * a.q_sb[1] +
                    (int64_t)(it.h * G + r % G) * a.q_sb[2] + unit * 16;
            cp_async16(sbase + kOffQ + g * kQBytes + sw128_offset((uint32_t)r, (uint32_t)unit, kQRegion), src,
                       valid);
          }
        }
        cp_async_arrive_noinc(q_full);
      };
      auto issue_tile = [&](const TcCursor& c, int64_t j, bool is_v) {
        const int stages = is_v ? kStagesV : kStagesK;
        const int st = (int)(j % stages);
        if (j >= stages) mbar_wait(is_v ? &v_empty[st] : &k_empty[st], ((j / stages) - 1) & 1, aborted);
        const TcPair& u = c.it.u;
        const int t = c.it.t_begin + c.i;
        const uint32_t dst = sbase + (is_v ? kOffV : kOffK) + st * kKvBytes;
        const int rows_end = (int)max(u.tok_end[0], u.tok_end[kPair - 1]);
        if (t < u.row.hist_tiles)
          stage_hist_cp<T>(a, ba, u.b, c.it.h, u.row.start, t, is_v ? a.v_pool : a.k_pool, dst, lane, pages);
        else
          stage_chunk_cp(a, u.b, c.it.h, u.row.first, t - u.row.hist_tiles, rows_end, is_v ? a.v_chunk : a.k_chunk,
                         dst, lane);
        cp_async_arrive_noinc(is_v ? &v_full[st] : &k_full[st]);
      };
      int64_t jk = 0;
      load_q(cv.it);
      for (; jk < min(n_tiles, (int64_t)kStagesK); ++jk) {
        issue_tile(ck, jk, false);
        ck.advance(a);
      }
      issue_tile(cv, 0, true);
      cv.advance(a);
      for (int64_t j = 0; j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
          const bool opens = cv.i == 0;
          issue_tile(cv, j + 1, true);
          if (opens) {
            mbar_wait(&k_empty[j % kStagesK], (j / kStagesK) & 1, aborted);
            load_q(cv.it);
          }
          cv.advance(a);
        }
        if (jk < n_tiles) {
          issue_tile(ck, jk, false);
          ++jk;
          ck.advance(a);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer: the row tiles alternate PV_g(i), S_g(i+1) ----------------
    // The whole warp runs the loop (warp-uniform control flow); elected lanes issue.
    constexpr bool kBf16 = !std::is_same<T, __half>::value;
    const uint32_t idesc_qk = idesc_f16(kBf16, false, kTcRows, kTcKv);
    const uint32_t idesc_pv = idesc_f16(kBf16, true, kTcRows, kTcDim);
    // Shared-memory descriptors: the start-address field holds address >> 4 (14 bits, every
    // address here is below 256 KiB), so the descriptor of base + off is desc(base) + off / 16.
    const uint64_t dq = desc_kmajor(sbase + kOffQ);
    const uint64_t dk = desc_kmajor(sbase + kOffK);
    const uint64_t dv = desc_mnmajor(sbase + kOffV);
    TcWalker w = walk0;
    TcItem it;
    int64_t j0 = 0;            // CTA tile index of the item's first tile (ring positions)
    int cnt[kPair] = {0, 0};   // tiles of row tile g so far (phases of s_full, p_half, p_full, o_done)
    int fin[kPair] = {0, 0};   // items with tiles of row tile g so far (phases of o_final, o_free)
    int items = 0;
    while (w.next(a, it)) {
      auto issue_s = [&](int g, int i) {  // S_g(i) = Q_g K(i)^T into g's S columns
        const int ks = (int)((j0 + i) % kStagesK);
        fence_async_smem();
        tc_fence_after();
        const uint64_t dks = dk + (uint64_t)(ks * (kKvBytes >> 4));
#pragma unroll
        for (int s = 0; s < kTcDim / 16; ++s)
          umma_f16(tmem + g * 128, dq + (uint64_t)((g * kQBytes + (s >> 2) * kQRegion + (s & 3) * 32) >> 4),
                   dks + (uint64_t)(((s >> 2) * kKvRegion + (s & 3) * 32) >> 4), idesc_qk, s > 0 ? 1u : 0u);
        umma_commit(&s_full[g]);
        // K(i) is free once every row tile that uses tile i has issued its S (row tile 1 issues last)
        if (g == kPair - 1 || i >= it.ng[kPair - 1]) umma_commit(&k_empty[ks]);
      };
      auto issue_pv_half = [&](int g, int i, int h) {  // O_g += P_g(i) V(i) over keys 64h .. 64h+63
        const int vs = (int)((j0 + i) % kStagesV);
        tc_fence_after();
        const uint64_t dvs = dv + (uint64_t)(vs * (kKvBytes >> 4));
#pragma unroll
        for (int s = h * 4; s < h * 4 + 4; ++s)  // P: 16-bit pairs in the first 64 of g's S columns
          umma_f16_tmem_a(tmem + kTmemO + g * 128, tmem + g * 128 + s * 8, dvs + (uint64_t)((s * 2048) >> 4),
                          idesc_pv, (i > 0 || s > 0) ? 1u : 0u);
      };
      auto issue_pv = [&](int g, int i) {  // the second half of PV_g(i), then its commits
        const int vs = (int)((j0 + i) % kStagesV);
        issue_pv_half(g, i, 1);
        umma_commit(&o_done[g]);
        if (g == kPair - 1 || i >= it.ng[kPair - 1]) umma_commit(&v_empty[vs]);
        if (i + 1 == it.ng[g]) umma_commit(&o_final[g]);
      };
      // S_g(i+1) overwrites P_g(i) in g's S columns, so it follows PV_g(i); PV_g(i) is issued in
      // two halves, keys 0-63 after p_half and keys 64-127 after p_full.  The waits suspend the
      // warp instead of spinning.
      mbar_wait_warp(q_full, items & 1, aborted);
      mbar_wait_warp(&k_full[j0 % kStagesK], (j0 / kStagesK) & 1, aborted);
#pragma unroll
      for (int g = 0; g < kPair; ++g)
        if (it.ng[g] > 0) issue_s(g, 0);
      for (int i = 0; i < it.n; ++i) {
#pragma unroll
        for (int g = 0; g < kPair; ++g) {
          if (i >= it.ng[g]) continue;
          mbar_wait_warp(&p_half[g], (cnt[g] + i) & 1, aborted);
          mbar_wait_warp(&v_full[(j0 + i) % kStagesV], ((j0 + i) / kStagesV) & 1, aborted);
          // the previous item's O of this row tile has been read out before PV overwrites it
          if (i == 0 && fin[g] > 0) mbar_wait_warp(&o_free[g], (fin[g] - 1) & 1, aborted);
          issue_pv_half(g, i, 0);  // under the softmax's second half
          mbar_wait_warp(&p_full[g], (cnt[g] + i) & 1, aborted);
          issue_pv(g, i);
          if (i + 1 < it.ng[g]) {
            mbar_wait_warp(&k_full[(j0 + i + 1) % kStagesK], ((j0 + i + 1) / kStagesK) & 1, aborted);
            issue_s(g, i + 1);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kPair; ++g) {
        cnt[g] += it.ng[g];
        fin[g] += it.ng[g] > 0 ? 1 : 0;
      }
      j0 += it.n;
      ++items;
    }
  } else {
    // ---------------- softmax warpgroup g: thread <-> row <-> TMEM lane ----------------
    const int g = (warp - kFirstSoftmaxWarp) / 4;
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;            // row of the tile
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t s_col = (uint32_t)g * 128;
    const uint32_t o_col = kTmemO + (uint32_t)g * 128;
    const float scale = a.scale_log2;
    TcWalker w = walk0;
    TcItem it;
    int cnt = 0, fin = 0;  // tiles and items of this row tile so far (barrier phases)
    while (w.next(a, it)) {
      const TcPair& u = it.u;
      // selects, not indexing by the warp-dependent g (which would put the item in local memory)
      const int my_n = g ? it.ng[1] : it.ng[0];
      const int64_t my_tok0 = g ? u.tok0[1] : u.tok0[0];
      const int64_t my_tok = my_tok0 + r / G;
      const bool row_valid = my_tok < (g ? u.tok_end[1] : u.tok_end[0]);
      const int start = u.row.start;
      const int hist_tiles = u.row.hist_tiles;
      float m_ref = -INFINITY, l_run = 0.f;
      for (int i = 0; i < my_n; ++i) {
        const int t = it.t_begin + i;
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
        mbar_wait(&s_full[g], (cnt + i) & 1, aborted);
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
          for (int e = 0; e < 32; e += 2)
            mx[(e >> 1) & 3] = fmax3(mx[(e >> 1) & 3], __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
        }
        const float tile_max = fmax3(fmaxf(mx[0], mx[1]), mx[2], mx[3]) * scale;
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
        // A warp that rescales O releases its half of P only after the rescale (PV must not add
        // into O before it); the others release keys 0-63 as soon as they are stored.
        const bool warp_need = __any_sync(0xffffffffu, need);
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
          if (c == 1 && !warp_need) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_half[g]);
          }
        }
        l_run += (ps[0] + ps[1]) + (ps[2] + ps[3]);
        // The running O is rescaled after P is out of registers; PV(i) waits for both.
        if (warp_need) {  // warp-collective TMEM access
          mbar_wait(&o_done[g], (cnt + i - 1) & 1, aborted);  // PV(i-1) of this row tile finished writing O
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
        if (warp_need) mbar_arrive(&p_half[g]);
        mbar_arrive(&p_full[g]);
      }
      cnt += my_n;
      // ---- epilogue of the item: O out of TMEM (then free for the next item), then global stores
      if (my_n > 0) {
        mbar_wait(&o_final[g], fin & 1, aborted);
        tc_fence_after();
        ++fin;
        // O 32 columns at a time; TMEM is handed back once the last columns are loaded
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        T* dst = out + (u.b * a.padded_len + u.row.first + my_tok) * row_elems + (int64_t)(it.h * G + r % G) * kTcDim;
        const int64_t part = (int64_t)it.slot * kPair + g;
        float* po = ws_o + (part * kTcRows + r) * kTcDim;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32_async(tmem + o_col + lane_base + c * 32, ov);
          tmem_wait_ld();
          if (c == 3) {
            tc_fence_before();
            mbar_arrive(&o_free[g]);
          }
          if (it.slot < 0) {
            if (row_valid) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const uint32_t* f = &ov[v * 8];
                uint4 pk;
                pk.x = pack2<T>(__uint_as_float(f[0]) * inv, __uint_as_float(f[1]) * inv);
                pk.y = pack2<T>(__uint_as_float(f[2]) * inv, __uint_as_float(f[3]) * inv);
                pk.z = pack2<T>(__uint_as_float(f[4]) * inv, __uint_as_float(f[5]) * inv);
                pk.w = pack2<T>(__uint_as_float(f[6]) * inv, __uint_as_float(f[7]) * inv);
                *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = pk;
              }
            }
          } else {
#pragma unroll
            for (int v = 0; v < 8; ++v)
              *reinterpret_cast<uint4*>(po + c * 32 + v * 4) = make_uint4(ov[v * 4], ov[v * 4 + 1], ov[v * 4 + 2], ov[v * 4 + 3]);
          }
        }
        if (it.slot >= 0) *reinterpret_cast<float2*>(ws_ml + (part * kTcRows + r) * 2) = make_float2(m_ref, l_run);
      } else if (it.slot >= 0) {  // no tiles of this row tile in the piece: an empty partial
        *reinterpret_cast<float2*>(ws_ml + (((int64_t)it.slot * kPair + g) * kTcRows + r) * 2) =
            make_float2(-INFINITY, 0.f);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Merge the pieces of units cut by CTA boundaries.  CTA (c, g, row group) reads CTA c's
// descriptor (the unit c opened and left unfinished, and the last CTA c1 of the same head holding
// a piece of it) and merges row tile g's rows [8 * group, 8 * group + 8) over the pieces in
// slots 2c + 1 and 2c' (c' = c + hkv, c + 2 hkv, ..., c1); each thread merges (row, 16-byte column chunk) items in one online pass
// (running max, rescaled sums), so a warp reads 512 contiguous bytes of one row per piece.
constexpr int kCombineThreads = 128;
constexpr int kCombineRows = 8;

template <typename T>
__global__ void __launch_bounds__(kCombineThreads) prefill_combine_kernel(const PrefillArgs a, const float* ws_o,
                                                                          const float* ws_ml,
                                                                          const int64_t* ws_desc, int pairs) {
  // Launched as a programmatic dependent of the tc kernel: the CTAs start while it drains and
  // wait here for its completion (partials and descriptors written and visible).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int c = blockIdx.x;
  const int g = blockIdx.y;
  const int r0 = blockIdx.z * kCombineRows;
  const int64_t rp = ws_desc[c * 4 + 0];
  if (rp < 0) return;  // uniform for the CTA
  const int h = (int)ws_desc[c * 4 + 1];
  const int c1 = (int)ws_desc[c * 4 + 2];
  const TcPair u = tc_pair(a, (int)rp, pairs);
  const int G = a.groups;
  const int rows = max(0, min(kTcRows, (u.tok_end[g] - u.tok0[g]) * G));  // valid rows
  T* out = reinterpret_cast<T*>(a.out);
  constexpr int kChunks = kTcDim / 4;  // float4 chunks of a row
  for (int item = threadIdx.x; item < kCombineRows * kChunks; item += kCombineThreads) {
    const int r = r0 + item / kChunks;
    const int cc = item % kChunks;
    if (r >= rows) break;  // items are row-major: the rest of this thread's items are past the end too
    float m = -INFINITY, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int p = c; p <= c1; p += a.hkv) {
      const int64_t slot = p == c ? 2 * (int64_t)c + 1 : 2 * (int64_t)p;
      const int64_t row = (slot * kPair + g) * kTcRows + r;
      const float2 ml = *reinterpret_cast<const float2*>(ws_ml + row * 2);
      if (ml.x == -INFINITY) continue;  // an empty piece contributes nothing
      const float4 o = *reinterpret_cast<const float4*>(ws_o + row * kTcDim + cc * 4);
      const float m_new = fmaxf(m, ml.x);
      const float alpha = exp2f(m - m_new);  // 0 on the first contribution (m = -inf)
      const float wt = exp2f(ml.x - m_new);
      l = l * alpha + wt * ml.y;
      acc.x = acc.x * alpha + wt * o.x;
      acc.y = acc.y * alpha + wt * o.y;
      acc.z = acc.z * alpha + wt * o.z;
      acc.w = acc.w * alpha + wt * o.w;
      m = m_new;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t tok = u.tok0[g] + r / G;
    T* dst = out + (u.b * a.padded_len + u.row.first + tok) * (int64_t)(a.hq * kTcDim) +
             (int64_t)(h * G + r % G) * kTcDim + cc * 4;
    uint2 pk;
    pk.x = pack2<T>(acc.x * inv, acc.y * inv);
    pk.y = pack2<T>(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(dst) = pk;
  }
}

// Workspace: partial O [2 * kMaxCtas slots][kPair][128 rows][128] fp32, then (m, l) per row, then
// one descriptor (4 int64) per CTA.
constexpr int kMaxCtas = 148;  // persistent CTAs: one per SM of a B200
constexpr size_t kWsOBytes = (size_t)2 * kMaxCtas * kPair * kTcRows * kTcDim * sizeof(float);
constexpr size_t kWsMlBytes = (size_t)2 * kMaxCtas * kPair * kTcRows * 2 * sizeof(float);
constexpr size_t kWsDescBytes = (size_t)kMaxCtas * 4 * sizeof(int64_t);

int log2_if_pow2(int x) {
  if (x <= 0 || (x & (x - 1))) return -1;
  int s = 0;
  while ((1 << s) < x) ++s;
  return s;
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return kMaxCtas;
  return n;
}

template <typename T, bool kTma>
cudaError_t launch_tc(const PrefillArgs& a, float* ws, const PrefillMaps& maps, cudaStream_t s) {
  auto kern = prefill_tc_kernel<T, kTma>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes);
  if (e != cudaSuccess) return e;
  static const int sms = std::min(kMaxCtas, num_sms());
  const int ctas = std::max(1, sms / a.hkv) * a.hkv;  // CTAs per head x heads
  float* ws_o = ws;
  float* ws_ml = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kWsOBytes);
  int64_t* ws_desc = reinterpret_cast<int64_t*>(reinterpret_cast<char*>(ws) + kWsOBytes + kWsMlBytes);
  const int64_t tokens_per_tile = kTcRows / a.groups;
  const int64_t qtiles = (a.padded_len + tokens_per_tile - 1) / tokens_per_tile;
  const int pairs = (int)((qtiles + kPair - 1) / kPair);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = kTcSmemBytes;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a, maps, ws_o, ws_ml, ws_desc, pairs, log2_if_pow2(a.block_size));
  }
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, kPair, kTcRows / kCombineRows);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_combine_kernel<T>, a, static_cast<const float*>(ws_o),
                            static_cast<const float*>(ws_ml), static_cast<const int64_t*>(ws_desc), pairs);
}

}  // namespace

size_t prefill_tc_workspace_bytes(const PrefillArgs& a) {
  (void)a;
  return kWsOBytes + kWsMlBytes + kWsDescBytes;
}

bool prefill_tc_supported(const PrefillArgs& a, int dtype) {
  if (dtype != MI_BF16 && dtype != MI_F16) return false;
  if (a.head_dim != kTcDim) return false;
  if (!(a.groups == 1 || a.groups == 2 || a.groups == 4 || a.groups == 8)) return false;
  if (a.batch > 65535 || a.hkv > kMaxCtas) return false;
  if (a.table_stride * a.block_size + a.padded_len >= (int64_t(1) << 30)) return false;
  {  // the stream of one head (pairs of the batch x their tiles) is counted in 32-bit integers
    const int64_t tpt = kTcRows / a.groups;
    const int64_t pairs = ((a.padded_len + tpt - 1) / tpt + kPair - 1) / kPair;
    const int64_t tiles = (a.table_stride * a.block_size + a.padded_len) / kTcKv + 2 + kUnitCost;
    if (a.batch * pairs * tiles >= (int64_t(1) << 31)) return false;
  }
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
