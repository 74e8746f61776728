// Chunked-prefill paged attention on CTA pairs (tcgen05.mma.cta_group::2), sm_100a.
//
// The same work split as prefill_tc_kernel (persistent owners over per-KV-head streams of units,
// a unit = one sequence's pair of 128-row query tiles of one KV head, pieces of units cut at owner
// boundaries merged by prefill_combine_kernel), but an owner is a cluster of two CTAs on two SMs:
// the unit's row tile g lives in CTA g.  The leader (rank 0) issues M = 256 MMAs that cover both
// row tiles: each SM's tensor core computes its CTA's 128 rows from its own shared memory and TMEM.
//   * staging: each CTA stages its own Q tile, HALF of every K tile (its 64 keys, all 128 dims)
//     and HALF of every V tile (all 128 keys, its 64 head dims): the B operand of a 2-CTA MMA is
//     split along N between the CTAs.  A K/V byte staged still serves 256 query rows, while each
//     SM stages and reads half the bytes of the one-CTA kernel per K/V tile.  TMA copies of both
//     CTAs complete on the leader's barriers (`.cta_group::2` loads, no multicast); the leader
//     posts the expected bytes of both.
//   * TMEM (each CTA, 512 columns): two S/P buffers of 128 columns (the CTA's tile c in buffer
//     c % 2) and two O buffers (item m in buffer m % 2).  With one row tile per SM there is room
//     for the second S buffer, so S(i+2) is issued right after PV(i) (which reads P(i) from the
//     same buffer; tcgen05.mma of one thread run in issue order) and the softmax finds its next S
//     computed; with the second O buffer the first PV of an item does not wait for the previous
//     item's epilogue, and with two Q buffers in shared memory (the halved K/V stages make room)
//     the next item's Q is loaded one item ahead: unit boundaries cost no pipeline refill.
//   * softmax: 8 warps per CTA, two per TMEM lane quadrant; a thread owns one row and half of
//     the tile's 128 key columns (and of O's 128 columns).  The halves of a row agree on its
//     running maximum through shared memory behind a named barrier of the quadrant's two warps.
//   * barriers: commits arrive on both CTAs' copies (`.multicast::cluster` commits); every
//     softmax warp of both CTAs arrives on the leader's p_full / o_free; one s_full / p_full
//     barrier per S buffer and one o_free per O buffer (a buffer's next use needs the consumer of
//     its previous one, so no barrier runs two phases ahead of its waiter).  Every wait is bounded.
// Warps: 0 Q + K loader, 1 MMA (issues in the leader; allocates TMEM in both), 2-9 softmax,
// 10 V loader.  The barrier protocol is restated and checked on the host by
// tests/test_prefill_protocol.py (run_pair).
#include "common.cuh"
#include "kernels.cuh"

namespace mi {
namespace {

constexpr int kP2SoftmaxWarps = 8;               // two sets of 4 (one warp per TMEM lane quadrant each)
constexpr int kP2Threads = 32 * (3 + kP2SoftmaxWarps);
constexpr int kP2VLoaderWarp = kFirstSoftmaxWarp + kP2SoftmaxWarps;
constexpr int kP2StagesK = 5;                     // depth of the K ring: K(i + 2) is needed with V(i)
constexpr int kP2StagesV = 4;                     // depth of the V ring
constexpr int kP2Half = 64;                       // keys (K) or head dims (V) a CTA stages per tile
constexpr int kP2KBytes = kP2Half * 128 * 2;      // 16 KiB: 64 keys x 128 dims, two 8 KiB regions
constexpr int kP2KRegion = kP2Half * 128;         // 8 KiB: 64 rows x 64 dims
constexpr int kP2VBytes = kTcKv * kP2Half * 2;    // 16 KiB: 128 keys x 64 dims, one region
constexpr int kP2OffQ = 0;                        // two Q buffers of 32 KiB
constexpr int kP2OffK = kP2OffQ + 2 * kQBytes;
constexpr int kP2OffV = kP2OffK + kP2StagesK * kP2KBytes;
constexpr int kP2OffBar = kP2OffV + kP2StagesV * kP2VBytes;
constexpr int kP2OffXchg = kP2OffBar + 256;       // row maxima and row sums [2 sets][128] for the merge
constexpr int kP2SmemBytes = kP2OffXchg + 2 * 2 * kTcRows * 4 + 1024;  // + alignment slack (~195 KiB)
static_assert(kP2SmemBytes <= 232448, "shared memory above the 227 KiB a CTA may use");
constexpr int kPolyEvery = 0;                     // every kPolyEvery-th exponential pair by exp2_poly (0: none)
constexpr int kP2HalfKeys = 64;                   // keys of a half tile: one S buffer, N of its S MMA
constexpr uint32_t kP2TmemO = 256;                // S buffers 2h + k % 2 at 64 (2h + k % 2); O_0 / O_1 at 256 / 384

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of a shared::cta variable's copy in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrival on a barrier of either CTA of the cluster (default semantics, as for a local arrival:
// the data it publishes is TMEM written by tcgen05.st and completed by tcgen05.wait::st, ordered
// by the tcgen05 fences around it).
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2^x on the FMA and integer pipes, for the share of the softmax exponentials taken off the
// MUFU unit (whose rate, 16 results per clock per SM, otherwise sets the softmax time).  Method:
// Cody-Waite range reduction x = j + f, j = round(x) (adding 1.5 * 2^23 rounds to an integer
// held in the low mantissa bits), f in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose
// coefficients were fitted to the relative error on [-0.5, 0.5] by iteratively reweighted least
// squares (Lawson's algorithm); 2^j by adding j to the exponent field.  Maximum relative error
// 7.5e-5 in fp32 (P is rounded to 16 bits after, relative step 2^-8).  x is clamped at -125
// (-inf from masking included) so the exponent stays normal: 2^-125 stands in for 0, which no
// row with a visible key can tell from 0.  x <= 8 here (the rescale threshold).
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;  // 1.5 * 2^23: round to nearest
  const float j = t - 12582912.f;
  const float f = x - j;
  float p = fmaf(0.05517132f, f, 0.24261054f);
  p = fmaf(p, f, 0.69326097f);
  p = fmaf(p, f, 0.99992812f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}
// Named barrier of the two softmax warps that share a TMEM lane quadrant.
__device__ __forceinline__ void pair_sync(uint32_t id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }
__device__ __forceinline__ void umma_pair_ss(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_pair_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}
// Commit of the leader's MMAs, arriving on the barrier at this offset in both CTAs.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "h"((unsigned short)0x3)
      : "memory");
}
// Non-multicast TMA loads into this CTA's shared memory whose bytes complete on the barrier at
// `bar_cluster` (the leader's copy).
__device__ __forceinline__ void tma_pair_3d(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_pair_4d(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// One loader warp's stream of its CTA's K or V halves over the cluster's items.  Lane q holds the
// block id of page q of the part of a tile this CTA stages, for the next kAhead tiles (a FIFO in
// registers: the table reads are issued kAhead tiles before their TMA boxes, so a loader that
// finds its ring stages free issues back to back instead of once per global-load latency); a
// tile goes out as one TMA box per lane.
//   K half: keys [128 t + 64 rank, + 64): 64 / bs pages x 2 dim halves (history), or 2 boxes of
//           64 tokens x 64 dims (chunk); stage = two 8 KiB regions (dims 0-63, 64-127) of 64 rows.
//   V half: all 128 keys, dims [64 rank, + 64): 128 / bs pages (history) or 2 boxes of 64 tokens
//           (chunk); stage = one 16 KiB region of 128 rows.
constexpr int64_t kNoPage = INT64_MIN;  // the lane's page is not history: the box reads zeros
struct PairLoader {
  TcCursor c;  // the next tile to issue
  TcCursor f;  // the next tile to read block ids for
  int64_t p0, p1, p2, p3;  // block ids of tiles c, c + 1, c + 2, c + 3 (this lane's page)
  int lane, shift, rank;
  bool is_v;
  __device__ __forceinline__ int pages(const PrefillArgs& a) const { return (is_v ? kTcKv : kP2Half) / a.block_size; }
  __device__ __forceinline__ int64_t fetch(const PrefillArgs& a) {
    int64_t id = kNoPage;
    if (f.valid && lane < pages(a)) {
      const int t = f.it.t_begin + f.i;
      const int pos0 = t * kTcKv + (is_v ? 0 : rank * kP2Half) + lane * a.block_size;
      if (t < f.it.u.row.hist_tiles && pos0 < f.it.u.row.start)
        id = a.block_tables[f.it.u.b * a.table_stride + (pos0 >> shift)];
    }
    if (f.valid) f.advance(a);
    return id;
  }
  __device__ __forceinline__ void init(const TcWalker& w0, const PrefillArgs& a, int lane_, int shift_, int rank_,
                                       bool is_v_) {
    lane = lane_;
    shift = shift_;
    rank = rank_;
    is_v = is_v_;
    c.init(w0, a);
    f.init(w0, a);
    p0 = fetch(a);
    p1 = fetch(a);
    p2 = fetch(a);
    p3 = fetch(a);
  }
  __device__ __forceinline__ void issue(const PrefillArgs& a, const CUtensorMap& pool_map, const CUtensorMap& chunk_map,
                                        uint8_t* dst, uint64_t* full_local, uint32_t full_leader) {
    const int np = pages(a);
    int my_row = (int)(a.num_blocks * a.block_size);  // past the pool: TMA reads zeros
    if (lane < np && p0 != kNoPage) {
      if (p0 < 0 || p0 >= a.num_blocks) record_status(MI_STATUS_BAD_BLOCK);
      else my_row = (int)(p0 * a.block_size);
    }
    const int t = c.it.t_begin + c.i;
    const bool hist = t < c.it.u.row.hist_tiles;
    const int h = c.it.h;
    const int b = c.it.u.b;
    const int pos = c.it.u.row.first + (t - c.it.u.row.hist_tiles) * kTcKv;
    if (rank == 0 && lane == 0) mbar_arrive_expect_tx(full_local, 2u * (uint32_t)(is_v ? kP2VBytes : kP2KBytes));
    __syncwarp();
    if (!is_v) {
      const int boxes = hist ? 2 * np : 2;
      const int q = lane >> 1, cc = lane & 1;
      const int row0 = __shfl_sync(0xffffffffu, my_row, q & 31);
      if (lane < boxes) {
        if (hist) tma_pair_3d(dst + cc * kP2KRegion + q * a.block_size * 128, &pool_map, full_leader, cc * 64, h, row0);
        else tma_pair_4d(dst + cc * kP2KRegion, &chunk_map, full_leader, cc * 64, h, pos + rank * kP2Half, b);
      }
    } else {
      const int boxes = hist ? np : 2;
      if (lane < boxes) {
        if (hist) tma_pair_3d(dst + lane * a.block_size * 128, &pool_map, full_leader, rank * kP2Half, h, my_row);
        else tma_pair_4d(dst + lane * 64 * 128, &chunk_map, full_leader, rank * kP2Half, h, pos + lane * 64, b);
      }
    }
    c.advance(a);
    p0 = p1;
    p1 = p2;
    p2 = p3;
    p3 = fetch(a);
  }
};

template <typename T>
__global__ void __launch_bounds__(kP2Threads, 1) prefill_tc2_kernel(const PrefillArgs a,
                                                                     const __grid_constant__ PrefillMaps maps,
                                                                     float* ws_o, float* ws_ml, int64_t* ws_desc,
                                                                     int pairs, int shift) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kP2OffBar);
  // leader-side barriers (both CTAs' TMA bytes, or one arrival per softmax warp of both CTAs)
  uint64_t* q_full = bars + 0;                 // [2] per Q buffer
  uint64_t* k_full = q_full + 2;               // [kP2StagesK]
  uint64_t* v_full = k_full + kP2StagesK;      // [kP2StagesV]
  uint64_t* p_full = v_full + kP2StagesV;      // [4] per S buffer 2h + k % 2
  uint64_t* o_free = p_full + 4;               // both O accumulators read out
  // barriers of each CTA, arrived on by the leader's multicast commits
  uint64_t* k_empty = o_free + 1;              // [kP2StagesK]
  uint64_t* v_empty = k_empty + kP2StagesK;    // [kP2StagesV]
  uint64_t* s_full = v_empty + kP2StagesV;     // [4] per S buffer
  uint64_t* o_done = s_full + 4;               // [2] per set: one phase per PV into O_set
  uint64_t* o_final = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);
  float* xmax = reinterpret_cast<float*>(smem + kP2OffXchg);  // [2 sets][128 rows]
  float* xsum = xmax + 2 * kTcRows;                           // [2 sets][128 rows]

  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent of the previous kernel
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = a.groups;
  const int row_elems = a.hq * kTcDim;
  const uint32_t rank = cluster_rank();
  const int cluster = (int)(blockIdx.x >> 1);
  const int clusters = (int)(gridDim.x >> 1);
  T* out = reinterpret_cast<T*>(a.out);

  zero_padding<T, kP2Threads>(a, tid);
  int64_t total, ctas;
  int64_t* const scratch = reinterpret_cast<int64_t*>(smem + kP2OffK);
  const TcWalker walk0 = tc_start<kP2Threads>(a, pairs, scratch, tid, total, ctas, cluster, clusters);
  if (tid == 0) {  // the cluster's tiles, and the unit it opens and leaves unfinished (for the combine)
    int64_t d0 = -1, d1 = 0, d2 = 0, tiles = 0;
    TcWalker w = walk0;
    TcItem it;
    const int64_t r = cluster / a.hkv;
    const int64_t x0 = r * total / max(ctas, (int64_t)1);
    while (w.next(a, it)) {
      tiles += it.n;
      if (it.slot == 2 * cluster + 1) {
        const int64_t first = x0 + w.used - it.n;
        d0 = it.u.b * pairs + it.u.pair;
        d1 = it.h;
        d2 = ((first + it.u.n) * ctas - 1) / total * a.hkv + it.h;
      }
    }
    if (rank == 0) {
      ws_desc[cluster * 4 + 0] = d0;
      ws_desc[cluster * 4 + 1] = d1;
      ws_desc[cluster * 4 + 2] = d2;
    }
    scratch[16] = tiles;
  }
  __syncthreads();
  const int64_t n_tiles = scratch[16];
  if (n_tiles == 0) return;  // uniform for the cluster: both CTAs walk the same items

  if (tid == 0) {
    for (int i = 0; i < kP2StagesK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kP2StagesV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&p_full[b], 2 * 4);  // the 4 warps of one set, in both CTAs
      mbar_init(&s_full[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&o_done[b], 1);
    }
    mbar_init(o_free, 2 * kP2SoftmaxWarps);
    mbar_init(o_final, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {  // both CTAs, same warp: the pair's TMEM columns
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_async_smem();  // the start scan's shared-memory words (K stage 0) before TMA writes them
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool aborted = false;

  if (warp == kLoaderWarp || warp == kP2VLoaderWarp) {
    const bool is_v = warp == kP2VLoaderWarp;
    if (lane == 0) {
      tma_prefetch_desc(&maps.q);
      tma_prefetch_desc(&maps.k_chunk);
      tma_prefetch_desc(&maps.v_chunk);
      tma_prefetch_desc(&maps.k_pool);
      tma_prefetch_desc(&maps.v_pool);
    }
    __syncwarp();
    PairLoader ld;
    ld.init(walk0, a, lane, shift, (int)rank, is_v);
    uint64_t* full = is_v ? v_full : k_full;
    uint64_t* empty = is_v ? v_empty : k_empty;
    const int stage_bytes = is_v ? kP2VBytes : kP2KBytes;
    uint8_t* ring = smem + (is_v ? kP2OffV : kP2OffK);
    // item m's Q (this CTA's row tile: box [64 d, G heads, 128/G tokens]) into buffer m % 2
    auto load_q = [&](const TcItem& it, int m) {
      uint64_t* bar = &q_full[m & 1];
      if (rank == 0 && lane == 0) mbar_arrive_expect_tx(bar, 2u * (uint32_t)kQBytes);
      __syncwarp();
      if (lane < 2) {
        const int tok0 = rank ? it.u.tok0[1] : it.u.tok0[0];
        tma_pair_4d(smem + kP2OffQ + (m & 1) * kQBytes + lane * kQRegion, &maps.q, mapa_rank(bar, 0), lane * 64,
                    it.h * G, it.u.row.first + tok0, it.u.b);
      }
    };
    const int stages = is_v ? kP2StagesV : kP2StagesK;
    auto issue = [&](int64_t j) {
      const int st = (int)(j % stages);
      ld.issue(a, is_v ? maps.v_pool : maps.k_pool, is_v ? maps.v_chunk : maps.k_chunk, ring + st * stage_bytes,
               &full[st], mapa_rank(&full[st], 0));
    };
    if (is_v) {
      for (int64_t j = 0; j < n_tiles; ++j) {
        if (j >= kP2StagesV) mbar_wait_warp(&empty[j % kP2StagesV], ((j / kP2StagesV) - 1) & 1, aborted);
        issue(j);
      }
    } else {
      // K(j + stages) reuses the stage of tile j once S(j) is done.  The Q of items 0 and 1 load
      // first; that of item m + 2 once every S of item m is done (S(j) of its last tile j: the S
      // MMAs complete in issue order), into the buffer item m used.
      TcWalker wq = walk0;
      TcItem qi;
      int nq = 0;
      for (int k = 0; k < 2 && wq.next(a, qi); ++k) load_q(qi, nq++);
      TcCursor cq;
      cq.init(walk0, a);
      for (int64_t j = 0; j < min(n_tiles, (int64_t)kP2StagesK); ++j) issue(j);
      for (int64_t j = 0; j < n_tiles; ++j) {
        const bool item_end = cq.last_of_item();
        cq.advance(a);
        if (item_end || j + kP2StagesK < n_tiles)
          mbar_wait_warp(&empty[j % kP2StagesK], (j / kP2StagesK) & 1, aborted);
        if (item_end && wq.next(a, qi)) load_q(qi, nq++);
        if (j + kP2StagesK < n_tiles) issue(j + kP2StagesK);
      }
    }
    // tail: every commit that frees a stage of this CTA has landed before the CTA may exit
    for (int64_t j = max((int64_t)0, n_tiles - stages); j < n_tiles; ++j)
      mbar_wait_warp(&empty[j % stages], (j / stages) & 1, aborted);
  } else if (warp == kMmaWarp) {
    if (rank == 0) {
      // ---------------- MMA issuer (leader): M = 256 over both CTAs' row tiles ----------------
      // Per tile k of the stream and half h: S_h(k) = Q K_h(k)^T (N = 64 keys: 32 from each CTA's
      // K piece h) into buffer 2h + k % 2, O_h += P_h(k) V_h(k) (K = the same 64 keys).
      constexpr bool kBf16 = !std::is_same<T, __half>::value;
      const uint32_t idesc_qk = idesc_f16(kBf16, false, 2 * kTcRows, kP2HalfKeys);
      const uint32_t idesc_pv = idesc_f16(kBf16, true, 2 * kTcRows, kTcDim);
      const uint64_t dk = desc_kmajor(sbase + kP2OffK);
      const uint64_t dv = desc_mnmajor(sbase + kP2OffV);
      TcWalker w = walk0;
      TcItem it;
      int64_t j0 = 0;  // the cluster's tile index of the item's first tile
      int c = 0;       // tiles so far (tile k of the stream uses S buffers 2h + k % 2)
      int items = 0;   // item m uses Q buffer m % 2
      while (w.next(a, it)) {
        const int n = it.n;
        const int qb = items & 1;
        const uint64_t dq = desc_kmajor(sbase + kP2OffQ + qb * kQBytes);
        auto issue_s = [&](int i, int h) {  // S_h(i) into buffer 2h + (c + i) % 2
          const int64_t jj = j0 + i;
          const int ks = (int)(jj % kP2StagesK);
          const int bb = 2 * h + ((c + i) & 1);
          tc_fence_after();
          // this CTA's piece h: rows [32 h, 32 h + 32) of both 64-dimension regions of the K stage
          const uint64_t dks = dk + (uint64_t)((ks * kP2KBytes + h * 32 * 128) >> 4);
#pragma unroll
          for (int s = 0; s < kTcDim / 16; ++s)
            umma_pair_ss(tmem + bb * kP2HalfKeys, dq + (uint64_t)(((s >> 2) * kQRegion + (s & 3) * 32) >> 4),
                         dks + (uint64_t)(((s >> 2) * kP2KRegion + (s & 3) * 32) >> 4), idesc_qk, s > 0 ? 1u : 0u);
          umma_commit_pair(&s_full[bb]);
          if (h == 1) umma_commit_pair(&k_empty[ks]);  // the stage's last S
        };
        mbar_wait_warp(&q_full[qb], (items >> 1) & 1, aborted);
        for (int i = 0; i < min(n, 2); ++i) {
          mbar_wait_warp(&k_full[(j0 + i) % kP2StagesK], ((j0 + i) / kP2StagesK) & 1, aborted);
          issue_s(i, 0);
          issue_s(i, 1);
        }
        for (int i = 0; i < n; ++i) {
          const int k = c + i;
          const int64_t jj = j0 + i;
          const int vs = (int)(jj % kP2StagesV);
          mbar_wait_warp(&v_full[vs], (jj / kP2StagesV) & 1, aborted);
          // both O accumulators read out by the previous item's epilogue
          if (i == 0 && items > 0) mbar_wait_warp(o_free, (items - 1) & 1, aborted);
          const uint64_t dvs = dv + (uint64_t)((vs * kP2VBytes) >> 4);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int bb = 2 * h + (k & 1);
            mbar_wait_warp(&p_full[bb], (k >> 1) & 1, aborted);  // set h's P(k) in both CTAs' TMEM
            tc_fence_after();
            // k-step s covers S_h columns [16 s, 16 s + 16): keys 64 (s / 2) + 32 h + 16 (s % 2) + [0, 16)
#pragma unroll
            for (int s = 0; s < kP2HalfKeys / 16; ++s)
              umma_pair_ts(tmem + kP2TmemO + h * 128, tmem + bb * kP2HalfKeys + s * 8,
                           dvs + (uint64_t)((((s >> 1) * 64 + 32 * h + (s & 1) * 16) * 128) >> 4), idesc_pv,
                           (i > 0 || s > 0) ? 1u : 0u);
            umma_commit_pair(&o_done[h]);
            if (h == 1) {
              umma_commit_pair(&v_empty[vs]);
              if (i + 1 == n) umma_commit_pair(o_final);
            }
            if (i + 2 < n) {
              if (h == 0)
                mbar_wait_warp(&k_full[(jj + 2) % kP2StagesK], ((jj + 2) / kP2StagesK) & 1, aborted);
              issue_s(i + 2, h);
            }
          }
        }
        c += n;
        j0 += n;
        ++items;
      }
    }
  } else if (warp >= kFirstSoftmaxWarp && warp < kFirstSoftmaxWarp + kP2SoftmaxWarps) {
    // ------- softmax set `set` (= h): half h of every tile, i.e. S_h columns j <-> tile keys
    // 64 (j / 32) + 32 h + j % 32; thread <-> row (TMEM lane) of this CTA's row tile; running max /
    // sum and O accumulator O_h of its own, merged with the other set's in the item's epilogue ----
    const int g = (int)rank;
    const int set = (warp - kFirstSoftmaxWarp) >> 2;
    const int quad = warp & 3;                        // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t bar_id = 1 + (uint32_t)quad;       // the two warps of one quadrant (one per set)
    const float scale = a.scale_log2;
    const uint32_t o_addr = tmem + kP2TmemO + (uint32_t)set * 128 + lane_base;
    const uint32_t p_full_leader[2] = {mapa_rank(&p_full[2 * set], 0), mapa_rank(&p_full[2 * set + 1], 0)};
    const uint32_t o_free_leader = mapa_rank(o_free, 0);
    TcWalker w = walk0;
    TcItem it;
    int c = 0, items = 0;  // tiles of the stream (barrier phases), items
    while (w.next(a, it)) {
      const TcPair& u = it.u;
      const int n = it.n;  // every tile of the unit's union range (tiles past this row tile's range are masked)
      const int64_t my_tok0 = g ? u.tok0[1] : u.tok0[0];
      const int64_t my_tok = my_tok0 + r / G;
      const bool row_valid = my_tok < (g ? u.tok_end[1] : u.tok_end[0]);
      const int start = u.row.start;
      const int hist_tiles = u.row.hist_tiles;
      float m_ref = -INFINITY, l_run = 0.f;
      for (int i = 0; i < n; ++i) {
        const int t = it.t_begin + i;
        const int k = c + i;
        const int par = k & 1;
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
        lim -= 32 * set;  // column j of chunk cc is visible while 64 cc + j < lim
        const uint32_t s_addr = tmem + (uint32_t)(2 * set + par) * kP2HalfKeys + lane_base;
        bool ab = aborted;
        mbar_wait(&s_full[2 * set + par], (k >> 1) & 1, ab);
        aborted = ab;
        tc_fence_after();
        uint32_t sr[2][32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) tmem_ld32_async(s_addr + cc * 32, sr[cc]);
        tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (cc * 64 + e >= lim) sr[cc][e] = 0xff800000u;
          }
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            mx[(e >> 1) & 3] = fmax3(mx[(e >> 1) & 3], __uint_as_float(sr[cc][e]), __uint_as_float(sr[cc][e + 1]));
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
        const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t pw[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float x0 = fmaf(__uint_as_float(sr[cc][2 * j]), scale, neg_m);
            const float x1 = fmaf(__uint_as_float(sr[cc][2 * j + 1]), scale, neg_m);
            // kPolyEvery-th pairs on the FMA pipe, the rest on MUFU
            const bool poly = kPolyEvery > 0 && (j % kPolyEvery) == kPolyEvery - 1;
            const float p0 = poly ? exp2_poly(x0) : fast_exp2(x0);
            const float p1 = poly ? exp2_poly(x1) : fast_exp2(x1);
            ps[j & 3] += p0 + p1;
            pw[j] = pack2<T>(p0, p1);
          }
          tmem_st16_async(s_addr + cc * 16, pw);  // P over the buffer's first 32 columns
        }
        l_run += (ps[0] + ps[1]) + (ps[2] + ps[3]);
        if (__any_sync(0xffffffffu, need)) {  // warp-collective TMEM access
          bool ab2 = aborted;
          mbar_wait(&o_done[set], (k - 1) & 1, ab2);  // PV_h(k - 1) finished writing O_h
          aborted = ab2;
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            float ov[32];
            tmem_ld32(o_addr + cc * 32, ov);
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] *= alpha;
            tmem_st32(o_addr + cc * 32, ov);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) remote_arrive(p_full_leader[par]);
      }
      c += n;
      // ---- epilogue of the item: merge the two sets' (m, l, O) per row; set s stores output
      // columns [64 s, 64 s + 64)
      {
        bool ab = aborted;
        mbar_wait(o_final, items & 1, ab);
        aborted = ab;
      }
      tc_fence_after();
      xmax[set * kTcRows + r] = m_ref;
      xsum[set * kTcRows + r] = l_run;
      pair_sync(bar_id);
      const float m0 = xmax[r], m1 = xmax[kTcRows + r];
      const float m = fmaxf(m0, m1);
      // a set with nothing visible for this row (or no tile in the item) contributes nothing: its
      // O columns are not read into the sum (they may hold an earlier item's values)
      const float a0 = m0 == -INFINITY ? 0.f : fast_exp2(m0 - m);
      const float a1 = m1 == -INFINITY ? 0.f : fast_exp2(m1 - m);
      const float l_all = xsum[r] * a0 + xsum[kTcRows + r] * a1;
      const float inv = l_all > 0.f ? 1.f / l_all : 0.f;
      uint32_t o0[2][32], o1[2][32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        tmem_ld32_async(tmem + kP2TmemO + lane_base + set * 64 + cc * 32, o0[cc]);
        tmem_ld32_async(tmem + kP2TmemO + 128 + lane_base + set * 64 + cc * 32, o1[cc]);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(o_free_leader);
      float ov[2][32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          ov[cc][e] = (a0 != 0.f ? __uint_as_float(o0[cc][e]) * a0 : 0.f) +
                      (a1 != 0.f ? __uint_as_float(o1[cc][e]) * a1 : 0.f);
      }
      const int64_t part = (int64_t)it.slot * kPair + g;
      if (it.slot < 0) {
        if (row_valid) {
          T* dst = out + (u.b * a.padded_len + u.row.first + my_tok) * row_elems + (int64_t)(it.h * G + r % G) * kTcDim +
                   set * 64;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const float* f = &ov[cc][v * 8];
              uint4 pk;
              pk.x = pack2<T>(f[0] * inv, f[1] * inv);
              pk.y = pack2<T>(f[2] * inv, f[3] * inv);
              pk.z = pack2<T>(f[4] * inv, f[5] * inv);
              pk.w = pack2<T>(f[6] * inv, f[7] * inv);
              *reinterpret_cast<uint4*>(dst + cc * 32 + v * 8) = pk;
            }
          }
        }
      } else {
        float* po = ws_o + (part * kTcRows + r) * kTcDim + set * 64;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
          for (int v = 0; v < 8; ++v)
            *reinterpret_cast<float4*>(po + cc * 32 + v * 4) =
                make_float4(ov[cc][v * 4], ov[cc][v * 4 + 1], ov[cc][v * 4 + 2], ov[cc][v * 4 + 3]);
        }
        if (set == 0) *reinterpret_cast<float2*>(ws_ml + (part * kTcRows + r) * 2) = make_float2(m, l_all);
      }
      // the exchange words are rewritten at the next epilogue, after at least one more pair
      // barrier; the next item's first pair barrier is this one's partner's too
      pair_sync(bar_id);
      ++items;
    }
    // tail: this set's last o_done arrival (committed before o_final) has landed as well
    mbar_wait(&o_done[set], (c - 1) & 1, aborted);
  }
  tc_fence_before();
  cluster_sync_all();  // every MMA into either CTA's TMEM has been waited for
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

int pair_clusters_for(int hkv) {
  static int max_clusters = -1;
  if (max_clusters < 0) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (kMaxCtas / 2));
    cfg.blockDim = dim3(kP2Threads);
    cfg.dynamicSmemBytes = kP2SmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaFuncSetAttribute(prefill_tc2_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kP2SmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(prefill_tc2_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kP2SmemBytes) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, prefill_tc2_kernel<__nv_bfloat16>, &cfg) != cudaSuccess)
      n = 0;
    (void)cudaGetLastError();
    max_clusters = std::min(n, kMaxCtas / 2);
  }
  return max_clusters >= hkv ? max_clusters / hkv * hkv : 0;
}

template <typename T>
cudaError_t launch_tc2(const PrefillArgs& a, float* ws, const PrefillMaps& maps, int clusters, cudaStream_t s) {
  auto kern = prefill_tc2_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kP2SmemBytes);
  if (e != cudaSuccess) return e;
  float* ws_o = ws;
  float* ws_ml = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kWsOBytes);
  int64_t* ws_desc = reinterpret_cast<int64_t*>(reinterpret_cast<char*>(ws) + kWsOBytes + kWsMlBytes);
  const int64_t tokens_per_tile = kTcRows / a.groups;
  const int64_t qtiles = (a.padded_len + tokens_per_tile - 1) / tokens_per_tile;
  const int pairs = (int)((qtiles + kPair - 1) / kPair);
  {
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(kP2Threads);
    cfg.dynamicSmemBytes = kP2SmemBytes;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, a, maps, ws_o, ws_ml, ws_desc, pairs, log2_if_pow2(a.block_size));
  }
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(clusters, kPair, kTcRows / kCombineRows);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_combine_kernel<T>, a, static_cast<const float*>(ws_o),
                            static_cast<const float*>(ws_ml), static_cast<const int64_t*>(ws_desc), pairs);
}

}  // namespace

// The CTA-pair kernel for TMA-staged operands (block sizes 16/32/64); 0 clusters: not available.
int prefill_tc2_clusters(const PrefillArgs& a, const PrefillMaps* maps) {
  if (!maps || a.block_size > kP2Half) return 0;
  return pair_clusters_for(a.hkv);
}

cudaError_t launch_paged_prefill_tc2(const PrefillArgs& a, float* ws, const PrefillMaps& maps, int clusters, int dtype,
                                     cudaStream_t s) {
  if (dtype == MI_BF16) return launch_tc2<__nv_bfloat16>(a, ws, maps, clusters, s);
  return launch_tc2<__half>(a, ws, maps, clusters, s);
}

}  // namespace mi
