// Chunked-prefill paged attention on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Variant: bf16 / fp16, head_dim 128, any block size, G = Hq/H_kv in {1, 2, 4, 8}.
// One CTA (128 threads) = one (sequence, KV head, tile of 128 query rows).  The 128 rows pack
// 128/G chunk tokens x G query heads of the KV head (row r = token r/G, head r%G), so the K/V
// tiles staged in shared memory serve the whole GQA group.  Per 128-position KV tile:
//   1. cp.async stages K and V rows (double-buffered, the next tile streams in during this one):
//      positions < start come from the pool through the block table, the rest from the chunk's
//      own K/V; rows past the causal end are zero-filled;
//   2. one thread issues S = Q K^T as 8 tcgen05.mma (M=128, N=128, K=16, kind::f16, fp32 accum)
//      into TMEM columns [0, 128); tcgen05.commit signals an mbarrier;
//   3. each thread owns one row (its TMEM lane): tcgen05.ld of the row, causal/length mask, online
//      softmax in the exp2 domain; the running O in TMEM is rescaled (tcgen05.ld/st) only when the
//      row maximum grew by more than 2^8 since the last rescale (otherwise p <= 2^8 stays exact
//      in fp32 and the final 1/l normalisation absorbs it); P is written as bf16 into shared
//      memory in the 128-byte-swizzled K-major layout;
//   4. one thread issues O += P V as 8 tcgen05.mma (V read MN-major) into TMEM columns [128, 256).
// Epilogue: tcgen05.ld of O, divide by l, store bf16 rows.  Padding positions get zeros.
//
// Shared-memory operand layout ("SW128"): a 128 x 128 tile of 16-bit elements is two 16 KiB
// regions (columns 0-63 and 64-127); row r of a region is 128 bytes at r*128, and its 16-byte unit
// u lives at unit u ^ (r % 8).  Every region starts 1024-byte aligned.  Descriptors:
//   K-major (Q, K, P):  start, LBO = 16 B (unused), SBO = 1024 B (8-row groups), swizzle 128B;
//                       k-step s (16 columns) starts at region(s/4) + (s%4)*32 B.
//   MN-major (V as the B operand of PV, N = head_dim):  LBO = 16 KiB (next 64 columns of N),
//                       SBO = 1024 B (next 8 K-rows); k-step s starts at s*16 rows = s*2048 B.
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace mi {
namespace {

constexpr int kTcRows = 128;       // query rows per CTA (MMA M)
constexpr int kTcKv = 128;         // KV positions per tile (MMA N of QK^T, K of PV)
constexpr int kTcDim = 128;        // head_dim
constexpr int kTcThreads = 128;
constexpr int kTileBytes = kTcRows * kTcDim * 2;  // 32 KiB per 128 x 128 operand
constexpr int kRegionBytes = kTileBytes / 2;      // 16 KiB per 64-column region
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;          // two buffers
constexpr int kOffV = kOffK + 2 * kTileBytes;      // two buffers
constexpr int kOffP = kOffV + 2 * kTileBytes;
constexpr int kOffBar = kOffP + kTileBytes;
constexpr int kTcSmemBytes = kOffBar + 64 + 1024;  // + barriers/TMEM slot + alignment slack
constexpr uint32_t kTmemCols = 256;                // S: [0,128), O: [128,256)
constexpr float kRescaleLog2 = 8.0f;

__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t unit16) {
  // unit16 in [0, 16): 16-byte unit of a 256-byte row (128 two-byte columns)
  return (unit16 >> 3) * kRegionBytes + row * 128 + (((unit16 & 7) ^ (row & 7)) << 4);
}

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (uint64_t(kRegionBytes >> 4) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// kind::f16 instruction descriptor: fp32 accumulate, A/B format, A K-major, B K- or MN-major, N, M.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, bool b_mn_major, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
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

__device__ __forceinline__ void cp_async16(uint32_t sdst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sdst), "l"(gsrc), "r"(valid ? 16u : 0u)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

struct TcRowMap {
  int groups;
  int64_t tok0;  // first chunk token of this tile
};

// Stage one 128-position KV tile (K and V) for KV head h: positions [j0, j0 + 128).  Thread t
// moves 16-byte unit (t % 16) of rows t/16, t/16 + 8, ...: 16 threads cover one 256-byte row.
template <typename T>
__device__ __forceinline__ void stage_kv(const PrefillArgs& a, int64_t b, int h, int64_t start, int64_t kv_end,
                                         int64_t first, int64_t j0, uint32_t k_dst, uint32_t v_dst) {
  const int unit = threadIdx.x & 15;
  const int64_t* table = a.block_tables + b * a.table_stride;
  const char* kc = a.k_chunk + b * a.kv_sb[0] + (int64_t)h * a.kv_sb[2];
  const char* vc = a.v_chunk + b * a.kv_sb[0] + (int64_t)h * a.kv_sb[2];
  const int64_t pool_row = (int64_t)a.hkv * kTcDim * sizeof(T);
#pragma unroll 4
  for (int rr = threadIdx.x >> 4; rr < kTcKv; rr += kTcThreads / 16) {
    const int64_t j = j0 + rr;
    const char* ksrc = a.k_chunk;  // any valid address for zero-fill
    const char* vsrc = a.k_chunk;
    bool valid = j < kv_end;
    if (valid && j < start) {
      const int64_t blk = table[j / a.block_size];
      if (blk < 0 || blk >= a.num_blocks) {
        if (unit == 0) record_status(MI_STATUS_BAD_BLOCK);
        valid = false;
      } else {
        const int64_t off = (blk * a.block_size + j % a.block_size) * pool_row + (int64_t)h * kTcDim * sizeof(T);
        ksrc = a.k_pool + off;
        vsrc = a.v_pool + off;
      }
    } else if (valid) {
      const int64_t p = first + (j - start);
      ksrc = kc + p * a.kv_sb[1];
      vsrc = vc + p * a.kv_sb[1];
    }
    const uint32_t o = sw128_offset((uint32_t)rr, (uint32_t)unit);
    cp_async16(k_dst + o, ksrc + (valid ? unit * 16 : 0), valid);
    cp_async16(v_dst + o, vsrc + (valid ? unit * 16 : 0), valid);
  }
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1) prefill_tc_kernel(const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);

  const int qtile = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = a.groups;
  const int tokens_per_tile = kTcRows / G;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;

  int64_t len = a.chunk_lens[b];
  if (len > a.padded_len) {
    if (tid == 0 && qtile == 0 && h == 0) record_status(MI_STATUS_BAD_LENGTH);
    len = a.padded_len;
  }
  if (len < 0) len = 0;
  const int64_t first = a.padded_len - len;
  int64_t start = a.starts[b];
  if (start < 0) start = 0;
  if (start > a.table_stride * a.block_size) {
    if (tid == 0 && qtile == 0 && h == 0) record_status(MI_STATUS_BAD_LENGTH);
    start = a.table_stride * a.block_size;
  }
  const int row_bytes_out = a.hq * kTcDim;  // elements per output position
  T* out = reinterpret_cast<T*>(a.out);

  // Padding positions of this KV head's query heads are zeros (the CTA of tile 0 writes them).
  if (qtile == 0) {
    for (int64_t i = tid; i < first * G * (kTcDim / 8); i += kTcThreads) {
      const int64_t p = i / (G * (kTcDim / 8));
      const int rem = (int)(i % (G * (kTcDim / 8)));
      const int g = rem / (kTcDim / 8);
      const int u = rem % (kTcDim / 8);
      *reinterpret_cast<uint4*>(out + (b * a.padded_len + p) * row_bytes_out + (int64_t)(h * G + g) * kTcDim + u * 8) =
          make_uint4(0, 0, 0, 0);
    }
  }
  const int64_t tok0 = (int64_t)qtile * tokens_per_tile;
  if (tok0 >= len) return;  // uniform for the CTA
  const int64_t tok_end = min(len, tok0 + tokens_per_tile);
  const int64_t kv_end = start + tok_end;  // causal end of the last token of the tile
  const int n_tiles = (int)((kv_end + kTcKv - 1) / kTcKv);

  // ---- setup: barriers, TMEM ----
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // ---- stage Q (row r = token r/G, head r%G) and the first KV tile ----
  {
    const int unit = tid & 15;
    for (int r = tid >> 4; r < kTcRows; r += kTcThreads / 16) {
      const int64_t tok = tok0 + r / G;
      const bool valid = tok < tok_end;
      const char* src = a.q;
      if (valid) src = a.q + b * a.q_sb[0] + (first + tok) * a.q_sb[1] + (int64_t)(h * G + r % G) * a.q_sb[2] + unit * 16;
      cp_async16(sbase + kOffQ + sw128_offset((uint32_t)r, (uint32_t)unit), src, valid);
    }
  }
  stage_kv<T>(a, b, h, start, kv_end, first, 0, sbase + kOffK, sbase + kOffV);
  cp_async_commit();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem;
  const uint32_t tmem_o = tmem + kTcKv;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
  const uint32_t idesc_qk = idesc_f16(kBf16, false, kTcRows, kTcKv);
  const uint32_t idesc_pv = idesc_f16(kBf16, true, kTcRows, kTcDim);

  // this thread's row
  const int r = tid;
  const int64_t my_tok = tok0 + r / G;
  const bool row_valid = my_tok < tok_end;
  const int64_t my_kv_end = row_valid ? start + my_tok + 1 : 0;  // keys [0, my_kv_end) are visible
  float m_ref = -INFINITY, l_run = 0.f;
  bool aborted = false;
  const float scale = a.scale_log2;

  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    cp_async_wait_all();  // tile j (and Q) landed
    fence_async_smem();
    __syncthreads();
    if (j > 0) {
      mbar_wait(bar_o, (j - 1) & 1, aborted);  // PV of tile j-1 finished: its V buffer and P are free
      tc_fence_after();
    }
    if (j + 1 < n_tiles) {
      stage_kv<T>(a, b, h, start, kv_end, first, (int64_t)(j + 1) * kTcKv, sbase + kOffK + (buf ^ 1) * kTileBytes,
                  sbase + kOffV + (buf ^ 1) * kTileBytes);
      cp_async_commit();
    }
    // ---- S = Q K^T ----
    if (tid == 0) {
      tc_fence_after();
      const uint32_t q0 = sbase + kOffQ, k0 = sbase + kOffK + buf * kTileBytes;
#pragma unroll
      for (int s = 0; s < kTcDim / 16; ++s) {
        const uint32_t off = (s >> 2) * kRegionBytes + (s & 3) * 32;
        umma_f16(tmem_s, desc_kmajor(q0 + off), desc_kmajor(k0 + off), idesc_qk, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_s);
    }
    mbar_wait(bar_s, j & 1, aborted);
    tc_fence_after();
    // ---- online softmax of this row: pass 1 (row max) and pass 2 (exp, sum, P) over TMEM ----
    const int64_t j0 = (int64_t)j * kTcKv;
    float tile_max = -INFINITY;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float sv[32];
      tmem_ld32(tmem_s + lane_base + c * 32, sv);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (j0 + c * 32 + i < my_kv_end) tile_max = fmaxf(tile_max, sv[i] * scale);
    }
    const float m_new = fmaxf(m_ref, tile_max);
    // tcgen05.ld/st are warp-collective: the warp rescales together if any of its rows must.
    const bool need = j > 0 && m_ref != -INFINITY && m_new > m_ref + kRescaleLog2;
    if (__any_sync(0xffffffffu, need)) {
      const float alpha = need ? exp2f(m_ref - m_new) : 1.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tmem_o + lane_base + c * 32, ov);
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
        tmem_st32(tmem_o + lane_base + c * 32, ov);
      }
    }
    if (need) {
      l_run *= exp2f(m_ref - m_new);
      m_ref = m_new;
    } else if (m_ref == -INFINITY) {
      m_ref = m_new;
    }
    float psum = 0.f;
    uint8_t* p_tile = smem + kOffP;
    const bool live = m_ref != -INFINITY;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float sv[32];
      tmem_ld32(tmem_s + lane_base + c * 32, sv);
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // 4 units of 8 columns per 32-column chunk
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i0 = u * 8 + 2 * e;
          const bool v0 = live && j0 + c * 32 + i0 < my_kv_end;
          const bool v1 = live && j0 + c * 32 + i0 + 1 < my_kv_end;
          const float p0 = v0 ? exp2f(sv[i0] * scale - m_ref) : 0.f;
          const float p1 = v1 ? exp2f(sv[i0 + 1] * scale - m_ref) : 0.f;
          psum += p0 + p1;
          w[e] = pack2<T>(p0, p1);
        }
        *reinterpret_cast<uint4*>(p_tile + sw128_offset((uint32_t)r, (uint32_t)(c * 4 + u))) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    l_run += psum;
    tc_fence_before();
    fence_async_smem();
    __syncthreads();
    // ---- O += P V ----
    if (tid == 0) {
      tc_fence_after();
      const uint32_t p0 = sbase + kOffP, v0 = sbase + kOffV + buf * kTileBytes;
#pragma unroll
      for (int s = 0; s < kTcKv / 16; ++s) {
        const uint32_t poff = (s >> 2) * kRegionBytes + (s & 3) * 32;
        umma_f16(tmem_o, desc_kmajor(p0 + poff), desc_mnmajor(v0 + s * 2048), idesc_pv, (j > 0 || s > 0) ? 1u : 0u);
      }
      umma_commit(bar_o);
    }
  }
  mbar_wait(bar_o, (n_tiles - 1) & 1, aborted);
  tc_fence_after();
  // ---- epilogue: O / l -> output row ----
  {
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    T* dst = out + (b * a.padded_len + first + my_tok) * row_bytes_out + (int64_t)(h * G + r % G) * kTcDim;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float ov[32];
      tmem_ld32(tmem_o + lane_base + c * 32, ov);
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <typename T>
cudaError_t launch_tc(const PrefillArgs& a, cudaStream_t s) {
  auto kern = prefill_tc_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes);
  if (e != cudaSuccess) return e;
  const int tokens_per_tile = kTcRows / a.groups;
  const int64_t qtiles = (a.padded_len + tokens_per_tile - 1) / tokens_per_tile;
  dim3 grid((unsigned)qtiles, (unsigned)a.hkv, (unsigned)a.batch);
  kern<<<grid, kTcThreads, kTcSmemBytes, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool prefill_tc_supported(const PrefillArgs& a, int dtype) {
  if (dtype != MI_BF16 && dtype != MI_F16) return false;
  if (a.head_dim != kTcDim) return false;
  if (!(a.groups == 1 || a.groups == 2 || a.groups == 4 || a.groups == 8)) return false;
  if (a.batch > 65535 || a.hkv > 65535) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a.q) || !al16(a.k_chunk) || !al16(a.v_chunk) || !al16(a.out)) return false;
  if (a.table_stride > 0 && (!al16(a.k_pool) || !al16(a.v_pool))) return false;
  for (int i = 0; i < 3; ++i)
    if ((a.q_sb[i] & 15) || (a.kv_sb[i] & 15)) return false;
  return true;
}

cudaError_t launch_paged_prefill_tc(const PrefillArgs& a, int dtype, cudaStream_t s) {
  if (dtype == MI_BF16) return launch_tc<__nv_bfloat16>(a, s);
  return launch_tc<__half>(a, s);
}

}  // namespace mi
