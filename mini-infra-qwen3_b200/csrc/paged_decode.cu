// Paged decode attention (one query token per sequence, GQA), sm_100a.
//
// Split kernel (bf16/fp16, head_dim 64/128, block_size a multiple of 16, G <= 8):
//   grid = (splits, kv-head blocks, batch); 4 consumer warps + 1 TMA producer warp per CTA.
//   The producer warp walks the split's pages of the block table and stages each page of each KV
//   head with non-multicast TMA tensor loads ([64 x 1 x block_size] boxes, 128-byte swizzle), one
//   box per lane, into an NSTAGE-deep shared-memory ring guarded by full/empty mbarriers; each lane
//   reads its next page's block id one stage ahead.  Each consumer warp owns one
//   KV head: its G query heads sit in mma.sync A fragments (rows = query heads), QK^T and PV run as
//   m16n8k16 tensor-core tiles with fp32 accumulation, and the online softmax (exp2 domain) keeps
//   its row max/sum in registers with quad shuffles.  Each warp writes an unnormalised partial
//   (m, l, acc[D]) per split to the workspace.
// Combine kernel: one warp per (sequence, query head) merges the partials (log-sum-exp) and
//   writes the bf16/fp16/fp32 output row.
// Scalar kernel (every other case, incl. fp32): one warp per (sequence, query head), lanes split
//   head_dim, single pass online softmax in fp32, reads the pool directly through the table.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace mi {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSmemTarget = 100 * 1024;  // two CTAs per SM

template <int D, int BS, int HB, int TG>
struct DecodeShape {
  static constexpr int kChunks = D / 64;                    // 128-byte column chunks of a row
  static constexpr int kChunkBytes = BS * 128;              // one chunk of one head's page
  static constexpr int kHeadPageBytes = kChunks * kChunkBytes;  // K (or V) page of one head
  static constexpr int kStageBytes = TG * HB * 2 * kHeadPageBytes;
  static constexpr int kStages = std::max(2, std::min(8, kSmemTarget / kStageBytes));
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 2 * kStages * 8;
};

template <typename T, int D, int BS, int HB, int TG>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                                const __grid_constant__ CUtensorMap tm_v,
                                                                const DecodeArgs a) {
  using S = DecodeShape<D, BS, HB, TG>;
  constexpr int NST = S::kStages;
  // Launched as a programmatic dependent of the stream's previous kernel (typically the one that
  // appended this step's K/V): nothing is read before that kernel has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + NST * S::kStageBytes);
  uint64_t* empty_bar = full_bar + NST;

  const int split = blockIdx.x;
  const int head_block = blockIdx.y;
  const int64_t b = blockIdx.z;
  int64_t ctx = a.context_lens[b];
  int64_t n_pages = ctx > 0 ? (ctx + BS - 1) / BS : 0;
  if (n_pages > a.max_blocks) {
    if (threadIdx.x == 0 && split == 0) record_status(MI_STATUS_BAD_LENGTH);
    n_pages = a.max_blocks;
    ctx = n_pages * BS;
  }
  const int64_t page_begin = (int64_t)split * a.split_pages;
  if (page_begin >= n_pages) return;  // uniform for the CTA
  const int64_t page_end = min(n_pages, page_begin + (int64_t)a.split_pages);
  const int n_iter = (int)((page_end - page_begin + TG - 1) / TG);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  bool aborted = false;

  if (warp == kConsumerWarps) {
    // ---------------- TMA producer: one box per lane ----------------
    // A stage is TG pages x HB heads x {K, V} x kChunks boxes of [64 x 1 x BS]; lane L issues box L
    // (page L / kBoxesPerPage).  Each lane loads the block id of its page one stage ahead, so the
    // table reads overlap the wait for a free stage instead of sitting between the wait and the
    // copies.
    constexpr int kBoxesPerPage = HB * 2 * S::kChunks;
    static_assert(TG * kBoxesPerPage <= 32, "one box per lane");
    const int my_page = lane / kBoxesPerPage;
    const int rem = lane - my_page * kBoxesPerPage;
    const int hl = rem / (2 * S::kChunks);
    const bool is_v = (rem / S::kChunks) & 1;
    const int c = rem % S::kChunks;
    const bool has_box = my_page < TG;
    const int64_t* table = a.block_tables + b * a.table_stride;
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    int64_t next_blk = 0;
    if (has_box && page_begin + my_page < page_end) next_blk = table[page_begin + my_page];
    for (int it = 0; it < n_iter; ++it) {
      const int st = it % NST;
      if (it >= NST) {
        mbar_wait(&empty_bar[st], ((it / NST) - 1) & 1, aborted);
        aborted = __any_sync(0xffffffffu, aborted);
      }
      const int64_t first = page_begin + (int64_t)it * TG;
      const int npg = (int)min((int64_t)TG, page_end - first);
      int64_t blk = next_blk;
      const int64_t ahead = first + TG + my_page;  // this lane's page of the next stage
      if (has_box && it + 1 < n_iter && ahead < page_end) next_blk = table[ahead];
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[st], (uint32_t)(npg * HB * 2 * S::kHeadPageBytes));
      __syncwarp();
      if (has_box && my_page < npg) {
        if (blk < 0 || blk >= a.num_blocks) {
          record_status(MI_STATUS_BAD_BLOCK);
          blk = a.num_blocks;  // outside the tensor map: TMA fills zeros
        }
        uint8_t* dst = smem + st * S::kStageBytes + ((my_page * HB + hl) * 2 + (is_v ? 1 : 0)) * S::kHeadPageBytes +
                       c * S::kChunkBytes;
        tma_load_3d(dst, is_v ? &tm_v : &tm_k, &full_bar[st], c * 64, head_block * HB + hl, (int)(blk * BS));
      }
    }
    return;
  }

  // ---------------- consumers: one warp per (KV head, page lane) ----------------
  const int hl = warp / TG;
  const int tg = warp % TG;
  const int h = head_block * HB + hl;
  const int r = lane >> 2;  // mma row = query head within the group
  const int q4 = lane & 3;
  const bool row_valid = r < a.groups;

  constexpr int KS = D / 16;  // k-steps over head_dim
  uint32_t qa[KS][2];
  {
    const char* qp = a.q + b * a.q_sb + (int64_t)(h * a.groups + (row_valid ? r : 0)) * a.q_sh;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const uint32_t lo = *reinterpret_cast<const uint32_t*>(qp + (ks * 16 + 2 * q4) * sizeof(T));
      const uint32_t hi = *reinterpret_cast<const uint32_t*>(qp + (ks * 16 + 8 + 2 * q4) * sizeof(T));
      qa[ks][0] = row_valid ? lo : 0u;
      qa[ks][1] = row_valid ? hi : 0u;
    }
  }

  float o[D / 8][2];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = 0.f;
  float m_run = -INFINITY;
  float l_run = 0.f;
  const float scale = a.scale_log2;

  for (int it = 0; it < n_iter; ++it) {
    const int st = it % NST;
    mbar_wait(&full_bar[st], (it / NST) & 1, aborted);
    const int64_t page = page_begin + (int64_t)it * TG + tg;
    if (page < page_end) {
      const uint8_t* kbase = smem + st * S::kStageBytes + ((tg * HB + hl) * 2) * S::kHeadPageBytes;
      const uint32_t k_addr = smem_u32(kbase);
      const uint32_t v_addr = k_addr + S::kHeadPageBytes;
#pragma unroll
      for (int step = 0; step < BS / 16; ++step) {
        // ---- S = Q K^T for 16 tokens (two n-tiles of 8) ----
        float s0[4] = {0.f, 0.f, 0.f, 0.f};
        float s1[4] = {0.f, 0.f, 0.f, 0.f};
        {
          const int mi = lane >> 3;
          const uint32_t tok = (uint32_t)((mi >> 1) * 8 + (lane & 7) + step * 16);
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            const uint32_t unit = (uint32_t)((ks & 3) * 2 + (mi & 1));
            uint32_t b00, b01, b10, b11;
            ldmatrix_x4(k_addr + (ks >> 2) * S::kChunkBytes + swz128(tok, unit), b00, b01, b10, b11);
            const uint32_t af[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
            Mma16816<T>::run(s0, af, b00, b01);
            Mma16816<T>::run(s1, af, b10, b11);
          }
        }
        // ---- online softmax over the 16 tokens (rows = query heads) ----
        const int64_t tok0 = page * BS + step * 16 + 2 * q4;
        float x0 = (tok0 < ctx) ? s0[0] * scale : -INFINITY;
        float x1 = (tok0 + 1 < ctx) ? s0[1] * scale : -INFINITY;
        float x2 = (tok0 + 8 < ctx) ? s1[0] * scale : -INFINITY;
        float x3 = (tok0 + 9 < ctx) ? s1[1] * scale : -INFINITY;
        float mt = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
        const float m_new = fmaxf(m_run, mt);
        float alpha, p0, p1, p2, p3;
        if (m_new == -INFINITY) {
          alpha = 1.f;
          p0 = p1 = p2 = p3 = 0.f;
        } else {
          alpha = exp2f(m_run - m_new);
          p0 = exp2f(x0 - m_new);
          p1 = exp2f(x1 - m_new);
          p2 = exp2f(x2 - m_new);
          p3 = exp2f(x3 - m_new);
        }
        m_run = m_new;
        l_run = l_run * alpha + ((p0 + p1) + (p2 + p3));
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int i = 0; i < D / 8; ++i) {
            o[i][0] *= alpha;
            o[i][1] *= alpha;
          }
        }
        // ---- O += P V ----
        const uint32_t pa[4] = {pack2<T>(p0, p1), 0u, pack2<T>(p2, p3), 0u};
        {
          const int mi = lane >> 3;
          const uint32_t tok = (uint32_t)((mi & 1) * 8 + (lane & 7) + step * 16);
#pragma unroll
          for (int np = 0; np < D / 16; ++np) {
            const uint32_t unit = (uint32_t)((np & 3) * 2 + (mi >> 1));
            uint32_t v0, v1, v2, v3;
            ldmatrix_x4_trans(v_addr + (np >> 2) * S::kChunkBytes + swz128(tok, unit), v0, v1, v2, v3);
            float c0[4] = {o[2 * np][0], o[2 * np][1], 0.f, 0.f};
            float c1[4] = {o[2 * np + 1][0], o[2 * np + 1][1], 0.f, 0.f};
            Mma16816<T>::run(c0, pa, v0, v1);
            Mma16816<T>::run(c1, pa, v2, v3);
            o[2 * np][0] = c0[0];
            o[2 * np][1] = c0[1];
            o[2 * np + 1][0] = c1[0];
            o[2 * np + 1][1] = c1[1];
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
  }

  // ---- write this warp's partial (rows = query heads of KV head h) ----
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (row_valid) {
    const int part = split * TG + tg;
    const int64_t idx = (b * a.hq + (int64_t)h * a.groups + r) * a.max_parts + part;
    float* dst = a.ws_o + idx * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<float2*>(dst + i * 8 + 2 * q4) = make_float2(o[i][0], o[i][1]);
    }
    if (q4 == 0) *reinterpret_cast<float2*>(a.ws_ml + idx * 2) = make_float2(m_run, l_run);
  }
}

// One warp per (sequence, query head): merge the split partials and write the output row.
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_combine_kernel(const DecodeArgs a) {
  constexpr int PER_LANE = D / 32;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // programmatic dependent of the split kernel
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= a.batch * a.hq) return;
  const int64_t b = gw / a.hq;
  const int hq = (int)(gw - b * a.hq);
  int64_t ctx = a.context_lens[b];
  int64_t n_pages = ctx > 0 ? (ctx + a.block_size - 1) / a.block_size : 0;
  n_pages = min(n_pages, a.max_blocks);
  const int n_parts = (int)((n_pages + a.split_pages - 1) / a.split_pages) * a.parts_per_split;
  const int64_t base = gw * a.max_parts;
  float m_all = -INFINITY;
  for (int p = lane; p < n_parts; p += 32) m_all = fmaxf(m_all, a.ws_ml[(base + p) * 2]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m_all = fmaxf(m_all, __shfl_xor_sync(0xffffffffu, m_all, off));
  float acc[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) acc[i] = 0.f;
  float l_all = 0.f;
  if (m_all != -INFINITY) {
    // lane j weighs part p0 + j; the O rows of 32 parts are then read with independent loads
    for (int p0 = 0; p0 < n_parts; p0 += 32) {
      float w = 0.f;
      if (p0 + lane < n_parts) {
        const float2 ml = *reinterpret_cast<const float2*>(a.ws_ml + (base + p0 + lane) * 2);
        w = exp2f(ml.x - m_all);
        l_all += w * ml.y;
      }
      const int cnt = min(32, n_parts - p0);
#pragma unroll 4
      for (int j = 0; j < cnt; ++j) {
        const float wj = __shfl_sync(0xffffffffu, w, j);
        const float* src = a.ws_o + (base + p0 + j) * D + lane * PER_LANE;
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) acc[i] += wj * src[i];
      }
    }
    l_all = warp_sum(l_all);
  }
  const float inv = l_all > 0.f ? 1.f / l_all : 0.f;
  if (a.world == 0) {
    T* dst = reinterpret_cast<T*>(a.out + b * a.out_sb) + (int64_t)hq * D + lane * PER_LANE;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) dst[i] = Elem<T>::from_f(acc[i] * inv);
    return;
  }
  // Exchange: the row slice goes to every rank's gathered buffer (peer stores over NVLink), one
  // vector store per lane and destination; the system-scope fence orders them before the barrier
  // kernel's release of this rank's flag.
  static_assert(PER_LANE * sizeof(T) == 8 || PER_LANE * sizeof(T) == 4, "16-bit rows of 64 or 128");
  using Vec = typename std::conditional<PER_LANE * sizeof(T) == 8, uint2, uint32_t>::type;
  union {
    Vec v;
    T e[PER_LANE];
  } pk;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) pk.e[i] = Elem<T>::from_f(acc[i] * inv);
  const int64_t col = ((int64_t)a.rank * a.hq + hq) * D + lane * PER_LANE;
  for (int p = 0; p < a.world; ++p)
    *reinterpret_cast<Vec*>(reinterpret_cast<T*>(a.gathered[p] + b * a.gathered_sb) + col) = pk.v;
  __threadfence_system();
}

// Barrier after an exchange: one warp, lane p signals and then waits for peer p.
__global__ void __launch_bounds__(32) peer_barrier_kernel(const PeerBarrierArgs a) {
  const int p = threadIdx.x;
  // Launched as a programmatic dependent of the combine kernel: placed while the combine drains,
  // it waits here for the combine's completion (its peer stores performed) before signalling.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  const unsigned int e = *reinterpret_cast<volatile unsigned int*>(a.epoch) + 1u;
  if (p < a.world && p != a.rank) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flags[p] + a.rank), "r"(e) : "memory");
    const unsigned int* mine = a.flags[a.rank] + p;
    const uint64_t start = globaltimer_ns();
    while (true) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int)(v - e) >= 0) break;
      if (globaltimer_ns() - start > a.timeout_ns) {
        record_status(MI_STATUS_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
  if (p == 0) *a.epoch = e;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Generic single-pass kernel: one warp per (sequence, query head); any dtype, head_dim <= 256,
// any block size.  Reads K/V rows straight from the pool through the block table.
template <typename T>
__global__ void __launch_bounds__(128) decode_scalar_kernel(const DecodeArgs a) {
  constexpr int MAXD = 256 / 32;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= a.batch * a.hq) return;
  const int64_t b = gw / a.hq;
  const int hq = (int)(gw - b * a.hq);
  const int h = hq / a.groups;
  const int D = a.head_dim;
  int64_t ctx = a.context_lens[b];
  if (ctx < 0) ctx = 0;
  if (ctx > a.max_blocks * a.block_size) {
    if (lane == 0) record_status(MI_STATUS_BAD_LENGTH);
    ctx = a.max_blocks * a.block_size;
  }
  const T* q = reinterpret_cast<const T*>(a.q + b * a.q_sb + (int64_t)hq * a.q_sh);
  float qv[MAXD], acc[MAXD];
#pragma unroll
  for (int i = 0; i < MAXD; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < D ? Elem<T>::to_f(q[d]) : 0.f;
    acc[i] = 0.f;
  }
  const int64_t* table = a.block_tables + b * a.table_stride;
  const int64_t row_elems = (int64_t)a.hkv * D;
  const T* kp = reinterpret_cast<const T*>(a.k_pool);
  const T* vp = reinterpret_cast<const T*>(a.v_pool);
  float m_run = -INFINITY, l_run = 0.f;
  for (int64_t t = 0; t < ctx; ++t) {
    int64_t blk = table[t / a.block_size];
    if (blk < 0 || blk >= a.num_blocks) {
      if (lane == 0) record_status(MI_STATUS_BAD_BLOCK);
      continue;
    }
    const int64_t off = (blk * a.block_size + t % a.block_size) * row_elems + (int64_t)h * D;
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < MAXD; ++i) {
      const int d = lane + 32 * i;
      if (d < D) part += qv[i] * Elem<T>::to_f(kp[off + d]);
    }
    const float s = warp_sum(part) * a.scale_log2;
    const float m_new = fmaxf(m_run, s);
    const float alpha = exp2f(m_run - m_new);
    const float p = exp2f(s - m_new);
    l_run = l_run * alpha + p;
#pragma unroll
    for (int i = 0; i < MAXD; ++i) {
      const int d = lane + 32 * i;
      if (d < D) acc[i] = acc[i] * alpha + p * Elem<T>::to_f(vp[off + d]);
    }
    m_run = m_new;
  }
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
  T* dst = reinterpret_cast<T*>(a.out + b * a.out_sb) + (int64_t)hq * D;
#pragma unroll
  for (int i = 0; i < MAXD; ++i) {
    const int d = lane + 32 * i;
    if (d < D) dst[d] = Elem<T>::from_f(acc[i] * inv);
  }
}

template <typename T, int D, int BS, int HB, int TG>
cudaError_t launch_split(const DecodeArgs& a, const CUtensorMap* tk, const CUtensorMap* tv, cudaStream_t s) {
  using S = DecodeShape<D, BS, HB, TG>;
  auto kern = decode_split_kernel<T, D, BS, HB, TG>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
  if (e != cudaSuccess) return e;
  // Both launches are programmatic dependents of their predecessor (their CTAs are placed while it
  // drains; each kernel waits for it before touching memory).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.max_splits, (unsigned)(a.hkv / HB), (unsigned)a.batch);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::kSmemBytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, *tk, *tv, a);
  if (e != cudaSuccess) return e;
  const int64_t warps = a.batch * a.hq;
  cfg.gridDim = dim3((unsigned)((warps + 3) / 4));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&cfg, decode_combine_kernel<T, D>, a);
}

template <typename T, int D, int BS>
cudaError_t launch_split_hb(const DecodeArgs& a, int hb, const CUtensorMap* tk, const CUtensorMap* tv,
                            cudaStream_t s) {
  switch (hb) {
    case 4: return launch_split<T, D, BS, 4, 1>(a, tk, tv, s);
    case 2: return launch_split<T, D, BS, 2, 2>(a, tk, tv, s);
    default: return launch_split<T, D, BS, 1, 4>(a, tk, tv, s);
  }
}

template <typename T>
cudaError_t launch_split_t(const DecodeArgs& a, const DecodePlan& p, const CUtensorMap* tk, const CUtensorMap* tv,
                           cudaStream_t s) {
  if (a.head_dim == 128) {
    if (a.block_size == 16) return launch_split_hb<T, 128, 16>(a, p.heads_per_cta, tk, tv, s);
    return launch_split_hb<T, 128, 32>(a, p.heads_per_cta, tk, tv, s);
  }
  if (a.block_size == 16) return launch_split_hb<T, 64, 16>(a, p.heads_per_cta, tk, tv, s);
  return launch_split_hb<T, 64, 32>(a, p.heads_per_cta, tk, tv, s);
}

}  // namespace

cudaError_t launch_peer_barrier(const PeerBarrierArgs& a, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, peer_barrier_kernel, a);
}

DecodePlan plan_decode(int64_t batch, int hq, int hkv, int head_dim, int64_t max_blocks, int block_size, int dtype) {
  DecodePlan p{};
  const int groups = hkv > 0 ? hq / hkv : 0;
  p.use_mma = (dtype == MI_BF16 || dtype == MI_F16) && (head_dim == 64 || head_dim == 128) &&
              (block_size == 16 || block_size == 32) && groups >= 1 && groups <= 8;
  if (!p.use_mma) {
    p.heads_per_cta = 1;
    p.parts_per_split = 1;
    p.split_pages = (int)std::max<int64_t>(1, max_blocks);
    p.max_splits = 1;
    p.ws_bytes = 0;
    return p;
  }
  p.heads_per_cta = (hkv % 4 == 0) ? 4 : (hkv % 2 == 0) ? 2 : 1;
  p.parts_per_split = 4 / p.heads_per_cta;
  // Splits of ~512 tokens x 4 KV heads of K/V per CTA (512 tokens at HB = 4, 2048 at HB = 1, so a
  // CTA's bytes do not shrink with the heads it holds) balance long and short sequences; shrink
  // them when the grid would be too small to cover the 148 SMs twice.
  const int64_t ctas_per_split = batch * (hkv / p.heads_per_cta);
  int64_t split_pages = std::max<int64_t>(p.parts_per_split, 512 * (4 / p.heads_per_cta) / block_size);
  const int64_t target_ctas = 2 * 148 * 2;
  while (split_pages > p.parts_per_split &&
         ctas_per_split * ((max_blocks + split_pages - 1) / split_pages) < target_ctas) {
    split_pages = std::max<int64_t>(p.parts_per_split, split_pages / 2);
  }
  p.split_pages = (int)std::min<int64_t>(split_pages, std::max<int64_t>(1, max_blocks));
  p.max_splits = (int)std::max<int64_t>(1, (max_blocks + p.split_pages - 1) / p.split_pages);
  const int64_t parts = (int64_t)p.max_splits * p.parts_per_split;
  const size_t o_bytes = (size_t)batch * hq * parts * head_dim * sizeof(float);
  const size_t ml_bytes = (size_t)batch * hq * parts * 2 * sizeof(float);
  p.ws_bytes = ((o_bytes + 255) & ~size_t(255)) + ((ml_bytes + 255) & ~size_t(255));
  return p;
}

cudaError_t launch_paged_decode(const DecodeArgs& a, const DecodePlan& plan, const CUtensorMap* tm_k,
                                const CUtensorMap* tm_v, int dtype, cudaStream_t s) {
  if (a.batch == 0) return cudaSuccess;
  if (plan.use_mma) {
    if (dtype == MI_BF16) return launch_split_t<__nv_bfloat16>(a, plan, tm_k, tm_v, s);
    return launch_split_t<__half>(a, plan, tm_k, tm_v, s);
  }
  const int64_t warps = a.batch * a.hq;
  const unsigned blocks = (unsigned)((warps + 3) / 4);
  switch (dtype) {
    case MI_BF16: decode_scalar_kernel<__nv_bfloat16><<<blocks, 128, 0, s>>>(a); break;
    case MI_F16: decode_scalar_kernel<__half><<<blocks, 128, 0, s>>>(a); break;
    default: decode_scalar_kernel<float><<<blocks, 128, 0, s>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace mi
