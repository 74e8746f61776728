// mi_paged_decode_static_scratch: the paged decode entry point for callers that cannot allocate
// device memory on the call path.
//
// Who needs it: hosts that bind the C ABI without any device allocator of their own (a C, Go or
// JNI caller has no caching allocator to hand a workspace from), and latency-critical loops that
// cannot afford cudaMalloc's implicit device synchronisation.  The regular entry point
// (mi_paged_decode) needs a caller-provided split-K workspace; this one uses a fixed scratch array
// compiled into the library instead and allocates nothing.
//
// The scratch array is a file-scope __device__ array of MI_STATIC_SCRATCH_BYTES (32 MiB).  Every GPU
// that loads this library holds it until the process exits.  Host code must not pass the array's
// name to a kernel (in host code that name is only a stand-in for the device symbol); the device
// address is looked up once per device with cudaGetSymbolAddress, with that device current, the
// first time this entry point runs on it — so make the first call on each device before any
// stream capture begins.  The cached address outlives a cudaDeviceReset of that device, after which
// it names a released module: this entry point must not be called on a device after resetting it.
// All calls share the array and it keeps the previous call's contents: nothing in it needs to
// start at zero (each split partial the combine step reads is written by the same call first), but
// calls that overlap on the GPU — two streams, or two host threads — race on it and must be
// serialised by the caller.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr size_t kStaticScratchBytes = MI_STATIC_SCRATCH_BYTES;  // 32 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (looked up once per device).
int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "mi_paged_decode_static_scratch: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(MI_ERR_UNSUPPORTED, "mi_paged_decode_static_scratch: device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "mi_paged_decode_static_scratch: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MI_OK;
}

}  // namespace

extern "C" {

int mi_paged_decode_static_scratch(const void* q, const int64_t* q_strides, const void* k_new, const void* v_new,
                                   const int64_t* new_strides, const int64_t* slot_mapping, void* k_pool,
                                   void* v_pool, int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                                   const int64_t* block_tables, int64_t table_stride, int64_t max_blocks_per_seq,
                                   const int64_t* context_lens, int64_t batch, int num_q_heads, float scale,
                                   void* out, int64_t out_stride, int dtype, void* stream) {
  if (batch > 0 && num_kv_heads > 0 && num_q_heads > 0) {
    const size_t need = mi::plan_decode(batch, num_q_heads, num_kv_heads, head_dim, max_blocks_per_seq, block_size,
                                        dtype)
                            .ws_bytes;
    if (need > kStaticScratchBytes)
      return fail(MI_ERR_UNSUPPORTED,
                  "mi_paged_decode_static_scratch: this call needs %zu bytes of split-K scratch but the static "
                  "scratch array holds %zu; use mi_paged_decode with a caller workspace",
                  need, kStaticScratchBytes);
  }
  void* scratch = nullptr;
  if (int rc = static_scratch_address(&scratch)) return rc;
  return mi_paged_decode(q, q_strides, k_new, v_new, new_strides, slot_mapping, k_pool, v_pool, num_blocks,
                         block_size, num_kv_heads, head_dim, block_tables, table_stride, max_blocks_per_seq,
                         context_lens, batch, num_q_heads, scale, out, out_stride, scratch, kStaticScratchBytes, dtype,
                         stream);
}

}  // extern "C"
