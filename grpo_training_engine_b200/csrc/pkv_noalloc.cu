// pkv_noalloc.cu — decode attention with library-owned scratch, for callers
// that cannot allocate device memory.
//
// pkv_decode needs a workspace (the split plan and the split-K partials) that
// the caller allocates. Some callers cannot do that: an FFI host that only
// hands over the tensors it already owns, or a process whose GPU memory
// belongs to another framework's allocator (which may hold nearly all of it,
// so a direct cudaMalloc fails or fragments its pool). pkv_decode_noalloc
// serves them from a fixed scratch array compiled into this library.
//
// The array is a file-scope __device__ variable: every GPU on which the
// library's device code is loaded keeps PKV_NOALLOC_SCRATCH_BYTES of memory
// for it until the process exits. Host code cannot use the array's name as a
// device address, so the first call on each device looks its address up with
// cudaGetSymbolAddress (with that device current) and caches it; that first
// call should come before any stream capture. All calls share the one array
// and leave their data in it; each call's plan kernel rewrites every field the
// decode reads (including the scheduling counters), so nothing has to be
// cleared between calls, but calls that overlap on the GPU (e.g. on two
// streams at once) race on it and must be serialised by the caller.
#include <mutex>

#include "pkv_common.cuh"

namespace {

static __device__ __align__(256) uint8_t g_decode_scratch[PKV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (set up once per device).
int scratch_on_current_device(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    pkv::set_error_detail("pkv_decode_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    pkv::set_error_detail("pkv_decode_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
    return PKV_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      pkv::set_error_detail("pkv_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                            cudaGetErrorString(e));
      return PKV_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PKV_OK;
}

}  // namespace

extern "C" int pkv_decode_noalloc(const void *q, const void *k_cache, const void *v_cache,
                                  const int32_t *block_tables, const int32_t *context_lens,
                                  float *out, int32_t batch, int32_t num_q_heads,
                                  int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                  int32_t num_blocks, int32_t max_blocks,
                                  const int64_t *q_strides, const int64_t *cache_strides,
                                  const int64_t *bt_strides, const int64_t *out_strides,
                                  int32_t q_dtype, int32_t kv_dtype, float scale,
                                  int32_t pages_per_split, int32_t flags, int32_t *status,
                                  void *stream) {
  const size_t need = pkv_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim,
                                                max_blocks, pages_per_split);
  if (need == 0) {
    pkv::set_error_detail("pkv_decode_noalloc: invalid sizes");
    return PKV_ERR_INVALID_ARG;
  }
  if (need > (size_t)PKV_NOALLOC_SCRATCH_BYTES) {
    pkv::set_error_detail(
        "pkv_decode_noalloc: this decode needs %zu bytes of scratch but the library's static "
        "scratch holds %zu; use pkv_decode with a caller-allocated workspace",
        need, (size_t)PKV_NOALLOC_SCRATCH_BYTES);
    return PKV_ERR_WORKSPACE;
  }
  void *ws = nullptr;
  const int rc = scratch_on_current_device(&ws);
  if (rc) return rc;
  return pkv_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch, num_q_heads,
                    num_kv_heads, head_dim, block_size, num_blocks, max_blocks, q_strides,
                    cache_strides, bt_strides, out_strides, q_dtype, kv_dtype, scale,
                    pages_per_split, flags, ws, (size_t)PKV_NOALLOC_SCRATCH_BYTES, status, stream);
}
