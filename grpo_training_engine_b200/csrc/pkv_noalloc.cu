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
// device address, so the first call in each CUDA context looks its address up
// with cudaGetSymbolAddress (with that context current) and caches it under the
// context's unique id: a __device__ variable has one address per context, so a
// context made with the driver API, or a primary context re-created after
// cudaDeviceReset, gets its own lookup instead of a stale address. That first
// call should come before any stream capture. All calls share the one array
// and leave their data in it; each call's plan kernel rewrites every field the
// decode reads (including the scheduling counters), so nothing has to be
// cleared between calls, but calls that overlap on the GPU (e.g. on two
// streams at once) race on it and must be serialised by the caller.
#include <mutex>

#include "pkv_common.cuh"

namespace {

static __device__ __align__(256) uint8_t g_decode_scratch[PKV_NOALLOC_SCRATCH_BYTES];

// Driver entry points resolved through the runtime (the library does not link
// libcuda): the current context and its process-unique id.
using CtxGetCurrentFn = int (*)(void **ctx);
using CtxGetIdFn = int (*)(void *ctx, unsigned long long *id);

struct ScratchEntry {
  unsigned long long ctx_id;
  void *ptr;
};
constexpr int kMaxContexts = 64;
std::mutex g_scratch_mu;
ScratchEntry g_scratch[kMaxContexts] = {};
int g_scratch_used = 0;
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;
bool g_entry_points_tried = false;

void resolve_entry_points() {
  if (g_entry_points_tried) return;
  g_entry_points_tried = true;
  void *f = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(f);
  f = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_id = reinterpret_cast<CtxGetIdFn>(f);
  cudaGetLastError();
}

// Unique id of the context current on this thread, 0 when none is current or
// the driver cannot say.
unsigned long long current_context_id() {
  if (g_ctx_current == nullptr || g_ctx_id == nullptr) return 0;
  void *ctx = nullptr;
  if (g_ctx_current(&ctx) != 0 || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (g_ctx_id(ctx, &id) != 0) return 0;
  return id;
}

// Device address of g_decode_scratch in the current context (looked up once
// per context; looked up on every call if the context cannot be identified).
int scratch_in_current_context(void **out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  resolve_entry_points();
  unsigned long long id = current_context_id();
  if (id != 0) {
    for (int i = 0; i < g_scratch_used; ++i) {
      if (g_scratch[i].ctx_id == id) {
        *out = g_scratch[i].ptr;
        return PKV_OK;
      }
    }
  }
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess || p == nullptr) {
    int dev = -1;
    cudaGetDevice(&dev);
    pkv::set_error_detail("pkv_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                          cudaGetErrorString(e));
    cudaGetLastError();
    return PKV_ERR_CUDA;
  }
  // the lookup made the runtime's context current if none was
  if (id == 0) id = current_context_id();
  if (id != 0) {
    const int slot = g_scratch_used < kMaxContexts ? g_scratch_used++ : (int)(id % kMaxContexts);
    g_scratch[slot] = ScratchEntry{id, p};
  }
  *out = p;
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
  const int rc = scratch_in_current_context(&ws);
  if (rc) return rc;
  return pkv_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch, num_q_heads,
                    num_kv_heads, head_dim, block_size, num_blocks, max_blocks, q_strides,
                    cache_strides, bt_strides, out_strides, q_dtype, kv_dtype, scale,
                    pages_per_split, flags, ws, (size_t)PKV_NOALLOC_SCRATCH_BYTES, status, stream);
}
