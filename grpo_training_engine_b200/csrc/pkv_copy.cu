// pkv_copy.cu — page append, bulk prompt append and dense gather (sm_100a).
//
// These three kernels move K/V payload bit for bit between dense tensors and
// the paged cache; none of them does arithmetic on the payload. One thread
// moves one 16-byte vector when every row is 16-byte aligned and
// contiguous in head_dim, otherwise one element, so the kernels are plain
// coalesced HBM streams. The addressing follows the reference:
//   append   src/triton_kernels/paged_kv.py:277-319 (slot = pre-append length)
//   prompt   src/triton_kernels/paged_kv.py:576-586 (position pos of sequence b)
//   gather   src/triton_kernels/paged_kv.py:98-131  (block_tables[b, t // bs], t % bs)
#include <stdarg.h>
#include <stdio.h>

#include "pkv_common.cuh"

namespace pkv {

static thread_local char g_detail[512] = "";

void set_error_detail(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_detail, sizeof(g_detail), fmt, ap);
  va_end(ap);
}

namespace {

constexpr int kCopyThreads = 256;

// Raw-bit vector types: a copy through them is bit exact for every dtype.
template <int BYTES> struct RawVec;
template <> struct RawVec<2> { using T = uint16_t; };
template <> struct RawVec<4> { using T = uint32_t; };
template <> struct RawVec<16> { using T = uint4; };

struct CopyGeom {
  int32_t batch, heads, tokens, chunks;  // chunks = head_dim / elements per vector
  int32_t block_size, num_blocks, max_blocks;
  int64_t s0, s1, s2, s3;  // dense-side strides (vector units) [B,H,(T),D]
  int64_t c0, c1, c2, c3;  // cache strides (vector units)
  int64_t bt0, bt1;        // block-table strides (elements)
  int32_t ctx_offset;      // append: slot = context_lens[b] + ctx_offset (0: pre-append lengths)
};

// Looks up the page of position `pos` of sequence b; -1 if out of range.
__device__ __forceinline__ int32_t page_of(const int32_t *bt, const CopyGeom &g, int32_t b,
                                           int32_t pos, int32_t *status, bool report) {
  if (pos < 0 || pos >= g.max_blocks * g.block_size) {
    if (report) flag_status(status, PKV_DEV_CTX_OUT_OF_RANGE);
    return -1;
  }
  int32_t page = bt[b * g.bt0 + (int64_t)(pos / g.block_size) * g.bt1];
  if (page < 0 || page >= g.num_blocks) {
    if (report) flag_status(status, PKV_DEV_PAGE_OUT_OF_RANGE);
    return -1;
  }
  return page;
}

template <typename V>
__global__ void __launch_bounds__(kCopyThreads)
append_kernel(const V *__restrict__ k_new, const V *__restrict__ v_new, V *__restrict__ kc,
              V *__restrict__ vc, const int32_t *__restrict__ bt, const int32_t *__restrict__ ctx,
              CopyGeom g, int32_t *status) {
  const int64_t total = (int64_t)g.batch * g.heads * g.chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t c = (int32_t)(i % g.chunks);
    const int64_t row = i / g.chunks;
    const int32_t h = (int32_t)(row % g.heads);
    const int32_t b = (int32_t)(row / g.heads);
    // with post-append lengths (ctx_offset -1) an empty sequence has no new token
    if (g.ctx_offset < 0 && ctx[b] <= 0) continue;
    const int32_t pos = ctx[b] + g.ctx_offset;
    const int32_t page = page_of(bt, g, b, pos, status, c == 0);
    if (page < 0) continue;
    const int64_t dst = page * g.c0 + h * g.c1 + (int64_t)(pos % g.block_size) * g.c2 + c * g.c3;
    const int64_t src = b * g.s0 + h * g.s1 + c * g.s3;
    kc[dst] = k_new[src];
    vc[dst] = v_new[src];
  }
}

template <typename V>
__global__ void __launch_bounds__(kCopyThreads)
append_prompt_kernel(const V *__restrict__ ks, const V *__restrict__ vs, V *__restrict__ kc,
                     V *__restrict__ vc, const int32_t *__restrict__ bt,
                     const int32_t *__restrict__ start, const int32_t *__restrict__ lens,
                     CopyGeom g, int32_t *status) {
  const int64_t total = (int64_t)g.batch * g.heads * g.tokens * g.chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t c = (int32_t)(i % g.chunks);
    int64_t r = i / g.chunks;
    const int32_t t = (int32_t)(r % g.tokens);
    r /= g.tokens;
    const int32_t h = (int32_t)(r % g.heads);
    const int32_t b = (int32_t)(r / g.heads);
    const int32_t n = lens ? lens[b] : g.tokens;
    if (t >= n) continue;
    const int32_t pos = (start ? start[b] : 0) + t;
    const int32_t page = page_of(bt, g, b, pos, status, c == 0);
    if (page < 0) continue;
    const int64_t dst = page * g.c0 + h * g.c1 + (int64_t)(pos % g.block_size) * g.c2 + c * g.c3;
    const int64_t src = b * g.s0 + h * g.s1 + t * g.s2 + c * g.s3;
    kc[dst] = ks[src];
    vc[dst] = vs[src];
  }
}

template <typename V>
__global__ void __launch_bounds__(kCopyThreads)
gather_kernel(const V *__restrict__ kc, const V *__restrict__ vc, const int32_t *__restrict__ bt,
              const int32_t *__restrict__ ctx, V *__restrict__ ko, V *__restrict__ vo, CopyGeom g,
              int32_t *status) {
  const int64_t total = (int64_t)g.batch * g.heads * g.tokens * g.chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t c = (int32_t)(i % g.chunks);
    int64_t r = i / g.chunks;
    const int32_t t = (int32_t)(r % g.tokens);
    r /= g.tokens;
    const int32_t h = (int32_t)(r % g.heads);
    const int32_t b = (int32_t)(r / g.heads);
    const int64_t dst = b * g.s0 + h * g.s1 + t * g.s2 + c * g.s3;
    int32_t n = ctx[b];
    const int32_t cap = g.max_blocks * g.block_size;
    if (n < 0 || n > cap) {
      if (t == 0 && h == 0 && c == 0) flag_status(status, PKV_DEV_CTX_OUT_OF_RANGE);
      n = n < 0 ? 0 : cap;
    }
    V kv{}, vv{};
    if (t < n) {
      const int32_t page = page_of(bt, g, b, t, status, c == 0);
      if (page >= 0) {
        const int64_t src = page * g.c0 + h * g.c1 + (int64_t)(t % g.block_size) * g.c2 + c * g.c3;
        kv = kc[src];
        vv = vc[src];
      }
    }
    ko[dst] = kv;
    vo[dst] = vv;
  }
}

// Chooses the widest vector (16 B or one element) that every pointer and
// stride allows. Strides are converted to vector units.
struct VecPlan {
  int vec_bytes;
  int elems_per_vec;
};

bool strides_allow(const int64_t *s, int n, int64_t elems_per_vec) {
  for (int i = 0; i < n - 1; ++i)
    if (s[i] % elems_per_vec != 0) return false;
  return s[n - 1] == 1;
}

VecPlan pick_vector(int esize, int32_t head_dim, const void *const *ptrs, int nptrs,
                    const int64_t *sa, int na, const int64_t *sb, int nb) {
  const int epv = 16 / esize;
  bool ok = head_dim % epv == 0 && strides_allow(sa, na, epv) && strides_allow(sb, nb, epv);
  for (int i = 0; ok && i < nptrs; ++i) ok = aligned_to(ptrs[i], 16);
  if (ok) return {16, epv};
  return {esize, 1};
}

int grid_for(int64_t total) {
  int64_t blocks = (total + kCopyThreads - 1) / kCopyThreads;
  if (blocks < 1) blocks = 1;
  if (blocks > (1 << 20)) blocks = 1 << 20;  // grid-stride loop covers the rest
  return (int)blocks;
}

int check_common(int32_t dtype, int32_t batch, int32_t heads, int32_t head_dim, int32_t bs,
                 int32_t num_blocks, int32_t max_blocks, const int64_t *cache_strides,
                 const int64_t *bt_strides) {
  if (dtype_size(dtype) == 0) {
    set_error_detail("unsupported dtype code %d", dtype);
    return PKV_ERR_UNSUPPORTED;
  }
  if (batch < 0 || heads <= 0 || head_dim <= 0 || bs <= 0 || num_blocks < 0 || max_blocks < 0) {
    set_error_detail("invalid sizes: batch=%d heads=%d head_dim=%d block_size=%d num_blocks=%d "
                     "max_blocks=%d",
                     batch, heads, head_dim, bs, num_blocks, max_blocks);
    return PKV_ERR_INVALID_ARG;
  }
  if (cache_strides == nullptr || bt_strides == nullptr) {
    set_error_detail("stride arrays must not be NULL");
    return PKV_ERR_INVALID_ARG;
  }
  if ((int64_t)max_blocks * bs > INT32_MAX) {
    set_error_detail("max_blocks * block_size overflows int32");
    return PKV_ERR_INVALID_ARG;
  }
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_abi_version(void) { return PKV_ABI_VERSION; }

extern "C" const char *pkv_error_string(int status) {
  switch (status) {
    case PKV_OK: return "ok";
    case PKV_ERR_INVALID_ARG: return "invalid argument";
    case PKV_ERR_UNSUPPORTED: return "unsupported dtype or shape";
    case PKV_ERR_ALIGNMENT: return "misaligned pointer";
    case PKV_ERR_WORKSPACE: return "workspace missing or too small";
    case PKV_ERR_CUDA: return "CUDA error";
    case PKV_ERR_TENSOR_MAP: return "tensor map encoding failed";
    default: return "unknown status";
  }
}

extern "C" const char *pkv_last_error_detail(void) { return g_detail; }

namespace pkv {

// Append launcher shared by pkv_append (slot = pre-append length, ctx_offset 0)
// and the fused append + decode fallback (post-append lengths, ctx_offset -1).
int append_launch(const void *k_new, const void *v_new, void *k_cache, void *v_cache,
                  const int32_t *block_tables, const int32_t *context_lens, int32_t ctx_offset,
                  int32_t batch, int32_t num_heads, int32_t head_dim, int32_t block_size,
                  int32_t num_blocks, int32_t max_blocks, const int64_t *new_strides,
                  const int64_t *cache_strides, const int64_t *bt_strides, int32_t dtype,
                  int32_t *status, void *stream) {
  int rc = check_common(dtype, batch, num_heads, head_dim, block_size, num_blocks, max_blocks,
                        cache_strides, bt_strides);
  if (rc) return rc;
  if (new_strides == nullptr) {
    set_error_detail("new_strides must not be NULL");
    return PKV_ERR_INVALID_ARG;
  }
  if (batch == 0) return PKV_OK;
  if (!k_new || !v_new || !k_cache || !v_cache || !block_tables || !context_lens) {
    set_error_detail("pkv_append: NULL tensor pointer");
    return PKV_ERR_INVALID_ARG;
  }
  const int es = dtype_size(dtype);
  const void *ptrs[] = {k_new, v_new, k_cache, v_cache};
  for (const void *p : ptrs)
    if (!aligned_to(p, es)) return PKV_ERR_ALIGNMENT;
  VecPlan vp = pick_vector(es, head_dim, ptrs, 4, new_strides, 3, cache_strides, 4);
  CopyGeom g{};
  g.batch = batch;
  g.heads = num_heads;
  g.tokens = 1;
  g.chunks = head_dim / vp.elems_per_vec;
  g.block_size = block_size;
  g.num_blocks = num_blocks;
  g.max_blocks = max_blocks;
  g.ctx_offset = ctx_offset;
  const int64_t e = vp.elems_per_vec;
  g.s0 = new_strides[0] / e; g.s1 = new_strides[1] / e; g.s2 = 0; g.s3 = vp.vec_bytes == 16 ? 1 : new_strides[2];
  g.c0 = cache_strides[0] / e; g.c1 = cache_strides[1] / e; g.c2 = cache_strides[2] / e;
  g.c3 = vp.vec_bytes == 16 ? 1 : cache_strides[3];
  g.bt0 = bt_strides[0]; g.bt1 = bt_strides[1];
  const int grid = grid_for((int64_t)batch * num_heads * g.chunks);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (vp.vec_bytes) {
    case 16:
      append_kernel<uint4><<<grid, kCopyThreads, 0, st>>>(
          (const uint4 *)k_new, (const uint4 *)v_new, (uint4 *)k_cache, (uint4 *)v_cache,
          block_tables, context_lens, g, status);
      break;
    case 4:
      append_kernel<uint32_t><<<grid, kCopyThreads, 0, st>>>(
          (const uint32_t *)k_new, (const uint32_t *)v_new, (uint32_t *)k_cache,
          (uint32_t *)v_cache, block_tables, context_lens, g, status);
      break;
    default:
      append_kernel<uint16_t><<<grid, kCopyThreads, 0, st>>>(
          (const uint16_t *)k_new, (const uint16_t *)v_new, (uint16_t *)k_cache,
          (uint16_t *)v_cache, block_tables, context_lens, g, status);
      break;
  }
  return check_launch("pkv_append");
}

}  // namespace pkv

extern "C" int pkv_append(const void *k_new, const void *v_new, void *k_cache, void *v_cache,
                          const int32_t *block_tables, const int32_t *context_lens,
                          int32_t batch, int32_t num_heads, int32_t head_dim, int32_t block_size,
                          int32_t num_blocks, int32_t max_blocks, const int64_t *new_strides,
                          const int64_t *cache_strides, const int64_t *bt_strides, int32_t dtype,
                          int32_t *status, void *stream) {
  return pkv::append_launch(k_new, v_new, k_cache, v_cache, block_tables, context_lens, 0, batch,
                            num_heads, head_dim, block_size, num_blocks, max_blocks, new_strides,
                            cache_strides, bt_strides, dtype, status, stream);
}

extern "C" int pkv_append_prompt(const void *k_src, const void *v_src, void *k_cache,
                                 void *v_cache, const int32_t *block_tables,
                                 const int32_t *start_pos, const int32_t *lens, int32_t batch,
                                 int32_t num_heads, int32_t seq_len, int32_t head_dim,
                                 int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                                 const int64_t *src_strides, const int64_t *cache_strides,
                                 const int64_t *bt_strides, int32_t dtype, int32_t *status,
                                 void *stream) {
  int rc = check_common(dtype, batch, num_heads, head_dim, block_size, num_blocks, max_blocks,
                        cache_strides, bt_strides);
  if (rc) return rc;
  if (src_strides == nullptr || seq_len < 0) {
    set_error_detail("pkv_append_prompt: bad src_strides or seq_len=%d", seq_len);
    return PKV_ERR_INVALID_ARG;
  }
  if (batch == 0 || seq_len == 0) return PKV_OK;
  if (!k_src || !v_src || !k_cache || !v_cache || !block_tables) {
    set_error_detail("pkv_append_prompt: NULL tensor pointer");
    return PKV_ERR_INVALID_ARG;
  }
  const int es = dtype_size(dtype);
  const void *ptrs[] = {k_src, v_src, k_cache, v_cache};
  for (const void *p : ptrs)
    if (!aligned_to(p, es)) return PKV_ERR_ALIGNMENT;
  VecPlan vp = pick_vector(es, head_dim, ptrs, 4, src_strides, 4, cache_strides, 4);
  const int64_t e = vp.elems_per_vec;
  CopyGeom g{};
  g.batch = batch;
  g.heads = num_heads;
  g.tokens = seq_len;
  g.chunks = head_dim / vp.elems_per_vec;
  g.block_size = block_size;
  g.num_blocks = num_blocks;
  g.max_blocks = max_blocks;
  g.s0 = src_strides[0] / e; g.s1 = src_strides[1] / e; g.s2 = src_strides[2] / e;
  g.s3 = vp.vec_bytes == 16 ? 1 : src_strides[3];
  g.c0 = cache_strides[0] / e; g.c1 = cache_strides[1] / e; g.c2 = cache_strides[2] / e;
  g.c3 = vp.vec_bytes == 16 ? 1 : cache_strides[3];
  g.bt0 = bt_strides[0]; g.bt1 = bt_strides[1];
  const int grid = grid_for((int64_t)batch * num_heads * seq_len * g.chunks);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (vp.vec_bytes) {
    case 16:
      append_prompt_kernel<uint4><<<grid, kCopyThreads, 0, st>>>(
          (const uint4 *)k_src, (const uint4 *)v_src, (uint4 *)k_cache, (uint4 *)v_cache,
          block_tables, start_pos, lens, g, status);
      break;
    case 4:
      append_prompt_kernel<uint32_t><<<grid, kCopyThreads, 0, st>>>(
          (const uint32_t *)k_src, (const uint32_t *)v_src, (uint32_t *)k_cache,
          (uint32_t *)v_cache, block_tables, start_pos, lens, g, status);
      break;
    default:
      append_prompt_kernel<uint16_t><<<grid, kCopyThreads, 0, st>>>(
          (const uint16_t *)k_src, (const uint16_t *)v_src, (uint16_t *)k_cache,
          (uint16_t *)v_cache, block_tables, start_pos, lens, g, status);
      break;
  }
  return check_launch("pkv_append_prompt");
}

extern "C" int pkv_gather(const void *k_cache, const void *v_cache, const int32_t *block_tables,
                          const int32_t *context_lens, void *k_out, void *v_out, int32_t batch,
                          int32_t num_heads, int32_t head_dim, int32_t block_size,
                          int32_t num_blocks, int32_t max_blocks, int32_t max_tokens,
                          const int64_t *cache_strides, const int64_t *bt_strides,
                          const int64_t *out_strides, int32_t dtype, int32_t *status,
                          void *stream) {
  int rc = check_common(dtype, batch, num_heads, head_dim, block_size, num_blocks, max_blocks,
                        cache_strides, bt_strides);
  if (rc) return rc;
  if (out_strides == nullptr || max_tokens < 0) {
    set_error_detail("pkv_gather: bad out_strides or max_tokens=%d", max_tokens);
    return PKV_ERR_INVALID_ARG;
  }
  if (batch == 0 || max_tokens == 0) return PKV_OK;
  if (!k_cache || !v_cache || !block_tables || !context_lens || !k_out || !v_out) {
    set_error_detail("pkv_gather: NULL tensor pointer");
    return PKV_ERR_INVALID_ARG;
  }
  const int es = dtype_size(dtype);
  const void *ptrs[] = {k_cache, v_cache, k_out, v_out};
  for (const void *p : ptrs)
    if (!aligned_to(p, es)) return PKV_ERR_ALIGNMENT;
  VecPlan vp = pick_vector(es, head_dim, ptrs, 4, out_strides, 4, cache_strides, 4);
  const int64_t e = vp.elems_per_vec;
  CopyGeom g{};
  g.batch = batch;
  g.heads = num_heads;
  g.tokens = max_tokens;
  g.chunks = head_dim / vp.elems_per_vec;
  g.block_size = block_size;
  g.num_blocks = num_blocks;
  g.max_blocks = max_blocks;
  g.s0 = out_strides[0] / e; g.s1 = out_strides[1] / e; g.s2 = out_strides[2] / e;
  g.s3 = vp.vec_bytes == 16 ? 1 : out_strides[3];
  g.c0 = cache_strides[0] / e; g.c1 = cache_strides[1] / e; g.c2 = cache_strides[2] / e;
  g.c3 = vp.vec_bytes == 16 ? 1 : cache_strides[3];
  g.bt0 = bt_strides[0]; g.bt1 = bt_strides[1];
  const int grid = grid_for((int64_t)batch * num_heads * max_tokens * g.chunks);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (vp.vec_bytes) {
    case 16:
      gather_kernel<uint4><<<grid, kCopyThreads, 0, st>>>(
          (const uint4 *)k_cache, (const uint4 *)v_cache, block_tables, context_lens,
          (uint4 *)k_out, (uint4 *)v_out, g, status);
      break;
    case 4:
      gather_kernel<uint32_t><<<grid, kCopyThreads, 0, st>>>(
          (const uint32_t *)k_cache, (const uint32_t *)v_cache, block_tables, context_lens,
          (uint32_t *)k_out, (uint32_t *)v_out, g, status);
      break;
    default:
      gather_kernel<uint16_t><<<grid, kCopyThreads, 0, st>>>(
          (const uint16_t *)k_cache, (const uint16_t *)v_cache, block_tables, context_lens,
          (uint16_t *)k_out, (uint16_t *)v_out, g, status);
      break;
  }
  return check_launch("pkv_gather");
}
