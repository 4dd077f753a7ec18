/*
 * pkv.h — C ABI of the B200 paged-KV library (libpkv.so).
 *
 * The library implements the rollout hot path of the GRPO trainer: the paged
 * KV-cache page append and the paged-KV (GQA) single-query decode attention.
 * Every entry point takes plain device pointers, element strides and sizes,
 * enqueues its kernels on the given CUDA stream (a cudaStream_t passed as
 * void*; NULL = legacy default stream) and returns without synchronising.
 *
 * Conventions shared by all entry points
 *   - Strides are in ELEMENTS (not bytes), exactly like torch.Tensor.stride().
 *   - The KV cache of one layer has the logical shape
 *         [num_blocks, num_kv_heads, block_size, head_dim]
 *     (the layout of the reference's per-layer k_cache/v_cache,
 *     src/triton_kernels/paged_kv.py:378-381,412). k_cache and v_cache share
 *     one set of strides, as they share stride_kb/kh/kt/kd in the reference
 *     kernels (paged_kv.py:74-77,264-267).
 *   - block_tables is int32 [batch, max_blocks]; context_lens is int32 [batch].
 *   - Page ids outside [0, num_blocks) and context lengths outside
 *     [0, max_blocks * block_size] never cause an out-of-bounds access: the
 *     kernel skips the access (append/gather) or treats the page as empty
 *     (decode) and ORs a PKV_DEV_* bit into *status when status != NULL.
 *   - Return value: PKV_OK (0) or a negative PKV_ERR_* code. The library never
 *     traps on the device and never allocates device memory: scratch space
 *     (the decode workspace) is provided by the caller.
 *   - Launch failures are reported through cudaGetLastError() as PKV_ERR_CUDA;
 *     pkv_last_error_detail() returns a thread-local description of the most
 *     recent error on the calling thread.
 */
#ifndef PKV_H_
#define PKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PKV_ABI_VERSION 10 /* 2: pkv_append_decode_run, 3: pkv_sample_top_p, 4: rmsnorm, rope, 5: silu_mul,
                              6: pkv_sample_top_p flags, 7: pkv_rope_qk output strides,
                              8: pkv_rope_append_decode_run, 9: pkv_linear,
                              10: PKV_LINEAR_WEIGHTS_STATIC, PKV_DECODE_EARLY_START */

/* Element types. The reference stores the cache in bfloat16
 * (paged_kv.py:409-410, 629-633); float32 is accepted because the reference
 * kernels themselves are dtype-agnostic (they cast to fp32, paged_kv.py:120,132,240). */
enum {
    PKV_DTYPE_F32 = 0,
    PKV_DTYPE_BF16 = 1,
    PKV_DTYPE_F16 = 2
};

/* Host-side status codes. */
enum {
    PKV_OK = 0,
    PKV_ERR_INVALID_ARG = -1, /* null pointer, negative size, bad stride     */
    PKV_ERR_UNSUPPORTED = -2, /* dtype / head_dim combination not built      */
    PKV_ERR_ALIGNMENT = -3,   /* pointer not aligned to its element size     */
    PKV_ERR_WORKSPACE = -4,   /* workspace missing or smaller than required  */
    PKV_ERR_CUDA = -5,        /* a CUDA runtime call or launch failed        */
    PKV_ERR_TENSOR_MAP = -6   /* cuTensorMapEncodeTiled rejected the layout  */
};

/* Device-side status bits, OR-ed into the optional int32 *status word. */
enum {
    PKV_DEV_CTX_OUT_OF_RANGE = 1,  /* context_lens[b] < 0 or > max_blocks*block_size */
    PKV_DEV_PAGE_OUT_OF_RANGE = 2, /* block_tables entry outside [0, num_blocks)      */
    PKV_DEV_WAIT_TIMEOUT = 4       /* a bounded device-side wait gave up              */
};

/* Decode flags. */
enum {
    PKV_DECODE_FORCE_GENERIC = 1, /* use the CUDA-core kernel even when the
                                     tensor-core kernel could run            */
    PKV_DECODE_EXACT_P = 2,       /* tensor-core kernel: multiply the softmax
                                     weights as a 16-bit head plus 16-bit
                                     remainder (~17 significant bits instead
                                     of 8); slower, closer to fp32           */
    PKV_DECODE_OUT_Q_DTYPE = 4,   /* out holds q's dtype (bf16 or fp16; fp32 q:
                                     no change): each fp32 result rounded to
                                     nearest, as a cast of the fp32 output   */
    PKV_DECODE_EARLY_START = 8,   /* tensor-core kernel: the caller promises
                                     that the previous kernel in the stream
                                     wrote none of the plan (workspace),
                                     block tables, context lengths and
                                     caches, and that every kernel before it
                                     is complete once it lets this launch
                                     start. Both hold when it is an earlier
                                     decode launch after the plan (a decode
                                     launch lets the next launch start only
                                     after its own wait): the layers after the
                                     first of a step, not the first (behind the
                                     plan) nor one behind a separate append.
                                     The launch then schedules its first unit
                                     and starts loading its pages before
                                     waiting for that kernel; q, the new rows
                                     and cos / sin are read after the wait. */
    PKV_DECODE_TEST_WAIT_TIMEOUT = 1 << 30 /* TEST ONLY (tensor-core kernel):
                                     every device wait gives up after 4096
                                     polls instead of seconds' worth, and the
                                     first CTA's producer never publishes one
                                     pipeline element, so waits run out: the
                                     launch returns, ORs PKV_DEV_WAIT_TIMEOUT
                                     into *status, and its output is
                                     undefined. Exercises the timeout path;
                                     never set it otherwise. */
};

/* Sampling flags. */
enum {
    PKV_SAMPLE_FORCE_RADIX = 1 /* 16-bit logits: take the radix-select path even
                                  when the per-pattern counts fit (same tokens) */
};

int pkv_abi_version(void);
const char *pkv_error_string(int status);
const char *pkv_last_error_detail(void);

/*
 * pkv_append — write one new K and V token per (sequence, head) into its page.
 *
 * Replaces the reference's _paged_kv_update_kernel
 * (src/triton_kernels/paged_kv.py:253-319) and its launch
 * (paged_kv.py:730-752, 914-936): for every b < batch, h < num_heads the slot
 * is position context_lens[b] (the PRE-append length): page
 * block_tables[b, ctx / block_size], offset ctx % block_size
 * (paged_kv.py:277-284); k_cache[page, h, off, :] = k_new[b, h, :] and the
 * same for v (paged_kv.py:286-319). The payload is copied bit for bit.
 *
 * new_strides[3]  : strides of k_new / v_new [batch, num_heads, head_dim]
 * cache_strides[4]: strides of k_cache / v_cache
 * bt_strides[2]   : strides of block_tables
 * dtype           : element type of k_new, v_new and the caches (all equal)
 */
int pkv_append(const void *k_new, const void *v_new, void *k_cache, void *v_cache,
               const int32_t *block_tables, const int32_t *context_lens,
               int32_t batch, int32_t num_heads, int32_t head_dim,
               int32_t block_size, int32_t num_blocks, int32_t max_blocks,
               const int64_t *new_strides, const int64_t *cache_strides,
               const int64_t *bt_strides, int32_t dtype, int32_t *status,
               void *stream);

/*
 * pkv_append_prompt — bulk write of a prompt's K/V into pages.
 *
 * Replaces the B x T x L host loop of the reference's _prefill_paged_cache
 * (src/triton_kernels/paged_kv.py:572-586): for b < batch, t < lens[b],
 * h < num_heads, position pos = start_pos[b] + t goes to page
 * block_tables[b, pos / block_size], offset pos % block_size, and
 * k_cache[page, h, off, :] = k_src[b, h, t, :] (same for v).
 * k_src/v_src have the [batch, num_heads, seq_len, head_dim] layout of a
 * HuggingFace past_key_values layer. start_pos == NULL means 0 for every
 * sequence; lens == NULL means seq_len for every sequence.
 * src_strides[4]: strides of k_src / v_src.
 */
int pkv_append_prompt(const void *k_src, const void *v_src, void *k_cache,
                      void *v_cache, const int32_t *block_tables,
                      const int32_t *start_pos, const int32_t *lens,
                      int32_t batch, int32_t num_heads, int32_t seq_len,
                      int32_t head_dim, int32_t block_size, int32_t num_blocks,
                      int32_t max_blocks, const int64_t *src_strides,
                      const int64_t *cache_strides, const int64_t *bt_strides,
                      int32_t dtype, int32_t *status, void *stream);

/*
 * pkv_gather — dense copy of the paged cache: k_out[b, h, t, :] =
 * k_cache[block_tables[b, t / bs], h, t % bs, :] for t < context_lens[b],
 * zero for context_lens[b] <= t < max_tokens (same for v). This is the
 * addressing of the reference decode kernel (paged_kv.py:98-131) written out
 * densely; the reference uses it implicitly in its dense parity test
 * (tests/test_triton_performance.py:196-219).
 * out_strides[4]: strides of k_out / v_out [batch, num_heads, max_tokens, head_dim].
 */
int pkv_gather(const void *k_cache, const void *v_cache,
               const int32_t *block_tables, const int32_t *context_lens,
               void *k_out, void *v_out, int32_t batch, int32_t num_heads,
               int32_t head_dim, int32_t block_size, int32_t num_blocks,
               int32_t max_blocks, int32_t max_tokens,
               const int64_t *cache_strides, const int64_t *bt_strides,
               const int64_t *out_strides, int32_t dtype, int32_t *status,
               void *stream);

/*
 * Decode attention: out[b, h, :] = sum_{t < ctx_b} softmax_t(scale * q[b,h] . K[t]) V[t]
 * with K/V the pages of sequence b for kv head h / (num_q_heads / num_kv_heads),
 * fp32 accumulation and an fp32 output; out = acc / max(sum, 1e-6), so an
 * empty context yields zeros. Replaces _paged_attention_decode_kernel
 * (src/triton_kernels/paged_kv.py:63-251) and its launches
 * (paged_kv.py:754-783, 939-969). context_lens is the POST-append length
 * (paged_kv.py:697,761,938). num_q_heads == num_kv_heads reproduces the
 * reference's head-replicated cache; num_q_heads = G * num_kv_heads is the
 * grouped-query layout (one cache head serves G consecutive query heads).
 *
 * Long contexts are split into chunks of pages_per_split pages; partial
 * (max, sum, acc) triples go to the caller's workspace and are combined in
 * chunk order. pages_per_split == 0 selects the library's heuristic for the
 * current device.
 *
 * pkv_decode = pkv_decode_plan + pkv_decode_run. The plan depends only on
 * context_lens (and the sizes), so a caller that runs many layers with the
 * same context_lens may plan once and run per layer on the same workspace.
 * After a launch that set PKV_DEV_WAIT_TIMEOUT, plan again before the next
 * run on that workspace (the plan's scheduling and merge counters may have
 * been left mid-count).
 *
 * pages_per_split == 0: pkv_decode_pages_per_split returns the library's
 * estimate for sequences of max_blocks pages. For batches of at most 1024
 * sequences the plan kernel instead picks the split length (a multiple of 8,
 * up to 512) from the actual lengths, by simulating its schedule; the
 * workspace size accounts for that. With the tensor-core kernel the last split of a sequence to finish
 * merges the split partials inside the same launch; the CUDA-core kernel
 * launches the merge kernel after it.
 */
int32_t pkv_decode_pages_per_split(int32_t batch, int32_t num_q_heads,
                                   int32_t num_kv_heads, int32_t head_dim,
                                   int32_t max_blocks, int32_t pages_per_split);

size_t pkv_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                 int32_t num_kv_heads, int32_t head_dim,
                                 int32_t max_blocks, int32_t pages_per_split);

int pkv_decode_plan(const int32_t *context_lens, int32_t batch,
                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                    int32_t block_size, int32_t max_blocks,
                    int32_t pages_per_split, void *workspace,
                    size_t workspace_bytes, int32_t *status, void *stream);

int pkv_decode_run(const void *q, const void *k_cache, const void *v_cache,
                   const int32_t *block_tables, const int32_t *context_lens,
                   float *out, int32_t batch, int32_t num_q_heads,
                   int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                   int32_t num_blocks, int32_t max_blocks,
                   const int64_t *q_strides, const int64_t *cache_strides,
                   const int64_t *bt_strides, const int64_t *out_strides,
                   int32_t q_dtype, int32_t kv_dtype, float scale,
                   int32_t pages_per_split, int32_t flags, void *workspace,
                   size_t workspace_bytes, int32_t *status, void *stream);

/*
 * pkv_append_decode_run: one decode step of one layer, the append included.
 * Writes k_new[b] / v_new[b] ([batch, num_kv_heads, head_dim], cache dtype)
 * into the cache at position context_lens[b] - 1, then decodes exactly as
 * pkv_decode_run over context_lens[b] positions (POST-append lengths; a
 * sequence of length 0 appends nothing). The pair it replaces is the
 * reference's per-layer _paged_kv_update_kernel launch with the pre-append
 * lengths followed by _paged_attention_decode_kernel with the post-append
 * ones (src/triton_kernels/paged_kv.py:730-783). On the tensor-core kernel
 * (and D-contiguous, 16-byte aligned k_new / v_new rows) this is one launch:
 * the kernel writes the token into its page and uses it in the same pass;
 * otherwise the append kernel runs first on the same stream. The cache
 * bytes written are those pkv_append would write.
 */
int pkv_append_decode_run(const void *q, const void *k_new, const void *v_new,
                          void *k_cache, void *v_cache,
                          const int32_t *block_tables, const int32_t *context_lens,
                          float *out, int32_t batch, int32_t num_q_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                          int32_t num_blocks, int32_t max_blocks,
                          const int64_t *q_strides, const int64_t *new_strides,
                          const int64_t *cache_strides, const int64_t *bt_strides,
                          const int64_t *out_strides, int32_t q_dtype, int32_t kv_dtype,
                          float scale, int32_t pages_per_split, int32_t flags,
                          void *workspace, size_t workspace_bytes, int32_t *status,
                          void *stream);

/*
 * pkv_sample_top_p: one token per row of logits [batch, vocab] (row stride
 * row_stride elements, any dtype code), sampled from softmax(logits / T)
 * restricted to the nucleus the reference keeps: tokens in descending order
 * while their running probability is <= top_p, and always the most likely
 * one (src/triton_kernels/paged_kv.py:418-450). Ties at the cut are kept in
 * index order. uniforms[b] in [0, 1) picks the token by the inverse CDF of the
 * kept tokens in index order. out_tokens is int64 [batch]. temperature and
 * top_p must be > 0; top_p >= 1 keeps every token. One launch, no sort.
 * flags: PKV_SAMPLE_* (0 for the default).
 */
int pkv_sample_top_p(const void *logits, int32_t dtype, int32_t batch, int32_t vocab,
                     int64_t row_stride, float temperature, float top_p,
                     const float *uniforms, int64_t *out_tokens, int32_t flags, void *stream);

/*
 * Decode-step element-wise steps around the decode launch (one launch each).
 *
 * pkv_add_rmsnorm: for each row, s = x + residual (rounded to dtype; skipped
 * when residual is NULL; written to sum_out when that is not NULL), then
 * out = weight * dtype(s * rsqrt(mean(s^2) + eps)) with fp32 statistics, the
 * rounding points of HF's Qwen2RMSNorm (the reference's fused_ops rmsnorm).
 * Rows are read as 16-byte vectors: 16-byte aligned rows whose byte length is a
 * multiple of 16, hidden <= 8192 bytes' worth (4096 bf16). Strides in elements.
 *
 * pkv_rope_qk: RoPE of one new query row [num_q_heads * head_dim] and key row
 * [num_kv_heads * head_dim] per sequence with cos/sin [rows, head_dim] (row
 * stride cs_stride), written as q_out [rows, Hq, D] and k_out [rows, Hkv, D]
 * (row strides q_out_stride / k_out_stride, heads contiguous: the layout
 * pkv_append_decode_run reads), with the element-wise rounding of HF's
 * apply_rotary_pos_emb. k_out may be k itself (rotation in place).
 */
int pkv_add_rmsnorm(const void *x, const void *residual, const void *weight, void *sum_out, void *out,
                    int32_t rows, int32_t hidden, int64_t x_stride, int64_t residual_stride,
                    int64_t sum_stride, int64_t out_stride, float eps, int32_t dtype, void *stream);

/* pkv_silu_mul: out [rows, cols] (contiguous) = dtype(dtype(silu(gate)) * up), the
 * gated activation of a Qwen2 MLP; rows of 16-byte multiples, 16-byte aligned. */
int pkv_silu_mul(const void *gate, const void *up, void *out, int32_t rows, int32_t cols,
                 int64_t gate_stride, int64_t up_stride, int32_t dtype, void *stream);

int pkv_rope_qk(const void *q, const void *k, const void *cos_, const void *sin_, void *q_out,
                void *k_out, int32_t rows, int32_t num_q_heads, int32_t num_kv_heads,
                int32_t head_dim, int64_t q_stride, int64_t k_stride, int64_t cs_stride,
                int64_t q_out_stride, int64_t k_out_stride, int32_t dtype, void *stream);

int pkv_decode(const void *q, const void *k_cache, const void *v_cache,
               const int32_t *block_tables, const int32_t *context_lens,
               float *out, int32_t batch, int32_t num_q_heads,
               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
               int32_t num_blocks, int32_t max_blocks,
               const int64_t *q_strides, const int64_t *cache_strides,
               const int64_t *bt_strides, const int64_t *out_strides,
               int32_t q_dtype, int32_t kv_dtype, float scale,
               int32_t pages_per_split, int32_t flags, void *workspace,
               size_t workspace_bytes, int32_t *status, void *stream);

/*
 * pkv_rope_append_decode_run: pkv_append_decode_run for q and k_new rows taken
 * before RoPE (the projections' outputs), rotated inside the launch with
 * cos / sin [batch, head_dim] (q's dtype, row stride rope_stride) exactly as
 * pkv_rope_qk rotates them (HF apply_rotary_pos_emb's rounding): one launch
 * for the per-layer RoPE, page append and decode of the reference's model loop
 * (paged_kv.py:720-783). Only on the tensor-core kernel: 16-bit q and cache of
 * one dtype, 16-byte aligned rows with contiguous head_dim for q, k_new, v_new,
 * cos and sin; anything else returns PKV_ERR_UNSUPPORTED without launching.
 */
int pkv_rope_append_decode_run(const void *q, const void *k_new, const void *v_new,
                               const void *rope_cos, const void *rope_sin, int64_t rope_stride,
                               void *k_cache, void *v_cache, const int32_t *block_tables,
                               const int32_t *context_lens, float *out, int32_t batch,
                               int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                               int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                               const int64_t *q_strides, const int64_t *new_strides,
                               const int64_t *cache_strides, const int64_t *bt_strides,
                               const int64_t *out_strides, int32_t q_dtype, int32_t kv_dtype,
                               float scale, int32_t pages_per_split, int32_t flags, void *workspace,
                               size_t workspace_bytes, int32_t *status, void *stream);

/*
 * pkv_decode_noalloc — pkv_decode without a caller workspace. No counterpart
 * in the reference: it exists for callers that cannot allocate device memory
 * themselves (an FFI host that only passes in the tensors it owns, or a
 * process whose GPU memory is held by another framework's allocator, where a
 * direct cudaMalloc fails or fragments that allocator's pool).
 *
 * The split plan and split-K partials live in a static device array of
 * PKV_NOALLOC_SCRATCH_BYTES inside the library; every GPU that loads the
 * library's device code keeps that much memory for it until the process
 * exits. Decodes whose workspace (pkv_decode_workspace_size) exceeds it are
 * rejected with PKV_ERR_WORKSPACE. The first call in a CUDA context looks up
 * the array's device address in that context (cudaGetSymbolAddress, with the
 * caller's device and context current) and caches it under the context's
 * unique id, so a context made with the driver API, or a primary context
 * re-created after cudaDeviceReset, gets its own lookup. Make that first call
 * before any stream capture. All calls share the array:
 * calls that run concurrently on the GPU race on it and must be serialised by
 * the caller. Arguments and results are those of pkv_decode.
 */
#define PKV_NOALLOC_SCRATCH_BYTES (32u << 20)

int pkv_decode_noalloc(const void *q, const void *k_cache, const void *v_cache,
                       const int32_t *block_tables, const int32_t *context_lens,
                       float *out, int32_t batch, int32_t num_q_heads,
                       int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                       int32_t num_blocks, int32_t max_blocks,
                       const int64_t *q_strides, const int64_t *cache_strides,
                       const int64_t *bt_strides, const int64_t *out_strides,
                       int32_t q_dtype, int32_t kv_dtype, float scale,
                       int32_t pages_per_split, int32_t flags, int32_t *status,
                       void *stream);

/*
 * pkv_linear — one projection of a rollout decode step on the tcgen05 tensor
 * cores: out[r, j] = sum_k x[r, k] * W[j, k] (+ bias[j]) for r < rows <= 128,
 * j < n, with fp32 accumulation and the result rounded to the 16-bit dtype of
 * x, W and out (bf16 or fp16, all the same). W has nn.Linear's layout
 * [out_features, in_features] (row stride w_stride elements), so the weights
 * are read as they lie. Replaces the nn.Linear calls of the reference's fused
 * decode step: q/k/v (src/triton_kernels/fused_ops.py:198-219), o_proj
 * (paged_kv.py:789), gate/up and down (fused_ops.py:184-195) and the LM head
 * (fused_ops.py:231).
 *
 * act = PKV_LINEAR_SILU_GATE: W holds the gate rows [n, k] and the up rows
 * come from w_up ([n, k], same row stride), or, with w_up NULL, W is the gate
 * rows stacked over the up rows ([2 n, k]); out[r, j] = T(T(silu(g)) * u) with
 * g = T(x . gate[j]) and u = T(x . up[j]) — the MLP's act_fn(gate_proj(x)) *
 * up_proj(x) rounded as HF Qwen2MLP rounds it (the reference's fused_silu_mul,
 * fused_ops.py:79-103); n a multiple of 64, no bias. w_up must be NULL for
 * PKV_LINEAR_NONE.
 *
 * act | PKV_LINEAR_WEIGHTS_STATIC: the caller guarantees that no kernel still
 * in flight in `stream` writes W or w_up (model weights during generation).
 * The launch is a programmatic dependent launch either way; with this flag
 * each CTA starts streaming its first W tiles into shared memory before it
 * waits for the previous kernel in the stream, so the weight stream overlaps
 * that kernel's tail and this launch's own ramp. x, the bias and out are
 * touched only after the wait.
 *
 * Requirements: in_features a multiple of 64; x, W and out 16-byte aligned
 * with row strides that are multiples of 8 elements. No workspace: the split-K
 * partials stay on chip (the splits of a column tile are one thread-block
 * cluster that adds them in split order, so results are deterministic).
 */
enum {
    PKV_LINEAR_NONE = 0,
    PKV_LINEAR_SILU_GATE = 1,
    PKV_LINEAR_WEIGHTS_STATIC = 0x100  /* flag, OR'd into act */
};

int pkv_linear(const void *x, const void *w, const void *w_up, const void *bias, void *out,
               int32_t rows, int32_t n, int32_t k, int64_t x_stride, int64_t w_stride,
               int64_t out_stride, int32_t dtype, int32_t act, int32_t *status, void *stream);

/*
 * Which decode kernel pkv_decode_run would launch for these arguments:
 * 1 = tensor-core kernel (cp.async page staging, mma.sync), 0 = CUDA-core kernel, <0 = error code.
 */
int pkv_decode_kernel_kind(const void *k_cache, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, const int64_t *cache_strides,
                           int32_t q_dtype, int32_t kv_dtype, int32_t flags);

#ifdef __cplusplus
}
#endif

#endif /* PKV_H_ */
