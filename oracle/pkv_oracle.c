/*
 * pkv_oracle.c — CPU restatement of the reference paged-KV decode attention.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA path in
 * libpkv.so and the timed CPU baseline of bench.py; nothing in the product
 * package loads it.
 *
 * It restates _paged_attention_decode_kernel of the reference
 * (src/triton_kernels/paged_kv.py:63-251) for one (sequence b, query head h)
 * at a time, pass by pass:
 *   pass 1 (paged_kv.py:96-138):  m = max_t  (sum_d q[d] * K[t][d]) * scale
 *   pass 2 (paged_kv.py:140-182): s = sum_t exp(logit_t - m)
 *   pass 3 (paged_kv.py:184-251): out[d] = sum_t exp(logit_t - m) V[t][d] / max(s, 1e-6)
 * recomputing q.K in every pass as the reference does. K and V rows of
 * position t come from page block_tables[b, t / block_size], slot
 * t % block_size (paged_kv.py:100-131). Positions t >= context_lens[b] are
 * masked, so an empty context gives out = 0 (paged_kv.py:136,181,228,243).
 * Query head h reads cache head h / (Hq / Hkv); with Hq == Hkv this is the
 * reference's head-replicated cache. Inputs are converted to fp32 before any
 * arithmetic (paged_kv.py:120,132,176,240).
 *
 * Strides are in elements; the argument list is the one of pkv_decode in
 * include/pkv.h, with host pointers.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <unistd.h>

enum { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

/* IEEE 754 binary16 -> binary32, from the format definition. */
static float half_bits_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float load_f32(const void *base, int64_t idx, int dtype) {
    if (dtype == DT_BF16) {
        uint32_t u = (uint32_t)((const uint16_t *)base)[idx] << 16;
        float f;
        memcpy(&f, &u, 4);
        return f;
    }
    if (dtype == DT_F16) return half_bits_to_float(((const uint16_t *)base)[idx]);
    return ((const float *)base)[idx];
}

/* Row of cache position t of sequence b, or -1 when the page id is invalid. */
static int64_t row_offset(const int32_t *bt, const int64_t *bts, const int64_t *cs, int32_t b,
                          int32_t t, int32_t kvh, int32_t bs, int32_t num_blocks) {
    int32_t page = bt[b * bts[0] + (int64_t)(t / bs) * bts[1]];
    if (page < 0 || page >= num_blocks) return -1;
    return page * cs[0] + kvh * cs[1] + (int64_t)(t % bs) * cs[2];
}

static float logit_at(const float *qf, const void *kc, int64_t row, const int64_t *cs, int32_t D,
                      int kv_dtype, float scale) {
    float dot = 0.f;
    for (int32_t d = 0; d < D; ++d) dot += qf[d] * load_f32(kc, row + d * cs[3], kv_dtype);
    return dot * scale; /* scale applied after the dot product (paged_kv.py:135) */
}

typedef struct {
    const void *q, *k_cache, *v_cache;
    const int32_t *block_tables, *context_lens;
    float *out;
    int32_t batch, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, max_blocks;
    const int64_t *q_strides, *cache_strides, *bt_strides, *out_strides;
    int32_t q_dtype, kv_dtype;
    float scale;
    int64_t next; /* next (b, h) unit to take; shared work counter */
} DecodeJob;

/* One (sequence b, query head h) of the reference decode kernel. */
static void decode_unit(const DecodeJob *j, int64_t u, float *qf, float *acc) {
    const int32_t G = j->num_q_heads / j->num_kv_heads;
    const int32_t cap = j->max_blocks * j->block_size;
    const int32_t b = (int32_t)(u / j->num_q_heads);
    const int32_t h = (int32_t)(u % j->num_q_heads);
    const int32_t kvh = h / G;
    const int32_t D = j->head_dim;
    const int64_t *cs = j->cache_strides;
    int32_t n = j->context_lens[b];
    if (n < 0) n = 0;
    if (n > cap) n = cap;
    for (int32_t d = 0; d < D; ++d)
        qf[d] = load_f32(j->q, b * j->q_strides[0] + h * j->q_strides[1] + d * j->q_strides[2],
                         j->q_dtype);

    float m = -INFINITY; /* pass 1 */
    for (int32_t t = 0; t < n; ++t) {
        int64_t row = row_offset(j->block_tables, j->bt_strides, cs, b, t, kvh, j->block_size,
                                 j->num_blocks);
        if (row < 0) continue;
        float l = logit_at(qf, j->k_cache, row, cs, D, j->kv_dtype, j->scale);
        if (l > m) m = l;
    }
    float s = 0.f; /* pass 2 */
    for (int32_t t = 0; t < n; ++t) {
        int64_t row = row_offset(j->block_tables, j->bt_strides, cs, b, t, kvh, j->block_size,
                                 j->num_blocks);
        if (row < 0) continue;
        s += expf(logit_at(qf, j->k_cache, row, cs, D, j->kv_dtype, j->scale) - m);
    }
    for (int32_t d = 0; d < D; ++d) acc[d] = 0.f; /* pass 3 */
    for (int32_t t = 0; t < n; ++t) {
        int64_t row = row_offset(j->block_tables, j->bt_strides, cs, b, t, kvh, j->block_size,
                                 j->num_blocks);
        if (row < 0) continue;
        const float w = expf(logit_at(qf, j->k_cache, row, cs, D, j->kv_dtype, j->scale) - m);
        for (int32_t d = 0; d < D; ++d)
            acc[d] += w * load_f32(j->v_cache, row + d * cs[3], j->kv_dtype);
    }
    const float denom = s > 1e-6f ? s : 1e-6f; /* paged_kv.py:243 */
    for (int32_t d = 0; d < D; ++d)
        j->out[b * j->out_strides[0] + h * j->out_strides[1] + d * j->out_strides[2]] =
            acc[d] / denom;
}

static void *decode_worker(void *arg) {
    DecodeJob *j = (DecodeJob *)arg;
    float *qf = (float *)malloc(sizeof(float) * (size_t)j->head_dim);
    float *acc = (float *)malloc(sizeof(float) * (size_t)j->head_dim);
    const int64_t units = (int64_t)j->batch * j->num_q_heads;
    for (;;) {
        int64_t u = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        if (u >= units) break;
        decode_unit(j, u, qf, acc);
    }
    free(qf);
    free(acc);
    return NULL;
}

int oracle_max_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

int oracle_decode(const void *q, const void *k_cache, const void *v_cache,
                  const int32_t *block_tables, const int32_t *context_lens, float *out,
                  int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                  int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                  const int64_t *q_strides, const int64_t *cache_strides,
                  const int64_t *bt_strides, const int64_t *out_strides, int32_t q_dtype,
                  int32_t kv_dtype, float scale, int32_t nthreads) {
    if (num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || head_dim <= 0 || block_size <= 0)
        return -1;
    DecodeJob job = {q, k_cache, v_cache, block_tables, context_lens, out, batch, num_q_heads,
                     num_kv_heads, head_dim, block_size, num_blocks, max_blocks, q_strides,
                     cache_strides, bt_strides, out_strides, q_dtype, kv_dtype, scale, 0};
    int n = nthreads > 0 ? nthreads : oracle_max_threads();
    const int64_t units = (int64_t)batch * num_q_heads;
    if (n > units) n = units > 0 ? (int)units : 1;
    if (n <= 1) {
        decode_worker(&job);
        return 0;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n);
    int started = 0;
    for (int i = 0; i < n; ++i)
        if (pthread_create(&th[i], NULL, decode_worker, &job) == 0) ++started;
    if (started == 0) decode_worker(&job);
    for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
    free(th);
    return 0;
}
