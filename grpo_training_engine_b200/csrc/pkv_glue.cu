// pkv_glue.cu — the per-layer element-wise steps around the decode launch in a
// rollout step: residual add + RMSNorm, and RoPE of the new query/key rows.
//
// In the reference model loop (src/triton_kernels/paged_kv.py:699-808, with
// fused_ops.py's rmsnorm and q/k/v + RoPE) and in an HF Qwen2 layer these are
// each a handful of small torch kernels per layer (pow, mean, add, rsqrt, two
// multiplies and a cast for one RMSNorm; a concatenation, four multiplies and
// adds and two copies for RoPE). Here each is one launch. The arithmetic keeps
// the HF module's rounding points:
//   RMSNorm (Qwen2RMSNorm): s = x + r rounded to the dtype when there is a
//     residual; v = fp32(s); y = dtype(v * rsqrt(mean(v^2) + eps));
//     out = dtype(w * y);
//   RoPE (apply_rotary_pos_emb): out = dtype(dtype(q * cos) + dtype(rot(q) * sin)),
//     rot(q) = (-q[D/2:], q[:D/2]), every product and sum rounded to the dtype
//     as torch's bf16 element-wise ops do.
#include "pkv_common.cuh"

namespace pkv {
namespace {

template <typename T> struct Cvt;
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 t(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half t(float v) { return __float2half_rn(v); }
};
template <> struct Cvt<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float t(float v) { return v; }
};

constexpr int kNormThreads = 256;
constexpr int kNormPerThread = 16;  // hidden sizes up to 4096

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const T *x, const T *res, const T *w,
                                                                    T *sum_out, T *out, int H, int64_t xs,
                                                                    int64_t rs, int64_t ss, int64_t os,
                                                                    float eps) {
  __shared__ float red[kNormThreads / 32];
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  float v[kNormPerThread];
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kNormPerThread; ++j) {
    const int i = tid + j * kNormThreads;
    v[j] = 0.f;
    if (i < H) {
      float s = Cvt<T>::f(x[b * xs + i]);
      if (res != nullptr) {
        const T st = Cvt<T>::t(s + Cvt<T>::f(res[b * rs + i]));
        if (sum_out != nullptr) sum_out[b * ss + i] = st;
        s = Cvt<T>::f(st);
      }
      v[j] = s;
      acc += s * s;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((tid & 31) == 0) red[tid >> 5] = acc;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) tot += red[k];
  const float r = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kNormPerThread; ++j) {
    const int i = tid + j * kNormThreads;
    if (i < H) out[b * os + i] = Cvt<T>::t(Cvt<T>::f(w[i]) * Cvt<T>::f(Cvt<T>::t(v[j] * r)));
  }
}

// One CTA per row: threads over (head, d < D/2) pairs of the query and key heads.
template <typename T>
__global__ void rope_qk_kernel(const T *q, const T *k, const T *cosv, const T *sinv, T *qo, T *ko, int Hq,
                               int Hkv, int D, int64_t qs, int64_t ks, int64_t cs) {
  const int64_t b = blockIdx.x;
  const int half = D / 2;
  const int pairs = (Hq + Hkv) * half;
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const int h = p / half, d = p - h * half;
    const bool isq = h < Hq;
    const int hh = isq ? h : h - Hq;
    const T *src = isq ? q + b * qs + (int64_t)hh * D : k + b * ks + (int64_t)hh * D;
    T *dst = isq ? qo + (b * Hq + hh) * D : ko + (b * Hkv + hh) * D;
    const float x1 = Cvt<T>::f(src[d]), x2 = Cvt<T>::f(src[d + half]);
    const float c1 = Cvt<T>::f(cosv[b * cs + d]), c2 = Cvt<T>::f(cosv[b * cs + d + half]);
    const float s1 = Cvt<T>::f(sinv[b * cs + d]), s2 = Cvt<T>::f(sinv[b * cs + d + half]);
    const float a1 = Cvt<T>::f(Cvt<T>::t(x1 * c1)), b1 = Cvt<T>::f(Cvt<T>::t(-x2 * s1));
    const float a2 = Cvt<T>::f(Cvt<T>::t(x2 * c2)), b2 = Cvt<T>::f(Cvt<T>::t(x1 * s2));
    dst[d] = Cvt<T>::t(a1 + b1);
    dst[d + half] = Cvt<T>::t(a2 + b2);
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_add_rmsnorm(const void *x, const void *residual, const void *weight, void *sum_out,
                               void *out, int32_t rows, int32_t hidden, int64_t x_stride,
                               int64_t residual_stride, int64_t sum_stride, int64_t out_stride, float eps,
                               int32_t dtype, void *stream) {
  if (rows < 0 || hidden <= 0 || hidden > kNormThreads * kNormPerThread) {
    set_error_detail("pkv_add_rmsnorm: rows %d, hidden %d (at most %d)", rows, hidden,
                     kNormThreads * kNormPerThread);
    return PKV_ERR_INVALID_ARG;
  }
  if (rows == 0) return PKV_OK;
  if (!x || !weight || !out || (sum_out && !residual)) {
    set_error_detail("pkv_add_rmsnorm: NULL pointer");
    return PKV_ERR_INVALID_ARG;
  }
  const int es = dtype_size(dtype);
  if (es == 0) return PKV_ERR_UNSUPPORTED;
  const void *ptrs[] = {x, residual, weight, sum_out, out};
  for (const void *p : ptrs)
    if (p && !aligned_to(p, es)) return PKV_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PKV_DTYPE_BF16:
      add_rmsnorm_kernel<__nv_bfloat16><<<rows, kNormThreads, 0, st>>>(
          (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)residual, (const __nv_bfloat16 *)weight,
          (__nv_bfloat16 *)sum_out, (__nv_bfloat16 *)out, hidden, x_stride, residual_stride, sum_stride,
          out_stride, eps);
      break;
    case PKV_DTYPE_F16:
      add_rmsnorm_kernel<__half><<<rows, kNormThreads, 0, st>>>(
          (const __half *)x, (const __half *)residual, (const __half *)weight, (__half *)sum_out,
          (__half *)out, hidden, x_stride, residual_stride, sum_stride, out_stride, eps);
      break;
    default:
      add_rmsnorm_kernel<float><<<rows, kNormThreads, 0, st>>>(
          (const float *)x, (const float *)residual, (const float *)weight, (float *)sum_out, (float *)out,
          hidden, x_stride, residual_stride, sum_stride, out_stride, eps);
      break;
  }
  return check_launch("pkv_add_rmsnorm");
}

extern "C" int pkv_rope_qk(const void *q, const void *k, const void *cos_, const void *sin_, void *q_out,
                           void *k_out, int32_t rows, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t head_dim, int64_t q_stride, int64_t k_stride, int64_t cs_stride,
                           int32_t dtype, void *stream) {
  if (rows < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0) {
    set_error_detail("pkv_rope_qk: invalid sizes");
    return PKV_ERR_INVALID_ARG;
  }
  if (rows == 0) return PKV_OK;
  if (!q || !k || !cos_ || !sin_ || !q_out || !k_out) {
    set_error_detail("pkv_rope_qk: NULL pointer");
    return PKV_ERR_INVALID_ARG;
  }
  const int es = dtype_size(dtype);
  if (es == 0) return PKV_ERR_UNSUPPORTED;
  const void *ptrs[] = {q, k, cos_, sin_, q_out, k_out};
  for (const void *p : ptrs)
    if (!aligned_to(p, es)) return PKV_ERR_ALIGNMENT;
  const int pairs = (num_q_heads + num_kv_heads) * head_dim / 2;
  const int threads = pairs >= 512 ? 512 : ((pairs + 31) / 32) * 32;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PKV_DTYPE_BF16:
      rope_qk_kernel<__nv_bfloat16><<<rows, threads, 0, st>>>(
          (const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k, (const __nv_bfloat16 *)cos_,
          (const __nv_bfloat16 *)sin_, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)k_out, num_q_heads,
          num_kv_heads, head_dim, q_stride, k_stride, cs_stride);
      break;
    case PKV_DTYPE_F16:
      rope_qk_kernel<__half><<<rows, threads, 0, st>>>(
          (const __half *)q, (const __half *)k, (const __half *)cos_, (const __half *)sin_, (__half *)q_out,
          (__half *)k_out, num_q_heads, num_kv_heads, head_dim, q_stride, k_stride, cs_stride);
      break;
    default:
      rope_qk_kernel<float><<<rows, threads, 0, st>>>((const float *)q, (const float *)k, (const float *)cos_,
                                                      (const float *)sin_, (float *)q_out, (float *)k_out,
                                                      num_q_heads, num_kv_heads, head_dim, q_stride,
                                                      k_stride, cs_stride);
      break;
  }
  return check_launch("pkv_rope_qk");
}
