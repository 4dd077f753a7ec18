// pkv_glue.cu — the per-layer element-wise steps around the decode launch in a
// rollout step: residual add + RMSNorm, and RoPE of the new query/key rows.
//
// In the reference model loop (src/triton_kernels/paged_kv.py:699-808, with
// fused_ops.py's rmsnorm and q/k/v + RoPE) and in an HF Qwen2 layer these are
// each a handful of small torch kernels per layer (pow, mean, add, rsqrt, two
// multiplies and a cast for one RMSNorm; a concatenation, four multiplies and
// adds and two copies for RoPE, SiLU and a multiply in the MLP). Here each is
// one launch. The arithmetic keeps
// the HF module's rounding points:
//   RMSNorm (Qwen2RMSNorm): s = x + r rounded to the dtype when there is a
//     residual; v = fp32(s); y = dtype(v * rsqrt(mean(v^2) + eps));
//     out = dtype(w * y);
//   SiLU * up (Qwen2MLP): out = dtype(dtype(silu(gate)) * up);
//   RoPE (apply_rotary_pos_emb): out = dtype(dtype(q * cos) + dtype(rot(q) * sin)),
//     rot(q) = (-q[D/2:], q[:D/2]), every product and sum rounded to the dtype
//     as torch's bf16 element-wise ops do.
#include <algorithm>

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
constexpr int kNormVecs = 2;  // 16-byte vectors per thread: hidden sizes up to 256 x 2 x 16 B

// Loads / stores of 16 bytes as kV elements of T (the row offsets used are
// multiples of kV, and the host checks 16-byte alignment of rows).
template <typename T> struct Vec16 {
  static constexpr int kV = 16 / (int)sizeof(T);
  T e[kV];
};

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const T *x, const T *res, const T *w,
                                                                    T *sum_out, T *out, int H, int64_t xs,
                                                                    int64_t rs, int64_t ss, int64_t os,
                                                                    float eps) {
  using V = Vec16<T>;
  constexpr int kV = V::kV;
  __shared__ float red[kNormThreads / 32];
  // Programmatic dependent launch: the next kernel (a projection) may place
  // its CTAs and start its weight stream now; this grid waits for the
  // previous one before its first load.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  float v[kNormVecs][kV];
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kNormVecs; ++j) {
    const int i = (tid + j * kNormThreads) * kV;
    if (i < H) {
      const V xv = *reinterpret_cast<const V *>(x + b * xs + i);
      V rv;
      if (res != nullptr) rv = *reinterpret_cast<const V *>(res + b * rs + i);
      V sv;
#pragma unroll
      for (int e = 0; e < kV; ++e) {
        float s = Cvt<T>::f(xv.e[e]);
        if (res != nullptr) {
          sv.e[e] = Cvt<T>::t(s + Cvt<T>::f(rv.e[e]));  // the residual sum, rounded to T
          s = Cvt<T>::f(sv.e[e]);
        }
        v[j][e] = s;
        acc += s * s;
      }
      if (sum_out != nullptr) *reinterpret_cast<V *>(sum_out + b * ss + i) = sv;
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
  for (int j = 0; j < kNormVecs; ++j) {
    const int i = (tid + j * kNormThreads) * kV;
    if (i < H) {
      const V wv = *reinterpret_cast<const V *>(w + i);
      V ov;
#pragma unroll
      for (int e = 0; e < kV; ++e) ov.e[e] = Cvt<T>::t(Cvt<T>::f(wv.e[e]) * Cvt<T>::f(Cvt<T>::t(v[j][e] * r)));
      *reinterpret_cast<V *>(out + b * os + i) = ov;
    }
  }
}

// out = dtype(dtype(silu(gate)) * up), the rounding of HF's act_fn(gate) * up.
template <typename T>
__global__ void silu_mul_kernel(const T *gate, const T *up, T *out, int64_t n_vec, int cols, int64_t gs,
                                int64_t us) {
  using V = Vec16<T>;
  constexpr int kV = V::kV;
  const int vpr = cols / kV;  // vectors per row
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n_vec; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / vpr, c = (v - r * vpr) * kV;
    const V g = *reinterpret_cast<const V *>(gate + r * gs + c);
    const V u = *reinterpret_cast<const V *>(up + r * us + c);
    V o;
#pragma unroll
    for (int e = 0; e < kV; ++e) {
      const float x = Cvt<T>::f(g.e[e]);
      const float a = Cvt<T>::f(Cvt<T>::t(x / (1.f + expf(-x))));
      o.e[e] = Cvt<T>::t(a * Cvt<T>::f(u.e[e]));
    }
    *reinterpret_cast<V *>(out + r * (int64_t)cols + c) = o;
  }
}

// One CTA per row: threads over (head, d < D/2) pairs of the query and key heads.
template <typename T>
__global__ void rope_qk_kernel(const T *q, const T *k, const T *cosv, const T *sinv, T *qo, T *ko, int Hq,
                               int Hkv, int D, int64_t qs, int64_t ks, int64_t cs, int64_t qos, int64_t kos) {
  // the decode launch that follows may start its CTAs' setup now (it waits
  // for this grid before reading the rows written here)
  asm volatile("griddepcontrol.launch_dependents;");
  const int64_t b = blockIdx.x;
  const int half = D / 2;
  const int pairs = (Hq + Hkv) * half;
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const int h = p / half, d = p - h * half;
    const bool isq = h < Hq;
    const int hh = isq ? h : h - Hq;
    const T *src = isq ? q + b * qs + (int64_t)hh * D : k + b * ks + (int64_t)hh * D;
    // one thread reads and writes both elements of its pair: out may alias in
    T *dst = isq ? qo + b * qos + (int64_t)hh * D : ko + b * kos + (int64_t)hh * D;
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
  const int es = dtype_size(dtype);
  if (es == 0) return PKV_ERR_UNSUPPORTED;
  const int max_hidden = kNormThreads * kNormVecs * 16 / es;
  if (rows < 0 || hidden <= 0 || hidden > max_hidden || (hidden * es) % 16 != 0) {
    set_error_detail("pkv_add_rmsnorm: rows %d, hidden %d (a multiple of 16 bytes, at most %d elements)", rows,
                     hidden, max_hidden);
    return PKV_ERR_INVALID_ARG;
  }
  if (rows == 0) return PKV_OK;
  if (!x || !weight || !out || (sum_out && !residual)) {
    set_error_detail("pkv_add_rmsnorm: NULL pointer");
    return PKV_ERR_INVALID_ARG;
  }
  // rows are read and written as 16-byte vectors
  const void *ptrs[] = {x, residual, weight, sum_out, out};
  for (const void *p : ptrs)
    if (p && !aligned_to(p, 16)) return PKV_ERR_ALIGNMENT;
  const int64_t strides[] = {x_stride, residual ? residual_stride : 0, sum_out ? sum_stride : 0, out_stride};
  for (int64_t st : strides)
    if ((st * es) % 16 != 0) return PKV_ERR_ALIGNMENT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)rows);
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (dtype) {
    case PKV_DTYPE_BF16:
      e = cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<__nv_bfloat16>, (const __nv_bfloat16 *)x,
                             (const __nv_bfloat16 *)residual, (const __nv_bfloat16 *)weight,
                             (__nv_bfloat16 *)sum_out, (__nv_bfloat16 *)out, (int)hidden, x_stride,
                             residual_stride, sum_stride, out_stride, eps);
      break;
    case PKV_DTYPE_F16:
      e = cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<__half>, (const __half *)x, (const __half *)residual,
                             (const __half *)weight, (__half *)sum_out, (__half *)out, (int)hidden, x_stride,
                             residual_stride, sum_stride, out_stride, eps);
      break;
    default:
      e = cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel<float>, (const float *)x, (const float *)residual,
                             (const float *)weight, (float *)sum_out, (float *)out, (int)hidden, x_stride,
                             residual_stride, sum_stride, out_stride, eps);
      break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error_detail("pkv_add_rmsnorm: %s", cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return check_launch("pkv_add_rmsnorm");
}

extern "C" int pkv_silu_mul(const void *gate, const void *up, void *out, int32_t rows, int32_t cols,
                            int64_t gate_stride, int64_t up_stride, int32_t dtype, void *stream) {
  const int es = dtype_size(dtype);
  if (es == 0) return PKV_ERR_UNSUPPORTED;
  if (rows < 0 || cols <= 0 || (cols * es) % 16 != 0) {
    set_error_detail("pkv_silu_mul: rows %d, cols %d (a multiple of 16 bytes)", rows, cols);
    return PKV_ERR_INVALID_ARG;
  }
  if (rows == 0) return PKV_OK;
  if (!gate || !up || !out) {
    set_error_detail("pkv_silu_mul: NULL pointer");
    return PKV_ERR_INVALID_ARG;
  }
  const void *ptrs[] = {gate, up, out};
  for (const void *p : ptrs)
    if (!aligned_to(p, 16)) return PKV_ERR_ALIGNMENT;
  if ((gate_stride * es) % 16 != 0 || (up_stride * es) % 16 != 0) return PKV_ERR_ALIGNMENT;
  const int64_t n_vec = (int64_t)rows * cols * es / 16;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n_vec + threads - 1) / threads, 148 * 16);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PKV_DTYPE_BF16:
      silu_mul_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(
          (const __nv_bfloat16 *)gate, (const __nv_bfloat16 *)up, (__nv_bfloat16 *)out, n_vec, cols, gate_stride,
          up_stride);
      break;
    case PKV_DTYPE_F16:
      silu_mul_kernel<__half><<<(unsigned)blocks, threads, 0, st>>>((const __half *)gate, (const __half *)up,
                                                                    (__half *)out, n_vec, cols, gate_stride,
                                                                    up_stride);
      break;
    default:
      silu_mul_kernel<float><<<(unsigned)blocks, threads, 0, st>>>((const float *)gate, (const float *)up,
                                                                   (float *)out, n_vec, cols, gate_stride,
                                                                   up_stride);
      break;
  }
  return check_launch("pkv_silu_mul");
}

extern "C" int pkv_rope_qk(const void *q, const void *k, const void *cos_, const void *sin_, void *q_out,
                           void *k_out, int32_t rows, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t head_dim, int64_t q_stride, int64_t k_stride, int64_t cs_stride,
                           int64_t q_out_stride, int64_t k_out_stride, int32_t dtype, void *stream) {
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
          num_kv_heads, head_dim, q_stride, k_stride, cs_stride, q_out_stride, k_out_stride);
      break;
    case PKV_DTYPE_F16:
      rope_qk_kernel<__half><<<rows, threads, 0, st>>>(
          (const __half *)q, (const __half *)k, (const __half *)cos_, (const __half *)sin_, (__half *)q_out,
          (__half *)k_out, num_q_heads, num_kv_heads, head_dim, q_stride, k_stride, cs_stride, q_out_stride,
          k_out_stride);
      break;
    default:
      rope_qk_kernel<float><<<rows, threads, 0, st>>>((const float *)q, (const float *)k, (const float *)cos_,
                                                      (const float *)sin_, (float *)q_out, (float *)k_out,
                                                      num_q_heads, num_kv_heads, head_dim, q_stride,
                                                      k_stride, cs_stride, q_out_stride, k_out_stride);
      break;
  }
  return check_launch("pkv_rope_qk");
}
