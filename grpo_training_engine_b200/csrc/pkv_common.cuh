// pkv_common.cuh — shared device helpers for the paged-KV kernels (sm_100a).
//
// Element conversion, bounded mbarrier waits, ldmatrix / mma.sync wrappers and the host-side error plumbing used by every
// entry point of libpkv.so.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pkv.h"

namespace pkv {

// ---------------------------------------------------------------------------
// host-side error detail (thread-local, read back by pkv_last_error_detail)
// ---------------------------------------------------------------------------
void set_error_detail(const char *fmt, ...);

// Launches the append kernel (pkv_copy.cu): writes k_new/v_new[b] at slot
// context_lens[b] + ctx_offset of sequence b.
int append_launch(const void *k_new, const void *v_new, void *k_cache, void *v_cache,
                  const int32_t *block_tables, const int32_t *context_lens, int32_t ctx_offset,
                  int32_t batch, int32_t num_heads, int32_t head_dim, int32_t block_size,
                  int32_t num_blocks, int32_t max_blocks, const int64_t *new_strides,
                  const int64_t *cache_strides, const int64_t *bt_strides, int32_t dtype,
                  int32_t *status, void *stream);

inline int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error_detail("%s: %s", what, cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

inline int dtype_size(int32_t dtype) {
  switch (dtype) {
    case PKV_DTYPE_F32: return 4;
    case PKV_DTYPE_BF16: return 2;
    case PKV_DTYPE_F16: return 2;
    default: return 0;
  }
}

inline bool aligned_to(const void *p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// ---------------------------------------------------------------------------
// element loads as fp32
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f32(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
};

__device__ __forceinline__ float load_as_f32(const void *base, int64_t idx, int32_t dtype) {
  switch (dtype) {
    case PKV_DTYPE_BF16:
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(base)[idx]);
    case PKV_DTYPE_F16:
      return __half2float(reinterpret_cast<const __half *>(base)[idx]);
    default:
      return reinterpret_cast<const float *>(base)[idx];
  }
}

__device__ __forceinline__ void flag_status(int32_t *status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---------------------------------------------------------------------------
// shared-memory addresses and mbarriers (PTX ISA 8.x)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Make mbarrier initialisation visible before other threads use the barriers.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that gives up after about ns nanoseconds (the suspend-time hint)
// instead of the hardware-defined interval
__device__ __forceinline__ bool mbar_try_wait_ns(uint64_t *bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Each try_wait suspends the thread for a
// hardware-defined interval, so kMaxTries bounds the wait to well under a
// minute. Returns false if the phase never completed.
constexpr uint32_t kMaxWaitTries = 1u << 22;

// Bounded wait for a thread on the critical path (a consumer waiting for its
// next element or for the group): polls every ~100 ns, so it resumes soon
// after the phase completes; 2^24 polls bound the wait to a few seconds.
constexpr uint32_t kPollNs = 100;
constexpr uint32_t kMaxPolls = 1u << 24;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint32_t max_polls = kMaxPolls) {
  for (uint32_t i = 0; i < max_polls; ++i) {
    if (mbar_try_wait_ns(bar, parity, kPollNs)) return true;
  }
  return false;
}

// Bounded wait for a thread that is usually AHEAD of the threads it waits for
// (a producer whose ring is full): after a few polls it sleeps with growing
// back-off, so it does not take issue slots from the warps it is waiting on.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t *bar, uint32_t parity,
                                                  uint32_t max_tries = kMaxWaitTries) {
  uint32_t sleep_ns = 32;
  for (uint32_t i = 0; i < max_tries; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 4) {
      __nanosleep(sleep_ns);
      if (sleep_ns < 512) sleep_ns <<= 1;
    }
  }
  return false;
}

// ---------------------------------------------------------------------------
// warp-level matrix helpers (bf16 / fp16 operands, fp32 accumulate)
// ---------------------------------------------------------------------------
// In-register transpose of an 8x8 matrix of 16-bit values held as m16n8k16
// fragments (lane 4r + c holds row r, columns 2c and 2c + 1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                              uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct Mma16816;

template <> struct Mma16816<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
  static __device__ __forceinline__ float unpack_lo(uint32_t v) { return __uint_as_float(v << 16); }
  static __device__ __forceinline__ float unpack_hi(uint32_t v) {
    return __uint_as_float(v & 0xffff0000u);
  }
};

template <> struct Mma16816<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
  static __device__ __forceinline__ float unpack_lo(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xffffu)));
  }
  static __device__ __forceinline__ float unpack_hi(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
  }
};

// 2^x with the hardware approximation (ex2.approx.ftz: relative error ~2^-22;
// -inf -> 0, results below 2^-126 flush to 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp2 that maps the fully-masked case (x = -inf) to 0 without NaNs.
__device__ __forceinline__ float exp2_or_zero(float x) { return x == -INFINITY ? 0.f : exp2f(x); }

}  // namespace pkv
