// pkv_linear.cu — the projections of a rollout decode step on 5th-generation
// tensor cores (tcgen05, sm_100a).
//
// A decode step multiplies a handful of activation rows (one per sequence of
// the batch, at most 128) by every weight matrix of the model once: q/k/v,
// o_proj, gate/up, down and the LM head (the nn.Linear calls of the
// reference's fused step, src/triton_kernels/paged_kv.py:699-808 and
// fused_ops.py:184-251). With so few rows this is weight streaming: each
// weight element is read once from HBM and used for <= 128 multiply-adds, so
// the bound is HBM bandwidth, and reaching it needs ~830 TFLOP/s of bf16
// tensor throughput at 6.5 TB/s — tcgen05 territory.
//
//   out[r, j] = sum_k x[r, k] * W[j, k]  (+ bias[j])        (act = 0)
//   out[r, j] = T(T(silu(T(g))) * T(u)),  g / u the same with the rows j and
//               n + j of W (the stacked gate / up weights)   (act = SiLU gate)
//
// W keeps nn.Linear's [out_features, in_features] layout (K contiguous): it is
// the K-major B operand as it lies in memory, so no transposed copy is made.
//
// One CTA computes one (column tile, K split) work item: all rows (the MMA M
// of 128; rows past `rows` are zero-filled by TMA) by BN columns.
//   warp 0, one thread : TMA loads of 64-wide K blocks of x and W into an
//                        S-stage shared-memory ring (128-byte swizzle)
//   warp 1             : allocates the TMEM accumulator; one thread issues
//                        tcgen05.mma (M 128, N BN, K 16) per 16 K and commits
//                        each stage back to the producer
//   warps 2-17 / 2-9   : epilogue: tcgen05.ld of the accumulator (warp w reads
//                        TMEM lanes 32 (w % 4) ..., four (two with a K split)
//                        warps per lane group on interleaved 16- (32-) column
//                        chunks), bias / activation, bf16 stores.
// Narrow matrices (N of a few thousand) are split along K so that ~148 CTAs
// stream every weight matrix. The splits of a tile are the CTAs of one thread-
// block cluster: each leaves its fp32 partial tile in its own shared memory,
// and after a cluster barrier every CTA sums a share of the rows over all the
// splits in split order (reading its peers' shared memory), so the result
// does not depend on which split finishes first and nothing goes through
// global memory. (A first version wrote the partials to global memory and let
// the last split add them: its fences, count and serial reduction took longer
// than the weight streaming.)
//
// Every wait is bounded; a wait that runs out sets PKV_DEV_WAIT_TIMEOUT, the
// thread stops issuing, waits (bounded) for its own copies / MMAs in flight,
// and the CTA frees its TMEM and returns.
#include <cuda.h>  // CUtensorMap and its enums (the encoder is reached through the runtime)

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int kLinBM = 128;      // rows of the MMA (all activation rows)
constexpr int kLinBK = 64;       // K elements per stage: one 128-byte swizzle row of 16-bit values
// Warp 0 TMA, warp 1 MMA, warps 2 .. 2 + EW - 1 epilogue: EW / 4 warps per
// 32-lane TMEM group, each taking every (EW / 4)-th chunk of accumulator
// columns. With one warp per group the epilogue's dependent convert / SiLU
// chains took ~5 us of a gate/up launch; tiles stored straight from TMEM use
// 16 warps on 16-column chunks (3.6 -> 3.0 us), split-K tiles, whose partials
// go to shared memory and whose cluster reduction uses every thread, 8 warps
// on 32-column chunks (16 measured slower there).
template <int EW>
struct LinEpi {
  static constexpr int kParts = EW / 4;              // warps per TMEM lane group
  static constexpr int kChunk = EW >= 16 ? 16 : 32;  // accumulator columns per tcgen05.ld
  static constexpr int kThreads = 64 + 32 * EW;      // threads of the CTA
  static constexpr int kEpiThreads = 32 * EW;
  static_assert(EW % 4 == 0 && 64 + 32 * EW <= 1024, "epilogue warps: a multiple of 4, at most 30");
};
constexpr int kLinEpiBarrier = 1;  // named barrier of the epilogue warps
constexpr int kLinMaxSplits = 8;   // K splits of a tile: the CTAs of one (portable) cluster

struct LinArgs {
  const void *bias;    // [n] or nullptr
  void *out;           // [rows, n] (row stride out_stride elements)
  int32_t *status;
  int64_t out_stride;
  int32_t rows, n, kblocks, tiles, splits;
  int32_t up_row;      // SiLU gate: first up row in the up tensor map (n when stacked under gate)
  int32_t static_w;    // W / w_up are written by no kernel in flight: stream them before the dependency wait
  uint32_t max_polls;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// 2-D tiled TMA load of box (x, y) of the tensor map into shared memory,
// completing on `bar`; this CTA's own shared memory is the only destination.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, M 128, N and formats in idesc; accumulate
// when `acc` is non-zero.
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor of a K-major tile stored as rows of 128
// bytes with the 128-byte swizzle (what TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B into a 1024-byte aligned buffer): 8-row groups
// 1024 bytes apart (stride byte offset), descriptor version 1, layout
// SWIZZLE_128B (2). The leading byte offset is unused for this layout.
__device__ __forceinline__ uint64_t sw128_desc(const void *tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor of a dense kind::f16 MMA: fp32 accumulator, A and B
// of the same 16-bit type (bf16 or f16), both K-major, M 128, N n.
__host__ __device__ constexpr uint32_t mma_idesc(bool bf16, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kLinBM >> 4) << 24);
}

// NC (16 or 32) consecutive fp32 columns of this thread's TMEM lane.
template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[NC]) {
  static_assert(NC == 16 || NC == 32, "tcgen05.ld 32x32b .x16 or .x32");
  if constexpr (NC == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Barrier of the epilogue threads. One lane may arrive later than the
// rest of its warp (it waited on an mbarrier alone), so the warp reconverges
// first and the barrier is the non-aligned form.
template <int NT>
__device__ __forceinline__ void epi_sync() {
  __syncwarp();
  asm volatile("barrier.sync %0, %1;" ::"n"(kLinEpiBarrier), "n"(NT) : "memory");
}

// Barrier over every thread of every CTA of the cluster, with release /
// acquire ordering of their shared-memory writes.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of this CTA's shared-memory location `addr` in the CTA of `rank`
// of the cluster.
__device__ __forceinline__ uint32_t map_cluster(uint32_t addr, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <typename T> struct LinCvt;
template <> struct LinCvt<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 t(float v) { return __float2bfloat16_rn(v); }
};
template <> struct LinCvt<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half t(float v) { return __float2half_rn(v); }
};


// One ring of S stages, each an x tile and a W tile. (Separate x and W rings,
// with the W ring deeper, measured slower: both streams are bound by their
// bytes in flight, and the x stream then ran short.)
template <int BN, int S>
struct LinSmem {
  static constexpr int kA = kLinBM * kLinBK * 2;  // one x stage: 128 rows x 128 bytes
  static constexpr int kB = BN * kLinBK * 2;      // one W stage: BN rows x 128 bytes
  static constexpr size_t kW = (size_t)S * kA;    // W tiles after the x tiles
  static constexpr size_t kFull = kW + (size_t)S * kB;
  static constexpr size_t kEmpty = kFull + 8 * S;
  static constexpr size_t kAcc = kEmpty + 8 * S;
  static constexpr size_t kTmem = kAcc + 8;   // TMEM base address written by tcgen05.alloc
  static constexpr size_t kFlag = kTmem + 4;  // epilogue broadcast
  static constexpr size_t kBytes = kFlag + 4 + 1024;  // + alignment slack
};

constexpr int kActNone = 0, kActSiluGate = 1;

// TMEM columns of the accumulator: a power of two >= 32, >= BN
template <int BN> struct TmemCols {
  static constexpr uint32_t value = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

__device__ __forceinline__ uint32_t bits16(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }
__device__ __forceinline__ uint32_t bits16(__half v) { return __half_as_ushort(v); }

// Final value of NC columns of one row: bias / activation, rounding, store.
template <typename T, int ACT, int NC>
__device__ __forceinline__ void store_row(const LinArgs &a, int row, int col0, const float (&v)[NC],
                                          const float (&up)[NC]) {
  using C = LinCvt<T>;
  T *out = reinterpret_cast<T *>(a.out) + row * a.out_stride;
  const T *bias = reinterpret_cast<const T *>(a.bias);
  T o[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    if constexpr (ACT == kActSiluGate) {
      // HF Qwen2MLP: gate and up rounded as GEMM outputs, silu rounded, product rounded
      const float g = C::f(C::t(v[j]));
      const float s = C::f(C::t(g / (1.f + expf(-g))));
      o[j] = C::t(s * C::f(C::t(up[j])));
    } else {
      const int c = col0 + j;
      o[j] = C::t(bias != nullptr && c < a.n ? v[j] + C::f(bias[c]) : v[j]);
    }
  }
  if (col0 + NC <= a.n && (reinterpret_cast<uintptr_t>(out + col0) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < NC / 8; ++q) {
      uint4 w;
      w.x = bits16(o[8 * q + 0]) | (bits16(o[8 * q + 1]) << 16);
      w.y = bits16(o[8 * q + 2]) | (bits16(o[8 * q + 3]) << 16);
      w.z = bits16(o[8 * q + 4]) | (bits16(o[8 * q + 5]) << 16);
      w.w = bits16(o[8 * q + 6]) | (bits16(o[8 * q + 7]) << 16);
      reinterpret_cast<uint4 *>(out + col0)[q] = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < NC; ++j)
      if (col0 + j < a.n) out[col0 + j] = o[j];
  }
}

// Four consecutive results of one row (+ bias), rounded, at column col (a
// multiple of 4; out rows are 16-byte aligned, so 8 bytes when in range).
template <typename T>
__device__ __forceinline__ void store_4(const LinArgs &a, int row, int col, float4 v) {
  using C = LinCvt<T>;
  T *out = reinterpret_cast<T *>(a.out) + row * a.out_stride + col;
  const T *bias = reinterpret_cast<const T *>(a.bias);
  const float e[4] = {v.x, v.y, v.z, v.w};
  T o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = C::t(bias != nullptr && col + j < a.n ? e[j] + C::f(bias[col + j]) : e[j]);
  if (col + 4 <= a.n) {
    *reinterpret_cast<uint2 *>(out) =
        make_uint2(bits16(o[0]) | (bits16(o[1]) << 16), bits16(o[2]) | (bits16(o[3]) << 16));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (col + j < a.n) out[j] = o[j];
  }
}

template <typename T, int BN, int S, int ACT, int EW>
__global__ void __launch_bounds__(LinEpi<EW>::kThreads, 1)
linear_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
              const __grid_constant__ CUtensorMap tu, LinArgs a) {
  using L = LinSmem<BN, S>;
  using E = LinEpi<EW>;
  extern __shared__ uint8_t lin_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(lin_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *sa = smem;           // S x tiles (1024-byte aligned: kA is a multiple of 1024)
  uint8_t *sb = smem + L::kW;   // S W tiles
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kFull);
  uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L::kEmpty);
  uint64_t *acc_full = reinterpret_cast<uint64_t *>(smem + L::kAcc);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kTmem);
  int32_t *flag = reinterpret_cast<int32_t *>(smem + L::kFlag);
  static_assert(L::kA % 1024 == 0 && L::kB % 1024 == 0, "swizzled tiles stay 1024-byte aligned");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / a.splits, split = blockIdx.x - tile * a.splits;
  constexpr int kCols = ACT == kActSiluGate ? BN / 2 : BN;  // output columns of a tile
  const int n0 = tile * kCols;
  const int kb0 = (int)((int64_t)split * a.kblocks / a.splits);
  const int kb1 = (int)((int64_t)(split + 1) * a.kblocks / a.splits);
  const int nkb = kb1 - kb0;  // >= 1: the host keeps splits <= kblocks

  // W tiles of K block i (the gate and up rows for the SiLU gate) into stage s
  auto load_w = [&](int s, int i) {
    const int kx = (kb0 + i) * kLinBK;
    if constexpr (ACT == kActSiluGate) {
      tma_load_2d(sb + s * L::kB, &tw, kx, n0, &full[s]);                          // gate rows
      tma_load_2d(sb + s * L::kB + L::kB / 2, &tu, kx, a.up_row + n0, &full[s]);  // up rows
    } else {
      tma_load_2d(sb + s * L::kB, &tw, kx, n0, &full[s]);
    }
  };
  // stages whose W tiles are issued before the dependency wait
  const int pre = a.static_w ? (nkb < S ? nkb : S) : 0;

  // Programmatic dependent launch: the next kernel in the stream may place its
  // CTAs on SMs this grid frees, and it waits (griddepcontrol.wait) for this
  // grid to complete before it reads memory; this grid likewise initialises
  // its barriers and TMEM (and, with static weights, starts its weight
  // stream) before waiting for the previous kernel.
  asm volatile("griddepcontrol.launch_dependents;");
  if (threadIdx.x == 32) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
    if (ACT == kActSiluGate) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tu)) : "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    // make the initialised barriers visible to the async proxy (TMA, tcgen05)
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // the first stages' weights: each stage's barrier expects its x tile too,
    // which is loaded after the wait
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&full[i], L::kA + L::kB);
      load_w(i, i);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TmemCols<BN>::value)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // from here on the previous kernel (which may have written x, W, the bias or
  // the output) is complete and its writes are visible
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ============================ TMA producer ============================
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S, use = i / S;
        if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1, a.max_polls)) {
          flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
          break;
        }
        if (i >= pre) {  // (stages below `pre` have their W tiles and byte count already)
          mbar_expect_tx(&full[s], L::kA + L::kB);
          load_w(s, i);
        }
        tma_load_2d(sa + s * L::kA, &tx, (kb0 + i) * kLinBK, 0, &full[s]);
        ++issued;
      }
      // the last load of each stage has landed before the CTA (and its shared
      // memory) goes away, also if the MMA thread stopped consuming
      for (int i = issued > S ? issued - S : 0; i < issued; ++i) {
        if (!mbar_wait_bounded(&full[i % S], (i / S) & 1, a.max_polls)) flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
      }
    }
  } else if (warp == 1) {
    // ============================ MMA issuer ==============================
    if (lane == 0) {
      constexpr uint32_t idesc = mma_idesc(std::is_same<T, __nv_bfloat16>::value, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (!mbar_wait_bounded(&full[s], (i / S) & 1, a.max_polls)) {
          flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint64_t ad = sw128_desc(sa + s * L::kA), bd = sw128_desc(sb + s * L::kB);
#pragma unroll
        for (int kk = 0; kk < kLinBK / 16; ++kk)  // K 16 per MMA: 32 bytes further along the swizzled rows
          tc_mma(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
      }
      tc_commit(acc_full);  // the accumulator is complete once every MMA above is
    }
  } else {
    // ============================ epilogue ================================
    const int lg = warp & 3;  // TMEM lanes 32 lg .. 32 lg + 31 are readable by this warp
    const int part = (warp - 2) >> 2;  // which of the group's warps: its column chunks
    const int row = lg * 32 + lane;
    if (threadIdx.x == 64) *flag = mbar_wait_bounded(acc_full, 0, a.max_polls) ? 1 : 0;
    epi_sync<E::kEpiThreads>();
    const bool ready = *flag != 0;
    epi_sync<E::kEpiThreads>();  // every epilogue thread has read the flag before it is reused
    if (!ready) {
      if (threadIdx.x == 64) flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
    } else {
      tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(lg * 32) << 16);
      if (a.splits == 1) {
        for (int c0 = E::kChunk * part; c0 < kCols; c0 += E::kChunk * E::kParts) {
          uint32_t r[E::kChunk];
          float v[E::kChunk], u[E::kChunk];
          tmem_ld<E::kChunk>(trow + c0, r);
#pragma unroll
          for (int j = 0; j < E::kChunk; ++j) v[j] = __uint_as_float(r[j]);
          if constexpr (ACT == kActSiluGate) {
            tmem_ld<E::kChunk>(trow + BN / 2 + c0, r);
#pragma unroll
            for (int j = 0; j < E::kChunk; ++j) u[j] = __uint_as_float(r[j]);
          }
          if (row < a.rows && n0 + c0 < a.n) store_row<T, ACT, E::kChunk>(a, row, n0 + c0, v, u);
        }
      } else {
        // split-K: this split's fp32 partial tile into its own shared memory
        // (the stage buffers are idle once every MMA has completed), summed
        // across the cluster below
        float *tile_s = reinterpret_cast<float *>(smem) + row * (BN + 4);
        for (int c0 = E::kChunk * part; c0 < BN; c0 += E::kChunk * E::kParts) {
          uint32_t r[E::kChunk];
          tmem_ld<E::kChunk>(trow + c0, r);
#pragma unroll
          for (int q = 0; q < E::kChunk / 4; ++q)
            reinterpret_cast<float4 *>(tile_s + c0)[q] =
                make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                            __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
        }
      }
    }
    tc_fence_before();
  }
  __syncwarp();  // warps 0 and 1: lane 0 rejoins the rest of its warp
  __syncthreads();
  if (a.splits > 1) {
    // The K splits of a tile are the CTAs of one cluster (rank = split). Every
    // partial tile is in its CTA's shared memory; CTA `split` sums the rows
    // r = split, split + splits, ... of all of them in split order (shared
    // memory of the peers through the cluster window), adds the bias and
    // stores the 16-bit result. The second cluster barrier keeps every tile
    // alive until its peers have read it.
    cluster_sync();
    const uint32_t base = smem_u32(smem);
    constexpr int kC4 = kCols / 4;
    const int my_rows = (kLinBM - split + a.splits - 1) / a.splits;
    for (int it = threadIdx.x; it < my_rows * kC4; it += E::kThreads) {
      const int row = split + (it / kC4) * a.splits, c4 = it % kC4;
      if (row >= a.rows || n0 + 4 * c4 >= a.n) continue;
      const uint32_t off = (uint32_t)((row * (BN + 4) + 4 * c4) * sizeof(float));
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp = 0; sp < a.splits; ++sp) {
        const float4 p = ld_cluster_f4(map_cluster(base + off, sp));
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
      store_4<T>(a, row, n0 + 4 * c4, acc);
    }
    cluster_sync();
  }
  if (warp == 1) {
    // every MMA has completed before the accumulator's columns are freed
    if (lane == 0 && !mbar_wait_bounded(acc_full, 0, a.max_polls)) flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TmemCols<BN>::value)
                 : "memory");
  }
}


// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
    cudaGetLastError();
  });
  return fn;
}

// 2-D map of a row-major [rows, k] matrix of 16-bit values, boxes of 64 (k)
// by box_rows rows, 128-byte swizzle, zero fill outside the matrix.
int encode_2d(CUtensorMap *map, const void *base, bool bf16, int64_t k, int64_t rows, int64_t row_stride,
              uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error_detail("pkv_linear: cuTensorMapEncodeTiled is not available from the driver");
    return PKV_ERR_TENSOR_MAP;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kLinBK, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void *>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error_detail("pkv_linear: cuTensorMapEncodeTiled failed (%d) for a [%lld, %lld] matrix", (int)r,
                     (long long)rows, (long long)k);
    return PKV_ERR_TENSOR_MAP;
  }
  return PKV_OK;
}

int lin_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return 148;
  }
  return sms;
}

// Tile width and K splits of one call. The SiLU gate uses 64 gate +
// 64 up rows per tile (MMA N 128) and no split (its K of a few thousand and N
// of ~9000 columns give ~140 tiles); wide matrices (the LM head) use tiles of
// 256 columns; the rest 64-column tiles with K split so that tiles x splits
// fill the SMs once (q/k/v 32 x 4, o_proj and down_proj 24 x 6 on B200).
struct LinPlan {
  int bn, tiles, splits, kblocks;
};

LinPlan lin_plan(int32_t n, int32_t k, int32_t act, int sms) {
  LinPlan p{};
  p.kblocks = k / kLinBK;
  if (act == kActSiluGate) {
    // 64 gate + 64 up rows per tile, no split (8960 columns: 140 tiles). 128 +
    // 128 rows with K split in two (a cluster of 2) measured slower on B200:
    // 20.1 us against 16.3 for the 1.5B model's gate / up at 128 rows.
    p.bn = 128;
    p.tiles = (n + 63) / 64;
    p.splits = 1;
  } else if ((int64_t)n >= (int64_t)sms * 128) {
    p.bn = 256;
    p.tiles = (n + 255) / 256;
    p.splits = 1;
  } else {
    // measured on B200 at 128 rows: long K (down_proj, K 8960) is fastest as
    // 128-column tiles x 8 splits (12 clusters of 8), short K (q/k/v, o_proj)
    // as 64-column tiles x 4 splits; clusters of 6 or of 8 with 16 or more
    // clusters did not all fit at once (one 200 KB CTA per SM)
    const bool long_k = p.kblocks >= 64;
    p.bn = long_k ? 128 : 64;
    p.tiles = (n + p.bn - 1) / p.bn;
    p.splits = std::max(1, std::min({p.kblocks, long_k ? kLinMaxSplits : 4, sms / std::max(1, p.tiles)}));
  }
  return p;
}

template <typename T, int BN, int S, int ACT, int EW>
int lin_launch(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &tu, const LinArgs &a,
               cudaStream_t st) {
  using L = LinSmem<BN, S>;
  static_assert(L::kBytes <= 227 * 1024, "linear kernel exceeds 227 KB of shared memory");
  static_assert(kLinBM * (BN + 4) * sizeof(float) <= L::kFull, "the split-K partial tile fits the ring");
  auto kern = linear_kernel<T, BN, S, ACT, EW>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kBytes) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute(linear)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.tiles * a.splits));
  cfg.blockDim = dim3(LinEpi<EW>::kThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // the K splits of a tile: one cluster
  attr[1].val.clusterDim.x = (unsigned)a.splits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.splits > 1 ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, tx, tw, tu, a) != cudaSuccess) return check_launch("linear_kernel");
  return check_launch("linear_kernel");
}

template <typename T>
int lin_dispatch(const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &tu, const LinArgs &a, int bn,
                 int act, cudaStream_t st) {
  // 16 epilogue warps where tiles are stored from TMEM, 8 where they are summed
  // across a K-split cluster (the plan never splits gate/up or 256-column tiles)
  if (act == kActSiluGate) return lin_launch<T, 128, 6, kActSiluGate, 16>(tx, tw, tu, a, st);
  if (bn == 256) return lin_launch<T, 256, 4, kActNone, 16>(tx, tw, tu, a, st);
  if (bn == 128)
    return a.splits > 1 ? lin_launch<T, 128, 6, kActNone, 8>(tx, tw, tu, a, st)
                        : lin_launch<T, 128, 6, kActNone, 16>(tx, tw, tu, a, st);
  return a.splits > 1 ? lin_launch<T, 64, 8, kActNone, 8>(tx, tw, tu, a, st)
                      : lin_launch<T, 64, 8, kActNone, 16>(tx, tw, tu, a, st);
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_linear(const void *x, const void *w, const void *w_up, const void *bias, void *out,
                          int32_t rows, int32_t n, int32_t k, int64_t x_stride, int64_t w_stride,
                          int64_t out_stride, int32_t dtype, int32_t act, int32_t *status, void *stream) {
  if (rows <= 0 || rows > kLinBM || n <= 0 || k <= 0) {
    set_error_detail("pkv_linear: rows must be in [1, %d] and n, k positive (rows %d, n %d, k %d)", kLinBM, rows,
                     n, k);
    return PKV_ERR_INVALID_ARG;
  }
  if (dtype != PKV_DTYPE_BF16 && dtype != PKV_DTYPE_F16) {
    set_error_detail("pkv_linear: x, W and out must be bf16 or fp16");
    return PKV_ERR_UNSUPPORTED;
  }
  const bool static_w = (act & PKV_LINEAR_WEIGHTS_STATIC) != 0;
  act &= ~PKV_LINEAR_WEIGHTS_STATIC;
  if (act != PKV_LINEAR_NONE && act != PKV_LINEAR_SILU_GATE) {
    set_error_detail("pkv_linear: unknown activation %d", act);
    return PKV_ERR_INVALID_ARG;
  }
  if (k % kLinBK != 0) {
    set_error_detail("pkv_linear: in_features %d is not a multiple of %d", k, kLinBK);
    return PKV_ERR_UNSUPPORTED;
  }
  if (act == 1 && (n % 64 != 0 || bias != nullptr)) {
    set_error_detail("pkv_linear: the SiLU gate needs n a multiple of 64 and no bias");
    return PKV_ERR_UNSUPPORTED;
  }
  if (!x || !w || !out) {
    set_error_detail("pkv_linear: NULL tensor pointer");
    return PKV_ERR_INVALID_ARG;
  }
  // TMA: 16-byte aligned bases and row strides; 16-byte output rows for the vector stores
  if (w_up != nullptr && act != 1) {
    set_error_detail("pkv_linear: w_up is only used by the SiLU gate");
    return PKV_ERR_INVALID_ARG;
  }
  if (!aligned_to(x, 16) || !aligned_to(w, 16) || !aligned_to(out, 16) || x_stride < k || w_stride < k ||
      (w_up != nullptr && !aligned_to(w_up, 16)) ||
      out_stride < n || (x_stride * 2) % 16 != 0 || (w_stride * 2) % 16 != 0 || (out_stride * 2) % 16 != 0 ||
      (bias != nullptr && !aligned_to(bias, 2))) {
    set_error_detail("pkv_linear: x, W and out need 16-byte aligned bases and row strides (elements: x %lld, "
                     "W %lld, out %lld)", (long long)x_stride, (long long)w_stride, (long long)out_stride);
    return PKV_ERR_ALIGNMENT;
  }
  const LinPlan p = lin_plan(n, k, act, lin_sms());
  const bool bf16 = dtype == PKV_DTYPE_BF16;
  CUtensorMap tx, tw;
  int rc = encode_2d(&tx, x, bf16, k, rows, x_stride, kLinBM);
  if (rc) return rc;
  // the SiLU gate's up rows: a separate [n, k] matrix (same row stride), or
  // rows n .. 2n - 1 of W
  const int64_t w_rows = (act == 1 && w_up == nullptr) ? 2 * (int64_t)n : n;
  rc = encode_2d(&tw, w, bf16, k, w_rows, w_stride, act == 1 ? p.bn / 2 : p.bn);
  if (rc) return rc;
  CUtensorMap tu = tw;
  if (w_up != nullptr) {
    rc = encode_2d(&tu, w_up, bf16, k, n, w_stride, p.bn / 2);
    if (rc) return rc;
  }
  LinArgs a{};
  a.bias = bias;
  a.out = out;
  a.status = status;
  a.out_stride = out_stride;
  a.rows = rows;
  a.n = n;
  a.kblocks = p.kblocks;
  a.tiles = p.tiles;
  a.splits = p.splits;
  a.up_row = w_up != nullptr ? 0 : n;
  a.static_w = static_w ? 1 : 0;
  a.max_polls = kMaxPolls;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return bf16 ? lin_dispatch<__nv_bfloat16>(tx, tw, tu, a, p.bn, act, st)
              : lin_dispatch<__half>(tx, tw, tu, a, p.bn, act, st);
}
