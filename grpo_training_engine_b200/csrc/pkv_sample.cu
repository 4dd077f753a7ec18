// pkv_sample.cu — temperature + top-p (nucleus) sampling of one token per row.
//
// The reference samples with a full sort of the vocabulary per row
// (src/triton_kernels/paged_kv.py:418-450, the same rule as
// fused_ops.py:236-248): scaled = logits / max(T, 1e-6) in the logits dtype,
// sort descending, softmax, running sum, drop every sorted token whose running
// sum exceeds top_p except the first, renormalise, multinomial draw. At a
// 151,936-token vocabulary that sort is most of a rollout step's sampling time.
//
// Here one CTA handles one row without sorting. A token's mass is the fp32
// exp of its scaled logit minus the row max, as 40-bit fixed point, so sums
// are exact and independent of the order of summation (a probability is a
// mass over the row total; below 2^-40 counts as 0). The cut is the scaled
// value of the first token, in descending order, whose running mass exceeds
// top_p x total: tokens above it are kept, and of the tokens tied at it the
// ones that fit under top_p in index order (the order a stable sort gives
// equal keys), and always the most likely token. The draw scales the caller's
// uniform u in [0, 1) by the kept mass and inverts it over the kept tokens in
// index order. The reference rounds probabilities and their running sum to
// the logits dtype, so a token whose running probability lies within that
// rounding of top_p can fall on the other side of the cut.
//
// 16-bit logits (top_p16_kernel): a scaled logit and its mass depend only on
// the token's 16-bit pattern, and the scaling is monotone in it. So the CTA
//   1. finds the largest pattern (in value order) of the row;
//   2. counts the row's tokens per pattern in a window of the 49,152 patterns
//      below it (every pattern under the window has zero mass; otherwise the
//      radix path below runs);
//   3. finds the cut from the counts alone: a scan of count x mass over the
//      window, then a warp's search for the tie group's pattern range;
//   4. reads the row once more for the draw, looking each kept token's mass
//      up by its pattern.
// Three passes over the row, with a shared-memory increment as the only
// per-token work besides the loads.
//
// fp32 logits, and rows whose window does not fit (fp16 at high temperature;
// a +inf or NaN logit; all -inf), take the radix path: the max, then the cut
// by a radix select over 8-bit digits of the order key of the scaled logit
// (two passes for bf16, three for fp16, four for fp32), each pass a 256-bin
// histogram of mass (one per warp, lanes with equal digits summed with warp
// match / reduce), then the draw with masses computed per token.
#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kBins = 256;
constexpr int kTableBytes = 65536 * 2;
constexpr int kHistBytes = kSampleWarps * kBins * 8;  // per-warp fixed-point mass histograms

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Scaled logit as the reference computes it: logits / T rounded to the logits
// dtype. For 16-bit logits it depends only on the 16-bit pattern, so it is
// looked up in a 65,536-entry table that each CTA fills once (128 KB of smem).
template <typename L> struct Scaled;
template <> struct Scaled<float> {
  static constexpr bool kTable = false;
  static __device__ __forceinline__ float get(const float *row, int i, float t, const uint16_t *) {
    return __fdiv_rn(row[i], t);
  }
  static __device__ __forceinline__ uint16_t scale_bits(uint16_t, float) { return 0; }
};
template <> struct Scaled<__nv_bfloat16> {
  static constexpr bool kTable = true;
  static __device__ __forceinline__ uint16_t scale_bits(uint16_t raw, float t) {
    const float v = __bfloat162float(__ushort_as_bfloat16(raw));
    return __bfloat16_as_ushort(__float2bfloat16_rn(__fdiv_rn(v, t)));
  }
  static __device__ __forceinline__ float get(const __nv_bfloat16 *row, int i, float, const uint16_t *tbl) {
    return __bfloat162float(__ushort_as_bfloat16(tbl[__bfloat16_as_ushort(row[i])]));
  }
};
template <> struct Scaled<__half> {
  static constexpr bool kTable = true;
  static __device__ __forceinline__ uint16_t scale_bits(uint16_t raw, float t) {
    const float v = __half2float(__ushort_as_half(raw));
    return __half_as_ushort(__float2half_rn(__fdiv_rn(v, t)));
  }
  static __device__ __forceinline__ float get(const __half *row, int i, float, const uint16_t *tbl) {
    return __half2float(__ushort_as_half(tbl[__half_as_ushort(row[i])]));
  }
};

struct SampleArgs {
  const void *logits;
  int64_t row_stride;
  int32_t vocab;
  float temperature;
  float top_p;
  const float *uniforms;
  int64_t *out;
  int32_t flags;
};

// Masses are exp(x - row max) as 40-bit fixed point: integer sums are exact
// and independent of the order of summation (below 2^-40 counts as 0).

// The radix path for one row (the CTA's), all threads of the CTA.
template <typename L, int KEY_BITS>
__device__ __forceinline__ void radix_top_p(const SampleArgs &a, uint8_t *sample_smem) {
  unsigned long long *whist = reinterpret_cast<unsigned long long *>(sample_smem);  // [warps][bins]
  uint16_t *scaled_tbl = reinterpret_cast<uint16_t *>(sample_smem + kHistBytes);    // 16-bit logits
  __shared__ float redm[kSampleWarps];
  __shared__ unsigned long long s_top;  // top_p x the row's total mass
  __shared__ unsigned long long hmass[kBins];
  __shared__ unsigned long long wmass[kSampleWarps];
  __shared__ int wties[kSampleWarps];
  __shared__ uint32_t s_prefix;
  __shared__ unsigned long long s_above;
  __shared__ int s_found;
  __shared__ int s_pick;
  const L *row = reinterpret_cast<const L *>(a.logits) + (int64_t)blockIdx.x * a.row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.vocab;
  const float t = a.temperature;
  if constexpr (Scaled<L>::kTable) {
    for (int r = tid; r < 65536; r += kSampleThreads) scaled_tbl[r] = Scaled<L>::scale_bits((uint16_t)r, t);
    __syncthreads();
  }
  auto scaled = [&](int i) { return Scaled<L>::get(row, i, t, scaled_tbl); };
  // The row is read as 16-byte vectors of kVec tokens (scalar loads when the
  // row is not 16-byte aligned), two vectors per thread per step, so each
  // thread keeps two loads in flight instead of one token.
  constexpr int kVec = 16 / (int)sizeof(L);
  constexpr int kStep = kSampleThreads * kVec;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  // scaled values of tokens [base, base + kVec); n of them are < V
  auto fetch = [&](int base, float (&x)[kVec]) -> int {
    const int n = max(0, min(kVec, V - base));
    if (vec_ok && n == kVec) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(row + base);
      const L *e = reinterpret_cast<const L *>(&raw);
#pragma unroll
      for (int j = 0; j < kVec; ++j) x[j] = Scaled<L>::get(e, j, t, scaled_tbl);
    } else {
#pragma unroll
      for (int j = 0; j < kVec; ++j) x[j] = j < n ? scaled(base + j) : -INFINITY;
    }
    return n;
  };

  // ---- 1. row max. Masses below are e = exp(x - max) in 40-bit fixed point
  // (e <= 1); the row sum of e comes out of the first histogram as its total,
  // and the nucleus bound is top_p times that sum, so no division per token.
  float m = -INFINITY;
  for (int b0 = tid * kVec; b0 < V; b0 += 2 * kStep) {
    float x0[kVec], x1[kVec];
    fetch(b0, x0);
    fetch(b0 + kStep, x1);
#pragma unroll
    for (int j = 0; j < kVec; ++j) m = fmaxf(m, fmaxf(x0[j], x1[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) redm[warp] = m;
  __syncthreads();
  m = lane < kSampleWarps ? redm[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float row_max = m;
  auto pfix = [&](float x) -> unsigned long long {
    return __float2ull_rn(expf(x - row_max) * 1099511627776.0f);  // * 2^40
  };

  // ---- 2. radix select of the cut key, 8 bits per pass from the top
  if (tid == 0) {
    s_prefix = 0;
    s_above = 0;
    s_found = 0;
  }
  unsigned long long *myhist = whist + warp * kBins;
  constexpr int kPasses = KEY_BITS / 8;
  // Keys of 16-bit values converted to fp32 carry their information in the top
  // KEY_BITS bits; the rest are 0 for positive values and 1 for negative ones
  // (the order key complements those). They are cleared, so every token of one
  // scaled value has the same key and the selected prefix is that key.
  constexpr uint32_t kLowMask = KEY_BITS >= 32 ? 0u : (1u << (32 - KEY_BITS)) - 1u;
  auto rkey = [](float x) { return order_key(x) & ~kLowMask; };
#pragma unroll 1
  for (int pass = 0; pass < kPasses; ++pass) {
    const int shift = 32 - 8 * (pass + 1);
    for (int b = tid; b < kSampleWarps * kBins; b += kSampleThreads) whist[b] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    // every lane of the warp runs the same number of steps (the sync ops below)
    for (int s0 = 0; s0 < V; s0 += 2 * kStep) {
      float xs[2][kVec];
      const int n0 = fetch(s0 + tid * kVec, xs[0]);
      const int n1 = fetch(s0 + kStep + tid * kVec, xs[1]);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const float x = xs[h][j];
          const uint32_t k = rkey(x);
          const bool in = j < (h ? n1 : n0) && (pass == 0 || (k >> (shift + 8)) == (prefix >> (shift + 8)));
          const uint32_t digit = in ? (k >> shift) & 0xffu : kBins;  // kBins: a group of its own
          const unsigned long long p = in ? pfix(x) : 0ull;
          // lanes with the same digit sum their masses (two 20-bit halves,
          // exact) and the lowest of them adds the sum to the warp's histogram
          const unsigned grp = __match_any_sync(0xffffffffu, digit);
          const unsigned hs = __reduce_add_sync(grp, (unsigned)(p >> 20));
          const unsigned ls = __reduce_add_sync(grp, (unsigned)(p & 0xfffffu));
          if (in && lane == __ffs(grp) - 1) myhist[digit] += ((unsigned long long)hs << 20) + ls;
        }
      }
    }
    __syncthreads();
    for (int b = tid; b < kBins; b += kSampleThreads) {
      unsigned long long h = 0;
#pragma unroll 8
      for (int w = 0; w < kSampleWarps; ++w) h += whist[w * kBins + b];
      hmass[b] = h;
    }
    __syncthreads();
    if (tid == 0) {
      if (pass == 0) {  // the row's total mass; the nucleus bound top_p x total
        unsigned long long tot = 0;
        for (int b = 0; b < kBins; ++b) tot += hmass[b];
        s_top = (unsigned long long)fmin((double)a.top_p * (double)tot, 4.0 * (double)tot);
      }
      const unsigned long long top_p = s_top;
      // first digit, from the top, at which the running mass exceeds top_p
      unsigned long long run = s_above;
      int d = kBins - 1;
      for (; d >= 0; --d) {
        if (hmass[d] == 0) continue;
        if (run + hmass[d] > top_p) break;
        run += hmass[d];
      }
      if (d < 0) {  // everything fits: the cut is below the smallest key
        s_found = 0;
      } else {
        s_found = 1;
        s_above = run;
        s_prefix = (pass == 0 ? 0u : s_prefix) | ((uint32_t)d << shift);
      }
    }
    __syncthreads();
    if (!s_found) break;
  }
  const bool found = s_found != 0;
  const uint32_t cut = s_prefix;
  const unsigned long long above = s_above;
  const unsigned long long top_p = s_top;
  // tokens tied at the cut key that stay: while the running mass is <= top_p,
  // and at least one token overall (the most likely one); the final pass caps
  // it by the number of ties there are
  const unsigned long long pc = found ? pfix(key_value((cut & 0x80000000u) ? cut : (cut | kLowMask))) : 0;
  int keep_ties = 0;
  if (found) {
    if (pc > 0 && top_p > above) {
      const unsigned long long n = (top_p - above) / pc;
      keep_ties = n >= (unsigned long long)V ? V : (int)n;
    }
    if (above == 0 && keep_ties == 0) keep_ties = 1;  // the most likely token always stays
  }
  auto kept_mass = [&](unsigned long long nontie, int ties) {
    return nontie + (unsigned long long)min(ties, keep_ties) * pc;
  };
  // a token's share: its mass if above the cut (or no cut), flags a tie at it
  auto classify = [&](float x, unsigned long long &p, bool &tie) {
    const uint32_t k = rkey(x);
    p = 0;
    tie = false;
    if (x == -INFINITY) return;
    if (!found || k > cut) p = pfix(x);
    else if (k == cut) tie = true;
  };

  // ---- 3. inverse CDF over the kept tokens in index order. Warp w owns the
  // contiguous range [w * span, (w + 1) * span) (span a whole number of
  // vectors per lane); the warp totals are scanned in warp order, and in the
  // warp whose range holds the target each lane sums a contiguous 1/32 of the
  // range, a lane scan finds the lane that holds it, and that lane walks.
  const int sub = ((V + kSampleThreads - 1) / kSampleThreads + kVec - 1) / kVec * kVec;  // per lane
  const int span = 32 * sub;
  const int wlo = min(V, warp * span), whi = min(V, wlo + span);
  unsigned long long lmass = 0;
  int lties = 0;
  for (int b0 = wlo + lane * kVec; b0 < whi; b0 += 32 * kVec) {
    float x[kVec];
    const int n = min(fetch(b0, x), whi - b0);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      unsigned long long p;
      bool tie;
      classify(x[j], p, tie);
      if (j < n) {
        lmass += p;
        lties += tie ? 1 : 0;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lmass += __shfl_xor_sync(0xffffffffu, lmass, o);
    lties += __shfl_xor_sync(0xffffffffu, lties, o);
  }
  if (lane == 0) {
    wmass[warp] = lmass;
    wties[warp] = lties;
  }
  if (tid == 0) s_pick = -1;
  __syncthreads();
  // warp scan of the warp totals: non-tie mass and ties before warp w
  unsigned long long mi = lane < kSampleWarps ? wmass[lane] : 0;
  int ti = lane < kSampleWarps ? wties[lane] : 0;
  const unsigned long long mv = mi;
  const int tv = ti;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long a2 = __shfl_up_sync(0xffffffffu, mi, o);
    const int b2 = __shfl_up_sync(0xffffffffu, ti, o);
    if (lane >= o) {
      mi += a2;
      ti += b2;
    }
  }
  const unsigned long long wm_before = __shfl_sync(0xffffffffu, mi - mv, warp);
  const int wt_before = __shfl_sync(0xffffffffu, ti - tv, warp);
  const unsigned long long wm_incl = __shfl_sync(0xffffffffu, mi, warp);
  const int wt_incl = __shfl_sync(0xffffffffu, ti, warp);
  const unsigned long long total = kept_mass(__shfl_sync(0xffffffffu, mi, 31), __shfl_sync(0xffffffffu, ti, 31));
  const unsigned long long target =
      (unsigned long long)((double)a.uniforms[blockIdx.x] * (double)total);  // < total
  const unsigned long long kb = kept_mass(wm_before, wt_before), ki = kept_mass(wm_incl, wt_incl);
  if (ki > kb && kb <= target && target < ki) {
    const int llo = min(whi, wlo + lane * sub), lhi = min(whi, llo + sub);
    unsigned long long lm = 0;
    int lt = 0;
    for (int b0 = llo; b0 < lhi; b0 += kVec) {
      float x[kVec];
      const int n = min(fetch(b0, x), lhi - b0);
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        unsigned long long p;
        bool tie;
        classify(x[j], p, tie);
        if (j < n) {
          lm += p;
          lt += tie ? 1 : 0;
        }
      }
    }
    unsigned long long sm = lm;
    int st = lt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long a2 = __shfl_up_sync(0xffffffffu, sm, o);
      const int b2 = __shfl_up_sync(0xffffffffu, st, o);
      if (lane >= o) {
        sm += a2;
        st += b2;
      }
    }
    const unsigned long long nb = wm_before + sm - lm;
    const int tb = wt_before + st - lt;
    const unsigned long long lkb = kept_mass(nb, tb), lki = kept_mass(nb + lm, tb + lt);
    if (lki > lkb && lkb <= target && target < lki) {
      unsigned long long run = lkb;
      int ties = tb, pick = -1, last = -1;
      for (int b0 = llo; b0 < lhi && pick < 0; b0 += kVec) {
        float x[kVec];
        const int n = min(fetch(b0, x), lhi - b0);
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          unsigned long long p;
          bool tie;
          classify(x[j], p, tie);
          if (j >= n || pick >= 0) continue;
          if (tie) {
            if (ties < keep_ties) p = pc;
            ++ties;
          }
          if (p > 0) {
            last = b0 + j;
            run += p;
            if (target < run) pick = b0 + j;
          }
        }
      }
      s_pick = pick >= 0 ? pick : last;  // exactly one lane of the CTA gets here
    }
  }
  __syncthreads();
  if (tid == 0) a.out[blockIdx.x] = s_pick >= 0 ? s_pick : 0;
}

template <typename L, int KEY_BITS>
__global__ void __launch_bounds__(kSampleThreads, 1) top_p_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t sample_smem[];
  radix_top_p<L, KEY_BITS>(a, sample_smem);
}

// ---------------------------------------------------------------------------
// 16-bit logits: counts per bit pattern
// ---------------------------------------------------------------------------
constexpr int kWindow = 49152;  // patterns counted per row: 192 KB of counts
static_assert(kWindow * 4 <= kHistBytes + kTableBytes, "both paths share one dynamic smem size");
static_assert(kWindow % (4 * kSampleThreads) == 0 && kWindow <= 64 * kSampleThreads, "window layout");

// order key of a 16-bit float pattern (larger value, larger key) and back
__device__ __forceinline__ uint32_t key16(uint32_t u) {
  return (u & 0x8000u) ? (~u & 0xffffu) : (u | 0x8000u);
}
__device__ __forceinline__ uint32_t raw16(uint32_t k) {
  return (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu);
}
template <typename L> struct Bits16;
template <> struct Bits16<__nv_bfloat16> {
  static constexpr uint32_t kPosInf = 0x7f80u, kNegInf = 0xff80u;
  static __device__ __forceinline__ float to_float(uint32_t b) {
    return __bfloat162float(__ushort_as_bfloat16((uint16_t)b));
  }
};
template <> struct Bits16<__half> {
  static constexpr uint32_t kPosInf = 0x7c00u, kNegInf = 0xfc00u;
  static __device__ __forceinline__ float to_float(uint32_t b) { return __half2float(__ushort_as_half((uint16_t)b)); }
};

template <typename L, int KEY_BITS>
__global__ void __launch_bounds__(kSampleThreads, 1) top_p16_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t sample_smem[];
  uint32_t *cnt = reinterpret_cast<uint32_t *>(sample_smem);  // [kWindow] token count per pattern
  float *etab = reinterpret_cast<float *>(sample_smem);       // later: exp(scaled - max) per kept pattern
  __shared__ unsigned long long tex[kSampleThreads];  // exclusive prefix of each thread's window mass
  __shared__ unsigned long long wsum[kSampleWarps];
  __shared__ uint32_t redk[kSampleWarps];
  __shared__ unsigned long long wmass[kSampleWarps];
  __shared__ int wties[kSampleWarps];
  __shared__ int s_owner, s_glo, s_ghi, s_pick;
  __shared__ unsigned long long s_above, s_pc;

  const uint32_t FULL = 0xffffffffu;
  const uint16_t *row = reinterpret_cast<const uint16_t *>(a.logits) + (int64_t)blockIdx.x * a.row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.vocab;
  const float t = a.temperature;
  constexpr int kVec = 8;  // tokens per 16-byte vector
  constexpr int kStep = kSampleThreads * kVec;
  constexpr uint32_t kNoKey = 0x10000u;  // past the end of the row: above every pattern's key
  const bool vec_ok = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  auto fetch = [&](int base, uint32_t(&k)[kVec]) -> int {
    const int n = max(0, min(kVec, V - base));
    if (vec_ok && n == kVec) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(row + base);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        k[2 * j] = key16(w[j] & 0xffffu);
        k[2 * j + 1] = key16(w[j] >> 16);
      }
    } else {
#pragma unroll
      for (int j = 0; j < kVec; ++j) k[j] = j < n ? key16(row[base + j]) : kNoKey;
    }
    return n;
  };

  // ---- 1. the row's largest pattern
  uint32_t km = 0;
  for (int b0 = tid * kVec; b0 < V; b0 += 2 * kStep) {
    uint32_t k0[kVec], k1[kVec];
    fetch(b0, k0);
    fetch(b0 + kStep, k1);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      if (k0[j] != kNoKey) km = max(km, k0[j]);
      if (k1[j] != kNoKey) km = max(km, k1[j]);
    }
  }
  km = __reduce_max_sync(FULL, km);
  if (lane == 0) redk[warp] = km;
  __syncthreads();
  const uint32_t kmax = __reduce_max_sync(FULL, lane < kSampleWarps ? redk[lane] : 0u);

  // scaled value of the pattern with key k, and its mass relative to the max
  auto sbits = [&](uint32_t k) -> uint32_t { return Scaled<L>::scale_bits((uint16_t)raw16(k), t); };
  const float smax = Bits16<L>::to_float(sbits(kmax));
  auto emass = [&](uint32_t k) { return expf(Bits16<L>::to_float(sbits(k)) - smax); };
  auto pfix = [](float e) -> unsigned long long { return __float2ull_rn(e * 1099511627776.0f); };  // * 2^40

  // the window: the kWindow patterns up to the max; everything below must be
  // massless, and the max finite (no +inf or NaN, not all -inf)
  const int nb = (int)min((uint32_t)kWindow, kmax + 1);
  const int klo = (int)kmax - nb + 1;
  const bool window_ok = !(a.flags & PKV_SAMPLE_FORCE_RADIX) && kmax < key16(Bits16<L>::kPosInf) &&
                         kmax > key16(Bits16<L>::kNegInf) && (klo == 0 || pfix(emass(klo - 1)) == 0);
  if (!window_ok) {  // uniform across the CTA
    radix_top_p<L, KEY_BITS>(a, sample_smem);
    return;
  }

  // ---- 2. token counts per pattern (runs of equal neighbours added at once)
  for (int i = tid * 4; i < nb; i += kSampleThreads * 4) *reinterpret_cast<uint4 *>(cnt + i) = make_uint4(0, 0, 0, 0);
  __syncthreads();
  auto add_run = [&](uint32_t k, uint32_t n) {
    if (k >= (uint32_t)klo && k <= kmax) atomicAdd(&cnt[k - klo], n);
  };
  for (int b0 = tid * kVec; b0 < V; b0 += 2 * kStep) {
    uint32_t ks[2][kVec];
    fetch(b0, ks[0]);
    fetch(b0 + kStep, ks[1]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t prev = ks[h][0], run = 1;
#pragma unroll
      for (int j = 1; j < kVec; ++j) {
        if (ks[h][j] == prev) {
          ++run;
        } else {
          add_run(prev, run);
          prev = ks[h][j];
          run = 1;
        }
      }
      add_run(prev, run);
    }
  }
  __syncthreads();

  // ---- 3. the cut. Position j = 0, 1, ... is pattern kmax - j (descending);
  // thread i owns positions [i * cs, (i + 1) * cs).
  const int cs = (nb + kSampleThreads - 1) / kSampleThreads;  // <= 48
  auto pos_mass = [&](int j) -> unsigned long long {
    const uint32_t c = cnt[nb - 1 - j];
    return c ? (unsigned long long)c * pfix(emass(kmax - j)) : 0ull;
  };
  const int j0 = min(nb, tid * cs), j1 = min(nb, j0 + cs);
  unsigned long long S = 0;
  for (int j = j0; j < j1; ++j) S += pos_mass(j);
  unsigned long long inc = S;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long v = __shfl_up_sync(FULL, w, o);
      if (lane >= o) w += v;
    }
    wsum[lane] = w;
  }
  if (tid == 0) s_owner = -1;
  __syncthreads();
  const unsigned long long texcl = (warp ? wsum[warp - 1] : 0ull) + inc - S;
  tex[tid] = texcl;
  const unsigned long long total = wsum[kSampleWarps - 1];
  const unsigned long long top_p = (unsigned long long)fmin((double)a.top_p * (double)total, 4.0 * (double)total);
  const bool found = total > top_p;
  if (found && texcl <= top_p && top_p < texcl + S) s_owner = tid;
  __syncthreads();
  if (found && warp == (s_owner >> 5)) {
    // the owner's positions, two per lane, in order: the first whose running mass exceeds top_p
    const int ow = s_owner, oj0 = min(nb, ow * cs), oj1 = min(nb, oj0 + cs);
    const int pa = oj0 + lane, pb = oj0 + 32 + lane;
    const unsigned long long ma = pa < oj1 ? pos_mass(pa) : 0ull, mb = pb < oj1 ? pos_mass(pb) : 0ull;
    unsigned long long ia = ma, ib = mb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long va = __shfl_up_sync(FULL, ia, o), vb = __shfl_up_sync(FULL, ib, o);
      if (lane >= o) {
        ia += va;
        ib += vb;
      }
    }
    const unsigned long long base = tex[ow], ta = __shfl_sync(FULL, ia, 31);
    const unsigned ba = __ballot_sync(FULL, pa < oj1 && base + ia > top_p);
    const unsigned bb = __ballot_sync(FULL, pb < oj1 && base + ta + ib > top_p);
    const int jstar = ba ? oj0 + __ffs(ba) - 1 : oj0 + 32 + __ffs(bb) - 1;  // exists: the owner's range crosses top_p
    const uint32_t kstar = kmax - (uint32_t)jstar;
    const uint32_t sstar = key16(sbits(kstar));
    // the patterns tied with it (same scaled value) form a range [glo, ghi]
    int lo = (int)kstar, hi = (int)kmax;
    while (lo < hi) {
      const int step = (hi - lo + 31) / 32;
      const int c = lo + (lane + 1) * step;
      const int n = __popc(__ballot_sync(FULL, c <= hi && key16(sbits((uint32_t)c)) == sstar));
      lo += n * step;
      hi = min(hi, lo + step - 1);
    }
    const int ghi = lo;
    lo = klo;
    hi = (int)kstar;
    while (lo < hi) {
      const int step = (hi - lo + 31) / 32;
      const int c = hi - (lane + 1) * step;
      const int n = __popc(__ballot_sync(FULL, c >= lo && key16(sbits((uint32_t)c)) == sstar));
      hi -= n * step;
      lo = max(lo, hi - step + 1);
    }
    const int glo = hi;
    // mass above the tie group: positions before jhi = kmax - ghi
    const int jhi = (int)kmax - ghi, th = jhi / cs, hj0 = th * cs;
    unsigned long long part = (hj0 + lane < jhi ? pos_mass(hj0 + lane) : 0ull) +
                              (hj0 + 32 + lane < jhi ? pos_mass(hj0 + 32 + lane) : 0ull);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(FULL, part, o);
    if (lane == 0) {
      s_glo = glo;
      s_ghi = ghi;
      s_above = (th < kSampleThreads ? tex[th] : total) + part;
      s_pc = pfix(emass(kstar));
    }
  } else if (!found && tid == 0) {
    s_glo = klo - 1;
    s_ghi = klo - 1;
    s_above = 0;
    s_pc = 0;
  }
  __syncthreads();
  const int glo = s_glo, ghi = s_ghi;
  const unsigned long long above = s_above, pc = s_pc;
  int keep_ties = 0;
  if (found) {
    if (pc > 0 && top_p > above) {
      const unsigned long long n = (top_p - above) / pc;
      keep_ties = n >= (unsigned long long)V ? V : (int)n;
    }
    if (above == 0 && keep_ties == 0) keep_ties = 1;  // the most likely token always stays
  }
  // masses of the kept patterns, in place of their counts
  for (int j = j0; j < min(j1, (int)kmax - ghi); ++j) {
    const int b = nb - 1 - j;
    if (cnt[b]) etab[b] = emass(kmax - j);
  }
  __syncthreads();
  auto kept_mass = [&](unsigned long long nontie, int ties) {
    return nontie + (unsigned long long)min(ties, keep_ties) * pc;
  };
  auto classify = [&](uint32_t k, unsigned long long &p, bool &tie) {
    p = 0;
    tie = false;
    if (k > kmax) return;  // past the end of the row
    if ((int)k > ghi) p = pfix(etab[k - klo]);
    else if (found && (int)k >= glo) tie = true;
  };

  // ---- 4. inverse CDF over the kept tokens in index order: per-warp totals
  // over contiguous ranges, the warp holding the target splits its range into
  // lane slices, and the lane holding it walks its slice.
  const int sub = ((V + kSampleThreads - 1) / kSampleThreads + kVec - 1) / kVec * kVec;  // per lane
  const int span = 32 * sub;
  const int wlo = min(V, warp * span), whi = min(V, wlo + span);
  unsigned long long lmass = 0;
  int lties = 0;
  for (int b0 = wlo + lane * kVec; b0 < whi; b0 += 32 * kVec) {
    uint32_t k[kVec];
    const int n = min(fetch(b0, k), whi - b0);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      unsigned long long p;
      bool tie;
      classify(k[j], p, tie);
      if (j < n) {
        lmass += p;
        lties += tie ? 1 : 0;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lmass += __shfl_xor_sync(FULL, lmass, o);
    lties += __shfl_xor_sync(FULL, lties, o);
  }
  if (lane == 0) {
    wmass[warp] = lmass;
    wties[warp] = lties;
  }
  if (tid == 0) s_pick = -1;
  __syncthreads();
  unsigned long long mi = lane < kSampleWarps ? wmass[lane] : 0;
  int ti = lane < kSampleWarps ? wties[lane] : 0;
  const unsigned long long mv = mi;
  const int tv = ti;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long a2 = __shfl_up_sync(FULL, mi, o);
    const int b2 = __shfl_up_sync(FULL, ti, o);
    if (lane >= o) {
      mi += a2;
      ti += b2;
    }
  }
  const unsigned long long wm_before = __shfl_sync(FULL, mi - mv, warp);
  const int wt_before = __shfl_sync(FULL, ti - tv, warp);
  const unsigned long long wm_incl = __shfl_sync(FULL, mi, warp);
  const int wt_incl = __shfl_sync(FULL, ti, warp);
  const unsigned long long kept = kept_mass(__shfl_sync(FULL, mi, 31), __shfl_sync(FULL, ti, 31));
  const unsigned long long target = (unsigned long long)((double)a.uniforms[blockIdx.x] * (double)kept);
  const unsigned long long kb = kept_mass(wm_before, wt_before), ki = kept_mass(wm_incl, wt_incl);
  if (ki > kb && kb <= target && target < ki) {
    const int llo = min(whi, wlo + lane * sub), lhi = min(whi, llo + sub);
    unsigned long long lm = 0;
    int lt = 0;
    for (int b0 = llo; b0 < lhi; b0 += kVec) {
      uint32_t k[kVec];
      const int n = min(fetch(b0, k), lhi - b0);
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        unsigned long long p;
        bool tie;
        classify(k[j], p, tie);
        if (j < n) {
          lm += p;
          lt += tie ? 1 : 0;
        }
      }
    }
    unsigned long long sm = lm;
    int st = lt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long a2 = __shfl_up_sync(FULL, sm, o);
      const int b2 = __shfl_up_sync(FULL, st, o);
      if (lane >= o) {
        sm += a2;
        st += b2;
      }
    }
    const unsigned long long nb0 = wm_before + sm - lm;
    const int tb = wt_before + st - lt;
    const unsigned long long lkb = kept_mass(nb0, tb), lki = kept_mass(nb0 + lm, tb + lt);
    if (lki > lkb && lkb <= target && target < lki) {
      unsigned long long run = lkb;
      int ties = tb, pick = -1, last = -1;
      for (int b0 = llo; b0 < lhi && pick < 0; b0 += kVec) {
        uint32_t k[kVec];
        const int n = min(fetch(b0, k), lhi - b0);
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          unsigned long long p;
          bool tie;
          classify(k[j], p, tie);
          if (j >= n || pick >= 0) continue;
          if (tie) {
            if (ties < keep_ties) p = pc;
            ++ties;
          }
          if (p > 0) {
            last = b0 + j;
            run += p;
            if (target < run) pick = b0 + j;
          }
        }
      }
      s_pick = pick >= 0 ? pick : last;  // exactly one lane of the CTA gets here
    }
  }
  __syncthreads();
  if (tid == 0) a.out[blockIdx.x] = s_pick >= 0 ? s_pick : 0;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_sample_top_p(const void *logits, int32_t dtype, int32_t batch, int32_t vocab,
                                int64_t row_stride, float temperature, float top_p,
                                const float *uniforms, int64_t *out_tokens, int32_t flags,
                                void *stream) {
  if (batch < 0 || vocab <= 0 || row_stride < vocab) {
    set_error_detail("pkv_sample_top_p: invalid sizes (batch %d, vocab %d, row stride %lld)", batch,
                     vocab, (long long)row_stride);
    return PKV_ERR_INVALID_ARG;
  }
  if (!(temperature > 0.f) || !(top_p > 0.f)) {
    set_error_detail("pkv_sample_top_p: temperature and top_p must be > 0 (got %g, %g)",
                     (double)temperature, (double)top_p);
    return PKV_ERR_INVALID_ARG;
  }
  if (batch == 0) return PKV_OK;
  if (!logits || !uniforms || !out_tokens) {
    set_error_detail("pkv_sample_top_p: NULL pointer");
    return PKV_ERR_INVALID_ARG;
  }
  if (dtype_size(dtype) == 0) {
    set_error_detail("pkv_sample_top_p: unsupported dtype %d", dtype);
    return PKV_ERR_UNSUPPORTED;
  }
  if (!aligned_to(logits, dtype_size(dtype))) return PKV_ERR_ALIGNMENT;
  SampleArgs a{logits, row_stride, vocab, fmaxf(temperature, 1e-6f), top_p, uniforms, out_tokens, flags};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PKV_DTYPE_BF16:
      if (cudaFuncSetAttribute(top_p16_kernel<__nv_bfloat16, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kHistBytes + kTableBytes) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(top_p)");
      top_p16_kernel<__nv_bfloat16, 16><<<batch, kSampleThreads, kHistBytes + kTableBytes, st>>>(a);
      break;
    case PKV_DTYPE_F16:
      if (cudaFuncSetAttribute(top_p16_kernel<__half, 24>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kHistBytes + kTableBytes) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(top_p)");
      top_p16_kernel<__half, 24><<<batch, kSampleThreads, kHistBytes + kTableBytes, st>>>(a);
      break;
    default:
      if (cudaFuncSetAttribute(top_p_kernel<float, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kHistBytes) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(top_p)");
      top_p_kernel<float, 32><<<batch, kSampleThreads, kHistBytes, st>>>(a);
      break;
  }
  return check_launch("pkv_sample_top_p");
}
