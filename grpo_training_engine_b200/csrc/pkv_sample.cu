// pkv_sample.cu — temperature + top-p (nucleus) sampling of one token per row.
//
// The reference samples with a full sort of the vocabulary per row
// (src/triton_kernels/paged_kv.py:418-450, the same rule as
// fused_ops.py:236-248): scaled = logits / max(T, 1e-6) in the logits dtype,
// sort descending, softmax, running sum, drop every sorted token whose running
// sum exceeds top_p except the first, renormalise, then a multinomial draw
// over the sorted probabilities. At a 151,936-token vocabulary that sort is
// most of a rollout step's sampling time.
//
// Here one CTA handles one row without sorting. A token's mass is the fp32
// exp of its scaled logit minus the row max, as 40-bit fixed point, so sums
// are exact and independent of the order of summation (a probability is a
// mass over the row total; below 2^-40 counts as 0). Tokens are ordered as
// the reference's stable sort orders them: by scaled value descending, equal
// values (a "group") by index. The cut is the group of the first token whose
// running mass exceeds top_p x total: groups above it are kept, and of the
// cut group the tokens that fit under top_p, in index order, and always the
// most likely token. The draw scales the caller's uniform u in [0, 1) by the
// kept mass and inverts it in the same order: the group where the running
// mass passes the target, then the r-th token of that group in index order,
// r = (target - mass above the group) / the group's per-token mass. The
// reference rounds probabilities and their running sum to the logits dtype,
// so a token whose running probability lies within that rounding of top_p can
// fall on the other side of the cut.
//
// 16-bit logits (top_p16_kernel): a scaled logit and its mass depend only on
// the token's 16-bit pattern, and the scaling is monotone in it, so a group is
// a range of patterns. The CTA
//   1. finds the largest pattern (in value order) of the row;
//   2. counts the row's tokens per pattern in a window of the 49,152 patterns
//      below it (every pattern under the window has zero mass; otherwise the
//      radix path below runs);
//   3. scans count x mass over the window, and one warp finds the cut, the
//      kept mass, the target's group and r from the counts alone;
//   4. finds the r-th token of that group's pattern range in index order:
//      per-warp, per-sub-range and per-lane counts of matching keys.
// Three passes over the row; the only per-token shared-memory work is the
// count increment.
//
// fp32 logits (top_p32_kernel) sum exact masses per bin of the distance
// below the row max and sort only the tokens of the bin where the cut, and
// then the draw, falls (described above the kernel).
//
// Rows neither count path serves (fp16 at high temperature; a +inf or NaN
// logit; all -inf; fp32 rows whose cut bin holds more tokens than the sort
// buffer), and PKV_SAMPLE_FORCE_RADIX, take the radix path: the max, then the cut
// by a radix select over 8-bit digits of the order key of the scaled logit
// (two passes for bf16, three for fp16, four for fp32), each pass a 256-bin
// histogram of mass (one per warp, lanes with equal digits summed with warp
// match / reduce), a count of the cut group, the same radix select at the
// target, and the same r-th token search.
#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kBins = 256;
constexpr int kTableBytes = 65536 * 2;
constexpr int kHistBytes = kSampleWarps * kBins * 8;  // per-warp fixed-point mass histograms
constexpr uint32_t FULL = 0xffffffffu;

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Scaled logit as the reference computes it: logits / T rounded to the logits
// dtype. For 16-bit logits it depends only on the 16-bit pattern.
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

// low n bits (n >= 0) of a per-vector match mask
__device__ __forceinline__ uint32_t low_bits(int n) { return n >= 32 ? FULL : (1u << max(n, 0)) - 1u; }

// The index of the r-th (0-based) token of the row, in index order, among the
// tokens that match, or -1; every thread of the CTA calls it and gets the
// answer. load(b) gives the 16-byte vector of tokens [b, b + KV) (b a multiple
// of KV; anything past the row), match(v, b) a bit per token of it. Three
// levels of counts: contiguous warp ranges of the row, the 32 sub-ranges of
// the chosen warp's range, the 32 lane slices of the chosen sub-range; the
// chosen lane walks its slice. count_full(v, b) gives the number of matching
// tokens of a vector wholly inside the range being counted (popc of match by
// default; the 16-bit path counts with per-halfword min / max).
template <int KV, typename Load, typename Match, typename CountFull>
__device__ __forceinline__ int find_rth(int V, int r, Load load, Match match, CountFull count_full, int *s_cnt,
                                        int *s_res) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kInFlight = 4;
  const int sub = ((V + kSampleThreads - 1) / kSampleThreads + KV - 1) / KV * KV;  // per lane
  const int span = 32 * sub;
  // matches in [lo, hi), lanes strided by vectors, summed over the warp
  auto count_range = [&](int lo, int hi) -> int {
    int c = 0;
    for (int b0 = lo + lane * KV; b0 < hi; b0 += kInFlight * 32 * KV) {
      uint4 v[kInFlight];
#pragma unroll
      for (int h = 0; h < kInFlight; ++h) {
        const int b = b0 + h * 32 * KV;
        v[h] = b < hi ? load(b) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int h = 0; h < kInFlight; ++h) {
        const int b = b0 + h * 32 * KV;
        if (b + KV <= hi) {
          c += count_full(v[h], b);
        } else if (b < hi) {
          c += __popc(match(v[h], b) & low_bits(hi - b));
        }
      }
    }
    return __reduce_add_sync(FULL, c);
  };
  // the lane whose inclusive count passes rr (counts one per lane), and the count before it
  auto pick = [&](int c, int rr, int &before) -> int {
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(FULL, inc, o);
      if (lane >= o) inc += u;
    }
    const int l = __ffs(__ballot_sync(FULL, rr < inc && rr >= inc - c)) - 1;
    before = l >= 0 ? __shfl_sync(FULL, inc - c, l) : 0;
    return l;
  };
  if (tid == 0) *s_res = -1;
  const int wlo = min(V, warp * span), whi = min(V, wlo + span);
  const int c1 = count_range(wlo, whi);
  if (lane == 0) s_cnt[warp] = c1;
  __syncthreads();
  int b1 = 0;
  const int W = pick(s_cnt[lane], r, b1);
  if (W >= 0) {  // uniform across the CTA
    const int r2 = r - b1;
    const int Wlo = min(V, W * span), Whi = min(V, Wlo + span);
    const int lo2 = min(Whi, Wlo + warp * sub), hi2 = min(Whi, lo2 + sub);
    const int c2 = count_range(lo2, hi2);
    __syncthreads();  // every warp has read the level-1 counts
    if (lane == 0) s_cnt[warp] = c2;
    __syncthreads();
    int b2 = 0;
    const int W2 = pick(s_cnt[lane], r2, b2);
    if (W2 >= 0 && warp == W2) {
      const int r3 = r2 - b2;
      const int sub3 = ((sub + 31) / 32 + KV - 1) / KV * KV;
      const int lo3 = min(Whi, Wlo + W2 * sub), hi3 = min(Whi, lo3 + sub);
      const int llo = min(hi3, lo3 + lane * sub3), lhi = min(hi3, llo + sub3);
      int c3 = 0;
      for (int b0 = llo; b0 < lhi; b0 += KV) c3 += __popc(match(load(b0), b0) & low_bits(lhi - b0));
      int b3 = 0;
      const int L3 = pick(c3, r3, b3);
      if (L3 >= 0 && lane == L3) {
        int rr = r3 - b3, res = -1;
        for (int b0 = llo; b0 < lhi && res < 0; b0 += KV) {
          uint32_t m = match(load(b0), b0) & low_bits(lhi - b0);
          const int n = __popc(m);
          if (rr < n) {
            for (; rr > 0; --rr) m &= m - 1;  // drop the rr lowest set bits
            res = b0 + __ffs(m) - 1;
          } else {
            rr -= n;
          }
        }
        *s_res = res;
      }
    }
  }
  __syncthreads();
  return *s_res;
}

// ---------------------------------------------------------------------------
// radix path
// ---------------------------------------------------------------------------
// One row (the CTA's), all threads of the CTA.
template <typename L, int KEY_BITS>
__device__ __forceinline__ void radix_top_p(const SampleArgs &a, uint8_t *sample_smem) {
  unsigned long long *whist = reinterpret_cast<unsigned long long *>(sample_smem);  // [warps][bins]
  uint16_t *scaled_tbl = reinterpret_cast<uint16_t *>(sample_smem + kHistBytes);    // 16-bit logits
  __shared__ float redm[kSampleWarps];
  __shared__ unsigned long long hmass[kBins];
  __shared__ unsigned long long s_tot, s_thr, s_above;
  __shared__ uint32_t s_prefix;
  __shared__ int s_found;
  __shared__ int s_cnt[kSampleWarps];
  __shared__ int s_res;
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
  // row is not 16-byte aligned), two vectors per thread per step.
  constexpr int kVec = 16 / (int)sizeof(L);
  constexpr int kStep = kSampleThreads * kVec;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  auto load = [&](int base) -> uint4 {
    if (vec_ok && base + kVec <= V) return __ldg(reinterpret_cast<const uint4 *>(row + base));
    uint4 v = make_uint4(0, 0, 0, 0);
    L *e = reinterpret_cast<L *>(&v);
#pragma unroll
    for (int j = 0; j < kVec; ++j)
      if (base + j < V) e[j] = row[base + j];
    return v;
  };
  // scaled values of tokens [base, base + kVec); n of them are < V
  auto fetch = [&](int base, float(&x)[kVec]) -> int {
    const int n = max(0, min(kVec, V - base));
    const uint4 raw = load(base);
    const L *e = reinterpret_cast<const L *>(&raw);
#pragma unroll
    for (int j = 0; j < kVec; ++j) x[j] = j < n ? Scaled<L>::get(e, j, t, scaled_tbl) : -INFINITY;
    return n;
  };

  // ---- row max; masses are e = exp(x - max) in 40-bit fixed point (e <= 1)
  float m = -INFINITY;
  for (int b0 = tid * kVec; b0 < V; b0 += 2 * kStep) {
    float x0[kVec], x1[kVec];
    fetch(b0, x0);
    fetch(b0 + kStep, x1);
#pragma unroll
    for (int j = 0; j < kVec; ++j) m = fmaxf(m, fmaxf(x0[j], x1[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, o));
  if (lane == 0) redm[warp] = m;
  __syncthreads();
  m = lane < kSampleWarps ? redm[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, o));
  const float row_max = m;
  auto pfix = [&](float x) -> unsigned long long {
    return __float2ull_rn(expf(x - row_max) * 1099511627776.0f);  // * 2^40
  };
  // Keys of 16-bit values converted to fp32 carry their information in the top
  // KEY_BITS bits; the rest are 0 for positive values and 1 for negative ones
  // (the order key complements those). They are cleared, so every token of one
  // scaled value (a group) has the same key.
  constexpr uint32_t kLowMask = KEY_BITS >= 32 ? 0u : (1u << (32 - KEY_BITS)) - 1u;
  auto rkey = [](float x) { return order_key(x) & ~kLowMask; };
  auto group_value = [](uint32_t k) { return key_value((k & 0x80000000u) ? k : (k | kLowMask)); };

  // ---- radix select, 8 bits per pass from the top: the key of the group
  // holding the first token, in descending order, whose running mass exceeds
  // thr (s_prefix; s_found = 0 when none does) and the mass above that group
  // (s_above). With first set, the threshold is top_p x the row's total,
  // taken from the first pass (s_tot).
  unsigned long long *myhist = whist + warp * kBins;
  constexpr int kPasses = KEY_BITS / 8;
  auto radix_select = [&](unsigned long long thr, bool first) {
    if (tid == 0) {
      s_prefix = 0;
      s_above = 0;
      s_found = 0;
      s_thr = thr;
    }
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
            const unsigned grp = __match_any_sync(FULL, digit);
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
        if (pass == 0 && first) {  // the row's total mass; the nucleus bound top_p x total
          unsigned long long tot = 0;
          for (int b = 0; b < kBins; ++b) tot += hmass[b];
          s_tot = tot;
          s_thr = (unsigned long long)fmin((double)a.top_p * (double)tot, 4.0 * (double)tot);
        }
        const unsigned long long th = s_thr;
        // first digit, from the top, at which the running mass exceeds th
        unsigned long long run = s_above;
        int d = kBins - 1;
        for (; d >= 0; --d) {
          if (hmass[d] == 0) continue;
          if (run + hmass[d] > th) break;
          run += hmass[d];
        }
        if (d < 0) {  // everything fits under th
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
  };
  auto match_key = [&](uint32_t key) {
    return [&, key](const uint4 &v, int b0) -> uint32_t {
      const L *e = reinterpret_cast<const L *>(&v);
      uint32_t msk = 0;
#pragma unroll
      for (int j = 0; j < kVec; ++j)
        if (b0 + j < V && rkey(Scaled<L>::get(e, j, t, scaled_tbl)) == key) msk |= 1u << j;
      return msk;
    };
  };

  // ---- the cut
  radix_select(0ull, true);
  const bool found = s_found != 0;
  const uint32_t cut = s_prefix;
  const unsigned long long top_p = s_thr, total = s_tot;
  const unsigned long long above = found ? s_above : total;
  const unsigned long long pc = found ? pfix(group_value(cut)) : 0;
  // tokens in the cut group, and how many of them stay: while the running mass
  // is <= top_p, and at least one token overall (the most likely one)
  int n_ties = 0;
  if (found) {
    const auto mt = match_key(cut);
    int c = 0;
    for (int b0 = tid * kVec; b0 < V; b0 += kStep) c += __popc(mt(load(b0), b0));
    c = __reduce_add_sync(FULL, c);
    __syncthreads();
    if (lane == 0) s_cnt[warp] = c;
    __syncthreads();
    n_ties = __reduce_add_sync(FULL, s_cnt[lane]);
  }
  int keep_ties = 0;
  if (found) {
    if (pc > 0 && top_p > above) {
      const unsigned long long n = (top_p - above) / pc;
      keep_ties = n >= (unsigned long long)V ? V : (int)n;
    }
    if (above == 0 && keep_ties == 0) keep_ties = 1;
  }
  const unsigned long long kept = above + (unsigned long long)min(n_ties, keep_ties) * pc;
  // ---- the draw
  int token = -1;
  if (kept > 0) {  // uniform
    const unsigned long long target = (unsigned long long)((double)a.uniforms[blockIdx.x] * (double)kept);
    uint32_t gkey;
    unsigned long long r;
    if (target < above) {
      radix_select(target, false);  // found: target < above <= total
      gkey = s_prefix;
      r = (target - s_above) / pfix(group_value(gkey));
    } else {
      gkey = cut;
      r = (target - above) / pc;
    }
    __syncthreads();
    const auto mk = match_key(gkey);
    token = find_rth<kVec>(V, (int)min(r, (unsigned long long)V), load, mk,
                           [&](const uint4 &v, int b) { return __popc(mk(v, b)); }, s_cnt, &s_res);
  }
  if (tid == 0) a.out[blockIdx.x] = token >= 0 ? token : 0;
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
static_assert(kWindow % (4 * kSampleThreads) == 0, "window layout");

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
  uint32_t *cnt = reinterpret_cast<uint32_t *>(sample_smem);  // [kWindow] token count per pattern key - klo
  // Positions (patterns in descending order from the max) in groups of 128,
  // one uint4 of counts per lane; group g is summed by warp g % 32, and warp
  // w's prefix range is groups [w * kWarpGroups, (w + 1) * kWarpGroups).
  constexpr int kGroup = 128;
  constexpr int kNumGroups = kWindow / kGroup;
  constexpr int kWarpGroups = kNumGroups / kSampleWarps;
  static_assert(kWarpGroups <= 32, "one group per lane in a warp's prefix range");
  __shared__ unsigned long long gsum[kNumGroups];  // window mass per group
  __shared__ unsigned long long wsum[kSampleWarps];
  __shared__ uint32_t redk[kSampleWarps];
  __shared__ int s_lo, s_hi, s_r;
  __shared__ int s_cnt[kSampleWarps];
  __shared__ int s_res;

  const uint16_t *row = reinterpret_cast<const uint16_t *>(a.logits) + (int64_t)blockIdx.x * a.row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.vocab;
  const float t = a.temperature;
  constexpr int kVec = 8;  // tokens per 16-byte vector
  constexpr int kStep = kSampleThreads * kVec;
  constexpr int kInFlight = 4;  // vectors per thread per step of a pass
  constexpr uint32_t kNoKey = 0x10000u;  // past the end of the row: above every pattern's key
  const bool vec_ok = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  // the row is read twice: start pulling all of it into L2 now
  if (vec_ok && warp == 0) {
    const uint32_t bytes = (uint32_t)V * 2u & ~15u;
    const uint32_t chunk = ((bytes + 31u) / 32u + 15u) & ~15u;
    const uint32_t off = (uint32_t)lane * chunk;
    if (off < bytes)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<const uint8_t *>(row) + off),
                   "r"(min(chunk, bytes - off))
                   : "memory");
  }
  // 16-byte vector of tokens [base, base + 8); 0 past the row
  auto load = [&](int base) -> uint4 {
    if (vec_ok && base + kVec <= V) return __ldg(reinterpret_cast<const uint4 *>(row + base));
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < kVec; ++j)
      if (base + j < V) w[j >> 1] |= (uint32_t)row[base + j] << (16 * (j & 1));
    return make_uint4(w[0], w[1], w[2], w[3]);
  };
  auto half_at = [](const uint4 &v, int j) -> uint32_t {
    const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
    return (j & 1) ? w >> 16 : w & 0xffffu;
  };
  // key of token j of a loaded vector; kNoKey past the end of the row
  auto key_at = [&](const uint4 &v, int base, int j) -> uint32_t {
    return base + j < V ? key16(half_at(v, j)) : kNoKey;
  };
  auto sbits = [&](uint32_t k) -> uint32_t { return Scaled<L>::scale_bits((uint16_t)raw16(k), t); };
  auto pfix = [](float e) -> unsigned long long { return __float2ull_rn(e * 1099511627776.0f); };  // * 2^40
  auto block_max = [&](uint32_t v) {
    v = __reduce_max_sync(FULL, v);
    __syncthreads();  // redk is free
    if (lane == 0) redk[warp] = v;
    __syncthreads();
    return __reduce_max_sync(FULL, redk[lane]);
  };
  for (int i = tid * 4; i < kWindow; i += kSampleThreads * 4) *reinterpret_cast<uint4 *>(cnt + i) = make_uint4(0, 0, 0, 0);

  // ---- 1. token counts per pattern key in a window [klo, khi] of kWindow keys,
  // with the row max found in the same pass. The window's top is the max of
  // the first step's tokens plus a margin; if the row max lies above it, or a
  // pattern under the window has mass, the row is counted again below.
  uint4 v0[kInFlight];
#pragma unroll
  for (int h = 0; h < kInFlight; ++h) v0[h] = load(tid * kVec + h * kStep);
  uint32_t km = 0;
#pragma unroll
  for (int h = 0; h < kInFlight; ++h)
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const uint32_t k = key_at(v0[h], tid * kVec + h * kStep, j);
      if (k != kNoKey) km = max(km, k);
    }
  const uint32_t kmax0 = block_max(km);  // also orders the zeroing before the counting
  constexpr uint32_t kMargin = 1024;     // 8 binades of bf16 above the first step's max
  int khi = (int)min(kmax0 + kMargin, 0xffffu);
  int klo = max(khi - kWindow + 1, 0);
  // count the tokens of one vector: a vector of one pattern (flat or padded
  // rows) takes one increment, any other one increment per token. A full
  // vector's keys are made two per 32-bit word (each 16-bit half h becomes
  // h ^ 0xffff when negative, h ^ 0x8000 otherwise), and their running max is
  // a per-halfword max; a token outside the window [klo, khi] (k - klo wraps
  // past the span) is not counted.
  uint32_t span = (uint32_t)(khi - klo);  // (reset when the window moves)
  uint32_t km2 = 0;  // per-halfword max of the full vectors' keys
  auto count_vec = [&](const uint4 &v, int base) {
    if (base + kVec <= V) {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t kw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) kw[q] = w[q] ^ ((((w[q] >> 15) & 0x10001u) * 0x7fffu) | 0x80008000u);
      km2 = __vimax3_u16x2(km2, __vimax3_u16x2(kw[0], kw[1], kw[2]), kw[3]);
      if (((kw[0] ^ kw[1]) | (kw[0] ^ kw[2]) | (kw[0] ^ kw[3]) | ((kw[0] ^ (kw[0] >> 16)) & 0xffffu)) == 0u) {
        const uint32_t i = (kw[0] & 0xffffu) - (uint32_t)klo;
        if (i <= span) atomicAdd(&cnt[i], (uint32_t)kVec);
        return;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t i0 = (kw[q] & 0xffffu) - (uint32_t)klo, i1 = (kw[q] >> 16) - (uint32_t)klo;
        if (i0 <= span) atomicAdd(&cnt[i0], 1u);
        if (i1 <= span) atomicAdd(&cnt[i1], 1u);
      }
      return;
    }
#pragma unroll
    for (int j = 0; j < kVec; ++j) {  // the row's last, partial vector
      const uint32_t k = key_at(v, base, j);
      if (k == kNoKey) continue;
      km = max(km, k);
      if (k - (uint32_t)klo <= span) atomicAdd(&cnt[k - klo], 1u);
    }
  };
  auto count_rest = [&](int from) {
    for (int b0 = from + tid * kVec; b0 < V; b0 += kInFlight * kStep) {
      uint4 v[kInFlight];
#pragma unroll
      for (int h = 0; h < kInFlight; ++h) v[h] = load(b0 + h * kStep);
#pragma unroll
      for (int h = 0; h < kInFlight; ++h) count_vec(v[h], b0 + h * kStep);
    }
  };
#pragma unroll
  for (int h = 0; h < kInFlight; ++h) count_vec(v0[h], tid * kVec + h * kStep);
  count_rest(kInFlight * kStep);
  const uint32_t kmax = block_max(max(km, max(km2 & 0xffffu, km2 >> 16)));

  // scaled value of the pattern with key k, and its mass relative to the max
  const float smax = Bits16<L>::to_float(sbits(kmax));
  auto emass = [&](uint32_t k) { return expf(Bits16<L>::to_float(sbits(k)) - smax); };
  // rows the window cannot serve: a +inf or NaN max, all -inf, forced radix
  if ((a.flags & PKV_SAMPLE_FORCE_RADIX) || kmax >= key16(Bits16<L>::kPosInf) || kmax <= key16(Bits16<L>::kNegInf)) {
    radix_top_p<L, KEY_BITS>(a, sample_smem);
    return;
  }
  if ((int)kmax > khi || (klo > 0 && pfix(emass((uint32_t)klo - 1)) != 0)) {  // uniform
    // the window from the row max: [kmax - kWindow + 1, kmax]
    khi = (int)kmax;
    klo = max(khi - kWindow + 1, 0);
    span = (uint32_t)(khi - klo);
    if (klo > 0 && pfix(emass((uint32_t)klo - 1)) != 0) {  // massful patterns beyond any window
      radix_top_p<L, KEY_BITS>(a, sample_smem);
      return;
    }
    for (int i = tid * 4; i < kWindow; i += kSampleThreads * 4) *reinterpret_cast<uint4 *>(cnt + i) = make_uint4(0, 0, 0, 0);
    __syncthreads();
    count_rest(0);
    __syncthreads();
  }

  // ---- 2. masses over the window. Position j = 0, 1, ... is pattern kmax - j
  // (bin jmax - j); positions past jmax count nothing.
  const int jmax = (int)kmax - klo;
  auto count_at = [&](int j) -> uint32_t { return j <= jmax ? cnt[jmax - j] : 0u; };
  auto warp_sum = [&](unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
  };
  // the counts of positions [j, j + 4) (bins jmax - 3 - j .. jmax - j), one 16-byte read when aligned
  auto counts4 = [&](int j, uint32_t(&c)[4]) {
    if (j + 3 <= jmax && ((jmax - 3 - j) & 3) == 0) {
      const uint4 q = *reinterpret_cast<const uint4 *>(cnt + jmax - 3 - j);
      c[0] = q.w;
      c[1] = q.z;
      c[2] = q.y;
      c[3] = q.x;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) c[e] = count_at(j + e);
    }
  };
  for (int g = warp; g < kNumGroups; g += kSampleWarps) {
    const int j = g * kGroup + 4 * lane;
    uint32_t c[4];
    counts4(j, c);
    const bool has = (c[0] | c[1] | c[2] | c[3]) != 0u;
    unsigned long long m = 0;
    if (__any_sync(FULL, has)) {
      if (has) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (c[e]) m += (unsigned long long)c[e] * pfix(emass(kmax - (j + e)));
      }
      m = warp_sum(m);
    }
    if (lane == 0) gsum[g] = m;
  }
  __syncthreads();
  {
    const unsigned long long v = warp_sum(lane < kWarpGroups ? gsum[warp * kWarpGroups + lane] : 0ull);
    if (lane == 0) wsum[warp] = v;
  }
  __syncthreads();

  // ---- 3. one warp: the cut, the kept mass, the target's group and r
  if (warp == 0) {
    unsigned long long wincl = wsum[lane];  // inclusive prefix of the warp totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long v = __shfl_up_sync(FULL, wincl, o);
      if (lane >= o) wincl += v;
    }
    const unsigned long long total = __shfl_sync(FULL, wincl, 31);
    auto wexcl_of = [&](int w) { return __shfl_sync(FULL, wincl, w) - wsum[w]; };  // warp-uniform w
    auto excl_scan = [&](unsigned long long v) {
      unsigned long long i = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long u = __shfl_up_sync(FULL, i, o);
        if (lane >= o) i += u;
      }
      return i - v;
    };
    // The first position whose running mass exceeds thr (thr < total), the
    // mass of the positions before it and its per-token mass.
    auto first_over = [&](unsigned long long thr, unsigned long long &before, unsigned long long &per) -> int {
      const int ow = __ffs(__ballot_sync(FULL, wincl > thr && wincl - wsum[lane] <= thr)) - 1;
      const unsigned long long base = wexcl_of(ow);
      const unsigned long long gv = lane < kWarpGroups ? gsum[ow * kWarpGroups + lane] : 0ull;
      const unsigned long long gex = excl_scan(gv);
      const int gl = __ffs(__ballot_sync(FULL, lane < kWarpGroups && base + gex + gv > thr)) - 1;
      const int jg = (ow * kWarpGroups + gl) * kGroup;
      const unsigned long long gbase = base + __shfl_sync(FULL, gex, gl);
      uint32_t c[4];
      counts4(jg + 4 * lane, c);
      unsigned long long pf[4], lm = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pf[e] = c[e] ? pfix(emass(kmax - (jg + 4 * lane + e))) : 0ull;
        lm += c[e] * pf[e];
      }
      const unsigned long long lex = excl_scan(lm);
      const int ll = __ffs(__ballot_sync(FULL, gbase + lex + lm > thr)) - 1;
      int j = 0;
      unsigned long long run = 0, p = 0;
      if (lane == ll) {
        run = gbase + lex;
        int e = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (e == q && run + c[q] * pf[q] <= thr) {
            run += c[q] * pf[q];
            ++e;
          }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q == e) p = pf[q];
        j = jg + 4 * lane + e;
      }
      before = __shfl_sync(FULL, run, ll);
      per = __shfl_sync(FULL, p, ll);
      return __shfl_sync(FULL, j, ll);
    };
    // the pattern range [glo, ghi] of the group (same scaled value) of
    // position j, and the mass above the group (before: the mass of the
    // positions before j)
    auto group_of = [&](int j, unsigned long long before, int &glo, int &ghi) -> unsigned long long {
      const uint32_t k = kmax - (uint32_t)j;
      const uint32_t sk = sbits(k);
      // neighbours first: a group is usually one pattern
      const int nbk = lane == 0 ? (int)k + 1 : (int)k - 1;
      const bool same = lane < 2 && nbk >= klo && nbk <= (int)kmax && sbits((uint32_t)nbk) == sk;
      const unsigned nbr = __ballot_sync(FULL, same);
      ghi = (int)k;
      glo = (int)k;
      if (nbr & 1u) {
        int lo = (int)k + 1, hi = (int)kmax;
        while (lo < hi) {
          const int step = (hi - lo + 31) / 32;
          const int c = lo + (lane + 1) * step;
          const int n = __popc(__ballot_sync(FULL, c <= hi && sbits((uint32_t)c) == sk));
          lo += n * step;
          hi = min(hi, lo + step - 1);
        }
        ghi = lo;
      }
      if (nbr & 2u) {
        int lo = klo, hi = (int)k - 1;
        while (lo < hi) {
          const int step = (hi - lo + 31) / 32;
          const int c = hi - (lane + 1) * step;
          const int n = __popc(__ballot_sync(FULL, c >= lo && sbits((uint32_t)c) == sk));
          hi -= n * step;
          lo = max(lo, hi - step + 1);
        }
        glo = hi;
      }
      if (ghi == (int)k) return before;
      // the mass of positions [kmax - ghi, j): patterns above k in the group
      unsigned long long part = 0;
      for (int q = (int)kmax - ghi + lane; q < j; q += 32) part += (unsigned long long)count_at(q) * pfix(emass(kmax - q));
      return before - warp_sum(part);
    };
    // tokens with a pattern in [lo, hi]
    auto tokens_in = [&](int lo, int hi) {
      unsigned c = 0;
      for (int k = lo + lane; k <= hi; k += 32) c += cnt[k - klo];
      return (int)__reduce_add_sync(FULL, c);
    };
    const unsigned long long top_p = (unsigned long long)fmin((double)a.top_p * (double)total, 4.0 * (double)total);
    const bool found = total > top_p;
    int glo = 0, ghi = -1, n_ties = 0, keep_ties = 0;
    unsigned long long above = total, pc = 0;
    if (found) {
      unsigned long long before;
      const int jc = first_over(top_p, before, pc);
      above = group_of(jc, before, glo, ghi);
      n_ties = tokens_in(glo, ghi);
      if (pc > 0 && top_p > above) {
        const unsigned long long n = (top_p - above) / pc;
        keep_ties = n >= (unsigned long long)V ? V : (int)n;
      }
      if (above == 0 && keep_ties == 0) keep_ties = 1;  // the most likely token always stays
    }
    const unsigned long long kept = above + (unsigned long long)min(n_ties, keep_ties) * pc;
    const unsigned long long target = (unsigned long long)((double)a.uniforms[blockIdx.x] * (double)kept);
    int lo = glo, hi = ghi;
    unsigned long long r = 0;
    if (target < above) {
      unsigned long long before, per;
      const int jt = first_over(target, before, per);
      r = (target - group_of(jt, before, lo, hi)) / per;
    } else if (pc > 0) {
      r = (target - above) / pc;
    }
    if (lane == 0) {
      s_lo = lo;
      s_hi = hi;
      s_r = (int)min(r, (unsigned long long)V);
    }
  }
  __syncthreads();

  // ---- 4. the r-th token, in index order, with a pattern key in [lo, hi]. A
  // group's patterns share a sign, so the key range is one range of raw
  // patterns (increasing with the key for positive values, decreasing for
  // negative ones).
  const uint32_t rk0 = raw16((uint32_t)s_lo), rk1 = raw16((uint32_t)s_hi);
  const uint32_t rlo = min(rk0, rk1), rspan = max(rk0, rk1) - rlo;
  const auto match = [&](const uint4 &v, int b0) -> uint32_t {
    uint32_t msk = 0;
#pragma unroll
    for (int j = 0; j < kVec; ++j)
      if (((half_at(v, j) - rlo) & 0xffffu) <= rspan) msk |= 1u << j;
    return msk;  // bits past the row are masked by the caller
  };
  // a full vector's matches: per halfword, min(max(h, rlo), rlo + rspan) == h
  // exactly for the matching patterns (rlo + rspan <= 0xffff); the other
  // halfwords leave a non-zero xor, clamped to 1 and summed
  const uint32_t rlo2 = rlo * 0x10001u, rhi2 = (rlo + rspan) * 0x10001u;
  const auto count_full = [&](const uint4 &v, int) -> int {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t miss = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t c = __vimin3_u16x2(__vimax3_u16x2(w[q], rlo2, rlo2), rhi2, rhi2);
      miss += __vimin3_u16x2(c ^ w[q], 0x10001u, 0x10001u);
    }
    return kVec - (int)((miss & 0xffffu) + (miss >> 16));
  };
  const int token = s_hi >= s_lo ? find_rth<kVec>(V, s_r, load, match, count_full, s_cnt, &s_res) : -1;
  if (tid == 0) a.out[blockIdx.x] = token >= 0 ? token : 0;
}

// ---------------------------------------------------------------------------
// fp32 logits: exact masses per value bin, the tokens of one or two bins sorted
// ---------------------------------------------------------------------------
// A token's mass depends on its distance d = max - x below the row max (x the
// scaled logit), and is 0 in 2^-40 fixed point once d > 28.4. The span
// [0, kSpan32) of d is cut into kBins32 equal bins; a bin index is
// floor(d x kBins32 / kSpan32), monotone in x, so tokens of one scaled value
// (a group) share a bin, and bins run from the max downwards. One pass sums
// the exact fixed-point masses per bin (64-bit shared atomics); a block scan
// of the bins finds the bin where the running mass passes a threshold (the
// cut, then the draw's target) exactly; one more pass collects that bin's
// tokens (order key, index) into shared memory, where they are sorted by value
// (descending) and index (ascending) and walked group by group with the
// masses, cut and draw rule of the other paths. Rows it cannot serve (a NaN
// or +inf, all -inf, a bin with more tokens than the buffer holds: flat or
// tie-heavy rows) take the radix path.
constexpr int kBins32 = 16384;     // 128 KB of 64-bit masses
constexpr float kSpan32 = 28.5f;   // e^-28.5 x 2^40 < 0.5: no mass beyond
constexpr int kCand = 8192;        // tokens of a bin held for sorting: 64 KB
static_assert(kBins32 * 8 + kCand * 8 <= kHistBytes + kTableBytes, "the fp32 path uses the same dynamic smem");

__global__ void __launch_bounds__(kSampleThreads, 1) top_p32_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t sample_smem[];
  unsigned long long *bmass = reinterpret_cast<unsigned long long *>(sample_smem);  // [kBins32]
  unsigned long long *cand = bmass + kBins32;                                       // [kCand]
  __shared__ unsigned long long red64[kSampleWarps];
  __shared__ unsigned long long s_u64;
  __shared__ uint32_t redk[kSampleWarps];
  __shared__ int s_hit, s_n;

  if (a.flags & PKV_SAMPLE_FORCE_RADIX) {
    radix_top_p<float, 32>(a, sample_smem);
    return;
  }
  const float *row = reinterpret_cast<const float *>(a.logits) + (int64_t)blockIdx.x * a.row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.vocab;
  const float t = a.temperature;
  constexpr int kVec = 4;
  constexpr int kStep = kSampleThreads * kVec;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  const uint32_t kPosInfKey = order_key(INFINITY), kNegInfKey = order_key(-INFINITY);
  auto pfix = [](float e) -> unsigned long long { return __float2ull_rn(e * 1099511627776.0f); };  // * 2^40

  // raw logits of tokens [base, base + 4); -inf past the row
  auto fetch_raw = [&](int base, float(&r)[kVec]) {
    if (vec_ok && base + kVec <= V) {
      const float4 v = __ldg(reinterpret_cast<const float4 *>(row + base));
      r[0] = v.x;
      r[1] = v.y;
      r[2] = v.z;
      r[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < kVec; ++j) r[j] = base + j < V ? row[base + j] : -INFINITY;
    }
  };
  // ---- 1. the row max; any NaN (a key below -inf's or above +inf's). The
  // scaling by 1 / T (T > 0) is monotone and correctly rounded, so the max
  // scaled value is the scaled max raw value: no division here.
  uint32_t km = 0;
  bool nan_seen = false;
  for (int b0 = tid * kVec; b0 < V; b0 += kStep) {
    float r[kVec];
    fetch_raw(b0, r);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      if (b0 + j >= V) continue;
      const uint32_t k = order_key(r[j]);
      km = max(km, k);
      nan_seen |= k < kNegInfKey;
    }
  }
  km = __reduce_max_sync(FULL, km);
  if (lane == 0) redk[warp] = km;
  for (int i = tid; i < kBins32; i += kSampleThreads) bmass[i] = 0ull;
  const bool any_nan = __syncthreads_or(nan_seen ? 1 : 0) != 0;
  const uint32_t kmax = __reduce_max_sync(FULL, redk[lane]);  // of the raw values
  if (any_nan || kmax >= kPosInfKey || kmax <= kNegInfKey) {
    radix_top_p<float, 32>(a, sample_smem);
    return;
  }
  const float smax = __fdiv_rn(key_value(kmax), t);
  const float inv_w = (float)kBins32 / kSpan32;
  // raw values that certainly lie below the span (scaled distance > 28.5 by a
  // margin): massless, no division needed
  const float raw_floor = (smax - kSpan32 - 1.f) * t - 1e-5f * fabsf((smax - kSpan32 - 1.f) * t);
  auto bin_of = [&](float x) -> int {  // kBins32: beyond the span (no mass)
    const float d = smax - x;
    return d < kSpan32 ? min((int)(d * inv_w), kBins32 - 1) : kBins32;
  };

  // ---- 2. exact masses per bin and of the row
  unsigned long long tot = 0;
  for (int b0 = tid * kVec; b0 < V; b0 += kStep) {
    float x[kVec];
    fetch_raw(b0, x);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      if (b0 + j >= V || x[j] < raw_floor) continue;
      x[j] = __fdiv_rn(x[j], t);
      const int b = bin_of(x[j]);
      if (b < kBins32) {
        const unsigned long long p = pfix(expf(x[j] - smax));
        if (p) atomicAdd(&bmass[b], p);
        tot += p;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(FULL, tot, o);
  if (lane == 0) red64[warp] = tot;
  __syncthreads();
  unsigned long long total = red64[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(FULL, total, o);
  __syncthreads();

  // exclusive block scan of one value per thread: (the thread's prefix, the
  // per-thread inclusive value is prefix + v)
  auto block_excl = [&](unsigned long long v) -> unsigned long long {
    unsigned long long inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long u = __shfl_up_sync(FULL, inc, o);
      if (lane >= o) inc += u;
    }
    if (lane == 31) red64[warp] = inc;
    __syncthreads();
    unsigned long long wpre = 0;
    for (int w = 0; w < warp; ++w) wpre += red64[w];
    __syncthreads();
    return wpre + inc - v;
  };

  // ---- the first bin whose running mass (inclusive) exceeds thr, and the
  // mass of the bins before it; -1 when none does
  constexpr int kBinsPerThread = kBins32 / kSampleThreads;
  auto first_bin_over = [&](unsigned long long thr, unsigned long long &before) -> int {
    unsigned long long local = 0;
#pragma unroll
    for (int q = 0; q < kBinsPerThread; ++q) local += bmass[tid * kBinsPerThread + q];
    const unsigned long long pre = block_excl(local);
    if (tid == 0) s_hit = INT32_MAX;
    __syncthreads();
    unsigned long long run = pre;
    for (int q = 0; q < kBinsPerThread; ++q) {
      const unsigned long long m = bmass[tid * kBinsPerThread + q];
      if (run + m > thr) {
        atomicMin(&s_hit, tid * kBinsPerThread + q);
        break;
      }
      run += m;
    }
    __syncthreads();
    const int b = s_hit;
    if (b != INT32_MAX && tid == b / kBinsPerThread) {
      unsigned long long r = pre;
      for (int q = 0; q < b % kBinsPerThread; ++q) r += bmass[tid * kBinsPerThread + q];
      s_u64 = r;
    }
    __syncthreads();
    before = s_u64;
    __syncthreads();
    return b == INT32_MAX ? -1 : b;
  };

  // ---- the tokens of bin b into cand, sorted by value (descending) then
  // index (ascending); their count, or -1 when they do not fit
  auto collect = [&](int bin) -> int {
    if (tid == 0) s_n = 0;
    // raw values of the bin, widened by a whole bin on either side and a
    // relative 1e-5 (the scaling rounds by half an ulp): only tokens in there
    // are divided and binned exactly
    const float xl = smax - (float)(bin + 2) / inv_w, xh = smax - (float)(bin - 1) / inv_w;
    const float rl = xl * t - 1e-5f * fabsf(xl * t) - 1e-30f, rh = xh * t + 1e-5f * fabsf(xh * t) + 1e-30f;
    __syncthreads();
    for (int b0 = tid * kVec; b0 < V; b0 += kStep) {
      float x[kVec];
      fetch_raw(b0, x);
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        if (b0 + j < V && x[j] >= rl && x[j] <= rh && bin_of(x[j] = __fdiv_rn(x[j], t)) == bin) {
          const int pos = atomicAdd(&s_n, 1);
          if (pos < kCand)
            cand[pos] = ((unsigned long long)order_key(x[j]) << 32) | (uint32_t)(0xffffffffu - (uint32_t)(b0 + j));
        }
      }
    }
    __syncthreads();
    const int n = s_n;
    if (n > kCand) return -1;
    int np = 2;
    while (np < n) np <<= 1;
    for (int i = n + tid; i < np; i += kSampleThreads) cand[i] = 0ull;
    __syncthreads();
    for (int k = 2; k <= np; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < np; i += kSampleThreads) {
          const int p = i ^ j;
          if (p > i) {
            const unsigned long long u = cand[i], w = cand[p];
            if ((i & k) == 0 ? u < w : u > w) {
              cand[i] = w;
              cand[p] = u;
            }
          }
        }
        __syncthreads();
      }
    }
    return n;
  };

  // ---- walk the n sorted tokens from `base` (the mass before them): the
  // first whose running mass (inclusive) exceeds thr, its group (equal values)
  // [gs, ge], the mass before the group and its per-token mass. False when
  // none does.
  constexpr int kPerThread = kCand / kSampleThreads;
  auto walk = [&](int n, unsigned long long base, unsigned long long thr, int &gs, int &ge,
                  unsigned long long &gbefore, unsigned long long &per) -> bool {
    unsigned long long m[kPerThread], local = 0;
#pragma unroll
    for (int q = 0; q < kPerThread; ++q) {
      const int i = tid * kPerThread + q;
      m[q] = i < n ? pfix(expf(key_value((uint32_t)(cand[i] >> 32)) - smax)) : 0ull;
      local += m[q];
    }
    const unsigned long long pre = base + block_excl(local);
    if (tid == 0) s_hit = INT32_MAX;
    __syncthreads();
    unsigned long long run = pre;
#pragma unroll
    for (int q = 0; q < kPerThread; ++q) {
      run += m[q];
      const int i = tid * kPerThread + q;
      if (i < n && run > thr) {
        atomicMin(&s_hit, i);
        break;
      }
    }
    __syncthreads();
    const int hit = s_hit;
    if (hit == INT32_MAX) return false;
    const uint32_t key = (uint32_t)(cand[hit] >> 32);
    int lo = 0, hi = hit;  // first index with this key (keys descending)
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((uint32_t)(cand[mid] >> 32) > key) lo = mid + 1; else hi = mid;
    }
    gs = lo;
    lo = hit;
    hi = n - 1;  // last index with this key
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((uint32_t)(cand[mid] >> 32) < key) hi = mid - 1; else lo = mid;
    }
    ge = lo;
    per = pfix(expf(key_value(key) - smax));
    if (tid == hit / kPerThread) {  // the running mass through the hit: every token of a group weighs the same
      unsigned long long r = pre;
      for (int q = 0; q <= hit % kPerThread; ++q) r += m[q];
      s_u64 = r;
    }
    __syncthreads();
    gbefore = s_u64 - (unsigned long long)(hit - gs + 1) * per;
    __syncthreads();
    return true;
  };
  auto token_of = [&](int i) { return (int)(0xffffffffu - (uint32_t)(cand[i] & 0xffffffffu)); };

  // ---- 3. the cut
  const unsigned long long top_p = (unsigned long long)fmin((double)a.top_p * (double)total, 4.0 * (double)total);
  const bool found = total > top_p;
  int cbin = -1, cgs = 0, cge = -1, n_ties = 0, keep_ties = 0, ncand = 0;
  unsigned long long above = total, pc = 0;
  if (found) {
    unsigned long long bbefore = 0;
    cbin = first_bin_over(top_p, bbefore);
    ncand = cbin >= 0 ? collect(cbin) : -1;
    if (ncand < 0 || !walk(ncand, bbefore, top_p, cgs, cge, above, pc)) {
      radix_top_p<float, 32>(a, sample_smem);
      return;
    }
    n_ties = cge - cgs + 1;
    if (pc > 0 && top_p > above) {
      const unsigned long long nk = (top_p - above) / pc;
      keep_ties = nk >= (unsigned long long)V ? V : (int)nk;
    }
    if (above == 0 && keep_ties == 0) keep_ties = 1;  // the most likely token always stays
  }
  const unsigned long long kept = above + (unsigned long long)min(n_ties, keep_ties) * pc;

  // ---- 4. the draw
  const unsigned long long target = (unsigned long long)((double)a.uniforms[blockIdx.x] * (double)kept);
  int token;
  if (found && target >= above) {  // in the cut group
    const unsigned long long r = pc > 0 ? (target - above) / pc : 0;
    token = token_of(cgs + (int)min(r, (unsigned long long)(n_ties - 1)));
  } else {
    unsigned long long bbefore = 0;
    const int tbin = first_bin_over(target, bbefore);
    int n = ncand;
    if (tbin != cbin) n = tbin >= 0 ? collect(tbin) : -1;
    int gs = 0, ge = -1;
    unsigned long long gb = 0, per = 0;
    if (n < 0 || !walk(n, bbefore, target, gs, ge, gb, per)) {
      radix_top_p<float, 32>(a, sample_smem);
      return;
    }
    const unsigned long long r = per > 0 ? (target - gb) / per : 0;
    token = token_of(gs + (int)min(r, (unsigned long long)(ge - gs)));
  }
  if (tid == 0) a.out[blockIdx.x] = token;
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
      if (cudaFuncSetAttribute(top_p32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kHistBytes + kTableBytes) != cudaSuccess)
        return check_launch("cudaFuncSetAttribute(top_p)");
      top_p32_kernel<<<batch, kSampleThreads, kHistBytes + kTableBytes, st>>>(a);
      break;
  }
  return check_launch("pkv_sample_top_p");
}
