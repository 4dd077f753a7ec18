// pkv_decode.cu — paged-KV single-query decode attention for sm_100a.
//
// Computes, for every sequence b and query head h,
//     out[b, h, :] = sum_{t < ctx_b} softmax_t(scale * q[b,h] . K[t]) V[t]
// over the pages listed in block_tables[b], with fp32 accumulation, fp32
// output and out = acc / max(sum, 1e-6) — the arithmetic of the reference's
// _paged_attention_decode_kernel (src/triton_kernels/paged_kv.py:63-251).
// The reference makes three passes over K (max, sum, weighted V,
// paged_kv.py:97-251) per query head; this file makes ONE pass with an online
// (running max) softmax and lets one CTA serve all G = Hq / Hkv query heads
// that share a KV head, so every K/V byte is read from HBM once.
//
// Work decomposition (shared by both kernels):
//   plan kernel   : per sequence, n_b = ceil(pages_b / P) chunks of P pages
//                   ("splits"); a flat list of item descriptors
//                   (b, split, length, n_b) is written into the caller's
//                   workspace together with per-sequence offsets.
//   decode kernel : persistent CTAs take work units (item, kv head, head
//                   group). A unit whose sequence has one split writes the
//                   final output; otherwise it writes a partial
//                   (max, sum, unnormalised acc).
//   merge kernel  : one CTA per (sequence, head group) combines the partials
//                   of multi-split sequences, in split order.
//
// Two decode kernels:
//   decode_tc_kernel      bf16/fp16 cache, block_size 16, head_dim 64/128.
//                         A producer warp schedules units and publishes, per
//                         consumer warp, the pages to read (plus staged
//                         query rows); each of 9 (head_dim 128; 7 when it
//                         also applies RoPE) or 8 (64) consumer warps
//                         streams its own K and V pages into a
//                         smem ring with 16-byte cp.async (one commit group per
//                         page, issued S - 1 pages ahead) and computes
//                         K.q^T and V^T.P^T with m16n8k16 tensor-core MMAs
//                         (tokens, resp. head_dim, on M; query heads on N).
//                         Optionally it also appends the step's new K/V row
//                         (and rotates q and that K row by RoPE first), and it
//                         is launched as a programmatic dependent launch.
//   decode_generic_kernel any dtype (fp32/bf16/fp16), any block size,
//                         head_dim <= 256: CUDA-core FMAs, plain coalesced
//                         loads, per-warp online softmax.
#include <algorithm>
#include <climits>
#include <cstddef>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kTcRows = 16;   // query heads per head group in the tensor-core kernel (MMA M)
constexpr int kGenThreads = 128;
constexpr int kGenWarps = kGenThreads / 32;
// Block-table entries of a unit held in the tensor-core producer's registers,
// lane-strided: kBtRegs per lane, so a split has at most kMaxPagesPerSplit pages.
constexpr int kBtRegs = 16;
constexpr int32_t kMaxPagesPerSplit = kBtRegs * 32;
// wait bound of every device wait under PKV_DECODE_TEST_WAIT_TIMEOUT
constexpr uint32_t kTestWaitPolls = 4096;
// Split-length cost model, in pages' worth of one CTA's streaming: the fixed
// cost of a unit (cross-warp combine and pipeline refill, measured on B200 at
// about 16 pages) and of merging split partials (the last split of a sequence
// counts in, reads the others' partials back from L2 and writes the output:
// ~2 us in a per-warp trace, about 16 pages), and the extra cost of every unit
// of a split sequence (its partial store, fence and count-in barrier: ~1.5 us
// more per unit than an unsplit one in the same trace, about 12 pages).
constexpr int64_t kUnitCost = 16, kMergeCost = 16, kSplitUnitCost = 12;
// Candidate split lengths the plan kernel weighs (multiples of 8 pages).
constexpr int kMaxSplitCandidates = 64;

// ---------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------
struct WsLayout {
  size_t hdr, seq_off, seq_nsplit, merge_cnt, items, partials, total;
  int64_t max_items;
  int32_t units_per_item;  // num_kv_heads * head_groups
  int32_t group_rows;      // query heads per head group (partial row count)
  int32_t part_o;          // offset of the accumulator rows in a partial unit (16-byte aligned)
  int32_t part_floats;     // floats per partial unit: [max GR][sum GR][pad][acc GR x D]
};

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline int32_t group_rows_for(int32_t G, int32_t D) {
  // Rows per head group: 16 (one MMA M tile) in general; the CUDA-core kernel
  // keeps G x D/32 accumulators per lane, so wide heads use groups of 8.
  int32_t cap = D > 128 ? 8 : kTcRows;
  return G < cap ? G : cap;
}

WsLayout ws_layout(int32_t B, int32_t Hq, int32_t Hkv, int32_t D, int32_t max_blocks, int32_t P) {
  WsLayout w{};
  const int32_t G = Hq / Hkv;
  w.group_rows = group_rows_for(G, D);
  const int32_t HG = (G + w.group_rows - 1) / w.group_rows;
  w.units_per_item = Hkv * HG;
  const int64_t per_seq = max_blocks > 0 ? (max_blocks + P - 1) / P : 1;
  w.max_items = (int64_t)B * per_seq;
  w.part_o = (int32_t)align_up(2 * (size_t)w.group_rows, 4);
  w.part_floats = w.part_o + w.group_rows * D;
  size_t off = 0;
  w.hdr = off; off += 256;
  w.seq_off = off; off = align_up(off + sizeof(int32_t) * (size_t)B, 256);
  w.seq_nsplit = off; off = align_up(off + sizeof(int32_t) * (size_t)B, 256);
  w.merge_cnt = off; off = align_up(off + sizeof(int32_t) * (size_t)B * w.units_per_item, 256);
  w.items = off; off = align_up(off + sizeof(int4) * (size_t)w.max_items, 256);
  w.partials = off;
  off = align_up(off + sizeof(float) * (size_t)w.max_items * w.units_per_item * w.part_floats, 256);
  w.total = off;
  return w;
}

// ---------------------------------------------------------------------------
// kernel arguments
// ---------------------------------------------------------------------------
struct DecodeArgs {
  const void *q;
  const int32_t *bt;
  const int32_t *ctx;
  float *out;
  const void *kc;
  const void *vc;
  // P: the longest split the plan may choose (shared-memory sizing); the
  // plan's choice is hdr[1], which the kernels read
  int32_t B, Hq, Hkv, G, GR, HG, D, bs, num_blocks, max_blocks, P, upi, part_o, part_floats;
  int32_t q_dtype, kv_dtype;
  int32_t q_vec;    // q rows are 16-byte aligned and contiguous in head_dim
  int32_t out_vec;  // out rows are aligned for 4-element stores and contiguous in head_dim
  int32_t out16;    // out element type: 0 fp32, 1 bf16, 2 fp16 (rounded to nearest)
  int64_t q0, q1, q2;
  int64_t c0, c1, c2, c3;
  int64_t bt0, bt1;
  int64_t o0, o1, o2;
  float scale, scale_log2;
  const int32_t *hdr;
  const int32_t *seq_off;
  const int32_t *seq_nsplit;
  const int4 *items;  // per item {b, split, clamped ctx, splits of b}
  int64_t max_items;  // entries the item array holds (the plan fills the first total / upi)
  float *partials;
  // splits of (sequence b, unit r) that finished, at b * upi + r: the last one
  // merges (tensor-core kernel); zeroed by the plan, reset by the merging unit
  int32_t *merge_cnt;
  int32_t *status;
  int32_t *sched;  // {next tail unit, CTAs done claiming}: the dynamic tail of the schedule
  // fused append (tensor-core kernel): the new token of sequence b, written at
  // position context_lens[b] - 1; kn == nullptr when there is none
  const void *kn;
  const void *vn;
  int64_t n0, n1;  // k_new / v_new strides [B, Hkv, D] (elements; D contiguous)
  // RoPE of q and k_new in the producer (nullptr: q and k_new are final):
  // cos / sin [B, D] in q's dtype, row stride rcs elements
  const void *rcos;
  const void *rsin;
  int64_t rcs;
  // bounds of the tensor-core kernel's device waits (polls of a consumer wait,
  // tries of a producer wait); withhold != 0 (PKV_DECODE_TEST_WAIT_TIMEOUT
  // only): CTA 0's producer never publishes consumer warp 0's first element
  uint32_t max_polls, max_tries;
  int32_t withhold;
  // PKV_DECODE_EARLY_START (tensor-core kernel): the plan, block tables,
  // context lengths and caches are not written by the previous kernel in the
  // stream, so the first unit's pages are scheduled and loaded before the
  // dependency wait
  int32_t early;
};

struct Unit {
  int32_t b, s, kvh, hg, nsplit, ctx, p_begin, p_end, gcount, qh0;
};

// One output element, in the output's type.
__device__ __forceinline__ void store_out(const DecodeArgs &a, int64_t idx, float v) {
  if (a.out16 == 1)
    reinterpret_cast<__nv_bfloat16 *>(a.out)[idx] = __float2bfloat16_rn(v);
  else if (a.out16 == 2)
    reinterpret_cast<__half *>(a.out)[idx] = __float2half_rn(v);
  else
    a.out[idx] = v;
}

// Four consecutive output elements starting at element idx (a multiple of 4
// on a row of 4-element-aligned stores).
__device__ __forceinline__ void store_out4(const DecodeArgs &a, int64_t idx, float4 r) {
  if (a.out16 == 1) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(r.x, r.y), hi = __floats2bfloat162_rn(r.z, r.w);
    *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(a.out) + idx) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
  } else if (a.out16 == 2) {
    const __half2 lo = __floats2half2_rn(r.x, r.y), hi = __floats2half2_rn(r.z, r.w);
    *reinterpret_cast<uint2 *>(reinterpret_cast<__half *>(a.out) + idx) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
  } else {
    *reinterpret_cast<float4 *>(a.out + idx) = r;
  }
}

// Work unit w = (item, kv head, head group); the item descriptor comes from the
// plan, P is the plan's split length.
__device__ __forceinline__ Unit unit_from(const DecodeArgs &a, int32_t P, int32_t w, int4 it) {
  Unit u;
  const int32_t item = w / a.upi;
  const int32_t r = w - item * a.upi;
  u.kvh = r / a.HG;
  u.hg = r - u.kvh * a.HG;
  u.b = it.x;
  u.s = it.y;
  u.ctx = it.z;
  u.nsplit = it.w;
  const int32_t npages = (u.ctx + a.bs - 1) / a.bs;
  u.p_begin = u.s * P;
  u.p_end = min(u.p_begin + P, npages);
  if (u.p_end < u.p_begin) u.p_end = u.p_begin;
  const int32_t g0 = u.hg * a.GR;
  u.gcount = min(a.GR, a.G - g0);
  u.qh0 = u.kvh * a.G + g0;
  return u;
}

__device__ __forceinline__ Unit decode_unit(const DecodeArgs &a, int32_t P, int32_t w) {
  return unit_from(a, P, w, a.items[w / a.upi]);
}

// ---------------------------------------------------------------------------
// plan: per-sequence split counts, prefix offsets, item descriptors
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;

// Block-wide exclusive scan of one value per thread (kPlanThreads threads);
// returns the thread's exclusive prefix, *total gets the block sum.
__device__ __forceinline__ int32_t block_exclusive_scan(int32_t v, int32_t *warp_tot, int32_t *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int32_t t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_tot[lane] = t;  // inclusive totals per warp
  }
  __syncthreads();
  const int32_t excl = (warp > 0 ? warp_tot[warp - 1] : 0) + x - v;
  *total = warp_tot[kPlanThreads / 32 - 1];
  __syncthreads();  // warp_tot is reused by the next scan
  return excl;
}

// Splits of sequence b: n in total, `full` of them P pages long; when n > full
// the last split is partial with `rest` pages (an empty sequence is one
// partial split of 0 pages).
struct SeqSplits {
  int32_t ctx, n, full, rest;
};

__device__ __forceinline__ SeqSplits seq_splits(const int32_t *ctx, int32_t b, int32_t bs,
                                                int32_t cap, int32_t P, int32_t *status,
                                                bool report) {
  SeqSplits r;
  int32_t c = ctx[b];
  if (c < 0 || c > cap) {
    if (report) flag_status(status, PKV_DEV_CTX_OUT_OF_RANGE);
    c = c < 0 ? 0 : cap;
  }
  const int32_t pages = (c + bs - 1) / bs;
  r.ctx = c;
  r.n = pages > 0 ? (pages + P - 1) / P : 1;
  r.rest = pages % P;
  r.full = pages / P;
  return r;
}

// Split length for these lengths: P in {p_lo, p_lo + 8, ..., p_hi}, the one
// whose launch the tensor-core kernel's schedule finishes first. Each of
// kSimWarps warps takes candidates in turn and simulates the schedule: items
// are the full P-page splits, then the partial last splits by decreasing
// length (the order this kernel writes), each expanded to upi units; CTA c of
// `slots` takes unit c in round 0, 2 slots - 1 - c in round 1, and so on (the
// snake). A CTA's time is its units' pages plus kUnitCost per unit (plus
// kSplitUnitCost for a unit of a split sequence); the launch takes the largest
// CTA time, plus kMergeCost when some sequence is split. The partial splits are
// ordered by a counting sort of their costs in 8-page bins (a unit's cost is
// taken as its bin's upper edge, within 8 pages), so a candidate costs
// O(B / 32 + rounds) per lane. Ties go to the longer split. B <= kMaxSimSeqs
// (the host enables this only for such batches). Whole block.
constexpr int kSimWarps = 16;
constexpr int kMaxSimSeqs = kPlanThreads;
constexpr int kSimBins = (kMaxPagesPerSplit + (int)kSplitUnitCost) / 8 + 2;

__device__ int32_t choose_split(const int32_t *__restrict__ ctx, int32_t B, int32_t bs, int32_t cap,
                                int32_t p_lo, int32_t p_hi, int32_t upi, int32_t slots) {
  static_assert(kSimBins <= 96 && kSimBins * 8 < 32768, "three bins per lane; int16 costs");
  __shared__ int32_t s_pages[kMaxSimSeqs];
  __shared__ int32_t s_hist[kSimWarps][kSimBins];        // partial splits per cost bin
  __shared__ int16_t s_sorted[kSimWarps][kMaxSimSeqs];  // partial split costs, highest first
  __shared__ long long s_cost[kMaxSplitCandidates];
  __shared__ int32_t s_maxp, s_choice;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int32_t ncand = min(kMaxSplitCandidates, (p_hi - p_lo) / 8 + 1);
  if (tid == 0) s_maxp = 0;
  __syncthreads();
  int32_t mp = 0;
  if (tid < B) {
    const int32_t c = min(max(ctx[tid], 0), cap);
    mp = (c + bs - 1) / bs;
    s_pages[tid] = mp;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mp = max(mp, __shfl_xor_sync(0xffffffffu, mp, o));
  if (lane == 0 && mp > 0) atomicMax(&s_maxp, mp);
  __syncthreads();
  const int32_t maxp = s_maxp;
  if (warp < kSimWarps) {
    int32_t *hist = s_hist[warp];
    int16_t *sorted = s_sorted[warp];
    for (int32_t k = warp; k < ncand; k += kSimWarps) {
      const int32_t P = p_lo + 8 * k;
      for (int i = lane; i < kSimBins; i += 32) hist[i] = 0;
      __syncwarp();
      int32_t full = 0, parts = 0;
      for (int32_t b = lane; b < B; b += 32) {
        const int32_t pg = s_pages[b];
        const int32_t f = pg / P, n = pg > 0 ? (pg + P - 1) / P : 1;
        full += f;
        if (n > f) {
          // the last split's cost: its pages, plus the split overhead when the
          // sequence has other splits
          const int32_t cost = pg - f * P + (f > 0 ? (int32_t)kSplitUnitCost : 0);
          atomicAdd(&hist[cost >> 3], 1);
          ++parts;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        full += __shfl_xor_sync(0xffffffffu, full, o);
        parts += __shfl_xor_sync(0xffffffffu, parts, o);
      }
      __syncwarp();
      {
        // counting sort: lane l owns bins 3l .. 3l + 2; the partials in higher
        // bins come first (a suffix scan over the lanes), then each lane writes
        // its bins' costs in place
        int32_t h[3], own = 0;
#pragma unroll
        for (int e = 0; e < 3; ++e) {
          const int i = 3 * lane + e;
          h[e] = i < kSimBins ? hist[i] : 0;
          own += h[e];
        }
        int32_t suf = own;  // inclusive sum over lanes >= this one
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int32_t y = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += y;
        }
        int32_t pos = suf - own;  // partials in the bins of higher lanes
#pragma unroll
        for (int e = 2; e >= 0; --e) {
          for (int32_t x = 0; x < h[e]; ++x) sorted[pos + x] = (int16_t)((3 * lane + e) * 8 + 7);
          pos += h[e];
        }
      }
      __syncwarp();
      // P >= lo keeps the full splits within 16 rounds of the CTAs, so the
      // units (full + one partial per sequence and unit) fit 32 bits
      const int32_t units = upi * (full + parts);
      const int32_t rounds = (units + slots - 1) / slots;
      long long worst = 0;
      for (int32_t c = lane; c < slots; c += 32) {
        long long load = 0;
        for (int32_t r = 0; r < rounds; ++r) {
          const int32_t w = r * slots + ((r & 1) ? slots - 1 - c : c);
          if (w >= units) continue;
          const int32_t item = w / upi;
          // full splits are (nearly always) of longer sequences
          const int32_t cost = item < full ? P + (int32_t)kSplitUnitCost : (int32_t)sorted[item - full];
          load += cost + kUnitCost;
        }
        worst = max(worst, load);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) worst = max(worst, __shfl_xor_sync(0xffffffffu, worst, o));
      if (lane == 0) s_cost[k] = worst + (maxp > P ? kMergeCost : 0);
      __syncwarp();  // hist / sorted are rewritten for the next candidate
    }
  }
  __syncthreads();
  if (warp == 0) {
    long long best = LLONG_MAX;
    int32_t bestP = p_hi;
    for (int32_t k = lane; k < ncand; k += 32) {
      const int32_t Pc = p_lo + 8 * k;
      if (s_cost[k] < best || (s_cost[k] == best && Pc > bestP)) {
        best = s_cost[k];
        bestP = Pc;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const long long ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int32_t op = __shfl_xor_sync(0xffffffffu, bestP, o);
      if (ob < best || (ob == best && op > bestP)) {
        best = ob;
        bestP = op;
      }
    }
    if (lane == 0) s_choice = bestP;
  }
  __syncthreads();
  return s_choice;
}

// Items are ordered for the tensor-core kernel's snake schedule: every full P-page split first
// (sequence order), then the partial last splits by decreasing length, so the
// units left for the end of a launch are the shortest. Partial-result slots do
// not depend on this order (they are indexed by seq_off[b] + split). P is p_hi,
// or, when p_lo < p_hi, chosen from the lengths (choose_split); hdr[1] records it.
__global__ void __launch_bounds__(kPlanThreads)
plan_kernel(const int32_t *__restrict__ ctx, int32_t B, int32_t bs, int32_t max_blocks, int32_t p_lo,
            int32_t p_hi, int32_t slots, int32_t upi, int32_t *hdr, int32_t *seq_off,
            int32_t *seq_nsplit, int32_t *merge_cnt, int4 *items, int32_t *status) {
  __shared__ int32_t warp_tot[kPlanThreads / 32];
  __shared__ int32_t bucket[kMaxPagesPerSplit + 1];  // partial splits per length, then cursors
  __shared__ int32_t carry_all, carry_full;
  // the decode launch that follows may start its CTAs' setup now (it waits
  // for this grid before reading the plan)
  asm volatile("griddepcontrol.launch_dependents;");
  const int tid = threadIdx.x;
  const int32_t cap = max_blocks * bs;
  const int32_t P = (p_lo < p_hi && B <= kMaxSimSeqs) ? choose_split(ctx, B, bs, cap, p_lo, p_hi, upi, slots)
                                                        : p_hi;
  for (int i = tid; i <= P; i += kPlanThreads) bucket[i] = 0;
  for (int64_t i = tid; i < (int64_t)B * upi; i += kPlanThreads) merge_cnt[i] = 0;
  if (tid == 0) carry_all = carry_full = 0;
  __syncthreads();
  // pass 1: per-sequence offsets, full-split count, histogram of partial lengths
  for (int32_t base = 0; base < B; base += kPlanThreads) {
    const int32_t b = base + tid;
    SeqSplits q{0, 0, 0, 0};
    if (b < B) q = seq_splits(ctx, b, bs, cap, P, status, true);
    int32_t tot_n, tot_f;
    const int32_t off = carry_all + block_exclusive_scan(q.n, warp_tot, &tot_n);
    block_exclusive_scan(q.full, warp_tot, &tot_f);
    if (b < B) {
      seq_off[b] = off;
      seq_nsplit[b] = q.n;
      if (q.n > q.full) atomicAdd(&bucket[q.rest], 1);
    }
    __syncthreads();
    if (tid == 0) {
      carry_all += tot_n;
      carry_full += tot_f;
    }
    __syncthreads();
  }
  // bucket -> first item index of each partial length, longest first
  if (tid == 0) {
    int32_t pos = carry_full;
    for (int32_t r = P; r >= 0; --r) {
      const int32_t cnt = bucket[r];
      bucket[r] = pos;
      pos += cnt;
    }
    carry_full = 0;
  }
  __syncthreads();
  // pass 2: write the items
  for (int32_t base = 0; base < B; base += kPlanThreads) {
    const int32_t b = base + tid;
    SeqSplits q{0, 0, 0, 0};
    if (b < B) q = seq_splits(ctx, b, bs, cap, P, status, false);
    int32_t tot_f;
    const int32_t foff = carry_full + block_exclusive_scan(q.full, warp_tot, &tot_f);
    if (b < B) {
      for (int32_t s = 0; s < q.full; ++s) items[foff + s] = make_int4(b, s, q.ctx, q.n);
      if (q.n > q.full) items[atomicAdd(&bucket[q.rest], 1)] = make_int4(b, q.n - 1, q.ctx, q.n);
    }
    __syncthreads();
    if (tid == 0) carry_full += tot_f;
    __syncthreads();
  }
  if (tid == 0) {
    hdr[0] = carry_all * upi;  // total work units
    hdr[1] = P;
    hdr[2] = B;
    hdr[3] = upi;
    hdr[4] = 0;  // next tail unit to hand out (tensor-core kernel)
    hdr[5] = 0;  // CTAs done claiming tail units
  }
}

// ---------------------------------------------------------------------------
// split-K epilogue shared by both kernels.
// xm/xl hold each warp's running max (log2 units) and sum per head row, xo
// each warp's unnormalised accumulator; rows are [warp][row], xo rows padded
// to xd floats. `split_row` = seq_off[b] + split, the sequence's partial-result
// row (unused when the sequence has one split); callers load it ahead of time
// so no global load sits in the epilogue. `sync` is a barrier over the
// participating threads.
// ---------------------------------------------------------------------------
template <typename Sync>
__device__ bool unit_epilogue(const DecodeArgs &a, const Unit &u, int32_t split_row, int nwarps,
                              int xr, const float *xm, const float *xl, const float *const *xo,
                              int xd, int tid, int nthreads, Sync &sync) {
  const int32_t D = a.D;
  const int32_t GR = a.GR;
  const int32_t n = u.gcount * D;
  const int64_t unit_idx = (int64_t)split_row * a.upi + u.kvh * a.HG + u.hg;
  float *part = a.partials + unit_idx * a.part_floats;
  for (int32_t i = tid; i < n; i += nthreads) {
    const int32_t g = i / D, d = i - g * D;
    float M = -INFINITY;
    for (int w = 0; w < nwarps; ++w) M = fmaxf(M, xm[w * xr + g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < nwarps; ++w) {
        const float f = exp2_or_zero(xm[w * xr + g] - M);
        L += f * xl[w * xr + g];
        O += f * xo[w][g * xd + d];
      }
    }
    if (u.nsplit == 1) {
      store_out(a, u.b * a.o0 + (int64_t)(u.qh0 + g) * a.o1 + d * a.o2, O / fmaxf(L, 1e-6f));
    } else {  // merged by merge_kernel after the launch
      part[a.part_o + g * D + d] = O;
      if (d == 0) {
        part[g] = M;
        part[GR + g] = L;
      }
    }
  }
  return sync();
}

// ---------------------------------------------------------------------------
// split-K merge: one CTA per (sequence, kv head x head group); sequences with a
// single split were finished by the decode kernel and return at once.
// ---------------------------------------------------------------------------
constexpr int kMergeThreads = 128;

__global__ void __launch_bounds__(kMergeThreads) merge_kernel(DecodeArgs a) {
  const int32_t b = blockIdx.x;
  const int32_t r = blockIdx.y;
  const int32_t n = a.seq_nsplit[b];
  if (n <= 1) return;
  const int32_t kvh = r / a.HG, hg = r - kvh * a.HG;
  const int32_t gcount = min(a.GR, a.G - hg * a.GR);
  const int32_t qh0 = kvh * a.G + hg * a.GR;
  const int32_t D = a.D, GR = a.GR;
  const float *base = a.partials + ((int64_t)a.seq_off[b] * a.upi + r) * a.part_floats;
  const int64_t stride = (int64_t)a.upi * a.part_floats;  // next split of the same head group
  for (int32_t i = threadIdx.x; i < gcount * D; i += kMergeThreads) {
    const int32_t g = i / D, d = i - g * D;
    float M = -INFINITY;
    for (int32_t s = 0; s < n; ++s) M = fmaxf(M, base[s * stride + g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll 4
      for (int32_t s = 0; s < n; ++s) {
        const float *p = base + s * stride;
        const float f = exp2_or_zero(p[g] - M);
        L += f * p[GR + g];
        O += f * p[a.part_o + g * D + d];
      }
    }
    store_out(a, b * a.o0 + (int64_t)(qh0 + g) * a.o1 + d * a.o2, O / fmaxf(L, 1e-6f));
  }
}

struct CtaSync {
  __device__ bool operator()() {
    __syncthreads();
    return true;
  }
};

// Barrier over the consumer warps of the tensor-core kernel, built on an
// mbarrier (one arrival per warp) so that every wait is bounded.
struct GroupSync {
  uint64_t *bar;
  uint32_t phase;
  int32_t *status;
  uint32_t max_polls;
  __device__ bool operator()() {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    const bool ok = mbar_wait_bounded(bar, phase & 1u, max_polls);
    ++phase;
    if (!ok) flag_status(status, PKV_DEV_WAIT_TIMEOUT);
    return ok;
  }
};

// ---------------------------------------------------------------------------
// CUDA-core kernel (any dtype, any block size, head_dim <= 32*DJ)
// ---------------------------------------------------------------------------
template <typename KT, int DJ, int GM>
__global__ void __launch_bounds__(kGenThreads)
decode_generic_kernel(DecodeArgs a) {
  extern __shared__ float gsm[];
  constexpr int DP = DJ * 32;
  float *q_s = gsm;                          // [GM][DP]
  float *xm = q_s + GM * DP;                 // [NW][16]
  float *xl = xm + kGenWarps * kTcRows;      // [NW][16]
  float *xo = xl + kGenWarps * kTcRows;      // [NW][16][DP]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const KT *kc = reinterpret_cast<const KT *>(a.kc);
  const KT *vc = reinterpret_cast<const KT *>(a.vc);
  const int32_t total = a.hdr[0];
  const int32_t P = a.hdr[1];
  CtaSync sync;

  for (int32_t w = blockIdx.x; w < total; w += gridDim.x) {
    const Unit u = decode_unit(a, P, w);
    const int32_t split_row = u.nsplit > 1 ? a.seq_off[u.b] + u.s : 0;  // used at the end
    for (int i = tid; i < GM * DP; i += kGenThreads) {
      const int g = i / DP, d = i - g * DP;
      float v = 0.f;
      if (g < u.gcount && d < a.D)
        v = load_as_f32(a.q, u.b * a.q0 + (int64_t)(u.qh0 + g) * a.q1 + d * a.q2, a.q_dtype);
      q_s[i] = v;
    }
    __syncthreads();

    float m[GM], l[GM], acc[GM][DJ];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int j = 0; j < DJ; ++j) acc[g][j] = 0.f;
    }

    const int32_t t_begin = u.p_begin * a.bs;
    const int32_t t_end = min(u.p_end * a.bs, u.ctx);
    for (int32_t t = t_begin + warp; t < t_end; t += kGenWarps) {
      const int32_t pg = t / a.bs;
      const int32_t page = a.bt[u.b * a.bt0 + (int64_t)pg * a.bt1];
      if (page < 0 || page >= a.num_blocks) {
        if (lane == 0) flag_status(a.status, PKV_DEV_PAGE_OUT_OF_RANGE);
        continue;
      }
      const int64_t base = page * a.c0 + u.kvh * a.c1 + (int64_t)(t - pg * a.bs) * a.c2;
      float kr[DJ], vr[DJ];
#pragma unroll
      for (int j = 0; j < DJ; ++j) {
        const int d = lane + 32 * j;
        kr[j] = d < a.D ? Elem<KT>::to_f32(kc[base + d * a.c3]) : 0.f;
        vr[j] = d < a.D ? Elem<KT>::to_f32(vc[base + d * a.c3]) : 0.f;
      }
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        if (g < u.gcount) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < DJ; ++j) s = fmaf(q_s[g * DP + lane + 32 * j], kr[j], s);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          // logits = (q . k) * scale (paged_kv.py:133-135), kept in log2 units
          const float x = s * a.scale_log2;
          const float mn = fmaxf(m[g], x);
          const float alpha = (mn == m[g]) ? 1.f : exp2_or_zero(m[g] - mn);
          const float p = exp2f(x - mn);
          l[g] = l[g] * alpha + p;
#pragma unroll
          for (int j = 0; j < DJ; ++j) acc[g][j] = fmaf(p, vr[j], acc[g][j] * alpha);
          m[g] = mn;
        }
      }
    }

#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < u.gcount) {
        if (lane == 0) {
          xm[warp * kTcRows + g] = m[g];
          xl[warp * kTcRows + g] = l[g];
        }
#pragma unroll
        for (int j = 0; j < DJ; ++j) xo[(warp * kTcRows + g) * DP + lane + 32 * j] = acc[g][j];
      }
    }
    __syncthreads();
    const float *xo_w[kGenWarps];
#pragma unroll
    for (int w = 0; w < kGenWarps; ++w) xo_w[w] = xo + w * kTcRows * DP;
    unit_epilogue(a, u, split_row, kGenWarps, kTcRows, xm, xl, xo_w, DP, tid, kGenThreads, sync);
  }
}

size_t generic_smem_bytes(int DJ, int GM) {
  const int DP = DJ * 32;
  return sizeof(float) * ((size_t)GM * DP + 2 * kGenWarps * kTcRows + (size_t)kGenWarps * kTcRows * DP) +
         16;
}

// ---------------------------------------------------------------------------
// cp.async + tensor-core kernel (bf16 / fp16 cache, block_size 16, head_dim 64/128)
// ---------------------------------------------------------------------------
enum : int32_t { kElemPage = 0, kElemEmpty = 1, kElemStop = 2 };

// One pipeline element as the producer publishes it to a consumer warp: the
// page (or its absence) plus everything the consumer needs about the unit,
// so consumers never touch global memory for bookkeeping.
struct __align__(16) SlotMeta {
  int32_t kind;    // kElemPage / kElemEmpty / kElemStop
  int32_t valid;   // valid tokens in the page (1..16)
  int32_t last;    // last element of this warp for the unit
  int32_t work;    // work-unit id
  int32_t qslot;   // smem slot holding the unit's query rows
  int32_t b, s, nsplit;
  int32_t kvh, hg, gcount, qh0;
  int32_t page;       // physical page id (kElemPage only)
  int32_t newrow;     // row of this page that takes the appended token, or -1
  int32_t split_row;  // seq_off[b] + s: the unit's partial-result row (nsplit > 1)
  int32_t pad;
};

static_assert(sizeof(SlotMeta) == 64, "SlotMeta layout");
static_assert(offsetof(SlotMeta, qslot) == 16 && offsetof(SlotMeta, kvh) == 32 &&
                  offsetof(SlotMeta, page) == 48,
              "SlotMeta fields read as 16-byte blocks must stay 16-byte aligned");

constexpr int kBoxRows = 16;               // tokens per page (block_size)
constexpr int kBoxBytes = kBoxRows * 128;  // one [16][64] 16-bit box, 128-byte swizzled rows

template <int D> struct TcShape {
  static constexpr int kBoxes = D / 64;
  static constexpr int kTile = kBoxes * kBoxBytes;  // one K (or V) page of one head
  static constexpr int kSlot = 2 * kTile;           // K + V
  static constexpr int kKSteps = D / 16;
  static constexpr int kMTiles = D / 16;
  static constexpr int kQRow = D * 2 + 16;    // padded query row (bytes): conflict-free ldmatrix
  static constexpr int kQNew = kTcRows * kQRow;  // then the appended token's K row and V row
  static constexpr int kQSlot = kQNew + 2 * D * 2;
};

// Shared-memory plan of the kernel: per consumer warp a ring of S data slots
// (one K+V page each, filled by the warp itself with cp.async) and a deeper
// ring of MD metadata entries (filled by the producer warp); query rows of
// QS = S + 1 units (the consumers' look-ahead of S - 1 elements can reach S - 1
// units ahead, so the producer must be able to stage that many more). A
// deeper metadata ring lets the producer publish a whole unit and go on to the
// next one sooner: 4 S for head_dim 128 (+2.4% config 3, +1.3% config 5,
// +0.6% config 4 against 2 S on B200; 8 S measured the same as 4 S); head_dim
// 64 keeps 2 S, its 6 data slots leave no shared memory for more.
template <int D, int NW, int S>
struct TcSmem {
  static constexpr int MD = (D == 128 ? 4 : 2) * S;
  static constexpr int QS = S + 1;
  static constexpr size_t kTiles = (size_t)NW * S * TcShape<D>::kSlot;
  static constexpr size_t kQ = kTiles;
  static constexpr size_t kMeta = kQ + (size_t)QS * TcShape<D>::kQSlot;
  static constexpr size_t kFull = align_up(kMeta + sizeof(SlotMeta) * NW * MD, 16);
  static constexpr size_t kEmpty = kFull + 8 * NW * MD;
  static constexpr size_t kQEmpty = kEmpty + 8 * NW * MD;
  static constexpr size_t kQFull = kQEmpty + 8 * QS;
  static constexpr size_t kGroup = kQFull + 8 * QS;
  // [NW] slot holding each warp's exchange rows, then the merge flag
  static constexpr size_t kXSlot = kGroup + 8;
  static constexpr size_t kXm = align_up(kXSlot + 4 * (NW + 1), 16);
  static constexpr size_t kXl = kXm + sizeof(float) * NW * kTcRows;
  static constexpr size_t kBt = kXl + sizeof(float) * NW * kTcRows;
  static size_t bytes(int32_t P) { return kBt + sizeof(int32_t) * (size_t)P + 1024; }
};

// Byte offset, inside a K or V tile, of 16-byte chunk c of a page slab
// (16 rows of D contiguous 16-bit values): row r, chunk cc of the row, stored
// in [D/64 boxes][16 rows][128 bytes] with chunk (cc % 8) ^ (r % 8).
template <int D>
__device__ __forceinline__ uint32_t slab_chunk_offset(int c) {
  constexpr int kRowChunks = D / 8;
  const int r = c / kRowChunks, cc = c % kRowChunks;
  return (cc >> 3) * kBoxBytes + r * 128 + (((cc & 7) ^ (r & 7)) << 4);
}

// 16-byte copy of which only the first src_bytes are read; the rest are zero
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Packs (x, y) into a 16-bit pair `hi` and the rounding remainders into `lo`.
template <typename M>
__device__ __forceinline__ void split_pair(float x, float y, uint32_t &hi, uint32_t &lo) {
  hi = M::pack(x, y);
  const float hx = M::unpack_lo(hi), hy = M::unpack_hi(hi);
  lo = M::pack(x - hx, y - hy);
}


// RoPE of one 16-byte chunk x (8 elements of one head) with the chunk p at the
// same place in the other half of the head, and the cos / sin chunks of those
// 8 positions; second: x lies in the second half. The rounding points of HF's
// apply_rotary_pos_emb: x * cos and rotate_half(x) * sin rounded to T, then
// their sum.
template <typename T>
__device__ __forceinline__ uint4 rope_chunk(uint4 x, uint4 p, uint4 cs, uint4 sn, bool second) {
  const T *xe = reinterpret_cast<const T *>(&x), *pe = reinterpret_cast<const T *>(&p);
  const T *ce = reinterpret_cast<const T *>(&cs), *se = reinterpret_cast<const T *>(&sn);
  uint4 out;
  T *oe = reinterpret_cast<T *>(&out);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float a = Elem<T>::to_f32(T(Elem<T>::to_f32(xe[j]) * Elem<T>::to_f32(ce[j])));
    const float pv = Elem<T>::to_f32(pe[j]);
    const float b = Elem<T>::to_f32(T((second ? pv : -pv) * Elem<T>::to_f32(se[j])));
    oe[j] = T(a + b);
  }
  return out;
}

__device__ __forceinline__ uint4 shfl_xor_u4(uint4 v, int m) {
  return make_uint4(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m),
                    __shfl_xor_sync(0xffffffffu, v.z, m), __shfl_xor_sync(0xffffffffu, v.w, m));
}

template <typename T, int D, int NW, int S, bool kExactP, int NT, bool kRope>
__global__ void __launch_bounds__((NW + 1) * 32, 1)
decode_tc_kernel(DecodeArgs a) {
  static_assert(NT == 1 || NT == 2, "one or two tiles of 8 query heads");
  using Sh = TcShape<D>;
  using L = TcSmem<D, NW, S>;
  extern __shared__ uint8_t tc_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *tiles = smem;
  uint8_t *qbuf = smem + L::kQ;
  SlotMeta *meta = reinterpret_cast<SlotMeta *>(smem + L::kMeta);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kFull);
  uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L::kEmpty);
  uint64_t *qempty = reinterpret_cast<uint64_t *>(smem + L::kQEmpty);
  uint64_t *qfull = reinterpret_cast<uint64_t *>(smem + L::kQFull);  // query slot staged
  uint64_t *group = reinterpret_cast<uint64_t *>(smem + L::kGroup);
  int32_t *xslot = reinterpret_cast<int32_t *>(smem + L::kXSlot);
  float *xm = reinterpret_cast<float *>(smem + L::kXm);
  float *xl = reinterpret_cast<float *>(smem + L::kXl);
  int32_t *btbuf = reinterpret_cast<int32_t *>(smem + L::kBt);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int MD = L::MD, QS = L::QS;
  static_assert(NW * MD <= (NW + 1) * 32 && QS <= (NW + 1) * 32, "one thread per mbarrier");
  // Programmatic dependent launch. Each thread first waits for the previous
  // kernel in the stream (griddepcontrol.wait: it is complete and its writes
  // are visible) and only then lets the next launch place its CTAs on the SMs
  // this grid frees. A launch queued behind this one therefore finds every
  // kernel before this one complete, which is what PKV_DECODE_EARLY_START on
  // the next layer's launch relies on.
  auto dep_wait = [] {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
  };
  const bool early = a.early != 0;
  if (tid < NW * MD) {
    mbar_init(&full[tid], 1);
    mbar_init(&empty[tid], 1);
  }
  if (tid < QS) {
    mbar_init(&qempty[tid], 1);
    mbar_init(&qfull[tid], 1);
  }
  if (tid == 0) mbar_init(group, NW);
  fence_mbar_init();
  __syncthreads();
  // Only shared memory was touched so far. Past dep_wait() the previous
  // kernel in the stream (which may have written q, the new rows, the caches
  // or the plan) is complete and its writes are visible. With early start the
  // producer reads the plan and the first unit's block-table entries and
  // publishes its pages, and each consumer warp issues its first page, before
  // waiting; q, the new rows, RoPE's cos / sin, the schedule counters and
  // every global write stay behind the wait.
  if (!early) dep_wait();

  if (warp == NW) {
    const int32_t total = a.hdr[0];
    const int32_t P = a.hdr[1];  // the plan's split length
    // =========================== producer warp ===========================
    // Schedule: the plan numbers units longest first. CTA c takes unit c in
    // round 0, 2G-1-c in round 1, 2G+c in round 2, ... (G = gridDim.x, "snake"
    // order: the CTAs given the longest units of one round get the shortest of
    // the next). With at least six rounds of units, only the first R = U/G - 1
    // rounds are assigned this way; the remaining, shortest units are handed
    // out in order by a global counter, so the CTAs that run ahead take more of
    // them and the launch ends within about one short unit. The warp runs a
    // three-deep software pipeline so no global-load latency is exposed at a
    // unit boundary: while lane 0 publishes unit r, the descriptor of r+2 is
    // being loaded, the block-table entries and query rows of r+1 are in flight
    // into registers, and the claim of round r+3 (if it is a counted one) is
    // outstanding.
    const uint32_t FULL = 0xffffffffu;
    const int32_t G = (int32_t)gridDim.x;
    const int4 none = make_int4(0, 0, 0, 1);

    // registers holding the NEXT unit's block-table entries, query rows and
    // partial-result row
    int32_t btr[kBtRegs];
    uint4 qr[(kTcRows * D * 2 / 16 + 31) / 32];
    int32_t srow = 0;
    uint4 nkv = make_uint4(0, 0, 0, 0);  // appended token: lane < D/8 a K chunk, then V chunks
    // RoPE: the cos / sin chunk (lane % (D/8)) of the next unit's sequence; a
    // lane's query chunks and its K chunk all sit at that chunk index
    uint4 rc = make_uint4(0, 0, 0, 0), rs = make_uint4(0, 0, 0, 0);
    constexpr int kRowChunks = D / 8;    // 16-byte chunks of one K or V row
    constexpr int kQVec = kTcRows * D * 2 / 16;  // 16-byte vectors of a query block
    constexpr int kQPerLane = (kQVec + 31) / 32;
    // plan-side loads of a unit: its partial-result row and block-table entries
    auto load_bt = [&](int32_t w, int4 d) {
      Unit u = unit_from(a, P, w, d);
      const int32_t np = u.p_end - u.p_begin;
      srow = (w < total && u.nsplit > 1) ? a.seq_off[u.b] + u.s : 0;
#pragma unroll
      for (int i = 0; i < kBtRegs; ++i) {
        const int32_t pi = lane + 32 * i;
        btr[i] = (w < total && pi < np) ? a.bt[u.b * a.bt0 + (int64_t)(u.p_begin + pi) * a.bt1] : -1;
      }
    };
    // input-side loads (what the previous kernel may have written): the new
    // K / V rows, RoPE's cos / sin and the query rows
    auto load_in = [&](int32_t w, int4 d) {
      Unit u = unit_from(a, P, w, d);
      if (a.kn != nullptr && w < total && u.s == u.nsplit - 1 && u.ctx > 0 && lane < 2 * kRowChunks) {
        const int which = lane / kRowChunks, cc = lane % kRowChunks;
        const uint8_t *src = reinterpret_cast<const uint8_t *>(which ? a.vn : a.kn);
        nkv = *reinterpret_cast<const uint4 *>(src + (u.b * a.n0 + (int64_t)u.kvh * a.n1) * 2 + 16 * cc);
      }
      if (kRope && a.rcos != nullptr && w < total) {
        const int64_t off = (u.b * a.rcs + 8 * (lane % kRowChunks)) * 2;
        rc = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(a.rcos) + off);
        rs = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(a.rsin) + off);
      }
      const uint8_t *qb = reinterpret_cast<const uint8_t *>(a.q);
#pragma unroll
      for (int i = 0; i < kQPerLane; ++i) {
        const int v = lane + 32 * i;
        const int r = v / (D / 8), c = v % (D / 8);
        uint4 x = make_uint4(0, 0, 0, 0);
        if (w < total && v < kQVec && r < u.gcount) {
          const int64_t row = u.b * a.q0 + (int64_t)(u.qh0 + r) * a.q1;
          if (a.q_vec) {
            x = *reinterpret_cast<const uint4 *>(qb + 2 * row + 16 * c);
          } else {  // arbitrary strides: eight 16-bit loads
            const uint16_t *qh = reinterpret_cast<const uint16_t *>(a.q);
            uint32_t wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              wv[e] = (uint32_t)qh[row + (int64_t)(8 * c + 2 * e) * a.q2] |
                      ((uint32_t)qh[row + (int64_t)(8 * c + 2 * e + 1) * a.q2] << 16);
            x = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
        qr[i] = x;
      }
    };
    auto load_next = [&](int32_t w, int4 d) {
      load_bt(w, d);
      load_in(w, d);
    };
    const int32_t c = (int32_t)blockIdx.x;
    // the descriptors of rounds 0 and 1 are loaded together with the unit
    // count instead of after it (indices clamped into the item array; a
    // descriptor past the count is never used)
    const int4 r0 = a.items[min((int64_t)c / a.upi, a.max_items - 1)];
    const int4 r1 = a.items[min((int64_t)(2 * G - 1 - c) / a.upi, a.max_items - 1)];
    // rounds assigned statically; claims run three rounds ahead of use, so a
    // counted tail only pays off once the CTAs have progressed for a few rounds
    const int32_t R = total / G >= 6 ? total / G - 1 : INT32_MAX;
    // unit of static round r < R (r * G + ... < total)
    auto unit_at = [&](int32_t r) -> int32_t {
      const int64_t w = (int64_t)r * G + ((r & 1) ? G - 1 - c : c);
      return w < total ? (int32_t)w : total;
    };
    // unit of counted round r >= R from the counter value f claimed for it
    auto tail_unit = [&](int32_t f) -> int32_t {
      const int64_t w = (int64_t)R * G + f;
      return w < total ? (int32_t)w : total;
    };
    int32_t fetched = 0;  // lane 0: the outstanding claim
    int32_t round = 0;
    int32_t w1 = unit_at(0), w2 = unit_at(1);
    int4 d1 = w1 < total ? r0 : none;
    int4 d2 = w2 < total ? r1 : none;
    bool waited = !early;  // past dep_wait()
    if (waited) {
      if (lane == 0 && R <= 2) fetched = atomicAdd(&a.sched[0], 1);  // round 2 is counted
      load_next(w1, d1);
    } else {
      load_bt(w1, d1);  // the rest after the first unit's pages are out
    }

    int32_t kcount = 0;  // lane cw < NW: elements published to consumer warp cw
    bool ok = true;
    int32_t nunit = 0;  // units issued by this CTA (query slot = nunit % QS)
    while (w1 < total && ok) {
      const Unit u = unit_from(a, P, w1, d1);
      const int32_t npages = u.p_end - u.p_begin;
      const int qs = nunit % QS;
      const int32_t split_row = srow;
      // (1) the unit's block-table entries and query rows -> smem
      if (nunit >= QS) {
        if (!mbar_wait_backoff(&qempty[qs], ((nunit / QS) - 1) & 1, a.max_tries)) {
          flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
          ok = false;
        }
      }
#pragma unroll
      for (int i = 0; i < kBtRegs; ++i) {
        const int32_t pi = lane + 32 * i;
        if (pi < npages) {
          int32_t page = btr[i];
          if (page < 0 || page >= a.num_blocks) {
            flag_status(a.status, PKV_DEV_PAGE_OUT_OF_RANGE);
            page = -1;
          }
          btbuf[pi] = page;
        }
      }
      // fused append: this unit holds the sequence's last page (its last split)
      const bool app = a.kn != nullptr && u.s == u.nsplit - 1 && u.ctx > 0;
      const int32_t app_pi = app ? (u.ctx - 1) / kBoxRows - u.p_begin : -1;  // page within the unit
      const int32_t app_row = (u.ctx - 1) % kBoxRows;
      __syncwarp();  // btbuf written
      // (2) publish the unit's pages to the consumer warps (page p -> warp p % NW),
      //     lane cw filling warp cw's ring; each consumer loads its pages itself
      //     with cp.async. The first page of every warp goes out before the
      //     query rows are staged, so the first loads overlap the staging; a
      //     consumer waits for qfull[qs] before it reads the rows.
      const int32_t rounds = npages > 0 ? (npages + NW - 1) / NW : 1;
      auto publish = [&](int32_t j0, int32_t j1) {
        if (lane >= NW || !ok) return;
        for (int32_t j = j0; j < j1; ++j) {
          const int32_t pi = j * NW + lane;
          const bool has = pi < npages;
          const bool last = (j == rounds - 1);
          if (!has && !last) continue;
          const int32_t k = kcount++;
          // test of the bounded waits: an element that is never published
          if (a.withhold && k == 0 && lane == 0 && blockIdx.x == 0) continue;
          const int slot = lane * MD + (k % MD);
          const int32_t use = k / MD;
          if (use > 0 && !mbar_wait_backoff(&empty[slot], (use - 1) & 1, a.max_tries)) {
            flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
            ok = false;
            return;
          }
          const int32_t page = has ? btbuf[pi] : -1;
          SlotMeta md;
          md.kind = page >= 0 ? kElemPage : kElemEmpty;
          md.valid = has ? min(kBoxRows, u.ctx - (u.p_begin + pi) * kBoxRows) : 0;
          md.last = last ? 1 : 0;
          md.work = w1;
          md.qslot = qs;
          md.b = u.b;
          md.s = u.s;
          md.nsplit = u.nsplit;
          md.kvh = u.kvh;
          md.hg = u.hg;
          md.gcount = u.gcount;
          md.qh0 = u.qh0;
          md.page = page;
          md.newrow = (pi == app_pi) ? app_row : -1;
          md.split_row = split_row;
          md.pad = (nunit / QS) & 1;  // phase of qfull[qs] that stages this unit's rows
          meta[slot] = md;
          mbar_arrive(&full[slot]);
        }
      };
      // early start, first unit: every round that fits the (still empty) ring
      // goes out before the wait, so no consumer waits for the producer's
      // post-wait staging to get its next element; more would have to wait for
      // ring space, which consumers free only after reading this unit's rows
      const int32_t first_rounds = waited ? 1 : min(rounds, (int32_t)MD);
      publish(0, first_rounds);
      __syncwarp();
      if (!waited) {
        // early start: the first unit's pages are being loaded; now the
        // previous kernel, then what it may have written
        dep_wait();
        waited = true;
        if (lane == 0 && R <= 2) fetched = atomicAdd(&a.sched[0], 1);
        load_in(w1, d1);
      }
      // query rows (and the appended K/V row) -> the unit's query slot
      if (kRope && a.rcos != nullptr) {  // RoPE: the partner chunk (other half of the head) is in lane ^ D/16
        const bool second = (lane % kRowChunks) >= kRowChunks / 2;
#pragma unroll
        for (int i = 0; i < kQPerLane; ++i)
          qr[i] = rope_chunk<T>(qr[i], shfl_xor_u4(qr[i], kRowChunks / 2), rc, rs, second);
        const uint4 pk = shfl_xor_u4(nkv, kRowChunks / 2);
        if (lane < kRowChunks) nkv = rope_chunk<T>(nkv, pk, rc, rs, second);
      }
#pragma unroll
      for (int i = 0; i < kQPerLane; ++i) {
        const int v = lane + 32 * i;
        if (v < kQVec) {
          const int r = v / (D / 8), c = v % (D / 8);
          *reinterpret_cast<uint4 *>(qbuf + qs * Sh::kQSlot + r * Sh::kQRow + 16 * c) = qr[i];
        }
      }
      if (app && lane < 2 * kRowChunks)
        *reinterpret_cast<uint4 *>(qbuf + qs * Sh::kQSlot + Sh::kQNew + 16 * lane) = nkv;
      __syncwarp();
      if (lane == 0) mbar_arrive(&qfull[qs]);
      if (app && u.hg == 0 && lane < 2 * kRowChunks) {
        // one unit per (sequence, kv head) writes the token into the cache for
        // later steps; every unit reading the page patches its own smem copy
        const int32_t page = btbuf[app_pi];
        if (page >= 0) {
          const int which = lane / kRowChunks, cc = lane % kRowChunks;
          uint8_t *dst = reinterpret_cast<uint8_t *>(const_cast<void *>(which ? a.vc : a.kc));
          *reinterpret_cast<uint4 *>(dst + ((int64_t)page * a.c0 + (int64_t)u.kvh * a.c1 +
                                            (int64_t)app_row * a.c2) * 2 + 16 * cc) = nkv;
        }
      }
      publish(first_rounds, rounds);
      // (3) prefetch: the next unit's block-table entries and query rows, the
      //     descriptor of the one after
      load_next(w2, d2);
      int32_t w3;
      if (round + 2 < R) {
        w3 = unit_at(round + 2);
      } else {
        w3 = tail_unit(__shfl_sync(FULL, fetched, 0));
      }
      // the claim for round r + 3 is consumed at the next iteration
      if (lane == 0 && round + 3 >= R && w3 < total) fetched = atomicAdd(&a.sched[0], 1);
      const int4 d3 = w3 < total ? a.items[w3 / a.upi] : none;
      ok = __all_sync(FULL, ok);
      __syncwarp();  // btbuf / qbuf are rewritten for the next unit
      ++nunit;
      ++round;
      w1 = w2;
      d1 = d2;
      w2 = w3;
      d2 = d3;
    }
    if (lane < NW && ok) {  // a stop element to each consumer warp
      const int32_t k = kcount++;
      const int slot = lane * MD + (k % MD);
      const int32_t use = k / MD;
      if (use > 0 && !mbar_wait_backoff(&empty[slot], (use - 1) & 1, a.max_tries)) {
        flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
      } else {
        SlotMeta md{};
        md.kind = kElemStop;
        md.last = 1;
        md.work = -1;
        meta[slot] = md;
        mbar_arrive(&full[slot]);
      }
    }
    // (a CTA without units, or stopped by a timeout, under early start)
    if (!waited) dep_wait();
    if (lane == 0) {
      // This CTA claims no more units. The last CTA to get here resets the
      // counters so the plan can drive the next launch.
      __threadfence();
      const int done = atomicAdd(&a.sched[1], 1);
      if (done == (int)gridDim.x - 1) {
        atomicExch(&a.sched[0], 0);
        atomicExch(&a.sched[1], 0);
      }
    }
    return;
  }

  // =========================== consumer warps ===========================
  using M = Mma16816<T>;
  const int cw = warp;
  // m16n8k16 fragment coordinates: lane = 4 * fr + fq
  const int fr = lane >> 2, fq = lane & 3;
  GroupSync sync{group, 0u, a.status, a.max_polls};

  // A page is processed transposed: S^T = K Q^T (the 16 tokens on M, up to 8
  // query heads per head tile on N) and O^T = V^T P^T (head_dim on M), so one
  // page costs 2 * D/16 MMAs per head tile. Per-lane byte offsets inside a
  // swizzled tile (128-byte rows, 16-byte chunk c of row r stored at chunk
  // c ^ (r % 8)) for the ldmatrix.x4 of k-step / m-tile j; the box offset
  // (j / 4) * 2 KB is a compile-time constant:
  //   K, A operand, plain:      token (lane & 7) + 8 ((lane >> 3) & 1), chunk 2j + (lane >> 4)
  //   V, A operand, transposed: token (lane & 7) + 8 (lane >> 4),       chunk 2j + ((lane >> 3) & 1)
  uint32_t k_off[4], v_off[4];
  {
    const uint32_t kr = (lane & 7) + 8 * ((lane >> 3) & 1), kh = lane >> 4;
    const uint32_t vr = (lane & 7) + 8 * (lane >> 4), vh = (lane >> 3) & 1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      k_off[j] = kr * 128 + (((2 * j + kh) ^ (lane & 7)) << 4);
      v_off[j] = vr * 128 + (((2 * j + vh) ^ (lane & 7)) << 4);
    }
  }
  // query rows, B operand, plain ldmatrix.x4 over two k-steps: head (lane & 7)
  // (+8 for the second head tile), chunk 2 ks + (lane >> 3)
  const uint32_t q_off = (lane & 7) * Sh::kQRow + 16 * (lane >> 3);

  uint32_t qb[NT][Sh::kKSteps][2];
  float o[NT][Sh::kMTiles][4];  // O^T: d = 16 mt + fr (+8), head 8 nt + 2 fq (+1)
  float m[NT][2], l[NT][2];     // running max and this lane's partial sum, head 8 nt + 2 fq + j
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m[nt][0] = m[nt][1] = -INFINITY;
    l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
    for (int i = 0; i < Sh::kMTiles; ++i) o[nt][i][0] = o[nt][i][1] = o[nt][i][2] = o[nt][i][3] = 0.f;
  }
  int32_t cur_work = -1, cur_qslot = 0;
  const float sl2 = a.scale_log2;

  // Each consumer warp loads its own pages: element e's K and V slabs go into
  // data slot e % S with 16-byte cp.async copies (each instruction moves 512
  // contiguous bytes of one slab, written straight into the swizzled tile
  // layout), one commit group per element, issued S - 1 elements ahead.
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(a.kc);
  const uint8_t *vbase = reinterpret_cast<const uint8_t *>(a.vc);
  int32_t stop_at = INT32_MAX;
  bool alive = true;
  // destination offsets of this lane's chunks c = lane + 32 i: rows r and r + 8
  // share the swizzle pattern, so chunk i + 4 lands 1024 bytes after chunk i
  uint32_t dst_off[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dst_off[i] = slab_chunk_offset<D>(lane + 32 * i);
  auto issue = [&](int32_t e) {
    if (e <= stop_at && alive) {
      const int ms = cw * MD + (e % MD);
      if (!mbar_wait_bounded(&full[ms], (e / MD) & 1, a.max_polls)) {
        flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
        alive = false;
      } else {
        const int32_t kind = meta[ms].kind;
        if (kind == kElemStop) {
          stop_at = e;
        } else if (kind == kElemPage) {
          const int64_t off =
              ((int64_t)meta[ms].page * a.c0 + (int64_t)meta[ms].kvh * a.c1) * 2 + 16 * lane;
          const uint8_t *ks = kbase + off;
          const uint8_t *vs = vbase + off;
          const uint32_t dst = smem_u32(tiles + (size_t)(cw * S + (e % S)) * Sh::kSlot);
          // rows past the context are zero-filled, not read: their weights are
          // 0, but 0 x (a NaN or Inf left in an unused cache slot) is not, and
          // the reference's masked loads read 0 there
          const int32_t valid = meta[ms].valid;
#pragma unroll
          for (int i = 0; i < D / 16; ++i) {
            const uint32_t o = dst + dst_off[i & 3] + 1024 * (i >> 2);
            const uint32_t n = (32 * i + lane) / (D / 8) < valid ? 16u : 0u;  // token row of this chunk
            cp_async16_zfill(o, ks + 512 * i, n);
            cp_async16_zfill(o + Sh::kTile, vs + 512 * i, n);
          }
        }
      }
    }
    cp_async_commit();  // one group per element, possibly empty
  };
  if (early) {
    // the first element is published before the producer's dependency wait:
    // its page loads start now, the rest after this warp's own wait
    issue(0);
    dep_wait();
#pragma unroll 1
    for (int32_t e = 1; e < S - 1; ++e) issue(e);
  } else {
#pragma unroll 1
    for (int32_t e = 0; e < S - 1; ++e) issue(e);
  }

  for (int32_t k = 0;; ++k) {
    issue(k + S - 1);
    if (!alive) {
      cp_async_wait_all();
      return;
    }
    cp_async_wait<S - 1>();  // element k's group (and all older) has landed
    __syncwarp();
    const int ms = cw * MD + (k % MD);
    // per page only the first 16 bytes are needed; the unit fields are read
    // below for a unit's first and last element
    const int4 head = *reinterpret_cast<const int4 *>(&meta[ms]);
    SlotMeta md;
    md.kind = head.x;
    md.valid = head.y;
    md.last = head.z;
    md.work = head.w;
    const int4 tailv = *reinterpret_cast<const int4 *>(&meta[ms].page);  // bytes 48..63
    md.newrow = tailv.y;
    md.split_row = tailv.z;
    md.pad = tailv.w;
    if (md.last || md.work != cur_work) {
      // 16-byte aligned blocks of SlotMeta: bytes 16..31 and 32..47
      const int4 m1v = *reinterpret_cast<const int4 *>(&meta[ms].qslot);
      const int4 m2v = *reinterpret_cast<const int4 *>(&meta[ms].kvh);
      md.qslot = m1v.x;
      md.b = m1v.y;
      md.s = m1v.z;
      md.nsplit = m1v.w;
      md.kvh = m2v.x;
      md.hg = m2v.y;
      md.gcount = m2v.z;
      md.qh0 = m2v.w;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[ms]);  // metadata copied: the producer may reuse the entry
    if (md.kind == kElemStop) break;
    const int slot = cw * S + (k % S);
    if (md.work != cur_work) {
      cur_work = md.work;
      cur_qslot = md.qslot;
      if (!mbar_wait_bounded(&qfull[md.qslot], (uint32_t)md.pad, a.max_polls)) {  // the unit's rows are staged
        flag_status(a.status, PKV_DEV_WAIT_TIMEOUT);
        cp_async_wait_all();
        return;
      }
      const uint32_t qs0 = smem_u32(qbuf + md.qslot * Sh::kQSlot) + q_off;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int kp = 0; kp < Sh::kKSteps / 2; ++kp)
          ldsm_x4(qs0 + nt * 8 * Sh::kQRow + kp * 64, qb[nt][2 * kp][0], qb[nt][2 * kp][1],
                  qb[nt][2 * kp + 1][0], qb[nt][2 * kp + 1][1]);
    }
    if (md.kind == kElemPage && md.newrow >= 0) {
      // fused append: the page's copy in smem may predate the token (the cache
      // write happens in whichever CTA owns it, unordered with this copy), so
      // put the appended K and V rows, staged with the query rows, into the tile
      constexpr int kRowChunks = D / 8;
      if (lane < 2 * kRowChunks) {
        const int which = lane / kRowChunks, cc = lane % kRowChunks;
        const uint4 v = *reinterpret_cast<const uint4 *>(qbuf + cur_qslot * Sh::kQSlot + Sh::kQNew + 16 * lane);
        *reinterpret_cast<uint4 *>(tiles + (size_t)slot * Sh::kSlot + which * Sh::kTile +
                                   slab_chunk_offset<D>(md.newrow * kRowChunks + cc)) = v;
      }
      __syncwarp();
    }

    if (md.kind == kElemPage) {
      const uint32_t kt = smem_u32(tiles + (size_t)slot * Sh::kSlot);
      const uint32_t vt = kt + Sh::kTile;
      // ---- S^T = K Q^T; even and odd k-steps accumulate separately (two
      // short MMA chains) and are added
      float st[NT][2][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) st[nt][c][0] = st[nt][c][1] = st[nt][c][2] = st[nt][c][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < Sh::kKSteps; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kt + (ks >> 2) * kBoxBytes + k_off[ks & 3], a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          M::run(st[nt][ks & 1], a0, a1, a2, a3, qb[nt][ks][0], qb[nt][ks][1]);
      }
      // ---- online softmax of each head over the page: this lane holds tokens
      // fr and fr + 8 of heads 2 fq, 2 fq + 1; the 8 lanes with the same fq
      // hold the other tokens
      bool moved = false;
      float al[NT][2];
      uint32_t pb[NT][2], pbl[NT][2];  // P^T as B fragments: tokens 2 fq (+1), +8; head fr
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float x[4], p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const bool in = (i < 2 ? fr : fr + 8) < md.valid;
          x[i] = in ? (st[nt][0][i] + st[nt][1][i]) * sl2 : -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float mx = fmaxf(x[j], x[2 + j]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          // a page element has a valid token, so n is finite: masked logits
          // (-inf) give exp2 = 0 and the first page's alpha is 0
          const float n = fmaxf(m[nt][j], mx);
          al[nt][j] = fast_exp2(m[nt][j] - n);
          p[j] = fast_exp2(x[j] - n);
          p[2 + j] = fast_exp2(x[2 + j] - n);
          l[nt][j] = l[nt][j] * al[nt][j] + (p[j] + p[2 + j]);
          m[nt][j] = n;
          moved |= al[nt][j] != 1.f;
        }
        // P rounded to 16 bits (relative error <= 2^-9 per weight); with
        // kExactP also the 16-bit remainder (P = hi + lo, ~17 significant
        // bits). The accumulator rows (tokens fr, fr + 8) become the B
        // operand's columns by an in-register 8x8 transpose.
        if constexpr (kExactP) {
          uint32_t h0, l0, h1, l1;
          split_pair<M>(p[0], p[1], h0, l0);
          split_pair<M>(p[2], p[3], h1, l1);
          pb[nt][0] = movmatrix_trans(h0);
          pb[nt][1] = movmatrix_trans(h1);
          pbl[nt][0] = movmatrix_trans(l0);
          pbl[nt][1] = movmatrix_trans(l1);
        } else {
          pb[nt][0] = movmatrix_trans(M::pack(p[0], p[1]));
          pb[nt][1] = movmatrix_trans(M::pack(p[2], p[3]));
        }
      }
      // the running max settles after a few pages: rescale only when it moved
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int mt = 0; mt < Sh::kMTiles; ++mt) {
            o[nt][mt][0] *= al[nt][0];
            o[nt][mt][1] *= al[nt][1];
            o[nt][mt][2] *= al[nt][0];
            o[nt][mt][3] *= al[nt][1];
          }
      }
      // ---- O^T += V^T P^T, one m-tile per 16 columns of head_dim
#pragma unroll
      for (int mt = 0; mt < Sh::kMTiles; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(vt + (mt >> 2) * kBoxBytes + v_off[mt & 3], a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          M::run(o[nt][mt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
          if constexpr (kExactP) M::run(o[nt][mt], a0, a1, a2, a3, pbl[nt][0], pbl[nt][1]);
        }
      }
    }
    __syncwarp();
    // A unit's last element: its data slot (8 KB, 4 KB for head_dim 64) holds
    // this warp's exchange rows until the unit epilogue is done; the warp's next
    // load into that slot is only issued in the next iteration.
    if (md.last) {
      // ---- this warp is done with the unit: publish its state, then combine
      Unit u;
      u.b = md.b;
      u.s = md.s;
      u.kvh = md.kvh;
      u.hg = md.hg;
      u.nsplit = md.nsplit;
      u.gcount = md.gcount;
      u.qh0 = md.qh0;
      const int xr = a.GR;
      // padded rows when they fit in the slot (fewer bank conflicts), else dense
      const int xd = (a.GR * (D + 4) * 4 <= Sh::kSlot) ? D + 4 : D;
      float *xo = reinterpret_cast<float *>(tiles + (size_t)slot * Sh::kSlot);
      if (lane == 0) xslot[cw] = slot;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float ls = l[nt][j];
          ls += __shfl_xor_sync(0xffffffffu, ls, 4);
          ls += __shfl_xor_sync(0xffffffffu, ls, 8);
          ls += __shfl_xor_sync(0xffffffffu, ls, 16);
          const int h = 8 * nt + 2 * fq + j;
          if (fr == 0 && h < u.gcount) {
            xm[cw * xr + h] = m[nt][j];
            xl[cw * xr + h] = ls;
          }
        }
        const int h0 = 8 * nt + 2 * fq;
#pragma unroll
        for (int mt = 0; mt < Sh::kMTiles; ++mt) {
          const int d = 16 * mt + fr;
          if (h0 < u.gcount) {
            xo[h0 * xd + d] = o[nt][mt][0];
            xo[h0 * xd + d + 8] = o[nt][mt][2];
          }
          if (h0 + 1 < u.gcount) {
            xo[(h0 + 1) * xd + d] = o[nt][mt][1];
            xo[(h0 + 1) * xd + d + 8] = o[nt][mt][3];
          }
        }
      }
      if (!sync()) {
        cp_async_wait_all();
        return;
      }
      // ---- combine the NW warps' states (same arithmetic as unit_epilogue):
      // thread t owns query row g = t / (D/4) and columns 4c..4c+3, c = t % (D/4),
      // so the exchange reads and the output stores are 16 bytes wide and a
      // row's scale factors are computed once per thread for four columns
      constexpr int kC4 = D / 4;
      constexpr int kRowsPerPass = NW * 32 / kC4;
      const int c4 = tid % kC4;
      {
        const float *xw[NW];  // each warp's exchange rows
#pragma unroll
        for (int w = 0; w < NW; ++w)
          xw[w] = reinterpret_cast<const float *>(tiles + (size_t)xslot[w] * Sh::kSlot) + 4 * c4;
        for (int g = tid / kC4; g < u.gcount; g += kRowsPerPass) {
          float M = -INFINITY;
#pragma unroll
          for (int w = 0; w < NW; ++w) M = fmaxf(M, xm[w * xr + g]);
          float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
          float Ls = 0.f;
          if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
              const float f = exp2_or_zero(xm[w * xr + g] - M);
              Ls += f * xl[w * xr + g];
              const float4 x = *reinterpret_cast<const float4 *>(xw[w] + g * xd);
              O.x += f * x.x;
              O.y += f * x.y;
              O.z += f * x.z;
              O.w += f * x.w;
            }
          }
          if (u.nsplit == 1) {
            const float inv = 1.f / fmaxf(Ls, 1e-6f);
            const float4 r = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
            const int64_t op = u.b * a.o0 + (int64_t)(u.qh0 + g) * a.o1;
            if (a.out_vec) {
              store_out4(a, op + 4 * c4, r);
            } else {
              store_out(a, op + (4 * c4 + 0) * a.o2, r.x);
              store_out(a, op + (4 * c4 + 1) * a.o2, r.y);
              store_out(a, op + (4 * c4 + 2) * a.o2, r.z);
              store_out(a, op + (4 * c4 + 3) * a.o2, r.w);
            }
          } else {  // one split of several: merged by the last split to finish
            float *part = a.partials +
                          ((int64_t)md.split_row * a.upi + u.kvh * a.HG + u.hg) * a.part_floats;
            *reinterpret_cast<float4 *>(part + a.part_o + g * D + 4 * c4) = O;
            if (c4 == 0) {
              part[g] = M;
              part[a.GR + g] = Ls;
            }
          }
        }
      }
      // the partial is visible to every CTA before this unit counts itself in
      if (u.nsplit > 1) __threadfence();
      if (!sync()) {
        cp_async_wait_all();
        return;
      }
      // every consumer warp has read the unit's query rows and all exchange
      // rows: the query slot may be refilled
      if (tid == 0) mbar_arrive(&qempty[md.qslot]);
      if (u.nsplit > 1) {
        // ---- split-K merge by the last of the sequence's splits to finish:
        // the splits' partials combined in split order, the arithmetic of
        // merge_kernel (so the result does not depend on which split is last)
        int32_t *cnt = a.merge_cnt + (int64_t)u.b * a.upi + u.kvh * a.HG + u.hg;
        if (tid == 0) {
          __threadfence();
          const int32_t prev = atomicAdd(cnt, 1);
          const bool last = prev == u.nsplit - 1;
          if (last) *cnt = 0;  // all splits counted in: ready for the plan's next launch
          __threadfence();
          xslot[NW] = last ? 1 : 0;
        }
        if (!sync()) {
          cp_async_wait_all();
          return;
        }
        if (xslot[NW]) {
          const int64_t stride = (int64_t)a.upi * a.part_floats;  // next split of the unit
          const float *base = a.partials +
                              ((int64_t)(md.split_row - u.s) * a.upi + u.kvh * a.HG + u.hg) * a.part_floats;
          for (int g = tid / kC4; g < u.gcount; g += kRowsPerPass) {
            float M = -INFINITY;
            for (int32_t sp = 0; sp < u.nsplit; ++sp) M = fmaxf(M, __ldcg(base + sp * stride + g));
            float L = 0.f;
            float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
            if (M != -INFINITY) {
              for (int32_t sp = 0; sp < u.nsplit; ++sp) {
                const float *p = base + sp * stride;
                const float f = exp2_or_zero(__ldcg(p + g) - M);
                L += f * __ldcg(p + a.GR + g);
                const float4 x = __ldcg(reinterpret_cast<const float4 *>(p + a.part_o + g * D + 4 * c4));
                O.x += f * x.x;
                O.y += f * x.y;
                O.z += f * x.z;
                O.w += f * x.w;
              }
            }
            const float den = fmaxf(L, 1e-6f);
            const float4 r = make_float4(O.x / den, O.y / den, O.z / den, O.w / den);
            const int64_t op = u.b * a.o0 + (int64_t)(u.qh0 + g) * a.o1;
            if (a.out_vec) {
              store_out4(a, op + 4 * c4, r);
            } else {
              store_out(a, op + (4 * c4 + 0) * a.o2, r.x);
              store_out(a, op + (4 * c4 + 1) * a.o2, r.y);
              store_out(a, op + (4 * c4 + 2) * a.o2, r.z);
              store_out(a, op + (4 * c4 + 3) * a.o2, r.w);
            }
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        m[nt][0] = m[nt][1] = -INFINITY;
        l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
        for (int i = 0; i < Sh::kMTiles; ++i) o[nt][i][0] = o[nt][i][1] = o[nt][i][2] = o[nt][i][3] = 0.f;
      }
    }
  }
  cp_async_wait_all();
}

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
int device_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return 148;  // B200
  }
  return sms;
}


// Default pages per split: the P in {8, 16, ..., 512} with the smallest
// estimated launch time, assuming every sequence is max_blocks pages long (the
// host does not see the lengths). With U units on `sms` persistent CTAs the
// launch takes ceil(U / sms) rounds; a round costs its unit's pages plus a
// fixed unit overhead (the cross-warp combine and pipeline refill, measured on
// B200 at about 16 pages' worth of streaming), and any splitting adds the merge
// launch (about 32 pages' worth). This keeps whole sequences in one unit when
// there are enough of them to fill the GPU (config 3: 64 pages, 31 us per layer
// vs 68 us with 8-page splits; config 5: 256 pages, 89% vs 85% of HBM peak
// with 152) and splits just enough to fill every SM when there are few.
int32_t resolve_pps(int32_t B, int32_t Hq, int32_t Hkv, int32_t D, int32_t max_blocks,
                    int32_t pps) {
  if (pps > 0) return pps < kMaxPagesPerSplit ? pps : kMaxPagesPerSplit;
  const int32_t G = Hq / Hkv;
  const int32_t rows = group_rows_for(G, D);
  const int64_t u0 = std::max<int64_t>(1, (int64_t)B * Hkv * ((G + rows - 1) / rows));
  const int64_t mb = std::max<int32_t>(max_blocks, 1);
  const int64_t sms = device_sms();
  int64_t best_cost = INT64_MAX;
  int32_t best = kMaxPagesPerSplit;
  for (int32_t P = 8; P <= kMaxPagesPerSplit; P += 8) {
    const int64_t per = (mb + P - 1) / P;
    const int64_t rounds = (u0 * per + sms - 1) / sms;
    const int64_t cost = rounds * (std::min<int64_t>(P, mb) + kUnitCost) + (per > 1 ? kMergeCost : 0);
    if (cost < best_cost) {
      best_cost = cost;
      best = P;
    }
  }
  return best;
}

// Range of split lengths a plan may use. An explicit pages_per_split fixes it.
// Otherwise it is resolve_pps's length, except for batches of at most
// kMaxSimSeqs sequences: there a few units more or less per CTA decide the
// launch time, and the host's assumption that every sequence is max_blocks
// long can be far off in either direction (ragged lengths), so the plan kernel
// picks the length in [lo, top] from the actual lengths by simulating its
// schedule. top = max_blocks rounded up to 8 (longer splits split nothing),
// at most kMaxPagesPerSplit; lo keeps the launch at no more than 16 rounds of
// units even if every sequence were max_blocks long, which also bounds the
// workspace (sized for lo).
struct SplitRange {
  int32_t lo, hi;
};

SplitRange resolve_split(int32_t B, int32_t Hq, int32_t Hkv, int32_t D, int32_t max_blocks, int32_t pps) {
  const int32_t hi = resolve_pps(B, Hq, Hkv, D, max_blocks, pps);
  if (pps > 0 || max_blocks <= 8) return {hi, hi};
  const int32_t G = Hq / Hkv;
  const int32_t rows = group_rows_for(G, D);
  const int64_t u0 = std::max<int64_t>(1, (int64_t)B * Hkv * ((G + rows - 1) / rows));
  const int64_t sms = device_sms();
  if (B > kMaxSimSeqs) return {hi, hi};
  // no split needed and at least one unit per SM: splitting can only add
  // units and merges (and the simulation costs plan time), so keep hi
  if (hi >= max_blocks && u0 >= sms) return {hi, hi};
  const int32_t top = std::min<int32_t>(kMaxPagesPerSplit, (max_blocks + 7) / 8 * 8);
  int64_t lo = ((int64_t)max_blocks * u0 + 16 * sms - 1) / (16 * sms);
  lo = (lo + 7) / 8 * 8;
  // at most kMaxSplitCandidates multiples of 8 up to the top
  lo = std::max<int64_t>({8, lo, (int64_t)top - 8 * (kMaxSplitCandidates - 1)});
  if (lo >= top) return {hi, hi};
  return {(int32_t)lo, top};
}

// The tensor-core kernel copies whole (page, head) slabs of 16 x D 16-bit
// values with 16-byte cp.async: rows must be contiguous and every slab
// 16-byte aligned.
bool tc_eligible(const void *k_cache, const void *v_cache, int32_t Hq, int32_t Hkv, int32_t D,
                 int32_t bs, const int64_t *cs, int32_t q_dtype, int32_t kv_dtype, int32_t flags) {
  if (flags & PKV_DECODE_FORCE_GENERIC) return false;
  if (kv_dtype != PKV_DTYPE_BF16 && kv_dtype != PKV_DTYPE_F16) return false;
  if (q_dtype != kv_dtype) return false;
  if (bs != kBoxRows || (D != 64 && D != 128)) return false;
  if (Hq % Hkv != 0) return false;
  if (cs[3] != 1 || cs[2] != D) return false;
  if (cs[0] % 8 != 0 || cs[1] % 8 != 0 || cs[0] <= 0 || cs[1] <= 0) return false;
  if (!aligned_to(k_cache, 16) || (v_cache != nullptr && !aligned_to(v_cache, 16))) return false;
  return true;
}

int validate_decode(const void *q, const void *kc, const void *vc, const int32_t *bt,
                    const int32_t *ctx, const float *out, int32_t B, int32_t Hq, int32_t Hkv,
                    int32_t D, int32_t bs, int32_t num_blocks, int32_t max_blocks,
                    const int64_t *qs, const int64_t *cs, const int64_t *bts, const int64_t *os,
                    int32_t q_dtype, int32_t kv_dtype) {
  if (dtype_size(q_dtype) == 0 || dtype_size(kv_dtype) == 0) {
    set_error_detail("unsupported dtype codes q=%d kv=%d", q_dtype, kv_dtype);
    return PKV_ERR_UNSUPPORTED;
  }
  if (B < 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || bs <= 0 || num_blocks < 0 || max_blocks < 0) {
    set_error_detail("invalid sizes");
    return PKV_ERR_INVALID_ARG;
  }
  if (Hq % Hkv != 0) {
    set_error_detail("num_q_heads (%d) must be a multiple of num_kv_heads (%d)", Hq, Hkv);
    return PKV_ERR_INVALID_ARG;
  }
  if (D > 256) {
    set_error_detail("head_dim %d > 256 is not supported", D);
    return PKV_ERR_UNSUPPORTED;
  }
  if ((int64_t)max_blocks * bs > INT32_MAX) {
    set_error_detail("max_blocks * block_size overflows int32");
    return PKV_ERR_INVALID_ARG;
  }
  if (!qs || !cs || !bts || !os) {
    set_error_detail("stride arrays must not be NULL");
    return PKV_ERR_INVALID_ARG;
  }
  if (B > 0 && (!q || !kc || !vc || !bt || !ctx || !out)) {
    set_error_detail("NULL tensor pointer");
    return PKV_ERR_INVALID_ARG;
  }
  if (B > 0 && (!aligned_to(q, dtype_size(q_dtype)) || !aligned_to(kc, dtype_size(kv_dtype)) ||
                !aligned_to(vc, dtype_size(kv_dtype)) || !aligned_to(out, 4)))
    return PKV_ERR_ALIGNMENT;
  return PKV_OK;
}

template <typename KT, int DJ, int GM>
int launch_generic_t(const DecodeArgs &a, cudaStream_t st, int64_t max_units) {
  const size_t smem = generic_smem_bytes(DJ, GM);
  auto kern = decode_generic_kernel<KT, DJ, GM>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return check_launch("cudaFuncSetAttribute(generic)");
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGenThreads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  int64_t grid = (int64_t)device_sms() * per_sm;
  if (grid > max_units) grid = max_units;
  if (grid < 1) grid = 1;
  kern<<<(unsigned)grid, kGenThreads, smem, st>>>(a);
  return check_launch("decode_generic_kernel");
}

template <typename KT, int DJ>
int launch_generic_g(const DecodeArgs &a, cudaStream_t st, int64_t max_units) {
  if (a.GR <= 2) return launch_generic_t<KT, DJ, 2>(a, st, max_units);
  if (a.GR <= 4) return launch_generic_t<KT, DJ, 4>(a, st, max_units);
  if (a.GR <= 8) return launch_generic_t<KT, DJ, 8>(a, st, max_units);
  if constexpr (DJ <= 4) return launch_generic_t<KT, DJ, 16>(a, st, max_units);
  set_error_detail("head group of %d rows with head_dim %d is not supported", a.GR, a.D);
  return PKV_ERR_UNSUPPORTED;
}

template <typename KT>
int launch_generic_d(const DecodeArgs &a, cudaStream_t st, int64_t max_units) {
  if (a.D <= 32) return launch_generic_g<KT, 1>(a, st, max_units);
  if (a.D <= 64) return launch_generic_g<KT, 2>(a, st, max_units);
  if (a.D <= 128) return launch_generic_g<KT, 4>(a, st, max_units);
  return launch_generic_g<KT, 8>(a, st, max_units);
}

// Tensor-core kernel configuration: consumer warps and a per-warp ring of S
// pages. head_dim 128 without RoPE (158 registers for one head tile): 9
// consumer warps x 2 x 8 KB = 144 KB of K/V staging; measured on B200 against
// 7 x 3, 8 x 3 and 11 x 2 it is the fastest (config 4 694 us per layer vs 704
// for 7 x 3, config 5 292 vs 295, their 8-GPU shards 1.5-2% faster, config 3
// unchanged). With RoPE in the producer the kernel takes 218 registers, which
// leaves room for 7 consumer warps (+ the producer: two warps per SM
// sub-partition) x 3 x 8 KB = 168 KB. head_dim 64: 8 x 6 x 4 KB.
template <typename T, int D, bool kExactP, int NT, bool kRope>
int launch_tc_x(const DecodeArgs &a, cudaStream_t st, int64_t max_units) {
  constexpr int kTcWarps = D == 128 ? (kRope ? 7 : 9) : 8;
  constexpr int S = D == 128 ? (kRope ? 3 : 2) : 6;
  using L = TcSmem<D, kTcWarps, S>;
  static_assert(L::kBt + sizeof(int32_t) * kMaxPagesPerSplit + 1024 <= 227 * 1024,
                "tensor-core decode exceeds the 227 KB of shared memory per CTA");
  const size_t smem = L::bytes(a.P);
  auto kern = decode_tc_kernel<T, D, kTcWarps, S, kExactP, NT, kRope>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return check_launch("cudaFuncSetAttribute(tc)");
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (kTcWarps + 1) * 32, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  int64_t grid = (int64_t)device_sms() * per_sm;
  if (grid > max_units) grid = max_units;
  if (grid < 1) grid = 1;
  // launched with programmatic stream serialization: its CTAs may become
  // resident while the previous kernel finishes (the kernel waits for it)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((kTcWarps + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return check_launch("decode_tc_kernel");
  return check_launch("decode_tc_kernel");
}

template <typename T, int D, bool kRope>
int launch_tc_r(const DecodeArgs &a, cudaStream_t st, int64_t max_units, int32_t flags) {
  // query heads of a head group: up to 8 in one MMA n-tile, up to 16 in two
  const bool two = a.GR > 8;
  if (flags & PKV_DECODE_EXACT_P)
    return two ? launch_tc_x<T, D, true, 2, kRope>(a, st, max_units)
               : launch_tc_x<T, D, true, 1, kRope>(a, st, max_units);
  return two ? launch_tc_x<T, D, false, 2, kRope>(a, st, max_units)
             : launch_tc_x<T, D, false, 1, kRope>(a, st, max_units);
}

template <typename T, int D>
int launch_tc_t(const DecodeArgs &a, cudaStream_t st, int64_t max_units, int32_t flags) {
  return a.rcos != nullptr ? launch_tc_r<T, D, true>(a, st, max_units, flags)
                           : launch_tc_r<T, D, false>(a, st, max_units, flags);
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int32_t pkv_decode_pages_per_split(int32_t batch, int32_t num_q_heads,
                                              int32_t num_kv_heads, int32_t head_dim,
                                              int32_t max_blocks, int32_t pages_per_split) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_blocks < 0 ||
      num_q_heads % num_kv_heads != 0)
    return PKV_ERR_INVALID_ARG;
  return resolve_pps(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pages_per_split);
}

extern "C" size_t pkv_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                            int32_t num_kv_heads, int32_t head_dim,
                                            int32_t max_blocks, int32_t pages_per_split) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_blocks < 0 ||
      num_q_heads % num_kv_heads != 0)
    return 0;
  const SplitRange r =
      resolve_split(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pages_per_split);
  return ws_layout(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, r.lo).total;
}

extern "C" int pkv_decode_kernel_kind(const void *k_cache, int32_t num_q_heads,
                                      int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                      const int64_t *cache_strides, int32_t q_dtype,
                                      int32_t kv_dtype, int32_t flags) {
  if (!cache_strides || num_kv_heads <= 0) return PKV_ERR_INVALID_ARG;
  return tc_eligible(k_cache, nullptr, num_q_heads, num_kv_heads, head_dim, block_size,
                     cache_strides, q_dtype, kv_dtype, flags)
             ? 1
             : 0;
}

extern "C" int pkv_decode_plan(const int32_t *context_lens, int32_t batch, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int32_t max_blocks, int32_t pages_per_split, void *workspace,
                               size_t workspace_bytes, int32_t *status, void *stream) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      max_blocks < 0 || num_q_heads % num_kv_heads != 0) {
    set_error_detail("pkv_decode_plan: invalid sizes");
    return PKV_ERR_INVALID_ARG;
  }
  if ((int64_t)max_blocks * block_size > INT32_MAX) {
    set_error_detail("max_blocks * block_size overflows int32");
    return PKV_ERR_INVALID_ARG;
  }
  const SplitRange r =
      resolve_split(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pages_per_split);
  const WsLayout w = ws_layout(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, r.lo);
  if (workspace == nullptr || workspace_bytes < w.total || !aligned_to(workspace, 256)) {
    set_error_detail("workspace needs %zu bytes (256-byte aligned), got %zu", w.total,
                     workspace_bytes);
    return PKV_ERR_WORKSPACE;
  }
  if (batch > 0 && context_lens == nullptr) {
    set_error_detail("pkv_decode_plan: NULL context_lens");
    return PKV_ERR_INVALID_ARG;
  }
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  plan_kernel<<<1, kPlanThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      context_lens, batch, block_size, max_blocks, r.lo, r.hi,
      (int32_t)std::min<int64_t>(device_sms(), w.max_items * w.units_per_item), w.units_per_item,
      reinterpret_cast<int32_t *>(ws + w.hdr), reinterpret_cast<int32_t *>(ws + w.seq_off),
      reinterpret_cast<int32_t *>(ws + w.seq_nsplit), reinterpret_cast<int32_t *>(ws + w.merge_cnt),
      reinterpret_cast<int4 *>(ws + w.items), status);
  return check_launch("plan_kernel");
}

namespace {

// pkv_decode_run, optionally with the fused append of k_new / v_new (kn != nullptr).
int decode_run_impl(const void *q, const void *kn, const void *vn, const void *k_cache,
                    const void *v_cache, const int32_t *block_tables, const int32_t *context_lens,
                    float *out, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                    const int64_t *q_strides, const int64_t *new_strides,
                    const int64_t *cache_strides, const int64_t *bt_strides,
                    const int64_t *out_strides, int32_t q_dtype, int32_t kv_dtype, float scale,
                    int32_t pages_per_split, int32_t flags, void *workspace,
                    size_t workspace_bytes, int32_t *status, void *stream,
                    const void *rope_cos = nullptr, const void *rope_sin = nullptr,
                    int64_t rope_stride = 0) {
  int rc = validate_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                           num_q_heads, num_kv_heads, head_dim, block_size, num_blocks,
                           max_blocks, q_strides, cache_strides, bt_strides, out_strides, q_dtype,
                           kv_dtype);
  if (rc) return rc;
  if (kn != nullptr || vn != nullptr) {
    if (new_strides == nullptr) {
      set_error_detail("new_strides must not be NULL");
      return PKV_ERR_INVALID_ARG;
    }
    if (batch > 0 && (kn == nullptr || vn == nullptr)) {
      set_error_detail("k_new and v_new must both be given");
      return PKV_ERR_INVALID_ARG;
    }
    if (batch > 0 && (!aligned_to(kn, dtype_size(kv_dtype)) || !aligned_to(vn, dtype_size(kv_dtype))))
      return PKV_ERR_ALIGNMENT;
  }
  if (batch == 0) return PKV_OK;
  const SplitRange r =
      resolve_split(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pages_per_split);
  const WsLayout w = ws_layout(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, r.lo);
  if (workspace == nullptr || workspace_bytes < w.total || !aligned_to(workspace, 256)) {
    set_error_detail("workspace needs %zu bytes (256-byte aligned), got %zu", w.total,
                     workspace_bytes);
    return PKV_ERR_WORKSPACE;
  }
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  DecodeArgs a{};
  a.q = q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.bt = block_tables;
  a.ctx = context_lens;
  a.out = out;
  a.B = batch;
  a.Hq = num_q_heads;
  a.Hkv = num_kv_heads;
  a.G = num_q_heads / num_kv_heads;
  a.GR = w.group_rows;
  a.HG = (a.G + a.GR - 1) / a.GR;
  a.D = head_dim;
  a.bs = block_size;
  a.num_blocks = num_blocks;
  a.max_blocks = max_blocks;
  a.P = r.hi;
  a.upi = w.units_per_item;
  a.part_o = w.part_o;
  a.part_floats = w.part_floats;
  a.q_dtype = q_dtype;
  a.kv_dtype = kv_dtype;
  a.q0 = q_strides[0]; a.q1 = q_strides[1]; a.q2 = q_strides[2];
  a.q_vec = (a.q2 == 1 && a.q0 % 8 == 0 && a.q1 % 8 == 0 && aligned_to(q, 16)) ? 1 : 0;
  a.c0 = cache_strides[0]; a.c1 = cache_strides[1]; a.c2 = cache_strides[2]; a.c3 = cache_strides[3];
  a.bt0 = bt_strides[0]; a.bt1 = bt_strides[1];
  a.o0 = out_strides[0]; a.o1 = out_strides[1]; a.o2 = out_strides[2];
  a.out16 = (flags & PKV_DECODE_OUT_Q_DTYPE) ? (q_dtype == PKV_DTYPE_BF16 ? 1 : q_dtype == PKV_DTYPE_F16 ? 2 : 0) : 0;
  a.out_vec = (a.o2 == 1 && a.o0 % 4 == 0 && a.o1 % 4 == 0 && aligned_to(out, a.out16 ? 8 : 16)) ? 1 : 0;
  a.scale = scale;
  a.scale_log2 = scale * kLog2e;
  a.hdr = reinterpret_cast<const int32_t *>(ws + w.hdr);
  a.seq_off = reinterpret_cast<const int32_t *>(ws + w.seq_off);
  a.seq_nsplit = reinterpret_cast<const int32_t *>(ws + w.seq_nsplit);
  a.items = reinterpret_cast<const int4 *>(ws + w.items);
  a.max_items = w.max_items;
  a.partials = reinterpret_cast<float *>(ws + w.partials);
  a.merge_cnt = reinterpret_cast<int32_t *>(ws + w.merge_cnt);
  a.sched = reinterpret_cast<int32_t *>(ws + w.hdr) + 4;
  a.status = status;
  a.max_polls = kMaxPolls;
  a.max_tries = kMaxWaitTries;
  if (flags & PKV_DECODE_TEST_WAIT_TIMEOUT) {
    // a few thousand polls (well under a millisecond) instead of seconds, and
    // one element withheld, so the launch ends by its wait limits
    a.max_polls = kTestWaitPolls;
    a.max_tries = kTestWaitPolls;
    a.withhold = 1;
  }
  a.early = (flags & PKV_DECODE_EARLY_START) ? 1 : 0;
  const int64_t max_units = w.max_items * w.units_per_item;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool tc = tc_eligible(k_cache, v_cache, num_q_heads, num_kv_heads, head_dim, block_size,
                              cache_strides, q_dtype, kv_dtype, flags);
  if (rope_cos != nullptr) {
    // RoPE in the producer: the tensor-core kernel with 16-byte query and new
    // rows and 16-byte cos / sin rows, nothing else
    const bool rope_ok = kn != nullptr && rope_sin != nullptr && tc && q_dtype == kv_dtype && a.q_vec &&
                         new_strides[2] == 1 && new_strides[0] % 8 == 0 && new_strides[1] % 8 == 0 &&
                         aligned_to(kn, 16) && aligned_to(vn, 16) && rope_stride >= head_dim &&
                         rope_stride % 8 == 0 && aligned_to(rope_cos, 16) && aligned_to(rope_sin, 16);
    if (!rope_ok) {
      set_error_detail("RoPE in the decode needs the tensor-core kernel (16-bit q and cache of one dtype), "
                       "16-byte aligned contiguous q and new rows, and 16-byte aligned cos / sin rows");
      return PKV_ERR_UNSUPPORTED;
    }
    a.rcos = rope_cos;
    a.rsin = rope_sin;
    a.rcs = rope_stride;
  }
  if (kn != nullptr) {
    // the tensor-core kernel takes the new token rows as 16-byte vectors;
    // anything else appends with the append kernel first (slot = length - 1)
    if (tc && new_strides[2] == 1 && new_strides[0] % 8 == 0 && new_strides[1] % 8 == 0 &&
        aligned_to(kn, 16) && aligned_to(vn, 16)) {
      a.kn = kn;
      a.vn = vn;
      a.n0 = new_strides[0];
      a.n1 = new_strides[1];
    } else {
      rc = append_launch(kn, vn, const_cast<void *>(k_cache), const_cast<void *>(v_cache),
                         block_tables, context_lens, -1, batch, num_kv_heads, head_dim,
                         block_size, num_blocks, max_blocks, new_strides, cache_strides,
                         bt_strides, kv_dtype, status, stream);
      if (rc) return rc;
    }
  }

  if (tc) {
    if (kv_dtype == PKV_DTYPE_BF16)
      rc = head_dim == 128 ? launch_tc_t<__nv_bfloat16, 128>(a, st, max_units, flags)
                           : launch_tc_t<__nv_bfloat16, 64>(a, st, max_units, flags);
    else
      rc = head_dim == 128 ? launch_tc_t<__half, 128>(a, st, max_units, flags)
                           : launch_tc_t<__half, 64>(a, st, max_units, flags);
  } else {
    switch (kv_dtype) {
      case PKV_DTYPE_BF16: rc = launch_generic_d<__nv_bfloat16>(a, st, max_units); break;
      case PKV_DTYPE_F16: rc = launch_generic_d<__half>(a, st, max_units); break;
      default: rc = launch_generic_d<float>(a, st, max_units); break;
    }
  }
  if (rc) return rc;
  // the CUDA-core kernel leaves the partials of split sequences to the merge
  // kernel (stream-ordered); the tensor-core kernel merges them itself
  if (!tc && max_blocks > r.lo) {
    if (w.units_per_item > 65535) {
      set_error_detail("num_kv_heads x head groups = %d exceeds the merge grid", w.units_per_item);
      return PKV_ERR_UNSUPPORTED;
    }
    merge_kernel<<<dim3((unsigned)batch, (unsigned)w.units_per_item), kMergeThreads, 0, st>>>(a);
    rc = check_launch("merge_kernel");
  }
  return rc;
}

}  // namespace

extern "C" int pkv_decode_run(const void *q, const void *k_cache, const void *v_cache,
                              const int32_t *block_tables, const int32_t *context_lens,
                              float *out, int32_t batch, int32_t num_q_heads,
                              int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                              int32_t num_blocks, int32_t max_blocks, const int64_t *q_strides,
                              const int64_t *cache_strides, const int64_t *bt_strides,
                              const int64_t *out_strides, int32_t q_dtype, int32_t kv_dtype,
                              float scale, int32_t pages_per_split, int32_t flags,
                              void *workspace, size_t workspace_bytes, int32_t *status,
                              void *stream) {
  return decode_run_impl(q, nullptr, nullptr, k_cache, v_cache, block_tables, context_lens, out,
                         batch, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks,
                         max_blocks, q_strides, nullptr, cache_strides, bt_strides, out_strides,
                         q_dtype, kv_dtype, scale, pages_per_split, flags, workspace,
                         workspace_bytes, status, stream);
}

extern "C" int pkv_append_decode_run(const void *q, const void *k_new, const void *v_new,
                                     void *k_cache, void *v_cache, const int32_t *block_tables,
                                     const int32_t *context_lens, float *out, int32_t batch,
                                     int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                     int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                                     const int64_t *q_strides, const int64_t *new_strides,
                                     const int64_t *cache_strides, const int64_t *bt_strides,
                                     const int64_t *out_strides, int32_t q_dtype,
                                     int32_t kv_dtype, float scale, int32_t pages_per_split,
                                     int32_t flags, void *workspace, size_t workspace_bytes,
                                     int32_t *status, void *stream) {
  if (batch > 0 && (k_new == nullptr || v_new == nullptr)) {
    set_error_detail("pkv_append_decode_run: k_new and v_new must not be NULL");
    return PKV_ERR_INVALID_ARG;
  }
  return decode_run_impl(q, k_new, v_new, k_cache, v_cache, block_tables, context_lens, out,
                         batch, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks,
                         max_blocks, q_strides, new_strides, cache_strides, bt_strides,
                         out_strides, q_dtype, kv_dtype, scale, pages_per_split, flags,
                         workspace, workspace_bytes, status, stream);
}

extern "C" int pkv_rope_append_decode_run(
    const void *q, const void *k_new, const void *v_new, const void *rope_cos, const void *rope_sin,
    int64_t rope_stride, void *k_cache, void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, float *out, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t block_size, int32_t num_blocks, int32_t max_blocks,
    const int64_t *q_strides, const int64_t *new_strides, const int64_t *cache_strides,
    const int64_t *bt_strides, const int64_t *out_strides, int32_t q_dtype, int32_t kv_dtype, float scale,
    int32_t pages_per_split, int32_t flags, void *workspace, size_t workspace_bytes, int32_t *status,
    void *stream) {
  if (batch > 0 && (k_new == nullptr || v_new == nullptr || rope_cos == nullptr || rope_sin == nullptr)) {
    set_error_detail("pkv_rope_append_decode_run: k_new, v_new, cos and sin must not be NULL");
    return PKV_ERR_INVALID_ARG;
  }
  if (batch == 0) return PKV_OK;
  return decode_run_impl(q, k_new, v_new, k_cache, v_cache, block_tables, context_lens, out, batch,
                         num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, max_blocks,
                         q_strides, new_strides, cache_strides, bt_strides, out_strides, q_dtype,
                         kv_dtype, scale, pages_per_split, flags, workspace, workspace_bytes, status,
                         stream, rope_cos, rope_sin, rope_stride);
}

extern "C" int pkv_decode(const void *q, const void *k_cache, const void *v_cache,
                          const int32_t *block_tables, const int32_t *context_lens, float *out,
                          int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                          int32_t head_dim, int32_t block_size, int32_t num_blocks,
                          int32_t max_blocks, const int64_t *q_strides,
                          const int64_t *cache_strides, const int64_t *bt_strides,
                          const int64_t *out_strides, int32_t q_dtype, int32_t kv_dtype,
                          float scale, int32_t pages_per_split, int32_t flags, void *workspace,
                          size_t workspace_bytes, int32_t *status, void *stream) {
  int rc = validate_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                           num_q_heads, num_kv_heads, head_dim, block_size, num_blocks,
                           max_blocks, q_strides, cache_strides, bt_strides, out_strides, q_dtype,
                           kv_dtype);
  if (rc) return rc;
  if (batch == 0) return PKV_OK;
  rc = pkv_decode_plan(context_lens, batch, num_q_heads, num_kv_heads, head_dim, block_size,
                       max_blocks, pages_per_split, workspace, workspace_bytes, status, stream);
  if (rc) return rc;
  return pkv_decode_run(q, k_cache, v_cache, block_tables, context_lens, out, batch, num_q_heads,
                        num_kv_heads, head_dim, block_size, num_blocks, max_blocks, q_strides,
                        cache_strides, bt_strides, out_strides, q_dtype, kv_dtype, scale,
                        pages_per_split, flags, workspace, workspace_bytes, status, stream);
}
