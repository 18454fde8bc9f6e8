// Pieces shared by the decode kernels: arguments, workspace layout, the
// split-KV work plan every CTA derives from context_lens, and the last-CTA
// log-sum-exp combine of split partials.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace b200kv {

constexpr int kMaxBatch = 1024;
constexpr int kMaxWorkItems = 8192;
constexpr int kDefaultItemsPerCta = 4;
// The completion counters always occupy the same fixed-size region at the
// start of the workspace, whatever the call's shape, so a workspace shared by
// calls of different shapes never sees partials where counters are expected.
constexpr int64_t kMaxCounters = 131072;  // batch * num_kv_heads limit
constexpr float kLn2 = 0.69314718055994530942f;

struct DecodeArgs {
  const __half *q;
  int64_t q_sb, q_sh;
  const int32_t *block_table;
  int64_t bt_stride;
  const int32_t *ctx_lens;
  __half *out;
  int64_t o_sb, o_sh;
  float *lse;
  int batch, hkv, hq, max_blocks;
  int64_t num_blocks;
  float scale_log2;  // scale * log2(e)
  int target_items;
  int *counters;     // [batch * hkv] completion tickets, zero between calls
  float2 *part_ml;   // [slots][G] (max in log2 units, sum of exp2)
  float *part_o;     // [slots][G][128] unnormalised partial outputs
  int32_t *error_flag;
};

struct WorkspaceLayout {
  int64_t counters_off, ml_off, o_off, total;
};

inline WorkspaceLayout workspace_layout(int64_t batch, int64_t hq, int64_t hkv) {
  const int64_t g = hq / hkv;
  const int64_t slots = kMaxWorkItems + batch * hkv;
  auto up = [](int64_t x) { return (x + 255) & ~int64_t(255); };
  WorkspaceLayout w;
  w.counters_off = 0;
  w.ml_off = up(kMaxCounters * 4);
  w.o_off = up(w.ml_off + slots * g * 8);
  w.total = up(w.o_off + slots * g * kHeadDim * 4);
  return w;
}

// Shared-memory footprint of the plan (per-sequence pages, splits, clamped
// context length, item prefix, scratch).
constexpr int kPlanBytes = (4 * kMaxBatch + 1) * 4 + 64 * 4;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Pages of sequence b (its context length clamped to the block table).
__device__ __forceinline__ int clamped_ctx(const DecodeArgs &a, int b, bool flag_errors) {
  int ctx = __ldg(a.ctx_lens + b);
  const int cap = a.max_blocks * kPageTokens;
  if (ctx < 0 || ctx > cap) {
    if (flag_errors && a.error_flag) atomicOr(a.error_flag, B200KV_DEVERR_BAD_LEN);
    ctx = ctx < 0 ? 0 : cap;
  }
  return ctx;
}

struct Plan {
  int *nb;       // [batch] pages per sequence
  int *splits;   // [batch] splits per sequence
  int *ctx;      // [batch] context length clamped to the block table
  int *prefix;   // [batch + 1] first item of each sequence (b-major, then kv head)
  int *scratch;  // [64]
  int chunk;     // pages per split
  int total_items;
};

__device__ __forceinline__ Plan plan_view(uint8_t *base) {
  Plan p;
  p.nb = reinterpret_cast<int *>(base);
  p.splits = p.nb + kMaxBatch;
  p.ctx = p.splits + kMaxBatch;
  p.prefix = p.ctx + kMaxBatch;
  p.scratch = p.prefix + kMaxBatch + 1;
  p.chunk = 0;
  p.total_items = 0;
  return p;
}

// Every CTA derives the same split-KV partition from context_lens: the chunk
// C (pages per split) is the page-head count divided by the target number of
// work items; sequence b gets max(1, ceil(pages_b / C)) splits per KV head.
// All NT threads of the CTA must call this (it synchronises).
template <int NT>
__device__ __forceinline__ void build_plan(const DecodeArgs &a, Plan &p) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = NT / 32;
  int local_pages = 0;
  for (int b = tid; b < a.batch; b += NT) {
    const int ctx = clamped_ctx(a, b, blockIdx.x == 0);
    const int nb = (ctx + kPageTokens - 1) / kPageTokens;
    p.ctx[b] = ctx;
    p.nb[b] = nb;
    local_pages += nb;
  }
  {
    int v = local_pages;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    if (lane == 0) p.scratch[warp] = v;
  }
  __syncthreads();
  int total_pages = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) total_pages += p.scratch[w];
  const long long page_heads = static_cast<long long>(total_pages) * a.hkv;
  const int chunk = max(1, static_cast<int>((page_heads + a.target_items - 1) / a.target_items));
  constexpr int kPer = (kMaxBatch + NT - 1) / NT;
  int cnt[kPer];
  int run = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    int items = 0;
    if (b < a.batch) {
      const int ns = max(1, (p.nb[b] + chunk - 1) / chunk);
      p.splits[b] = ns;
      items = ns * a.hkv;
    }
    cnt[i] = run;
    run += items;
  }
  int incl = run;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, m);
    if (lane >= m) incl += y;
  }
  __syncthreads();  // page sums read; scratch reused below
  if (lane == 31) p.scratch[warp] = incl;
  __syncthreads();
  int warp_base = 0;
  for (int w = 0; w < warp; ++w) warp_base += p.scratch[w];
  const int thread_base = warp_base + incl - run;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    if (b < a.batch) p.prefix[b] = thread_base + cnt[i];
  }
  if (tid == NT - 1) p.prefix[a.batch] = thread_base + run;
  __syncthreads();
  p.chunk = chunk;
  p.total_items = p.prefix[a.batch];
}

struct Item {
  int b, kvh, split, nsplit, p, p_end, ctx;
};

// Work item `it` (b-major, then KV head, then split) of the plan.
__device__ __forceinline__ Item decode_item(const DecodeArgs &a, const Plan &pl, int it) {
  int lo = 0, hi = a.batch - 1;  // largest b with prefix[b] <= it
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pl.prefix[mid] <= it) lo = mid; else hi = mid - 1;
  }
  Item r;
  r.b = lo;
  r.nsplit = pl.splits[lo];
  const int rem = it - pl.prefix[lo];
  r.kvh = rem / r.nsplit;
  r.split = rem - r.kvh * r.nsplit;
  const int nb = pl.nb[lo];
  r.p = r.split * pl.chunk;
  r.p_end = min(r.p + pl.chunk, nb);
  if (r.p > r.p_end) r.p = r.p_end;
  r.ctx = pl.ctx[lo];
  return r;
}

// ---------------------------------------------------------------------------
// Balanced ("stream-K") partition used by the tensor-core kernel.
//
// The work is a sequence of units: (b, kv head) pairs in b-major order, pair j
// contributing w_b = max(pages_b, 1) units (an empty sequence still costs one
// unit so its zero output has an owner).  CTA c of the grid takes the units
// [c * per, (c + 1) * per), per = ceil(total / grid), so every CTA streams the
// same number of pages whatever the spread of context lengths.  A pair cut by
// CTA boundaries is a split: its piece in CTA c writes a partial to slot
// j + c (unique, and contiguous from j + c_lo for the pair's pieces), and the
// CTA that finishes last merges them.
// ---------------------------------------------------------------------------

// Fills pl.ctx / pl.nb and, in pl.prefix, the exclusive prefix over sequences
// of w_b; pl.total_items is set to the total number of units (all pairs).
template <int NT>
__device__ __forceinline__ void build_unit_plan(const DecodeArgs &a, Plan &p) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kPer = (kMaxBatch + NT - 1) / NT;
  int cnt[kPer];
  int run = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    int w = 0;
    if (b < a.batch) {
      const int ctx = clamped_ctx(a, b, blockIdx.x == 0);
      const int nb = (ctx + kPageTokens - 1) / kPageTokens;
      p.ctx[b] = ctx;
      p.nb[b] = nb;
      w = max(nb, 1);
    }
    cnt[i] = run;
    run += w;
  }
  int incl = run;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, m);
    if (lane >= m) incl += y;
  }
  if (lane == 31) p.scratch[warp] = incl;
  __syncthreads();
  int warp_base = 0;
  for (int w = 0; w < warp; ++w) warp_base += p.scratch[w];
  const int thread_base = warp_base + incl - run;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    if (b < a.batch) p.prefix[b] = thread_base + cnt[i];
  }
  if (tid == NT - 1) p.prefix[a.batch] = thread_base + run;
  __syncthreads();
  p.total_items = p.prefix[a.batch] * a.hkv;
  p.chunk = 0;
}

struct Seg {
  int b, kvh, pair;     // sequence, KV head, pair index b * Hkv + kvh
  int p, p_end, ctx;    // pages [p, p_end) of the pair streamed by this piece
  int nsplit, split;    // pieces of the pair, index of this one
  int first_slot, slot; // partial slots: pair's first, this piece's
  int u_next;           // first unit after this piece
};

// The piece of work that starts at unit u inside CTA c's range [.., u_end).
__device__ __forceinline__ Seg locate_seg(const DecodeArgs &a, const Plan &pl, int u, int u_end,
                                          int c, int per) {
  int lo = 0, hi = a.batch - 1;  // largest b whose first unit is <= u
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.hkv * pl.prefix[mid] <= u) lo = mid; else hi = mid - 1;
  }
  Seg s;
  s.b = lo;
  const int nb = pl.nb[lo];
  const int w = max(nb, 1);
  const int base = a.hkv * pl.prefix[lo];
  s.kvh = (u - base) / w;
  const int pj = base + s.kvh * w;  // first unit of the pair
  const int hi_u = min(u_end, pj + w);
  s.pair = lo * a.hkv + s.kvh;
  s.p = min(u - pj, nb);
  s.p_end = min(hi_u - pj, nb);
  s.ctx = pl.ctx[lo];
  const int c_lo = pj / per, c_hi = (pj + w - 1) / per;
  s.nsplit = c_hi - c_lo + 1;
  s.split = c - c_lo;
  s.first_slot = s.pair + c_lo;
  s.slot = s.pair + c;
  s.u_next = hi_u;
  return s;
}

// Block id of page p of sequence b, clamped into the pool (bad ids are
// flagged and replaced by block 0 so no transfer leaves the pool).
__device__ __forceinline__ int page_block(const DecodeArgs &a, int b, int p) {
  int blk = __ldg(a.block_table + static_cast<int64_t>(b) * a.bt_stride + p);
  if (blk < 0 || blk >= a.num_blocks) {
    if (a.error_flag) atomicOr(a.error_flag, B200KV_DEVERR_BAD_BLOCK);
    blk = 0;
  }
  return blk;
}

// Final output of (b, head h0 + g, d) from an unnormalised accumulator.
__device__ __forceinline__ void store_out(const DecodeArgs &a, int b, int h, int d, float acc,
                                          float l) {
  a.out[b * a.o_sb + h * a.o_sh + d] = __float2half_rn(l > 0.f ? acc / l : 0.f);
}
__device__ __forceinline__ void store_lse(const DecodeArgs &a, int b, int h, float m, float l) {
  if (a.lse)
    a.lse[static_cast<int64_t>(b) * a.hq + h] = l > 0.f ? (m + log2f(l)) * kLn2 : -CUDART_INF_F;
}

// Log-sum-exp merge of the nsplit partials of (b, kv head), run by the CTA
// that finished last.  Threads [0, NT) cover the G x 128 outputs.
template <int G, int NT>
__device__ __forceinline__ void combine_partials(const DecodeArgs &a, const Item &it, int first,
                                                 int tid) {
  const int h0 = it.kvh * G;
  for (int i = tid; i < G * kHeadDim; i += NT) {
    const int g = i / kHeadDim, d = i % kHeadDim;
    float mx = -CUDART_INF_F;
    for (int s = 0; s < it.nsplit; ++s)
      mx = fmaxf(mx, __ldcg(a.part_ml + static_cast<int64_t>(first + s) * G + g).x);
    float lsum = 0.f, acc = 0.f;
    for (int s = 0; s < it.nsplit; ++s) {
      const float2 ml = __ldcg(a.part_ml + static_cast<int64_t>(first + s) * G + g);
      const float w = ml.x == -CUDART_INF_F ? 0.f : exp2f(ml.x - mx);
      lsum = fmaf(ml.y, w, lsum);
      acc = fmaf(__ldcg(a.part_o + static_cast<int64_t>(first + s) * G * kHeadDim + i), w, acc);
    }
    store_out(a, it.b, h0 + g, d, acc, lsum);
    if (d == 0) store_lse(a, it.b, h0 + g, mx, lsum);
  }
}

// Merge of at most MAXS partials by 128 threads, thread d producing output dim
// d of every head: all partial loads are issued before any is used, so the
// merge costs one memory round trip and no barrier.
template <int G, int MAXS>
__device__ __forceinline__ void combine_partials_regs(const DecodeArgs &a, const Item &it,
                                                      int first, int d) {
  const int ns = it.nsplit;
  float2 ml[MAXS][G];
  float ov[MAXS][G];
  const float2 *mls = a.part_ml + static_cast<int64_t>(first) * G;
  const float *po = a.part_o + static_cast<int64_t>(first) * G * kHeadDim + d;
#pragma unroll
  for (int s = 0; s < MAXS; ++s)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const bool in = s < ns;
      ml[s][g] = in ? __ldcg(mls + s * G + g) : make_float2(-CUDART_INF_F, 0.f);
      ov[s][g] = in ? __ldcg(po + (s * G + g) * kHeadDim) : 0.f;
    }
  const int h0 = it.kvh * G;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int s = 0; s < MAXS; ++s) mx = fmaxf(mx, ml[s][g].x);
    float l = 0.f, acc = 0.f;
#pragma unroll
    for (int s = 0; s < MAXS; ++s) {
      const float w = ml[s][g].x == -CUDART_INF_F ? 0.f : exp2f(ml[s][g].x - mx);
      l = fmaf(ml[s][g].y, w, l);
      acc = fmaf(ov[s][g], w, acc);
    }
    store_out(a, it.b, h0 + g, d, acc, l);
    if (d == 0) store_lse(a, it.b, h0 + g, mx, l);
  }
}

// Same merge with the split weights staged in shared memory (`scratch`,
// capacity `cap` floats, shared by the NT threads, which must all call this):
// the per-split max/sum are read once, each thread then streams its partial
// outputs with independent, unrolled loads.  Falls back to combine_partials
// when the splits do not fit.
template <int G, int NT, typename SyncFn>
__device__ __forceinline__ void combine_partials_staged(const DecodeArgs &a, const Item &it,
                                                        int first, int tid, float *scratch,
                                                        int cap, SyncFn sync) {
  const int ns = it.nsplit;
  if (3 * ns * G + 2 * G > cap) {
    combine_partials<G, NT>(a, it, first, tid);
    return;
  }
  float *w = scratch;                 // [ns][G] weights exp2(m_s - M) / L
  float *stat = scratch + ns * G;     // M[G], L[G]
  float *mls = stat + 2 * G;          // [ns][G] (m, l) pairs
  const float2 *src = a.part_ml + static_cast<int64_t>(first) * G;
  for (int i = tid; i < ns * G; i += NT) {
    const float2 ml = __ldcg(src + i);
    mls[2 * i] = ml.x;
    mls[2 * i + 1] = ml.y;
  }
  sync();
  if (tid < G) {
    float mx = -CUDART_INF_F;
    for (int s = 0; s < ns; ++s) mx = fmaxf(mx, mls[2 * (s * G + tid)]);
    float l = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float m = mls[2 * (s * G + tid)];
      l = fmaf(mls[2 * (s * G + tid) + 1], m == -CUDART_INF_F ? 0.f : exp2f(m - mx), l);
    }
    stat[tid] = mx;
    stat[G + tid] = l;
  }
  sync();
  for (int i = tid; i < ns * G; i += NT) {
    const int g = i % G;
    const float m = mls[2 * i], mx = stat[g], l = stat[G + g];
    w[i] = (m == -CUDART_INF_F || !(l > 0.f)) ? 0.f : exp2f(m - mx) / l;
  }
  sync();
  const int h0 = it.kvh * G;
  for (int i = tid; i < G * kHeadDim; i += NT) {
    const int g = i / kHeadDim, d = i % kHeadDim;
    const float *po = a.part_o + static_cast<int64_t>(first) * G * kHeadDim + i;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    int s = 0;
    for (; s + 4 <= ns; s += 4) {
      const float v0 = __ldcg(po + (s + 0) * G * kHeadDim);
      const float v1 = __ldcg(po + (s + 1) * G * kHeadDim);
      const float v2 = __ldcg(po + (s + 2) * G * kHeadDim);
      const float v3 = __ldcg(po + (s + 3) * G * kHeadDim);
      acc0 = fmaf(v0, w[(s + 0) * G + g], acc0);
      acc1 = fmaf(v1, w[(s + 1) * G + g], acc1);
      acc2 = fmaf(v2, w[(s + 2) * G + g], acc2);
      acc3 = fmaf(v3, w[(s + 3) * G + g], acc3);
    }
    for (; s < ns; ++s) acc0 = fmaf(__ldcg(po + s * G * kHeadDim), w[s * G + g], acc0);
    const float l = stat[G + g];
    a.out[it.b * a.o_sb + (h0 + g) * a.o_sh + d] =
        __float2half_rn(l > 0.f ? (acc0 + acc1) + (acc2 + acc3) : 0.f);
    if (d == 0) store_lse(a, it.b, h0 + g, stat[g], l);
  }
  sync();
}

}  // namespace b200kv
