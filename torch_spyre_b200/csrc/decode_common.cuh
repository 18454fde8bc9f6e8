// Pieces shared by the decode kernels: arguments, workspace layout, the
// split-KV work plan every CTA derives from context_lens, and the last-CTA
// log-sum-exp combine of split partials.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace b200kv {

constexpr int kMaxBatch = 1024;
constexpr int kMaxWorkItems = 1024;   // partial slots beyond one per pair
constexpr int kMaxPartitions = 1024;  // CTAs of a decode launch (one slot each)
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
  // Fused append (null when not appending): the rows of the token at position
  // context_len - 1 of each sequence, written into the pools and used for it.
  const __half *k_new = nullptr, *v_new = nullptr;
  int64_t new_sb = 0, new_sh = 0;
  __half *k_pool_w = nullptr, *v_pool_w = nullptr;
  // FP8 pages (null for fp16 pages): the pools hold e4m3 values whose fp16
  // dequantisation scales are *k_scale / *v_scale; the fused append writes the
  // quantised new rows through k_pool8_w / v_pool8_w.
  const __half *k_scale = nullptr, *v_scale = nullptr;
  uint8_t *k_pool8_w = nullptr, *v_pool8_w = nullptr;
  // Rotary embedding on append (null: none): q and the new K row are rotated
  // with rope_freqs[context_len - 1] ([max_pos][2][2][64] fp16, rope.cuh).
  const __half *rope_freqs = nullptr;
  int64_t rope_max_pos = 0;
  // Early start: the pools, block table and context lengths were written
  // before the preceding kernel on the stream began, so the plan and the
  // first stages' page loads may run before griddepcontrol.wait; q, the
  // appended rows, the scales, the workspace and every write wait.
  int early = 0;
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

// The partition of one launch over `grid` CTAs ("stream-K"): CTA c streams
// the units [c * per, (c + 1) * per), per = ceil(units / grid), so every CTA
// streams the same number of pages whatever the spread of context lengths.
// A pair cut by a CTA boundary is a split: its piece in CTA c writes slot
// pair + c.  Along the unit stream pair and c never decrease and each new
// piece increases one of them, so slots are unique and a pair's pieces occupy
// the contiguous slots pair + c_lo .. pair + c_hi.
struct Partition {
  int units, grid, per;
  __device__ __forceinline__ int lo(int c) const { return min(c * per, units); }
  __device__ __forceinline__ int hi(int c) const { return min((c + 1) * per, units); }
};

__device__ __forceinline__ Partition make_partition(int units, int grid) {
  Partition P;
  P.units = units;
  P.grid = grid;
  P.per = max(1, (units + grid - 1) / grid);
  return P;
}

struct SlotMap {
  int first, count;
  __device__ __forceinline__ int n() const { return count; }
  __device__ __forceinline__ int operator()(int s) const { return first + s; }
};

__device__ __forceinline__ SlotMap pair_slots(const Partition &P, int pair, int pj, int w) {
  const int c_lo = pj / P.per, c_hi = (pj + w - 1) / P.per;
  return SlotMap{pair + c_lo, c_hi - c_lo + 1};
}

// First unit and unit count of a pair.
__device__ __forceinline__ void pair_units(const DecodeArgs &a, const Plan &pl, int pair, int *pj,
                                           int *w) {
  const int b = pair / a.hkv, kvh = pair - (pair / a.hkv) * a.hkv;
  *w = max(pl.nb[b], 1);
  *pj = a.hkv * pl.prefix[b] + kvh * *w;
}

struct Piece {
  int b, kvh, pair;     // sequence, KV head, pair index b * Hkv + kvh
  int p, p_end, ctx;    // pages [p, p_end) of the pair streamed by this piece
  int nsplit, slot;     // pieces of the pair, this piece's partial slot
  int u_next;           // first unit after this piece
};

// The piece that starts at unit u of CTA c's range, which ends at u_hi.
__device__ __forceinline__ Piece locate_piece(const DecodeArgs &a, const Plan &pl,
                                              const Partition &P, int u, int u_hi, int c) {
  int lo = 0, hi = a.batch - 1;  // largest b whose first unit is <= u
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.hkv * pl.prefix[mid] <= u) lo = mid; else hi = mid - 1;
  }
  Piece s;
  s.b = lo;
  const int nb = pl.nb[lo];
  const int w = max(nb, 1);
  const int base = a.hkv * pl.prefix[lo];
  s.kvh = (u - base) / w;
  const int pj = base + s.kvh * w;  // first unit of the pair
  const int hi_u = min(u_hi, pj + w);
  s.pair = lo * a.hkv + s.kvh;
  s.p = min(u - pj, nb);
  s.p_end = min(hi_u - pj, nb);
  s.ctx = pl.ctx[lo];
  s.nsplit = pair_slots(P, s.pair, pj, w).n();
  s.slot = s.pair + c;
  s.u_next = hi_u;
  return s;
}

// Block id of page p of sequence b as stored (may be out of range).
__device__ __forceinline__ int page_block_raw(const DecodeArgs &a, int b, int p) {
  return __ldg(a.block_table + static_cast<int64_t>(b) * a.bt_stride + p);
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
// The reciprocal of a head's sum (one division per head, applied by store_out4_inv).
__device__ __forceinline__ float inv_sum(float l) { return l > 0.f ? __frcp_rn(l) : 0.f; }
// Dims d0..d0+3 of (b, head h) from unnormalised accumulators: one 8-byte
// store where the output row allows it, else four 2-byte stores (the values
// are the same either way).
__device__ __forceinline__ void store_out4_inv(const DecodeArgs &a, int b, int h, int d0, const float (&acc)[4],
                                               float inv) {
  __half *p = a.out + b * a.o_sb + h * a.o_sh + d0;
  const __half2 lo = __floats2half2_rn(__fmul_rn(acc[0], inv), __fmul_rn(acc[1], inv));
  const __half2 hi = __floats2half2_rn(__fmul_rn(acc[2], inv), __fmul_rn(acc[3], inv));
  if ((reinterpret_cast<uintptr_t>(p) & 7u) == 0) {
    *reinterpret_cast<uint2 *>(p) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
  } else {
    p[0] = __low2half(lo);
    p[1] = __high2half(lo);
    p[2] = __low2half(hi);
    p[3] = __high2half(hi);
  }
}
__device__ __forceinline__ void store_lse(const DecodeArgs &a, int b, int h, float m, float l) {
  if (a.lse)
    a.lse[static_cast<int64_t>(b) * a.hq + h] = l > 0.f ? (m + log2f(l)) * kLn2 : -CUDART_INF_F;
}

// Log-sum-exp merge of the nsplit partials of (b, kv head), run by the CTA
// that finished last.  Threads [0, NT) cover the G x 128 outputs.
template <int G, int NT>
__device__ __forceinline__ void combine_partials(const DecodeArgs &a, const Item &it,
                                                 const SlotMap &sm, int tid) {
  const int h0 = it.kvh * G;
  for (int i = tid; i < G * kHeadDim; i += NT) {
    const int g = i / kHeadDim, d = i % kHeadDim;
    float mx = -CUDART_INF_F;
    for (int s = 0; s < it.nsplit; ++s)
      mx = fmaxf(mx, __ldcg(a.part_ml + static_cast<int64_t>(sm(s)) * G + g).x);
    float lsum = 0.f, acc = 0.f;
    for (int s = 0; s < it.nsplit; ++s) {
      const float2 ml = __ldcg(a.part_ml + static_cast<int64_t>(sm(s)) * G + g);
      const float w = ml.x == -CUDART_INF_F ? 0.f : exp2f(ml.x - mx);
      lsum = fmaf(ml.y, w, lsum);
      acc = fmaf(__ldcg(a.part_o + static_cast<int64_t>(sm(s)) * G * kHeadDim + i), w, acc);
    }
    store_out(a, it.b, h0 + g, d, acc, lsum);
    if (d == 0) store_lse(a, it.b, h0 + g, mx, lsum);
  }
}

// Log-sum-exp merge of a pair's split partials by one warp: lane l produces
// output dims 4l .. 4l + 3 of every head of the pair (one 16-byte load per
// partial row, one 8-byte store per output row).  Splits are
// read two at a time (every load of a batch issued before any is used) and
// folded into a running (max, sum, accumulator) per head, so any number of
// splits merges without shared memory.  The running state starts from
// (M, Ls, acc): empty for the ticket holder, or the merged state of a piece
// that knows it is the pair's last, which then skips its own slot (`skip`;
// -1 skips none).
template <int G>
__device__ __forceinline__ void combine_online_warp_from(const DecodeArgs &a, int b, int kvh, const SlotMap &sm,
                                                         int lane, int skip, float (&M)[G], float (&Ls)[G],
                                                         float (&acc)[G][4]) {
  const int ns = sm.n();
  for (int s0 = 0; s0 < ns; s0 += 2) {
    float2 ml[2][G];
    float ov[2][G][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const bool in = s0 + j < ns && sm(s0 + j) != skip;
      const int64_t slot = sm(s0 + j < ns ? s0 + j : s0);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        ml[j][g] = in ? __ldcg(a.part_ml + slot * G + g) : make_float2(-CUDART_INF_F, 0.f);
        const float4 v = in ? __ldcg(reinterpret_cast<const float4 *>(a.part_o + (slot * G + g) * kHeadDim) + lane)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        ov[j][g][0] = v.x;
        ov[j][g][1] = v.y;
        ov[j][g][2] = v.z;
        ov[j][g][3] = v.w;
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float m = ml[j][g].x;
        if (m != -CUDART_INF_F) {
          const float mn = fmaxf(M[g], m);
          const float w_old = M[g] == -CUDART_INF_F ? 0.f : exp2f(M[g] - mn);
          const float w_new = exp2f(m - mn);
          // explicit roundings: every merge path computes the same bits
          Ls[g] = fmaf(Ls[g], w_old, __fmul_rn(ml[j][g].y, w_new));
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[g][k] = fmaf(acc[g][k], w_old, __fmul_rn(ov[j][g][k], w_new));
          M[g] = mn;
        }
      }
  }
  const int h0 = kvh * G;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    store_out4_inv(a, b, h0 + g, 4 * lane, acc[g], inv_sum(Ls[g]));
    if (lane == 0) store_lse(a, b, h0 + g, M[g], Ls[g]);
  }
}

template <int G>
__device__ __forceinline__ void combine_online_warp(const DecodeArgs &a, int b, int kvh,
                                                    const SlotMap &sm, int lane) {
  float M[G], Ls[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    M[g] = -CUDART_INF_F;
    Ls[g] = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[g][k] = 0.f;
  }
  combine_online_warp_from<G>(a, b, kvh, sm, lane, -1, M, Ls, acc);
}

}  // namespace b200kv
