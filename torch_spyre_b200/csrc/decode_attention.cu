// Split-KV paged decode attention for B200 (sm_100a).
//
// Computes, for every sequence b and query head h (GQA group g = h % G of KV
// head h / G, G = Hq / Hkv),
//     out[b, h, :] = softmax(scale * q[b, h, :] . K_b^T) . V_b
// over the ctx_b tokens of sequence b, whose K/V rows live in 64-token pages
// of the paged stick layout (see include/b200kv.h).  This is the decode case of
// the reference's SDPA decomposition spyre__sdpa_overrideable
// (torch_spyre/_inductor/decompositions.py:523-611): scores -> softmax -> P.V,
// GQA by KV-head expansion (560-563), computed here in fp32 with one scale.
//
// Design (one persistent launch):
//   * work items = (b, kv_head, split); a split is a run of C consecutive pages.
//     Every CTA derives the same partition from context_lens (C is chosen so the
//     grid gets ~num_splits items per CTA), so no host synchronisation and no
//     planning launch are needed;
//   * pages are carried through an NST-stage shared-memory ring ("carousel"):
//     thread 0 issues one 3-D TMA load per K page and per V page (16 KiB each,
//     128-byte swizzle, L2 evict-first) up to NST pages ahead, across item
//     boundaries; each stage completes on its own mbarrier;
//   * the G query heads of a KV head share every staged byte (the KV stream is
//     read once per group);
//   * Q.K^T: 8 threads per token, 16 dims each, fp32 FMA, then a warp-shuffle
//     reduce-scatter so each lane ends with one head's score;
//   * online softmax (exp2 domain) per page, one warp per head, shuffle
//     max/sum; P.V: each thread owns one 8-dim chunk for all G heads and a
//     quarter of the tokens; lazy rescale only when a running max moves;
//   * a split that is not the only one of its (b, kv_head) writes its
//     unnormalised partial (O, m, l) to the workspace; the last CTA to finish a
//     (b, kv_head) (atomic ticket, self-resetting) merges the partials with a
//     log-sum-exp combine in fp32 and writes the fp16 output.
#include <math_constants.h>

#include <cmath>

#include "common.cuh"

namespace b200kv {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxBatch = 1024;
constexpr int kMaxWorkItems = 8192;
constexpr int kDefaultItemsPerCta = 4;

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
  int *counters;     // [batch * hkv], zero between calls
  float2 *part_ml;   // [slots][G] (running max in log2 units, running sum)
  float *part_o;     // [slots][G][128] unnormalised partial output
  int32_t *error_flag;
};

struct WorkspaceLayout {
  int64_t counters_off, ml_off, o_off, total;
};

WorkspaceLayout workspace_layout(int64_t batch, int64_t hq, int64_t hkv) {
  const int64_t g = hq / hkv;
  const int64_t slots = kMaxWorkItems + batch * hkv;
  auto up = [](int64_t x) { return (x + 255) & ~int64_t(255); };
  WorkspaceLayout w;
  w.counters_off = 0;
  w.ml_off = up(batch * hkv * 4);
  w.o_off = up(w.ml_off + slots * g * 8);
  w.total = up(w.o_off + slots * g * kHeadDim * 4);
  return w;
}

template <int G, int NST>
struct Smem {
  static constexpr int kStageBytes = 2 * kPageBytes;  // K page + V page
  static constexpr int kStages = 0;
  static constexpr int kScore = kStages + NST * kStageBytes;    // float [G][64]
  static constexpr int kP = kScore + G * 64 * 4;                // float [64][G]
  static constexpr int kORed = kP + 64 * G * 4;                 // float [G][128]
  static constexpr int kWRed = kORed + G * kHeadDim * 4;        // float [8 warps][G][128]
  static constexpr int kStats = kWRed + 8 * G * kHeadDim * 4;   // float m[G], l[G], alpha[G]
  static constexpr int kNb = kStats + 3 * 16 * 4;               // int [kMaxBatch]
  static constexpr int kSplits = kNb + kMaxBatch * 4;           // int [kMaxBatch]
  static constexpr int kPrefix = kSplits + kMaxBatch * 4;       // int [kMaxBatch + 1]
  static constexpr int kScratch = kPrefix + (kMaxBatch + 1) * 4 + 4;  // int [64]
  static constexpr int kBars = (kScratch + 64 * 4 + 7) & ~7;    // uint64 [NST]
  static constexpr int kBytes = kBars + NST * 8;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

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

// Reduce-scatter of N per-lane values over the 8-lane group (lane bits 0..2).
// Each halving step sends half of the remaining values to the partner lane
// (xor MASK) and adds what comes back; `head` accumulates which value index
// this lane keeps.  When one value is left the remaining masks all-reduce it.
template <int N, int MASK>
struct ReduceScatter8 {
  __device__ __forceinline__ static float run(const float *v, int lane, int &head) {
    if constexpr (N == 1) {
      float x = v[0];
#pragma unroll
      for (int m = MASK; m >= 1; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
      return x;
    } else {
      static_assert(MASK >= 1, "more values than lanes");
      constexpr int H = N / 2;
      const bool up = (lane & MASK) != 0;
      float nv[H];
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float send = up ? v[i] : v[i + H];
        const float keep = up ? v[i + H] : v[i];
        nv[i] = keep + __shfl_xor_sync(0xffffffffu, send, MASK);
      }
      if (up) head += H;
      return ReduceScatter8<H, MASK / 2>::run(nv, lane, head);
    }
  }
};

__device__ __forceinline__ void h8_to_f32(const uint4 &u, float *f) {
  const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __half22float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

// Number of pages of sequence b (context length clamped to the block table).
__device__ __forceinline__ int seq_pages(const DecodeArgs &a, int b, int *ctx_out) {
  int ctx = __ldg(a.ctx_lens + b);
  const int cap = a.max_blocks * kPageTokens;
  if (ctx < 0 || ctx > cap) {
    if (a.error_flag) atomicOr(a.error_flag, B200KV_DEVERR_BAD_LEN);
    ctx = ctx < 0 ? 0 : cap;
  }
  if (ctx_out) *ctx_out = ctx;
  return (ctx + kPageTokens - 1) / kPageTokens;
}

struct Item {
  int b, kvh, split, nsplit, p, p_end, ctx;
};

// Decodes work item `it` (b-major, then kv head, then split) from the plan.
__device__ __forceinline__ Item decode_item(const DecodeArgs &a, int it, const int *s_nb,
                                            const int *s_splits, const int *s_prefix, int chunk) {
  int lo = 0, hi = a.batch - 1;  // largest b with prefix[b] <= it
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_prefix[mid] <= it) lo = mid; else hi = mid - 1;
  }
  Item r;
  r.b = lo;
  r.nsplit = s_splits[lo];
  const int rem = it - s_prefix[lo];
  r.kvh = rem / r.nsplit;
  r.split = rem - r.kvh * r.nsplit;
  const int nb = s_nb[lo];
  r.p = r.split * chunk;
  r.p_end = min(r.p + chunk, nb);
  if (r.p > r.p_end) r.p = r.p_end;
  r.ctx = min(nb * kPageTokens, __ldg(a.ctx_lens + lo) < 0 ? 0 : __ldg(a.ctx_lens + lo));
  return r;
}

template <int G, int NST>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  using L = Smem<G, NST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *s_score = reinterpret_cast<float *>(smem + L::kScore);
  float *s_p = reinterpret_cast<float *>(smem + L::kP);
  float *s_ored = reinterpret_cast<float *>(smem + L::kORed);
  float *s_wred = reinterpret_cast<float *>(smem + L::kWRed);
  float *s_m = reinterpret_cast<float *>(smem + L::kStats);
  float *s_l = s_m + 16;
  float *s_alpha = s_l + 16;
  int *s_nb = reinterpret_cast<int *>(smem + L::kNb);
  int *s_splits = reinterpret_cast<int *>(smem + L::kSplits);
  int *s_prefix = reinterpret_cast<int *>(smem + L::kPrefix);
  int *s_scratch = reinterpret_cast<int *>(smem + L::kScratch);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBars);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  if (tid == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < NST; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }

  // ---- plan: pages per sequence, chunk size, splits, item prefix ----------
  int local_pages = 0;
  for (int b = tid; b < a.batch; b += kThreads) {
    const int nb = seq_pages(a, b, nullptr);
    s_nb[b] = nb;
    local_pages += nb;
  }
  {
    int v = local_pages;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    if (lane == 0) s_scratch[warp] = v;
  }
  __syncthreads();
  int total_pages = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) total_pages += s_scratch[w];
  const long long page_heads = static_cast<long long>(total_pages) * a.hkv;
  const int chunk = max(1, static_cast<int>((page_heads + a.target_items - 1) / a.target_items));
  // splits per sequence and exclusive prefix of item counts (4 sequences per thread)
  constexpr int kPer = kMaxBatch / kThreads;
  int cnt[kPer];
  int run = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    int items = 0;
    if (b < a.batch) {
      const int ns = max(1, (s_nb[b] + chunk - 1) / chunk);
      s_splits[b] = ns;
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
  __syncthreads();  // s_scratch reuse
  if (lane == 31) s_scratch[warp] = incl;
  __syncthreads();
  int warp_base = 0;
  for (int w = 0; w < warp; ++w) warp_base += s_scratch[w];
  const int thread_base = warp_base + incl - run;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = tid * kPer + i;
    if (b < a.batch) s_prefix[b] = thread_base + cnt[i];
  }
  if (tid == kThreads - 1) s_prefix[a.batch] = thread_base + run;
  if (tid < G) {
    s_m[tid] = -CUDART_INF_F;
    s_l[tid] = 0.f;
  }
  __syncthreads();
  const int total_items = s_prefix[a.batch];

  // ---- producer (thread 0): page cursor over this CTA's items --------------
  int prod_item = blockIdx.x, prod_p = 0, prod_end = 0, prod_b = 0, prod_kvh = 0;
  bool prod_live = false;
  uint64_t policy = 0;
  auto prod_seek = [&]() {  // advance to the next page that exists
    while (prod_p >= prod_end) {
      if (prod_live) prod_item += gridDim.x;
      prod_live = true;
      if (prod_item >= total_items) {
        prod_live = false;
        return;
      }
      const Item it = decode_item(a, prod_item, s_nb, s_splits, s_prefix, chunk);
      prod_b = it.b;
      prod_kvh = it.kvh;
      prod_p = it.p;
      prod_end = it.p_end;
    }
  };
  auto prod_issue = [&](int stage) {
    prod_seek();
    if (!prod_live) return;
    int blk = __ldg(a.block_table + static_cast<int64_t>(prod_b) * a.bt_stride + prod_p);
    if (blk < 0 || blk >= a.num_blocks) {
      if (a.error_flag) atomicOr(a.error_flag, B200KV_DEVERR_BAD_BLOCK);
      blk = 0;
    }
    const int page = blk * a.hkv + prod_kvh;
    uint8_t *dst = smem + stage * L::kStageBytes;
    mbar_arrive_expect_tx(&bars[stage], 2 * kPageBytes);
    tma_load_3d(dst, &kmap, &bars[stage], 0, 0, page, policy);
    tma_load_3d(dst + kPageBytes, &vmap, &bars[stage], 0, 0, page, policy);
    ++prod_p;
  };
  if (tid == 0) {
    policy = l2_policy_evict_first();
    prod_item = blockIdx.x;
    prod_live = false;
    prod_p = prod_end = 0;
    for (int s = 0; s < NST; ++s) prod_issue(s);
  }

  // ---- consumer: all threads ------------------------------------------------
  const int qk_part = tid & 7;          // 16-dim slice of the head
  const int qk_stick = qk_part >> 2;
  const int qk_c0 = (qk_part & 3) * 2;  // first 16-byte chunk of the slice
  const int pv_c = tid & 15;            // 8-dim chunk owned in P.V
  const int pv_stick = pv_c >> 3;
  const int pv_ch = pv_c & 7;
  const int pv_tg = tid >> 4;           // token group (tokens tg + 16 j)

  int stage = 0;
  uint32_t phase = 0;
  for (int item = blockIdx.x; item < total_items; item += gridDim.x) {
    const Item it = decode_item(a, item, s_nb, s_splits, s_prefix, chunk);
    const int h0 = it.kvh * G;
    // q slice of this thread, fp32: qf[g][0..15] = q[b, h0 + g, 16 * part ...]
    float qf[G][16];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const __half *qp = a.q + it.b * a.q_sb + (h0 + g) * a.q_sh + qk_part * 16;
      const uint4 u0 = __ldg(reinterpret_cast<const uint4 *>(qp));
      const uint4 u1 = __ldg(reinterpret_cast<const uint4 *>(qp + 8));
      h8_to_f32(u0, qf[g]);
      h8_to_f32(u1, qf[g] + 8);
    }
    float o[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < 8; ++e) o[g][e] = 0.f;

    for (int p = it.p; p < it.p_end; ++p) {
      const int valid = min(kPageTokens, it.ctx - p * kPageTokens);
      mbar_wait_bounded(&bars[stage], phase, a.error_flag);
      const uint8_t *kpage = smem + stage * L::kStageBytes;
      const uint8_t *vpage = kpage + kPageBytes;

      // -- scores: 2 passes of 32 tokens, 8 threads per token -------------
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int t = pass * 32 + (tid >> 3);
        float acc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g] = 0.f;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const uint4 kv = *reinterpret_cast<const uint4 *>(kpage + swz_off(qk_stick, t, qk_c0 + cc));
          float kf[8];
          h8_to_f32(kv, kf);
#pragma unroll
          for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int g = 0; g < G; ++g) acc[g] = fmaf(qf[g][cc * 8 + e], kf[e], acc[g]);
        }
        int head = 0;
        const float s = ReduceScatter8<G, 4>::run(acc, lane, head);
        if ((qk_part & (8 / G - 1)) == 0)
          s_score[head * 64 + t] = t < valid ? s * a.scale_log2 : -CUDART_INF_F;
      }
      __syncthreads();

      // -- online softmax, one warp per head -------------------------------
      for (int g = warp; g < G; g += kThreads / 32) {
        const float s0 = s_score[g * 64 + lane];
        const float s1 = s_score[g * 64 + lane + 32];
        const float mx = warp_max(fmaxf(s0, s1));
        const float m_old = s_m[g];
        const float m_new = fmaxf(m_old, mx);
        float p0 = 0.f, p1 = 0.f, alpha = 1.f;
        if (m_new != -CUDART_INF_F) {
          p0 = exp2f(s0 - m_new);
          p1 = exp2f(s1 - m_new);
          alpha = exp2f(m_old - m_new);
        }
        const float sum = warp_sum(p0 + p1);
        s_p[lane * G + g] = p0;
        s_p[(lane + 32) * G + g] = p1;
        __syncwarp();
        if (lane == 0) {
          s_l[g] = s_l[g] * alpha + sum;
          s_m[g] = m_new;
          s_alpha[g] = alpha;
        }
      }
      __syncthreads();

      // -- P.V ------------------------------------------------------------
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float al = s_alpha[g];
        if (al != 1.f) {
#pragma unroll
          for (int e = 0; e < 8; ++e) o[g][e] *= al;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = pv_tg + 16 * j;
        if (t < valid) {
          const uint4 vv = *reinterpret_cast<const uint4 *>(vpage + swz_off(pv_stick, t, pv_ch));
          float vf[8];
          h8_to_f32(vv, vf);
          float pw[G];
#pragma unroll
          for (int g = 0; g < G; ++g) pw[g] = s_p[t * G + g];
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < 8; ++e) o[g][e] = fmaf(pw[g], vf[e], o[g][e]);
        }
      }
      __syncthreads();  // stage fully consumed
      if (tid == 0) prod_issue(stage);
      if (++stage == NST) {
        stage = 0;
        phase ^= 1u;
      }
    }

    // ---- finish the item: reduce the 16 token groups in a fixed order -------
    // (lanes 0-15 and 16-31 of a warp hold two token groups: add them with a
    // shuffle, then sum the 8 warps' partials in warp order -> deterministic)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < 8; ++e) o[g][e] += __shfl_xor_sync(0xffffffffu, o[g][e], 16);
    if (lane < 16) {
      float *dst = s_wred + warp * (G * kHeadDim) + pv_stick * 64 + pv_ch * 8;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        *reinterpret_cast<float4 *>(dst + g * kHeadDim) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
        *reinterpret_cast<float4 *>(dst + g * kHeadDim + 4) = make_float4(o[g][4], o[g][5], o[g][6], o[g][7]);
      }
    }
    __syncthreads();
    for (int i = tid; i < G * kHeadDim; i += kThreads) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) acc += s_wred[w * (G * kHeadDim) + i];
      s_ored[i] = acc;
    }
    __syncthreads();
    constexpr float kLn2 = 0.69314718055994530942f;
    if (it.nsplit == 1) {
      for (int i = tid; i < G * kHeadDim; i += kThreads) {
        const int g = i / kHeadDim, d = i % kHeadDim;
        const float l = s_l[g];
        const float v = l > 0.f ? s_ored[i] / l : 0.f;
        a.out[it.b * a.o_sb + (h0 + g) * a.o_sh + d] = __float2half_rn(v);
      }
      if (a.lse && tid < G) {
        const float l = s_l[tid];
        a.lse[static_cast<int64_t>(it.b) * a.hq + h0 + tid] =
            l > 0.f ? (s_m[tid] + log2f(l)) * kLn2 : -CUDART_INF_F;
      }
    } else {
      float *po = a.part_o + static_cast<int64_t>(item) * G * kHeadDim;
      for (int i = tid; i < G * kHeadDim; i += kThreads) __stcg(po + i, s_ored[i]);
      if (tid < G) __stcg(a.part_ml + static_cast<int64_t>(item) * G + tid, make_float2(s_m[tid], s_l[tid]));
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const int ticket = atomicAdd(a.counters + it.b * a.hkv + it.kvh, 1);
        s_scratch[0] = ticket == it.nsplit - 1;
      }
      __syncthreads();
      if (s_scratch[0]) {
        __threadfence();
        const int first = item - it.split;
        for (int i = tid; i < G * kHeadDim; i += kThreads) {
          const int g = i / kHeadDim;
          float mx = -CUDART_INF_F;
          for (int s = 0; s < it.nsplit; ++s)
            mx = fmaxf(mx, __ldcg(a.part_ml + static_cast<int64_t>(first + s) * G + g).x);
          float lsum = 0.f, acc = 0.f;
          for (int s = 0; s < it.nsplit; ++s) {
            const float2 ml = __ldcg(a.part_ml + static_cast<int64_t>(first + s) * G + g);
            const float w = ml.x == -CUDART_INF_F ? 0.f : exp2f(ml.x - mx);
            lsum = fmaf(ml.y, w, lsum);
            acc = fmaf(__ldcg(a.part_o + (static_cast<int64_t>(first + s) * G) * kHeadDim + i), w, acc);
          }
          const float v = lsum > 0.f ? acc / lsum : 0.f;
          a.out[it.b * a.o_sb + (h0 + g) * a.o_sh + (i % kHeadDim)] = __float2half_rn(v);
          if (a.lse && (i % kHeadDim) == 0)
            a.lse[static_cast<int64_t>(it.b) * a.hq + h0 + g] =
                lsum > 0.f ? (mx + log2f(lsum)) * kLn2 : -CUDART_INF_F;
        }
        if (tid == 0) atomicExch(a.counters + it.b * a.hkv + it.kvh, 0);
      }
    }
    __syncthreads();
    if (tid < G) {
      s_m[tid] = -CUDART_INF_F;
      s_l[tid] = 0.f;
    }
    __syncthreads();
  }
}

constexpr int kStagesDefault = 4;

template <int G>
int launch_decode(const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a, int items_per_cta,
                  cudaStream_t stream) {
  constexpr int NST = kStagesDefault;
  using L = Smem<G, NST>;
  auto kern = decode_kernel<G, NST>;
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  static int configured[64] = {0};  // per device: smem attribute set
  if (!__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    B200KV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  const int grid = sms;  // one 256-thread CTA per SM (smem-limited)
  long long target = static_cast<long long>(grid) * items_per_cta;
  if (target > kMaxWorkItems) target = kMaxWorkItems;
  a.target_items = static_cast<int>(target);
  kern<<<grid, kThreads, L::kAlloc, stream>>>(km, vm, a);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int64_t b200kv_decode_workspace_bytes(int64_t batch, int64_t num_q_heads,
                                                 int64_t num_kv_heads, int64_t head_dim) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 ||
      head_dim != kHeadDim)
    return -1;
  return workspace_layout(batch, num_q_heads, num_kv_heads).total;
}

extern "C" int b200kv_decode_attention_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool, const void *v_pool,
    const int32_t *block_table, int64_t block_table_stride, const int32_t *context_lens, void *out,
    int64_t out_stride_b, int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq,
    float scale, int64_t num_splits, void *workspace, int64_t workspace_bytes,
    int32_t *error_flag, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(batch >= 0, "batch must be >= 0");
  B200KV_CHECK_ARG(num_q_heads > 0 && num_kv_heads > 0, "head counts must be > 0");
  B200KV_CHECK_ARG(num_q_heads % num_kv_heads == 0,
                   "num_q_heads (%lld) must be a multiple of num_kv_heads (%lld)",
                   (long long)num_q_heads, (long long)num_kv_heads);
  if (head_dim != kHeadDim)
    return set_error(B200KV_ERR_UNSUPPORTED, "head_dim %lld unsupported (only %d)",
                     (long long)head_dim, kHeadDim);
  const int64_t group = num_q_heads / num_kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return set_error(B200KV_ERR_UNSUPPORTED, "GQA group size %lld unsupported (1, 2, 4, 8)",
                     (long long)group);
  if (batch > kMaxBatch)
    return set_error(B200KV_ERR_UNSUPPORTED, "batch %lld > %d unsupported", (long long)batch,
                     kMaxBatch);
  B200KV_CHECK_ARG(num_blocks > 0 && max_blocks_per_seq > 0, "num_blocks and max_blocks_per_seq must be > 0");
  B200KV_CHECK_ARG(max_blocks_per_seq * kPageTokens < (int64_t{1} << 31), "max_blocks_per_seq too large");
  B200KV_CHECK_ARG(block_table_stride >= max_blocks_per_seq, "block_table_stride < max_blocks_per_seq");
  B200KV_CHECK_ARG(num_splits >= 0 && num_splits <= 64, "num_splits must be in [0, 64]");
  B200KV_CHECK_ARG(std::isfinite(scale), "scale must be finite");
  if (batch == 0) return B200KV_OK;
  B200KV_CHECK_ARG(q && k_pool && v_pool && block_table && context_lens && out,
                   "null pointer argument");
  B200KV_CHECK_ARG(aligned16(q) && q_stride_b % 8 == 0 && q_stride_h % 8 == 0,
                   "q must be 16-byte aligned with strides that are multiples of 8 elements");
  const WorkspaceLayout wl = workspace_layout(batch, num_q_heads, num_kv_heads);
  if (!workspace || workspace_bytes < wl.total)
    return set_error(B200KV_ERR_WORKSPACE, "workspace of %lld bytes required (got %lld)",
                     (long long)wl.total, (long long)workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error(B200KV_ERR_WORKSPACE, "workspace must be 256-byte aligned");

  CUtensorMap km, vm;
  int st = make_page_pool_map(&km, k_pool, num_blocks, num_kv_heads);
  if (st != B200KV_OK) return st;
  st = make_page_pool_map(&vm, v_pool, num_blocks, num_kv_heads);
  if (st != B200KV_OK) return st;

  DecodeArgs a;
  a.q = static_cast<const __half *>(q);
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.block_table = block_table;
  a.bt_stride = block_table_stride;
  a.ctx_lens = context_lens;
  a.out = static_cast<__half *>(out);
  a.o_sb = out_stride_b;
  a.o_sh = out_stride_h;
  a.lse = lse;
  a.batch = static_cast<int>(batch);
  a.hkv = static_cast<int>(num_kv_heads);
  a.hq = static_cast<int>(num_q_heads);
  a.max_blocks = static_cast<int>(max_blocks_per_seq);
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.target_items = 0;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  a.counters = reinterpret_cast<int *>(ws + wl.counters_off);
  a.part_ml = reinterpret_cast<float2 *>(ws + wl.ml_off);
  a.part_o = reinterpret_cast<float *>(ws + wl.o_off);
  a.error_flag = error_flag;
  const int per_cta = num_splits > 0 ? static_cast<int>(num_splits) : kDefaultItemsPerCta;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (group) {
    case 1: return launch_decode<1>(km, vm, a, per_cta, s);
    case 2: return launch_decode<2>(km, vm, a, per_cta, s);
    case 4: return launch_decode<4>(km, vm, a, per_cta, s);
    default: return launch_decode<8>(km, vm, a, per_cta, s);
  }
}
