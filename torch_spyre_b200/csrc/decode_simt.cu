// Decode attention, CUDA-core variant (fp32 FMA on 256 threads).
//
// Kept beside the tensor-core kernel (decode_mma.cu) as the measured baseline
// of the "CUDA cores in fp32" design: per page, Q.K^T with 8 threads per
// token (16 dims each) and a warp-shuffle reduce-scatter, an online softmax
// with one warp per head, and P.V with one 8-dim chunk per thread for all G
// heads.  Pages arrive through the same TMA stage ring; thread 0 refills a
// stage after the CTA-wide barrier that ends the page.  Selected with
// B200KV_DECODE_KERNEL=simt.
#include "decode_common.cuh"
#include "decode_kernels.h"

namespace b200kv {
namespace {

constexpr int kThreads = 256;

template <int G, int NST>
struct SimtSmem {
  static constexpr int kStageBytes = 2 * kPageBytes;            // K page + V page
  static constexpr int kScore = NST * kStageBytes;              // float [G][64]
  static constexpr int kP = kScore + G * 64 * 4;                // float [64][G]
  static constexpr int kORed = kP + 64 * G * 4;                 // float [G][128]
  static constexpr int kWRed = kORed + G * kHeadDim * 4;        // float [8 warps][G][128]
  static constexpr int kStats = kWRed + 8 * G * kHeadDim * 4;   // float m[16], l[16], alpha[16]
  static constexpr int kPlan = kStats + 3 * 16 * 4;
  static constexpr int kBars = (kPlan + kPlanBytes + 7) & ~7;  // uint64 [NST]
  static constexpr int kBytes = kBars + NST * 8;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

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

template <int G, int NST>
__global__ void __launch_bounds__(kThreads, 1)
    decode_simt_kernel(const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  using L = SimtSmem<G, NST>;
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
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBars);
  Plan pl = plan_view(smem + L::kPlan);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  if (tid == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < NST; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  if (tid < G) {
    s_m[tid] = -CUDART_INF_F;
    s_l[tid] = 0.f;
  }
  build_plan<kThreads>(a, pl);  // synchronises the CTA
  const int total_items = pl.total_items;

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
      const Item it = decode_item(a, pl, prod_item);
      prod_b = it.b;
      prod_kvh = it.kvh;
      prod_p = it.p;
      prod_end = it.p_end;
    }
  };
  auto prod_issue = [&](int stage) {
    prod_seek();
    if (!prod_live) return;
    const int page = page_block(a, prod_b, prod_p) * a.hkv + prod_kvh;
    uint8_t *dst = smem + stage * L::kStageBytes;
    mbar_arrive_expect_tx(&bars[stage], 2 * kPageBytes);
    tma_load_3d(dst, &kmap, &bars[stage], 0, 0, page, policy);
    tma_load_3d(dst + kPageBytes, &vmap, &bars[stage], 0, 0, page, policy);
    ++prod_p;
  };
  if (tid == 0) {
    policy = l2_policy_evict_first();
    for (int s = 0; s < NST; ++s) prod_issue(s);
  }

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
    const Item it = decode_item(a, pl, item);
    const int h0 = it.kvh * G;
    float qf[G][16];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const __half *qp = a.q + it.b * a.q_sb + (h0 + g) * a.q_sh + qk_part * 16;
      h8_to_f32(__ldg(reinterpret_cast<const uint4 *>(qp)), qf[g]);
      h8_to_f32(__ldg(reinterpret_cast<const uint4 *>(qp + 8)), qf[g] + 8);
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

    // ---- finish the item: reduce the 16 token groups in a fixed order -----
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
    if (it.nsplit == 1) {
      for (int i = tid; i < G * kHeadDim; i += kThreads)
        store_out(a, it.b, h0 + i / kHeadDim, i % kHeadDim, s_ored[i], s_l[i / kHeadDim]);
      if (tid < G) store_lse(a, it.b, h0 + tid, s_m[tid], s_l[tid]);
    } else {
      float *po = a.part_o + static_cast<int64_t>(item) * G * kHeadDim;
      for (int i = tid; i < G * kHeadDim; i += kThreads) __stcg(po + i, s_ored[i]);
      if (tid < G)
        __stcg(a.part_ml + static_cast<int64_t>(item) * G + tid, make_float2(s_m[tid], s_l[tid]));
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const int ticket = atomicAdd(a.counters + it.b * a.hkv + it.kvh, 1);
        pl.scratch[0] = ticket == it.nsplit - 1;
      }
      __syncthreads();
      if (pl.scratch[0]) {
        __threadfence();
        combine_partials<G, kThreads>(a, it, SlotMap{item - it.split, it.nsplit}, tid);
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

template <int G>
int launch_simt(const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a, int items_per_cta,
                cudaStream_t stream) {
  constexpr int NST = 4;
  using L = SimtSmem<G, NST>;
  auto kern = decode_simt_kernel<G, NST>;
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  static int configured[64] = {0};
  if (!__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    B200KV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  const int grid = sms;
  const long long target = static_cast<long long>(grid) * items_per_cta;
  a.target_items = static_cast<int>(target > kMaxWorkItems ? kMaxWorkItems : target);
  kern<<<grid, kThreads, L::kAlloc, stream>>>(km, vm, a);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}

}  // namespace

int launch_decode_simt(int group, const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a,
                       int items_per_cta, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_simt<1>(km, vm, a, items_per_cta, stream);
    case 2: return launch_simt<2>(km, vm, a, items_per_cta, stream);
    case 4: return launch_simt<4>(km, vm, a, items_per_cta, stream);
    case 8: return launch_simt<8>(km, vm, a, items_per_cta, stream);
    default: return set_error(B200KV_ERR_UNSUPPORTED, "group %d", group);
  }
}

}  // namespace b200kv
