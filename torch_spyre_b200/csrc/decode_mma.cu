// Decode attention, tensor-core variant (the default).
//
// Why tensor cores: a KV head with G query heads does 2*G flops per fp16 KV
// element (G flop per byte).  On CUDA cores that is G fp32 FMAs plus a
// conversion per element; at G = 8 and 80% of HBM bandwidth that is ~90% of
// the SMs' fp32 issue rate before any softmax or reduction work, so the
// CUDA-core kernel (decode_simt.cu) cannot keep up with HBM.  Here the grouped
// tile runs on mma.sync m16n8k16 (fp16 in, fp32 accumulate), with the G heads
// in the n = 8 dimension (G < 8 is zero-padded), which leaves the SMs almost
// idle and the kernel bound by HBM.
//
// CTA = 1 producer warp + 4 consumer warps, one CTA per SM (persistent):
// Work partition: the balanced unit split of decode_common.cuh (every CTA
// streams the same number of pages; a sequence-head cut by a CTA boundary is
// a split).
//   producer  walks this CTA's pieces page by page: block ids are fetched
//             32 at a time by the whole warp, the piece's q rows are staged
//             with its first page, and lane 0 issues two 3-D TMA loads per page (K, V;
//             16 KiB each, 128-byte swizzle, L2 evict-first) into an NST-stage
//             ring, waiting on each stage's "empty" mbarrier and arming its
//             "full" mbarrier with the bytes;
//   consumer  warp w owns tokens [16w, 16w + 16) of every page and keeps its
//             own online-softmax state, so no CTA barrier is taken per page:
//               S^T[16 t x 8 h] = K[16 t x 128 d] . Q^T   (8 mma, ldmatrix)
//               mask t >= ctx, exp2-domain online softmax (shuffles over t)
//               P^T fragment from S^T by movmatrix.trans
//               O^T[128 d x 8 h] += V^T[128 d x 16 t] . P^T (8 mma, ldmatrix.trans)
//             then one arrive on the stage's empty barrier.
// At the end of a piece the 4 warps' (m, l, O) are merged in shared
// memory; a single split writes the fp16 output, otherwise the unnormalised
// partial goes to the workspace and the CTA that takes the last ticket of the
// (b, kv head) merges all partials (decode_common.cuh); the ticket is read one
// piece later so its atomic round trip overlaps useful work.
#include "decode_kernels.h"

namespace b200kv {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kMmaThreads = (kConsumerWarps + 1) * 32;

// Staged q of one piece: G rows of 128 fp16, row stride padded to 272 B so
// the Q^T fragment loads (8 heads x 4 lanes) hit 32 distinct banks.
constexpr int kQRowBytes = 272;
constexpr int kQSlotBytes = 8 * kQRowBytes;

template <int NST>
struct MmaSmem {
  static constexpr int kStageBytes = 2 * kPageBytes;                     // K page + V page
  static constexpr int kQ = NST * kStageBytes;                           // q slot per stage
  static constexpr int kWO = kQ + NST * kQSlotBytes;                     // float [4][128][8]
  static constexpr int kWML = kWO + kConsumerWarps * kHeadDim * 8 * 4;   // float2 [4][8]
  static constexpr int kPlan = kWML + kConsumerWarps * 8 * 8;
  static constexpr int kBars = (kPlan + kPlanBytes + 7) & ~7;            // full[NST], empty[NST]
  static constexpr int kBytes = kBars + 2 * NST * 8;
  static constexpr int kAlloc = kBytes + 1024;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}
__device__ __forceinline__ float quad_max(float v) {  // over lanes with equal lane % 4
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  return v + __shfl_xor_sync(0xffffffffu, v, 16);
}

template <int G, int NST>
__global__ void __launch_bounds__(kMmaThreads, 1)
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  static_assert(G >= 1 && G <= 8, "the head group sits in one n = 8 MMA tile");
  using L = MmaSmem<NST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *s_wo = reinterpret_cast<float *>(smem + L::kWO);
  float2 *s_wml = reinterpret_cast<float2 *>(smem + L::kWML);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBars);
  uint64_t *empty = full + NST;
  Plan pl = plan_view(smem + L::kPlan);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  if (tid == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  build_unit_plan<kMmaThreads>(a, pl);  // synchronises the CTA
  const int total_units = pl.total_items;
  const int per = max(1, (total_units + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x));
  const int c = blockIdx.x;
  const int u_begin = min(c * per, total_units);
  const int u_end = min(u_begin + per, total_units);

  // ------------------------------------------------------------ producer --
  // The whole warp fetches the next 32 block ids of a piece in one coalesced
  // load (so page issue never waits on a block-table read); lane 0 arms the
  // stage's full barrier and issues the two page loads, plus, with the first
  // page of a piece, one bulk copy per q row into the stage's q slot.
  if (warp == kConsumerWarps) {
    const uint64_t policy = l2_policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    for (int u = u_begin; u < u_end;) {
      const Seg it = locate_seg(a, pl, u, u_end, c, per);
      u = it.u_next;
      for (int base = it.p; base < it.p_end; base += 32) {
        const int n = min(32, it.p_end - base);
        const int my_blk = lane < n ? page_block(a, it.b, base + lane) : 0;
        for (int j = 0; j < n; ++j) {
          const int blk = __shfl_sync(0xffffffffu, my_blk, j);
          if (lane == 0) {
            mbar_wait_bounded(&empty[stage], phase ^ 1u, a.error_flag);
            const int page = blk * a.hkv + it.kvh;
            uint8_t *dst = smem + stage * L::kStageBytes;
            const bool first = base + j == it.p;
            mbar_arrive_expect_tx(&full[stage], 2 * kPageBytes + (first ? G * kHeadDim * 2 : 0));
            if (first) {  // the piece's q rows ride on its first page's barrier
              uint8_t *qs = smem + L::kQ + stage * kQSlotBytes;
              const __half *qg = a.q + it.b * a.q_sb + (it.kvh * G) * a.q_sh;
#pragma unroll
              for (int g = 0; g < G; ++g) bulk_load(qs + g * kQRowBytes, qg + g * a.q_sh, kHeadDim * 2, &full[stage]);
            }
            tma_load_3d(dst, &kmap, &full[stage], 0, 0, page, policy);
            tma_load_3d(dst + kPageBytes, &vmap, &full[stage], 0, 0, page, policy);
          }
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    return;
  }

  // ----------------------------------------------------------- consumers --
  const int t0 = warp * 16;          // this warp's 16 tokens of each page
  const int mi = lane >> 3;          // ldmatrix: which 8x8 matrix this lane addresses
  const int mr = lane & 7;           // ldmatrix: row within that matrix
  const int k_row = t0 + mr + (mi & 1) * 8;   // K rows (A of Q.K^T, non-transposed)
  const int k_dof = (mi >> 1) * 8;
  const int v_row = t0 + mr + (mi >> 1) * 8;  // V rows (A = V^T of P.V, transposed)
  const int v_dof = (mi & 1) * 8;
  const int qh = lane >> 2;          // head of this lane's Q^T fragment (n index)
  const int hc = (lane & 3) * 2;     // heads of this lane's accumulator columns
  const int tr = t0 + (lane >> 2);   // token of this lane's S^T rows (and +8)
  const float sc = a.scale_log2;
  // Completion ticket of the previous split piece, checked one piece later so
  // the atomic's round trip overlaps the next piece's pages (thread 0 only).
  bool pend = false;
  int pend_ticket = 0, pend_b = 0, pend_kvh = 0, pend_nsplit = 0, pend_first = 0;
  int *s_flag = pl.scratch + 8;  // [0] combine? [1] b [2] kvh [3] nsplit [4] first slot [5] more

  int stage = 0;
  uint32_t phase = 0;
  for (int u = u_begin;;) {
    const bool live = u < u_end;
    Seg it;
    if (live) {
      it = locate_seg(a, pl, u, u_end, c, per);
      u = it.u_next;
      const int h0 = it.kvh * G;
      uint32_t qb[8][2];
      float o[8][4];
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;

      for (int p = it.p; p < it.p_end; ++p) {
        const int valid = min(kPageTokens, it.ctx - p * kPageTokens);
        mbar_wait_bounded(&full[stage], phase, a.error_flag);
        const uint32_t kbase = smem_u32(smem + stage * L::kStageBytes);
        const uint32_t vbase = kbase + kPageBytes;
        if (p == it.p) {  // q of this piece, staged with its first page
          const uint32_t qs = smem_u32(smem + L::kQ + stage * kQSlotBytes) + qh * kQRowBytes + hc * 2;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            uint32_t x0 = 0u, x1 = 0u;
            if (qh < G) {
              asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x0) : "r"(qs + ks * 32));
              asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x1) : "r"(qs + ks * 32 + 16));
            }
            qb[ks][0] = x0;
            qb[ks][1] = x1;
          }
        }
        const bool partial = valid < t0 + 16;
        if (partial) {  // zero this warp's V rows past the context (0 * NaN = NaN in the MMA)
          for (int idx = lane; idx < 16 * 16; idx += 32) {
            const int t = t0 + (idx >> 4), c = idx & 15;
            if (t >= valid) st_shared_zero16(vbase + swz_off(c >> 3, t, c & 7));
          }
          __syncwarp();
        }
        // S^T = K . Q^T over the 128 dims (two independent accumulation chains)
        float s[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 8; ks += 2) {
          uint32_t ka[4], kb[4];
          const int d = ks * 16 + k_dof;
          ldsm_x4(kbase + swz_off(d >> 6, k_row, (d & 63) >> 3), ka);
          ldsm_x4(kbase + swz_off((d + 16) >> 6, k_row, ((d + 16) & 63) >> 3), kb);
          mma16816(s, ka, qb[ks][0], qb[ks][1]);
          mma16816(s2, kb, qb[ks + 1][0], qb[ks + 1][1]);
        }
        // online softmax over this warp's 16 tokens, heads hc and hc + 1
        const float x0 = tr < valid ? (s[0] + s2[0]) * sc : -CUDART_INF_F;
        const float x1 = tr < valid ? (s[1] + s2[1]) * sc : -CUDART_INF_F;
        const float x2 = tr + 8 < valid ? (s[2] + s2[2]) * sc : -CUDART_INF_F;
        const float x3 = tr + 8 < valid ? (s[3] + s2[3]) * sc : -CUDART_INF_F;
        const float mn0 = fmaxf(m0, quad_max(fmaxf(x0, x2)));
        const float mn1 = fmaxf(m1, quad_max(fmaxf(x1, x3)));
        float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f, al0 = 1.f, al1 = 1.f;
        if (mn0 != -CUDART_INF_F) {
          p0 = exp2f(x0 - mn0);
          p2 = exp2f(x2 - mn0);
          al0 = exp2f(m0 - mn0);
        }
        if (mn1 != -CUDART_INF_F) {
          p1 = exp2f(x1 - mn1);
          p3 = exp2f(x3 - mn1);
          al1 = exp2f(m1 - mn1);
        }
        l0 = l0 * al0 + quad_sum(p0 + p2);
        l1 = l1 * al1 + quad_sum(p1 + p3);
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[mt][0] *= al0;
          o[mt][1] *= al1;
          o[mt][2] *= al0;
          o[mt][3] *= al1;
        }
        const uint32_t pb0 = movmatrix_trans(pack_half2(p0, p1));  // tokens 0-7 of the warp
        const uint32_t pb1 = movmatrix_trans(pack_half2(p2, p3));  // tokens 8-15
        // O^T += V^T . P^T, 8 tiles of 16 dims
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d = mt * 16 + v_dof;
          uint32_t va[4];
          ldsm_x4_t(vbase + swz_off(d >> 6, v_row, (d & 63) >> 3), va);
          mma16816(o[mt], va, pb0, pb1);
        }
        if (partial) fence_proxy_async_smem();  // zero stores before the next TMA write
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == NST) {
          stage = 0;
          phase ^= 1u;
        }
      }

      // ---- merge the 4 warps' states -----------------------------------
      if (lane < 4) {
        s_wml[warp * 8 + hc] = make_float2(m0, l0);
        s_wml[warp * 8 + hc + 1] = make_float2(m1, l1);
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d = mt * 16 + (lane >> 2);
        float *w = s_wo + (warp * kHeadDim + d) * 8 + hc;
        *reinterpret_cast<float2 *>(w) = make_float2(o[mt][0], o[mt][1]);
        *reinterpret_cast<float2 *>(w + 8 * 8) = make_float2(o[mt][2], o[mt][3]);
      }
      consumer_sync();
      const int d = tid;  // 128 consumer threads, one output dim each
      float acc[G], mx[G], ls[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float m = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) m = fmaxf(m, s_wml[w * 8 + g].x);
        float l = 0.f, x = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float2 ml = s_wml[w * 8 + g];
          const float sc_w = ml.x == -CUDART_INF_F ? 0.f : exp2f(ml.x - m);
          l = fmaf(ml.y, sc_w, l);
          x = fmaf(s_wo[(w * kHeadDim + d) * 8 + g], sc_w, x);
        }
        acc[g] = x;
        mx[g] = m;
        ls[g] = l;
      }
      if (it.nsplit == 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          store_out(a, it.b, h0 + g, d, acc[g], ls[g]);
          if (d == 0) store_lse(a, it.b, h0 + g, mx[g], ls[g]);
        }
      } else {
        float *po = a.part_o + static_cast<int64_t>(it.slot) * G * kHeadDim;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          __stcg(po + g * kHeadDim + d, acc[g]);
          if (d == 0) __stcg(a.part_ml + static_cast<int64_t>(it.slot) * G + g, make_float2(mx[g], ls[g]));
        }
      }
    }
    // ---- completion tickets (split pieces) and deferred combine -----------
    consumer_sync();  // partial stores of every consumer thread precede the ticket
    if (tid == 0) {
      s_flag[0] = 0;
      if (pend) {
        if (pend_ticket == pend_nsplit - 1) {
          s_flag[0] = 1;
          s_flag[1] = pend_b;
          s_flag[2] = pend_kvh;
          s_flag[3] = pend_nsplit;
          s_flag[4] = pend_first;
        }
        pend = false;
      }
      if (live && it.nsplit > 1) {
        // releases this CTA's partial (cumulative over the barrier above)
        pend_ticket = atomic_add_acq_rel_gpu(a.counters + it.pair, 1);
        pend = true;
        pend_b = it.b;
        pend_kvh = it.kvh;
        pend_nsplit = it.nsplit;
        pend_first = it.first_slot;
      }
      s_flag[5] = live || pend;  // one drain round settles the last ticket
    }
    consumer_sync();
    if (s_flag[0]) {
      Item cit;
      cit.b = s_flag[1];
      cit.kvh = s_flag[2];
      cit.nsplit = s_flag[3];
      cit.split = cit.p = cit.p_end = cit.ctx = 0;
      __threadfence();  // acquire the other CTAs' partials
      if (cit.nsplit <= 4)
        combine_partials_regs<G, 4>(a, cit, s_flag[4], tid);
      else
        combine_partials_staged<G, kConsumerWarps * 32>(a, cit, s_flag[4], tid, s_wo,
                                                        kConsumerWarps * kHeadDim * 8, consumer_sync);
      if (tid == 0) atomicExch(a.counters + cit.b * a.hkv + cit.kvh, 0);
    }
    const bool more = s_flag[5] != 0;
    consumer_sync();  // s_wo / s_wml / flags are reused by the next round
    if (!more) break;
  }
}

template <int G, int NST>
int launch_mma(const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a, int partitions,
               cudaStream_t stream) {
  using L = MmaSmem<NST>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  auto kern = decode_mma_kernel<G, NST>;
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  static int configured[64] = {0};
  if (!__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    B200KV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  // one partition (CTA) per SM by default; `partitions` overrides the count
  const int grid = partitions > 0 ? partitions : sms;
  a.target_items = grid;
  kern<<<grid, kMmaThreads, L::kAlloc, stream>>>(km, vm, a);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}

#ifndef B200KV_MMA_STAGES
#define B200KV_MMA_STAGES 5
#endif
constexpr int kMmaStages = B200KV_MMA_STAGES;  // 5 stages (160 KiB) fit beside the q slots

}  // namespace

int launch_decode_mma(int group, const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a,
                      int partitions, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_mma<1, kMmaStages>(km, vm, a, partitions, stream);
    case 2: return launch_mma<2, kMmaStages>(km, vm, a, partitions, stream);
    case 4: return launch_mma<4, kMmaStages>(km, vm, a, partitions, stream);
    case 8: return launch_mma<8, kMmaStages>(km, vm, a, partitions, stream);
    default: return set_error(B200KV_ERR_UNSUPPORTED, "group %d", group);
  }
}

}  // namespace b200kv
