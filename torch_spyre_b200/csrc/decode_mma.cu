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
// CTA = 1 producer warp + 4 consumer warps + 2 epilogue warps, one CTA per SM
// (persistent).  Work partition: the balanced unit split of decode_common.cuh
// (every CTA streams the same number of pages; a sequence-head cut by a CTA
// boundary is a split).
//   producer  walks this CTA's pieces page by page: block ids are fetched 32 at
//             a time by the whole warp; lane 0 writes a small descriptor per
//             stage (piece, page, flags), issues two 3-D TMA loads per page
//             (K, V; 16 KiB each, 128-byte swizzle, L2 evict-first) and, with
//             the first page of a piece, one bulk copy per q row, into an
//             NST-stage ring with "full"/"empty" mbarriers;
//   consumers take the ring's stages in turn: warp w processes the whole
//             pages of stages w, w + 4, w + 8, ... (and only reads the
//             descriptors of the others), each with its own online-softmax
//             state per piece, so no CTA barrier is taken per page.  Per page:
//               S^T[64 t x 8 h] = K[64 t x 128 d] . Q^T   (four 16-token MMA
//                                 chains, ldmatrix at precomputed offsets)
//               mask t >= ctx, one exp2-domain online-softmax update for the
//               page (quad shuffles)
//               P^T fragments from S^T by movmatrix.trans
//               O^T[128 d x 8 h] += V^T[128 d x 64 t] . P^T (ldmatrix.trans,
//                                 eight dim tiles x four token steps)
//             then one arrive on the stage's empty barrier; at the end of a
//             piece the warp drops its state into one of two piece buffers
//             and goes on with its next page;
//   epilogue  merges the 4 warps' states of a finished piece, writes the fp16
//             output (unsplit pair) or the fp32 partial, takes the pair's
//             completion ticket and, holding the last one, merges the pair's
//             partials (online log-sum-exp, decode_common.cuh).  Two epilogue
//             warps take the pieces in turn (warp e owns piece buffer e), so a
//             piece whose merge waits on L2 round trips does not hold up the
//             next one -- the CTA's final piece in particular.
//
// Fused append (kAppend) may also apply the rotary embedding (rope.cuh) of
// position context_len - 1 to q and to the new K row: q in its MMA fragments
// (dims j and j + 64 sit in the same lane, in steps ks and ks + 4), the K row
// in the append path (16-byte chunks c and c ^ 8 meet by one shuffle).
//
// FP8 pages (kFp8): the pools hold e4m3 values, one 128-byte stick per token
// row (8 KiB pages).  The consumers widen them to fp16 in registers (exact) and
// run the same fp16 MMAs; because both contractions are sums, the order of
// their reduction index inside a fragment is free:
//   K: ldmatrix on the fp8 rows gives lane (r, j) bytes d = 4j..4j+3 of a
//      16-byte chunk; they serve as fragment columns k = 2j, 2j+1 (low pair)
//      and 2j+8, 2j+9 (high pair), and the Q^T fragment is loaded with the
//      same order (fp16 elements 4j..4j+3 of the chunk);
//   V: ldmatrix.trans of the b16 view gives lane (i, j) tokens 2j, 2j+1 of
//      dims 2i, 2i+1; a byte permute splits them into dims 2i (fragment row
//      i) and 2i+1 (row i + 8), so O^T row r of m-tile mt is d = 16 mt + 2r
//      and row r + 8 is d = 16 mt + 2r + 1.
// The K scale folds into the softmax scale, the V scale into the epilogue.
#include "decode_kernels.h"
#include "fp8.cuh"
#include "rope.cuh"

namespace b200kv {
namespace {

constexpr int kConsumerWarps = 4;

constexpr int kEpilogueWarps = 2;
constexpr int kProducerWarp = kConsumerWarps;      // warp 4
constexpr int kEpilogueWarp = kConsumerWarps + 1;  // warps 5, 6
constexpr int kMmaThreads = (kConsumerWarps + 1 + kEpilogueWarps) * 32;

// Staged q of one piece: G rows of 128 fp16, row stride padded to 272 B so
// the Q^T fragment loads (8 heads x 4 lanes) hit 32 distinct banks.
constexpr int kQRowBytes = 272;
constexpr int kQSlotBytes = 8 * kQRowBytes;

// Hand-off of a finished piece from the consumer warps to an epilogue warp:
// every warp's unnormalised output rows O [8 h][128 d], its (max, sum) per
// head and the piece's identity.  Piece k goes to buffer k & 1, which
// epilogue warp k & 1 drains.  Rows are padded to 132 floats: the consumers'
// scalar writes (lanes of 8 dims x 4 head pairs) fall in 32 distinct banks,
// and the epilogue reads 4 consecutive dims per lane with one conflict-free
// 16-byte load.
struct PieceHeader {
  int b, kvh, pair, nsplit, slot, end, tail, own_first;
};
constexpr int kPieceRow = kHeadDim + 4;
constexpr int kPieceO = 0;                                    // float [4][8][kPieceRow]
constexpr int kPieceML = kConsumerWarps * 8 * kPieceRow * 4;  // float2 [4][8]
constexpr int kPieceHdr = kPieceML + kConsumerWarps * 8 * 8;
constexpr int kPieceBytes = (kPieceHdr + 64 + 127) & ~127;
constexpr int kPieceBufs = kEpilogueWarps;

template <int NST, bool kFp8>
struct MmaSmem {
  static constexpr int kPage = kFp8 ? kPageBytesFp8 : kPageBytes;
  static constexpr int kStageBytes = 2 * kPage;                          // K page + V page
  static constexpr int kQ = NST * kStageBytes;                           // q slot per stage
  static constexpr int kPiece = kQ + NST * kQSlotBytes;                  // piece buffers
  static constexpr int kNew = kPiece + kPieceBufs * kPieceBytes;         // new K+V row per stage
  static constexpr int kDesc = kNew + NST * 2 * kHeadDim * 2;            // StageDesc [NST]
  static constexpr int kPlan = kDesc + NST * 48;
  static constexpr int kBars = (kPlan + kPlanBytes + 7) & ~7;  // full, empty [NST]; pfull, pempty [2]
  static constexpr int kBytes = kBars + (2 * NST + 2 * kPieceBufs) * 8;
  static constexpr int kAlloc = kBytes + 1024;
};

// What one stage carries, written by the producer before it arms the stage's
// full barrier: the piece (pair, slot, split count), the page and flags.
struct StageDesc {
  int b, kvh, pair, page, ctx, nsplit, slot, flags, blk, pad[3];
};
constexpr int kDescFirst = 1;  // first page of a piece
constexpr int kDescLast = 2;   // last page of a piece
constexpr int kDescPage = 4;   // the stage holds a page (an empty sequence has none)
constexpr int kDescEnd = 8;    // no more work for this CTA
constexpr int kDescNew = 16;   // the stage carries the appended token's K/V rows
constexpr int kDescTail = 32;  // the page belongs to the CTA's final piece
constexpr int kDescOwnFirst = 64;  // the piece holds its pair's lowest partial slot

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
__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

template <int G, int NST, bool kAppend, bool kFp8>
__global__ void __launch_bounds__(kMmaThreads, 1)
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  static_assert(G >= 1 && G <= 8, "the head group sits in one n = 8 MMA tile");
  using L = MmaSmem<NST, kFp8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  StageDesc *descs = reinterpret_cast<StageDesc *>(smem + L::kDesc);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBars);
  uint64_t *empty = full + NST;
  uint64_t *pfull = empty + NST;         // piece handed to the epilogue (4 arrivals)
  uint64_t *pempty = pfull + kPieceBufs; // piece buffer free again (1 arrival)
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
    for (int s = 0; s < kPieceBufs; ++s) {
      mbar_init(&pfull[s], kConsumerWarps);
      mbar_init(&pempty[s], 1);
    }
    fence_mbar_init();
  }
  // Programmatic dependent launch.  Nothing above reads global memory.  By
  // default every thread waits here for the preceding grid on the stream to
  // finish (a no-op when this launch has no programmatic predecessor).  With
  // an early start the plan and the producer's first NST stages of page
  // loads run before the wait -- they read only inputs written before the
  // preceding kernel began -- and every role waits before it touches q, the
  // appended rows, the scales, the workspace, the pools' new rows or the
  // outputs.  The next grid may be scheduled at once so its CTAs take over
  // SMs as soon as ours exit (it waits for this grid before it reads what
  // this grid writes, unless its own caller vouched that it does not).
  const bool early = a.early != 0;
  if (!early) asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  build_unit_plan<kMmaThreads>(a, pl);  // synchronises the CTA
  const Partition P = make_partition(pl.total_items, static_cast<int>(gridDim.x));
  const int c = blockIdx.x;

  // ------------------------------------------------------------ producer --
  // Streams this CTA's range of units.  Per page: the whole warp fetches block ids 32 at
  // a time in one coalesced load; lane 0 waits for the stage to be free,
  // writes its descriptor, arms its full barrier and issues the two page
  // loads, plus, with the first page of a piece, one bulk copy per q row.
  if (warp == kProducerWarp) {
    const uint64_t policy = l2_policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    // early start: the stages issued before griddepcontrol.wait -- stages
    // 0 .. issued - 1, at most one trip round the ring -- get their q rows and
    // appended rows after it (their full barriers already expect those bytes;
    // their descriptors stay in place until those bytes land)
    bool waited = !early;
    int issued = 0;
    auto q_rows = [&](int st, const __half *qg) {
      uint8_t *qs = smem + L::kQ + st * kQSlotBytes;
#pragma unroll
      for (int g = 0; g < G; ++g) bulk_load(qs + g * kQRowBytes, qg + g * a.q_sh, kHeadDim * 2, &full[st]);
    };
    auto new_rows = [&](int st, int64_t off) {
      uint8_t *ns = smem + L::kNew + st * 2 * kHeadDim * 2;
      bulk_load(ns, a.k_new + off, kHeadDim * 2, &full[st]);
      bulk_load(ns + kHeadDim * 2, a.v_new + off, kHeadDim * 2, &full[st]);
    };
    auto finish_wait = [&]() {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      waited = true;
      for (int st = 0; st < issued; ++st) {
        const StageDesc &d = descs[st];
        if (kAppend && (d.flags & kDescNew)) new_rows(st, d.b * a.new_sb + d.kvh * a.new_sh);
        if ((d.flags & (kDescFirst | kDescPage)) == (kDescFirst | kDescPage))
          q_rows(st, a.q + d.b * a.q_sb + (d.kvh * G) * a.q_sh);
      }
    };
    auto emit_range = [&](int u_lo, int u_hi, int owner) {
      for (int u = u_lo; u < u_hi;) {
        const Piece pc = locate_piece(a, pl, P, u, u_hi, owner);
        u = pc.u_next;
        // kDescTail: the CTA's final piece; kDescOwnFirst: the piece starts at
        // the pair's first page, so it holds the pair's lowest partial slot
        const int tail_flag = (u >= u_hi ? kDescTail : 0) | (pc.p == 0 ? kDescOwnFirst : 0);
        const int npages = pc.p_end - pc.p;
        const int nstages = max(npages, 1);  // an empty sequence still takes one stage
        for (int base = 0; base < nstages; base += 32) {
          const int n = min(32, nstages - base);
          const int my_raw = (lane < n && npages > 0) ? page_block_raw(a, pc.b, pc.p + base + lane) : 0;
          const int my_blk = (my_raw < 0 || my_raw >= a.num_blocks) ? page_block(a, pc.b, pc.p + base + lane) : my_raw;
          for (int j = 0; j < n; ++j) {
            const int blk = __shfl_sync(0xffffffffu, my_blk, j);
            const int raw = kAppend ? __shfl_sync(0xffffffffu, my_raw, j) : 0;
            if (lane == 0) {
              mbar_wait_bounded(&empty[stage], phase ^ 1u, a.error_flag);
              const int i = base + j;
              const bool has = npages > 0;
              StageDesc &d = descs[stage];
              d.b = pc.b;
              d.kvh = pc.kvh;
              d.pair = pc.pair;
              d.page = pc.p + i;
              d.ctx = pc.ctx;
              d.nsplit = pc.nsplit;
              d.slot = pc.slot;
              // the appended token (position ctx - 1) lies on this page
              const bool app = kAppend && has && (pc.ctx - 1) / kPageTokens == pc.p + i;
              if (kAppend) d.blk = (raw >= 0 && raw < a.num_blocks) ? raw : -1;
              d.flags = (i == 0 ? kDescFirst : 0) | (i == nstages - 1 ? kDescLast : 0) |
                        (has ? kDescPage : 0) | (app ? kDescNew : 0) | tail_flag;
              uint32_t tx = has ? 2 * L::kPage : 0;
              if (has && i == 0) tx += G * kHeadDim * 2;
              if (app) tx += 2 * kHeadDim * 2;
              mbar_arrive_expect_tx(&full[stage], tx);
              // q rows (first page of a piece) and the appended token's rows ride
              // on the stage's barrier; before the wait they are deferred
              if (waited) {
                if (kAppend && app) new_rows(stage, pc.b * a.new_sb + pc.kvh * a.new_sh);
                if (has && i == 0) q_rows(stage, a.q + pc.b * a.q_sb + (pc.kvh * G) * a.q_sh);
              }
              if (has) {
                uint8_t *dst = smem + stage * L::kStageBytes;
                const int page = blk * a.hkv + pc.kvh;
                tma_load_3d(dst, &kmap, &full[stage], 0, 0, page, policy);
                tma_load_3d(dst + L::kPage, &vmap, &full[stage], 0, 0, page, policy);
              }
              if (!waited && ++issued == NST) finish_wait();
            }
            if (++stage == NST) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
    };
    emit_range(P.lo(c), P.hi(c), c);
    if (lane == 0 && !waited) finish_wait();
    if (lane == 0) {  // end marker
      mbar_wait_bounded(&empty[stage], phase ^ 1u, a.error_flag);
      descs[stage].flags = kDescEnd;
      mbar_arrive_expect_tx(&full[stage], 0);
    }
    return;
  }

  // ------------------------------------------------------------ epilogue --
  // Takes finished pieces from the consumers: merges the 4 warps' states,
  // writes the fp16 output (single piece) or the fp32 partial, takes the
  // pair's completion ticket and, holding the last one, merges the pair's
  // partials.  Epilogue warp e takes pieces e, e + 2, e + 4, ... from buffer
  // e.  Runs beside the consumers, which never wait for it unless a warp
  // falls a whole piece behind.
  if (early) asm volatile("griddepcontrol.wait;" ::: "memory");  // consumers and epilogue
  if (warp >= kEpilogueWarp) {
    const float vsc = kFp8 ? __half2float(*a.v_scale) : 1.f;  // V dequantisation scale
    const int pb = warp - kEpilogueWarp;
    for (uint32_t j = 0;; ++j) {
      mbar_wait_bounded(&pfull[pb], j & 1u, a.error_flag);
      const uint8_t *buf = smem + L::kPiece + pb * kPieceBytes;
      const PieceHeader hd = *reinterpret_cast<const PieceHeader *>(buf + kPieceHdr);
      if (hd.end) break;
      const float *wo = reinterpret_cast<const float *>(buf + kPieceO);
      const float2 *wml = reinterpret_cast<const float2 *>(buf + kPieceML);
      // lane l holds dims 4l .. 4l + 3 of every head
      float acc[G][4], mx[G], ls[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float m = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) m = fmaxf(m, wml[w * 8 + g].x);
        float l = 0.f, x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float2 ml = wml[w * 8 + g];
          const float sw = ml.x == -CUDART_INF_F ? 0.f : exp2f(ml.x - m);
          l = fmaf(ml.y, sw, l);
          const float4 v = reinterpret_cast<const float4 *>(wo + (w * 8 + g) * kPieceRow)[lane];
          x[0] = fmaf(v.x, sw, x[0]);
          x[1] = fmaf(v.y, sw, x[1]);
          x[2] = fmaf(v.z, sw, x[2]);
          x[3] = fmaf(v.w, sw, x[3]);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) acc[g][kk] = kFp8 ? x[kk] * vsc : x[kk];
        mx[g] = m;
        ls[g] = l;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[pb]);  // buffer read: the consumers may refill it
      const int h0 = hd.kvh * G;
      if (hd.nsplit == 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          store_out4_inv(a, hd.b, h0 + g, 4 * lane, acc[g], inv_sum(ls[g]));
          if (lane == 0) store_lse(a, hd.b, h0 + g, mx[g], ls[g]);
        }
        continue;
      }
      // every other piece of the pair already in (their partials stored and
      // fenced before their tickets): this piece is the last, so it merges
      // its own state with their partials at once -- no store, fence, ticket
      // or reload of its own partial.  Each lane's acquire load sees the
      // counter; any lane that saw less sends the piece down the ticket path.
      // (tried on the CTA's final piece only: the pair it starts was finished
      // early by the next CTA, so it is almost always the pair's last)
      // Every merge folds the pair's partials in ascending slot order from the
      // empty state, so the output bits do not depend on which piece merges:
      // this shortcut starts from the piece's own state only when it holds
      // the pair's lowest slot.
      if (hd.tail && hd.own_first &&
          __all_sync(0xffffffffu, ld_acquire_gpu(a.counters + hd.pair) == hd.nsplit - 1)) {
        int pj, w;
        pair_units(a, pl, hd.pair, &pj, &w);
        combine_online_warp_from<G>(a, hd.b, hd.kvh, pair_slots(P, hd.pair, pj, w), lane, hd.slot, mx, ls, acc);
        if (lane == 0) atomicExch(a.counters + hd.pair, 0);
        continue;
      }
      float *po = a.part_o + static_cast<int64_t>(hd.slot) * G * kHeadDim;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        __stcg(reinterpret_cast<float4 *>(po + g * kHeadDim) + lane,
               make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]));
        if (lane == 0) __stcg(a.part_ml + static_cast<int64_t>(hd.slot) * G + g, make_float2(mx[g], ls[g]));
      }
      __syncwarp();  // the warp's partial stores precede lane 0's release
      int ticket = 0;
      if (lane == 0) {
        __threadfence();
        ticket = atomicAdd(a.counters + hd.pair, 1);
      }
      ticket = __shfl_sync(0xffffffffu, ticket, 0);
      if (ticket == hd.nsplit - 1) {  // last piece of the pair: merge all partials
        __threadfence();
        int pj, w;
        pair_units(a, pl, hd.pair, &pj, &w);
        combine_online_warp<G>(a, hd.b, hd.kvh, pair_slots(P, hd.pair, pj, w), lane);
        if (lane == 0) atomicExch(a.counters + hd.pair, 0);
      }
    }
    return;
  }

  // ----------------------------------------------------------- consumers --
  // The stages are taken in turn: warp w processes the pages of stages
  // number w, w + 4, w + 8, ... (counted from the kernel start) and passes
  // over the others after reading their descriptors.  Each warp keeps its own
  // online-softmax state per piece.
  const int mi = lane >> 3;          // ldmatrix: which 8x8 matrix this lane addresses
  const int mr = lane & 7;           // ldmatrix: row within that matrix
  const int qh = lane >> 2;          // head of this lane's Q^T fragment (n index)
  const int hc = (lane & 3) * 2;     // heads of this lane's accumulator columns
  const int tr = lane >> 2;          // token (within a 16-token tile) of this lane's S^T rows (and +8)
  const float sc = kFp8 ? a.scale_log2 * __half2float(*a.k_scale) : a.scale_log2;
  __half2 kinv = {}, vinv = {};      // fp8 fused append: quantisation scales of the new rows
  if (kFp8 && kAppend) {
    kinv = fp8_inv_scale2(*a.k_scale);
    vinv = fp8_inv_scale2(*a.v_scale);
  }
  // Byte offsets, in a staged page, of this lane's ldmatrix rows.  Token tile
  // mt (16 tokens) adds 2048 * mt: its rows share the swizzle phase (row & 7).
  //   fp16 K (non-transposed, A of S^T = K Q^T): 16-dim step ks
  //   fp16 V (transposed, A = V^T of O^T = V^T P^T): 16-dim tile mt
  //   fp8 K and V: 32-dim step cc (chunk pair 2cc, 2cc + 1)
  uint32_t koff[kFp8 ? 4 : 8], voff[kFp8 ? 4 : 8];
  if (kFp8) {
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) koff[cc] = voff[cc] = swz_off(0, mr + (mi & 1) * 8, 2 * cc + (mi >> 1));
  } else {
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int dk = ks * 16 + (mi >> 1) * 8;
      koff[ks] = swz_off(dk >> 6, mr + (mi & 1) * 8, (dk & 63) >> 3);
      const int dv = ks * 16 + (mi & 1) * 8;
      voff[ks] = swz_off(dv >> 6, mr + (mi >> 1) * 8, (dv & 63) >> 3);
    }
  }

  // Hands this warp's state of the finished piece (or an end marker) to
  // epilogue warp k & 1 through piece buffer k & 1.
  auto hand_off = [&](int k, const StageDesc &d, bool end, const float (&o)[8][4], float m0,
                      float m1, float l0, float l1) {
    const int pb = k & 1;
    mbar_wait_bounded(&pempty[pb], ((k >> 1) & 1) ^ 1u, a.error_flag);
    uint8_t *buf = smem + L::kPiece + pb * kPieceBytes;
    if (!end) {
      float *wo = reinterpret_cast<float *>(buf + kPieceO);
      float2 *wml = reinterpret_cast<float2 *>(buf + kPieceML);
      if (lane < 4) {
        wml[warp * 8 + hc] = make_float2(m0, l0);
        wml[warp * 8 + hc + 1] = make_float2(m1, l1);
      }
      // accumulator rows of m-tile mt: d = 16 mt + r and + 8 (fp16 pages),
      // d = 16 mt + 2r and + 1 (fp8 pages), r = lane / 4; columns: heads hc, hc + 1
      float *w0 = wo + (warp * 8 + hc) * kPieceRow;
      float *w1 = w0 + kPieceRow;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int dd = mt * 16 + (kFp8 ? 2 * (lane >> 2) : (lane >> 2));
        const int d2 = dd + (kFp8 ? 1 : 8);
        w0[dd] = o[mt][0];
        w1[dd] = o[mt][1];
        w0[d2] = o[mt][2];
        w1[d2] = o[mt][3];
      }
    }
    if (warp == 0 && lane == 0) {
      PieceHeader *hd = reinterpret_cast<PieceHeader *>(buf + kPieceHdr);
      hd->b = d.b;
      hd->kvh = d.kvh;
      hd->pair = d.pair;
      hd->nsplit = d.nsplit;
      hd->slot = d.slot;
      hd->end = end;
      hd->tail = (d.flags & kDescTail) != 0;
      hd->own_first = (d.flags & kDescOwnFirst) != 0;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&pfull[pb]);
  };

  uint32_t qb[8][2];
  float o[8][4];
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;

  // Row of the rotary table for a sequence of `ctx` tokens (its new token at
  // ctx - 1); out of range is flagged and clamped.
  auto rope_pos = [&](int ctx) -> int64_t {
    int64_t pos = int64_t(ctx) - 1;
    if (pos < 0 || pos >= a.rope_max_pos) {
      if (lane == 0 && a.error_flag) atomicOr(a.error_flag, B200KV_DEVERR_BAD_LEN);
      pos = pos < 0 ? 0 : a.rope_max_pos - 1;
    }
    return pos;
  };

  // The appended token's rows replace the staged ones (the page's warp writes
  // them into the stage's K/V pages and into the pools).
  auto apply_append = [&](int st, const StageDesc &dd) {
    const int t_new = (dd.ctx - 1) % kPageTokens;
    const int c = lane & 15;  // 16-byte chunk of the row; lanes 0-15 K, 16-31 V
    const int kv = lane >> 4;
    const uint8_t *src = smem + L::kNew + st * 2 * kHeadDim * 2 + kv * kHeadDim * 2 + c * 16;
    uint4 v = *reinterpret_cast<const uint4 *>(src);
    if (a.rope_freqs != nullptr) {  // rotate the K row: chunk c pairs with chunk c ^ 8
      uint32_t w[4] = {v.x, v.y, v.z, v.w}, pw[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pw[i] = __shfl_xor_sync(0xffffffffu, w[i], 8);
      if (kv == 0) {
        const __half *f = a.rope_freqs + rope_pos(dd.ctx) * 4 * (kHeadDim / 2);
        const bool lo = c < 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t x0 = lo ? w[i] : pw[i], x1 = lo ? pw[i] : w[i];
          rope_pair(f, kHeadDim / 2, 8 * (c & 7) + 2 * i, x0, x1);
          w[i] = lo ? x0 : x1;
        }
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    if (kFp8) {  // quantise: dims 8c..8c+7 are bytes 8c..8c+7 of the page row
      const uint2 q8 = quantize8_e4m3(v, kv ? vinv : kinv);
      *reinterpret_cast<uint2 *>(smem + st * L::kStageBytes + kv * L::kPage + swz_off(0, t_new, c >> 1) +
                                 (c & 1) * 8) = q8;
      if (dd.blk >= 0) {
        uint8_t *pool = kv ? a.v_pool8_w : a.k_pool8_w;
        const int64_t off =
            ((static_cast<int64_t>(dd.blk) * a.hkv + dd.kvh) * kPageTokens + t_new) * kHeadDim + c * 8;
        *reinterpret_cast<uint2 *>(pool + off) = q8;
      }
    } else {
      *reinterpret_cast<uint4 *>(smem + st * L::kStageBytes + kv * kPageBytes + swz_off(c >> 3, t_new, c & 7)) =
          v;
      if (dd.blk >= 0) {
        __half *pool = kv ? a.v_pool_w : a.k_pool_w;
        const int64_t off = ((static_cast<int64_t>(dd.blk) * a.hkv + dd.kvh) * kSticks + (c >> 3)) *
                                (kPageTokens * kStickElems) +
                            t_new * kStickElems + (c & 7) * 8;
        *reinterpret_cast<uint4 *>(pool + off) = v;
      }
    }
    __syncwarp();
  };

  int stage = 0, piece = 0, seq = 0;
  uint32_t phase = 0;
  for (;; ++seq) {
    mbar_wait_bounded(&full[stage], phase, a.error_flag);
    const StageDesc d = descs[stage];
    if (d.flags & kDescEnd) {  // one end marker per epilogue warp
      hand_off(piece, d, true, o, m0, m1, l0, l1);
      hand_off(piece + 1, d, true, o, m0, m1, l0, l1);
      break;
    }
    const bool first = d.flags & kDescFirst, last = d.flags & kDescLast;
    const bool has = d.flags & kDescPage;
    if (first) {
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      m0 = m1 = -CUDART_INF_F;
      l0 = l1 = 0.f;
      if (has) {  // q of this piece, staged with its first page (every warp reads it)
        // fragment columns 2j, 2j+1 / 2j+8, 2j+9 of each 16-dim step are dims
        // 2j, 2j+1 / 2j+8, 2j+9 (fp16 pages) or 4j..4j+3 (fp8 pages)
        const uint32_t qs = smem_u32(smem + L::kQ + stage * kQSlotBytes) + qh * kQRowBytes +
                            (kFp8 ? 4 * (lane & 3) : hc) * 2;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          uint32_t x0 = 0u, x1 = 0u;
          if (qh < G) {
            asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x0) : "r"(qs + ks * 32));
            asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x1) : "r"(qs + ks * 32 + (kFp8 ? 4 : 16)));
          }
          qb[ks][0] = x0;
          qb[ks][1] = x1;
        }
        if (kAppend && a.rope_freqs != nullptr) {  // rotate q: dims e and e + 64 are steps ks, ks + 4
          const __half *f = a.rope_freqs + rope_pos(d.ctx) * 4 * (kHeadDim / 2);
          if (qh < G) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const int e0 = kFp8 ? 16 * ks + 4 * (lane & 3) : 16 * ks + hc;
              rope_pair(f, kHeadDim / 2, e0, qb[ks][0], qb[ks + 4][0]);
              rope_pair(f, kHeadDim / 2, kFp8 ? e0 + 2 : e0 + 8, qb[ks][1], qb[ks + 4][1]);
            }
          }
        }
      }
    }
    if (has && (seq & (kConsumerWarps - 1)) == warp) {  // this warp's page
      bool wrote_smem = false;
      if (kAppend && (d.flags & kDescNew)) {
        apply_append(stage, d);
        wrote_smem = true;
      }
      const uint32_t kbase = smem_u32(smem + stage * L::kStageBytes);
      const uint32_t vbase = kbase + L::kPage;
      const int valid = min(kPageTokens, d.ctx - d.page * kPageTokens);
      if (valid < kPageTokens) {  // zero the V rows past the context (0 * NaN = NaN in the MMA)
        constexpr int kRowChunks = kFp8 ? 8 : 16;
        for (int idx = valid * kRowChunks + lane; idx < kPageTokens * kRowChunks; idx += 32) {
          const int t = idx / kRowChunks, cc = idx % kRowChunks;
          st_shared_zero16(vbase + (kFp8 ? swz_off(0, t, cc) : swz_off(cc >> 3, t, cc & 7)));
        }
        __syncwarp();
        wrote_smem = true;
      }
      // S^T [64 t x 8 h] = K . Q^T: four token tiles, one accumulation chain each
      float sacc[4][4];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) sacc[mt][0] = sacc[mt][1] = sacc[mt][2] = sacc[mt][3] = 0.f;
      if (kFp8) {
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            uint32_t x[4], ka[4], kc[4];
            ldsm_x4(kbase + koff[cc] + 2048 * mt, x);
            // {dims 4j, 4j+1 | 4j+2, 4j+3} of rows r (x0, x2) and r + 8 (x1, x3)
            e4m3x4_to_half2x2(x[0], ka[0], ka[2]);
            e4m3x4_to_half2x2(x[1], ka[1], ka[3]);
            e4m3x4_to_half2x2(x[2], kc[0], kc[2]);
            e4m3x4_to_half2x2(x[3], kc[1], kc[3]);
            mma16816(sacc[mt], ka, qb[2 * cc][0], qb[2 * cc][1]);
            mma16816(sacc[mt], kc, qb[2 * cc + 1][0], qb[2 * cc + 1][1]);
          }
        }
      } else {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            uint32_t ka[4];
            ldsm_x4(kbase + koff[ks] + 2048 * mt, ka);
            mma16816(sacc[mt], ka, qb[ks][0], qb[ks][1]);
          }
        }
      }
      // online softmax over the page's 64 tokens, heads hc and hc + 1
      float mx0 = -CUDART_INF_F, mx1 = -CUDART_INF_F;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const int t = mt * 16 + tr;
        sacc[mt][0] = t < valid ? sacc[mt][0] * sc : -CUDART_INF_F;
        sacc[mt][1] = t < valid ? sacc[mt][1] * sc : -CUDART_INF_F;
        sacc[mt][2] = t + 8 < valid ? sacc[mt][2] * sc : -CUDART_INF_F;
        sacc[mt][3] = t + 8 < valid ? sacc[mt][3] * sc : -CUDART_INF_F;
        mx0 = fmaxf(mx0, fmaxf(sacc[mt][0], sacc[mt][2]));
        mx1 = fmaxf(mx1, fmaxf(sacc[mt][1], sacc[mt][3]));
      }
      const float mn0 = fmaxf(m0, quad_max(mx0));
      const float mn1 = fmaxf(m1, quad_max(mx1));
      const float e0 = mn0 == -CUDART_INF_F ? 0.f : mn0;  // exp2(-inf - 0) = 0 for an all-masked head
      const float e1 = mn1 == -CUDART_INF_F ? 0.f : mn1;
      const float al0 = exp2f(m0 - e0), al1 = exp2f(m1 - e1);
      float ps0 = 0.f, ps1 = 0.f;
      uint32_t pfr[4][2];  // P^T fragments of the four token tiles
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const float p0 = exp2f(sacc[mt][0] - e0), p1 = exp2f(sacc[mt][1] - e1);
        const float p2 = exp2f(sacc[mt][2] - e0), p3 = exp2f(sacc[mt][3] - e1);
        ps0 += p0 + p2;
        ps1 += p1 + p3;
        pfr[mt][0] = movmatrix_trans(pack_half2(p0, p1));  // tokens 0-7 of the tile
        pfr[mt][1] = movmatrix_trans(pack_half2(p2, p3));  // tokens 8-15
      }
      l0 = l0 * al0 + quad_sum(ps0);
      l1 = l1 * al1 + quad_sum(ps1);
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
      }
      // O^T [128 d x 8 h] += V^T . P^T: eight dim tiles, four token steps each
      if (kFp8) {
        // ldmatrix.trans (b16 view) of a token tile x chunk pair 2cc, 2cc+1;
        // byte permute {t2j d2i, t2j d2i+1, t2j+1 d2i, t2j+1 d2i+1} ->
        // {d2i: t2j, t2j+1 | d2i+1: t2j, t2j+1}
#pragma unroll
        for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t x[4], va[4], vc[4];
            ldsm_x4_t(vbase + voff[cc] + 2048 * kt, x);
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = __byte_perm(x[i], 0u, 0x3120);
            e4m3x4_to_half2x2(x[0], va[0], va[1]);
            e4m3x4_to_half2x2(x[1], va[2], va[3]);
            e4m3x4_to_half2x2(x[2], vc[0], vc[1]);
            e4m3x4_to_half2x2(x[3], vc[2], vc[3]);
            mma16816(o[2 * cc], va, pfr[kt][0], pfr[kt][1]);
            mma16816(o[2 * cc + 1], vc, pfr[kt][0], pfr[kt][1]);
          }
        }
      } else {
#pragma unroll
        for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            uint32_t va[4];
            ldsm_x4_t(vbase + voff[mt] + 2048 * kt, va);
            mma16816(o[mt], va, pfr[kt][0], pfr[kt][1]);
          }
        }
      }
      if (wrote_smem) fence_proxy_async_smem();  // st.shared before the next TMA write
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == NST) {
      stage = 0;
      phase ^= 1u;
    }
    if (last) hand_off(piece++, d, false, o, m0, m1, l0, l1);
  }
}

template <int G, int NST, bool kAppend, bool kFp8>
int launch_mma_impl(const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a, int partitions,
                    cudaStream_t stream) {
  using L = MmaSmem<NST, kFp8>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  auto kern = decode_mma_kernel<G, NST, kAppend, kFp8>;
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  static int configured[64] = {0};
  if (!__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    B200KV_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  // one CTA per SM by default; `partitions` (<= kMaxPartitions) overrides it
  const int grid = partitions > 0 ? partitions : sms;
  a.target_items = grid;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMmaThreads);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200KV_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, km, vm, a));
  return B200KV_OK;
}

#ifndef B200KV_MMA_STAGES
#define B200KV_MMA_STAGES 5
#endif
#ifndef B200KV_MMA_STAGES_FP8
#define B200KV_MMA_STAGES_FP8 8
#endif
constexpr int kMmaStages = B200KV_MMA_STAGES;        // fp16: 5 stages (160 KiB) beside the q slots
constexpr int kMmaStagesFp8 = B200KV_MMA_STAGES_FP8; // fp8: 8 stages (128 KiB)

template <int G>
int launch_mma(const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a, int partitions,
               cudaStream_t stream) {
  const bool app = a.k_new != nullptr;
  if (a.k_scale != nullptr)
    return app ? launch_mma_impl<G, kMmaStagesFp8, true, true>(km, vm, a, partitions, stream)
               : launch_mma_impl<G, kMmaStagesFp8, false, true>(km, vm, a, partitions, stream);
  return app ? launch_mma_impl<G, kMmaStages, true, false>(km, vm, a, partitions, stream)
             : launch_mma_impl<G, kMmaStages, false, false>(km, vm, a, partitions, stream);
}

}  // namespace

int launch_decode_mma(int group, const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a,
                      int partitions, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_mma<1>(km, vm, a, partitions, stream);
    case 2: return launch_mma<2>(km, vm, a, partitions, stream);
    case 4: return launch_mma<4>(km, vm, a, partitions, stream);
    case 8: return launch_mma<8>(km, vm, a, partitions, stream);
    default: return set_error(B200KV_ERR_UNSUPPORTED, "group %d", group);
  }
}

}  // namespace b200kv
