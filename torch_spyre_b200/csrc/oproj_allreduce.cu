// Fused o_proj GEMM + tensor-parallel all-reduce: out = sum over ranks of
// attn_r [B, K] . W_r[N, K]^T, one kernel per rank.
//
// The reference's TP step is the o_proj of each rank's heads followed by a SUM
// all-reduce of the [B, N] partial (SpyreCCLBackend::allreduce,
// torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494).  Here every CTA owns
// one 128 x 64 output tile (rows = the batch, zero-padded to 128 by the TMA).
//
// Split-K over a thread-block cluster of C CTAs (C = 1, 2 or 4): the cluster
// computes a 128 x 64C super-tile, CTA r of the cluster over the K blocks
// [r K/C, (r+1) K/C), so each SM pulls 1/C of the attn slab (the operand every
// CTA shares, read from L2) plus 64C rows of W over 1/C of K: 1 MB per SM at
// C = 2 instead of 1.5 MB.  The C partial super-tiles are reduce-scattered
// through distributed shared memory: after a cluster barrier (every CTA's MMAs
// are done, so its operand ring is free) CTA r stores its fp32 partial of
// column block q into CTA q's ring (st.shared::cluster), and after a second
// barrier each CTA sums the C partials of its own 128 x 64 tile in
// cluster-rank order.
//   warp 4   TMA producer: K-slabs of attn (128 x 64) and W (64C x 64), 128-byte
//            swizzle, into a ring with full/empty mbarriers;
//   warp 5   allocates 64C TMEM columns; one lane issues tcgen05.mma
//            (kind::f16, M = 128, N = 64C, K = 16, fp32 accumulate in TMEM) and
//            tcgen05.commit frees each stage and finally signals the tile;
//   warps 0-3  read the accumulator (tcgen05.ld, TMEM lane = row), reduce the
//            split (C > 1) and run the tile's all-reduce at once, so a tile's
//            exchange overlaps the other tiles' GEMM: the tile is owned by rank
//            tile / (T / N); a non-owner sends its fp16 partial rows to the
//            owner, the owner sums the N partials (rank order, fp32, rounded
//            once), writes its output rows and sends the sum to every other
//            rank, which polls it into its output.
// Transfers are the flagged 8-byte packets of peer_allreduce.cu (data + epoch,
// receiver polls, no fences, no multicast) in the same peer buffers, receive
// regions and epoch counter, so fused and unfused calls interleave.  Inside a
// tile's region packet j of row r sits at j * 128 + r, so a warp's stores and
// polls cover 512 contiguous bytes, and a row's packets are polled as a batch.  All CTAs
// are resident at once (checked on the host: N / 64 <= SMs for C = 1, enough
// co-resident clusters for C > 1), so no CTA waits on one that cannot run.
// Every mbarrier / packet wait is bounded (2 s); every thread of a cluster
// reaches both cluster barriers on every path; TMEM is freed on every path.
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace b200kv {
namespace {

constexpr int kOpM = 128, kOpN = 64, kOpK = 64;
constexpr int kOpATile = kOpM * kOpK * 2;  // 16 KiB
constexpr int kOpThreads = 192;
constexpr int kOpMaxRanks = 8;
constexpr int kOpPktPerRow = kOpN * 2 / 8;           // 16 packets of 8 data bytes per tile row
constexpr int kOpPktPerTile = kOpM * kOpPktPerRow;   // 2048

// Shapes of the split-K variant over a cluster of C CTAs.
template <int C>
struct OpCfg {
  static constexpr int kN = kOpN * C;                  // columns of the cluster's super-tile
  static constexpr int kBTile = kN * kOpK * 2;         // W slab: 8 KiB per CTA of the cluster
  static constexpr int kStage = kOpATile + kBTile;
  static constexpr int kStages = C == 4 ? 4 : 6;
  static constexpr int kRing = kStages * kStage;
  static constexpr int kSmem = kRing + 1024 + 256;
  static constexpr uint32_t kTmemCols = 64u * C;       // 128 lanes x 64C fp32 columns
  // kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both
  // K-major, N = 64C, M = 128.
  static constexpr uint32_t kIdesc = (1u << 4) | (uint32_t(kN >> 3) << 17) | (uint32_t(kOpM >> 4) << 24);
  // reduction slot of one source CTA: a 128 x 64 fp32 partial, 256 B per row
  static constexpr int kRecvSlot = kOpM * kOpN * 4;
  static_assert(C == 1 || C == 2 || C == 4, "cluster split of 1, 2 or 4");
  static_assert(C == 1 || C * kRecvSlot <= kRing, "the reduction slots reuse the operand ring");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

struct OpArgs {
  uint8_t *peers[kOpMaxRanks];
  int rank, world, tiles, batch;
  int kblocks;
  __half *out;
  int64_t out_sb;
  int64_t recv1_off, recv2_off, region_bytes, counter_off;
  int32_t *error_flag;
};

// K-major operand tile of 128-byte rows in the 128-byte swizzle (8-row atoms
// of 1024 bytes): start address >> 4, LBO 1 (unused for this layout), SBO
// 1024 >> 4, descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void st_volatile_v4(uint4 *p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_v4(const uint4 *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Receives kOpPktHalf packets of one tile row (packet j at p + j * stride;
// each packet is two 8-byte {data, epoch} words, complete when both carry
// `epoch`): the loads are issued at once and only the packets not yet complete
// are polled again, so packets that have arrived cost one memory round trip
// (polling them one by one would chain a round trip per packet).  Gives up
// after kWaitLimitNs (sets B200KV_DEVERR_TIMEOUT and `dead`, which also stops
// the thread's later waits).
constexpr int kOpPktHalf = kOpPktPerRow / 2;
__device__ __forceinline__ void recv_packets(const uint4 *p, int stride, uint32_t epoch, uint64_t t0, bool &dead,
                                             int32_t *err, uint2 (&out)[kOpPktHalf]) {
  uint4 v[kOpPktHalf];
#pragma unroll
  for (int j = 0; j < kOpPktHalf; ++j) v[j] = ld_volatile_v4(p + j * stride);
  for (uint32_t i = 0; !dead; ++i) {
    bool ok = true;
#pragma unroll
    for (int j = 0; j < kOpPktHalf; ++j) ok = ok && v[j].y == epoch && v[j].w == epoch;
    if (ok) break;
    if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
      dead = true;
      if (err) atomicOr(err, B200KV_DEVERR_TIMEOUT);
      break;
    }
#pragma unroll
    for (int j = 0; j < kOpPktHalf; ++j)
      if (v[j].y != epoch || v[j].w != epoch) v[j] = ld_volatile_v4(p + j * stride);
  }
#pragma unroll
  for (int j = 0; j < kOpPktHalf; ++j) out[j] = make_uint2(v[j].x, v[j].z);
}

// One warp reads 64 consecutive fp32 columns of its 32 TMEM lanes (lane = row).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,"
      "%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]),
        "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]),
        "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]),
        "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]),
        "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Every thread of every CTA of the cluster arrives (release) and waits
// (acquire); not .aligned, so warps whose lanes took different roles may call it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Address, in the shared::cluster window, of the same offset in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_cluster(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

template <int C>
__global__ void __launch_bounds__(kOpThreads, 1)
    oproj_allreduce_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
                           const OpArgs a) {
  using Cfg = OpCfg<C>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Cfg::kRing);
  uint64_t *empty = full + kStages;
  uint64_t *accum = empty + kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  uint32_t *epoch_slot = tmem_slot + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x;
  const int n0 = tile * kOpN;
  // (C, 1, 1) clusters over a 1-D grid: the CTA's rank in its cluster is
  // tile % C; the cluster's super-tile starts at column (tile - crank) * 64
  const int crank = tile % C;
  const int cn0 = (tile - crank) * kOpN;
  const int kpc = a.kblocks / C;  // K blocks of this CTA's split
  const int kb0 = crank * kpc;

  if (tid == 0) {
    prefetch_tensormap(&amap);
    prefetch_tensormap(&wmap);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
    *epoch_slot = static_cast<uint32_t>(*reinterpret_cast<volatile int32_t *>(a.peers[a.rank] + a.counter_off)) + 1u;
  }
  if (warp == 5) {  // 64C TMEM columns for the 128 x 64C fp32 accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(Cfg::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t epoch = *epoch_slot;

  if (warp == 4) {
    if (lane == 0) {  // producer
      for (int i = 0; i < kpc; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1u;
        mbar_wait_bounded(&empty[s], ph ^ 1u, a.error_flag);
        mbar_arrive_expect_tx(&full[s], Cfg::kStage);
        uint8_t *st = smem + s * Cfg::kStage;
        tma_load_2d(st, &amap, &full[s], (kb0 + i) * kOpK, 0);
        tma_load_2d(st + kOpATile, &wmap, &full[s], (kb0 + i) * kOpK, cn0);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // MMA issuer
      for (int i = 0; i < kpc; ++i) {
        const int s = i % kStages;
        mbar_wait_bounded(&full[s], (i / kStages) & 1u, a.error_flag);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t abase = smem_u32(smem + s * Cfg::kStage), bbase = abase + kOpATile;
#pragma unroll
        for (int ki = 0; ki < kOpK / 16; ++ki) {
          const uint64_t ad = kmajor_sw128_desc(abase + ki * 32), bd = kmajor_sw128_desc(bbase + ki * 32);
          const uint32_t acc = (i > 0 || ki > 0) ? 1u : 0u;
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
              "l"(ad), "l"(bd), "r"(Cfg::kIdesc), "r"(acc)
              : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&empty[s]))
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(accum))
                   : "memory");
    }
  } else {
    // ------------------------------------------------ epilogue: warps 0-3 --
    mbar_wait_bounded(accum, 0, a.error_flag);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }

  // This CTA's 128 x 64 tile, row `row` (TMEM lane), summed over the K split.
  const int row = (warp & 3) * 32 + lane;
  const uint32_t tlane = tmem + (uint32_t((warp & 3) * 32) << 16);
  float v[64];
  if constexpr (C == 1) {
    if (warp < 4) {
      uint32_t r[64];
      tmem_ld64(tlane, r);
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
    }
  } else {
    // Reduce-scatter of the split through distributed shared memory.  The
    // slot of source CTA s in CTA q's ring holds s's fp32 partial of q's
    // columns: 128 rows of 256 B, 16-byte chunk j of a row stored at chunk
    // j ^ (row % 16), so the 8 lanes of a store or load wavefront hit
    // distinct banks.
    cluster_sync_all();  // every CTA's MMAs are done: the rings are free
    const uint32_t row_base = smem_u32(smem) + uint32_t(row) * 256u;
    if (warp < 4) {
#pragma unroll 1
      for (int d = 1; d < C; ++d) {
        const int q = (crank + d) % C;
        uint32_t r[64];
        tmem_ld64(tlane + uint32_t(q * kOpN), r);
        const uint32_t dst = mapa_cluster(row_base + uint32_t(crank * Cfg::kRecvSlot), uint32_t(q));
#pragma unroll
        for (int j = 0; j < 16; ++j)
          st_cluster_v4(dst + (uint32_t(j ^ (row & 15)) << 4), r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
      }
    }
    cluster_sync_all();  // every partial has landed
    if (warp < 4) {
      uint32_t own[64];
      tmem_ld64(tlane + uint32_t(crank * kOpN), own);
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = 0.f;
#pragma unroll
      for (int src = 0; src < C; ++src) {
        if (src == crank) {
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] += __uint_as_float(own[i]);
        } else {
          const uint8_t *slot = smem + src * Cfg::kRecvSlot + row * 256;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float4 p = *reinterpret_cast<const float4 *>(slot + ((j ^ (row & 15)) << 4));
            v[4 * j] += p.x;
            v[4 * j + 1] += p.y;
            v[4 * j + 2] += p.z;
            v[4 * j + 3] += p.w;
          }
        }
      }
    }
  }

  if (warp < 4) {
    // this rank's partial row, rounded to fp16 (as the unfused path's GEMM
    // output), 32 words of two halves
    uint32_t h[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const __half2 hv = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      h[i] = *reinterpret_cast<const uint32_t *>(&hv);
    }
    const bool live = row < a.batch;
    const int N = a.world, me = a.rank;
    const int per_owner = a.tiles / N;
    const int owner = tile / per_owner, local = tile - owner * per_owner;
    const int64_t par_off = int64_t(epoch & 1u) * a.region_bytes;
    const int64_t slot_pk = int64_t(per_owner) * kOpPktPerTile;  // packets per source slot
    // packet j of row r of a tile sits at j * 128 + r: the 32 lanes of a warp
    // (32 consecutive rows) move 512 contiguous bytes per packet index
    const int64_t pk0 = int64_t(local) * kOpPktPerTile + row;
    __half *orow = a.out + int64_t(row) * a.out_sb + n0;
    const uint64_t t0 = global_timer_ns();
    bool dead = false;
    if (live) {
      if (owner != me) {
        // send the partial row to the owner, then take the sum back
        uint4 *dst = reinterpret_cast<uint4 *>(a.peers[owner] + a.recv1_off + par_off) + int64_t(me) * slot_pk + pk0;
#pragma unroll
        for (int j = 0; j < kOpPktPerRow; ++j)
          st_volatile_v4(dst + j * kOpM, make_uint4(h[2 * j], epoch, h[2 * j + 1], epoch));
        const uint4 *src = reinterpret_cast<const uint4 *>(a.peers[me] + a.recv2_off + par_off) + int64_t(owner) * slot_pk + pk0;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint2 got[kOpPktHalf];
          recv_packets(src + hf * kOpPktHalf * kOpM, kOpM, epoch, t0, dead, a.error_flag, got);
#pragma unroll
          for (int j = 0; j < kOpPktHalf; ++j) *reinterpret_cast<uint2 *>(orow + 4 * (hf * kOpPktHalf + j)) = got[j];
        }
      } else {
        // owner: sum the N partial rows in rank order, keep and send the sum
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = 0.f;
        for (int q = 0; q < N; ++q) {
          const uint4 *src = reinterpret_cast<const uint4 *>(a.peers[me] + a.recv1_off + par_off) + int64_t(q) * slot_pk + pk0;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint2 got[kOpPktHalf];
            if (q != me) recv_packets(src + hf * kOpPktHalf * kOpM, kOpM, epoch, t0, dead, a.error_flag, got);
#pragma unroll
            for (int jj = 0; jj < kOpPktHalf; ++jj) {
              const int j = hf * kOpPktHalf + jj;
              const uint2 v = q == me ? make_uint2(h[2 * j], h[2 * j + 1]) : got[jj];
              const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
              const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
              acc[4 * j] += f0.x;
              acc[4 * j + 1] += f0.y;
              acc[4 * j + 2] += f1.x;
              acc[4 * j + 3] += f1.y;
            }
          }
        }
        uint32_t s[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const __half2 v = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
          s[i] = *reinterpret_cast<const uint32_t *>(&v);
        }
#pragma unroll
        for (int j = 0; j < kOpPktPerRow; ++j)
          *reinterpret_cast<uint2 *>(orow + 4 * j) = make_uint2(s[2 * j], s[2 * j + 1]);
        for (int q = 0; q < N; ++q) {
          if (q == me) continue;
          uint4 *dst = reinterpret_cast<uint4 *>(a.peers[q] + a.recv2_off + par_off) + int64_t(me) * slot_pk + pk0;
#pragma unroll
          for (int j = 0; j < kOpPktPerRow; ++j)
            st_volatile_v4(dst + j * kOpM, make_uint4(s[2 * j], epoch, s[2 * j + 1], epoch));
        }
      }
    }
  }

  // the last CTA to finish publishes the epoch; warp 5 frees the TMEM
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0) {
    int32_t *counter = reinterpret_cast<int32_t *>(a.peers[a.rank] + a.counter_off);
    __threadfence();
    if (atomicAdd(counter + 1, 1) == a.tiles - 1) {
      counter[1] = 0;
      __threadfence();
      *reinterpret_cast<volatile int32_t *>(counter) = static_cast<int32_t>(epoch);
    }
  }
  if (warp == 5) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmemCols)
                 : "memory");
  }
}

int make_rowmajor_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t row_stride_elems,
                      uint32_t box_rows) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return set_error(B200KV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kOpK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(B200KV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return B200KV_OK;
}

// The peer-buffer regions of peer_allreduce.cu (same layout function there).
void peer_regions(int64_t capacity, int world, int64_t *recv1, int64_t *recv2, int64_t *region, int64_t *counter) {
  auto up = [](int64_t x) { return (x + 255) & ~int64_t(255); };
  const int64_t part_cap = (capacity + world - 1) / world;
  *region = int64_t(world) * (part_cap / 4) * 16;
  *recv1 = up(capacity * 2);
  *recv2 = up(*recv1 + 2 * *region);
  *counter = up(*recv2 + 2 * *region);
}


// Sets the kernel's shared-memory limit once per device.
template <int C>
int configure_oproj(int dev) {
  static int configured[64] = {0};
  if (dev < 0 || dev >= 64) return set_error(B200KV_ERR_UNSUPPORTED, "device ordinal %d", dev);
  if (!__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    B200KV_CUDA_TRY(cudaFuncSetAttribute(oproj_allreduce_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         OpCfg<C>::kSmem));
    __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  return B200KV_OK;
}

template <int C>
void fill_launch(cudaLaunchConfig_t *cfg, cudaLaunchAttribute *attr, int tiles, cudaStream_t stream) {
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3(static_cast<unsigned>(tiles));
  cfg->blockDim = dim3(kOpThreads);
  cfg->dynamicSmemBytes = OpCfg<C>::kSmem;
  cfg->stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg->attrs = attr;
  cfg->numAttrs = C > 1 ? 1 : 0;
}

// How many clusters of C CTAs of this kernel fit on the device at once
// (cached per device; 0 if the query fails).
template <int C>
int max_active_clusters(int dev) {
  static int cached[64];
  static int known[64] = {0};
  if (__atomic_load_n(&known[dev], __ATOMIC_ACQUIRE)) return cached[dev];
  int n = 0;
  if (configure_oproj<C>(dev) == B200KV_OK) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    fill_launch<C>(&cfg, attr, 128, nullptr);
    if (cudaOccupancyMaxActiveClusters(&n, oproj_allreduce_kernel<C>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
  }
  cached[dev] = n;
  __atomic_store_n(&known[dev], 1, __ATOMIC_RELEASE);
  return n;
}

// Split-K cluster size.  Measured on B200 (world 1, hidden 8192, graph
// replays, W rotated through more than L2): K = 1024 / 2048 / 4096 / 8192 ran
// 11.8 / 16.6 / 26.4 / 45.7 us with C = 1, 13.2 / 15.8 / 20.8 / 32.7 us with
// C = 2 and 17.7 / 20.1 / 25.2 / 35.6 us with C = 4 (ncu: DRAM 27-35 % and L2
// 20-25 % busy, tensor pipe 17-23 %: the kernel is bound by the bytes each SM
// keeps in flight, not by a bandwidth, and C = 4 pays a deeper reduction and a
// shallower ring).  So C = 2 from 32 K blocks of 64 on, else 1; a split is used
// only if it divides the tile count and the K blocks and all its clusters fit
// on the device at once (every CTA must be resident: tiles wait on the other
// ranks' tiles).  B200KV_OPROJ_SPLIT=1|2|4 asks for one size (still checked).
int pick_split(int dev, int sms, int tiles, int kblocks, int *split) {
  int want = 0;
  if (const char *e = std::getenv("B200KV_OPROJ_SPLIT")) want = std::atoi(e);
  B200KV_CHECK_ARG(want == 0 || want == 1 || want == 2 || want == 4, "B200KV_OPROJ_SPLIT must be 1, 2 or 4");
  if (dev < 0 || dev >= 64) return set_error(B200KV_ERR_UNSUPPORTED, "device ordinal %d", dev);
  auto fits = [&](int c) {
    if (tiles % c != 0 || kblocks % c != 0) return false;
    if (c == 1) return tiles <= sms;
    const int n = c == 4 ? max_active_clusters<4>(dev) : max_active_clusters<2>(dev);
    return n * c >= tiles;
  };
  if (want != 0) {
    if (!fits(want))
      return set_error(B200KV_ERR_UNSUPPORTED, "split %d does not fit %d tiles x %d K blocks on this device", want,
                       tiles, kblocks);
    *split = want;
    return B200KV_OK;
  }
  for (int c : {2, 1}) {
    if ((c == 1 || kblocks >= 32) && fits(c)) {
      *split = c;
      return B200KV_OK;
    }
  }
  return set_error(B200KV_ERR_UNSUPPORTED, "%d output tiles need as many co-resident CTAs (%d SMs)", tiles, sms);
}

template <int C>
int launch_oproj(const CUtensorMap &am, const CUtensorMap &wm, const OpArgs &a, int tiles, cudaStream_t stream) {
  int dev = 0;
  B200KV_CUDA_TRY(cudaGetDevice(&dev));
  int st = configure_oproj<C>(dev);
  if (st != B200KV_OK) return st;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  fill_launch<C>(&cfg, attr, tiles, stream);
  B200KV_CUDA_TRY(cudaLaunchKernelEx(&cfg, oproj_allreduce_kernel<C>, am, wm, a));
  return B200KV_OK;
}
}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int b200kv_oproj_allreduce_f16(const void *attn, int64_t attn_stride_b, const void *w,
                                          int64_t w_stride_n, void *out, int64_t out_stride_b, int64_t batch,
                                          int64_t hidden, int64_t k, void *const *peer_buffers, int32_t rank,
                                          int32_t world, int64_t capacity_elems, int32_t *error_flag,
                                          void *stream) {
  clear_error();
  B200KV_CHECK_ARG(world >= 1 && world <= kOpMaxRanks, "world must be in [1, %d]", kOpMaxRanks);
  B200KV_CHECK_ARG(rank >= 0 && rank < world, "rank %d outside [0, %d)", rank, world);
  B200KV_CHECK_ARG(batch >= 0 && batch <= kOpM, "batch must be in [0, %d]", kOpM);
  B200KV_CHECK_ARG(k > 0 && k % kOpK == 0, "k (%lld) must be a positive multiple of %d", (long long)k, kOpK);
  B200KV_CHECK_ARG(hidden > 0 && hidden % (kOpN * world) == 0,
                   "hidden (%lld) must be a multiple of %d * world", (long long)hidden, kOpN);
  const int64_t tiles = hidden / kOpN;
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  B200KV_CHECK_ARG(capacity_elems >= int64_t(kOpM) * hidden && capacity_elems % (int64_t(world) * 8) == 0,
                   "the peer buffers must hold 128 x hidden elements (capacity %lld)", (long long)capacity_elems);
  if (batch == 0) return B200KV_OK;
  B200KV_CHECK_ARG(attn && w && out && peer_buffers, "null pointer argument");
  B200KV_CHECK_ARG((reinterpret_cast<uintptr_t>(attn) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
                       attn_stride_b % 8 == 0 && w_stride_n % 8 == 0 && attn_stride_b >= k && w_stride_n >= k,
                   "attn / w must be 16-byte aligned with row strides that are multiples of 8 elements >= k");
  B200KV_CHECK_ARG((reinterpret_cast<uintptr_t>(out) & 7u) == 0 && out_stride_b % 4 == 0 && out_stride_b >= hidden,
                   "out must be 8-byte aligned with a row stride that is a multiple of 4 elements >= hidden");
  OpArgs a{};
  for (int p = 0; p < world; ++p) {
    B200KV_CHECK_ARG(peer_buffers[p] && (reinterpret_cast<uintptr_t>(peer_buffers[p]) & 255u) == 0,
                     "peer buffer %d is null or not 256-byte aligned", p);
    a.peers[p] = static_cast<uint8_t *>(peer_buffers[p]);
  }
  int split = 1;
  st = pick_split(dev, sms, static_cast<int>(tiles), static_cast<int>(k / kOpK), &split);
  if (st != B200KV_OK) return st;
  CUtensorMap am, wm;
  st = make_rowmajor_map(&am, attn, batch, k, attn_stride_b, kOpM);
  if (st != B200KV_OK) return st;
  st = make_rowmajor_map(&wm, w, hidden, k, w_stride_n, static_cast<uint32_t>(kOpN * split));
  if (st != B200KV_OK) return st;
  a.rank = rank;
  a.world = world;
  a.tiles = static_cast<int>(tiles);
  a.batch = static_cast<int>(batch);
  a.kblocks = static_cast<int>(k / kOpK);
  a.out = static_cast<__half *>(out);
  a.out_sb = out_stride_b;
  peer_regions(capacity_elems, world, &a.recv1_off, &a.recv2_off, &a.region_bytes, &a.counter_off);
  a.error_flag = error_flag;
  const cudaStream_t cs = static_cast<cudaStream_t>(stream);
  switch (split) {
    case 4: return launch_oproj<4>(am, wm, a, static_cast<int>(tiles), cs);
    case 2: return launch_oproj<2>(am, wm, a, static_cast<int>(tiles), cs);
    default: return launch_oproj<1>(am, wm, a, static_cast<int>(tiles), cs);
  }
}
