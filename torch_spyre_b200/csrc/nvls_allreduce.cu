// Tensor-parallel all-reduce (SUM) of an fp16 tensor through NVLink SHARP:
// the NVSwitch adds the ranks' values in the switch and multicasts the sum.
// The reference's TP collective is an all-reduce SUM of one tensor
// (torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494); this is the B200
// form of it for the o_proj partials of the head-sharded decode step.
//
// Every rank holds the same buffer layout in memory that is bound to one
// NVLink multicast object (allocated and mapped by the host, e.g. through
// PyTorch's symmetric memory):
//   data    [n] fp16 at offset 0: the rank's partial on entry, the sum on exit
//   signals a separate per-rank area (b200kv_nvls_signal_bytes), zeroed once:
//           word 0 the epoch of the last completed call, word 1 a CTA ticket,
//           then flags [2 phases][kNvlsMaxCtas][kNvlsMaxRanks] (uint32)
// One kernel per rank, `ctas` CTAs.  Rank r owns slice r of the data
// (elements [r n/N, (r+1) n/N)); CTA c takes chunk c of it:
//   phase 0  CTA c of every rank tells CTA c of every other rank that its
//            data is in place (the producer of the partial ran before this
//            kernel) and waits for theirs;
//   reduce   multimem.ld_reduce (add, fp32 accumulation in the switch) of the
//            chunk through the multicast address, rounded once to fp16, and
//            multimem.st of the sum to every rank's buffer;
//   phase 1  after a system-scope fence CTA c signals again and waits until
//            every rank's CTA c has stored its chunk here.
// Every rank thus ends with the same bits: each element is reduced once, by
// its owner, and multicast.  Flags carry the call's epoch (counter + 1, the
// counter lives in device memory and the last CTA stores it back), so a
// captured CUDA graph replays correctly, and they are compared with >= so a
// rank that runs one call ahead cannot be missed.  Every wait is bounded
// (2 s of %globaltimer) and sets B200KV_DEVERR_TIMEOUT instead of hanging.
// Loads and stores on peer memory are plain flag stores and the multimem
// instructions; there is no TMA and no multicast TMA anywhere in this file.
#include "common.cuh"

namespace b200kv {
namespace {

constexpr int kNvlsMaxRanks = 8;
constexpr int kNvlsMaxCtas = 256;
constexpr int kNvlsThreads = 512;
constexpr int kNvlsFlagWord = 64;  // flags start 256 bytes into the signal area
constexpr int64_t kNvlsSignalBytes = (kNvlsFlagWord + 2 * kNvlsMaxCtas * kNvlsMaxRanks) * 4;

struct NvlsArgs {
  uint4 *mc;                              // multicast address of the data
  uint32_t *signals[kNvlsMaxRanks];       // every rank's signal area, mapped here
  int rank, world, ctas;
  int64_t n;                              // elements (n % (8 * world) == 0)
  int32_t *error_flag;
};

__device__ __forceinline__ void st_relaxed_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Signals CTA c of every rank for `phase` and waits (bounded) for their
// signals; thread q < world handles rank q.  Returns false after a timeout.
__device__ __forceinline__ bool cta_exchange(const NvlsArgs &a, int phase, int c, uint32_t epoch) {
  const int tid = threadIdx.x;
  bool ok = true;
  if (tid < a.world) {
    const int slot = kNvlsFlagWord + (phase * kNvlsMaxCtas + c) * kNvlsMaxRanks;
    st_relaxed_sys(a.signals[tid] + slot + a.rank, epoch);
    const uint32_t *mine = a.signals[a.rank] + slot + tid;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0; static_cast<int32_t>(ld_acquire_sys(mine) - epoch) < 0; ++i) {
      if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
        if (a.error_flag) atomicOr(a.error_flag, B200KV_DEVERR_TIMEOUT);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ uint4 ld_reduce_add_f16x8(const uint4 *p) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}
__device__ __forceinline__ void st_multicast_f16x8(uint4 *p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

constexpr int kNvlsUnroll = 4;

// Low-latency variant: the sentinel that marks a value not yet arrived in a
// receive region (fp16 0xFFFF, a NaN payload that data never carries there).
constexpr uint32_t kNvlsSentinel = 0xFFFFu;
__device__ __forceinline__ uint32_t canonical_nan_f16x2(uint32_t w) {
  uint32_t lo = w & 0xFFFFu, hi = w >> 16;
  if ((lo & 0x7FFFu) > 0x7C00u) lo = 0x7E00u;  // any NaN -> the canonical quiet NaN
  if ((hi & 0x7FFFu) > 0x7C00u) hi = 0x7E00u;
  return lo | (hi << 16);
}
__device__ __forceinline__ bool half_is_sentinel(uint32_t w) {
  return (w & 0xFFFFu) == kNvlsSentinel || (w >> 16) == kNvlsSentinel;
}
__device__ __forceinline__ bool has_sentinel(uint4 v) {
  return half_is_sentinel(v.x) | half_is_sentinel(v.y) | half_is_sentinel(v.z) | half_is_sentinel(v.w);
}
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const uint4 *p) {
  uint4 r;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}

__global__ void __launch_bounds__(kNvlsThreads) nvls_allreduce_kernel(const __grid_constant__ NvlsArgs a) {
  // Launched as a programmatic dependent: wait for the producer of the partial
  // (a no-op after a kernel that does not trigger early), then let the next
  // grid start -- it must itself wait before it reads this kernel's output.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int c = blockIdx.x, tid = threadIdx.x;
  uint32_t *own = a.signals[a.rank];
  __shared__ uint32_t epoch_s;
  if (tid == 0) epoch_s = *reinterpret_cast<volatile uint32_t *>(own) + 1u;
  __syncthreads();
  const uint32_t epoch = epoch_s;

  // phase 0: every rank's partial is in place
  bool ok = cta_exchange(a, 0, c, epoch);

  // reduce chunk c of this rank's slice and multicast the sum
  const int64_t vslice = a.n / 8 / a.world;
  const int64_t per = (vslice + a.ctas - 1) / a.ctas;
  const int64_t v0 = int64_t(a.rank) * vslice + min(vslice, int64_t(c) * per);
  const int64_t v1 = int64_t(a.rank) * vslice + min(vslice, int64_t(c + 1) * per);
  if (ok) {
    for (int64_t base = v0 + tid; base < v1; base += int64_t(kNvlsThreads) * kNvlsUnroll) {
      uint4 r[kNvlsUnroll];
#pragma unroll
      for (int u = 0; u < kNvlsUnroll; ++u) {
        const int64_t v = base + int64_t(u) * kNvlsThreads;
        if (v < v1) r[u] = ld_reduce_add_f16x8(a.mc + v);
      }
#pragma unroll
      for (int u = 0; u < kNvlsUnroll; ++u) {
        const int64_t v = base + int64_t(u) * kNvlsThreads;
        if (v < v1) st_multicast_f16x8(a.mc + v, r[u]);
      }
    }
  }
  // phase 1: the CTA's stores are performed system-wide before its signal
  __syncthreads();
  if (tid < a.world) asm volatile("fence.acq_rel.sys;" ::: "memory");
  ok = cta_exchange(a, 1, c, epoch) && ok;

  // the last CTA to finish publishes the epoch for the next call
  __shared__ int last;
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(own + 1, 1u) == static_cast<uint32_t>(a.ctas - 1);
  }
  __syncthreads();
  if (last && tid == 0) {
    own[1] = 0;
    __threadfence();
    *reinterpret_cast<volatile uint32_t *>(own) = epoch;
  }
}

// Low-latency variant: two-shot with the arrival marker in the data, no
// flag exchange and no fence.  Every rank owns, in the multicast-bound
// memory, a reduce-scatter region and an all-gather region per parity of the
// call's epoch (double buffered), both holding the sentinel between calls.
//   1. chunk c of every other slice j of the rank's partial goes straight
//      into rank j's reduce-scatter region, slot `rank` (peer stores);
//   2. the owner of slice r polls its slots until the sentinel is gone from
//      every element, sums the ranks' values in rank order in fp32, rounds
//      once to fp16 and multicasts the sum into every rank's all-gather
//      region (multimem.st), putting the sentinel back in its slots;
//   3. every rank polls its all-gather region for chunk c of every slice,
//      copies the sums into its data and puts the sentinel back.
// CTA c of every rank handles chunk c of every slice, so the CTAs of one
// index form an independent group.  Values equal to the sentinel are sent
// as the canonical NaN (their sums are NaN either way) and NaN sums are
// multicast as the canonical NaN, so the sentinel never stands for data.
// Why the regions can be reused without a barrier: a region of parity p is
// written for call k + 2 only by a rank that has finished call k + 1, which
// needs data that the reading rank sent after finishing call k -- its reads
// and sentinel resets of parity p included.  Each 2-byte element is written
// whole, so a vector whose 8 elements all differ from the sentinel has fully
// arrived.  After a timeout the regions may hold stale values: the caller
// must rebuild them (the error flag says so).
struct LlArgs {
  const uint4 *data_in;                 // local data (partial), read
  uint4 *data_out;                      // local data (sum), written
  uint4 *rs[kNvlsMaxRanks];             // every rank's reduce-scatter region, mapped here
  uint4 *ag, *ag_mc;                    // this rank's all-gather region, its multicast address
  int64_t region;                       // vectors per parity in each region
  uint32_t *signal;                     // this rank's signal area: epoch, CTA ticket
  int rank, world, ctas;
  int64_t n;
  int32_t *error_flag;
};

__device__ __forceinline__ uint4 canonical_nan_f16x8(uint4 v) {
  return make_uint4(canonical_nan_f16x2(v.x), canonical_nan_f16x2(v.y), canonical_nan_f16x2(v.z),
                    canonical_nan_f16x2(v.w));
}
__device__ __forceinline__ void add_f16x2(float &lo, float &hi, uint32_t w) {
  lo += __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
  hi += __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}
__device__ __forceinline__ void add_f16x8(float (&acc)[8], uint4 v) {
  add_f16x2(acc[0], acc[1], v.x);
  add_f16x2(acc[2], acc[3], v.y);
  add_f16x2(acc[4], acc[5], v.z);
  add_f16x2(acc[6], acc[7], v.w);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(lo))) |
         (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(hi))) << 16);
}
__device__ __forceinline__ uint4 pack_f16x8(const float (&acc)[8]) {
  return make_uint4(pack_f16x2(acc[0], acc[1]), pack_f16x2(acc[2], acc[3]), pack_f16x2(acc[4], acc[5]),
                    pack_f16x2(acc[6], acc[7]));
}
// Polls *p until none of its 8 elements is the sentinel; false after the
// time limit (t0 is the kernel's start).
__device__ __forceinline__ bool poll_arrived(const uint4 *p, uint4 &x, uint64_t t0, int32_t *error_flag) {
  x = ld_relaxed_sys_v4(p);
  for (uint32_t i = 0; has_sentinel(x); ++i) {
    if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
      if (error_flag) atomicOr(error_flag, B200KV_DEVERR_TIMEOUT);
      return false;
    }
    x = ld_relaxed_sys_v4(p);
  }
  return true;
}

__global__ void __launch_bounds__(kNvlsThreads, 1) nvls_allreduce_ll_kernel(const __grid_constant__ LlArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int c = blockIdx.x, tid = threadIdx.x;
  const uint64_t t0 = global_timer_ns();
  __shared__ uint32_t epoch_s;
  if (tid == 0) epoch_s = *reinterpret_cast<volatile uint32_t *>(a.signal) + 1u;
  __syncthreads();
  const uint32_t epoch = epoch_s;
  // the CTA's ticket, taken now (every CTA has read the epoch before its
  // ticket) and used at the end: the last CTA publishes the epoch
  uint32_t ticket = 0;
  if (tid == 0) ticket = atomicAdd(a.signal + 1, 1u);

  const int64_t pbase = int64_t(epoch & 1u) * a.region;
  const int64_t vslice = a.n / 8 / a.world;
  const int64_t per = (vslice + a.ctas - 1) / a.ctas;
  const int64_t c0 = min(vslice, int64_t(c) * per), c1 = min(vslice, int64_t(c + 1) * per);
  const uint4 sentinel = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);

  // 1. chunk c of every other slice to its owner, slot `rank`
  for (int jj = 1; jj < a.world; ++jj) {
    const int j = (a.rank + jj) % a.world;
    uint4 *dst = a.rs[j] + pbase + int64_t(a.rank) * vslice;
    for (int64_t v = c0 + tid; v < c1; v += kNvlsThreads)
      dst[v] = canonical_nan_f16x8(a.data_in[int64_t(j) * vslice + v]);
  }
  // 2. chunk c of this rank's slice: sum in rank order, multicast the sum
  bool ok = true;
  uint4 *own_rs = a.rs[a.rank] + pbase;
  for (int64_t v = c0 + tid; v < c1 && ok; v += kNvlsThreads) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < a.world; ++q) {
      uint4 x;
      if (q == a.rank) {
        x = a.data_in[int64_t(a.rank) * vslice + v];
      } else {
        uint4 *src = own_rs + int64_t(q) * vslice + v;
        if (!(ok = poll_arrived(src, x, t0, a.error_flag))) break;
        *src = sentinel;
      }
      add_f16x8(acc, x);
    }
    if (ok) st_multicast_f16x8(a.ag_mc + pbase + int64_t(a.rank) * vslice + v, canonical_nan_f16x8(pack_f16x8(acc)));
  }
  // 3. chunk c of every slice: the sums into the data, the sentinel back
  for (int jj = 0; jj < a.world && ok; ++jj) {
    const int j = (a.rank + jj) % a.world;
    for (int64_t v = c0 + tid; v < c1 && ok; v += kNvlsThreads) {
      uint4 *src = a.ag + pbase + int64_t(j) * vslice + v;
      uint4 x;
      if (!(ok = poll_arrived(src, x, t0, a.error_flag))) break;
      a.data_out[int64_t(j) * vslice + v] = x;
      *src = sentinel;
    }
  }
  if (tid == 0 && ticket == static_cast<uint32_t>(a.ctas - 1)) {
    a.signal[1] = 0;
    __threadfence();
    *reinterpret_cast<volatile uint32_t *>(a.signal) = epoch;
  }
}

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int64_t b200kv_nvls_signal_bytes(void) { return kNvlsSignalBytes; }

extern "C" int b200kv_nvls_allreduce_f16(void *multicast_data, void *const *signal_areas, int32_t rank,
                                         int32_t world, int64_t num_elems, int32_t ctas, int32_t *error_flag,
                                         void *stream) {
  clear_error();
  B200KV_CHECK_ARG(world >= 1 && world <= kNvlsMaxRanks, "world must be in [1, %d]", kNvlsMaxRanks);
  B200KV_CHECK_ARG(rank >= 0 && rank < world, "rank %d outside [0, %d)", rank, world);
  B200KV_CHECK_ARG(num_elems >= 0 && num_elems % (int64_t(world) * 8) == 0,
                   "num_elems (%lld) must be a non-negative multiple of 8 * world", (long long)num_elems);
  B200KV_CHECK_ARG(ctas >= 0 && ctas <= kNvlsMaxCtas, "ctas must be in [0, %d]", kNvlsMaxCtas);
  B200KV_CHECK_ARG(multicast_data && (reinterpret_cast<uintptr_t>(multicast_data) & 15u) == 0,
                   "the multicast data address must be 16-byte aligned");
  B200KV_CHECK_ARG(signal_areas, "null signal area table");
  if (num_elems == 0) return B200KV_OK;
  NvlsArgs a{};
  for (int p = 0; p < world; ++p) {
    B200KV_CHECK_ARG(signal_areas[p] && (reinterpret_cast<uintptr_t>(signal_areas[p]) & 255u) == 0,
                     "signal area %d is null or not 256-byte aligned", p);
    a.signals[p] = static_cast<uint32_t *>(signal_areas[p]);
  }
  a.mc = static_cast<uint4 *>(multicast_data);
  a.rank = rank;
  a.world = world;
  a.n = num_elems;
  a.ctas = ctas > 0 ? ctas : 32;
  a.error_flag = error_flag;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.ctas);
  cfg.blockDim = dim3(kNvlsThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200KV_CUDA_TRY(cudaLaunchKernelEx(&cfg, nvls_allreduce_kernel, static_cast<const NvlsArgs>(a)));
  return B200KV_OK;
}

extern "C" int b200kv_nvls_allreduce_ll_f16(void *data, void *const *rs_regions, void *ag_region,
                                            void *ag_multicast, int64_t region_elems, void *signal_area,
                                            int32_t rank, int32_t world, int64_t num_elems, int32_t ctas,
                                            int32_t *error_flag, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(world >= 1 && world <= kNvlsMaxRanks, "world must be in [1, %d]", kNvlsMaxRanks);
  B200KV_CHECK_ARG(rank >= 0 && rank < world, "rank %d outside [0, %d)", rank, world);
  B200KV_CHECK_ARG(num_elems >= 0 && num_elems % (int64_t(world) * 8) == 0,
                   "num_elems (%lld) must be a non-negative multiple of 8 * world", (long long)num_elems);
  B200KV_CHECK_ARG(region_elems >= num_elems && region_elems % 8 == 0,
                   "region_elems (%lld) must be a multiple of 8 holding num_elems", (long long)region_elems);
  B200KV_CHECK_ARG(ctas >= 0 && ctas <= kNvlsMaxCtas, "ctas must be in [0, %d]", kNvlsMaxCtas);
  for (void *p : {data, ag_region, ag_multicast, signal_area})
    B200KV_CHECK_ARG(p && (reinterpret_cast<uintptr_t>(p) & 15u) == 0,
                     "the data, all-gather and signal addresses must be non-null and 16-byte aligned");
  B200KV_CHECK_ARG(rs_regions, "null reduce-scatter region table");
  if (num_elems == 0) return B200KV_OK;
  LlArgs a{};
  for (int p = 0; p < world; ++p) {
    B200KV_CHECK_ARG(rs_regions[p] && (reinterpret_cast<uintptr_t>(rs_regions[p]) & 15u) == 0,
                     "reduce-scatter region %d is null or not 16-byte aligned", p);
    a.rs[p] = static_cast<uint4 *>(rs_regions[p]);
  }
  a.data_in = static_cast<const uint4 *>(data);
  a.data_out = static_cast<uint4 *>(data);
  a.ag = static_cast<uint4 *>(ag_region);
  a.ag_mc = static_cast<uint4 *>(ag_multicast);
  a.region = region_elems / 8;
  a.signal = static_cast<uint32_t *>(signal_area);
  a.rank = rank;
  a.world = world;
  a.n = num_elems;
  a.ctas = ctas > 0 ? ctas : 32;
  a.error_flag = error_flag;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.ctas);
  cfg.blockDim = dim3(kNvlsThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200KV_CUDA_TRY(cudaLaunchKernelEx(&cfg, nvls_allreduce_ll_kernel, static_cast<const LlArgs>(a)));
  return B200KV_OK;
}
