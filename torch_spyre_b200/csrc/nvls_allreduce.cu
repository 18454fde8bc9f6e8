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
constexpr int kNvlsMaxCtas = 64;
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

__global__ void __launch_bounds__(kNvlsThreads) nvls_allreduce_kernel(const NvlsArgs a) {
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
