// Tensor-parallel all-reduce (SUM) of an fp16 tensor over peer memory, for the
// o_proj partials of the head-sharded decode step.  The reference's TP
// collective is an all-reduce SUM of one tensor (torch_spyre/csrc/
// spyre_ccl.cpp:470-494); here it is one kernel per rank over buffers the
// ranks map into each other's address space with CUDA IPC, moving data with
// plain peer stores over NVLink (no multicast, no library kernel on peer
// memory).
//
// Every rank owns one "peer buffer" (allocated by b200kv_peer_alloc):
//   data    [S] fp16        the rank's partial on entry, the sum on exit
//   staging [N][S / N] fp16 the slices of its own part pushed by every rank
//   flags1  [N][kMaxCtas]   "slice chunk from rank q staged" (epoch values)
//   flags2  [N][kMaxCtas]   "reduced chunk of rank q's part written"
//   counter                 epoch of the last completed call, and a ticket
// Two-shot algorithm (CTA c owns chunk c of every part; part p = elements
// [p*S/N, (p+1)*S/N) is reduced by rank p):
//   1. push chunk c of part p of `data` into rank p's staging[me], then set
//      rank p's flags1[me][c] = epoch (release, system scope);
//   2. wait flags1[q][c] == epoch for every q, sum staging[*] chunk c in fp32
//      (rank order, so every rank rounds the same way), write the fp16 sum
//      into data of every rank (own included), set flags2[me][c] on every
//      rank;
//   3. wait flags2[q][c] == epoch for every q: chunk c of every part is home.
// The epoch comes from device memory (counter + 1) and the last CTA to
// finish stores it back, so a captured CUDA graph replays correctly.  Every
// wait is bounded (2 s of %globaltimer) and sets B200KV_DEVERR_TIMEOUT.
#include <cstring>

#include "common.cuh"

namespace b200kv {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 64;
constexpr int kArThreads = 256;

struct PeerLayout {
  int64_t data_off, staging_off, flags1_off, flags2_off, counter_off, total;
};

PeerLayout peer_layout(int64_t capacity_elems, int world) {
  auto up = [](int64_t x) { return (x + 255) & ~int64_t(255); };
  PeerLayout l;
  const int64_t part = (capacity_elems + world - 1) / world;
  l.data_off = 0;
  l.staging_off = up(capacity_elems * 2);
  l.flags1_off = up(l.staging_off + int64_t(world) * part * 2);
  l.flags2_off = up(l.flags1_off + int64_t(kMaxRanks) * kMaxCtas * 4);
  l.counter_off = up(l.flags2_off + int64_t(kMaxRanks) * kMaxCtas * 4);
  l.total = up(l.counter_off + 64);
  return l;
}

struct PeerArgs {
  uint8_t *peers[kMaxRanks];  // every rank's peer buffer, mapped here (own included)
  int rank, world, ctas;
  int64_t n;                  // elements (n % (world * 8) == 0)
  int64_t cap;                // capacity the buffers were laid out for
  PeerLayout lay;
  int32_t *error_flag;
};

__device__ __forceinline__ void st_release_sys(int32_t *p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t *p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0 waits until flags[q * kMaxCtas + c] == epoch for every rank q
// (bounded); the CTA then proceeds.  Returns false after a timeout.
__device__ bool wait_flags(const int32_t *flags, int world, int c, int32_t epoch, int32_t *error_flag) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = global_timer_ns();
    for (int q = 0; q < world; ++q) {
      const int32_t *f = flags + q * kMaxCtas + c;
      for (uint32_t i = 0;; ++i) {
        if (ld_acquire_sys(f) == epoch) break;
        if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
          if (error_flag) atomicOr(error_flag, B200KV_DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
      if (!ok) break;
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(kArThreads) peer_allreduce_kernel(const PeerArgs a) {
  const int c = blockIdx.x, tid = threadIdx.x;
  const int me = a.rank, N = a.world;
  uint8_t *mine = a.peers[me];
  int32_t *counter = reinterpret_cast<int32_t *>(mine + a.lay.counter_off);
  const int32_t epoch = ld_acquire_sys(counter) + 1;

  const int64_t part = a.n / N;                 // elements of one rank's part
  const int64_t vec_part = part / 8;            // 16-byte vectors per part
  const int64_t per = (vec_part + a.ctas - 1) / a.ctas;
  const int64_t v0 = min(vec_part, int64_t(c) * per), v1 = min(vec_part, v0 + per);
  const uint4 *data_me = reinterpret_cast<const uint4 *>(mine + a.lay.data_off);
  const int64_t part_stride = ((a.cap + N - 1) / N) / 8;  // staging slot stride in vectors

  // 1. push chunk c of part p to rank p's staging[me]
  for (int p = 0; p < N; ++p) {
    uint4 *dst = reinterpret_cast<uint4 *>(a.peers[p] + a.lay.staging_off) + int64_t(me) * part_stride;
    const uint4 *src = data_me + int64_t(p) * vec_part;
    for (int64_t v = v0 + tid; v < v1; v += kArThreads) dst[v] = src[v];
  }
  __threadfence_system();
  __syncthreads();
  if (tid < N) st_release_sys(reinterpret_cast<int32_t *>(a.peers[tid] + a.lay.flags1_off) + me * kMaxCtas + c, epoch);

  // 2. reduce chunk c of my part and write it into every rank's data
  const int32_t *flags1 = reinterpret_cast<const int32_t *>(mine + a.lay.flags1_off);
  const bool ok1 = wait_flags(flags1, N, c, epoch, a.error_flag);
  if (ok1) {
    const uint4 *stg = reinterpret_cast<const uint4 *>(mine + a.lay.staging_off);
    for (int64_t v = v0 + tid; v < v1; v += kArThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int q = 0; q < N; ++q) {
        const uint4 x = stg[int64_t(q) * part_stride + v];
        const __half2 *h = reinterpret_cast<const __half2 *>(&x);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
      uint4 r;
      __half2 *rh = reinterpret_cast<__half2 *>(&r);
#pragma unroll
      for (int i = 0; i < 4; ++i) rh[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
      for (int p = 0; p < N; ++p)
        reinterpret_cast<uint4 *>(a.peers[p] + a.lay.data_off)[int64_t(me) * vec_part + v] = r;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (tid < N) st_release_sys(reinterpret_cast<int32_t *>(a.peers[tid] + a.lay.flags2_off) + me * kMaxCtas + c, epoch);

  // 3. wait until every rank's reduced chunk c is home
  const int32_t *flags2 = reinterpret_cast<const int32_t *>(mine + a.lay.flags2_off);
  wait_flags(flags2, N, c, epoch, a.error_flag);

  // the last CTA to finish publishes the epoch for the next call
  __shared__ int last;
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(counter + 1, 1) == a.ctas - 1;
  }
  __syncthreads();
  if (last && tid == 0) {
    counter[1] = 0;
    __threadfence();
    st_release_sys(counter, epoch);
  }
}

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int64_t b200kv_peer_buffer_bytes(int64_t capacity_elems, int32_t world) {
  if (capacity_elems <= 0 || world < 1 || world > kMaxRanks) return -1;
  return peer_layout(capacity_elems, world).total;
}

extern "C" int b200kv_peer_alloc(int64_t capacity_elems, int32_t world, void **buffer_out) {
  clear_error();
  B200KV_CHECK_ARG(buffer_out, "null output pointer");
  *buffer_out = nullptr;
  B200KV_CHECK_ARG(capacity_elems > 0 && world >= 1 && world <= kMaxRanks,
                   "capacity must be > 0 and world in [1, %d]", kMaxRanks);
  const PeerLayout l = peer_layout(capacity_elems, world);
  void *p = nullptr;
  B200KV_CUDA_TRY(cudaMalloc(&p, l.total));
  const cudaError_t e = cudaMemset(p, 0, l.total);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "cudaMemset");
  }
  *buffer_out = p;
  return B200KV_OK;
}

extern "C" int b200kv_peer_free(void *buffer) {
  clear_error();
  if (buffer) B200KV_CUDA_TRY(cudaFree(buffer));
  return B200KV_OK;
}

extern "C" int32_t b200kv_ipc_handle_bytes(void) { return static_cast<int32_t>(sizeof(cudaIpcMemHandle_t)); }

extern "C" int b200kv_ipc_get_handle(void *buffer, void *handle_out) {
  clear_error();
  B200KV_CHECK_ARG(buffer && handle_out, "null pointer argument");
  cudaIpcMemHandle_t h;
  B200KV_CUDA_TRY(cudaIpcGetMemHandle(&h, buffer));
  memcpy(handle_out, &h, sizeof(h));
  return B200KV_OK;
}

extern "C" int b200kv_ipc_open_handle(const void *handle, void **buffer_out) {
  clear_error();
  B200KV_CHECK_ARG(handle && buffer_out, "null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  B200KV_CUDA_TRY(cudaIpcOpenMemHandle(buffer_out, h, cudaIpcMemLazyEnablePeerAccess));
  return B200KV_OK;
}

extern "C" int b200kv_ipc_close_handle(void *buffer) {
  clear_error();
  if (buffer) B200KV_CUDA_TRY(cudaIpcCloseMemHandle(buffer));
  return B200KV_OK;
}

extern "C" int b200kv_peer_allreduce_f16(void *const *peer_buffers, int32_t rank, int32_t world,
                                         int64_t num_elems, int64_t capacity_elems, int32_t ctas,
                                         int32_t *error_flag, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(world >= 1 && world <= kMaxRanks, "world must be in [1, %d]", kMaxRanks);
  B200KV_CHECK_ARG(rank >= 0 && rank < world, "rank %d outside [0, %d)", rank, world);
  B200KV_CHECK_ARG(num_elems >= 0 && num_elems <= capacity_elems, "num_elems must be in [0, capacity]");
  B200KV_CHECK_ARG(num_elems % (int64_t(world) * 8) == 0,
                   "num_elems (%lld) must be a multiple of 8 * world", (long long)num_elems);
  B200KV_CHECK_ARG(capacity_elems % (int64_t(world) * 8) == 0,
                   "capacity (%lld) must be a multiple of 8 * world", (long long)capacity_elems);
  B200KV_CHECK_ARG(ctas >= 0 && ctas <= kMaxCtas, "ctas must be in [0, %d]", kMaxCtas);
  B200KV_CHECK_ARG(peer_buffers, "null peer buffer table");
  if (num_elems == 0) return B200KV_OK;
  PeerArgs a{};
  for (int p = 0; p < world; ++p) {
    B200KV_CHECK_ARG(peer_buffers[p] && (reinterpret_cast<uintptr_t>(peer_buffers[p]) & 255u) == 0,
                     "peer buffer %d is null or not 256-byte aligned", p);
    a.peers[p] = static_cast<uint8_t *>(peer_buffers[p]);
  }
  a.rank = rank;
  a.world = world;
  a.n = num_elems;
  a.cap = capacity_elems;
  a.lay = peer_layout(capacity_elems, world);
  a.ctas = ctas > 0 ? ctas : 32;
  a.error_flag = error_flag;
  peer_allreduce_kernel<<<a.ctas, kArThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}
