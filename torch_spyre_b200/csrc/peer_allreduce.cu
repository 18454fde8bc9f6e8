// Tensor-parallel all-reduce (SUM) of an fp16 tensor over peer memory, for the
// o_proj partials of the head-sharded decode step.  The reference's TP
// collective is an all-reduce SUM of one tensor (torch_spyre/csrc/
// spyre_ccl.cpp:470-494); here it is one kernel per rank over buffers the
// ranks map into each other's address space with CUDA IPC, moving data with
// plain peer stores over NVLink (no multicast, no library kernel on peer
// memory).
//
// Transfers use flagged packets instead of fences: every 16-byte peer store
// carries two 8-byte words {4 bytes of data, the call's epoch}.  An aligned
// 8-byte store is seen whole, so a receiver that polls a word until its flag
// equals the epoch has the data: no system-scope fence or flag array is
// needed (a system fence costs microseconds per signal on this path).
//
// Every rank owns one "peer buffer" (allocated by b200kv_peer_alloc):
//   data    [S] fp16                         the partial on entry, the sum on exit
//   recv1   [2][N][S/N / 4] 16-byte packets  slices of its part, from rank q
//   recv2   [2][N][S/N / 4] packets          rank q's reduced part
//   counter                                  epoch of the last completed call, a ticket
// Receive regions alternate with the epoch's parity: a rank cannot start call
// k + 2 (reusing call k's region) before every rank finished call k + 1, by
// which time every rank finished reading call k's packets.  Peers never write
// `data`, so a rank's next producer (the o_proj GEMM) cannot race with them.
// Two-shot algorithm (part p = elements [p*S/N, (p+1)*S/N) is reduced by
// rank p; CTA c takes chunk c of every part):
//   1. send chunk c of part p != me to rank p's recv1[par][me];
//   2. sum chunk c of the parts in rank order (own partial read in place,
//      the others polled from recv1) in fp32, round once to fp16, write it
//      into data and send it to every rank's recv2[par][me];
//   3. poll recv2[par][q] for chunk c of every other part q into data.
// The epoch comes from device memory (counter + 1) and the last CTA to finish
// stores it back, so a captured CUDA graph replays correctly.  Every poll is
// bounded (2 s of %globaltimer per thread); a timeout sets
// B200KV_DEVERR_TIMEOUT and the thread stops waiting (its output is undefined).
#include <cstring>

#include "common.cuh"

namespace b200kv {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 128;
constexpr int kArThreads = 256;

struct PeerLayout {
  int64_t part_cap;      // elements of one part (capacity / world)
  int64_t region_bytes;  // one [N][part_cap / 4] packet region
  int64_t data_off, recv1_off, recv2_off, counter_off, total;
};

PeerLayout peer_layout(int64_t capacity_elems, int world) {
  auto up = [](int64_t x) { return (x + 255) & ~int64_t(255); };
  PeerLayout l;
  l.part_cap = (capacity_elems + world - 1) / world;
  l.region_bytes = int64_t(world) * (l.part_cap / 4) * 16;
  l.data_off = 0;
  l.recv1_off = up(capacity_elems * 2);
  l.recv2_off = up(l.recv1_off + 2 * l.region_bytes);
  l.counter_off = up(l.recv2_off + 2 * l.region_bytes);
  l.total = up(l.counter_off + 64);
  return l;
}

struct PeerArgs {
  uint8_t *peers[kMaxRanks];  // every rank's peer buffer, mapped here (own included)
  int rank, world, ctas;
  int64_t n;                  // elements (n % (world * 8) == 0)
  PeerLayout lay;
  int32_t *error_flag;
};

__device__ __forceinline__ void st_volatile_v4(uint4 *p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
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

// One 16-byte data vector (8 fp16) travels as packets 2v, 2v + 1.
__device__ __forceinline__ void send_vec(uint4 *region, int64_t v, uint4 x, uint32_t epoch) {
  st_volatile_v4(region + 2 * v, make_uint4(x.x, epoch, x.y, epoch));
  st_volatile_v4(region + 2 * v + 1, make_uint4(x.z, epoch, x.w, epoch));
}

// Polls packets 2v, 2v + 1 until both words of both carry `epoch` (bounded by
// the thread's deadline; after a timeout `dead` is set and polling stops).
__device__ __forceinline__ uint4 recv_vec(const uint4 *region, int64_t v, uint32_t epoch, uint64_t t0,
                                          bool &dead, int32_t *error_flag) {
  uint4 a, b;
  for (uint32_t i = 0;; ++i) {
    a = ld_volatile_v4(region + 2 * v);
    b = ld_volatile_v4(region + 2 * v + 1);
    if ((a.y == epoch && a.w == epoch && b.y == epoch && b.w == epoch) || dead) break;
    if ((i & 255u) == 255u && global_timer_ns() - t0 > kWaitLimitNs) {
      dead = true;
      if (error_flag) atomicOr(error_flag, B200KV_DEVERR_TIMEOUT);
      break;
    }
  }
  return make_uint4(a.x, a.z, b.x, b.z);
}

__device__ __forceinline__ void add_half8(float (&acc)[8], uint4 x) {
  const __half2 *h = reinterpret_cast<const __half2 *>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

__global__ void __launch_bounds__(kArThreads) peer_allreduce_kernel(const PeerArgs a) {
  // Launched as a programmatic dependent: wait for the producer of the partial
  // (a no-op after a kernel that does not trigger early), then let the next
  // grid start -- it must itself wait before it reads this kernel's output.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int c = blockIdx.x, tid = threadIdx.x;
  const int me = a.rank, N = a.world;
  uint8_t *mine = a.peers[me];
  int32_t *counter = reinterpret_cast<int32_t *>(mine + a.lay.counter_off);
  __shared__ uint32_t epoch_s;
  if (tid == 0) epoch_s = static_cast<uint32_t>(*reinterpret_cast<volatile int32_t *>(counter)) + 1u;
  __syncthreads();
  const uint32_t epoch = epoch_s;
  const int64_t par_off = int64_t(epoch & 1u) * a.lay.region_bytes;
  const int64_t slot_pk = a.lay.part_cap / 4;  // packets per source slot

  const int64_t part = a.n / N;       // elements of one part
  const int64_t vec_part = part / 8;  // 16-byte vectors per part
  const int64_t per = (vec_part + a.ctas - 1) / a.ctas;
  const int64_t v0 = min(vec_part, int64_t(c) * per), v1 = min(vec_part, v0 + per);
  uint4 *data_me = reinterpret_cast<uint4 *>(mine + a.lay.data_off);
  const uint64_t t0 = global_timer_ns();
  bool dead = false;

  // 1. send chunk c of part p != me to rank p's recv1[par][me]
  for (int p = 0; p < N; ++p) {
    if (p == me) continue;
    uint4 *dst = reinterpret_cast<uint4 *>(a.peers[p] + a.lay.recv1_off + par_off) + int64_t(me) * slot_pk;
    const uint4 *src = data_me + int64_t(p) * vec_part;
    for (int64_t v = v0 + tid; v < v1; v += kArThreads) send_vec(dst, v, __ldcs(src + v), epoch);
  }

  // 2. reduce chunk c of my part in rank order; keep it and send it to every rank
  const uint4 *recv1 = reinterpret_cast<const uint4 *>(mine + a.lay.recv1_off + par_off);
  for (int64_t v = v0 + tid; v < v1; v += kArThreads) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < N; ++q) {
      const uint4 x = q == me ? data_me[int64_t(me) * vec_part + v]
                              : recv_vec(recv1 + int64_t(q) * slot_pk, v, epoch, t0, dead, a.error_flag);
      add_half8(acc, x);
    }
    uint4 r;
    __half2 *rh = reinterpret_cast<__half2 *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) rh[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
    data_me[int64_t(me) * vec_part + v] = r;
    for (int p = 0; p < N; ++p) {
      if (p == me) continue;
      send_vec(reinterpret_cast<uint4 *>(a.peers[p] + a.lay.recv2_off + par_off) + int64_t(me) * slot_pk, v, r,
               epoch);
    }
  }

  // 3. collect chunk c of every other rank's reduced part
  const uint4 *recv2 = reinterpret_cast<const uint4 *>(mine + a.lay.recv2_off + par_off);
  for (int q = 0; q < N; ++q) {
    if (q == me) continue;
    for (int64_t v = v0 + tid; v < v1; v += kArThreads)
      data_me[int64_t(q) * vec_part + v] = recv_vec(recv2 + int64_t(q) * slot_pk, v, epoch, t0, dead, a.error_flag);
  }

  // the last CTA to finish publishes the epoch for the next call
  __shared__ int last;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(counter + 1, 1) == a.ctas - 1;
  }
  __syncthreads();
  if (last && tid == 0) {
    counter[1] = 0;
    __threadfence();
    *reinterpret_cast<volatile int32_t *>(counter) = static_cast<int32_t>(epoch);
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
  B200KV_CHECK_ARG(capacity_elems % (int64_t(world) * 8) == 0,
                   "capacity (%lld) must be a multiple of 8 * world", (long long)capacity_elems);
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
  a.lay = peer_layout(capacity_elems, world);
  a.ctas = ctas > 0 ? ctas : 128;
  a.error_flag = error_flag;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.ctas);
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200KV_CUDA_TRY(cudaLaunchKernelEx(&cfg, peer_allreduce_kernel, static_cast<const PeerArgs>(a)));
  return B200KV_OK;
}
