// Decode attention for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc or an allocator at the
// point where they launch decode attention: an inference engine that must
// not allocate while it replays pre-planned memory, a plugin host that hands
// out only the tensors it owns, or code that runs inside another framework's
// memory budget.  b200kv_decode_attention_f16 needs a caller-provided
// workspace for its split-KV partials; this variant takes no workspace and
// uses a fixed-size scratch array that lives in the library's own device
// memory instead.
//
// The scratch is a file-scope __device__ array, so every GPU that loads the
// library holds it (kScratchBytes) until the process exits.  Its device
// address is looked up with cudaGetSymbolAddress (host code may not use the
// array's name as a device pointer) by the first call on each device, with
// that device current, so make that first call before any stream capture.
// Only a successful lookup is kept: a call whose lookup failed returns the
// CUDA error and the next call on that device tries again.
// All calls on a device share the array and it keeps the last call's data:
// each call clears the completion counters it uses, and calls that overlap on
// the GPU (different streams, no ordering between them) race on the scratch.
// The caller still passes all inputs and outputs.
// Limit: batch * num_kv_heads <= 16384 and
//   64 KiB + (batch * num_kv_heads + SMs) * G * 520 bytes <= 16 MiB
// (G = num_q_heads / num_kv_heads, SMs = 148 on B200; 520 = 128 fp32 outputs
// plus one (max, sum) pair per query head, the 256-byte alignment of the
// partial region aside): at most about 15900 (sequence, KV head) pairs at
// G = 2, 7880 at G = 4, 3860 at G = 8.  Larger sizes are rejected with
// B200KV_ERR_UNSUPPORTED before anything is launched.
#include <atomic>
#include <cmath>
#include <mutex>

#include "decode_kernels.h"

namespace b200kv {
namespace {

constexpr int64_t kScratchBytes = 16ll << 20;          // 16 MiB per device
constexpr int64_t kNoAllocMaxPairs = 16384;            // batch * num_kv_heads
constexpr int64_t kCounterBytes = kNoAllocMaxPairs * 4;

static __device__ __align__(256) uint8_t g_decode_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<uint8_t *> g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device `dev`.  A
// successful lookup is cached; a failed one is not, so a later call retries.
int scratch_address(int dev, uint8_t **out) {
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(B200KV_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  uint8_t *p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void *addr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&addr, g_decode_scratch);
      if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress");
      p = static_cast<uint8_t *>(addr);
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return B200KV_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int b200kv_decode_attention_f16_noalloc(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool, const void *v_pool,
    const int32_t *block_table, int64_t block_table_stride, const int32_t *context_lens, void *out,
    int64_t out_stride_b, int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq,
    float scale, int32_t *error_flag, void *stream) {
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
  B200KV_CHECK_ARG(num_blocks > 0 && max_blocks_per_seq > 0,
                   "num_blocks and max_blocks_per_seq must be > 0");
  B200KV_CHECK_ARG(max_blocks_per_seq * kPageTokens < (int64_t{1} << 31), "max_blocks_per_seq too large");
  B200KV_CHECK_ARG(block_table_stride >= max_blocks_per_seq, "block_table_stride < max_blocks_per_seq");
  B200KV_CHECK_ARG(std::isfinite(scale), "scale must be finite");
  if (batch * num_kv_heads * max_blocks_per_seq >= (int64_t{1} << 31))
    return set_error(B200KV_ERR_UNSUPPORTED, "batch * num_kv_heads * max_blocks_per_seq >= 2^31");
  if (batch == 0) return B200KV_OK;
  B200KV_CHECK_ARG(q && k_pool && v_pool && block_table && context_lens && out,
                   "null pointer argument");
  B200KV_CHECK_ARG(aligned16(q) && q_stride_b % 8 == 0 && q_stride_h % 8 == 0,
                   "q must be 16-byte aligned with strides that are multiples of 8 elements");

  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  // Scratch need: completion counters for every (sequence, KV head) pair and
  // one partial (G x 128 outputs + G (max, sum) pairs) per pair and per CTA.
  const int64_t pairs = batch * num_kv_heads;
  const int64_t slots = pairs + sms;
  const int64_t ml_off = kCounterBytes;
  const int64_t o_off = (ml_off + slots * group * 8 + 255) & ~int64_t(255);
  const int64_t need = o_off + slots * group * kHeadDim * 4;
  if (pairs > kNoAllocMaxPairs || need > kScratchBytes)
    return set_error(B200KV_ERR_UNSUPPORTED,
                     "batch %lld x %lld KV heads needs %lld scratch bytes; the no-allocation "
                     "entry point has %lld (use b200kv_decode_attention_f16 with a workspace)",
                     (long long)batch, (long long)num_kv_heads, (long long)need,
                     (long long)kScratchBytes);
  uint8_t *scratch = nullptr;
  st = scratch_address(dev, &scratch);
  if (st != B200KV_OK) return st;

  CUtensorMap km, vm;
  st = make_page_pool_map(&km, k_pool, num_blocks, num_kv_heads);
  if (st != B200KV_OK) return st;
  st = make_page_pool_map(&vm, v_pool, num_blocks, num_kv_heads);
  if (st != B200KV_OK) return st;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The counters must start at zero; the previous call's contents may remain.
  B200KV_CUDA_TRY(cudaMemsetAsync(scratch, 0, pairs * 4, s));

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
  a.counters = reinterpret_cast<int *>(scratch);
  a.part_ml = reinterpret_cast<float2 *>(scratch + ml_off);
  a.part_o = reinterpret_cast<float *>(scratch + o_off);
  a.error_flag = error_flag;
  // one partition per SM, the same partition as the default entry point
  return launch_decode_mma(static_cast<int>(group), km, vm, a, sms, s);
}
