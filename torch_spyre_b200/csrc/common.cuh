// Shared helpers of libb200kv: status reporting, PTX wrappers for mbarriers and
// TMA (cp.async.bulk.tensor), cached device attributes.  sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/b200kv.h"

namespace b200kv {

constexpr int kPageTokens = 64;    // tokens per page (one block-table entry)
constexpr int kStickElems = 64;    // fp16 elements per 128-byte stick
constexpr int kHeadDim = 128;      // the head_dim the kernels are built for
constexpr int kSticks = kHeadDim / kStickElems;               // 2
constexpr int kPageElems = kPageTokens * kHeadDim;            // 8192
constexpr int kPageBytes = kPageElems * 2;                    // 16 KiB
constexpr int kStickBytes = kPageTokens * kStickElems * 2;    // 8 KiB per stick column
// fp8 (e4m3) pages: a 128-byte stick holds 128 elements, so a D = 128 page is
// one stick column of 64 token rows.
constexpr int kStickElemsFp8 = 128;
constexpr int kSticksFp8 = kHeadDim / kStickElemsFp8;         // 1
constexpr int kPageBytesFp8 = kPageTokens * kHeadDim;         // 8 KiB

// ---------------------------------------------------------------- status ----
// Sets the calling thread's last-error message and returns `code`.
int set_error(int code, const char *fmt, ...);
int clear_error();
int cuda_status(cudaError_t err, const char *what);

#define B200KV_CHECK_ARG(cond, ...)                          \
  do {                                                       \
    if (!(cond)) return ::b200kv::set_error(B200KV_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define B200KV_CUDA_TRY(expr)                                          \
  do {                                                                 \
    cudaError_t e_ = (expr);                                           \
    if (e_ != cudaSuccess) return ::b200kv::cuda_status(e_, #expr);    \
  } while (0)

// Number of SMs of the current device (cached per device ordinal).
int current_device_sm_count(int *device_out, int *sms_out);

// cuTensorMapEncodeTiled resolved through the runtime's driver entry point
// (no link-time dependency on libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t,
                                   void *, const cuuint64_t *, const cuuint64_t *,
                                   const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// Tensor map over a page pool viewed as 3-D (one 128-byte stick of elements,
// 64*S stick rows, NB*Hkv pages) with a box of one whole page and the 128-byte
// swizzle.  elem_bytes 2: fp16 pages (64-element sticks, S = D/64);
// elem_bytes 1: fp8 pages (128-element sticks, S = D/128).
int make_page_pool_map(CUtensorMap *map, const void *pool, int64_t num_blocks,
                       int64_t num_kv_heads, int elem_bytes = 2);

// --------------------------------------------------------------- device ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: gives up after kWaitLimitNs of wall
// clock (%globaltimer), records B200KV_DEVERR_TIMEOUT and lets the caller go on
// (its shared-memory reads stay in bounds), so a lost transfer can never hang
// the GPU.  A healthy page transfer completes in microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ void mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  int32_t *error_flag) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) break;
  }
  if (error_flag) atomicOr(error_flag, B200KV_DEVERR_TIMEOUT);
}

// L2 policy of the streamed KV pages (read once per launch): evict first.
#ifndef B200KV_KV_POLICY
#define B200KV_KV_POLICY "evict_first"
#endif
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::" B200KV_KV_POLICY ".b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 3-D tiled TMA load of one box into shared memory, completing on `bar`.
// No multicast: every CTA fetches its own pages.
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map,
                                            uint64_t *bar, int c0, int c1, int c2,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// Untiled bulk copy global -> shared of `bytes` (both addresses 16-byte
// aligned, bytes a multiple of 16), completing on `bar`.  No multicast.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Byte offset, inside a page staged with the 128-byte swizzle, of 16-byte chunk
// `chunk` (0..7) of stick `stick` of token row `t`.  The swizzle XORs the chunk
// index with the row index modulo 8 (rows are 128 B, atoms 1024 B).
__device__ __forceinline__ uint32_t swz_off(int stick, int t, int chunk) {
  return static_cast<uint32_t>(stick * kStickBytes + t * 128 + ((chunk ^ (t & 7)) << 4));
}

}  // namespace b200kv
