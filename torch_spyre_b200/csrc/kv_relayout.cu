// KV append (slot write) and bulk relayout between a row-major KV cache and the
// paged stick layout.  Pure data movement, bit-exact: every thread moves
// 16-byte vectors, reads and writes are coalesced into 128-byte stick rows.
//
// Reference behaviour replaced:
//   append   -- spyre::overwrite / overwrite_cpu (torch_spyre/_inductor/
//               customops.py:262-308) and the aten.index_copy.out CPU fallback
//               (torch_spyre/ops/fallbacks.py:237-259) that HF KV caches hit;
//   relayout -- the host<->device stick relayout loop nest of generate_dci
//               (torch_spyre/csrc/spyre_mem.cpp:176-440), here HBM -> HBM.
#include "common.cuh"

namespace b200kv {
namespace {

constexpr int kChunks = kHeadDim / 8;  // 16-byte chunks per head row (16)

// Element offset of (page, stick, slot, elem) inside a pool.
__device__ __forceinline__ int64_t pool_offset(int64_t page, int chunk, int slot) {
  return (page * kSticks + (chunk >> 3)) * (kPageTokens * kStickElems) +
         static_cast<int64_t>(slot) * kStickElems + (chunk & 7) * 8;
}

// One thread per (token, head, 16-byte chunk); K and V moved by the same thread.
__global__ void __launch_bounds__(256) kv_append_kernel(
    const __half *__restrict__ k_new, const __half *__restrict__ v_new, int64_t stride_n,
    int64_t stride_h, __half *__restrict__ k_pool, __half *__restrict__ v_pool,
    const int64_t *__restrict__ slots, int64_t num_tokens, int num_kv_heads,
    int64_t num_slots, int32_t *error_flag) {
  const int64_t total = num_tokens * num_kv_heads * kChunks;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % kChunks);
    const int64_t nh = i / kChunks;
    const int h = static_cast<int>(nh % num_kv_heads);
    const int64_t n = nh / num_kv_heads;
    const int64_t slot = __ldg(slots + n);
    if (slot < 0) continue;  // padding token
    if (slot >= num_slots) {
      if (error_flag && c == 0 && h == 0) atomicOr(error_flag, B200KV_DEVERR_BAD_SLOT);
      continue;
    }
    const int64_t page = (slot >> 6) * num_kv_heads + h;
    const int64_t dst = pool_offset(page, c, static_cast<int>(slot & 63));
    const int64_t src = n * stride_n + h * stride_h + c * 8;
    const uint4 kv = __ldg(reinterpret_cast<const uint4 *>(k_new + src));
    const uint4 vv = __ldg(reinterpret_cast<const uint4 *>(v_new + src));
    *reinterpret_cast<uint4 *>(k_pool + dst) = kv;
    *reinterpret_cast<uint4 *>(v_pool + dst) = vv;
  }
}

// One thread moves kUnroll 16-byte chunks (grid-stride), all loads issued
// before the stores for memory-level parallelism.
constexpr int kUnroll = 4;

template <int kDir>
__global__ void __launch_bounds__(256) relayout_kernel(
    __half *__restrict__ rows, __half *__restrict__ pool, const int32_t *__restrict__ block_ids,
    int64_t num_tokens, int num_kv_heads, int64_t num_blocks, int32_t *error_flag) {
  const int64_t total = num_tokens * num_kv_heads * kChunks;
  const int64_t step = int64_t(gridDim.x) * blockDim.x;
  for (int64_t base = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; base < total;
       base += step * kUnroll) {
    uint4 v[kUnroll];
    int64_t dst[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * step;
      dst[u] = -1;
      if (i >= total) continue;
      const int c = static_cast<int>(i % kChunks);
      const int64_t th = i / kChunks;
      const int h = static_cast<int>(th % num_kv_heads);
      const int64_t t = th / num_kv_heads;
      const int32_t blk = __ldg(block_ids + (t >> 6));
      if (blk < 0 || blk >= num_blocks) {
        if (error_flag && c == 0 && h == 0 && (t & 63) == 0)
          atomicOr(error_flag, B200KV_DEVERR_BAD_BLOCK);
        continue;
      }
      const int64_t poff = pool_offset(int64_t(blk) * num_kv_heads + h, c, int(t & 63));
      const int64_t roff = i * 8;
      if (kDir == 0) {
        v[u] = __ldcs(reinterpret_cast<const uint4 *>(rows + roff));
        dst[u] = poff;
      } else {
        v[u] = __ldcs(reinterpret_cast<const uint4 *>(pool + poff));
        dst[u] = roff;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (dst[u] < 0) continue;
      __half *out = kDir == 0 ? pool : rows;
      __stcs(reinterpret_cast<uint4 *>(out + dst[u]), v[u]);
    }
  }
}

int grid_for(int64_t work_items, int threads, int per_thread) {
  int dev = 0, sms = 0;
  if (current_device_sm_count(&dev, &sms) != B200KV_OK) return -1;
  const int64_t want = (work_items + int64_t(threads) * per_thread - 1) / (int64_t(threads) * per_thread);
  const int64_t cap = int64_t(sms) * 8;  // 8 resident 256-thread CTAs per SM
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int b200kv_kv_append_f16(const void *k_new, const void *v_new, int64_t new_stride_n,
                                    int64_t new_stride_h, void *k_pool, void *v_pool,
                                    const int64_t *slot_mapping, int64_t num_tokens,
                                    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
                                    int32_t *error_flag, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(num_tokens >= 0, "num_tokens must be >= 0 (got %lld)", (long long)num_tokens);
  B200KV_CHECK_ARG(num_kv_heads > 0 && num_blocks > 0, "num_kv_heads and num_blocks must be > 0");
  if (head_dim != kHeadDim)
    return set_error(B200KV_ERR_UNSUPPORTED, "head_dim %lld unsupported (only %d)",
                     (long long)head_dim, kHeadDim);
  if (num_tokens == 0) return B200KV_OK;
  B200KV_CHECK_ARG(k_new && v_new && k_pool && v_pool && slot_mapping, "null pointer argument");
  B200KV_CHECK_ARG(aligned16(k_new) && aligned16(v_new) && aligned16(k_pool) && aligned16(v_pool),
                   "buffers must be 16-byte aligned");
  B200KV_CHECK_ARG(new_stride_n % 8 == 0 && new_stride_h % 8 == 0 && new_stride_h >= kHeadDim &&
                       new_stride_n >= 0,
                   "new-row strides must be multiples of 8 elements (got %lld, %lld)",
                   (long long)new_stride_n, (long long)new_stride_h);
  const int threads = 256;
  const int grid = grid_for(num_tokens * num_kv_heads * 16, threads, 1);
  if (grid < 0) return B200KV_ERR_CUDA;
  kv_append_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half *>(k_new), static_cast<const __half *>(v_new), new_stride_n,
      new_stride_h, static_cast<__half *>(k_pool), static_cast<__half *>(v_pool), slot_mapping,
      num_tokens, static_cast<int>(num_kv_heads), num_blocks * kPageTokens, error_flag);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}

extern "C" int b200kv_relayout_f16(void *rows, void *pool, const int32_t *block_ids,
                                   int64_t num_tokens, int64_t num_kv_heads, int64_t head_dim,
                                   int64_t num_blocks, int32_t direction, int32_t *error_flag,
                                   void *stream) {
  clear_error();
  B200KV_CHECK_ARG(direction == 0 || direction == 1, "direction must be 0 or 1 (got %d)",
                   direction);
  B200KV_CHECK_ARG(num_tokens >= 0, "num_tokens must be >= 0");
  B200KV_CHECK_ARG(num_kv_heads > 0 && num_blocks > 0, "num_kv_heads and num_blocks must be > 0");
  if (head_dim != kHeadDim)
    return set_error(B200KV_ERR_UNSUPPORTED, "head_dim %lld unsupported (only %d)",
                     (long long)head_dim, kHeadDim);
  if (num_tokens == 0) return B200KV_OK;
  B200KV_CHECK_ARG(rows && pool && block_ids, "null pointer argument");
  B200KV_CHECK_ARG(aligned16(rows) && aligned16(pool), "buffers must be 16-byte aligned");
  const int threads = 256;
  const int grid = grid_for(num_tokens * num_kv_heads * 16, threads, kUnroll);
  if (grid < 0) return B200KV_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (direction == 0)
    relayout_kernel<0><<<grid, threads, 0, s>>>(static_cast<__half *>(rows),
                                                static_cast<__half *>(pool), block_ids, num_tokens,
                                                static_cast<int>(num_kv_heads), num_blocks,
                                                error_flag);
  else
    relayout_kernel<1><<<grid, threads, 0, s>>>(static_cast<__half *>(rows),
                                                static_cast<__half *>(pool), block_ids, num_tokens,
                                                static_cast<int>(num_kv_heads), num_blocks,
                                                error_flag);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}
