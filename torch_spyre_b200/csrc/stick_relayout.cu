// General stick relayout: a strided host-order tensor <-> a device buffer laid
// out by an arbitrary (device_size, stride_map) stick layout, on the GPU; and
// restickify, the device -> device move of a tensor from one stick layout to
// another (spyre::restickify, torch_spyre/_inductor/customops.py:338-342,
// whose target layouts torch_spyre/_inductor/pass_utils.py:749-835 derives).
//
// Restates the element map that the reference's DMA descriptors encode for
// every host<->device copy (generate_dci / get_device_stride_infos,
// torch_spyre/csrc/spyre_mem.cpp:176-440; dim matching get_dim_map 60-96):
// device dim j walks the host dim whose contiguous stride is the largest one
// <= stride_map[j], advancing it by stride_map[j] / that stride per step; the
// stick dim appears twice (stick index and element in stick); dims with
// stride_map -1 (size one, or the sparse stick) or 0 (expanded) do not move.
// Device positions that fall outside the host tensor (stick padding) are zero
// when writing the device buffer and skipped when reading it back.
#include "common.cuh"

namespace b200kv {
namespace {

constexpr int kMaxRank = 8;

struct RelayoutMap {
  int dev_rank, host_rank;
  int64_t dev_size[kMaxRank];
  int64_t dev_stride[kMaxRank];   // contiguous strides of the device buffer
  int dim[kMaxRank];              // host dim walked by device dim j, -1 = none
  int64_t mult[kMaxRank];         // host coordinate step per device step
  int64_t host_size[kMaxRank];
  int64_t host_stride[kMaxRank];  // actual element strides of the host tensor
  int64_t total;                  // device elements
  int vec;                        // 1: 8-element runs may be contiguous on both sides
};

// Host coordinates of device element e; false for padding.
__device__ __forceinline__ bool host_coords(const RelayoutMap &m, int64_t e, int64_t (&coord)[kMaxRank]) {
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) coord[d] = 0;
#pragma unroll
  for (int j = 0; j < kMaxRank; ++j) {
    if (j >= m.dev_rank) break;
    const int64_t ij = (e / m.dev_stride[j]) % m.dev_size[j];
    const int d = m.dim[j];
#pragma unroll
    for (int k = 0; k < kMaxRank; ++k)
      if (k == d) coord[k] += ij * m.mult[j];
  }
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) {
    if (d >= m.host_rank) break;
    if (coord[d] >= m.host_size[d]) return false;
  }
  return true;
}

// Device element offset of host coordinates in layout m: every device dim j
// that walks host dim d contributes ((coord_d / mult_j) % size_j) * stride_j
// (the stick dim and its outer dim split the coordinate in mixed radix).
__device__ __forceinline__ int64_t device_offset(const RelayoutMap &m, const int64_t (&coord)[kMaxRank]) {
  int64_t off = 0;
#pragma unroll
  for (int j = 0; j < kMaxRank; ++j) {
    if (j >= m.dev_rank) break;
    const int d = m.dim[j];
    int64_t c = 0;
#pragma unroll
    for (int k = 0; k < kMaxRank; ++k)
      if (k == d) c = coord[k];
    if (d >= 0) off += ((c / m.mult[j]) % m.dev_size[j]) * m.dev_stride[j];
  }
  return off;
}

// Restickify: dst device element e <- the src device element holding the
// same host element (0 for dst padding).
template <typename T>
__global__ void __launch_bounds__(256) restickify_kernel(const T *__restrict__ src, T *__restrict__ dst,
                                                         const RelayoutMap sm, const RelayoutMap dm) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < dm.total;
       e += int64_t(gridDim.x) * blockDim.x) {
    int64_t coord[kMaxRank];
    dst[e] = host_coords(dm, e, coord) ? src[device_offset(sm, coord)] : T(0);
  }
}

// Host element offset of device element e, or -1 for padding.
__device__ __forceinline__ int64_t host_offset(const RelayoutMap &m, int64_t e) {
  int64_t coord[kMaxRank];
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) coord[d] = 0;
#pragma unroll
  for (int j = 0; j < kMaxRank; ++j) {
    if (j >= m.dev_rank) break;
    const int64_t ij = (e / m.dev_stride[j]) % m.dev_size[j];
    const int d = m.dim[j];
#pragma unroll
    for (int k = 0; k < kMaxRank; ++k)
      if (k == d) coord[k] += ij * m.mult[j];
  }
  int64_t off = 0;
#pragma unroll
  for (int d = 0; d < kMaxRank; ++d) {
    if (d >= m.host_rank) break;
    if (coord[d] >= m.host_size[d]) return -1;
    off += coord[d] * m.host_stride[d];
  }
  return off;
}

// One thread per run of 8 device elements; a run that is contiguous and
// 16-byte aligned on both sides moves as one vector.
template <typename T, int kDir>
__global__ void __launch_bounds__(256) stick_relayout_kernel(const T *__restrict__ src,
                                                             T *__restrict__ dst,
                                                             const RelayoutMap m) {
  const int64_t runs = (m.total + 7) / 8;
  for (int64_t r = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; r < runs;
       r += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e0 = r * 8;
    if (m.vec && e0 + 8 <= m.total) {
      const int64_t h0 = host_offset(m, e0);
      const int64_t h7 = host_offset(m, e0 + 7);
      if (h0 >= 0 && h7 == h0 + 7 && ((h0 * static_cast<int64_t>(sizeof(T))) & 15) == 0) {
        if (kDir == 0)
          *reinterpret_cast<uint4 *>(dst + e0) = *reinterpret_cast<const uint4 *>(src + h0);
        else
          *reinterpret_cast<uint4 *>(dst + h0) = *reinterpret_cast<const uint4 *>(src + e0);
        continue;
      }
    }
    for (int k = 0; k < 8; ++k) {
      const int64_t e = e0 + k;
      if (e >= m.total) break;
      const int64_t h = host_offset(m, e);
      if (kDir == 0)
        dst[e] = h >= 0 ? src[h] : T(0);
      else if (h >= 0)
        dst[h] = src[e];
    }
  }
}

template <typename T>
void launch_typed(const void *src, void *dst, const RelayoutMap &m, int dir, int grid,
                  cudaStream_t s) {
  if (dir == 0)
    stick_relayout_kernel<T, 0><<<grid, 256, 0, s>>>(static_cast<const T *>(src), static_cast<T *>(dst), m);
  else
    stick_relayout_kernel<T, 1><<<grid, 256, 0, s>>>(static_cast<const T *>(src), static_cast<T *>(dst), m);
}

}  // namespace
}  // namespace b200kv

namespace b200kv {
namespace {

// Builds the element map of a device layout over a host tensor (dim matching
// as get_dim_map, torch_spyre/csrc/spyre_mem.cpp:60-96); returns a status.
int build_map(RelayoutMap &m, int32_t host_rank, const int64_t *host_size, const int64_t *host_stride,
              int32_t device_rank, const int64_t *device_size, const int64_t *stride_map) {
  B200KV_CHECK_ARG(host_rank >= 1 && host_rank <= kMaxRank && device_rank >= 1 && device_rank <= kMaxRank,
                   "ranks must be in [1, %d]", kMaxRank);
  B200KV_CHECK_ARG(host_size && device_size && stride_map, "null size/stride array");
  m = RelayoutMap{};
  m.dev_rank = device_rank;
  m.host_rank = host_rank;
  int64_t host_elems = 1, cstride[kMaxRank];
  for (int d = host_rank - 1; d >= 0; --d) {
    B200KV_CHECK_ARG(host_size[d] >= 0, "negative host size");
    cstride[d] = host_elems;
    host_elems *= host_size[d];
    m.host_size[d] = host_size[d];
    m.host_stride[d] = host_stride ? host_stride[d] : cstride[d];
    B200KV_CHECK_ARG(m.host_stride[d] >= 0, "negative host stride");
  }
  int64_t total = 1;
  for (int j = device_rank - 1; j >= 0; --j) {
    B200KV_CHECK_ARG(device_size[j] >= 1, "device sizes must be >= 1");
    m.dev_size[j] = device_size[j];
    m.dev_stride[j] = total;
    total *= device_size[j];
  }
  m.total = host_elems == 0 ? 0 : total;
  for (int j = 0; j < device_rank; ++j) {
    m.dim[j] = -1;
    m.mult[j] = 0;
    if (stride_map[j] <= 0 || device_size[j] == 1) continue;
    int best = -1;
    for (int d = 0; d < host_rank; ++d) {
      if (host_size[d] == 1) continue;
      if (cstride[d] <= stride_map[j] && (best < 0 || cstride[d] > cstride[best])) best = d;
    }
    if (best < 0) continue;
    if (stride_map[j] % cstride[best] != 0)
      return set_error(B200KV_ERR_UNSUPPORTED,
                       "stride_map[%d] = %lld is not a multiple of host stride %lld (folded "
                       "layouts are not supported)",
                       j, (long long)stride_map[j], (long long)cstride[best]);
    m.dim[j] = best;
    m.mult[j] = stride_map[j] / cstride[best];
  }
  for (int j = device_rank; j < kMaxRank; ++j) {
    m.dim[j] = -1;
    m.dev_size[j] = 1;
    m.dev_stride[j] = 1;
  }
  return B200KV_OK;
}

int grid_for_elems(int64_t work, int *grid) {
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  const int64_t want = (work + 255) / 256;
  *grid = static_cast<int>(want < 1 ? 1 : (want > int64_t(sms) * 16 ? int64_t(sms) * 16 : want));
  return B200KV_OK;
}

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int b200kv_stick_relayout(const void *src, void *dst, int32_t elem_bytes,
                                     int32_t host_rank, const int64_t *host_size,
                                     const int64_t *host_stride, int32_t device_rank,
                                     const int64_t *device_size, const int64_t *stride_map,
                                     int32_t direction, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(direction == 0 || direction == 1, "direction must be 0 or 1");
  B200KV_CHECK_ARG(host_stride, "null host stride array");
  B200KV_CHECK_ARG(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4, "element size %d", elem_bytes);
  RelayoutMap m;
  int st = build_map(m, host_rank, host_size, host_stride, device_rank, device_size, stride_map);
  if (st != B200KV_OK) return st;
  // 8-element runs of the innermost device dim can be contiguous in the host
  // when that dim walks a host dim of unit stride with step 1, sticks hold a
  // multiple of 8 elements and the elements are 2 bytes (one 16-byte vector)
  const int jl = device_rank - 1;
  m.vec = (m.dim[jl] >= 0 && m.mult[jl] == 1 && host_stride[m.dim[jl]] == 1 &&
           device_size[jl] % 8 == 0 && elem_bytes == 2 &&
           (reinterpret_cast<uintptr_t>(src) & 15u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0)
              ? 1
              : 0;
  if (m.total == 0) return B200KV_OK;
  B200KV_CHECK_ARG(src && dst, "null buffer");
  int grid = 0;
  st = grid_for_elems((m.total + 7) / 8, &grid);
  if (st != B200KV_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (elem_bytes) {
    case 1: launch_typed<uint8_t>(src, dst, m, direction, grid, s); break;
    case 2: launch_typed<uint16_t>(src, dst, m, direction, grid, s); break;
    default: launch_typed<uint32_t>(src, dst, m, direction, grid, s); break;
  }
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}

extern "C" int b200kv_stick_restickify(const void *src, void *dst, int32_t elem_bytes, int32_t host_rank,
                                       const int64_t *host_size, int32_t src_rank,
                                       const int64_t *src_device_size, const int64_t *src_stride_map,
                                       int32_t dst_rank, const int64_t *dst_device_size,
                                       const int64_t *dst_stride_map, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4, "element size %d", elem_bytes);
  RelayoutMap sm, dm;
  int st = build_map(sm, host_rank, host_size, nullptr, src_rank, src_device_size, src_stride_map);
  if (st != B200KV_OK) return st;
  st = build_map(dm, host_rank, host_size, nullptr, dst_rank, dst_device_size, dst_stride_map);
  if (st != B200KV_OK) return st;
  if (dm.total == 0) return B200KV_OK;
  B200KV_CHECK_ARG(src && dst, "null buffer");
  int grid = 0;
  st = grid_for_elems(dm.total, &grid);
  if (st != B200KV_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (elem_bytes) {
    case 1:
      restickify_kernel<uint8_t><<<grid, 256, 0, s>>>(static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst), sm, dm);
      break;
    case 2:
      restickify_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t *>(src), static_cast<uint16_t *>(dst), sm, dm);
      break;
    default:
      restickify_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t *>(src), static_cast<uint32_t *>(dst), sm, dm);
      break;
  }
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}
