// Host-side part of the C ABI: error reporting, cached device attributes,
// tensor-map encoding and the stick-layout algebra (no GPU needed for the
// latter).
#include <mutex>
#include <vector>

#include "common.cuh"

namespace b200kv {

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int clear_error() {
  g_last_error.clear();
  return B200KV_OK;
}

int cuda_status(cudaError_t err, const char *what) {
  return set_error(B200KV_ERR_CUDA, "CUDA error %d (%s) in %s", static_cast<int>(err),
                   cudaGetErrorString(err), what);
}

int current_device_sm_count(int *device_out, int *sms_out) {
  constexpr int kMaxDevices = 64;
  static int cached[kMaxDevices] = {0};  // cached device attribute, 0 = unknown
  int dev = 0;
  B200KV_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(B200KV_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  int sms = __atomic_load_n(&cached[dev], __ATOMIC_RELAXED);
  if (sms == 0) {
    B200KV_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    __atomic_store_n(&cached[dev], sms, __ATOMIC_RELAXED);
  }
  *device_out = dev;
  *sms_out = sms;
  return B200KV_OK;
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

#ifndef B200KV_L2_PROMOTION
#define B200KV_L2_PROMOTION CU_TENSOR_MAP_L2_PROMOTION_L2_256B
#endif
constexpr CUtensorMapL2promotion kPagePromotion = B200KV_L2_PROMOTION;

int make_page_pool_map(CUtensorMap *map, const void *pool, int64_t num_blocks,
                       int64_t num_kv_heads, int elem_bytes) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return set_error(B200KV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(pool) & 15u) != 0)
    return set_error(B200KV_ERR_INVALID_ARG, "KV pool must be 16-byte aligned");
  const int64_t pages = num_blocks * num_kv_heads;
  if (pages <= 0 || pages > (int64_t{1} << 31) - 1)
    return set_error(B200KV_ERR_INVALID_ARG, "pool page count %lld out of range",
                     static_cast<long long>(pages));
  if (elem_bytes != 1 && elem_bytes != 2)
    return set_error(B200KV_ERR_INVALID_ARG, "page element size %d", elem_bytes);
  // dim0: the elements of one 128-byte stick, dim1: S*64 stick rows of a page,
  // dim2: pages (block * Hkv + head).
  const bool fp8 = elem_bytes == 1;
  const cuuint32_t stick = fp8 ? kStickElemsFp8 : kStickElems;
  const cuuint32_t rows = (fp8 ? kSticksFp8 : kSticks) * kPageTokens;
  cuuint64_t dims[3] = {stick, rows, static_cast<cuuint64_t>(pages)};
  cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(fp8 ? kPageBytesFp8 : kPageBytes)};
  cuuint32_t box[3] = {stick, rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void *>(pool), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, kPagePromotion,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(B200KV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return B200KV_OK;
}

}  // namespace b200kv

using namespace b200kv;

extern "C" int b200kv_version(void) { return 100; }  // 0.1.0

extern "C" int b200kv_last_error(char *buf, size_t len) {
  const std::string &m = g_last_error;
  if (buf && len > 0) {
    size_t n = m.size() < len - 1 ? m.size() : len - 1;
    memcpy(buf, m.data(), n);
    buf[n] = '\0';
  }
  return static_cast<int>(m.size());
}

// Stick layout algebra.  The tiling rule: with host dim order o[0..r-1], the
// device dims are o[1], ..., o[r-1], o[0], o[r-1]; the last entry is the stick
// (elements inside one 128-byte stick) and the other occurrence of the stick
// dim counts sticks.  A trailing -1 in the dim order makes the layout sparse
// (one element per stick).  Strides of the stride map are host element strides:
// the innermost occurrence of a host dim gets that dim's host stride, each
// outer occurrence the inner stride times the inner device size; a size-1 host
// dim (or the sparse -1) gets -1.
extern "C" int b200kv_stick_layout(const int64_t *host_size, const int64_t *host_stride,
                                   int32_t rank, const int32_t *dim_order, int32_t order_len,
                                   int32_t elem_bytes, int64_t *device_size,
                                   int64_t *stride_map, int32_t cap, int32_t *out_rank) {
  clear_error();
  B200KV_CHECK_ARG(rank >= 0 && rank <= 6, "Unsupported tensor rank: %d", rank);
  B200KV_CHECK_ARG(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8,
                   "unsupported element size %d", elem_bytes);
  B200KV_CHECK_ARG(device_size && stride_map && out_rank, "null output pointer");
  B200KV_CHECK_ARG(rank == 0 || host_size, "null host_size");
  const int64_t elems_per_stick = 128 / elem_bytes;
  if (rank == 0) {  // scalar: one stick, no strides
    B200KV_CHECK_ARG(cap >= 2, "output capacity %d < 2", cap);
    device_size[0] = 1;
    device_size[1] = elems_per_stick;
    stride_map[0] = -1;
    stride_map[1] = -1;
    *out_rank = 2;
    return B200KV_OK;
  }
  std::vector<int32_t> order;
  if (dim_order) {
    order.assign(dim_order, dim_order + order_len);
  } else {
    for (int32_t i = 0; i < rank; ++i) order.push_back(i);
  }
  const int32_t n_order = static_cast<int32_t>(order.size());
  const bool sparse = n_order == rank + 1 && order.back() == -1;
  B200KV_CHECK_ARG(n_order == rank || sparse, "Incompatible host_size and dim_order");
  for (int32_t i = 0; i < n_order; ++i)
    B200KV_CHECK_ARG(order[i] >= -1 && order[i] < rank, "dim_order entry %d out of range",
                     order[i]);
  std::vector<int64_t> hstride(rank);
  if (host_stride) {
    hstride.assign(host_stride, host_stride + rank);
  } else {
    int64_t s = 1;
    for (int32_t i = rank - 1; i >= 0; --i) {
      hstride[i] = s;
      s *= host_size[i];
    }
  }
  // Tiling (dim map): the order's dims after the first, then the first, then
  // the stick dim (the order's last entry) again.
  std::vector<int32_t> dmap;
  for (int32_t i = 1; i < n_order; ++i) dmap.push_back(order[i]);
  dmap.push_back(order[0]);
  dmap.push_back(order[n_order - 1]);
  const int32_t n = static_cast<int32_t>(dmap.size());
  B200KV_CHECK_ARG(cap >= n, "output capacity %d < device rank %d", cap, n);
  const int32_t stick_dim = dmap[n - 1];
  device_size[n - 1] = elems_per_stick;
  for (int32_t i = 0; i < n - 1; ++i) {
    const int32_t d = dmap[i];
    if (d == stick_dim)
      device_size[i] = sparse ? 1 : (host_size[d] + elems_per_stick - 1) / elems_per_stick;
    else
      device_size[i] = host_size[d];
  }
  std::vector<int64_t> outer(rank, -1);  // stride of the next outer occurrence
  for (int32_t j = n - 1; j >= 0; --j) {
    const int32_t d = dmap[j];
    if (d < 0 || host_size[d] == 1) {
      stride_map[j] = -1;
      continue;
    }
    stride_map[j] = outer[d] == -1 ? hstride[d] : outer[d];
    outer[d] = stride_map[j] * device_size[j];
  }
  *out_rank = n;
  return B200KV_OK;
}

extern "C" int64_t b200kv_device_size_in_bytes(const int64_t *device_size, int32_t device_rank) {
  if (!device_size || device_rank < 1) return -1;
  int64_t sticks = 1;
  for (int32_t i = 0; i < device_rank - 1; ++i) sticks *= device_size[i];
  return sticks * 128;
}
