// Standalone rotary position embedding of fp16 head rows (rope.cuh has the
// formula and its rounding).  One thread per (token, head, pair of adjacent
// frequencies): it loads both halves' pairs, rotates them and stores them.
#include "rope.cuh"

namespace b200kv {
namespace {

__global__ void __launch_bounds__(256) rope_kernel(const __half *__restrict__ x, int64_t xs_t, int64_t xs_h,
                                                   __half *__restrict__ out, int64_t os_t, int64_t os_h,
                                                   const __half *__restrict__ freqs, int64_t max_pos,
                                                   const int32_t *__restrict__ positions, int64_t tokens,
                                                   int heads, int half_d, int32_t *error_flag) {
  const int pairs = half_d / 2;
  const int64_t total = tokens * heads * pairs;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(i % pairs) * 2;
    const int64_t th = i / pairs;
    const int h = static_cast<int>(th % heads);
    const int64_t t = th / heads;
    int64_t pos = __ldg(positions + t);
    if (pos < 0 || pos >= max_pos) {
      if (error_flag && e == 0 && h == 0) atomicOr(error_flag, B200KV_DEVERR_BAD_LEN);
      pos = pos < 0 ? 0 : max_pos - 1;
    }
    const __half *row = x + t * xs_t + h * xs_h;
    uint32_t x0 = *reinterpret_cast<const uint32_t *>(row + e);
    uint32_t x1 = *reinterpret_cast<const uint32_t *>(row + half_d + e);
    rope_pair(freqs + pos * 4 * half_d, half_d, e, x0, x1);
    __half *orow = out + t * os_t + h * os_h;
    *reinterpret_cast<uint32_t *>(orow + e) = x0;
    *reinterpret_cast<uint32_t *>(orow + half_d + e) = x1;
  }
}

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int b200kv_rope_f16(const void *x, int64_t x_stride_t, int64_t x_stride_h, void *out,
                               int64_t out_stride_t, int64_t out_stride_h, const void *freqs, int64_t max_pos,
                               const int32_t *positions, int64_t num_tokens, int64_t num_heads, int64_t head_dim,
                               int32_t *error_flag, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(num_tokens >= 0 && num_heads > 0, "num_tokens must be >= 0 and num_heads > 0");
  B200KV_CHECK_ARG(head_dim > 0 && head_dim % 4 == 0 && head_dim <= 4096,
                   "head_dim (%lld) must be a positive multiple of 4", (long long)head_dim);
  B200KV_CHECK_ARG(max_pos > 0, "max_pos must be > 0");
  if (num_tokens == 0) return B200KV_OK;
  B200KV_CHECK_ARG(x && out && freqs && positions, "null pointer argument");
  B200KV_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 3u) == 0 && (reinterpret_cast<uintptr_t>(out) & 3u) == 0 &&
                       (reinterpret_cast<uintptr_t>(freqs) & 3u) == 0 && x_stride_t % 2 == 0 &&
                       x_stride_h % 2 == 0 && out_stride_t % 2 == 0 && out_stride_h % 2 == 0,
                   "x / out / freqs must be 4-byte aligned with even strides");
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  const int64_t work = num_tokens * num_heads * (head_dim / 4);
  const int64_t want = (work + 255) / 256;
  const int grid = static_cast<int>(want < 1 ? 1 : (want > int64_t(sms) * 8 ? int64_t(sms) * 8 : want));
  rope_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half *>(x), x_stride_t, x_stride_h, static_cast<__half *>(out), out_stride_t,
      out_stride_h, static_cast<const __half *>(freqs), max_pos, positions, num_tokens, static_cast<int>(num_heads),
      static_cast<int>(head_dim / 2), error_flag);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}
