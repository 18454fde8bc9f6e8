// Merge of attention outputs computed over disjoint KV sets, through their
// log-sum-exps: for row r (a (sequence, head) pair) with parts i = 0..n-1,
//     m   = max_i lse_i,   w_i = exp(lse_i - m),
//     out = sum_i w_i * o_i / sum_i w_i,   lse = m + log(sum_i w_i).
// This is the split-KV combine of the decode kernel (which runs it on its own
// partials internally) exposed for callers that split the KV themselves, e.g.
// a shared-prefix cache decoded separately from each sequence's own pages.
// A part with lse = -inf (no keys) has weight 0; a row whose parts are all
// empty gives a zero output and lse -inf.  One warp per row, dims strided by
// lane, parts folded in order.
#include "common.cuh"

namespace b200kv {
namespace {

template <typename Tin>
__global__ void __launch_bounds__(256) lse_combine_kernel(const Tin *__restrict__ part_o,
                                                          const float *__restrict__ part_lse, int64_t n,
                                                          int64_t rows, int64_t d, __half *__restrict__ out,
                                                          float *__restrict__ lse_out) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) / 32; r < rows;
       r += int64_t(gridDim.x) * blockDim.x / 32) {
    float m = -INFINITY;
    for (int64_t i = 0; i < n; ++i) m = fmaxf(m, __ldg(part_lse + i * rows + r));
    float wsum = 0.f;
    for (int64_t i = 0; i < n; ++i) {
      const float l = __ldg(part_lse + i * rows + r);
      wsum += l == -INFINITY ? 0.f : expf(l - m);
    }
    for (int64_t k = lane; k < d; k += 32) {
      float acc = 0.f;
      for (int64_t i = 0; i < n; ++i) {
        const float l = __ldg(part_lse + i * rows + r);
        if (l == -INFINITY) continue;
        const float o = static_cast<float>(part_o[(i * rows + r) * d + k]);
        acc = fmaf(expf(l - m), o, acc);
      }
      out[r * d + k] = __float2half_rn(wsum > 0.f ? acc / wsum : 0.f);
    }
    if (lane == 0 && lse_out) lse_out[r] = wsum > 0.f ? m + logf(wsum) : -INFINITY;
  }
}

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int b200kv_lse_combine_f32(const void *part_o, int32_t part_elem_bytes, const float *part_lse,
                                      int64_t num_parts, int64_t rows, int64_t head_dim, void *out,
                                      float *lse_out, void *stream) {
  clear_error();
  B200KV_CHECK_ARG(part_elem_bytes == 2 || part_elem_bytes == 4,
                   "part_elem_bytes must be 2 (fp16 parts) or 4 (fp32 parts), got %d", part_elem_bytes);
  B200KV_CHECK_ARG(num_parts >= 1 && rows >= 0 && head_dim >= 1, "num_parts >= 1, rows >= 0, head_dim >= 1");
  if (rows == 0) return B200KV_OK;
  B200KV_CHECK_ARG(part_o && part_lse && out, "null pointer argument");
  int dev = 0, sms = 0;
  int st = current_device_sm_count(&dev, &sms);
  if (st != B200KV_OK) return st;
  const int64_t want = (rows * 32 + 255) / 256;
  const int grid = static_cast<int>(want > int64_t(sms) * 8 ? int64_t(sms) * 8 : want);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (part_elem_bytes == 2)
    lse_combine_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half *>(part_o), part_lse, num_parts, rows,
                                                    head_dim, static_cast<__half *>(out), lse_out);
  else
    lse_combine_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float *>(part_o), part_lse, num_parts, rows,
                                                   head_dim, static_cast<__half *>(out), lse_out);
  B200KV_CUDA_TRY(cudaGetLastError());
  return B200KV_OK;
}
