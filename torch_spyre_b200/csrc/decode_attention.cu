// C-ABI entry of paged decode attention: argument validation, tensor maps
// over the two page pools, and dispatch to the decode kernel.
//
// Computes, for every sequence b and query head h (GQA group g = h % G of KV
// head h / G, G = Hq / Hkv),
//     out[b, h, :] = softmax(scale * q[b, h, :] . K_b^T) . V_b
// over the ctx_b tokens of sequence b, whose K/V rows live in 64-token pages
// of the paged stick layout (include/b200kv.h).  This is the decode case of the
// reference's SDPA decomposition spyre__sdpa_overrideable
// (torch_spyre/_inductor/decompositions.py:523-611): scores -> softmax -> P.V
// with GQA by KV-head expansion (560-563), computed here with fp32
// accumulation and the scale applied once.
//
// Kernels: decode_mma.cu (tensor cores, default) and decode_simt.cu (CUDA-core
// fp32, selected with the environment variable B200KV_DECODE_KERNEL=simt).
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "decode_kernels.h"

namespace b200kv {
namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool use_simt_kernel() {
  static const bool simt = [] {
    const char *v = std::getenv("B200KV_DECODE_KERNEL");
    return v && std::strcmp(v, "simt") == 0;
  }();
  return simt;
}

}  // namespace
}  // namespace b200kv

using namespace b200kv;

extern "C" int64_t b200kv_decode_workspace_bytes(int64_t batch, int64_t num_q_heads,
                                                 int64_t num_kv_heads, int64_t head_dim) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 ||
      head_dim != kHeadDim)
    return -1;
  return workspace_layout(batch, num_q_heads, num_kv_heads).total;
}

// The name the build contract gives the workspace query (same arguments).
extern "C" int64_t b200kv_query_workspace_bytes(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                                int64_t head_dim) {
  return b200kv_decode_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim);
}

static int decode_entry(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool, const void *v_pool,
    const int32_t *block_table, int64_t block_table_stride, const int32_t *context_lens, void *out,
    int64_t out_stride_b, int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq,
    float scale, int64_t num_splits, void *workspace, int64_t workspace_bytes,
    int32_t *error_flag, void *stream, const void *k_new, const void *v_new, int64_t new_sb,
    int64_t new_sh, bool append, bool fp8 = false, const void *k_scale = nullptr,
    const void *v_scale = nullptr, const void *rope_freqs = nullptr, int64_t rope_max_pos = 0,
    uint32_t flags = 0) {
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
  if (batch * num_kv_heads > kMaxCounters)
    return set_error(B200KV_ERR_UNSUPPORTED, "batch * num_kv_heads %lld > %lld unsupported",
                     (long long)(batch * num_kv_heads), (long long)kMaxCounters);
  B200KV_CHECK_ARG(num_blocks > 0 && max_blocks_per_seq > 0, "num_blocks and max_blocks_per_seq must be > 0");
  B200KV_CHECK_ARG(max_blocks_per_seq * kPageTokens < (int64_t{1} << 31), "max_blocks_per_seq too large");
  B200KV_CHECK_ARG(block_table_stride >= max_blocks_per_seq, "block_table_stride < max_blocks_per_seq");
  B200KV_CHECK_ARG(num_splits >= 0 && num_splits <= kMaxPartitions, "num_splits must be in [0, %d]",
                   kMaxPartitions);
  if (batch * num_kv_heads * max_blocks_per_seq >= (int64_t{1} << 31))
    return set_error(B200KV_ERR_UNSUPPORTED, "batch * num_kv_heads * max_blocks_per_seq >= 2^31");
  B200KV_CHECK_ARG(std::isfinite(scale), "scale must be finite");
  if (batch == 0) return B200KV_OK;
  B200KV_CHECK_ARG(q && k_pool && v_pool && block_table && context_lens && out,
                   "null pointer argument");
  B200KV_CHECK_ARG(aligned16(q) && q_stride_b % 8 == 0 && q_stride_h % 8 == 0,
                   "q must be 16-byte aligned with strides that are multiples of 8 elements");
  const WorkspaceLayout wl = workspace_layout(batch, num_q_heads, num_kv_heads);
  if (!workspace || workspace_bytes < wl.total)
    return set_error(B200KV_ERR_WORKSPACE, "workspace of %lld bytes required (got %lld)",
                     (long long)wl.total, (long long)workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error(B200KV_ERR_WORKSPACE, "workspace must be 256-byte aligned");

  if (append) {
    B200KV_CHECK_ARG(k_new && v_new, "k_new / v_new must not be null");
    B200KV_CHECK_ARG((reinterpret_cast<uintptr_t>(k_new) & 15u) == 0 &&
                         (reinterpret_cast<uintptr_t>(v_new) & 15u) == 0 && new_sb % 8 == 0 &&
                         new_sh % 8 == 0,
                     "new K/V rows must be 16-byte aligned with strides that are multiples of 8");
    if (use_simt_kernel())
      return set_error(B200KV_ERR_UNSUPPORTED, "fused append needs the tensor-core kernel");
  }
  if (rope_freqs) {
    B200KV_CHECK_ARG(append, "the rotary embedding applies to the fused append only");
    B200KV_CHECK_ARG(rope_max_pos > 0, "rope_max_pos must be > 0");
    B200KV_CHECK_ARG((reinterpret_cast<uintptr_t>(rope_freqs) & 3u) == 0, "rope_freqs must be 4-byte aligned");
  }
  if (fp8) {
    B200KV_CHECK_ARG(k_scale && v_scale, "k_scale / v_scale must not be null");
    if (use_simt_kernel())
      return set_error(B200KV_ERR_UNSUPPORTED, "fp8 pages need the tensor-core kernel");
  }
  CUtensorMap km, vm;
  int st = make_page_pool_map(&km, k_pool, num_blocks, num_kv_heads, fp8 ? 1 : 2);
  if (st != B200KV_OK) return st;
  st = make_page_pool_map(&vm, v_pool, num_blocks, num_kv_heads, fp8 ? 1 : 2);
  if (st != B200KV_OK) return st;

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
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  a.counters = reinterpret_cast<int *>(ws + wl.counters_off);
  a.part_ml = reinterpret_cast<float2 *>(ws + wl.ml_off);
  a.part_o = reinterpret_cast<float *>(ws + wl.o_off);
  a.error_flag = error_flag;
  a.early = (flags & B200KV_DECODE_INPUTS_READY) != 0;
  if (append) {
    a.k_new = static_cast<const __half *>(k_new);
    a.v_new = static_cast<const __half *>(v_new);
    a.new_sb = new_sb;
    a.new_sh = new_sh;
    a.k_pool_w = static_cast<__half *>(const_cast<void *>(k_pool));
    a.v_pool_w = static_cast<__half *>(const_cast<void *>(v_pool));
  }
  if (rope_freqs) {
    a.rope_freqs = static_cast<const __half *>(rope_freqs);
    a.rope_max_pos = rope_max_pos;
  }
  if (fp8) {
    a.k_scale = static_cast<const __half *>(k_scale);
    a.v_scale = static_cast<const __half *>(v_scale);
    if (append) {
      a.k_pool8_w = static_cast<uint8_t *>(const_cast<void *>(k_pool));
      a.v_pool8_w = static_cast<uint8_t *>(const_cast<void *>(v_pool));
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (use_simt_kernel()) {
    // CUDA-core variant: num_splits is its target number of work items per CTA
    const int per_cta = num_splits > 0 ? static_cast<int>(num_splits < 64 ? num_splits : 64)
                                       : kDefaultItemsPerCta;
    return launch_decode_simt(static_cast<int>(group), km, vm, a, per_cta, s);
  }
  // tensor-core kernel: num_splits is the number of equal KV partitions (CTAs)
  return launch_decode_mma(static_cast<int>(group), km, vm, a, static_cast<int>(num_splits), s);
}

extern "C" int b200kv_decode_attention_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool, const void *v_pool,
    const int32_t *block_table, int64_t block_table_stride, const int32_t *context_lens, void *out,
    int64_t out_stride_b, int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq,
    float scale, int64_t num_splits, void *workspace, int64_t workspace_bytes,
    int32_t *error_flag, void *stream) {
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, nullptr, nullptr, 0, 0, false);
}

extern "C" int b200kv_decode_attention_ex_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool, const void *v_pool,
    const int32_t *block_table, int64_t block_table_stride, const int32_t *context_lens, void *out,
    int64_t out_stride_b, int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq,
    float scale, int64_t num_splits, void *workspace, int64_t workspace_bytes,
    int32_t *error_flag, uint32_t flags, void *stream) {
  if (flags & ~uint32_t(B200KV_DECODE_INPUTS_READY))
    return set_error(B200KV_ERR_INVALID_ARG, "unknown flags 0x%x", flags);
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, nullptr, nullptr, 0, 0, false, false,
                      nullptr, nullptr, nullptr, 0, flags);
}

extern "C" int b200kv_decode_attention_append_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new, const void *v_new,
    int64_t new_stride_b, int64_t new_stride_h, void *k_pool, void *v_pool,
    const int32_t *block_table, int64_t block_table_stride, const int32_t *context_lens, void *out,
    int64_t out_stride_b, int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq,
    float scale, int64_t num_splits, void *workspace, int64_t workspace_bytes,
    int32_t *error_flag, void *stream) {
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, k_new, v_new, new_stride_b,
                      new_stride_h, true);
}

extern "C" int b200kv_decode_attention_append_ex_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new, const void *v_new,
    int64_t new_stride_b, int64_t new_stride_h, void *k_pool, void *v_pool,
    const int32_t *block_table, int64_t block_table_stride, const int32_t *context_lens, void *out,
    int64_t out_stride_b, int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq,
    float scale, int64_t num_splits, void *workspace, int64_t workspace_bytes,
    int32_t *error_flag, uint32_t flags, void *stream) {
  if (flags & ~uint32_t(B200KV_DECODE_INPUTS_READY))
    return set_error(B200KV_ERR_INVALID_ARG, "unknown flags 0x%x", flags);
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, k_new, v_new, new_stride_b,
                      new_stride_h, true, false, nullptr, nullptr, nullptr, 0, flags);
}

extern "C" int b200kv_decode_attention_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool, const void *v_pool,
    const void *k_scale, const void *v_scale, const int32_t *block_table,
    int64_t block_table_stride, const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq, float scale,
    int64_t num_splits, void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    void *stream) {
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, nullptr, nullptr, 0, 0, false,
                      true, k_scale, v_scale);
}

extern "C" int b200kv_decode_attention_ex_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool, const void *v_pool,
    const void *k_scale, const void *v_scale, const int32_t *block_table,
    int64_t block_table_stride, const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq, float scale,
    int64_t num_splits, void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    uint32_t flags, void *stream) {
  if (flags & ~uint32_t(B200KV_DECODE_INPUTS_READY))
    return set_error(B200KV_ERR_INVALID_ARG, "unknown flags 0x%x", flags);
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, nullptr, nullptr, 0, 0, false,
                      true, k_scale, v_scale, nullptr, 0, flags);
}

extern "C" int b200kv_decode_attention_append_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new, const void *v_new,
    int64_t new_stride_b, int64_t new_stride_h, void *k_pool, void *v_pool, const void *k_scale,
    const void *v_scale, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b, int64_t out_stride_h,
    float *lse, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
    int64_t num_blocks, int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag, void *stream) {
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, k_new, v_new, new_stride_b,
                      new_stride_h, true, true, k_scale, v_scale);
}

extern "C" int b200kv_decode_attention_append_rope_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new, const void *v_new,
    int64_t new_stride_b, int64_t new_stride_h, void *k_pool, void *v_pool, const void *rope_freqs,
    int64_t rope_max_pos, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b, int64_t out_stride_h, float *lse,
    int64_t batch, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits, void *workspace,
    int64_t workspace_bytes, int32_t *error_flag, void *stream) {
  B200KV_CHECK_ARG(rope_freqs, "rope_freqs must not be null");
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, k_new, v_new, new_stride_b,
                      new_stride_h, true, false, nullptr, nullptr, rope_freqs, rope_max_pos);
}

extern "C" int b200kv_decode_attention_append_rope_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new, const void *v_new,
    int64_t new_stride_b, int64_t new_stride_h, void *k_pool, void *v_pool, const void *k_scale,
    const void *v_scale, const void *rope_freqs, int64_t rope_max_pos, const int32_t *block_table,
    int64_t block_table_stride, const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_dim, int64_t num_blocks, int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag, void *stream) {
  B200KV_CHECK_ARG(rope_freqs, "rope_freqs must not be null");
  return decode_entry(q, q_stride_b, q_stride_h, k_pool, v_pool, block_table, block_table_stride,
                      context_lens, out, out_stride_b, out_stride_h, lse, batch, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, max_blocks_per_seq, scale, num_splits,
                      workspace, workspace_bytes, error_flag, stream, k_new, v_new, new_stride_b,
                      new_stride_h, true, true, k_scale, v_scale, rope_freqs, rope_max_pos);
}
