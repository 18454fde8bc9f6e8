/*
 * b200kv.h -- C ABI of the B200 paged-KV decode library (libb200kv.so).
 *
 * The library implements one hot path of torch-spyre for NVIDIA B200 (sm_100a):
 * single-token decode attention over a paged fp16 KV cache that is tiled in
 * 64-element "sticks", plus the on-device KV append and relayout that feed it.
 *
 * Conventions (every entry point):
 *   - plain C types only; device buffers are raw device pointers, sizes are
 *     int64_t, the CUDA stream is passed as an opaque `void *` (a cudaStream_t,
 *     NULL = legacy default stream);
 *   - return an int status (enum b200kv_status); 0 means success.  A non-zero
 *     status leaves a message that b200kv_last_error() returns (thread-local);
 *   - argument validation happens on the host before any launch; nothing is
 *     allocated and the stream is never synchronised by a compute entry point;
 *   - device-side index errors (a block id or slot outside the pool) never
 *     fault: the access is skipped (TMA out-of-bounds fill, or an explicit
 *     bounds test) and, when `error_flag` is non-NULL, a bit is OR-ed into that
 *     device int32 (B200KV_DEVERR_*).  The caller reads it when it chooses.
 *
 * KV pool layout ("paged stick layout").  One page holds P = 64 consecutive
 * tokens of one KV head.  Inside a page the head dimension D (= 64 * S) is split
 * into S sticks of 64 fp16 (128 bytes); the page is the reference's default
 * stick tiling of a [64, D] fp16 tile: device_size [S, 64, 64], stride_map
 * [64, D, 1] (torch_spyre/csrc/spyre_tensor_impl.cpp:46-175).  The pool is
 *     k_pool, v_pool : fp16 [num_blocks, num_kv_heads, S, 64, 64]
 * so token t of sequence b, element d of head h lives at element offset
 *     ((blk * Hkv + h) * S + d / 64) * 4096 + (t % 64) * 64 + d % 64,
 *     blk = block_table[b * block_table_stride + t / 64].
 * A slot is blk * 64 + (t % 64) (the kv_append addressing).
 */
#ifndef B200KV_H_
#define B200KV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define B200KV_API __attribute__((visibility("default")))
#else
#define B200KV_API
#endif

#define B200KV_PAGE_TOKENS 64
#define B200KV_STICK_ELEMS 64

enum b200kv_status {
  B200KV_OK = 0,
  B200KV_ERR_INVALID_ARG = 1,   /* null pointer, bad size, bad stride        */
  B200KV_ERR_UNSUPPORTED = 2,   /* legal but not implemented (e.g. D != 128) */
  B200KV_ERR_WORKSPACE = 3,     /* workspace missing or too small            */
  B200KV_ERR_CUDA = 4,          /* a CUDA runtime / driver call failed       */
};

/* Bits OR-ed into the optional device-side error flag. */
#define B200KV_DEVERR_BAD_BLOCK 0x1 /* block id outside [0, num_blocks)       */
#define B200KV_DEVERR_BAD_SLOT 0x2  /* slot outside [0, num_blocks * 64)      */
#define B200KV_DEVERR_BAD_LEN 0x4   /* context_len < 0 or > capacity of table */
#define B200KV_DEVERR_TIMEOUT 0x8   /* a bounded wait on a page transfer expired */

/* Library version: major * 10000 + minor * 100 + patch. */
B200KV_API int b200kv_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated to
 * len) into buf.  Returns the full message length.  Replaces the reference's
 * TORCH_CHECK / RuntimeError reporting (torch_spyre/csrc/spyre_mem.cpp:266-293). */
B200KV_API int b200kv_last_error(char *buf, size_t len);

/* ------------------------------------------------------------------------ *
 * Stick layout algebra (host only, no GPU needed).
 * Restates SpyreTensorLayout::init (torch_spyre/csrc/spyre_tensor_impl.cpp:
 * 126-175; tiling rule get_generic_stick_layout 46-82, stride map 104-124).
 *   host_size[rank], host_stride[rank] (NULL = contiguous),
 *   dim_order[order_len] (NULL = identity; order_len == rank, or rank + 1 with
 *   a trailing -1 for the sparse layout), elem_bytes (2 for fp16, 4 for fp32).
 * Writes device_rank (= rank + 1, or 2 for a scalar) entries into
 * device_size / stride_map (capacity `cap`) and returns device_rank through
 * *out_rank.
 * ------------------------------------------------------------------------ */
B200KV_API int b200kv_stick_layout(const int64_t *host_size, const int64_t *host_stride,
                        int32_t rank, const int32_t *dim_order,
                        int32_t order_len, int32_t elem_bytes,
                        int64_t *device_size, int64_t *stride_map, int32_t cap,
                        int32_t *out_rank);

/* General stick relayout between a strided tensor in host dim order and a
 * device buffer laid out by (device_size, stride_map) -- the device-side form
 * of the reference's `x.to(device_layout=stl)` / `.cpu()` copies, whose
 * element map its DMA descriptors encode (generate_dci /
 * get_device_stride_infos, torch_spyre/csrc/spyre_mem.cpp:176-440; dim
 * matching get_dim_map 60-96; pinned by tests/tensor/test_tensor_layout.py:
 * 152-280).  Both buffers are device memory.
 *   direction 0: src = host-order tensor (sizes host_size, element strides
 *                host_stride), dst = device buffer of prod(device_size)
 *                elements; stick padding is written as zero.
 *   direction 1: src = device buffer, dst = host-order tensor; only elements
 *                inside the host tensor are written.
 * elem_bytes 1, 2 or 4; ranks <= 8.  A stride_map entry that is not a
 * multiple of the host stride it matches (a folded layout) is
 * B200KV_ERR_UNSUPPORTED. */
B200KV_API int b200kv_stick_relayout(const void *src, void *dst, int32_t elem_bytes,
                                     int32_t host_rank, const int64_t *host_size,
                                     const int64_t *host_stride, int32_t device_rank,
                                     const int64_t *device_size, const int64_t *stride_map,
                                     int32_t direction, void *stream);

/* Bytes a layout occupies on the device: 128 B per stick times the product of
 * the non-stick device dims (spyre_tensor_impl.cpp:287-293). */
/* Restickify: moves a tensor that lives in device layout (src_device_size,
 * src_stride_map) into device layout (dst_device_size, dst_stride_map) of the
 * same host tensor (host_size, contiguous strides), on the device in one
 * pass; destination padding is zero.  Replaces spyre::restickify
 * (torch_spyre/_inductor/customops.py:338-342), whose target layouts come
 * from restickify_device_size / restickify_stride_map
 * (torch_spyre/_inductor/pass_utils.py:749-781).  Bit-exact. */
B200KV_API int b200kv_stick_restickify(const void *src, void *dst, int32_t elem_bytes,
                                       int32_t host_rank, const int64_t *host_size,
                                       int32_t src_rank, const int64_t *src_device_size,
                                       const int64_t *src_stride_map, int32_t dst_rank,
                                       const int64_t *dst_device_size,
                                       const int64_t *dst_stride_map, void *stream);

B200KV_API int64_t b200kv_device_size_in_bytes(const int64_t *device_size,
                                    int32_t device_rank);

/* ------------------------------------------------------------------------ *
 * Decode attention.
 * Replaces the decode case of aten::_scaled_dot_product_fused_attention_
 * overrideable as decomposed by spyre__sdpa_overrideable
 * (torch_spyre/_inductor/decompositions.py:523-611; backend selection
 * torch_spyre/csrc/attn_utils.cpp:22-37): out = softmax(q k^T * scale) v with
 * GQA head mapping kv_head = q_head / (Hq / Hkv) (decompositions.py:560-563),
 * over a paged KV cache instead of dense k/v.
 * ------------------------------------------------------------------------ */

/* Workspace bytes the decode call needs (split-KV partials, per-sequence split
 * metadata, self-resetting completion counters).  The workspace must be zeroed
 * once before its first use; every successful call leaves it re-usable (the
 * counters return to zero).  Calls that share a workspace must be ordered on
 * one stream. */
B200KV_API int64_t b200kv_decode_workspace_bytes(int64_t batch, int64_t num_q_heads,
                                      int64_t num_kv_heads, int64_t head_dim);

/* Same as b200kv_decode_workspace_bytes (the name of the build contract). */
B200KV_API int64_t b200kv_query_workspace_bytes(int64_t batch, int64_t num_q_heads,
                                                int64_t num_kv_heads, int64_t head_dim);

/* Merge of attention outputs over disjoint KV sets through their
 * log-sum-exps (the split-KV combine, exposed): part_o [num_parts][rows]
 * [head_dim] (fp16 when part_elem_bytes is 2, fp32 when 4), part_lse fp32
 * [num_parts][rows] (natural log, -inf for an empty part) ->
 * out fp16 [rows][head_dim] = sum_i exp(lse_i - m) o_i / sum_i exp(lse_i - m)
 * and, when lse_out is not NULL, lse_out fp32 [rows] = m + log(sum_i ...).
 * Rows whose parts are all empty give zeros and -inf.  Replaces nothing in
 * the reference (it has no split KV); it lets a caller decode a shared
 * prefix and per-sequence pages separately and merge the results. */
B200KV_API int b200kv_lse_combine_f32(const void *part_o, int32_t part_elem_bytes,
                                      const float *part_lse, int64_t num_parts, int64_t rows,
                                      int64_t head_dim, void *out, float *lse_out,
                                      void *stream);

/*
 * q            fp16, element (b, h, d) at q[b * q_stride_b + h * q_stride_h + d]
 * k_pool/v_pool fp16 [num_blocks, num_kv_heads, D/64, 64, 64] (16-byte aligned)
 * block_table  int32 [batch, *] row stride block_table_stride (elements)
 * context_lens int32 [batch], each in [0, max_blocks_per_seq * 64]
 * out          fp16, element (b, h, d) at out[b * out_stride_b + h * out_stride_h + d]
 * lse          optional fp32 [batch, num_q_heads] (natural-log logsumexp of the
 *              scaled scores; -inf for an empty context), may be NULL
 * scale        softmax scale (the reference default is 1/sqrt(D))
 * num_splits   0 = automatic: one partition (CTA) per SM; n > 0 = n partitions
 *              (n <= 1024).  The KV pages of the whole batch are cut into equal
 *              contiguous shares, one per partition; a sequence-head cut by a
 *              share boundary is a split whose partials are merged with a
 *              log-sum-exp combine.
 * workspace    device buffer of at least b200kv_decode_workspace_bytes()
 * error_flag   optional device int32 (B200KV_DEVERR_* bits are OR-ed in)
 * Supported: head_dim 128, Hq % Hkv == 0, Hq / Hkv in {1, 2, 4, 8}, batch <= 1024,
 * batch * Hkv <= 131072.
 * An empty context (len 0) yields a zero output row, matching torch CPU SDPA.
 */
B200KV_API int b200kv_decode_attention_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool,
    const void *v_pool, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    void *stream);

/* Decode attention fused with the KV append of the token being decoded (one
 * launch instead of an append kernel followed by decode).  Each sequence's
 * context length includes the new token, at position context_lens[b] - 1;
 * its K/V rows k_new/v_new[b * new_stride_b + h * new_stride_h + d] are written
 * into that position of the pools (page block_table[b][(len - 1) / 64]) and
 * used for the attention of this step.  Replaces the reference's two-step HF
 * path: cache.index_copy_ (torch_spyre/ops/fallbacks.py:256; test pattern
 * tests/inductor/test_inductor_ops.py:5715-5740) followed by SDPA
 * (torch_spyre/_inductor/decompositions.py:523-611).  Other arguments as in
 * b200kv_decode_attention_f16; the pools are written.  A block id out of range
 * skips the write (B200KV_DEVERR_BAD_BLOCK). */
B200KV_API int b200kv_decode_attention_append_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new,
    const void *v_new, int64_t new_stride_b, int64_t new_stride_h, void *k_pool,
    void *v_pool, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    void *stream);

/* Decode attention with options: the arguments of b200kv_decode_attention_f16
 * plus `flags`, the same computation and result.
 *   B200KV_DECODE_INPUTS_READY  the pools, block table and context lengths were
 *     written before the preceding kernel on `stream` began (q may still be
 *     written by it).  The decode kernel is launched as a programmatic
 *     dependent of that kernel; with this flag each CTA plans its work and
 *     starts loading its first pages while the preceding kernel finishes, and
 *     only q, the scales, the workspace and the outputs wait for it.  Without
 *     the flag (or under the CUDA-core kernel) everything waits.  Mind that
 *     the fused append of this library writes pool rows: a decode of the same
 *     pools right after it must not pass this flag.
 * Same reference interface as b200kv_decode_attention_f16
 * (decompositions.py:523-611); the flag has no reference counterpart (the
 * reference has no programmatic dependent launch). */
#define B200KV_DECODE_INPUTS_READY 1u
B200KV_API int b200kv_decode_attention_ex_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool,
    const void *v_pool, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    uint32_t flags, void *stream);

/* Fused append + decode with options: the arguments of
 * b200kv_decode_attention_append_f16 plus `flags`.  With
 * B200KV_DECODE_INPUTS_READY the caller vouches that the pools (other than the
 * rows this call appends), block table and context lengths were written before
 * the preceding kernel on `stream` began; q and the new K/V rows may be written
 * by it.  The kernel then plans and loads its first pages while that kernel
 * finishes; the new rows, q and every write wait for it.  Same reference
 * interface as b200kv_decode_attention_append_f16. */
B200KV_API int b200kv_decode_attention_append_ex_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new,
    const void *v_new, int64_t new_stride_b, int64_t new_stride_h, void *k_pool,
    void *v_pool, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    uint32_t flags, void *stream);

/* Decode attention that allocates nothing.  No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc or any allocator when they
 * launch decode (an engine replaying pre-planned memory, a plugin host that
 * only hands over the tensors it owns), so they cannot provide the workspace
 * of b200kv_decode_attention_f16.  Same arguments minus num_splits and the
 * workspace; the caller still passes every input and output.  The split-KV
 * partials go to a 16 MiB scratch array the library keeps on each device that
 * loads it (until process exit).  Limit, else B200KV_ERR_UNSUPPORTED before any
 * launch: pairs = batch * num_kv_heads <= 16384 and
 * 64 KiB + (pairs + SMs) * G * 520 B <= 16 MiB (G = num_q_heads / num_kv_heads,
 * 148 SMs on B200): about 15900 pairs at G = 2, 7880 at G = 4, 3860 at G = 8.
 * The first call on a device looks up the scratch address, so make it before
 * any stream capture (a failed lookup is retried by the next call).  Calls
 * share the scratch: calls that overlap on the GPU race. */
B200KV_API int b200kv_decode_attention_f16_noalloc(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool,
    const void *v_pool, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int32_t *error_flag, void *stream);

/* ------------------------------------------------------------------------ *
 * KV append: write one new token row per entry of slot_mapping into the pools.
 * Replaces the KV-cache write paths of the reference: spyre::overwrite
 * (torch_spyre/_inductor/customops.py:262-308) and the aten.index_copy.out
 * CPU fallback used by HF caches (torch_spyre/ops/fallbacks.py:237-259).
 *   k_new/v_new fp16, row n head h at k_new[n * new_stride_n + h * new_stride_h]
 *               (head_dim contiguous, 16-byte aligned rows)
 *   slot_mapping int64 [num_tokens]; slot = block * 64 + offset; a negative
 *               slot means "padding token, skip"; slot >= num_blocks * 64 sets
 *               B200KV_DEVERR_BAD_SLOT and is skipped.
 * Bit-exact copy.  Duplicate slots in one call: last writer is unspecified.
 * ------------------------------------------------------------------------ */
B200KV_API int b200kv_kv_append_f16(const void *k_new, const void *v_new,
                         int64_t new_stride_n, int64_t new_stride_h,
                         void *k_pool, void *v_pool,
                         const int64_t *slot_mapping, int64_t num_tokens,
                         int64_t num_kv_heads, int64_t head_dim,
                         int64_t num_blocks, int32_t *error_flag, void *stream);

/* ------------------------------------------------------------------------ *
 * Bulk relayout between a row-major cache [num_tokens, Hkv, D] fp16 and the
 * paged stick layout.  Token t goes to page block_ids[t / 64], slot t % 64.
 * Replaces the host<->device stick relayout the reference does in its DMA
 * descriptors (generate_dci / get_device_stride_infos,
 * torch_spyre/csrc/spyre_mem.cpp:176-440) with an HBM->HBM kernel.
 *   direction 0: rows -> pages (pool slots past num_tokens are untouched)
 *   direction 1: pages -> rows
 * block_ids int32 [ceil(num_tokens / 64)]; an id outside [0, num_blocks) sets
 * B200KV_DEVERR_BAD_BLOCK and that page is skipped.  Bit-exact.
 * ------------------------------------------------------------------------ */
B200KV_API int b200kv_relayout_f16(void *rows, void *pool, const int32_t *block_ids,
                        int64_t num_tokens, int64_t num_kv_heads,
                        int64_t head_dim, int64_t num_blocks, int32_t direction,
                        int32_t *error_flag, void *stream);

/* ------------------------------------------------------------------------ *
 * FP8 (e4m3) KV pages.
 *
 * An fp8 pool uses the reference's stick tiling for 1-byte elements: a stick
 * is 128 elements (128 bytes), so a page of 64 tokens x D holds D/128 sticks:
 *     k_pool, v_pool : e4m3 [num_blocks, num_kv_heads, D/128, 64, 128]
 * (device_size [D/128, 64, 128], stride_map [128, D, 1];
 * torch_spyre/csrc/spyre_tensor_impl.cpp:46-175).  Element (t, d) of page
 * (blk, h) is at byte ((blk * Hkv + h) * D/128 + d / 128) * 8192 +
 * (t % 64) * 128 + d % 128.  Each pool carries one fp16 scale (a device
 * scalar): the stored value q stands for fp16(q) * scale, the reference's
 * dequantize_fp8_with_scale (torch_spyre/_inductor/customops.py:624-653,
 * decompositions.py:846-858); values are written with its
 * quantize_fp8_with_scale (customops.py:587-621, decompositions.py:897-904):
 *     q = e4m3_rne(clamp(fp16(x * fp16(1 / scale)), -448, 448)).
 * ------------------------------------------------------------------------ */

/* Quantize fp16 x [rows, cols] (contiguous) to e4m3 out [rows, cols] with the
 * fp16 scale of row r at scale[r * scale_stride] (scale_stride 0: one scale
 * for the whole tensor).  Replaces spyre::quantize_fp8_with_scale.  Bit-exact
 * with the reference's CPU decomposition. */
B200KV_API int b200kv_quantize_fp8_f16(const void *x, void *out, int64_t rows,
                                       int64_t cols, const void *scale,
                                       int64_t scale_stride, void *stream);

/* Dequantize e4m3 x [rows, cols] to fp16 out: fp16(x) * scale[r * scale_stride].
 * Replaces spyre::dequantize_fp8_with_scale.  Bit-exact. */
B200KV_API int b200kv_dequantize_fp8_f16(const void *x, void *out, int64_t rows,
                                         int64_t cols, const void *scale,
                                         int64_t scale_stride, void *stream);

/* KV append into fp8 pools: as b200kv_kv_append_f16, with each fp16 row
 * quantized with the pool's scale (k_scale / v_scale: device fp16 scalars). */
B200KV_API int b200kv_kv_append_fp8(const void *k_new, const void *v_new,
                                    int64_t new_stride_n, int64_t new_stride_h,
                                    void *k_pool, void *v_pool,
                                    const void *k_scale, const void *v_scale,
                                    const int64_t *slot_mapping, int64_t num_tokens,
                                    int64_t num_kv_heads, int64_t head_dim,
                                    int64_t num_blocks, int32_t *error_flag,
                                    void *stream);

/* Decode attention over fp8 pools: as b200kv_decode_attention_f16 with
 * K = fp16(k_pool) * k_scale and V = fp16(v_pool) * v_scale (device fp16
 * scalars).  q, out, lse and the workspace are as in the fp16 call.  The
 * scales are applied in fp32 (to the scores and to the output) instead of
 * rounding each dequantized element to fp16. */
B200KV_API int b200kv_decode_attention_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool,
    const void *v_pool, const void *k_scale, const void *v_scale,
    const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    void *stream);

/* b200kv_decode_attention_fp8 with launch flags (the same interface as
 * above; flags as b200kv_decode_attention_ex_f16): B200KV_DECODE_INPUTS_READY
 * lets the kernel plan and start its page loads before the preceding kernel
 * on the stream finishes; the pools, block table and context lengths must
 * then have been written before that kernel began (q and the scales may be
 * written by it).  Same result either way. */
B200KV_API int b200kv_decode_attention_ex_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_pool,
    const void *v_pool, const void *k_scale, const void *v_scale,
    const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    uint32_t flags, void *stream);

/* Fused append + decode over fp8 pools: as
 * b200kv_decode_attention_append_f16, the new fp16 rows quantized into the
 * pools (as b200kv_kv_append_fp8) and used, quantized, for this step. */
B200KV_API int b200kv_decode_attention_append_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new,
    const void *v_new, int64_t new_stride_b, int64_t new_stride_h, void *k_pool,
    void *v_pool, const void *k_scale, const void *v_scale,
    const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    void *stream);

/* ------------------------------------------------------------------------ *
 * Rotary position embedding (RoPE) with the reference's formulation (the
 * rope dataflow of tests/inductor/test_inductor_ops.py:5447-5456): a head row
 * x of D elements is two halves x_0 = x[0 : D/2], x_1 = x[D/2 : D] and
 *     out[i * D/2 + j] = sum_k freqs[pos][i][k][j] * x_k[j]    (i, k in {0, 1})
 * with freqs fp16 [max_pos][2][2][D/2] (a 2x2 matrix per position and
 * frequency); each product is rounded to fp16, the two products are summed
 * in fp32 and the sum is rounded to fp16 (bit-exact with the reference's CPU
 * path).  A position outside [0, max_pos) is clamped and sets
 * B200KV_DEVERR_BAD_LEN.
 * ------------------------------------------------------------------------ */

/* Rotates rows x[t * x_stride_t + h * x_stride_h + d] (fp16, t < num_tokens,
 * h < num_heads, d < head_dim) at positions[t] (int32) into out (may equal x).
 * head_dim a multiple of 4; x, out and freqs 4-byte aligned, even strides. */
B200KV_API int b200kv_rope_f16(const void *x, int64_t x_stride_t, int64_t x_stride_h,
                               void *out, int64_t out_stride_t, int64_t out_stride_h,
                               const void *freqs, int64_t max_pos,
                               const int32_t *positions, int64_t num_tokens,
                               int64_t num_heads, int64_t head_dim,
                               int32_t *error_flag, void *stream);

/* Fused append + decode with RoPE: as b200kv_decode_attention_append_f16 /
 * _fp8, with q and the new K row rotated at position context_lens[b] - 1
 * (rope_freqs fp16 [rope_max_pos][2][2][64]) before the K row is written and
 * attention is computed.  Equals b200kv_rope_f16 on q and k_new followed by
 * the plain fused call. */
B200KV_API int b200kv_decode_attention_append_rope_f16(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new,
    const void *v_new, int64_t new_stride_b, int64_t new_stride_h, void *k_pool,
    void *v_pool, const void *rope_freqs, int64_t rope_max_pos,
    const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    void *stream);
B200KV_API int b200kv_decode_attention_append_rope_fp8(
    const void *q, int64_t q_stride_b, int64_t q_stride_h, const void *k_new,
    const void *v_new, int64_t new_stride_b, int64_t new_stride_h, void *k_pool,
    void *v_pool, const void *k_scale, const void *v_scale, const void *rope_freqs,
    int64_t rope_max_pos, const int32_t *block_table, int64_t block_table_stride,
    const int32_t *context_lens, void *out, int64_t out_stride_b,
    int64_t out_stride_h, float *lse, int64_t batch, int64_t num_q_heads,
    int64_t num_kv_heads, int64_t head_dim, int64_t num_blocks,
    int64_t max_blocks_per_seq, float scale, int64_t num_splits,
    void *workspace, int64_t workspace_bytes, int32_t *error_flag,
    void *stream);

/* ------------------------------------------------------------------------ *
 * Tensor-parallel all-reduce over peer memory.
 *
 * Replaces the o_proj all-reduce of the head-sharded decode step: the
 * reference's TP collective is a SUM all-reduce of one tensor
 * (SpyreCCLBackend::allreduce, torch_spyre/csrc/distributed/
 * spyre_ccl.cpp:470-494).  Each rank (one process per GPU) allocates a peer
 * buffer, exports it with b200kv_ipc_get_handle, exchanges the handle bytes
 * with the other ranks by any host channel, maps theirs with
 * b200kv_ipc_open_handle, and passes the table of all ranks' buffers (own
 * included, in rank order) to b200kv_peer_allreduce_f16.  The tensor is the
 * first num_elems fp16 of the rank's buffer (its "data" region, at offset
 * 0): the rank's partial on entry, the elementwise sum over ranks on exit
 * (fp32 accumulation in rank order, rounded to fp16 once; bit-identical on
 * every rank).  Data moves with peer stores over NVLink; no multicast.
 * Every rank must make the same calls (same num_elems, capacity and ctas) in
 * the same order, like a collective; a call waits for its peers at most 2 s
 * (then B200KV_DEVERR_TIMEOUT is OR-ed into error_flag and the result is
 * undefined).  Calls replay correctly from CUDA graphs.
 * ------------------------------------------------------------------------ */

/* Bytes of one peer buffer for tensors of up to capacity_elems fp16 over
 * world ranks (-1 on bad arguments). */
B200KV_API int64_t b200kv_peer_buffer_bytes(int64_t capacity_elems, int32_t world);

/* Allocates (cudaMalloc) and zeroes a peer buffer on the current device. */
B200KV_API int b200kv_peer_alloc(int64_t capacity_elems, int32_t world, void **buffer_out);
B200KV_API int b200kv_peer_free(void *buffer);

/* CUDA IPC handle of a buffer (b200kv_ipc_handle_bytes() bytes) and the
 * mapping of a peer's buffer into this process. */
B200KV_API int32_t b200kv_ipc_handle_bytes(void);
B200KV_API int b200kv_ipc_get_handle(void *buffer, void *handle_out);
B200KV_API int b200kv_ipc_open_handle(const void *handle, void **buffer_out);
B200KV_API int b200kv_ipc_close_handle(void *buffer);

/* In-place SUM all-reduce of the first num_elems fp16 of every rank's buffer.
 * peer_buffers: host array of world device pointers (rank order).
 * num_elems and capacity_elems: multiples of 8 * world; ctas: CTAs per rank
 * (0 = 128, at most 128). */
B200KV_API int b200kv_peer_allreduce_f16(void *const *peer_buffers, int32_t rank,
                                         int32_t world, int64_t num_elems,
                                         int64_t capacity_elems, int32_t ctas,
                                         int32_t *error_flag, void *stream);

/* ------------------------------------------------------------------------ *
 * Tensor-parallel all-reduce through NVLink SHARP (multimem).
 *
 * The same collective as b200kv_peer_allreduce_f16 -- the reference's TP
 * SUM all-reduce of one tensor (SpyreCCLBackend::allreduce,
 * torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494) -- with the adds done
 * inside the NVSwitch: every element is reduced once by its owning rank
 * (multimem.ld_reduce, fp32 accumulation, rounded once to fp16) and the sum
 * is multicast to every rank (multimem.st), so all ranks end with the same
 * bits.  The caller allocates, on every rank, the data buffer of num_elems
 * fp16 at the same offset of memory bound to one NVLink multicast object
 * (e.g. PyTorch symmetric memory) and passes its multicast address, plus a
 * separate zero-initialised signal area of b200kv_nvls_signal_bytes() per
 * rank, mapped into every rank (table of all ranks' areas, own included, in
 * rank order, 256-byte aligned).  num_elems must be a multiple of 8 * world;
 * ctas in [0, 256] (0 = 32).  The data buffer holds the partial on entry and
 * the sum on exit.  Every rank must make the same calls in the same order;
 * waits are bounded (2 s, then B200KV_DEVERR_TIMEOUT in error_flag and the
 * output is undefined).  Calls replay correctly from CUDA graphs.
 * ------------------------------------------------------------------------ */
B200KV_API int64_t b200kv_nvls_signal_bytes(void);
B200KV_API int b200kv_nvls_allreduce_f16(void *multicast_data, void *const *signal_areas,
                                         int32_t rank, int32_t world, int64_t num_elems,
                                         int32_t ctas, int32_t *error_flag, void *stream);

/* The same collective in its low-latency form (same reference interface as
 * above): two-shot with the arrival marker in the data -- no flag exchange,
 * no fence, no in-switch reduction.  Each rank writes slice j of its partial
 * into rank j's reduce-scatter region (peer stores); the owner polls its
 * region until every element has arrived, sums the ranks' values in rank
 * order in fp32, rounds once to fp16 and multicasts the sum (multimem.st)
 * into every rank's all-gather region, which every rank polls and copies
 * into its data.  Sums are the fp32 rank-order sums rounded once, the same
 * bits on every rank; NaN sums come out as the canonical NaN 0x7E00.
 * Memory, allocated by the caller on every rank in memory bound to one NVLink
 * multicast object: the data (num_elems fp16), a reduce-scatter and an
 * all-gather region of 2 * region_elems fp16 each (region_elems >=
 * num_elems, a multiple of 8), both filled with 0xFF bytes before the first
 * call on any rank, and a zero-initialised signal area of
 * b200kv_nvls_signal_bytes().  Arguments: this rank's data, the table of all
 * ranks' reduce-scatter regions mapped here (rank order), this rank's
 * all-gather region and the multicast address of the all-gather regions,
 * region_elems, this rank's signal area.  ctas in [0, 256] (0 = 32).  Waits
 * are bounded (2 s, then B200KV_DEVERR_TIMEOUT); after a timeout the regions
 * may hold stale values: refill them before the next call. */
B200KV_API int b200kv_nvls_allreduce_ll_f16(void *data, void *const *rs_regions, void *ag_region,
                                            void *ag_multicast, int64_t region_elems, void *signal_area,
                                            int32_t rank, int32_t world, int64_t num_elems, int32_t ctas,
                                            int32_t *error_flag, void *stream);

/* Fused o_proj GEMM + SUM all-reduce of the tensor-parallel step, one kernel
 * per rank: out[b, n] = sum over ranks of sum_k attn[b, k] * w[n, k]
 * (attn fp16 [batch, k] row stride attn_stride_b; w fp16 [hidden, k] row
 * stride w_stride_n, the rank's input columns of W_o; out fp16 [batch, hidden]
 * row stride out_stride_b), with the peer buffers of b200kv_peer_alloc
 * (capacity >= 128 * hidden).  Each rank's partial is rounded to fp16, the
 * partials are summed in fp32 in rank order and rounded once, as
 * b200kv_peer_allreduce_f16 does.  The GEMM runs on the tensor cores
 * (tcgen05, fp32 accumulate); each 128 x 64 output tile is exchanged as soon
 * as it is computed.  batch <= 128, k a multiple of 64, hidden a multiple of
 * 64 * world and at most 64 * (SM count).  Replaces the o_proj + allreduce
 * pair of the reference's TP step (SpyreCCLBackend::allreduce,
 * torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494).  Shares the peer
 * buffers' epoch with b200kv_peer_allreduce_f16 (calls of both kinds may
 * interleave, in the same order on every rank). */
B200KV_API int b200kv_oproj_allreduce_f16(const void *attn, int64_t attn_stride_b, const void *w,
                                          int64_t w_stride_n, void *out, int64_t out_stride_b,
                                          int64_t batch, int64_t hidden, int64_t k,
                                          void *const *peer_buffers, int32_t rank, int32_t world,
                                          int64_t capacity_elems, int32_t *error_flag,
                                          void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B200KV_H_ */
