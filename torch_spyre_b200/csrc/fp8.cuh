// FP8 (e4m3) conversions with the reference's quantize / dequantize semantics
// (spyre::quantize_fp8_with_scale / dequantize_fp8_with_scale, decomposed in
// torch_spyre/_inductor/decompositions.py:846-858 and 897-904):
//   quantize    q = e4m3(clamp(fp16(x * fp16(1 / scale)), -448, 448))
//   dequantize  y = fp16(fp16(q) * scale)
// with fp16 arithmetic rounded to nearest even at every step and the e4m3
// conversion rounded to nearest even, as the reference's CPU path computes.
// The hardware conversions (cvt ... e4m3x2) are reached through cuda_fp8.h.
#pragma once

#include <cuda_fp8.h>

#include "common.cuh"

namespace b200kv {

constexpr float kFp8E4M3Max = 448.f;  // FP8_E4M3_MAX, torch_spyre/_inductor/constants.py:90

// fp16 reciprocal of an fp16 scale, as torch.reciprocal computes it on a Half
// tensor: fp32 division, rounded to fp16.
__device__ __forceinline__ __half2 fp8_inv_scale2(__half scale) {
  return __half2half2(__float2half_rn(1.0f / __half2float(scale)));
}

// Two fp16 (packed in x, element 0 in the low half) -> two e4m3 (element 0 in
// the low byte).  NaN propagates through the clamp as in torch.clamp.
__device__ __forceinline__ uint32_t quantize2_e4m3(uint32_t x, __half2 inv2) {
  __half2 h = __halves2half2(__ushort_as_half(static_cast<unsigned short>(x & 0xffffu)),
                             __ushort_as_half(static_cast<unsigned short>(x >> 16)));
  h = __hmul2(h, inv2);
  h = __hmin2_nan(__hmax2_nan(h, __float2half2_rn(-kFp8E4M3Max)), __float2half2_rn(kFp8E4M3Max));
  const __half2_raw r = h;
  return __nv_cvt_halfraw2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3);
}

// Eight fp16 (one 16-byte vector) -> eight e4m3 (one 8-byte vector).
__device__ __forceinline__ uint2 quantize8_e4m3(uint4 v, __half2 inv2) {
  return make_uint2(quantize2_e4m3(v.x, inv2) | (quantize2_e4m3(v.y, inv2) << 16),
                    quantize2_e4m3(v.z, inv2) | (quantize2_e4m3(v.w, inv2) << 16));
}

// Two e4m3 (byte 0 in the low 8 bits of x) -> fp16x2 bits (element 0 in the
// low half), by the hardware conversion.  Exact: every e4m3 value is an fp16
// value.
__device__ __forceinline__ uint32_t e4m3x2_to_half2(uint32_t x) {
  uint32_t r;
  const unsigned short pair = static_cast<unsigned short>(x & 0xffffu);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(pair));
  return r;
}

// Four e4m3 (bytes 0..3 of x) -> fp16x2 of bytes 0, 1 (lo) and 2, 3 (hi), by
// two hardware conversions on the halves of x.
__device__ __forceinline__ void e4m3x4_to_half2x2(uint32_t x, uint32_t &lo, uint32_t &hi) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(x));
}

// fp16x2 bits times an fp16x2 scale, as bits.
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t x, __half2 s) {
  const __half2 h = __hmul2(__halves2half2(__ushort_as_half(static_cast<unsigned short>(x & 0xffffu)),
                                           __ushort_as_half(static_cast<unsigned short>(x >> 16))),
                            s);
  return static_cast<uint32_t>(__half_as_ushort(__low2half(h))) |
         (static_cast<uint32_t>(__half_as_ushort(__high2half(h))) << 16);
}

// Eight e4m3 -> eight fp16 times an fp16 scale.
__device__ __forceinline__ uint4 dequantize8_e4m3(uint2 v, __half2 scale2) {
  return make_uint4(hmul2_bits(e4m3x2_to_half2(v.x), scale2), hmul2_bits(e4m3x2_to_half2(v.x >> 16), scale2),
                    hmul2_bits(e4m3x2_to_half2(v.y), scale2), hmul2_bits(e4m3x2_to_half2(v.y >> 16), scale2));
}

}  // namespace b200kv
