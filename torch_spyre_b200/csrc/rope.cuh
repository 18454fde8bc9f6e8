// Rotary position embedding with the reference's formulation (the rope
// dataflow of tests/inductor/test_inductor_ops.py:5447-5456, FMS style): a
// head row x of D elements is two halves x0 = x[0 : D/2], x1 = x[D/2 : D];
// freqs[pos] is [2][2][D/2] (a 2x2 matrix per frequency j) and
//     out[i * D/2 + j] = sum_k freqs[pos][i][k][j] * x_k[j]      (i, k in {0, 1})
// computed as the reference's CPU path does it: each product rounded to fp16,
// the two products summed in fp32 from a +0 accumulator, the sum rounded to
// fp16.
#pragma once

#include "common.cuh"

namespace b200kv {

// Two adjacent elements (e, e + 1 < D/2) of both halves: x0/x1 are the fp16x2
// pairs of the first / second half, f points at freqs[pos] ([2][2][D/2]).
// Returns the rotated pairs in x0 / x1.
__device__ __forceinline__ void rope_pair(const __half *__restrict__ f, int half_d, int e, uint32_t &x0,
                                          uint32_t &x1) {
  const __half2 a = __halves2half2(__ushort_as_half(static_cast<unsigned short>(x0 & 0xffffu)),
                                   __ushort_as_half(static_cast<unsigned short>(x0 >> 16)));
  const __half2 b = __halves2half2(__ushort_as_half(static_cast<unsigned short>(x1 & 0xffffu)),
                                   __ushort_as_half(static_cast<unsigned short>(x1 >> 16)));
  const __half2 f00 = __ldg(reinterpret_cast<const __half2 *>(f + 0 * half_d + e));
  const __half2 f01 = __ldg(reinterpret_cast<const __half2 *>(f + 1 * half_d + e));
  const __half2 f10 = __ldg(reinterpret_cast<const __half2 *>(f + 2 * half_d + e));
  const __half2 f11 = __ldg(reinterpret_cast<const __half2 *>(f + 3 * half_d + e));
  const float2 p00 = __half22float2(__hmul2(f00, a)), p01 = __half22float2(__hmul2(f01, b));
  const float2 p10 = __half22float2(__hmul2(f10, a)), p11 = __half22float2(__hmul2(f11, b));
  // the CPU sum starts from +0: (0 + p0) + p1, so -0 + -0 gives +0 as there
  const __half2 o0 = __floats2half2_rn(__fadd_rn(__fadd_rn(0.f, p00.x), p01.x), __fadd_rn(__fadd_rn(0.f, p00.y), p01.y));
  const __half2 o1 = __floats2half2_rn(__fadd_rn(__fadd_rn(0.f, p10.x), p11.x), __fadd_rn(__fadd_rn(0.f, p10.y), p11.y));
  x0 = static_cast<uint32_t>(__half_as_ushort(__low2half(o0))) |
       (static_cast<uint32_t>(__half_as_ushort(__high2half(o0))) << 16);
  x1 = static_cast<uint32_t>(__half_as_ushort(__low2half(o1))) |
       (static_cast<uint32_t>(__half_as_ushort(__high2half(o1))) << 16);
}

}  // namespace b200kv
