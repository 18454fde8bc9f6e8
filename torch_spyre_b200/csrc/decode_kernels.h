// Launchers of the decode kernels (internal to libb200kv).
#pragma once

#include "decode_common.cuh"

namespace b200kv {

// Tensor-core variant (decode_mma.cu): the default.
int launch_decode_mma(int group, const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a,
                      int items_per_cta, cudaStream_t stream);
// CUDA-core fp32 variant (decode_simt.cu), B200KV_DECODE_KERNEL=simt.
int launch_decode_simt(int group, const CUtensorMap &km, const CUtensorMap &vm, DecodeArgs &a,
                       int items_per_cta, cudaStream_t stream);

}  // namespace b200kv
