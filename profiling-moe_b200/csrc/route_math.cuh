// Scalar routing arithmetic shared by the router kernels (routing.cu) and the decode-chain
// kernel (chain.cu), so that both rank and weigh experts identically.
#pragma once

#include "kb_common.cuh"

namespace kb {

// ------------------------------------------------------------------------------------
// Ordering keys.  okey: a larger float gives a larger key, NaN the largest (torch.sort puts
// NaN first in a descending sort), -0 and +0 share a key; key 0 marks "taken".
// fkey: the same map for values known to be neither NaN nor -0.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t okey(float s) {
    uint32_t u = __float_as_uint(s);
    if (u == 0x80000000u) u = 0u;
    uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (s != s) ? 0xffffffffu : k;
}
__device__ __forceinline__ uint32_t fkey(float s) {
    const uint32_t u = __float_as_uint(s);
    return u ^ ((uint32_t)((int32_t)u >> 31) | 0x80000000u);
}

// Router weight: sigmoid of the raw (un-biased) logit, with the accurate expf.
__device__ __forceinline__ float sigmoid_acc(float x) { return 1.0f / (1.0f + expf(-x)); }

}  // namespace kb
