// MoE finalize (combine) for sm_100a: the weighted sum of each token's K expert-output rows,
//   out[t, :] = dtype( sum_{k < K} float(expert_out[u2p[k*T + t], :]) * w[t, k] )
// in fp32 with the products rounded first and the sum taken in slot order k = 0 .. K-1, as
// the reference harness computes it: (expert_out[u2p.view(K, T)].float() *
// weights.float().t().unsqueeze(-1)).sum(0).to(dtype)  (benchmarks/11_profile_2block_e2e.py:
// 259-262).  A slot whose u2p is negative (an id outside [0, E) at routing) contributes 0.
//
// One CTA per token; each thread owns 16-byte vectors of the row (row_shape), gathers the K
// source vectors (all loads in flight together), and writes the combined vector once
// (finalize_math.cuh).
// HBM bound: K + 1 row transfers per token.
#include "finalize_math.cuh"
#include "norm_math.cuh"

#include <algorithm>

namespace kb {

template <typename T, int VPT, int KMAX>
__global__ void __launch_bounds__(512) moe_finalize_kernel(const T* __restrict__ expert_out,
                                                           const int32_t* __restrict__ u2p,
                                                           const float* __restrict__ w,
                                                           T* __restrict__ out, int64_t ntok,
                                                           int K, int64_t rows, int H) {
    pdl_wait();
    pdl_launch();
    for (int64_t t = blockIdx.x; t < ntok; t += gridDim.x)
        finalize_token<T, VPT, KMAX>(expert_out, u2p, w, out, t, ntok, K, rows, H);
}

namespace {

template <typename T, int KMAX>
int finalize_launch(const void* eo, const int32_t* u2p, const float* w, void* out, int64_t T_,
                    int K, int64_t H, cudaStream_t st) {
    constexpr int N = 16 / sizeof(T);
    const RowShape rs = row_shape((int)(H / N));
    const unsigned grid = (unsigned)std::min<int64_t>(T_, (int64_t)INT32_MAX);
    const int64_t rows = T_ * K;
#define KB_FIN(V)                                                                               \
    case V:                                                                                     \
        return launch(moe_finalize_kernel<T, V, KMAX>, dim3(grid), dim3(rs.threads), 0, st,      \
                      static_cast<const T*>(eo), u2p, w, static_cast<T*>(out), T_, K, rows,    \
                      (int)H);
    switch (rs.vpt) {
        KB_FIN(1) KB_FIN(2) KB_FIN(3) KB_FIN(4) KB_FIN(6) KB_FIN(8)
        default: break;
    }
#undef KB_FIN
    return KB_ERR_UNSUPPORTED;
}

template <typename T>
int finalize_k(const void* eo, const int32_t* u2p, const float* w, void* out, int64_t T_, int K,
               int64_t H, cudaStream_t st) {
    if (K <= 8) return finalize_launch<T, 8>(eo, u2p, w, out, T_, K, H, st);
    return finalize_launch<T, 32>(eo, u2p, w, out, T_, K, H, st);
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int kb_moe_finalize(const void* expert_out, const int32_t* u2p, const float* weights,
                               void* out, int64_t T, int K, int64_t H, int dtype,
                               kb_stream_t stream) {
    if (T < 0 || K <= 0 || H <= 0) return KB_ERR_INVALID_ARG;
    if (K > 32) return KB_ERR_UNSUPPORTED;
    if (T == 0) return KB_OK;
    if (!expert_out || !u2p || !weights || !out) return KB_ERR_INVALID_ARG;
    if (T * K >= (int64_t)INT32_MAX) return KB_ERR_TOO_LARGE;
    if (!aligned16(expert_out) || !aligned16(out)) return KB_ERR_ALIGNMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case KB_BF16:
            if (H % 8) return KB_ERR_ALIGNMENT;
            return finalize_k<__nv_bfloat16>(expert_out, u2p, weights, out, T, K, H, st);
        case KB_F16:
            if (H % 8) return KB_ERR_ALIGNMENT;
            return finalize_k<__half>(expert_out, u2p, weights, out, T, K, H, st);
        case KB_F32:
            if (H % 4) return KB_ERR_ALIGNMENT;
            return finalize_k<float>(expert_out, u2p, weights, out, T, K, H, st);
        default:
            return KB_ERR_UNSUPPORTED;
    }
}
