// The per-token arithmetic of the MoE finalize, shared by kb_moe_finalize and the
// expert-parallel combine (kb_ep_combine), so that both produce the same bits:
//   out[t, :] = dtype( sum_{k < K} float(expert_out[u2p[k*T + t], :]) * w[t, k] )
// fp32 products rounded first, summed in slot order k = 0 .. K-1, one rounding to dtype
// (benchmarks/11_profile_2block_e2e.py:259-262).  A slot whose u2p is negative or >= rows
// contributes nothing.  Each thread of the CTA owns VPT 16-byte vectors of the row; the K
// source vectors of one output vector are loaded together.
#pragma once

#include "kb_common.cuh"

namespace kb {

template <typename T, int VPT, int KMAX>
__device__ __forceinline__ void finalize_token(const T* __restrict__ expert_out,
                                               const int32_t* __restrict__ u2p,
                                               const float* __restrict__ w, T* __restrict__ out,
                                               int64_t t, int64_t ntok, int K, int64_t rows,
                                               int H) {
    using V = Vec16<T>;
    constexpr int N = V::N;
    const int nvec = H / N;
    int64_t src[KMAX];
    float wk[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        src[k] = -1;
        wk[k] = 0.0f;
        if (k < K) {
            const int64_t r = __ldg(u2p + (int64_t)k * ntok + t);
            src[k] = (r >= 0 && r < rows) ? r : -1;
            wk[k] = __ldg(w + t * K + k);
        }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int v = threadIdx.x + i * blockDim.x;
        if (v >= nvec) continue;
        V x[KMAX];
#pragma unroll
        for (int k = 0; k < KMAX; ++k)
            if (src[k] >= 0) x[k].u = ld_stream(reinterpret_cast<const uint4*>(expert_out + src[k] * H) + v);
        float acc[N];
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] = 0.0f;
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
            if (src[k] >= 0) {
#pragma unroll
                for (int e = 0; e < N; ++e)
                    acc[e] = __fadd_rn(acc[e], __fmul_rn(Elem<T>::to_f(x[k].e[e]), wk[k]));
            }
        }
        V o;
#pragma unroll
        for (int e = 0; e < N; ++e) o.e[e] = Elem<T>::from_f(acc[e]);
        st_stream(reinterpret_cast<uint4*>(out + t * H) + v, o.u);
    }
}

}  // namespace kb
