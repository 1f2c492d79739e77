// Warp-per-token ranking shared by the router kernels (routing.cu) and the epilogue of the
// tensor-core router GEMM (router_gemm.cu): the exact K-round warp ranking (route_exact), the
// fast lane-top-3 ranking (route_fast) and the routing weight of a pick (pick_weight).  Both
// give the order of torch.sort(scores, descending=True, stable=True): larger key first, the
// lower expert first among equal keys, NaN above +inf.
#pragma once

#include "kb_common.cuh"
#include "route_math.cuh"

namespace kb {

__device__ __forceinline__ float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Element j of a lane's register row.  VEC: 4 consecutive experts per float4, lane-major
// (expert 4*(lane + 32*(j/4)) + j%4); SCALAR: expert lane + 32*j.  Both ascend with j.
template <bool VEC>
__device__ __forceinline__ int expert_of(int lane, int j) {
    return VEC ? 4 * (lane + 32 * (j >> 2)) + (j & 3) : lane + 32 * j;
}

template <int VPL, bool VEC>
__device__ __forceinline__ void load_row(const float* __restrict__ row, int E, int lane,
                                         float (&x)[VPL]) {
    if constexpr (VEC) {
#pragma unroll
        for (int q = 0; q < VPL / 4; ++q) {
            float4 v = __ldg(reinterpret_cast<const float4*>(row) + lane + 32 * q);
            x[4 * q + 0] = v.x; x[4 * q + 1] = v.y; x[4 * q + 2] = v.z; x[4 * q + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            int e = lane + 32 * j;
            x[j] = (e < E) ? __ldg(row + e) : 0.0f;
        }
    }
}

// Bias registers; b + 0.0f turns a -0 bias into +0, so that no score x + b is ever -0.
template <int VPL, bool VEC>
__device__ __forceinline__ void load_bias(const float* __restrict__ bias, int E, int lane,
                                          float (&b)[VPL]) {
    if (bias == nullptr) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) b[j] = 0.0f;
        return;
    }
    load_row<VPL, VEC>(bias, E, lane, b);
#pragma unroll
    for (int j = 0; j < VPL; ++j) b[j] = b[j] + 0.0f;
}

// Exact top-K: K rounds of (lane argmax over keys, warp max, lowest index among equal keys).
// Reads the row again from `row` (shared or global memory) and the bias from `bias` (or
// zero), so no register array crosses the call.  Writes sel[r] (r < K) = r-th pick.
template <int VPL, bool VEC>
__device__ __noinline__ void route_exact(const float* row, const float* __restrict__ bias, int E,
                                         int K, int lane, int* sel) {
    uint32_t key[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
        const int e = expert_of<VEC>(lane, j);
        float v = 0.0f;
        if (e < E) v = row[e] + (bias ? bias[e] + 0.0f : 0.0f);
        key[j] = (e < E) ? okey(v) : 0u;
    }
    for (int r = 0; r < K; ++r) {
        uint32_t best = 0u;
        int bj = 0;
#pragma unroll
        for (int j = 0; j < VPL; ++j)
            if (key[j] > best) { best = key[j]; bj = j; }
        uint32_t wmax = __reduce_max_sync(FULL_MASK, best);
        unsigned cand = (best == wmax && best != 0u) ? (unsigned)expert_of<VEC>(lane, bj)
                                                      : 0xffffffffu;
        unsigned widx = __reduce_min_sync(FULL_MASK, cand);
        if (cand == widx) {
#pragma unroll
            for (int j = 0; j < VPL; ++j)
                if (j == bj) key[j] = 0u;
        }
        if (lane == 0) sel[r] = (int)widx;
    }
    __syncwarp();
}

// Fast top-K (VEC layout, K <= 8; KT = K at compile time, or 0 for a runtime K).  Lane-local
// top-3 values by a min/max network, then K warp rounds: the lane holding the largest
// current candidate consumes it and offers its next one.  Each lane only records which rounds
// it won; the register positions of its picks are recovered once at the end.  Returns false
// (nothing written) if the row holds a NaN, two lanes offered equal values in a round, or a
// lane ran out of its three values before the last round -- route_exact then decides.
template <int VPL, int KT>
__device__ __forceinline__ bool route_fast(const float (&s)[VPL], int K_rt, int lane, int* sel) {
    const int K = KT ? KT : K_rt;
    constexpr int KMAX = KT ? KT : 8;
    float b1 = s[0], b2 = -INFINITY, b3 = -INFINITY;
#pragma unroll
    for (int j = 1; j < VPL; ++j) {
        const float v = s[j];
        const float t1 = fminf(b1, v);
        b1 = fmax_nan(b1, v);
        const float t2 = fminf(b2, t1);
        b2 = fmaxf(b2, t1);
        b3 = fmaxf(b3, t2);
    }
    if (__any_sync(FULL_MASK, b1 != b1)) return false;
    uint32_t cur = fkey(b1), nx2 = fkey(b2), nx3 = fkey(b3);
    unsigned won = 0u, clash = 0u;
    bool exhausted = false;
#pragma unroll
    for (int r = 0; r < KMAX; ++r) {
        if (KT || r < K) {
            if (KT ? (r == KT - 1) : (r == K - 1)) exhausted = __any_sync(FULL_MASK, cur == 0u);
            const uint32_t wmax = __reduce_max_sync(FULL_MASK, cur);
            const bool eq = (cur == wmax);
            const unsigned m = __ballot_sync(FULL_MASK, eq);
            clash |= m & (m - 1u);
            if (eq) {
                won |= 1u << r;
                cur = nx2;
                nx2 = nx3;
                nx3 = 0u;
            }
        }
    }
    if (clash != 0u || exhausted) return false;
    const int nwon = __popc(won);
    int i1 = 0, i2 = 0, i3 = 0;
#pragma unroll
    for (int j = VPL - 1; j >= 0; --j)
        if (s[j] == b1) i1 = j;
    if (__any_sync(FULL_MASK, nwon >= 2)) {
#pragma unroll
        for (int j = VPL - 1; j >= 0; --j)
            if (s[j] == b2 && j != i1) i2 = j;
        if (__any_sync(FULL_MASK, nwon >= 3)) {
#pragma unroll
            for (int j = VPL - 1; j >= 0; --j)
                if (s[j] == b3 && j != i1 && j != i2) i3 = j;
        }
    }
    if (won) {
        unsigned wv = won;
        sel[__ffs(wv) - 1] = expert_of<true>(lane, i1);
        wv &= wv - 1u;
        if (wv) {
            sel[__ffs(wv) - 1] = expert_of<true>(lane, i2);
            wv &= wv - 1u;
            if (wv) sel[__ffs(wv) - 1] = expert_of<true>(lane, i3);
        }
    }
    __syncwarp();
    return true;
}


// Lane r < K holds pick r: weight = sigmoid(raw logit); optional renorm over the K picks.
__device__ __forceinline__ float pick_weight(float x, int K, int lane, int renorm) {
    float w = (lane < K) ? sigmoid_acc(x) : 0.0f;
    if (renorm) {
        const float sum = warp_sum(w);
        w = w * (1.0f / (sum + 1e-20f));
    }
    return w;
}

}  // namespace kb
