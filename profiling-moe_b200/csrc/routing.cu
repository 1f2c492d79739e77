// Router (top-K of biased logits, sigmoid of the raw logit) and expert-map build
// (histogram -> exclusive offsets -> stable permutation -> inverse map), for sm_100a.
//
// Semantics follow the reference's eager definitions:
//   router  benchmarks/01_benchmark_router.py:33-37 (scores = x + bias; top-k; sigmoid(x[ids])),
//           kernels/triton/fused_kolibri_router.py:38-95 (optional renorm 1/(sum+1e-20)),
//           tie-break: the lower expert index wins (kernels/cuda/moeTopKFuncs.cuh:54-61 packs
//           65535-idx into the key; torch.sort(stable) gives the same order).
//   maps    kernels/cuda/customKolibriBuildExpertMapsKernels.cuh:16-83 (histogram, exclusive
//           offsets int64, unpermuted row = slot*T + token, ids outside [0,E) skipped),
//           with the (expert, token, slot) order of the CUB rank kernel
//           kernels/cuda/customKolibriBuildExpertMapsKernel.cu:96-156 instead of atomic order.
//
// Design (B200): one warp per token with the 384 logits register-resident (3 x float4 per
// lane).  A lane-local top-3 plus K warp-wide redux.sync rounds picks the top-K; ties, NaN
// rows and lanes holding more than three winners fall back to an exact key-based path.
// Maps: per-tile smem histograms; the last CTA of each super-tile (arrival counter, no spin)
// folds its tiles into one row; a second kernel (one CTA per super-tile) scans the super-tile
// rows and ranks selections stably with __match_any_sync in input order.
#include "kb_common.cuh"

#include <algorithm>
#include <math.h>

namespace kb {

// ------------------------------------------------------------------------------------
// Ordering key: a larger float gives a larger key, NaN gives the largest key (torch.sort
// puts NaN first in a descending sort), -0 and +0 share a key.  Key 0 marks "taken".
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t okey(float s) {
    uint32_t u = __float_as_uint(s);
    if (u == 0x80000000u) u = 0u;
    uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (s != s) ? 0xffffffffu : k;
}

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

// Bias registers; b + 0.0f turns a -0 bias into +0 so that no score is ever -0.
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
// Writes sel[r] (r < K) = expert id of the r-th pick.
template <int VPL, bool VEC>
__device__ __noinline__ void route_exact(const float (&s)[VPL], int E, int K, int lane,
                                         int* sel) {
    uint32_t key[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) key[j] = (expert_of<VEC>(lane, j) < E) ? okey(s[j]) : 0u;
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

// Fast top-K (VEC layout, K <= 8): lane-local top-3 by value (min/max network), then K warp
// rounds over the lanes' current candidates.  Returns false (nothing written) when the row
// holds a NaN, when two lanes offer equal values in a round, or when a lane would need its
// fourth value; the caller then runs route_exact.  Both paths produce the same result.
template <int VPL>
__device__ __forceinline__ bool route_fast(const float (&s)[VPL], int K, int lane, int* sel) {
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
    const uint32_t k1 = okey(b1), k2 = okey(b2), k3 = okey(b3);
    uint32_t cur = k1;
    int c = 0, r0 = 0, r1 = 0, r2 = 0;
    bool exhausted_early = false;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        if (r >= K) break;
        const uint32_t wmax = __reduce_max_sync(FULL_MASK, cur);
        const bool eq = (cur == wmax);
        const unsigned m = __ballot_sync(FULL_MASK, eq);
        if (m & (m - 1u)) return false;  // two lanes offer the same value
        if (eq) {
            if (c == 0) { r0 = r; cur = k2; }
            else if (c == 1) { r1 = r; cur = k3; }
            else { r2 = r; cur = 0u; exhausted_early = (r + 1 < K); }
            ++c;
        }
    }
    if (__any_sync(FULL_MASK, exhausted_early)) return false;
    // Register positions of the taken values: the first occurrence of b1, the first other
    // occurrence of b2, then of b3 (equal values inside a lane keep index order).
    int i1 = 0, i2 = 0, i3 = 0;
#pragma unroll
    for (int j = VPL - 1; j >= 0; --j)
        if (s[j] == b1) i1 = j;
    if (__any_sync(FULL_MASK, c >= 2)) {
#pragma unroll
        for (int j = VPL - 1; j >= 0; --j)
            if (s[j] == b2 && j != i1) i2 = j;
        if (__any_sync(FULL_MASK, c >= 3)) {
#pragma unroll
            for (int j = VPL - 1; j >= 0; --j)
                if (s[j] == b3 && j != i1 && j != i2) i3 = j;
        }
    }
    if (c >= 1) sel[r0] = expert_of<true>(lane, i1);
    if (c >= 2) sel[r1] = expert_of<true>(lane, i2);
    if (c >= 3) sel[r2] = expert_of<true>(lane, i3);
    __syncwarp();
    return true;
}

// Route one token: sel[0..K) <- expert ids, best first.
template <int VPL, bool VEC>
__device__ __forceinline__ void route_token(const float* __restrict__ row, const float (&b)[VPL],
                                            int E, int K, int lane, int* sel) {
    float s[VPL];
    {
        float x[VPL];
        load_row<VPL, VEC>(row, E, lane, x);
#pragma unroll
        for (int j = 0; j < VPL; ++j) s[j] = x[j] + b[j];
    }
    bool done = false;
    if constexpr (VEC) {
        if (K <= 8) done = route_fast<VPL>(s, K, lane, sel);
    }
    if (!done) route_exact<VPL, VEC>(s, E, K, lane, sel);
}

__device__ __forceinline__ float sigmoid_acc(float x) { return 1.0f / (1.0f + expf(-x)); }

// Lane r < K: weight of the r-th pick from the raw (un-biased) logit; optional renorm.
__device__ __forceinline__ float pick_weight(const float* __restrict__ row, int id, int K,
                                             int lane, int renorm) {
    float w = 0.0f;
    if (lane < K) w = sigmoid_acc(row[id]);
    if (renorm) {
        const float sum = warp_sum(w);
        w = w * (1.0f / (sum + 1e-20f));
    }
    return w;
}

template <typename WT>
__device__ __forceinline__ void store_w(WT* p, float v) { *p = Elem<WT>::from_f(v); }

// ------------------------------------------------------------------------------------
// kb_router kernel: 8 warps per CTA, one token per warp per iteration.
// ------------------------------------------------------------------------------------
template <int VPL, bool VEC, typename WT>
__global__ void __launch_bounds__(256) router_kernel(const float* __restrict__ logits,
                                                     const float* __restrict__ bias,
                                                     int32_t* __restrict__ ids,
                                                     WT* __restrict__ w, int64_t T, int E,
                                                     int K, int renorm) {
    pdl_wait();
    pdl_launch();
    __shared__ int sel_sm[8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* sel = sel_sm[warp];
    float b[VPL];
    load_bias<VPL, VEC>(bias, E, lane, b);
    for (int64_t t = (int64_t)blockIdx.x * 8 + warp; t < T; t += (int64_t)gridDim.x * 8) {
        const float* row = logits + t * E;
        route_token<VPL, VEC>(row, b, E, K, lane, sel);
        const int id = (lane < K) ? sel[lane] : 0;
        const float wv = pick_weight(row, id, K, lane, renorm);
        if (lane < K) {
            ids[t * K + lane] = id;
            store_w(w + t * K + lane, wv);
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------------------------
// Expert-map building blocks (block-wide; blockDim a multiple of 32).
// ------------------------------------------------------------------------------------

// Phase A: per-warp histograms of the selections sel[0..n) (contiguous warp ranges of
// 32-wide chunks).  whist: [nwarps][E] in smem, zeroed here.
__device__ __forceinline__ void warp_ranges(int n, int& c0, int& c1) {
    const int nwarps = blockDim.x >> 5, warp = threadIdx.x >> 5;
    const int chunks = (n + 31) >> 5;
    const int per = (chunks + nwarps - 1) / nwarps;
    c0 = min(chunks, warp * per);
    c1 = min(chunks, c0 + per);
}

__device__ void count_per_warp(const int* sel, int n, int E, int* whist) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* h = whist + warp * E;
    for (int e = lane; e < E; e += 32) h[e] = 0;
    __syncwarp();
    int c0, c1;
    warp_ranges(n, c0, c1);
    for (int c = c0; c < c1; ++c) {
        const int i = c * 32 + lane;
        const int e = (i < n) ? sel[i] : -1;
        const bool valid = (e >= 0 && e < E);
        const unsigned peers = __match_any_sync(FULL_MASK, valid ? e : -1);
        const int leader = 31 - __clz(peers);
        if (valid && lane == leader) h[e] += __popc(peers);
        __syncwarp();
    }
}

// Phase B (after __syncthreads): whist[w][e] <- sum_{w'<w} whist[w'][e] (exclusive over
// warps); tot[e] <- column total.
__device__ void scan_over_warps(int E, int* whist, int* tot) {
    const int nwarps = blockDim.x >> 5;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < nwarps; ++w) {
            const int v = whist[w * E + e];
            whist[w * E + e] = run;
            run += v;
        }
        tot[e] = run;
    }
}

// Exclusive block scan of tot[0..E) into offs[0..E], offs[E] = sum.  Uses the first
// ceil(E/32) warps; needs __syncthreads before and after.  scratch: >= 16 ints.
__device__ void scan_experts(const int* tot, int E, int* offs, int* scratch) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = (E + 31) >> 5;
    int v = 0, incl = 0;
    if (warp < nw) {
        const int e = warp * 32 + lane;
        v = (e < E) ? tot[e] : 0;
        incl = warp_incl_scan(v, lane);
        if (lane == 31) scratch[warp] = incl;
    }
    __syncthreads();
    if (warp == 0) {
        int s = (lane < nw) ? scratch[lane] : 0;
        s = warp_incl_scan(s, lane);
        if (lane < nw) scratch[16 + lane] = s;  // inclusive warp totals
    }
    __syncthreads();
    if (warp < nw) {
        const int e = warp * 32 + lane;
        const int before = (warp > 0) ? scratch[16 + warp - 1] : 0;
        if (e < E) offs[e] = before + incl - v;
        if (e == E - 1) offs[E] = before + incl;
    }
}

// Phase C: stable ranks and scatter.  whist[w][e] holds the first permuted row of warp
// w's selections of expert e (base already added).  sel0 = global index of sel[0].
__device__ void rank_scatter(const int* sel, int n, int64_t sel0, int64_t T, int E, int K,
                             int* whist, int32_t* __restrict__ p2u,
                             int32_t* __restrict__ u2p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* h = whist + warp * E;
    const unsigned lt = (1u << lane) - 1u;
    int c0, c1;
    warp_ranges(n, c0, c1);
    for (int c = c0; c < c1; ++c) {
        const int i = c * 32 + lane;
        const int e = (i < n) ? sel[i] : -1;
        const bool valid = (e >= 0 && e < E);
        const unsigned peers = __match_any_sync(FULL_MASK, valid ? e : -1);
        const int leader = 31 - __clz(peers);
        const int base = valid ? h[e] : 0;
        __syncwarp();
        if (valid && lane == leader) h[e] = base + __popc(peers);
        __syncwarp();
        if (i < n) {
            const int64_t g = sel0 + i;
            const int64_t tok = g / K;
            const int slot = (int)(g - tok * K);
            const int32_t u = (int32_t)(slot * T + tok);
            if (valid) {
                const int rank = base + __popc(peers & lt);
                p2u[rank] = u;
                if (u2p) u2p[u] = rank;
            } else if (u2p) {
                u2p[u] = -1;
            }
        }
    }
}

__device__ void write_offsets(const int* offs, const int* tot, int E, int64_t nsel,
                              int32_t* counts, int64_t* offsets, int32_t* p2u) {
    for (int e = threadIdx.x; e <= E; e += blockDim.x) {
        offsets[e] = (int64_t)offs[e];
        if (counts && e < E) counts[e] = tot[e];
    }
    // Rows past the last valid selection (ids outside [0, E)) are marked -1.
    for (int64_t r = (int64_t)offs[E] + threadIdx.x; r < nsel; r += blockDim.x) p2u[r] = -1;
}

// ------------------------------------------------------------------------------------
// Single-CTA maps (small T): optional routing, then all phases in shared memory.
// smem: sel[T*K] | whist[32][E] | tot[E] | offs[E+1] | scratch[32]
// ------------------------------------------------------------------------------------
template <int VPL, bool VEC, bool ROUTE>
__global__ void __launch_bounds__(1024) maps_single_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias,
    const int32_t* __restrict__ ids_in, int32_t* __restrict__ ids_out, float* __restrict__ w,
    int64_t T, int E, int K, int renorm, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p) {
    pdl_wait();
    pdl_launch();
    extern __shared__ int smem[];
    const int n = (int)(T * K);
    const int nwarps = blockDim.x >> 5;
    int* sel = smem;
    int* whist = sel + ((n + 3) & ~3);
    int* tot = whist + nwarps * E;
    int* offs = tot + E;
    int* scratch = offs + E + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if constexpr (ROUTE) {
        float b[VPL];
        load_bias<VPL, VEC>(bias, E, lane, b);
        __shared__ int sel_sm[32][32];
        for (int64_t t = warp; t < T; t += nwarps) {
            const float* row = logits + t * E;
            route_token<VPL, VEC>(row, b, E, K, lane, sel_sm[warp]);
            const int id = (lane < K) ? sel_sm[warp][lane] : 0;
            const float wv = pick_weight(row, id, K, lane, renorm);
            if (lane < K) {
                sel[t * K + lane] = id;
                ids_out[t * K + lane] = id;
                w[t * K + lane] = wv;
            }
            __syncwarp();
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) sel[i] = ids_in[i];
    }
    __syncthreads();
    count_per_warp(sel, n, E, whist);
    __syncthreads();
    scan_over_warps(E, whist, tot);
    __syncthreads();
    scan_experts(tot, E, offs, scratch);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int base = offs[e];
        for (int wv = 0; wv < nwarps; ++wv) whist[wv * E + e] += base;
    }
    write_offsets(offs, tot, E, n, counts, offsets, p2u);
    __syncthreads();
    rank_scatter(sel, n, 0, T, E, K, whist, p2u, u2p);
}

// ------------------------------------------------------------------------------------
// Multi-CTA maps, kernel 1: per-tile histogram (optionally routing the tile first).
// Tile = TT tokens; super-tile = tiles_per_super consecutive tiles.  The last CTA of a
// super-tile to arrive sums the super-tile's rows into super_hist and resets the counter.
// ------------------------------------------------------------------------------------
struct MapsWs {
    unsigned* arrive;   // [S]      zero between calls
    int* tile_counts;   // [num_tiles][E]
    int* super_hist;    // [S][E]
};

template <int VPL, bool VEC, bool ROUTE>
__global__ void __launch_bounds__(256) maps_count_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias,
    const int32_t* __restrict__ ids_in, int32_t* __restrict__ ids_out, float* __restrict__ w,
    int64_t T, int E, int K, int renorm, int TT, int tiles_per_super, int num_tiles,
    MapsWs ws) {
    pdl_wait();
    pdl_launch();
    __shared__ int hist[E_MAX];
    __shared__ int sel_sm[8][32];
    __shared__ int is_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int64_t t0 = (int64_t)tile * TT;
    const int64_t t1 = (T < t0 + TT ? T : t0 + TT);
    if constexpr (ROUTE) {
        float b[VPL];
        load_bias<VPL, VEC>(bias, E, lane, b);
        for (int64_t t = t0 + warp; t < t1; t += 8) {
            const float* row = logits + t * E;
            route_token<VPL, VEC>(row, b, E, K, lane, sel_sm[warp]);
            const int id = (lane < K) ? sel_sm[warp][lane] : 0;
            const float wv = pick_weight(row, id, K, lane, renorm);
            if (lane < K) {
                ids_out[t * K + lane] = id;
                w[t * K + lane] = wv;
                atomicAdd(&hist[id], 1);
            }
            __syncwarp();
        }
    } else {
        for (int64_t i = t0 * K + threadIdx.x; i < t1 * K; i += blockDim.x) {
            const int e = __ldg(ids_in + i);
            if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
        }
    }
    __syncthreads();
    int* row = ws.tile_counts + (size_t)tile * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) row[e] = hist[e];
    __threadfence();
    __syncthreads();
    const int s = tile / tiles_per_super;
    const int first = s * tiles_per_super;
    const int members = min(num_tiles, first + tiles_per_super) - first;
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(ws.arrive + s, 1u);
        is_last = (prev == (unsigned)(members - 1));
    }
    __syncthreads();
    if (is_last) {
        __threadfence();
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            int sum = 0;
            for (int q = 0; q < members; ++q)
                sum += __ldcg(ws.tile_counts + (size_t)(first + q) * E + e);
            ws.super_hist[(size_t)s * E + e] = sum;
        }
        if (threadIdx.x == 0) ws.arrive[s] = 0u;
    }
}

// Multi-CTA maps, kernel 2: one CTA per super-tile.  Scans the super-tile rows, writes
// counts/offsets (CTA 0), ranks the super-tile's selections and scatters p2u/u2p.
// smem: sel[G*K] | whist[32][E] | tot[E] | pre[E] | offs[E+1] | scratch[32]
__global__ void __launch_bounds__(1024) maps_scatter_kernel(
    const int32_t* __restrict__ ids, int64_t T, int E, int K, int super_tokens, int S,
    const int* __restrict__ super_hist, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p) {
    pdl_wait();
    pdl_launch();
    extern __shared__ int smem[];
    const int s = blockIdx.x;
    const int nwarps = blockDim.x >> 5;
    const int64_t tok0 = (int64_t)s * super_tokens;
    const int ntok = (int)((T - tok0) < super_tokens ? (T - tok0) : (int64_t)super_tokens);
    const int n = ntok * K;
    const int cap = super_tokens * K;
    int* sel = smem;
    int* whist = sel + ((cap + 3) & ~3);
    int* tot = whist + nwarps * E;
    int* pre = tot + E;
    int* offs = pre + E;
    int* scratch = offs + E + 1;
    // Selections of this super-tile (contiguous in ids).
    const int32_t* src = ids + tok0 * K;
    for (int i = threadIdx.x; i < n; i += blockDim.x) sel[i] = __ldcg(src + i);
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int t_all = 0, t_pre = 0;
#pragma unroll 8
        for (int q = 0; q < S; ++q) {
            const int v = __ldcg(super_hist + (size_t)q * E + e);
            t_all += v;
            t_pre += (q < s) ? v : 0;
        }
        tot[e] = t_all;
        pre[e] = t_pre;
    }
    __syncthreads();
    scan_experts(tot, E, offs, scratch);
    __syncthreads();
    if (s == 0) write_offsets(offs, tot, E, T * K, counts, offsets, p2u);
    count_per_warp(sel, n, E, whist);
    __syncthreads();
    scan_over_warps(E, whist, tot);  // tot is reused as scratch here
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int base = offs[e] + pre[e];
        for (int wv = 0; wv < nwarps; ++wv) whist[wv * E + e] += base;
    }
    __syncthreads();
    rank_scatter(sel, n, tok0 * K, T, E, K, whist, p2u, u2p);
}

// ------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------
namespace {

constexpr int kSingleThreads = 1024;
constexpr int kScatterThreads = 1024;
constexpr int kTargetSupers = 64;
constexpr int kMaxSingleSel = 12288;  // single-CTA path: T*K selections held in smem

struct MapsPlan {
    bool single;
    int TT;               // tokens per tile (kernel 1)
    int num_tiles;
    int tiles_per_super;
    int S;
    int super_tokens;
    size_t ws_bytes;
    size_t smem_single;
    size_t smem_scatter;
};

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

size_t single_smem(int64_t T, int E, int K) {
    const size_t n = (size_t)T * K;
    return (((n + 3) & ~size_t(3)) + (size_t)32 * E + 2 * E + 1 + 32) * sizeof(int);
}

MapsPlan make_plan(int64_t T, int E, int K, int mode, bool route) {
    MapsPlan p{};
    const int64_t n = T * K;
    const bool fits_single = n <= kMaxSingleSel;
    const int64_t auto_single_T = route ? 32 : 768;
    p.single = (mode == KB_MAPS_SINGLE_CTA) ? fits_single
             : (mode == KB_MAPS_MULTI_CTA) ? false
             : (fits_single && T <= auto_single_T);
    p.smem_single = single_smem(T, E, K);
    if (p.single) return p;
    if (route) {
        // 8 warps per tile; tokens per warp grows with T so that ~2 CTAs per SM remain.
        int64_t tpw = (T + 148 * 2 * 8 - 1) / (148 * 2 * 8);
        tpw = std::max<int64_t>(1, std::min<int64_t>(16, tpw));
        p.TT = (int)(8 * tpw);
    } else {
        p.TT = 256;
    }
    p.num_tiles = (int)((T + p.TT - 1) / p.TT);
    // Kernel 2 holds a super-tile's selections in shared memory: cap them at 24576 (96 KB);
    // beyond that the number of super-tiles grows instead.
    const int max_tps = std::max(1, 24576 / (K * p.TT));
    p.tiles_per_super = std::min(max_tps, (p.num_tiles + kTargetSupers - 1) / kTargetSupers);
    p.S = (p.num_tiles + p.tiles_per_super - 1) / p.tiles_per_super;
    p.super_tokens = p.TT * p.tiles_per_super;
    p.ws_bytes = align256((size_t)p.S * sizeof(unsigned)) +
                 align256((size_t)p.num_tiles * E * sizeof(int)) +
                 align256((size_t)p.S * E * sizeof(int));
    const size_t cap = (size_t)p.super_tokens * K;
    p.smem_scatter = (((cap + 3) & ~size_t(3)) + (size_t)(kScatterThreads / 32) * E + 3 * E + 1 + 32) * sizeof(int);
    return p;
}

MapsWs carve(void* ws, const MapsPlan& p, int E) {
    char* b = static_cast<char*>(ws);
    MapsWs w;
    w.arrive = reinterpret_cast<unsigned*>(b);
    b += align256((size_t)p.S * sizeof(unsigned));
    w.tile_counts = reinterpret_cast<int*>(b);
    b += align256((size_t)p.num_tiles * E * sizeof(int));
    w.super_hist = reinterpret_cast<int*>(b);
    return w;
}

int check_common(int64_t T, int E, int K) {
    if (T < 0 || E <= 0 || K <= 0) return KB_ERR_INVALID_ARG;
    if (E > E_MAX || K > 32 || K > E) return KB_ERR_UNSUPPORTED;
    if (T * (int64_t)K >= (int64_t)INT32_MAX) return KB_ERR_TOO_LARGE;
    return KB_OK;
}

// Dispatch on the register layout for E.
template <template <int, bool> class Fn, typename... Args>
int with_layout(int E, Args&&... args) {
    if (E == 384) return Fn<12, true>::run(std::forward<Args>(args)...);
    if (E == 256) return Fn<8, true>::run(std::forward<Args>(args)...);
    if (E == 512) return Fn<16, true>::run(std::forward<Args>(args)...);
    if (E == 128) return Fn<4, true>::run(std::forward<Args>(args)...);
    return Fn<16, false>::run(std::forward<Args>(args)...);
}

template <int VPL, bool VEC>
struct RouterLaunch {
    static int run(const float* logits, const float* bias, int32_t* ids, void* w, int w_dtype,
                   int64_t T, int E, int K, int renorm, cudaStream_t st) {
        const int64_t ctas = std::min<int64_t>((T + 7) / 8, 148 * 64);
        dim3 grid((unsigned)std::max<int64_t>(1, ctas)), block(256);
        switch (w_dtype) {
            case KB_F32:
                return launch(router_kernel<VPL, VEC, float>, grid, block, 0, st, logits, bias,
                              ids, static_cast<float*>(w), T, E, K, renorm);
            case KB_BF16:
                return launch(router_kernel<VPL, VEC, __nv_bfloat16>, grid, block, 0, st, logits,
                              bias, ids, static_cast<__nv_bfloat16*>(w), T, E, K, renorm);
            case KB_F16:
                return launch(router_kernel<VPL, VEC, __half>, grid, block, 0, st, logits, bias,
                              ids, static_cast<__half*>(w), T, E, K, renorm);
            default:
                return KB_ERR_UNSUPPORTED;
        }
    }
};

template <bool ROUTE>
struct MapsLaunchT {
    template <int VPL, bool VEC>
    struct Impl {
        static int run(const float* logits, const float* bias, const int32_t* ids_in,
                       int32_t* ids_out, float* w, int32_t* counts, int64_t* offsets,
                       int32_t* p2u, int32_t* u2p, void* ws, size_t ws_bytes, int64_t T,
                       int E, int K, int renorm, int mode, cudaStream_t st) {
            const MapsPlan p = make_plan(T, E, K, mode, ROUTE);
            if (p.single) {
                auto* kern = maps_single_kernel<VPL, VEC, ROUTE>;
                int err = allow_smem(kern, p.smem_single);
                if (err) return err;
                return launch(kern, dim3(1), dim3(kSingleThreads), p.smem_single, st, logits, bias,
                              ids_in, ids_out, w, T, E, K, renorm, counts, offsets, p2u, u2p);
            }
            if (ws == nullptr || ws_bytes < p.ws_bytes) return KB_ERR_WORKSPACE;
            if (!aligned16(ws)) return KB_ERR_ALIGNMENT;
            const MapsWs w_ = carve(ws, p, E);
            int err = launch(maps_count_kernel<VPL, VEC, ROUTE>, dim3(p.num_tiles), dim3(256), 0,
                             st, logits, bias, ids_in, ids_out, w, T, E, K, renorm, p.TT,
                             p.tiles_per_super, p.num_tiles, w_);
            if (err) return err;
            err = allow_smem(maps_scatter_kernel, p.smem_scatter);
            if (err) return err;
            const int32_t* ids_src = ROUTE ? ids_out : ids_in;
            return launch(maps_scatter_kernel, dim3(p.S), dim3(kScatterThreads), p.smem_scatter, st,
                          ids_src, T, E, K, p.super_tokens, p.S,
                          static_cast<const int*>(w_.super_hist), counts, offsets, p2u, u2p);
        }
    };
};

template <int VPL, bool VEC>
using MapsOnly = MapsLaunchT<false>::Impl<VPL, VEC>;
template <int VPL, bool VEC>
using RouterMaps = MapsLaunchT<true>::Impl<VPL, VEC>;

// T == 0: offsets are all zero.
__global__ void zero_offsets_kernel(int64_t* offsets, int32_t* counts, int E) {
    pdl_wait();
    pdl_launch();
    for (int e = threadIdx.x; e <= E; e += blockDim.x) {
        offsets[e] = 0;
        if (counts && e < E) counts[e] = 0;
    }
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int kb_router(const float* logits, const float* bias, int32_t* ids, void* weights,
                         int w_dtype, int64_t T, int E, int K, int renorm, kb_stream_t stream) {
    int st = check_common(T, E, K);
    if (st) return st;
    if (T == 0) return KB_OK;
    if (!logits || !ids || !weights) return KB_ERR_INVALID_ARG;
    if (w_dtype != KB_F32 && w_dtype != KB_BF16 && w_dtype != KB_F16) return KB_ERR_UNSUPPORTED;
    if ((E % 128 == 0) && (!aligned16(logits) || (bias && !aligned16(bias)))) return KB_ERR_ALIGNMENT;
    return with_layout<RouterLaunch>(E, logits, bias, ids, weights, w_dtype, T, E, K, renorm,
                                     (cudaStream_t)stream);
}

extern "C" size_t kb_expert_maps_workspace_bytes(int64_t T, int E, int K) {
    if (check_common(T, E, K) != KB_OK || T == 0) return 0;
    return make_plan(T, E, K, KB_MAPS_MULTI_CTA, false).ws_bytes;
}

extern "C" size_t kb_router_maps_workspace_bytes(int64_t T, int E, int K) {
    if (check_common(T, E, K) != KB_OK || T == 0) return 0;
    return make_plan(T, E, K, KB_MAPS_MULTI_CTA, true).ws_bytes;
}

extern "C" int kb_expert_maps(const int32_t* ids, int32_t* counts, int64_t* offsets, int32_t* p2u,
                              int32_t* u2p, void* workspace, size_t workspace_bytes, int64_t T,
                              int E, int K, int mode, kb_stream_t stream) {
    int st = check_common(T, E, K);
    if (st) return st;
    if (mode < KB_MAPS_AUTO || mode > KB_MAPS_MULTI_CTA) return KB_ERR_INVALID_ARG;
    if (!offsets) return KB_ERR_INVALID_ARG;
    if (T == 0)
        return launch(zero_offsets_kernel, dim3(1), dim3(512), 0, (cudaStream_t)stream, offsets,
                      counts, E);
    if (!ids || !p2u) return KB_ERR_INVALID_ARG;
    if (mode == KB_MAPS_SINGLE_CTA && T * K > kMaxSingleSel) return KB_ERR_UNSUPPORTED;
    return with_layout<MapsOnly>(E, nullptr, nullptr, ids, nullptr, nullptr, counts, offsets, p2u,
                                 u2p, workspace, workspace_bytes, T, E, K, 0, mode,
                                 (cudaStream_t)stream);
}

extern "C" int kb_router_maps(const float* logits, const float* bias, int32_t* ids, float* weights,
                              int32_t* counts, int64_t* offsets, int32_t* p2u, int32_t* u2p,
                              void* workspace, size_t workspace_bytes, int64_t T, int E, int K,
                              int renorm, int mode, kb_stream_t stream) {
    int st = check_common(T, E, K);
    if (st) return st;
    if (mode < KB_MAPS_AUTO || mode > KB_MAPS_MULTI_CTA) return KB_ERR_INVALID_ARG;
    if (!offsets) return KB_ERR_INVALID_ARG;
    if (T == 0)
        return launch(zero_offsets_kernel, dim3(1), dim3(512), 0, (cudaStream_t)stream, offsets,
                      counts, E);
    if (!logits || !ids || !weights || !p2u) return KB_ERR_INVALID_ARG;
    if ((E % 128 == 0) && (!aligned16(logits) || (bias && !aligned16(bias)))) return KB_ERR_ALIGNMENT;
    if (mode == KB_MAPS_SINGLE_CTA && T * K > kMaxSingleSel) return KB_ERR_UNSUPPORTED;
    return with_layout<RouterMaps>(E, logits, bias, nullptr, ids, weights, counts, offsets, p2u,
                                   u2p, workspace, workspace_bytes, T, E, K, renorm, mode,
                                   (cudaStream_t)stream);
}
