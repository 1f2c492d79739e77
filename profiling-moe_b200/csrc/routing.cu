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
// Design (B200):
//  * Router: one warp per token, the row of E logits spread over the lanes as float4s.  Rows
//    stream through a per-warp cp.async double buffer in shared memory, so the next row is
//    in flight while the current one is ranked and the raw logit of a pick is a shared-memory
//    read.  Ranking: lane-local top-3 (min/max network), then K warp rounds of redux.sync over
//    the lanes' current candidates; a row with a NaN, a tie between lanes, or a lane holding
//    more than three picks is re-ranked by an exact key-based path.  Both give the same answer.
//  * Maps at large T: one persistent cooperative kernel.  Phase 1 routes (or loads ids) and
//    builds a per-CTA histogram; phase 2 scans each expert's column of CTA histograms; phase 3
//    ranks the CTA's selections stably in input order (expert lanes of a chunk found by
//    ballots over the expert bits) and scatters.
//    Phases are separated by a grid barrier whose wait is bounded (on timeout the kernel sets
//    an error flag in the workspace and returns; later calls then poison the offsets).
//  * Small T: one CTA does everything in shared memory.  A two-kernel variant (tile
//    histograms, last-arriving CTA folds super-tiles, one CTA per super-tile scatters) remains
//    as the path for shapes the persistent kernel cannot hold.
#include "ep_common.cuh"
#include "kb_common.cuh"
#include "route_math.cuh"
#include "warp_route.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <math.h>
#include <map>
#include <mutex>
#include <tuple>

namespace kb {

// Where the picks of a token go.  Lanes < K hold pick `lane`.  MAPS additionally appends
// the id to this CTA's shared-memory selection list and histogram.
template <typename WT, bool SEL, bool HIST>
struct RouteSink {
    int32_t* ids;    // global [T, K]
    WT* w;           // global [T, K]
    int* sel;        // shared memory, selections of tokens sel_t0.. (SEL)
    int64_t sel_t0;
    int* hist;       // shared memory histogram (HIST)
    __device__ __forceinline__ void put(int64_t t, int K, int lane, int id, float wv) const {
        if (lane < K) {
            const int64_t o = t * K + lane;
            ids[o] = id;
            w[o] = Elem<WT>::from_f(wv);
            if constexpr (SEL) sel[(int)(t - sel_t0) * K + lane] = id;
            if constexpr (HIST) atomicAdd(&hist[id], 1);
        }
    }
};

// ------------------------------------------------------------------------------------
// cp.async helpers (16-byte global -> shared copies, L1 bypass)
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

#include "trouter.cuh"

// ------------------------------------------------------------------------------------
// Warp router loop over tokens t_begin, t_begin+t_step, ... < t_end.
// VEC: rows stream through ring[2][E] (this warp's shared-memory double buffer); the next
// row's copy is issued before the current row is ranked.  sel: a 32-int scratch per warp.
// ------------------------------------------------------------------------------------
template <int VPL, bool VEC, int KT, typename Sink>
__device__ __forceinline__ void route_tokens(const float* __restrict__ logits,
                                             const float* __restrict__ bias,
                                             const float (&b)[VPL], int E, int K, int renorm,
                                             int64_t t_begin, int64_t t_end, int64_t t_step,
                                             float* ring, int* sel, const Sink& sink) {
    const int lane = threadIdx.x & 31;
    if constexpr (VEC) {
        const float* src = logits + t_begin * E + 4 * lane;
        const int64_t src_step = t_step * E;
        float* dst0 = ring + 4 * lane;
        if (t_begin < t_end) {
#pragma unroll
            for (int q = 0; q < VPL / 4; ++q) cp_async16(dst0 + 128 * q, src + 128 * q);
        }
        cp_async_commit();
        int slot = 0;
        for (int64_t t = t_begin; t < t_end; t += t_step, slot ^= 1) {
            src += src_step;
            if (t + t_step < t_end) {
                float* dst = dst0 + (slot ^ 1) * E;
#pragma unroll
                for (int q = 0; q < VPL / 4; ++q) cp_async16(dst + 128 * q, src + 128 * q);
            }
            cp_async_commit();
            cp_async_wait<1>();
            __syncwarp();
            const float* rb = ring + slot * E;
            float s[VPL];
#pragma unroll
            for (int q = 0; q < VPL / 4; ++q) {
                const float4 v = reinterpret_cast<const float4*>(rb)[lane + 32 * q];
                s[4 * q + 0] = v.x + b[4 * q + 0];
                s[4 * q + 1] = v.y + b[4 * q + 1];
                s[4 * q + 2] = v.z + b[4 * q + 2];
                s[4 * q + 3] = v.w + b[4 * q + 3];
            }
            bool done = false;
            if (KT || K <= 8) done = route_fast<VPL, KT>(s, K, lane, sel);
            if (!done) route_exact<VPL, true>(rb, bias, E, K, lane, sel);
            const int id = (lane < K) ? sel[lane] : 0;
            const float wv = pick_weight((lane < K) ? rb[id] : 0.0f, K, lane, renorm);
            sink.put(t, K, lane, id, wv);
            __syncwarp();
        }
        cp_async_wait<0>();
    } else {
        for (int64_t t = t_begin; t < t_end; t += t_step) {
            const float* row = logits + t * E;
            route_exact<VPL, false>(row, bias, E, K, lane, sel);
            const int id = (lane < K) ? sel[lane] : 0;
            const float wv = pick_weight((lane < K) ? __ldg(row + id) : 0.0f, K, lane, renorm);
            sink.put(t, K, lane, id, wv);
            __syncwarp();
        }
    }
}

// ------------------------------------------------------------------------------------
// kb_router kernel: 8 warps per CTA, grid-stride over tokens, one token per warp at a time.
// ------------------------------------------------------------------------------------
template <int VPL, bool VEC, int KT, typename WT>
__global__ void __launch_bounds__(256) router_kernel(const float* __restrict__ logits,
                                                     const float* __restrict__ bias,
                                                     int32_t* __restrict__ ids,
                                                     WT* __restrict__ w, int64_t T, int E,
                                                     int K, int renorm) {
    pdl_wait();
    pdl_launch();
    extern __shared__ __align__(16) float rsmem[];
    __shared__ int sel_sm[8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float b[VPL];
    load_bias<VPL, VEC>(bias, E, lane, b);
    float* ring = VEC ? rsmem + (size_t)warp * 2 * E : nullptr;
    const int64_t first = (int64_t)blockIdx.x * 8 + warp;
    const int64_t step = (int64_t)gridDim.x * 8;
    const RouteSink<WT, false, false> sink{ids, w, nullptr, 0, nullptr};
    route_tokens<VPL, VEC, KT>(logits, bias, b, E, K, renorm, first, T, step, ring, sel_sm[warp],
                               sink);
}

// ------------------------------------------------------------------------------------
// Expert-map building blocks (block-wide; blockDim a multiple of 32).
// ------------------------------------------------------------------------------------

// Contiguous range of 32-wide selection chunks handled by this warp.
__device__ __forceinline__ void warp_ranges(int n, int& c0, int& c1) {
    const int nwarps = blockDim.x >> 5, warp = threadIdx.x >> 5;
    const int chunks = (n + 31) >> 5;
    const int per = (chunks + nwarps - 1) / nwarps;
    c0 = min(chunks, warp * per);
    c1 = min(chunks, c0 + per);
}

// Lanes of the warp holding the same expert as this lane (meaningful for valid lanes; e in
// [0, E_MAX)): one ballot per bit of e.  Nine ballots issue back to back; match.any on
// sm_100 has a dependent latency of about 380 cycles against about 25 for a ballot, and
// shared-memory atomics on random experts serialise (about 2 us for 2.6k selections a CTA).
__device__ __forceinline__ unsigned same_expert_lanes(int e, bool valid) {
    static_assert(E_MAX <= 512, "nine expert bits");
    unsigned m = __ballot_sync(FULL_MASK, valid);
#pragma unroll
    for (int b = 0; b < 9; ++b) {
        const bool bit = (e >> b) & 1;
        const unsigned vb = __ballot_sync(FULL_MASK, bit);
        m &= bit ? vb : ~vb;
    }
    return m;
}

// Per-warp histograms of sel[0..n) over each warp's chunk range.  whist: [nwarps][E].
// One shared-memory atomic per selection (cheaper on sm_100 than finding equal lanes).
template <typename SelT>
__device__ void count_per_warp(const SelT* sel, int n, int E, int* whist) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* h = whist + warp * E;
    for (int e = lane; e < E; e += 32) h[e] = 0;
    __syncwarp();
    int c0, c1;
    warp_ranges(n, c0, c1);
    const int end = min(n, c1 * 32);
    for (int i = c0 * 32 + lane; i < end; i += 32) {
        const int e = (int)sel[i];
        if (e >= 0 && e < E) atomicAdd(h + e, 1);
    }
    __syncwarp();
}

// whist[w][e] <- sum_{w'<w} whist[w'][e] (exclusive over warps); tot[e] <- column total.
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

// Exclusive block scan of tot[0..E) into offs[0..E], offs[E] = sum, for any blockDim (each
// thread scans a contiguous run of experts).  Needs __syncthreads before and after.
// scratch: >= 64 ints.
__device__ void scan_experts(const int* tot, int E, int* offs, int* scratch) {
    const int nthr = blockDim.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, nw = nthr >> 5;
    const int per = (E + nthr - 1) / nthr;
    const int e0 = min(E, tid * per), e1 = min(E, e0 + per);
    int sum = 0;
    for (int e = e0; e < e1; ++e) sum += tot[e];
    const int incl = warp_incl_scan(sum, lane);
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int s = (lane < nw) ? scratch[lane] : 0;
        s = warp_incl_scan(s, lane);
        if (lane < nw) scratch[32 + lane] = s;  // inclusive warp totals
    }
    __syncthreads();
    int run = incl - sum + ((warp > 0) ? scratch[32 + warp - 1] : 0);
    for (int e = e0; e < e1; ++e) {
        offs[e] = run;
        run += tot[e];
    }
    if (tid == 0) offs[E] = scratch[32 + nw - 1];
}

// Stable ranks and scatter.  whist[w][e] holds the first permuted row of warp w's
// selections of expert e (base already added).  Selection i of the block is token t0 + i/K,
// slot i%K.  A warp walks its chunks in order; inside a chunk, lanes of one expert rank by
// lane (same_expert_lanes), and the chunk's last lane of the expert advances the running row.
// The next chunk's expert lanes are computed before this chunk's shared-memory update, so
// the ballots overlap the update chain.
template <typename SelT>
__device__ void rank_scatter(const SelT* sel, int n, int64_t t0, int64_t T, int E, int K,
                             int* whist, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* h = whist + warp * E;
    const unsigned lt = (1u << lane) - 1u;
    int c0, c1;
    warp_ranges(n, c0, c1);
    if (c0 >= c1) return;
    int i = c0 * 32 + lane;
    int e = (i < n) ? (int)sel[i] : -1;
    bool valid = (e >= 0 && e < E);
    unsigned peers = same_expert_lanes(e, valid);
    for (int c = c0; c < c1; ++c) {
        const int i_n = i + 32;
        const int e_n = (c + 1 < c1 && i_n < n) ? (int)sel[i_n] : -1;
        const bool valid_n = (e_n >= 0 && e_n < E);
        const unsigned peers_n = same_expert_lanes(e_n, valid_n);
        const int leader = 31 - __clz(peers);
        const int base = valid ? h[e] : 0;
        __syncwarp();
        if (valid && lane == leader) h[e] = base + __popc(peers);
        __syncwarp();
        if (i < n) {
            const unsigned tl = (unsigned)i / (unsigned)K;
            const int slot = i - (int)tl * K;
            const int32_t u = (int32_t)((int64_t)slot * T + t0 + tl);
            if (valid) {
                const int rank = base + __popc(peers & lt);
                p2u[rank] = u;
                if (u2p) u2p[u] = rank;
            } else if (u2p) {
                u2p[u] = -1;
            }
        }
        i = i_n;
        e = e_n;
        valid = valid_n;
        peers = peers_n;
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
// smem: sel[T*K] | whist[32][E] | tot[E] | offs[E+1] | scratch[64] | ring[32][2][E] (VEC route)
// ------------------------------------------------------------------------------------
template <int VPL, bool VEC, bool ROUTE, int KT>
__global__ void __launch_bounds__(1024) maps_single_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias,
    const int32_t* __restrict__ ids_in, int32_t* __restrict__ ids_out, float* __restrict__ w,
    int64_t T, int E, int K, int renorm, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p,
    CountPush cp) {
    pdl_wait();
    pdl_launch();
    extern __shared__ __align__(16) int smem[];
    const int n = (int)(T * K);
    const int nwarps = blockDim.x >> 5;
    int* sel = smem;
    int* whist = sel + ((n + 3) & ~3);
    int* tot = whist + nwarps * E;
    int* offs = tot + E;
    int* scratch = offs + E + 1;
    float* ring = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(scratch + 64) + 15) & ~uintptr_t(15));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if constexpr (ROUTE) {
        __shared__ int sel_sm[32][32];
        float b[VPL];
        load_bias<VPL, VEC>(bias, E, lane, b);
        const RouteSink<float, true, false> sink{ids_out, w, sel, 0, nullptr};
        route_tokens<VPL, VEC, KT>(logits, bias, b, E, K, renorm, warp, T, nwarps,
                                   VEC ? ring + (size_t)warp * 2 * E : nullptr, sel_sm[warp],
                                   sink);
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) sel[i] = ids_in[i];
    }
    __syncthreads();
    count_per_warp(sel, n, E, whist);
    __syncthreads();
    scan_over_warps(E, whist, tot);
    __syncthreads();
    // Fused count all-gather (kb_router_maps_allgather): the totals go to every rank now, a
    // quarter of the CTA per destination, and the rows of the others are collected at the end.
    if (cp.world > 0) {
        const unsigned tag = count_push_tag(cp);
        const int per = blockDim.x / 4;
        for (int q = threadIdx.x / per; q < cp.world; q += 4)
            count_push_send(cp, tot, q, tag, threadIdx.x % per, per);
    }
    scan_experts(tot, E, offs, scratch);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int base = offs[e];
        for (int wv = 0; wv < nwarps; ++wv) whist[wv * E + e] += base;
    }
    write_offsets(offs, tot, E, n, counts, offsets, p2u);
    __syncthreads();
    rank_scatter(sel, n, 0, T, E, K, whist, p2u, u2p);
    if (cp.world > 0) count_push_gather(cp, count_push_tag(cp));
}

// ------------------------------------------------------------------------------------
// Persistent cooperative maps kernel (large T).
// ------------------------------------------------------------------------------------
__host__ __device__ constexpr size_t tile_align_c(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct PersistWs {
    unsigned* bar;   // arrival counter; 0 between calls (the last CTA out resets it)
    int* err;        // non-zero after a barrier wait gave up; the workspace must be re-zeroed
    int* rowhist;    // [grid][E] per-CTA histograms, CTA-major
    int* gsum;       // [ceil(grid/kGS)][E] histogram sums of kGS-CTA groups; zero between calls
    long long spin;  // poll limit of the bounded waits (kb_set_wait_limit)
    CountPush cp;    // tile kernel: the count all-gather fused into its tail (cp.world == 0: off)
};

constexpr int kPW = 8;                      // warps per persistent CTA
constexpr int kGS = 16;                     // CTAs per group of the two-level CTA prefix
constexpr long long kSpinLimit = 2000000;   // bounded barrier wait (about a second of polling)

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier over co-resident CTAs (cooperative launch).  Returns false if the wait gave
// up; the error flag is then set for the host and for later calls.
__device__ bool grid_barrier(const PersistWs& ws, unsigned target) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ws.bar, 1u);
        unsigned v = ld_acquire_gpu(ws.bar);
        long long it = 0;
        while (v < target && it < ws.spin) {
            __nanosleep(64);
            v = ld_acquire_gpu(ws.bar);
            ++it;
        }
        if (v < target) atomicExch(ws.err, 1);
        ok = (v >= target) && (*(volatile int*)ws.err == 0);
        __threadfence();
    }
    __syncthreads();
    return ok != 0;
}

// Maps phases of the persistent kernels, after this CTA's selections sel[0..n) (tokens
// t0..) are in shared memory.
//   before the barrier  stable ranks inside the CTA (per-warp histograms, exclusive over
//                       warps) and its histogram: published as row c of rowhist and added
//                       into the sum of its group of kGS CTAs
//   one grid barrier
//   after it            CTA base of expert e = sum of the groups before this CTA's group +
//                       the rows of the CTAs of its group before it (at most
//                       ceil(grid/kGS) + kGS - 1 independent L2 reads per expert); expert
//                       totals = sum of all groups; global offsets; scatter
// The last CTA out zeroes the group sums and resets the arrival counter.
template <typename SelT>
__device__ void maps_finish(const PersistWs& ws, int64_t T, int E, int K, int64_t t0, int n,
                            const SelT* sel, int* hist, int* totsm, int* offs, int* scratch, int* whist,
                            int32_t* counts, int64_t* offsets, int32_t* p2u, int32_t* u2p) {
    const int grid = gridDim.x, c = blockIdx.x;
    const int nwarps = blockDim.x >> 5;
    const int g = c / kGS, ng = (grid + kGS - 1) / kGS;
    __syncthreads();  // selections complete; the phase-1 buffers aliased by whist are free
    count_per_warp(sel, n, E, whist);
    __syncthreads();
    scan_over_warps(E, whist, hist);
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int v = hist[e];
        __stcg(ws.rowhist + (size_t)c * E + e, v);
        if (v) atomicAdd(ws.gsum + (size_t)g * E + e, v);
    }
    if (!grid_barrier(ws, (unsigned)grid)) return;
    pdl_launch();

    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int before = 0, total = 0;
        for (int q = 0; q < ng; ++q) {
            const int v = __ldcg(ws.gsum + (size_t)q * E + e);
            total += v;
            before += (q < g) ? v : 0;
        }
        for (int cc = g * kGS; cc < c; ++cc) before += __ldcg(ws.rowhist + (size_t)cc * E + e);
        hist[e] = before;
        totsm[e] = total;
    }
    __syncthreads();
    scan_experts(totsm, E, offs, scratch);
    __syncthreads();
    if (c == 0) write_offsets(offs, totsm, E, T * K, counts, offsets, p2u);
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int base = offs[e] + hist[e];
        for (int wv = 0; wv < nwarps; ++wv) whist[wv * E + e] += base;
    }
    __syncthreads();
    rank_scatter(sel, n, t0, T, E, K, whist, p2u, u2p);

    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = (atomicAdd(ws.bar, 1u) == 2u * (unsigned)grid - 1u);
    }
    __syncthreads();
    if (last) {
        for (int i = threadIdx.x; i < ng * E; i += blockDim.x) ws.gsum[i] = 0;
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            atomicExch(ws.bar, 0u);
        }
    }
}

// Split grid barrier: arrive once this CTA's stores are issued, do local work, then wait.
__device__ __forceinline__ void grid_arrive(const PersistWs& ws) {
    __syncthreads();
    if (threadIdx.x == 0)   // release: the CTA's writes (ordered before by the barrier) first
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ws.bar) : "memory");
}
__device__ bool grid_wait(const PersistWs& ws, unsigned target) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        unsigned v = ld_acquire_gpu(ws.bar);
        long long it = 0;
        while (v < target && it < ws.spin) {
            __nanosleep(32);
            v = ld_acquire_gpu(ws.bar);
            ++it;
        }
        if (v < target) atomicExch(ws.err, 1);
        ok = (v >= target) && (*(volatile int*)ws.err == 0);
        __threadfence();
    }
    __syncthreads();
    return ok != 0;
}

// Shared-memory ints the tile kernel's map phases need beyond the selections: whist, local
// offsets, prefix partial sums, and (staged) the token masks and prefixes of the CTA's 32-token
// tiles.
__host__ __device__ constexpr size_t tile_maps_ints(int nthreads, int E, int n, int K, bool staged) {
    return (size_t)(nthreads / 32) * E + tile_align_c(E + 1, 4) +
           (size_t)2 * (nthreads / (E / 4)) * E +
           (staged ? (size_t)2 * ((n / (K > 0 ? K : 1) + 31) / 32) * E : 0);
}

// Token masks of the CTA's 32-token tiles: mask[tile][e] bit l is set when token l of the tile
// selected expert e.  A warp takes tiles w, w + nwarps, ...; lane l ORs its bit into the
// word of each of its token's experts (shared-memory atomics, all K issued back to back; OR
// is order-free, so the masks do not depend on timing).  A token's experts are distinct, so
// every bit is set once.  mask: [ntiles][E], zero on entry.  (One match.any per slot, the
// earlier form, cost ~380 cycles each and 4.6 us of the kernel's tail at T = 65536.)
__device__ void build_tile_masks(const uint16_t* sel, int ntok, int K, int E, unsigned* mask) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int ntiles = (ntok + 31) >> 5;
    for (int tile = warp; tile < ntiles; tile += nw) {
        const int tok = tile * 32 + lane;
        if (tok >= ntok) continue;
        unsigned* m = mask + (size_t)tile * E;
        for (int k = 0; k < K; ++k) {
            const int e = (int)sel[tok * K + k];
            if (e < E) atomicOr(m + e, 1u << lane);
        }
    }
}

// Per expert e: tbase[tile][e] = selections of e in the tiles before `tile`; returns the
// CTA total of e (thread e, e + blockDim, ...).
__device__ void tile_prefix(const unsigned* __restrict__ mask, int ntiles, int E,
                            unsigned* __restrict__ tbase, int* __restrict__ hist) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        unsigned run = 0;
        int t = 0;
        for (; t + 4 <= ntiles; t += 4) {   // four tiles' masks loaded before they are summed
            unsigned m[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) m[u] = mask[(size_t)(t + u) * E + e];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                tbase[(size_t)(t + u) * E + e] = run;
                run += (unsigned)__popc(m[u]);
            }
        }
        for (; t < ntiles; ++t) {
            const unsigned m = mask[(size_t)t * E + e];
            tbase[(size_t)t * E + e] = run;
            run += (unsigned)__popc(m);
        }
        hist[e] = (int)run;
    }
}

// Maps phases of the tile kernel (E % 4 == 0, blockDim >= E/4), after the CTA's selections
// sel[0..n) (16-bit experts, tokens t0..) are in shared memory.  free_sm: the ring, free now.
// As maps_finish, with:
//   tile masks     (staged) per 32-token tile and expert, the mask of tokens that selected it
//                  (build_tile_masks: one match.any per slot per tile, no shared-memory
//                  atomics and no per-selection warp votes, which serialise on this GPU), and
//                  per expert the counts of the earlier tiles (tile_prefix), which give the
//                  CTA histogram
//   arrive early   the CTA histogram (counted as the selections were made) is published and
//                  the grid barrier entered before the masks are built
//   prefix         every thread issues its 128-bit loads of group sums and earlier rows of
//                  its group before summing; partial sums meet in shared memory
//   writes         each selection's row from the masks (expert offset + earlier CTAs + the
//                  tile bases + the tile's earlier tokens), in slot-major order so that u2p is
//                  written coalesced.  Without room for the masks, or with a token that names
//                  an expert twice: per-warp counts and rank_scatter.
template <int E>
__device__ void maps_finish_tile(const PersistWs& ws, int64_t T, int K, int64_t t0, int n,
                                 const uint16_t* sel, int* hist, int* totsm, int* offs,
                                 int* scratch, int* free_sm, bool staged, bool hist_ready,
                                 int32_t* counts, int64_t* offsets, int32_t* p2u, int32_t* u2p) {
    static_assert(E % 4 == 0, "int4 rows");
    constexpr int Q4 = E / 4;
    const int grid = gridDim.x, c = blockIdx.x, nthr = blockDim.x, tid = threadIdx.x;
    const int nwarps = nthr >> 5;
    const int g = c / kGS, ng = (grid + kGS - 1) / kGS;
    const int R = nthr / Q4;
    int* whist = free_sm;
    int* loc = whist + nwarps * E;
    int* part_b = loc + tile_align_c(E + 1, 4);
    int* part_t = part_b + R * E;

    // Tile masks (staged path): [ntiles][E] masks and tile prefixes after the staging arrays.
    const int ntok = n / K, ntiles = (ntok + 31) >> 5;
    unsigned* tmask = reinterpret_cast<unsigned*>(part_t + R * E);
    unsigned* tbase = tmask + (size_t)ntiles * E;
    __syncthreads();  // selections complete; the ring is free
    // Publish the CTA histogram (row of rowhist, group sum) and enter the grid barrier.
    // Atomics reach L2 at once, so the release of grid_arrive does not wait behind stores
    // that are still buffered.
    auto publish_and_arrive = [&]() {
        for (int e = tid; e < E; e += nthr) {
            const int v = hist[e];
            atomicExch(ws.rowhist + (size_t)c * E + e, v);
            if (v) atomicAdd(ws.gsum + (size_t)g * E + e, v);
        }
        grid_arrive(ws);
    };
    // hist_ready: the histogram was counted while the selections were made, so it is published
    // at once and the masks and the CTA-local placement below overlap the other CTAs' arrival.
    if (hist_ready) publish_and_arrive();
    if (staged) {
        for (int i = tid; i < ntiles * E; i += nthr) tmask[i] = 0u;
        __syncthreads();
        build_tile_masks(sel, ntok, K, E, tmask);
        __syncthreads();
        tile_prefix(tmask, ntiles, E, tbase, hist);  // hist = CTA histogram
    } else {
        count_per_warp(sel, n, E, whist);
        __syncthreads();
        scan_over_warps(E, whist, hist);  // hist = CTA histogram, whist exclusive over warps
    }
    if (!hist_ready) publish_and_arrive();
    // While the other CTAs arrive: CTA-local expert offsets, CTA-sorted positions.
    // (staged: every selection's row is computed after the barrier from the masks, so no
    // CTA-local placement here)
    if (!staged) {
        scan_experts(hist, E, loc, scratch);  // barriers inside
        __syncthreads();
        for (int e = tid; e < E; e += nthr) {
            const int l = loc[e];
            for (int wv = 0; wv < nwarps; ++wv) whist[wv * E + e] += l;
        }
    }
    if (!grid_wait(ws, (unsigned)grid)) return;
    pdl_launch();

    // Rows before this CTA: group sums 0..g-1 and rows g*kGS..c-1; totals: all group sums.
    const int nrows = ng + (c - g * kGS);
    if (tid < R * Q4) {
        const int qd = tid % Q4, r0 = tid / Q4;
        const int4* gs4 = reinterpret_cast<const int4*>(ws.gsum);
        const int4* rh4 = reinterpret_cast<const int4*>(ws.rowhist + (size_t)g * kGS * E);
        int4 bs = make_int4(0, 0, 0, 0), ts = make_int4(0, 0, 0, 0);
        for (int rb = r0; rb < nrows; rb += 10 * R) {   // kGS + ceil(148/kGS) rows: one round
            int4 v[10];
#pragma unroll
            for (int u = 0; u < 10; ++u) {
                const int r = rb + u * R;
                v[u] = make_int4(0, 0, 0, 0);
                if (r < nrows)
                    v[u] = __ldcg(r < ng ? gs4 + (size_t)r * Q4 + qd : rh4 + (size_t)(r - ng) * Q4 + qd);
            }
#pragma unroll
            for (int u = 0; u < 10; ++u) {
                const int r = rb + u * R;
                const bool tot = r < ng, bef = (r < g) || (r >= ng);
                if (tot) { ts.x += v[u].x; ts.y += v[u].y; ts.z += v[u].z; ts.w += v[u].w; }
                if (bef) { bs.x += v[u].x; bs.y += v[u].y; bs.z += v[u].z; bs.w += v[u].w; }
            }
        }
        reinterpret_cast<int4*>(part_b)[r0 * Q4 + qd] = bs;
        reinterpret_cast<int4*>(part_t)[r0 * Q4 + qd] = ts;
    }
    __syncthreads();
    for (int e = tid; e < E; e += nthr) {
        int b = 0, t = 0;
        for (int r = 0; r < R; ++r) {
            b += part_b[r * E + e];
            t += part_t[r * E + e];
        }
        hist[e] = b;
        totsm[e] = t;
    }
    __syncthreads();
    scan_experts(totsm, E, offs, scratch);
    __syncthreads();
    if (c == 0) write_offsets(offs, totsm, E, T * K, counts, offsets, p2u);
    // Fused count all-gather: CTA q < N stores this rank's totals into rank q's buffer now,
    // so the transfer overlaps the placement below; the last CTA out collects every rank's.
    if (c < ws.cp.world) count_push_send(ws.cp, totsm, c, count_push_tag(ws.cp), tid, nthr);
    if (staged) {
        // Row of selection (token tl, slot sl) of expert e: the expert's global offset + its
        // selections in earlier CTAs (hist[e], from the prefix above) + those in this CTA's
        // earlier tiles (tbase) + this tile's earlier tokens with e (popcount of the mask below
        // the token's bit).  Slot-major order: u2p is written coalesced; ids outside [0, E)
        // get u2p = -1.
        for (int e = tid; e < E; e += nthr) hist[e] = offs[e] + hist[e];
        __syncthreads();
        const uint16_t* __restrict__ se = sel;
        const int* __restrict__ hb = hist;
        const unsigned* __restrict__ tb = tbase;
        const unsigned* __restrict__ tm = tmask;
#pragma unroll 4
        for (int j = tid; j < n; j += nthr) {
            const int sl = j / ntok, tl = j - sl * ntok;
            const int e = (int)se[tl * K + sl];
            int r = -1;
            if (e < E) {
                const size_t te = (size_t)(tl >> 5) * E + e;
                r = hb[e] + (int)tb[te] + __popc(tm[te] & ((1u << (tl & 31)) - 1u));
                p2u[r] = (int32_t)((int64_t)sl * T + t0 + tl);
            }
            if (u2p) u2p[(int64_t)sl * T + t0 + tl] = r;
        }
    } else {
        // Global row of CTA-sorted position lpos of expert e = offs[e] + hist[e] + lpos - loc[e].
        for (int e = tid; e < E; e += nthr) hist[e] = offs[e] + hist[e] - loc[e];
        __syncthreads();
        for (int e = tid; e < E; e += nthr) {
            const int d = hist[e];
            for (int wv = 0; wv < nwarps; ++wv) whist[wv * E + e] += d;
        }
        __syncthreads();
        rank_scatter(sel, n, t0, T, E, K, whist, p2u, u2p);
    }

    // Every CTA has used the group sums it loaded before it counts itself out here; kernel
    // completion makes the last CTA's reset visible to the next call.
    __shared__ int last;
    __syncthreads();
    if (tid == 0) last = (atomicAdd(ws.bar, 1u) == 2u * (unsigned)grid - 1u);
    __syncthreads();
    if (last) {
        for (int i = tid; i < ng * E; i += nthr) ws.gsum[i] = 0;
        if (tid == 0) atomicExch(ws.bar, 0u);
        if (ws.cp.world > 0) count_push_gather(ws.cp, count_push_tag(ws.cp));
    }
}

// A workspace whose earlier barrier gave up stays poisoned until re-zeroed: report it
// through offsets (all -1) and do nothing else.
__device__ __forceinline__ bool ws_poisoned(const PersistWs& ws, int E, int64_t* offsets) {
    if (*(volatile int*)ws.err == 0) return false;
    if (blockIdx.x == 0)
        for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = -1;
    return true;
}

// Warp-per-token persistent kernel (any E <= 512, any K <= 32; also the ids-only maps).
// smem: sel[tpc*K] | hist[E] | totsm[E] | offs[E+1] | scratch[64] | ring (phase 1) = whist (phase 3)
template <int VPL, bool VEC, bool ROUTE, int KT>
__global__ void __launch_bounds__(kPW * 32) maps_persistent_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias,
    const int32_t* __restrict__ ids_in, int32_t* __restrict__ ids_out, float* __restrict__ w,
    int64_t T, int E, int K, int renorm, int tpc, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p,
    PersistWs ws) {
    pdl_wait();
    extern __shared__ __align__(16) int smem[];
    const int c = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int selcap = (tpc * K + 3) & ~3;
    int* sel = smem;
    int* hist = sel + selcap;
    int* totsm = hist + E;
    int* offs = totsm + E;
    int* scratch = offs + ((E + 1 + 3) & ~3);
    float* ring = reinterpret_cast<float*>(scratch + 64);  // phase 1
    int* whist = scratch + 64;                             // phase 3 (aliases the ring)
    if (ws_poisoned(ws, E, offsets)) return;
    const int64_t t0 = (int64_t)c * tpc;
    const int64_t t1 = min(T, t0 + tpc);
    const int n = (t1 > t0) ? (int)((t1 - t0) * K) : 0;

    // Phase 1: route (or load ids) this CTA's tokens into sel.
    if constexpr (ROUTE) {
        __shared__ int sel_sm[kPW][32];
        float b[VPL];
        load_bias<VPL, VEC>(bias, E, lane, b);
        const RouteSink<float, true, false> sink{ids_out, w, sel, t0, nullptr};
        route_tokens<VPL, VEC, KT>(logits, bias, b, E, K, renorm, t0 + warp, t1, kPW,
                                   VEC ? ring + (size_t)warp * 2 * E : nullptr, sel_sm[warp],
                                   sink);
    } else {
        const int32_t* src = ids_in + t0 * K;
        for (int i = threadIdx.x; i < n; i += blockDim.x) sel[i] = __ldg(src + i);
    }
    maps_finish(ws, T, E, K, t0, n, sel, hist, totsm, offs, scratch, whist, counts, offsets, p2u,
                u2p);
}

// Maps from ids for E in {128, 256, 384} (kb_expert_maps at T > 768): the map phases of the
// tile kernel (maps_finish_tile: token masks per 32-token tile, the histogram published and the
// grid barrier entered before the CTA-local placement, staged coalesced writes) on the CTA's
// ids, loaded as 16-bit experts (ids outside [0, E) become 0xFFFF and are skipped).  One
// cooperative launch, one CTA of 256 threads per SM.
// smem: sel (u16)[tpc*K, padded to 8] | hist[E] | totsm[E] | offs[E+1, padded to 4]
//       | scratch[64] | the map phases' arrays (tile_maps_ints, staged)
template <int E_>
__global__ void __launch_bounds__(256) maps_ids_tile_kernel(
    const int32_t* __restrict__ ids_in, int64_t T, int K, int tpc, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p,
    PersistWs ws) {
    pdl_wait();
    extern __shared__ __align__(16) int ism[];
    const int selw = (int)(tile_align_c((size_t)tpc * K, 8) / 2);
    uint16_t* sel = reinterpret_cast<uint16_t*>(ism);
    int* hist = ism + selw;
    int* totsm = hist + E_;
    int* offs = totsm + E_;
    int* scratch = offs + tile_align_c(E_ + 1, 4);
    int* free_sm = scratch + 64;
    if (ws_poisoned(ws, E_, offsets)) return;
    const int c = blockIdx.x;
    const int64_t t0 = (int64_t)c * tpc;
    const int64_t t1 = min(T, t0 + tpc);
    const int n = (t1 > t0) ? (int)((t1 - t0) * K) : 0;
    for (int e = threadIdx.x; e < E_; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int32_t* src = ids_in + t0 * K;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = __ldg(src + i);
        const bool ok = e >= 0 && e < E_;
        sel[i] = ok ? (uint16_t)e : (uint16_t)0xFFFFu;
        if (ok) atomicAdd(&hist[e], 1);   // the CTA histogram, published before the masks
    }
    __syncthreads();
    // The token masks count tokens, so they need a token's experts to be distinct (as a
    // router's are).  A CTA holding a token that names one expert twice places its selections
    // with the per-warp counts instead (maps_finish_tile's unstaged placement).
    bool dup = false;
    const int ntok = n / K;
    for (int tk = threadIdx.x; tk < ntok; tk += blockDim.x) {
        const uint16_t* r = sel + tk * K;
        for (int a = 1; a < K; ++a)
            for (int b = 0; b < a; ++b) dup |= (r[a] == r[b]) && (r[a] != 0xFFFFu);
    }
    const bool staged = __syncthreads_or(dup) == 0;
    maps_finish_tile<E_>(ws, T, K, t0, n, sel, hist, totsm, offs, scratch, free_sm, staged, true,
                         counts, offsets, p2u, u2p);
}

// Hybrid-router persistent kernel (see trouter.cuh).
// smem: bias[E] | wsm[nw][hwarp] (phase 1) = whist[nw][E] (phase 3) | sel_tmp[nw][32]
//       | sel[tpc*K] | hist[E] | totsm[E] | offs[E+1] | scratch[64]
template <int E_, int KT>
__global__ void __launch_bounds__(256) maps_tpersist_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int32_t* __restrict__ ids_out,
    float* __restrict__ w, int64_t T, int K, int renorm, int tpc, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p,
    PersistWs ws) {
    pdl_wait();
    extern __shared__ __align__(16) float tsm[];
    constexpr size_t HW = hwarp_smem_floats<E_>();
    const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* bias_sm = tsm;
    float* wsm = bias_sm + E_;
    int* whist = reinterpret_cast<int*>(wsm);
    int* sel_tmp = reinterpret_cast<int*>(wsm + nw * HW);
    int* sel = sel_tmp + nw * 32;
    const int selcap = (tpc * K + 3) & ~3;
    int* hist = sel + selcap;
    int* totsm = hist + E_;
    int* offs = totsm + E_;
    int* scratch = offs + ((E_ + 1 + 3) & ~3);
    if (ws_poisoned(ws, E_, offsets)) return;
    const int c = blockIdx.x;
    const int64_t t0 = (int64_t)c * tpc;
    const int64_t t1 = min(T, t0 + tpc);
    const int n = (t1 > t0) ? (int)((t1 - t0) * K) : 0;
    troute_setup<E_>(bias, bias_sm);
    float b[E_ / 32];
    load_bias<E_ / 32, true>(bias, E_, lane, b);

    // Phase 1: this warp's contiguous share of the CTA's tokens.
    const int64_t tpw = (t1 - t0 + nw - 1) / nw;
    const int64_t tb0 = t0 + warp * tpw;
    const int64_t te = min(t1, tb0 + tpw);
    troute_range<E_, KT, true, false, float>(logits, b, bias_sm, K, renorm, tb0, te,
                                             wsm + warp * HW, sel_tmp + warp * 32, ids_out, w,
                                             sel, t0, nullptr);
    maps_finish(ws, T, E_, K, t0, n, sel, hist, totsm, offs, scratch, whist, counts, offsets, p2u,
                u2p);
}

// ------------------------------------------------------------------------------------
// mbarrier helpers of the tile kernel (bounded waits).
// ------------------------------------------------------------------------------------
constexpr long long kMbarSpin = 1LL << 20;

__device__ __forceinline__ unsigned smem_u32(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Waits for the phase of parity `parity` to complete; false (and the error word set) if it
// did not within `limit` polls (kMbarSpin when limit <= 0), or as soon as another wait gave
// up.  err may be null (the router-only launches have no workspace): nothing is read or set.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, int* err,
                                          long long limit = kMbarSpin) {
    const unsigned a = smem_u32(bar);
    if (limit <= 0) limit = kMbarSpin;
    for (long long it = 0; it < limit; ++it) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
        if ((it & 255) == 255 && err && *(volatile int*)err) return false;
        __nanosleep(40);  // a waiting warp leaves the issue slots to the working ones
    }
    if (err) atomicExch(err, 1);
    return false;
}
// The drain after a wait gave up: waits for a copy this CTA issued to land whatever the error
// word says (a CTA must not leave with a copy still writing its shared memory); bounded.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, unsigned parity) {
    const unsigned a = smem_u32(bar);
    for (long long it = 0; it < kMbarSpin; ++it) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return;
        __nanosleep(40);
    }
}
// ------------------------------------------------------------------------------------
// Tile maps kernel (routing, E = 32*VPL in {128, 256, 384}, K <= 8): one CTA per SM.
//
// Warp 0 streams the CTA's tokens in tiles of kTileRows = 32 rows through an nslot-deep
// ring: one 2-D tensor copy per 32-column box (E/32 boxes per tile), with the 128-byte
// swizzle, so that 32 lanes each reading their own row hit 8 distinct 16-byte bank groups
// per quarter-warp (conflict-free lane-per-row float4 reads).  Consumer pair p (warps 1+2p
// and 2+2p) owns slot p and routes tiles p, p + nslot, ...; lane l ranks token l of the tile:
//   stage 1     warp h of the pair takes the 16-expert groups [h*G/2, (h+1)*G/2) of its
//               row: group maxima of s = x + b (NaN-propagating), into gm
//   tau         both warps read all G maxima: tau = K-th largest, a lower bound of the K-th
//               largest score (the top-K groups each hold an element >= tau)
//   candidates  the qualifying groups (maximum >= tau) alternate between the two warps in
//               index order; elements >= tau enter a register top-K in ascending index
//               order, so a strict key comparison keeps the lower index first
//   merge       warp 1 hands its list to warp 0 through shared memory; warp 0 merges it
//               (key, then lower index), releases the slot, weighs sigmoid(raw logit) and
//               writes the tile's ids and weights as whole lines
// Rows holding a NaN take the exact warp-cooperative path on the global row.  Then the maps
// phases (maps_finish) with the CTA's selections as 16-bit expert ids.
// smem (base rounded up to 1024 bytes):
//   ring[nslot][E/32 boxes][32 rows][32] | gm[nslot][32][G+1] | xk[nslot][KM][32]
//   | xi[nslot][KM][32] | bias[E] | sel_tmp[nslot][32] | sel (u16)[tpc*K, padded to 8]
//   | hist[E] | totsm[E] | offs[E+1, padded to 4] | scratch[64] | full[nslot], empty[nslot]
// whist (maps phases) aliases the ring.
// ------------------------------------------------------------------------------------
constexpr int kTileRows = 32;
constexpr int kTileMaxSlots = 6;
constexpr int kTileMaxThreads = 32 * (1 + 2 * kTileMaxSlots);

template <int E_, int KT>
struct TileCfg {
    static constexpr int G = E_ / 16;                 // 16-expert groups
    static constexpr int H = G / 2;                   // groups per warp of a pair
    static constexpr int GP = G + 1;                  // gm row stride (odd)
    static constexpr int BOXES = E_ / 32;             // 32-column boxes per tile
    static constexpr int BOX_FLOATS = kTileRows * 32;
    static constexpr int SLOT_FLOATS = kTileRows * E_;
    static constexpr int KM = TCfg<E_, KT>::KM;       // register top-K capacity
    static_assert(E_ % 32 == 0 && G % 2 == 0, "tile shape");
};

__host__ __device__ constexpr size_t tile_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Byte sizes of the tile kernel's shared-memory regions (before the 1024-byte alignment slack).
template <int E_, int KT>
__host__ __device__ constexpr size_t tile_smem_bytes(int nslot, int tpc, int K) {
    using C = TileCfg<E_, KT>;
    return (size_t)nslot * C::SLOT_FLOATS * 4 + (size_t)nslot * 32 * C::GP * 4 +
           (size_t)2 * nslot * C::KM * 32 * 4 + (size_t)E_ * 4 + (size_t)nslot * 32 * 4 +
           tile_align((size_t)tpc * K, 8) * 2 +
           ((size_t)2 * E_ + tile_align(E_ + 1, 4) + 64) * 4 + (size_t)2 * nslot * 8;
}

// Float offset of (row r, column col) in a tile slot: box col/32, 128-byte swizzle (the
// 16-byte chunk index within a 128-byte row is XORed with r mod 8).
__device__ __forceinline__ int tile_off(int r, int col) {
    return (col >> 5) * (kTileRows * 32) + r * 32 + ((((col >> 2) & 7) ^ (r & 7)) << 2) + (col & 3);
}

__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
    float r;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// One 2-D tensor copy (box at column x, row y) into this CTA's shared memory, completing on bar.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
          "r"(smem_u32(bar)) : "memory");
}

// Barrier over the two warps of consumer pair p (named barrier 1 + p).
__device__ __forceinline__ void pair_sync(int p) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + p) : "memory");
}
static_assert(kTileMaxSlots < 15, "named barriers 1..kTileMaxSlots must exist");
constexpr int kTileSetupBar = 15;  // the tile kernel's set-up barrier (the pairs use 1..nslot)

// Insert (kk, jj) into a top-KM list sorted by key descending; candidates arrive in ascending
// index order, so a strict comparison keeps the earlier (lower) index first among equal keys.
// The comparisons are independent: positions at and after the first smaller key shift down.
template <int KM>
__device__ __forceinline__ void topk_insert(uint32_t (&key)[KM], int (&idx)[KM], uint32_t kk,
                                            int jj) {
    bool gt[KM];
#pragma unroll
    for (int i = 0; i < KM; ++i) gt[i] = kk > key[i];
#pragma unroll
    for (int i = KM - 1; i > 0; --i) {
        key[i] = gt[i] ? (gt[i - 1] ? key[i - 1] : kk) : key[i];
        idx[i] = gt[i] ? (gt[i - 1] ? idx[i - 1] : jj) : idx[i];
    }
    key[0] = gt[0] ? kk : key[0];
    idx[0] = gt[0] ? jj : idx[0];
}

// As topk_insert for an entry of any index: ties go to the lower index.
template <int KM>
__device__ __forceinline__ void topk_merge(uint32_t (&key)[KM], int (&idx)[KM], uint32_t kk,
                                           int jj) {
    bool gt[KM];
#pragma unroll
    for (int i = 0; i < KM; ++i) gt[i] = kk > key[i] || (kk == key[i] && jj < idx[i]);
#pragma unroll
    for (int i = KM - 1; i > 0; --i) {
        key[i] = gt[i] ? (gt[i - 1] ? key[i - 1] : kk) : key[i];
        idx[i] = gt[i] ? (gt[i - 1] ? idx[i - 1] : jj) : idx[i];
    }
    key[0] = gt[0] ? kk : key[0];
    idx[0] = gt[0] ? jj : idx[0];
}

// MAPS = false: the router alone (kb_router), a plain launch: no selections, no map phases;
// WT: the weights' type (fp32 with the maps; fp32, bf16 or fp16 for the router alone).
template <int E_, int KT, bool MAPS = true, typename WT = float>
__global__ void __launch_bounds__(kTileMaxThreads, 1) maps_tile_kernel(
    const __grid_constant__ CUtensorMap tmap, const float* __restrict__ logits,
    const float* __restrict__ bias, int32_t* __restrict__ ids_out, WT* __restrict__ w,
    int64_t T, int K_rt, int renorm, int tpc, int nslot, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p,
    PersistWs ws) {
    using C = TileCfg<E_, KT>;
    constexpr int G = C::G, H = C::H, GP = C::GP, KM = C::KM;
    const int K = KT ? KT : K_rt;
    pdl_wait();
    extern __shared__ __align__(16) unsigned char tile_raw[];
    unsigned char* base = tile_raw + ((1024u - (smem_u32(tile_raw) & 1023u)) & 1023u);
    float* ring = reinterpret_cast<float*>(base);
    float* gm = ring + (size_t)nslot * C::SLOT_FLOATS;
    uint32_t* xk = reinterpret_cast<uint32_t*>(gm + (size_t)nslot * 32 * GP);
    int* xi = reinterpret_cast<int*>(xk + (size_t)nslot * KM * 32);
    float* bias_sm = reinterpret_cast<float*>(xi + (size_t)nslot * KM * 32);
    int* sel_tmp = reinterpret_cast<int*>(bias_sm + E_);
    uint16_t* sel = reinterpret_cast<uint16_t*>(sel_tmp + nslot * 32);
    int* hist = reinterpret_cast<int*>(sel + tile_align((size_t)tpc * K, 8));
    int* totsm = hist + E_;
    int* offs = totsm + E_;
    int* scratch = offs + tile_align(E_ + 1, 4);
    uint64_t* full = reinterpret_cast<uint64_t*>(scratch + 64);
    uint64_t* empty = full + nslot;
    int* whist = reinterpret_cast<int*>(ring);
    if constexpr (MAPS) {
        if (ws_poisoned(ws, E_, offsets)) return;
    } else {
        pdl_launch();
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const int64_t t0 = (int64_t)c * tpc;
    const int64_t t1 = min(T, t0 + tpc);
    const int n = (t1 > t0) ? (int)((t1 - t0) * K) : 0;
    const int nbat = (t1 > t0) ? (int)((t1 - t0 + kTileRows - 1) / kTileRows) : 0;
    // Set-up: the producer warp initialises the mbarriers and only arrives on the set-up
    // barrier (named barrier kTileSetupBar), so its first copies are issued while the other
    // warps zero the CTA histogram and load the bias; they wait on the barrier, which also
    // publishes the mbarriers' initialisation to them.
    if (warp == 0) {
        if (lane == 0) {
            for (int st = 0; st < nslot; ++st) {
                mbar_init(full + st, 1);
                mbar_init(empty + st, 2);
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncwarp();
        asm volatile("bar.arrive %0, %1;" ::"r"(kTileSetupBar), "r"((int)blockDim.x) : "memory");
    } else {
        const int nt = blockDim.x - 32, t = threadIdx.x - 32;
        for (int e = t; e < E_; e += nt) {
            bias_sm[e] = bias ? __ldg(bias + e) + 0.0f : 0.0f;
            if constexpr (MAPS) hist[e] = 0;   // counted as the selections are made
        }
        asm volatile("bar.sync %0, %1;" ::"r"(kTileSetupBar), "r"((int)blockDim.x) : "memory");
    }

    if (warp == 0) {
        // Producer: every tile of this CTA in order; lane 0 waits for the slot, posts the
        // byte count of the whole tile (rows past T are zero-filled and still counted) and
        // issues one tensor copy per box.
        bool ok = true;
        int issued = 0;
        for (int bi = 0; bi < nbat && ok; ++bi) {
            const int st = bi % nslot, k = bi / nslot;
            if (lane == 0 && k > 0) ok = mbar_wait(empty + st, (unsigned)((k - 1) & 1), ws.err, ws.spin);
            ok = __shfl_sync(FULL_MASK, ok, 0);
            if (!ok) break;
            const int y = (int)(t0 + (int64_t)bi * kTileRows);
            if (lane == 0) {
                mbar_expect_tx(full + st, (unsigned)(C::SLOT_FLOATS * sizeof(float)));
                float* dst = ring + (size_t)st * C::SLOT_FLOATS;
#pragma unroll 1
                for (int bx = 0; bx < C::BOXES; ++bx)
                    tma_load_2d(dst + bx * C::BOX_FLOATS, &tmap, 32 * bx, y, full + st);
            }
            issued = bi + 1;
        }
        // Drain: no copy may still be writing when the CTA moves on, also when a consumer gave
        // up on a tile (the last phase of each slot is complete or current, so its parity
        // waits only for a copy still in flight).
        if (lane == 0) {
            for (int bi = max(0, issued - nslot); bi < issued; ++bi)
                mbar_drain(full + bi % nslot, (unsigned)((bi / nslot) & 1));
        }
        __syncwarp();
    } else if (warp <= 2 * nslot) {
        const int p = (warp - 1) >> 1, h = (warp - 1) & 1;
        const float* slot = ring + (size_t)p * C::SLOT_FLOATS;
        float* gms = gm + (size_t)p * 32 * GP;
        uint32_t* xks = xk + (size_t)p * KM * 32;
        int* xis = xi + (size_t)p * KM * 32;
        const float4* bias4 = reinterpret_cast<const float4*>(bias_sm);
        const int sw = lane & 7;
        const float* myrow = slot + lane * 32;  // this lane's row inside box 0
        __shared__ int pair_ok[kTileMaxSlots];
        for (int bi = p; bi < nbat; bi += nslot) {
            const unsigned par = (unsigned)((bi / nslot) & 1);
            // The pair's first warp decides whether the tile arrived (bounded wait); the
            // decision reaches the second through the pair barrier, so both take one branch.
            if (h == 0) {
                const bool ok = mbar_wait(full + p, par, ws.err, ws.spin);
                if (lane == 0) pair_ok[p] = ok ? 1 : 0;
            }
            pair_sync(p);
            if (!pair_ok[p]) break;
            if (h == 1) mbar_wait(full + p, par, ws.err);  // completed: returns at once
            const int64_t tb = t0 + (int64_t)bi * kTileRows;
            const int rows = (int)min((int64_t)kTileRows, t1 - tb);
            const bool valid = lane < rows;

            // ---- stage 1: maxima of this warp's groups of the lane's row ----
#pragma unroll
            for (int gg = 0; gg < H; ++gg) {
                const int g = h * H + gg;
                const float* rp = myrow + (g >> 1) * C::BOX_FLOATS;
                const int j0 = (g & 1) * 4;
                float m[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 x = *reinterpret_cast<const float4*>(rp + (((j0 + q) ^ sw) << 2));
                    const float4 b = bias4[4 * g + q];
                    m[q] = fmax3_nan(x.x + b.x, x.y + b.y, fmax_nan(x.z + b.z, x.w + b.w));
                }
                gms[lane * GP + g] = fmax3_nan(m[0], m[1], fmax_nan(m[2], m[3]));
            }
            pair_sync(p);

            // ---- tau: K-th largest group maximum (both warps, all groups) ----
            float gmax[G];
#pragma unroll
            for (int g = 0; g < G; ++g) gmax[g] = gms[lane * GP + g];
            bool nan_row = false;
            float tk[KM];
#pragma unroll
            for (int i = 0; i < KM; ++i) tk[i] = -INFINITY;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float v = gmax[g];
                nan_row |= (v != v);
#pragma unroll
                for (int i = 0; i < KM; ++i) {
                    const float hi = fmaxf(tk[i], v);
                    v = fminf(tk[i], v);
                    tk[i] = hi;
                }
            }
            float tau = tk[0];
#pragma unroll
            for (int i = 1; i < KM; ++i)
                if (i == K - 1) tau = tk[i];
            // Qualifying groups in index order alternate between the pair's warps (warp h
            // takes the (h+1)-th, (h+3)-th, ...), which splits them evenly; each warp's
            // candidates still arrive in ascending index order.
            unsigned gq = 0u;
#pragma unroll
            for (int g = 0; g < G; ++g) gq |= (gmax[g] >= tau) ? (1u << g) : 0u;
            if (h == 1) gq &= gq - 1u;

            // ---- candidates of this warp's qualifying groups ----
            uint32_t key[KM];
            int idx[KM];
#pragma unroll
            for (int i = 0; i < KM; ++i) { key[i] = 0u; idx[i] = 0; }
            if (valid && !nan_row) {
                while (gq) {
                    const int g = __ffs(gq) - 1;
                    gq &= gq - 1u;
                    gq &= gq - 1u;  // the next qualifying group belongs to the other warp
                    const float* rp = myrow + (g >> 1) * C::BOX_FLOATS;
                    const int j0 = (g & 1) * 4;
                    float sv[16];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 x = *reinterpret_cast<const float4*>(rp + (((j0 + q) ^ sw) << 2));
                        const float4 b = bias4[4 * g + q];
                        sv[4 * q + 0] = x.x + b.x;
                        sv[4 * q + 1] = x.y + b.y;
                        sv[4 * q + 2] = x.z + b.z;
                        sv[4 * q + 3] = x.w + b.w;
                    }
                    // Mask of the elements >= tau, built as a tree (no 16-deep OR chain).
                    unsigned mq[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        mq[q] = ((sv[4 * q] >= tau) ? 1u : 0u) | ((sv[4 * q + 1] >= tau) ? 2u : 0u) |
                                ((sv[4 * q + 2] >= tau) ? 4u : 0u) | ((sv[4 * q + 3] >= tau) ? 8u : 0u);
                    unsigned msk = (mq[0] | (mq[1] << 4)) | ((mq[2] << 8) | (mq[3] << 12));
                    while (msk) {
                        const int k = __ffs(msk) - 1;
                        msk &= msk - 1u;
                        // sv[k] by a 4-level select on the bits of k (registers, no reload)
                        float a8[8], a4[4], a2[2];
#pragma unroll
                        for (int u = 0; u < 8; ++u) a8[u] = (k & 1) ? sv[2 * u + 1] : sv[2 * u];
#pragma unroll
                        for (int u = 0; u < 4; ++u) a4[u] = (k & 2) ? a8[2 * u + 1] : a8[2 * u];
#pragma unroll
                        for (int u = 0; u < 2; ++u) a2[u] = (k & 4) ? a4[2 * u + 1] : a4[2 * u];
                        const float v = (k & 8) ? a2[1] : a2[0];
                        topk_insert<KM>(key, idx, fkey(v), g * 16 + k);
                    }
                }
            }

            // ---- merge, weights, outputs ----
            if (h == 1) {
#pragma unroll
                for (int i = 0; i < KM; ++i) {
                    xks[i * 32 + lane] = key[i];
                    xis[i * 32 + lane] = idx[i];
                }
            }
            pair_sync(p);
            if (h == 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + p);
                continue;
            }
            const bool bad = valid && nan_row;
            // The tile's ids and weights are staged in the pair's exchange buffers (32 x KM
            // entries each, row-major [token][K]) and leave as whole 128-byte lines.
            int32_t* oi = reinterpret_cast<int32_t*>(xks);
            float* ow = reinterpret_cast<float*>(xis);
            float xr[KM];  // raw logits of the picks: the last reads of the slot
            if (valid && !nan_row) {
#pragma unroll
                for (int i = 0; i < KM; ++i)
                    if (i < K) topk_merge<KM>(key, idx, xks[i * 32 + lane], xis[i * 32 + lane]);
#pragma unroll
                for (int i = 0; i < KM; ++i) xr[i] = (i < K) ? slot[tile_off(lane, idx[i])] : 0.0f;
            }
            __syncwarp();  // slot and exchange buffers read: release the slot, reuse the buffers
            if (lane == 0) mbar_arrive(empty + p);
            if (valid && !nan_row) {
                float wv[KM];
                float sum = 0.0f;
#pragma unroll
                for (int i = 0; i < KM; ++i) {
                    wv[i] = 0.0f;
                    if (i < K) {
                        wv[i] = sigmoid_acc(xr[i]);
                        sum += wv[i];
                    }
                }
                if (renorm) {
                    const float inv = 1.0f / (sum + 1e-20f);
#pragma unroll
                    for (int i = 0; i < KM; ++i) wv[i] = wv[i] * inv;
                }
                uint16_t* sp = sel + (int)(tb + lane - t0) * K;
#pragma unroll
                for (int i = 0; i < KM; ++i) {
                    if (i < K) {
                        oi[lane * K + i] = idx[i];
                        ow[lane * K + i] = wv[i];
                        if constexpr (MAPS) {
                            sp[i] = (uint16_t)idx[i];
                            atomicAdd(&hist[idx[i]], 1);
                        }
                    }
                }
            }
            // Rows holding a NaN: the exact warp-cooperative ranking on the global row.
            unsigned badm = __ballot_sync(FULL_MASK, bad);
            while (badm) {
                const int l = __ffs(badm) - 1;
                badm &= badm - 1u;
                const float* brow = logits + (tb + l) * E_;
                route_exact<E_ / 32, true>(brow, bias_sm, E_, K, lane, sel_tmp + p * 32);
                const int id = (lane < K) ? sel_tmp[p * 32 + lane] : 0;
                const float wl = pick_weight((lane < K) ? __ldg(brow + id) : 0.0f, K, lane, renorm);
                if (lane < K) {
                    oi[l * K + lane] = id;
                    ow[l * K + lane] = wl;
                    if constexpr (MAPS) {
                        sel[(int)(tb + l - t0) * K + lane] = (uint16_t)id;
                        atomicAdd(&hist[id], 1);
                    }
                }
                __syncwarp();
            }
            __syncwarp();
            {
                const int cnt = rows * K;
                int32_t* gi = ids_out + tb * K;
                WT* gw = w + tb * K;
                if (sizeof(WT) == 4 &&
                    ((reinterpret_cast<uintptr_t>(gi) | reinterpret_cast<uintptr_t>(gw)) & 15u) == 0 &&
                    (cnt & 3) == 0) {  // 16-byte stores when both rows start aligned
                    for (int j = lane; j < (cnt >> 2); j += 32) {
                        reinterpret_cast<int4*>(gi)[j] = reinterpret_cast<const int4*>(oi)[j];
                        reinterpret_cast<float4*>(gw)[j] = reinterpret_cast<const float4*>(ow)[j];
                    }
                } else {
                    for (int j = lane; j < cnt; j += 32) {
                        gi[j] = oi[j];
                        gw[j] = Elem<WT>::from_f(ow[j]);
                    }
                }
            }
            __syncwarp();
        }
    }
    if constexpr (MAPS) {
        const bool staged =
            tile_maps_ints(blockDim.x, E_, n, K, true) <= (size_t)nslot * C::SLOT_FLOATS;
        maps_finish_tile<E_>(ws, T, K, t0, n, sel, hist, totsm, offs, scratch, whist, staged, true,
                             counts, offsets, p2u, u2p);
    }
}

// Hybrid router for kb_router: each warp takes a contiguous range of tokens.
// smem: bias[E] | wsm[nw][hwarp] | sel_tmp[nw][32]
template <int E_, int KT, typename WT>
__global__ void __launch_bounds__(256) router_t_kernel(const float* __restrict__ logits,
                                                       const float* __restrict__ bias,
                                                       int32_t* __restrict__ ids,
                                                       WT* __restrict__ w, int64_t T, int K,
                                                       int renorm, int64_t tpw) {
    pdl_wait();
    pdl_launch();
    extern __shared__ __align__(16) float tsm[];
    constexpr size_t HW = hwarp_smem_floats<E_>();
    const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* bias_sm = tsm;
    float* wsm = bias_sm + E_;
    int* sel_tmp = reinterpret_cast<int*>(wsm + nw * HW);
    troute_setup<E_>(bias, bias_sm);
    float b[E_ / 32];
    load_bias<E_ / 32, true>(bias, E_, lane, b);
    const int64_t tb0 = ((int64_t)blockIdx.x * nw + warp) * tpw;
    const int64_t te = min(T, tb0 + tpw);
    troute_range<E_, KT, false, false, WT>(logits, b, bias_sm, K, renorm, tb0, te, wsm + warp * HW,
                                           sel_tmp + warp * 32, ids, w, nullptr, 0, nullptr);
}

// ------------------------------------------------------------------------------------
// Two-kernel maps (fallback).  Kernel 1: per-tile histogram (optionally routing the tile);
// the last CTA of a super-tile to arrive sums its tiles into super_hist and resets the
// counter.  Kernel 2: one CTA per super-tile scans the super-tile rows and scatters.
// ------------------------------------------------------------------------------------
struct MapsWs {
    unsigned* arrive;   // [S]      zero between calls
    int* tile_counts;   // [num_tiles][E]
    int* super_hist;    // [S][E]
};

template <int VPL, bool VEC, bool ROUTE, int KT>
__global__ void __launch_bounds__(256) maps_count_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias,
    const int32_t* __restrict__ ids_in, int32_t* __restrict__ ids_out, float* __restrict__ w,
    int64_t T, int E, int K, int renorm, int TT, int tiles_per_super, int num_tiles,
    MapsWs ws) {
    pdl_wait();
    pdl_launch();
    extern __shared__ __align__(16) float csmem[];
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
        const RouteSink<float, false, true> sink{ids_out, w, nullptr, 0, hist};
        route_tokens<VPL, VEC, KT>(logits, bias, b, E, K, renorm, t0 + warp, t1, 8,
                                   VEC ? csmem + (size_t)warp * 2 * E : nullptr, sel_sm[warp],
                                   sink);
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

// smem: sel[G*K] | whist[32][E] | tot[E] | pre[E] | offs[E+1] | scratch[64]
__global__ void __launch_bounds__(1024) maps_scatter_kernel(
    const int32_t* __restrict__ ids, int64_t T, int E, int K, int super_tokens, int S,
    const int* __restrict__ super_hist, int32_t* __restrict__ counts,
    int64_t* __restrict__ offsets, int32_t* __restrict__ p2u, int32_t* __restrict__ u2p) {
    pdl_wait();
    pdl_launch();
    extern __shared__ __align__(16) int smem[];
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
    rank_scatter(sel, n, tok0, T, E, K, whist, p2u, u2p);
}

// ------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------
namespace {

constexpr int kSingleThreads = 1024;
constexpr int kScatterThreads = 1024;
constexpr int kTargetSupers = 64;
constexpr int kMaxSingleSel = 12288;   // single-CTA path: T*K selections held in smem
constexpr int kMaxPersistSel = 16384;  // persistent path: selections per CTA held in smem
constexpr int kMaxPersistGrid = 1024;  // bounds the workspace (rowhist) and the prefix reads
constexpr size_t kMaxSmem = 227 * 1024;  // opt-in shared memory per CTA on sm_100

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct DevInfo {
    int sms = 0;
};

DevInfo dev_info() {
    static std::mutex mu;
    static DevInfo cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    DevInfo& d = cache[dev & 63];
    if (d.sms == 0) {
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        if (d.sms <= 0) d.sms = 148;
    }
    return d;
}

enum class Path { Single, Persistent, TPersistent, Tile, IdsTile, TwoKernel };

struct MapsPlan {
    Path path;
    // single
    size_t smem_single;
    // persistent (warp-per-token or transposed)
    int grid, tpc, tnw;
    size_t smem_persist;
    // two-kernel
    int TT, num_tiles, tiles_per_super, S, super_tokens;
    size_t smem_scatter, smem_count;
    size_t ws_bytes;   // workspace for the chosen multi-CTA path
    CUtensorMap tmap;  // tile path: the logits tensor map
};

size_t single_smem(int64_t T, int E, int K, bool route, bool vec) {
    const size_t n = (size_t)T * K;
    size_t words = ((n + 3) & ~size_t(3)) + (size_t)32 * E + E + (E + 1) + 64 + 8;
    size_t bytes = words * sizeof(int) + 16;
    if (route && vec) bytes += (size_t)32 * 2 * E * sizeof(float);
    return bytes;
}

// Hybrid-router shared memory: bias[E] | wsm[nw][hwarp] | sel_tmp[nw][32]
// [ | sel[tpc*K] | hist[E] | totsm[E] | offs[E+1] | scratch[64]  when persistent; whist[nw][E]
//   aliases wsm ]
template <int E_>
size_t troute_smem(int nw, int tpc, int K) {
    const size_t wsm = std::max((size_t)nw * hwarp_smem_floats<E_>(), (size_t)nw * E_);
    size_t b = (size_t)E_ * sizeof(float) + wsm * sizeof(float) + (size_t)nw * 32 * sizeof(int);
    if (tpc > 0)
        b += ((((size_t)tpc * K + 3) & ~size_t(3)) + 2 * (size_t)E_ + ((E_ + 1 + 3) & ~3) + 64) *
             sizeof(int);
    return b;
}

// sel | hist | totsm | offs | scratch | union { ring (phase 1), whist (phase 3) }
size_t persist_smem(int tpc, int E, int K, bool route, bool vec) {
    size_t words = (((size_t)tpc * K + 3) & ~size_t(3)) + 2 * (size_t)E + ((E + 1 + 3) & ~3) + 64;
    const size_t whist = (size_t)kPW * E * sizeof(int);
    const size_t ring = (route && vec) ? (size_t)kPW * 2 * E * sizeof(float) : 0;
    return words * sizeof(int) + std::max(whist, ring);
}

// Workspace layout shared by every multi-CTA maps path, so that paths, shapes and E can
// alternate on one buffer.  The zero zone holds zeros between calls (every call restores
// what it changes in it); the scratch zone behind it is written before it is read.
//   [0, 256)                     bar, err (persistent kernels)
//   [kArriveOff, kGsumOff)       arrival counters of the two-kernel super-tiles
//   [kGsumOff, kScratchOff)      group sums of the persistent kernels ([group][E], E <= E_MAX)
//   [kScratchOff, ...)           rowhist | tile_counts, super_hist
constexpr int kMaxSupers = 4096;
constexpr int kMaxGroups = (kMaxPersistGrid + kGS - 1) / kGS;
constexpr size_t kArriveOff = 256;
constexpr size_t kGsumOff = kArriveOff + (size_t)kMaxSupers * sizeof(unsigned);
constexpr size_t kScratchOff = kGsumOff + (size_t)kMaxGroups * E_MAX * sizeof(int);

size_t persist_ws_bytes(int grid, int E) {
    return kScratchOff + align256((size_t)E * grid * sizeof(int));
}

PersistWs carve_persist(void* ws, int grid, int E) {
    (void)grid;
    (void)E;
    char* b = static_cast<char*>(ws);
    PersistWs w;
    w.bar = reinterpret_cast<unsigned*>(b);
    w.err = reinterpret_cast<int*>(b + sizeof(int));
    w.gsum = reinterpret_cast<int*>(b + kGsumOff);
    w.rowhist = reinterpret_cast<int*>(b + kScratchOff);
    w.spin = wait_limit(kSpinLimit);
    w.cp = CountPush{};
    return w;
}

// Largest cooperative grid for a persistent kernel instance (per device, cached by the
// caller's static).  Returns CTAs per SM.
template <typename KernelT>
int coop_blocks_per_sm(KernelT kern, size_t smem) {
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kPW * 32, smem) != cudaSuccess)
        return 0;
    return nb;
}

// 2-D tensor map of a [T][E] fp32 logits matrix for the tile kernel: 32 x 32 boxes, 128-byte
// swizzle, rows past T zero-filled.  The encoder comes from the driver at first use.
bool make_tile_map(CUtensorMap* map, const float* logits, int64_t T, int E) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (encode == nullptr) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)E, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)E * sizeof(float)};
    const cuuint32_t box[2] = {32, (cuuint32_t)kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(logits),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Two-kernel plan (also the workspace bound).
void plan_two_kernel(MapsPlan& p, int64_t T, int E, int K, bool route, bool vec) {
    if (route) {
        int64_t tpw = (T + 148 * 2 * 8 - 1) / (148 * 2 * 8);
        tpw = std::max<int64_t>(1, std::min<int64_t>(16, tpw));
        p.TT = (int)(8 * tpw);
    } else {
        p.TT = 256;
    }
    p.num_tiles = (int)((T + p.TT - 1) / p.TT);
    const int max_tps = std::max(1, 24576 / (K * p.TT));
    p.tiles_per_super = std::min(max_tps, (p.num_tiles + kTargetSupers - 1) / kTargetSupers);
    p.S = (p.num_tiles + p.tiles_per_super - 1) / p.tiles_per_super;
    p.super_tokens = p.TT * p.tiles_per_super;
    const size_t cap = (size_t)p.super_tokens * K;
    p.smem_scatter = (((cap + 3) & ~size_t(3)) + (size_t)(kScatterThreads / 32) * E + 3 * E + 1 + 64) * sizeof(int);
    p.smem_count = (route && vec) ? (size_t)8 * 2 * E * sizeof(float) : 0;
}

size_t two_kernel_ws(const MapsPlan& p, int E) {
    return kScratchOff + align256((size_t)p.num_tiles * E * sizeof(int)) +
           align256((size_t)p.S * E * sizeof(int));
}

MapsWs carve_two(void* ws, const MapsPlan& p, int E) {
    char* b = static_cast<char*>(ws);
    MapsWs w;
    w.arrive = reinterpret_cast<unsigned*>(b + kArriveOff);
    b += kScratchOff;
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
    template <int KT>
    static int run_kt(const float* logits, const float* bias, int32_t* ids, void* w, int w_dtype,
                      int64_t T, int E, int K, int renorm, cudaStream_t st) {
        const int64_t ctas = std::min<int64_t>((T + 7) / 8, (int64_t)dev_info().sms * 8);
        dim3 grid((unsigned)std::max<int64_t>(1, ctas)), block(256);
        const size_t smem = VEC ? (size_t)8 * 2 * E * sizeof(float) : 0;
        switch (w_dtype) {
            case KB_F32:
                return launch(router_kernel<VPL, VEC, KT, float>, grid, block, smem, st, logits,
                              bias, ids, static_cast<float*>(w), T, E, K, renorm);
            case KB_BF16:
                return launch(router_kernel<VPL, VEC, KT, __nv_bfloat16>, grid, block, smem, st,
                              logits, bias, ids, static_cast<__nv_bfloat16*>(w), T, E, K, renorm);
            case KB_F16:
                return launch(router_kernel<VPL, VEC, KT, __half>, grid, block, smem, st, logits,
                              bias, ids, static_cast<__half*>(w), T, E, K, renorm);
            default:
                return KB_ERR_UNSUPPORTED;
        }
    }
    // Lane-per-token router (trouter.cuh) for E = 32*VPL in {128, 256, 384, 512}, K <= 8.
    template <int KT, typename WT>
    static int run_t(const float* logits, const float* bias, int32_t* ids, WT* w, int64_t T,
                     int K, int renorm, cudaStream_t st) {
        constexpr int E_ = 32 * VPL;
        constexpr int nw = 8;
        const int sms = dev_info().sms;
        auto* kern = router_t_kernel<E_, KT, WT>;
        const size_t smem = troute_smem<E_>(nw, 0, 0);
        int err = allow_smem(kern, smem);
        if (err) return err;
        static int bps = 0;  // co-resident CTAs per SM (per instance)
        if (bps == 0) {
            int v = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, 32 * nw, smem);
            bps = v > 0 ? v : 1;
        }
        const int64_t slots = (int64_t)sms * bps * nw;   // resident warps
        const int64_t tpw = std::max<int64_t>(std::min<int64_t>(32, T), (T + slots - 1) / slots);
        const int64_t warps = (T + tpw - 1) / tpw;
        const int64_t ctas = (warps + nw - 1) / nw;
        return launch(kern, dim3((unsigned)ctas), dim3(32 * nw), smem, st, logits, bias, ids, w, T,
                      K, renorm, tpw);
    }
    template <typename WT>
    static int run_t_any(const float* logits, const float* bias, int32_t* ids, WT* w, int64_t T,
                         int K, int renorm, cudaStream_t st) {
        if (K == 6) return run_t<6, WT>(logits, bias, ids, w, T, K, renorm, st);
        return run_t<0, WT>(logits, bias, ids, w, T, K, renorm, st);
    }
    static int run(const float* logits, const float* bias, int32_t* ids, void* w, int w_dtype,
                   int64_t T, int E, int K, int renorm, cudaStream_t st) {
        if constexpr (VEC) {
            if (K <= 8) {
                switch (w_dtype) {
                    case KB_F32: return run_t_any<float>(logits, bias, ids, static_cast<float*>(w), T, K, renorm, st);
                    case KB_BF16: return run_t_any<__nv_bfloat16>(logits, bias, ids, static_cast<__nv_bfloat16*>(w), T, K, renorm, st);
                    case KB_F16: return run_t_any<__half>(logits, bias, ids, static_cast<__half*>(w), T, K, renorm, st);
                    default: return KB_ERR_UNSUPPORTED;
                }
            }
        }
        if (VEC && K == 6) return run_kt<6>(logits, bias, ids, w, w_dtype, T, E, K, renorm, st);
        return run_kt<0>(logits, bias, ids, w, w_dtype, T, E, K, renorm, st);
    }
};

template <typename... KArgs, typename... Args>
int launch_coop(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

template <bool ROUTE>
struct MapsLaunchT {
    template <int VPL, bool VEC>
    struct Impl {
        template <int KT>
        static auto persistent_kernel() { return maps_persistent_kernel<VPL, VEC, ROUTE, KT>; }

        // Co-resident CTAs per SM of the persistent kernel at a given shared-memory size.
        static int blocks_per_sm(int E, int K, size_t smem) {
            static std::mutex mu;
            static std::map<std::tuple<int, int, int, size_t>, int> cache;
            int dev = 0;
            cudaGetDevice(&dev);
            std::lock_guard<std::mutex> lk(mu);
            int& v = cache[std::make_tuple(dev, E, K, smem)];
            if (v == 0) {
                int occ = 0;
                if (VEC && ROUTE && K == 6) {
                    auto* kern = persistent_kernel<6>();
                    allow_smem(kern, smem);
                    occ = coop_blocks_per_sm(kern, smem);
                } else {
                    auto* kern = persistent_kernel<0>();
                    allow_smem(kern, smem);
                    occ = coop_blocks_per_sm(kern, smem);
                }
                v = occ > 0 ? occ : -1;
            }
            return v;
        }

        // Largest co-resident grid (<= 8 CTAs/SM) whose footprint still fits at that occupancy.
        static bool plan_persist(MapsPlan& p, int64_t T, int E, int K) {
            const int sms = dev_info().sms;
            const int64_t min_tpc = 2 * kPW;
            for (int bps = 8; bps >= 1; --bps) {
                int grid = (int)std::min<int64_t>(std::min(kMaxPersistGrid, bps * sms),
                                                  (T + min_tpc - 1) / min_tpc);
                grid = std::max(grid, 1);
                const int64_t tpc = (T + grid - 1) / grid;
                if (tpc * K > kMaxPersistSel) return false;
                const size_t smem = persist_smem((int)tpc, E, K, ROUTE, VEC);
                if (smem > kMaxSmem) return false;
                const int occ = blocks_per_sm(E, K, smem);
                if (occ <= 0) return false;
                if ((int64_t)occ * sms >= grid) {
                    p.grid = (int)((T + tpc - 1) / tpc);
                    p.tpc = (int)tpc;
                    p.smem_persist = smem;
                    return true;
                }
            }
            return false;
        }

        // Transposed-router persistent kernel (routing, E = 32*VPL, K <= 8): one CTA per SM,
        // up to 4 router warps, whatever fits in shared memory.
        static bool plan_tpersist(MapsPlan& p, int64_t T, int E, int K) {
            if constexpr (!(ROUTE && VEC)) {
                return false;
            } else {
                constexpr int E_ = 32 * VPL;
                constexpr int nw = 8;
                if (K > 8 || E != E_) return false;
                const int sms = dev_info().sms;
                for (int bps = 4; bps >= 1; --bps) {
                    int grid = (int)std::min<int64_t>(std::min(kMaxPersistGrid, bps * sms),
                                                      (T + 31) / 32);
                    grid = std::max(grid, 1);
                    const int64_t tpc = (T + grid - 1) / grid;
                    if (tpc * K > kMaxPersistSel) return false;
                    const size_t smem = troute_smem<E_>(nw, (int)tpc, K);
                    if (smem > kMaxSmem) return false;
                    const int occ = tblocks_per_sm(K, smem);
                    if (occ <= 0) return false;
                    if ((int64_t)occ * sms >= grid) {
                        p.grid = (int)((T + tpc - 1) / tpc);
                        p.tpc = (int)tpc;
                        p.tnw = nw;
                        p.smem_persist = smem;
                        return true;
                    }
                }
                return false;
            }
        }

        // Co-resident CTAs per SM of the transposed persistent kernel.
        static int tblocks_per_sm(int K, size_t smem) {
            if constexpr (!(ROUTE && VEC)) {
                return 0;
            } else {
                constexpr int E_ = 32 * VPL;
                static std::mutex mu;
                static std::map<std::tuple<int, int, size_t>, int> cache;
                int dev = 0;
                cudaGetDevice(&dev);
                std::lock_guard<std::mutex> lk(mu);
                int& v = cache[std::make_tuple(dev, K == 6 ? 6 : 0, smem)];
                if (v == 0) {
                    int occ = 0;
                    if (K == 6) {
                        auto* kern = maps_tpersist_kernel<E_, 6>;
                        allow_smem(kern, smem);
                        occ = coop_blocks_per_sm(kern, smem);
                    } else {
                        auto* kern = maps_tpersist_kernel<E_, 0>;
                        allow_smem(kern, smem);
                        occ = coop_blocks_per_sm(kern, smem);
                    }
                    v = occ > 0 ? occ : -1;
                }
                return v;
            }
        }

        // Tile kernel (routing, E = 32*VPL in {128, 256, 384}, K <= 8, T >= 32): one CTA per
        // SM with as many 32-row ring slots (and consumer pairs) as shared memory holds.
        static size_t tile_smem(int nslot, int tpc, int K) {
            constexpr int E_ = 32 * VPL;
            return 1024 + (K == 6 ? tile_smem_bytes<E_, 6>(nslot, tpc, K)
                                  : tile_smem_bytes<E_, 0>(nslot, tpc, K));
        }
        static int tile_blocks_per_sm(int K, int nslot, size_t smem) {
            if constexpr (!(ROUTE && VEC && 32 * VPL <= 384)) {
                return 0;
            } else {
                constexpr int E_ = 32 * VPL;
                static std::mutex mu;
                static std::map<std::tuple<int, int, int, size_t>, int> cache;
                int dev = 0;
                cudaGetDevice(&dev);
                std::lock_guard<std::mutex> lk(mu);
                int& v = cache[std::make_tuple(dev, K == 6 ? 6 : 0, nslot, smem)];
                if (v == 0) {
                    int occ = 0;
                    auto* kern = (K == 6) ? maps_tile_kernel<E_, 6> : maps_tile_kernel<E_, 0>;
                    allow_smem(kern, smem);
                    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 32 * (1 + 2 * nslot),
                                                                      smem) != cudaSuccess)
                        occ = 0;
                    v = occ > 0 ? occ : -1;
                }
                return v;
            }
        }
        static bool plan_tile(MapsPlan& p, int64_t T, int E, int K) {
            if constexpr (!(ROUTE && VEC && 32 * VPL <= 384)) {
                return false;
            } else {
                constexpr int E_ = 32 * VPL;
                if (E != E_ || K > 8 || T < kTileRows || T > (int64_t)INT32_MAX) return false;
                const int sms = dev_info().sms;
                int grid = (int)std::min<int64_t>(std::min(kMaxPersistGrid, sms),
                                                  (T + kTileRows - 1) / kTileRows);
                grid = std::max(grid, 1);
                const int64_t tpc = (T + grid - 1) / grid;
                if (tpc * K > kMaxPersistSel) return false;
                for (int ns = kTileMaxSlots; ns >= 2; --ns) {
                    const size_t smem = tile_smem(ns, (int)tpc, K);
                    if (smem > kMaxSmem) continue;
                    if (tile_blocks_per_sm(K, ns, smem) < 1) return false;
                    p.grid = (int)((T + tpc - 1) / tpc);
                    p.tpc = (int)tpc;
                    p.tnw = ns;
                    p.smem_persist = smem;
                    return true;
                }
                return false;
            }
        }

        // Maps from ids through the tile kernel's map phases (E = 32*VPL in {128, 256, 384}).
        static size_t ids_tile_smem(int tpc, int K) {
            constexpr int E_ = 32 * VPL;
            return (tile_align((size_t)tpc * K, 8) / 2 + 2 * (size_t)E_ + tile_align(E_ + 1, 4) +
                    64 + tile_maps_ints(256, E_, tpc * K, K, true)) * sizeof(int);
        }
        static bool plan_ids_tile(MapsPlan& p, int64_t T, int E, int K) {
            if constexpr (ROUTE || !VEC || 32 * VPL > 384) {
                return false;
            } else {
                constexpr int E_ = 32 * VPL;
                if (E != E_ || T < kTileRows || T > (int64_t)INT32_MAX) return false;
                const int sms = dev_info().sms;
                int grid = (int)std::min<int64_t>(std::min(kMaxPersistGrid, sms),
                                                  (T + kTileRows - 1) / kTileRows);
                grid = std::max(grid, 1);
                const int64_t tpc = (T + grid - 1) / grid;
                if (tpc * K > kMaxPersistSel) return false;
                const size_t smem = ids_tile_smem((int)tpc, K);
                if (smem > kMaxSmem) return false;
                static std::mutex mu;
                static std::map<std::tuple<int, size_t>, int> cache;
                int dev = 0;
                cudaGetDevice(&dev);
                {
                    std::lock_guard<std::mutex> lk(mu);
                    int& v = cache[std::make_tuple(dev, smem)];
                    if (v == 0) {
                        int occ = 0;
                        auto* kern = maps_ids_tile_kernel<E_>;
                        allow_smem(kern, smem);
                        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, smem) !=
                            cudaSuccess)
                            occ = 0;
                        v = occ > 0 ? occ : -1;
                    }
                    if (v < 1) return false;
                }
                p.grid = (int)((T + tpc - 1) / tpc);
                p.tpc = (int)tpc;
                p.smem_persist = smem;
                return true;
            }
        }

        static MapsPlan plan(int64_t T, int E, int K, int mode, bool allow_tile = true) {
            MapsPlan p{};
            const bool fits_single = T * K <= kMaxSingleSel;
            const int64_t auto_single_T = ROUTE ? 32 : 768;
            if (mode == KB_MAPS_SINGLE_CTA || (mode == KB_MAPS_AUTO && fits_single && T <= auto_single_T)) {
                p.path = Path::Single;
                p.smem_single = single_smem(T, E, K, ROUTE, VEC);
                return p;
            }
            plan_two_kernel(p, T, E, K, ROUTE, VEC);
            // Forced routing paths: KB_MAPS_HYBRID_ROUTER skips the tile kernel,
            // KB_MAPS_WARP_ROUTER skips both the tile and the hybrid-router kernels.
            const bool multi = mode != KB_MAPS_TWO_KERNEL;
            const bool tile_ok = multi && mode != KB_MAPS_HYBRID_ROUTER && mode != KB_MAPS_WARP_ROUTER;
            const bool hybrid_ok = multi && mode != KB_MAPS_WARP_ROUTER;
            if (tile_ok && allow_tile && plan_tile(p, T, E, K)) {
                p.path = Path::Tile;
                p.ws_bytes = persist_ws_bytes(p.grid, E);
            } else if (!ROUTE && (mode == KB_MAPS_AUTO || mode == KB_MAPS_MULTI_CTA) &&
                       plan_ids_tile(p, T, E, K)) {
                // ids only: the tile kernel's map phases (KB_MAPS_WARP_ROUTER / HYBRID_ROUTER
                // keep the warp-per-token persistent kernel's map phases reachable)
                p.path = Path::IdsTile;
                p.ws_bytes = persist_ws_bytes(p.grid, E);
            } else if (hybrid_ok && plan_tpersist(p, T, E, K)) {
                p.path = Path::TPersistent;
                p.ws_bytes = persist_ws_bytes(p.grid, E);
            } else if (multi && plan_persist(p, T, E, K)) {
                p.path = Path::Persistent;
                p.ws_bytes = persist_ws_bytes(p.grid, E);
            } else {
                p.path = Path::TwoKernel;
                p.ws_bytes = two_kernel_ws(p, E);
            }
            return p;
        }

        template <int KT>
        static int run_kt(const MapsPlan& p, const float* logits, const float* bias,
                          const int32_t* ids_in, int32_t* ids_out, float* w, int32_t* counts,
                          int64_t* offsets, int32_t* p2u, int32_t* u2p, void* ws, int64_t T, int E,
                          int K, int renorm, cudaStream_t st, CountPush* push) {
            if (p.path == Path::Single) {
                auto* kern = maps_single_kernel<VPL, VEC, ROUTE, KT>;
                int err = allow_smem(kern, p.smem_single);
                if (err) return err;
                CountPush cp{};
                if (push) {
                    cp = *push;
                    push->fused = 1;
                }
                return launch(kern, dim3(1), dim3(kSingleThreads), p.smem_single, st, logits, bias,
                              ids_in, ids_out, w, T, E, K, renorm, counts, offsets, p2u, u2p, cp);
            }
            if constexpr (ROUTE && VEC && 32 * VPL <= 384) {
                if (p.path == Path::Tile) {
                    constexpr int E_ = 32 * VPL;
                    auto* kern = maps_tile_kernel<E_, (KT == 6 ? 6 : 0)>;
                    int err = allow_smem(kern, p.smem_persist);
                    if (err) return err;
                    PersistWs pw = carve_persist(ws, p.grid, E);
                    if (push && p.grid >= push->world) {
                        pw.cp = *push;
                        push->fused = 1;
                    }
                    return launch_coop(kern, dim3(p.grid), dim3(32 * (1 + 2 * p.tnw)),
                                       p.smem_persist, st, p.tmap, logits, bias, ids_out, w, T, K,
                                       renorm, p.tpc, p.tnw, counts, offsets, p2u, u2p, pw);
                }
                if (p.path == Path::TPersistent) {
                    constexpr int E_ = 32 * VPL;
                    auto* kern = maps_tpersist_kernel<E_, (KT == 6 ? 6 : 0)>;
                    int err = allow_smem(kern, p.smem_persist);
                    if (err) return err;
                    return launch_coop(kern, dim3(p.grid), dim3(32 * p.tnw), p.smem_persist, st,
                                       logits, bias, ids_out, w, T, K, renorm, p.tpc, counts,
                                       offsets, p2u, u2p, carve_persist(ws, p.grid, E));
                }
            }
            if constexpr (!ROUTE && VEC && 32 * VPL <= 384) {
                if (p.path == Path::IdsTile) {
                    constexpr int E_ = 32 * VPL;
                    auto* kern = maps_ids_tile_kernel<E_>;
                    int err = allow_smem(kern, p.smem_persist);
                    if (err) return err;
                    return launch_coop(kern, dim3(p.grid), dim3(256), p.smem_persist, st, ids_in, T,
                                       K, p.tpc, counts, offsets, p2u, u2p,
                                       carve_persist(ws, p.grid, E));
                }
            }
            if (p.path == Path::Persistent) {
                auto* kern = persistent_kernel<KT>();
                int err = allow_smem(kern, p.smem_persist);
                if (err) return err;
                return launch_coop(kern, dim3(p.grid), dim3(kPW * 32), p.smem_persist, st, logits,
                                   bias, ids_in, ids_out, w, T, E, K, renorm, p.tpc, counts,
                                   offsets, p2u, u2p, carve_persist(ws, p.grid, E));
            }
            const MapsWs w_ = carve_two(ws, p, E);
            auto* k1 = maps_count_kernel<VPL, VEC, ROUTE, KT>;
            int err = allow_smem(k1, p.smem_count);
            if (err) return err;
            err = launch(k1, dim3(p.num_tiles), dim3(256), p.smem_count, st, logits, bias, ids_in,
                         ids_out, w, T, E, K, renorm, p.TT, p.tiles_per_super, p.num_tiles, w_);
            if (err) return err;
            err = allow_smem(maps_scatter_kernel, p.smem_scatter);
            if (err) return err;
            const int32_t* ids_src = ROUTE ? ids_out : ids_in;
            return launch(maps_scatter_kernel, dim3(p.S), dim3(kScatterThreads), p.smem_scatter, st,
                          ids_src, T, E, K, p.super_tokens, p.S,
                          static_cast<const int*>(w_.super_hist), counts, offsets, p2u, u2p);
        }

        static int run(const float* logits, const float* bias, const int32_t* ids_in,
                       int32_t* ids_out, float* w, int32_t* counts, int64_t* offsets,
                       int32_t* p2u, int32_t* u2p, void* ws, size_t ws_bytes, int64_t T,
                       int E, int K, int renorm, int mode, cudaStream_t st,
                       CountPush* push = nullptr) {
            // The tile path's tensor copies need a 16-byte aligned logits base and the
            // driver's tensor-map encoder; without either the next path is taken.
            MapsPlan p = plan(T, E, K, mode, !ROUTE || aligned16(logits));
            if (p.path == Path::Tile && !make_tile_map(&p.tmap, logits, T, E))
                p = plan(T, E, K, mode, false);
            if (p.path == Path::Single) {
                if (T * K > kMaxSingleSel || p.smem_single > kMaxSmem) return KB_ERR_UNSUPPORTED;
            } else {
                if (p.path == Path::TwoKernel && p.S > kMaxSupers) return KB_ERR_TOO_LARGE;
                if (ws == nullptr || ws_bytes < p.ws_bytes) return KB_ERR_WORKSPACE;
                if (!aligned16(ws)) return KB_ERR_ALIGNMENT;
            }
            if (VEC && ROUTE && K == 6)
                return run_kt<6>(p, logits, bias, ids_in, ids_out, w, counts, offsets, p2u, u2p,
                                 ws, T, E, K, renorm, st, push);
            if (p.path == Path::TPersistent ||
                p.path == Path::Tile)  // runtime-K (K <= 8)
                return run_kt<0>(p, logits, bias, ids_in, ids_out, w, counts, offsets, p2u, u2p,
                                 ws, T, E, K, renorm, st, push);
            return run_kt<0>(p, logits, bias, ids_in, ids_out, w, counts, offsets, p2u, u2p, ws,
                             T, E, K, renorm, st, push);
        }

        // Workspace large enough for every multi-CTA path at this T.
        static size_t ws_bound(int64_t T, int E, int K) {
            MapsPlan p{};
            plan_two_kernel(p, T, E, K, ROUTE, VEC);
            size_t b = two_kernel_ws(p, E);
            MapsPlan q{};
            if (plan_persist(q, T, E, K)) b = std::max(b, persist_ws_bytes(q.grid, E));
            MapsPlan r{};
            if (plan_tpersist(r, T, E, K)) b = std::max(b, persist_ws_bytes(r.grid, E));
            MapsPlan v{};
            if (plan_tile(v, T, E, K)) b = std::max(b, persist_ws_bytes(v.grid, E));
            MapsPlan u{};
            if (plan_ids_tile(u, T, E, K)) b = std::max(b, persist_ws_bytes(u.grid, E));
            return b;
        }

        // Path, launches and grid the library would use (introspection for benchmarks).
        static void describe(int64_t T, int E, int K, int mode, int* path, int* launches,
                             int* grid) {
            const MapsPlan p = plan(T, E, K, mode);
            const bool pers = p.path == Path::Persistent || p.path == Path::TPersistent ||
                              p.path == Path::Tile || p.path == Path::IdsTile;
            // Routing paths name their router kernel: the hybrid and the warp-per-token router.
            const int pk = p.path == Path::Single ? KB_MAPS_SINGLE_CTA
                         : (ROUTE && p.path == Path::TPersistent) ? KB_MAPS_HYBRID_ROUTER
                         : (ROUTE && p.path == Path::Persistent) ? KB_MAPS_WARP_ROUTER
                         : pers ? KB_MAPS_MULTI_CTA : KB_MAPS_TWO_KERNEL;
            if (path) *path = pk;
            if (launches) *launches = (p.path == Path::TwoKernel) ? 2 : 1;
            if (grid) *grid = p.path == Path::Single ? 1 : pers ? p.grid : p.num_tiles;
        }
    };
};

template <int VPL, bool VEC>
using MapsOnly = MapsLaunchT<false>::Impl<VPL, VEC>;
template <int VPL, bool VEC>
using RouterMaps = MapsLaunchT<true>::Impl<VPL, VEC>;

template <template <int, bool> class Fn>
void describe_for(int64_t T, int E, int K, int mode, int* path, int* launches, int* grid) {
    if (E == 384) return Fn<12, true>::describe(T, E, K, mode, path, launches, grid);
    if (E == 256) return Fn<8, true>::describe(T, E, K, mode, path, launches, grid);
    if (E == 512) return Fn<16, true>::describe(T, E, K, mode, path, launches, grid);
    if (E == 128) return Fn<4, true>::describe(T, E, K, mode, path, launches, grid);
    return Fn<16, false>::describe(T, E, K, mode, path, launches, grid);
}

template <template <int, bool> class Fn>
size_t ws_bound_for(int64_t T, int E, int K) {
    if (E == 384) return Fn<12, true>::ws_bound(T, E, K);
    if (E == 256) return Fn<8, true>::ws_bound(T, E, K);
    if (E == 512) return Fn<16, true>::ws_bound(T, E, K);
    if (E == 128) return Fn<4, true>::ws_bound(T, E, K);
    return Fn<16, false>::ws_bound(T, E, K);
}

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

namespace kb {
namespace {
// kb_router through the tile kernel without its map phases (E = 32*VPL in {128, 256, 384},
// K <= 8, T >= 32, when its shared memory fits; weights rounded to WT at the store).  Returns
// KB_ERR_UNSUPPORTED, having launched nothing, when that path does not apply.
template <int VPL, typename WT>
int tile_router(const float* logits, const float* bias, int32_t* ids, WT* w, int64_t T, int E,
                int K, int renorm, cudaStream_t st) {
    constexpr int E_ = 32 * VPL;
    if constexpr (E_ > 384) {
        return KB_ERR_UNSUPPORTED;
    } else {
        MapsPlan p{};
        if (!aligned16(logits) || !RouterMaps<VPL, true>::plan_tile(p, T, E, K))
            return KB_ERR_UNSUPPORTED;
        if (!make_tile_map(&p.tmap, logits, T, E)) return KB_ERR_UNSUPPORTED;
        auto* kern = (K == 6) ? maps_tile_kernel<E_, 6, false, WT> : maps_tile_kernel<E_, 0, false, WT>;
        int err = allow_smem(kern, p.smem_persist);
        if (err) return err;
        PersistWs nows{};  // no workspace: no error word, only the wait limit
        nows.spin = wait_limit(kMbarSpin);
        return launch(kern, dim3(p.grid), dim3(32 * (1 + 2 * p.tnw)), p.smem_persist, st, p.tmap,
                      logits, bias, ids, w, T, K, renorm, p.tpc, p.tnw,
                      static_cast<int32_t*>(nullptr), static_cast<int64_t*>(nullptr),
                      static_cast<int32_t*>(nullptr), static_cast<int32_t*>(nullptr), nows);
    }
}
template <typename WT>
int tile_router_any(const float* logits, const float* bias, int32_t* ids, WT* w, int64_t T,
                    int E, int K, int renorm, cudaStream_t st) {
    if (E == 384) return tile_router<12, WT>(logits, bias, ids, w, T, E, K, renorm, st);
    if (E == 256) return tile_router<8, WT>(logits, bias, ids, w, T, E, K, renorm, st);
    if (E == 128) return tile_router<4, WT>(logits, bias, ids, w, T, E, K, renorm, st);
    return KB_ERR_UNSUPPORTED;
}
}  // namespace
}  // namespace kb

extern "C" int kb_router(const float* logits, const float* bias, int32_t* ids, void* weights,
                         int w_dtype, int64_t T, int E, int K, int renorm, kb_stream_t stream) {
    int st = check_common(T, E, K);
    if (st) return st;
    if (T == 0) return KB_OK;
    if (!logits || !ids || !weights) return KB_ERR_INVALID_ARG;
    if (w_dtype != KB_F32 && w_dtype != KB_BF16 && w_dtype != KB_F16) return KB_ERR_UNSUPPORTED;
    if ((E % 128 == 0) && (!aligned16(logits) || (bias && !aligned16(bias)))) return KB_ERR_ALIGNMENT;
    if (K <= 8) {  // large T: the tile kernel's routing phase alone
        const cudaStream_t cs = (cudaStream_t)stream;
        const int tr =
            w_dtype == KB_F32 ? tile_router_any(logits, bias, ids, static_cast<float*>(weights), T, E, K, renorm, cs)
            : w_dtype == KB_BF16 ? tile_router_any(logits, bias, ids, static_cast<__nv_bfloat16*>(weights), T, E, K, renorm, cs)
                                 : tile_router_any(logits, bias, ids, static_cast<__half*>(weights), T, E, K, renorm, cs);
        if (tr != KB_ERR_UNSUPPORTED) return tr;
    }
    return with_layout<RouterLaunch>(E, logits, bias, ids, weights, w_dtype, T, E, K, renorm,
                                     (cudaStream_t)stream);
}

// The workspace bound covers every multi-CTA path (host-only computation; it queries the
// device's occupancy only when a GPU is present).
extern "C" size_t kb_expert_maps_workspace_bytes(int64_t T, int E, int K) {
    if (check_common(T, E, K) != KB_OK || T == 0) return 0;
    return ws_bound_for<MapsOnly>(T, E, K);
}

extern "C" size_t kb_router_maps_workspace_bytes(int64_t T, int E, int K) {
    if (check_common(T, E, K) != KB_OK || T == 0) return 0;
    return ws_bound_for<RouterMaps>(T, E, K);
}

extern "C" int kb_expert_maps(const int32_t* ids, int32_t* counts, int64_t* offsets, int32_t* p2u,
                              int32_t* u2p, void* workspace, size_t workspace_bytes, int64_t T,
                              int E, int K, int mode, kb_stream_t stream) {
    int st = check_common(T, E, K);
    if (st) return st;
    if (mode < KB_MAPS_AUTO || mode > KB_MAPS_WARP_ROUTER) return KB_ERR_INVALID_ARG;
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
    if (mode < KB_MAPS_AUTO || mode > KB_MAPS_WARP_ROUTER) return KB_ERR_INVALID_ARG;
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

extern "C" int kb_router_maps_allgather(const kb_ep_group_t* g, const float* logits,
                                        const float* bias, int32_t* ids, float* weights,
                                        int32_t* counts, int64_t* offsets, int32_t* p2u,
                                        int32_t* u2p, void* workspace, size_t workspace_bytes,
                                        int64_t T, int renorm, int mode, int32_t* gathered,
                                        kb_stream_t stream) {
    CountPush cp;
    if (const int s = make_count_push(g, gathered, &cp)) return s;
    if (!counts) return KB_ERR_INVALID_ARG;
    const int E = g->num_experts, K = g->top_k;
    int st = check_common(T, E, K);
    if (st) return st;
    if (mode < KB_MAPS_AUTO || mode > KB_MAPS_WARP_ROUTER) return KB_ERR_INVALID_ARG;
    if (T > 0) {
        if (!logits || !ids || !weights || !p2u || !offsets) return KB_ERR_INVALID_ARG;
        if ((E % 128 == 0) && (!aligned16(logits) || (bias && !aligned16(bias))))
            return KB_ERR_ALIGNMENT;
        if (mode == KB_MAPS_SINGLE_CTA && T * K > kMaxSingleSel) return KB_ERR_UNSUPPORTED;
        st = with_layout<RouterMaps>(E, logits, bias, nullptr, ids, weights, counts, offsets, p2u,
                                     u2p, workspace, workspace_bytes, T, E, K, renorm, mode,
                                     (cudaStream_t)stream, &cp);
    } else {
        st = kb_router_maps(logits, bias, ids, weights, counts, offsets, p2u, u2p, workspace,
                            workspace_bytes, T, E, K, renorm, mode, stream);
    }
    if (st || cp.fused) return st;
    return kb_ep_counts_allgather(g, counts, gathered, stream);
}

extern "C" int kb_maps_describe(int64_t T, int E, int K, int route, int mode, int* path,
                                int* launches, int* grid) {
    int st = check_common(T, E, K);
    if (st) return st;
    if (mode < KB_MAPS_AUTO || mode > KB_MAPS_WARP_ROUTER) return KB_ERR_INVALID_ARG;
    if (T == 0) {
        if (path) *path = KB_MAPS_SINGLE_CTA;
        if (launches) *launches = 1;
        if (grid) *grid = 1;
        return KB_OK;
    }
    if (route) describe_for<RouterMaps>(T, E, K, mode, path, launches, grid);
    else describe_for<MapsOnly>(T, E, K, mode, path, launches, grid);
    return KB_OK;
}

// ------------------------------------------------------------------------------------
// kb_expert_maps_noalloc: kb_expert_maps (mode AUTO) with its workspace in a static
// device array, for callers that may not allocate device memory.
// ------------------------------------------------------------------------------------
namespace kb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB on each device
constexpr int64_t kNoAllocMaxTokens = int64_t(1) << 19;   // 524288 tokens per call

// Workspace of every kb_expert_maps_noalloc call on a device.  The CUDA runtime reserves
// one copy in each device context when it loads this library's device code; the library
// never allocates it.  It must hold zeros before the first call (the first call on each
// device fills it), and every completed call leaves it zero-filled again.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

__global__ void zero_scratch_kernel(uint4* __restrict__ p, size_t n16) {
    pdl_wait();
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16;
         i += (size_t)gridDim.x * blockDim.x)
        p[i] = z;
    pdl_launch();
}

// Device address of the scratch for the current device, resolved once per device with
// cudaGetSymbolAddress; the first call on a device (and any call with KB_NOALLOC_REZERO)
// zero-fills it on `st` before the maps kernels run.
int noalloc_scratch(cudaStream_t st, int flags, void** out) {
    static std::mutex mu;
    static void* ptrs[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (dev < 0 || dev >= 64) return KB_ERR_UNSUPPORTED;
    if (st != nullptr) {  // the scratch address is per device: the stream must be this device's
        int sdev = -1;
        e = cudaStreamGetDevice(st, &sdev);
        if (e != cudaSuccess) return static_cast<int>(e);
        if (sdev != dev) return KB_ERR_INVALID_ARG;
    }
    std::lock_guard<std::mutex> lk(mu);
    void* p = ptrs[dev];
    const bool first = (p == nullptr);
    if (first) {
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return static_cast<int>(e);
        if (p == nullptr || !aligned16(p)) return KB_ERR_ALIGNMENT;
    }
    if (first || (flags & KB_NOALLOC_REZERO)) {
        const int err = launch(zero_scratch_kernel, dim3((unsigned)dev_info().sms * 4), dim3(256),
                               0, st, static_cast<uint4*>(p), kNoAllocScratchBytes / 16);
        if (err) return err;
    }
    ptrs[dev] = p;  // published only once the zero fill is enqueued
    *out = p;
    return KB_OK;
}


}  // namespace

size_t maps_err_offset() { return sizeof(unsigned); }

// The scratch address of the current device for kb_workspace_status (no zero fill: a scratch
// that no call has used yet holds zeros).
int noalloc_scratch_address(void** out) {
    return static_cast<int>(cudaGetSymbolAddress(out, g_noalloc_scratch));
}
}  // namespace kb

extern "C" int kb_expert_maps_noalloc(const int32_t* ids, int32_t* counts, int64_t* offsets,
                                      int32_t* p2u, int32_t* u2p, int64_t T, int E, int K,
                                      int flags, kb_stream_t stream) {
    int st = check_common(T, E, K);
    if (st) return st;
    if ((flags & ~KB_NOALLOC_REZERO) != 0 || !offsets) return KB_ERR_INVALID_ARG;
    if (T > 0 && (!ids || !p2u)) return KB_ERR_INVALID_ARG;
    if (T > kNoAllocMaxTokens) return KB_ERR_SCRATCH_LIMIT;
    const size_t need = T > 0 ? ws_bound_for<MapsOnly>(T, E, K) : 0;
    if (need > kNoAllocScratchBytes) return KB_ERR_SCRATCH_LIMIT;
    void* scratch = nullptr;
    st = noalloc_scratch(static_cast<cudaStream_t>(stream), flags, &scratch);
    if (st) return st;
    return kb_expert_maps(ids, counts, offsets, p2u, u2p, scratch, kNoAllocScratchBytes, T, E, K,
                          KB_MAPS_AUTO, stream);
}
