// Expert-parallel exchange over peer memory for sm_100a: the per-expert count all-gather,
// the dispatch of routed rows to their owners and the combine back, as kernels of this GPU
// storing into the other ranks' exchange buffers (mapped through CUDA IPC, so the stores
// travel over NVLink / NVSwitch), with release increments of per-rank arrival counters and
// bounded acquire polls on the receiving side.  No NCCL call and no host round trip: the
// send and receive splits, and the final row of every transfer, follow on the device from
// the all-gathered counts.
//
// Row placement (N ranks, rank r owns experts [r*Er, (r+1)*Er), Er = E/N; c[q][e] = count of
// expert e on rank q; tot[e] = sum_q c[q][e]; S = exclusive scan of tot over all experts):
//   dispatch  permuted row i of expert e on rank q (loff_q[e] <= i < loff_q[e+1], loff_q the
//             exclusive scan of c[q]) lands on owner o = e / Er at grouped row
//             (S[e] - S[o*Er]) + sum_{q' < q} c[q'][e] + (i - loff_q[e])
//             i.e. by local expert, then by sender, then in the sender's (expert, token,
//             slot) order -- the order of an all-to-all of the expert-sorted rows followed by
//             a stable grouping by local expert (the reference's map order,
//             kernels/cuda/customKolibriBuildExpertMapsKernel.cu:96-156).
//   combine   the inverse: grouped row g of the owner goes back to sender q's permuted row
//             loff_q[e] + j, where g is the j-th row of sender q in expert e's segment; the
//             sender then finalizes from its returned rows exactly as kb_moe_finalize
//             (benchmarks/11_profile_2block_e2e.py:259-262).
//
// Synchronisation.  Counts travel as 64-bit words (epoch << 32 | count) into one of two slots
// chosen by epoch parity, so one word carries its own validity.  Rows are followed, per call
// and per sending rank, by one red.release.sys increment of the receiver's arrival counter,
// made by the sender's last CTA after every CTA of the sender fenced its stores; the receiver
// polls its counters with ld.acquire.sys until they reach the call's epoch.  Every call waits
// for every rank, and a rank's next send into a buffer region happens only after the owner of
// that region has finished reading it (see the hazard notes at each kernel).
#include "ep_common.cuh"
#include "finalize_math.cuh"
#include "norm_math.cuh"

#include <algorithm>
#include <cstring>

namespace kb {
namespace {

constexpr int kMaxRanks = kEpMaxRanks;
constexpr long long kPeerSpin = kEpSpin;
constexpr size_t kErr = kEpErr, kDispEpoch = kEpDispEpoch, kCombEpoch = kEpCombEpoch;
constexpr size_t kDispTicket = kEpDispTicket, kCombTicket = kEpCombTicket, kFinTicket = kEpFinTicket;
constexpr size_t kDispArrive = kEpDispArrive, kCombArrive = kEpCombArrive, kCountsOff = kEpCountsOff;

constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Layout {
    size_t recv, back, total;
    int64_t cap_recv, cap_back;   // rows
};

Layout layout(int world, int E, int K, int64_t max_tokens, int64_t row_bytes) {
    Layout L;
    L.cap_recv = (int64_t)world * max_tokens * K;
    L.cap_back = max_tokens * K;
    L.recv = align_up(kCountsOff + (size_t)2 * kMaxRanks * E * 8, 256);
    L.back = align_up(L.recv + (size_t)L.cap_recv * row_bytes, 256);
    L.total = align_up(L.back + (size_t)L.cap_back * row_bytes, 256);
    return L;
}

// Kernel view of a group.
struct EpDev {
    char* buf[kMaxRanks];
    int world, rank, E, K, Er;
    int64_t cap_recv, cap_back, vpr;   // capacities in rows, 16-byte vectors per row
    size_t recv, back;                 // byte offsets of the row areas
    long long spin;
};

__device__ __forceinline__ unsigned* word(const EpDev& g, int q, size_t off) {
    return reinterpret_cast<unsigned*>(g.buf[q] + off);
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_volatile(const unsigned* p) { return ep_ld_volatile(p); }
__device__ __forceinline__ void set_err(const EpDev& g, unsigned code) {
    atomicCAS(word(g, g.rank, kErr), 0u, code);
}

// One thread: poll this rank's arrival counters [q] at `off` until each reaches `target`
// (wrap-safe).  False if the wait gave up: after g.spin polls, or at once when another CTA's
// wait has already given up (the error word is set), so a failed exchange ends in one wait.
__device__ bool wait_arrivals(const EpDev& g, size_t off, unsigned target) {
    const unsigned* a = word(g, g.rank, off);
    const unsigned* err = word(g, g.rank, kErr);
    long long it = 0;
    for (int q = 0; q < g.world; ++q) {
        unsigned v = ld_acquire_sys(a + q);
        while ((int)(v - target) < 0) {
            if (++it > g.spin || ((it & 63) == 0 && ld_volatile(err) != 0u)) return false;
            __nanosleep(128);
            v = ld_acquire_sys(a + q);
        }
    }
    return true;
}

// Exclusive scan of a[0..n) in place, a[n] = total, by one whole warp (the caller brackets it
// with barriers).
__device__ void warp_excl_scan(int* a, int n) {
    const int lane = threadIdx.x & 31;
    const int per = (n + 31) / 32;
    const int b = lane * per, e = min(b + per, n);
    int s = 0;
    for (int i = b; i < e; ++i) s += a[i];
    const int incl = warp_incl_scan(s, lane);
    int run = incl - s;
    for (int i = b; i < e; ++i) {
        const int v = a[i];
        a[i] = run;
        run += v;
    }
    if (lane == 31) a[n] = incl;
}

// Largest i in [0, n) with a[i] <= v (a non-decreasing, a[0] <= v).
__device__ __forceinline__ int last_le(const int* a, int n, int v) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a[mid] <= v) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Copy one row of vpr 16-byte vectors with one warp, UNROLL vectors per lane in flight; the
// destination is written once and not read again by this kernel (evict-first stores).
template <int UNROLL>
__device__ __forceinline__ void warp_copy_row(const uint4* __restrict__ src, uint4* dst,
                                              int64_t vpr, int lane) {
    int64_t v = lane;
    for (; v + 32 * (UNROLL - 1) < vpr; v += 32 * UNROLL) {
        uint4 buf[UNROLL];
#pragma unroll
        for (int i = 0; i < UNROLL; ++i) buf[i] = __ldg(src + v + 32 * i);
#pragma unroll
        for (int i = 0; i < UNROLL; ++i) st_stream(dst + v + 32 * i, buf[i]);
    }
    for (; v < vpr; v += 32) st_stream(dst + v, __ldg(src + v));
}

// ------------------------------------------------------------------------------------
// Count all-gather: one CTA (the protocol of ep_common.cuh).
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) ep_counts_kernel(CountPush cp, const int32_t* __restrict__ counts) {
    pdl_wait();
    __shared__ unsigned tag_s;
    __shared__ int bad;
    __shared__ int sc[E_MAX];
    if (threadIdx.x == 0) {
        tag_s = count_push_tag(cp);
        bad = ep_ld_volatile(reinterpret_cast<const unsigned*>(cp.buf[cp.rank] + kEpErr)) != 0u;
    }
    for (int e = threadIdx.x; e < cp.E; e += blockDim.x) sc[e] = __ldg(counts + e);
    __syncthreads();
    if (bad) {
        for (int i = threadIdx.x; i < cp.world * cp.E; i += blockDim.x) cp.gathered[i] = -1;
        return;
    }
    // this rank's row into every rank's buffer: warp group q % 4 of the CTA sends to rank q
    const int per = blockDim.x / 4;
    for (int q = threadIdx.x / per; q < cp.world; q += 4)
        count_push_send(cp, sc, q, tag_s, threadIdx.x % per, per);
    pdl_launch();
    count_push_gather(cp, tag_s);
}

// Shared tables of the row kernels, built by every CTA from gathered [N][E]:
//   S[0..E]        exclusive scan of tot[e] = sum_q c[q][e]
//   mine[0..E]     exclusive scan of this rank's counts (its permuted-row offsets)
//   before[e]      sum_{q < rank} c[q][e]
// Returns false (error word set by the caller's CTA 0) if a count is negative.
__device__ bool build_tables(const EpDev& g, const int32_t* __restrict__ gathered, int* S,
                             int* mine, int* before) {
    __shared__ int neg;
    if (threadIdx.x == 0) neg = 0;
    __syncthreads();
    for (int e = threadIdx.x; e < g.E; e += blockDim.x) {
        int tot = 0, bef = 0, my = 0;
        for (int q = 0; q < g.world; ++q) {
            const int c = __ldg(gathered + (size_t)q * g.E + e);
            if (c < 0) neg = 1;
            tot += c;
            if (q < g.rank) bef += c;
            if (q == g.rank) my = c;
        }
        S[e] = tot;
        mine[e] = my;
        before[e] = bef;
    }
    __syncthreads();
    if (threadIdx.x < 32) warp_excl_scan(S, g.E);
    else if (threadIdx.x < 64) warp_excl_scan(mine, g.E);
    __syncthreads();
    return neg == 0;
}

// ------------------------------------------------------------------------------------
// Dispatch.  Hazard: the owner reads its received rows until its kb_ep_combine has sent
// them all back; a sender writes them again only in its next dispatch, which follows its
// own combine, which waited for the owner's completed combine send (one arrival per owner,
// made after all of the owner's CTAs finished sending).
// ------------------------------------------------------------------------------------
template <int UNROLL>
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpDev g, const uint4* __restrict__ x,
                                                          int64_t T, const int32_t* __restrict__ p2u,
                                                          const int32_t* __restrict__ gathered,
                                                          int64_t* __restrict__ recv_offsets) {
    pdl_wait();
    extern __shared__ int sm[];
    int* S = sm;                     // [E+1]
    int* mine = S + g.E + 1;         // [E+1]
    int* pos = mine + g.E + 1;       // [E]: before[e], then the row base of expert e
    __shared__ unsigned epoch_s;
    __shared__ int bad, last;
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid == 0) {
        epoch_s = ld_volatile(word(g, g.rank, kDispEpoch));
        bad = ld_volatile(word(g, g.rank, kErr)) != 0u;
    }
    __syncthreads();
    if (bad) return;
    const bool counts_ok = build_tables(g, gathered, S, mine, pos);
    const int Er = g.Er;
    // Received rows of every owner must fit its buffer; a bad count stops the exchange.
    if (tid == 0) {
        bool ok = counts_ok;
        for (int o = 0; o < g.world; ++o)
            ok = ok && (int64_t)(S[(o + 1) * Er] - S[o * Er]) <= g.cap_recv;
        if (!ok) {
            bad = 1;
            if (blockIdx.x == 0) set_err(g, KB_WS_CAPACITY);
        }
    }
    for (int e = tid; e < g.E; e += blockDim.x) pos[e] = S[e] - S[(e / Er) * Er] + pos[e] - mine[e];
    if (blockIdx.x == 0)
        for (int l = tid; l <= Er; l += blockDim.x)
            recv_offsets[l] = (int64_t)(S[g.rank * Er + l] - S[g.rank * Er]);
    __syncthreads();
    pdl_launch();
    if (!bad) {
        // The rows of each owner are one contiguous run of the permuted order.  Warp gw walks
        // the owners starting at gw mod N, so at every moment the warps spread over all
        // owners: NVLink to every peer and this GPU's own HBM are busy together (walking the
        // rows in order would feed one owner at a time).
        const int64_t TK = T * g.K;
        const int warps = gridDim.x * (blockDim.x >> 5);
        const int gw = blockIdx.x * (blockDim.x >> 5) + (tid >> 5);
        for (int oo = 0; oo < g.world; ++oo) {
            const int o = (gw + oo) % g.world;
            const int r1 = mine[(o + 1) * Er];
            for (int r = mine[o * Er] + gw; r < r1; r += warps) {
                const int64_t u = __ldg(p2u + r);
                if (u < 0 || u >= TK) continue;
                const int e = last_le(mine, g.E, r);
                const int64_t dest = (int64_t)pos[e] + r;
                uint4* dst = reinterpret_cast<uint4*>(g.buf[o] + g.recv) + dest * g.vpr;
                warp_copy_row<UNROLL>(x + (u % T) * g.vpr, dst, g.vpr, lane);
            }
        }
    }
    // Count this CTA out; the last one signals every owner, then waits for every sender.
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        last = atomicAdd(word(g, g.rank, kDispTicket), 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && tid == 0) {
        __threadfence_system();
        for (int q = 0; q < g.world; ++q) red_release_sys_add(word(g, q, kDispArrive) + g.rank, 1u);
        if (!wait_arrivals(g, kDispArrive, epoch_s + 1u)) set_err(g, KB_WS_TIMEOUT);
        *reinterpret_cast<volatile unsigned*>(word(g, g.rank, kDispTicket)) = 0u;
        *reinterpret_cast<volatile unsigned*>(word(g, g.rank, kDispEpoch)) = epoch_s + 1u;
    }
}

// ------------------------------------------------------------------------------------
// Combine, part 1: every grouped row back to its sender's permuted position.  Hazard: the
// sender reads its returned rows in part 2 until its finalize is done; an owner writes them
// again only in its next combine, which follows its next dispatch, which waited for that
// sender's next dispatch, which the sender starts after its finalize.
// ------------------------------------------------------------------------------------
template <int UNROLL>
__global__ void __launch_bounds__(256) ep_combine_send_kernel(EpDev g, const uint4* __restrict__ eo,
                                                              const int32_t* __restrict__ gathered) {
    pdl_wait();
    extern __shared__ int sm[];
    const int E = g.E, Er = g.Er, W = g.world, tid = threadIdx.x, lane = tid & 31;
    int* S = sm;                      // [E+1] exclusive scan of the totals
    int* start = S + E + 1;           // [Er][W]: first grouped row of sender q in local expert l
    int* dbase = start + E;           // [Er][W]: sender q's permuted offset of that expert
    int* scan = dbase + E;            // [W][E+1]: exclusive scans of every sender's counts
    __shared__ int bad, last;
    if (tid == 0) bad = ld_volatile(word(g, g.rank, kErr)) != 0u;
    __syncthreads();
    if (bad) return;
    for (int i = tid; i < W * E; i += blockDim.x) {
        const int q = i / E, e = i - q * E;
        const int c = __ldg(gathered + i);
        if (c < 0) bad = 1;
        scan[q * (E + 1) + e] = c;
    }
    __syncthreads();
    if ((tid >> 5) < W) warp_excl_scan(scan + (tid >> 5) * (E + 1), E);
    __syncthreads();
    for (int e = tid; e <= E; e += blockDim.x) {
        int s = 0;
        for (int q = 0; q < W; ++q) s += scan[q * (E + 1) + e];
        S[e] = s;
    }
    __syncthreads();
    const int base = S[g.rank * Er];
    for (int i = tid; i < Er * W; i += blockDim.x) {
        const int l = i / W, q = i - l * W, e = g.rank * Er + l;
        int st = S[e] - base;
        for (int qq = 0; qq < q; ++qq) st += scan[qq * (E + 1) + e + 1] - scan[qq * (E + 1) + e];
        start[i] = st;
        dbase[i] = scan[q * (E + 1) + e];
    }
    __syncthreads();
    pdl_launch();
    if (!bad) {
        const int R = S[(g.rank + 1) * Er] - base;
        const int warps = gridDim.x * (blockDim.x >> 5);
        for (int r = blockIdx.x * (blockDim.x >> 5) + (tid >> 5); r < R; r += warps) {
            const int l = last_le(S + g.rank * Er, Er, r + base);
            int q = 0;
            while (q + 1 < W && start[l * W + q + 1] <= r) ++q;
            const int64_t dest = (int64_t)dbase[l * W + q] + (r - start[l * W + q]);
            if (dest >= g.cap_back) continue;
            uint4* dst = reinterpret_cast<uint4*>(g.buf[q] + g.back) + dest * g.vpr;
            warp_copy_row<UNROLL>(eo + (int64_t)r * g.vpr, dst, g.vpr, lane);
        }
    } else if (blockIdx.x == 0 && tid == 0) {
        set_err(g, KB_WS_CAPACITY);
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        last = atomicAdd(word(g, g.rank, kCombTicket), 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && tid == 0) {
        __threadfence_system();
        for (int q = 0; q < W; ++q) red_release_sys_add(word(g, q, kCombArrive) + g.rank, 1u);
        *reinterpret_cast<volatile unsigned*>(word(g, g.rank, kCombTicket)) = 0u;
    }
}

// Combine, part 2: wait for every owner's rows, then the finalize of kb_moe_finalize on the
// returned rows.
template <typename T, int VPT, int KMAX>
__global__ void __launch_bounds__(512) ep_finalize_kernel(EpDev g, const int32_t* __restrict__ u2p,
                                                          const float* __restrict__ w,
                                                          T* __restrict__ out, int64_t ntok, int H) {
    pdl_wait();
    __shared__ unsigned epoch_s;
    __shared__ int bad, last;
    const int tid = threadIdx.x;
    if (tid == 0) {
        epoch_s = ld_volatile(word(g, g.rank, kCombEpoch));
        bad = ld_volatile(word(g, g.rank, kErr)) != 0u;
        if (!bad && !wait_arrivals(g, kCombArrive, epoch_s + 1u)) {
            set_err(g, KB_WS_TIMEOUT);
            bad = 1;
        }
    }
    __syncthreads();
    pdl_launch();
    if (!bad) {
        const T* back = reinterpret_cast<const T*>(g.buf[g.rank] + g.back);
        for (int64_t t = blockIdx.x; t < ntok; t += gridDim.x)
            finalize_token<T, VPT, KMAX>(back, u2p, w, out, t, ntok, g.K, ntok * g.K, H);
    }
    __syncthreads();
    if (tid == 0) last = atomicAdd(word(g, g.rank, kFinTicket), 1u) == gridDim.x - 1;
    __syncthreads();
    if (last && tid == 0) {
        *reinterpret_cast<volatile unsigned*>(word(g, g.rank, kFinTicket)) = 0u;
        *reinterpret_cast<volatile unsigned*>(word(g, g.rank, kCombEpoch)) = epoch_s + 1u;
    }
}

// Device barrier of the group: one thread signals every rank, then waits for every rank's
// signal of this call.  Work queued behind it on the stream starts on all ranks together.
__global__ void ep_barrier_kernel(EpDev g) {
    pdl_wait();
    if (threadIdx.x != 0) return;
    if (ld_volatile(word(g, g.rank, kErr)) != 0u) return;
    const unsigned epoch = ld_volatile(word(g, g.rank, kEpBarEpoch));
    for (int q = 0; q < g.world; ++q) red_release_sys_add(word(g, q, kEpBarArrive) + g.rank, 1u);
    if (!wait_arrivals(g, kEpBarArrive, epoch + 1u)) set_err(g, KB_WS_TIMEOUT);
    *reinterpret_cast<volatile unsigned*>(word(g, g.rank, kEpBarEpoch)) = epoch + 1u;
}

// ------------------------------------------------------------------------------------
// Host side.
// ------------------------------------------------------------------------------------
int check_group(const kb_ep_group_t* g) {
    if (!g) return KB_ERR_INVALID_ARG;
    if (g->world < 1 || g->world > kMaxRanks || g->rank < 0 || g->rank >= g->world)
        return KB_ERR_INVALID_ARG;
    if (g->num_experts < g->world || g->num_experts > E_MAX || g->num_experts % g->world)
        return KB_ERR_UNSUPPORTED;
    if (g->top_k < 1 || g->top_k > 32 || g->max_tokens < 0 || g->row_bytes <= 0)
        return KB_ERR_INVALID_ARG;
    if (g->row_bytes % 16) return KB_ERR_ALIGNMENT;
    if ((int64_t)g->world * g->max_tokens * g->top_k >= (int64_t)INT32_MAX) return KB_ERR_TOO_LARGE;
    for (int q = 0; q < g->world; ++q) {
        if (!g->buf[q]) return KB_ERR_INVALID_ARG;
        if (reinterpret_cast<uintptr_t>(g->buf[q]) & 255u) return KB_ERR_ALIGNMENT;
    }
    return KB_OK;
}

EpDev make_dev(const kb_ep_group_t* g) {
    const Layout L = layout(g->world, g->num_experts, g->top_k, g->max_tokens, g->row_bytes);
    EpDev d;
    for (int q = 0; q < kMaxRanks; ++q) d.buf[q] = q < g->world ? static_cast<char*>(g->buf[q]) : nullptr;
    d.world = g->world;
    d.rank = g->rank;
    d.E = g->num_experts;
    d.K = g->top_k;
    d.Er = g->num_experts / g->world;
    d.cap_recv = L.cap_recv;
    d.cap_back = L.cap_back;
    d.vpr = g->row_bytes / 16;
    d.recv = L.recv;
    d.back = L.back;
    d.spin = wait_limit(kPeerSpin);
    return d;
}

// CTAs of the row kernels: about eight rows per CTA (one per warp), at most eight CTAs of
// 256 threads per SM (all resident at once).
unsigned row_grid(int64_t rows) {
    const int64_t cap = (int64_t)device_sm_count() * 8;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, cap));
}

// Grid of the finalize: the CTAs that are resident at once (each waits for the arrivals
// once, then walks tokens with a stride of the grid), at most one per token.
template <typename... KArgs>
unsigned resident_grid(void (*kern)(KArgs...), int threads, int64_t ntok) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0) != cudaSuccess ||
        per_sm <= 0)
        per_sm = 1;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ntok, (int64_t)device_sm_count() * per_sm));
}

template <typename T, int KMAX>
int finalize_launch(const EpDev& d, const int32_t* u2p, const float* w, void* out, int64_t ntok,
                    int H, cudaStream_t st) {
    constexpr int N = 16 / sizeof(T);
    const RowShape rs = row_shape(H / N);
#define KB_EPF(V)                                                                              \
    case V:                                                                                    \
        return launch(ep_finalize_kernel<T, V, KMAX>,                                           \
                      dim3(resident_grid(ep_finalize_kernel<T, V, KMAX>, rs.threads, ntok)),    \
                      dim3(rs.threads), 0, st, d, u2p, w, static_cast<T*>(out), ntok, H);
    switch (rs.vpt) {
        KB_EPF(1) KB_EPF(2) KB_EPF(3) KB_EPF(4) KB_EPF(6) KB_EPF(8)
        default: break;
    }
#undef KB_EPF
    return KB_ERR_UNSUPPORTED;
}

template <typename T>
int finalize_k(const EpDev& d, const int32_t* u2p, const float* w, void* out, int64_t ntok,
               int H, cudaStream_t st) {
    if (d.K <= 8) return finalize_launch<T, 8>(d, u2p, w, out, ntok, H, st);
    return finalize_launch<T, 32>(d, u2p, w, out, ntok, H, st);
}

}  // namespace

size_t ep_err_offset() { return kErr; }

int make_count_push(const kb_ep_group_t* g, int32_t* gathered, CountPush* cp) {
    if (const int s = check_group(g)) return s;
    if (!gathered) return KB_ERR_INVALID_ARG;
    *cp = CountPush{};
    for (int q = 0; q < g->world; ++q) cp->buf[q] = static_cast<char*>(g->buf[q]);
    cp->gathered = gathered;
    cp->world = g->world;
    cp->rank = g->rank;
    cp->E = g->num_experts;
    cp->spin = wait_limit(kEpSpin);
    return KB_OK;
}

}  // namespace kb

using namespace kb;

extern "C" size_t kb_ep_buffer_bytes(int world, int E, int K, int64_t max_tokens,
                                     int64_t row_bytes) {
    if (world < 1 || world > kMaxRanks || E < 1 || E > E_MAX || K < 1 || max_tokens < 0 ||
        row_bytes <= 0)
        return 0;
    return layout(world, E, K, max_tokens, row_bytes).total;
}

extern "C" int kb_ep_alloc(size_t bytes, void** buf) {
    if (!buf || bytes == 0) return KB_ERR_INVALID_ARG;
    *buf = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return static_cast<int>(e);
    }
    *buf = p;
    return KB_OK;
}

extern "C" int kb_ep_free(void* buf) {
    if (!buf) return KB_OK;
    return static_cast<int>(cudaFree(buf));
}

extern "C" int kb_ipc_export(const void* buf, void* handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == KB_IPC_HANDLE_BYTES, "IPC handle size");
    if (!buf || !handle) return KB_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(buf));
    if (e != cudaSuccess) return static_cast<int>(e);
    std::memcpy(handle, &h, sizeof(h));
    return KB_OK;
}

extern "C" int kb_ipc_import(const void* handle, void** buf) {
    if (!buf || !handle) return KB_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    *buf = nullptr;
    return static_cast<int>(cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int kb_ipc_close(void* buf) {
    if (!buf) return KB_OK;
    return static_cast<int>(cudaIpcCloseMemHandle(buf));
}

extern "C" int kb_ep_counts_allgather(const kb_ep_group_t* g, const int32_t* counts,
                                      int32_t* gathered, kb_stream_t stream) {
    CountPush cp;
    if (const int s = make_count_push(g, gathered, &cp)) return s;
    if (!counts) return KB_ERR_INVALID_ARG;
    return launch(ep_counts_kernel, dim3(1), dim3(512), 0, static_cast<cudaStream_t>(stream),
                  cp, counts);
}

extern "C" int kb_ep_dispatch(const kb_ep_group_t* g, const void* x, int64_t T, const int32_t* p2u,
                              const int32_t* gathered, int64_t* recv_offsets, kb_stream_t stream) {
    if (const int s = check_group(g)) return s;
    if (T < 0 || T > g->max_tokens) return KB_ERR_INVALID_ARG;
    if (!gathered || !recv_offsets || (T > 0 && (!x || !p2u))) return KB_ERR_INVALID_ARG;
    if (x && !aligned16(x)) return KB_ERR_ALIGNMENT;
    const EpDev d = make_dev(g);
    const size_t smem = (size_t)(3 * d.E + 2) * sizeof(int);
    return launch(ep_dispatch_kernel<4>, dim3(row_grid(T * d.K)), dim3(256), smem,
                  static_cast<cudaStream_t>(stream), d, static_cast<const uint4*>(x), T, p2u,
                  gathered, recv_offsets);
}

extern "C" int kb_ep_recv_rows(const kb_ep_group_t* g, void** rows) {
    if (const int s = check_group(g)) return s;
    if (!rows) return KB_ERR_INVALID_ARG;
    *rows = static_cast<char*>(g->buf[g->rank]) +
            layout(g->world, g->num_experts, g->top_k, g->max_tokens, g->row_bytes).recv;
    return KB_OK;
}

extern "C" int kb_ep_combine(const kb_ep_group_t* g, const void* expert_out, const int32_t* gathered,
                             int64_t T, const int32_t* u2p, const float* weights, void* out,
                             int dtype, kb_stream_t stream) {
    if (const int s = check_group(g)) return s;
    if (T < 0 || T > g->max_tokens) return KB_ERR_INVALID_ARG;
    if (!expert_out || !gathered || (T > 0 && (!u2p || !weights || !out))) return KB_ERR_INVALID_ARG;
    if (!aligned16(expert_out) || (out && !aligned16(out))) return KB_ERR_ALIGNMENT;
    const int esize = dtype == KB_F32 ? 4 : (dtype == KB_BF16 || dtype == KB_F16) ? 2 : 0;
    if (!esize) return KB_ERR_UNSUPPORTED;
    if (g->row_bytes % esize || g->row_bytes / esize > INT32_MAX) return KB_ERR_UNSUPPORTED;
    const int H = (int)(g->row_bytes / esize);
    if (row_shape(H / (16 / esize)).vpt == 0) return KB_ERR_UNSUPPORTED;
    const EpDev d = make_dev(g);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t smem = (size_t)(3 * d.E + 1 + d.world * (d.E + 1)) * sizeof(int);
    int s = launch(ep_combine_send_kernel<4>, dim3(row_grid(g->max_tokens * d.K)), dim3(256), smem,
                   st, d, static_cast<const uint4*>(expert_out), gathered);
    if (s) return s;
    switch (dtype) {
        case KB_BF16: return finalize_k<__nv_bfloat16>(d, u2p, weights, out, T, H, st);
        case KB_F16: return finalize_k<__half>(d, u2p, weights, out, T, H, st);
        default: return finalize_k<float>(d, u2p, weights, out, T, H, st);
    }
}

extern "C" int kb_ep_barrier(const kb_ep_group_t* g, kb_stream_t stream) {
    if (const int s = check_group(g)) return s;
    return launch(ep_barrier_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                  make_dev(g));
}
