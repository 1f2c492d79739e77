// Router projection on the fifth-generation tensor cores, with the routing epilogue fused.
//
// The reference computes the gate as `(x @ W_g).float()` (a bf16 GEMM: fp32 accumulation,
// one rounding to bf16, then widened) and routes the result: s = logits + bias, top-K of s
// (descending, lower expert first among equals), w = sigmoid(logits[id])
// (benchmarks/11_profile_2block_e2e.py:236-246 gate_gemm + R2_moe_prologue;
// benchmarks/01_benchmark_router.py:33-37).  kb_router_gemm does both in one launch:
//
//   mainloop   one CTA per (128-token tile m, expert tile n, hidden split z).  Warp 0 streams
//              x[m-tile, k-block] (128 x 64 bf16) and W[n-tile, k-block] (BN x 64 bf16) into an
//              S-deep shared-memory ring with 2-D tensor copies (128-byte swizzle, rows past T
//              zero-filled); warp 1 issues tcgen05.mma (M = 128, N = BN, K = 16, bf16 inputs,
//              fp32 accumulator in tensor memory) and releases each slot with tcgen05.commit.
//   epilogue   TMEM lane r of the CTA is token m*128 + r; warps w and w + 4 read the two
//              halves of lane quarter w % 4's accumulators with tcgen05.ld into a shared-memory
//              tile, which leaves for global memory as coalesced row segments.  Two forms:
//     cooperative (the grid fits the SMs; T <= 9472 at E = 384; coop_epilogue)
//              the tile goes out rounded to bf16 as the logits, or, with several hidden splits,
//              as fp32 partials; after a grid barrier every CTA sums a share of the partials in
//              split order (independent of timing) and rounds it; after a second barrier one
//              warp per token ranks the whole row with the library's warp router.
//     per tile (more tiles than SMs; one hidden split)
//              each thread ranks its row segment: a 16-column group-maximum threshold, then a
//              register top-K of the candidates, kept sorted by (key desc, expert asc); each
//              tile's K candidates go to the workspace and the last tile of a token tile to
//              finish (a ticket per m) merges them in tile order and writes ids and weights.
//              Exact: every top-K element of the row is a top-K element of its own tile.
//
// Every wait is bounded: a wait that gives up sets the workspace error word, the CTA stops
// issuing work, waits (bounded) for its own tensor copies and frees its tensor memory.
#include "kb_common.cuh"
#include "route_math.cuh"
#include "warp_route.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

namespace kb {
namespace rg {

constexpr int BM = 128;            // tokens per tile (UMMA M)
constexpr int BK = 64;             // hidden elements per k-block: one 128-byte swizzle row
constexpr int UK = 16;             // UMMA K of 16-bit inputs
constexpr int THREADS = 256;       // eight warps: warp w reads TMEM lane quarter w % 4,
                                   // warps 4..7 the second half of each row's columns
constexpr int KMAX = 8;            // largest top-K
constexpr int A_BYTES = BM * BK * 2;
constexpr size_t kSmemCap = 200 * 1024;
constexpr long long kSpin = 1LL << 22;

// Workspace: a zero zone of fixed size (error word, tickets) left zero by every call, then
// scratch.  The zone does not depend on the shape, so calls of different shapes can share one
// workspace: no call's scratch overlaps another call's counters.
constexpr size_t kErrOff = 0;
constexpr size_t kSplitBarOff = 128;   // cooperative path: grid-barrier counter, then exits
constexpr size_t kTicketOff = 256;
constexpr size_t kZeroBytes = 256 * 1024;
constexpr int64_t kMaxTokens = 524288;   // its tickets fit the zero zone at every tile shape

__host__ __device__ constexpr size_t align256(size_t v) { return (v + 255) / 256 * 256; }

struct Plan {
    int bn = 0, n_tiles = 0, ks = 0, kb_per = 0, stages = 0, tmem_cols = 0;
    int coop = 0;   // the grid fits the SMs: cooperative launch, whole-token routing
    int64_t m_tiles = 0;
    size_t smem = 0;
    // workspace layout
    size_t tk_m = 0, zero_bytes = 0, part = 0, lgs = 0, cand = 0, total = 0;
};

// ------------------------------------------------------------------------------------
// Device helpers: mbarriers, tensor copies, tensor-core descriptors and tensor memory.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned su32(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint64_t* b, unsigned n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, unsigned parity) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(su32(b)), "r"(parity) : "memory");
    return done != 0;
}
// Bounded wait for the phase of `parity`; false (error word set) if it did not complete
// within `limit` polls, or as soon as another wait of the launch gave up.
__device__ __forceinline__ bool bar_wait(uint64_t* b, unsigned parity, int* err, long long limit) {
    for (long long it = 0; it < limit; ++it) {
        if (bar_try(b, parity)) return true;
        if ((it & 255) == 255 && *(volatile int*)err) return false;
        if (it > 64) __nanosleep(32);
    }
    atomicExch(err, KB_WS_TIMEOUT);
    return false;
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(b))
        : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by a 128-byte-swizzled tensor
// copy: rows of 128 bytes, 8-row core groups 1024 bytes apart (stride byte offset), leading
// byte offset unused by swizzled K-major layouts (1), descriptor version 1, layout 2 =
// 128-byte swizzle.  The tile base must be 1024-byte aligned; a K step of 16 elements inside
// the swizzle row advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t sw128_desc(unsigned saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}
// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A and B
// (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrives on `b` once every tensor-core operation issued before it by this thread completed.
__device__ __forceinline__ void umma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane (32x32b shape: warp w reads lanes
// 32w..32w+31, lane l of the warp gets lane 32w+l).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
    float r;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// The float whose okey is k (k from okey of a float; the NaN key gives a NaN).
__device__ __forceinline__ float okey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ float bf16_round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

// ------------------------------------------------------------------------------------
// Register top-K of one row, kept sorted by (key desc, expert asc).  Elements are offered in
// ascending expert order (or, when merging, in tile order of sorted lists), so a strict key
// comparison keeps the lower expert first among equal keys.  Key 0 never belongs to a real
// score (okey maps every float, NaN included, to a key >= 0x00800000).
// ------------------------------------------------------------------------------------
struct TopK {
    // positions 0..7 as scalars (never an indexed array, so the list stays in registers)
    uint32_t k0, k1, k2, k3, k4, k5, k6, k7;
    int i0, i1, i2, i3, i4, i5, i6, i7;
    float r0, r1, r2, r3, r4, r5, r6, r7;
    uint32_t thr;   // key of position K-1: an element enters only above it
    __device__ __forceinline__ void init() {
        k0 = k1 = k2 = k3 = k4 = k5 = k6 = k7 = 0u;
        i0 = i1 = i2 = i3 = i4 = i5 = i6 = i7 = 0;
        r0 = r1 = r2 = r3 = r4 = r5 = r6 = r7 = 0.0f;
        thr = 0u;
    }
    __device__ __forceinline__ uint32_t key_at(int j) const {
        switch (j) {
            case 0: return k0; case 1: return k1; case 2: return k2; case 3: return k3;
            case 4: return k4; case 5: return k5; case 6: return k6; default: return k7;
        }
    }
    __device__ __forceinline__ int idx_at(int j) const {
        switch (j) {
            case 0: return i0; case 1: return i1; case 2: return i2; case 3: return i3;
            case 4: return i4; case 5: return i5; case 6: return i6; default: return i7;
        }
    }
    __device__ __forceinline__ float raw_at(int j) const {
        switch (j) {
            case 0: return r0; case 1: return r1; case 2: return r2; case 3: return r3;
            case 4: return r4; case 5: return r5; case 6: return r6; default: return r7;
        }
    }
    // The new element goes before the first smaller key; from there on every element moves
    // down one place (a displaced element must not be compared again: it could fail to pass
    // an equal key with a higher expert and land after it).
    __device__ __forceinline__ void offer(uint32_t k, int i, float r, int K) {
        if (k <= thr) return;
        bool sh = false;
#define KB_TOPK_STEP(KJ, IJ, RJ)                                                     \
        {                                                                            \
            sh = sh || k > KJ;                                                       \
            const uint32_t tk_ = KJ;                                                 \
            const int ti_ = IJ;                                                      \
            const float tr_ = RJ;                                                    \
            if (sh) { KJ = k; IJ = i; RJ = r; k = tk_; i = ti_; r = tr_; }           \
        }
        KB_TOPK_STEP(k0, i0, r0) KB_TOPK_STEP(k1, i1, r1) KB_TOPK_STEP(k2, i2, r2)
        KB_TOPK_STEP(k3, i3, r3) KB_TOPK_STEP(k4, i4, r4) KB_TOPK_STEP(k5, i5, r5)
        KB_TOPK_STEP(k6, i6, r6) KB_TOPK_STEP(k7, i7, r7)
#undef KB_TOPK_STEP
        thr = key_at(K - 1);
    }
};

// The K-th largest 16-column group maximum (as a key) of s = row + bias over a BN-wide
// segment in shared memory (K <= BN / 16).  The K largest maxima are kept sorted in g0..g7.
template <int BN>
__device__ __forceinline__ uint32_t group_tau(const float* row, const float* bias_sm, int K) {
    uint32_t g0 = 0, g1 = 0, g2 = 0, g3 = 0, g4 = 0, g5 = 0, g6 = 0, g7 = 0;
#pragma unroll 1
    for (int g = 0; g < BN / 16; ++g) {
        float sv[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 x = reinterpret_cast<const float4*>(row + 16 * g)[q];
            const float4 b = reinterpret_cast<const float4*>(bias_sm + 16 * g)[q];
            sv[4 * q] = x.x + b.x; sv[4 * q + 1] = x.y + b.y;
            sv[4 * q + 2] = x.z + b.z; sv[4 * q + 3] = x.w + b.w;
        }
        float mx = sv[0];
#pragma unroll
        for (int j = 1; j < 15; j += 2) mx = fmax3_nan(mx, sv[j], sv[j + 1]);
        mx = fmax3_nan(mx, sv[15], sv[15]);
        uint32_t k = okey(mx), o;
        // sorted insertion of a bare key: a max/min ladder
        o = min(k, g0); g0 = max(k, g0); k = o;
        o = min(k, g1); g1 = max(k, g1); k = o;
        o = min(k, g2); g2 = max(k, g2); k = o;
        o = min(k, g3); g3 = max(k, g3); k = o;
        o = min(k, g4); g4 = max(k, g4); k = o;
        o = min(k, g5); g5 = max(k, g5); k = o;
        o = min(k, g6); g6 = max(k, g6); k = o;
        g7 = max(k, g7);
    }
    switch (K) {
        case 1: return g0; case 2: return g1; case 3: return g2; case 4: return g3;
        case 5: return g4; case 6: return g5; case 7: return g6; default: return g7;
    }
}

// Sum of K <= 8 weights in the order of a 32-lane xor butterfly (lanes >= K hold zero), the
// order in which the warp routers renormalise.
__device__ __forceinline__ float butterfly_sum8(const float (&w)[KMAX]) {
    const float b0 = w[0] + w[4], b1 = w[1] + w[5], b2 = w[2] + w[6], b3 = w[3] + w[7];
    return (b0 + b2) + (b1 + b3);
}

__device__ __forceinline__ void write_row(const TopK& tk, int64_t t, int K, int renorm,
                                          int32_t* __restrict__ ids, float* __restrict__ w) {
    float wv[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j) wv[j] = (j < K) ? sigmoid_acc(tk.raw_at(j)) : 0.0f;
    if (renorm) {
        const float inv = 1.0f / (butterfly_sum8(wv) + 1e-20f);
#pragma unroll
        for (int j = 0; j < KMAX; ++j) wv[j] = wv[j] * inv;
    }
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
        if (j < K) {
            ids[t * K + j] = tk.idx_at(j);
            w[t * K + j] = wv[j];
        }
}

struct Args {
    const float* bias;       // [E] or null
    float* logits;           // [T, E] or null
    int32_t* ids;            // [T, K] or null (no routing)
    float* weights;          // [T, K]
    unsigned char* ws;
    int64_t T;
    int E, K, renorm, nkb;   // nkb: k-blocks of the whole hidden dimension
    long long spin;
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Barrier over the whole (co-resident) grid: the arrival counter reaches `target`.  Bounded:
// false (error word set) if it did not within the poll limit or another wait gave up.
__device__ __forceinline__ bool grid_sync(unsigned* cnt, unsigned target, int* err, long long spin,
                                          int* flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        // release: this CTA's stores (ordered before by the CTA barrier) precede the arrival
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
        unsigned v = ld_acquire_gpu(cnt);
        long long it = 0;
        while (v < target && it < spin) {
            if ((it & 255) == 255 && *(volatile int*)err) break;
            if (it > 256) __nanosleep(32);
            v = ld_acquire_gpu(cnt);
            ++it;
        }
        if (v < target) atomicExch(err, KB_WS_TIMEOUT);
        flag[2] = (v >= target) && *(volatile int*)err == 0;
        __threadfence();
    }
    __syncthreads();
    return flag[2] != 0;
}

// A 384-wide row in the warp routers' layout (lane l holds experts 4*(l + 32q) + i), read
// through L2: other CTAs of this launch wrote it.
__device__ __forceinline__ void load_row_cg(const float* row, int lane, float (&x)[12]) {
#pragma unroll
    for (int q = 0; q < 3; ++q) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(row) + lane + 32 * q);
        x[4 * q] = v.x; x[4 * q + 1] = v.y; x[4 * q + 2] = v.z; x[4 * q + 3] = v.w;
    }
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 ::"r"(su32(smem_dst)), "l"(gmem_src) : "memory");
}

// The epilogue of a cooperative launch (every CTA resident: the grid fits the SMs).
//   1. the CTA's tile goes from TMEM to shared memory (rounded to bf16 when the hidden
//      dimension is not split) and from there, row segments coalesced, to global memory: the
//      logits (or the workspace when the caller wants none), or with several hidden splits
//      the fp32 partial part[z][t][e]
//   2. (several splits) grid barrier; each CTA sums a contiguous share of the [T][E] logits
//      over the splits in split order (so the sum does not depend on timing): cp.async copies
//      gather all splits of a chunk into shared memory at once, one thread per float4 adds
//      them up, rounds to bf16 and stores
//   3. grid barrier; one warp per token ranks the whole row with the library's warp router
//      (route_fast; route_exact when it cannot decide: the order of torch.sort) and weighs
//      the picks with pick_weight, the next token's row loaded while this one is ranked
//   4. the last CTA out resets the barrier counters
__device__ __forceinline__ void coop_epilogue(const Args& a, const Plan& p, uint32_t trow, int r,
                                             int64_t m0, int z, int n0, int* flag, float* red,
                                             int rs, size_t region) {
    const int E = a.E, K = a.K;
    int* err = reinterpret_cast<int*>(a.ws + kErrOff);
    unsigned* bar = reinterpret_cast<unsigned*>(a.ws + kSplitBarOff);
    unsigned* leave = bar + 1;
    float* part = reinterpret_cast<float*>(a.ws + p.part);
    float* out = a.logits ? a.logits : reinterpret_cast<float*>(a.ws + p.lgs);
    const int bn = p.bn;
    const bool split = p.ks > 1;
    const int half = bn / 2, c_lo = (int)(threadIdx.x >> 7) * half;
#pragma unroll 1
    for (int c = c_lo; c < c_lo + half; c += 32) {
        float v[32];
        tmem_ld32(trow + (uint32_t)c, v);
        if (!split) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);
        }
        float4* srow = reinterpret_cast<float4*>(red + r * rs + c);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            srow[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    __syncthreads();
    {
        const int rows = (int)(a.T - m0 < BM ? a.T - m0 : (int64_t)BM);
        const int q4 = bn / 4;
        float* dst = split ? part + (int64_t)z * a.T * E : out;
        for (int i = threadIdx.x; i < rows * q4; i += THREADS) {
            const int rr = i / q4, qq = i - rr * q4;
            reinterpret_cast<float4*>(dst + (m0 + rr) * E + n0)[qq] =
                reinterpret_cast<const float4*>(red + rr * rs)[qq];
        }
    }
    const unsigned G = gridDim.x * gridDim.y * gridDim.z;
    const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (!grid_sync(bar, G, err, a.spin, flag)) return;

    if (split) {
        const int64_t n4 = a.T * (int64_t)E / 4;
        const int64_t per = (n4 + G - 1) / G;
        const int64_t lo = (int64_t)cta * per, hi = min(n4, lo + per);
        const float4* p4 = reinterpret_cast<const float4*>(part);
        float4* buf = reinterpret_cast<float4*>(red);   // the tile is in global memory now
        const int64_t chunk = (int64_t)(region / (16 * (size_t)p.ks));
        for (int64_t c0 = lo; c0 < hi; c0 += chunk) {
            const int nch = (int)min(chunk, hi - c0);
            for (int q = threadIdx.x; q < nch * p.ks; q += THREADS) {
                const int zz = q / nch, ii = q - zz * nch;
                cp_async16(buf + q, p4 + (int64_t)zz * n4 + c0 + ii);
            }
            asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
            __syncthreads();
            for (int ii = threadIdx.x; ii < nch; ii += THREADS) {
                float4 acc = buf[ii];
                for (int zz = 1; zz < p.ks; ++zz) {
                    const float4 v = buf[zz * nch + ii];
                    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                }
                reinterpret_cast<float4*>(out)[c0 + ii] =
                    make_float4(bf16_round(acc.x), bf16_round(acc.y), bf16_round(acc.z),
                                bf16_round(acc.w));
            }
            __syncthreads();
        }
        if (!grid_sync(bar, 2 * G, err, a.spin, flag)) return;
    }

    if (a.ids) {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        int* sel = reinterpret_cast<int*>(red) + warp * 32;   // per-warp pick scratch
        const int64_t nw = (int64_t)G * (THREADS / 32);
        int64_t tt = (int64_t)cta * (THREADS / 32) + warp;
        if (E == 384 && K <= 8) {
            // E = 384: 12 experts per lane as three float4 (expert 4*(lane + 32q) + i)
            float b[12];
            load_bias<12, true>(a.bias, E, lane, b);
            float nxt[12];
            if (tt < a.T) load_row_cg(out + tt * E, lane, nxt);
            for (; tt < a.T; tt += nw) {
                float sv[12];
#pragma unroll
                for (int j = 0; j < 12; ++j) sv[j] = nxt[j] + b[j];
                const float* row = out + tt * E;
                if (tt + nw < a.T) load_row_cg(out + (tt + nw) * E, lane, nxt);
                const bool done = K == 6 ? route_fast<12, 6>(sv, K, lane, sel)
                                         : route_fast<12, 0>(sv, K, lane, sel);
                if (!done) route_exact<12, true>(row, a.bias, E, K, lane, sel);
                const int id = lane < K ? sel[lane] : 0;
                const float wv = pick_weight(lane < K ? row[id] : 0.0f, K, lane, a.renorm);
                if (lane < K) {
                    a.ids[tt * K + lane] = id;
                    a.weights[tt * K + lane] = wv;
                }
                __syncwarp();
            }
        } else {
            for (; tt < a.T; tt += nw) {
                const float* row = out + tt * E;
                route_exact<16, false>(row, a.bias, E, K, lane, sel);
                const int id = lane < K ? sel[lane] : 0;
                const float wv = pick_weight(lane < K ? row[id] : 0.0f, K, lane, a.renorm);
                if (lane < K) {
                    a.ids[tt * K + lane] = id;
                    a.weights[tt * K + lane] = wv;
                }
                __syncwarp();
            }
        }
    }
    // the last CTA out resets the counters (every CTA has passed the barriers by then)
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atomicAdd(leave, 1u) == G - 1) {
            atomicExch(bar, 0u);
            atomicExch(leave, 0u);
        }
    }
}

// ------------------------------------------------------------------------------------
// The kernel.  grid = (m_tiles, n_tiles, ks); BN experts per tile; S ring slots.
// ------------------------------------------------------------------------------------
template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
router_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                   const Args a, const Plan p) {
    constexpr int B_BYTES = BN * BK * 2;
    constexpr int STAGE = A_BYTES + B_BYTES;
    constexpr uint32_t IDESC = f16_idesc(BM, BN);
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    // the ring, and after the mainloop the split-sum tile, then the barriers
    const size_t region = max((size_t)S * STAGE, (size_t)BM * (BN + 4) * sizeof(float));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + region);
    uint64_t* empty = full + S;
    uint64_t* accum = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    int* flag = reinterpret_cast<int*>(tmem_slot + 1);
    // the bias tile is read as float4: 16-byte aligned
    float* bias_sm = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(flag + 4) + 15) & ~uintptr_t(15));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m = blockIdx.x;
    const int n = blockIdx.y, z = blockIdx.z;
    const int64_t m0 = m * BM;
    const int n0 = n * BN;
    const int kb0 = z * p.kb_per;
    const int nkb = min(p.kb_per, a.nkb - kb0);
    int* err = reinterpret_cast<int*>(a.ws + kErrOff);

    if (warp == 0 && lane == 0) {
        prefetch_map(&tmx);
        prefetch_map(&tmw);
        for (int s = 0; s < S; ++s) { bar_init(full + s, 1); bar_init(empty + s, 1); }
        bar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(su32(tmem_slot)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_wait();   // x (and possibly the bias) come from earlier kernels
    for (int j = threadIdx.x; j < BN; j += THREADS)
        bias_sm[j] = a.bias ? a.bias[n0 + j] + 0.0f : 0.0f;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const bool dead = *(volatile int*)err != 0;   // a poisoned workspace: no work at all
    if (warp == 0 && lane == 0 && !dead) {
        // producer
        int issued = 0;
        for (int i = 0; i < nkb; ++i) {
            const int s = i % S;
            if (i >= S && !bar_wait(empty + s, (unsigned)(((i / S) - 1) & 1), err, a.spin)) break;
            unsigned char* st = sm + (size_t)s * STAGE;
            bar_expect_tx(full + s, STAGE);
            tma_2d(st, &tmx, (kb0 + i) * BK, (int)m0, full + s);
            tma_2d(st + A_BYTES, &tmw, (kb0 + i) * BK, n0, full + s);
            issued = i + 1;
        }
        // every copy issued must have landed before the CTA leaves (normally the MMA warp
        // consumed them all already; this only waits after an error)
        for (int i = max(0, issued - S); i < issued; ++i) {
            const int s = i % S;
            for (long long it = 0; it < kSpin && !bar_try(full + s, (unsigned)((i / S) & 1)); ++it)
                __nanosleep(32);
        }
    } else if (warp == 1 && lane == 0 && !dead) {
        // tensor-core issue
        for (int i = 0; i < nkb; ++i) {
            const int s = i % S;
            if (!bar_wait(full + s, (unsigned)((i / S) & 1), err, a.spin)) break;
            tc_fence_after();
            const unsigned sa = su32(sm + (size_t)s * STAGE);
            const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + A_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / UK; ++kk)
                umma_bf16(tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), IDESC,
                          (i | kk) != 0 ? 1u : 0u);
            umma_commit(empty + s);
        }
        umma_commit(accum);   // all MMAs above complete (or none were issued)
    }
    __syncwarp();

    // ---------------- epilogue: thread r = TMEM lane r = token m0 + r ----------------
    const int r = threadIdx.x & (BM - 1);          // TMEM lane = token row of the tile
    const int ch = threadIdx.x >> 7;               // which half of the row's columns
    const int64_t t = m0 + r;
    const bool valid = t < a.T;
    bool ok = !dead && bar_wait(accum, 0u, err, a.spin);
    tc_fence_after();
    ok = __syncthreads_and(ok) != 0;
    pdl_launch();
    const int E = a.E, K = a.K;
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    constexpr int RS = BN + 4;                     // padded row stride of the tile (floats)
    float* red = reinterpret_cast<float*>(sm);     // the tile's logits [BM][RS] (ring is free)
    bool have = false;                             // red holds the rounded tile (per-tile path)

    if (ok && p.coop) {
        // the grid fits the SMs: tokens are routed whole after a grid barrier
        coop_epilogue(a, p, trow, r, m0, z, n0, flag, red, RS, region);
        ok = false;
    } else if (ok) {
        // one hidden split, more tiles than SMs: TMEM -> bf16-rounded row in shared memory
#pragma unroll 1
        for (int c = ch * (BN / 2); c < (ch + 1) * (BN / 2); c += 32) {
            float v[32];
            tmem_ld32(trow + (uint32_t)c, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);
            float4* srow = reinterpret_cast<float4*>(red + r * RS + c);
#pragma unroll
            for (int q = 0; q < 8; ++q)
                srow[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        have = true;
    }
    __syncthreads();   // the tile in shared memory is complete
    if (have && a.logits) {   // the rounded logits, row segments stored coalesced
        const int rows = (int)(a.T - m0 < BM ? a.T - m0 : (int64_t)BM);
        constexpr int Q4 = BN / 4;
        for (int i = threadIdx.x; i < rows * Q4; i += THREADS) {
            const int rr = i / Q4, qq = i - rr * Q4;
            reinterpret_cast<float4*>(a.logits + (m0 + rr) * E + n0)[qq] =
                reinterpret_cast<const float4*>(red + rr * RS)[qq];
        }
    }

    // ---------------- per-tile path: rank this thread's row segment ----------------
    // tau = the K-th largest 16-column group maximum of s = logit + bias: each of those K
    // groups holds an element >= tau, so every top-K element is >= tau (a lower bound; all
    // elements pass when the segment has fewer than K groups).  Only elements >= tau (and NaN,
    // which ranks first) enter the register top-K, in ascending column order.
    TopK tk;
    tk.init();
    const bool have_row = have && a.ids && valid && ch == 0;   // one thread per row ranks
    if (have_row) {
        const float* row = red + r * RS;
        const uint32_t tau = (BN / 16 >= K) ? group_tau<BN>(row, bias_sm, K) : 0u;
        const float tf = tau == 0u ? -INFINITY : okey_inv(tau);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            unsigned mask = 0u;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 x = reinterpret_cast<const float4*>(row + c)[q];
                const float4 b = reinterpret_cast<const float4*>(bias_sm + c)[q];
                const float s0 = x.x + b.x, s1 = x.y + b.y, s2 = x.z + b.z, s3 = x.w + b.w;
                mask |= (unsigned)((s0 >= tf) | (s0 != s0)) << (4 * q);
                mask |= (unsigned)((s1 >= tf) | (s1 != s1)) << (4 * q + 1);
                mask |= (unsigned)((s2 >= tf) | (s2 != s2)) << (4 * q + 2);
                mask |= (unsigned)((s3 >= tf) | (s3 != s3)) << (4 * q + 3);
            }
            while (mask) {
                const int j = c + __ffs(mask) - 1;
                mask &= mask - 1u;
                const float v = row[j];
                tk.offer(okey(v + bias_sm[j]), n0 + j, v, K);
            }
        }
    }

    // ---------------- per-tile path: merge the expert tiles, write ids / weights ----------
    if (have && a.ids) {
        if (p.n_tiles == 1) {
            if (have_row) write_row(tk, t, K, a.renorm, a.ids, a.weights);
        } else {
            uint64_t* ck = reinterpret_cast<uint64_t*>(a.ws + p.cand);
            float* cr = reinterpret_cast<float*>(ck + (size_t)p.n_tiles * a.T * K);
            if (have_row) {
                const int64_t o = ((int64_t)n * a.T + t) * K;
#pragma unroll
                for (int j = 0; j < KMAX; ++j)
                    if (j < K) {
                        ck[o + j] = ((uint64_t)tk.key_at(j) << 32) | (uint32_t)tk.idx_at(j);
                        cr[o + j] = tk.raw_at(j);
                    }
            }
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                int* tkt = reinterpret_cast<int*>(a.ws + p.tk_m) + m;
                const int old = atomicAdd(tkt, 1);
                const bool last = old == p.n_tiles - 1;
                if (last) *tkt = 0;
                flag[1] = last;
            }
            __syncthreads();
            if (flag[1] && valid && ch == 0) {
                __threadfence();
                TopK f;
                f.init();
#pragma unroll 1
                for (int nn = 0; nn < p.n_tiles; ++nn) {
                    // the tile's K candidates are loaded together (one round trip per tile)
                    const int64_t o = ((int64_t)nn * a.T + t) * K;
                    uint64_t cv[KMAX];
                    float rv[KMAX];
#pragma unroll
                    for (int j = 0; j < KMAX; ++j)
                        if (j < K) { cv[j] = __ldcg(ck + o + j); rv[j] = __ldcg(cr + o + j); }
#pragma unroll
                    for (int j = 0; j < KMAX; ++j)
                        if (j < K) f.offer((uint32_t)(cv[j] >> 32), (int)(uint32_t)cv[j], rv[j], K);
                }
                write_row(f, t, K, a.renorm, a.ids, a.weights);
            }
        }
    }

    // Before its tensor memory is freed, every MMA the CTA issued must have completed: the
    // MMA thread always commits to `accum`, so after an epilogue wait that gave up this waits
    // for that phase (bounded by the default limit, not the caller's).
    if (!dead && threadIdx.x == 64)
        for (long long it = 0; it < kSpin && !bar_try(accum, 0u); ++it) __nanosleep(32);
    tc_fence_before();
    __syncthreads();
    if (warp == 2)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     ::"r"(tmem), "r"(p.tmem_cols) : "memory");
}

// ------------------------------------------------------------------------------------
// Host side.
// ------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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
    return encode;
}

// 2-D map of a bf16 [rows][H] matrix with 64 x box_rows boxes and the 128-byte swizzle;
// rows past `rows` read as zero.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int H, int box_rows) {
    auto encode = encoder();
    if (!encode) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)H * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

// Tile shape and hidden split for T tokens: enough CTAs to cover the SMs, every split a
// whole number of k-blocks.  KB_RGEMM_BN / KB_RGEMM_KS force a shape (tests).
bool make_plan(Plan& p, int64_t T, int H, int E, int K, int sms) {
    const int nkb = H / BK;
    p.m_tiles = (T + BM - 1) / BM;
    int bn = env_int("KB_RGEMM_BN", 0);
    int ks = env_int("KB_RGEMM_KS", 0);
    if (bn == 0)   // the widest tile: the fewest re-reads of x and of the gate weight
        bn = E % 192 == 0 ? 192 : E % 128 == 0 ? 128 : 64;
    if (bn != 64 && bn != 128 && bn != 192 && bn != 256) return false;
    if (E % bn != 0) return false;
    p.bn = bn;
    p.n_tiles = E / bn;
    if (ks == 0) {
        const int64_t tiles = p.m_tiles * p.n_tiles;
        const int want = (int)std::max<int64_t>(1, sms / std::max<int64_t>(1, tiles));
        ks = 1;
        for (int d = 1; d <= nkb; ++d)   // largest divisor of nkb not above want
            if (nkb % d == 0 && d <= want) ks = d;
    }
    ks = std::max(1, std::min(ks, nkb));
    // several splits run as one cooperative launch of at most one CTA per SM
    const int64_t tiles = p.m_tiles * p.n_tiles;
    if (ks > 1 && tiles * ks > sms) ks = (int)std::max<int64_t>(1, sms / tiles);
    p.ks = ks;
    p.kb_per = (nkb + ks - 1) / ks;
    p.ks = (nkb + p.kb_per - 1) / p.kb_per;   // no empty split
    // a grid that fits the SMs routes whole tokens after a grid barrier (KB_RGEMM_COOP=0
    // forces the per-tile path when the hidden dimension is not split: tests)
    p.coop = (tiles * p.ks <= sms && (p.ks > 1 || env_int("KB_RGEMM_COOP", 1) != 0)) ? 1 : 0;
    const size_t stage = (size_t)A_BYTES + (size_t)bn * BK * 2;
    p.stages = (int)std::max<size_t>(2, std::min<size_t>((size_t)p.kb_per, kSmemCap / stage));
    p.stages = std::min(p.stages, 8);
    const size_t ring = (size_t)p.stages * stage;
    const size_t red = (size_t)BM * (bn + 4) * sizeof(float);
    p.smem = 1024 + std::max(ring, red) + (size_t)(2 * p.stages + 1) * 8 + 4 + 16 + 16 +
             (size_t)bn * sizeof(float);
    p.tmem_cols = bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
    // workspace
    p.tk_m = kTicketOff;   // per token tile: expert tiles merged (per-tile epilogue)
    p.zero_bytes = kZeroBytes;
    if (p.tk_m + (size_t)p.m_tiles * sizeof(int) > kZeroBytes) return false;   // T too large
    p.part = p.zero_bytes;
    const size_t part_bytes = p.ks > 1 ? align256((size_t)p.ks * T * E * sizeof(float)) : 0;
    p.lgs = p.part + part_bytes;
    const size_t lgs_bytes = p.coop ? align256((size_t)T * E * sizeof(float)) : 0;
    p.cand = p.lgs + lgs_bytes;
    const size_t cand_bytes =
        (!p.coop && p.n_tiles > 1)
            ? align256((size_t)p.n_tiles * T * K * (sizeof(uint64_t) + sizeof(float))) : 0;
    p.total = p.cand + cand_bytes;
    (void)K;
    return true;
}

template <int BN>
int launch_bn(const CUtensorMap& mx, const CUtensorMap& mw, const Args& a, const Plan& p,
              cudaStream_t stream) {
    auto kern = router_gemm_kernel<BN>;
    static std::once_flag once;
    static int attr_err = 0;
    std::call_once(once, [&] {
        attr_err = static_cast<int>(cudaFuncSetAttribute(
            kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    });
    if (attr_err) return attr_err;
    const dim3 grid((unsigned)p.m_tiles, (unsigned)p.n_tiles, (unsigned)p.ks);
    if (!p.coop) return launch(kern, grid, dim3(THREADS), p.smem, stream, mx, mw, a, p);
    // the CTAs wait for one another at grid barriers: a cooperative launch guarantees that
    // every CTA is resident (the plan keeps the grid within one CTA per SM)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, mx, mw, a, p));
}

}  // namespace rg
}  // namespace kb

using namespace kb;

extern "C" size_t kb_router_gemm_workspace_bytes(int64_t T, int H, int E, int K) {
    rg::Plan p;
    if (T <= 0 || H <= 0 || E <= 0 || K <= 0 || K > rg::KMAX) return 256;
    if (!rg::make_plan(p, T, H, E, K, device_sm_count())) return 256;
    return p.total;
}

extern "C" int kb_router_gemm(const void* x, const void* w_gate, const float* bias, float* logits,
                              int32_t* ids, float* weights, void* workspace, size_t ws_bytes,
                              int64_t T, int H, int E, int K, int renorm, kb_stream_t stream) {
    if (T < 0 || H <= 0 || E <= 0) return KB_ERR_INVALID_ARG;
    if (!x || !w_gate || !workspace) return KB_ERR_INVALID_ARG;
    if (ids && (!weights || K <= 0)) return KB_ERR_INVALID_ARG;
    if (!ids && !logits) return KB_ERR_INVALID_ARG;   // nothing to produce
    if (ids && K > rg::KMAX) return KB_ERR_UNSUPPORTED;
    if (ids && K > E) return KB_ERR_UNSUPPORTED;
    if (H % rg::BK != 0 || E % 64 != 0 || E > 512) return KB_ERR_UNSUPPORTED;
    if (T > rg::kMaxTokens) return KB_ERR_TOO_LARGE;
    if (!aligned16(x) || !aligned16(w_gate) || (logits && !aligned16(logits)) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return KB_ERR_ALIGNMENT;
    if (T == 0) return KB_OK;
    rg::Plan p;
    const int Kp = ids ? K : 1;
    if (!rg::make_plan(p, T, H, E, Kp, device_sm_count())) return KB_ERR_UNSUPPORTED;
    if (ws_bytes < p.total) return KB_ERR_WORKSPACE;
    CUtensorMap mx, mw;
    if (!rg::make_map(&mx, x, T, H, rg::BM) || !rg::make_map(&mw, w_gate, E, H, p.bn))
        return KB_ERR_UNSUPPORTED;
    rg::Args a;
    a.bias = bias;
    a.logits = logits;
    a.ids = ids;
    a.weights = weights;
    a.ws = static_cast<unsigned char*>(workspace);
    a.T = T;
    a.E = E;
    a.K = Kp;
    a.renorm = renorm ? 1 : 0;
    a.nkb = H / rg::BK;
    a.spin = wait_limit(rg::kSpin);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (p.bn) {
        case 64: return rg::launch_bn<64>(mx, mw, a, p, st);
        case 128: return rg::launch_bn<128>(mx, mw, a, p, st);
        case 192: return rg::launch_bn<192>(mx, mw, a, p, st);
        case 256: return rg::launch_bn<256>(mx, mw, a, p, st);
        default: return KB_ERR_UNSUPPORTED;
    }
}

extern "C" int kb_router_gemm_describe(int64_t T, int H, int E, int K, int* bn, int* ks,
                                       int* grid) {
    rg::Plan p;
    if (T <= 0 || H <= 0 || E <= 0 || H % rg::BK != 0) return KB_ERR_INVALID_ARG;
    if (!rg::make_plan(p, T, H, E, K > 0 ? K : 1, device_sm_count())) return KB_ERR_UNSUPPORTED;
    if (bn) *bn = p.bn;
    if (ks) *ks = p.ks;
    if (grid) *grid = (int)(p.m_tiles * p.n_tiles * p.ks);
    return KB_OK;
}
