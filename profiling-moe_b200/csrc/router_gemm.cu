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
//   epilogue   thread r of the CTA owns TMEM lane r = token m*128 + r and reads its BN
//              accumulators with tcgen05.ld.  With one hidden split they are rounded to bf16
//              at once; with several, each split stores its fp32 partial tile and the last
//              split to finish (an atomic ticket per (m, n)) sums the partials in split order,
//              so the result does not depend on which CTA finishes first.  The rounded logits
//              are stored (optional), and each thread ranks its row segment: a register top-K
//              of keys (score order, NaN first) kept sorted by (key desc, expert asc).
//   merge      with several expert tiles, each tile's K candidates go to the workspace and the
//              last tile of a token tile to finish (a ticket per m) merges them in tile order
//              and writes ids and weights.  Exact: every top-K element of the row is a top-K
//              element of its own tile.
//
// Every wait is bounded: a wait that gives up sets the workspace error word, the CTA stops
// issuing work, waits (bounded) for its own tensor copies and frees its tensor memory.
#include "kb_common.cuh"
#include "route_math.cuh"

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
constexpr int THREADS = 128;       // four warps: TMEM lane quarters 0..3
constexpr int KMAX = 8;            // largest top-K
constexpr int A_BYTES = BM * BK * 2;
constexpr size_t kSmemCap = 200 * 1024;
constexpr long long kSpin = 1LL << 22;

// Workspace: a zero zone of fixed size (error word, tickets) left zero by every call, then
// scratch.  The zone does not depend on the shape, so calls of different shapes can share one
// workspace: no call's scratch overlaps another call's counters.
constexpr size_t kErrOff = 0;
constexpr size_t kTicketOff = 256;
constexpr size_t kZeroBytes = 256 * 1024;
constexpr int64_t kMaxTokens = 524288;   // its tickets fit the zero zone at every tile shape

__host__ __device__ constexpr size_t align256(size_t v) { return (v + 255) / 256 * 256; }

struct Plan {
    int bn = 0, n_tiles = 0, ks = 0, kb_per = 0, stages = 0, tmem_cols = 0;
    int64_t m_tiles = 0;
    size_t smem = 0;
    // workspace layout
    size_t tk_mn = 0, tk_m = 0, zero_bytes = 0, part = 0, cand = 0, total = 0;
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
    uint32_t key[KMAX];
    int idx[KMAX];
    float raw[KMAX];
    uint32_t thr;   // key of position K-1: an element enters only above it
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int j = 0; j < KMAX; ++j) { key[j] = 0u; idx[j] = 0; raw[j] = 0.0f; }
        thr = 0u;
    }
    __device__ __forceinline__ void offer(uint32_t k, int i, float r, int K) {
        if (k <= thr) return;
        // the new element goes before the first smaller key; from there on every element
        // moves down one place (a displaced element must not be compared again: it could
        // fail to pass an equal key with a higher expert and land after it)
        bool shift = false;
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
            shift = shift || k > key[j];
            const uint32_t tk = key[j];
            const int ti = idx[j];
            const float tr = raw[j];
            if (shift) { key[j] = k; idx[j] = i; raw[j] = r; k = tk; i = ti; r = tr; }
        }
#pragma unroll
        for (int j = 0; j < KMAX; ++j)
            if (j == K - 1) thr = key[j];
    }
};

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
    for (int j = 0; j < KMAX; ++j) wv[j] = (j < K) ? sigmoid_acc(tk.raw[j]) : 0.0f;
    if (renorm) {
        const float inv = 1.0f / (butterfly_sum8(wv) + 1e-20f);
#pragma unroll
        for (int j = 0; j < KMAX; ++j) wv[j] = wv[j] * inv;
    }
#pragma unroll
    for (int j = 0; j < KMAX; ++j)
        if (j < K) {
            ids[t * K + j] = tk.idx[j];
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
    float* bias_sm = reinterpret_cast<float*>(flag + 4);

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
    const int r = threadIdx.x;
    const int64_t t = m0 + r;
    const bool valid = t < a.T;
    bool ok = !dead && bar_wait(accum, 0u, err, a.spin);
    tc_fence_after();
    ok = __syncthreads_and(ok) != 0;
    pdl_launch();
    const int E = a.E, K = a.K;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    TopK tk;
    tk.init();
    bool have_row = false;   // tk holds this row's tile candidates

    if (ok && p.ks == 1) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(trow + (uint32_t)c, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = bf16_round(v[j]);
            if (valid) {
                if (a.logits) {
                    float4* dst = reinterpret_cast<float4*>(a.logits + t * E + n0 + c);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                }
                if (a.ids) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        tk.offer(okey(v[j] + bias_sm[c + j]), n0 + c + j, v[j], K);
                }
            }
        }
        have_row = valid && a.ids;
    } else if (ok) {
        // several hidden splits: store this split's fp32 partial, the last split sums them
        float* part = reinterpret_cast<float*>(a.ws + p.part);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(trow + (uint32_t)c, v);
            if (valid) {
                float4* dst = reinterpret_cast<float4*>(part + ((int64_t)z * a.T + t) * E + n0 + c);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            int* tkt = reinterpret_cast<int*>(a.ws + p.tk_mn) + m * p.n_tiles + n;
            const int old = atomicAdd(tkt, 1);
            const bool last = old == p.ks - 1;
            if (last) *tkt = 0;   // left zero for the next call
            flag[0] = last;
        }
        __syncthreads();
        if (flag[0]) {
            __threadfence();
            // cooperative, coalesced sum of the ks partial tiles (split order) into shared
            // memory (the ring is free: every MMA completed), rounded to bf16
            const int rows = (int)(a.T - m0 < BM ? a.T - m0 : (int64_t)BM);
            constexpr int Q = BN / 4;              // float4 per row segment
            constexpr int RS = BN + 4;             // padded row stride (floats)
            float* red = reinterpret_cast<float*>(sm);
            for (int e4 = threadIdx.x; e4 < rows * Q; e4 += THREADS) {
                const int rr = e4 / Q, qq = e4 % Q;
                const float* src = part + (m0 + rr) * E + n0 + 4 * qq;
                const int64_t zs = a.T * (int64_t)E;
                float4 acc = __ldcg(reinterpret_cast<const float4*>(src));
                int zz = 1;
                for (; zz + 4 <= p.ks; zz += 4) {
                    const float4 v1 = __ldcg(reinterpret_cast<const float4*>(src + zz * zs));
                    const float4 v2 = __ldcg(reinterpret_cast<const float4*>(src + (zz + 1) * zs));
                    const float4 v3 = __ldcg(reinterpret_cast<const float4*>(src + (zz + 2) * zs));
                    const float4 v4 = __ldcg(reinterpret_cast<const float4*>(src + (zz + 3) * zs));
                    acc.x = (((acc.x + v1.x) + v2.x) + v3.x) + v4.x;
                    acc.y = (((acc.y + v1.y) + v2.y) + v3.y) + v4.y;
                    acc.z = (((acc.z + v1.z) + v2.z) + v3.z) + v4.z;
                    acc.w = (((acc.w + v1.w) + v2.w) + v3.w) + v4.w;
                }
                for (; zz < p.ks; ++zz) {
                    const float4 v1 = __ldcg(reinterpret_cast<const float4*>(src + zz * zs));
                    acc.x += v1.x; acc.y += v1.y; acc.z += v1.z; acc.w += v1.w;
                }
                acc = make_float4(bf16_round(acc.x), bf16_round(acc.y), bf16_round(acc.z),
                                  bf16_round(acc.w));
                *reinterpret_cast<float4*>(red + rr * RS + 4 * qq) = acc;
                if (a.logits)
                    *reinterpret_cast<float4*>(a.logits + (m0 + rr) * E + n0 + 4 * qq) = acc;
            }
            __syncthreads();
            if (valid && a.ids) {
                const float* row = red + r * RS;
#pragma unroll 4
                for (int j = 0; j < BN; ++j) tk.offer(okey(row[j] + bias_sm[j]), n0 + j, row[j], K);
                have_row = true;
            }
        } else {
            ok = false;   // another split finishes this tile
        }
    }

    // ---------------- merge the expert tiles and write ids / weights ----------------
    if (ok && a.ids) {
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
                        ck[o + j] = ((uint64_t)tk.key[j] << 32) | (uint32_t)tk.idx[j];
                        cr[o + j] = tk.raw[j];
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
            if (flag[1] && valid) {
                __threadfence();
                TopK f;
                f.init();
                for (int nn = 0; nn < p.n_tiles; ++nn) {
                    const int64_t o = ((int64_t)nn * a.T + t) * K;
                    for (int j = 0; j < K; ++j) {
                        const uint64_t c = __ldcg(ck + o + j);
                        f.offer((uint32_t)(c >> 32), (int)(uint32_t)c, __ldcg(cr + o + j), K);
                    }
                }
                write_row(f, t, K, a.renorm, a.ids, a.weights);
            }
        }
    }

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
    if (bn == 0) {
        if (E % 192 == 0 && p.m_tiles * (E / 192) >= sms / 2) bn = 192;
        else if (E % 128 == 0 && p.m_tiles * (E / 128) >= sms / 2) bn = 128;
        else bn = 64;
    }
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
    p.ks = ks;
    p.kb_per = (nkb + ks - 1) / ks;
    p.ks = (nkb + p.kb_per - 1) / p.kb_per;   // no empty split
    const size_t stage = (size_t)A_BYTES + (size_t)bn * BK * 2;
    p.stages = (int)std::max<size_t>(2, std::min<size_t>((size_t)p.kb_per, kSmemCap / stage));
    p.stages = std::min(p.stages, 8);
    const size_t ring = (size_t)p.stages * stage;
    const size_t red = (size_t)BM * (bn + 4) * sizeof(float);
    p.smem = 1024 + std::max(ring, red) + (size_t)(2 * p.stages + 1) * 8 + 4 + 16 +
             (size_t)bn * sizeof(float);
    p.tmem_cols = bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
    // workspace
    p.tk_mn = kTicketOff;
    p.tk_m = p.tk_mn + (size_t)p.m_tiles * p.n_tiles * sizeof(int);
    p.zero_bytes = kZeroBytes;
    if (p.tk_m + (size_t)p.m_tiles * sizeof(int) > kZeroBytes) return false;   // T too large
    p.part = p.zero_bytes;
    const size_t part_bytes = p.ks > 1 ? align256((size_t)p.ks * T * E * sizeof(float)) : 0;
    p.cand = p.part + part_bytes;
    const size_t cand_bytes =
        p.n_tiles > 1 ? align256((size_t)p.n_tiles * T * K * (sizeof(uint64_t) + sizeof(float))) : 0;
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
    return launch(kern, grid, dim3(THREADS), p.smem, stream, mx, mw, a, p);
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
