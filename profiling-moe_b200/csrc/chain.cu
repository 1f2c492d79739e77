// Decode-chain kernel for sm_100a: every layer of the non-GEMM decode chain of a Kolibri-style
// MoE decoder in ONE persistent launch, for decode batches of T <= 4 tokens.
//
// Per layer, in the order of the reference harness's decoder_layer
// (benchmarks/11_profile_2block_e2e.py:215-266, with the next layer's input_layernorm
// :222-227 fused into the post-MoE pair), each stage starting after the previous one ended:
//   A  Q/K RMSNorm + NeoX RoPE of q, k (RNoPE layers: the norm only)           main CTA
//   B  sandwich: h = r + RMSNorm(attn_out)*g1 ; moe_in = RMSNorm(h)*g2          main CTA
//   C  router GEMV: logits[t][e] = float(bf16(moe_in[t] . W[e]))                gate CTAs
//   D  router (top-K of logits + bias, sigmoid weights) and expert maps         main CTA
//   E  activation expansion: permuted[r] = moe_in[p2u[r] % T]     main CTA (gate CTAs at T=1)
//   F  post-MoE pair: r = h + RMSNorm(moe_out)*g3 ; next = RMSNorm(r)*g4         main CTA
// The main CTA (block 0) runs every stage but C and keeps r, h and moe_in of its rows in
// shared memory.  Every other CTA (one per remaining SM) owns up to four experts of the
// router GEMV: it streams its rows of W for the next layer into shared memory while the main
// CTA works, waits for the layer's `go` word, computes its logits and publishes each one with
// the layer's tag in a 64-bit record, which the main CTA polls (the logits arrive with the
// tag).  `go` and the records are the only cross-CTA synchronisation; every wait is bounded
// and sets an error word when it gives up.  The arithmetic is that of the stand-alone kernels
// (norm_math.cuh, route_math.cuh, the Q/K formula of qk_norm_rope.cu), so each stage gives
// the same bits as its own kernel would on the same inputs.
#include "kb_common.cuh"
#include "norm_math.cuh"
#include "route_math.cuh"

#include <algorithm>
#include <mutex>

namespace kb {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kCT = 512;                     // threads per CTA
constexpr int kCW = kCT / 32;                // warps per CTA
constexpr int kMaxGateCtas = 960;            // gate CTAs with logit records in the workspace
constexpr int kChainMaxLayers = 256;         // layer descriptors held in shared memory
constexpr int kMaxChunks = E_MAX / 32;       // 32-expert chunks of the router
constexpr int kChainMaxT = 4;                // tokens per call
constexpr int kChainMaxK = 8;                // top-K
constexpr int kGateMaxExperts = 4;           // experts per gate CTA
constexpr int kHalfD = 64;                   // head_dim 128
constexpr long long kChainSpin = 1LL << 21;  // bounded waits (about a second of polling)
constexpr int kRedRows = kChainMaxT * kGateMaxExperts;

struct ChainParams {
    const kb_chain_layer_t* layers;
    int L, T, H, Hq, Hkv, E, K;
    int pair_threads;  // threads owning row vectors in the norm stages (row_shape)
    float eps;
    const bf16* attn_out;
    const bf16* moe_out;
    const bf16* q;
    const bf16* k;
    const int32_t* pos;
    const float* inv_freq;
    const bf16* r_in;
    bf16* r_out;
    bf16* h;
    bf16* moe_in;
    bf16* nxt;
    bf16* q_out;
    bf16* k_out;
    bf16* permuted;
    float* logits;
    int32_t* ids;
    float* w;
    int32_t* counts;
    int64_t* offsets;
    int32_t* p2u;
    int32_t* u2p;
    float* trace_logits;
    unsigned* go;    // layers whose moe_in rows are published; 0 between calls
    // [gate CTAs][kGateMaxExperts][kChainMaxT] logit records: (layer + 1) << 32 | float bits,
    // written by the gate CTAs with one 64-bit store each; 0 between calls
    unsigned long long* rec;
    int* err;        // non-zero once a wait gave up (the workspace must be re-zeroed)
};

__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_rel(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// 64-bit accesses are single-copy atomic: a record's tag and value are seen together.
__device__ __forceinline__ void st_rec(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_rec(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void cp16(void* dst, const void* src) {
    const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp4(void* dst, const void* src) {
    const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Thread 0 waits until *p >= target.  Gives up (sets err) after kChainSpin polls, or as soon
// as another CTA has given up.
__device__ bool wait_geq(const unsigned* p, unsigned target, int* err) {
    unsigned v = ld_acq(p);
    long long it = 0;
    while (v < target) {
        if (++it > kChainSpin) {
            atomicExch(err, 1);
            return false;
        }
        if ((it & 1023) == 0 && *(volatile int*)err) return false;
        __nanosleep(32);
        v = ld_acq(p);
    }
    return true;
}

// Block-wide sums of n values at once; each value is reduced exactly as block_sum reduces
// it (warp butterfly, then a butterfly over the warp partials, lanes past the last warp
// adding 0).  Every warp runs the second butterfly itself: a butterfly leaves the same bits
// in every lane, so each warp gets warp 0's result, and one barrier does.  red: MAXN*33
// floats, read after the barrier; the next call must take another buffer (two calls in
// turn on two buffers are safe: a call's barrier follows every read of the buffer before).
template <int MAXN>
__device__ __forceinline__ void block_sum_n(float (&v)[MAXN], int n, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int m = 0; m < MAXN; ++m) {
        if (m < n) {
            const float s = warp_sum(v[m]);
            if (lane == 0) red[m * 33 + warp] = s;
        }
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MAXN; ++m)
        if (m < n) v[m] = warp_sum((lane < nw) ? red[m * 33 + lane] : 0.0f);
}

union V8 {
    uint4 u;
    bf16 e[8];
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

// ------------------------------------------------------------------------------------
// Main CTA stages.
// ------------------------------------------------------------------------------------
struct MainSmem {
    bf16* r;      // [kChainMaxT][H] residual stream
    bf16* h;      // [kChainMaxT][H] sandwich sum
    bf16* x;      // [kChainMaxT][H] moe_in
    float* cs;    // [kChainMaxT][64]
    float* sn;    // [kChainMaxT][64]
    float* red;   // [kRedRows][33]
    int* hist;    // [E_MAX]  routing: group maxima [kChainMaxT][32]
    int* offs;    // [E_MAX + 4]  routing: candidates (u64) [kChainMaxT][32]
    int* sel;     // [32]
    int* perm;    // [32]  token of each permuted row
    int* scratch; // [64]
    int* flag;    // [4]
    kb_chain_layer_t* layers;  // [kChainMaxLayers]
    float* xrow;  // [kChainMaxT][E_MAX] logits of the layer
    float* bias;  // [E_MAX] gate bias of the layer (+0 for -0), 0 without one
};

__host__ __device__ constexpr size_t main_smem_bytes(int H) {
    return (size_t)3 * kChainMaxT * H * sizeof(bf16) + 2 * kChainMaxT * kHalfD * sizeof(float) +
           (size_t)kRedRows * 33 * sizeof(float) + (2 * E_MAX + 4 + 32 + 32 + 64 + 4) * sizeof(int) +
           (size_t)kChainMaxLayers * sizeof(kb_chain_layer_t) +
           (size_t)(kChainMaxT * E_MAX + E_MAX) * 4;
}
__host__ __device__ constexpr size_t gate_smem_bytes(int H) {
    return (size_t)2 * kGateMaxExperts * H * sizeof(bf16) + (size_t)kRedRows * 33 * sizeof(float) +
           16;
}

__device__ MainSmem carve_main(unsigned char* smem, int H) {
    MainSmem m;
    m.r = reinterpret_cast<bf16*>(smem);
    m.h = m.r + (size_t)kChainMaxT * H;
    m.x = m.h + (size_t)kChainMaxT * H;
    m.cs = reinterpret_cast<float*>(m.x + (size_t)kChainMaxT * H);
    m.sn = m.cs + kChainMaxT * kHalfD;
    m.red = m.sn + kChainMaxT * kHalfD;
    m.hist = reinterpret_cast<int*>(m.red + kRedRows * 33);
    m.offs = m.hist + E_MAX;
    m.sel = m.offs + E_MAX + 4;
    m.perm = m.sel + 32;
    m.scratch = m.perm + 32;
    m.flag = m.scratch + 64;
    m.layers = reinterpret_cast<kb_chain_layer_t*>(m.flag + 4);
    m.xrow = reinterpret_cast<float*>(m.layers + kChainMaxLayers);
    m.bias = m.xrow + kChainMaxT * E_MAX;
    return m;
}

// A: per-head RMSNorm + NeoX RoPE.  Four lanes per (token, head), 32 elements per lane,
// eight heads per warp.  Lane p of a head holds the elements of lanes 8p..8p+7 of the
// one-warp-per-head kernel (qk_norm_rope.cu); its butterfly levels 16, 8 become lane
// exchanges 2, 1 and levels 4, 2, 1 register adds, so the sum of squares, and with it every
// output, has the same bits.  The NeoX partner of element j (j +- 64) sits in lane p^2.
constexpr int kQkChunk = 1;  // head groups per warp with loads in flight together

__device__ __forceinline__ void stage_qk(const ChainParams& p, const kb_chain_layer_t& Ly,
                                     const MainSmem& s) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = lane >> 2, pl = lane & 3;  // head slot in the warp, lane in the head
    const int HH = p.Hq + p.Hkv, nh = p.T * HH;
    const int ngroups = (nh + 7) >> 3;
    const bool rope = !Ly.rnope && p.pos != nullptr;
    for (int g0 = warp; g0 < ngroups; g0 += kCW * kQkChunk) {
        V8 xv[kQkChunk][4], gv[kQkChunk][4];
#pragma unroll
        for (int c = 0; c < kQkChunk; ++c) {  // clamped heads: every load in flight at once
            const int hd = min((g0 + c * kCW) * 8 + slot, nh - 1);
            const int t = hd / HH, hh = hd - t * HH;
            const bf16* src = hh < p.Hq ? p.q + ((size_t)t * p.Hq + hh) * 128
                                        : p.k + ((size_t)t * p.Hkv + (hh - p.Hq)) * 128;
            const bf16* gsrc = static_cast<const bf16*>(hh < p.Hq ? Ly.g_q : Ly.g_k) + pl * 32;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                xv[c][u].u = ld_stream(reinterpret_cast<const uint4*>(src + pl * 32) + u);
                gv[c][u].u = __ldg(reinterpret_cast<const uint4*>(gsrc) + u);
            }
        }
#pragma unroll
        for (int c = 0; c < kQkChunk; ++c) {
            if (g0 + c * kCW >= ngroups) break;
            const int hd = (g0 + c * kCW) * 8 + slot;
            const bool act = hd < nh;
            const int t = act ? hd / HH : 0, hh = act ? hd - t * HH : 0;
            const bool is_q = hh < p.Hq;
            float y[32];
            float part[8];
#pragma unroll
            for (int sub = 0; sub < 8; ++sub) {
                part[sub] = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int k = sub * 4 + i;
                    y[k] = act ? __bfloat162float(xv[c][k >> 3].e[k & 7]) : 0.0f;
                    part[sub] = fmaf(y[k], y[k], part[sub]);
                }
            }
#pragma unroll
            for (int o = 2; o > 0; o >>= 1)  // levels 16, 8
#pragma unroll
                for (int sub = 0; sub < 8; ++sub)
                    part[sub] += __shfl_xor_sync(FULL_MASK, part[sub], o);
            float a4[4];
#pragma unroll
            for (int sub = 0; sub < 4; ++sub) a4[sub] = part[sub] + part[sub + 4];  // level 4
            const float a20 = a4[0] + a4[2], a21 = a4[1] + a4[3];                  // level 2
            const float ss = a20 + a21;                                             // level 1
            const float r = 1.0f / sqrtf(ss / 128.0f + p.eps);
            const V8* g = gv[c];  // this lane's gamma slice, loaded with the head
#pragma unroll
            for (int k = 0; k < 32; ++k)
                y[k] = __fmul_rn(__fmul_rn(y[k], r), __bfloat162float(g[k >> 3].e[k & 7]));
            V8 o[4];
            if (rope) {
                const bool first_half = pl < 2;
                // cos/sin of this lane's elements k: angles j = (pl*32 + k) mod 64, 4 at a time
                const float4* cs4 = reinterpret_cast<const float4*>(s.cs + t * kHalfD + ((pl * 32) & (kHalfD - 1)));
                const float4* sn4 = reinterpret_cast<const float4*>(s.sn + t * kHalfD + ((pl * 32) & (kHalfD - 1)));
#pragma unroll
                for (int m = 0; m < 8; ++m) {  // four elements per float4 of cos and of sin
                    const float4 a = cs4[m], b = sn4[m];
                    const float cc4[4] = {a.x, a.y, a.z, a.w}, sv4[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int k = 4 * m + q;
                        const float other = __shfl_xor_sync(FULL_MASK, y[k], 2);
                        const float cc = cc4[q], sv = sv4[q];
                        const float v = first_half ? __fsub_rn(__fmul_rn(y[k], cc), __fmul_rn(other, sv))
                                                   : __fadd_rn(__fmul_rn(y[k], cc), __fmul_rn(other, sv));
                        o[k >> 3].e[k & 7] = __float2bfloat16_rn(v);
                    }
                }
            } else {
#pragma unroll
                for (int k = 0; k < 32; ++k) o[k >> 3].e[k & 7] = __float2bfloat16_rn(y[k]);
            }
            if (act) {
                bf16* dst = is_q ? p.q_out + ((size_t)t * p.Hq + hh) * 128
                                 : p.k_out + ((size_t)t * p.Hkv + (hh - p.Hq)) * 128;
#pragma unroll
                for (int u = 0; u < 4; ++u) reinterpret_cast<uint4*>(dst + pl * 32)[u] = o[u].u;
            }
        }
    }
}

// B / F: sum = res + RMSNorm(a)*g1 (rounded) ; norm = RMSNorm(sum)*g2, for the T rows.
// Threads below pair_threads own vectors tid + i*pair_threads, exactly as the stand-alone
// kernel's threads do (row_shape); the others add zeros to the reductions, which changes no
// bit.
// a comes from global memory (read-only during the launch), res from shared memory.
// sum goes to sum_sm (and sum_g if non-null), norm to norm_g (and norm_sm if non-null).
template <int VPT, int TT>
__device__ __forceinline__ void stage_pair(const ChainParams& p, const bf16* a, const bf16* res_sm,
                           const bf16* g1, const bf16* g2, bf16* sum_sm, bf16* sum_g,
                           bf16* norm_g, bf16* norm_sm, float* red) {
    const int T = p.T, H = p.H, nvec = H / 8;
    // Threads past pair_threads own no vector: their index lands past the row.
    const int PT = p.pair_threads;
    const int tid = (int)threadIdx.x < PT ? (int)threadIdx.x : nvec;
    V8 va[TT][VPT];
    V8 vg1[VPT], vg2[VPT];
    float ss[TT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {  // weights first: every load of the stage is in flight at once
        const int v = min(tid + i * PT, nvec - 1);
        vg1[i].u = __ldg(reinterpret_cast<const uint4*>(g1) + v);
        vg2[i].u = __ldg(reinterpret_cast<const uint4*>(g2) + v);
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {  // clamped addresses: every load in flight at once
        ss[t] = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i)
            va[t][i].u = ld_stream(reinterpret_cast<const uint4*>(a + (size_t)min(t, T - 1) * H) +
                                   min(tid + i * PT, nvec - 1));
    }
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int i = 0; i < VPT; ++i)
            if (tid + i * PT >= nvec) va[t][i].u = make_uint4(0, 0, 0, 0);
    static_assert(2 * TT <= kRedRows, "two reduction buffers of TT rows");
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        if (t < T) {
#pragma unroll
            for (int i = 0; i < VPT; ++i)
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float x = __bfloat162float(va[t][i].e[e]);
                    ss[t] = fmaf(x, x, ss[t]);
                }
        }
    }
    block_sum_n<TT>(ss, T, red);
    float ss2[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        ss2[t] = 0.0f;
        if (t < T) {
            const float r1 = rms_scale(ss[t], H, p.eps);
#pragma unroll
            for (int i = 0; i < VPT; ++i) {
                const int v = tid + i * PT;
                if (v < nvec) {
                    V8 vr, vh;
                    const V8& vg = vg1[i];
                    vr.u = reinterpret_cast<const uint4*>(res_sm + (size_t)t * H)[v];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float post = rnd<bf16>(__fmul_rn(
                            __fmul_rn(__bfloat162float(va[t][i].e[e]), r1), __bfloat162float(vg.e[e])));
                        const bf16 hv = __float2bfloat16_rn(__fadd_rn(__bfloat162float(vr.e[e]), post));
                        vh.e[e] = hv;
                        const float hf = __bfloat162float(hv);
                        ss2[t] = fmaf(hf, hf, ss2[t]);
                    }
                    va[t][i].u = vh.u;
                    reinterpret_cast<uint4*>(sum_sm + (size_t)t * H)[v] = vh.u;
                    if (sum_g) reinterpret_cast<uint4*>(sum_g + (size_t)t * H)[v] = vh.u;
                }
            }
        }
    }
    block_sum_n<TT>(ss2, T, red + TT * 33);
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        if (t < T) {
            const float r2 = rms_scale(ss2[t], H, p.eps);
#pragma unroll
            for (int i = 0; i < VPT; ++i) {
                const int v = tid + i * PT;
                if (v < nvec) {
                    V8 vx;
                    const V8& vg = vg2[i];
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        vx.e[e] = __float2bfloat16_rn(__fmul_rn(
                            __fmul_rn(__bfloat162float(va[t][i].e[e]), r2), __bfloat162float(vg.e[e])));
                    reinterpret_cast<uint4*>(norm_g + (size_t)t * H)[v] = vx.u;
                    if (norm_sm) reinterpret_cast<uint4*>(norm_sm + (size_t)t * H)[v] = vx.u;
                }
            }
        }
    }
}

// Top-K of token t by K rounds over all of its keys (lane l holds experts l, l + 32, ...):
// each round takes the warp's largest key, the lowest expert among equal keys (redux max,
// then redux min), and clears it.  The path for rows whose keys tie at the threshold.
__device__ void topk_rounds(const MainSmem& s, const float* bias_sm, int t, int E, int K) {
    const int lane = threadIdx.x & 31;
    uint32_t key[kMaxChunks];
#pragma unroll
    for (int j = 0; j < kMaxChunks; ++j) {
        const int e = lane + 32 * j;
        key[j] = (e < E) ? okey(s.xrow[t * E_MAX + e] + (bias_sm[e] + 0.0f)) : 0u;
    }
    static_assert(kMaxChunks == 16, "four-level tournament");
    for (int r = 0; r < K; ++r) {
        // Lane maximum by a 4-level tournament of (key, j); the right side wins only on a
        // strictly larger key, so the lowest j (expert) of the lane wins ties.
        uint32_t k8[8], k4[4], k2[2];
        int j8[8], j4[4], j2[2];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const bool rt = key[2 * u + 1] > key[2 * u];
            k8[u] = rt ? key[2 * u + 1] : key[2 * u];
            j8[u] = rt ? 2 * u + 1 : 2 * u;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const bool rt = k8[2 * u + 1] > k8[2 * u];
            k4[u] = rt ? k8[2 * u + 1] : k8[2 * u];
            j4[u] = rt ? j8[2 * u + 1] : j8[2 * u];
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const bool rt = k4[2 * u + 1] > k4[2 * u];
            k2[u] = rt ? k4[2 * u + 1] : k4[2 * u];
            j2[u] = rt ? j4[2 * u + 1] : j4[2 * u];
        }
        const bool rt = k2[1] > k2[0];
        const uint32_t best = rt ? k2[1] : k2[0];
        const int bj = rt ? j2[1] : j2[0];
        const uint32_t wmax = __reduce_max_sync(FULL_MASK, best);
        const unsigned cand = (best == wmax && best != 0u) ? (unsigned)(lane + 32 * bj) : 0xffffffffu;
        const unsigned widx = __reduce_min_sync(FULL_MASK, cand);
        if (cand == widx) {
#pragma unroll
            for (int j = 0; j < kMaxChunks; ++j)
                if (j == bj) key[j] = 0u;
        }
        if (lane == 0) s.sel[t * K + r] = (int)widx;
    }
}

// D: exact top-K per token, then the weights and the maps of the T*K <= 32 selections.
// Same keys and tie rule as the router kernels: score = logit + (bias + 0), ordered by okey
// (NaN highest), the lower expert index first.  The bias row (bias_sm) and the layer's
// logits (xrow, filled from the gate records) sit in shared memory, complete at entry.
//  1. Every warp, per (token, 32-expert chunk): the key of each expert and the maximum of
//     each group of G consecutive experts, G the smallest power of two giving ng <= 32
//     groups (so ng >= K: ng > 16 whenever G > 1, and ng = E >= K when G = 1).
//  2. Per (token, chunk) again: tau = the K-th largest group maximum (the least maximum
//     with fewer than K maxima above it).  The K groups with the largest maxima hold K keys
//     >= tau, so every key of the top K is >= tau; those keys are the candidates, appended
//     to the token's list (a shared-memory counter hands out the slots).
//  3. Warp t: with C <= 32 candidates, each one's rank is the number of candidates above it
//     in (key, then lower expert) order, found in one pass; ranks below K are the output.
//     Rows with more candidates (ties at tau) take the K rounds of topk_rounds.
__device__ __forceinline__ void stage_route_maps(const ChainParams& p, const float* bias_sm,
                                             const MainSmem& s) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int T = p.T, E = p.E, K = p.K, n = T * K;
    const int nch = (E + 31) >> 5, units = T * nch;
    int lg = 0;  // log2 G
    while (((E + (1 << lg) - 1) >> lg) > 32) ++lg;
    const int ng = (E + (1 << lg) - 1) >> lg;
    uint32_t* gmax = reinterpret_cast<uint32_t*>(s.hist);                  // [kChainMaxT][32]
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(s.offs);  // [kChainMaxT][32]
    int* ncand = s.scratch;                                                 // [kChainMaxT]
    if ((int)threadIdx.x < T) ncand[threadIdx.x] = 0;
    for (int u = warp; u < units; u += kCW) {  // 1: uniform trip count within the warp
        const int t = u / nch, e = (u - t * nch) * 32 + lane;
        uint32_t k = (e < E) ? okey(s.xrow[t * E_MAX + e] + (bias_sm[e] + 0.0f)) : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
            if (o < (1 << lg)) k = max(k, __shfl_xor_sync(FULL_MASK, k, o));
        if ((lane & ((1 << lg) - 1)) == 0 && e < E) gmax[t * 32 + (e >> lg)] = k;
    }
    __syncthreads();
    for (int u = warp; u < units; u += kCW) {  // 2
        const int t = u / nch, e = (u - t * nch) * 32 + lane;
        const uint32_t m = lane < ng ? gmax[t * 32 + lane] : 0u;  // valid maxima are > 0
        int above = 0;
#pragma unroll
        for (int h = 0; h < 32; ++h) above += (__shfl_sync(FULL_MASK, m, h) > m) ? 1 : 0;
        const uint32_t tau = __reduce_min_sync(FULL_MASK, (lane < ng && above < K) ? m : 0xffffffffu);
        const uint32_t k = (e < E) ? okey(s.xrow[t * E_MAX + e] + (bias_sm[e] + 0.0f)) : 0u;
        const bool take = e < E && k >= tau;
        const unsigned b = __ballot_sync(FULL_MASK, take);
        int base = 0;
        if (lane == 0 && b) base = atomicAdd(ncand + t, __popc(b));
        base = __shfl_sync(FULL_MASK, base, 0);
        const int slot = base + __popc(b & ((1u << lane) - 1u));
        if (take && slot < 32)
            cand[t * 32 + slot] = ((unsigned long long)k << 32) | (unsigned)(0xffffffffu - (unsigned)e);
    }
    __syncthreads();
    if (warp < T) {  // 3
        const int t = warp;
        const int C = ncand[t];
        if (C <= 32) {
            const unsigned long long mine = lane < C ? cand[t * 32 + lane] : 0ull;
            int rank = 0;
            for (int j = 0; j < C; ++j) rank += (cand[t * 32 + j] > mine) ? 1 : 0;
            if (lane < C && rank < K) s.sel[t * K + rank] = (int)(0xffffffffu - (unsigned)mine);
        } else {
            topk_rounds(s, bias_sm, t, E, K);
        }
        __syncwarp();
        if (lane < K) {
            const int id = s.sel[t * K + lane];
            p.ids[t * K + lane] = id;
            p.w[t * K + lane] = sigmoid_acc(s.xrow[t * E_MAX + id]);
        }
    }
    __syncthreads();
    // Maps of n <= 32 selections without a scan: offsets[e] = selections below e,
    // counts[e] = selections equal to e, rank of selection i = selections below its expert
    // + equal ones before it (selections are in (token, slot) order).
    for (int e = threadIdx.x; e <= E; e += kCT) {
        int below = 0, equal = 0;
        for (int i = 0; i < n; ++i) {
            const int v = s.sel[i];
            below += (v < e) ? 1 : 0;
            equal += (v == e) ? 1 : 0;
        }
        p.offsets[e] = (int64_t)below;
        if (p.counts && e < E) p.counts[e] = equal;
    }
    if (warp == 0) {
        const int e = (lane < n) ? s.sel[lane] : 0x7fffffff;
        int rank = 0;
        for (int i = 0; i < n; ++i) {
            const int v = s.sel[i];
            rank += (v < e || (v == e && i < lane)) ? 1 : 0;
        }
        if (lane < n) {
            const int tok = lane / K, slot = lane - tok * K;
            const int u = slot * T + tok;
            p.p2u[rank] = u;
            if (p.u2p) p.u2p[u] = rank;
            s.perm[rank] = tok;
        }
    }
    __syncthreads();
}

// E: permuted rows straight from the moe_in rows held in shared memory (T > 1).  At T == 1
// every selection is token 0, so the K permuted rows are copies of moe_in whatever the
// routing: the gate CTAs write them while they compute the router GEMV (chain_gate).
__device__ __forceinline__ void stage_expand(const ChainParams& p, const MainSmem& s) {
    const int nvec = p.H / 8, n = p.T * p.K;
    for (int r = 0; r < n; ++r) {
        const uint4* src = reinterpret_cast<const uint4*>(s.x + (size_t)s.perm[r] * p.H);
        uint4* dst = reinterpret_cast<uint4*>(p.permuted + (size_t)r * p.H);
        for (int v = threadIdx.x; v < nvec; v += kCT) st_stream(dst + v, src[v]);
    }
}

// Waits (bounded) until every logit record of gate CTA c carries `tag`, then stores the
// logits in xrow[t][e].  A failed wait sets the error word.
__device__ bool take_records(const ChainParams& p, unsigned c, unsigned gate_ctas, unsigned tag,
                             float* xrow) {
    const unsigned long long* rc = p.rec + (size_t)c * kGateMaxExperts * kChainMaxT;
    const int T = p.T, E = p.E;
    long long it = 0;
    while (true) {
        unsigned long long r[kGateMaxExperts][kChainMaxT];
        bool all = true;
#pragma unroll
        for (int m = 0; m < kGateMaxExperts; ++m)
#pragma unroll
            for (int t = 0; t < kChainMaxT; ++t) {
                const bool used = (int)(c + m * gate_ctas) < E && t < T;
                r[m][t] = used ? ld_rec(rc + m * kChainMaxT + t) : ((unsigned long long)tag << 32);
                all = all && (unsigned)(r[m][t] >> 32) == tag;
            }
        if (all) {
#pragma unroll
            for (int m = 0; m < kGateMaxExperts; ++m)
#pragma unroll
                for (int t = 0; t < kChainMaxT; ++t) {
                    const int e = (int)(c + m * gate_ctas);
                    if (e < E && t < T) xrow[t * E_MAX + e] = __uint_as_float((unsigned)r[m][t]);
                }
            return true;
        }
        if (++it > kChainSpin || ((it & 1023) == 0 && *(volatile int*)p.err)) {
            atomicExch(p.err, 1);
            return false;
        }
        __nanosleep(32);
    }
}

template <int VPT, int TT>
__device__ __forceinline__ void chain_main(const ChainParams& p, unsigned char* smem) {
    const int T = p.T, H = p.H, nvec = H / 8;
    const MainSmem s = carve_main(smem, H);
    const unsigned gate_ctas = gridDim.x - 1;
    {  // every layer descriptor into shared memory once
        const int words = p.L * (int)(sizeof(kb_chain_layer_t) / sizeof(int));
        for (int i = threadIdx.x; i < words; i += kCT)
            reinterpret_cast<int*>(s.layers)[i] = reinterpret_cast<const int*>(p.layers)[i];
    }
    for (int i = threadIdx.x; i < T * nvec; i += kCT) {
        const int t = i / nvec, v = i - t * nvec;
        reinterpret_cast<uint4*>(s.r + (size_t)t * H)[v] =
            reinterpret_cast<const uint4*>(p.r_in + (size_t)t * H)[v];
    }
    if (p.pos) {
        for (int i = threadIdx.x; i < T * kHalfD; i += kCT) {
            const int t = i / kHalfD, j = i - t * kHalfD;
            float sv, cv;
            sincosf(__fmul_rn((float)__ldg(p.pos + t), __ldg(p.inv_freq + j)), &sv, &cv);
            s.cs[i] = cv;
            s.sn[i] = sv;
        }
    }
    if (threadIdx.x == 0) s.flag[0] = 1;  // cleared only on a failed wait, which returns
    __syncthreads();
    for (int l = 0; l < p.L; ++l) {
        const kb_chain_layer_t& Ly = s.layers[l];
        // This layer's gate bias into shared memory, in the background until the router.
        if (Ly.gate_bias) {
            for (int e = threadIdx.x; e < p.E; e += kCT) cp4(s.bias + e, Ly.gate_bias + e);
        } else {
            for (int e = threadIdx.x; e < p.E; e += kCT) s.bias[e] = 0.0f;
        }
        cp_commit();
        if (l + 1 < p.L) {  // the next layer's small weights into L2
            const kb_chain_layer_t& Ln = s.layers[l + 1];
            if (Ln.gate_bias && threadIdx.x < (p.E * 4 + 127) / 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(
                    reinterpret_cast<const char*>(Ln.gate_bias) + threadIdx.x * 128));
            const int lines = (H * 2 + 127) / 128;
            for (int i = threadIdx.x; i < 4 * lines; i += kCT) {
                const int w = i / lines;  // selects, not an indexed array (which lives on the stack)
                const void* base = w == 0 ? Ln.g_post_attn : w == 1 ? Ln.g_pre_moe
                                 : w == 2 ? Ln.g_post_ffn : Ln.g_input_ln;
                asm volatile("prefetch.global.L2 [%0];" ::"l"(
                    static_cast<const char*>(base) + (size_t)(i - w * lines) * 128));
            }
        }
        stage_qk(p, Ly, s);
        __syncthreads();
        stage_pair<VPT, TT>(p, p.attn_out, s.r, static_cast<const bf16*>(Ly.g_post_attn),
                        static_cast<const bf16*>(Ly.g_pre_moe), s.h, p.h, p.moe_in, s.x, s.red);
        __syncthreads();
        // The barrier above orders every thread's rows before the release.
        if (threadIdx.x == 0) st_rel(p.go, (unsigned)(l + 1));
        // One thread per gate CTA polls that CTA's logit records (all loads of a poll in
        // flight at once) until each carries this layer's tag; the logits arrive with it.
        for (unsigned c = threadIdx.x; c < gate_ctas; c += kCT)
            if (!take_records(p, c, gate_ctas, (unsigned)(l + 1), s.xrow)) s.flag[0] = 0;
        cp_wait<0>();  // this thread's part of the bias row; the barrier shares it
        __syncthreads();
        if (!s.flag[0]) {
            for (int e = threadIdx.x; e <= p.E; e += kCT) p.offsets[e] = -1;
            return;
        }
        stage_route_maps(p, s.bias, s);
        if (p.T > 1) stage_expand(p, s);  // T == 1: the gate CTAs wrote it
        stage_pair<VPT, TT>(p, p.moe_out, s.h, static_cast<const bf16*>(Ly.g_post_ffn),
                        static_cast<const bf16*>(Ly.g_input_ln), s.r, p.r_out, p.nxt, nullptr,
                        s.red);
        __syncthreads();
    }
    // Every gate CTA has written its last records: they and go can return to zero.
    for (unsigned i = threadIdx.x; i < gate_ctas * kGateMaxExperts * kChainMaxT; i += kCT)
        p.rec[i] = 0ull;
    if (threadIdx.x == 0) *p.go = 0u;
}

// ------------------------------------------------------------------------------------
// Gate CTAs: router GEMV for experts j, j + G1, ... (G1 = gate CTAs).
// ------------------------------------------------------------------------------------

template <int VQ, int TT>
__device__ __forceinline__ void chain_gate(const ChainParams& p, unsigned char* smem) {
    const int G1 = gridDim.x - 1, j = blockIdx.x - 1;
    const int H = p.H, E = p.E, T = p.T, nvec = H / 8;
    bf16* wb = reinterpret_cast<bf16*>(smem);  // [2][kGateMaxExperts][H]
    float* red = reinterpret_cast<float*>(wb + (size_t)2 * kGateMaxExperts * H);
    __shared__ int ok;
    int ne = 0;  // this CTA's experts: j + m * G1 for m < ne
#pragma unroll
    for (int m = 0; m < kGateMaxExperts; ++m)
        if (j + m * G1 < E) ne = m + 1;
    auto issue = [&](int l) {
        const bf16* W = static_cast<const bf16*>(p.layers[l].w_gate_t);
        bf16* dst = wb + (size_t)(l & 1) * kGateMaxExperts * H;
        for (int m = 0; m < ne; ++m)
            for (int v = threadIdx.x; v < nvec; v += kCT)
                cp16(dst + (size_t)m * H + v * 8, W + (size_t)(j + m * G1) * H + v * 8);
        cp_commit();
    };
    issue(0);
    for (int l = 0; l < p.L; ++l) {
        if (l + 1 < p.L) issue(l + 1);
        else cp_commit();
        if (threadIdx.x == 0) ok = wait_geq(p.go, (unsigned)(l + 1), p.err) ? 1 : 0;
        cp_wait<1>();
        __syncthreads();
        if (!ok) {
            cp_wait<0>();
            return;
        }
        // T == 1: this CTA's share [x0, x1) of the K copies of moe_in (the expansion).  The
        // first vector of each thread is loaded here and stored after the dot products, so
        // its L2 round trip overlaps them; every copy is stored before the barrier that
        // precedes this CTA's records, so moe_in is read before the main CTA can move on.
        const int xtotal = (T == 1 && p.permuted) ? p.K * nvec : 0;
        const int xper = (xtotal + G1 - 1) / G1;
        const int x0 = min(xtotal, j * xper), x1 = min(xtotal, x0 + xper);
        const int xi = x0 + (int)threadIdx.x;
        uint4 xcopy = make_uint4(0, 0, 0, 0);
        if (xi < x1) xcopy = __ldcg(reinterpret_cast<const uint4*>(p.moe_in) + xi % nvec);
        const bf16* wl = wb + (size_t)(l & 1) * kGateMaxExperts * H;
        // Warp w takes slice w of H (kCW slices) for every expert of the CTA and every token:
        // its moe_in vectors once from L2 (one read of moe_in per CTA), the experts' W
        // vectors from shared memory, one accumulator per (expert, token), a warp sum; the
        // slices are then added in order by one thread per (expert, token).
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const int S = (nvec + kCW - 1) / kCW;  // vectors per slice
        const int v0 = warp * S, v1 = min(v0 + S, nvec);
        float acc[kGateMaxExperts][TT];
#pragma unroll
        for (int m = 0; m < kGateMaxExperts; ++m)
#pragma unroll
            for (int t = 0; t < TT; ++t) acc[m][t] = 0.0f;
#pragma unroll
        for (int i = 0; i < VQ; ++i) {
            const int v = v0 + lane + 32 * i;
            const bool in = v < v1;
            const int vc = in ? v : v0;  // clamped: every load in flight at once
            V8 xv[TT];
#pragma unroll
            for (int t = 0; t < TT; ++t)
                xv[t].u = __ldcg(reinterpret_cast<const uint4*>(p.moe_in + (size_t)min(t, T - 1) * H) + vc);
#pragma unroll
            for (int m = 0; m < kGateMaxExperts; ++m) {
                if (m < ne && in) {
                    V8 wv;
                    wv.u = reinterpret_cast<const uint4*>(wl + (size_t)m * H)[vc];
#pragma unroll
                    for (int t = 0; t < TT; ++t)
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            acc[m][t] = fmaf(__bfloat162float(xv[t].e[e]), __bfloat162float(wv.e[e]), acc[m][t]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < kGateMaxExperts; ++m)
#pragma unroll
            for (int t = 0; t < TT; ++t)
                if (m < ne && t < T) {  // ne and T are uniform over the CTA
                    const float sum = warp_sum(acc[m][t]);
                    if (lane == 0) red[(m * kCW + warp) * TT + t] = sum;
                }
        if (xi < x1) st_stream(reinterpret_cast<uint4*>(p.permuted) + xi, xcopy);
        for (int i = xi + kCT; i < x1; i += kCT)  // shares longer than one vector per thread
            st_stream(reinterpret_cast<uint4*>(p.permuted) + i,
                      __ldcg(reinterpret_cast<const uint4*>(p.moe_in) + i % nvec));
        __syncthreads();
        if (threadIdx.x < ne * TT) {
            const int mm = threadIdx.x / TT, t = threadIdx.x - mm * TT;
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) sum += red[(mm * kCW + w) * TT + t];
            const float v = __bfloat162float(__float2bfloat16_rn(sum));
            const int e = j + mm * G1;
            p.logits[(size_t)t * E + e] = v;
            if (p.trace_logits) p.trace_logits[((size_t)l * T + t) * E + e] = v;
            st_rec(p.rec + ((size_t)j * kGateMaxExperts + mm) * kChainMaxT + t,
                   ((unsigned long long)(l + 1) << 32) | __float_as_uint(v));
        }
        __syncthreads();  // this layer's reads of moe_in and of the W buffer are over
    }
}

template <int VPT, int TT>
__global__ void __launch_bounds__(kCT, 1) decode_chain_kernel(const __grid_constant__ ChainParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    if (*(volatile int*)p.err) {  // an earlier call gave up: report and do nothing
        if (blockIdx.x == 0)
            for (int e = threadIdx.x; e <= p.E; e += kCT) p.offsets[e] = -1;
        return;
    }
    // The stages read the parameters from a shared-memory copy (short, fixed latency).
    __shared__ ChainParams ps;
    constexpr int kWords = (int)(sizeof(ChainParams) / sizeof(int));
    static_assert(sizeof(ChainParams) % sizeof(int) == 0, "ChainParams copy");
    for (int i = threadIdx.x; i < kWords; i += kCT)
        reinterpret_cast<int*>(&ps)[i] = reinterpret_cast<const int*>(&p)[i];
    __syncthreads();
    if (blockIdx.x == 0) chain_main<VPT, TT>(ps, smem);
    else chain_gate<VPT, TT>(ps, smem);  // a slice of H / kCW vectors: at most VPT per lane
}

// ------------------------------------------------------------------------------------
// Host
// ------------------------------------------------------------------------------------
template <int VPT, int TT>
int run_chain(const ChainParams& prm, size_t smem, int grid, cudaStream_t st) {
    auto* kern = decode_chain_kernel<VPT, TT>;
    int err = allow_smem(kern, smem);
    if (err) return err;
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kCT, smem) != cudaSuccess || nb < 1)
        return KB_ERR_UNSUPPORTED;
    return launch_coop(kern, dim3((unsigned)grid), dim3(kCT), smem, st, prm);
}

template <int VPT>
int run_tokens(int T, const ChainParams& prm, size_t smem, int grid, cudaStream_t st) {
    switch (T) {
        case 1: return run_chain<VPT, 1>(prm, smem, grid, st);
        case 2: return run_chain<VPT, 2>(prm, smem, grid, st);
        case 3: return run_chain<VPT, 3>(prm, smem, grid, st);
        case 4: return run_chain<VPT, 4>(prm, smem, grid, st);
        default: return KB_ERR_UNSUPPORTED;
    }
}

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    int& v = cache[dev & 63];
    if (v == 0) {
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (v <= 0) v = 148;
    }
    return v;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" size_t kb_decode_chain_workspace_bytes(void) {
    return 256 + (size_t)8 * kMaxGateCtas * kGateMaxExperts * kChainMaxT;
}

extern "C" int kb_decode_chain(const kb_chain_layer_t* layers, int n_layers, const void* attn_out,
                               const void* moe_out, const void* q, const void* k,
                               const int32_t* pos, const float* inv_freq,
                               const void* residual_in, void* residual_out, void* h,
                               void* moe_in, void* next, void* q_out, void* k_out, float* logits,
                               int32_t* ids, float* weights, int32_t* counts, int64_t* offsets,
                               int32_t* p2u, int32_t* u2p, void* permuted, float* trace_logits,
                               void* workspace, size_t workspace_bytes, int64_t T, int H,
                               int Hq, int Hkv, int D, int E, int K, float eps,
                               kb_stream_t stream) {
    if (n_layers > kChainMaxLayers) return KB_ERR_UNSUPPORTED;
    if (T < 1 || n_layers < 1 || H <= 0 || Hq < 0 || Hkv < 0 || E <= 0 || K <= 0)
        return KB_ERR_INVALID_ARG;
    if (T > kChainMaxT || D != 128 || H % 8 != 0 || row_shape(H / 8).vpt == 0 || row_shape(H / 8).vpt > 3 || E > E_MAX ||
        K > kChainMaxK || K > E || Hq + Hkv <= 0)
        return KB_ERR_UNSUPPORTED;
    if (!layers || !attn_out || !moe_out || !q || !k || !residual_in || !residual_out || !h ||
        !moe_in || !next || !q_out || !k_out || !logits || !ids || !weights || !offsets ||
        !p2u || !permuted || (pos && !inv_freq))
        return KB_ERR_INVALID_ARG;
    if (!workspace || workspace_bytes < kb_decode_chain_workspace_bytes()) return KB_ERR_WORKSPACE;
    const void* vec_ptrs[] = {attn_out, moe_out, q, k, residual_in, residual_out, h, moe_in,
                              next, q_out, k_out, permuted, workspace};
    for (const void* v : vec_ptrs)
        if (!aligned16(v)) return KB_ERR_ALIGNMENT;
    const int sms = sm_count();
    const int gate = std::min(std::min(sms - 1, E), kMaxGateCtas);
    if (gate < 1 || (int64_t)gate * kGateMaxExperts < E) return KB_ERR_UNSUPPORTED;
    ChainParams prm;
    prm.layers = layers;
    prm.L = n_layers;
    prm.T = (int)T;
    prm.H = H;
    prm.Hq = Hq;
    prm.Hkv = Hkv;
    prm.E = E;
    prm.K = K;
    prm.eps = eps;
    prm.attn_out = static_cast<const bf16*>(attn_out);
    prm.moe_out = static_cast<const bf16*>(moe_out);
    prm.q = static_cast<const bf16*>(q);
    prm.k = static_cast<const bf16*>(k);
    prm.pos = pos;
    prm.inv_freq = inv_freq;
    prm.r_in = static_cast<const bf16*>(residual_in);
    prm.r_out = static_cast<bf16*>(residual_out);
    prm.h = static_cast<bf16*>(h);
    prm.moe_in = static_cast<bf16*>(moe_in);
    prm.nxt = static_cast<bf16*>(next);
    prm.q_out = static_cast<bf16*>(q_out);
    prm.k_out = static_cast<bf16*>(k_out);
    prm.permuted = static_cast<bf16*>(permuted);
    prm.logits = logits;
    prm.ids = ids;
    prm.w = weights;
    prm.counts = counts;
    prm.offsets = offsets;
    prm.p2u = p2u;
    prm.u2p = u2p;
    prm.trace_logits = trace_logits;
    unsigned char* wsb = static_cast<unsigned char*>(workspace);
    prm.go = reinterpret_cast<unsigned*>(wsb);
    prm.err = reinterpret_cast<int*>(wsb + 128);
    prm.rec = reinterpret_cast<unsigned long long*>(wsb + 256);
    const size_t smem = std::max(main_smem_bytes(H), gate_smem_bytes(H));
    const RowShape rs = row_shape(H / 8);
    const int vpt = rs.vpt;
    prm.pair_threads = rs.threads;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (vpt) {
        case 1: return run_tokens<1>((int)T, prm, smem, 1 + gate, st);
        case 2: return run_tokens<2>((int)T, prm, smem, 1 + gate, st);
        case 3: return run_tokens<3>((int)T, prm, smem, 1 + gate, st);
        default: return KB_ERR_UNSUPPORTED;
    }
}
