// Decode-chain kernel for sm_100a: every layer of the non-GEMM decode chain of a Kolibri-style
// MoE decoder in ONE persistent launch, for decode batches of T <= 4 tokens.
//
// Per layer, in the order of the reference harness's decoder_layer
// (benchmarks/11_profile_2block_e2e.py:215-266, with the next layer's input_layernorm
// :222-227 fused into the post-MoE pair), each stage starting after the previous one ended:
//   A  Q/K RMSNorm + NeoX RoPE of q, k (RNoPE layers: the norm only)
//   B  sandwich: h = r + RMSNorm(attn_out)*g1 ; moe_in = RMSNorm(h)*g2
//   C  router GEMV: logits[t][e] = float(bf16(moe_in[t] . W[e]))
//   D  router (top-K of logits + bias, sigmoid weights) and expert maps
//   E  activation expansion: permuted[r] = moe_in[p2u[r] % T]
//   F  post-MoE pair: r = h + RMSNorm(moe_out)*g3 ; next = RMSNorm(r)*g4
//
// Every CTA (one per SM) runs every stage on whole rows.  The residual stream, h and moe_in of
// the T tokens stay in its registers, so a stage never waits for another CTA except where the
// data really is spread over the GPU: the router GEMV.  CTA c owns experts c, c + G, ... (G
// CTAs); it keeps their W rows in shared memory, computes their logits and publishes each one
// as a 64-bit record: the call's layer tag in the high word, the value in the low word.
// 64-bit accesses are single-copy atomic, so the poll that sees the tag also delivers the
// value.  Every CTA then polls the E records of the layer, and all CTAs rank the same logits
// with the same code, so they all hold the same selections.  That all-gather is the only
// cross-CTA wait of a layer; records alternate between two banks by layer parity, and a CTA
// can be at most one layer ahead of another (it needs the other's records to leave a layer).
//
// Each output element is written once, by an owner CTA: vector v of token t of h, moe_in,
// next and the residual by CTA (t*nvec + v) mod G, Q/K head j by CTA j mod G, map entries and
// logits by the CTA that owns them, so the writes are spread over all SMs.
// The next layer's weights (gammas, the owned W rows, the bias) arrive in shared memory by bulk
// copies (plain cp.async.bulk from this GPU's memory into this CTA's own) while the current
// layer runs; loads of the GEMM stand-ins (q, k, attn_out, moe_out) are issued only when their
// stage starts and bypass L1, as loads of a tensor that a GEMM has just written would.
//
// The arithmetic is that of the stand-alone kernels (norm_math.cuh and the row shape of
// norms.cu, route_math.cuh, the Q/K formula and lane layout of qk_norm_rope.cu), so every
// routing-independent output is bit-identical to the stage-by-stage path.  Every wait is
// bounded; a wait that gives up sets the workspace error word, the CTAs leave at the end of
// the layer, and later calls report offsets = -1 until the workspace is zero-filled again.
#include "f32x2.cuh"
#include "kb_common.cuh"
#include "norm_math.cuh"
#include "route_math.cuh"

#include <algorithm>

namespace kb {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kCT = 384;                     // threads per CTA (a 6144-wide row: 2 vectors each)
constexpr int kCW = kCT / 32;                // warps per CTA
constexpr int kChainMaxLayers = 256;         // layer descriptors held in shared memory
constexpr int kChainMaxT = 4;                // tokens per call
constexpr int kChainMaxK = 8;                // top-K
constexpr int kMaxOwn = 4;                   // router experts per CTA
constexpr int kHalfD = 64;                   // head_dim 128
constexpr int kQkChunk = 6;                  // heads per warp with their loads in flight together
constexpr int kMaxChunks = E_MAX / 32;       // 32-expert chunks of a router row
constexpr long long kChainSpin = 1LL << 21;  // bounded waits (about a second of polling)
constexpr int kRedVals = kMaxOwn * kChainMaxT;
// The threshold of the router stage is the K-th largest of the kCW warp maxima.
static_assert(kChainMaxK <= kCW, "the router threshold needs at least K expert groups");
static_assert(kChainMaxK * kChainMaxT <= 32, "the selections of one call fit one warp");

// Workspace (zero-filled before the first call): epoch word (+1 per completed call), exit
// counter, error word, then the logit records [2 banks][kChainMaxT][E_MAX].
constexpr size_t kWsEpoch = 0, kWsDone = 64, kWsErr = 128, kWsRec = 256;
constexpr size_t kWsBytes = kWsRec + sizeof(unsigned long long) * 2 * kChainMaxT * E_MAX;
// Error-word values.
constexpr int kErrTimeout = 1;    // a bounded wait gave up
constexpr int kErrAlignment = 2;  // a layer's weight pointer is not 16-byte aligned

enum : int { kBarQK = 0, kBarA = 1, kBarW = 2, kBarB = 3, kNumBars = 4 };

struct ChainParams {
    const kb_chain_layer_t* layers;
    int L, T, H, Hq, Hkv, E, K;
    int pt;    // threads owning row vectors (row_shape of the stand-alone norm kernels)
    int vpt;   // row vectors per such thread (1 or 2)
    int nown;  // router experts per CTA
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
    unsigned* epoch;
    unsigned* done;
    int* err;
    unsigned long long* rec;
    long long spin;  // poll limit of the bounded waits (kb_set_wait_limit)
};

// ------------------------------------------------------------------------------------
// Shared memory
// ------------------------------------------------------------------------------------
struct SmemLayout {
    size_t bar, gqk, ga, gb, w, bias, layers, xrow, cs, sn, red, wmax, cand, ncand, sel, perm,
        flag, total;
};
__host__ __device__ constexpr size_t al128(size_t v) { return (v + 127) & ~size_t(127); }
__host__ __device__ inline SmemLayout smem_layout(int H, int nown, int L) {
    SmemLayout s{};
    size_t o = 0;
    s.bar = o;    o = al128(o + kNumBars * sizeof(uint64_t));
    s.gqk = o;    o = al128(o + 2 * 128 * sizeof(bf16));
    s.ga = o;     o = al128(o + (size_t)2 * H * sizeof(bf16));
    s.gb = o;     o = al128(o + (size_t)2 * H * sizeof(bf16));
    s.w = o;      o = al128(o + (size_t)nown * H * sizeof(bf16));
    s.bias = o;   o = al128(o + E_MAX * sizeof(float));
    s.layers = o; o = al128(o + (size_t)L * sizeof(kb_chain_layer_t));
    s.xrow = o;   o = al128(o + (size_t)kChainMaxT * E_MAX * sizeof(float));
    s.cs = o;     o = al128(o + kChainMaxT * kHalfD * sizeof(float));
    s.sn = o;     o = al128(o + kChainMaxT * kHalfD * sizeof(float));
    s.red = o;    o = al128(o + (size_t)2 * kRedVals * 33 * sizeof(float));
    s.wmax = o;   o = al128(o + kChainMaxT * 32 * sizeof(uint32_t));
    s.cand = o;   o = al128(o + kChainMaxT * 32 * sizeof(unsigned long long));
    s.ncand = o;  o = al128(o + kChainMaxT * sizeof(int));
    s.sel = o;    o = al128(o + 32 * sizeof(int));
    s.perm = o;   o = al128(o + 32 * sizeof(int));
    s.flag = o;   o = al128(o + 8 * sizeof(int));
    s.total = o;
    return s;
}

struct Smem {
    uint64_t* bar;             // [kNumBars] one mbarrier per weight buffer
    bf16* gqk;                 // [2][128]  g_q, g_k
    bf16* ga;                  // [2][H]    g_post_attn, g_pre_moe
    bf16* gb;                  // [2][H]    g_post_ffn, g_input_ln
    bf16* w;                   // [nown][H] router rows of the owned experts
    float* bias;               // [E_MAX]   gate bias (+0 for -0), zeros without one
    kb_chain_layer_t* layers;  // [L]
    float* xrow;               // [kChainMaxT][E_MAX] logits of the layer
    float* cs;                 // [kChainMaxT][64]
    float* sn;                 // [kChainMaxT][64]
    float* red;                // [2][kRedVals][33] block reductions, two buffers in turn
    uint32_t* wmax;            // [kChainMaxT][32] warp maxima of the router keys
    unsigned long long* cand;  // [kChainMaxT][32] router candidates
    int* ncand;                // [kChainMaxT]
    int* sel;                  // [32] selections, (token, slot) order
    int* perm;                 // [32] token of each permuted row
    int* flag;                 // [8]  flag[0]: leave at the end of this layer;
                               //      flag[4 + b]: bulk-copy phases issued on buffer b
};

__device__ __forceinline__ Smem carve(unsigned char* base, const SmemLayout& l) {
    Smem s;
    s.bar = reinterpret_cast<uint64_t*>(base + l.bar);
    s.gqk = reinterpret_cast<bf16*>(base + l.gqk);
    s.ga = reinterpret_cast<bf16*>(base + l.ga);
    s.gb = reinterpret_cast<bf16*>(base + l.gb);
    s.w = reinterpret_cast<bf16*>(base + l.w);
    s.bias = reinterpret_cast<float*>(base + l.bias);
    s.layers = reinterpret_cast<kb_chain_layer_t*>(base + l.layers);
    s.xrow = reinterpret_cast<float*>(base + l.xrow);
    s.cs = reinterpret_cast<float*>(base + l.cs);
    s.sn = reinterpret_cast<float*>(base + l.sn);
    s.red = reinterpret_cast<float*>(base + l.red);
    s.wmax = reinterpret_cast<uint32_t*>(base + l.wmax);
    s.cand = reinterpret_cast<unsigned long long*>(base + l.cand);
    s.ncand = reinterpret_cast<int*>(base + l.ncand);
    s.sel = reinterpret_cast<int*>(base + l.sel);
    s.perm = reinterpret_cast<int*>(base + l.perm);
    s.flag = reinterpret_cast<int*>(base + l.flag);
    return s;
}

// ------------------------------------------------------------------------------------
// Memory primitives
// ------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned su32(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mb_init(uint64_t* b, unsigned n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mb_expect(uint64_t* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
                 : "memory");
}
// Non-blocking test of the phase of parity `parity`.
__device__ __forceinline__ bool mb_try(uint64_t* b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(su32(b)), "r"(parity) : "memory");
    return ok != 0;
}
// One bulk copy global -> this CTA's shared memory (16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(su32(dst)), "l"(src), "r"(bytes), "r"(su32(b)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void cp4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Loads of the GEMM stand-ins: cached in L2 only.
__device__ __forceinline__ uint4 ld_cg16(const void* p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ld_cg8(const void* p) {
    uint2 r;
    asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
// 64-bit accesses are single-copy atomic: a record's tag and value are seen together.  The
// record is published with an atomic exchange, which is performed at L2 at once (a plain
// relaxed store measured up to ~3 us before other SMs saw it).
__device__ __forceinline__ void st_rec(unsigned long long* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.relaxed.gpu.global.exch.b64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    (void)old;
}
__device__ __forceinline__ unsigned long long ld_rec(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

union V8 {
    uint4 u;
    uint32_t w[4];
    bf16 e[8];
};

union V4 {
    uint2 u;
    bf16 e[4];
};

// Marks this CTA to leave at the end of the layer, and the call as failed (error word).
__device__ __forceinline__ void give_up(const ChainParams& p, const Smem& s, int code) {
    s.flag[0] = 1;
    atomicCAS(p.err, 0, code);
}
__device__ __forceinline__ bool leaving(const ChainParams& p, const Smem& s) {
    return *(volatile int*)s.flag || *(volatile int*)p.err;
}

// Every thread waits for the phase of parity `par` of weight buffer b (bounded).
__device__ __forceinline__ void wait_weights(const ChainParams& p, const Smem& s, int b, unsigned par) {
    long long it = 0;
    while (!mb_try(s.bar + b, par)) {
        if (++it > p.spin || ((it & 255) == 0 && leaving(p, s))) {
            give_up(p, s, kErrTimeout);
            return;
        }
        __nanosleep(20);
    }
}

// Thread 0: bulk copies of layer l's weights for buffer b.  Issued only after every thread
// saw the buffer's previous phase complete (no wait of this CTA gave up), so a buffer never
// has two phases in flight.
__device__ void issue_weights(const ChainParams& p, const Smem& s, int b, int l) {
    const kb_chain_layer_t& Ly = s.layers[l];
    const unsigned row = (unsigned)p.H * (unsigned)sizeof(bf16);
    s.flag[4 + b] += 1;
    fence_proxy_async();  // earlier generic reads of the buffer come before the copy's writes
    if (b == kBarQK) {
        mb_expect(s.bar + b, 2 * 128 * sizeof(bf16));
        bulk_g2s(s.gqk, Ly.g_q, 128 * sizeof(bf16), s.bar + b);
        bulk_g2s(s.gqk + 128, Ly.g_k, 128 * sizeof(bf16), s.bar + b);
    } else if (b == kBarA || b == kBarB) {
        bf16* dst = b == kBarA ? s.ga : s.gb;
        mb_expect(s.bar + b, 2 * row);
        bulk_g2s(dst, b == kBarA ? Ly.g_post_attn : Ly.g_post_ffn, row, s.bar + b);
        bulk_g2s(dst + p.H, b == kBarA ? Ly.g_pre_moe : Ly.g_input_ln, row, s.bar + b);
    } else {
        const int c = blockIdx.x, G = gridDim.x;
        int mine = 0;
        for (int m = 0; m < p.nown; ++m)
            if (c + m * G < p.E) mine = m + 1;
        mb_expect(s.bar + b, (unsigned)mine * row);
        const bf16* W = static_cast<const bf16*>(Ly.w_gate_t);
        for (int m = 0; m < mine; ++m)
            bulk_g2s(s.w + (size_t)m * p.H, W + (size_t)(c + m * G) * p.H, row, s.bar + b);
    }
}

// Layer l's gate bias into shared memory (+0 for -0, zeros without a bias): 4-byte
// asynchronous copies, completed by cp_wait_all before the router reads them.
__device__ __forceinline__ void issue_bias(const ChainParams& p, const Smem& s, int l) {
    const float* b = s.layers[l].gate_bias;
    for (int e = threadIdx.x; e < p.E; e += kCT) {
        if (b) cp4(s.bias + e, b + e);
        else s.bias[e] = 0.0f;
    }
    cp_commit();
}

// Block-wide sums of n values at once; each value is reduced exactly as block_sum reduces it
// (warp butterfly, then a butterfly over the warp partials, lanes past the last warp adding
// 0).  One barrier; the next call must take the other buffer.
// The butterfly of warp_sum over the kCW warp partials w[0..kCW) (lanes past kCW holding
// 0.0f), as lane 0 would compute it, from shared memory: the same additions in the same tree,
// so the same bits (every lane of a xor butterfly ends with identical bits).
__device__ __forceinline__ float butterfly_of_partials(const float* w) {
    static_assert(kCW <= 16, "partials fit the lower half-warp");
    float a[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = (i < kCW ? w[i] : 0.0f) + 0.0f;  // level 16: + lane i+16
    float b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = a[i] + a[i + 8];  // level 8
    float c4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) c4[i] = b[i] + b[i + 4];  // level 4
    const float d0 = c4[0] + c4[2], d1 = c4[1] + c4[3];  // level 2
    return d0 + d1;                                       // level 1
}

// Block-wide sums of MAXN values at once; each value is reduced exactly as block_sum reduces
// it (warp butterfly, then a butterfly over the warp partials, lanes past the last warp
// adding 0), the second butterfly replayed from shared memory.  One barrier; the next call
// must take the other buffer.
template <int MAXN>
__device__ __forceinline__ void block_sum_n(float (&v)[MAXN], float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int m = 0; m < MAXN; ++m) {
        const float s = warp_sum(v[m]);
        if (lane == 0) red[m * 33 + warp] = s;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < MAXN; ++m) v[m] = butterfly_of_partials(red + m * 33);
}

// ------------------------------------------------------------------------------------
// Stages
// ------------------------------------------------------------------------------------

// A: per-head RMSNorm + NeoX RoPE of every head of the T tokens (one warp per head, four
// consecutive elements per lane, as qk_norm_rope_kernel<128>: the NeoX partner of lane l is
// lane l^16).  Head j (over tokens and q then k heads) is stored by CTA j mod G (j < 3G).  A
// warp takes QC heads at once and runs each step for all of them together (independent
// chains side by side); lane i < QC computes head i's 1/sqrt and hands it out by a shuffle.
// The sum of squares of each head is the butterfly of warp_sum, so every bit matches; the
// products run on fp32 pairs (the scalar kernel's roundings; the first half's y*c - o*s is
// y*c + o*(-s), the same bits).  The q/k loads are issued before the wait for g_q/g_k.
// rot (TT == 1): the lane's rotation pairs (cos, then sin negated on the first half).
template <int TT>
__device__ __forceinline__ void stage_qk(const ChainParams& p, const Smem& s, bool rope, unsigned par,
                                         const f2_t (&rot)[4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const int HH = p.Hq + p.Hkv, nh = TT * HH;
    // Nothing in the chain reads q_out / k_out, so a CTA computes only the heads it owns
    // (head hd belongs to CTA hd mod G): at most ceil(nh / G) of them, warp w taking its w-th.
    const int n_own = c < nh ? (nh - c + G - 1) / G : 0;
    constexpr int QC = TT <= 2 ? kQkChunk : kQkChunk / 2;  // fewer heads at once at larger T
    bool waited = false;
    f2_t gq[2], gk[2];
    for (int base = warp; base < n_own; base += kCW * QC) {
        V4 xv[QC];
        int tt[QC], hq[QC];
#pragma unroll
        for (int cc = 0; cc < QC; ++cc) {  // clamped heads: all loads in flight at once
            const int hd = c + min(base + cc * kCW, n_own - 1) * G;
            const int t = TT == 1 ? 0 : (hd >= HH) + (hd >= 2 * HH) + (hd >= 3 * HH);
            tt[cc] = t;
            hq[cc] = hd - t * HH;
            const bf16* src = hq[cc] < p.Hq ? p.q + ((size_t)t * p.Hq + hq[cc]) * 128
                                            : p.k + ((size_t)t * p.Hkv + (hq[cc] - p.Hq)) * 128;
            xv[cc].u = ld_cg8(src + lane * 4);
        }
        if (!waited) {
            wait_weights(p, s, kBarQK, par);
            waited = true;
            const uint2 a = reinterpret_cast<const uint2*>(s.gqk)[lane];
            const uint2 b = reinterpret_cast<const uint2*>(s.gqk + 128)[lane];
            gq[0] = bf2_to_f2(a.x);
            gq[1] = bf2_to_f2(a.y);
            gk[0] = bf2_to_f2(b.x);
            gk[1] = bf2_to_f2(b.y);
        }
        f2_t y[QC][2];
        float ss[QC];
#pragma unroll
        for (int cc = 0; cc < QC; ++cc) {
            y[cc][0] = bf2_to_f2(xv[cc].u.x);
            y[cc][1] = bf2_to_f2(xv[cc].u.y);
            float a0, a1, a2, a3;
            f2_unpack(y[cc][0], a0, a1);
            f2_unpack(y[cc][1], a2, a3);
            ss[cc] = fmaf(a3, a3, fmaf(a2, a2, fmaf(a1, a1, fmaf(a0, a0, 0.0f))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int cc = 0; cc < QC; ++cc) ss[cc] += __shfl_xor_sync(FULL_MASK, ss[cc], o);
        float mine = ss[0];
#pragma unroll
        for (int cc = 1; cc < QC; ++cc) mine = (lane == cc) ? ss[cc] : mine;
        const float rl = 1.0f / sqrtf(mine / 128.0f + p.eps);
#pragma unroll
        for (int cc = 0; cc < QC; ++cc) {
            const float r = __shfl_sync(FULL_MASK, rl, cc);
            const f2_t rr = f2_pack(r, r);
            const bool is_q = hq[cc] < p.Hq;
            y[cc][0] = f2_mul(f2_mul(y[cc][0], rr), is_q ? gq[0] : gk[0]);
            y[cc][1] = f2_mul(f2_mul(y[cc][1], rr), is_q ? gq[1] : gk[1]);
        }
        uint2 o[QC];
        if (rope) {
#pragma unroll
            for (int cc = 0; cc < QC; ++cc) {
                f2_t cp0, cp1, sp0, sp1;
                if (TT == 1) {
                    cp0 = rot[0]; cp1 = rot[1]; sp0 = rot[2]; sp1 = rot[3];
                } else {
                    const float4 c4 = reinterpret_cast<const float4*>(s.cs + tt[cc] * kHalfD)[lane & 15];
                    const float4 s4 = reinterpret_cast<const float4*>(s.sn + tt[cc] * kHalfD)[lane & 15];
                    const float sg = lane < 16 ? -1.0f : 1.0f;
                    cp0 = f2_pack(c4.x, c4.y);
                    cp1 = f2_pack(c4.z, c4.w);
                    sp0 = f2_pack(sg * s4.x, sg * s4.y);
                    sp1 = f2_pack(sg * s4.z, sg * s4.w);
                }
                float y0, y1, y2, y3;
                f2_unpack(y[cc][0], y0, y1);
                f2_unpack(y[cc][1], y2, y3);
                const f2_t o0 = f2_pack(__shfl_xor_sync(FULL_MASK, y0, 16), __shfl_xor_sync(FULL_MASK, y1, 16));
                const f2_t o1 = f2_pack(__shfl_xor_sync(FULL_MASK, y2, 16), __shfl_xor_sync(FULL_MASK, y3, 16));
                o[cc].x = f2_to_bf2(f2_add(f2_mul(y[cc][0], cp0), f2_mul(o0, sp0)));
                o[cc].y = f2_to_bf2(f2_add(f2_mul(y[cc][1], cp1), f2_mul(o1, sp1)));
            }
        } else {
#pragma unroll
            for (int cc = 0; cc < QC; ++cc) {
                o[cc].x = f2_to_bf2(y[cc][0]);
                o[cc].y = f2_to_bf2(y[cc][1]);
            }
        }
#pragma unroll
        for (int cc = 0; cc < QC; ++cc) {
            if (base + cc * kCW < n_own) {  // each owned head once (the clamped ones repeat)
                const int t = tt[cc];
                bf16* dst = hq[cc] < p.Hq ? p.q_out + ((size_t)t * p.Hq + hq[cc]) * 128
                                          : p.k_out + ((size_t)t * p.Hkv + (hq[cc] - p.Hq)) * 128;
                reinterpret_cast<uint2*>(dst)[lane] = o[cc];
            }
        }
    }
    if (!waited) wait_weights(p, s, kBarQK, par);
}

// Row vectors of this thread: k-th = tid + k*pt (k < 2), valid if ok[k]; voff = v (uint4 index).
struct RowSlots {
    int v[2];
    bool ok[2];
};

// B / F: sum = res + RMSNorm(a)*g1 (rounded) ; norm = RMSNorm(sum)*g2 for the TT rows.  Thread
// i < pt owns row vectors i + k*pt (k < vpt), as the stand-alone kernel's threads do; the
// others add zeros to the reductions, which changes no bit.  a comes from global memory, res
// from registers, g1/g2 from shared memory.  sum goes to registers (and the owned vectors to
// sum_g); norm to registers if NORM_ALL (else only the owned vectors are computed), and the
// owned vectors to norm_g.  own: bit 2t+k marks vector k of token t as owned by this CTA.
// Products and sums run on fp32 pairs with the scalar kernel's roundings; the sums of squares
// stay sequential fmaf in element order, as in the stand-alone kernel.
template <int TT, bool NORM_ALL>
__device__ __forceinline__ void stage_pair(const ChainParams& p, const Smem& s, const RowSlots& rs,
                                           const bf16* a, const V8 (&res)[TT][2], int gbar,
                                           unsigned par, const bf16* g1, const bf16* g2,
                                           V8 (&sum)[TT][2], V8 (&norm)[TT][2], bf16* sum_g,
                                           bf16* norm_g, unsigned own, float* red_a, float* red_b) {
    const int H = p.H;
    V8 va[TT][2];
    float ss[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int k = 0; k < 2; ++k)
            va[t][k].u = rs.ok[k] ? ld_cg16(a + (size_t)t * H + (size_t)rs.v[k] * 8) : make_uint4(0, 0, 0, 0);
    wait_weights(p, s, gbar, par);  // the gammas are read after the first reduction
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        ss[t] = 0.0f;
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float x0 = __uint_as_float(va[t][k].w[j] << 16);
                const float x1 = __uint_as_float(va[t][k].w[j] & 0xffff0000u);
                ss[t] = fmaf(x0, x0, ss[t]);
                ss[t] = fmaf(x1, x1, ss[t]);
            }
    }
    block_sum_n<TT>(ss, red_a);
    float ss2[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        ss2[t] = 0.0f;
        const float r1 = rms_scale(ss[t], H, p.eps);
        const f2_t r1r1 = f2_pack(r1, r1);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            V8 vh;
            vh.u = make_uint4(0, 0, 0, 0);
            if (rs.ok[k]) {
                V8 vg;
                vg.u = reinterpret_cast<const uint4*>(g1)[rs.v[k]];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const f2_t m = f2_mul(f2_mul(bf2_to_f2(va[t][k].w[j]), r1r1), bf2_to_f2(vg.w[j]));
                    const f2_t post = bf2_to_f2(f2_to_bf2(m));
                    const uint32_t hb = f2_to_bf2(f2_add(bf2_to_f2(res[t][k].w[j]), post));
                    vh.w[j] = hb;
                    const float h0 = __uint_as_float(hb << 16), h1 = __uint_as_float(hb & 0xffff0000u);
                    ss2[t] = fmaf(h0, h0, ss2[t]);
                    ss2[t] = fmaf(h1, h1, ss2[t]);
                }
                if (sum_g && ((own >> (2 * t + k)) & 1u))
                    reinterpret_cast<uint4*>(sum_g + (size_t)t * H)[rs.v[k]] = vh.u;
            }
            sum[t][k] = vh;
        }
    }
    block_sum_n<TT>(ss2, red_b);
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        const float r2 = rms_scale(ss2[t], H, p.eps);
        const f2_t r2r2 = f2_pack(r2, r2);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const bool mine = (own >> (2 * t + k)) & 1u;
            V8 vx;
            vx.u = make_uint4(0, 0, 0, 0);
            if (rs.ok[k] && (NORM_ALL || mine)) {
                V8 vg;
                vg.u = reinterpret_cast<const uint4*>(g2)[rs.v[k]];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    vx.w[j] = f2_to_bf2(f2_mul(f2_mul(bf2_to_f2(sum[t][k].w[j]), r2r2), bf2_to_f2(vg.w[j])));
                if (norm_g && mine) reinterpret_cast<uint4*>(norm_g + (size_t)t * H)[rs.v[k]] = vx.u;
            }
            if (NORM_ALL) norm[t][k] = vx;
        }
    }
}

// Top-K of token t by K rounds over all of its keys (lane l holds experts l, l + 32, ...):
// each round takes the warp's largest key, the lowest expert among equal keys (redux max,
// then redux min), and clears it.  The path for rows whose keys tie at the threshold.
__device__ void topk_rounds(const Smem& s, int t, int E, int K) {
    const int lane = threadIdx.x & 31;
    uint32_t key[kMaxChunks];
#pragma unroll
    for (int j = 0; j < kMaxChunks; ++j) {
        const int e = lane + 32 * j;
        key[j] = (e < E) ? okey(s.xrow[t * E_MAX + e] + (s.bias[e] + 0.0f)) : 0u;
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
        const uint32_t wmx = __reduce_max_sync(FULL_MASK, best);
        const unsigned cnd = (best == wmx && best != 0u) ? (unsigned)(lane + 32 * bj) : 0xffffffffu;
        const unsigned widx = __reduce_min_sync(FULL_MASK, cnd);
        if (cnd == widx) {
#pragma unroll
            for (int j = 0; j < kMaxChunks; ++j)
                if (j == bj) key[j] = 0u;
        }
        if (lane == 0) s.sel[t * K + r] = (int)widx;
    }
}

// D: exact top-K of every token; the same keys and tie rule as the router kernels: score =
// logit + (bias + 0), ordered by okey (NaN highest), the lower expert first.
//  1. (In the all-gather, as each record arrives.)  Thread i keys experts i and i + kCT; each
//     warp's largest key of token t is its group maximum (warp w's group: experts 32w.. and
//     kCT + 32w..), in wmax[t][w].
//  2. tau = the K-th largest group maximum: the K groups with the largest maxima each hold a
//     key >= tau, so every key of the top K is >= tau.  With fewer than K groups, tau = 0
//     (every key is a candidate).
//  3. Keys >= tau are the candidates, appended to the token's list.
//  4. Warp t: with C <= 32 candidates, each one's rank is the number of candidates above it
//     in (key, then lower expert) order, found in one pass; ranks below K are the output.
//     More candidates (ties at tau) take the K rounds of topk_rounds.
// Leaves sel (all tokens) complete for every thread; writes ids and weights (CTA 0).
template <int TT>
__device__ __forceinline__ void stage_route(const ChainParams& p, const Smem& s,
                                            const uint32_t (&key)[TT][2]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, K = p.K;
    const int ng = min(kCW, (E + 31) >> 5);  // warps holding at least one expert
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        const uint32_t mj = lane < ng ? s.wmax[t * 32 + lane] : 0u;
        int above = 0;
#pragma unroll
        for (int i = 0; i < kCW; ++i) above += (__shfl_sync(FULL_MASK, mj, i) > mj) ? 1 : 0;
        const uint32_t tau = (ng >= K)
            ? __reduce_min_sync(FULL_MASK, (lane < ng && above < K) ? mj : 0xffffffffu) : 0u;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int e = tid + j * kCT;
            const bool take = e < E && key[t][j] >= tau;
            const unsigned b = __ballot_sync(FULL_MASK, take);
            if (b) {  // uniform over the warp
                int base = 0;
                if (lane == 0) base = atomicAdd(s.ncand + t, __popc(b));
                base = __shfl_sync(FULL_MASK, base, 0);
                const int slot = base + __popc(b & ((1u << lane) - 1u));
                if (take && slot < 32)
                    s.cand[t * 32 + slot] =
                        ((unsigned long long)key[t][j] << 32) | (unsigned)(0xffffffffu - (unsigned)e);
            }
        }
    }
    __syncthreads();
    if (warp < TT) {
        const int t = warp;
        const int C = s.ncand[t];
        if (C <= 32) {
            const unsigned long long mine = lane < C ? s.cand[t * 32 + lane] : 0ull;
            int rank = 0;
#pragma unroll 8
            for (int j = 0; j < C; ++j) rank += (s.cand[t * 32 + j] > mine) ? 1 : 0;
            if (lane < C && rank < K) s.sel[t * K + rank] = (int)(0xffffffffu - (unsigned)mine);
        } else {
            topk_rounds(s, t, E, K);
        }
        __syncwarp();
        if (lane < K && blockIdx.x == 0) {
            const int id = s.sel[t * K + lane];
            p.ids[t * K + lane] = id;
            p.w[t * K + lane] = sigmoid_acc(s.xrow[t * E_MAX + id]);
        }
    }
    __syncthreads();
}

// D (maps) + E: maps of the n = T*K <= 32 selections without a scan: offsets[e] = selections
// below e, counts[e] = selections equal to e, rank of selection i = selections below its
// expert + equal ones before it (selections are in (token, slot) order).  Entry e of offsets
// and counts is written by CTA e mod G, p2u and u2p by CTA 0.  Every CTA derives the token of
// each permuted row and stores its share of the expansion from the moe_in rows it holds.
template <int TT>
__device__ __forceinline__ void stage_maps_expand(const ChainParams& p, const Smem& s,
                                                  const V8 (&x)[TT][2], unsigned long long own_perm) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    constexpr int T = TT;
    const int E = p.E, K = p.K, n = T * K, nvec = p.H / 8;
    for (int e = c + tid * G; e <= E; e += kCT * G) {
        int below = 0, equal = 0;
#pragma unroll
        for (int i = 0; i < kChainMaxK * TT; ++i) {
            if (i < n) {
                const int v = s.sel[i];
                below += (v < e) ? 1 : 0;
                equal += (v == e) ? 1 : 0;
            }
        }
        p.offsets[e] = (int64_t)below;
        if (p.counts && e < E) p.counts[e] = equal;
    }
    if (TT > 1 || c == 0) {
        if (warp == 0) {
            const int e = (lane < n) ? s.sel[lane] : 0x7fffffff;
            int rank = 0;
#pragma unroll
            for (int i = 0; i < kChainMaxK * TT; ++i) {
                if (i < n) {
                    const int v = s.sel[i];
                    rank += (v < e || (v == e && i < lane)) ? 1 : 0;
                }
            }
            if (lane < n) {
                const int tok = lane / K, slot = lane - tok * K;
                const int u = slot * T + tok;
                if (c == 0) {
                    p.p2u[rank] = u;
                    if (p.u2p) p.u2p[u] = rank;
                }
                s.perm[rank] = tok;
            }
        }
        if (TT > 1) __syncthreads();
    }
    if (p.permuted) {
        // own_perm bit 2r+k: vector k of this thread in permuted row r is this CTA's to store.
        unsigned long long bits = own_perm;
        while (bits) {
            const int b = __ffsll((long long)bits) - 1;
            bits &= bits - 1ull;
            const int r = b >> 1, k = b & 1;
            const int tok = TT > 1 ? s.perm[r] : 0;
            uint4 val = k ? x[0][1].u : x[0][0].u;
#pragma unroll
            for (int t = 1; t < TT; ++t)
                if (t == tok) val = k ? x[t][1].u : x[t][0].u;
            st_stream(reinterpret_cast<uint4*>(p.permuted) + (size_t)r * nvec + tid + k * p.pt, val);
        }
    }
}

template <int TT>
__global__ void __launch_bounds__(kCT, 1) decode_chain_kernel(const __grid_constant__ ChainParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int tid = threadIdx.x;
    const int c = blockIdx.x, G = gridDim.x;
    const int H = p.H, E = p.E, nvec = H / 8;  // p.T == TT
    if (*(volatile int*)p.err) {  // an earlier call gave up: report and do nothing
        if (c == 0)
            for (int e = tid; e <= E; e += kCT) p.offsets[e] = -1;
        return;
    }
    const Smem s = carve(smem_raw, smem_layout(H, p.nown, p.L));
    {  // every layer descriptor into shared memory once
        const int words = p.L * (int)(sizeof(kb_chain_layer_t) / sizeof(int));
        for (int i = tid; i < words; i += kCT)
            reinterpret_cast<int*>(s.layers)[i] = reinterpret_cast<const int*>(p.layers)[i];
    }
    if (tid == 0) {
        for (int b = 0; b < kNumBars; ++b) mb_init(s.bar + b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < 8) s.flag[tid] = 0;
    if (p.pos) {
        for (int i = tid; i < TT * kHalfD; i += kCT) {
            const int t = i / kHalfD, j = i - t * kHalfD;
            float sv, cv;
            sincosf(__fmul_rn((float)__ldg(p.pos + t), __ldg(p.inv_freq + j)), &sv, &cv);
            s.cs[i] = cv;
            s.sn[i] = sv;
        }
    }
    __syncthreads();
    // Bulk copies need 16-byte aligned sources: check every layer's weights before any copy.
    int bad = 0;
    for (int l = tid; l < p.L; l += kCT) {
        const kb_chain_layer_t& Ly = s.layers[l];
        const uintptr_t a16 = reinterpret_cast<uintptr_t>(Ly.g_post_attn) |
                              reinterpret_cast<uintptr_t>(Ly.g_pre_moe) |
                              reinterpret_cast<uintptr_t>(Ly.g_post_ffn) |
                              reinterpret_cast<uintptr_t>(Ly.g_input_ln) |
                              reinterpret_cast<uintptr_t>(Ly.g_q) | reinterpret_cast<uintptr_t>(Ly.g_k) |
                              reinterpret_cast<uintptr_t>(Ly.w_gate_t);
        const bool nul = !Ly.g_post_attn || !Ly.g_pre_moe || !Ly.g_post_ffn || !Ly.g_input_ln ||
                         !Ly.g_q || !Ly.g_k || !Ly.w_gate_t;
        if ((a16 & 15u) || (reinterpret_cast<uintptr_t>(Ly.gate_bias) & 3u) || nul) bad = 1;
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0) atomicCAS(p.err, 0, kErrAlignment);
        if (c == 0)
            for (int e = tid; e <= E; e += kCT) p.offsets[e] = -1;
        return;
    }
    if (tid == 0)
        for (int b = 0; b < kNumBars; ++b) issue_weights(p, s, b, 0);
    issue_bias(p, s, 0);
    const unsigned epoch = *(volatile unsigned*)p.epoch;

    // Vectors of this thread: k-th = tid + k*pt; own bit 2t+k: vector (t, k) of a row output
    // is this CTA's to store; own_perm bit 2r+k: the same in permuted row r.
    RowSlots rs;
    unsigned own = 0u;
    unsigned long long own_perm = 0ull;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int v = tid + k * p.pt;
        rs.v[k] = v;
        rs.ok[k] = tid < p.pt && k < p.vpt && v < nvec;
        if (rs.ok[k]) {
            for (int t = 0; t < TT; ++t)
                if ((t * nvec + v) % G == c) own |= 1u << (2 * t + k);
            for (int rr = 0; rr < TT * p.K; ++rr)
                if ((rr * nvec + v) % G == c) own_perm |= 1ull << (2 * rr + k);
        }
    }
    V8 r[TT][2], hh[TT][2], x[TT][2];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int k = 0; k < 2; ++k)
            r[t][k].u = rs.ok[k] ? reinterpret_cast<const uint4*>(p.r_in + (size_t)t * H)[rs.v[k]]
                                 : make_uint4(0, 0, 0, 0);
    f2_t rot[4] = {0ull, 0ull, 0ull, 0ull};  // TT == 1: this lane's rotation pairs
    if (TT == 1 && p.pos) {
        const int lane_ = tid & 31;
        const float4 c4 = reinterpret_cast<const float4*>(s.cs)[lane_ & 15];
        const float4 s4 = reinterpret_cast<const float4*>(s.sn)[lane_ & 15];
        const float sg = lane_ < 16 ? -1.0f : 1.0f;
        rot[0] = f2_pack(c4.x, c4.y);
        rot[1] = f2_pack(c4.z, c4.w);
        rot[2] = f2_pack(sg * s4.x, sg * s4.y);
        rot[3] = f2_pack(sg * s4.z, sg * s4.w);
    }
    int mine = 0;  // experts owned: c + m*G, m < mine
    for (int m = 0; m < p.nown; ++m)
        if (c + m * G < E) mine = m + 1;
    const int warp = tid >> 5, lane = tid & 31;

    float* red0 = s.red;
    float* red1 = s.red + kRedVals * 33;
    int l = 0;
    for (; l < p.L; ++l) {
        const kb_chain_layer_t& Ly = s.layers[l];
        const unsigned par = (unsigned)(l & 1);
        const unsigned tag = epoch * 256u + (unsigned)l + 1u;
        const bool more = l + 1 < p.L;

        // ---- A: Q/K norm + RoPE ----
        stage_qk<TT>(p, s, !Ly.rnope && p.pos != nullptr, par, rot);
        __syncthreads();
        if (s.flag[0]) break;  // uniform: read after the barrier, written before it
        // Every read of the previous layer's post-MoE gammas is behind the barrier above.
        if (tid == 0) {
            if (more) issue_weights(p, s, kBarQK, l + 1);
            if (l > 0) issue_weights(p, s, kBarB, l);
        }

        // ---- B: sandwich ----
        stage_pair<TT, true>(p, s, rs, p.attn_out, r, kBarA, par, s.ga, s.ga + H, hh, x, p.h, p.moe_in,
                             own, red0, red1);

        // ---- C: router GEMV over the owned experts, records out ----
        // Each thread's dot products run on fp32 pairs (even and odd elements), added at the end.
        wait_weights(p, s, kBarW, par);
        float acc[kMaxOwn * TT];
        {
            f2_t acc2[kMaxOwn][TT];
#pragma unroll
            for (int m = 0; m < kMaxOwn; ++m)
#pragma unroll
                for (int t = 0; t < TT; ++t) acc2[m][t] = 0ull;  // (+0, +0)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                if (rs.ok[k]) {
                    f2_t xf[TT][4];
#pragma unroll
                    for (int t = 0; t < TT; ++t)
#pragma unroll
                        for (int j = 0; j < 4; ++j) xf[t][j] = bf2_to_f2(x[t][k].w[j]);
#pragma unroll
                    for (int m = 0; m < kMaxOwn; ++m) {
                        if (m < mine) {
                            V8 wv;
                            wv.u = reinterpret_cast<const uint4*>(s.w + (size_t)m * H)[rs.v[k]];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const f2_t wf = bf2_to_f2(wv.w[j]);
#pragma unroll
                                for (int t = 0; t < TT; ++t) acc2[m][t] = f2_fma(xf[t][j], wf, acc2[m][t]);
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < kMaxOwn; ++m)
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    float lo, hi;
                    f2_unpack(acc2[m][t], lo, hi);
                    acc[m * TT + t] = lo + hi;
                }
        }
        // Warp partials of every (expert, token) value; thread m*TT + t then replays the
        // cross-warp butterfly of its own value only.
#pragma unroll
        for (int i = 0; i < kMaxOwn * TT; ++i) {
            const float wsum = warp_sum(acc[i]);
            if (lane == 0) red0[i * 33 + warp] = wsum;
        }
        __syncthreads();
        unsigned long long* bank = p.rec + (size_t)par * kChainMaxT * E_MAX;
        if (tid < mine * TT) {
            const int m = tid / TT, t = tid - m * TT;
            const float v = __bfloat162float(__float2bfloat16_rn(butterfly_of_partials(red0 + tid * 33)));
            const int e = c + m * G;
            st_rec(bank + (size_t)t * E_MAX + e, ((unsigned long long)tag << 32) | __float_as_uint(v));
            p.logits[(size_t)t * E + e] = v;
            if (p.trace_logits) p.trace_logits[((size_t)l * TT + t) * E + e] = v;
        }
        // Every read of ga and of the W rows is behind the barrier above; the copies are issued
        // by the last warp, after the records are out.
        if (tid == kCT - 32 && more && !s.flag[0]) {
            issue_weights(p, s, kBarA, l + 1);
            issue_weights(p, s, kBarW, l + 1);
        }

        // ---- all-gather of the layer's logits: thread i polls records i and i + kCT ----
        {
            unsigned pending = 0u;
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int t = 0; t < TT; ++t)
                    if (tid + j * kCT < E) pending |= 1u << (j * TT + t);
            long long it = 0;
            while (pending) {
                unsigned long long v[2][TT];
#pragma unroll
                for (int j = 0; j < 2; ++j)
#pragma unroll
                    for (int t = 0; t < TT; ++t)
                        v[j][t] = ((pending >> (j * TT + t)) & 1u)
                                      ? ld_rec(bank + (size_t)t * E_MAX + tid + j * kCT) : 0ull;
#pragma unroll
                for (int j = 0; j < 2; ++j)
#pragma unroll
                    for (int t = 0; t < TT; ++t)
                        if (((pending >> (j * TT + t)) & 1u) && (unsigned)(v[j][t] >> 32) == tag) {
                            s.xrow[t * E_MAX + tid + j * kCT] = __uint_as_float((unsigned)v[j][t]);
                            pending &= ~(1u << (j * TT + t));
                        }
                if (pending) {
                    if (++it > p.spin || ((it & 1023) == 0 && leaving(p, s))) {
                        give_up(p, s, kErrTimeout);
                        break;
                    }
                    __nanosleep(32);
                }
            }
        }
        // Router step 1 on the gathered logits: keys and the warp maxima (this thread's bias
        // entries are its own 4-byte copies).
        cp_wait_all();
        uint32_t key[TT][2];
#pragma unroll
        for (int t = 0; t < TT; ++t) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int e = tid + j * kCT;
                key[t][j] = e < E ? okey(s.xrow[t * E_MAX + e] + (s.bias[e] + 0.0f)) : 0u;
            }
            const uint32_t m = __reduce_max_sync(FULL_MASK, max(key[t][0], key[t][1]));
            if (lane == 0) s.wmax[t * 32 + warp] = m;
        }
        if (tid < TT) s.ncand[tid] = 0;
        __syncthreads();

        // ---- D: router, maps; E: expansion ----
        stage_route<TT>(p, s, key);
        if (more) issue_bias(p, s, l + 1);  // every bias read is behind stage_route's barrier
        stage_maps_expand<TT>(p, s, x, own_perm);

        // ---- F: post-MoE + next layer's input norm ----
        V8 unused[TT][2];
        stage_pair<TT, false>(p, s, rs, p.moe_out, hh, kBarB, par, s.gb, s.gb + H, r, unused, p.r_out,
                              p.nxt, own, red1, red0);
    }
    __syncthreads();
    if (s.flag[0] && l == p.L) l = p.L - 1;  // a wait of the last layer gave up
    if (l < p.L) {  // left early: no copy may still be writing when the CTA exits
        if (tid == 0) {
            // The last phase issued on each buffer (every earlier one completed) is the current
            // phase or, complete, the one before it; its parity waits only in the first case.
            for (int b = 0; b < kNumBars; ++b) {
                const int n = s.flag[4 + b];
                long long it = 0;
                while (n > 0 && !mb_try(s.bar + b, (unsigned)((n - 1) & 1)) && ++it < kChainSpin)
                    __nanosleep(20);
            }
        }
        cp_wait_all();
        for (int e = c + tid * G; e <= E; e += kCT * G) p.offsets[e] = -1;
        __syncthreads();
    }
    // The last CTA out advances the epoch (every CTA read it at the start) and resets the exit
    // counter; the kernel boundary publishes both to the next call.
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(p.done, 1u) == (unsigned)G - 1u) {
            atomicExch(p.done, 0u);
            atomicAdd(p.epoch, 1u);
        }
    }
}

// ------------------------------------------------------------------------------------
// Host
// ------------------------------------------------------------------------------------
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

template <int TT>
int run_chain(const ChainParams& prm, size_t smem, int grid, cudaStream_t st) {
    auto* kern = decode_chain_kernel<TT>;
    int err = allow_smem(kern, smem);
    if (err) return err;
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kCT, smem) != cudaSuccess || nb < 1)
        return KB_ERR_UNSUPPORTED;
    return launch_coop(kern, dim3((unsigned)grid), dim3(kCT), smem, st, prm);
}

bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
    const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + nb && y < x + na;
}

}  // namespace
}  // namespace kb

namespace kb {
size_t chain_err_offset() { return kWsErr; }
}  // namespace kb

using namespace kb;

extern "C" size_t kb_decode_chain_workspace_bytes(void) { return kWsBytes; }

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
    const RowShape rs = H % 8 == 0 ? row_shape(H / 8) : RowShape{0, 0};
    if (T > kChainMaxT || D != 128 || H % 8 != 0 || rs.vpt == 0 || rs.vpt > 2 || rs.threads > kCT ||
        E > E_MAX || K > kChainMaxK || K > E || Hq + Hkv <= 0)
        return KB_ERR_UNSUPPORTED;
    if (!layers || !attn_out || !moe_out || !q || !k || !residual_in || !residual_out || !h ||
        !moe_in || !next || !q_out || !k_out || !logits || !ids || !weights || !offsets ||
        !p2u || !permuted || (pos && !inv_freq))
        return KB_ERR_INVALID_ARG;
    if (!workspace || workspace_bytes < kWsBytes) return KB_ERR_WORKSPACE;
    const void* vec_ptrs[] = {attn_out, moe_out, q, k, residual_in, residual_out, h, moe_in,
                              next, q_out, k_out, permuted, workspace};
    for (const void* v : vec_ptrs)
        if (!aligned16(v)) return KB_ERR_ALIGNMENT;
    // Every CTA reads the GEMM stand-ins in every layer while owners store the outputs, so no
    // output may overlap an input (the residual stream may be updated in place: every CTA
    // reads residual_in before any CTA can finish the first layer's router all-gather).
    const size_t row = (size_t)T * H * sizeof(bf16);
    const size_t qb = (size_t)T * Hq * D * sizeof(bf16), kbb = (size_t)T * Hkv * D * sizeof(bf16);
    const void* ins[] = {attn_out, moe_out, q, k};
    const size_t in_b[] = {row, row, qb, kbb};
    const void* outs[] = {h, moe_in, next, q_out, k_out, permuted, residual_out};
    const size_t out_b[] = {row, row, row, qb, kbb, (size_t)T * K * H * sizeof(bf16), row};
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 7; ++j)
            if (in_b[i] && out_b[j] && overlaps(ins[i], in_b[i], outs[j], out_b[j])) return KB_ERR_INVALID_ARG;
    const int G = device_sm_count();
    const int nown = (E + G - 1) / G;
    if ((int64_t)T * (Hq + Hkv) > 3 * (int64_t)G) return KB_ERR_UNSUPPORTED;  // head owners
    if (nown > kMaxOwn) return KB_ERR_UNSUPPORTED;
    const size_t smem = smem_layout(H, nown, n_layers).total;
    if (smem > (size_t)227 * 1024) return KB_ERR_UNSUPPORTED;
    ChainParams prm;
    prm.layers = layers;
    prm.L = n_layers;
    prm.T = (int)T;
    prm.H = H;
    prm.Hq = Hq;
    prm.Hkv = Hkv;
    prm.E = E;
    prm.K = K;
    prm.pt = rs.threads;
    prm.vpt = rs.vpt;
    prm.nown = nown;
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
    prm.epoch = reinterpret_cast<unsigned*>(wsb + kWsEpoch);
    prm.done = reinterpret_cast<unsigned*>(wsb + kWsDone);
    prm.err = reinterpret_cast<int*>(wsb + kWsErr);
    prm.rec = reinterpret_cast<unsigned long long*>(wsb + kWsRec);
    prm.spin = wait_limit(kChainSpin);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (T) {
        case 1: return run_chain<1>(prm, smem, G, st);
        case 2: return run_chain<2>(prm, smem, G, st);
        case 3: return run_chain<3>(prm, smem, G, st);
        case 4: return run_chain<4>(prm, smem, G, st);
        default: return KB_ERR_UNSUPPORTED;
    }
}
