// Per-head Q/K RMSNorm fused with NeoX RoPE (bf16 in/out, fp32 math) for sm_100a.
//
// Math (scratch/diag_rope_fusion.py:31-38, the local statement of TensorRT-LLM's
// fusedQKNormRopeKernel as driven from benchmarks/02_benchmark_attention_norm.py:105-112):
//   y   = (x * (1/sqrt(mean(x^2) + eps))) * gamma              per head of D elements
//   a_j = float(pos) * inv_freq[j]                              j < D/2
//   out = [y1*cos(a) - y2*sin(a), y2*cos(a) + y1*sin(a)]  ->  bf16
// RNoPE layers pass no positions (pos == NULL): the rotation is the identity and the kernel
// is the harness's per-head F.rms_norm (benchmarks/11_profile_2block_e2e.py:195-196).
//
// Layout: a warp normalises whole heads, D/32 consecutive elements per lane, so the NeoX
// partner of lane l is lane l^16.  A CTA of HPC warps covers HPC*hpw heads of one token (warp w
// takes heads w, w+HPC, ...) and computes the D/2 (cos, sin) pairs of that token once in shared
// memory with the accurate sincosf.  At large T, hpw = ceil(heads/HPC): one CTA per token, so
// the trigonometry runs once per token instead of once per group of HPC heads (it dominated
// the instruction count).  At decode T, hpw = 1: the heads spread over more CTAs.
//
// Instruction count per head (the large-T kernel is issue-bound): the gammas are unpacked once
// per CTA; the products run as packed f32x2 pairs (two IEEE round-to-nearest operations per
// instruction, so the same bits as the scalar __fmul_rn / __fadd_rn); the (cos, sin) table is
// laid out in each lane's element order with the first half's sine negated, so the rotation is
// one uniform out = y*c + other*s' (y*c - other*s = y*c + other*(-s) exactly) read with one
// vector load per table.  Sums of squares keep the scalar fmaf order of the reference kernel.
#include "f32x2.cuh"
#include "kb_common.cuh"

#include <algorithm>
#include <type_traits>

namespace kb {

template <int EPL> struct LaneWords;
template <> struct LaneWords<2> { using T = uint32_t; };
template <> struct LaneWords<4> { using T = uint2; };
template <> struct LaneWords<8> { using T = uint4; };

template <int D, int HPC, int MAXW>
__global__ void __launch_bounds__(HPC * 32) qk_norm_rope_kernel(
    const __nv_bfloat16* q_in, __nv_bfloat16* q_out, const __nv_bfloat16* k_in,
    __nv_bfloat16* k_out, const __nv_bfloat16* __restrict__ gq,
    const __nv_bfloat16* __restrict__ gk, const int32_t* __restrict__ pos,
    const float* __restrict__ inv_freq, int64_t T, int Hq, int Hkv, int64_t qs, int64_t ks,
    float eps, int groups, int hpw) {
    constexpr int EPL = D / 32;  // elements per lane
    constexpr int NP = EPL / 2;  // packed pairs per lane
    static_assert(EPL == 2 || EPL == 4 || EPL == 8, "D must be 64, 128 or 256");
    using Lane = typename LaneWords<EPL>::T;
    union LaneU {
        Lane l;
        uint32_t w[NP];
    };
    pdl_wait();
    pdl_launch();
    // The rotation table in lane-element order: entry e = l*EPL + i holds cos(a_j) and
    // -sin(a_j) (first half, e < D/2) or +sin(a_j) (second half), j = e mod D/2.
    __shared__ __align__(16) float cs[D], sn[D];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = blockIdx.x / groups;
    const int head0 = (int)(blockIdx.x % groups) * HPC * hpw + warp;
    const int heads = Hq + Hkv;
    const __nv_bfloat16* qt = q_in + t * qs;
    const __nv_bfloat16* kt = k_in + t * ks;

    // Issue every head's loads (and both gammas) before the trigonometry.
    LaneU xl[MAXW];
#pragma unroll
    for (int i = 0; i < MAXW; ++i) {
        const int head = head0 + i * HPC;
        xl[i].l = Lane{};
        if (i < hpw && head < heads) {
            const __nv_bfloat16* src = head < Hq ? qt + head * D : kt + (head - Hq) * D;
            xl[i].l = *(reinterpret_cast<const Lane*>(src) + lane);
        }
    }
    LaneU glq, glk;
    glq.l = Lane{};
    glk.l = Lane{};
    if (Hq > 0) glq.l = __ldg(reinterpret_cast<const Lane*>(gq) + lane);
    if (Hkv > 0) glk.l = __ldg(reinterpret_cast<const Lane*>(gk) + lane);
    f2_t gqp[NP], gkp[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) {
        gqp[k] = bf2_to_f2(glq.w[k]);
        gkp[k] = bf2_to_f2(glk.w[k]);
    }
    const bool rope = pos != nullptr;
    if (rope) {
        const float p = (float)__ldg(pos + t);
        for (int j = threadIdx.x; j < D / 2; j += blockDim.x) {
            float s_, c_;
            sincosf(__fmul_rn(p, __ldg(inv_freq + j)), &s_, &c_);
            cs[j] = c_;
            sn[j] = -s_;
            cs[j + D / 2] = c_;
            sn[j + D / 2] = s_;
        }
        __syncthreads();
    }
    f2_t csp[NP], snp[NP];
    if (rope) {
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            csp[k] = f2_pack(cs[lane * EPL + 2 * k], cs[lane * EPL + 2 * k + 1]);
            snp[k] = f2_pack(sn[lane * EPL + 2 * k], sn[lane * EPL + 2 * k + 1]);
        }
    }

#pragma unroll
    for (int i = 0; i < MAXW; ++i) {
        const int head = head0 + i * HPC;
        if (!(i < hpw && head < heads)) continue;
        const bool is_q = head < Hq;
        f2_t y[NP];
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            y[k] = bf2_to_f2(xl[i].w[k]);
            float lo, hi;
            f2_unpack(y[k], lo, hi);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
        }
        ss = warp_sum(ss);
        const float r = 1.0f / sqrtf(ss / (float)D + eps);
        const f2_t rr = f2_pack(r, r);
        LaneU ov;
#pragma unroll
        for (int k = 0; k < NP; ++k) {
            f2_t v = f2_mul(f2_mul(y[k], rr), is_q ? gqp[k] : gkp[k]);
            if (rope) {
                const f2_t other = (f2_t)__shfl_xor_sync(FULL_MASK, (unsigned long long)v, 16);
                v = f2_add(f2_mul(v, csp[k]), f2_mul(other, snp[k]));
            }
            ov.w[k] = f2_to_bf2(v);
        }
        __nv_bfloat16* dst = is_q ? q_out + t * qs + head * D : k_out + t * ks + (head - Hq) * D;
        *(reinterpret_cast<Lane*>(dst) + lane) = ov.l;
    }
}

namespace {

template <int D>
int qk_launch(const void* q_in, void* q_out, const void* k_in, void* k_out, const void* gq,
              const void* gk, const int32_t* pos, const float* inv_freq, int64_t T, int Hq,
              int Hkv, int64_t qs, int64_t ks, float eps, cudaStream_t st) {
    constexpr int HPC = 8, MAXW = 9;
    const int heads = Hq + Hkv;
    const int per_warp = (heads + HPC - 1) / HPC;
    // Decode batches: one head per warp over more CTAs; otherwise one CTA per token (up to
    // HPC*MAXW heads), so the token's (cos, sin) pairs are computed once.
    const bool spread = T * per_warp <= 4LL * device_sm_count();
    const int hpw = spread ? 1 : std::min(per_warp, MAXW);
    const int groups = (heads + HPC * hpw - 1) / (HPC * hpw);
    const int64_t ctas = T * groups;
    if (ctas > (int64_t)INT32_MAX) return KB_ERR_TOO_LARGE;
    return launch(qk_norm_rope_kernel<D, HPC, MAXW>, dim3((unsigned)ctas), dim3(HPC * 32), 0, st,
                  static_cast<const __nv_bfloat16*>(q_in), static_cast<__nv_bfloat16*>(q_out),
                  static_cast<const __nv_bfloat16*>(k_in), static_cast<__nv_bfloat16*>(k_out),
                  static_cast<const __nv_bfloat16*>(gq), static_cast<const __nv_bfloat16*>(gk),
                  pos, inv_freq, T, Hq, Hkv, qs, ks, eps, groups, hpw);
}

inline bool aligned_to(const void* p, unsigned a) {
    return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int kb_qk_norm_rope(const void* q_in, void* q_out, const void* k_in, void* k_out,
                               const void* gamma_q, const void* gamma_k, const int32_t* pos,
                               const float* inv_freq, int64_t T, int Hq, int Hkv, int D,
                               int64_t q_tok_stride, int64_t k_tok_stride, float eps,
                               kb_stream_t stream) {
    if (T < 0 || Hq < 0 || Hkv < 0) return KB_ERR_INVALID_ARG;
    if (D != 64 && D != 128 && D != 256) return KB_ERR_UNSUPPORTED;
    if (T == 0 || Hq + Hkv == 0) return KB_OK;
    if ((Hq > 0 && (!q_in || !q_out || !gamma_q)) || (Hkv > 0 && (!k_in || !k_out || !gamma_k)))
        return KB_ERR_INVALID_ARG;
    if (pos && !inv_freq) return KB_ERR_INVALID_ARG;
    if (q_tok_stride < (int64_t)Hq * D || k_tok_stride < (int64_t)Hkv * D) return KB_ERR_INVALID_ARG;
    // Each lane moves D/32 bf16 = D/16 bytes: rows and strides must keep that alignment.
    const unsigned al = (unsigned)(D / 16);
    const int64_t se = al / 2;  // stride alignment in elements
    if (Hq > 0 && (!aligned_to(q_in, al) || !aligned_to(q_out, al) || q_tok_stride % se)) return KB_ERR_ALIGNMENT;
    if (Hkv > 0 && (!aligned_to(k_in, al) || !aligned_to(k_out, al) || k_tok_stride % se)) return KB_ERR_ALIGNMENT;
    if ((Hq > 0 && !aligned_to(gamma_q, al)) || (Hkv > 0 && !aligned_to(gamma_k, al))) return KB_ERR_ALIGNMENT;
    cudaStream_t st = (cudaStream_t)stream;
    switch (D) {
        case 64: return qk_launch<64>(q_in, q_out, k_in, k_out, gamma_q, gamma_k, pos, inv_freq, T, Hq, Hkv, q_tok_stride, k_tok_stride, eps, st);
        case 128: return qk_launch<128>(q_in, q_out, k_in, k_out, gamma_q, gamma_k, pos, inv_freq, T, Hq, Hkv, q_tok_stride, k_tok_stride, eps, st);
        default: return qk_launch<256>(q_in, q_out, k_in, k_out, gamma_q, gamma_k, pos, inv_freq, T, Hq, Hkv, q_tok_stride, k_tok_stride, eps, st);
    }
}
