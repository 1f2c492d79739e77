// Residual RMSNorm fusions for sm_100a, one CTA per row, 16-byte vectors held in registers.
//
//   kb_residual_norm_pair: sum = residual + RMSNorm(a)*g1 ; norm = RMSNorm(sum)*g2
//     = fused_sandwich_norm (fusions/01_sandwich_norm/fused/fused_sandwich_norm.py:46-72) and the
//       post-MoE + next-layer pre-attention pair (benchmarks/11_profile_2block_e2e.py:229-231,269-270)
//   kb_add_rms_norm:       sum = a + b ; out = RMSNorm(sum)*g
//     = fused_add_post_moe_norm (fusions/02_post_moe_norm/fused/fused_post_moe_norm.py:54-77)
//
// Rounding follows the eager reference (fusions/01_sandwich_norm/baseline/trtllm_baseline.py:78-95,
// fusions/02_post_moe_norm/baseline/trtllm_baseline.py:77-90): F.rms_norm computes
// dtype((x_f32 * (1/sqrt(mean(x_f32^2) + eps))) * g_f32) with one rounding, the residual add is
// rounded to the activation dtype, and the second norm reads the rounded sum.  Products use
// __fmul_rn so that no FMA contraction changes the rounding.
#include "kb_common.cuh"
#include "norm_math.cuh"

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

namespace kb {

// ------------------------------------------------------------------------------------
// Register kernels: each thread owns VPT 16-byte vectors v = tid + i*blockDim.
// ------------------------------------------------------------------------------------
// This thread's vectors of row `row` of x and y (zeros past the row or past `rows`).
template <typename T, int VPT>
__device__ __forceinline__ void load_row_pair(const T* __restrict__ x, const T* __restrict__ y,
                                              int64_t row, int64_t rows, int H, int nvec,
                                              Vec16<T>* vx, Vec16<T>* vy) {
    const bool in = row < rows;
    const uint4* px = reinterpret_cast<const uint4*>(x + (in ? row : 0) * H);
    const uint4* py = reinterpret_cast<const uint4*>(y + (in ? row : 0) * H);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int v = threadIdx.x + i * blockDim.x;
        if (in && v < nvec) {
            vx[i].u = ld_stream(px + v);
            vy[i].u = ld_stream(py + v);
        } else {
            vx[i].u = make_uint4(0, 0, 0, 0);
            vy[i].u = make_uint4(0, 0, 0, 0);
        }
    }
}

template <typename T, int VPT>
__global__ void __launch_bounds__(512) residual_norm_pair_kernel(
    const T* __restrict__ a, const T* __restrict__ res, const T* __restrict__ g1,
    const T* __restrict__ g2, T* sum_out, T* norm_out, int64_t rows, int H, float eps) {
    pdl_wait();
    pdl_launch();
    using V = Vec16<T>;
    constexpr int N = V::N;
    __shared__ float red[64];
    int turn = 0;
    const int nvec = H / N;
    // The CTA walks rows blockIdx.x, + gridDim.x, ...; the next row's loads are issued before
    // the current row's reductions, so two rows per CTA are in flight.
    V na[VPT], nr[VPT];
    load_row_pair<T, VPT>(a, res, (int64_t)blockIdx.x, rows, H, nvec, na, nr);
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        V va[VPT], vr[VPT];
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            va[i].u = na[i].u;
            vr[i].u = nr[i].u;
        }
        load_row_pair<T, VPT>(a, res, row + gridDim.x, rows, H, nvec, na, nr);
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
#pragma unroll
            for (int e = 0; e < N; ++e) {
                const float x = Elem<T>::to_f(va[i].e[e]);
                ss = fmaf(x, x, ss);
            }
        }
        const float r1 = rms_scale(block_sum(ss, red, turn), H, eps);
        float ss2 = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int v = threadIdx.x + i * blockDim.x;
            if (v < nvec) {
                V vg;
                vg.u = __ldg(reinterpret_cast<const uint4*>(g1) + v);
                V vh;
#pragma unroll
                for (int e = 0; e < N; ++e) {
                    const float post = rnd<T>(__fmul_rn(__fmul_rn(Elem<T>::to_f(va[i].e[e]), r1),
                                                       Elem<T>::to_f(vg.e[e])));
                    const T h = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(vr[i].e[e]), post));
                    vh.e[e] = h;
                    const float hf = Elem<T>::to_f(h);
                    ss2 = fmaf(hf, hf, ss2);
                }
                vr[i].u = vh.u;
                reinterpret_cast<uint4*>(sum_out + row * H)[v] = vh.u;
            }
        }
        const float r2 = rms_scale(block_sum(ss2, red, turn), H, eps);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int v = threadIdx.x + i * blockDim.x;
            if (v < nvec) {
                V vg;
                vg.u = __ldg(reinterpret_cast<const uint4*>(g2) + v);
                V vx;
#pragma unroll
                for (int e = 0; e < N; ++e)
                    vx.e[e] = Elem<T>::from_f(__fmul_rn(__fmul_rn(Elem<T>::to_f(vr[i].e[e]), r2),
                                                        Elem<T>::to_f(vg.e[e])));
                reinterpret_cast<uint4*>(norm_out + row * H)[v] = vx.u;
            }
        }
    }
}

template <typename T, int VPT>
__global__ void __launch_bounds__(512) add_rms_norm_kernel(
    const T* __restrict__ a, const T* __restrict__ b, const T* __restrict__ g, T* out, T* sum_out,
    int64_t rows, int H, float eps) {
    pdl_wait();
    pdl_launch();
    using V = Vec16<T>;
    constexpr int N = V::N;
    __shared__ float red[64];
    int turn = 0;
    const int nvec = H / N;
    V na[VPT], nb[VPT];   // next row, loaded one row ahead (see residual_norm_pair_kernel)
    load_row_pair<T, VPT>(a, b, (int64_t)blockIdx.x, rows, H, nvec, na, nb);
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        V ca[VPT], cb[VPT];
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            ca[i].u = na[i].u;
            cb[i].u = nb[i].u;
        }
        load_row_pair<T, VPT>(a, b, row + gridDim.x, rows, H, nvec, na, nb);
        V vs[VPT];
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int v = threadIdx.x + i * blockDim.x;
            if (v < nvec) {
                const V& va = ca[i];
                const V& vb = cb[i];
#pragma unroll
                for (int e = 0; e < N; ++e) {
                    vs[i].e[e] = Elem<T>::from_f(
                        __fadd_rn(Elem<T>::to_f(va.e[e]), Elem<T>::to_f(vb.e[e])));
                    const float x = Elem<T>::to_f(vs[i].e[e]);
                    ss = fmaf(x, x, ss);
                }
                if (sum_out) reinterpret_cast<uint4*>(sum_out + row * H)[v] = vs[i].u;
            } else {
                vs[i].u = make_uint4(0, 0, 0, 0);
            }
        }
        const float r = rms_scale(block_sum(ss, red, turn), H, eps);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int v = threadIdx.x + i * blockDim.x;
            if (v < nvec) {
                V vg, vo;
                vg.u = __ldg(reinterpret_cast<const uint4*>(g) + v);
#pragma unroll
                for (int e = 0; e < N; ++e)
                    vo.e[e] = Elem<T>::from_f(__fmul_rn(__fmul_rn(Elem<T>::to_f(vs[i].e[e]), r),
                                                        Elem<T>::to_f(vg.e[e])));
                reinterpret_cast<uint4*>(out + row * H)[v] = vo.u;
            }
        }
    }
}

// ------------------------------------------------------------------------------------
// Generic kernels (any H, any alignment): the row is staged in shared memory as fp32.
// ------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(512) residual_norm_pair_generic(
    const T* __restrict__ a, const T* __restrict__ res, const T* __restrict__ g1,
    const T* __restrict__ g2, T* sum_out, T* norm_out, int64_t rows, int H, float eps) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float rowbuf[];
    __shared__ float red[64];
    int turn = 0;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            const float x = Elem<T>::to_f(a[row * H + i]);
            rowbuf[i] = x;
            ss = fmaf(x, x, ss);
        }
        const float r1 = rms_scale(block_sum(ss, red, turn), H, eps);
        float ss2 = 0.0f;
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            const float post = rnd<T>(__fmul_rn(__fmul_rn(rowbuf[i], r1), Elem<T>::to_f(g1[i])));
            const T h = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(res[row * H + i]), post));
            const float hf = Elem<T>::to_f(h);
            rowbuf[i] = hf;
            sum_out[row * H + i] = h;
            ss2 = fmaf(hf, hf, ss2);
        }
        const float r2 = rms_scale(block_sum(ss2, red, turn), H, eps);
        for (int i = threadIdx.x; i < H; i += blockDim.x)
            norm_out[row * H + i] =
                Elem<T>::from_f(__fmul_rn(__fmul_rn(rowbuf[i], r2), Elem<T>::to_f(g2[i])));
        __syncthreads();
    }
}

template <typename T>
__global__ void __launch_bounds__(512) add_rms_norm_generic(
    const T* __restrict__ a, const T* __restrict__ b, const T* __restrict__ g, T* out, T* sum_out,
    int64_t rows, int H, float eps) {
    pdl_wait();
    pdl_launch();
    extern __shared__ float rowbuf[];
    __shared__ float red[64];
    int turn = 0;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            const T s = Elem<T>::from_f(
                __fadd_rn(Elem<T>::to_f(a[row * H + i]), Elem<T>::to_f(b[row * H + i])));
            if (sum_out) sum_out[row * H + i] = s;
            const float x = Elem<T>::to_f(s);
            rowbuf[i] = x;
            ss = fmaf(x, x, ss);
        }
        const float r = rms_scale(block_sum(ss, red, turn), H, eps);
        for (int i = threadIdx.x; i < H; i += blockDim.x)
            out[row * H + i] =
                Elem<T>::from_f(__fmul_rn(__fmul_rn(rowbuf[i], r), Elem<T>::to_f(g[i])));
        __syncthreads();
    }
}

namespace {

constexpr int kMaxGenericH = 48 * 1024;  // fp32 row in <= 192 KB of shared memory

inline unsigned row_grid(int64_t rows) {
    return (unsigned)std::min<int64_t>(rows, (int64_t)INT32_MAX);
}

// Grid of the register kernels: at most the CTAs that are resident at once (every CTA then
// walks rows with a stride of the grid and keeps the next row's loads in flight).
template <typename... KArgs>
unsigned resident_grid(void (*kern)(KArgs...), int threads, int64_t rows) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        int& v = cache[std::make_tuple(reinterpret_cast<const void*>(kern), threads, dev)];
        if (v == 0) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kern, threads, 0) != cudaSuccess ||
                v <= 0)
                v = 1;
        }
        per_sm = v;
    }
    return (unsigned)std::min<int64_t>(rows, (int64_t)device_sm_count() * per_sm);
}

template <typename T>
int pair_launch(const void* a, const void* res, const void* g1, const void* g2, void* sum_out,
                void* norm_out, int64_t rows, int H, float eps, cudaStream_t st) {
    constexpr int N = 16 / sizeof(T);
    const bool vec = (H % N == 0) && aligned16(a) && aligned16(res) && aligned16(g1) &&
                     aligned16(g2) && aligned16(sum_out) && aligned16(norm_out);
    const RowShape rs = vec ? row_shape(H / N) : RowShape{0, 0};
    const T* A = static_cast<const T*>(a);
    const T* R = static_cast<const T*>(res);
    const T* G1 = static_cast<const T*>(g1);
    const T* G2 = static_cast<const T*>(g2);
    T* S = static_cast<T*>(sum_out);
    T* O = static_cast<T*>(norm_out);
    dim3 grid(row_grid(rows));
#define KB_PAIR(V)                                                                           \
    case V:                                                                                  \
        return launch(residual_norm_pair_kernel<T, V>,                                       \
                      dim3(resident_grid(residual_norm_pair_kernel<T, V>, rs.threads, rows)),  \
                      dim3(rs.threads), 0, st, A, R, G1, G2, S, O, rows, H, eps);
    switch (rs.vpt) {
        KB_PAIR(1) KB_PAIR(2) KB_PAIR(3) KB_PAIR(4) KB_PAIR(6) KB_PAIR(8)
        default: break;
    }
#undef KB_PAIR
    if (H > kMaxGenericH) return KB_ERR_UNSUPPORTED;
    const size_t smem = (size_t)H * sizeof(float);
    int err = allow_smem(residual_norm_pair_generic<T>, smem);
    if (err) return err;
    return launch(residual_norm_pair_generic<T>, grid, dim3(512), smem, st, A, R, G1, G2, S, O,
                  rows, H, eps);
}

template <typename T>
int add_launch(const void* a, const void* b, const void* g, void* out, void* sum_out,
               int64_t rows, int H, float eps, cudaStream_t st) {
    constexpr int N = 16 / sizeof(T);
    const bool vec = (H % N == 0) && aligned16(a) && aligned16(b) && aligned16(g) &&
                     aligned16(out) && (sum_out == nullptr || aligned16(sum_out));
    const RowShape rs = vec ? row_shape(H / N) : RowShape{0, 0};
    const T* A = static_cast<const T*>(a);
    const T* B = static_cast<const T*>(b);
    const T* G = static_cast<const T*>(g);
    T* O = static_cast<T*>(out);
    T* S = static_cast<T*>(sum_out);
    dim3 grid(row_grid(rows));
#define KB_ADD(V)                                                                              \
    case V:                                                                                    \
        return launch(add_rms_norm_kernel<T, V>,                                               \
                      dim3(resident_grid(add_rms_norm_kernel<T, V>, rs.threads, rows)),         \
                      dim3(rs.threads), 0, st, A, B, G, O, S, rows, H, eps);
    switch (rs.vpt) {
        KB_ADD(1) KB_ADD(2) KB_ADD(3) KB_ADD(4) KB_ADD(6) KB_ADD(8)
        default: break;
    }
#undef KB_ADD
    if (H > kMaxGenericH) return KB_ERR_UNSUPPORTED;
    const size_t smem = (size_t)H * sizeof(float);
    int err = allow_smem(add_rms_norm_generic<T>, smem);
    if (err) return err;
    return launch(add_rms_norm_generic<T>, grid, dim3(512), smem, st, A, B, G, O, S, rows, H, eps);
}

int check_rows(int64_t T, int64_t H, int dtype) {
    if (T < 0 || H <= 0) return KB_ERR_INVALID_ARG;
    if (H >= (int64_t)INT32_MAX) return KB_ERR_TOO_LARGE;
    if (dtype != KB_BF16 && dtype != KB_F16 && dtype != KB_F32) return KB_ERR_UNSUPPORTED;
    return KB_OK;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int kb_residual_norm_pair(const void* a, const void* residual, const void* g1,
                                     const void* g2, void* sum_out, void* norm_out, int64_t T,
                                     int64_t H, float eps, int dtype, kb_stream_t stream) {
    int st = check_rows(T, H, dtype);
    if (st) return st;
    if (T == 0) return KB_OK;
    if (!a || !residual || !g1 || !g2 || !sum_out || !norm_out) return KB_ERR_INVALID_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    switch (dtype) {
        case KB_BF16: return pair_launch<__nv_bfloat16>(a, residual, g1, g2, sum_out, norm_out, T, (int)H, eps, s);
        case KB_F16: return pair_launch<__half>(a, residual, g1, g2, sum_out, norm_out, T, (int)H, eps, s);
        default: return pair_launch<float>(a, residual, g1, g2, sum_out, norm_out, T, (int)H, eps, s);
    }
}

extern "C" int kb_add_rms_norm(const void* a, const void* b, const void* g, void* out,
                               void* sum_out, int64_t T, int64_t H, float eps, int dtype,
                               kb_stream_t stream) {
    int st = check_rows(T, H, dtype);
    if (st) return st;
    if (T == 0) return KB_OK;
    if (!a || !b || !g || !out) return KB_ERR_INVALID_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    switch (dtype) {
        case KB_BF16: return add_launch<__nv_bfloat16>(a, b, g, out, sum_out, T, (int)H, eps, s);
        case KB_F16: return add_launch<__half>(a, b, g, out, sum_out, T, (int)H, eps, s);
        default: return add_launch<float>(a, b, g, out, sum_out, T, (int)H, eps, s);
    }
}
