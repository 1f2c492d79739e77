// Activation expansion (MoE dispatch gather) for sm_100a:
//   out[r, :] = x[p2u[r] % T, :]    r in [0, rows), p2u[r] in [0, rows)
// Same contract as kolibri_activation_expansion_kernel
// (fusions/03_moe_prologue/fused/custom_moe_prologue.cu:453-478): the unpermuted row index is
// slot*T + token, so the source token is p2u % T.  A row with p2u outside [0, rows) is left
// untouched (the reference would read out of bounds).
//
// One warp per output row, 16-byte vectors, 4 vectors in flight per lane; source rows are
// re-read up to K times, so they are loaded through L2 with normal caching while the output
// (written once) uses evict-first stores.
#include "kb_common.cuh"

#include <algorithm>

namespace kb {

// With w != nullptr the kernel also gathers the routing weight of every permuted row:
// scales[r] = w[token*K + slot] for p2u[r] = slot*T + token (0 for a row without a source).
template <int UNROLL>
__global__ void __launch_bounds__(256) expand_rows_vec_kernel(const uint4* __restrict__ x,
                                                              uint4* __restrict__ out,
                                                              const int32_t* __restrict__ p2u,
                                                              int64_t T, int64_t rows,
                                                              int64_t vpr,
                                                              const float* __restrict__ w = nullptr,
                                                              int K = 0,
                                                              float* __restrict__ scales = nullptr) {
    pdl_wait();
    pdl_launch();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const int64_t u = __ldg(p2u + r);
        if (w != nullptr && lane == 0)
            scales[r] = (u < 0 || u >= rows) ? 0.0f : __ldg(w + (u % T) * K + u / T);
        if (u < 0 || u >= rows) continue;
        const uint4* src = x + (u % T) * vpr;
        uint4* dst = out + r * vpr;
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
}

__global__ void __launch_bounds__(256) expand_rows_byte_kernel(const uint8_t* __restrict__ x,
                                                               uint8_t* __restrict__ out,
                                                               const int32_t* __restrict__ p2u,
                                                               int64_t T, int64_t rows,
                                                               int64_t row_bytes) {
    pdl_wait();
    pdl_launch();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const int64_t u = __ldg(p2u + r);
        if (u < 0 || u >= rows) continue;
        const uint8_t* src = x + (u % T) * row_bytes;
        uint8_t* dst = out + r * row_bytes;
        for (int64_t b = lane; b < row_bytes; b += 32) dst[b] = src[b];
    }
}

}  // namespace kb

using namespace kb;

extern "C" int kb_expand_rows(const void* x, void* out, const int32_t* p2u, int64_t T,
                              int64_t rows, int64_t row_bytes, kb_stream_t stream) {
    if (T < 0 || rows < 0 || row_bytes < 0) return KB_ERR_INVALID_ARG;
    if (rows == 0 || row_bytes == 0) return KB_OK;
    if (T == 0 || !x || !out || !p2u) return KB_ERR_INVALID_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    // Eight rows per CTA (one per warp), at most 8 resident CTAs of 256 threads per SM.
    const int64_t ctas = std::min<int64_t>((rows + 7) / 8, (int64_t)device_sm_count() * 8);
    dim3 grid((unsigned)ctas), block(256);
    if (row_bytes % 16 == 0 && aligned16(x) && aligned16(out)) {
        return launch(expand_rows_vec_kernel<4>, grid, block, 0, st,
                      static_cast<const uint4*>(x), static_cast<uint4*>(out), p2u, T, rows,
                      row_bytes / 16, static_cast<const float*>(nullptr), 0,
                      static_cast<float*>(nullptr));
    }
    return launch(expand_rows_byte_kernel, grid, block, 0, st, static_cast<const uint8_t*>(x),
                  static_cast<uint8_t*>(out), p2u, T, rows, row_bytes);
}

extern "C" int kb_expand_rows_scaled(const void* x, void* out, const int32_t* p2u,
                                     const float* weights, float* scales, int64_t T, int K,
                                     int64_t row_bytes, kb_stream_t stream) {
    if (T < 0 || K <= 0 || row_bytes < 0) return KB_ERR_INVALID_ARG;
    const int64_t rows = T * K;
    if (rows == 0) return KB_OK;
    if (!x || !out || !p2u || !weights || !scales) return KB_ERR_INVALID_ARG;
    if (rows >= (int64_t)INT32_MAX) return KB_ERR_TOO_LARGE;
    if (row_bytes % 16 || !aligned16(x) || !aligned16(out)) return KB_ERR_ALIGNMENT;
    const int64_t ctas = std::min<int64_t>((rows + 7) / 8, (int64_t)device_sm_count() * 8);
    return launch(expand_rows_vec_kernel<4>, dim3((unsigned)ctas), dim3(256), 0,
                  (cudaStream_t)stream, static_cast<const uint4*>(x), static_cast<uint4*>(out),
                  p2u, T, rows, row_bytes / 16, weights, K, scales);
}
