// RMSNorm building blocks shared by the residual-norm kernels (norms.cu) and the
// decode-chain kernel (chain.cu), so that both reduce and round identically.
#pragma once

#include "kb_common.cuh"

namespace kb {

// Block-wide fp32 sum: a warp butterfly, then a butterfly over the warp partials (lanes past
// the last warp adding 0).  Every warp runs the second butterfly itself, which leaves the
// same bits in every lane of every warp, so one barrier does.  `red` is a 64-float smem
// scratch of two 32-float buffers taken in turn (`turn` flips on each call and must start
// equal in every thread): a call's barrier follows every read of the buffer it leaves
// behind, so the call after it may write that buffer again.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red, int& turn) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = (blockDim.x + 31) >> 5;
    float* buf = red + 32 * turn;
    turn ^= 1;
    v = warp_sum(v);
    if (lane == 0) buf[warp] = v;
    __syncthreads();
    return warp_sum((lane < nw) ? buf[lane] : 0.0f);
}

__device__ __forceinline__ float rms_scale(float ss, int H, float eps) {
    return 1.0f / sqrtf(ss / (float)H + eps);
}

template <typename T>
__device__ __forceinline__ float rnd(float v) { return Elem<T>::to_f(Elem<T>::from_f(v)); }

// Launch shape of a row of nvec 16-byte vectors: vpt vectors per thread, threads a multiple
// of 32 (at most 512).  Thread i owns vectors i + k*threads, k < vpt.  The stand-alone norm
// kernels and the decode-chain kernel both use it, so their reductions add in one order.
// vpt == 0: the row is too long for the register kernels.
struct RowShape {
    int vpt, threads;
};
inline RowShape row_shape(int nvec) {
    int vpt = (nvec + 511) / 512;
    if (vpt > 8) return {0, 0};
    if (vpt == 5) vpt = 6;
    if (vpt == 7) vpt = 8;
    int threads = (nvec + vpt - 1) / vpt;
    threads = (threads + 31) & ~31;
    return {vpt, threads};
}

}  // namespace kb
