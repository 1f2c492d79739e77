// Packed fp32 pairs for sm_100a: the f32x2 arithmetic performs two IEEE round-to-nearest
// operations per instruction, with the same results as the scalar __fmul_rn / __fadd_rn /
// fmaf on each half, so kernels can halve their multiply and add count without changing a
// rounding.  Shared by the decode chain and the Q/K norm + RoPE kernel.
#pragma once

#include "kb_common.cuh"

namespace kb {

typedef unsigned long long f2_t;
__device__ __forceinline__ f2_t f2_pack(float lo, float hi) {
    f2_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(f2_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2_t f2_mul(f2_t a, f2_t b) {
    f2_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2_t f2_add(f2_t a, f2_t b) {
    f2_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
    f2_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// bf16 pair (element 2j in the low half) -> fp32 pair, exactly.
__device__ __forceinline__ f2_t bf2_to_f2(uint32_t u) {
    return f2_pack(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
// fp32 pair -> bf16 pair, round to nearest even (as __float2bfloat16_rn on each).
__device__ __forceinline__ uint32_t f2_to_bf2(f2_t v) {
    float lo, hi;
    f2_unpack(v, lo, hi);
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
}  // namespace kb
