// dev_math.h -- device math shared by kernels that must agree bit for bit
// (an activation applied in a GEMM epilogue and in the stand-alone kernel).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace rt {

// tanh-approximated GELU with the reference's constants
// (csrc/ops/elementwise.c:186-189): 0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))).
// tanh(y) is evaluated as 1 - 2 / (1 + e^{2y}) with the hardware exp2 and
// reciprocal approximations (a few instructions instead of a full tanhf,
// which matters inside a GEMM epilogue).  For large |y| the quotient goes to
// 0 or 2 and tanh to +-1 exactly; near 0 the subtraction cancels to an
// absolute error of ~1e-7, so GELU's error stays ~1e-7 |x| -- far inside the
// 1e-4 / 1e-3 parity tolerance.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float y = 0.7978845608f * (x + 0.044715f * x * x * x);
    const float e = __expf(2.0f * y);                 // e^{2y}; inf for large y
    const float t = 1.0f - __fdividef(2.0f, 1.0f + e);  // -> 1 as e -> inf, -1 as e -> 0
    return 0.5f * x * (1.0f + t);
}

// Operand split shared by the GEMM's split pass and producers that write a
// GEMM's split A operand directly: hi = x rounded to tf32 (nearest, ties away),
// lo = x - hi, and bf16 (round to nearest even) bit patterns.
__device__ __forceinline__ float split_hi(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}
__device__ __forceinline__ uint32_t bf16_pair(float a, float b) {   // a in the low half
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
}

// Four consecutive A-operand elements (k % 4 == 0) of a row of K into the
// split planes: hi (fp32 slots) and plane 1 -- lo as fp32 (cross == false) or
// the cross layout, per 16-wide K block of width w = min(16, K - 16*kb):
// bf16 [hi(0..w-1) | lo(0..w-1)] in the block's 64 bytes.
__device__ __forceinline__ void store_split4(float* hi_row, uint16_t* x_row, int64_t k, int64_t K, float4 v,
                                             bool cross) {
    const float4 h = make_float4(split_hi(v.x), split_hi(v.y), split_hi(v.z), split_hi(v.w));
    const float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    *reinterpret_cast<float4*>(hi_row + k) = h;
    if (!cross) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(x_row) + k) = l;
        return;
    }
    const int64_t kb = k >> 4;
    const int j = (int)(k & 15);
    const int w = (int)(K - kb * 16 < 16 ? K - kb * 16 : 16);
    uint16_t* blk = x_row + kb * 32;
    *reinterpret_cast<uint2*>(blk + j) = make_uint2(bf16_pair(h.x, h.y), bf16_pair(h.z, h.w));
    *reinterpret_cast<uint2*>(blk + w + j) = make_uint2(bf16_pair(l.x, l.y), bf16_pair(l.z, l.w));
}

}  // namespace rt
