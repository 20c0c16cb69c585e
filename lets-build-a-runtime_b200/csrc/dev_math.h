// dev_math.h -- device math shared by kernels that must agree bit for bit
// (an activation applied in a GEMM epilogue and in the stand-alone kernel).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
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

// ---- element-wise arithmetic shared by the element-wise kernels and the
// small-graph kernel (csrc/ops/elementwise.c, csrc/ops/shape.c:46-51) ----
enum UnaryKind { U_RELU, U_EXP, U_TANH, U_POW, U_GELU, U_RSQRT, U_SILU, U_NEG, U_COS, U_SIN };

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

template <int K>
__device__ __forceinline__ float unary_op(float v, float p) {
    if (K == U_RELU) return v > 0.0f ? v : 0.0f;
    if (K == U_EXP) return expf(v);
    if (K == U_TANH) return tanhf(v);
    if (K == U_POW) return powf(v, p);
    if (K == U_GELU) return gelu_tanh(v);
    if (K == U_RSQRT) return 1.0f / sqrtf(v);
    if (K == U_SILU) return silu(v);
    if (K == U_NEG) return -v;
    if (K == U_COS) return cosf(v);
    return sinf(v);
}

enum BinKind { B_ADD = 0, B_SUB = 1, B_MUL = 2, B_DIV = 3, B_ADD_RELU = 4 };

template <int K>
__device__ __forceinline__ float bin_op(float a, float b) {
    if (K == B_ADD) return a + b;
    if (K == B_SUB) return a - b;
    if (K == B_MUL) return a * b;
    if (K == B_DIV) return a / b;
    float v = a + b;
    return v > 0.0f ? v : 0.0f;
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

// ---- fp16 split (the default GEMM operand form) -----------------------------
// An operand row x is scaled by a power of two 2^e so that its largest
// magnitude lies in [2^14, 2^15) (exact: only the exponent changes), then
// written as h = fp16(x 2^e) and l = fp16(x 2^e - h): |x 2^e - h - l| <=
// 2^-22 |x 2^e|, and the MMA products h.h, h.l, l.h are exact in fp32.  The
// GEMM multiplies its result by 2^-e (per A row, per B tensor).  Elements far
// below the row maximum lose relative precision once h or l turns subnormal,
// but never more than ~2^-39 of the row maximum in absolute terms.
//
// e for a maximum magnitude m (0 when m is 0, subnormal-small or not finite).
__device__ __forceinline__ int f16_scale_exp(float m) {
    const uint32_t eb = (__float_as_uint(m) >> 23) & 0xffu;
    if (!(m > 0.0f) || eb == 0xffu) return 0;
    const int e = 141 - (int)eb;                 // m in [2^(eb-127), 2^(eb-126)) -> [2^14, 2^15)
    return e < -120 ? -120 : (e > 120 ? 120 : e);
}
__device__ __forceinline__ float pow2i(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }
// h = x rounded to 11 significant bits (ties away) by integer arithmetic on
// its bits -- the fp16 value of x for |x| in the fp16 normal range -- and
// l = x - h, exact.  The conversion instructions then only pack: one
// cvt.rn.f16x2 per two values (exact for h; l keeps 11 bits of the residual).
__device__ __forceinline__ float round11(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ uint32_t f16x2_rn(float lo, float hi) {   // lo in the low half
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
// Four consecutive elements k..k+3 (k % 4 == 0, already scaled) of a row into
// its fp16 plane: per 16-wide K block 32 halves, [h(16) | l(16)] when
// first_hi (A operands), [l(16) | h(16)] otherwise (B operands).
__device__ __forceinline__ void store_f16x4(uint16_t* row, int64_t k, float4 v, bool first_hi) {
    const float h0 = round11(v.x), h1 = round11(v.y), h2 = round11(v.z), h3 = round11(v.w);
    const uint2 hh = make_uint2(f16x2_rn(h0, h1), f16x2_rn(h2, h3));
    const uint2 ll = make_uint2(f16x2_rn(v.x - h0, v.y - h1), f16x2_rn(v.z - h2, v.w - h3));
    uint16_t* blk = row + (k >> 4) * 32 + (k & 15);
    *reinterpret_cast<uint2*>(blk + (first_hi ? 0 : 16)) = hh;
    *reinterpret_cast<uint2*>(blk + (first_hi ? 16 : 0)) = ll;
}
// One element: its h and l halves (h in the low 16 bits of the result).
__device__ __forceinline__ uint32_t f16_hl(float x) {
    const float h = round11(x);
    return f16x2_rn(h, x - h);
}

// Blackwell's three-input maximum and paired fp32 arithmetic (one
// instruction for two values), for loops bounded by their instruction count
// (the attention softmax, the GEMM epilogue's chunk sums).
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(unsigned long long r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

}  // namespace rt
