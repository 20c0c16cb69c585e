// dev_math.h -- device math shared by kernels that must agree bit for bit
// (an activation applied in a GEMM epilogue and in the stand-alone kernel).
#pragma once

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

}  // namespace rt
