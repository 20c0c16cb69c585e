// k_elementwise.cu -- element-wise kernels: unary ops, binary ops in every
// mode of the reference dispatch, fused bias+ReLU and the gated activations.
//
// Reference semantics:
//   unary   csrc/executor.c:57-81, csrc/ops/elementwise.c (relu :23, exp :63,
//           pow :139, tanh :150, gelu_tanh :167-191, rsqrt :196, silu :203,
//           neg :210, cos/sin :217-226)
//   ADD     csrc/executor.c:96-117  modes 0 bias / 1 same-shape / 2 scalar / 3 broadcast
//   SUB/MUL/DIV csrc/executor.c:119-168  modes 0 same / 1 scalar / 2 broadcast
//   broadcast csrc/ops/shape.c:32-62 (per-dimension strides, 0 = broadcast)
//   FUSED_BIAS_RELU csrc/ops/elementwise.c:81-90
//   GATED_ACT csrc/executor.c:354-369, csrc/ops/elementwise.c:96-136
//
// All are HBM-bound: one read per input element, one write per output
// element, 16-byte vector accesses when every pointer is 16-byte aligned and
// the element count is a multiple of 4, grid-stride loops over a grid sized
// in multiples of the SM count.  The arithmetic is the reference's, in fp32,
// using CUDA's IEEE-accurate library functions (no fast-math intrinsics).
#include "rt_internal.h"

#include "dev_math.h"

namespace rt {
namespace {

template <int K>
__global__ void unary_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n, float p,
                             bool vec) {
    int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {
        int64_t n4 = n >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        float4* y4 = reinterpret_cast<float4*>(y);
        for (int64_t i = tid; i < n4; i += stride) {
            float4 v = x4[i];
            v.x = unary_op<K>(v.x, p);
            v.y = unary_op<K>(v.y, p);
            v.z = unary_op<K>(v.z, p);
            v.w = unary_op<K>(v.w, p);
            y4[i] = v;
        }
    } else {
        for (int64_t i = tid; i < n; i += stride) y[i] = unary_op<K>(x[i], p);
    }
}

template <int K>
__device__ __forceinline__ float4 bin_op4(float4 a, float4 b) {
    return make_float4(bin_op<K>(a.x, b.x), bin_op<K>(a.y, b.y), bin_op<K>(a.z, b.z),
                       bin_op<K>(a.w, b.w));
}

// b indexed as b[i % period] (period = n: same shape; period = N: bias row;
// period = 0: scalar `s`).
template <int K>
__global__ void binary_kernel(const float* __restrict__ a, const float* __restrict__ b, float s,
                              float* __restrict__ y, int64_t n, int64_t period, bool vec) {
    int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {
        int64_t n4 = n >> 2;
        const float4* a4 = reinterpret_cast<const float4*>(a);
        float4* y4 = reinterpret_cast<float4*>(y);
        for (int64_t i = tid; i < n4; i += stride) {
            float4 bv;
            if (period == 0) {
                bv = make_float4(s, s, s, s);
            } else {
                int64_t j = (i << 2) % period;   // period % 4 == 0 on this path
                bv = *reinterpret_cast<const float4*>(b + j);
            }
            y4[i] = bin_op4<K>(a4[i], bv);
        }
    } else {
        for (int64_t i = tid; i < n; i += stride) {
            float bv = period == 0 ? s : b[i % period];
            y[i] = bin_op<K>(a[i], bv);
        }
    }
}

struct BcastParams {
    int ndim;
    int shape[8];
    int as[8];
    int bs[8];
};

// General broadcast (csrc/ops/shape.c:32-62).  When the innermost dimension
// is contiguous for a, b (stride 1 or 0) and a multiple of 4 long, each
// thread handles 4 consecutive outputs with one coordinate decode.
template <int K>
__global__ void broadcast_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                 float* __restrict__ y, int64_t n, BcastParams p, bool vec) {
    int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int w = vec ? 4 : 1;
    int64_t groups = n / w;
    for (int64_t g = tid; g < groups; g += stride) {
        int64_t idx = g * w;
        int64_t rem = idx, ao = 0, bo = 0;
#pragma unroll
        for (int d = 7; d >= 0; d--) {
            if (d < p.ndim) {
                int64_t c = rem % p.shape[d];
                rem /= p.shape[d];
                ao += c * p.as[d];
                bo += c * p.bs[d];
            }
        }
        if (vec) {
            int last = p.ndim - 1;
            float4 av = p.as[last] ? *reinterpret_cast<const float4*>(a + ao)
                                   : make_float4(a[ao], a[ao], a[ao], a[ao]);
            float4 bv = p.bs[last] ? *reinterpret_cast<const float4*>(b + bo)
                                   : make_float4(b[bo], b[bo], b[bo], b[bo]);
            *reinterpret_cast<float4*>(y + idx) = bin_op4<K>(av, bv);
        } else {
            y[idx] = bin_op<K>(a[ao], b[bo]);
        }
    }
}

// GATED_ACT: y = act(x + bias?) * up ; act 0 = SiLU, 1 = tanh-GELU.
template <int ACT>
__global__ void gated_kernel(const float* __restrict__ x, const float* __restrict__ up,
                             const float* __restrict__ bias, float* __restrict__ y, int64_t n,
                             int64_t N, bool vec) {
    int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {
        int64_t n4 = n >> 2;
        for (int64_t i = tid; i < n4; i += stride) {
            float4 v = reinterpret_cast<const float4*>(x)[i];
            float4 u = reinterpret_cast<const float4*>(up)[i];
            if (bias) {
                float4 bb = *reinterpret_cast<const float4*>(bias + ((i << 2) % N));
                v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
            }
            float4 o;
            o.x = (ACT == 0 ? silu(v.x) : gelu_tanh(v.x)) * u.x;
            o.y = (ACT == 0 ? silu(v.y) : gelu_tanh(v.y)) * u.y;
            o.z = (ACT == 0 ? silu(v.z) : gelu_tanh(v.z)) * u.z;
            o.w = (ACT == 0 ? silu(v.w) : gelu_tanh(v.w)) * u.w;
            reinterpret_cast<float4*>(y)[i] = o;
        }
    } else {
        for (int64_t i = tid; i < n; i += stride) {
            float v = x[i] + (bias ? bias[i % N] : 0.0f);
            y[i] = (ACT == 0 ? silu(v) : gelu_tanh(v)) * up[i];
        }
    }
}

constexpr int kThreads = 256;

template <int K>
Status run_unary(const float* x, float* y, int64_t n, float p, cudaStream_t st) {
    bool vec = aligned16(x) && aligned16(y) && (n % 4 == 0);
    int grid = grid_for(vec ? n / 4 : n, kThreads);
    unary_kernel<K><<<grid, kThreads, 0, st>>>(x, y, n, p, vec);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

template <int K>
Status run_binary(const float* a, const float* b, float s, float* y, int64_t n, int64_t period,
                  cudaStream_t st) {
    bool vec = aligned16(a) && aligned16(y) && (n % 4 == 0) &&
               (period == 0 || (aligned16(b) && period % 4 == 0));
    int grid = grid_for(vec ? n / 4 : n, kThreads);
    binary_kernel<K><<<grid, kThreads, 0, st>>>(a, b, s, y, n, period, vec);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

template <int K>
Status run_broadcast(const OpNode& nd, int base, cudaStream_t st) {
    int ndim = nd.extra[base];
    if (ndim < 1 || ndim > 7 || base + 1 + 3 * ndim > RT_MAX_DIMS)
        return Status::err(RT_ERR_BAD_NODE, "broadcast: bad ndim in extras");
    BcastParams p{};
    p.ndim = ndim;
    int64_t n = 1;
    for (int d = 0; d < ndim; d++) {
        p.as[d] = nd.extra[base + 1 + d];
        p.bs[d] = nd.extra[base + 1 + ndim + d];
        p.shape[d] = nd.extra[base + 1 + 2 * ndim + d];
        if (p.shape[d] <= 0) return Status::err(RT_ERR_BAD_NODE, "broadcast: bad shape");
        n *= p.shape[d];
    }
    const float* a = (const float*)nd.inputs[0];
    const float* b = (const float*)nd.inputs[1];
    float* y = (float*)nd.output;
    int last = ndim - 1;
    // a vector group of 4 must stay inside one innermost row and step both
    // operands by 1 (or 0) element
    bool vec = p.shape[last] % 4 == 0 && (p.as[last] == 1 || p.as[last] == 0) &&
               (p.bs[last] == 1 || p.bs[last] == 0) && aligned16(y);
    if (vec) {
        // every group start must be 16-byte aligned in the strided operands
        for (int d = 0; d < ndim && vec; d++) {
            if (p.as[last] == 1 && (int64_t)p.as[d] % 4 != 0 && d != last) vec = false;
            if (p.bs[last] == 1 && (int64_t)p.bs[d] % 4 != 0 && d != last) vec = false;
        }
        if (p.as[last] == 1 && !aligned16(a)) vec = false;
        if (p.bs[last] == 1 && !aligned16(b)) vec = false;
    }
    int grid = grid_for(vec ? n / 4 : n, kThreads);
    broadcast_kernel<K><<<grid, kThreads, 0, st>>>(a, b, y, n, p, vec);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

template <int K>
Status run_binop_node(const OpNode& nd, int mode_same, int mode_scalar, int mode_bcast,
                      cudaStream_t st) {
    int mode = nd.extra[0];
    int64_t n = total_elements(nd);
    const float* a = (const float*)nd.inputs[0];
    float* y = (float*)nd.output;
    if (mode == mode_scalar) return run_binary<K>(a, nullptr, extra_float(nd, 1), y, n, 0, st);
    if (mode == mode_same) return run_binary<K>(a, (const float*)nd.inputs[1], 0.f, y, n, n, st);
    if (mode == mode_bcast) return run_broadcast<K>(nd, 1, st);
    return Status::err(RT_ERR_BAD_NODE, "binary op: unknown mode");
}

}  // namespace

Status launch_elementwise(const OpNode& nd, cudaStream_t st, int* launches) {
    *launches += 1;
    const float* x = (const float*)nd.inputs[0];
    float* y = (float*)nd.output;
    int64_t n = total_elements(nd);
    switch (nd.op) {
        case RT_OP_RELU: return run_unary<U_RELU>(x, y, n, 0.f, st);
        case RT_OP_EXP: return run_unary<U_EXP>(x, y, n, 0.f, st);
        case RT_OP_TANH: return run_unary<U_TANH>(x, y, n, 0.f, st);
        case RT_OP_POW: return run_unary<U_POW>(x, y, n, extra_float(nd, 0), st);
        case RT_OP_GELU: return run_unary<U_GELU>(x, y, n, 0.f, st);
        case RT_OP_RSQRT: return run_unary<U_RSQRT>(x, y, n, 0.f, st);
        case RT_OP_SILU: return run_unary<U_SILU>(x, y, n, 0.f, st);
        case RT_OP_NEG: return run_unary<U_NEG>(x, y, n, 0.f, st);
        case RT_OP_COS: return run_unary<U_COS>(x, y, n, 0.f, st);
        case RT_OP_SIN: return run_unary<U_SIN>(x, y, n, 0.f, st);
        case RT_OP_ADD: {
            int mode = nd.extra[0];
            if (mode == 0)  // bias broadcast along the last dim (executor.c:110-114)
                return run_binary<B_ADD>(x, (const float*)nd.inputs[1], 0.f, y, n, last_dim(nd), st);
            if (mode == 1) return run_binary<B_ADD>(x, (const float*)nd.inputs[1], 0.f, y, n, n, st);
            if (mode == 2) return run_binary<B_ADD>(x, nullptr, extra_float(nd, 1), y, n, 0, st);
            if (mode == 3) return run_broadcast<B_ADD>(nd, 1, st);
            return Status::err(RT_ERR_BAD_NODE, "ADD: unknown mode");
        }
        case RT_OP_SUB: return run_binop_node<B_SUB>(nd, 0, 1, 2, st);
        case RT_OP_MUL: return run_binop_node<B_MUL>(nd, 0, 1, 2, st);
        case RT_OP_DIV: return run_binop_node<B_DIV>(nd, 0, 1, 2, st);
        case RT_OP_FUSED_BIAS_RELU:
            return run_binary<B_ADD_RELU>(x, (const float*)nd.inputs[1], 0.f, y, n, last_dim(nd), st);
        case RT_OP_GATED_ACT: {
            int has_bias = nd.extra[0], act = nd.extra[1];
            const float* up = (const float*)(has_bias ? nd.inputs[2] : nd.inputs[1]);
            const float* bias = has_bias ? (const float*)nd.inputs[1] : nullptr;
            int64_t N = last_dim(nd);
            bool vec = aligned16(x) && aligned16(up) && aligned16(y) && n % 4 == 0 &&
                       (!bias || (aligned16(bias) && N % 4 == 0));
            int grid = grid_for(vec ? n / 4 : n, kThreads);
            if (act == 0)
                gated_kernel<0><<<grid, kThreads, 0, st>>>(x, up, bias, y, n, N, vec);
            else
                gated_kernel<1><<<grid, kThreads, 0, st>>>(x, up, bias, y, n, N, vec);
            RT_LAUNCH_CHECK();
            return Status::ok();
        }
        default:
            return Status::err(RT_ERR_BAD_OP, "elementwise: unexpected op");
    }
}

namespace {

// gated activation with row-strided inputs (see GatedViews); 4 columns per
// thread when every row start is 16-byte aligned.
template <int ACT>
__global__ void gated_views_kernel(GatedViews v, const float* __restrict__ bias, float* __restrict__ y,
                                   int64_t rows, int64_t N, bool vec) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {
        const int64_t per_row = N >> 2, total = rows * per_row;
        for (int64_t i = tid; i < total; i += stride) {
            const int64_t r = i / per_row, c = (i - r * per_row) << 2;
            float4 a = *reinterpret_cast<const float4*>(v.x + r * v.x_ld + c);
            const float4 u = *reinterpret_cast<const float4*>(v.up + r * v.up_ld + c);
            if (bias) {
                const float4 bb = *reinterpret_cast<const float4*>(bias + c);
                a.x += bb.x; a.y += bb.y; a.z += bb.z; a.w += bb.w;
            }
            float4 o;
            o.x = (ACT == 0 ? silu(a.x) : gelu_tanh(a.x)) * u.x;
            o.y = (ACT == 0 ? silu(a.y) : gelu_tanh(a.y)) * u.y;
            o.z = (ACT == 0 ? silu(a.z) : gelu_tanh(a.z)) * u.z;
            o.w = (ACT == 0 ? silu(a.w) : gelu_tanh(a.w)) * u.w;
            *reinterpret_cast<float4*>(y + r * N + c) = o;
        }
    } else {
        for (int64_t i = tid; i < rows * N; i += stride) {
            const int64_t r = i / N, c = i - r * N;
            const float a = v.x[r * v.x_ld + c] + (bias ? bias[c] : 0.0f);
            y[i] = (ACT == 0 ? silu(a) : gelu_tanh(a)) * v.up[r * v.up_ld + c];
        }
    }
}

}  // namespace

Status launch_gated_views(const OpNode& nd, const GatedViews& v, cudaStream_t st, int* launches) {
    const int has_bias = nd.extra[0], act = nd.extra[1];
    const float* bias = has_bias ? (const float*)nd.inputs[1] : nullptr;
    float* y = (float*)nd.output;
    const int64_t N = last_dim(nd), rows = N ? total_elements(nd) / N : 0;
    const bool vec = N % 4 == 0 && v.x_ld % 4 == 0 && v.up_ld % 4 == 0 && aligned16(v.x) && aligned16(v.up) &&
                     aligned16(y) && (!bias || aligned16(bias));
    const int grid = grid_for(vec ? rows * N / 4 : rows * N, kThreads);
    if (act == 0) gated_views_kernel<0><<<grid, kThreads, 0, st>>>(v, bias, y, rows, N, vec);
    else gated_views_kernel<1><<<grid, kThreads, 0, st>>>(v, bias, y, rows, N, vec);
    RT_LAUNCH_CHECK();
    *launches += 1;
    return Status::ok();
}

}  // namespace rt
