// k_norm.cu -- row-wise normalisations and reductions.
//
// Reference semantics:
//   LAYERNORM csrc/ops/norm.c:48-63 (non-Apple): mean, centred variance,
//             (x-mean) * (1/sqrt(var/C + eps)) * gamma + beta; eps = extra[0] bits
//             (csrc/executor.c:296-301)
//   RMSNORM   csrc/ops/norm.c:100-107: x * (1/sqrt(sum(x^2)/C + eps)) * w
//   SOFTMAX   csrc/ops/reduce.c:84-96: exp(x - max) / sum, along the last dim
//   MAX/SUM   csrc/ops/reduce.c:8-36 over [outer, axis, inner], extras [axis, axis_size]
//             (csrc/executor.c:172-190)
//
// A row is read from HBM once and kept in registers: one warp per row when
// the row fits 32 lanes x VPT floats, one 256-thread CTA per row up to 4096
// floats, and a three-pass loop beyond that.  Reductions are warp shuffles
// (+ shared memory across warps); everything accumulates in fp32.
#include "dev_math.h"
#include "rt_internal.h"

namespace rt {
namespace {

enum NormKind { N_LAYER = 0, N_RMS = 1, N_SOFTMAX = 2 };

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Reduction across the threads of a CTA (THREADS/32 warps); all threads get it.
template <int THREADS, bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* sh) {
    v = MAX ? warp_max(v) : warp_sum(v);
    if (THREADS == 32) return v;
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();  // sh may still be read from a previous reduction
    if (l == 0) sh[w] = v;
    __syncthreads();
    float r = l < THREADS / 32 ? sh[l] : (MAX ? -INFINITY : 0.0f);
    return MAX ? warp_max(r) : warp_sum(r);
}

// Two sums and one maximum across the threads of a group (a warp or the
// CTA) in one round: one barrier pair instead of one per quantity.  All
// threads get the results.  sh holds 24 floats.
template <int THREADS>
__device__ __forceinline__ void group_reduce_ssm(float& s, float& q, float& m, float* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        q += __shfl_xor_sync(0xffffffffu, q, o);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    if constexpr (THREADS != 32) {
    static_assert(THREADS == 256, "whole-CTA rows are 256 threads");
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();  // sh may still be read from the previous row
    if (l == 0) {
        sh[w] = s;
        sh[8 + w] = q;
        sh[16 + w] = m;
    }
    __syncthreads();
    const float4* s4 = reinterpret_cast<const float4*>(sh);
    const float4 a0 = s4[0], a1 = s4[1], b0 = s4[2], b1 = s4[3], c0 = s4[4], c1 = s4[5];
    s = ((a0.x + a0.y) + (a0.z + a0.w)) + ((a1.x + a1.y) + (a1.z + a1.w));
    q = ((b0.x + b0.y) + (b0.z + b0.w)) + ((b1.x + b1.y) + (b1.z + b1.w));
    m = fmaxf(fmaxf(fmaxf(c0.x, c0.y), fmaxf(c0.z, c0.w)), fmaxf(fmaxf(c1.x, c1.y), fmaxf(c1.z, c1.w)));
    }
}

// One row per group of THREADS threads (a warp or the whole CTA); each
// thread holds VPT floats of the row: elements (v*THREADS + t)*4 .. +3 when
// VEC (C % 4 == 0; x, y, gamma, beta 16-byte aligned), else elements v*THREADS + t.
// PLANES: the row is a GEMM's A operand; write its split planes (hi to y,
// plane 1 to `x1`, mode `cross`) instead of the fp32 row -- or, with F16P,
// its fp16 plane to y (2*C halves per row, C % 16 == 0) and its 2^-e scale
// to ((float*)x1)[row], from the maximum of the normalised row.
template <int KIND, int THREADS, int VPT, bool VEC, bool PLANES = false, bool F16P = false>
__global__ void __launch_bounds__(256, THREADS == 256 ? (VPT <= 8 ? 5 : 1) : (VPT <= 24 ? 3 : VPT <= 32 ? 2 : 1)) row_kernel(const float* __restrict__ x,
                                                  const float* __restrict__ g,
                                                  const float* __restrict__ b,
                                                  float* __restrict__ y, int64_t rows, int C,
                                                  float eps, uint16_t* __restrict__ x1 = nullptr,
                                                  bool cross = true) {
    __shared__ __align__(16) float sh[32];
    constexpr int GROUPS = 256 / THREADS;  // rows handled by one CTA at a time
    // Whole-CTA rows (few values per thread) load the CTA's next row while
    // this one is reduced and stored: a row in flight per CTA at all times.
    constexpr bool PF = THREADS == 256 && VPT <= 16;
    int group = threadIdx.x / THREADS;
    int t = threadIdx.x % THREADS;
    auto load = [&](int64_t rw, float (&a)[VPT]) {
        const float* xr = x + rw * C;
        if (VEC) {
#pragma unroll
            for (int i = 0; i < VPT / 4; i++) {
                int c = (i * THREADS + t) * 4;
                float4 q = c < C ? *reinterpret_cast<const float4*>(xr + c)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
                a[4 * i] = q.x; a[4 * i + 1] = q.y; a[4 * i + 2] = q.z; a[4 * i + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < VPT; i++) {
                int c = i * THREADS + t;
                a[i] = c < C ? xr[c] : 0.0f;
            }
        }
    };
    // Whole-CTA F16P rows take their fp16 scale from a bound instead of a
    // further reduction: |y| <= scale * (max|x| + |mean|) * max|gamma| +
    // max|beta|; the gamma / beta maxima over the row once per CTA.
    // Whole-CTA rows: one reduction round per row (two sums and a maximum).
    // Warp rows keep the sequential warp reductions, which need fewer
    // registers (occupancy decides the warp form's speed).
    constexpr bool STATS1 = VEC && THREADS == 256 && (KIND == N_LAYER || KIND == N_RMS);
    constexpr bool ONE_PASS = STATS1 && PLANES && F16P;
    float gmax = 0.0f, bmax = 0.0f;
    if constexpr (ONE_PASS) {
#pragma unroll
        for (int i = 0; i < VPT / 4; i++) {
            const int c = (i * THREADS + t) * 4;
            if (c < C) {
                const float4 g4 = *reinterpret_cast<const float4*>(g + c);
                gmax = fmaxf(gmax, fmaxf(fmaxf(fabsf(g4.x), fabsf(g4.y)), fmaxf(fabsf(g4.z), fabsf(g4.w))));
                if (KIND == N_LAYER) {
                    const float4 b4 = *reinterpret_cast<const float4*>(b + c);
                    bmax = fmaxf(bmax, fmaxf(fmaxf(fabsf(b4.x), fabsf(b4.y)), fmaxf(fabsf(b4.z), fabsf(b4.w))));
                }
            }
        }
        float unused = 0.0f;
        group_reduce_ssm<THREADS>(unused, unused, gmax, sh);
        if (KIND == N_LAYER) group_reduce_ssm<THREADS>(unused, unused, bmax, sh);
    }
    const int64_t row0 = (int64_t)blockIdx.x * GROUPS + group, stride = (int64_t)gridDim.x * GROUPS;
    float nxt[PF ? VPT : 1];
    if constexpr (PF) {
        if (row0 < rows) load(row0, *reinterpret_cast<float(*)[VPT]>(nxt));
    }
    for (int64_t row = row0; row < rows; row += stride) {
        float* yr = y + row * C;
        float v[VPT];
        if constexpr (PF) {
#pragma unroll
            for (int i = 0; i < VPT; i++) v[i] = nxt[i];
            if (row + stride < rows) load(row + stride, *reinterpret_cast<float(*)[VPT]>(nxt));
        } else {
            load(row, v);
        }
        auto col = [&](int i) -> int {
            return VEC ? ((i / 4) * THREADS + t) * 4 + (i % 4) : i * THREADS + t;
        };
        float scale = 1.0f, shift = 0.0f;
        float bound = 0.0f;   // F16P: an upper bound of the normalised row's magnitudes
        if (STATS1 && KIND == N_LAYER) {
            // One reduction round: sums of d = x - x[0] and d^2 (shifted sums:
            // no cancellation unless the mean is far from x[0] relative to the
            // spread), and max |x| for the plane's scale bound.
            const float k0 = __ldg(x + row * C);
            float s = 0.0f, q = 0.0f, xm = 0.0f;
#pragma unroll
            for (int i = 0; i < VPT; i++) {
                const float d = col(i) < C ? v[i] - k0 : 0.0f;
                s += d;
                q = fmaf(d, d, q);
                xm = fmaxf(xm, fabsf(v[i]));   // padding lanes hold 0
            }
            group_reduce_ssm<THREADS>(s, q, xm, sh);
            const float mean = k0 + s / C;
            const float var = fmaxf(q - s * (s / C), 0.0f);
            scale = 1.0f / sqrtf(var / C + eps);
#pragma unroll
            for (int i = 0; i < VPT; i++) v[i] = col(i) < C ? v[i] - mean : 0.0f;
            bound = fmaf(scale * (xm + fabsf(mean)), gmax, bmax);
        } else if (STATS1 && KIND == N_RMS) {
            float q = 0.0f, xm = 0.0f, unused = 0.0f;
#pragma unroll
            for (int i = 0; i < VPT; i++) {
                q = fmaf(v[i], v[i], q);
                xm = fmaxf(xm, fabsf(v[i]));
            }
            group_reduce_ssm<THREADS>(q, unused, xm, sh);
            scale = 1.0f / sqrtf(q / C + eps);
            bound = scale * xm * gmax;
        } else if (KIND == N_LAYER) {
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < VPT; i++) s += v[i];
            float mean = block_reduce<THREADS, false>(s, sh) / C;
            float q = 0.0f;
#pragma unroll
            for (int i = 0; i < VPT; i++) {
                float d = col(i) < C ? v[i] - mean : 0.0f;
                v[i] = d;
                q += d * d;
            }
            float var = block_reduce<THREADS, false>(q, sh);
            scale = 1.0f / sqrtf(var / C + eps);
        } else if (KIND == N_RMS) {
            float q = 0.0f;
#pragma unroll
            for (int i = 0; i < VPT; i++) q += v[i] * v[i];
            float ss = block_reduce<THREADS, false>(q, sh);
            scale = 1.0f / sqrtf(ss / C + eps);
        } else {
            float m = -INFINITY;
#pragma unroll
            for (int i = 0; i < VPT; i++)
                if (col(i) < C) m = fmaxf(m, v[i]);
            m = block_reduce<THREADS, true>(m, sh);
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < VPT; i++) {
                v[i] = col(i) < C ? expf(v[i] - m) : 0.0f;
                s += v[i];
            }
            s = block_reduce<THREADS, false>(s, sh);
            scale = s;  // divided below, as the reference does (reduce.c:95)
            shift = 0.0f;
        }
        if (VEC && PLANES && F16P) {
            float m = 0.0f;
#pragma unroll
            for (int i = 0; i < VPT / 4; i++) {
                const int c = (i * THREADS + t) * 4;
                if (c < C) {   // gamma / beta as 16-byte vectors (aligned on this path)
                    const float4 g4 = *reinterpret_cast<const float4*>(g + c);
                    const float4 b4 = KIND == N_LAYER ? *reinterpret_cast<const float4*>(b + c)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                    const float gg[4] = {g4.x, g4.y, g4.z, g4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        float val = v[4 * i + k] * scale * gg[k];
                        if (KIND == N_LAYER) val += bv[k];
                        v[4 * i + k] = val;
                        if (!ONE_PASS) m = fmaxf(m, fabsf(val));
                    }
                }
            }
            if (!ONE_PASS) m = block_reduce<THREADS, true>(m, sh);
            const int e = f16_scale_exp(ONE_PASS ? bound : m);
            const float sc = pow2i(e);
            if (t == 0) reinterpret_cast<float*>(x1)[row] = pow2i(-e);
            uint16_t* pr = reinterpret_cast<uint16_t*>(y) + row * C * 2;
#pragma unroll
            for (int i = 0; i < VPT / 4; i++) {
                const int c = (i * THREADS + t) * 4;
                if (c < C)
                    store_f16x4(pr, c, make_float4(v[4 * i] * sc, v[4 * i + 1] * sc, v[4 * i + 2] * sc,
                                                   v[4 * i + 3] * sc), true);
            }
        } else if (VEC) {
#pragma unroll
            for (int i = 0; i < VPT / 4; i++) {
                int c = (i * THREADS + t) * 4;
                if (c < C) {
                    float4 o;
                    float* op = &o.x;
                    float4 g4 = make_float4(0.f, 0.f, 0.f, 0.f), b4 = g4;
                    if (KIND != N_SOFTMAX) g4 = *reinterpret_cast<const float4*>(g + c);   // aligned on this path
                    if (KIND == N_LAYER) b4 = *reinterpret_cast<const float4*>(b + c);
                    const float gg[4] = {g4.x, g4.y, g4.z, g4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        float val = v[4 * i + k];
                        if (KIND == N_LAYER) val = val * scale * gg[k] + bv[k];
                        else if (KIND == N_RMS) val = val * scale * gg[k];
                        else val = val / scale;
                        op[k] = val + shift;
                    }
                    if (PLANES) store_split4(yr, x1 + row * C * 2, c, C, o, cross);
                    else *reinterpret_cast<float4*>(yr + c) = o;
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < VPT; i++) {
                int c = i * THREADS + t;
                if (c < C) {
                    float val = v[i];
                    if (KIND == N_LAYER) val = val * scale * g[c] + b[c];
                    else if (KIND == N_RMS) val = val * scale * g[c];
                    else val = val / scale;
                    yr[c] = val;
                }
            }
        }
    }
}

// Rows longer than the register budget: one CTA per row, three passes over HBM.
template <int KIND>
__global__ void __launch_bounds__(256) row_loop_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ g,
                                                       const float* __restrict__ b,
                                                       float* __restrict__ y, int64_t rows,
                                                       int C, float eps) {
    __shared__ float sh[32];
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float* xr = x + row * C;
        float* yr = y + row * C;
        float a = 0.0f, scale = 1.0f;
        if (KIND == N_LAYER) {
            for (int c = threadIdx.x; c < C; c += 256) a += xr[c];
            float mean = block_reduce<256, false>(a, sh) / C;
            float q = 0.0f;
            for (int c = threadIdx.x; c < C; c += 256) {
                float d = xr[c] - mean;
                q += d * d;
            }
            scale = 1.0f / sqrtf(block_reduce<256, false>(q, sh) / C + eps);
            for (int c = threadIdx.x; c < C; c += 256) yr[c] = (xr[c] - mean) * scale * g[c] + b[c];
        } else if (KIND == N_RMS) {
            for (int c = threadIdx.x; c < C; c += 256) a += xr[c] * xr[c];
            scale = 1.0f / sqrtf(block_reduce<256, false>(a, sh) / C + eps);
            for (int c = threadIdx.x; c < C; c += 256) yr[c] = xr[c] * scale * g[c];
        } else {
            float m = -INFINITY;
            for (int c = threadIdx.x; c < C; c += 256) m = fmaxf(m, xr[c]);
            m = block_reduce<256, true>(m, sh);
            for (int c = threadIdx.x; c < C; c += 256) a += expf(xr[c] - m);
            float s = block_reduce<256, false>(a, sh);
            for (int c = threadIdx.x; c < C; c += 256) yr[c] = expf(xr[c] - m) / s;
        }
    }
}

template <int KIND, int THREADS, int VPT, bool VEC, bool PLANES = false, bool F16P = false>
void launch_rows(const float* x, const float* g, const float* b, float* y, int64_t rows, int C,
                 float eps, cudaStream_t st, uint16_t* x1 = nullptr, bool cross = true) {
    constexpr int GROUPS = 256 / THREADS;
    int64_t blocks = (rows + GROUPS - 1) / GROUPS;
    int64_t cap = (int64_t)g_num_sms * (THREADS == 32 ? 8 : 4) * 4;
    int grid = (int)(blocks < cap ? blocks : cap);
    row_kernel<KIND, THREADS, VPT, VEC, PLANES, F16P><<<grid, 256, 0, st>>>(x, g, b, y, rows, C, eps, x1, cross);
}

// Rows of 1024 < C <= 2048 run on a whole 256-thread CTA (8 values per
// thread, the next row prefetched); shorter rows on one warp.  RT_NORM_CTA=1
// extends the CTA form down to C > 512, RT_NORM_CTA=0 turns it off.
int norm_cta_min() {
    static const int c = [] {
        const char* e = getenv("RT_NORM_CTA");
        return e && e[0] == '1' ? 512 : e && e[0] == '0' ? 1 << 30 : 1024;
    }();
    return c;
}

template <int KIND, bool F16P>
void run_rows_planes_t(const float* x, const float* g, const float* b, float* hi, uint16_t* x1, int64_t rows,
                       int C, float eps, bool cross, cudaStream_t st) {
    if (C > norm_cta_min() && C <= 2048) {
        if (C <= 1024) launch_rows<KIND, 256, 4, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
        else launch_rows<KIND, 256, 8, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
        return;
    }
    if (C <= 128) launch_rows<KIND, 32, 4, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
    else if (C <= 256) launch_rows<KIND, 32, 8, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
    else if (C <= 512) launch_rows<KIND, 32, 16, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
    else if (C <= 768) launch_rows<KIND, 32, 24, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
    else if (C <= 1024) launch_rows<KIND, 32, 32, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
    else if (C <= 2048) launch_rows<KIND, 32, 64, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
    else launch_rows<KIND, 256, 16, true, true, F16P>(x, g, b, hi, rows, C, eps, st, x1, cross);
}
template <int KIND>
void run_rows_planes(const float* x, const float* g, const float* b, float* hi, uint16_t* x1, int64_t rows,
                     int C, float eps, int scheme, cudaStream_t st) {
    if (scheme == 2) run_rows_planes_t<KIND, true>(x, g, b, hi, x1, rows, C, eps, false, st);
    else run_rows_planes_t<KIND, false>(x, g, b, hi, x1, rows, C, eps, scheme == 1, st);
}

template <int KIND>
Status run_rows(const float* x, const float* g, const float* b, float* y, int64_t rows, int C,
                float eps, cudaStream_t st) {
    if (rows == 0 || C == 0) return Status::ok();
    bool vec = C % 4 == 0 && aligned16(x) && aligned16(y) && (!g || aligned16(g)) && (!b || aligned16(b));
    if (vec) {
        if (C <= 128) launch_rows<KIND, 32, 4, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 256) launch_rows<KIND, 32, 8, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 512) launch_rows<KIND, 32, 16, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 1024 && C > norm_cta_min()) launch_rows<KIND, 256, 4, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 2048 && C > norm_cta_min()) launch_rows<KIND, 256, 8, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 768) launch_rows<KIND, 32, 24, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 1024) launch_rows<KIND, 32, 32, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 2048) launch_rows<KIND, 32, 64, true>(x, g, b, y, rows, C, eps, st);
        else if (C <= 4096) launch_rows<KIND, 256, 16, true>(x, g, b, y, rows, C, eps, st);
        else vec = false;
    }
    if (!vec) {
        if (C <= 128) launch_rows<KIND, 32, 4, false>(x, g, b, y, rows, C, eps, st);
        else if (C <= 512) launch_rows<KIND, 32, 16, false>(x, g, b, y, rows, C, eps, st);
        else {
            int grid = (int)(rows < (int64_t)g_num_sms * 8 ? rows : (int64_t)g_num_sms * 8);
            row_loop_kernel<KIND><<<grid, 256, 0, st>>>(x, g, b, y, rows, C, eps);
        }
    }
    RT_LAUNCH_CHECK();
    return Status::ok();
}

template <bool MAX>
__global__ void reduce_axis_kernel(const float* __restrict__ x, float* __restrict__ y,
                                   int64_t outer, int64_t axis, int64_t inner) {
    int64_t n = outer * inner;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = i / inner, j = i % inner;
        const float* p = x + o * axis * inner + j;
        float acc = MAX ? -3.402823466e+38f : 0.0f;
        for (int64_t a = 0; a < axis; a++) {
            float v = p[a * inner];
            acc = MAX ? (v > acc ? v : acc) : acc + v;
        }
        y[i] = acc;
    }
}

}  // namespace

Status launch_norm(const OpNode& nd, cudaStream_t st, int* launches) {
    *launches += 1;
    const float* x = (const float*)nd.inputs[0];
    float* y = (float*)nd.output;
    int C = last_dim(nd);
    int64_t rows = leading_dims(nd);
    switch (nd.op) {
        case RT_OP_LAYERNORM:
            return run_rows<N_LAYER>(x, (const float*)nd.inputs[1], (const float*)nd.inputs[2], y,
                                     rows, C, extra_float(nd, 0), st);
        case RT_OP_RMSNORM:
            return run_rows<N_RMS>(x, (const float*)nd.inputs[1], nullptr, y, rows, C,
                                   extra_float(nd, 0), st);
        case RT_OP_SOFTMAX:
            return run_rows<N_SOFTMAX>(x, nullptr, nullptr, y, rows, C, 0.f, st);
        default:
            return Status::err(RT_ERR_BAD_OP, "norm: unexpected op");
    }
}

Status launch_reduce(const OpNode& nd, cudaStream_t st, int* launches) {
    *launches += 1;
    // csrc/executor.c:172-190: outer = prod(out_shape[:axis]),
    // inner = prod(out_shape[axis:]) (the reduced dim is absent from out_shape)
    int axis = nd.extra[0];
    int64_t axis_size = nd.extra[1];
    if (axis < 0 || axis > nd.n_dims) return Status::err(RT_ERR_BAD_NODE, "reduce: bad axis");
    int64_t outer = 1, inner = 1;
    for (int i = 0; i < axis; i++) outer *= nd.out_shape[i];
    for (int i = axis; i < nd.n_dims; i++) inner *= nd.out_shape[i];
    int grid = grid_for(outer * inner, 256);
    if (nd.op == RT_OP_MAX)
        reduce_axis_kernel<true><<<grid, 256, 0, st>>>((const float*)nd.inputs[0],
                                                       (float*)nd.output, outer, axis_size, inner);
    else
        reduce_axis_kernel<false><<<grid, 256, 0, st>>>((const float*)nd.inputs[0],
                                                        (float*)nd.output, outer, axis_size, inner);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

namespace {

// One warp per (b, s, h) row of D = 32 * VPT elements (warps in (b, s, h)
// order: consecutive warps read consecutive heads of one position).  The
// RMSNorm arithmetic is the warp-per-row path of row_kernel (same lane
// mapping, same sum order); the rotation pairs element d with d +- D/2,
// which lives VPT*16 elements = 16 lanes away.  Products and the sum are
// rounded as the separate MUL / NEG / CAT / ADD nodes would round them.
template <int VPT>
__global__ void __launch_bounds__(256) norm_rope_kernel(RopeFold r) {
    constexpr int D = 32 * VPT;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t rows = (int64_t)r.B * r.S * r.H;
    if (row >= rows) return;
    const int lane = threadIdx.x & 31;
    const int h = (int)(row % r.H);
    const int64_t bs = row / r.H;
    const int s = (int)(bs % r.S), b = (int)(bs / r.S);
    const float* yr = r.y + b * r.y_sb + (int64_t)s * r.y_ss + (int64_t)h * D + lane * VPT;
    float v[VPT];
    if (VPT == 4) {
        const float4 t = *reinterpret_cast<const float4*>(yr);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
        for (int i = 0; i < VPT; i++) v[i] = yr[i];
    }
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; i++) q += v[i] * v[i];
    const float ss = warp_sum(q);
    const float scale = 1.0f / sqrtf(ss / D + r.eps);
    const float* cr = r.cos + (int64_t)s * r.cs_ss + lane * VPT;
    const float* sr = r.sin + (int64_t)s * r.cs_ss + lane * VPT;
    const bool first_half = lane < 16;
    float o[VPT];
#pragma unroll
    for (int i = 0; i < VPT; i++) {
        const float n = v[i] * scale * r.w[lane * VPT + i];
        const float partner = __shfl_xor_sync(0xffffffffu, n, 16);
        const float rot = first_half ? -partner : partner;
        o[i] = __fadd_rn(__fmul_rn(n, cr[i]), __fmul_rn(rot, sr[i]));
    }
    float* orow = r.out + (((int64_t)b * r.H + h) * r.S + s) * D + lane * VPT;
    if (VPT == 4) {
        *reinterpret_cast<float4*>(orow) = make_float4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
        for (int i = 0; i < VPT; i++) orow[i] = o[i];
    }
}

}  // namespace

Status launch_norm_rope(const RopeFold& r, cudaStream_t st, int* launches) {
    const int64_t rows = (int64_t)r.B * r.S * r.H;
    if (rows == 0) return Status::ok();
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (r.D == 128) norm_rope_kernel<4><<<grid, 256, 0, st>>>(r);
    else if (r.D == 64) norm_rope_kernel<2><<<grid, 256, 0, st>>>(r);
    else return Status::err(RT_ERR_UNSUPPORTED, "norm_rope: head_dim must be 64 or 128");
    RT_LAUNCH_CHECK();
    *launches += 1;
    return Status::ok();
}

// LAYERNORM / RMSNORM whose output only feeds a GEMM's A operand: the rows
// go out as that GEMM's split planes (see row_kernel PLANES).
bool norm_planes_supported(const OpNode& n) {
    const int C = last_dim(n);
    // (fp16 scheme: whole 16-wide K blocks, so the plane is exactly 4 bytes per element)
    return (n.op == RT_OP_LAYERNORM || n.op == RT_OP_RMSNORM) && n.elem_size == 4 && C > 0 && C <= 4096 &&
           C % (gemm_scheme() == 2 ? 16 : 4) == 0 && aligned16(n.inputs[0]) && aligned16(n.inputs[1]) &&
           (n.op != RT_OP_LAYERNORM || aligned16(n.inputs[2]));
}

Status launch_norm_planes(const OpNode& nd, float* hi, void* x1, int scheme, cudaStream_t st, int* launches) {
    const int C = last_dim(nd);
    const int64_t rows = total_elements(nd) / C;
    if (rows == 0) return Status::ok();
    const float* x = (const float*)nd.inputs[0];
    const float eps = extra_float(nd, 0);
    uint16_t* xp = static_cast<uint16_t*>(x1);
    if (nd.op == RT_OP_LAYERNORM)
        run_rows_planes<N_LAYER>(x, (const float*)nd.inputs[1], (const float*)nd.inputs[2], hi, xp, rows, C, eps,
                                 scheme, st);
    else
        run_rows_planes<N_RMS>(x, (const float*)nd.inputs[1], nullptr, hi, xp, rows, C, eps, scheme, st);
    RT_LAUNCH_CHECK();
    *launches += 1;
    return Status::ok();
}

}  // namespace rt
