// k_layout.cu -- data movement: TRANSPOSE, SLICE, CAT, RESHAPE copy, EMBEDDING.
//
// Reference semantics:
//   TRANSPOSE 2-D  csrc/ops/shape.c:8-13 (extras [rows, cols])
//   TRANSPOSE N-D  csrc/executor.c:237-261: [outer, A, mid, B, inner] ->
//                  [outer, B, mid, A, inner], `inner` contiguous elements moved as a unit
//   SLICE          csrc/ops/shape.c:92-106, extras [outer, dim, start, len, inner]
//   CAT            csrc/ops/shape.c:121-138, extras [dim, size_0, size_1, ...]
//   RESHAPE        csrc/executor.c:228-235 (copy only when the input is external)
//   EMBEDDING      csrc/ops/shape.c:72-79 (int64 ids, extras [embed_dim])
//
// All are pure copies, bound by HBM bandwidth: each output element is
// written once and read from one place.  Work is expressed in "units" of
// the widest access (16, 8 or 4 bytes ... 1) that divides every run length
// and every base address, so head-split transposes of 64/128-float rows move
// 16-byte vectors with fully coalesced reads and writes.
#include <initializer_list>
#include <type_traits>

#include "rt_internal.h"

namespace rt {
namespace {

// Largest power-of-two unit (<= 16 bytes) dividing all of `vals`.
inline int pick_unit(std::initializer_list<uint64_t> vals) {
    int u = 16;
    for (uint64_t v : vals)
        while (u > 1 && (v % u) != 0) u >>= 1;
    return u;
}

template <typename T>
__global__ void transpose_nd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t A,
                                    int64_t M, int64_t B, int64_t inner, int64_t total) {
    // output order: [o][b][m][a][i]  (i in units of T)
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = idx % inner;
        int64_t r = idx / inner;
        int64_t a = r % A;
        r /= A;
        int64_t m = r % M;
        r /= M;
        int64_t b = r % B;
        int64_t o = r / B;
        y[idx] = x[(((o * A + a) * M + m) * B + b) * inner + i];
    }
}

__global__ void transpose_2d_kernel(const float* __restrict__ x, float* __restrict__ y, int R,
                                    int C) {
    __shared__ float tile[32][33];
    for (int64_t tr = blockIdx.y; tr * 32 < R; tr += gridDim.y)
        for (int64_t tc = blockIdx.x; tc * 32 < C; tc += gridDim.x) {
            for (int k = threadIdx.y; k < 32; k += blockDim.y) {
                int64_t r = tr * 32 + k, c = tc * 32 + threadIdx.x;
                if (r < R && c < C) tile[k][threadIdx.x] = x[r * C + c];
            }
            __syncthreads();
            for (int k = threadIdx.y; k < 32; k += blockDim.y) {
                int64_t c = tc * 32 + k, r = tr * 32 + threadIdx.x;
                if (r < R && c < C) y[c * R + r] = tile[threadIdx.x][k];
            }
            __syncthreads();
        }
}

// y[o][j] = x[o][start + j] for j < len (all counted in units of T).
template <typename T>
__global__ void strided_rows_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                    int64_t len, int64_t src_stride, int64_t start) {
    int64_t total = rows * len;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = idx / len, j = idx % len;
        y[idx] = x[o * src_stride + start + j];
    }
}

// One CAT input: y[o][off + j] = x[o][j], j < len (units of T).
template <typename T>
__global__ void cat_piece_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                 int64_t len, int64_t dst_stride, int64_t off) {
    int64_t total = rows * len;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = idx / len, j = idx % len;
        y[o * dst_stride + off + j] = x[idx];
    }
}

__global__ void embedding_kernel(const int64_t* __restrict__ ids, const float* __restrict__ table,
                                 float* __restrict__ y, int64_t n_tok, int64_t E) {
    int64_t total = n_tok * E;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = idx / E, e = idx % E;
        y[idx] = table[ids[t] * E + e];
    }
}

template <typename F>
Status dispatch_unit(int unit, F&& f) {
    switch (unit) {
        case 16: f((float4*)nullptr); break;
        case 8: f((float2*)nullptr); break;
        case 4: f((float*)nullptr); break;
        case 2: f((uint16_t*)nullptr); break;
        default: f((uint8_t*)nullptr); break;
    }
    RT_LAUNCH_CHECK();
    return Status::ok();
}

constexpr int kT = 256;

Status copy_bytes(const void* src, void* dst, size_t bytes, cudaStream_t st) {
    if (src == dst || bytes == 0) return Status::ok();
    int unit = pick_unit({(uint64_t)(uintptr_t)src, (uint64_t)(uintptr_t)dst, bytes});
    return dispatch_unit(unit, [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        int64_t n = bytes / sizeof(T);
        strided_rows_kernel<T><<<grid_for(n, kT), kT, 0, st>>>((const T*)src, (T*)dst, 1, n, n, 0);
    });
}

}  // namespace

Status launch_layout(const OpNode& nd, cudaStream_t st, int* launches) {
    *launches += 1;
    const int es = nd.elem_size;
    if (es <= 0) return Status::err(RT_ERR_BAD_NODE, "layout: elem_size <= 0");
    switch (nd.op) {
        case RT_OP_RESHAPE:
            return copy_bytes(nd.inputs[0], nd.output, (size_t)total_elements(nd) * es, st);
        case RT_OP_TRANSPOSE: {
            if (nd.n_dims == 2) {
                if (es != 4) return Status::err(RT_ERR_UNSUPPORTED, "2-D transpose of non-fp32");
                int R = nd.extra[0], C = nd.extra[1];
                dim3 grid((C + 31) / 32 < 1024 ? (C + 31) / 32 : 1024,
                          (R + 31) / 32 < 1024 ? (R + 31) / 32 : 1024);
                transpose_2d_kernel<<<grid, dim3(32, 8), 0, st>>>((const float*)nd.inputs[0],
                                                                   (float*)nd.output, R, C);
                RT_LAUNCH_CHECK();
                return Status::ok();
            }
            int64_t O = nd.extra[0], A = nd.extra[1], M = nd.extra[2], B = nd.extra[3],
                    I = nd.extra[4];
            uint64_t run = (uint64_t)I * es;
            int unit = pick_unit({run, (uint64_t)(uintptr_t)nd.inputs[0],
                                  (uint64_t)(uintptr_t)nd.output});
            int64_t inner = run / unit;
            int64_t total = O * A * M * B * inner;
            return dispatch_unit(unit, [&](auto* tag) {
                using T = std::remove_pointer_t<decltype(tag)>;
                transpose_nd_kernel<T><<<grid_for(total, kT), kT, 0, st>>>(
                    (const T*)nd.inputs[0], (T*)nd.output, A, M, B, inner, total);
            });
        }
        case RT_OP_SLICE: {
            int64_t O = nd.extra[0], D = nd.extra[1], s = nd.extra[2], L = nd.extra[3],
                    I = nd.extra[4];
            if (s < 0 || L < 0 || s + L > D) return Status::err(RT_ERR_BAD_NODE, "SLICE: bad range");
            uint64_t row = (uint64_t)L * I * es, src_row = (uint64_t)D * I * es,
                     start = (uint64_t)s * I * es;
            int unit = pick_unit({row, src_row, start, (uint64_t)(uintptr_t)nd.inputs[0],
                                  (uint64_t)(uintptr_t)nd.output});
            return dispatch_unit(unit, [&](auto* tag) {
                using T = std::remove_pointer_t<decltype(tag)>;
                int64_t len = row / unit;
                strided_rows_kernel<T><<<grid_for(O * len, kT), kT, 0, st>>>(
                    (const T*)nd.inputs[0], (T*)nd.output, O, len, src_row / unit, start / unit);
            });
        }
        case RT_OP_CAT: {
            int dim = nd.extra[0];
            if (dim < 0 || dim >= nd.n_dims || nd.n_inputs < 1 || nd.n_inputs > RT_MAX_DIMS - 1)
                return Status::err(RT_ERR_BAD_NODE, "CAT: bad dim/inputs");
            int64_t outer = 1, inner = 1, tot = 0;
            for (int i = 0; i < dim; i++) outer *= nd.out_shape[i];
            for (int i = dim + 1; i < nd.n_dims; i++) inner *= nd.out_shape[i];
            for (int k = 0; k < nd.n_inputs; k++) tot += nd.extra[1 + k];
            uint64_t dst_row = (uint64_t)tot * inner * es;
            uint64_t off = 0;
            *launches -= 1;
            for (int k = 0; k < nd.n_inputs; k++) {
                uint64_t len = (uint64_t)nd.extra[1 + k] * inner * es;
                int unit = pick_unit({len, dst_row, off, (uint64_t)(uintptr_t)nd.inputs[k],
                                      (uint64_t)(uintptr_t)nd.output});
                Status s = dispatch_unit(unit, [&](auto* tag) {
                    using T = std::remove_pointer_t<decltype(tag)>;
                    int64_t l = len / unit;
                    cat_piece_kernel<T><<<grid_for(outer * l, kT), kT, 0, st>>>(
                        (const T*)nd.inputs[k], (T*)nd.output, outer, l, dst_row / unit,
                        off / unit);
                });
                if (!s.good()) return s;
                *launches += 1;
                off += len;
            }
            return Status::ok();
        }
        case RT_OP_EMBEDDING: {
            int64_t E = nd.extra[0];
            int64_t n_tok = leading_dims(nd);
            embedding_kernel<<<grid_for(n_tok * E, kT), kT, 0, st>>>(
                (const int64_t*)nd.inputs[0], (const float*)nd.inputs[1], (float*)nd.output, n_tok, E);
            RT_LAUNCH_CHECK();
            return Status::ok();
        }
        default:
            return Status::err(RT_ERR_BAD_OP, "layout: unexpected op");
    }
}

}  // namespace rt
