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
#include <algorithm>
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

// A layout op as a list of runs: the output is `runs` runs of `len` units,
// each copied from one contiguous source run.  Index arithmetic (64-bit
// divisions) happens once per run and thread, not per element: a group of G
// lanes (a power of two, <= 32) copies one run, each lane moving up to four
// units per round with all loads issued before the stores.
//   MODE 0 TRANSPOSE N-D: run r = (((o*B + b)*M + m)*A + a), source run
//          (((o*A + a)*M + m)*B + b); runs are contiguous in the output
//   MODE 1 SLICE:  run o at y + o*len, from x + o*stride + off
//   MODE 2 CAT piece: run o from x + o*len, to y + o*stride + off
struct RunMap {
    int64_t A, M, B;      // MODE 0
    int64_t stride, off;  // MODES 1 / 2 (units)
};

template <typename T, int MODE>
__global__ void __launch_bounds__(256) runs_kernel(const T* __restrict__ x, T* __restrict__ y, RunMap p,
                                                   int64_t runs, int64_t len, int lg_g, int parts,
                                                   int64_t chunk) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int G = 1 << lg_g, lane = (int)(tid & (G - 1));
    const int64_t groups = ((int64_t)gridDim.x * blockDim.x) >> lg_g;
    const int64_t W = runs * parts;   // work items: a run, or a piece of one
    for (int64_t w = tid >> lg_g; w < W; w += 4 * groups) {
        // four work items at a time, so a lane has four loads in flight
        const T* src[4];
        T* dst[4];
        int64_t n[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t wk = w + k * groups;
            n[k] = 0;
            src[k] = x;
            dst[k] = y;
            if (wk >= W) continue;
            const int64_t r = parts == 1 ? wk : wk / parts;
            const int64_t i0 = parts == 1 ? 0 : (wk % parts) * chunk;
            n[k] = (parts == 1 || i0 + chunk > len ? len : i0 + chunk) - i0;
            if (MODE == 0) {
                int64_t q = r;
                const int64_t a = q % p.A;
                q /= p.A;
                const int64_t m = q % p.M;
                q /= p.M;
                const int64_t b = q % p.B, o = q / p.B;
                src[k] = x + (((o * p.A + a) * p.M + m) * p.B + b) * len + i0;
                dst[k] = y + r * len + i0;
            } else if (MODE == 1) {
                src[k] = x + r * p.stride + p.off + i0;
                dst[k] = y + r * len + i0;
            } else {
                src[k] = x + r * len + i0;
                dst[k] = y + r * p.stride + p.off + i0;
            }
        }
        const int64_t span = parts == 1 ? len : chunk;
        for (int64_t i = lane; i < span; i += G) {
            T v[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (i < n[k]) v[k] = src[k][i];
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (i < n[k]) dst[k][i] = v[k];
        }
    }
}

template <typename T, int MODE>
void launch_runs(const T* x, T* y, RunMap p, int64_t runs, int64_t len, cudaStream_t st) {
    if (runs <= 0 || len <= 0) return;
    int lg_g = 0;
    while (lg_g < 5 && ((int64_t)1 << lg_g) < len) lg_g++;
    // Few long runs: cut each into `parts` pieces of `chunk` units (a multiple
    // of 4*G) so that every SM gets work (four pieces per group round).
    const int64_t want = (int64_t)g_num_sms * 2048 * 4;       // resident threads x 4 items
    const int64_t round_units = (int64_t)4 << lg_g;
    int parts = 1;
    int64_t chunk = len;
    if ((runs << lg_g) < want && len > round_units) {
        const int64_t max_parts = (len + round_units - 1) / round_units;
        const int64_t need = (want + (runs << lg_g) - 1) / (runs << lg_g);
        parts = (int)std::min<int64_t>(max_parts, std::min<int64_t>(need, 1 << 20));
        chunk = ((len + parts - 1) / parts + round_units - 1) / round_units * round_units;
        parts = (int)((len + chunk - 1) / chunk);
    }
    const int64_t threads = (((runs * parts) + 3) / 4) << lg_g;   // four work items per group round
    runs_kernel<T, MODE><<<grid_for(threads, 256), 256, 0, st>>>(x, y, p, runs, len, lg_g, parts, chunk);
}

// Plain copy of n units.
template <typename T>
__global__ void copy_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = x[i];
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
        copy_kernel<T><<<grid_for(n, kT), kT, 0, st>>>((const T*)src, (T*)dst, n);
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
            return dispatch_unit(unit, [&](auto* tag) {
                using T = std::remove_pointer_t<decltype(tag)>;
                RunMap p{A, M, B, 0, 0};
                launch_runs<T, 0>((const T*)nd.inputs[0], (T*)nd.output, p, O * A * M * B, inner, st);
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
                RunMap p{1, 1, 1, (int64_t)(src_row / unit), (int64_t)(start / unit)};
                launch_runs<T, 1>((const T*)nd.inputs[0], (T*)nd.output, p, O, (int64_t)(row / unit), st);
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
                    RunMap p{1, 1, 1, (int64_t)(dst_row / unit), (int64_t)(off / unit)};
                    launch_runs<T, 2>((const T*)nd.inputs[k], (T*)nd.output, p, outer, (int64_t)(len / unit), st);
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
