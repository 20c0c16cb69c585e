// k_tiny.cu -- a whole small graph in one launch.
//
// When every node of a plan is tiny (the toy block: 20 nodes, ~1.7 M
// multiply-adds, 32 tokens), the forward is bound by per-kernel launch and
// ramp-up time, not by arithmetic or bandwidth: 20 kernels of a few
// microseconds each.  Such a plan runs instead as ONE launch of a cluster of
// TC CTAs that walks the node array on the device, node after node, with a
// cluster barrier (barrier.cluster release / acquire: every global write of a
// node is visible to the whole cluster before the next node starts) between
// nodes.  Each node's work is spread over the cluster's threads
// (RT_TINY_CTAS=1: a single CTA instead).
//
// Semantics are the reference's dispatch (csrc/executor.c:54-397), node for
// node, on the same OpNode array the other kernels run:
//   element-wise and binary modes  csrc/ops/elementwise.c, csrc/ops/shape.c:32-62
//   LAYERNORM / RMSNORM / SOFTMAX  csrc/ops/norm.c:48-63, :100-107, csrc/ops/reduce.c:84-96
//   MATMUL / MATMUL_ADD            csrc/executor.c:197-224, :312-346 (alpha / bias)
//   ATTENTION (S <= 128)           csrc/ops/attn.c:26-80: scores = scale * Q K^T,
//                                  + mask or causal -inf, softmax, P V
//   TRANSPOSE / SLICE / CAT / RESHAPE  csrc/executor.c:228-282, csrc/ops/shape.c
// all in fp32 with the element-wise arithmetic shared with k_elementwise.cu.
// The plan's other launch path (one kernel per node) stays available for
// per-node profiling and is what every larger plan uses.
#include "dev_math.h"
#include "gemm.h"
#include "sm100_ptx.h"

namespace rt {
namespace {

constexpr int TT = 512;                 // threads per CTA
constexpr int TC = 8;                   // CTAs per cluster (portable maximum) of the cluster form
constexpr int TSMEM = 80 * 1024;        // dynamic shared memory per CTA (attention scores, GEMM tiles)
constexpr int KC = 256;                 // K per GEMM shared-memory chunk: the toy's GEMMs load A and B once
constexpr int MAX_NODES = 48;               // node array held in shared memory (48 x 312 B)
constexpr size_t NODES_SMEM = (MAX_NODES * sizeof(OpNode) + 15) / 16 * 16;
constexpr size_t MIRROR_MAX = 128 * 1024;   // largest arena held in shared memory (opt-in, RT_TINY_MIRROR=1)
constexpr int ATT_S_MAX = 128;          // S x S fp32 scores of one head fit TSMEM
constexpr int64_t MAX_NODE_ELEMS = (int64_t)1 << 18;
constexpr int64_t MAX_NODE_MACS = (int64_t)1 << 22;
constexpr int64_t MAX_TOTAL_MACS = (int64_t)1 << 23;

struct Th {
    int rank, C, tid, g, G;   // CTA rank, CTAs, thread in the CTA, thread over all CTAs, all threads
};

__device__ __forceinline__ int64_t numel_d(const OpNode& n) {
    int64_t t = 1;
    for (int i = 0; i < n.n_dims; i++) t *= n.out_shape[i];
    return t;
}
__device__ __forceinline__ float xfloat(const OpNode& n, int i) { return __int_as_float(n.extra[i]); }

__device__ __forceinline__ float warp_sum_d(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max_d(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int K>
__device__ void unary_d(const OpNode& n, const Th& t) {
    const float* x = (const float*)n.inputs[0];
    float* y = (float*)n.output;
    const float p = K == U_POW ? xfloat(n, 0) : 0.0f;
    const int64_t N = numel_d(n);
    for (int64_t e = t.g; e < N; e += t.G) y[e] = unary_op<K>(x[e], p);
}

// b indexed as b[e % period] (period = N same shape, = C bias row), or the
// scalar s when period == 0.
template <int K>
__device__ void binary_d(const float* a, const float* b, float s, float* y, int64_t N, int64_t period, const Th& t) {
    for (int64_t e = t.g; e < N; e += t.G) y[e] = bin_op<K>(a[e], period ? b[e % period] : s);
}

// General broadcast, extras from `base`: [ndim, a_strides, b_strides, out_shape].
template <int K>
__device__ void broadcast_d(const OpNode& n, int base, const Th& t) {
    const int nd = n.extra[base];
    const float* a = (const float*)n.inputs[0];
    const float* b = (const float*)n.inputs[1];
    float* y = (float*)n.output;
    int64_t N = 1;
    for (int d = 0; d < nd; d++) N *= n.extra[base + 1 + 2 * nd + d];
    for (int64_t e = t.g; e < N; e += t.G) {
        int64_t rem = e, ao = 0, bo = 0;
        for (int d = nd - 1; d >= 0; d--) {
            const int64_t sh = n.extra[base + 1 + 2 * nd + d];
            const int64_t c = rem % sh;
            rem /= sh;
            ao += c * n.extra[base + 1 + d];
            bo += c * n.extra[base + 1 + nd + d];
        }
        y[e] = bin_op<K>(a[ao], b[bo]);
    }
}

// SUB / MUL / DIV: modes 0 same shape, 1 scalar, 2 broadcast.
template <int K>
__device__ void binop_node_d(const OpNode& n, const Th& t) {
    const int mode = n.extra[0];
    const int64_t N = numel_d(n);
    if (mode == 1) binary_d<K>((const float*)n.inputs[0], nullptr, xfloat(n, 1), (float*)n.output, N, 0, t);
    else if (mode == 0) binary_d<K>((const float*)n.inputs[0], (const float*)n.inputs[1], 0.f, (float*)n.output, N, N, t);
    else broadcast_d<K>(n, 1, t);
}

// Row ops: one warp per row, all warps of the cluster.
template <int KIND>   // 0 LayerNorm, 1 RMSNorm, 2 softmax
__device__ void rows_d(const OpNode& n, const Th& t) {
    const int C = n.out_shape[n.n_dims - 1];
    const int64_t rows = C ? numel_d(n) / C : 0;
    const float* x = (const float*)n.inputs[0];
    float* y = (float*)n.output;
    const int lane = t.tid & 31;
    const float eps = KIND < 2 ? xfloat(n, 0) : 0.0f;
    const float* g = KIND < 2 ? (const float*)n.inputs[1] : nullptr;
    const float* bb = KIND == 0 ? (const float*)n.inputs[2] : nullptr;
    for (int64_t r = t.g >> 5; r < rows; r += t.G >> 5) {
        const float* xr = x + r * C;
        float* yr = y + r * C;
        if (KIND == 0) {
            float s = 0.f;
            for (int c = lane; c < C; c += 32) s += xr[c];
            const float mean = warp_sum_d(s) / C;
            float q = 0.f;
            for (int c = lane; c < C; c += 32) {
                const float d = xr[c] - mean;
                q += d * d;
            }
            const float sc = 1.0f / sqrtf(warp_sum_d(q) / C + eps);
            for (int c = lane; c < C; c += 32) yr[c] = (xr[c] - mean) * sc * g[c] + bb[c];
        } else if (KIND == 1) {
            float q = 0.f;
            for (int c = lane; c < C; c += 32) q += xr[c] * xr[c];
            const float sc = 1.0f / sqrtf(warp_sum_d(q) / C + eps);
            for (int c = lane; c < C; c += 32) yr[c] = xr[c] * sc * g[c];
        } else {
            float m = -INFINITY;
            for (int c = lane; c < C; c += 32) m = fmaxf(m, xr[c]);
            m = warp_max_d(m);
            float s = 0.f;
            for (int c = lane; c < C; c += 32) s += expf(xr[c] - m);
            s = warp_sum_d(s);
            for (int c = lane; c < C; c += 32) yr[c] = expf(xr[c] - m) / s;
        }
    }
}

// C[b] = alpha * A[b] . op(B[b]) (+ bias): 32 x 32 output tiles spread over
// the CTAs; per CTA A and B chunks of up to KC along K in shared memory (one
// chunk for K <= KC: all loads in flight at once), two outputs per thread.
__device__ void gemm_d(const OpNode& n, const Th& t, float* sm) {
    const bool with_bias = n.op == RT_OP_MATMUL_ADD;
    const int64_t N = n.out_shape[n.n_dims - 1], K = n.extra[0];
    const bool tb = n.extra[1] != 0, b2d = n.extra[2] != 0;
    const float alpha = (!with_bias && n.extra[3]) ? xfloat(n, 3) : 1.0f;
    int64_t M, batches = 1;
    if (b2d) {
        M = 1;
        for (int i = 0; i < n.n_dims - 1; i++) M *= n.out_shape[i];
    } else {
        M = n.out_shape[n.n_dims - 2];
        for (int i = 0; i < n.n_dims - 2; i++) batches *= n.out_shape[i];
    }
    const float* A = (const float*)n.inputs[0];
    const float* B = (const float*)n.inputs[1];
    const float* bias = with_bias ? (const float*)n.inputs[2] : nullptr;
    float* Cp = (float*)n.output;
    float(*As)[33] = reinterpret_cast<float(*)[33]>(sm);             // [KC k][32 m]
    float(*Bs)[33] = reinterpret_cast<float(*)[33]>(sm + KC * 33);   // [KC k][32 n]
    const int64_t mt = (M + 31) / 32, nt = (N + 31) / 32, tiles = batches * mt * nt;
    const int ty = t.tid >> 4, tx = (t.tid & 15) * 2;
    for (int64_t tile = t.rank; tile < tiles; tile += t.C) {
        const int64_t bz = tile / (mt * nt), rem = tile % (mt * nt);
        const int64_t m0 = (rem / nt) * 32, n0 = (rem % nt) * 32;
        const float* Ab = A + bz * M * K;
        const float* Bb = B + (b2d ? 0 : bz * N * K);
        float acc0 = 0.f, acc1 = 0.f;
        for (int64_t k0 = 0; k0 < K; k0 += KC) {
            // every load of the chunk in flight before the first shared store
            // (KC * 32 / TT = 16 values of A and of B per thread)
            constexpr int PER = KC * 32 / TT;
            float ra[PER], rb[PER];
#pragma unroll
            for (int i = 0; i < PER; i++) {
                const int e = t.tid + i * TT;
                const int k = e % KC, r = e / KC;   // A: consecutive threads walk K of one row
                const int64_t gm = m0 + r, gk = k0 + k;
                ra[i] = (gm < M && gk < K) ? Ab[gm * K + gk] : 0.f;
                if (tb) {
                    const int64_t gn = n0 + r;
                    rb[i] = (gn < N && gk < K) ? Bb[gn * K + gk] : 0.f;
                } else {
                    const int c = e & 31, kk = e >> 5;   // B [K][N]: consecutive threads walk N
                    const int64_t gn = n0 + c, gk2 = k0 + kk;
                    rb[i] = (gn < N && gk2 < K) ? Bb[gk2 * N + gn] : 0.f;
                }
            }
#pragma unroll
            for (int i = 0; i < PER; i++) {
                const int e = t.tid + i * TT;
                As[e % KC][e / KC] = ra[i];
                if (tb) Bs[e % KC][e / KC] = rb[i];
                else Bs[e >> 5][e & 31] = rb[i];
            }
            __syncthreads();
            const int kmax = (int)min((int64_t)KC, K - k0);
            for (int k = 0; k < kmax; k++) {
                const float a = As[k][ty];
                acc0 = fmaf(a, Bs[k][tx], acc0);
                acc1 = fmaf(a, Bs[k][tx + 1], acc1);
            }
            __syncthreads();
        }
        const int64_t gm = m0 + ty;
        if (gm < M) {
            float* cr = Cp + bz * M * N + gm * N;
            if (n0 + tx < N) cr[n0 + tx] = alpha * acc0 + (bias ? bias[n0 + tx] : 0.f);
            if (n0 + tx + 1 < N) cr[n0 + tx + 1] = alpha * acc1 + (bias ? bias[n0 + tx + 1] : 0.f);
        }
    }
}

// Standard attention, one (batch, head) per CTA at a time, scores in shared memory.
__device__ void attention_d(const OpNode& n, const Th& t, float* sm) {
    const int S = n.extra[0], D = n.extra[1], causal = n.extra[2], has_mask = n.extra[3];
    const int group = n.extra[4] > 0 ? n.extra[4] : 1;
    int64_t BH = 1;
    for (int i = 0; i < n.n_dims - 2; i++) BH *= n.out_shape[i];
    const float* Q = (const float*)n.inputs[0];
    const float* Kp = (const float*)n.inputs[1];
    const float* V = (const float*)n.inputs[2];
    const float* mask = has_mask ? (const float*)n.inputs[3] : nullptr;
    float* O = (float*)n.output;
    const float scale = 1.0f / sqrtf((float)D);
    const int lane = t.tid & 31, warp = t.tid >> 5;
    for (int64_t bh = t.rank; bh < BH; bh += t.C) {
        const float* q = Q + bh * S * D;
        const float* k = Kp + (bh / group) * S * D;
        const float* v = V + (bh / group) * S * D;
        if (S * S + 3 * S * D <= TSMEM / 4) {   // the head's Q, K, V staged in shared memory first
            float* sq = sm + S * S;
            float* sk = sq + S * D;
            float* svv = sk + S * D;
            for (int e = t.tid; e < S * D; e += TT) {
                const float a = q[e], b = k[e], c = v[e];
                sq[e] = a;
                sk[e] = b;
                svv[e] = c;
            }
            __syncthreads();
            q = sq;
            k = sk;
            v = svv;
        }
        for (int e = t.tid; e < S * S; e += TT) {
            const int i = e / S, j = e % S;
            float dot = 0.f;
            for (int d = 0; d < D; d++) dot = fmaf(q[i * D + d], k[j * D + d], dot);
            float s = scale * dot;
            if (mask) s += mask[bh * S * S + e];
            else if (causal && j > i) s = -INFINITY;
            sm[e] = s;
        }
        __syncthreads();
        for (int i = warp; i < S; i += TT / 32) {
            float* row = sm + i * S;
            float m = -INFINITY;
            for (int j = lane; j < S; j += 32) m = fmaxf(m, row[j]);
            m = warp_max_d(m);
            float s = 0.f;
            for (int j = lane; j < S; j += 32) {
                const float p = expf(row[j] - m);
                row[j] = p;
                s += p;
            }
            s = warp_sum_d(s);
            for (int j = lane; j < S; j += 32) row[j] /= s;
        }
        __syncthreads();
        for (int e = t.tid; e < S * D; e += TT) {
            const int i = e / D, d = e % D;
            float acc = 0.f;
            for (int j = 0; j < S; j++) acc = fmaf(sm[i * S + j], v[j * D + d], acc);
            O[bh * S * D + e] = acc;
        }
        __syncthreads();
    }
}

__device__ void layout_d(const OpNode& n, const Th& t) {
    const float* x = (const float*)n.inputs[0];
    float* y = (float*)n.output;
    switch (n.op) {
        case RT_OP_RESHAPE: {
            if (x == y) return;
            const int64_t N = numel_d(n);
            for (int64_t e = t.g; e < N; e += t.G) y[e] = x[e];
            return;
        }
        case RT_OP_TRANSPOSE: {
            if (n.n_dims == 2) {   // [R, C] -> [C, R]
                const int64_t R = n.extra[0], C = n.extra[1];
                for (int64_t e = t.g; e < R * C; e += t.G) {
                    const int64_t c = e / R, r = e % R;   // output [c][r]
                    y[e] = x[r * C + c];
                }
                return;
            }
            const int64_t A = n.extra[1], M = n.extra[2], B = n.extra[3], I = n.extra[4];
            const int64_t N = numel_d(n);
            for (int64_t e = t.g; e < N; e += t.G) {   // output [o][b][m][a][i]
                int64_t r = e;
                const int64_t i = r % I; r /= I;
                const int64_t a = r % A; r /= A;
                const int64_t m = r % M; r /= M;
                const int64_t b = r % B;
                const int64_t o = r / B;
                y[e] = x[(((o * A + a) * M + m) * B + b) * I + i];
            }
            return;
        }
        case RT_OP_SLICE: {
            const int64_t O = n.extra[0], D = n.extra[1], s = n.extra[2], L = n.extra[3], I = n.extra[4];
            for (int64_t e = t.g; e < O * L * I; e += t.G) {
                const int64_t o = e / (L * I), r = e % (L * I);
                y[e] = x[o * D * I + s * I + r];
            }
            return;
        }
        case RT_OP_CAT: {
            const int dim = n.extra[0];
            int64_t outer = 1, inner = 1, tot = 0;
            for (int i = 0; i < dim; i++) outer *= n.out_shape[i];
            for (int i = dim + 1; i < n.n_dims; i++) inner *= n.out_shape[i];
            for (int k = 0; k < n.n_inputs; k++) tot += n.extra[1 + k];
            int64_t off = 0;
            for (int k = 0; k < n.n_inputs; k++) {
                const int64_t len = (int64_t)n.extra[1 + k] * inner;
                const float* src = (const float*)n.inputs[k];
                for (int64_t e = t.g; e < outer * len; e += t.G) {
                    const int64_t o = e / len, r = e % len;
                    y[o * tot * inner + off + r] = src[e];
                }
                off += len;
            }
            return;
        }
        default:
            return;
    }
}

__device__ void run_node(const OpNode& n, const Th& t, float* sm) {
    const int64_t N = numel_d(n);
    const int C = n.out_shape[n.n_dims - 1];
    switch (n.op) {
        case RT_OP_RELU: unary_d<U_RELU>(n, t); break;
        case RT_OP_EXP: unary_d<U_EXP>(n, t); break;
        case RT_OP_TANH: unary_d<U_TANH>(n, t); break;
        case RT_OP_POW: unary_d<U_POW>(n, t); break;
        case RT_OP_GELU: unary_d<U_GELU>(n, t); break;
        case RT_OP_RSQRT: unary_d<U_RSQRT>(n, t); break;
        case RT_OP_SILU: unary_d<U_SILU>(n, t); break;
        case RT_OP_NEG: unary_d<U_NEG>(n, t); break;
        case RT_OP_COS: unary_d<U_COS>(n, t); break;
        case RT_OP_SIN: unary_d<U_SIN>(n, t); break;
        case RT_OP_ADD: {
            const int mode = n.extra[0];
            const float* a = (const float*)n.inputs[0];
            const float* b = (const float*)n.inputs[1];
            if (mode == 0) binary_d<B_ADD>(a, b, 0.f, (float*)n.output, N, C, t);
            else if (mode == 1) binary_d<B_ADD>(a, b, 0.f, (float*)n.output, N, N, t);
            else if (mode == 2) binary_d<B_ADD>(a, nullptr, xfloat(n, 1), (float*)n.output, N, 0, t);
            else broadcast_d<B_ADD>(n, 1, t);
            break;
        }
        case RT_OP_SUB: binop_node_d<B_SUB>(n, t); break;
        case RT_OP_MUL: binop_node_d<B_MUL>(n, t); break;
        case RT_OP_DIV: binop_node_d<B_DIV>(n, t); break;
        case RT_OP_FUSED_BIAS_RELU:
            binary_d<B_ADD_RELU>((const float*)n.inputs[0], (const float*)n.inputs[1], 0.f, (float*)n.output, N, C,
                                 t);
            break;
        case RT_OP_GATED_ACT: {
            const int has_bias = n.extra[0], act = n.extra[1];
            const float* x = (const float*)n.inputs[0];
            const float* up = (const float*)(has_bias ? n.inputs[2] : n.inputs[1]);
            const float* bias = has_bias ? (const float*)n.inputs[1] : nullptr;
            float* y = (float*)n.output;
            for (int64_t e = t.g; e < N; e += t.G) {
                const float v = x[e] + (bias ? bias[e % C] : 0.0f);
                y[e] = (act == 0 ? silu(v) : gelu_tanh(v)) * up[e];
            }
            break;
        }
        case RT_OP_LAYERNORM: rows_d<0>(n, t); break;
        case RT_OP_RMSNORM: rows_d<1>(n, t); break;
        case RT_OP_SOFTMAX: rows_d<2>(n, t); break;
        case RT_OP_MATMUL: case RT_OP_MATMUL_ADD: gemm_d(n, t, sm); break;
        case RT_OP_ATTENTION: attention_d(n, t, sm); break;
        default: layout_d(n, t); break;
    }
}

// NC == 1: one CTA, a CTA barrier between nodes; NC > 1: a cluster of NC
// CTAs (launched with the cluster attribute), a cluster barrier.
// Generic address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ void* map_rank(void* p, uint32_t rank) {
    uint64_t r;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
    return reinterpret_cast<void*>(r);
}

// The arena mirror: while the launch runs, every node pointer into the
// mirrored allocation is redirected to the same offset of a shared-memory
// copy of it (CTA 0's, reached through distributed shared memory by the other
// CTAs of a cluster); generic loads and stores then stay on the SM.  The
// allocation is copied in first (nodes only read what earlier nodes wrote,
// but the copy also keeps any never-written bytes identical) and out last.
template <int NC>
__global__ void __launch_bounds__(TT, 1) tiny_graph_kernel(const OpNode* __restrict__ nodes, int n_nodes,
                                                           char* __restrict__ mirror, size_t mirror_bytes) {
    extern __shared__ __align__(16) float sm[];
    Th t;
    t.rank = NC > 1 ? (int)ptx::cluster_ctarank() : 0;
    t.C = NC;
    t.tid = threadIdx.x;
    t.g = t.rank * TT + t.tid;
    t.G = NC * TT;
    OpNode* snodes = reinterpret_cast<OpNode*>(reinterpret_cast<char*>(sm) + TSMEM);   // [n_nodes]
    char* local_mirror = reinterpret_cast<char*>(sm) + TSMEM + NODES_SMEM;   // CTA 0's copy is the one used
    char* smirror = mirror_bytes ? (NC > 1 ? static_cast<char*>(map_rank(local_mirror, 0)) : local_mirror) : nullptr;
    if (mirror_bytes && t.rank == 0) {
        for (size_t o = (size_t)t.tid * 16; o < mirror_bytes; o += (size_t)TT * 16)
            *reinterpret_cast<uint4*>(local_mirror + o) = *reinterpret_cast<const uint4*>(mirror + o);
    }
    // the whole node array into shared memory at once (all loads in flight),
    // pointers redirected to the mirror when there is one
    for (size_t o = (size_t)t.tid * 16; o < (size_t)n_nodes * sizeof(OpNode); o += (size_t)TT * 16)
        *reinterpret_cast<uint4*>(reinterpret_cast<char*>(snodes) + o) =
            *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(nodes) + o);
    __syncthreads();
    if (smirror && t.tid < n_nodes) {
        OpNode& nd = snodes[t.tid];
        const uintptr_t b = reinterpret_cast<uintptr_t>(mirror);
        auto redirect = [&](void* p) -> void* {
            const uintptr_t x = reinterpret_cast<uintptr_t>(p);
            return (x >= b && x < b + mirror_bytes) ? static_cast<void*>(smirror + (x - b)) : p;
        };
        for (int k = 0; k < nd.n_inputs && k < RT_MAX_INPUTS; k++) nd.inputs[k] = redirect(nd.inputs[k]);
        nd.output = redirect(nd.output);
    }
    if (NC > 1) ptx::cluster_sync();
    else __syncthreads();
    for (int i = 0; i < n_nodes; i++) {
        run_node(snodes[i], t, sm);
        if (NC > 1) ptx::cluster_sync();   // release / acquire at cluster scope: node i's writes before node i+1
        else __syncthreads();              // CTA scope
    }
    if (mirror_bytes && t.rank == 0) {
        for (size_t o = (size_t)t.tid * 16; o < mirror_bytes; o += (size_t)TT * 16)
            *reinterpret_cast<uint4*>(mirror + o) = *reinterpret_cast<const uint4*>(local_mirror + o);
    }
    if (NC > 1) ptx::cluster_sync();   // CTA 0's shared memory outlives the other CTAs' last remote access
}

// The cluster of TC CTAs by default; RT_TINY_CTAS=1 runs one CTA with CTA
// barriers.  Measured on the toy block: 88 us per forward with 8 CTAs, 162 us
// with one (the GEMM and attention nodes need the extra SMs; every node
// costs ~2 us either way, its L2 round trips and the barrier).
int tiny_ctas() {
    static const int v = [] {
        const char* e = getenv("RT_TINY_CTAS");
        return e && atoi(e) == 1 ? 1 : TC;
    }();
    return v;
}

int64_t numel_h(const OpNode& n) { return total_elements(n); }

}  // namespace

// Whether the whole node array can run as one tiny-graph launch: every op has
// a device implementation here, every tensor is fp32, every node is small and
// the total multiply-adds stay within what one cluster does faster than a
// launch per node.  RT_TINY=0 turns the path off; RT_TINY=force also takes
// plans of fewer than four nodes (tests of the device implementations).
bool tiny_graph_applicable(const std::vector<OpNode>& nodes) {
    const char* env = getenv("RT_TINY");
    if (env && env[0] == '0') return false;
    const bool force = env && !strcmp(env, "force");
    if (nodes.empty() || nodes.size() > (size_t)MAX_NODES || (!force && nodes.size() < 4)) return false;
    int64_t macs = 0;
    for (const OpNode& n : nodes) {
        if (n.elem_size != 4 || n.n_dims < 1 || numel_h(n) > MAX_NODE_ELEMS) return false;
        switch (n.op) {
            case RT_OP_RELU: case RT_OP_EXP: case RT_OP_TANH: case RT_OP_POW: case RT_OP_GELU:
            case RT_OP_RSQRT: case RT_OP_SILU: case RT_OP_NEG: case RT_OP_COS: case RT_OP_SIN:
            case RT_OP_FUSED_BIAS_RELU: case RT_OP_GATED_ACT:
            case RT_OP_LAYERNORM: case RT_OP_RMSNORM: case RT_OP_SOFTMAX:
            case RT_OP_RESHAPE: case RT_OP_SLICE: case RT_OP_CAT:
                break;
            case RT_OP_TRANSPOSE:
                if (n.n_dims != 2 && n.n_dims < 1) return false;
                break;
            case RT_OP_ADD:
                if (n.extra[0] < 0 || n.extra[0] > 3) return false;
                if (n.extra[0] == 3 && (n.extra[1] < 1 || n.extra[1] > 7)) return false;
                break;
            case RT_OP_SUB: case RT_OP_MUL: case RT_OP_DIV:
                if (n.extra[0] < 0 || n.extra[0] > 2) return false;
                if (n.extra[0] == 2 && (n.extra[1] < 1 || n.extra[1] > 7)) return false;
                break;
            case RT_OP_MATMUL: case RT_OP_MATMUL_ADD: {
                GemmProblem p;
                if (!decode_gemm(n, &p).good()) return false;
                const int64_t m = p.batches * p.M * p.N * p.K;
                if (m > MAX_NODE_MACS) return false;
                macs += m;
                break;
            }
            case RT_OP_ATTENTION: {
                const int64_t S = n.extra[0], D = n.extra[1], group = n.extra[4] > 0 ? n.extra[4] : 1;
                int64_t BH = 1;
                for (int i = 0; i < n.n_dims - 2; i++) BH *= n.out_shape[i];
                if (S < 1 || S > ATT_S_MAX || D < 1 || D > 256 || BH % group) return false;
                macs += 2 * BH * S * S * D;
                break;
            }
            default:
                return false;   // EMBEDDING (int64 ids), MAX / SUM, PERMUTE
        }
    }
    return macs <= MAX_TOTAL_MACS;
}

Status tiny_graph_build(const std::vector<OpNode>& nodes, TinyPlan* out) {
    TinyPlan t;
    const size_t bytes = nodes.size() * sizeof(OpNode);
    RT_CUDA_CHECK(cudaMalloc(&t.dev_nodes, (bytes + 15) / 16 * 16));   // read in 16-byte units
    cudaError_t e = cudaMemcpy(t.dev_nodes, nodes.data(), bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tiny_graph_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(TSMEM + NODES_SMEM + MIRROR_MAX));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tiny_graph_kernel<TC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(TSMEM + NODES_SMEM + MIRROR_MAX));
    // Opt-in (RT_TINY_MIRROR=1): mirror the arena in shared memory when every
    // node writes into one allocation of this library that fits.  Measured on
    // the toy: slower (165 against 129 us per forward with 8 CTAs) -- the
    // other CTAs reach CTA 0's copy through distributed shared memory, whose
    // latency the dot-product loops of the attention and GEMM nodes expose.
    const char* mv = getenv("RT_TINY_MIRROR");
    uintptr_t base = 0;
    size_t abytes = 0;
    bool mirror = mv && mv[0] == '1';
    for (size_t i = 0; i < nodes.size() && mirror; i++) {
        uintptr_t b;
        size_t n;
        if (!allocation_of(nodes[i].output, &b, &n) || (i > 0 && b != base)) mirror = false;
        base = b;
        abytes = n;
    }
    if (mirror && abytes <= MIRROR_MAX && abytes % 16 == 0 && base % 16 == 0) {
        t.mirror = reinterpret_cast<char*>(base);
        t.mirror_bytes = abytes;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(t.dev_nodes);
        return Status::err(RT_ERR_CUDA, std::string("tiny graph: ") + cudaGetErrorString(e));
    }
    t.n = (int)nodes.size();
    *out = t;
    return Status::ok();
}

Status launch_tiny(const TinyPlan& t, cudaStream_t st, int* launches) {
    if (tiny_ctas() == 1) {
        tiny_graph_kernel<1><<<1, TT, TSMEM + NODES_SMEM + t.mirror_bytes, st>>>(t.dev_nodes, t.n, t.mirror, t.mirror_bytes);
    } else {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(TC);
        cfg.blockDim = dim3(TT);
        cfg.dynamicSmemBytes = TSMEM + NODES_SMEM + t.mirror_bytes;
        cfg.stream = st;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = TC;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        RT_CUDA_CHECK(cudaLaunchKernelEx(&cfg, tiny_graph_kernel<TC>, (const OpNode*)t.dev_nodes, t.n, t.mirror,
                                         t.mirror_bytes));
    }
    RT_LAUNCH_CHECK();
    *launches += 1;
    return Status::ok();
}

void free_tiny(TinyPlan& t) {
    if (t.dev_nodes) cudaFree(t.dev_nodes);
    t.dev_nodes = nullptr;
    t.n = 0;
}

}  // namespace rt
