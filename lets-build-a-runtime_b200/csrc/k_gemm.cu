// k_gemm.cu -- MATMUL and MATMUL_ADD: problem decoding and path selection,
// plus the exact-fp32 CUDA-core GEMM used where the tensor-core path does
// not apply (tiny or TMA-unaligned problems).
//
// Reference semantics (csrc/executor.c:197-224, :312-346; csrc/ops/matmul.c:19-79):
//   extras [K, trans_b, b_is_2d, alpha_bits (0 = 1.0)]
//   b_is_2d: M = prod(out_shape[:-1]), one batch;  else M = out_shape[-2],
//            batches = prod(out_shape[:-2]), A/B/C strided per batch
//   trans_b: B stored [N, K] (nn.Linear weight) else [K, N]
//   MATMUL:     C = alpha * A.op(B)
//   MATMUL_ADD: C = bias[col] + A.op(B)   (bias prefill then sgemm beta=1; alpha is 1)
#include "gemm.h"

namespace rt {
namespace {

// ---- CUDA-core fp32 GEMM: 128x128 tile, BK=8, 256 threads, 8x8 per thread.
constexpr int SB_M = 128, SB_N = 128, SB_K = 8;

__global__ void __launch_bounds__(256) simt_gemm_kernel(GemmProblem p) {
    __shared__ float As[2][SB_K][SB_M];
    __shared__ float Bs[2][SB_K][SB_N];
    const int tid = threadIdx.x;
    const int64_t bz = blockIdx.z;
    const float* A = p.a + bz * p.stride_a;
    const float* B = p.b + bz * p.stride_b;
    float* C = p.c + bz * p.stride_c;
    const int64_t m0 = (int64_t)blockIdx.y * SB_M, n0 = (int64_t)blockIdx.x * SB_N;
    const int tx = tid % 16, ty = tid / 16;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

    float ra[4], rb[4];
    auto load_global = [&](int64_t k0) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int idx = tid * 4 + i;          // 0..1023 over the 128x8 A tile
            int r = idx / SB_K, k = idx % SB_K;
            int64_t gm = m0 + r, gk = k0 + k;
            ra[i] = (gm < p.M && gk < p.K) ? A[gm * p.K + gk] : 0.0f;
            if (p.trans_b) {
                int64_t gn = n0 + r;
                rb[i] = (gn < p.N && gk < p.K) ? B[gn * p.K + gk] : 0.0f;
            } else {
                int kk = idx / SB_N, n = idx % SB_N;
                int64_t gn = n0 + n, gk2 = k0 + kk;
                rb[i] = (gn < p.N && gk2 < p.K) ? B[gk2 * p.N + gn] : 0.0f;
            }
        }
    };
    auto store_shared = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int idx = tid * 4 + i;
            As[buf][idx % SB_K][idx / SB_K] = ra[i];
            if (p.trans_b) Bs[buf][idx % SB_K][idx / SB_K] = rb[i];
            else Bs[buf][idx / SB_N][idx % SB_N] = rb[i];
        }
    };

    load_global(0);
    store_shared(0);
    __syncthreads();
    int buf = 0;
    for (int64_t k0 = 0; k0 < p.K; k0 += SB_K) {
        bool more = k0 + SB_K < p.K;
        if (more) load_global(k0 + SB_K);
#pragma unroll
        for (int k = 0; k < SB_K; k++) {
            float a[8], b[8];
            float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
            float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
            float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
            float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
            b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            store_shared(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (gm >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int64_t gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (gn >= p.N) continue;
            float v = p.alpha * acc[i][j];
            if (p.bias) v += p.bias[gn];
            C[gm * p.N + gn] = v;
        }
    }
}

}  // namespace

Status decode_gemm(const OpNode& n, GemmProblem* p) {
    if (n.n_dims < 2 && !(n.n_dims >= 1 && n.extra[2]))
        return Status::err(RT_ERR_BAD_NODE, "matmul: out_shape needs >= 2 dims");
    bool with_bias = n.op == RT_OP_MATMUL_ADD;
    if (n.n_inputs < (with_bias ? 3 : 2)) return Status::err(RT_ERR_BAD_NODE, "matmul: inputs");
    GemmProblem q{};
    q.N = last_dim(n);
    q.K = n.extra[0];
    q.trans_b = n.extra[1] != 0;
    bool b2d = n.extra[2] != 0;
    q.alpha = (!with_bias && n.extra[3]) ? extra_float(n, 3) : 1.0f;
    if (b2d) {
        q.M = leading_dims(n);
        q.batches = 1;
    } else {
        q.M = n.out_shape[n.n_dims - 2];
        q.batches = 1;
        for (int i = 0; i < n.n_dims - 2; i++) q.batches *= n.out_shape[i];
    }
    if (q.K <= 0 || q.N <= 0 || q.M < 0) return Status::err(RT_ERR_BAD_NODE, "matmul: bad sizes");
    q.a = (const float*)n.inputs[0];
    q.b = (const float*)n.inputs[1];
    q.c = (float*)n.output;
    q.bias = with_bias ? (const float*)n.inputs[2] : nullptr;
    q.stride_a = q.M * q.K;
    q.stride_b = q.N * q.K;
    q.stride_c = q.M * q.N;
    *p = q;
    return Status::ok();
}

Status launch_simt_gemm(const GemmProblem& p, cudaStream_t st) {
    if (p.M == 0) return Status::ok();
    if (p.batches > 65535) return Status::err(RT_ERR_UNSUPPORTED, "matmul: > 65535 batches");
    dim3 grid((unsigned)((p.N + SB_N - 1) / SB_N), (unsigned)((p.M + SB_M - 1) / SB_M),
              (unsigned)p.batches);
    simt_gemm_kernel<<<grid, 256, 0, st>>>(p);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

size_t gemm_workspace_bytes(const OpNode& n) {
    GemmProblem p;
    if (!decode_gemm(n, &p).good()) return 0;
    return tc_gemm_workspace_bytes(p);
}

Status prepare_gemm(const OpNode& n, cudaStream_t st, int gate) {
    GemmProblem p;
    Status s = decode_gemm(n, &p);
    if (!s.good()) return s;
    return tc_gemm_prepare(p, st, gate);
}

bool gemm_fusable(const OpNode& n) {
    GemmProblem p;
    return decode_gemm(n, &p).good() && tc_gemm_applicable(p);
}

Status launch_gemm(const OpNode& n, cudaStream_t st, Workspace ws, int* launches, const GemmFusion* f) {
    GemmProblem p;
    Status s = decode_gemm(n, &p);
    if (!s.good()) return s;
    if (tc_gemm_applicable(p)) return tc_gemm_launch(p, st, ws, launches, f);
    if (f) return Status::err(RT_ERR_ARGUMENT, "gemm: fused epilogue needs the tensor-core path");
    *launches += 1;
    return launch_simt_gemm(p, st);
}

}  // namespace rt
