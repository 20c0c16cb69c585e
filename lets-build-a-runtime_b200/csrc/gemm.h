// gemm.h -- GEMM problem description shared by the GEMM paths.
#pragma once
#include "rt_internal.h"

namespace rt {

// C[b] = alpha * A[b] . op(B[b]) (+ bias[col]) for b < batches;
// A [M,K] row-major; B [N,K] if trans_b else [K,N]; C [M,N].
struct GemmProblem {
    const float* a;
    const float* b;
    float* c;
    const float* bias;
    int64_t M, N, K, batches;
    int64_t stride_a, stride_b, stride_c;
    float alpha;
    int trans_b;
};

Status decode_gemm(const OpNode& n, GemmProblem* p);
Status launch_simt_gemm(const GemmProblem& p, cudaStream_t st);

// tcgen05 3xTF32 path (k_gemm_tc.cu)
bool tc_gemm_applicable(const GemmProblem& p);
size_t tc_gemm_workspace_bytes(const GemmProblem& p);
Status tc_gemm_prepare(const GemmProblem& p, cudaStream_t st, int gate = 0);
Status tc_gemm_launch(const GemmProblem& p, cudaStream_t st, Workspace ws, int* launches,
                      const GemmFusion* f = nullptr);

}  // namespace rt

#include <cuda.h>
namespace rt {
// [batches][rows][K] -> hi/lo of the same layout, or (transpose) [batches][K][rows] -> [batches][rows][K].
Status split_operand(const float* x, float* hi, float* lo, int64_t batches, int64_t rows, int64_t K,
                     bool transpose, cudaStream_t st);
// fp32 3-D tensor map {d0 (contiguous), d1, d2}, box {box0, box1, 1}, swizzle 0/64/128 bytes.
Status encode_tmap_f32_3d(CUtensorMap* m, const float* base, int64_t d0, int64_t d1, int64_t d2, int box0,
                          int box1, int swizzle_bytes);
// fp32 tensor map of any rank (<= 5) with explicit byte strides of dims 1..rank-1
// (multiples of 16; dim 0 contiguous); out-of-range elements read as zero.
Status encode_tmap_f32(CUtensorMap* m, const float* base, int rank, const int64_t* dims,
                       const int64_t* byte_strides, const int* box, int swizzle_bytes);
}  // namespace rt
