// k_gemm_tc.cu -- placeholder until the tcgen05 path lands.
#include "gemm.h"
namespace rt {
bool tc_gemm_applicable(const GemmProblem&) { return false; }
size_t tc_gemm_workspace_bytes(const GemmProblem&) { return 0; }
Status tc_gemm_prepare(const GemmProblem&, cudaStream_t) { return Status::ok(); }
Status tc_gemm_launch(const GemmProblem&, cudaStream_t, Workspace, int*) {
    return Status::err(RT_ERR_UNSUPPORTED, "tcgen05 GEMM not built");
}
}  // namespace rt
