// rt_internal.h -- shared declarations of the CUDA backend (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <string>
#include <vector>

#include "b200exec.h"

namespace rt {

// Number of SMs on a B200; grids of bandwidth kernels are sized as
// multiples of it (queried at init, this is only the default).
extern int g_num_sms;

inline float extra_float(const OpNode& n, int i) {
    float f;
    memcpy(&f, &n.extra[i], 4);
    return f;
}
inline int64_t total_elements(const OpNode& n) {
    int64_t t = 1;
    for (int i = 0; i < n.n_dims; i++) t *= n.out_shape[i];
    return t;
}
inline int64_t leading_dims(const OpNode& n) {
    int64_t t = 1;
    for (int i = 0; i < n.n_dims - 1; i++) t *= n.out_shape[i];
    return t;
}
inline int last_dim(const OpNode& n) { return n.out_shape[n.n_dims - 1]; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Status carried out of planning/launch helpers.
struct Status {
    int code = RT_OK;
    std::string msg;
    static Status ok() { return {}; }
    static Status err(int c, std::string m) {
        Status s;
        s.code = c;
        s.msg = std::move(m);
        return s;
    }
    bool good() const { return code == RT_OK; }
};

// Scratch requirements a node reports at plan time and receives at launch.
struct Workspace {
    char* base = nullptr;
    size_t bytes = 0;
};

// Derived (split) forms of constant matrix operands, cached by the runtime
// for as long as the constant range stays registered and plans are kept.
struct SplitOperand {
    float* hi = nullptr;   // [batches][rows][K] tf32-exact high parts, K-major
    float* lo = nullptr;   // residuals a - hi
};
struct SplitKey {
    const void* src;
    int64_t batches, rows, k;
    int trans;
    bool operator<(const SplitKey& o) const;
};
// Returns the cached split of `key`, or null.
const SplitOperand* find_constant_split(const SplitKey& key);
// Allocates (device) and registers an empty split of `hi_elems` / `lo_elems`
// floats; the caller fills it.
Status create_constant_split(const SplitKey& key, size_t hi_elems, size_t lo_elems, SplitOperand* out);
// True when [p, p+bytes) lies inside a range marked with rt_mark_constant.
bool is_constant_range(const void* p, size_t bytes);

// ---- kernel families: each returns a Status; `ws` is the node's scratch.
// Planning hooks report scratch bytes a node needs beyond its arena buffers.
size_t gemm_workspace_bytes(const OpNode& n);
// Epilogue / prologue fusion of one GEMM launch (from a PlanItem).
struct GemmFusion {
    int act = 0;                    // 1: tanh-GELU after alpha and bias
    float* out = nullptr;           // write C here instead of the node's output
    float* plane_hi = nullptr;      // write the result as split A planes of a later GEMM
    void* plane_x = nullptr;
    const float* pre_hi = nullptr;  // this GEMM's A, already split
    const void* pre_x = nullptr;
    bool pre_seg = false;           // fp16 scheme: pre_x holds 2^-e per (row, 128 K) (a GEMM producer's
                                    // epilogue), not per row (a norm's)
    const float* bias = nullptr;    // bias to add (a node without one: a folded bias)
    const float* res = nullptr;     // residual added after the bias (same layout as C): a folded ADD
    int gate = 0;                   // 1 / 2: a folded GATED_ACT (SiLU / tanh-GELU): B's rows are taken in
                                    // the gated order and `out` receives act(gate) * up, N / 2 columns
};
Status launch_gemm(const OpNode& n, cudaStream_t st, Workspace ws, int* launches,
                   const GemmFusion* f = nullptr);
// Whether a GEMM node can take a GemmFusion (tensor-core path).
bool gemm_fusable(const OpNode& n);
bool gemm_cross_scheme();   // plane 1 of split operands: cross (true) or lo (false)
int gemm_scheme();          // 0 3xTF32, 1 tf32 + bf16 cross terms, 2 fp16 (one scaled plane + row scales)
bool gemm_planes_from_epilogues();   // GEMM / attention epilogues may write a GEMM's split A operand
bool norm_planes_supported(const OpNode& n);
// The split A operand of the GEMM reading this norm's output: for schemes
// 0/1 the hi plane at `hi` and plane 1 at `x1`; for the fp16 scheme (2) the
// fp16 plane at `hi` and the per-row 2^-e scales at `x1`.
Status launch_norm_planes(const OpNode& n, float* hi, void* x1, int scheme, cudaStream_t st, int* launches);
// constant splits, before capture (gate: the node's B in the gated row order, see GemmFusion)
Status prepare_gemm(const OpNode& n, cudaStream_t st, int gate = 0);

Status launch_attention(const OpNode& n, cudaStream_t st, Workspace ws, int* launches);

// Small graphs (k_tiny.cu): the whole node array in one cluster launch.
struct TinyPlan {
    OpNode* dev_nodes = nullptr;   // device copy of the node array
    int n = 0;                     // 0: not used by this plan
    char* mirror = nullptr;        // the allocation all node outputs live in (the arena), held in
    size_t mirror_bytes = 0;       //   shared memory during the launch when it fits (0: not mirrored)
};
// The allocation containing [p, p+1) made through this library: base and size.
bool allocation_of(const void* p, uintptr_t* base, size_t* bytes);
bool tiny_graph_applicable(const std::vector<OpNode>& nodes);
Status tiny_graph_build(const std::vector<OpNode>& nodes, TinyPlan* out);   // before any capture
Status launch_tiny(const TinyPlan& t, cudaStream_t st, int* launches);
void free_tiny(TinyPlan& t);
// Strided operands of a fused attention: element (b, h, s, d) of X lives at
// X + b*X_sb + h*X_sh + s*X_ss + d.  Produced by the plan's layout fusion.
struct AttnViews {
    const float* q;
    const float* k;
    const float* v;
    float* o;
    int64_t q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss, o_sb, o_sh, o_ss;
    int H;   // query heads per batch element
    // Non-null: O is the A operand of a following GEMM, written as its split
    // planes -- hi at `o` (same view), plane 1 here at the same element
    // offsets x 4 bytes (O contiguous [rows][K], K % 16 == 0).
    uint8_t* ox = nullptr;
    int ox_cross = 1;   // plane 1 layout: 1 cross (bf16 [hi | lo] per 16 block), 0 lo (fp32)
};
// Contiguous [B, H, S, D] views of an ATTENTION node's operands (4-D nodes only).
bool attention_default_views(const OpNode& n, AttnViews* v);
// Whether the tensor-core kernel (which takes strided views) runs this node.
bool attention_takes_views(const OpNode& n);
Status launch_attention_views(const OpNode& n, const AttnViews& v, cudaStream_t st, Workspace ws, int* launches);

// Fused per-head RMSNorm + rotary embedding + head split (fusion.cu folds the
// exporter's SLICE -> RMSNORM -> TRANSPOSE -> MUL(cos) / SLICE,SLICE,NEG,CAT,
// MUL(sin) -> ADD chain into the final ADD):
//   out[b,h,s,:] = rope(rmsnorm(y[b,s,h,:]) * w), rope(x) = x*cos[s] + rot(x)*sin[s],
//   rot(x)[d] = d < D/2 ? -x[d+D/2] : x[d-D/2].
struct RopeFold {
    const float* y;              // element (b, s, h, d) at y + b*y_sb + s*y_ss + h*D + d
    int64_t y_sb, y_ss;
    const float* w;              // RMSNorm weight [D]
    float eps;
    const float* cos;            // row s at cos + s*cs_ss (likewise sin)
    const float* sin;
    int64_t cs_ss;
    float* out;                  // [B, H, S, D] contiguous
    int B, H, S, D;
};
Status launch_norm_rope(const RopeFold& r, cudaStream_t st, int* launches);

// GATED_ACT reading x / up through row-strided views (a folded last-dim SLICE
// each): element (r, c) of x at x + r*x_ld + c; the output stays contiguous.
struct GatedViews {
    const float* x;
    const float* up;
    int64_t x_ld, up_ld;
};
Status launch_gated_views(const OpNode& n, const GatedViews& v, cudaStream_t st, int* launches);

// Per-node outcome of the plan-time layout fusion (fusion.cu).
struct PlanItem {
    bool skip = false;    // producer folded into its consumer: not launched
    bool views = false;   // attention launched with `attn` (strided operands)
    AttnViews attn{};
    int redirect_slot = -1;        // input slot now reading `redirect_ptr` (a folded producer's source)
    void* redirect_ptr = nullptr;
    // GEMM epilogue fusion: a GEMM that applies the folded activation node's
    // op and writes its output (`epi_out`), or -- when that output only feeds
    // the A operand of a later GEMM -- writes the split A planes of that GEMM
    // into the plan's carry buffer at `carry_off` (hi, then plane 1).
    int epi_act = 0;               // 0 none, 1 tanh-GELU
    void* epi_out = nullptr;
    int64_t carry_off = -1;        // producer: write A planes here (byte offset into the carry buffer)
    int64_t presplit_off = -1;     // consumer: A planes are already here; no split pre-pass
    bool presplit_seg = false;     //   fp16 scheme, written by a GEMM epilogue: scales per (row, 128 K)
    int64_t carry_plane_bytes = 0; // producer: bytes of the first plane it writes at carry_off / norm_planes_off / attn_planes_off
    int64_t presplit_plane_bytes = 0;  // consumer: bytes of the first plane at presplit_off (a GEMM can
                                       // both read split planes and write the next GEMM's)
    int64_t norm_planes_off = -1;  // LAYERNORM / RMSNORM: write the consumer GEMM's split A planes here
    int64_t attn_planes_off = -1;  // ATTENTION (merged-layout views): the same, from its O store
    int64_t epi_bias_off = -1;     // GEMM adds this merged bias (byte offset into the plan's bias buffer)
    const void* epi_res = nullptr; // GEMM adds this residual (a folded same-shape ADD) and writes epi_out
    bool rope = false;             // this (ADD) node launches the fused norm + rotary kernel instead
    RopeFold rp{};
    int epi_gate = 0;              // GEMM: a folded GATED_ACT, 1 + its act (see GemmFusion::gate); writes epi_out
    bool gated = false;            // this GATED_ACT reads its inputs through `gv`
    GatedViews gv{};
};
// Merged biases of bias folds: a plan-owned device buffer of `bytes`, zeroed
// in `zero` ranges then filled by device-to-device `copies` (dst offset, src, bytes).
struct BiasPlan {
    size_t bytes = 0;
    std::vector<std::pair<int64_t, int64_t>> zero;
    struct Copy { int64_t dst; const void* src; int64_t bytes; };
    std::vector<Copy> copies;
};
// `carry_bytes` receives the carry buffer size the items need (0 if none).
std::vector<PlanItem> plan_fusions(const std::vector<OpNode>& nodes,
                                   const std::vector<std::pair<uintptr_t, size_t>>& protected_ranges,
                                   size_t* carry_bytes = nullptr, BiasPlan* bias_plan = nullptr);
size_t attention_workspace_bytes(const OpNode& n);
Status prepare_attention(const OpNode& n);
Status launch_elementwise(const OpNode& n, cudaStream_t st, int* launches);
Status launch_norm(const OpNode& n, cudaStream_t st, int* launches);
Status launch_reduce(const OpNode& n, cudaStream_t st, int* launches);
Status launch_layout(const OpNode& n, cudaStream_t st, int* launches);

inline int grid_for(int64_t work_items, int threads, int per_sm = 8) {
    int64_t blocks = (work_items + threads - 1) / threads;
    int64_t cap = (int64_t)g_num_sms * per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

#define RT_CUDA_CHECK(expr)                                                           \
    do {                                                                              \
        cudaError_t _e = (expr);                                                      \
        if (_e != cudaSuccess)                                                        \
            return ::rt::Status::err(RT_ERR_CUDA, std::string(#expr ": ") +           \
                                                      cudaGetErrorString(_e));        \
    } while (0)

#define RT_LAUNCH_CHECK()                                                             \
    do {                                                                              \
        cudaError_t _e = cudaGetLastError();                                          \
        if (_e != cudaSuccess)                                                        \
            return ::rt::Status::err(RT_ERR_CUDA, std::string("launch: ") +           \
                                                      cudaGetErrorString(_e));        \
    } while (0)

}  // namespace rt
