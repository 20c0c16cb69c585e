// runtime.cu -- the C ABI of libb200exec.so: device memory, node-array
// validation, the launch sequence and its CUDA graph, profiling, errors.
//
// The reference's executor (csrc/executor.c:409-467) is a loop over the
// OpNode array calling dispatch_table[op].  Here the same loop runs once per
// distinct node array, at plan time, inside a CUDA stream capture; the
// resulting graph is instantiated and every later `execute` with the same
// array replays it with one cudaGraphLaunch.  Node arrays are identified by
// their contents (a 64-bit FNV-1a hash plus a full compare), so the caller
// may rebuild the array between calls, as the reference's compiled executor
// does when it patches input pointers (runtime/executor/compiled.py:77-82);
// with device staging buffers for graph inputs those pointers never change.
#include <stdio.h>
#include <stdlib.h>

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "gemm.h"
#include "rt_internal.h"
#include "sm100_ptx.h"

namespace rt {

int g_num_sms = 148;


namespace {

struct Alloc {
    size_t bytes;
    bool host;
    bool constant;
};

struct Plan {
    std::vector<OpNode> nodes;
    std::vector<size_t> ws_offset;   // per node, into `ws`
    std::vector<size_t> ws_bytes;
    char* ws = nullptr;
    size_t ws_total = 0;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    std::vector<PlanItem> items;   // per node: skipped by layout fusion / strided attention
    char* carry = nullptr;         // split A planes handed from one GEMM's epilogue to the next GEMM
    size_t carry_bytes = 0;
    char* bias = nullptr;          // merged biases of folded bias ADDs
    BiasPlan bias_plan;
    TinyPlan tiny;                 // set: the graph runs as one small-graph launch (per-node
                                   // profiling still launches the nodes one by one)
};

struct State {
    bool initialized = false;
    int device = -1;
    cudaStream_t stream = nullptr;
    std::map<uintptr_t, Alloc> allocs;                        // base -> info
    std::map<SplitKey, SplitOperand> splits;                 // derived constants
    std::unordered_map<uint64_t, std::vector<std::unique_ptr<Plan>>> plans;
    int last_error = RT_OK;
    std::string last_msg;
    std::vector<std::pair<uintptr_t, size_t>> protect;   // graph outputs (rt_protect)
    volatile int* kerr_host = nullptr;   // host-mapped error word written by kernels
    int* kerr_dev = nullptr;
    std::vector<cudaStream_t> chunk_streams;   // rt_execute_chunks, created on first use
};

State& S() {
    static State s;
    return s;
}

std::recursive_mutex& M() {
    static std::recursive_mutex m;
    return m;
}

int fail(int code, const std::string& msg) {
    S().last_error = code;
    S().last_msg = msg;
    return code;
}
int fail(const Status& s) { return fail(s.code, s.msg); }

uint64_t fnv1a(const void* data, size_t n, uint64_t h = 1469598103934665603ull) {
    const unsigned char* p = static_cast<const unsigned char*>(data);
    for (size_t i = 0; i < n; i++) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

// The allocation registered by this library that contains [p, p+bytes).
const Alloc* find_alloc(const void* p, size_t bytes, uintptr_t* base_out = nullptr) {
    auto& a = S().allocs;
    uintptr_t x = reinterpret_cast<uintptr_t>(p);
    auto it = a.upper_bound(x);
    if (it == a.begin()) return nullptr;
    --it;
    if (x < it->first || x + bytes > it->first + it->second.bytes) return nullptr;
    if (base_out) *base_out = it->first;
    return &it->second;
}

// Device-memory check for a buffer a node reads or writes.
Status check_buffer(const void* p, size_t bytes, int node, const char* what) {
    char buf[160];
    if (!p) {
        snprintf(buf, sizeof buf, "node %d: %s is NULL", node, what);
        return Status::err(RT_ERR_NULL_POINTER, buf);
    }
    uintptr_t base;
    const Alloc* a = find_alloc(p, 1, &base);
    if (a) {
        if (a->host) {
            snprintf(buf, sizeof buf, "node %d: %s points into pinned host memory", node, what);
            return Status::err(RT_ERR_HOST_POINTER, buf);
        }
        if (reinterpret_cast<uintptr_t>(p) + bytes > base + a->bytes) {
            snprintf(buf, sizeof buf, "node %d: %s [%p, +%zu) leaves its allocation", node, what, p,
                     bytes);
            return Status::err(RT_ERR_OUT_OF_RANGE, buf);
        }
        return Status::ok();
    }
    // not ours: accept device memory of this device allocated elsewhere
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        snprintf(buf, sizeof buf, "node %d: %s %p is not a device pointer", node, what, p);
        return Status::err(RT_ERR_HOST_POINTER, buf);
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
        snprintf(buf, sizeof buf, "node %d: %s %p is not device memory", node, what, p);
        return Status::err(RT_ERR_HOST_POINTER, buf);
    }
    if (attr.device != S().device) {
        snprintf(buf, sizeof buf, "node %d: %s lives on device %d, not %d", node, what, attr.device,
                 S().device);
        return Status::err(RT_ERR_HOST_POINTER, buf);
    }
    return Status::ok();
}

enum Family { F_NONE, F_ELEM, F_NORM, F_REDUCE, F_GEMM, F_ATTN, F_LAYOUT };

Family family_of(int op) {
    switch (op) {
        case RT_OP_RELU: case RT_OP_EXP: case RT_OP_TANH: case RT_OP_POW: case RT_OP_GELU:
        case RT_OP_RSQRT: case RT_OP_SILU: case RT_OP_NEG: case RT_OP_COS: case RT_OP_SIN:
        case RT_OP_ADD: case RT_OP_SUB: case RT_OP_MUL: case RT_OP_DIV:
        case RT_OP_FUSED_BIAS_RELU: case RT_OP_GATED_ACT:
            return F_ELEM;
        case RT_OP_LAYERNORM: case RT_OP_RMSNORM: case RT_OP_SOFTMAX:
            return F_NORM;
        case RT_OP_MAX: case RT_OP_SUM:
            return F_REDUCE;
        case RT_OP_MATMUL: case RT_OP_MATMUL_ADD:
            return F_GEMM;
        case RT_OP_ATTENTION:
            return F_ATTN;
        case RT_OP_RESHAPE: case RT_OP_TRANSPOSE: case RT_OP_SLICE: case RT_OP_CAT:
        case RT_OP_EMBEDDING:
            return F_LAYOUT;
        default:
            return F_NONE;   // includes PERMUTE (502): no dispatch entry in the reference
    }
}

// Per-node buffer extents (bytes) the kernels will touch; 0 = not checked
// beyond being device memory.  Mirrors what each reference dispatch_*
// function reads (csrc/executor.c:54-397).
Status validate_node(const OpNode& n, int i) {
    char buf[160];
    Family f = family_of(n.op);
    if (f == F_NONE) {
        snprintf(buf, sizeof buf, "node %d: unknown op %d", i, n.op);
        return Status::err(RT_ERR_BAD_OP, buf);
    }
    if (n.n_inputs < 0 || n.n_inputs > RT_MAX_INPUTS || n.n_dims < 1 || n.n_dims > RT_MAX_DIMS ||
        n.elem_size <= 0) {
        snprintf(buf, sizeof buf, "node %d (op %d): bad n_inputs/n_dims/elem_size", i, n.op);
        return Status::err(RT_ERR_BAD_NODE, buf);
    }
    int64_t numel = total_elements(n);
    for (int d = 0; d < n.n_dims; d++)
        if (n.out_shape[d] < 0) {
            snprintf(buf, sizeof buf, "node %d: negative out_shape", i);
            return Status::err(RT_ERR_BAD_NODE, buf);
        }
    size_t out_bytes = (size_t)numel * n.elem_size;
    std::vector<size_t> need(n.n_inputs, 1);
    int required = 1;
    int64_t C = last_dim(n);
    switch (n.op) {
        case RT_OP_ADD:
            required = n.extra[0] == 2 ? 1 : 2;
            if (n.extra[0] == 1 && n.n_inputs >= 2) need[1] = out_bytes;
            if (n.extra[0] == 0 && n.n_inputs >= 2) need[1] = C * 4;
            if (n.extra[0] != 3 && n.n_inputs >= 1) need[0] = out_bytes;
            break;
        case RT_OP_SUB: case RT_OP_MUL: case RT_OP_DIV:
            required = n.extra[0] == 1 ? 1 : 2;
            if (n.extra[0] == 0 && n.n_inputs >= 2) need[1] = out_bytes;
            if (n.extra[0] != 2 && n.n_inputs >= 1) need[0] = out_bytes;
            break;
        case RT_OP_FUSED_BIAS_RELU:
            required = 2;
            if (n.n_inputs >= 2) { need[0] = out_bytes; need[1] = C * 4; }
            break;
        case RT_OP_GATED_ACT:
            required = n.extra[0] ? 3 : 2;
            if (n.n_inputs >= required) {
                need[0] = out_bytes;
                need[required - 1] = out_bytes;
                if (n.extra[0]) need[1] = C * 4;
            }
            break;
        case RT_OP_LAYERNORM: case RT_OP_RMSNORM:
            required = n.op == RT_OP_LAYERNORM ? 3 : 2;
            if (n.n_inputs >= required) {
                need[0] = out_bytes;
                for (int k = 1; k < required; k++) need[k] = C * 4;
            }
            break;
        case RT_OP_MATMUL: case RT_OP_MATMUL_ADD: {
            // A [batches][M][K], B [N][K] or [K][N] (one per batch unless
            // b_is_2d), bias [N] -- csrc/executor.c:197-224, :312-346
            required = n.op == RT_OP_MATMUL ? 2 : 3;
            GemmProblem g;
            if (n.n_inputs >= required && decode_gemm(n, &g).good()) {
                need[0] = (size_t)(g.batches * g.M * g.K) * 4;
                need[1] = (size_t)(g.batches * g.N * g.K) * 4;
                if (required == 3) need[2] = (size_t)g.N * 4;
                if (g.M == 0) need[0] = 1;
            }
            break;
        }
        case RT_OP_ATTENTION: {
            // Q/O [BH][S][D], K/V [BH/group][S][D], mask [BH][S][S] --
            // csrc/executor.c:371-397, csrc/ops/attn.c:64-80, :238-253
            required = 3 + (n.extra[3] ? 1 : 0);
            const int64_t S = n.extra[0], D = n.extra[1], group = n.extra[4] > 0 ? n.extra[4] : 1;
            int64_t BH = 1;
            for (int d = 0; d < n.n_dims - 2; d++) BH *= n.out_shape[d];
            if (n.n_inputs >= required && S > 0 && D > 0 && BH % group == 0) {
                need[0] = out_bytes;
                need[1] = need[2] = (size_t)((BH / group) * S * D) * 4;
                if (n.extra[3]) need[3] = (size_t)(BH * S * S) * 4;
            }
            break;
        }
        case RT_OP_CAT:
            required = n.n_inputs;
            break;
        case RT_OP_EMBEDDING:
            required = 2;
            break;
        default:   // unary, softmax, reductions, reshape, transpose, slice
            required = 1;
            if (n.n_inputs >= 1 && (f == F_ELEM || n.op == RT_OP_SOFTMAX || n.op == RT_OP_RESHAPE ||
                                    n.op == RT_OP_TRANSPOSE))
                need[0] = out_bytes;
            break;
    }
    if (n.n_inputs < required) {
        snprintf(buf, sizeof buf, "node %d (op %d): %d inputs, needs %d", i, n.op, n.n_inputs, required);
        return Status::err(RT_ERR_BAD_NODE, buf);
    }
    // elementwise/norm/gemm/attention kernels compute in fp32 only
    if ((f == F_ELEM || f == F_NORM || f == F_REDUCE || f == F_GEMM || f == F_ATTN) &&
        n.elem_size != 4) {
        snprintf(buf, sizeof buf, "node %d (op %d): elem_size %d, only fp32 supported", i, n.op,
                 n.elem_size);
        return Status::err(RT_ERR_UNSUPPORTED, buf);
    }
    Status s = check_buffer(n.output, out_bytes ? out_bytes : 1, i, "output");
    if (!s.good()) return s;
    for (int k = 0; k < required; k++) {
        char what[32];
        snprintf(what, sizeof what, "input %d", k);
        s = check_buffer(n.inputs[k], need[k] ? need[k] : 1, i, what);
        if (!s.good()) return s;
    }
    return Status::ok();
}

size_t node_workspace(const OpNode& n) {
    if (family_of(n.op) == F_GEMM) return gemm_workspace_bytes(n);
    if (family_of(n.op) == F_ATTN) return attention_workspace_bytes(n);
    return 0;
}

Status launch_node(const OpNode& n, cudaStream_t st, Workspace ws, int* launches) {
    switch (family_of(n.op)) {
        case F_ELEM: return launch_elementwise(n, st, launches);
        case F_NORM: return launch_norm(n, st, launches);
        case F_REDUCE: return launch_reduce(n, st, launches);
        case F_GEMM: return launch_gemm(n, st, ws, launches);
        case F_ATTN: return launch_attention(n, st, ws, launches);
        case F_LAYOUT: return launch_layout(n, st, launches);
        default: return Status::err(RT_ERR_BAD_OP, "no kernel for op");
    }
}

Status launch_item(Plan& p, size_t i, cudaStream_t st, int* launches) {
    Workspace ws{p.ws + p.ws_offset[i], p.ws_bytes[i]};
    if (i < p.items.size()) {
        if (p.items[i].skip) return Status::ok();
        if (p.items[i].rope) return launch_norm_rope(p.items[i].rp, st, launches);
        if (p.items[i].gated) return launch_gated_views(p.nodes[i], p.items[i].gv, st, launches);
        if (p.items[i].norm_planes_off >= 0) {
            char* base = p.carry + p.items[i].norm_planes_off;
            return launch_norm_planes(p.nodes[i], reinterpret_cast<float*>(base), base + p.items[i].carry_plane_bytes,
                                      gemm_scheme(), st, launches);
        }
        if (p.items[i].views) {
            AttnViews v = p.items[i].attn;
            if (p.items[i].attn_planes_off >= 0) {
                char* base = p.carry + p.items[i].attn_planes_off;
                v.o = reinterpret_cast<float*>(base);
                v.ox = reinterpret_cast<uint8_t*>(base + p.items[i].carry_plane_bytes);
                v.ox_cross = gemm_cross_scheme() ? 1 : 0;
            }
            return launch_attention_views(p.nodes[i], v, st, ws, launches);
        }
        const PlanItem& it = p.items[i];
        if (it.epi_act || it.epi_out || it.carry_off >= 0 || it.presplit_off >= 0 || it.epi_bias_off >= 0 ||
            it.epi_gate) {
            GemmFusion f;
            f.act = it.epi_act;
            f.gate = it.epi_gate;
            if (it.epi_bias_off >= 0) f.bias = reinterpret_cast<const float*>(p.bias + it.epi_bias_off);
            f.out = static_cast<float*>(it.epi_out);
            f.res = static_cast<const float*>(it.epi_res);
            if (it.carry_off >= 0) {
                f.plane_hi = reinterpret_cast<float*>(p.carry + it.carry_off);
                f.plane_x = p.carry + it.carry_off + it.carry_plane_bytes;
            }
            if (it.presplit_off >= 0) {
                f.pre_hi = reinterpret_cast<const float*>(p.carry + it.presplit_off);
                f.pre_x = p.carry + it.presplit_off + it.presplit_plane_bytes;
                f.pre_seg = it.presplit_seg;
            }
            OpNode n = p.nodes[i];
            if (it.redirect_slot >= 0) n.inputs[it.redirect_slot] = it.redirect_ptr;
            return launch_gemm(n, st, ws, launches, &f);
        }
        if (p.items[i].redirect_slot >= 0) {
            OpNode n = p.nodes[i];
            n.inputs[p.items[i].redirect_slot] = p.items[i].redirect_ptr;
            return launch_node(n, st, ws, launches);
        }
    }
    return launch_node(p.nodes[i], st, ws, launches);
}

Status launch_all(Plan& p, cudaStream_t st, int* launches) {
    if (p.tiny.n) return launch_tiny(p.tiny, st, launches);
    for (size_t i = 0; i < p.nodes.size(); i++) {
        Status s = launch_item(p, i, st, launches);
        if (!s.good()) {
            s.msg = "node " + std::to_string(i) + " (op " + std::to_string(p.nodes[i].op) + "): " + s.msg;
            return s;
        }
    }
    return Status::ok();
}

void free_plan(Plan& p) {
    if (p.exec) cudaGraphExecDestroy(p.exec);
    if (p.ws) cudaFree(p.ws);
    if (p.carry) cudaFree(p.carry);
    if (p.bias) cudaFree(p.bias);
    free_tiny(p.tiny);
    p.exec = nullptr;
    p.ws = nullptr;
    p.carry = nullptr;
    p.bias = nullptr;
}

Status build_plan(const OpNode* nodes, int n, bool capture, Plan** out) {
    auto plan = std::make_unique<Plan>();
    plan->nodes.assign(nodes, nodes + n);
    for (int i = 0; i < n; i++) {
        Status s = validate_node(nodes[i], i);
        if (!s.good()) return s;
    }
    plan->items = plan_fusions(plan->nodes, S().protect, &plan->carry_bytes, &plan->bias_plan);
    if (getenv("RT_FUSE_VERBOSE")) {
        int skipped = 0, viewed = 0;
        for (auto& it : plan->items) { skipped += it.skip; viewed += it.views; }
        fprintf(stderr, "[b200exec] plan of %d nodes: %d skipped by layout fusion, %d strided attention\n", n,
                skipped, viewed);
    }
    size_t total = 0;
    for (int i = 0; i < n; i++) {
        // sized for the node as launched: a redirected input can change the
        // GEMM's choice of path (A overlapping C needs the split pre-pass)
        OpNode eff = nodes[i];
        if (i < (int)plan->items.size() && plan->items[i].redirect_slot >= 0)
            eff.inputs[plan->items[i].redirect_slot] = plan->items[i].redirect_ptr;
        size_t b = (node_workspace(eff) + 255) & ~(size_t)255;
        plan->ws_offset.push_back(total);
        plan->ws_bytes.push_back(b);
        total += b;
    }
    // Nodes run one after another on one stream, so their scratch can share
    // one region: every node gets offset 0 of a region sized for the largest.
    size_t peak = 0;
    for (size_t i = 0; i < plan->ws_bytes.size(); i++) {
        plan->ws_offset[i] = 0;
        if (plan->ws_bytes[i] > peak) peak = plan->ws_bytes[i];
    }
    plan->ws_total = peak;
    if (peak) {
        cudaError_t e = cudaMalloc(&plan->ws, peak);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return Status::err(RT_ERR_OOM, "workspace allocation failed");
        }
    }
    if (plan->carry_bytes) {
        cudaError_t e = cudaMalloc(&plan->carry, plan->carry_bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            free_plan(*plan);
            return Status::err(RT_ERR_OOM, "carry buffer allocation failed");
        }
    }
    if (plan->bias_plan.bytes) {   // merged biases: built once, before any capture
        const BiasPlan& bp = plan->bias_plan;
        cudaError_t e = cudaMalloc(&plan->bias, bp.bytes);
        for (auto& z : bp.zero)
            if (e == cudaSuccess) e = cudaMemsetAsync(plan->bias + z.first, 0, (size_t)z.second, S().stream);
        for (auto& c : bp.copies)
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(plan->bias + c.dst, c.src, (size_t)c.bytes, cudaMemcpyDeviceToDevice, S().stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(S().stream);
        if (e != cudaSuccess) {
            cudaGetLastError();
            free_plan(*plan);
            return Status::err(RT_ERR_CUDA, std::string("merged bias: ") + cudaGetErrorString(e));
        }
    }
    cudaStream_t st = S().stream;
    for (int i = 0; i < n; i++) {
        if (family_of(nodes[i].op) == F_GEMM || family_of(nodes[i].op) == F_ATTN) {
            Status s = family_of(nodes[i].op) == F_GEMM
                           ? prepare_gemm(nodes[i], st, i < (int)plan->items.size() ? plan->items[i].epi_gate : 0)
                           : prepare_attention(nodes[i]);
            if (!s.good()) {
                free_plan(*plan);
                return s;
            }
        }
    }
    if (tiny_graph_applicable(plan->nodes)) {
        Status s = tiny_graph_build(plan->nodes, &plan->tiny);
        if (!s.good()) {
            free_plan(*plan);
            return s;
        }
    }
    if (capture) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
            free_plan(*plan);
            return Status::err(RT_ERR_CUDA, std::string("prepare: ") + cudaGetErrorString(e));
        }
        e = cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed);
        if (e != cudaSuccess) {
            free_plan(*plan);
            return Status::err(RT_ERR_CUDA, std::string("begin capture: ") + cudaGetErrorString(e));
        }
        int launches = 0;
        Status s = launch_all(*plan, st, &launches);
        cudaGraph_t graph = nullptr;
        cudaError_t e2 = cudaStreamEndCapture(st, &graph);
        if (!s.good() || e2 != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            cudaGetLastError();
            free_plan(*plan);
            if (!s.good()) return s;
            return Status::err(RT_ERR_CUDA, std::string("end capture: ") + cudaGetErrorString(e2));
        }
        e = cudaGraphInstantiate(&plan->exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) {
            cudaGetLastError();
            free_plan(*plan);
            return Status::err(RT_ERR_CUDA, std::string("instantiate: ") + cudaGetErrorString(e));
        }
        plan->launches = launches;
    }
    uint64_t h = fnv1a(nodes, sizeof(OpNode) * (size_t)n, (uint64_t)n);
    *out = plan.get();
    S().plans[h].push_back(std::move(plan));
    return Status::ok();
}

Plan* find_plan(const OpNode* nodes, int n) {
    uint64_t h = fnv1a(nodes, sizeof(OpNode) * (size_t)n, (uint64_t)n);
    auto it = S().plans.find(h);
    if (it == S().plans.end()) return nullptr;
    for (auto& p : it->second)
        if ((int)p->nodes.size() == n && memcmp(p->nodes.data(), nodes, sizeof(OpNode) * n) == 0)
            return p.get();
    return nullptr;
}

Status get_plan(const OpNode* nodes, int n, Plan** out) {
    if (!S().initialized) return Status::err(RT_ERR_NOT_INITIALIZED, "rt_init not called");
    if (n < 0 || (n > 0 && !nodes)) return Status::err(RT_ERR_ARGUMENT, "bad node array");
    Plan* p = find_plan(nodes, n);
    if (p) {
        *out = p;
        return Status::ok();
    }
    return build_plan(nodes, n, true, out);
}

// Plans (and for constants, cached splits) that touch [lo, hi): a node
// writing into it, or any node pointer inside it.
bool plan_touches(const Plan& p, uintptr_t lo, uintptr_t hi) {
    for (const OpNode& nd : p.nodes) {
        const uintptr_t o = reinterpret_cast<uintptr_t>(nd.output);
        int64_t numel = 1;
        for (int d = 0; d < nd.n_dims && d < 24; d++) numel *= nd.out_shape[d];
        const uintptr_t oe = o + (uintptr_t)(numel * (nd.elem_size > 0 ? nd.elem_size : 1));
        if (o < hi && lo < oe) return true;
        for (int i = 0; i < nd.n_inputs && i < 12; i++) {
            const uintptr_t a = reinterpret_cast<uintptr_t>(nd.inputs[i]);
            if (a >= lo && a < hi) return true;
        }
    }
    return false;
}

void drop_plans_touching(uintptr_t lo, uintptr_t hi, bool splits_too) {
    bool synced = false;
    for (auto it = S().plans.begin(); it != S().plans.end();) {
        auto& v = it->second;
        for (size_t k = 0; k < v.size();) {
            if (plan_touches(*v[k], lo, hi)) {
                if (!synced) { cudaStreamSynchronize(S().stream); synced = true; }
                free_plan(*v[k]);
                v.erase(v.begin() + k);
            } else {
                k++;
            }
        }
        it = v.empty() ? S().plans.erase(it) : std::next(it);
    }
    if (!splits_too) return;
    for (auto it = S().splits.begin(); it != S().splits.end();) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(it->first.src);
        if (a >= lo && a < hi) {
            if (!synced) { cudaStreamSynchronize(S().stream); synced = true; }
            cudaFree(it->second.hi);
            cudaFree(it->second.lo);
            it = S().splits.erase(it);
        } else {
            ++it;
        }
    }
}

void clear_plans() {
    for (auto& kv : S().plans)
        for (auto& p : kv.second) free_plan(*p);
    S().plans.clear();
    for (auto& kv : S().splits) {
        cudaFree(kv.second.hi);
        cudaFree(kv.second.lo);
    }
    S().splits.clear();
}

}  // namespace

bool allocation_of(const void* p, uintptr_t* base, size_t* bytes) {
    uintptr_t b;
    const Alloc* a = find_alloc(p, 1, &b);
    if (!a || a->host) return false;
    *base = b;
    *bytes = a->bytes;
    return true;
}


bool SplitKey::operator<(const SplitKey& o) const {
    if (src != o.src) return src < o.src;
    if (batches != o.batches) return batches < o.batches;
    if (rows != o.rows) return rows < o.rows;
    if (k != o.k) return k < o.k;
    return trans < o.trans;
}

const SplitOperand* find_constant_split(const SplitKey& key) {
    auto it = S().splits.find(key);
    return it == S().splits.end() ? nullptr : &it->second;
}

Status create_constant_split(const SplitKey& key, size_t hi_elems, size_t lo_elems, SplitOperand* out) {
    SplitOperand s;
    if (cudaMalloc(&s.hi, hi_elems * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&s.lo, lo_elems * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        if (s.hi) cudaFree(s.hi);
        return Status::err(RT_ERR_OOM, "split operand allocation failed");
    }
    S().splits[key] = s;
    *out = s;
    return Status::ok();
}

bool is_constant_range(const void* p, size_t bytes) {
    const Alloc* a = find_alloc(p, bytes);
    return a && a->constant;
}

int* kernel_error_flag() { return S().kerr_dev; }

// After a synchronise: a kernel that gave up a bounded wait left its code.
int take_kernel_error() {
    if (!S().kerr_host) return 0;
    int v = *S().kerr_host;
    if (v) *S().kerr_host = 0;
    return v;
}

// A wait that nothing will ever complete: one thread waits on an mbarrier
// that no thread arrives on, through the same bounded wait the tensor-core
// kernels use.  After limit_ns it records ERR_PROBE in the error word and
// returns; it exercises the timeout path without any fault.
constexpr int ERR_PROBE = 0x301;
__global__ void unsatisfied_wait_kernel(uint64_t limit_ns, int* err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        abort_flag = 0;
        ptx::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) ptx::wait_bounded(&bar, 0, &abort_flag, err, ERR_PROBE, limit_ns);
    __syncthreads();
}

}  // namespace rt

// ============================================================== C ABI
using namespace rt;

#define RT_GUARD std::lock_guard<std::recursive_mutex> _g(M())
#define RT_NEED_INIT \
    if (!S().initialized) return fail(RT_ERR_NOT_INITIALIZED, "rt_init not called")

extern "C" {

const char* rt_version(void) { return "b200exec 0.1 (sm_100a)"; }

int rt_init(int device) {
    RT_GUARD;
    if (S().initialized) {
        if (S().device == device) return RT_OK;
        return fail(RT_ERR_ARGUMENT, "already initialised on another device; rt_destroy first");
    }
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    e = cudaStreamCreateWithFlags(&S().stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(e));
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0)
        g_num_sms = sms;
    void* flag = nullptr;
    e = cudaHostAlloc(&flag, 64, cudaHostAllocMapped);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("mapped flag: ") + cudaGetErrorString(e));
    memset(flag, 0, 64);
    void* dflag = nullptr;
    e = cudaHostGetDevicePointer(&dflag, flag, 0);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("mapped flag: ") + cudaGetErrorString(e));
    S().kerr_host = static_cast<volatile int*>(flag);
    S().kerr_dev = static_cast<int*>(dflag);
    S().device = device;
    S().initialized = true;
    return RT_OK;
}

int rt_destroy(void) {
    RT_GUARD;
    if (!S().initialized) return RT_OK;
    cudaStreamSynchronize(S().stream);
    for (cudaStream_t st : S().chunk_streams) {
        cudaStreamSynchronize(st);
        cudaStreamDestroy(st);
    }
    S().chunk_streams.clear();
    clear_plans();
    for (auto& kv : S().allocs) {
        if (kv.second.host) cudaFreeHost(reinterpret_cast<void*>(kv.first));
        else cudaFree(reinterpret_cast<void*>(kv.first));
    }
    S().allocs.clear();
    cudaStreamDestroy(S().stream);
    S().stream = nullptr;
    if (S().kerr_host) cudaFreeHost(const_cast<int*>(S().kerr_host));
    S().kerr_host = nullptr;
    S().kerr_dev = nullptr;
    S().initialized = false;
    S().device = -1;
    return RT_OK;
}

void* rt_alloc(size_t bytes) {
    RT_GUARD;
    if (!S().initialized) { fail(RT_ERR_NOT_INITIALIZED, "rt_init not called"); return nullptr; }
    void* p = nullptr;
    size_t b = bytes ? bytes : 1;
    if (cudaMalloc(&p, b) != cudaSuccess) {
        cudaGetLastError();
        fail(RT_ERR_OOM, "cudaMalloc failed for " + std::to_string(bytes) + " bytes");
        return nullptr;
    }
    // the reference arena is zero-initialised (runtime/executor/common.py:86).
    // On the library stream and waited for: the stream does not synchronise
    // with the legacy default stream, so a plain cudaMemset could still be
    // running when the first graph writes this memory.
    if (cudaMemsetAsync(p, 0, b, S().stream) != cudaSuccess || cudaStreamSynchronize(S().stream) != cudaSuccess) {
        cudaFree(p);
        fail(RT_ERR_CUDA, "cudaMemset failed");
        return nullptr;
    }
    S().allocs[reinterpret_cast<uintptr_t>(p)] = Alloc{b, false, false};
    return p;
}

int rt_free(void* dev) {
    RT_GUARD;
    RT_NEED_INIT;
    auto it = S().allocs.find(reinterpret_cast<uintptr_t>(dev));
    if (it == S().allocs.end() || it->second.host) return fail(RT_ERR_ARGUMENT, "rt_free: unknown pointer");
    // Plans that use this memory, and derived forms (splits) of a constant,
    // go with it; other graphs keep their captured plans.  Graph outputs
    // registered inside it go too (a later allocation at the same address
    // belongs to another graph).
    const uintptr_t lo = it->first, hi = lo + it->second.bytes;
    drop_plans_touching(lo, hi, it->second.constant);
    auto& pr = S().protect;
    for (size_t k = 0; k < pr.size();)
        if (pr[k].first >= lo && pr[k].first < hi) pr.erase(pr.begin() + k);
        else k++;
    cudaFree(dev);
    S().allocs.erase(it);
    return RT_OK;
}

void* rt_host_alloc(size_t bytes) {
    RT_GUARD;
    if (!S().initialized) { fail(RT_ERR_NOT_INITIALIZED, "rt_init not called"); return nullptr; }
    void* p = nullptr;
    size_t b = bytes ? bytes : 1;
    if (cudaMallocHost(&p, b) != cudaSuccess) {
        cudaGetLastError();
        fail(RT_ERR_OOM, "cudaMallocHost failed");
        return nullptr;
    }
    memset(p, 0, b);
    S().allocs[reinterpret_cast<uintptr_t>(p)] = Alloc{b, true, false};
    return p;
}

int rt_host_free(void* host) {
    RT_GUARD;
    RT_NEED_INIT;
    auto it = S().allocs.find(reinterpret_cast<uintptr_t>(host));
    if (it == S().allocs.end() || !it->second.host) return fail(RT_ERR_ARGUMENT, "rt_host_free: unknown pointer");
    cudaFreeHost(host);
    S().allocs.erase(it);
    return RT_OK;
}

int rt_upload(void* dst, const void* src, size_t bytes) {
    RT_GUARD;
    RT_NEED_INIT;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, S().stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(S().stream);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("upload: ") + cudaGetErrorString(e));
    return RT_OK;
}

int rt_download(void* dst, const void* src, size_t bytes) {
    RT_GUARD;
    RT_NEED_INIT;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, S().stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(S().stream);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("download: ") + cudaGetErrorString(e));
    return RT_OK;
}

int rt_mark_constant(void* dev, size_t bytes) {
    RT_GUARD;
    RT_NEED_INIT;
    auto it = S().allocs.find(reinterpret_cast<uintptr_t>(dev));
    if (it == S().allocs.end() || it->second.host || it->second.bytes < bytes)
        return fail(RT_ERR_ARGUMENT, "rt_mark_constant: not the base of a library device allocation");
    it->second.constant = true;
    return RT_OK;
}

int rt_prepare(const OpNode* nodes, int n) {
    RT_GUARD;
    Plan* p;
    Status s = get_plan(nodes, n, &p);
    return s.good() ? RT_OK : fail(s);
}

int rt_execute(const OpNode* nodes, int n, int flags) {
    RT_GUARD;
    RT_NEED_INIT;
    cudaStream_t st = S().stream;
    if (flags & RT_FLAG_EAGER) {
        Plan* p = find_plan(nodes, n);
        Status s;
        if (!p) {
            s = build_plan(nodes, n, false, &p);
            if (!s.good()) return fail(s);
        }
        int launches = 0;
        s = launch_all(*p, st, &launches);
        if (!s.good()) return fail(s);
    } else {
        Plan* p;
        Status s = get_plan(nodes, n, &p);
        if (!s.good()) return fail(s);
        if (p->exec) {
            cudaError_t e = cudaGraphLaunch(p->exec, st);
            if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("graph launch: ") + cudaGetErrorString(e));
        } else {
            int launches = 0;
            s = launch_all(*p, st, &launches);
            if (!s.good()) return fail(s);
        }
    }
    if (!(flags & RT_FLAG_ASYNC)) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("execute: ") + cudaGetErrorString(e));
        if (int k = take_kernel_error())
            return fail(RT_ERR_KERNEL_TIMEOUT, "a kernel abandoned a bounded wait, code " + std::to_string(k));
    }
    return RT_OK;
}

void execute(OpNode* nodes, int n_nodes) { rt_execute(nodes, n_nodes, 0); }

int rt_execute_io(const OpNode* nodes, int n, const RtCopy* h2d, int n_in, const RtCopy* d2h,
                  int n_out) {
    RT_GUARD;
    RT_NEED_INIT;
    cudaStream_t st = S().stream;
    Plan* p;
    Status s = get_plan(nodes, n, &p);
    if (!s.good()) return fail(s);
    for (int i = 0; i < n_in; i++) {
        cudaError_t e = cudaMemcpyAsync(h2d[i].dst, h2d[i].src, h2d[i].bytes, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("h2d: ") + cudaGetErrorString(e));
    }
    if (p->exec) {
        cudaError_t e = cudaGraphLaunch(p->exec, st);
        if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("graph launch: ") + cudaGetErrorString(e));
    }
    for (int i = 0; i < n_out; i++) {
        cudaError_t e = cudaMemcpyAsync(d2h[i].dst, d2h[i].src, d2h[i].bytes, cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("d2h: ") + cudaGetErrorString(e));
    }
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("execute_io: ") + cudaGetErrorString(e));
    if (int k = take_kernel_error())
        return fail(RT_ERR_KERNEL_TIMEOUT, "a kernel abandoned a bounded wait, code " + std::to_string(k));
    return RT_OK;
}

int rt_execute_chunks(const RtChunk* chunks, int n_chunks) {
    RT_GUARD;
    RT_NEED_INIT;
    if (n_chunks < 0 || (n_chunks > 0 && !chunks)) return fail(RT_ERR_ARGUMENT, "rt_execute_chunks: bad chunk array");
    std::vector<Plan*> plans((size_t)n_chunks);
    for (int c = 0; c < n_chunks; c++) {   // plan (and capture) before anything is enqueued
        Status s = get_plan(chunks[c].nodes, chunks[c].n_nodes, &plans[c]);
        if (!s.good()) {
            s.msg = "chunk " + std::to_string(c) + ": " + s.msg;
            return fail(s);
        }
    }
    auto& ss = S().chunk_streams;
    while ((int)ss.size() < n_chunks) {
        cudaStream_t st = nullptr;
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess)
            return fail(RT_ERR_CUDA, "rt_execute_chunks: stream creation failed");
        ss.push_back(st);
    }
    // work already queued on the library stream comes first
    cudaEvent_t ready = nullptr;
    if (cudaEventCreateWithFlags(&ready, cudaEventDisableTiming) != cudaSuccess)
        return fail(RT_ERR_CUDA, "rt_execute_chunks: event creation failed");
    cudaEventRecord(ready, S().stream);
    cudaError_t e = cudaSuccess;
    for (int c = 0; c < n_chunks && e == cudaSuccess; c++) {
        cudaStream_t st = ss[c];
        e = cudaStreamWaitEvent(st, ready, 0);
        for (int i = 0; i < chunks[c].n_in && e == cudaSuccess; i++)
            e = cudaMemcpyAsync(chunks[c].h2d[i].dst, chunks[c].h2d[i].src, chunks[c].h2d[i].bytes,
                                cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess && plans[c]->exec) e = cudaGraphLaunch(plans[c]->exec, st);
        for (int i = 0; i < chunks[c].n_out && e == cudaSuccess; i++)
            e = cudaMemcpyAsync(chunks[c].d2h[i].dst, chunks[c].d2h[i].src, chunks[c].d2h[i].bytes,
                                cudaMemcpyDeviceToHost, st);
    }
    for (int c = 0; c < n_chunks; c++) {
        cudaError_t e2 = cudaStreamSynchronize(ss[c]);
        if (e == cudaSuccess) e = e2;
    }
    cudaEventDestroy(ready);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("execute_chunks: ") + cudaGetErrorString(e));
    if (int k = take_kernel_error())
        return fail(RT_ERR_KERNEL_TIMEOUT, "a kernel abandoned a bounded wait, code " + std::to_string(k));
    return RT_OK;
}

int rt_kernel_launches(const OpNode* nodes, int n) {
    RT_GUARD;
    Plan* p;
    Status s = get_plan(nodes, n, &p);
    if (!s.good()) return -fail(s);
    return p->launches;
}

int rt_profile(const OpNode* nodes, int n, int reps, float* ms_per_node) {
    RT_GUARD;
    RT_NEED_INIT;
    if (reps < 1 || !ms_per_node) return fail(RT_ERR_ARGUMENT, "rt_profile: reps >= 1 and an output array");
    Plan* p;
    Status s = get_plan(nodes, n, &p);
    if (!s.good()) return fail(s);
    cudaStream_t st = S().stream;
    std::vector<cudaEvent_t> ev(n + 1);
    for (auto& e : ev) cudaEventCreate(&e);
    std::vector<double> acc(n, 0.0);
    for (int r = 0; r < reps && s.good(); r++) {
        cudaEventRecord(ev[0], st);
        int launches = 0;
        for (int i = 0; i < n && s.good(); i++) {
            s = launch_item(*p, (size_t)i, st, &launches);
            cudaEventRecord(ev[i + 1], st);
        }
        if (cudaEventSynchronize(ev[n]) != cudaSuccess) s = Status::err(RT_ERR_CUDA, "profile sync");
        for (int i = 0; i < n && s.good(); i++) {
            float ms = 0;
            cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            acc[i] += ms;
        }
    }
    for (auto& e : ev) cudaEventDestroy(e);
    if (!s.good()) return fail(s);
    for (int i = 0; i < n; i++) ms_per_node[i] = (float)(acc[i] / reps);
    return RT_OK;
}

int rt_release(const OpNode* nodes, int n) {
    RT_GUARD;
    if (!S().initialized || n < 0 || (n > 0 && !nodes)) return RT_OK;
    uint64_t h = fnv1a(nodes, sizeof(OpNode) * (size_t)n, (uint64_t)n);
    auto it = S().plans.find(h);
    if (it == S().plans.end()) return RT_OK;
    cudaStreamSynchronize(S().stream);
    auto& v = it->second;
    for (size_t k = 0; k < v.size();) {
        if ((int)v[k]->nodes.size() == n && memcmp(v[k]->nodes.data(), nodes, sizeof(OpNode) * n) == 0) {
            free_plan(*v[k]);
            v.erase(v.begin() + k);
        } else {
            k++;
        }
    }
    if (v.empty()) S().plans.erase(it);
    return RT_OK;
}

int rt_plan_count(void) {
    int c = 0;
    for (auto& kv : S().plans) c += (int)kv.second.size();
    return c;
}

int rt_reset_plans(void) {
    RT_GUARD;
    RT_NEED_INIT;
    cudaStreamSynchronize(S().stream);
    clear_plans();
    return RT_OK;
}

int rt_synchronize(void) {
    RT_GUARD;
    RT_NEED_INIT;
    cudaError_t e = cudaStreamSynchronize(S().stream);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, cudaGetErrorString(e));
    if (int k = take_kernel_error())
        return fail(RT_ERR_KERNEL_TIMEOUT, "a kernel abandoned a bounded wait, code " + std::to_string(k));
    return RT_OK;
}

void* rt_stream(void) { return S().stream; }

int rt_protect(const void* ptr, size_t bytes) {
    RT_GUARD;
    if (!ptr) return fail(RT_ERR_NULL_POINTER, "rt_protect: NULL");
    S().protect.push_back({reinterpret_cast<uintptr_t>(ptr), bytes});
    // plans built without this range may have folded a writer of it away
    const uintptr_t lo = reinterpret_cast<uintptr_t>(ptr);
    if (S().initialized) drop_plans_touching(lo, lo + bytes, false);
    return RT_OK;
}

int rt_unprotect_all(void) {
    RT_GUARD;
    S().protect.clear();
    if (S().initialized) {
        cudaStreamSynchronize(S().stream);
        clear_plans();
    }
    return RT_OK;
}

int rt_fusion_report(const OpNode* nodes, int n, int* skipped) {
    if (n < 0 || (n > 0 && !nodes)) return -RT_ERR_ARGUMENT;
    std::vector<OpNode> v(nodes, nodes + n);
    std::vector<PlanItem> items = plan_fusions(v, S().protect);
    int count = 0;
    for (int i = 0; i < n; i++) {
        const PlanItem& it = items[i];
        int f = it.skip ? 1
                : it.views ? 2
                : it.rope ? 5
                : it.gated ? 6
                : it.norm_planes_off >= 0 ? 8
                : it.epi_gate ? 7
                : (it.epi_act || it.epi_out || it.carry_off >= 0 || it.epi_bias_off >= 0) ? 3
                : it.presplit_off >= 0 ? 4
                                        : 0;
        if (skipped) skipped[i] = f;
        count += items[i].skip;
    }
    return count;
}

int rt_check_wait_timeout(unsigned long long limit_ns) {
    RT_GUARD;
    RT_NEED_INIT;
    if (limit_ns == 0 || limit_ns > 1000000000ull) return fail(RT_ERR_ARGUMENT, "limit_ns must be in (0, 1 s]");
    cudaStream_t st = S().stream;
    unsatisfied_wait_kernel<<<1, 32, 0, st>>>((uint64_t)limit_ns, kernel_error_flag());
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, std::string("wait probe: ") + cudaGetErrorString(e));
    if (int k = take_kernel_error())
        return fail(RT_ERR_KERNEL_TIMEOUT, "a kernel abandoned a bounded wait, code " + std::to_string(k));
    return RT_OK;
}

int rt_last_error(void) { return S().last_error; }
const char* rt_last_error_message(void) { return S().last_msg.c_str(); }
void rt_clear_error(void) {
    S().last_error = RT_OK;
    S().last_msg.clear();
}

}  // extern "C"
