/*
 * b200exec.h -- C ABI of libb200exec.so, the B200 (sm_100a) backend for the
 * compiled executor of lets-build-a-runtime.
 *
 * The reference runs a planned graph with ONE call,
 *     void execute(OpNode* nodes, int n_nodes)          (csrc/executor.c:458)
 * bound from Python by ctypes (runtime/executor/common.py:148-163) over an
 * OpNode array built by CompiledExecutor.compile (runtime/executor/
 * compiled.py:34-70).  This library exports the same symbol with the same
 * struct, op codes and extra[] encodings.  What changes is where memory
 * lives: every pointer in the node array is a DEVICE address (arena,
 * weights and input staging allocated through rt_alloc below, or any other
 * device allocation of the current device), and execution happens on the
 * GPU.  The reference's C side never allocates (the caller owns arena,
 * weights, inputs); here the caller still owns them, but allocates them
 * through this library so that they are device memory.
 *
 * Error convention: the reference aborts on an unknown op
 * (csrc/executor.c:461-464) and checks nothing else.  This library never
 * aborts: every entry point that can fail returns an RT_* status and
 * records it for rt_last_error()/rt_last_error_message(); `execute`, which
 * must keep its void signature for ctypes compatibility, only records it.
 *
 * Threading: like the reference, one call at a time per process; all work
 * runs on one library-owned CUDA stream of the device given to rt_init.
 */
#ifndef B200EXEC_H
#define B200EXEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RT_MAX_INPUTS 12   /* csrc/runtime.h:57  MAX_INPUTS */
#define RT_MAX_DIMS 24     /* csrc/runtime.h:58  MAX_DIMS   */

/* Byte-identical to OpNode (csrc/runtime.h:60-69) and COpNode
 * (runtime/executor/common.py:125-141). */
typedef struct OpNode {
    int op;
    int n_inputs;
    void* inputs[RT_MAX_INPUTS];
    void* output;
    int out_shape[RT_MAX_DIMS];
    int n_dims;
    int elem_size;
    int extra[RT_MAX_DIMS];
} OpNode;

/* Op codes: enum OpType of csrc/runtime.h:11-55 (= runtime/ir.py:36-78). */
enum RtOpType {
    RT_OP_RELU = 100, RT_OP_EXP = 101, RT_OP_TANH = 102, RT_OP_POW = 103,
    RT_OP_GELU = 104, RT_OP_RSQRT = 105, RT_OP_SILU = 106, RT_OP_NEG = 107,
    RT_OP_COS = 108, RT_OP_SIN = 109,
    RT_OP_ADD = 200, RT_OP_SUB = 201, RT_OP_MUL = 202, RT_OP_DIV = 203,
    RT_OP_MAX = 300, RT_OP_SUM = 301, RT_OP_SOFTMAX = 302,
    RT_OP_MATMUL = 400,
    RT_OP_RESHAPE = 500, RT_OP_TRANSPOSE = 501, RT_OP_PERMUTE = 502,
    RT_OP_SLICE = 503, RT_OP_EMBEDDING = 504, RT_OP_CAT = 505,
    RT_OP_LAYERNORM = 600, RT_OP_RMSNORM = 601,
    RT_OP_MATMUL_ADD = 1000, RT_OP_FUSED_BIAS_RELU = 1001,
    RT_OP_ATTENTION = 1002, RT_OP_GATED_ACT = 1003
};

/* Status codes. */
enum RtStatus {
    RT_OK = 0,
    RT_ERR_NOT_INITIALIZED = 1,
    RT_ERR_BAD_OP = 2,          /* op code with no dispatch entry (incl. PERMUTE) */
    RT_ERR_BAD_NODE = 3,        /* malformed node: dims, n_inputs, extras */
    RT_ERR_NULL_POINTER = 4,
    RT_ERR_HOST_POINTER = 5,    /* pointer is not device memory of this device */
    RT_ERR_OUT_OF_RANGE = 6,    /* buffer extent leaves its allocation */
    RT_ERR_UNSUPPORTED = 7,     /* valid reference node this build cannot run */
    RT_ERR_CUDA = 8,            /* a CUDA runtime/driver call failed */
    RT_ERR_OOM = 9,
    RT_ERR_ARGUMENT = 10,
    RT_ERR_KERNEL_TIMEOUT = 11  /* a kernel gave up a bounded wait (it recorded a code and returned) */
};

/* Execution flags for rt_execute. */
#define RT_FLAG_EAGER 1   /* launch node by node, no CUDA graph */
#define RT_FLAG_ASYNC 2   /* do not synchronise before returning */

/* One host<->device copy for rt_execute_io. */
typedef struct RtCopy {
    void* dst;
    const void* src;
    size_t bytes;
} RtCopy;

/* ---- lifecycle ---------------------------------------------------------- */
/* Select the device, create the stream.  Idempotent for the same device. */
int rt_init(int device);
/* Free every allocation, cached plan and graph; the library may be re-inited. */
int rt_destroy(void);
const char* rt_version(void);

/* ---- memory (replaces the host arena of runtime/executor/common.py:83-87
 *      and the numpy weight buffers) ------------------------------------- */
void* rt_alloc(size_t bytes);             /* device, 256-B aligned, zeroed; NULL on failure */
int rt_free(void* dev);
void* rt_host_alloc(size_t bytes);        /* pinned host memory; NULL on failure */
int rt_host_free(void* host);
int rt_upload(void* dst_dev, const void* src_host, size_t bytes);
int rt_download(void* dst_host, const void* src_dev, size_t bytes);
/* Declare [dev, dev+bytes) immutable (graph constants).  The library may
 * then cache derived forms of it (split matrix operands) across calls.
 * Writing to the range afterwards requires rt_reset_plans(). */
int rt_mark_constant(void* dev, size_t bytes);

/* ---- execution ---------------------------------------------------------- */
/* Drop-in for csrc/executor.c:458.  First call with a given node array
 * validates it, prepares derived operands and captures the launch sequence
 * into a CUDA graph; later calls with identical contents replay the graph.
 * Returns after the GPU finished.  Errors: see rt_last_error(). */
void execute(OpNode* nodes, int n_nodes);
/* Same, returning the status; flags = RT_FLAG_*. */
int rt_execute(const OpNode* nodes, int n_nodes, int flags);
/* End to end: n_in host->device copies, the graph of `nodes`, n_out
 * device->host copies, all on the library stream, then one synchronise. */
int rt_execute_io(const OpNode* nodes, int n_nodes,
                  const RtCopy* h2d, int n_in, const RtCopy* d2h, int n_out);
/* One batch as independent chunks (no counterpart in the reference): chunk c
 * runs its own node array -- the graph planned for that chunk's rows, with
 * its own arena -- between its host-to-device and device-to-host copies, on
 * its own stream, so one chunk's copies overlap another chunk's kernels.
 * Only valid when the chunks share no intermediate memory and the model
 * treats batch rows independently.  Synchronous, like rt_execute_io. */
typedef struct RtChunk {
    const OpNode* nodes;
    int n_nodes;
    const RtCopy* h2d;
    int n_in;
    const RtCopy* d2h;
    int n_out;
} RtChunk;
int rt_execute_chunks(const RtChunk* chunks, int n_chunks);
/* Validate and prepare (capture) without running. */
int rt_prepare(const OpNode* nodes, int n_nodes);
/* Kernel launches one execute of this node array issues (after prepare). */
int rt_kernel_launches(const OpNode* nodes, int n_nodes);
/* Per-node device time: runs the array `reps` times eagerly with CUDA
 * events around each node on the library stream; ms_per_node[i] receives
 * the mean over reps.  This fills RunProfile.op_timings
 * (runtime/executor/common.py:24-63) for the compiled path. */
int rt_profile(const OpNode* nodes, int n_nodes, int reps, float* ms_per_node);
/* Drop cached plans, graphs and derived constant forms. */
int rt_reset_plans(void);
/* Drop the cached plan (captured graph, scratch) of this node array only --
 * what an executor releases when it is closed while others keep theirs.
 * rt_plan_count() = plans currently cached (one per distinct node array). */
int rt_release(const OpNode* nodes, int n_nodes);
int rt_plan_count(void);
int rt_synchronize(void);
/* The library stream (a cudaStream_t), for callers that order work on it. */
void* rt_stream(void);
/* Declare [ptr, ptr+bytes) a graph output: plan-time layout fusion never
 * folds away a node that writes into it.  The output of the last node of an
 * array is always treated as a graph output; callers whose graphs return
 * more than that register the other outputs here before the first execute
 * (no counterpart in the reference, whose C side computes every node).
 * A registration lasts until rt_unprotect_all or until the rt_alloc memory
 * holding `ptr` is released with rt_free. */
int rt_protect(const void* ptr, size_t bytes);
int rt_unprotect_all(void);
/* Plan-time fusion, as execute would apply it to this node array:
 * flags[i] = 1 when node i is folded into another node and not launched (a
 * SLICE / TRANSPOSE around attention, a GELU after a GEMM), 2 for an
 * attention node launched with strided operands, 3 for a GEMM that applies a
 * folded activation and/or writes the split A operand of a later GEMM in its
 * epilogue (its A may arrive split as well), 4 for a GEMM whose only fusion is
 * that its A operand arrives split (no split pass),
 * 5 for the last node of a folded RMSNorm + rotary-embedding chain (it runs
 * the fused kernel), 6 for a gated activation reading its inputs through
 * strided views of the tensor its folded SLICEs took them from, 8 for a
 * LAYERNORM / RMSNORM writing the split A operand of the GEMM reading it
 * (that GEMM: 4), 7 for a GEMM whose epilogue applies a folded gated
 * activation (SLICE, SLICE, GATED_ACT of its output: 1 each), 0 otherwise.  Returns the number of folded nodes.  Host only: needs no
 * device and no rt_init.  RT_FUSE=0 turns all fusion off. */
int rt_fusion_report(const OpNode* nodes, int n_nodes, int* flags);

/* ---- allocation-free GEMM ------------------------------------------------ */
/* No counterpart in the reference.  C[M,N] = alpha * A[M,K] . op(B) + bias
 * (bias may be NULL; op(B) = B^T when trans_b, B stored [N,K], else B [K,N]),
 * computed by the same split-operand tensor-core kernel as MATMUL/MATMUL_ADD
 * (tf32 hi.hi product plus bf16 cross terms), for callers that may not
 * allocate device memory: plugins whose host application owns every device
 * allocation through its own pool, and processes that must not grow their
 * device footprint after start-up.  It allocates nothing and needs no
 * rt_init: it runs on the current device and `stream` (a cudaStream_t;
 * NULL = legacy default stream).  It is synchronous: it waits for `stream`
 * and returns after C is written, so it is a host-thread call, not one for a
 * CUDA host callback (which may not call CUDA).  Scratch: a fixed
 * RT_NOALLOC_SCRATCH_BYTES device array inside the library (held by every
 * GPU that loads it), so 8*(M*K + N*K) bytes must fit: larger problems
 * return RT_ERR_OUT_OF_RANGE; K % 4 != 0 returns RT_ERR_UNSUPPORTED.  A C
 * or bias off a 16-byte boundary is written / read with scalar accesses.
 * The first call on each device performs a one-time set-up (symbol address,
 * kernel attribute): make it before any stream capture.  All calls share
 * the scratch: calls that overlap on the GPU race.  Launches are checked
 * with cudaGetLastError, so an error left pending by earlier CUDA work of
 * the caller is reported as this call's RT_ERR_CUDA.  Returns an RT_*
 * status (not recorded in rt_last_error). */
#define RT_NOALLOC_SCRATCH_BYTES (32u << 20)
int rt_matmul_noalloc(const float* a, const float* b, const float* bias, float* c,
                      int M, int N, int K, int trans_b, float alpha, void* stream);

/* ---- errors ------------------------------------------------------------- */
/* No counterpart in the reference (which never waits on the device).  Runs
 * one kernel whose single bounded mbarrier wait is never satisfied, with a
 * limit of limit_ns (0 < limit_ns <= 1 s), through the same bounded-wait code
 * as the tensor-core kernels.  Returns RT_ERR_KERNEL_TIMEOUT (and records
 * it) when the timeout path works: the kernel records a code, returns, and
 * the context stays usable.  No fault, trap or hang is involved. */
int rt_check_wait_timeout(unsigned long long limit_ns);

int rt_last_error(void);                  /* status of the last failing call; 0 if none */
const char* rt_last_error_message(void);
void rt_clear_error(void);

#ifdef __cplusplus
}
#endif

#endif /* B200EXEC_H */
