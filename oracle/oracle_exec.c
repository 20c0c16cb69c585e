/*
 * oracle_exec.c -- TEST INFRASTRUCTURE ONLY: a plain-C restatement of the
 * reference compiled executor (kaselby/lets-build-a-runtime, csrc/), used by
 * tests/ and by bench.py's CPU-baseline leg as the checker.  Nothing in the
 * product links, loads or calls this file.
 *
 * It walks the same OpNode array (csrc/runtime.h:60-69) as the reference's
 * `execute` (csrc/executor.c:458-467) and restates each kernel's arithmetic
 * as the reference's non-Apple branch performs it, in this file's own code:
 * single-precision accumulation, the same loop orders for reductions, the
 * same flash-attention tiling (BR=128, BC=256) and online-softmax update.
 * The one deliberate difference: matrix products use a plain triple loop
 * (k innermost, fp32 accumulate) where the reference calls cblas_sgemm, so
 * results agree with the reference to BLAS summation-order rounding, not
 * bit for bit.
 *
 * Entry point: int oracle_execute(OpNode* nodes, int n) -> 0 on success,
 * else the 1-based index of the first node it could not run.
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MAX_INPUTS 12
#define MAX_DIMS 24

typedef struct {
    int op;
    int n_inputs;
    void* inputs[MAX_INPUTS];
    void* output;
    int out_shape[MAX_DIMS];
    int n_dims;
    int elem_size;
    int extra[MAX_DIMS];
} OpNode;

static long numel(const OpNode* n) {
    long t = 1;
    for (int i = 0; i < n->n_dims; i++) t *= n->out_shape[i];
    return t;
}
static long rows_of(const OpNode* n) {
    long t = 1;
    for (int i = 0; i < n->n_dims - 1; i++) t *= n->out_shape[i];
    return t;
}
static float fbits(int v) { float f; memcpy(&f, &v, 4); return f; }

/* C = alpha * A[M,K] . op(B) + beta * C ; op(B) = B^T when tb (B is [N,K]). */
static void gemm(const float* A, const float* B, float* C, long M, long N, long K,
                 int tb, float alpha, float beta) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < M; i++) {
        const float* a = A + i * K;
        for (long j = 0; j < N; j++) {
            float acc = 0.0f;
            if (tb) {
                const float* b = B + j * K;
                for (long k = 0; k < K; k++) acc += a[k] * b[k];
            } else {
                for (long k = 0; k < K; k++) acc += a[k] * B[k * N + j];
            }
            float prev = beta != 0.0f ? beta * C[i * N + j] : 0.0f;
            C[i * N + j] = alpha * acc + prev;
        }
    }
}

/* ---- matmul family: csrc/executor.c:197-224 (MATMUL), :312-346 (MATMUL_ADD),
 *      csrc/ops/matmul.c:19-40 (batched sgemm), :64-79 (M==1 sgemv) ---- */
static void op_matmul(OpNode* n, int with_bias) {
    long N = n->out_shape[n->n_dims - 1];
    long K = n->extra[0];
    int tb = n->extra[1], b2d = n->extra[2];
    float alpha = (!with_bias && n->extra[3]) ? fbits(n->extra[3]) : 1.0f;
    long M, batches = 1;
    if (b2d) {
        M = rows_of(n);
    } else {
        M = n->out_shape[n->n_dims - 2];
        for (int i = 0; i < n->n_dims - 2; i++) batches *= n->out_shape[i];
    }
    float* out = n->output;
    const float* A = n->inputs[0];
    const float* B = n->inputs[1];
    float beta = 0.0f;
    if (with_bias) {
        const float* bias = n->inputs[2];
        for (long r = 0; r < M * batches; r++)
            for (long c = 0; c < N; c++) out[r * N + c] = bias[c];
        beta = 1.0f;
    }
    for (long b = 0; b < batches; b++)
        gemm(A + b * M * K, B + b * N * K, out + b * M * N, M, N, K, tb, alpha, beta);
}

/* ---- row softmax: csrc/ops/reduce.c:53-98 (non-Apple branch) ---- */
static void softmax_rows(const float* x, float* y, long rows, long cols) {
    for (long i = 0; i < rows; i++) {
        const float* r = x + i * cols;
        float* o = y + i * cols;
        float mx = r[0];
        for (long j = 1; j < cols; j++) if (r[j] > mx) mx = r[j];
        float s = 0.0f;
        for (long j = 0; j < cols; j++) { o[j] = expf(r[j] - mx); s += o[j]; }
        for (long j = 0; j < cols; j++) o[j] /= s;
    }
}

/* ---- attention: csrc/executor.c:371-397 dispatch; standard path
 *      csrc/ops/attn.c:26-80; flash path csrc/ops/attn.c:106-253 ---- */
#define FL_BR 128
#define FL_BC 256
static void attn_standard(const float* Q, const float* K, const float* V, float* O,
                          const float* mask, long BH, long S, long D, int causal, int G) {
    float scale = 1.0f / sqrtf((float)D);
#pragma omp parallel for schedule(static)
    for (long bh = 0; bh < BH; bh++) {
        long kv = bh / G;
        float* P = malloc(sizeof(float) * S * S);
        gemm(Q + bh * S * D, K + kv * S * D, P, S, S, D, 1, scale, 0.0f);
        if (mask) {
            const float* m = mask + bh * S * S;
            for (long i = 0; i < S * S; i++) P[i] += m[i];
        } else if (causal) {
            for (long i = 0; i < S; i++)
                for (long j = i + 1; j < S; j++) P[i * S + j] = -INFINITY;
        }
        softmax_rows(P, P, S, S);
        gemm(P, V + kv * S * D, O + bh * S * D, S, D, S, 0, 1.0f, 0.0f);
        free(P);
    }
}

static void attn_flash(const float* Q, const float* K, const float* V, float* O,
                       long BH, long S, long D, int causal, int G) {
    float scale = 1.0f / sqrtf((float)D);
#pragma omp parallel for schedule(dynamic)
    for (long bh = 0; bh < BH; bh++) {
        long kvh = bh / G;
        const float* q = Q + bh * S * D;
        const float* k = K + kvh * S * D;
        const float* v = V + kvh * S * D;
        float* o = O + bh * S * D;
        float* T = malloc(sizeof(float) * FL_BR * FL_BC);
        float m[FL_BR], l[FL_BR];
        for (long q0 = 0; q0 < S; q0 += FL_BR) {
            long br = q0 + FL_BR <= S ? FL_BR : S - q0;
            for (long r = 0; r < br; r++) { m[r] = -FLT_MAX; l[r] = 0.0f; }
            memset(o + q0 * D, 0, sizeof(float) * br * D);
            for (long k0 = 0; k0 < S; k0 += FL_BC) {
                long bc = k0 + FL_BC <= S ? FL_BC : S - k0;
                if (causal && k0 > q0 + br - 1) break;
                gemm(q + q0 * D, k + k0 * D, T, br, bc, D, 1, scale, 0.0f);
                if (causal && k0 + bc > q0) {
                    for (long r = 0; r < br; r++) {
                        long last = q0 + r - k0;
                        for (long c = last < 0 ? 0 : last + 1; c < bc; c++) T[r * bc + c] = -INFINITY;
                    }
                }
                for (long r = 0; r < br; r++) {
                    float* t = T + r * bc;
                    float* orow = o + (q0 + r) * D;
                    float mt = t[0];
                    for (long c = 1; c < bc; c++) if (t[c] > mt) mt = t[c];
                    float mn = m[r] > mt ? m[r] : mt;
                    float corr = expf(m[r] - mn);
                    l[r] *= corr;
                    for (long d = 0; d < D; d++) orow[d] *= corr;
                    float ls = 0.0f;
                    for (long c = 0; c < bc; c++) { float p = expf(t[c] - mn); t[c] = p; ls += p; }
                    l[r] += ls;
                    m[r] = mn;
                }
                gemm(T, v + k0 * D, o + q0 * D, br, D, bc, 0, 1.0f, 1.0f);
            }
            for (long r = 0; r < br; r++) {
                float inv = 1.0f / l[r];
                for (long d = 0; d < D; d++) o[(q0 + r) * D + d] *= inv;
            }
        }
        free(T);
    }
}

static void op_attention(OpNode* n) {
    long S = n->extra[0], D = n->extra[1];
    int causal = n->extra[2], has_mask = n->extra[3];
    int G = n->extra[4] > 0 ? n->extra[4] : 1;
    long BH = 1;
    for (int i = 0; i < n->n_dims - 2; i++) BH *= n->out_shape[i];
    const float* mask = has_mask ? n->inputs[3] : NULL;
    if (S > 256 && !has_mask)
        attn_flash(n->inputs[0], n->inputs[1], n->inputs[2], n->output, BH, S, D, causal, G);
    else
        attn_standard(n->inputs[0], n->inputs[1], n->inputs[2], n->output, mask, BH, S, D, causal, G);
}

/* ---- norms: csrc/ops/norm.c:48-63 (LayerNorm, two-pass, centred variance),
 *      csrc/ops/norm.c:100-107 (RMSNorm) ---- */
static void op_layernorm(OpNode* n) {
    long C = n->out_shape[n->n_dims - 1], R = rows_of(n);
    const float *x = n->inputs[0], *g = n->inputs[1], *b = n->inputs[2];
    float* y = n->output;
    float eps = fbits(n->extra[0]);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < R; i++) {
        const float* xr = x + i * C;
        float* yr = y + i * C;
        float s = 0.0f;
        for (long j = 0; j < C; j++) s += xr[j];
        float mean = s / C;
        float v = 0.0f;
        for (long j = 0; j < C; j++) { float d = xr[j] - mean; yr[j] = d; v += d * d; }
        float inv = 1.0f / sqrtf(v / C + eps);
        for (long j = 0; j < C; j++) yr[j] = yr[j] * inv * g[j] + b[j];
    }
}

static void op_rmsnorm(OpNode* n) {
    long C = n->out_shape[n->n_dims - 1], R = rows_of(n);
    const float *x = n->inputs[0], *w = n->inputs[1];
    float* y = n->output;
    float eps = fbits(n->extra[0]);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < R; i++) {
        const float* xr = x + i * C;
        float ss = 0.0f;
        for (long j = 0; j < C; j++) ss += xr[j] * xr[j];
        float sc = 1.0f / sqrtf(ss / C + eps);
        for (long j = 0; j < C; j++) y[i * C + j] = xr[j] * sc * w[j];
    }
}

/* ---- elementwise: csrc/ops/elementwise.c ---- */
static float gelu_tanh(float x) {   /* elementwise.c:186-189 */
    return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}

static void op_unary(OpNode* n) {
    long t = numel(n);
    const float* x = n->inputs[0];
    float* y = n->output;
    float p = fbits(n->extra[0]);
    for (long i = 0; i < t; i++) {
        float v = x[i];
        switch (n->op) {
            case 100: y[i] = v > 0.0f ? v : 0.0f; break;           /* :23-27 */
            case 101: y[i] = expf(v); break;                        /* :63-67 */
            case 102: y[i] = tanhf(v); break;                       /* :150-154 */
            case 103: y[i] = powf(v, p); break;                     /* :139-143 */
            case 104: y[i] = gelu_tanh(v); break;
            case 105: y[i] = 1.0f / sqrtf(v); break;                /* :196-198 */
            case 106: y[i] = v / (1.0f + expf(-v)); break;          /* :203-205 */
            case 107: y[i] = -v; break;                             /* :210-212 */
            case 108: y[i] = cosf(v); break;
            case 109: y[i] = sinf(v); break;
        }
    }
}

/* binop: 0 add, 1 sub, 2 mul, 3 div (csrc/ops/shape.c:46-51) */
static float binop(int op, float a, float b) {
    switch (op) {
        case 0: return a + b;
        case 1: return a - b;
        case 2: return a * b;
        default: return a / b;
    }
}

/* general broadcast with per-dimension strides: csrc/ops/shape.c:32-62 */
static void broadcast(const float* a, const float* b, float* y, const int* as,
                      const int* bs, const int* shape, int nd, int op) {
    long total = 1;
    for (int d = 0; d < nd; d++) total *= shape[d];
    for (long i = 0; i < total; i++) {
        long rem = i, ao = 0, bo = 0;
        for (int d = nd - 1; d >= 0; d--) {
            long c = rem % shape[d];
            rem /= shape[d];
            ao += c * as[d];
            bo += c * bs[d];
        }
        y[i] = binop(op, a[ao], b[bo]);
    }
}

/* csrc/executor.c:96-168: ADD modes 0 bias/1 same/2 scalar/3 broadcast;
 * SUB/MUL/DIV modes 0 same/1 scalar/2 broadcast */
static void op_binary(OpNode* n) {
    int kind = n->op - 200;
    int mode = n->extra[0];
    long t = numel(n);
    const float* a = n->inputs[0];
    const float* b = n->inputs[1];
    float* y = n->output;
    int same, scalar, bcast, bias = 0;
    if (kind == 0) {
        same = mode == 1; scalar = mode == 2; bcast = mode == 3; bias = mode == 0;
    } else {
        same = mode == 0; scalar = mode == 1; bcast = mode == 2;
    }
    if (scalar) {
        float s = fbits(n->extra[1]);
        for (long i = 0; i < t; i++) y[i] = binop(kind, a[i], s);
    } else if (same) {
        for (long i = 0; i < t; i++) y[i] = binop(kind, a[i], b[i]);
    } else if (bias) {
        long N = n->out_shape[n->n_dims - 1];
        for (long i = 0; i < t; i++) y[i] = a[i] + b[i % N];
    } else if (bcast) {
        int nd = n->extra[1];
        broadcast(a, b, y, &n->extra[2], &n->extra[2 + nd], &n->extra[2 + 2 * nd], nd, kind);
    }
}

/* csrc/ops/elementwise.c:96-136 (gated SiLU / tanh-GELU) */
static void op_gated(OpNode* n) {
    int has_bias = n->extra[0], act = n->extra[1];
    long N = n->out_shape[n->n_dims - 1], t = numel(n);
    const float* x = n->inputs[0];
    const float* up = has_bias ? n->inputs[2] : n->inputs[1];
    const float* bias = has_bias ? n->inputs[1] : NULL;
    float* y = n->output;
    for (long i = 0; i < t; i++) {
        float v = x[i] + (bias ? bias[i % N] : 0.0f);
        float g = act == 0 ? v / (1.0f + expf(-v)) : gelu_tanh(v);
        y[i] = g * up[i];
    }
}

/* csrc/ops/elementwise.c:81-90 */
static void op_bias_relu(OpNode* n) {
    long N = n->out_shape[n->n_dims - 1], t = numel(n);
    const float* a = n->inputs[0];
    const float* b = n->inputs[1];
    float* y = n->output;
    for (long i = 0; i < t; i++) { float v = a[i] + b[i % N]; y[i] = v > 0.0f ? v : 0.0f; }
}

/* ---- reductions: csrc/executor.c:172-190, csrc/ops/reduce.c:8-36 ---- */
static void op_reduce(OpNode* n) {
    int axis = n->extra[0];
    long A = n->extra[1], outer = 1, inner = 1;
    for (int i = 0; i < axis; i++) outer *= n->out_shape[i];
    for (int i = axis; i < n->n_dims; i++) inner *= n->out_shape[i];
    const float* x = n->inputs[0];
    float* y = n->output;
    for (long o = 0; o < outer; o++)
        for (long j = 0; j < inner; j++) {
            float acc = n->op == 300 ? -FLT_MAX : 0.0f;
            for (long a = 0; a < A; a++) {
                float v = x[(o * A + a) * inner + j];
                if (n->op == 300) { if (v > acc) acc = v; } else acc += v;
            }
            y[o * inner + j] = acc;
        }
}

/* ---- data movement: csrc/executor.c:228-282, csrc/ops/shape.c ---- */
static void op_transpose(OpNode* n) {
    int es = n->elem_size;
    const char* x = n->inputs[0];
    char* y = n->output;
    if (n->n_dims == 2) {   /* shape.c:8-13 */
        long R = n->extra[0], C = n->extra[1];
        for (long i = 0; i < R; i++)
            for (long j = 0; j < C; j++) memcpy(y + (j * R + i) * es, x + (i * C + j) * es, es);
        return;
    }
    long O = n->extra[0], A = n->extra[1], Mi = n->extra[2], B = n->extra[3], I = n->extra[4];
    for (long o = 0; o < O; o++)
        for (long b = 0; b < B; b++)
            for (long m = 0; m < Mi; m++)
                for (long a = 0; a < A; a++)
                    memcpy(y + ((((o * B + b) * Mi + m) * A + a) * I) * es,
                           x + ((((o * A + a) * Mi + m) * B + b) * I) * es, I * es);
}

static void op_slice(OpNode* n) {   /* shape.c:92-106 */
    long O = n->extra[0], Dm = n->extra[1], st = n->extra[2], L = n->extra[3], I = n->extra[4];
    int es = n->elem_size;
    const char* x = n->inputs[0];
    char* y = n->output;
    for (long o = 0; o < O; o++) memcpy(y + o * L * I * es, x + (o * Dm + st) * I * es, L * I * es);
}

static void op_cat(OpNode* n) {     /* shape.c:121-138 */
    int dim = n->extra[0], es = n->elem_size;
    long outer = 1, inner = 1, tot = 0;
    for (int i = 0; i < dim; i++) outer *= n->out_shape[i];
    for (int i = dim + 1; i < n->n_dims; i++) inner *= n->out_shape[i];
    for (int k = 0; k < n->n_inputs; k++) tot += n->extra[1 + k];
    char* y = n->output;
    for (long o = 0; o < outer; o++) {
        long dst = o * tot * inner;
        for (int k = 0; k < n->n_inputs; k++) {
            long ch = (long)n->extra[1 + k] * inner;
            memcpy(y + dst * es, (const char*)n->inputs[k] + o * ch * es, ch * es);
            dst += ch;
        }
    }
}

static void op_embedding(OpNode* n) {  /* shape.c:72-79 */
    long E = n->extra[0], S = rows_of(n);
    const int64_t* ids = n->inputs[0];
    const float* tab = n->inputs[1];
    float* y = n->output;
    for (long i = 0; i < S; i++) memcpy(y + i * E, tab + ids[i] * E, E * sizeof(float));
}

int oracle_execute(OpNode* nodes, int n_nodes) {
    for (int i = 0; i < n_nodes; i++) {
        OpNode* n = &nodes[i];
        switch (n->op) {
            case 100: case 101: case 102: case 103: case 104:
            case 105: case 106: case 107: case 108: case 109: op_unary(n); break;
            case 200: case 201: case 202: case 203: op_binary(n); break;
            case 300: case 301: op_reduce(n); break;
            case 302: softmax_rows(n->inputs[0], n->output, rows_of(n), n->out_shape[n->n_dims - 1]); break;
            case 400: op_matmul(n, 0); break;
            case 500:
                if (n->inputs[0] != n->output) memcpy(n->output, n->inputs[0], numel(n) * n->elem_size);
                break;
            case 501: op_transpose(n); break;
            case 503: op_slice(n); break;
            case 504: op_embedding(n); break;
            case 505: op_cat(n); break;
            case 600: op_layernorm(n); break;
            case 601: op_rmsnorm(n); break;
            case 1000: op_matmul(n, 1); break;
            case 1001: op_bias_relu(n); break;
            case 1002: op_attention(n); break;
            case 1003: op_gated(n); break;
            default: return i + 1;
        }
    }
    return 0;
}
