// k_attention.cu -- fused attention (ATTENTION, op 1002).
//
// Reference semantics (csrc/executor.c:371-397; csrc/ops/attn.c):
//   extras [seq_len, head_dim, causal, has_mask, group_size]
//   inputs [Q, K, V, (mask,) scratch]; Q/O [BH, S, D], K/V [BH/group, S, D]
//   scores = (Q K^T) * (1/sqrtf(D)); + mask[bh] (additive, [S,S]) or causal
//   (key > query -> -inf); row softmax; O = P V.  GQA: kv head = bh / group.
//   The reference picks a standard (S <= 256 or masked) or a flash
//   (BR=128/BC=256 online softmax, attn.c:121-236) kernel; both compute the
//   same function, so one kernel serves both here and the planned scratch
//   buffer is not needed.
//
// This file holds the CUDA-core flash kernel (exact fp32 FMA): one CTA per
// (64 queries, batch-head), 8 warps x 8 query rows, key/value tiles of 64
// staged in shared memory, online softmax in registers (running max initial
// value -FLT_MAX as the reference), causal tiles beyond the diagonal skipped.
#include <float.h>

#include "rt_internal.h"

namespace rt {
namespace {

constexpr int AQ = 64;    // queries per CTA
constexpr int AK = 64;    // keys per tile
constexpr int AW = 8;     // warps
constexpr int AR = 8;     // query rows per warp

struct AttnParams {
    const float* q;
    const float* k;
    const float* v;
    const float* mask;   // [BH, S, S] or null
    float* o;
    int64_t S;
    int D;
    int group;
    int causal;
    float scale;
};

template <int DP>
__global__ void __launch_bounds__(AW * 32) attn_simt_kernel(AttnParams p) {
    extern __shared__ float4 smem4[];
    // layout: Qs [AQ][DP] | Ks4 [DP/4][AK] float4 | Vs [AK][DP] | Ps [AW][AR][AK]
    float* Qs = reinterpret_cast<float*>(smem4);
    float4* Ks4 = reinterpret_cast<float4*>(Qs + AQ * DP);
    float* Vs = reinterpret_cast<float*>(Ks4 + (DP / 4) * AK);
    float* Ps = Vs + AK * DP;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bh = blockIdx.y;
    const int64_t q0 = (int64_t)blockIdx.x * AQ;
    const int64_t S = p.S;
    const int D = p.D;
    const float* Qb = p.q + bh * S * D;
    const float* Kb = p.k + (bh / p.group) * S * D;
    const float* Vb = p.v + (bh / p.group) * S * D;
    const float* Mb = p.mask ? p.mask + bh * S * S : nullptr;

    // stage Q (zero padded in rows and dims)
    for (int i = threadIdx.x; i < AQ * DP; i += AW * 32) {
        int r = i / DP, d = i % DP;
        int64_t gq = q0 + r;
        Qs[i] = (gq < S && d < D) ? Qb[gq * D + d] : 0.0f;
    }

    float m[AR], l[AR], acc[AR][(DP + 31) / 32];
#pragma unroll
    for (int r = 0; r < AR; r++) {
        m[r] = -FLT_MAX;
        l[r] = 0.0f;
#pragma unroll
        for (int c = 0; c < (DP + 31) / 32; c++) acc[r][c] = 0.0f;
    }

    int64_t kv_end = S;
    if (p.causal) {
        int64_t last_q = q0 + AQ - 1 < S - 1 ? q0 + AQ - 1 : S - 1;
        kv_end = last_q + 1;
    }
    float* Pw = Ps + warp * AR * AK;
    for (int64_t k0 = 0; k0 < kv_end; k0 += AK) {
        __syncthreads();  // previous tile fully consumed
        for (int i = threadIdx.x; i < AK * DP; i += AW * 32) {
            int j = i / DP, d = i % DP;
            int64_t gk = k0 + j;
            bool ok = gk < S && d < D;
            float kv = ok ? Kb[gk * D + d] : 0.0f;
            reinterpret_cast<float*>(&Ks4[(d >> 2) * AK + j])[d & 3] = kv;
            Vs[j * DP + d] = ok ? Vb[gk * D + d] : 0.0f;
        }
        __syncthreads();

        // scores for keys (lane, lane+32) and the warp's 8 rows
        float s[AR][2];
#pragma unroll
        for (int r = 0; r < AR; r++) s[r][0] = s[r][1] = 0.0f;
#pragma unroll 4
        for (int d4 = 0; d4 < DP / 4; d4++) {
            float4 ka = Ks4[d4 * AK + lane];
            float4 kb = Ks4[d4 * AK + lane + 32];
#pragma unroll
            for (int r = 0; r < AR; r++) {
                float4 qv = *reinterpret_cast<const float4*>(&Qs[(warp * AR + r) * DP + d4 * 4]);
                s[r][0] = fmaf(qv.x, ka.x, s[r][0]);
                s[r][0] = fmaf(qv.y, ka.y, s[r][0]);
                s[r][0] = fmaf(qv.z, ka.z, s[r][0]);
                s[r][0] = fmaf(qv.w, ka.w, s[r][0]);
                s[r][1] = fmaf(qv.x, kb.x, s[r][1]);
                s[r][1] = fmaf(qv.y, kb.y, s[r][1]);
                s[r][1] = fmaf(qv.z, kb.z, s[r][1]);
                s[r][1] = fmaf(qv.w, kb.w, s[r][1]);
            }
        }
#pragma unroll
        for (int r = 0; r < AR; r++) {
            int64_t gq = q0 + warp * AR + r;
            float t[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                int64_t gk = k0 + lane + 32 * h;
                float val = s[r][h] * p.scale;
                if (gk >= S) val = -INFINITY;
                else if (Mb) val += gq < S ? Mb[gq * S + gk] : 0.0f;   // mask wins (attn.c:40-48)
                else if (p.causal && gk > gq) val = -INFINITY;
                t[h] = val;
            }
            float mt = fmaxf(t[0], t[1]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            float mn = m[r] > mt ? m[r] : mt;
            float corr = expf(m[r] - mn);
            float p0 = expf(t[0] - mn), p1 = expf(t[1] - mn);
            float ps = p0 + p1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l[r] = l[r] * corr + ps;
            m[r] = mn;
#pragma unroll
            for (int c = 0; c < (DP + 31) / 32; c++) acc[r][c] *= corr;
            Pw[r * AK + lane] = p0;
            Pw[r * AK + lane + 32] = p1;
        }
        __syncwarp();
#pragma unroll 2
        for (int j4 = 0; j4 < AK / 4; j4++) {
            float4 pr[AR];
#pragma unroll
            for (int r = 0; r < AR; r++) pr[r] = *reinterpret_cast<const float4*>(&Pw[r * AK + j4 * 4]);
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                int j = j4 * 4 + jj;
#pragma unroll
                for (int c = 0; c < (DP + 31) / 32; c++) {
                    int d = lane + 32 * c;
                    float vv = d < DP ? Vs[j * DP + d] : 0.0f;
#pragma unroll
                    for (int r = 0; r < AR; r++) {
                        float pv = jj == 0 ? pr[r].x : jj == 1 ? pr[r].y : jj == 2 ? pr[r].z : pr[r].w;
                        acc[r][c] = fmaf(pv, vv, acc[r][c]);
                    }
                }
            }
        }
        __syncwarp();
    }
#pragma unroll
    for (int r = 0; r < AR; r++) {
        int64_t gq = q0 + warp * AR + r;
        if (gq >= S) continue;
        float inv = 1.0f / l[r];
#pragma unroll
        for (int c = 0; c < (DP + 31) / 32; c++) {
            int d = lane + 32 * c;
            if (d < D) p.o[(bh * S + gq) * D + d] = acc[r][c] * inv;
        }
    }
}

template <int DP>
Status launch_simt(const AttnParams& p, int64_t BH, cudaStream_t st) {
    size_t smem = sizeof(float) * ((size_t)AQ * DP + (size_t)DP * AK + (size_t)AK * DP + AW * AR * AK);
    static bool configured = false;
    if (!configured) {
        RT_CUDA_CHECK(cudaFuncSetAttribute(attn_simt_kernel<DP>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = true;
    }
    dim3 grid((unsigned)((p.S + AQ - 1) / AQ), (unsigned)BH);
    attn_simt_kernel<DP><<<grid, AW * 32, smem, st>>>(p);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

}  // namespace

bool attention_tc_applicable(int64_t S, int D, bool has_mask, int64_t BH);
size_t attention_tc_workspace(int64_t BHkv, int64_t S, int D);
Status attention_tc_prepare();
Status launch_attention_tc(const AttnViews& vw, int64_t BH, int64_t S, int D, int group, int causal,
                           Workspace ws, cudaStream_t st, int* launches);

namespace {

Status decode_attention(const OpNode& n, AttnParams* out, int64_t* BH_out, bool* has_mask_out) {
    AttnParams p{};
    p.S = n.extra[0];
    p.D = n.extra[1];
    p.causal = n.extra[2];
    int has_mask = n.extra[3];
    p.group = n.extra[4] > 0 ? n.extra[4] : 1;
    int64_t BH = 1;
    for (int i = 0; i < n.n_dims - 2; i++) BH *= n.out_shape[i];
    if (n.n_dims < 2 || p.S <= 0 || p.D <= 0 || n.out_shape[n.n_dims - 2] != p.S ||
        n.out_shape[n.n_dims - 1] != p.D)
        return Status::err(RT_ERR_BAD_NODE, "attention: shape/extras mismatch");
    if (BH % p.group) return Status::err(RT_ERR_BAD_NODE, "attention: heads not divisible by group");
    if (BH > 65535) return Status::err(RT_ERR_UNSUPPORTED, "attention: > 65535 batch-heads");
    p.q = (const float*)n.inputs[0];
    p.k = (const float*)n.inputs[1];
    p.v = (const float*)n.inputs[2];
    p.mask = has_mask ? (const float*)n.inputs[3] : nullptr;
    p.o = (float*)n.output;
    if (p.mask) p.causal = 0;   // the reference applies a custom mask instead of causal
    p.scale = 1.0f / sqrtf((float)p.D);
    *out = p;
    *BH_out = BH;
    *has_mask_out = has_mask != 0;
    return Status::ok();
}

bool use_tc(const AttnParams& p, int64_t BH, bool has_mask) {
    // K and V are read as 16-byte vectors by the pack pass, Q by a tensor map
    // and O by vector stores: all four must start on a 16-byte boundary
    // (planner offsets need not), else the CUDA-core kernel runs.
    return attention_tc_applicable(p.S, p.D, has_mask, BH) && aligned16(p.q) && aligned16(p.o) &&
           aligned16(p.k) && aligned16(p.v);
}

}  // namespace

size_t attention_workspace_bytes(const OpNode& n) {
    AttnParams p;
    int64_t BH;
    bool m;
    if (!decode_attention(n, &p, &BH, &m).good() || !use_tc(p, BH, m)) return 0;
    return attention_tc_workspace(BH / p.group, p.S, p.D);
}

Status prepare_attention(const OpNode& n) {
    AttnParams p;
    int64_t BH;
    bool m;
    Status s = decode_attention(n, &p, &BH, &m);
    if (!s.good() || !use_tc(p, BH, m)) return s;
    return attention_tc_prepare();
}

Status launch_attention(const OpNode& n, cudaStream_t st, Workspace ws, int* launches) {
    AttnParams p;
    int64_t BH;
    bool has_mask;
    Status s = decode_attention(n, &p, &BH, &has_mask);
    if (!s.good()) return s;
    if (use_tc(p, BH, has_mask) && ws.bytes >= attention_tc_workspace(BH / p.group, p.S, p.D))
    {
        AttnViews vw;
        attention_default_views(n, &vw);
        return launch_attention_tc(vw, BH, p.S, p.D, p.group, p.causal, ws, st, launches);
    }
    *launches += 1;
    if (p.D <= 16) return launch_simt<16>(p, BH, st);
    if (p.D <= 32) return launch_simt<32>(p, BH, st);
    if (p.D <= 64) return launch_simt<64>(p, BH, st);
    if (p.D <= 128) return launch_simt<128>(p, BH, st);
    return Status::err(RT_ERR_UNSUPPORTED, "attention: head_dim > 128");
}

bool attention_default_views(const OpNode& n, AttnViews* v) {
    AttnParams p;
    int64_t BH;
    bool m;
    if (!decode_attention(n, &p, &BH, &m).good()) return false;
    const int64_t H = n.n_dims >= 4 ? n.out_shape[n.n_dims - 3] : BH;
    const int64_t S = p.S, D = p.D, Hkv = H / p.group;
    v->q = p.q;
    v->k = p.k;
    v->v = p.v;
    v->o = p.o;
    v->q_sb = H * S * D; v->q_sh = S * D; v->q_ss = D;
    v->o_sb = H * S * D; v->o_sh = S * D; v->o_ss = D;
    v->k_sb = Hkv * S * D; v->k_sh = S * D; v->k_ss = D;
    v->v_sb = Hkv * S * D; v->v_sh = S * D; v->v_ss = D;
    v->H = (int)H;
    return H % p.group == 0;
}

bool attention_takes_views(const OpNode& n) {
    AttnParams p;
    int64_t BH;
    bool m;
    if (!decode_attention(n, &p, &BH, &m).good()) return false;
    return n.n_dims >= 4 && use_tc(p, BH, m);
}

Status launch_attention_views(const OpNode& n, const AttnViews& vw, cudaStream_t st, Workspace ws, int* launches) {
    AttnParams p;
    int64_t BH;
    bool m;
    Status s = decode_attention(n, &p, &BH, &m);
    if (!s.good()) return s;
    if (!use_tc(p, BH, m)) return Status::err(RT_ERR_ARGUMENT, "attention: strided views need the tensor-core path");
    return launch_attention_tc(vw, BH, p.S, p.D, p.group, p.causal, ws, st, launches);
}

}  // namespace rt
