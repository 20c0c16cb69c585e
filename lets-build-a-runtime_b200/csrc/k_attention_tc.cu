// k_attention_tc.cu -- fused attention on the 5th-generation tensor cores.
//
// Same function as the reference's flash kernel (csrc/ops/attn.c:121-253):
// scores = (Q K^T) * 1/sqrtf(D), causal mask as -inf, online softmax with
// running max starting at -FLT_MAX, O = P V / l, GQA kv head = bh / group.
// Both products run as 3xTF32 on tcgen05 (hi.hi + hi.lo + lo.hi) so results
// stay at fp32 level; each P.V tile is accumulated in TMEM and folded into
// fp32 registers, like the GEMM's K chunks.
//
// One CTA = 128 queries of one (batch, head); 320 threads:
//   warp 0     TMA producer: per key tile (64 keys for D=64, 32 for D=128),
//              K (hi/lo, [keys][D]) and V^T (hi/lo, [D][keys]) in
//              128-byte-swizzled 32-float chunks, two slots each;
//   warp 1     allocates 512 TMEM columns and issues the MMAs from one
//              thread in the order S_0, S_1, PV_0, S_2, PV_1, ... so the next
//              score tile is computed while the softmax works on this one:
//              S = Q_hi.K_hi + Q_hi.K_lo (A from TMEM) + Q_lo.K_hi (A from
//              shared memory); O_tile = P_hi.V_hi + P_hi.V_lo + P_lo.V_hi;
//   warps 2-9  two threads per query row (half of the scores and half of
//              the output columns each; row maxima and sums exchanged through
//              shared memory behind bounded mbarrier waits): stage Q (hi to
//              TMEM, lo to shared memory), then per tile read S from TMEM,
//              mask, online softmax in log2 units (exp2f), write P hi/lo to
//              TMEM, fold the previous O tile into registers, rescaling only
//              when the running max grows.
// TMEM columns: Q_hi [0,D) | S x2 | P_hi | P_lo | O tile.
// K and V are split (and V transposed) into the node's workspace by a
// bandwidth-bound pre-pass.  All waits are bounded (see sm100_ptx.h).
#include <float.h>

#include "gemm.h"
#include "sm100_ptx.h"

namespace rt {

int* kernel_error_flag();

namespace {

constexpr int BQ = 128, SOFT_WARPS = 8, ATHREADS = 64 + 32 * SOFT_WARPS;
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr int ERR_A_PROD = 0x201, ERR_A_MMA = 0x202, ERR_A_SOFT = 0x203, ERR_A_DRAIN = 0x204;

template <int D>
struct AttnTcCfg {
    static constexpr int BKV = D == 128 ? 32 : 64;       // keys per tile
    static constexpr int QL_BYTES = D * BQ * 4;          // Q_lo, D/32 chunks of [128 rows][128 B]
    static constexpr int KH_BYTES = D * BKV * 4;         // one of K_hi / K_lo, one slot
    static constexpr int VH_BYTES = BKV * D * 4;         // one of V_hi / V_lo, one slot
    static constexpr int K_SLOT = 2 * KH_BYTES, V_SLOT = 2 * VH_BYTES;
    static constexpr int SMEM = QL_BYTES + 2 * K_SLOT + 2 * V_SLOT + 1024 + 256 + 6 * BQ * 4;
    // TMEM columns
    static constexpr uint32_t COL_S = D, COL_PH = D + 2 * BKV, COL_PL = D + 3 * BKV, COL_O = D + 4 * BKV;
    static_assert(2 * D + 4 * BKV <= 512, "TMEM budget");
};

struct AttnTcParams {
    CUtensorMap tk_hi, tk_lo;   // {D, S, BHkv}, box {32, BKV}
    CUtensorMap tv_hi, tv_lo;   // {S, D, BHkv}, box {32, D}
    const float* q;
    float* o;
    int S, group, causal, n_qblocks;
    float scale;
    int* err;
};

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Tile schedule (MMA issue order): S_0, S_1, PV_0, S_2, PV_1, ... so that
// S_{j+1} runs on the tensor cores while the softmax threads work on S_j.
template <int D>
__global__ void __launch_bounds__(ATHREADS, 1) attn_tc_kernel(const __grid_constant__ AttnTcParams p) {
    using C = AttnTcCfg<D>;
    constexpr int BKV = C::BKV;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* ql = smem;
    uint8_t* kbuf = ql + C::QL_BYTES;           // 2 slots: [hi | lo]
    uint8_t* vbuf = kbuf + 2 * C::K_SLOT;       // 2 slots: [hi | lo]
    uint64_t* bars = reinterpret_cast<uint64_t*>(vbuf + 2 * C::V_SLOT);
    uint64_t* k_full = bars + 0;    // [2]
    uint64_t* k_empty = bars + 2;   // [2]
    uint64_t* v_full = bars + 4;    // [2]
    uint64_t* v_empty = bars + 6;   // [2]
    uint64_t* s_full = bars + 8;    // [2]
    uint64_t* q_ready = bars + 10;
    uint64_t* p_full = bars + 11;
    uint64_t* pv_full = bars + 12;
    uint64_t* drain = bars + 13;
    uint64_t* pair_bar = bars + 14;   // [4 quarters][3]: row-pair exchange, tiles even/odd + final
    constexpr int NBAR = 26;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* k_issued = const_cast<int*>(abort_flag) + 1;   // [2] phase of the last load per slot, -1 none
    int* v_issued = k_issued + 2;                       // [2]
    // partial row maxima / sums exchanged by the two threads of a row: [tile even | odd | final][2 halves][128 rows]
    float* red = reinterpret_cast<float*>(smem + C::QL_BYTES + 2 * C::K_SLOT + 2 * C::V_SLOT + 256);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int qb = p.causal ? p.n_qblocks - 1 - (int)blockIdx.x : (int)blockIdx.x;   // long rows first
    const int q0 = qb * BQ;
    const int bhkv = bh / p.group;
    int kv_len = p.S;
    if (p.causal) kv_len = min(p.S, q0 + BQ);
    const int n_tiles = (kv_len + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; i++) ptx::mbar_init(&bars[i], (i == 10 || i == 11) ? 32 * SOFT_WARPS : i >= 14 ? 64 : 1);
        *abort_flag = 0;
        k_issued[0] = k_issued[1] = v_issued[0] = v_issued[1] = -1;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&p.tk_hi);
        ptx::prefetch_tmap(&p.tk_lo);
        ptx::prefetch_tmap(&p.tv_hi);
        ptx::prefetch_tmap(&p.tv_lo);
    }
    if (warp == 1) ptx::tmem_alloc(tmem_slot, 512);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            for (int j = 0; j < n_tiles; j++) {
                const int slot = j & 1;
                const uint32_t par = ((j >> 1) & 1) ^ 1;
                const int k0 = j * BKV;
                uint8_t* kh = kbuf + slot * C::K_SLOT;
                uint8_t* vh = vbuf + slot * C::V_SLOT;
                if (!ptx::wait_bounded(&k_empty[slot], par, abort_flag, p.err, ERR_A_PROD, WAIT_NS)) break;
                ptx::mbar_expect_tx(&k_full[slot], C::K_SLOT);
                k_issued[slot] = (j >> 1) & 1;
#pragma unroll
                for (int c = 0; c < D / 32; c++) {
                    ptx::tma_load_3d(kh + c * BKV * 128, &p.tk_hi, &k_full[slot], c * 32, k0, bhkv);
                    ptx::tma_load_3d(kh + C::KH_BYTES + c * BKV * 128, &p.tk_lo, &k_full[slot], c * 32, k0, bhkv);
                }
                if (!ptx::wait_bounded(&v_empty[slot], par, abort_flag, p.err, ERR_A_PROD, WAIT_NS)) break;
                ptx::mbar_expect_tx(&v_full[slot], C::V_SLOT);
                v_issued[slot] = (j >> 1) & 1;
#pragma unroll
                for (int c = 0; c < BKV / 32; c++) {
                    ptx::tma_load_3d(vh + c * D * 128, &p.tv_hi, &v_full[slot], k0 + c * 32, 0, bhkv);
                    ptx::tma_load_3d(vh + C::VH_BYTES + c * D * 128, &p.tv_lo, &v_full[slot], k0 + c * 32, 0, bhkv);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = ptx::idesc_tf32(BQ, BKV);
            constexpr uint32_t idesc_o = ptx::idesc_tf32(BQ, D);
            bool ok = ptx::wait_bounded(q_ready, 0, abort_flag, p.err, ERR_A_MMA, WAIT_NS);
            ptx::tc_fence_after();
            // S_j = Q.K_j^T into S buffer j&1
            auto issue_s = [&](int j) -> bool {
                const int slot = j & 1;
                if (!ptx::wait_bounded(&k_full[slot], (j >> 1) & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS))
                    return false;
                ptx::tc_fence_after();
                const uint8_t* kh = kbuf + slot * C::K_SLOT;
                const uint32_t d_s = tmem + C::COL_S + slot * BKV;
#pragma unroll
                for (int kk = 0; kk < D / 8; kk++) {
                    const int c = kk >> 2, off = (kk & 3) * 32;
                    uint64_t b_hi = ptx::smem_desc(kh + c * BKV * 128 + off, 1024, 2);
                    uint64_t b_lo = ptx::smem_desc(kh + C::KH_BYTES + c * BKV * 128 + off, 1024, 2);
                    uint64_t a_lo = ptx::smem_desc(ql + c * BQ * 128 + off, 1024, 2);
                    const uint32_t a_hi = tmem + kk * 8;
                    ptx::mma_tf32_ts(d_s, a_hi, b_hi, idesc_s, kk > 0 ? 1u : 0u);
                    ptx::mma_tf32_ts(d_s, a_hi, b_lo, idesc_s, 1u);
                    ptx::mma_tf32(d_s, a_lo, b_hi, idesc_s, 1u);
                }
                ptx::mma_commit(&k_empty[slot]);
                ptx::mma_commit(&s_full[slot]);
                return true;
            };
            if (ok && n_tiles > 0) ok = issue_s(0);
            for (int j = 0; j < n_tiles && ok; j++) {
                // S buffer (j+1)&1 was last read by softmax j-1, which finished before p_full j-1
                if (j + 1 < n_tiles && !(ok = issue_s(j + 1))) break;
                const int slot = j & 1;
                if (!(ok = ptx::wait_bounded(p_full, j & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS))) break;
                ptx::tc_fence_after();
                if (!(ok = ptx::wait_bounded(&v_full[slot], (j >> 1) & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS)))
                    break;
                ptx::tc_fence_after();
                const uint8_t* vh = vbuf + slot * C::V_SLOT;
#pragma unroll
                for (int kk = 0; kk < BKV / 8; kk++) {
                    const int c = kk >> 2, off = (kk & 3) * 32;
                    uint64_t b_hi = ptx::smem_desc(vh + c * D * 128 + off, 1024, 2);
                    uint64_t b_lo = ptx::smem_desc(vh + C::VH_BYTES + c * D * 128 + off, 1024, 2);
                    ptx::mma_tf32_ts(tmem + C::COL_O, tmem + C::COL_PH + kk * 8, b_hi, idesc_o, kk > 0 ? 1u : 0u);
                    ptx::mma_tf32_ts(tmem + C::COL_O, tmem + C::COL_PH + kk * 8, b_lo, idesc_o, 1u);
                    ptx::mma_tf32_ts(tmem + C::COL_O, tmem + C::COL_PL + kk * 8, b_hi, idesc_o, 1u);
                }
                ptx::mma_commit(&v_empty[slot]);
                ptx::mma_commit(pv_full);
            }
            ptx::mma_commit(drain);
            volatile int no_abort = 0;
            ptx::wait_bounded(drain, 0, &no_abort, p.err, ERR_A_DRAIN, WAIT_NS);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------- softmax rows
        // Two threads per query row (warps w and w+4 share TMEM lanes): each
        // owns half of the row's scores and half of its output columns.
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const int q = q0 + row;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        constexpr int DH = D / 2, KH = BKV / 2;   // per-thread output columns / score columns
        const float* qrow = p.q + ((int64_t)bh * p.S + (q < p.S ? q : 0)) * D;
        const float sl2 = p.scale * 1.4426950408889634f;   // scores in log2 units: exp(x) = 2^(x*log2 e)
        // exchange with the row's other thread through an mbarrier (bounded wait, never a hang)
        auto pair_sync = [&](int which, uint32_t parity) -> bool {
            uint64_t* b = &pair_bar[quarter * 3 + which];
            ptx::mbar_arrive(b);
            return ptx::wait_bounded(b, parity, abort_flag, p.err, ERR_A_SOFT, WAIT_NS);
        };
        // stage Q: hi -> TMEM [0, D), lo -> shared memory (128-byte swizzle)
#pragma unroll 1
        for (int c16 = half * (DH / 16); c16 < (half + 1) * (DH / 16); c16++) {
            uint32_t hi[16];
            float lo[16];
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                float4 v = q < p.S ? *reinterpret_cast<const float4*>(qrow + c16 * 16 + i)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    float h = tf32_round(x[k]);
                    hi[i + k] = __float_as_uint(h);
                    lo[i + k] = x[k] - h;
                }
            }
            ptx::tmem_st16(tmem + lane_off + c16 * 16, hi);
            const int chunk = c16 >> 1;
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int unit = (c16 & 1) * 4 + u;   // 16-byte unit within the 128-byte row
                uint8_t* dst = ql + chunk * BQ * 128 + row * 128 + ((unit ^ (row & 7)) << 4);
                *reinterpret_cast<float4*>(dst) = make_float4(lo[4 * u], lo[4 * u + 1], lo[4 * u + 2], lo[4 * u + 3]);
            }
        }
        ptx::tmem_st_wait();
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        ptx::mbar_arrive(q_ready);

        float m = -FLT_MAX, l = 0.0f;   // m in log2 units; -FLT_MAX as the reference's initial max
        float o[DH];
#pragma unroll
        for (int i = 0; i < DH; i++) o[i] = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_tiles; j++) {
            const uint32_t s_col = C::COL_S + (j & 1) * BKV + half * KH;
            if (!(ok = ptx::wait_bounded(&s_full[j & 1], (j >> 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS)))
                break;
            ptx::tc_fence_after();
            const int k0 = j * BKV + half * KH;
            // every key of this half-tile valid for this row: no mask arithmetic
            const bool full = k0 + KH <= p.S && (!p.causal || k0 + KH - 1 <= q);
            float sv[KH];
#pragma unroll
            for (int c16 = 0; c16 < KH / 16; c16++) {
                uint32_t r[16];
                ptx::tmem_ld16(tmem + lane_off + s_col + c16 * 16, r);
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; i++) sv[c16 * 16 + i] = __uint_as_float(r[i]) * sl2;
            }
            float mt = -INFINITY;
            if (full) {
#pragma unroll
                for (int i = 0; i < KH; i++) mt = fmaxf(mt, sv[i]);
            } else {
#pragma unroll
                for (int i = 0; i < KH; i++) {
                    const int kj = k0 + i;
                    if (kj >= p.S || (p.causal && kj > q)) sv[i] = -INFINITY;
                    mt = fmaxf(mt, sv[i]);
                }
            }
            red[((j & 1) * 2 + half) * BQ + row] = mt;
            if (!(ok = pair_sync(j & 1, (j >> 1) & 1))) break;
            mt = fmaxf(mt, red[((j & 1) * 2 + (half ^ 1)) * BQ + row]);
            if (j > 0) {   // O tile j-1: fold into registers (also frees P and the O tile)
                if (!(ok = ptx::wait_bounded(pv_full, (j - 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS))) break;
                ptx::tc_fence_after();
#pragma unroll
                for (int c16 = 0; c16 < DH / 16; c16++) {
                    uint32_t r[16];
                    ptx::tmem_ld16(tmem + lane_off + C::COL_O + half * DH + c16 * 16, r);
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; i++) o[c16 * 16 + i] += __uint_as_float(r[i]);
                }
            }
            if (mt > m) {   // running max grows: rescale (corr would be 1 otherwise)
                const float corr = exp2f(m - mt);
                l *= corr;
#pragma unroll
                for (int i = 0; i < DH; i++) o[i] *= corr;
                m = mt;
            }
#pragma unroll
            for (int c16 = 0; c16 < KH / 16; c16++) {
                uint32_t ph[16], pl[16];
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    float pv = exp2f(sv[c16 * 16 + i] - m);   // masked: 2^-inf = 0
                    l += pv;
                    float h = tf32_round(pv);
                    ph[i] = __float_as_uint(h);
                    pl[i] = __float_as_uint(pv - h);
                }
                ptx::tmem_st16(tmem + lane_off + C::COL_PH + half * KH + c16 * 16, ph);
                ptx::tmem_st16(tmem + lane_off + C::COL_PL + half * KH + c16 * 16, pl);
            }
            ptx::tmem_st_wait();
            ptx::tc_fence_before();
            ptx::mbar_arrive(p_full);
        }
        if (ok && n_tiles > 0 &&
            ptx::wait_bounded(pv_full, (n_tiles - 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS)) {
            ptx::tc_fence_after();
#pragma unroll
            for (int c16 = 0; c16 < DH / 16; c16++) {
                uint32_t r[16];
                ptx::tmem_ld16(tmem + lane_off + C::COL_O + half * DH + c16 * 16, r);
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; i++) o[c16 * 16 + i] += __uint_as_float(r[i]);
            }
            red[(4 + half) * BQ + row] = l;
            const bool paired = pair_sync(2, 0);
            l += red[(4 + (half ^ 1)) * BQ + row];
            if (paired && q < p.S) {
                const float inv = 1.0f / l;
                float* orow = p.o + ((int64_t)bh * p.S + q) * D + half * DH;
#pragma unroll
                for (int i = 0; i < DH; i += 4)
                    *reinterpret_cast<float4*>(orow + i) =
                        make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
            }
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        volatile int no_abort = 0;
        for (int sl = 0; sl < 2; sl++) {
            if (k_issued[sl] >= 0)
                ptx::wait_bounded(&k_full[sl], (uint32_t)k_issued[sl], &no_abort, nullptr, 0, 100000000ull);
            if (v_issued[sl] >= 0)
                ptx::wait_bounded(&v_full[sl], (uint32_t)v_issued[sl], &no_abort, nullptr, 0, 100000000ull);
        }
    }
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

template <int D>
Status launch_tc(const AttnTcParams& prm, int BH, cudaStream_t st) {
    dim3 grid((unsigned)prm.n_qblocks, (unsigned)BH);
    attn_tc_kernel<D><<<grid, ATHREADS, AttnTcCfg<D>::SMEM, st>>>(prm);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

}  // namespace

// Shapes this kernel takes: no custom mask, head_dim 64 or 128, S a multiple
// of 4 (TMA row stride of V^T), at least one full query block.
bool attention_tc_applicable(int64_t S, int D, bool has_mask, int64_t BH) {
    return !has_mask && (D == 64 || D == 128) && S % 4 == 0 && S >= 128 && BH <= 65535 && S < (1 << 30);
}

size_t attention_tc_workspace(int64_t BHkv, int64_t S, int D) { return 4 * (size_t)BHkv * S * D * 4 + 4 * 256; }

Status attention_tc_prepare() {
    static bool done = false;
    if (!done) {
        RT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           AttnTcCfg<64>::SMEM));
        RT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           AttnTcCfg<128>::SMEM));
        done = true;
    }
    return Status::ok();
}

Status launch_attention_tc(const float* q, const float* k, const float* v, float* o, int64_t BH, int64_t S,
                           int D, int group, int causal, Workspace ws, cudaStream_t st, int* launches) {
    const int64_t BHkv = BH / group;
    const size_t part = (((size_t)BHkv * S * D * 4) + 255) & ~(size_t)255;
    if (ws.bytes < 4 * part) return Status::err(RT_ERR_ARGUMENT, "attention: workspace too small");
    float* khi = reinterpret_cast<float*>(ws.base);
    float* klo = reinterpret_cast<float*>(ws.base + part);
    float* vhi = reinterpret_cast<float*>(ws.base + 2 * part);
    float* vlo = reinterpret_cast<float*>(ws.base + 3 * part);
    Status s = split_operand(k, khi, klo, 1, BHkv * S, D, false, st);
    if (!s.good()) return s;
    s = split_operand(v, vhi, vlo, BHkv, D, S, true, st);   // [BHkv][S][D] -> [BHkv][D][S]
    if (!s.good()) return s;
    *launches += 2;
    AttnTcParams prm;
    memset(&prm, 0, sizeof prm);
    if (!(s = encode_tmap_f32_3d(&prm.tk_hi, khi, D, S, BHkv, 32, D == 128 ? 32 : 64, 128)).good()) return s;
    if (!(s = encode_tmap_f32_3d(&prm.tk_lo, klo, D, S, BHkv, 32, D == 128 ? 32 : 64, 128)).good()) return s;
    if (!(s = encode_tmap_f32_3d(&prm.tv_hi, vhi, S, D, BHkv, 32, D, 128)).good()) return s;
    if (!(s = encode_tmap_f32_3d(&prm.tv_lo, vlo, S, D, BHkv, 32, D, 128)).good()) return s;
    prm.q = q;
    prm.o = o;
    prm.S = (int)S;
    prm.group = group;
    prm.causal = causal;
    prm.n_qblocks = (int)((S + BQ - 1) / BQ);
    prm.scale = 1.0f / sqrtf((float)D);
    prm.err = kernel_error_flag();
    *launches += 1;
    return D == 64 ? launch_tc<64>(prm, (int)BH, st) : launch_tc<128>(prm, (int)BH, st);
}

}  // namespace rt
