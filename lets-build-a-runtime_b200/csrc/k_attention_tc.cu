// k_attention_tc.cu -- fused attention on the 5th-generation tensor cores.
//
// Same function as the reference's flash kernel (csrc/ops/attn.c:121-253):
// scores = (Q K^T) * 1/sqrtf(D), causal mask as -inf, online softmax with
// running max starting at -FLT_MAX, O = P V / l, GQA kv head = bh / group.
// Both products run as 3xTF32 on tcgen05 (hi.hi + hi.lo + lo.hi) so results
// stay at fp32 level; each P.V tile is accumulated in TMEM and folded into
// fp32 registers, like the GEMM's K chunks.
//
// One CTA = 128 queries of one (batch, head); 352 threads:
//   warps 0,10 producers (K and V separately): one contiguous bulk copy per
//              key tile (64 keys for D=64, 32 for D=128) of a pre-packed,
//              pre-swizzled image, two slots each;
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
// TMEM columns: Q_hi [0,D) | S x2 | (P_hi, P_lo) x2 | O tile.
// K and V are split, V transposed and both packed into per-tile shared-memory
// images in the node's workspace by a bandwidth-bound pre-pass
// (pack_kv_kernel).  All waits are bounded (see sm100_ptx.h).
#include <float.h>

#include "gemm.h"
#include "sm100_ptx.h"

namespace rt {

int* kernel_error_flag();

namespace {

constexpr int BQ = 128, SOFT_WARPS = 8, ATHREADS = 96 + 32 * SOFT_WARPS;   // K producer, MMA, softmax x8, V producer
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
    // S x2 | (P_hi, P_lo) x2 | O tile
    static constexpr uint32_t COL_S = D, COL_P = D + 2 * BKV, COL_O = D + 6 * BKV;
    static_assert(2 * D + 6 * BKV <= 512, "TMEM budget");
};

struct AttnTcParams {
    const uint8_t* kv;          // packed tiles: [BHkv][n_kv][K image | V image] (pack_kv_kernel)
    int n_kv;                   // key tiles per head
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
    }
    if (warp == 1) ptx::tmem_alloc(tmem_slot, 512);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 || warp == 2 + SOFT_WARPS) {
        // ---------------------------------------------------- TMA producers
        // K and V tiles come from separate warps so that K loads run ahead:
        // a K slot frees when its S tile is done, a V slot only after P.V.
        const bool is_k = warp == 0;
        if (lane == 0) {
            for (int j = 0; j < n_tiles; j++) {
                const int slot = j & 1;
                const uint32_t par = ((j >> 1) & 1) ^ 1;
                const uint8_t* tile = p.kv + ((size_t)bhkv * p.n_kv + j) * (C::K_SLOT + C::V_SLOT);
                if (is_k) {
                    if (!ptx::wait_bounded(&k_empty[slot], par, abort_flag, p.err, ERR_A_PROD, WAIT_NS)) break;
                    ptx::mbar_expect_tx(&k_full[slot], C::K_SLOT);
                    k_issued[slot] = (j >> 1) & 1;
                    ptx::bulk_load(kbuf + slot * C::K_SLOT, tile, C::K_SLOT, &k_full[slot]);
                } else {
                    if (!ptx::wait_bounded(&v_empty[slot], par, abort_flag, p.err, ERR_A_PROD, WAIT_NS)) break;
                    ptx::mbar_expect_tx(&v_full[slot], C::V_SLOT);
                    v_issued[slot] = (j >> 1) & 1;
                    ptx::bulk_load(vbuf + slot * C::V_SLOT, tile + C::K_SLOT, C::V_SLOT, &v_full[slot]);
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
                // descriptors built once per tile; K steps advance the start address field
                const uint64_t bh0 = ptx::smem_desc(kh, 1024, 2);
                const uint64_t bl0 = ptx::smem_desc(kh + C::KH_BYTES, 1024, 2);
                const uint64_t al0 = ptx::smem_desc(ql, 1024, 2);
#pragma unroll
                for (int kk = 0; kk < D / 8; kk++) {
                    const uint64_t boff = (uint64_t)(((kk >> 2) * BKV * 128 + (kk & 3) * 32) >> 4);
                    const uint64_t aoff = (uint64_t)(((kk >> 2) * BQ * 128 + (kk & 3) * 32) >> 4);
                    const uint32_t a_hi = tmem + kk * 8;
                    ptx::mma_tf32_ts(d_s, a_hi, bh0 + boff, idesc_s, kk > 0 ? 1u : 0u);
                    ptx::mma_tf32_ts(d_s, a_hi, bl0 + boff, idesc_s, 1u);
                    ptx::mma_tf32(d_s, al0 + aoff, bh0 + boff, idesc_s, 1u);
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
                const uint32_t p_hi = tmem + C::COL_P + (j & 1) * 2 * BKV, p_lo = p_hi + BKV;
                const uint64_t vh0 = ptx::smem_desc(vh, 1024, 2);
                const uint64_t vl0 = ptx::smem_desc(vh + C::VH_BYTES, 1024, 2);
#pragma unroll
                for (int kk = 0; kk < BKV / 8; kk++) {
                    const uint64_t off = (uint64_t)(((kk >> 2) * D * 128 + (kk & 3) * 32) >> 4);
                    ptx::mma_tf32_ts(tmem + C::COL_O, p_hi + kk * 8, vh0 + off, idesc_o, kk > 0 ? 1u : 0u);
                    ptx::mma_tf32_ts(tmem + C::COL_O, p_hi + kk * 8, vl0 + off, idesc_o, 1u);
                    ptx::mma_tf32_ts(tmem + C::COL_O, p_lo + kk * 8, vh0 + off, idesc_o, 1u);
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
        // ---------------------------------------------------- softmax rows (warps 2 .. 1+SOFT_WARPS)
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
            {
                uint32_t r[KH];
#pragma unroll
                for (int c16 = 0; c16 < KH / 16; c16++)
                    ptx::tmem_ld16(tmem + lane_off + s_col + c16 * 16, *reinterpret_cast<uint32_t(*)[16]>(&r[c16 * 16]));
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < KH; i++) sv[i] = __uint_as_float(r[i]) * sl2;
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
            const float m_new = mt > m ? mt : m;
            // P_j (relative to m_new) into P buffer j&1; that buffer's last reader,
            // PV_{j-2}, finished before this thread's previous p_full arrive
            const uint32_t p_hi = tmem + lane_off + C::COL_P + (j & 1) * 2 * BKV + half * KH;
            float lt = 0.0f;
#pragma unroll
            for (int c16 = 0; c16 < KH / 16; c16++) {
                uint32_t ph[16], pl[16];
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    float pv = exp2f(sv[c16 * 16 + i] - m_new);   // masked: 2^-inf = 0
                    lt += pv;
                    float h = tf32_round(pv);
                    ph[i] = __float_as_uint(h);
                    pl[i] = __float_as_uint(pv - h);
                }
                ptx::tmem_st16(p_hi + c16 * 16, ph);
                ptx::tmem_st16(p_hi + BKV + c16 * 16, pl);
            }
            if (j > 0) {   // O tile j-1 (relative to the old max): fold into registers, freeing the tile
                if (!(ok = ptx::wait_bounded(pv_full, (j - 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS))) break;
                ptx::tc_fence_after();
                uint32_t r[DH];
#pragma unroll
                for (int c16 = 0; c16 < DH / 16; c16++)
                    ptx::tmem_ld16(tmem + lane_off + C::COL_O + half * DH + c16 * 16,
                                   *reinterpret_cast<uint32_t(*)[16]>(&r[c16 * 16]));
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < DH; i++) o[i] += __uint_as_float(r[i]);
            }
            if (m_new > m) {   // running max grew: rescale (corr would be 1 otherwise)
                const float corr = exp2f(m - m_new);
                l *= corr;
#pragma unroll
                for (int i = 0; i < DH; i++) o[i] *= corr;
                m = m_new;
            }
            l += lt;
            ptx::tmem_st_wait();
            ptx::tc_fence_before();
            ptx::mbar_arrive(p_full);
        }
        if (ok && n_tiles > 0 &&
            ptx::wait_bounded(pv_full, (n_tiles - 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS)) {
            ptx::tc_fence_after();
            {
                uint32_t r[DH];
#pragma unroll
                for (int c16 = 0; c16 < DH / 16; c16++)
                    ptx::tmem_ld16(tmem + lane_off + C::COL_O + half * DH + c16 * 16,
                                   *reinterpret_cast<uint32_t(*)[16]>(&r[c16 * 16]));
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < DH; i++) o[i] += __uint_as_float(r[i]);
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

// Packs K and V into per-tile images that are byte-for-byte the shared-memory
// layout the MMA reads (K: [D/32 chunks][BKV keys][128 B], V^T: [BKV/32
// chunks][D][128 B]; 16-byte units swizzled by row % 8 as the 128-byte
// swizzle mode expects; hi then lo), so each tile is one contiguous bulk copy.
// Keys past S are zero.
template <int D>
__global__ void pack_kv_kernel(const float* __restrict__ k, const float* __restrict__ v,
                               uint8_t* __restrict__ out, int S, int n_kv) {
    using C = AttnTcCfg<D>;
    constexpr int BKV = C::BKV;
    const int j = blockIdx.x, h = blockIdx.y;
    const int k0 = j * BKV;
    uint8_t* tile = out + ((size_t)h * n_kv + j) * (C::K_SLOT + C::V_SLOT);
    const float* kb = k + (size_t)h * S * D;
    const float* vb = v + (size_t)h * S * D;
    for (int e = threadIdx.x; e < BKV * D; e += blockDim.x) {
        const int r = e / D, d = e % D;   // key within tile, feature
        const bool ok = k0 + r < S;
        const float kx = ok ? kb[(size_t)(k0 + r) * D + d] : 0.0f;
        const float vx = ok ? vb[(size_t)(k0 + r) * D + d] : 0.0f;
        const float kh = tf32_round(kx), vh = tf32_round(vx);
        // K image: chunk d/32, row r, unit (d%32)/4
        {
            const int c = d >> 5, w = d & 31;
            const size_t off = (size_t)c * BKV * 128 + r * 128 + ((((w >> 2) ^ (r & 7))) << 4) + (w & 3) * 4;
            *reinterpret_cast<float*>(tile + off) = kh;
            *reinterpret_cast<float*>(tile + C::KH_BYTES + off) = kx - kh;
        }
        // V^T image: chunk r/32, row d, unit (r%32)/4
        {
            const int c = r >> 5, w = r & 31;
            const size_t off = (size_t)c * D * 128 + d * 128 + ((((w >> 2) ^ (d & 7))) << 4) + (w & 3) * 4;
            *reinterpret_cast<float*>(tile + C::K_SLOT + off) = vh;
            *reinterpret_cast<float*>(tile + C::K_SLOT + C::VH_BYTES + off) = vx - vh;
        }
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

size_t attention_tc_workspace(int64_t BHkv, int64_t S, int D) {
    const int bkv = D == 128 ? AttnTcCfg<128>::BKV : AttnTcCfg<64>::BKV;
    const size_t tile = D == 128 ? AttnTcCfg<128>::K_SLOT + AttnTcCfg<128>::V_SLOT
                                 : AttnTcCfg<64>::K_SLOT + AttnTcCfg<64>::V_SLOT;
    return (size_t)BHkv * ((S + bkv - 1) / bkv) * tile;
}

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
    if (ws.bytes < attention_tc_workspace(BHkv, S, D)) return Status::err(RT_ERR_ARGUMENT, "attention: workspace too small");
    const int bkv = D == 128 ? AttnTcCfg<128>::BKV : AttnTcCfg<64>::BKV;
    const int n_kv = (int)((S + bkv - 1) / bkv);
    dim3 pgrid((unsigned)n_kv, (unsigned)BHkv);
    if (D == 64)
        pack_kv_kernel<64><<<pgrid, 256, 0, st>>>(k, v, reinterpret_cast<uint8_t*>(ws.base), (int)S, n_kv);
    else
        pack_kv_kernel<128><<<pgrid, 256, 0, st>>>(k, v, reinterpret_cast<uint8_t*>(ws.base), (int)S, n_kv);
    RT_LAUNCH_CHECK();
    *launches += 1;
    AttnTcParams prm;
    memset(&prm, 0, sizeof prm);
    prm.kv = reinterpret_cast<const uint8_t*>(ws.base);
    prm.n_kv = n_kv;
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
