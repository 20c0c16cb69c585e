// k_attention_tc.cu -- fused attention on the 5th-generation tensor cores.
//
// Same function as the reference's flash kernel (csrc/ops/attn.c:121-253):
// scores = (Q K^T) * 1/sqrtf(D), causal mask as -inf, online softmax with
// running max starting at -FLT_MAX, O = P V / l, GQA kv head = bh / group.
// Both products keep fp32-level accuracy with the GEMM's operand split
// (x = hi + lo, hi = tf32(x)): hi.hi as a kind::tf32 MMA and the two cross
// terms as ONE kind::f16 MMA over a doubled K with bf16 operands
// [hi | lo] x [lo | hi] per 16-wide block (RT_ATTN_3XTF32=1: three tf32 MMAs,
// hi.hi + hi.lo + lo.hi).  Each P.V tile (128 keys) is accumulated in TMEM
// and folded into fp32 registers, like the GEMM's K chunks.
//
// Tiles are 128 queries x 128 keys, so every score MMA is M=128 x N=128
// (narrower MMAs are dominated by per-instruction cost on this hardware).
// One CTA = 128 queries of one (batch, head); 320 threads:
//   warp 0     producer: streams 32 KiB chunks through a shared-memory ring in
//              exactly the order the MMAs consume them -- K_0, K_1, V_0, K_2,
//              V_1, ... (K tile = D/32 chunks of 32 features x 128 keys, V^T
//              tile = chunks of 32 or 64 keys x D), each chunk one contiguous
//              bulk copy of a pre-packed, pre-swizzled image;
//   warp 1     allocates TMEM and issues the MMAs from one thread:
//              S = Q.K^T (Q from shared memory), O_tile = P.V (P from TMEM),
//              each as hi.hi + the cross terms;
//              S_{j+1} runs while the softmax works on S_j;
//   warps 2-9  two threads per query row (64 keys and D/2 output columns
//              each; row maxima / sums exchanged through shared memory behind
//              bounded mbarrier waits): stage Q hi/lo into shared memory, then
//              per tile read S from TMEM (freeing it), mask, online softmax in
//              log2 units, fold the previous O tile into registers, write P's
//              two planes to TMEM.
// TMEM columns: S [0,128) | P_hi [128,256) | P plane 1 [256,384) | O tile [384, 384+D).
// Plane 1 of every operand (Q, K, V in shared memory, P in TMEM) is lo as
// fp32, or for the cross scheme bf16 [hi | lo] (Q, P) / [lo | hi] (K, V) per
// 16-wide K block -- the same 4 bytes per element, so tiles and offsets are
// shared by both schemes.
// K and V are split, V transposed and both packed into per-tile images in the
// node's workspace by a bandwidth-bound pre-pass (pack_kv_kernel).  All waits
// are bounded (see sm100_ptx.h).
#include <float.h>

#include "gemm.h"
#include "sm100_ptx.h"

namespace rt {

int* kernel_error_flag();

namespace {

constexpr int BQ = 128, BKV = 128, SOFT_WARPS = 8, ATHREADS = 64 + 32 * SOFT_WARPS;
constexpr int CHUNK = 32 * 1024;                      // ring stage / packed chunk
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr int ERR_A_PROD = 0x201, ERR_A_MMA = 0x202, ERR_A_SOFT = 0x203, ERR_A_DRAIN = 0x204;
constexpr uint32_t COL_S = 0, COL_PH = 128, COL_PL = 256, COL_O = 384;

template <int D>
struct AttnTcCfg {
    static constexpr int Q_BYTES = D * BQ * 4;                  // one of Q_hi / Q_lo: D/32 x [128][128 B]
    static constexpr int K_CHUNKS = D / 32;                     // 32 features x 128 keys, hi | lo
    static constexpr int V_KEYS = D == 128 ? 32 : 64;           // keys per V chunk (D x keys, hi | lo)
    static constexpr int V_CHUNKS = BKV / V_KEYS;
    static constexpr int TILE_BYTES = (K_CHUNKS + V_CHUNKS) * CHUNK;
    static constexpr int STAGES = D == 128 ? 3 : 5;
    static constexpr int BODY = 2 * Q_BYTES + STAGES * CHUNK + 256 /*barriers*/ + 4 * BQ * 4 /*row exchange*/;
    static constexpr int SMEM = BODY + 768;   // + alignment slack; 232448 B, the per-CTA maximum
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(COL_O + D <= 512, "TMEM budget");
};

struct AttnTcParams {
    const uint8_t* kv;   // packed tiles [BHkv][n_kv][K chunks | V chunks]
    int n_kv;            // key tiles per head
    const float* q;
    float* o;
    int64_t q_sb, q_sh, q_ss;   // element strides of Q: batch, head, sequence (features contiguous)
    int64_t o_sb, o_sh, o_ss;   // same for O
    int H;                      // query heads per batch element
    int S, group, causal, n_qblocks;
    int heads_fast;             // grid (BH, q blocks) instead of (q blocks, BH)
    float scale;
    int* err;
};

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Byte offset of element (row, w) -- w = 0..31 within a 128-byte row -- in a
// [rows][128 B] block written the way the 128-byte swizzle mode reads it.
__device__ __forceinline__ uint32_t swz(int row, int w) {
    return (uint32_t)row * 128 + ((((uint32_t)w >> 2) ^ ((uint32_t)row & 7)) << 4) + ((uint32_t)w & 3) * 4;
}

// Packs K (as [K chunk c: 128 keys x 32 features]) and V^T (as [V chunk c:
// D x V_KEYS keys, in 32-key sub-blocks]) of one 128-key tile, hi then lo in
// each chunk, byte-for-byte the shared-memory image the MMAs read.  Keys
// past S are zero.  Every store is a whole 16-byte unit; V is transposed
// through shared memory 32 keys at a time so its global reads stay coalesced.
struct KvViews {
    const float* k;
    const float* v;
    int64_t k_sb, k_sh, k_ss, v_sb, v_sh, v_ss;   // element strides: batch, head, sequence
    int Hkv;                                      // kv heads per batch element
};

// bf16 (round to nearest even) of two values, `a` in the low half.
__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}

// Plane 1 of four consecutive K elements x (k % 4 == 0, k = position inside a
// 128-byte row of 32 elements) at row `row` of a swizzled [rows][128 B]
// block: lo as fp32, or the cross layout (first = hi (A role) / lo (B role)).
template <bool CROSS, bool A_ROLE>
__device__ __forceinline__ void put_plane1(uint8_t* blk, int row, int k, float4 h, float4 l) {
    if (!CROSS) {
        *reinterpret_cast<float4*>(blk + swz(row, k)) = l;
        return;
    }
    const float4 f = A_ROLE ? h : l, g = A_ROLE ? l : h;
    const int b = k >> 4, j = k & 15;   // 16-wide block inside the row, position in it
    // bf16 positions b*32 + j (first) and b*32 + 16 + j (second) = 4-byte slots / 2
    *reinterpret_cast<uint2*>(blk + swz(row, b * 16 + (j >> 1))) = make_uint2(bf16x2(f.x, f.y), bf16x2(f.z, f.w));
    *reinterpret_cast<uint2*>(blk + swz(row, b * 16 + 8 + (j >> 1))) =
        make_uint2(bf16x2(g.x, g.y), bf16x2(g.z, g.w));
}

template <int D, bool CROSS>
__global__ void __launch_bounds__(256) pack_kv_kernel(KvViews kv, uint8_t* __restrict__ out, int S, int n_kv) {
    using C = AttnTcCfg<D>;
    __shared__ float sv[32][D + 1];
    const int j = blockIdx.x, h = blockIdx.y;
    const int k0 = j * BKV;
    uint8_t* tile = out + ((size_t)h * n_kv + j) * C::TILE_BYTES;
    const int bb = h / kv.Hkv, hh = h % kv.Hkv;
    const float* kb = kv.k + bb * kv.k_sb + hh * kv.k_sh;
    const float* vb = kv.v + bb * kv.v_sb + hh * kv.v_sh;
    // K: unit = 4 consecutive features of one key
    for (int u = threadIdx.x; u < BKV * D / 4; u += blockDim.x) {
        const int r = u / (D / 4), d = (u % (D / 4)) * 4;
        float4 x = k0 + r < S ? *reinterpret_cast<const float4*>(kb + (int64_t)(k0 + r) * kv.k_ss + d)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 hi = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
        uint8_t* kc = tile + (size_t)(d >> 5) * CHUNK;
        *reinterpret_cast<float4*>(kc + swz(r, d & 31)) = hi;
        put_plane1<CROSS, false>(kc + CHUNK / 2, r, d & 31, hi,
                                 make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w));
    }
    // V^T: unit = 4 consecutive keys of one feature
    for (int kb32 = 0; kb32 < BKV; kb32 += 32) {
        __syncthreads();
        for (int u = threadIdx.x; u < 32 * D / 4; u += blockDim.x) {
            const int r = u / (D / 4), d = (u % (D / 4)) * 4;
            const int key = k0 + kb32 + r;
            float4 x = key < S ? *reinterpret_cast<const float4*>(vb + (int64_t)key * kv.v_ss + d)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            sv[r][d] = x.x; sv[r][d + 1] = x.y; sv[r][d + 2] = x.z; sv[r][d + 3] = x.w;
        }
        __syncthreads();
        const int vc = kb32 / C::V_KEYS, sub = (kb32 % C::V_KEYS) >> 5;
        uint8_t* vcp = tile + (size_t)(C::K_CHUNKS + vc) * CHUNK + (size_t)sub * D * 128;
        for (int u = threadIdx.x; u < D * 8; u += blockDim.x) {
            const int d = u >> 3, w = (u & 7) * 4;
            float4 x = make_float4(sv[w][d], sv[w + 1][d], sv[w + 2][d], sv[w + 3][d]);
            float4 hi = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
            *reinterpret_cast<float4*>(vcp + swz(d, w)) = hi;
            put_plane1<CROSS, false>(vcp + CHUNK / 2, d, w, hi,
                                     make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w));
        }
    }
}

template <int D, bool CROSS>
__global__ void __launch_bounds__(ATHREADS, 1) attn_tc_kernel(const __grid_constant__ AttnTcParams p) {
    using C = AttnTcCfg<D>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* qh = smem;
    uint8_t* ql = qh + C::Q_BYTES;
    uint8_t* ring = ql + C::Q_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + STAGES * CHUNK);
    uint64_t* full = bars;                        // [STAGES]
    uint64_t* empty = bars + STAGES;              // [STAGES]
    uint64_t* s_full = bars + 2 * STAGES;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_full + 2;
    uint64_t* pv_full = s_full + 3;
    uint64_t* q_ready = s_full + 4;
    uint64_t* drain = s_full + 5;
    uint64_t* pair_bar = s_full + 6;              // [4 quarters][3]
    constexpr int NBAR = 2 * STAGES + 6 + 12;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued = const_cast<int*>(abort_flag) + 1;    // [STAGES] phase of the last load, -1 none
    float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);   // [2][2][128]
    if ((smem - smem_raw) + C::BODY > C::SMEM) {   // dynamic shared memory less aligned than assumed
        if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, 0x205);
        return;
    }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Launch order.  Heads fastest: under a causal mask every head's longest
    // query blocks start before any shorter one (longest first), which evens
    // out the last wave -- when all heads' packed K/V stays in L2.  Otherwise
    // query blocks fastest, so the CTAs in flight share few heads' K/V.
    const int bh = p.heads_fast ? (int)blockIdx.x : (int)blockIdx.y;
    const int qi = p.heads_fast ? (int)blockIdx.y : (int)blockIdx.x;
    const int qb = p.causal ? p.n_qblocks - 1 - qi : qi;
    const int q0 = qb * BQ;
    const int bhkv = bh / p.group;
    const int kv_len = p.causal ? min(p.S, q0 + BQ) : p.S;
    const int n_tiles = (kv_len + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; i++) {
            uint32_t cnt = 1;
            if (&bars[i] == s_free || &bars[i] == p_full || &bars[i] == q_ready) cnt = 32 * SOFT_WARPS;
            if (&bars[i] >= pair_bar) cnt = 64;
            ptx::mbar_init(&bars[i], cnt);
        }
        for (int s = 0; s < STAGES; s++) issued[s] = -1;
        *abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 1) ptx::tmem_alloc(tmem_slot, 512);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------- producer
        if (lane == 0) {
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            auto push = [&](const uint8_t* src) {
                if (!ok) return;
                if (!(ok = ptx::wait_bounded(&empty[stage], ph ^ 1, abort_flag, p.err, ERR_A_PROD, WAIT_NS)))
                    return;
                ptx::mbar_expect_tx(&full[stage], CHUNK);
                issued[stage] = (int)ph;
                ptx::bulk_load(ring + stage * CHUNK, src, CHUNK, &full[stage]);
                if (++stage == STAGES) {
                    stage = 0;
                    ph ^= 1;
                }
            };
            auto tile = [&](int j) { return p.kv + ((size_t)bhkv * p.n_kv + j) * C::TILE_BYTES; };
            for (int c = 0; c < C::K_CHUNKS; c++) push(tile(0) + c * CHUNK);
            for (int j = 0; j < n_tiles && ok; j++) {
                if (j + 1 < n_tiles)
                    for (int c = 0; c < C::K_CHUNKS; c++) push(tile(j + 1) + c * CHUNK);
                for (int c = 0; c < C::V_CHUNKS; c++) push(tile(j) + (C::K_CHUNKS + c) * CHUNK);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = ptx::idesc_tf32(BQ, BKV);
            constexpr uint32_t idesc_o = ptx::idesc_tf32(BQ, D);
            constexpr uint32_t idesc_sx = ptx::idesc_bf16(BQ, BKV);
            constexpr uint32_t idesc_ox = ptx::idesc_bf16(BQ, D);
            int stage = 0;
            uint32_t ph = 0;
            bool ok = ptx::wait_bounded(q_ready, 0, abort_flag, p.err, ERR_A_MMA, WAIT_NS);
            ptx::tc_fence_after();
            auto pop = [&]() -> uint8_t* {
                if (!ok) return nullptr;
                if (!(ok = ptx::wait_bounded(&full[stage], ph, abort_flag, p.err, ERR_A_MMA, WAIT_NS)))
                    return nullptr;
                ptx::tc_fence_after();
                return ring + stage * CHUNK;
            };
            auto release = [&]() {
                ptx::mma_commit(&empty[stage]);
                if (++stage == STAGES) {
                    stage = 0;
                    ph ^= 1;
                }
            };
            auto issue_s = [&]() {
                for (int c = 0; c < C::K_CHUNKS; c++) {
                    uint8_t* buf = pop();
                    if (!buf) return;
                    const uint64_t ah = ptx::smem_desc(qh + c * BQ * 128, 1024, 2);
                    const uint64_t al = ptx::smem_desc(ql + c * BQ * 128, 1024, 2);
                    const uint64_t bh0 = ptx::smem_desc(buf, 1024, 2);
                    const uint64_t bl0 = ptx::smem_desc(buf + CHUNK / 2, 1024, 2);
                    // 32 bytes per K step in both kinds (8 tf32 / 16 bf16)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t off = (uint64_t)((kk * 32) >> 4);
                        ptx::mma_tf32(tmem + COL_S, ah + off, bh0 + off, idesc_s, (c | kk) ? 1u : 0u);
                        if (CROSS) {
                            ptx::mma_bf16(tmem + COL_S, al + off, bl0 + off, idesc_sx, 1u);
                        } else {
                            ptx::mma_tf32(tmem + COL_S, ah + off, bl0 + off, idesc_s, 1u);
                            ptx::mma_tf32(tmem + COL_S, al + off, bh0 + off, idesc_s, 1u);
                        }
                    }
                    release();
                }
                if (ok) ptx::mma_commit(s_full);
            };
            auto issue_pv = [&]() {
                for (int c = 0; c < C::V_CHUNKS; c++) {
                    uint8_t* buf = pop();
                    if (!buf) return;
                    const uint64_t bh0 = ptx::smem_desc(buf, 1024, 2);
                    const uint64_t bl0 = ptx::smem_desc(buf + CHUNK / 2, 1024, 2);
#pragma unroll
                    for (int kk = 0; kk < C::V_KEYS / 8; kk++) {
                        const uint64_t off = (uint64_t)((((kk >> 2) * D * 128) + (kk & 3) * 32) >> 4);
                        const uint32_t kc = c * C::V_KEYS + kk * 8;
                        ptx::mma_tf32_ts(tmem + COL_O, tmem + COL_PH + kc, bh0 + off, idesc_o, (c | kk) ? 1u : 0u);
                        if (CROSS) {
                            // doubled K: 8 columns = 16 bf16 of P plane 1 per step, 32 bytes of V plane 1
                            ptx::mma_bf16_ts(tmem + COL_O, tmem + COL_PL + kc, bl0 + off, idesc_ox, 1u);
                        } else {
                            ptx::mma_tf32_ts(tmem + COL_O, tmem + COL_PH + kc, bl0 + off, idesc_o, 1u);
                            ptx::mma_tf32_ts(tmem + COL_O, tmem + COL_PL + kc, bh0 + off, idesc_o, 1u);
                        }
                    }
                    release();
                }
                if (ok) ptx::mma_commit(pv_full);
            };
            if (ok && n_tiles > 0) issue_s();
            for (int j = 0; j < n_tiles && ok; j++) {
                if (j + 1 < n_tiles) {   // S_{j+1} once the softmax has read S_j out of TMEM
                    if (!(ok = ptx::wait_bounded(s_free, j & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS))) break;
                    ptx::tc_fence_after();
                    issue_s();
                }
                if (!ok) break;
                if (!(ok = ptx::wait_bounded(p_full, j & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS))) break;
                ptx::tc_fence_after();
                issue_pv();
            }
            ptx::mma_commit(drain);
            volatile int no_abort = 0;
            ptx::wait_bounded(drain, 0, &no_abort, p.err, ERR_A_DRAIN, WAIT_NS);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------- softmax rows (warps 2..9)
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const int q = q0 + row;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        constexpr int DH = D / 2, KH = BKV / 2;   // per-thread output columns / score columns
        const float* qrow = p.q + (bh / p.H) * p.q_sb + (bh % p.H) * p.q_sh + (int64_t)(q < p.S ? q : 0) * p.q_ss;
        const float sl2 = p.scale * 1.4426950408889634f;   // scores in log2 units: exp(x) = 2^(x log2 e)
        auto pair_sync = [&](int which, uint32_t parity) -> bool {
            uint64_t* b = &pair_bar[quarter * 3 + which];
            ptx::mbar_arrive(b);
            return ptx::wait_bounded(b, parity, abort_flag, p.err, ERR_A_SOFT, WAIT_NS);
        };
        // stage this thread's half of the Q row: hi and lo, 128-byte swizzled
#pragma unroll 4
        for (int d = half * DH; d < (half + 1) * DH; d += 4) {
            float4 v = q < p.S ? *reinterpret_cast<const float4*>(qrow + d) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 h = make_float4(tf32_round(v.x), tf32_round(v.y), tf32_round(v.z), tf32_round(v.w));
            const uint32_t blk = (uint32_t)(d >> 5) * BQ * 128;
            *reinterpret_cast<float4*>(qh + blk + swz(row, d & 31)) = h;
            put_plane1<CROSS, true>(ql + blk, row, d & 31, h, make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w));
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(q_ready);

        float m = -FLT_MAX, l = 0.0f;   // m in log2 units; -FLT_MAX as the reference's initial max
        float o[DH];
#pragma unroll
        for (int i = 0; i < DH; i++) o[i] = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_tiles; j++) {
            if (!(ok = ptx::wait_bounded(s_full, j & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS))) break;
            ptx::tc_fence_after();
            float sv[KH];
            {
                uint32_t r[KH];
#pragma unroll
                for (int c16 = 0; c16 < KH / 16; c16++)
                    ptx::tmem_ld16(tmem + lane_off + COL_S + half * KH + c16 * 16,
                                   *reinterpret_cast<uint32_t(*)[16]>(&r[c16 * 16]));
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < KH; i++) sv[i] = __uint_as_float(r[i]) * sl2;
            }
            ptx::tc_fence_before();
            ptx::mbar_arrive(s_free);   // S may be overwritten by the next tile's MMAs
            const int k0 = j * BKV + half * KH;
            const bool full = k0 + KH <= p.S && (!p.causal || k0 + KH - 1 <= q);
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
            float lt = 0.0f;
#pragma unroll
            for (int i = 0; i < KH; i++) {
                sv[i] = exp2f(sv[i] - m_new);   // masked: 2^-inf = 0
                lt += sv[i];
            }
            if (j > 0) {   // O tile j-1 (relative to the old max): fold, freeing the tile and P
                if (!(ok = ptx::wait_bounded(pv_full, (j - 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS))) break;
                ptx::tc_fence_after();
#pragma unroll
                for (int g = 0; g < DH / 32; g++) {   // 32 columns per batch keeps registers in bounds
                    uint32_t r[32];
                    ptx::tmem_ld16(tmem + lane_off + COL_O + half * DH + g * 32, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
                    ptx::tmem_ld16(tmem + lane_off + COL_O + half * DH + g * 32 + 16,
                                   *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; i++) o[g * 32 + i] += __uint_as_float(r[i]);
                }
            }
            if (m_new > m) {   // running max grew: rescale (corr would be 1 otherwise)
                const float corr = exp2f(m - m_new);
                l *= corr;
#pragma unroll
                for (int i = 0; i < DH; i++) o[i] *= corr;
                m = m_new;
            }
            l += lt;
#pragma unroll
            for (int c16 = 0; c16 < KH / 16; c16++) {
                uint32_t ph[16], pl[16];
                if (CROSS) {   // plane 1: 8 columns of bf16 pairs of hi, then 8 of lo
#pragma unroll
                    for (int i = 0; i < 16; i += 2) {
                        const float a = sv[c16 * 16 + i], b = sv[c16 * 16 + i + 1];
                        const float ha = tf32_round(a), hb = tf32_round(b);
                        ph[i] = __float_as_uint(ha);
                        ph[i + 1] = __float_as_uint(hb);
                        pl[i / 2] = bf16x2(ha, hb);
                        pl[8 + i / 2] = bf16x2(a - ha, b - hb);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float pv = sv[c16 * 16 + i];
                        const float h = tf32_round(pv);
                        ph[i] = __float_as_uint(h);
                        pl[i] = __float_as_uint(pv - h);
                    }
                }
                ptx::tmem_st16(tmem + lane_off + COL_PH + half * KH + c16 * 16, ph);
                ptx::tmem_st16(tmem + lane_off + COL_PL + half * KH + c16 * 16, pl);
            }
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
                    ptx::tmem_ld16(tmem + lane_off + COL_O + half * DH + c16 * 16,
                                   *reinterpret_cast<uint32_t(*)[16]>(&r[c16 * 16]));
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < DH; i++) o[i] += __uint_as_float(r[i]);
            }
            // the exchange buffer of parity n_tiles&1 was last read for tile n_tiles-2
            const int fb = n_tiles & 1;
            red[(fb * 2 + half) * BQ + row] = l;
            const bool paired = pair_sync(2, 0);
            l += red[(fb * 2 + (half ^ 1)) * BQ + row];
            if (paired && q < p.S) {
                const float inv = 1.0f / l;
                float* orow = p.o + (bh / p.H) * p.o_sb + (bh % p.H) * p.o_sh + (int64_t)q * p.o_ss + half * DH;
#pragma unroll
                for (int i = 0; i < DH; i += 4)
                    *reinterpret_cast<float4*>(orow + i) =
                        make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
            }
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        // copies still in flight land before the CTA's shared memory goes away
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; s++)
            if (issued[s] >= 0)
                ptx::wait_bounded(&full[s], (uint32_t)issued[s], &no_abort, nullptr, 0, 100000000ull);
    }
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

// Cross-term scheme unless RT_ATTN_3XTF32=1.
bool attn_cross() {
    static const bool on = [] {
        const char* e = getenv("RT_ATTN_3XTF32");
        return !(e && e[0] == '1');
    }();
    return on;
}

template <int D>
Status launch_tc(const AttnTcParams& prm, int BH, cudaStream_t st) {
    dim3 grid = prm.heads_fast ? dim3((unsigned)BH, (unsigned)prm.n_qblocks)
                               : dim3((unsigned)prm.n_qblocks, (unsigned)BH);
    if (attn_cross())
        attn_tc_kernel<D, true><<<grid, ATHREADS, AttnTcCfg<D>::SMEM, st>>>(prm);
    else
        attn_tc_kernel<D, false><<<grid, ATHREADS, AttnTcCfg<D>::SMEM, st>>>(prm);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

}  // namespace

// Shapes this kernel takes: no custom mask, head_dim 64 or 128, at least one
// full 128-query block.
bool attention_tc_applicable(int64_t S, int D, bool has_mask, int64_t BH) {
    return !has_mask && (D == 64 || D == 128) && S >= 128 && BH <= 65535 && (S + BQ - 1) / BQ <= 65535;
}

size_t attention_tc_workspace(int64_t BHkv, int64_t S, int D) {
    const size_t tile = D == 128 ? AttnTcCfg<128>::TILE_BYTES : AttnTcCfg<64>::TILE_BYTES;
    return (size_t)BHkv * ((S + BKV - 1) / BKV) * tile;
}

Status attention_tc_prepare() {
    static bool done = false;
    if (!done) {
        RT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           AttnTcCfg<64>::SMEM));
        RT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<128, true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, AttnTcCfg<128>::SMEM));
        RT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<64, false>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, AttnTcCfg<64>::SMEM));
        RT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<128, false>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, AttnTcCfg<128>::SMEM));
        done = true;
    }
    return Status::ok();
}

Status launch_attention_tc(const AttnViews& vw, int64_t BH, int64_t S, int D, int group, int causal,
                           Workspace ws, cudaStream_t st, int* launches) {
    const int64_t BHkv = BH / group;
    if (ws.bytes < attention_tc_workspace(BHkv, S, D))
        return Status::err(RT_ERR_ARGUMENT, "attention: workspace too small");
    const int n_kv = (int)((S + BKV - 1) / BKV);
    dim3 pgrid((unsigned)n_kv, (unsigned)BHkv);
    KvViews kv{vw.k, vw.v, vw.k_sb, vw.k_sh, vw.k_ss, vw.v_sb, vw.v_sh, vw.v_ss, vw.H / group};
    uint8_t* kvbuf = reinterpret_cast<uint8_t*>(ws.base);
    const bool cross = attn_cross();
    if (D == 64 && cross) pack_kv_kernel<64, true><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv);
    else if (D == 64) pack_kv_kernel<64, false><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv);
    else if (cross) pack_kv_kernel<128, true><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv);
    else pack_kv_kernel<128, false><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv);
    RT_LAUNCH_CHECK();
    *launches += 1;
    AttnTcParams prm;
    memset(&prm, 0, sizeof prm);
    prm.kv = reinterpret_cast<const uint8_t*>(ws.base);
    prm.n_kv = n_kv;
    prm.q = vw.q;
    prm.o = vw.o;
    prm.q_sb = vw.q_sb; prm.q_sh = vw.q_sh; prm.q_ss = vw.q_ss;
    prm.o_sb = vw.o_sb; prm.o_sh = vw.o_sh; prm.o_ss = vw.o_ss;
    prm.H = vw.H;
    prm.S = (int)S;
    prm.group = group;
    prm.causal = causal;
    prm.n_qblocks = (int)((S + BQ - 1) / BQ);
    prm.heads_fast = attention_tc_workspace(BHkv, S, D) <= ((size_t)512 << 20) ? 1 : 0;
    prm.scale = 1.0f / sqrtf((float)D);
    prm.err = kernel_error_flag();
    *launches += 1;
    return D == 64 ? launch_tc<64>(prm, (int)BH, st) : launch_tc<128>(prm, (int)BH, st);
}

}  // namespace rt
