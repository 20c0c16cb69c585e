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
// Work item = 128 queries of one (batch, head); the grid is persistent (one
// CTA per SM looping over items) so that one item's prologue (Q load, first
// scores) and epilogue (last P.V, O store) overlap its neighbours'.  384
// threads:
//   warp 0     producer: per item, the raw Q rows (one bulk copy per row, once
//              the previous item's score MMAs are done with the Q space), then
//              32 KiB chunks through a shared-memory ring in exactly the order
//              the MMAs consume them -- K_0, K_1, V_0, K_2, V_1, ... (K tile =
//              D/32 chunks of 32 features x 128 keys, V^T tile = chunks of 32
//              or 64 keys x D), each chunk one contiguous bulk copy of a
//              pre-packed, pre-swizzled image;
//   warp 1     allocates TMEM and issues the MMAs from one thread:
//              S = Q.K^T (Q from shared memory), O_tile = P.V (P from TMEM),
//              each as hi.hi + the cross terms;
//              S_{j+1} runs while the softmax works on S_j;
//   warps 4-11 two threads per query row (64 keys and D/2 output columns
//              each; row maxima / sums exchanged through shared memory behind
//              bounded mbarrier waits): split the raw Q rows into the hi /
//              plane-1 layouts, then per tile read S from TMEM (freeing it),
//              mask, online softmax in log2 units, fold the previous O tile
//              into registers, write P's two planes to TMEM; after an item's
//              last tile, stage the next item's Q before the final O fold.
// TMEM columns: S [0,128) | P_hi [128,256) | P plane 1 [256,384) | O tile [384, 384+D).
// Plane 1 of every operand (Q, K, V in shared memory, P in TMEM) is lo as
// fp32, or for the cross scheme bf16 [hi | lo] (Q, P) / [lo | hi] (K, V) per
// 16-wide K block -- the same 4 bytes per element, so tiles and offsets are
// shared by both schemes.
// K and V are split, V transposed and both packed into per-tile images in the
// node's workspace by a bandwidth-bound pre-pass (pack_kv_kernel).  All waits
// are bounded (see sm100_ptx.h).
#include <float.h>

#include <algorithm>

#include "dev_math.h"
#include "gemm.h"
#include "sm100_ptx.h"

namespace rt {

int* kernel_error_flag();

namespace {

// Warpgroup 0: producer (warp 0), MMA issuer (warp 1), two idle warps;
// warpgroups 1-2: the softmax.  Launched at 168 registers a thread (384 x 168
// fit the SM's 64 Ki), then rebalanced: warpgroup 0 down to REG_CTRL, the
// softmax up to REG_SOFT (128 x 120 + 256 x 192 = 384 x 168).
#ifndef RT_ATTN_RING128
#define RT_ATTN_RING128 3   // ring stages at head_dim 128 (what the shared memory left by Q allows)
#endif
constexpr int BQ = 128, BKV = 128, SOFT_WARPS = 8, ATHREADS = 128 + 32 * SOFT_WARPS;
constexpr int REG_CTRL = 120, REG_SOFT = 192;
static_assert(128 * REG_CTRL + 32 * SOFT_WARPS * REG_SOFT <= ATHREADS * 168, "register split");
constexpr int CHUNK = 32 * 1024;                      // ring stage / packed chunk
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr int ERR_A_PROD = 0x201, ERR_A_MMA = 0x202, ERR_A_SOFT = 0x203, ERR_A_DRAIN = 0x204;
constexpr uint32_t COL_S = 0, COL_PH = 128, COL_PL = 256, COL_O = 384;   // fp16 mode: P (h | l) at COL_PH
// fp16 mode: the Q plane is staged in TMEM (columns COL_QT.., 16 per 16
// features: 8 of h pairs, then 8 of l pairs), so the S MMAs read only K from
// shared memory (1B-8K B1: 801 -> 790 us).  RT_ATTN_QTMEM=0 builds the
// shared-memory form.
#ifndef RT_ATTN_QTMEM
#define RT_ATTN_QTMEM 1
#endif
constexpr bool Q_TMEM = RT_ATTN_QTMEM != 0;
constexpr uint32_t COL_QT = COL_PL;
// Operand modes: three tf32 MMAs, tf32 + bf16 cross terms, or scaled fp16
// hi / lo (three kind::f16 MMAs, one plane per operand: see below).
constexpr int AM_3XTF32 = 0, AM_CROSS = 1, AM_F16 = 2;
constexpr int FOLD_EVERY = 3;              // P.V tiles accumulated in TMEM between register folds
constexpr float RESCALE_LOG2 = 8.0f;       // a row keeps its reference max until a tile max exceeds it by this

// Tiles: tf32 modes -- Q hi and plane 1 (two Q_BYTES), K chunks of 32
// features x 128 keys (hi | plane 1), V^T chunks of D x V_KEYS keys (hi |
// plane 1); fp16 mode -- one Q plane, K chunks of 64 features x 128 keys,
// V^T chunks of D x 64 (D = 128) or D x 128 (D = 64) keys, each a 128-byte
// swizzled row per 32 elements of K holding [h | l] / [l | h] per 16.
template <int D, bool F16 = false>
struct AttnTcCfg {
    static constexpr int Q_BYTES = D * BQ * 4;                  // one Q plane: D/32 x [128][128 B]
    static constexpr int Q_PLANES = F16 ? 1 : 2;
    static constexpr int K_CHUNKS = F16 ? D / 64 : D / 32;
    static constexpr int V_KEYS = F16 ? (D == 128 ? 64 : 128) : (D == 128 ? 32 : 64);   // keys per V chunk
    static constexpr int V_CHUNKS = BKV / V_KEYS;
    static constexpr int TILE_BYTES = (K_CHUNKS + V_CHUNKS) * CHUNK;
    static constexpr int STAGES = F16 ? (D == 128 ? 4 : 5) : (D == 128 ? RT_ATTN_RING128 : 5);
    static constexpr int BAR_BYTES = 384;                       // mbarriers, TMEM slot, flags, item ring
    static constexpr int BODY = Q_PLANES * Q_BYTES + STAGES * CHUNK + BAR_BYTES +
                                (F16 ? 6 : 4) * BQ * 4 /*row exchange: maxima / sums (+ Q maxima)*/;
    static constexpr int SMEM = 232448;                         // the per-CTA maximum; BODY + alignment slack
    static_assert(BODY + 512 <= SMEM, "shared memory budget");
    static_assert(COL_O + D <= 512, "TMEM budget");
};

struct AttnTcParams {
    CUtensorMap tq;      // Q as {32-feature blocks: D, rows, heads, batch} (middle two in stride order)
    int q_rows_dim;      // which tensor-map dim (1 or 2) runs over rows; the other over heads
    const uint8_t* kv;   // packed tiles [BHkv][n_kv][K chunks | V chunks]
    int n_kv;            // key tiles per head
    const float* kscale; // fp16 mode: 2^-e per 32-key group [BHkv][n_kv][4]
    const unsigned* vmax;   // fp16 mode: |V| maximum per kv head (float bits) [BHkv]
    const float* q;
    float* o;
    int64_t q_sb, q_sh, q_ss;   // element strides of Q: batch, head, sequence (features contiguous)
    int64_t o_sb, o_sh, o_ss;   // same for O
    int H;                      // query heads per batch element
    int S, group, causal, n_qblocks;
    int BH, n_items;            // (batch, head) pairs; work items = BH x query blocks
    int head_group;             // item order: groups of this many (batch, head) pairs, heads fastest inside
    int* counter;               // next item to take (zeroed by the pack kernel before each launch)
    uint8_t* ox;                // non-null: O written as a GEMM's split A planes (hi at o, plane 1 here)
    int ox_cross;
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

// Softmax-side conversions on the integer / FMA pipes.  The conversion
// instructions (cvt to tf32 or bf16x2) issue on the same narrow pipe as ex2,
// and with one exponential per score that pipe bounded the softmax.
// tf32 (nearest, ties away) of a finite x by integer rounding of its magnitude
// bits: the same value cvt.rna.tf32.f32 gives.
__device__ __forceinline__ float tf32_rna_int(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}
// bf16 by truncation (upper halves) of two values, `a` in the low half.  Used
// for P's plane 1 only: the cross terms carry a relative weight of 2^-11, so
// truncation's 2^-8 (against 2^-9 for nearest) moves a product by ~2^-19.
__device__ __forceinline__ uint32_t bf16x2_trunc(float a, float b) {
    return __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x7632);
}
// bf16 (nearest, ties to even) of two finite values by integer rounding,
// `a` in the low half: the same bits as cvt.rn.bf16x2.f32.
__device__ __forceinline__ uint32_t bf16x2_rn_int(float a, float b) {
    const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    return ((ua + 0x7FFFu + ((ua >> 16) & 1u)) >> 16) | ((ub + 0x7FFFu + ((ub >> 16) & 1u)) & 0xFFFF0000u);
}
// 2^x with the hardware approximation (flushes results below 2^-126 to 0;
// 2^-inf = 0, which the causal mask relies on).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
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
__global__ void __launch_bounds__(256) pack_kv_kernel(KvViews kv, uint8_t* __restrict__ out, int S, int n_kv,
                                                      int* counter) {
    using C = AttnTcCfg<D>;
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *counter = 0;   // the attention kernel's item counter
    constexpr int PER = 32 * D / 4 / 256;   // 4-element units per thread, of K and of V
    __shared__ float sv[32][D + 1];
    // one block = 32 keys (sub-block `sub` of key tile j): all global loads first
    const int j = blockIdx.x >> 2, sub = blockIdx.x & 3, h = blockIdx.y;
    const int k0 = j * BKV + sub * 32;
    uint8_t* tile = out + ((size_t)h * n_kv + j) * C::TILE_BYTES;
    const int bb = h / kv.Hkv, hh = h % kv.Hkv;
    const float* kb = kv.k + bb * kv.k_sb + hh * kv.k_sh;
    const float* vb = kv.v + bb * kv.v_sb + hh * kv.v_sh;
    float4 xk[PER], xv[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int u = threadIdx.x + i * 256, r = u / (D / 4), d = (u % (D / 4)) * 4;
        const bool in = k0 + r < S;
        xk[i] = in ? *reinterpret_cast<const float4*>(kb + (int64_t)(k0 + r) * kv.k_ss + d) : make_float4(0.f, 0.f, 0.f, 0.f);
        xv[i] = in ? *reinterpret_cast<const float4*>(vb + (int64_t)(k0 + r) * kv.v_ss + d) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // K: unit = 4 consecutive features of one key
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int u = threadIdx.x + i * 256, r = u / (D / 4), d = (u % (D / 4)) * 4;
        sv[r][d] = xv[i].x; sv[r][d + 1] = xv[i].y; sv[r][d + 2] = xv[i].z; sv[r][d + 3] = xv[i].w;
        const float4 x = xk[i];
        const float4 hi = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
        uint8_t* kc = tile + (size_t)(d >> 5) * CHUNK;
        *reinterpret_cast<float4*>(kc + swz(sub * 32 + r, d & 31)) = hi;
        put_plane1<CROSS, false>(kc + CHUNK / 2, sub * 32 + r, d & 31, hi,
                                 make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w));
    }
    __syncthreads();
    // V^T: unit = 4 consecutive keys of one feature
    const int vc = (sub * 32) / C::V_KEYS, vsub = ((sub * 32) % C::V_KEYS) >> 5;
    uint8_t* vcp = tile + (size_t)(C::K_CHUNKS + vc) * CHUNK + (size_t)vsub * D * 128;
    for (int u = threadIdx.x; u < D * 8; u += blockDim.x) {
        const int d = u >> 3, w = (u & 7) * 4;
        const float4 x = make_float4(sv[w][d], sv[w + 1][d], sv[w + 2][d], sv[w + 3][d]);
        const float4 hi = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
        *reinterpret_cast<float4*>(vcp + swz(d, w)) = hi;
        put_plane1<CROSS, false>(vcp + CHUNK / 2, d, w, hi,
                                 make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w));
    }
}

// ---- fp16 mode: K / V packing --------------------------------------------
// Byte `b` (0..127) of row `row` of a [rows][128 B] block as the 128-byte
// swizzle mode reads it.
__device__ __forceinline__ uint32_t swzb(int row, int b) {
    return (uint32_t)row * 128 + ((((uint32_t)b >> 4) ^ ((uint32_t)row & 7)) << 4) + ((uint32_t)b & 15);
}
// Four consecutive K-dim elements e..e+3 (e % 4 == 0, e < 32: position in a
// 128-byte row of 32 elements), already scaled, as fp16 h / l into a B-role
// row ([l(16) | h(16)] per 16).
__device__ __forceinline__ void put_f16_b4(uint8_t* blk, int row, int e, float4 x) {
    const float h0 = round11(x.x), h1 = round11(x.y), h2 = round11(x.z), h3 = round11(x.w);
    const int b = (e >> 4) * 64 + (e & 15) * 2;
    *reinterpret_cast<uint2*>(blk + swzb(row, b)) =
        make_uint2(f16x2_rn(x.x - h0, x.y - h1), f16x2_rn(x.z - h2, x.w - h3));
    *reinterpret_cast<uint2*>(blk + swzb(row, b + 32)) = make_uint2(f16x2_rn(h0, h1), f16x2_rn(h2, h3));
}

// |V| maximum per kv head into vmax[h] (zeroed first; float bits).
template <int D>
__global__ void __launch_bounds__(256) v_absmax_kernel(KvViews kv, int S, unsigned* __restrict__ vmax) {
    const int h = blockIdx.y, bb = h / kv.Hkv, hh = h % kv.Hkv;
    const float* vb = kv.v + bb * kv.v_sb + hh * kv.v_sh;
    float m = 0.0f;
#pragma unroll 4
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)S * D / 4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t key = i / (D / 4), d = (i % (D / 4)) * 4;   // (D a constant: shifts)
        const float4 x = *reinterpret_cast<const float4*>(vb + key * kv.v_ss + d);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // one atomic per block (per-warp atomics on the BHkv words serialised)
    __shared__ float wm[8];
    if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
        for (int w = 1; w < 8; w++) m = fmaxf(m, wm[w]);
        atomicMax(vmax + h, __float_as_uint(m));
    }
}

// K (as K chunks of 64 features x 128 keys: two [128 keys][128 B] blocks) and
// V^T (V chunks of D x V_KEYS keys: [D][128 B] per 32 keys) of one 128-key
// tile in the fp16 mode.  K is scaled per 32 keys (this block's keys; its
// 2^-e to kscale), V per head (from vmax).  Keys past S are zero.
template <int D>
__global__ void __launch_bounds__(256) pack_kv16_kernel(KvViews kv, uint8_t* __restrict__ out, int S, int n_kv,
                                                        int* counter, float* __restrict__ kscale,
                                                        const unsigned* __restrict__ vmax) {
    using C = AttnTcCfg<D, true>;
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *counter = 0;   // the attention kernel's item counter
    constexpr int PER = 32 * D / 4 / 256;   // 4-element units per thread, of K and of V
    __shared__ float sv[32][D + 1];
    __shared__ float wmax[8];
    const int j = blockIdx.x >> 2, sub = blockIdx.x & 3, h = blockIdx.y;
    const int k0 = j * BKV + sub * 32;
    uint8_t* tile = out + ((size_t)h * n_kv + j) * C::TILE_BYTES;
    const int bb = h / kv.Hkv, hh = h % kv.Hkv;
    const float* kb = kv.k + bb * kv.k_sb + hh * kv.k_sh;
    const float* vb = kv.v + bb * kv.v_sb + hh * kv.v_sh;
    float4 xk[PER], xv[PER];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int u = threadIdx.x + i * 256, r = u / (D / 4), d = (u % (D / 4)) * 4;
        const bool in = k0 + r < S;
        xk[i] = in ? *reinterpret_cast<const float4*>(kb + (int64_t)(k0 + r) * kv.k_ss + d) : make_float4(0.f, 0.f, 0.f, 0.f);
        xv[i] = in ? *reinterpret_cast<const float4*>(vb + (int64_t)(k0 + r) * kv.v_ss + d) : make_float4(0.f, 0.f, 0.f, 0.f);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(xk[i].x), fabsf(xk[i].y)), fmaxf(fabsf(xk[i].z), fabsf(xk[i].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    m = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; w++) m = fmaxf(m, wmax[w]);
    const int ek = f16_scale_exp(m);
    const float sk = pow2i(ek);
    if (threadIdx.x == 0) kscale[((size_t)h * n_kv + j) * 4 + sub] = pow2i(-ek);
    const float svs = pow2i(f16_scale_exp(__uint_as_float(vmax[h])));
    // K: unit = 4 consecutive features of one key
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int u = threadIdx.x + i * 256, r = u / (D / 4), d = (u % (D / 4)) * 4;
        sv[r][d] = xv[i].x; sv[r][d + 1] = xv[i].y; sv[r][d + 2] = xv[i].z; sv[r][d + 3] = xv[i].w;
        const float4 x = make_float4(xk[i].x * sk, xk[i].y * sk, xk[i].z * sk, xk[i].w * sk);
        uint8_t* kc = tile + (size_t)(d >> 6) * CHUNK + (size_t)((d >> 5) & 1) * (BKV * 128);
        put_f16_b4(kc, sub * 32 + r, d & 31, x);
    }
    __syncthreads();
    // V^T: unit = 4 consecutive keys of one feature
    const int vc = (sub * 32) / C::V_KEYS, vsub = ((sub * 32) % C::V_KEYS) >> 5;
    uint8_t* vcp = tile + (size_t)(C::K_CHUNKS + vc) * CHUNK + (size_t)vsub * D * 128;
    for (int u = threadIdx.x; u < D * 8; u += blockDim.x) {
        const int d = u >> 3, w = (u & 7) * 4;
        const float4 x = make_float4(sv[w][d] * svs, sv[w + 1][d] * svs, sv[w + 2][d] * svs, sv[w + 3][d] * svs);
        put_f16_b4(vcp, d, w, x);
    }
}

// One work item = 128 queries of one (batch, head).  The grid is persistent
// (one CTA per SM); each CTA's producer takes the next item from a global
// counter, so items run in their list order across the GPU as on a plain
// grid -- longest causal blocks first, and the items in flight share few
// heads' K/V in L2 -- with no per-CTA start-up per item.  Item order: heads
// in groups whose packed K/V totals ~48 MB (RT_ATTN_GROUP_MB overrides),
// inside a group all heads' longest query block first, then the next
// longest; measured against all heads at once (GPT-2: 100 MB of K/V in
// flight) and 16 MB groups, 48 MB was fastest on every config here.
struct AttnItem {
    int bh, q0, n_tiles;
};

__device__ __forceinline__ void attn_decode(const AttnTcParams& p, int L, AttnItem& it) {
    const int per = p.head_group * p.n_qblocks;   // items per head group
    const int g = L / per, r = L - g * per;
    const int gh = min(p.head_group, p.BH - g * p.head_group);
    const int bh = g * p.head_group + r % gh;
    const int qi = r / gh;
    const int qb = p.causal ? p.n_qblocks - 1 - qi : qi;
    it.bh = bh;
    it.q0 = qb * BQ;
    const int kv_len = p.causal ? min(p.S, it.q0 + BQ) : p.S;
    it.n_tiles = (kv_len + BKV - 1) / BKV;
}

template <int D, int MODE>
__global__ void __launch_bounds__(ATHREADS, 1) attn_tc_kernel(const __grid_constant__ AttnTcParams p) {
    constexpr bool CROSS = MODE == AM_CROSS, F16 = MODE == AM_F16;
    using C = AttnTcCfg<D, F16>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* qh = smem;
    uint8_t* ql = qh + C::Q_BYTES;                // (tf32 modes: Q plane 1)
    uint8_t* ring = qh + C::Q_PLANES * C::Q_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + STAGES * CHUNK);
    uint64_t* full = bars;                        // [STAGES]
    uint64_t* empty = bars + STAGES;              // [STAGES]
    uint64_t* s_full = bars + 2 * STAGES;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_full + 2;
    uint64_t* pv_full = s_full + 3;
    uint64_t* q_ready = s_full + 4;               // Q planes written (per item)
    uint64_t* drain = s_full + 5;
    uint64_t* q_full = s_full + 6;                // raw Q block landed (per item)
    uint64_t* q_free = s_full + 7;                // the item's score MMAs done: Q space reusable
    uint64_t* pair_bar = s_full + 8;              // [4 quarters][3]
    uint64_t* item_full = pair_bar + 12;          // [4] item ring slot written (producer -> the other roles)
    uint64_t* qpair = item_full + 4;              // [4 quarters] Q row maxima exchanged (fp16 mode, per item)
    constexpr int NBAR = 2 * STAGES + 8 + 12 + 4 + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued = const_cast<int*>(abort_flag) + 1;    // [STAGES + 1] phase of the last load (ring, Q), -1 none
    volatile int* items = issued + STAGES + 1;         // [4] item ring: item r in slot r % 4, -1 = no more
    volatile int* pv_fresh = items + 4;                // [2] per tile parity: P.V starts a new O accumulator
    static_assert(NBAR * 8 + 8 + 4 * (STAGES + 1) + 16 + 8 <= C::BAR_BYTES, "barrier area");
    float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);   // [2][2][128]
    float* qred = red + 4 * BQ;                                                                  // [2][128]
    if ((smem - smem_raw) + C::BODY > C::SMEM) {   // dynamic shared memory less aligned than assumed
        if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, 0x205);
        return;
    }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; i++) {
            uint32_t cnt = 1;
            if (&bars[i] == s_free || &bars[i] == p_full || &bars[i] == q_ready) cnt = 32 * SOFT_WARPS;
            if ((&bars[i] >= pair_bar && &bars[i] < item_full) || (&bars[i] >= qpair && &bars[i] < qpair + 4)) cnt = 64;
            ptx::mbar_init(&bars[i], cnt);
        }
        for (int s = 0; s <= STAGES; s++) issued[s] = -1;
        *abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 1) ptx::tmem_alloc(tmem_slot, 512);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Item r for the MMA / softmax roles: 1 = got it, 0 = no more items, -1 = wait abandoned.
    // Slot r % 4 is rewritten for item r + 4 only after every role has moved past item r + 2.
    auto take = [&](int r, AttnItem& it, int code) -> int {
        if (!ptx::wait_bounded(&item_full[r & 3], (r >> 2) & 1, abort_flag, p.err, code, WAIT_NS)) return -1;
        const int L = items[r & 3];
        if (L < 0) return 0;
        attn_decode(p, L, it);
        return 1;
    };
    if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_CTRL));
    if (warp == 0) {
        // ---------------------------------------------------- producer
        // Per item: the raw Q block (D/32 tensor-map loads of 128 rows x 32
        // features, 128-byte swizzled into the hi plane's place, rows past S
        // zero-filled; once the previous item's score MMAs are done with the
        // Q planes), then the K/V chunks.
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
            AttnItem it;
            for (int r = 0; ok; r++) {
                const int L = atomicAdd(p.counter, 1);
                items[r & 3] = L < p.n_items ? L : -1;
                ptx::mbar_arrive(&item_full[r & 3]);
                if (L >= p.n_items) break;
                attn_decode(p, L, it);
                if (r > 0 && !(ok = ptx::wait_bounded(q_free, (r - 1) & 1, abort_flag, p.err, ERR_A_PROD, WAIT_NS)))
                    break;
                const int h = it.bh % p.H, b = it.bh / p.H;
                const int c1 = p.q_rows_dim == 1 ? it.q0 : h, c2 = p.q_rows_dim == 1 ? h : it.q0;
                ptx::mbar_expect_tx(q_full, (uint32_t)C::Q_BYTES);
                issued[STAGES] = r & 1;
                for (int blk = 0; blk < D / 32; blk++)
                    ptx::tma_load_4d(qh + blk * BQ * 128, &p.tq, q_full, blk * 32, c1, c2, b);
                const uint8_t* kv = p.kv + (size_t)(it.bh / p.group) * p.n_kv * C::TILE_BYTES;
                for (int c = 0; c < C::K_CHUNKS; c++) push(kv + c * CHUNK);
                for (int j = 0; j < it.n_tiles && ok; j++) {
                    if (j + 1 < it.n_tiles)
                        for (int c = 0; c < C::K_CHUNKS; c++) push(kv + (size_t)(j + 1) * C::TILE_BYTES + c * CHUNK);
                    for (int c = 0; c < C::V_CHUNKS; c++)
                        push(kv + (size_t)j * C::TILE_BYTES + (C::K_CHUNKS + c) * CHUNK);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = ptx::idesc_tf32(BQ, BKV);
            constexpr uint32_t idesc_o = ptx::idesc_tf32(BQ, D);
            constexpr uint32_t idesc_sx = ptx::idesc_bf16(BQ, BKV);
            constexpr uint32_t idesc_ox = ptx::idesc_bf16(BQ, D);
            constexpr uint32_t idesc_sh = ptx::idesc_f16(BQ, BKV);
            constexpr uint32_t idesc_oh = ptx::idesc_f16(BQ, D);
            int stage = 0;
            uint32_t ph = 0;
            bool ok = true;
            // 128-byte-swizzle descriptor of ring stage 0; stage s starts CHUNK * s
            // bytes later (the start-address field counts 16-byte units and the
            // whole shared window fits it, so the offset adds without carry)
            const uint64_t ring_desc0 = ptx::smem_desc(ring, 1024, 2);
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
                    if (F16) {
                        // 64 features: two 32-feature blocks of Q ([h | l] per 16) and of
                        // K ([l | h] per 16); per 16 features h.h, h.l, l.h
#pragma unroll
                        for (int cs = 0; cs < 2; cs++)
#pragma unroll
                            for (int j = 0; j < 2; j++) {
                                const uint8_t* a = qh + (c * 2 + cs) * BQ * 128 + j * 64;
                                const uint8_t* b = buf + cs * BKV * 128 + j * 64;
                                if (Q_TMEM) {
                                    // descriptors from the stage's precomputed base + constant offsets
                                    const uint64_t bl = ring_desc0 + (uint64_t)stage * (CHUNK >> 4) +
                                                        (uint64_t)((cs * BKV * 128 + j * 64) >> 4);
                                    ptx::mma_f16x3_ts(tmem + COL_S, tmem + COL_QT + (uint32_t)((c * 2 + cs) * 32 + j * 16),
                                                      bl + 2, bl, idesc_sh, (c | cs | j) ? 1u : 0u);
                                    continue;
                                }
                                ptx::mma_bf16(tmem + COL_S, ptx::smem_desc(a, 1024, 2), ptx::smem_desc(b + 32, 1024, 2),
                                              idesc_sh, (c | cs | j) ? 1u : 0u);
                                ptx::mma_bf16(tmem + COL_S, ptx::smem_desc(a, 1024, 2), ptx::smem_desc(b, 1024, 2),
                                              idesc_sh, 1u);
                                ptx::mma_bf16(tmem + COL_S, ptx::smem_desc(a + 32, 1024, 2),
                                              ptx::smem_desc(b + 32, 1024, 2), idesc_sh, 1u);
                            }
                        release();
                        continue;
                    }
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
            auto issue_pv = [&](bool fresh) {
                for (int c = 0; c < C::V_CHUNKS; c++) {
                    uint8_t* buf = pop();
                    if (!buf) return;
                    if (F16) {
                        // V_KEYS keys: [D][128 B] per 32 keys ([l | h] per 16); P in TMEM as
                        // 16 columns per 16 keys (8 of h, then 8 of l)
#pragma unroll
                        for (int sb = 0; sb < C::V_KEYS / 32; sb++)
#pragma unroll
                            for (int j = 0; j < 2; j++) {
                                const uint64_t bl = ring_desc0 + (uint64_t)stage * (CHUNK >> 4) +
                                                    (uint64_t)((sb * D * 128 + j * 64) >> 4);
                                ptx::mma_f16x3_ts(tmem + COL_O,
                                                  tmem + COL_PH + (uint32_t)((c * C::V_KEYS + sb * 32 + j * 16)),
                                                  bl + 2, bl, idesc_oh, (c | sb | j | !fresh) ? 1u : 0u);
                            }
                        release();
                        continue;
                    }
                    const uint64_t bh0 = ptx::smem_desc(buf, 1024, 2);
                    const uint64_t bl0 = ptx::smem_desc(buf + CHUNK / 2, 1024, 2);
#pragma unroll
                    for (int kk = 0; kk < C::V_KEYS / 8; kk++) {
                        const uint64_t off = (uint64_t)((((kk >> 2) * D * 128) + (kk & 3) * 32) >> 4);
                        const uint32_t kc = c * C::V_KEYS + kk * 8;
                        ptx::mma_tf32_ts(tmem + COL_O, tmem + COL_PH + kc, bh0 + off, idesc_o,
                                         (c | kk | !fresh) ? 1u : 0u);
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
            // T counts tiles over all items: the per-tile barriers flip once per tile.
            int T = 0;
            AttnItem it;
            for (int r = 0; ok; r++) {
                const int got = take(r, it, ERR_A_MMA);
                if (got <= 0) {
                    ok = got == 0;
                    break;
                }
                if (!(ok = ptx::wait_bounded(q_ready, r & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS))) break;
                // S of the previous item's last tile read out of TMEM
                if (T > 0 && !(ok = ptx::wait_bounded(s_free, (T - 1) & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS)))
                    break;
                ptx::tc_fence_after();
                issue_s();
                if (ok && it.n_tiles == 1) ptx::mma_commit(q_free);
                for (int j = 0; j < it.n_tiles && ok; j++, T++) {
                    if (j + 1 < it.n_tiles) {   // S_{j+1} once the softmax has read S_j out of TMEM
                        if (!(ok = ptx::wait_bounded(s_free, T & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS))) break;
                        ptx::tc_fence_after();
                        issue_s();
                        if (ok && j + 2 == it.n_tiles) ptx::mma_commit(q_free);
                    }
                    if (!ok) break;
                    if (!(ok = ptx::wait_bounded(p_full, T & 1, abort_flag, p.err, ERR_A_MMA, WAIT_NS))) break;
                    ptx::tc_fence_after();
                    issue_pv(pv_fresh[T & 1] != 0);
                }
            }
            ptx::mma_commit(drain);
            volatile int no_abort = 0;
            ptx::wait_bounded(drain, 0, &no_abort, p.err, ERR_A_DRAIN, WAIT_NS);
        }
        __syncwarp();
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_SOFT));
        // ---------------------------------------------------- softmax rows (warps 4..11)
        const int quarter = warp & 3;   // TMEM lanes 32*quarter.. are this warp's rows
        const int half = (warp - 4) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        constexpr int DH = D / 2, KH = BKV / 2;   // per-thread output columns / score columns
        const float sl2 = p.scale * 1.4426950408889634f;   // scores in log2 units: exp(x) = 2^(x log2 e)
        auto pair_sync = [&](int which, uint32_t parity) -> bool {
            uint64_t* b = &pair_bar[quarter * 3 + which];
            ptx::mbar_arrive(b);
            return ptx::wait_bounded(b, parity, abort_flag, p.err, ERR_A_SOFT, WAIT_NS);
        };
        // This thread's half of its Q row: the raw values sit where their hi
        // parts go (the load used the planes' swizzle), so each thread splits
        // its own elements in place and writes plane 1 beside them.
        float qinv_staged = 1.0f;   // fp16 mode: 2^-e of the staged item's Q row
        auto stage_q = [&](int r) -> bool {
            if (!ptx::wait_bounded(q_full, r & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS)) return false;
            if (F16) {
                // the row's maximum over both halves, then each 32-feature block of
                // this half rewritten in place as the fp16 plane ([h | l] per 16)
                float mx = 0.0f;
#pragma unroll 4
                for (int i = 0; i < DH; i += 4) {
                    const int d = half * DH + i;
                    const float4 v = *reinterpret_cast<const float4*>(qh + (uint32_t)(d >> 5) * BQ * 128 + swz(row, d & 31));
                    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                }
                qred[half * BQ + row] = mx;
                ptx::mbar_arrive(&qpair[quarter]);
                if (!ptx::wait_bounded(&qpair[quarter], r & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS)) return false;
                mx = fmaxf(mx, qred[(half ^ 1) * BQ + row]);
                const int e = f16_scale_exp(mx);
                const float sc = pow2i(e);
                qinv_staged = pow2i(-e);
#pragma unroll
                for (int cb = 0; cb < DH / 32; cb++) {
                    uint8_t* blk = qh + (uint32_t)(half * (DH / 32) + cb) * BQ * 128;
                    float x[32];
#pragma unroll
                    for (int w = 0; w < 32; w += 4) {
                        const float4 v = *reinterpret_cast<const float4*>(blk + swz(row, w));
                        x[w] = v.x * sc; x[w + 1] = v.y * sc; x[w + 2] = v.z * sc; x[w + 3] = v.w * sc;
                    }
#pragma unroll
                    for (int f16b = 0; f16b < 2; f16b++) {   // features 16*f16b .. +15
                        uint32_t hw[8], lw[8];
#pragma unroll
                        for (int t = 0; t < 8; t++) {
                            const float a = x[f16b * 16 + 2 * t], b = x[f16b * 16 + 2 * t + 1];
                            const float ha = round11(a), hb = round11(b);
                            hw[t] = f16x2_rn(ha, hb);
                            lw[t] = f16x2_rn(a - ha, b - hb);
                        }
                        if (Q_TMEM) {
                            uint32_t pr[16];
#pragma unroll
                            for (int t = 0; t < 8; t++) {
                                pr[t] = hw[t];
                                pr[8 + t] = lw[t];
                            }
                            ptx::tmem_st16(tmem + lane_off + COL_QT + (uint32_t)((half * (DH / 16) + cb * 2 + f16b) * 16),
                                           pr);
                            continue;
                        }
                        *reinterpret_cast<uint4*>(blk + swzb(row, f16b * 64)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                        *reinterpret_cast<uint4*>(blk + swzb(row, f16b * 64 + 16)) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                        *reinterpret_cast<uint4*>(blk + swzb(row, f16b * 64 + 32)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                        *reinterpret_cast<uint4*>(blk + swzb(row, f16b * 64 + 48)) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                    }
                }
                if (Q_TMEM) {
                    ptx::tmem_st_wait();
                    ptx::tc_fence_before();
                }
                ptx::fence_proxy_async_smem();
                ptx::mbar_arrive(q_ready);
                return true;
            }
#pragma unroll 4
            for (int i = 0; i < DH; i += 4) {
                const int d = half * DH + i;
                const uint32_t at = (uint32_t)(d >> 5) * BQ * 128 + swz(row, d & 31);
                const float4 v = *reinterpret_cast<const float4*>(qh + at);
                const float4 h = make_float4(tf32_round(v.x), tf32_round(v.y), tf32_round(v.z), tf32_round(v.w));
                *reinterpret_cast<float4*>(qh + at) = h;
                put_plane1<CROSS, true>(ql + (uint32_t)(d >> 5) * BQ * 128, row, d & 31, h,
                                        make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w));
            }
            ptx::fence_proxy_async_smem();
            ptx::mbar_arrive(q_ready);
            return true;
        };

        bool ok = true;
        int T = 0;
        AttnItem it;
        int got = take(0, it, ERR_A_SOFT);
        if (got < 0) ok = false;
        if (got > 0) ok = stage_q(0);
        for (int r = 0; ok; r++) {
            if ((got = take(r, it, ERR_A_SOFT)) <= 0) {
                ok = got == 0;
                break;
            }
            const int q = it.q0 + row;
            const float qinv = qinv_staged;   // fp16 mode: this item's Q row scale (1 otherwise)
            const int bhkv = it.bh / p.group;
            const float vinv = F16 ? pow2i(-f16_scale_exp(__uint_as_float(p.vmax[bhkv]))) : 1.0f;
            float m = -FLT_MAX, l = 0.0f;   // m in log2 units; -FLT_MAX as the reference's initial max
            int pend = 0;                   // P.V tiles accumulated in TMEM since the last fold
            float o[DH];
#pragma unroll
            for (int i = 0; i < DH; i++) o[i] = 0.0f;
            for (int j = 0; j < it.n_tiles; j++, T++) {
                // fp16 mode: scores in log2 units need 2^-e of the Q row and of the
                // tile's 32-key K groups (two per thread), loaded before the wait
                float f0 = sl2, f1 = sl2;
                if (F16) {
                    const float* ks = p.kscale + ((size_t)bhkv * p.n_kv + j) * 4 + half * 2;
                    f0 = sl2 * qinv * ks[0];
                    f1 = sl2 * qinv * ks[1];
                }
                if (!(ok = ptx::wait_bounded(s_full, T & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS))) break;
                ptx::tc_fence_after();
                float sv[KH];
                {
                    uint32_t rr[KH];
#pragma unroll
                    for (int c16 = 0; c16 < KH / 16; c16++)
                        ptx::tmem_ld16(tmem + lane_off + COL_S + half * KH + c16 * 16,
                                       *reinterpret_cast<uint32_t(*)[16]>(&rr[c16 * 16]));
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < KH; i++) sv[i] = __uint_as_float(rr[i]);   // raw: scaled in the exponent
                }
                ptx::tc_fence_before();
                ptx::mbar_arrive(s_free);   // S may be overwritten by the next tile's MMAs
                const int k0 = j * BKV + half * KH;
                const bool full_tile = k0 + KH <= p.S && (!p.causal || k0 + KH - 1 <= q);
                // maxima of the raw scores per 32-key group, then scaled (f0, f1 > 0)
                float g0 = -INFINITY, g1 = -INFINITY;
                if (full_tile) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        g0 = max3f(g0, sv[i], sv[i + 1]);
                        g1 = max3f(g1, sv[32 + i], sv[32 + i + 1]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < KH; i++) {
                        const int kj = k0 + i;
                        if (kj >= p.S || (p.causal && kj > q)) sv[i] = -INFINITY;
                        if (i < 32) g0 = fmaxf(g0, sv[i]);
                        else g1 = fmaxf(g1, sv[i]);
                    }
                }
                float mt = fmaxf(g0 * f0, g1 * f1);
                red[((T & 1) * 2 + half) * BQ + row] = mt;
                if (!(ok = pair_sync(T & 1, (T >> 1) & 1))) break;
                mt = fmaxf(mt, red[((T & 1) * 2 + (half ^ 1)) * BQ + row]);
                // Lazy rescaling: the row's reference max m stays put until a
                // tile's max exceeds it by more than 2^RESCALE_LOG2 (P <= 2^8
                // meanwhile), and O accumulates in TMEM over up to FOLD_EVERY
                // tiles before it is folded into registers (the same bounded
                // accumulation length as the GEMM's K chunks).  A row that does
                // rescale between folds scales its pending TMEM O in place.
                const bool first = j == 0;
                const bool fold = !first && pend >= FOLD_EVERY;   // uniform: one accumulator per tile
                float m_new = m;
                if (first || mt > m + RESCALE_LOG2 || (fold && mt > m)) m_new = mt > m ? mt : m;
                unsigned long long lt2 = pk2(0.0f, 0.0f);
                {
                    const unsigned long long ff0 = pk2(f0, f0), ff1 = pk2(f1, f1), mm = pk2(-m_new, -m_new);
#pragma unroll
                    for (int i = 0; i < KH; i += 2) {
                        float a, b;
                        upk2(fma2(pk2(sv[i], sv[i + 1]), i < 32 ? ff0 : ff1, mm), a, b);
                        sv[i] = ex2_approx(a);   // masked: 2^-inf = 0
                        sv[i + 1] = ex2_approx(b);
                        lt2 = add2(lt2, pk2(sv[i], sv[i + 1]));
                    }
                }
                float lt;
                {
                    float a, b;
                    upk2(lt2, a, b);
                    lt = a + b;
                }
                const float corr = m_new > m ? ex2_approx(m - m_new) : 1.0f;
                if (!first) {   // PV of tile j-1 done: P may be overwritten, pending O is complete
                    if (!(ok = ptx::wait_bounded(pv_full, (T - 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS)))
                        break;
                    ptx::tc_fence_after();
                }
                if (fold) {   // pending O (relative to the old max) into registers
#pragma unroll
                    for (int g = 0; g < DH / 32; g++) {   // 32 columns per batch keeps registers in bounds
                        uint32_t rr[32];
                        ptx::tmem_ld16(tmem + lane_off + COL_O + half * DH + g * 32,
                                       *reinterpret_cast<uint32_t(*)[16]>(&rr[0]));
                        ptx::tmem_ld16(tmem + lane_off + COL_O + half * DH + g * 32 + 16,
                                       *reinterpret_cast<uint32_t(*)[16]>(&rr[16]));
                        ptx::tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i += 2)
                            upk2(add2(pk2(o[g * 32 + i], o[g * 32 + i + 1]),
                                      pk2(__uint_as_float(rr[i]), __uint_as_float(rr[i + 1]))),
                                 o[g * 32 + i], o[g * 32 + i + 1]);
                    }
                } else if (!first && __any_sync(0xffffffffu, m_new > m)) {
                    // rescale this warp's rows of the pending TMEM O (warp-collective;
                    // corr is 1 for the rows that keep their max)
#pragma unroll
                    for (int g = 0; g < DH / 16; g++) {
                        uint32_t rr[16];
                        const uint32_t at = tmem + lane_off + COL_O + half * DH + g * 16;
                        ptx::tmem_ld16(at, rr);
                        ptx::tmem_ld_wait();
                        const unsigned long long cc = pk2(corr, corr);
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            float a, b;
                            upk2(mul2(pk2(__uint_as_float(rr[i]), __uint_as_float(rr[i + 1])), cc), a, b);
                            rr[i] = __float_as_uint(a);
                            rr[i + 1] = __float_as_uint(b);
                        }
                        ptx::tmem_st16(at, rr);
                    }
                    ptx::tmem_st_wait();
                }
                if (m_new > m) {   // running max grew: rescale the folded part (corr would be 1 otherwise)
                    l *= corr;
                    const unsigned long long cc = pk2(corr, corr);
#pragma unroll
                    for (int i = 0; i < DH; i += 2) upk2(mul2(pk2(o[i], o[i + 1]), cc), o[i], o[i + 1]);
                    m = m_new;
                }
                l += lt;
                pend = (first || fold) ? 1 : pend + 1;
                if (threadIdx.x == 128) pv_fresh[T & 1] = (first || fold) ? 1 : 0;   // PV_j starts a new accumulator
#pragma unroll
                for (int c16 = 0; c16 < KH / 16; c16++) {
                    uint32_t ph[16], pl[16];
                    if (F16) {   // 16 columns per 16 keys: 8 of h pairs, then 8 of l pairs
#pragma unroll
                        for (int t = 0; t < 8; t++) {
                            // h: 11 significant bits by truncation (exact in fp16), l = x - h >= 0
                            const float a = sv[c16 * 16 + 2 * t], b = sv[c16 * 16 + 2 * t + 1];
                            const float ha = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
                            const float hb = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
                            float la, lb;
                            upk2(sub2(pk2(a, b), pk2(ha, hb)), la, lb);
                            ph[t] = f16x2_rn(ha, hb);
                            ph[8 + t] = f16x2_rn(la, lb);
                        }
                        ptx::tmem_st16(tmem + lane_off + COL_PH + half * KH + c16 * 16, ph);
                        continue;
                    }
                    if (CROSS) {   // plane 1: 8 columns of bf16 pairs of hi, then 8 of lo
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            const float a = sv[c16 * 16 + i], b = sv[c16 * 16 + i + 1];
                            const float ha = tf32_rna_int(a), hb = tf32_rna_int(b);
                            ph[i] = __float_as_uint(ha);
                            ph[i + 1] = __float_as_uint(hb);
                            pl[i / 2] = bf16x2_trunc(ha, hb);
                            pl[8 + i / 2] = bf16x2_trunc(a - ha, b - hb);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            const float pv = sv[c16 * 16 + i];
                            const float h = tf32_rna_int(pv);
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
            if (!ok) break;
            // Row sum over both halves.  The exchange slot of parity T & 1 was
            // last read for tile T - 2; the next item's first tile reuses it only
            // after every softmax thread has arrived on q_ready in stage_q below.
            red[((T & 1) * 2 + half) * BQ + row] = l;
            const bool paired = pair_sync(2, r & 1);
            l += red[((T & 1) * 2 + (half ^ 1)) * BQ + row];
            if (!paired) {
                ok = false;
                break;
            }
            // The next item's Q while this item's last P.V runs.
            AttnItem nx;
            if ((got = take(r + 1, nx, ERR_A_SOFT)) < 0) {
                ok = false;
                break;
            }
            if (got > 0 && !(ok = stage_q(r + 1))) break;
            if (!(ok = ptx::wait_bounded(pv_full, (T - 1) & 1, abort_flag, p.err, ERR_A_SOFT, WAIT_NS))) break;
            ptx::tc_fence_after();
#pragma unroll
            for (int g = 0; g < DH / 32; g++) {
                uint32_t rr[32];
                ptx::tmem_ld16(tmem + lane_off + COL_O + half * DH + g * 32, *reinterpret_cast<uint32_t(*)[16]>(&rr[0]));
                ptx::tmem_ld16(tmem + lane_off + COL_O + half * DH + g * 32 + 16,
                               *reinterpret_cast<uint32_t(*)[16]>(&rr[16]));
                ptx::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) o[g * 32 + i] += __uint_as_float(rr[i]);
            }
            ptx::tc_fence_before();
            if (q < p.S) {
                const float inv = vinv / l;   // (fp16 mode: V was scaled by 1 / vinv)
                const int64_t e0 = (int64_t)(it.bh / p.H) * p.o_sb + (int64_t)(it.bh % p.H) * p.o_sh +
                                   (int64_t)q * p.o_ss + half * DH;
                float* orow = p.o + e0;
                if (!p.ox) {
#pragma unroll
                    for (int i = 0; i < DH; i += 4)
                        *reinterpret_cast<float4*>(orow + i) =
                            make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
                } else {
                    // split planes of the next GEMM's A operand: hi here, plane 1 at the
                    // same element offsets; e0 starts a 16-wide K block (D/2 is a multiple of 16)
#pragma unroll
                    for (int i = 0; i < DH; i += 16) {
                        uint32_t hb[8], lb[8];
#pragma unroll
                        for (int t = 0; t < 16; t += 4) {
                            const float4 v = make_float4(o[i + t] * inv, o[i + t + 1] * inv, o[i + t + 2] * inv,
                                                         o[i + t + 3] * inv);
                            const float4 h = make_float4(tf32_rna_int(v.x), tf32_rna_int(v.y), tf32_rna_int(v.z),
                                                         tf32_rna_int(v.w));
                            const float4 lo = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
                            *reinterpret_cast<float4*>(orow + i + t) = h;
                            if (p.ox_cross) {
                                hb[t / 2] = bf16x2_rn_int(h.x, h.y);
                                hb[t / 2 + 1] = bf16x2_rn_int(h.z, h.w);
                                lb[t / 2] = bf16x2_rn_int(lo.x, lo.y);
                                lb[t / 2 + 1] = bf16x2_rn_int(lo.z, lo.w);
                            } else {
                                *reinterpret_cast<float4*>(p.ox + (e0 + i + t) * 4) = lo;
                            }
                        }
                        if (p.ox_cross) {
                            uint4* blk = reinterpret_cast<uint4*>(p.ox + (e0 + i) * 4);   // 64 bytes: hi | lo
                            blk[0] = make_uint4(hb[0], hb[1], hb[2], hb[3]);
                            blk[1] = make_uint4(hb[4], hb[5], hb[6], hb[7]);
                            blk[2] = make_uint4(lb[0], lb[1], lb[2], lb[3]);
                            blk[3] = make_uint4(lb[4], lb[5], lb[6], lb[7]);
                        }
                    }
                }
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
        if (issued[STAGES] >= 0)
            ptx::wait_bounded(q_full, (uint32_t)issued[STAGES], &no_abort, nullptr, 0, 100000000ull);
    }
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

// Operand mode: fp16 (default), RT_ATTN_SCHEME=cross for tf32 + bf16 cross
// terms, RT_ATTN_3XTF32=1 (or RT_ATTN_SCHEME=3xtf32) for three tf32 MMAs.
int attn_mode() {
    static const int v = [] {
        const char* t = getenv("RT_ATTN_3XTF32");
        const char* e = getenv("RT_ATTN_SCHEME");
        if ((t && t[0] == '1') || (e && !strcmp(e, "3xtf32"))) return AM_3XTF32;
        if (e && !strcmp(e, "cross")) return AM_CROSS;
        return AM_F16;
    }();
    return v;
}

template <int D>
Status launch_tc(const AttnTcParams& prm, int BH, cudaStream_t st) {
    (void)BH;
    const dim3 grid((unsigned)min(prm.n_items, g_num_sms));   // persistent: one CTA per SM
    if (attn_mode() == AM_F16)
        attn_tc_kernel<D, AM_F16><<<grid, ATHREADS, AttnTcCfg<D, true>::SMEM, st>>>(prm);
    else if (attn_mode() == AM_CROSS)
        attn_tc_kernel<D, AM_CROSS><<<grid, ATHREADS, AttnTcCfg<D>::SMEM, st>>>(prm);
    else
        attn_tc_kernel<D, AM_3XTF32><<<grid, ATHREADS, AttnTcCfg<D>::SMEM, st>>>(prm);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

// fp16 mode workspace after the packed tiles: K group scales, V head maxima.
size_t tiles_bytes(int64_t BHkv, int64_t S, int D) {
    const bool f16 = attn_mode() == AM_F16;
    const size_t tile = D == 128 ? (f16 ? AttnTcCfg<128, true>::TILE_BYTES : AttnTcCfg<128>::TILE_BYTES)
                                 : (f16 ? AttnTcCfg<64, true>::TILE_BYTES : AttnTcCfg<64>::TILE_BYTES);
    return (size_t)BHkv * ((S + BKV - 1) / BKV) * tile;
}
size_t scales_bytes(int64_t BHkv, int64_t S) {
    if (attn_mode() != AM_F16) return 0;
    return ((size_t)BHkv * ((S + BKV - 1) / BKV) * 4 * 4 + (size_t)BHkv * 4 + 255) & ~(size_t)255;
}

}  // namespace

// Shapes this kernel takes: no custom mask, head_dim 64 or 128, at least one
// full 128-query block.
bool attention_tc_applicable(int64_t S, int D, bool has_mask, int64_t BH) {
    return !has_mask && (D == 64 || D == 128) && S >= 128 && BH * ((S + BQ - 1) / BQ) <= INT32_MAX;
}

size_t attention_tc_workspace(int64_t BHkv, int64_t S, int D) {
    return tiles_bytes(BHkv, S, D) + scales_bytes(BHkv, S) + 256;   // + the item counter
}

Status attention_tc_prepare() {
    static bool done = false;
    if (!done) {
        const void* ks[] = {(const void*)attn_tc_kernel<64, AM_F16>, (const void*)attn_tc_kernel<128, AM_F16>,
                            (const void*)attn_tc_kernel<64, AM_CROSS>, (const void*)attn_tc_kernel<128, AM_CROSS>,
                            (const void*)attn_tc_kernel<64, AM_3XTF32>, (const void*)attn_tc_kernel<128, AM_3XTF32>};
        for (const void* k : ks)   // every configuration uses the per-CTA maximum (AttnTcCfg::SMEM)
            RT_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnTcCfg<64>::SMEM));
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
    dim3 pgrid((unsigned)(n_kv * 4), (unsigned)BHkv);
    KvViews kv{vw.k, vw.v, vw.k_sb, vw.k_sh, vw.k_ss, vw.v_sb, vw.v_sh, vw.v_ss, vw.H / group};
    uint8_t* kvbuf = reinterpret_cast<uint8_t*>(ws.base);
    int* counter = reinterpret_cast<int*>(kvbuf + attention_tc_workspace(BHkv, S, D) - 256);
    const int mode = attn_mode();
    const bool cross = mode == AM_CROSS;
    float* kscale = reinterpret_cast<float*>(kvbuf + tiles_bytes(BHkv, S, D));
    unsigned* vmax = reinterpret_cast<unsigned*>(kscale + (size_t)BHkv * n_kv * 4);
    if (mode == AM_F16) {
        RT_CUDA_CHECK(cudaMemsetAsync(vmax, 0, (size_t)BHkv * 4, st));
        const int per_head = (int)std::max<int64_t>(1, std::min<int64_t>(128, (S * D / 4 + 2047) / 2048));
        if (D == 64) v_absmax_kernel<64><<<dim3((unsigned)per_head, (unsigned)BHkv), 256, 0, st>>>(kv, (int)S, vmax);
        else v_absmax_kernel<128><<<dim3((unsigned)per_head, (unsigned)BHkv), 256, 0, st>>>(kv, (int)S, vmax);
        RT_LAUNCH_CHECK();
        *launches += 1;
        if (D == 64) pack_kv16_kernel<64><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv, counter, kscale, vmax);
        else pack_kv16_kernel<128><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv, counter, kscale, vmax);
    } else if (D == 64 && cross) pack_kv_kernel<64, true><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv, counter);
    else if (D == 64) pack_kv_kernel<64, false><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv, counter);
    else if (cross) pack_kv_kernel<128, true><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv, counter);
    else pack_kv_kernel<128, false><<<pgrid, 256, 0, st>>>(kv, kvbuf, (int)S, n_kv, counter);
    RT_LAUNCH_CHECK();
    *launches += 1;
    AttnTcParams prm;
    memset(&prm, 0, sizeof prm);
    prm.kv = reinterpret_cast<const uint8_t*>(ws.base);
    prm.n_kv = n_kv;
    prm.kscale = kscale;
    prm.vmax = vmax;
    prm.q = vw.q;
    prm.o = vw.o;
    prm.q_sb = vw.q_sb; prm.q_sh = vw.q_sh; prm.q_ss = vw.q_ss;
    prm.o_sb = vw.o_sb; prm.o_sh = vw.o_sh; prm.o_ss = vw.o_ss;
    prm.H = vw.H;
    prm.S = (int)S;
    prm.group = group;
    prm.causal = causal;
    prm.n_qblocks = (int)((S + BQ - 1) / BQ);
    prm.BH = (int)BH;
    prm.n_items = (int)(BH * prm.n_qblocks);
    prm.counter = counter;
    prm.ox = vw.ox;
    prm.ox_cross = vw.ox_cross;
    {   // heads of one group together hold at most ~budget bytes of packed K/V
        size_t budget = (size_t)48 << 20;
        if (const char* e = getenv("RT_ATTN_GROUP_MB")) budget = (size_t)atoll(e) << 20;
        const size_t per_head = tiles_bytes(1, S, D) / group;
        prm.head_group = (int)std::max<int64_t>(1, std::min<int64_t>(BH, (int64_t)(budget / per_head)));
    }
    prm.scale = 1.0f / sqrtf((float)D);
    {   // Q tensor map: rows and heads ordered by stride (the driver wants them increasing)
        const bool rows_first = vw.q_ss <= vw.q_sh;
        const int64_t B = BH / vw.H;
        const int64_t dims[4] = {D, rows_first ? S : vw.H, rows_first ? vw.H : S, B};
        const int64_t strides[3] = {4 * (rows_first ? vw.q_ss : vw.q_sh), 4 * (rows_first ? vw.q_sh : vw.q_ss),
                                    4 * vw.q_sb};
        const int box[4] = {32, rows_first ? BQ : 1, rows_first ? 1 : BQ, 1};
        Status s = encode_tmap_f32(&prm.tq, vw.q, 4, dims, strides, box, 128);
        if (!s.good()) return s;
        prm.q_rows_dim = rows_first ? 1 : 2;
    }
    prm.err = kernel_error_flag();
    *launches += 1;
    return D == 64 ? launch_tc<64>(prm, (int)BH, st) : launch_tc<128>(prm, (int)BH, st);
}

}  // namespace rt
