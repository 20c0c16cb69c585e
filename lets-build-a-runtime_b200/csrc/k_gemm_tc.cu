// k_gemm_tc.cu -- MATMUL / MATMUL_ADD on the 5th-generation tensor cores.
//
// fp32 accuracy from reduced-precision tensor cores.  Every operand x is
// written as hi + lo with hi = x rounded to tf32 (cvt.rna.tf32.f32, low 13
// mantissa bits zero) and lo = x - hi (exact in fp32, |lo| <= 2^-11 |x|), and
//     A.B ~= A_hi.B_hi + A_hi.B_lo + A_lo.B_hi
// (the dropped A_lo.B_lo term is ~2^-22 relative).  Two ways to issue it:
//
//  * tf32 + bf16 cross terms (default): A_hi.B_hi is one kind::tf32 MMA (a
//    product of two tf32 values is exact in fp32); the two cross terms only
//    need ~8 significant bits each, so they run as ONE kind::f16 (bf16) MMA
//    over a doubled K: A' = [bf16(A_hi) | bf16(A_lo)], B' = [bf16(B_lo) |
//    bf16(B_hi)].  Rounding the cross operands to bf16 costs ~2^-19 of
//    |a||b| per product.  bf16 MMAs run at twice the tf32 rate, so a K block
//    takes 4 MMA instructions instead of 6 (1.5x less tensor time).
//  * 3xTF32 (RT_GEMM_3XTF32=1): three kind::tf32 MMAs, hi.hi + hi.lo + lo.hi.
//
// Both schemes store two planes per operand, K-major, 4 bytes per element:
// plane 0 = hi (tf32 in fp32 words); plane 1 = lo (fp32) for 3xTF32, or the
// "cross" plane for the default: per row and per K block of 16 (width w =
// min(16, K - 16*kb)), 2w bf16 values [first(0..w-1) | second(0..w-1)] in the
// block's 64 bytes, first/second = hi/lo for A and lo/hi for B.  The same
// 64-byte TMA box serves both; a short last block lands its second half where
// the first MMA still reads it and the rest is TMA zero fill.
//
// Constant B operands (weights) are split once per plan and cached; A
// (activations) is split per launch by a bandwidth-bound pre-pass into the
// node's workspace.
//
// The tensor core's fp32 accumulation does not round like IEEE adds, and its
// error grows with the number of MMAs summed into one accumulator (measured
// on B200: 1.5e-3 max abs at K=16384 with one accumulator per tile).  So each
// tile's K is accumulated in TMEM in chunks (256 by default) and the chunk
// sums are added in fp32 registers on the CUDA cores.  Measured max error
// against fp64, per sqrt(K), unit-variance operands, K = 768..16384: 4.8e-6
// (chunk 128), 7.2e-6 (256), 1.1e-5 (384), 1.9e-5 (768) -- numpy's fp32
// sgemm: 2.2e-6; a longer chunk means fewer accumulator hand-offs to the
// epilogue (GPT-2 body: 1.50 ms at 128, 1.45 ms at 256).
//
// Kernel: persistent, one CTA per SM, 320 threads in three roles:
//   warp 0     TMA producer: per K-block, four tile loads (A plane 0/1,
//              B plane 0/1; 64-byte swizzle, 64 bytes of K per row) into a
//              4-stage shared-memory ring;
//   warp 1     allocates 512 TMEM columns (two 128x256 fp32 accumulators)
//              and issues the tcgen05.mma (M=128, N=256) from one thread;
//              tcgen05.commit frees ring stages and publishes each finished
//              K chunk;
//   warps 2-9  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//              lanes 32*(w%4)..+31 = tile rows, one half of the columns),
//              sums the chunks in registers, then alpha / bias and one
//              store to C -- overlapping the next chunk's / tile's MMAs.
// Every mbarrier wait is bounded (ptx::wait_bounded); on timeout the kernel
// records an error code in host-mapped memory, drains its copies and MMAs
// (bounded), frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "dev_math.h"
#include "gemm.h"
#include "sm100_ptx.h"

namespace rt {

int* kernel_error_flag();   // runtime.cu: device view of the host-mapped error word

namespace {

constexpr int BM = 128, BK = 16;
constexpr int EPI_WARPS = 8;                          // 2 warps per TMEM lane quarter
constexpr int THREADS = 64 + 32 * EPI_WARPS;          // producer + MMA + epilogue
constexpr int A_TILE = BM * BK * 4;                   // 8 KiB

// Operand schemes (see the file comment): three tf32 MMAs, tf32 + bf16
// cross terms, or three fp16 MMAs over one scaled fp16 plane per operand.
constexpr int SCH_3XTF32 = 0, SCH_CROSS = 1, SCH_F16 = 2;

// N tile 256 or 128.  tf32 schemes: two 4-byte planes per operand, a 4-stage
// ring of 48 KiB (N 256) or 6 stages of 32 KiB; fp16: one plane, 8 stages of
// 24 KiB or 12 of 16 KiB.  K per stage: 16 (64-byte rows, 64-byte swizzle).
template <int BN_, int SCH>
struct GCfg {
    static constexpr int BN = BN_;
    static constexpr bool F16 = SCH == SCH_F16;
    static constexpr int STAGES = F16 ? (BN_ == 256 ? 8 : 12) : (BN_ == 256 ? 4 : 6);
    static constexpr int EPI_COLS = BN_ / 2;
    static constexpr int B_TILE = BN_ * BK * 4;
    static constexpr int STAGE_BYTES = (F16 ? 1 : 2) * (A_TILE + B_TILE);
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 512 /*barriers*/;
};
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;     // 2 s per wait
constexpr int ERR_PRODUCER = 0x101, ERR_MMA = 0x102, ERR_EPILOGUE = 0x103, ERR_DRAIN = 0x104;

struct TcParams {
    CUtensorMap ta_hi, ta_lo, tb_hi, tb_lo;   // 3-D {K, rows, batches}
    CUtensorMap tc;                           // C as 3-D {N, M, batches}, 32 x 32 boxes, 128-B swizzle
    int c_tma;                                // pair kernel: C through shared memory and TMA stores
    int vec_c;                                // 16-byte row accesses: N % 4 == 0 and C, bias, residual 16-byte aligned
    float* c;
    const float* bias;
    const float* res;             // non-null: residual [batches*M][N] added after the bias (first split)
    float alpha;
    int M, N, K, batches;
    int m_tiles, n_tiles, k_blocks, total_tiles;
    int kb_per_chunk, n_chunks;   // K accumulated in TMEM in chunks of kb_per_chunk blocks
    int splits, kb_split;         // split-K: work item = (tile, split); split s covers K blocks [s*kb_split, ...)
    int total_items;              // total_tiles * splits
    int act;                      // 1: tanh-GELU after alpha and bias
    int gate;                     // 1 / 2: gated output (B rows in the gated order): C[r][j] = act(g) * u,
                                  //   act SiLU / tanh-GELU, C has N / 2 columns
    const float* a_scale;         // fp16 scheme: 2^-e per A row ([batches*M]); null = 1
    const float* b_scale;         // fp16 scheme: 2^-e of the whole B operand (one float); null = 1
    float* plane_hi;              // non-null: write the result as split A planes (hi, plane 1) of a
    uint8_t* plane_x;             //   later GEMM instead of C (row-major [batches*M][N])
    int plane_mode;               //   plane 1: 0 = lo (fp32), 1 = cross (bf16 [hi | lo] per 16 block);
                                  //   2 = fp16 plane at plane_hi ([h | l] per 16 block, 2N halves per row)
                                  //   and 2^-e per 128-column segment at plane_x ([rows][N / 128] floats)
    const float* a_seg;           // A arrived as an fp16 plane with 2^-e per (row, 128 K): one TMEM chunk
    int a_segs;                   //   of 128 K per segment; a_segs = segments per row
    int* err;
};

__device__ __forceinline__ float tf32_hi(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}
__device__ __forceinline__ uint16_t bf16_bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// A folded residual (alpha == 1): on the first split, a full-width row's COLS
// residual values go straight into the accumulator registers before the
// tile's first TMEM chunk is awaited (the loads overlap the MMAs); the TMEM
// chunks are then added to them.  Returns whether it did (otherwise store_row
// adds the residual).
template <int COLS>
__device__ __forceinline__ bool load_residual(const TcParams& p, int64_t row, int bz, int col0, bool first_split,
                                              float* acc) {
    if (!first_split || row >= p.M || !p.vec_c || col0 + COLS > p.N) return false;
    const float* src = p.res + ((int64_t)bz * p.M + row) * p.N + col0;
#pragma unroll
    for (int j = 0; j < COLS; j += 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + j);
        acc[j] = v.x; acc[j + 1] = v.y; acc[j + 2] = v.z; acc[j + 3] = v.w;
    }
    return true;
}

// Factor applied to the accumulator of output row `row` (batch bz) as the
// TMEM chunks are summed: alpha, times the fp16 scheme's 2^-e of the A row
// and of the B operand.
__device__ __forceinline__ float epi_factor(const TcParams& p, int64_t row, int bz) {
    float f = p.alpha;
    if (p.a_scale && row < p.M) f *= p.a_scale[(int64_t)bz * p.M + row];
    if (p.b_scale) f *= *p.b_scale;
    return f;
}
// A given as an fp16 plane with one 2^-e per (row, 128-wide K segment): the
// row's segment factors (one TMEM chunk spans one segment), or null.
__device__ __forceinline__ const float* seg_row(const TcParams& p, int64_t row, int bz) {
    return p.a_seg && row < p.M ? p.a_seg + ((int64_t)bz * p.M + row) * p.a_segs : nullptr;
}

// One epilogue row: COLS consecutive columns from col0 of output row `row`
// (within batch bz), accumulator already scaled by epi_factor: bias (first
// split only), optional GELU, then C
// (plain store, or float4 atomics under split-K) or, for PLANES kernels, the
// split A planes (a separate instantiation: the plane code's registers would
// otherwise cost every GEMM's epilogue).
template <int COLS, bool PLANES, bool RESID = true>
__device__ __forceinline__ void store_row(const TcParams& p, int64_t row, int bz, int col0, float* acc,
                                          bool first_split, bool res_in_acc) {
    const bool add_bias = p.bias && first_split;
    const bool add_res = RESID && p.res && first_split && !res_in_acc;   // RESID: compiled in at all
    const int64_t r = (int64_t)bz * p.M + row;
    if (PLANES && COLS == 128 && p.plane_mode == 2) {
        // fp16 plane of the consuming GEMM's A: this thread's 128 columns are
        // one 128-wide K segment of that GEMM, scaled by their own maximum
        // (N % 128 == 0 here, so a segment is whole or past the end)
        if (col0 >= p.N) return;
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < COLS; j++) {
            float x = acc[j];
            if (add_bias) x += p.bias[col0 + j];
            if (p.act == 1) x = gelu_tanh(x);
            acc[j] = x;
            m = fmaxf(m, fabsf(x));
        }
        const int e = f16_scale_exp(m);
        const float sc = pow2i(e);
        reinterpret_cast<float*>(p.plane_x)[r * (p.N / 128) + col0 / 128] = pow2i(-e);
        uint16_t* prow = reinterpret_cast<uint16_t*>(p.plane_hi) + r * 2 * (int64_t)p.N;
        // one 16-column block = 64 bytes: 16 h halves, then 16 l halves
#pragma unroll
        for (int j = 0; j < COLS; j += 16) {
            uint32_t hw[8], lw[8];
#pragma unroll
            for (int t = 0; t < 16; t += 2) {
                const float x0 = acc[j + t] * sc, x1 = acc[j + t + 1] * sc;
                const float h0 = round11(x0), h1 = round11(x1);
                hw[t / 2] = f16x2_rn(h0, h1);
                lw[t / 2] = f16x2_rn(x0 - h0, x1 - h1);
            }
            uint4* blk = reinterpret_cast<uint4*>(prow + (int64_t)(col0 + j) * 2);
            blk[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            blk[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            blk[2] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            blk[3] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        }
        return;
    }
    if (PLANES) {
        // N % 4 == 0 here (it is the K of the consuming GEMM); splits == 1
        float* hrow = p.plane_hi + r * p.N;
        uint16_t* xrow = reinterpret_cast<uint16_t*>(p.plane_x + r * p.N * 4);
#pragma unroll
        for (int j = 0; j < COLS; j += 4) {
            const int col = col0 + j;
            if (col >= p.N) break;
            float h[4], l[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float v = acc[j + e];
                if (add_bias) v += p.bias[col + e];
                if (p.act == 1) v = gelu_tanh(v);
                h[e] = tf32_hi(v);
                l[e] = v - h[e];
            }
            *reinterpret_cast<float4*>(hrow + col) = make_float4(h[0], h[1], h[2], h[3]);
            if (p.plane_mode == 1) {
                // cross: bf16 [hi(0..w-1) | lo(0..w-1)] per 16-column block of width w
                const int kb = col >> 4, jj = col & 15, w = min(16, p.N - kb * 16);
                uint16_t* blk = xrow + kb * 32;
                uint2 f, g;
                f.x = (uint32_t)bf16_bits(h[0]) | ((uint32_t)bf16_bits(h[1]) << 16);
                f.y = (uint32_t)bf16_bits(h[2]) | ((uint32_t)bf16_bits(h[3]) << 16);
                g.x = (uint32_t)bf16_bits(l[0]) | ((uint32_t)bf16_bits(l[1]) << 16);
                g.y = (uint32_t)bf16_bits(l[2]) | ((uint32_t)bf16_bits(l[3]) << 16);
                *reinterpret_cast<uint2*>(blk + jj) = f;
                *reinterpret_cast<uint2*>(blk + w + jj) = g;
            } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(xrow) + col) =
                    make_float4(l[0], l[1], l[2], l[3]);
            }
        }
        return;
    }
    if (!PLANES && p.gate) {
        // this thread's COLS columns: COLS/2 gate values, then their COLS/2 up values
        constexpr int H = COLS / 2;
        const int64_t ldc = p.N / 2, c0 = col0 / 2;
        float* orow = p.c + r * ldc + c0;
#pragma unroll
        for (int j = 0; j < H; j += 4) {
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float g = acc[j + e], u = acc[H + j + e];
                o[e] = (p.gate == 1 ? silu(g) : gelu_tanh(g)) * u;
            }
            if (p.vec_c && c0 + j + 4 <= ldc) {
                *reinterpret_cast<float4*>(orow + j) = make_float4(o[0], o[1], o[2], o[3]);
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++)
                    if (c0 + j + e < ldc) orow[j + e] = o[e];
            }
        }
        return;
    }
    float* crow = p.c + r * p.N;
    if (p.vec_c && col0 + COLS <= p.N) {
#pragma unroll
        for (int j = 0; j < COLS; j += 4) {
            float4 v = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
            if (add_bias) {
                float4 bb = *reinterpret_cast<const float4*>(p.bias + col0 + j);
                v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
            }
            if (add_res) {   // alpha == 1 with a residual
                const float4 rr = *reinterpret_cast<const float4*>(p.res + r * p.N + col0 + j);
                v.x += rr.x; v.y += rr.y; v.z += rr.z; v.w += rr.w;
            }
            if (p.act == 1) {
                v.x = gelu_tanh(v.x); v.y = gelu_tanh(v.y); v.z = gelu_tanh(v.z); v.w = gelu_tanh(v.w);
            }
            // two splits add into a zeroed C: 0+x+y == 0+y+x, so the
            // result does not depend on which split lands first
            if (p.splits > 1) atomicAdd(reinterpret_cast<float4*>(crow + col0 + j), v);
            else *reinterpret_cast<float4*>(crow + col0 + j) = v;
        }
    } else {
#pragma unroll
        for (int j = 0; j < COLS; j++) {
            if (col0 + j < p.N) {
                float v = acc[j];
                if (add_bias) v += p.bias[col0 + j];
                if (add_res) v += p.res[r * p.N + col0 + j];   // alpha == 1 with a residual
                if (p.act == 1) v = gelu_tanh(v);
                if (p.splits > 1) atomicAdd(crow + col0 + j, v);
                else crow[col0 + j] = v;
            }
        }
    }
}

__device__ __forceinline__ void tile_coords(const TcParams& p, int item, int& m_blk, int& n_blk, int& bz,
                                            int& kb_lo, int& kb_hi) {
    const int t = item / p.splits, s = item % p.splits;
    n_blk = t % p.n_tiles;
    int rest = t / p.n_tiles;
    m_blk = rest % p.m_tiles;
    bz = rest / p.m_tiles;
    kb_lo = s * p.kb_split;
    kb_hi = min(p.k_blocks, kb_lo + p.kb_split);
}

template <int BN_, int SCH, bool PLANES>
__global__ void __launch_bounds__(THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
    using G = GCfg<BN_, SCH>;
    constexpr int BN = G::BN, STAGES = G::STAGES, EPI_COLS = G::EPI_COLS;
    constexpr int B_TILE = G::B_TILE, STAGE_BYTES = G::STAGE_BYTES;
    constexpr bool CROSS = SCH == SCH_CROSS, F16 = SCH == SCH_F16;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* full = bars;                        // [STAGES]
    uint64_t* empty = bars + STAGES;              // [STAGES]
    uint64_t* acc_full = bars + 2 * STAGES;       // [2]
    uint64_t* acc_empty = bars + 2 * STAGES + 2;  // [2]
    uint64_t* drain = bars + 2 * STAGES + 4;      // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued_phase = const_cast<int*>(abort_flag) + 1;   // [STAGES], -1 = nothing outstanding

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
            issued_phase[s] = -1;
        }
        for (int b = 0; b < 2; b++) {
            ptx::mbar_init(&acc_full[b], 1);
            ptx::mbar_init(&acc_empty[b], 32 * EPI_WARPS);
        }
        ptx::mbar_init(drain, 1);
        *abort_flag = 0;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&p.ta_hi);
        ptx::prefetch_tmap(&p.ta_lo);
        ptx::prefetch_tmap(&p.tb_hi);
        ptx::prefetch_tmap(&p.tb_lo);
    }
    if (warp == 1) ptx::tmem_alloc(tmem_slot, 512);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.total_items && ok; t += gridDim.x) {
                int m_blk, n_blk, bz, kb_lo, kb_hi;
                tile_coords(p, t, m_blk, n_blk, bz, kb_lo, kb_hi);
                for (int kb = kb_lo; kb < kb_hi; kb++) {
                    if (!ptx::wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, ERR_PRODUCER,
                                           WAIT_LIMIT_NS)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + stage * STAGE_BYTES;
                    ptx::mbar_expect_tx(&full[stage], STAGE_BYTES);
                    issued_phase[stage] = (int)phase;
                    int k0 = kb * BK;
                    if (F16) {   // one fp16 plane per operand: 2 halves per element of K
                        ptx::tma_load_3d(st, &p.ta_hi, &full[stage], 2 * k0, m_blk * BM, bz);
                        ptx::tma_load_3d(st + A_TILE, &p.tb_hi, &full[stage], 2 * k0, n_blk * BN, bz);
                    } else {
                        ptx::tma_load_3d(st, &p.ta_hi, &full[stage], k0, m_blk * BM, bz);
                        ptx::tma_load_3d(st + A_TILE, &p.ta_lo, &full[stage], k0, m_blk * BM, bz);
                        ptx::tma_load_3d(st + 2 * A_TILE, &p.tb_hi, &full[stage], k0, n_blk * BN, bz);
                        ptx::tma_load_3d(st + 2 * A_TILE + B_TILE, &p.tb_lo, &full[stage], k0, n_blk * BN, bz);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::idesc_tf32(BM, BN);
            constexpr uint32_t idesc_x = ptx::idesc_bf16(BM, BN);
            constexpr uint32_t idesc_h = ptx::idesc_f16(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int it = 0;   // accumulator hand-offs so far (one per K chunk)
            for (int t = blockIdx.x; t < p.total_items && ok; t += gridDim.x) {
                int m_blk, n_blk, bz, kb_lo, kb_hi;
                tile_coords(p, t, m_blk, n_blk, bz, kb_lo, kb_hi);
                const int n_chunks = (kb_hi - kb_lo + p.kb_per_chunk - 1) / p.kb_per_chunk;
                for (int c = 0; c < n_chunks && ok; c++, it++) {
                    int b = it & 1;
                    uint32_t acc_phase = (it >> 1) & 1;
                    if (!ptx::wait_bounded(&acc_empty[b], acc_phase ^ 1, abort_flag, p.err, ERR_MMA,
                                           WAIT_LIMIT_NS)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t d_tmem = tmem_base + b * BN;
                    const int kb0 = kb_lo + c * p.kb_per_chunk;
                    const int kb_end = min(kb_hi, kb0 + p.kb_per_chunk);
                    for (int kb = kb0; kb < kb_end; kb++) {
                        if (!ptx::wait_bounded(&full[stage], phase, abort_flag, p.err, ERR_MMA, WAIT_LIMIT_NS)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                        uint8_t* st = smem + stage * STAGE_BYTES;
                        const uint32_t acc0 = kb > kb0 ? 1u : 0u;
                        if (F16) {
                            // one 16-wide K block per stage: A row [h | l], B row [l | h]
                            // (32 bytes each): h.h, h.l, l.h
                            ptx::mma_bf16(d_tmem, ptx::smem_desc(st, 512, 4), ptx::smem_desc(st + A_TILE + 32, 512, 4),
                                          idesc_h, acc0);
                            ptx::mma_bf16(d_tmem, ptx::smem_desc(st, 512, 4), ptx::smem_desc(st + A_TILE, 512, 4),
                                          idesc_h, 1u);
                            ptx::mma_bf16(d_tmem, ptx::smem_desc(st + 32, 512, 4),
                                          ptx::smem_desc(st + A_TILE + 32, 512, 4), idesc_h, 1u);
                        } else if (CROSS) {
                            // hi.hi: two tf32 K=8 steps (+32 bytes each inside the 64-byte atom)
#pragma unroll
                            for (int kk = 0; kk < 2; kk++)
                                ptx::mma_tf32(d_tmem, ptx::smem_desc(st + kk * 32, 512, 4),
                                              ptx::smem_desc(st + 2 * A_TILE + kk * 32, 512, 4), idesc,
                                              (acc0 | kk) ? 1u : 0u);
                            // cross terms: two bf16 K=16 steps over the doubled K
#pragma unroll
                            for (int kk = 0; kk < 2; kk++)
                                ptx::mma_bf16(d_tmem, ptx::smem_desc(st + A_TILE + kk * 32, 512, 4),
                                              ptx::smem_desc(st + 2 * A_TILE + B_TILE + kk * 32, 512, 4),
                                              idesc_x, 1u);
                        } else {
#pragma unroll
                            for (int kk = 0; kk < BK / 8; kk++) {
                                uint64_t a_hi = ptx::smem_desc(st + kk * 32, 512, 4);
                                uint64_t a_lo = ptx::smem_desc(st + A_TILE + kk * 32, 512, 4);
                                uint64_t b_hi = ptx::smem_desc(st + 2 * A_TILE + kk * 32, 512, 4);
                                uint64_t b_lo = ptx::smem_desc(st + 2 * A_TILE + B_TILE + kk * 32, 512, 4);
                                ptx::mma_tf32(d_tmem, a_hi, b_hi, idesc, (acc0 | kk) ? 1u : 0u);
                                ptx::mma_tf32(d_tmem, a_hi, b_lo, idesc, 1u);
                                ptx::mma_tf32(d_tmem, a_lo, b_hi, idesc, 1u);
                            }
                        }
                        ptx::mma_commit(&empty[stage]);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    ptx::mma_commit(&acc_full[b]);
                }
            }
            // every MMA this thread issued has completed once `drain` flips
            ptx::mma_commit(drain);
            volatile int no_abort = 0;
            ptx::wait_bounded(drain, 0, &no_abort, p.err, ERR_DRAIN, WAIT_LIMIT_NS);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (warps 2..9)
        // Thread = one tile row (TMEM lane) x BN/2 columns.
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < p.total_items && ok; t += gridDim.x) {
            int m_blk, n_blk, bz, kb_lo, kb_hi;
            tile_coords(p, t, m_blk, n_blk, bz, kb_lo, kb_hi);
            const int n_chunks = (kb_hi - kb_lo + p.kb_per_chunk - 1) / p.kb_per_chunk;
            const bool first_split = kb_lo == 0;
            const int64_t erow = (int64_t)m_blk * BM + quarter * 32 + lane;
            const float fac = epi_factor(p, erow, bz);
            const float* segp = seg_row(p, erow, bz);
            const int seg0 = kb_lo / p.kb_per_chunk;
            float acc[EPI_COLS];
            for (int c = 0; c < n_chunks; c++, it++) {
                const float fc = segp ? fac * segp[seg0 + c] : fac;
                int b = it & 1;
                uint32_t acc_phase = (it >> 1) & 1;
                // warp-uniform outcome: the stores below are warp-collective
                const bool got = ptx::wait_bounded(&acc_full[b], acc_phase, abort_flag, p.err, ERR_EPILOGUE,
                                                   WAIT_LIMIT_NS);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t tbase =
                    tmem_base + ((uint32_t)(quarter * 32) << 16) + b * BN + half * EPI_COLS;
#pragma unroll
                for (int q = 0; q < EPI_COLS / 16; q++) {
                    uint32_t r[16];
                    ptx::tmem_ld16(tbase + q * 16, r);
                    ptx::tmem_ld_wait();
                    const unsigned long long f2 = pk2(fc, fc);
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        const unsigned long long rv = pk2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                        upk2(c == 0 ? mul2(f2, rv) : fma2(f2, rv, pk2(acc[q * 16 + j], acc[q * 16 + j + 1])),
                             acc[q * 16 + j], acc[q * 16 + j + 1]);
                    }
                }
                ptx::tc_fence_before();
                ptx::mbar_arrive(&acc_empty[b]);
            }
            if (!ok) break;
            const int64_t row = (int64_t)m_blk * BM + quarter * 32 + lane;
            if (row < p.M) store_row<EPI_COLS, PLANES>(p, row, bz, n_blk * BN + half * EPI_COLS, acc, first_split, false);
        }
    }

    __syncthreads();
    if (threadIdx.x == 0 && *abort_flag) {
        // drain: copies still in flight land before the CTA's smem goes away
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; s++)
            if (issued_phase[s] >= 0)
                ptx::wait_bounded(&full[s], (uint32_t)issued_phase[s], &no_abort, nullptr, 0, 100000000ull);
    }
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, 512);
    }
}

// ---- CTA-pair kernel: 256 x 256 tiles on tcgen05 cta_group::2 -------------
// A cluster of two CTAs on two SMs computes one 256x256 tile per work item:
// each CTA loads its own 128 rows of A and 128 rows of B (a 128x256 operand
// slice per SM instead of 128x384), so shared-memory traffic per flop drops
// by a third -- the 1-CTA kernel is bound by shared-memory bandwidth (TMA
// writes plus MMA operand reads), not by the tensor pipe.
//   * both CTAs' copies complete on the LEADER's (rank 0) full barrier, whose
//     producer posts the expected bytes of both;
//   * the leader's MMA thread issues M=256 MMAs over the pair; its commits
//     arrive on the empty / accumulator-full barriers of both CTAs;
//   * each CTA's epilogue drains its own TMEM (its 128 rows) and releases the
//     accumulator on the leader's barrier (one arrival per warp).
// K block of 32 fp32 = one 128-byte swizzle row: half the TMA requests per
// byte of the 64-byte rows (the request path to L2 limits the 1-CTA kernel).
constexpr int P_BK = 32;
// Stage ring: tf32 schemes 3 stages of four planes (A hi / A plane 1 / B hi /
// B plane 1, 64 KiB), the fp16 scheme 6 stages of two (A / B, 32 KiB).
template <int SCH>
struct PCfg {
    static constexpr int STAGES = SCH == SCH_F16 ? 6 : 3;
    static constexpr int STAGE_BYTES = (SCH == SCH_F16 ? 2 : 4) * 128 * 32 * 4;
    static constexpr int EPI_OFF = STAGES * STAGE_BYTES + 1024;   // after the barriers, 1024-aligned
    static constexpr int SMEM = EPI_OFF + 8 * 32 * 32 * 4 + 1024;
    static_assert(SMEM <= 232448, "shared memory budget");
};
constexpr int P_STAGES = 3;
constexpr int P_TILE = 128 * P_BK * 4;                 // 16 KiB: one plane of 128 rows
constexpr int P_STAGE_BYTES = 4 * P_TILE;              // A hi / A plane1 / B hi / B plane1
constexpr int P_EPI_STAGE = 32 * 32 * 4;               // per epilogue warp: 32 rows x 32 columns of C
constexpr int P_EPI_OFF = P_STAGES * P_STAGE_BYTES + 1024;   // after the barriers, 1024-aligned
constexpr int P_SMEM_BYTES = P_EPI_OFF + 8 * P_EPI_STAGE + 1024;
static_assert(P_SMEM_BYTES <= 232448, "shared memory budget");
constexpr int P_EPI_COLS = 128;   // (two 16-column TMEM loads per wait measured 20-35 % slower:
                                   //  the register cap of 168 leaves no room for them)

template <int SCH, bool PLANES, bool RES = false, bool TMA = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ TcParams p) {
    constexpr int P_STAGES = PCfg<SCH>::STAGES, P_STAGE_BYTES = PCfg<SCH>::STAGE_BYTES, P_EPI_OFF = PCfg<SCH>::EPI_OFF;
    constexpr bool CROSS = SCH == SCH_CROSS, F16 = SCH == SCH_F16;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem =
        reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
    uint64_t* full = bars;                          // [P_STAGES] (leader's are used)
    uint64_t* empty = bars + P_STAGES;              // [P_STAGES]
    uint64_t* acc_full = bars + 2 * P_STAGES;       // [2]
    uint64_t* acc_empty = bars + 2 * P_STAGES + 2;  // [2]   (leader's are used)
    uint64_t* drain = bars + 2 * P_STAGES + 4;      // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued_phase = const_cast<int*>(abort_flag) + 1;   // [P_STAGES]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = ptx::cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
            issued_phase[s] = -1;
        }
        for (int b = 0; b < 2; b++) {
            ptx::mbar_init(&acc_full[b], 1);
            ptx::mbar_init(&acc_empty[b], 2 * EPI_WARPS);
        }
        ptx::mbar_init(drain, 1);
        *abort_flag = 0;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&p.ta_hi);
        ptx::prefetch_tmap(&p.ta_lo);
        ptx::prefetch_tmap(&p.tb_hi);
        ptx::prefetch_tmap(&p.tb_lo);
    }
    if (warp == 1) ptx::tmem_alloc_pair(tmem_slot, 512);
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();   // barriers of both CTAs initialised, TMEM of both allocated
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = cluster; t < p.total_items && ok; t += n_clusters) {
                int m_blk, n_blk, bz, kb_lo, kb_hi;
                tile_coords(p, t, m_blk, n_blk, bz, kb_lo, kb_hi);
                const int arow = m_blk * 256 + (int)rank * 128, brow = n_blk * 256 + (int)rank * 128;
                for (int kb = kb_lo; kb < kb_hi; kb++) {
                    if (!ptx::wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, ERR_PRODUCER,
                                           WAIT_LIMIT_NS)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + stage * P_STAGE_BYTES;
                    const uint32_t bar = ptx::mapa_shared(ptx::smem_u32(&full[stage]), 0);
                    if (leader) {
                        ptx::mbar_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
                        issued_phase[stage] = (int)phase;
                    }
                    const int k0 = kb * P_BK;
                    if (F16) {   // one fp16 plane per operand: 2 halves per element of K
                        ptx::tma_load_3d_pair(st, &p.ta_hi, bar, 2 * k0, arow, bz);
                        ptx::tma_load_3d_pair(st + P_TILE, &p.tb_hi, bar, 2 * k0, brow, bz);
                    } else {
                        ptx::tma_load_3d_pair(st, &p.ta_hi, bar, k0, arow, bz);
                        ptx::tma_load_3d_pair(st + P_TILE, &p.ta_lo, bar, k0, arow, bz);
                        ptx::tma_load_3d_pair(st + 2 * P_TILE, &p.tb_hi, bar, k0, brow, bz);
                        ptx::tma_load_3d_pair(st + 3 * P_TILE, &p.tb_lo, bar, k0, brow, bz);
                    }
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (leader only)
        if (leader && lane == 0) {
            constexpr uint32_t idesc = ptx::idesc_tf32(256, 256);
            constexpr uint32_t idesc_x = ptx::idesc_bf16(256, 256);
            constexpr uint32_t idesc_h = ptx::idesc_f16(256, 256);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int it = 0;
            for (int t = cluster; t < p.total_items && ok; t += n_clusters) {
                int m_blk, n_blk, bz, kb_lo, kb_hi;
                tile_coords(p, t, m_blk, n_blk, bz, kb_lo, kb_hi);
                const int n_chunks = (kb_hi - kb_lo + p.kb_per_chunk - 1) / p.kb_per_chunk;
                for (int c = 0; c < n_chunks && ok; c++, it++) {
                    const int b = it & 1;
                    const uint32_t acc_phase = (it >> 1) & 1;
                    if (!ptx::wait_bounded(&acc_empty[b], acc_phase ^ 1, abort_flag, p.err, ERR_MMA,
                                           WAIT_LIMIT_NS)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t d_tmem = tmem_base + b * 256;
                    const int kb0 = kb_lo + c * p.kb_per_chunk;
                    const int kb_end = min(kb_hi, kb0 + p.kb_per_chunk);
                    for (int kb = kb0; kb < kb_end; kb++) {
                        if (!ptx::wait_bounded(&full[stage], phase, abort_flag, p.err, ERR_MMA, WAIT_LIMIT_NS)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                        uint8_t* st = smem + stage * P_STAGE_BYTES;
                        const uint32_t acc0 = kb > kb0 ? 1u : 0u;
                        // K advance inside the 128-byte swizzle atom: +32 bytes per step
                        if (F16) {
                            // two 16-wide K blocks per 128-byte row: A [h | l], B [l | h]
                            // (32 bytes each); per block h.h, h.l, l.h
#pragma unroll
                            for (int j = 0; j < 2; j++) {
                                const uint8_t* a = st + j * 64;
                                const uint8_t* bb = st + P_TILE + j * 64;
                                ptx::mma_bf16_pair(d_tmem, ptx::smem_desc(a, 1024, 2), ptx::smem_desc(bb + 32, 1024, 2),
                                                   idesc_h, (acc0 | j) ? 1u : 0u);
                                ptx::mma_bf16_pair(d_tmem, ptx::smem_desc(a, 1024, 2), ptx::smem_desc(bb, 1024, 2),
                                                   idesc_h, 1u);
                                ptx::mma_bf16_pair(d_tmem, ptx::smem_desc(a + 32, 1024, 2),
                                                   ptx::smem_desc(bb + 32, 1024, 2), idesc_h, 1u);
                            }
                        } else if (CROSS) {
#pragma unroll
                            for (int kk = 0; kk < 4; kk++)
                                ptx::mma_tf32_pair(d_tmem, ptx::smem_desc(st + kk * 32, 1024, 2),
                                                   ptx::smem_desc(st + 2 * P_TILE + kk * 32, 1024, 2), idesc,
                                                   (acc0 | kk) ? 1u : 0u);
#pragma unroll
                            for (int kk = 0; kk < 4; kk++)
                                ptx::mma_bf16_pair(d_tmem, ptx::smem_desc(st + P_TILE + kk * 32, 1024, 2),
                                                   ptx::smem_desc(st + 3 * P_TILE + kk * 32, 1024, 2), idesc_x,
                                                   1u);
                        } else {
#pragma unroll
                            for (int kk = 0; kk < 4; kk++) {
                                uint64_t a_hi = ptx::smem_desc(st + kk * 32, 1024, 2);
                                uint64_t a_lo = ptx::smem_desc(st + P_TILE + kk * 32, 1024, 2);
                                uint64_t b_hi = ptx::smem_desc(st + 2 * P_TILE + kk * 32, 1024, 2);
                                uint64_t b_lo = ptx::smem_desc(st + 3 * P_TILE + kk * 32, 1024, 2);
                                ptx::mma_tf32_pair(d_tmem, a_hi, b_hi, idesc, (acc0 | kk) ? 1u : 0u);
                                ptx::mma_tf32_pair(d_tmem, a_hi, b_lo, idesc, 1u);
                                ptx::mma_tf32_pair(d_tmem, a_lo, b_hi, idesc, 1u);
                            }
                        }
                        ptx::mma_commit_pair(&empty[stage], 0x3);
                        if (++stage == P_STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    ptx::mma_commit_pair(&acc_full[b], 0x3);
                }
            }
            ptx::mma_commit_pair(drain, 0x1);
            volatile int no_abort = 0;
            ptx::wait_bounded(drain, 0, &no_abort, p.err, ERR_DRAIN, WAIT_LIMIT_NS);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (warps 2..9, both CTAs)
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const uint32_t acc_empty_leader0 = ptx::mapa_shared(ptx::smem_u32(&acc_empty[0]), 0);
        int it = 0;
        bool ok = true;
        for (int t = cluster; t < p.total_items && ok; t += n_clusters) {
            int m_blk, n_blk, bz, kb_lo, kb_hi;
            tile_coords(p, t, m_blk, n_blk, bz, kb_lo, kb_hi);
            const int n_chunks = (kb_hi - kb_lo + p.kb_per_chunk - 1) / p.kb_per_chunk;
            const bool first_split = kb_lo == 0;
            const int64_t erow = (int64_t)m_blk * 256 + rank * 128 + quarter * 32 + lane;
            const float fac = epi_factor(p, erow, bz);
            const float* segp = seg_row(p, erow, bz);
            const int seg0 = kb_lo / p.kb_per_chunk;
            float acc[P_EPI_COLS];
            // RES: a folded residual preloaded into the accumulator registers
            // (zeros on a second split); the TMEM chunks add to it
            const bool res_in_acc =
                RES && load_residual<P_EPI_COLS>(p, (int64_t)m_blk * 256 + rank * 128 + quarter * 32 + lane, bz,
                                                 n_blk * 256 + half * P_EPI_COLS, first_split, acc);
            if (RES && !res_in_acc)
#pragma unroll
                for (int j = 0; j < P_EPI_COLS; j++) acc[j] = 0.0f;
            for (int c = 0; c < n_chunks; c++, it++) {
                const float fc = segp ? fac * segp[seg0 + c] : fac;
                const int b = it & 1;
                const uint32_t acc_phase = (it >> 1) & 1;
                // warp-uniform outcome: the stores below are warp-collective
                const bool got = ptx::wait_bounded(&acc_full[b], acc_phase, abort_flag, p.err, ERR_EPILOGUE,
                                                   WAIT_LIMIT_NS);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t tbase =
                    tmem_base + ((uint32_t)(quarter * 32) << 16) + b * 256 + half * P_EPI_COLS;
#pragma unroll
                for (int q = 0; q < P_EPI_COLS / 16; q++) {
                    uint32_t r[16];
                    ptx::tmem_ld16(tbase + q * 16, r);
                    ptx::tmem_ld_wait();
                    const unsigned long long f2 = pk2(fc, fc);
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        const unsigned long long rv = pk2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                        upk2(c == 0 && !RES ? mul2(f2, rv) : fma2(f2, rv, pk2(acc[q * 16 + j], acc[q * 16 + j + 1])),
                             acc[q * 16 + j], acc[q * 16 + j + 1]);
                    }
                }
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive_cluster(acc_empty_leader0 + b * 8);
            }
            if (!ok) break;
            if (TMA) {
                // 32 columns at a time: this warp's 32 rows into its staging block
                // (128-byte swizzle), then one TMA store (reduce-add under split-K)
                uint8_t* stg = smem + P_EPI_OFF + (warp - 2) * P_EPI_STAGE;
                const int col0 = n_blk * 256 + half * P_EPI_COLS;
                const int row0 = m_blk * 256 + rank * 128 + quarter * 32;
                const bool add_bias = p.bias && first_split;
#pragma unroll
                for (int c4 = 0; c4 < P_EPI_COLS / 32; c4++) {
                    if (col0 + c4 * 32 >= p.N) continue;   // (not break: acc stays statically indexed)
                    if (lane == 0) ptx::bulk_wait_read();   // the previous store has read the block
                    __syncwarp();
#pragma unroll
                    for (int w = 0; w < 32; w += 4) {
                        const int j = c4 * 32 + w, col = col0 + j;
                        float4 v = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                        if (add_bias && col < p.N) {   // N % 4 == 0 with a C tensor map
                            const float4 bb = *reinterpret_cast<const float4*>(p.bias + col);
                            v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
                        }
                        if (p.act == 1) {
                            v.x = gelu_tanh(v.x); v.y = gelu_tanh(v.y); v.z = gelu_tanh(v.z); v.w = gelu_tanh(v.w);
                        }
                        *reinterpret_cast<float4*>(stg + lane * 128 + ((((w >> 2) ^ (lane & 7))) << 4)) = v;
                    }
                    ptx::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (p.splits > 1) ptx::tma_reduce_add_3d(&p.tc, stg, col0 + c4 * 32, row0, bz);
                        else ptx::tma_store_3d(&p.tc, stg, col0 + c4 * 32, row0, bz);
                        ptx::bulk_commit();
                    }
                }
            } else if (const int64_t row = (int64_t)m_blk * 256 + rank * 128 + quarter * 32 + lane; row < p.M) {
                store_row<P_EPI_COLS, PLANES, RES>(p, row, bz, n_blk * 256 + half * P_EPI_COLS, acc, first_split,
                                                   res_in_acc);
            }
        }
    }

    if (TMA) ptx::bulk_wait_all();   // C stores done before the CTA's memory goes
    __syncthreads();
    if (threadIdx.x == 0 && leader && *abort_flag) {
        volatile int no_abort = 0;
        for (int s = 0; s < P_STAGES; s++)
            if (issued_phase[s] >= 0)
                ptx::wait_bounded(&full[s], (uint32_t)issued_phase[s], &no_abort, nullptr, 0, 100000000ull);
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();   // the peer's copies, MMA reads and remote arrivals are over
    ptx::tc_fence_after();
    if (warp == 1) ptx::tmem_dealloc_pair(tmem_base, 512);
}

// ---- operand split: hi = tf32(x) (round to nearest), lo = x - hi ----------

// Plane-1 writer for element k of a row whose plane-1 row starts at `row1`
// (2K bf16 slots).  mode 0: lo as fp32; mode 1 (A): cross [hi | lo];
// mode 2 (B): cross [lo | hi].  See the file comment for the block layout.
__device__ __forceinline__ void put_plane1(float* row1, int64_t k, int64_t K, float h, float l, int mode) {
    if (mode == 0) {
        row1[k] = l;
        return;
    }
    const int64_t kb = k >> 4;
    const int j = (int)(k & 15);
    const int w = (int)min((int64_t)16, K - kb * 16);
    uint16_t* blk = reinterpret_cast<uint16_t*>(row1) + kb * 32;
    blk[j] = bf16_bits(mode == 1 ? h : l);
    blk[w + j] = bf16_bits(mode == 1 ? l : h);
}

// [rows][K] -> planes of the same layout.  Vector path: 4 consecutive k of
// one row per thread (K % 4 == 0 keeps them in one 16-wide block).
__global__ void split_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ p1,
                             int64_t n, int64_t K, int mode, bool vec) {
    int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {
        for (int64_t i = tid; i < n / 4; i += stride) {
            float4 v = reinterpret_cast<const float4*>(x)[i];
            float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
            float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
            reinterpret_cast<float4*>(hi)[i] = h;
            if (mode == 0) {
                reinterpret_cast<float4*>(p1)[i] = l;
                continue;
            }
            const int64_t e = i * 4, row = e / K, k = e - row * K;
            const int64_t kb = k >> 4;
            const int j = (int)(k & 15);
            const int w = (int)min((int64_t)16, K - kb * 16);
            uint16_t* blk = reinterpret_cast<uint16_t*>(p1 + row * K) + kb * 32;
            const float4 f = mode == 1 ? h : l, g = mode == 1 ? l : h;
            uint2 fu, gu;
            fu.x = (uint32_t)bf16_bits(f.x) | ((uint32_t)bf16_bits(f.y) << 16);
            fu.y = (uint32_t)bf16_bits(f.z) | ((uint32_t)bf16_bits(f.w) << 16);
            gu.x = (uint32_t)bf16_bits(g.x) | ((uint32_t)bf16_bits(g.y) << 16);
            gu.y = (uint32_t)bf16_bits(g.z) | ((uint32_t)bf16_bits(g.w) << 16);
            *reinterpret_cast<uint2*>(blk + j) = fu;       // 8-byte aligned: j, w multiples of 4
            *reinterpret_cast<uint2*>(blk + w + j) = gu;
        }
    } else {
        for (int64_t i = tid; i < n; i += stride) {
            const int64_t row = i / K, k = i - row * K;
            float h = tf32_hi(x[i]);
            hi[i] = h;
            put_plane1(p1 + row * K, k, K, h, x[i] - h, mode);
        }
    }
}

// [batches][K][N] -> planes of the transpose, [batches][N][K]
__global__ void split_transpose_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                       float* __restrict__ p1, int K, int N, int mode) {
    __shared__ float tile[32][33];
    int64_t bz = blockIdx.z;
    const float* xb = x + bz * (int64_t)K * N;
    float* hb = hi + bz * (int64_t)K * N;
    float* pb = p1 + bz * (int64_t)K * N;
    int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        int k = k0 + r, n = n0 + threadIdx.x;
        tile[r][threadIdx.x] = (k < K && n < N) ? xb[(int64_t)k * N + n] : 0.0f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        int n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < K) {
            float v = tile[threadIdx.x][r];
            float h = tf32_hi(v);
            hb[(int64_t)n * K + k] = h;
            put_plane1(pb + (int64_t)n * K, k, K, h, v - h, mode);
        }
    }
}

Status run_split(const float* x, float* hi, float* p1, int64_t batches, int64_t rows, int64_t K, bool trans,
                 int mode, cudaStream_t st) {
    if (!trans) {
        int64_t n = batches * rows * K;
        bool vec = aligned16(x) && K % 4 == 0;
        int grid = grid_for(vec ? n / 4 : n, 256, 16);
        split_kernel<<<grid, 256, 0, st>>>(x, hi, p1, n, K, mode, vec);
    } else {
        // x is [batches][K][rows]; output [batches][rows][K]
        dim3 grid((unsigned)((rows + 31) / 32), (unsigned)((K + 31) / 32), (unsigned)batches);
        split_transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(x, hi, p1, (int)K, (int)rows, mode);
    }
    RT_LAUNCH_CHECK();
    return Status::ok();
}

// ---- fp16 split (SCH_F16): one plane per operand ---------------------------
// Row r of an operand becomes 2*K16 halves (K16 = K rounded up to 16): per
// 16-wide K block [h(16) | l(16)] for A, [l(16) | h(16)] for B, of x scaled by
// 2^e (dev_math.h); k >= K is zero.  A: e per row (its 2^-e in scale[row]),
// from the row's own maximum; B: one e for the whole operand, from the
// maximum an absmax pass left in tensor_max (its 2^-e in scale[1]).

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// |x| maximum over n elements into *out (zeroed first) as float bits
// (non-negative floats order like their bit patterns).
__global__ void absmax_kernel(const float* __restrict__ x, int64_t n, unsigned* out) {
    float m = 0.0f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(x[i]));
    m = warp_max_f(m);
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// One warp per row: the row's maximum (unless tensor_max), then the plane.
__global__ void split16_rows_kernel(const float* __restrict__ x, uint16_t* __restrict__ plane,
                                    float* __restrict__ scale, int64_t rows, int K, int K16,
                                    const float* __restrict__ tensor_max, bool first_hi, bool vec) {
    const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
    if (tensor_max && blockIdx.x == 0 && threadIdx.x == 0) scale[1] = pow2i(-f16_scale_exp(*tensor_max));
    for (int64_t row = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); row < rows; row += (int64_t)gridDim.x * wpb) {
        const float* xr = x + row * K;
        float m;
        if (tensor_max) {
            m = *tensor_max;
        } else {
            m = 0.0f;
            if (vec) {
#pragma unroll 4
                for (int c = lane; c < K / 4; c += 32) {
                    const float4 v = reinterpret_cast<const float4*>(xr)[c];
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                }
            } else {
                for (int k = lane; k < K; k += 32) m = fmaxf(m, fabsf(xr[k]));
            }
            m = warp_max_f(m);
        }
        const int e = f16_scale_exp(m);
        const float sc = pow2i(e);
        if (!tensor_max && lane == 0) scale[row] = pow2i(-e);
        uint16_t* pr = plane + row * (2 * (int64_t)K16);
#pragma unroll 4
        for (int c = lane; c < K16 / 4; c += 32) {
            const int k = 4 * c;
            float4 v;
            if (vec) {
                v = k < K ? reinterpret_cast<const float4*>(xr)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
                v.x = k < K ? xr[k] : 0.f;
                v.y = k + 1 < K ? xr[k + 1] : 0.f;
                v.z = k + 2 < K ? xr[k + 2] : 0.f;
                v.w = k + 3 < K ? xr[k + 3] : 0.f;
            }
            store_f16x4(pr, k, make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc), first_hi);
        }
    }
}

// Long rows (1024 < K16 <= 8192, 16-byte aligned, K % 4 == 0): one row per
// 256-thread block iteration, held in registers (V4 float4 per thread), so
// it is read from memory once -- the warp-per-row kernel above reads it twice
// (maximum, then planes) and keeps only a few loads in flight per warp.
template <int V4>
__global__ void __launch_bounds__(256) split16_rows_block_kernel(const float* __restrict__ x,
                                                                 uint16_t* __restrict__ plane,
                                                                 float* __restrict__ scale, int64_t rows, int K,
                                                                 int K16) {
    __shared__ float red[8];
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float4* xr = reinterpret_cast<const float4*>(x + row * K);
        float4 v[V4];
        float m = 0.0f;
#pragma unroll
        for (int i = 0; i < V4; i++) {
            const int c = t + i * 256;
            v[i] = c < K / 4 ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        }
        m = warp_max_f(m);
        if (lane == 0) red[w] = m;
        __syncthreads();
        m = red[0];
#pragma unroll
        for (int j = 1; j < 8; j++) m = fmaxf(m, red[j]);
        __syncthreads();   // red is rewritten by the next row
        const int e = f16_scale_exp(m);
        const float sc = pow2i(e);
        if (t == 0) scale[row] = pow2i(-e);
        uint16_t* pr = plane + row * (2 * (int64_t)K16);
#pragma unroll
        for (int i = 0; i < V4; i++) {
            const int c = t + i * 256;
            if (c < K16 / 4)
                store_f16x4(pr, 4 * c, make_float4(v[i].x * sc, v[i].y * sc, v[i].z * sc, v[i].w * sc), true);
        }
    }
}

// [batches][K][N] -> plane rows of the transpose ([batches][N][2*K16]), one
// scale for the whole operand (tensor_max).
__global__ void split16_transpose_kernel(const float* __restrict__ x, uint16_t* __restrict__ plane, int K, int N,
                                         int K16, const float* __restrict__ tensor_max, bool first_hi) {
    __shared__ float tile[32][33];
    const int64_t bz = blockIdx.z;
    const float* xb = x + bz * (int64_t)K * N;
    const float sc = pow2i(f16_scale_exp(*tensor_max));
    const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, n = n0 + threadIdx.x;
        tile[r][threadIdx.x] = (k < K && n < N) ? xb[(int64_t)k * N + n] : 0.0f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < K16) {
            const uint32_t hl = f16_hl(tile[threadIdx.x][r] * sc);
            const uint16_t hi = (uint16_t)(hl & 0xffffu), lo = (uint16_t)(hl >> 16);
            uint16_t* blk = plane + (bz * N + n) * (2 * (int64_t)K16) + (k >> 4) * 32 + (k & 15);
            blk[first_hi ? 0 : 16] = hi;
            blk[first_hi ? 16 : 0] = lo;
        }
    }
}

int64_t k16_of(int64_t K) { return (K + 15) / 16 * 16; }

// A operand: per-row scales into scale[batches*rows].
Status run_split16_rows(const float* x, uint16_t* plane, float* scale, int64_t rows, int64_t K, cudaStream_t st) {
    const bool vec = aligned16(x) && K % 4 == 0;
    const int64_t K16 = k16_of(K);
    if (rows == 0) return Status::ok();
    if (vec && K16 > 1024 && K16 <= 8192) {
        const int grid = (int)std::min<int64_t>(rows, (int64_t)g_num_sms * 8);
        if (K16 <= 2048)
            split16_rows_block_kernel<2><<<grid, 256, 0, st>>>(x, plane, scale, rows, (int)K, (int)K16);
        else if (K16 <= 4096)
            split16_rows_block_kernel<4><<<grid, 256, 0, st>>>(x, plane, scale, rows, (int)K, (int)K16);
        else
            split16_rows_block_kernel<8><<<grid, 256, 0, st>>>(x, plane, scale, rows, (int)K, (int)K16);
        RT_LAUNCH_CHECK();
        return Status::ok();
    }
    const int64_t blocks = (rows + 7) / 8;
    const int grid = (int)std::min<int64_t>(blocks, (int64_t)g_num_sms * 8);
    split16_rows_kernel<<<grid, 256, 0, st>>>(x, plane, scale, rows, (int)K, (int)K16, nullptr, true, vec);
    RT_LAUNCH_CHECK();
    return Status::ok();
}

// B operand ([batches][rows][K], or [batches][K][rows] when trans): one scale;
// scalars[0] = the absmax (float bits), scalars[1] = 2^-e.
Status run_split16_tensor(const float* x, uint16_t* plane, float* scalars, int64_t batches, int64_t rows, int64_t K,
                          bool trans, cudaStream_t st) {
    const int64_t n = batches * rows * K;
    RT_CUDA_CHECK(cudaMemsetAsync(scalars, 0, 2 * sizeof(float), st));
    absmax_kernel<<<grid_for(n, 256, 8), 256, 0, st>>>(x, n, reinterpret_cast<unsigned*>(scalars));
    RT_LAUNCH_CHECK();
    const int K16 = (int)k16_of(K);
    if (!trans) {
        const bool vec = aligned16(x) && K % 4 == 0;
        const int64_t all = batches * rows;
        const int grid = (int)std::min<int64_t>((all + 7) / 8, (int64_t)g_num_sms * 8);
        split16_rows_kernel<<<grid, 256, 0, st>>>(x, plane, scalars, all, (int)K, K16, scalars, false, vec);
    } else {
        dim3 grid((unsigned)((rows + 31) / 32), (unsigned)((K16 + 31) / 32), (unsigned)batches);
        split16_transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(x, plane, (int)K, (int)rows, K16, scalars, false);
        if (cudaPeekAtLastError() == cudaSuccess)   // scale[1] for the epilogue
            split16_rows_kernel<<<1, 32, 0, st>>>(x, plane, scalars, 0, (int)K, K16, scalars, false, false);
    }
    RT_LAUNCH_CHECK();
    return Status::ok();
}

// ---- tensor maps (driver entry point fetched through the runtime) --------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

Status make_tmap(CUtensorMap* m, const float* base, int64_t K, int64_t rows, int64_t batches, int box_rows,
                 int box_k = BK) {
    auto fn = encode_fn();
    if (!fn) return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)batches};
    cuuint64_t strides[2] = {(cuuint64_t)K * 4, (cuuint64_t)(rows * K * 4)};
    cuuint32_t box[3] = {(cuuint32_t)box_k, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE,
                    box_k * 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return Status::ok();
}

// fp16 plane tensor map: {2*K16 halves, rows, batches}, box {box_h, box_rows}.
Status make_tmap16(CUtensorMap* m, const void* base, int64_t K16, int64_t rows, int64_t batches, int box_rows,
                   int box_h) {
    auto fn = encode_fn();
    if (!fn) return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)(2 * K16), (cuuint64_t)rows, (cuuint64_t)batches};
    cuuint64_t strides[2] = {(cuuint64_t)K16 * 4, (cuuint64_t)(rows * K16 * 4)};
    cuuint32_t box[3] = {(cuuint32_t)box_h, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE,
                    box_h * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled (f16) failed: " + std::to_string((int)r));
    return Status::ok();
}

// Operand scheme: fp16 (default), RT_GEMM_SCHEME=cross for tf32 + bf16 cross
// terms, RT_GEMM_SCHEME=3xtf32 (or RT_GEMM_3XTF32=1) for three tf32 MMAs.
int scheme() {
    static const int v = [] {
        const char* e = getenv("RT_GEMM_SCHEME");
        const char* t = getenv("RT_GEMM_3XTF32");
        if (t && t[0] == '1') return SCH_3XTF32;
        if (e && !strcmp(e, "3xtf32")) return SCH_3XTF32;
        if (e && !strcmp(e, "cross")) return SCH_CROSS;
        return SCH_F16;
    }();
    return v;
}
bool cross_scheme() { return scheme() == SCH_CROSS; }

// K accumulated per TMEM chunk (see the file comment): 384 for the fp16
// scheme (its exact fp16 products leave the accumulation as the main error:
// 7.3e-6 per sqrt(K) against fp64 at 384, 4.9e-6 at 256, 1.1e-5 at 512; 384
// runs the 1b8k block 4 % faster than 256), 256 for the cross-term scheme,
// 128 for 3xTF32 (three accumulating MMAs per K step instead of two: its
// error at 256 exceeds the cross scheme's at 256).  RT_GEMM_KCHUNK (a
// multiple of 32) overrides all.
int k_chunk() {
    static int v = [] {
        const int dflt = scheme() == SCH_3XTF32 ? 128 : scheme() == SCH_F16 ? 384 : 256;
        const char* e = getenv("RT_GEMM_KCHUNK");
        int k = e ? atoi(e) : dflt;
        if (k < 32 || k % 32) k = dflt;
        return k;
    }();
    return v;
}

// RT_GEMM_SPLITK=0 turns the two-way split-K off.
bool split_k_enabled() {
    static const bool on = [] {
        const char* e = getenv("RT_GEMM_SPLITK");
        return !(e && e[0] == '0');
    }();
    return on;
}

int a_mode() { return cross_scheme() ? 1 : 0; }
int b_mode() { return cross_scheme() ? 2 : 0; }
SplitKey b_key(const GemmProblem& p, int gate = 0) {
    return SplitKey{p.b, p.batches, p.N, p.K, (p.trans_b ? 0 : 1) | (scheme() << 1) | (gate ? 8 : 0)};
}

// B rows ([N][K], N % 256 == 0) in the gated order read by a gated epilogue:
// per 256-row tile t and half h, 64 gate rows t*128 + h*64 + w (w < 64), then
// their up rows N/2 + t*128 + h*64 + w.
__global__ void gate_order_rows_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t N,
                                       int64_t K) {
    const int64_t Nh = N / 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N * K; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t q = i / K, k = i - q * K;
        const int64_t t = q / 256, h = (q % 256) / 128, w = q % 128;
        const int64_t row = (w < 64 ? 0 : Nh) + t * 128 + h * 64 + (w & 63);
        dst[i] = src[row * K + k];
    }
}

// Every kernel instantiation with its dynamic shared memory size.
template <class F>
cudaError_t for_each_kernel(F f) {
    constexpr int P0 = PCfg<SCH_3XTF32>::SMEM, P1 = PCfg<SCH_CROSS>::SMEM, P2 = PCfg<SCH_F16>::SMEM;
    const void* ks[] = {
        (const void*)tc_gemm_pair_kernel<SCH_3XTF32, false>, (const void*)tc_gemm_pair_kernel<SCH_CROSS, false>,
        (const void*)tc_gemm_pair_kernel<SCH_F16, false>,
        (const void*)tc_gemm_pair_kernel<SCH_3XTF32, true>, (const void*)tc_gemm_pair_kernel<SCH_CROSS, true>,
        (const void*)tc_gemm_pair_kernel<SCH_3XTF32, false, true>, (const void*)tc_gemm_pair_kernel<SCH_CROSS, false, true>,
        (const void*)tc_gemm_pair_kernel<SCH_F16, false, true>,
        (const void*)tc_gemm_pair_kernel<SCH_3XTF32, false, false, true>,
        (const void*)tc_gemm_pair_kernel<SCH_CROSS, false, false, true>,
        (const void*)tc_gemm_pair_kernel<SCH_F16, false, false, true>,
        (const void*)tc_gemm_kernel<256, SCH_3XTF32, false>, (const void*)tc_gemm_kernel<256, SCH_CROSS, false>,
        (const void*)tc_gemm_kernel<256, SCH_F16, false>,
        (const void*)tc_gemm_kernel<256, SCH_3XTF32, true>, (const void*)tc_gemm_kernel<256, SCH_CROSS, true>,
        (const void*)tc_gemm_kernel<128, SCH_3XTF32, false>, (const void*)tc_gemm_kernel<128, SCH_CROSS, false>,
        (const void*)tc_gemm_kernel<128, SCH_F16, false>,
        (const void*)tc_gemm_kernel<128, SCH_3XTF32, true>, (const void*)tc_gemm_kernel<128, SCH_CROSS, true>,
        (const void*)tc_gemm_pair_kernel<SCH_F16, true>, (const void*)tc_gemm_kernel<256, SCH_F16, true>,
        (const void*)tc_gemm_kernel<128, SCH_F16, true>};
    const int smem[] = {P0, P1, P2, P0, P1, P0, P1, P2, P0, P1, P2,
                        GCfg<256, SCH_3XTF32>::SMEM_BYTES, GCfg<256, SCH_CROSS>::SMEM_BYTES,
                        GCfg<256, SCH_F16>::SMEM_BYTES, GCfg<256, SCH_3XTF32>::SMEM_BYTES,
                        GCfg<256, SCH_CROSS>::SMEM_BYTES,
                        GCfg<128, SCH_3XTF32>::SMEM_BYTES, GCfg<128, SCH_CROSS>::SMEM_BYTES,
                        GCfg<128, SCH_F16>::SMEM_BYTES, GCfg<128, SCH_3XTF32>::SMEM_BYTES,
                        GCfg<128, SCH_CROSS>::SMEM_BYTES, P2, GCfg<256, SCH_F16>::SMEM_BYTES,
                        GCfg<128, SCH_F16>::SMEM_BYTES};
    static_assert(sizeof(ks) / sizeof(ks[0]) == sizeof(smem) / sizeof(smem[0]), "kernel table");
    for (size_t i = 0; i < sizeof(ks) / sizeof(ks[0]); i++) {
        cudaError_t e = f(ks[i], smem[i]);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <int SCH, bool PLANES>
void launch_tc_t(bool pair, int BN, int grid, const TcParams& prm, cudaStream_t st) {
    constexpr int PS = PCfg<SCH>::SMEM;
    if (pair && !PLANES && prm.res)
        tc_gemm_pair_kernel<SCH, false, true><<<2 * grid, THREADS, PS, st>>>(prm);
    else if (pair && !PLANES && prm.c_tma)
        tc_gemm_pair_kernel<SCH, false, false, true><<<2 * grid, THREADS, PS, st>>>(prm);
    else if (pair)
        tc_gemm_pair_kernel<SCH, PLANES><<<2 * grid, THREADS, PS, st>>>(prm);
    else if (BN == 128)
        tc_gemm_kernel<128, SCH, PLANES><<<grid, THREADS, GCfg<128, SCH>::SMEM_BYTES, st>>>(prm);
    else
        tc_gemm_kernel<256, SCH, PLANES><<<grid, THREADS, GCfg<256, SCH>::SMEM_BYTES, st>>>(prm);
}
void launch_tc(bool pair, int BN, int sch, bool planes, int grid, const TcParams& prm, cudaStream_t st) {
    if (sch == SCH_F16 && planes) launch_tc_t<SCH_F16, true>(pair, BN, grid, prm, st);
    else if (sch == SCH_F16) launch_tc_t<SCH_F16, false>(pair, BN, grid, prm, st);
    else if (sch == SCH_CROSS && planes) launch_tc_t<SCH_CROSS, true>(pair, BN, grid, prm, st);
    else if (sch == SCH_CROSS) launch_tc_t<SCH_CROSS, false>(pair, BN, grid, prm, st);
    else if (planes) launch_tc_t<SCH_3XTF32, true>(pair, BN, grid, prm, st);
    else launch_tc_t<SCH_3XTF32, false>(pair, BN, grid, prm, st);
}

// RT_GEMM_PAIR=0 keeps every GEMM on the one-CTA kernel.
bool pair_enabled() {
    static const bool on = [] {
        const char* e = getenv("RT_GEMM_PAIR");
        return !(e && e[0] == '0');
    }();
    return on;
}

// CTA pairs the device keeps resident at once (one pair per two SMs unless
// the GPC layout leaves some SMs unpaired).
int pair_clusters() {
    static int n = [] {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (g_num_sms / 2));
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = PCfg<SCH_CROSS>::SMEM;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int c = 0;
        if (cudaOccupancyMaxActiveClusters(&c, tc_gemm_pair_kernel<SCH_CROSS, false>, &cfg) != cudaSuccess ||
            c <= 0) {
            cudaGetLastError();
            c = g_num_sms / 2;
        }
        return c;
    }();
    return n;
}

bool b_is_constant(const GemmProblem& p) {
    return is_constant_range(p.b, (size_t)p.batches * p.N * p.K * 4);
}

size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }
// Bytes of one split plane: the tf32 schemes' fp32 planes hold K floats per
// row, the fp16 plane 2*K16 halves (the same bytes when K % 16 == 0).
size_t plane_bytes(int64_t batches, int64_t rows, int64_t K) {
    return (size_t)batches * rows * (scheme() == SCH_F16 ? k16_of(K) : K) * 4;
}
// fp16 scheme: the per-row A scales / the B scalars
size_t a_scale_bytes(const GemmProblem& p) { return round256((size_t)p.batches * p.M * 4); }
constexpr size_t B_SCALARS = 256;

}  // namespace

bool gemm_cross_scheme() { return cross_scheme(); }
int gemm_scheme() { return scheme(); }
bool gemm_planes_from_epilogues() { return scheme() != SCH_F16; }

bool tc_gemm_applicable(const GemmProblem& p) {
    // tf32 planes keep K fp32 per row (TMA row stride a 16-byte multiple);
    // the fp16 plane pads rows to 16-wide blocks
    if (scheme() != SCH_F16 && p.K % 4 != 0) return false;
    if ((double)p.M * p.N * p.K < 8.0 * 1024 * 1024) return false;   // tiny: the CUDA-core GEMM wins
    if (p.M > INT32_MAX / 2 || p.N > INT32_MAX / 2 || p.K > INT32_MAX / 4 || p.batches > 65535) return false;
    return true;
}

size_t tc_gemm_workspace_bytes(const GemmProblem& p) {
    if (!tc_gemm_applicable(p)) return 0;
    const bool f16 = scheme() == SCH_F16;
    size_t b = f16 ? round256(plane_bytes(p.batches, p.M, p.K)) + a_scale_bytes(p)
                   : 2 * round256(plane_bytes(p.batches, p.M, p.K));
    if (!b_is_constant(p))
        b += f16 ? round256(plane_bytes(p.batches, p.N, p.K)) + B_SCALARS
                 : 2 * round256(plane_bytes(p.batches, p.N, p.K));
    return b;
}

Status tc_gemm_prepare(const GemmProblem& p, cudaStream_t st, int gate) {
    if (!tc_gemm_applicable(p)) return Status::ok();
    static bool attr_set = false;
    if (!attr_set) {
        RT_CUDA_CHECK(for_each_kernel([](const void* k, int smem) {
            return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        }));
        attr_set = true;
        pair_clusters();   // occupancy query outside any stream capture
    }
    if (!b_is_constant(p)) {
        if (gate) return Status::err(RT_ERR_ARGUMENT, "gemm: a gated epilogue needs a constant B");
        return Status::ok();
    }
    SplitKey key = b_key(p, gate);
    if (find_constant_split(key)) return Status::ok();
    const float* src = p.b;
    float* tmp = nullptr;
    if (gate) {   // B in the gated row order, split once like any constant B
        if (!p.trans_b || p.batches != 1 || p.N % 256 != 0)
            return Status::err(RT_ERR_ARGUMENT, "gemm: a gated epilogue needs B [N][K], N % 256 == 0");
        RT_CUDA_CHECK(cudaMalloc(&tmp, (size_t)p.N * p.K * 4));
        gate_order_rows_kernel<<<grid_for(p.N * p.K, 256), 256, 0, st>>>(p.b, tmp, p.N, p.K);
        src = tmp;
    }
    SplitOperand s;
    Status r;
    if (scheme() == SCH_F16) {
        r = create_constant_split(key, plane_bytes(p.batches, p.N, p.K) / 4, B_SCALARS / 4, &s);
        if (r.good())
            r = run_split16_tensor(src, reinterpret_cast<uint16_t*>(s.hi), s.lo, p.batches, p.N, p.K, !p.trans_b, st);
    } else {
        const size_t elems = (size_t)p.batches * p.N * p.K;
        r = create_constant_split(key, elems, elems, &s);
        if (r.good()) r = run_split(src, s.hi, s.lo, p.batches, p.N, p.K, !p.trans_b, b_mode(), st);
    }
    if (tmp) {
        if (cudaStreamSynchronize(st) != cudaSuccess && r.good()) r = Status::err(RT_ERR_CUDA, "gemm: gated B order");
        cudaFree(tmp);
    }
    return r;
}

static bool prm_planes_out(const GemmFusion* f) { return f && f->plane_hi; }

Status tc_gemm_launch(const GemmProblem& p, cudaStream_t st, Workspace ws, int* launches,
                      const GemmFusion* f) {
    if (p.M == 0) return Status::ok();
    if (ws.bytes < tc_gemm_workspace_bytes(p)) return Status::err(RT_ERR_ARGUMENT, "gemm: workspace too small");
    if (f && f->plane_hi && p.N % 4 != 0) return Status::err(RT_ERR_ARGUMENT, "gemm: split-plane output needs N % 4 == 0");
    const int sch = scheme();
    const bool f16 = sch == SCH_F16;
    // fp16 scheme hand-offs: the output as the next GEMM's fp16 plane with
    // one scale per (row, 128 columns); an A operand given in that form
    if (f16 && f && f->plane_hi && p.N % 128 != 0)
        return Status::err(RT_ERR_ARGUMENT, "gemm: fp16 plane output needs N % 128 == 0");
    const bool a_seg = f16 && f && f->pre_hi && f->pre_seg;
    if (a_seg && p.K % 128 != 0) return Status::err(RT_ERR_ARGUMENT, "gemm: a segment-scaled A needs K % 128 == 0");
    const size_t abytes = round256(plane_bytes(p.batches, p.M, p.K));
    const size_t a2bytes = f16 ? a_scale_bytes(p) : abytes;   // second A region: scales or plane 1
    const void *a_hi, *a_lo;
    const void *b_hi, *b_lo;
    const float* a_scale = nullptr;
    const float* b_scale = nullptr;
    Status s;
    if (f && f->pre_hi) {   // A split by its producer (a norm: planes, or plane + row scales)
        a_hi = f->pre_hi;
        a_lo = f->pre_x;
    } else {
        char* ah = ws.base;
        char* al = ws.base + abytes;
        s = f16 ? run_split16_rows(p.a, reinterpret_cast<uint16_t*>(ah), reinterpret_cast<float*>(al),
                                   p.batches * p.M, p.K, st)
                : run_split(p.a, reinterpret_cast<float*>(ah), reinterpret_cast<float*>(al), p.batches, p.M, p.K,
                            false, a_mode(), st);
        if (!s.good()) return s;
        *launches += 1;
        a_hi = ah;
        a_lo = al;
    }
    if (f16 && !a_seg) a_scale = static_cast<const float*>(a_lo);
    const int gate = f ? f->gate : 0;
    if (gate && (!b_is_constant(p) || p.N % 256 != 0))
        return Status::err(RT_ERR_ARGUMENT, "gemm: a gated epilogue needs a constant B with N % 256 == 0");
    if (b_is_constant(p)) {
        const SplitOperand* so = find_constant_split(b_key(p, gate));
        if (!so) return Status::err(RT_ERR_ARGUMENT, "gemm: constant operand not prepared");
        b_hi = so->hi;
        b_lo = so->lo;
    } else {
        char* bh = ws.base + abytes + a2bytes;
        char* bl = bh + round256(plane_bytes(p.batches, p.N, p.K));
        s = f16 ? run_split16_tensor(p.b, reinterpret_cast<uint16_t*>(bh), reinterpret_cast<float*>(bl), p.batches,
                                     p.N, p.K, !p.trans_b, st)
                : run_split(p.b, reinterpret_cast<float*>(bh), reinterpret_cast<float*>(bl), p.batches, p.N, p.K,
                            !p.trans_b, b_mode(), st);
        if (!s.good()) return s;
        *launches += f16 ? 2 : 1;
        b_hi = bh;
        b_lo = bl;
    }
    if (f16) b_scale = static_cast<const float*>(b_lo) + 1;
    TcParams prm;
    memset(&prm, 0, sizeof prm);
    // N tile: 256 -- measured faster than 128 at every BASELINE shape, N=768
    // included (the 128-wide tile doubles A traffic per flop); short grids are
    // filled by split-K below instead.  RT_GEMM_BN=128 selects the narrow tile.
    static const int bn_force = [] {
        const char* e = getenv("RT_GEMM_BN");
        return e ? atoi(e) : 0;
    }();
    const int BN = bn_force == 128 && !(f16 && prm_planes_out(f)) ? 128 : 256;
    if (gate && BN != 256) return Status::err(RT_ERR_ARGUMENT, "gemm: a gated epilogue needs 256-wide N tiles");
    // CTA pairs (256x256 tiles) whenever A has more than one 128-row block.
    const bool pair = BN == 256 && p.M > BM && pair_enabled();
    const int b_box = pair ? 128 : BN;
    const int bk = pair ? P_BK : BK;
    if (f16) {
        const int64_t K16 = k16_of(p.K);
        if (!(s = make_tmap16(&prm.ta_hi, a_hi, K16, p.M, p.batches, BM, 2 * bk)).good()) return s;
        if (!(s = make_tmap16(&prm.tb_hi, b_hi, K16, p.N, p.batches, b_box, 2 * bk)).good()) return s;
    } else {
        const float *ah = static_cast<const float*>(a_hi), *al = static_cast<const float*>(a_lo);
        const float *bh = static_cast<const float*>(b_hi), *bl = static_cast<const float*>(b_lo);
        if (!(s = make_tmap(&prm.ta_hi, ah, p.K, p.M, p.batches, BM, bk)).good()) return s;
        if (!(s = make_tmap(&prm.ta_lo, al, p.K, p.M, p.batches, BM, bk)).good()) return s;
        if (!(s = make_tmap(&prm.tb_hi, bh, p.K, p.N, p.batches, b_box, bk)).good()) return s;
        if (!(s = make_tmap(&prm.tb_lo, bl, p.K, p.N, p.batches, b_box, bk)).good()) return s;
    }
    prm.a_scale = a_scale;
    prm.b_scale = b_scale;
    prm.a_seg = a_seg ? static_cast<const float*>(a_lo) : nullptr;
    prm.a_segs = a_seg ? (int)(p.K / 128) : 0;
    prm.c = f && f->out ? f->out : p.c;
    prm.bias = f && f->bias ? f->bias : p.bias;
    prm.res = f ? f->res : nullptr;
    prm.alpha = p.alpha;
    // Planner offsets are raw byte counts (first fit), so C, a bias or a
    // residual may sit off a 16-byte boundary: those rows take scalar accesses.
    prm.vec_c = (gate ? p.N / 2 : p.N) % 4 == 0 && aligned16(prm.c) && (!prm.bias || aligned16(prm.bias)) &&
                (!prm.res || aligned16(prm.res));
    prm.act = f ? f->act : 0;
    prm.gate = gate;
    if (gate && (prm.bias || prm.res || prm.alpha != 1.0f || prm.act || (f && f->plane_hi)))
        return Status::err(RT_ERR_ARGUMENT, "gemm: a gated epilogue takes no bias, residual, alpha or other activation");
    prm.plane_hi = f ? f->plane_hi : nullptr;
    prm.plane_x = f ? static_cast<uint8_t*>(f->plane_x) : nullptr;
    prm.plane_mode = f16 ? 2 : a_mode();
    prm.M = (int)p.M;
    prm.N = (int)p.N;
    prm.K = (int)p.K;
    prm.batches = (int)p.batches;
    const int tile_m = pair ? 2 * BM : BM;
    prm.m_tiles = (int)((p.M + tile_m - 1) / tile_m);
    prm.n_tiles = (int)((p.N + BN - 1) / BN);
    prm.k_blocks = (int)((p.K + bk - 1) / bk);
    // (a segment-scaled A: one chunk per 128-wide segment)
    prm.kb_per_chunk = a_seg ? 128 / bk : k_chunk() / bk > 0 ? k_chunk() / bk : 1;
    prm.n_chunks = (prm.k_blocks + prm.kb_per_chunk - 1) / prm.kb_per_chunk;
    int64_t total = (int64_t)prm.m_tiles * prm.n_tiles * p.batches;
    if (total > INT32_MAX / 2) return Status::err(RT_ERR_UNSUPPORTED, "gemm: too many tiles");
    prm.total_tiles = (int)total;
    // persistent workers: CTAs, or CTA pairs
    const int workers = pair ? pair_clusters() : g_num_sms;
    // Split K in two when the tiles alone fill well under 1.5 waves of the
    // persistent grid (two addends keep the fp32 sum order-independent).
    // (Not with a fused activation or split-plane output: both need the full sum.)
    prm.splits = 1;
    // A residual may be C itself (each element read, then written, by one
    // thread) but not partly overlap it; in place it also rules out split-K
    // (which zeroes C first).
    bool res_in_c = false;
    if (prm.res && prm.alpha != 1.0f) return Status::err(RT_ERR_ARGUMENT, "gemm: a residual needs alpha 1");
    if (prm.res) {
        const uintptr_t c0 = reinterpret_cast<uintptr_t>(prm.c), r0 = reinterpret_cast<uintptr_t>(prm.res);
        const uintptr_t nb = (uintptr_t)p.batches * p.M * p.N * 4;
        if (r0 < c0 + nb && c0 < r0 + nb) {
            if (r0 != c0) return Status::err(RT_ERR_ARGUMENT, "gemm: residual partly overlaps the output");
            res_in_c = true;
        }
    }
    const bool whole_sum = prm.act != 0 || prm.gate != 0 || prm.plane_hi != nullptr || res_in_c;
    if (total < (int64_t)workers * 3 / 2 && prm.n_chunks >= 2 && split_k_enabled() && !whole_sum) {
        prm.splits = 2;
        RT_CUDA_CHECK(cudaMemsetAsync(prm.c, 0, (size_t)p.batches * p.M * p.N * 4, st));
    }
    // equal halves of the K blocks (each split accumulates its own TMEM chunks)
    prm.kb_split = (prm.k_blocks + prm.splits - 1) / prm.splits;
    if (a_seg) prm.kb_split = (prm.kb_split + prm.kb_per_chunk - 1) / prm.kb_per_chunk * prm.kb_per_chunk;
    prm.total_items = prm.total_tiles * prm.splits;
    // Opt-in (RT_GEMM_TMA_STORE=1): C through shared memory and TMA stores
    // (pair kernel, plain C output, no split-K).  Alone, the 8192 x 2304 and
    // x 3072 (K = 768) GEMMs ran ~11 % faster than with per-row stores, but
    // whole forwards did not move (GPT-2 1.398 / 1.397 ms, Qwen3 2.825 /
    // 2.797, 7b 11.09 / 11.12), so per-row stores stay the default.
    static const bool c_tma_on = [] {
        const char* e = getenv("RT_GEMM_TMA_STORE");
        return e && e[0] == '1';
    }();
    prm.c_tma = 0;
    if (c_tma_on && pair && prm.splits == 1 && !prm.plane_hi && !prm.res && !prm.gate && prm.vec_c) {
        if (!(s = encode_tmap_f32_3d(&prm.tc, prm.c, p.N, p.M, p.batches, 32, 32, 128)).good()) return s;
        prm.c_tma = 1;
    }
    prm.err = kernel_error_flag();
    const int grid = prm.total_items < workers ? prm.total_items : workers;
    launch_tc(pair, BN, sch, prm.plane_hi != nullptr, grid, prm, st);
    RT_LAUNCH_CHECK();
    *launches += 1;
    return Status::ok();
}

}  // namespace rt

// ===========================================================================
// rt_matmul_noalloc: the same tensor-core GEMM for callers that cannot
// allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- a plugin
// whose host application owns all device memory through its own pool, or a
// process that must not grow its device footprint after start-up.
// rt_execute plans a workspace per node array (cudaMalloc), so those callers
// use this entry point instead.  It needs no rt_init either: it works on the
// current device and the stream it is given.  It is synchronous (it waits
// for that stream before returning), so it belongs on a host thread, not in
// a CUDA host callback, which may not call CUDA at all.
//
// Its scratch (the hi/lo split copies of both operands) lives in the file-
// scope device array below, NOALLOC_SCRATCH_BYTES (32 MiB) per GPU that loads
// the library, held until the process exits.  The caller passes inputs and
// output only.  Host code must not hand the array's name to a kernel (on the
// host it is a stand-in symbol, not a device address): the address is taken
// with cudaGetSymbolAddress once per device, on the first call made while
// that device is current -- that first call also sets the kernel's shared-
// memory attribute, so make it before any stream capture.  Nothing in the
// scratch has to start at zero (every word read is written first by the
// same call); the error word is cleared on the stream at the start of every
// call.  All calls share the one array, so calls whose GPU work overlaps
// (different streams, or host threads) race on it.  Each launch is checked
// with cudaGetLastError, which also returns an error that earlier CUDA work
// of the caller left pending: that is reported as this call's RT_ERR_CUDA.
// ===========================================================================
namespace rt {
namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)32 << 20;
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_BYTES / sizeof(float)];
static __device__ int g_noalloc_error;   // bounded-wait timeout code of the last call

struct NoallocDevice {
    float* scratch = nullptr;   // device address of g_noalloc_scratch on this device
    int* error = nullptr;       // device address of g_noalloc_error
    int sms = 0;
};

std::mutex& noalloc_mutex() {
    static std::mutex m;
    return m;
}

// Per-device set-up, run with the device current.  No allocation.
int noalloc_setup(int device, NoallocDevice** out) {
    static NoallocDevice table[64];
    if (device < 0 || device >= 64) return RT_ERR_ARGUMENT;
    NoallocDevice& d = table[device];
    if (!d.scratch) {
        float* s = nullptr;
        int* e = nullptr;
        if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s), g_noalloc_scratch) != cudaSuccess ||
            cudaGetSymbolAddress(reinterpret_cast<void**>(&e), g_noalloc_error) != cudaSuccess) {
            cudaGetLastError();
            return RT_ERR_CUDA;
        }
        if (cudaFuncSetAttribute(tc_gemm_kernel<256, SCH_CROSS, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 GCfg<256, SCH_CROSS>::SMEM_BYTES) !=
            cudaSuccess) {
            cudaGetLastError();
            return RT_ERR_CUDA;
        }
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0)
            sms = 148;
        d.error = e;
        d.sms = sms;
        d.scratch = s;   // published last: a set-up that failed is retried next call
    }
    *out = &d;
    return RT_OK;
}

}  // namespace
}  // namespace rt

extern "C" int rt_matmul_noalloc(const float* a, const float* b, const float* bias, float* c, int M, int N,
                                 int K, int trans_b, float alpha, void* stream) {
    using namespace rt;
    if (!a || !b || !c) return RT_ERR_NULL_POINTER;
    if (M < 0 || N <= 0 || K <= 0) return RT_ERR_ARGUMENT;
    if (K % 4 != 0) return RT_ERR_UNSUPPORTED;   // TMA rows must be a multiple of 16 bytes
    const size_t a_elems = round256((size_t)M * K * 4) / 4;
    const size_t b_elems = round256((size_t)N * K * 4) / 4;
    if (2 * (a_elems + b_elems) * sizeof(float) > NOALLOC_SCRATCH_BYTES)
        return RT_ERR_OUT_OF_RANGE;   // needs 8*(M*K + N*K) bytes <= 32 MiB of scratch
    if (M == 0) return RT_OK;
    std::lock_guard<std::mutex> lock(noalloc_mutex());
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return RT_ERR_CUDA;
    NoallocDevice* d = nullptr;
    int rc = noalloc_setup(device, &d);
    if (rc != RT_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    float* a_hi = d->scratch;
    float* a_lo = a_hi + a_elems;
    float* b_hi = a_lo + a_elems;
    float* b_lo = b_hi + b_elems;
    if (!run_split(a, a_hi, a_lo, 1, M, K, false, 1, st).good()) return RT_ERR_CUDA;
    if (!run_split(b, b_hi, b_lo, 1, N, K, !trans_b, 2, st).good()) return RT_ERR_CUDA;

    TcParams prm;
    memset(&prm, 0, sizeof prm);
    if (!make_tmap(&prm.ta_hi, a_hi, K, M, 1, BM).good() || !make_tmap(&prm.ta_lo, a_lo, K, M, 1, BM).good() ||
        !make_tmap(&prm.tb_hi, b_hi, K, N, 1, 256).good() || !make_tmap(&prm.tb_lo, b_lo, K, N, 1, 256).good())
        return RT_ERR_CUDA;
    prm.c = c;
    prm.bias = bias;
    prm.alpha = alpha;
    prm.vec_c = N % 4 == 0 && aligned16(c) && (!bias || aligned16(bias));
    prm.M = M;
    prm.N = N;
    prm.K = K;
    prm.batches = 1;
    prm.m_tiles = (M + BM - 1) / BM;
    prm.n_tiles = (N + 255) / 256;
    prm.k_blocks = (K + BK - 1) / BK;
    prm.kb_per_chunk = 256 / BK;   // the cross-term scheme's chunk (this entry point always uses that scheme)
    prm.n_chunks = (prm.k_blocks + prm.kb_per_chunk - 1) / prm.kb_per_chunk;
    int64_t total = (int64_t)prm.m_tiles * prm.n_tiles;
    prm.total_tiles = (int)total;
    prm.splits = 1;
    prm.kb_split = prm.k_blocks;
    prm.total_items = prm.total_tiles;
    prm.err = d->error;
    if (cudaMemsetAsync(d->error, 0, sizeof(int), st) != cudaSuccess) return RT_ERR_CUDA;
    int grid = prm.total_tiles < d->sms ? prm.total_tiles : d->sms;
    tc_gemm_kernel<256, SCH_CROSS, false><<<grid, THREADS, GCfg<256, SCH_CROSS>::SMEM_BYTES, st>>>(prm);
    if (cudaGetLastError() != cudaSuccess) return RT_ERR_CUDA;
    // synchronous: returns once C is written, and reports a kernel that gave
    // up a wait.  The error word comes back on the caller's stream (pageable
    // destination: the copy completes before the synchronize returns), so
    // the call never waits on work queued on other streams.
    int kerr = 0;
    if (cudaMemcpyAsync(&kerr, d->error, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return RT_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return RT_ERR_CUDA;
    return kerr ? RT_ERR_KERNEL_TIMEOUT : RT_OK;
}

namespace rt {

// Plain hi/lo split (3xTF32 form) and fp32 tensor maps for other kernels.
Status split_operand(const float* x, float* hi, float* lo, int64_t batches, int64_t rows, int64_t K,
                     bool transpose, cudaStream_t st) {
    return run_split(x, hi, lo, batches, rows, K, transpose, 0, st);
}

Status encode_tmap_f32(CUtensorMap* m, const float* base, int rank, const int64_t* dims,
                       const int64_t* byte_strides, const int* box, int swizzle_bytes) {
    auto fn = encode_fn();
    if (!fn) return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if (rank < 1 || rank > 5) return Status::err(RT_ERR_ARGUMENT, "tensor map rank");
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], estr[5];
    for (int i = 0; i < rank; i++) {
        d[i] = (cuuint64_t)dims[i];
        bx[i] = (cuuint32_t)box[i];
        estr[i] = 1;
        if (i > 0) st[i - 1] = (cuuint64_t)byte_strides[i - 1];
    }
    CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                            : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<float*>(base), d, st, bx, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return Status::ok();
}

Status encode_tmap_f32_3d(CUtensorMap* m, const float* base, int64_t d0, int64_t d1, int64_t d2, int box0,
                          int box1, int swizzle_bytes) {
    auto fn = encode_fn();
    if (!fn) return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)d0 * 4, (cuuint64_t)(d0 * d1 * 4)};
    cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                            : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return Status::err(RT_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return Status::ok();
}

}  // namespace rt
