// zz_gemm.cuh -- grouped block-scaled int8 GEMM over q4_0 / q8_0 / tq2 planes.
//
// C[o, n] = sum_b  dw[o,b] * dx[n,b] * <A_o,b , X_n,b>     (tq2: dx[n,b] only)
//
// The per-block scales vary along both o and n, so int32 partials cannot be carried
// across 32-wide K blocks: every block's integer product is converted and scaled into
// fp32 accumulators before the next block (the decomposition of q40.h:20-31).
//
// The tensor cores see the codes and activations as fp16 values that are exactly the
// integers the reference multiplies (q-8 in [-8,7], q8 codes and activations in
// [-127,127], tq2 codes {0,1,2}); each product and each 32-term block sum (|s| <
// 2^15) is exact in the f32 accumulator, so the MMA result of one block IS the
// reference's per-block integer, already in floating point. That removes the
// int->float conversion per (row, column, block) that an s8 MMA would need (a
// quarter-rate instruction that otherwise bounds the whole kernel); what remains per
// element and block is one packed fma.rn.f32x2 and one packed multiply.
//
// CTA tile: 128 weight rows x BN activation rows, 8 warps of 16 rows each. K moves in
// chunks of 4 blocks (128 weights) through a cp.async pipeline. The weight codes stay
// packed in shared memory and are widened to fp16 in registers straight into the
// m16n8k16 A fragment (q4_0: low nibbles of bytes j are k = j, high nibbles k = j+16,
// so one 16-bit load feeds both k16 steps of a block). Activations are fp16 in
// shared memory (ldmatrix.x4 fetches a whole block's B fragment) or int8 widened in
// registers for callers that hold only int8 rows.
//
// Work items (grid.y) name a group (expert) and a contiguous range of <= BN activation
// rows; grid.x walks 128-row weight tiles. Epilogues:
//   EPI_STORE  y[n, o] = C (tq2: alpha_o * (C - Sx_n))                 dense matmul
//   EPI_GATEUP rows 0-63 gate / 64-127 up of the same 64 features -> act -> q8_0
//              requant of h into hq/hs (+ per-block sums for tq2)      expert gate/up
//   EPI_DOWN   OUT[tok(n), o] += w(n) * C (float4 atomics)            expert down
#pragma once
#include "zz_common.cuh"

namespace zz {

enum { EPI_STORE = 0, EPI_GATEUP = 1, EPI_DOWN = 2 };

#ifndef ZZ_G_STAGES
#define ZZ_G_STAGES 2
#endif
constexpr int G_BM = 128, G_BKB = 4, G_STAGES = ZZ_G_STAGES, G_THREADS = 256;

template <int FMT>
struct FmtTraits {
    static constexpr int CB = FMT == GPU_FMT_Q40 ? 16 : FMT == GPU_FMT_Q80 ? 32 : 8;  // code bytes / block
    static constexpr int A_STRIDE = CB * G_BKB + 16;  // padded smem row (bank-conflict free)
    static constexpr bool HAS_WSCALE = FMT != GPU_FMT_TQ2;
};

struct WorkItem {
    int group;  // expert (or 0)
    int row0;   // first activation row (pair-sorted index)
    int count;  // rows in this item, 1..BN
    int pad;
};

struct GemmArgs {
    // weights: group g tensor = codes + g*codes_gstride, rows of code_row bytes
    const uint8_t *codes;
    const void *scale;       // fp16 [rows][nb] or f32 alpha [rows]
    long codes_gstride, scale_gstride;  // bytes
    int O, I;                // rows per group, K
    // activations: row r of the item -> X row xrow(r) (gather), scales likewise
    const void *xq;          // int8 rows [*, I] (B_HALF = false) or fp16 rows (B_HALF = true)
    const float *xs;
    const float *xsx;        // tq2 per-row Sx (EPI_STORE / EPI_GATEUP, indexed by X row)
    const int *xblk;         // tq2 down: per-block int sums of X rows; Sx is summed here
    const int *gather;       // NULL: X row = item row; else X row = gather[item row] / gather_div
    int gather_div;
    // work
    const WorkItem *items;
    const int *n_items;      // device count (NULL: use gridDim.y)
    int rows_total;          // items == NULL: item y covers rows [y*BN, min(rows_total, (y+1)*BN))
    // EPI_STORE
    float *y;                // [n][O]
    // EPI_GATEUP
    int act;
    float clamp;
    int8_t *hq;              // [pair][O/2]
    __half *hh;              // [pair][O/2] the same values as fp16 (the down GEMM's B)
    float *hs;               // [pair][O/64]
    int *hblk;               // [pair][O/64] (tq2 only)
    // EPI_DOWN
    float *out;              // [token][O]
    const float *pair_w;     // [pair]
    const int *pair_src;     // [pair] routing slot s*K+k of the pair
    int K;
    // tensor-core path: B rows in pair order and transposed block scales
    const __half *xg;        // [rows_cap][I] fp16
    const int8_t *xg8;       // [rows_cap][I] int8 (the int8 tensor-core engine's B rows)
    const float *xsT;        // [I/32][ldT]
    int ldT, rows_cap;
    float *hsT;              // gate/up: transposed hidden scales [O/64][ldT]
    // folded-scale fp16 engine: B operand planes of the pair rows, hi at xhs and lo at
    // xhs + rows_cap * I; gate/up also writes the down GEMM's planes to hhs likewise
    const __half *xhs;
    __half *hhs;
};


__device__ __forceinline__ void mma_f16(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1, float c0, float c1, float c2, float c3) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}
// int8 MMA onto the accumulator preset 0x4B400000 (fp32 1.5 * 2^23): for a block sum
// |I| < 2^22 the s32 result 0x4B400000 + I, read as fp32, is exactly 12582912 + I, so the
// block integer reaches fp32 without a conversion instruction
constexpr uint32_t S8_BIAS = 0x4B400000u;
constexpr float S8_BIAS_F = 12582912.0f;
__device__ __forceinline__ void mma_s8(int c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(S8_BIAS));
}
__device__ __forceinline__ void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(s));
}
// packed fp32 pair ops (sm_100 fma.rn.f32x2 / mul.rn.f32x2 through the compiler's own
// intrinsics, so operand pairs are allocated as register pairs with no packing moves)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ void cp_async4_zfill(void *smem, const void *gmem, bool valid) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async8_zfill(void *smem, const void *gmem, bool valid) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    int n = valid ? 8 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(s), "l"(gmem), "r"(n));
}

__device__ __forceinline__ float gelu_tanh_dev(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}
__device__ __forceinline__ float silu_dev(float x) { return x / (1.0f + expf(-x)); }
// gated activations of the expert FFN (gemma4.c:432-434, 637-644; maple.c:653-655)
__device__ __forceinline__ float gated_act(int act, float g, float u, float cl) {
    if (act == ZZ_ACT_GEGLU_TANH) return gelu_tanh_dev(g) * u;
    if (act == ZZ_ACT_SWIGLU_CLAMP) {
        g = g > cl ? cl : g;
        u = u < -cl ? -cl : (u > cl ? cl : u);
    }
    return silu_dev(g) * u;
}

// --- widening two packed codes (bytes b0, b1 of a 16-bit value) to an fp16 pair ---
__device__ __forceinline__ uint32_t spread2(uint32_t v) { return __byte_perm(v, 0u, 0x4140u); }  // 00 b1 00 b0
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t h2fma(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b),
                        *reinterpret_cast<__half2 *>(&c));
    return *reinterpret_cast<uint32_t *>(&r);
}
// 0x6400 is fp16 1024.0; OR-ing a small integer into its mantissa makes 1024 + v exactly
constexpr uint32_t H1024 = 0x64006400u, H1032 = 0x64086408u, H1152 = 0x64806480u;
constexpr uint32_t H_1_16 = 0x2C002C00u, H_NEG72 = 0xD480D480u;  // 1/16, -72
// q4_0 low nibbles -> q-8
__device__ __forceinline__ uint32_t q4lo_h2(uint32_t p) { return h2sub((p & 0x000F000Fu) | H1024, H1032); }
// q4_0 high nibbles: 1024 + 16q, times 1/16 minus 72 -> q-8
__device__ __forceinline__ uint32_t q4hi_h2(uint32_t p) { return h2fma((p & 0x00F000F0u) | H1024, H_1_16, H_NEG72); }
// signed int8 -> fp16: (x ^ 0x80) = x + 128 in [0, 255]; 1024 + x + 128 - 1152 = x
__device__ __forceinline__ uint32_t s8_h2(uint32_t p) { return h2sub((p ^ 0x00800080u) | H1024, H1152); }
// tq2 2-bit codes at bit offset sh -> c
__device__ __forceinline__ uint32_t c2_h2(uint32_t p, int sh) { return h2sub(((p >> sh) & 0x00030003u) | H1024, H1024); }

template <int FMT, int BN, bool B_HALF, bool S8 = false>
struct GemmSmem {
    using T = FmtTraits<FMT>;
    static constexpr int B_STRIDE = B_HALF ? (32 * G_BKB * 2 + 16) : (32 * G_BKB + 16);  // bytes per row
    static constexpr int A_BYTES = G_BM * T::A_STRIDE;
    static constexpr int AS_BYTES = T::HAS_WSCALE ? G_BM * G_BKB * 2 : 0;
    static constexpr int B_BYTES = BN * B_STRIDE;
    static constexpr int BS_BYTES = BN * G_BKB * 4;
    static constexpr int STAGE = A_BYTES + AS_BYTES + B_BYTES + BS_BYTES;
    static constexpr int PIPE = STAGE * G_STAGES;
    static constexpr int EPI = G_BM * (BN + 4) * 4;  // fp32 C tile, padded
    static constexpr int COL = PIPE > EPI ? PIPE : EPI;  // per-column info
    static constexpr int TOTAL = COL + BN * 16;
};

// S8: int8 tensor-core path (m16n8k32.s8, int8 activations in shared memory, int32
// block sums converted to fp32); else the fp16-exact path described above.
template <int FMT, int BN, int EPI, bool B_HALF, bool S8 = false>
__device__ __forceinline__ void gemm_item(const GemmArgs &a, int item_idx) {
    using T = FmtTraits<FMT>;
    using L = GemmSmem<FMT, BN, B_HALF, S8>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;

    WorkItem it;
    if (a.items) {
        it = a.items[item_idx];
    } else {
        it.group = 0;
        it.row0 = item_idx * BN;
        it.count = min(BN, a.rows_total - it.row0);
    }
    const int m0 = blockIdx.x * G_BM;
    if (m0 >= a.O) return;
    const int nb = a.I / ZZ_BLK;
    const int nchunks = (nb + G_BKB - 1) / G_BKB;
    const int ncols = it.count;

    const uint8_t *codes = a.codes + (long)it.group * a.codes_gstride;
    const size_t code_row = (size_t)nb * T::CB;
    const size_t xrow_bytes = (size_t)a.I * (B_HALF ? 2 : 1);
    const uint8_t *xbase = reinterpret_cast<const uint8_t *>(a.xq);

    // per-column info: X row index (after gather) and the tq2 offset total
    int *col_xrow = reinterpret_cast<int *>(smem + L::COL);
    float *col_sx = reinterpret_cast<float *>(smem + L::COL + BN * 4);
    for (int n = tid; n < BN; n += G_THREADS) {
        int r = it.row0 + (n < ncols ? n : 0);
        int xr = a.gather ? a.gather[r] / a.gather_div : r;
        col_xrow[n] = xr;
        float tot = 0.f;
        if (FMT == GPU_FMT_TQ2) {
            if (a.xblk) {  // Sx of a requantized hidden row, as tq2_quant_act sums it (tq2.h:103-107)
                double acc = 0;
                for (int b = 0; b < nb; b++)
                    acc += (double)a.xs[(size_t)xr * nb + b] * (double)a.xblk[(size_t)xr * nb + b];
                tot = (float)acc;
            } else {
                tot = a.xsx[xr];
            }
        }
        col_sx[n] = tot;
    }
    __syncthreads();

    auto stage_ptr = [&](int s) { return smem + s * L::STAGE; };

    auto load_chunk = [&](int c, int s) {
        uint8_t *sa = stage_ptr(s);
        uint8_t *sas = sa + L::A_BYTES;
        uint8_t *sb = sas + L::AS_BYTES;
        uint8_t *sbs = sb + L::B_BYTES;
        const int b0 = c * G_BKB;
        const int nbk = nb - b0 < G_BKB ? nb - b0 : G_BKB;
        // A codes: 128 rows x (G_BKB*CB) bytes in 16 B pieces
        constexpr int APR = T::CB * G_BKB / 16;  // pieces per row (4, 8, 2)
        for (int i = tid; i < G_BM * APR; i += G_THREADS) {
            int r = i / APR, p = i % APR;
            int row = m0 + r;
            int blk_in = (p * 16) / T::CB;  // a piece covers 16/CB blocks
            bool ok = row < a.O && blk_in < nbk;
            const uint8_t *src = codes + (size_t)(ok ? row : 0) * code_row + (size_t)b0 * T::CB + p * 16;
            cp_async16_zfill(sa + r * T::A_STRIDE + p * 16, ok ? src : codes, ok);
        }
        if (T::HAS_WSCALE) {
            // fp16 scale rows are padded to a multiple of 8 blocks (16 B), so the 4
            // scales of a chunk are one aligned 8-byte piece, tail chunks included
            const uint8_t *sc = reinterpret_cast<const uint8_t *>(a.scale) + (long)it.group * a.scale_gstride;
            const int nbp = (nb + 7) & ~7;
            for (int r = tid; r < G_BM; r += G_THREADS) {
                int row = m0 + r;
                bool ok = row < a.O;
                const uint8_t *src = sc + ((size_t)(ok ? row : 0) * nbp + b0) * 2;
                cp_async8_zfill(sas + r * 8, src, ok);
            }
        }
        // B: BN activation rows x 4 blocks, gathered, in 16 B pieces
        constexpr int BPR = B_HALF ? 16 : 8;
        constexpr int PPB = BPR / G_BKB;  // pieces per block
        for (int i = tid; i < BN * BPR; i += G_THREADS) {
            int n = i / BPR, p = i % BPR;
            bool ok = n < ncols && (p / PPB) < nbk;
            const uint8_t *src = xbase + (size_t)col_xrow[n] * xrow_bytes + (size_t)b0 * (B_HALF ? 64 : 32) + p * 16;
            cp_async16_zfill(sb + n * L::B_STRIDE + p * 16, ok ? (const void *)src : (const void *)xbase, ok);
        }
        // activation scales per block, [block][column] (a column pair is one 8-byte load)
        for (int i = tid; i < BN * G_BKB; i += G_THREADS) {
            int n = i / G_BKB, k = i % G_BKB;
            bool ok = n < ncols && k < nbk;
            const float *src = a.xs + (size_t)col_xrow[n] * nb + b0 + k;
            cp_async4_zfill(sbs + (k * BN + n) * 4, ok ? (const void *)src : (const void *)a.xs, ok);
        }
    };

    constexpr int NT = BN / 8;
    static_assert(!S8 || NT % 2 == 0, "int8 path pairs n8 tiles");
    float2 acc[NT][2];  // [n8 tile][row g | row g+8] x column pair (2t, 2t+1)
#pragma unroll
    for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = make_float2(0.f, 0.f);
    const int jv = (ncols + 7) >> 3;  // n8 tiles holding valid columns (warp-uniform)

    const int rA = warp * 16 + g;
    if constexpr (S8) {
        // ---- int8 path (m16n8k32.s8). Each thread's copies are fixed for the item, so a
        // chunk only moves the sources along K. The activation scales sit in shared memory
        // as [block][t][tile][pair]: the 2 NT scales of the column pairs (8j + 2t,
        // 8j + 2t + 1) that one thread uses in a block are 16-byte loads ----
        constexpr int APR = T::CB * G_BKB / 16;          // 16-byte code pieces per row and chunk
        constexpr int NA = G_BM * APR / G_THREADS;       // per thread: 2 (q4_0), 4 (q8_0), 1 (tq2)
        static_assert(NA >= 1 && G_BM * APR % G_THREADS == 0, "code pieces per thread");
        static_assert(BN * 8 % G_THREADS == 0, "whole activation pieces per thread");
        constexpr int NBP = BN * 8 / G_THREADS, BSTEP = G_THREADS / 8;  // pieces per thread, row step
        static_assert(BN * G_BKB <= G_THREADS, "one activation scale per thread");
        // piece k of this thread: row r0 + k * RSTEP, the same 16 bytes of it
        constexpr int RSTEP = G_THREADS / APR;
        const int r0 = tid / APR, ap = tid % APR, alim = (ap * 16) / T::CB;
        const uint8_t *asrc = codes + (size_t)(m0 + r0) * code_row + ap * 16;
        const uint32_t adst = r0 * T::A_STRIDE + ap * 16;
        const uint8_t *sc = T::HAS_WSCALE ? reinterpret_cast<const uint8_t *>(a.scale) + (long)it.group * a.scale_gstride
                                          : nullptr;
        const int nbp = (nb + 7) & ~7;
        const bool s_ok = T::HAS_WSCALE && tid < G_BM && m0 + tid < a.O;
        const uint8_t *ssrc = s_ok ? sc + (size_t)(m0 + tid) * nbp * 2 : sc;
        const int bn_ = tid >> 3, bp = tid & 7;  // piece k: row bn_ + k BSTEP, bytes 16 bp of the chunk
        const uint8_t *bsrc[NBP];
#pragma unroll
        for (int k = 0; k < NBP; k++) bsrc[k] = xbase + (size_t)col_xrow[bn_ + k * BSTEP] * xrow_bytes + bp * 16;
        const int sn = (tid >> 2) % BN, sk = tid & 3;
        const bool d_thr = tid < BN * G_BKB, d_ok = d_thr && sn < ncols;
        const float *dsrc = a.xs + (size_t)col_xrow[sn] * nb + sk;
        const int dpos = (sk * BN + ((sn % 8) / 2) * (2 * NT) + (sn / 8) * 2 + (sn % 2)) * 4;

        auto load8 = [&](int c, int s) {
            uint8_t *sa = stage_ptr(s);
            uint8_t *sas = sa + L::A_BYTES;
            uint8_t *sb = sas + L::AS_BYTES;
            uint8_t *sbs = sb + L::B_BYTES;
            const int b0 = c * G_BKB;
            const int nbk = nb - b0 < G_BKB ? nb - b0 : G_BKB;
#pragma unroll
            for (int k = 0; k < NA; k++) {
                const bool ok = alim < nbk && m0 + r0 + k * RSTEP < a.O;
                cp_async16_zfill(sa + adst + k * RSTEP * T::A_STRIDE,
                                 ok ? asrc + (size_t)k * RSTEP * code_row + (size_t)b0 * T::CB : codes, ok);
            }
            if (T::HAS_WSCALE && tid < G_BM) cp_async8_zfill(sas + tid * 8, ssrc + b0 * 2, s_ok);
#pragma unroll
            for (int k = 0; k < NBP; k++) {
                const bool ok = bn_ + k * BSTEP < ncols && (bp >> 1) < nbk;
                cp_async16_zfill(sb + (bn_ + k * BSTEP) * L::B_STRIDE + bp * 16, ok ? bsrc[k] + b0 * 32 : xbase, ok);
            }
            if (d_thr) {
                const bool ok = d_ok && sk < nbk;
                cp_async4_zfill(sbs + dpos, ok ? dsrc + b0 : a.xs, ok);
            }
        };

#pragma unroll
        for (int s = 0; s < G_STAGES - 1; s++) {
            if (s < nchunks) load8(s, s);
            cp_async_commit();
        }
        for (int c = 0; c < nchunks; c++) {
            cp_async_wait<G_STAGES - 2>();
            __syncthreads();
            {
                int cn = c + G_STAGES - 1;
                if (cn < nchunks) load8(cn, cn % G_STAGES);
                cp_async_commit();
            }
            const uint8_t *sa = stage_ptr(c % G_STAGES);
            const uint8_t *sas = sa + L::A_BYTES;
            const uint8_t *sb = sas + L::AS_BYTES;
            const float *sbs = reinterpret_cast<const float *>(sb + L::B_BYTES);
            const int nbk = nb - c * G_BKB < G_BKB ? nb - c * G_BKB : G_BKB;
            auto blk = [&](int kb) {
                uint32_t a0, a1, a2, a3;
                const uint8_t *r0 = sa + rA * T::A_STRIDE, *r1 = r0 + 8 * T::A_STRIDE;
                if (FMT == GPU_FMT_Q40) {
                    // low nibbles are k = j, high k = j + 16: the fragment split. Nibble q
                    // to the high half of its byte xor 8 gives the signed byte 16 (q - 8)
                    uint32_t w0 = *reinterpret_cast<const uint32_t *>(r0 + kb * 16 + 4 * t);
                    uint32_t w1 = *reinterpret_cast<const uint32_t *>(r1 + kb * 16 + 4 * t);
                    a0 = ((w0 << 4) & 0xF0F0F0F0u) ^ 0x80808080u; a2 = (w0 & 0xF0F0F0F0u) ^ 0x80808080u;
                    a1 = ((w1 << 4) & 0xF0F0F0F0u) ^ 0x80808080u; a3 = (w1 & 0xF0F0F0F0u) ^ 0x80808080u;
                } else if (FMT == GPU_FMT_Q80) {
                    const uint8_t *p0 = r0 + kb * 32 + 4 * t, *p1 = r1 + kb * 32 + 4 * t;
                    a0 = *reinterpret_cast<const uint32_t *>(p0); a2 = *reinterpret_cast<const uint32_t *>(p0 + 16);
                    a1 = *reinterpret_cast<const uint32_t *>(p1); a3 = *reinterpret_cast<const uint32_t *>(p1 + 16);
                } else {
                    const int sh = (kb & 1) * 4;
                    uint32_t w0 = *reinterpret_cast<const uint32_t *>(r0 + (kb >> 1) * 16 + 4 * t);
                    uint32_t w1 = *reinterpret_cast<const uint32_t *>(r1 + (kb >> 1) * 16 + 4 * t);
                    a0 = (w0 >> sh) & 0x03030303u; a2 = (w0 >> (sh + 2)) & 0x03030303u;
                    a1 = (w1 >> sh) & 0x03030303u; a3 = (w1 >> (sh + 2)) & 0x03030303u;
                }
                float2 dw0 = make_float2(1.f, 1.f), dw1 = dw0;
                float2 cm0 = make_float2(-S8_BIAS_F, -S8_BIAS_F), cm1 = cm0;
                if (T::HAS_WSCALE) {
                    const __half *hs = reinterpret_cast<const __half *>(sas);
                    float w0 = __half2float(hs[rA * G_BKB + kb]), w1 = __half2float(hs[(rA + 8) * G_BKB + kb]);
                    if (FMT == GPU_FMT_Q40) { w0 *= 0.0625f; w1 *= 0.0625f; }
                    dw0 = make_float2(w0, w0); dw1 = make_float2(w1, w1);
                    cm0 = make_float2(-S8_BIAS_F * w0, -S8_BIAS_F * w0); cm1 = make_float2(-S8_BIAS_F * w1, -S8_BIAS_F * w1);
                }
                auto tile = [&](int j, uint32_t b0, uint32_t b1, float2 dx) {
                    int cc[4];
                    mma_s8(cc, a0, a1, a2, a3, b0, b1);
                    const float2 f01 = make_float2(__int_as_float(cc[0]), __int_as_float(cc[1]));
                    const float2 f23 = make_float2(__int_as_float(cc[2]), __int_as_float(cc[3]));
                    // dw * I rounded once, then + dx * (dw * I)
                    acc[j][0] = ffma2(ffma2(f01, dw0, cm0), dx, acc[j][0]);
                    acc[j][1] = ffma2(ffma2(f23, dw1, cm1), dx, acc[j][1]);
                };
                // B fragments of n8 tiles jp, jp + 1 per ldmatrix.x4 and their 4 activation
                // scales per 16-byte load (columns 8j + 2t, 8j + 2t + 1)
#pragma unroll
                for (int jp = 0; jp < NT; jp += 2) {
                    if (jp < jv) {
                        uint32_t b0, b1, b2, b3;
                        const int lrow = (jp + (lane >> 4)) * 8 + (lane & 7);
                        ldsm_x4(b0, b1, b2, b3, sb + lrow * L::B_STRIDE + kb * 32 + ((lane >> 3) & 1) * 16);
                        const float4 dx = *reinterpret_cast<const float4 *>(sbs + kb * BN + t * 2 * NT + 2 * jp);
                        tile(jp, b0, b1, make_float2(dx.x, dx.y));
                        if (jp + 1 < jv) tile(jp + 1, b2, b3, make_float2(dx.z, dx.w));
                    }
                }
            };
            if (nbk == G_BKB) {
#pragma unroll
                for (int kb = 0; kb < G_BKB; kb++) blk(kb);
            } else {
                for (int kb = 0; kb < nbk; kb++) blk(kb);
            }
        }
    } else {
    #pragma unroll
        for (int s = 0; s < G_STAGES - 1; s++) {
            if (s < nchunks) load_chunk(s, s);
            cp_async_commit();
        }
        for (int c = 0; c < nchunks; c++) {
            cp_async_wait<G_STAGES - 2>();
            __syncthreads();
            {
                int cn = c + G_STAGES - 1;
                if (cn < nchunks) load_chunk(cn, cn % G_STAGES);
                cp_async_commit();
            }
            const uint8_t *sa = stage_ptr(c % G_STAGES);
            const uint8_t *sas = sa + L::A_BYTES;
            const uint8_t *sb = sas + L::AS_BYTES;
            const float *sbs = reinterpret_cast<const float *>(sb + L::B_BYTES);
            const int nbk = nb - c * G_BKB < G_BKB ? nb - c * G_BKB : G_BKB;
            // one K block: fragments, MMAs for the valid n8 tiles, block-scale epilogue
            auto block = [&](int kb) {
                // A fragments of the two k16 steps of this block: s0 = k 0..15, s1 = k 16..31
                uint32_t a0[4], a1[4];  // {row g k 2t.., row g+8 k 2t.., row g k 2t+8.., row g+8 k 2t+8..}
                {
                    const uint8_t *r0 = sa + rA * T::A_STRIDE, *r1 = r0 + 8 * T::A_STRIDE;
                    if (FMT == GPU_FMT_Q40) {
                        const int o = kb * 16 + 2 * t;
                        uint32_t p00 = spread2(*reinterpret_cast<const uint16_t *>(r0 + o));
                        uint32_t p10 = spread2(*reinterpret_cast<const uint16_t *>(r1 + o));
                        uint32_t p01 = spread2(*reinterpret_cast<const uint16_t *>(r0 + o + 8));
                        uint32_t p11 = spread2(*reinterpret_cast<const uint16_t *>(r1 + o + 8));
                        a0[0] = q4lo_h2(p00); a0[1] = q4lo_h2(p10); a0[2] = q4lo_h2(p01); a0[3] = q4lo_h2(p11);
                        a1[0] = q4hi_h2(p00); a1[1] = q4hi_h2(p10); a1[2] = q4hi_h2(p01); a1[3] = q4hi_h2(p11);
                    } else if (FMT == GPU_FMT_Q80) {
                        const int o = kb * 32 + 2 * t;
                        a0[0] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r0 + o)));
                        a0[1] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r1 + o)));
                        a0[2] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r0 + o + 8)));
                        a0[3] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r1 + o + 8)));
                        a1[0] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r0 + o + 16)));
                        a1[1] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r1 + o + 16)));
                        a1[2] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r0 + o + 24)));
                        a1[3] = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(r1 + o + 24)));
                    } else {
                        const int o = (kb >> 1) * 16 + 2 * t, sh = (kb & 1) * 4;
                        uint32_t p00 = spread2(*reinterpret_cast<const uint16_t *>(r0 + o));
                        uint32_t p10 = spread2(*reinterpret_cast<const uint16_t *>(r1 + o));
                        uint32_t p01 = spread2(*reinterpret_cast<const uint16_t *>(r0 + o + 8));
                        uint32_t p11 = spread2(*reinterpret_cast<const uint16_t *>(r1 + o + 8));
                        a0[0] = c2_h2(p00, sh); a0[1] = c2_h2(p10, sh); a0[2] = c2_h2(p01, sh); a0[3] = c2_h2(p11, sh);
                        a1[0] = c2_h2(p00, sh + 2); a1[1] = c2_h2(p10, sh + 2);
                        a1[2] = c2_h2(p01, sh + 2); a1[3] = c2_h2(p11, sh + 2);
                    }
                }
                float2 dw0 = make_float2(1.f, 1.f), dw1 = make_float2(1.f, 1.f);
                if (T::HAS_WSCALE) {
                    const __half *hs = reinterpret_cast<const __half *>(sas);
                    float w0 = __half2float(hs[rA * G_BKB + kb]), w1 = __half2float(hs[(rA + 8) * G_BKB + kb]);
                    dw0 = make_float2(w0, w0);
                    dw1 = make_float2(w1, w1);
                }
    #pragma unroll
                for (int j = 0; j < NT; j++) {
                    if (j < jv) {
                        uint32_t b00, b01, b10, b11;  // step 0: k 2t.., k 2t+8..; step 1: +16
                        if (B_HALF) {
                            // lanes 0-7 address k 0-7 of rows n, 8-15 k 8-15, 16-23 k 16-23, 24-31 k 24-31
                            const uint8_t *pb = sb + (j * 8 + (lane & 7)) * L::B_STRIDE + kb * 64 + (lane >> 3) * 16;
                            ldsm_x4(b00, b01, b10, b11, pb);
                        } else {
                            const uint8_t *pb = sb + (j * 8 + g) * L::B_STRIDE + kb * 32 + 2 * t;
                            b00 = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(pb)));
                            b01 = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(pb + 8)));
                            b10 = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(pb + 16)));
                            b11 = s8_h2(spread2(*reinterpret_cast<const uint16_t *>(pb + 24)));
                        }
                        float d[4];
                        mma_f16(d, a0[0], a0[1], a0[2], a0[3], b00, b01, 0.f, 0.f, 0.f, 0.f);
                        mma_f16(d, a1[0], a1[1], a1[2], a1[3], b10, b11, d[0], d[1], d[2], d[3]);
                        // d = this block's exact integer sums; scale by dw*dx and accumulate
                        const float2 dx = *reinterpret_cast<const float2 *>(sbs + kb * BN + j * 8 + 2 * t);
                        if (T::HAS_WSCALE) {
                            acc[j][0] = ffma2(fmul2(dw0, dx), make_float2(d[0], d[1]), acc[j][0]);
                            acc[j][1] = ffma2(fmul2(dw1, dx), make_float2(d[2], d[3]), acc[j][1]);
                        } else {
                            acc[j][0] = ffma2(dx, make_float2(d[0], d[1]), acc[j][0]);
                            acc[j][1] = ffma2(dx, make_float2(d[2], d[3]), acc[j][1]);
                        }
                    }
                }
            };
            if (nbk == G_BKB) {
                // full chunk: unrolled so the 4 blocks' MMA -> FMA chains interleave
    #pragma unroll
                for (int kb = 0; kb < G_BKB; kb++) block(kb);
            } else {
                for (int kb = 0; kb < nbk; kb++) block(kb);
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---- epilogue: C tile to shared memory [128][BN+4] fp32 ----
    float *ct = reinterpret_cast<float *>(smem);
    constexpr int CS = BN + 4;
#pragma unroll
    for (int j = 0; j < NT; j++) {
        *reinterpret_cast<float2 *>(ct + rA * CS + j * 8 + 2 * t) = acc[j][0];
        *reinterpret_cast<float2 *>(ct + (rA + 8) * CS + j * 8 + 2 * t) = acc[j][1];
    }
    __syncthreads();

    const float *alpha = FMT == GPU_FMT_TQ2 ? reinterpret_cast<const float *>(
                                                  reinterpret_cast<const uint8_t *>(a.scale) + (long)it.group * a.scale_gstride)
                                            : nullptr;
    if (EPI == EPI_STORE) {
        // each warp takes columns; lanes walk rows (coalesced along o)
        for (int n = warp; n < ncols; n += 8) {
            int xr = col_xrow[n];
            float tot = col_sx[n];
            for (int r = lane; r < G_BM; r += 32) {
                int o = m0 + r;
                if (o < a.O) {
                    float v = ct[r * CS + n];
                    if (FMT == GPU_FMT_TQ2) v = alpha[o] * (v - tot);
                    a.y[(size_t)xr * a.O + o] = v;
                }
            }
        }
    } else if (EPI == EPI_GATEUP) {
        // features f0 .. f0+63 of this tile; h = act(gate, up); requant per 32-block
        const int f0 = (m0 / 128) * 64;
        const int MI = a.O / 2, nbh = MI / 32;
        for (int wi = warp; wi < ncols * 2; wi += 8) {
            int n = wi >> 1, hb = wi & 1;
            int f = hb * 32 + lane;
            float gv = ct[f * CS + n], uv = ct[(64 + f) * CS + n];
            if (FMT == GPU_FMT_TQ2) {
                float tot = col_sx[n];
                // rows of the interleaved stack: gate feature f -> tile row f, up -> 64+f
                gv = alpha[m0 + f] * (gv - tot);
                uv = alpha[m0 + 64 + f] * (uv - tot);
            }
            float h = gated_act(a.act, gv, uv, a.clamp), d;
            int8_t q = quant_lane(h, d);
            const size_t pr = (size_t)(it.row0 + n);
            a.hq[pr * MI + f0 + f] = q;
            if (a.hh) a.hh[pr * MI + f0 + f] = __int2half_rn(q);
            if (a.hhs) {
                // the folded-scale down GEMM's B planes: fp16 hi and lo of d * q
                const float v = (float)q * d;
                const __half hi = __float2half_rn(v);
                a.hhs[pr * MI + f0 + f] = hi;
                a.hhs[(size_t)a.rows_cap * MI + pr * MI + f0 + f] = __float2half_rn(v - __half2float(hi));
            }
            if (lane == 0) a.hs[pr * nbh + f0 / 32 + hb] = d;
            if (FMT == GPU_FMT_TQ2) {
                int s = q;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0) a.hblk[pr * nbh + f0 / 32 + hb] = s;
            }
        }
    } else {  // EPI_DOWN
        for (int n = warp; n < ncols; n += 8) {
            const int pr = it.row0 + n;
            const float w = a.pair_w[pr];
            const int tok = a.pair_src[pr] / a.K;
            const float tot = col_sx[n];
            int r = lane * 4;
            int o = m0 + r;
            if (o + 3 < a.O) {
                float4 v;
                v.x = ct[r * CS + n]; v.y = ct[(r + 1) * CS + n]; v.z = ct[(r + 2) * CS + n]; v.w = ct[(r + 3) * CS + n];
                if (FMT == GPU_FMT_TQ2) {
                    v.x = alpha[o] * (v.x - tot); v.y = alpha[o + 1] * (v.y - tot);
                    v.z = alpha[o + 2] * (v.z - tot); v.w = alpha[o + 3] * (v.w - tot);
                }
                v.x *= w; v.y *= w; v.z *= w; v.w *= w;
                atomicAdd(reinterpret_cast<float4 *>(a.out + (size_t)tok * a.O + o), v);
            } else {
                for (int k = 0; k < 4; k++)
                    if (o + k < a.O) {
                        float v = ct[(r + k) * CS + n];
                        if (FMT == GPU_FMT_TQ2) v = alpha[o + k] * (v - tot);
                        atomicAdd(a.out + (size_t)tok * a.O + o + k, w * v);
                    }
            }
        }
    }
}

// One work item per grid row; with STRIDE the items are strided over grid.y instead (a
// grid capped below the worst-case item count then launches no CTA that finds no item;
// the loop costs a few registers, so exact grids use the plain form).
template <int FMT, int BN, int EPI, bool B_HALF, bool S8 = false, bool STRIDE = false>
// CTAs per SM the register budget targets (measured best): 3 for the 32-row gate/up GEMM
// (78 registers, no spills), 4 for the 32-row down GEMM (64), 3 for 64-row items and the
// dense matmul
__global__ void __launch_bounds__(G_THREADS, BN <= 32 ? (EPI == EPI_GATEUP ? 3 : 4) : 3) k_gemm(GemmArgs a) {
    const int n = a.n_items ? *a.n_items : (int)gridDim.y;
    if constexpr (!STRIDE) {
        if ((int)blockIdx.y < n) gemm_item<FMT, BN, EPI, B_HALF, S8>(a, blockIdx.y);
    } else {
        for (int y = blockIdx.y; y < n; y += gridDim.y) {
            gemm_item<FMT, BN, EPI, B_HALF, S8>(a, y);
            __syncthreads();  // shared memory is reused by the next item
        }
    }
}

}  // namespace zz
