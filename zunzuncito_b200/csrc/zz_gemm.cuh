// zz_gemm.cuh -- grouped block-scaled int8 GEMM over q4_0 / q8_0 / tq2 planes.
//
// C[o, n] = sum_b  dw[o,b] * dx[n,b] * <A_o,b , X_n,b>     (tq2: dx[n,b] only)
//
// The per-block scales vary along both o and n, so int32 partials cannot be carried
// across 32-wide K blocks: every block's integer product is converted and scaled into
// fp32 accumulators before the next block (the decomposition of q40.h:20-31). One
// tensor-core MMA of K=32 therefore matches exactly one q4_0 block.
//
// CTA tile: 128 weight rows x BN activation rows, 8 warps of 16 rows each. K moves in
// chunks of 4 blocks (128 weights) through a 4-stage cp.async pipeline; nibble / 2-bit
// codes are widened to int8 in registers straight into the MMA fragment (the q4_0
// byte layout -- low nibble k, high nibble k+16 -- is exactly the m16n8k32 A-fragment
// split, so one 32-bit shared load feeds two fragment registers).
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

constexpr int G_BM = 128, G_BKB = 4, G_STAGES = 4, G_THREADS = 256;

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
    const int8_t *xq;
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
    float *hs;               // [pair][O/64]
    int *hblk;               // [pair][O/64] (tq2 only)
    // EPI_DOWN
    float *out;              // [token][O]
    const float *pair_w;     // [pair]
    const int *pair_src;     // [pair] routing slot s*K+k of the pair
    int K;
};

__device__ __forceinline__ void mma_s8(int c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}
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
__device__ __forceinline__ float gated_act(int act, float g, float u, float cl) {
    if (act == ZZ_ACT_GEGLU_TANH) return gelu_tanh_dev(g) * u;
    if (act == ZZ_ACT_SWIGLU_CLAMP) {
        g = g > cl ? cl : g;
        u = u < -cl ? -cl : (u > cl ? cl : u);
    }
    return silu_dev(g) * u;
}

template <int FMT, int BN>
struct GemmSmem {
    using T = FmtTraits<FMT>;
    static constexpr int B_STRIDE = 32 * G_BKB + 16;
    static constexpr int A_BYTES = G_BM * T::A_STRIDE;
    static constexpr int AS_BYTES = T::HAS_WSCALE ? G_BM * G_BKB * 2 : 0;
    static constexpr int B_BYTES = BN * B_STRIDE;
    static constexpr int BS_BYTES = BN * G_BKB * 4;
    static constexpr int STAGE = A_BYTES + AS_BYTES + B_BYTES + BS_BYTES;
    static constexpr int PIPE = STAGE * G_STAGES;
    static constexpr int EPI = G_BM * (BN + 4) * 4;  // fp32 C tile, padded
    static constexpr int TOTAL = (PIPE > EPI ? PIPE : EPI) + BN * 16;  // + per-column info
};

template <int FMT, int BN, int EPI>
__global__ void __launch_bounds__(G_THREADS) k_gemm(GemmArgs a) {
    using T = FmtTraits<FMT>;
    using L = GemmSmem<FMT, BN>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;

    const int item_idx = blockIdx.y;
    if (a.n_items && item_idx >= *a.n_items) return;
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

    // per-column info: X row index (after gather)
    int *col_xrow = reinterpret_cast<int *>(smem + L::TOTAL - BN * 16);
    float *col_sx = reinterpret_cast<float *>(smem + L::TOTAL - BN * 12);
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
            // a 16 B piece covers 16/CB blocks (1 for q4, half for q8, 2 for tq2)
            int blk_in = (p * 16) / T::CB;
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
        // B: BN activation rows x 128 bytes (8 pieces), gathered
        for (int i = tid; i < BN * 8; i += G_THREADS) {
            int n = i >> 3, p = i & 7;
            bool ok = n < ncols && (p >> 1) < nbk;
            const int8_t *src = a.xq + (size_t)col_xrow[n] * a.I + (size_t)b0 * 32 + p * 16;
            cp_async16_zfill(sb + n * L::B_STRIDE + p * 16, ok ? (const void *)src : (const void *)a.xq, ok);
        }
        for (int i = tid; i < BN * G_BKB; i += G_THREADS) {
            int n = i / G_BKB, k = i % G_BKB;
            bool ok = n < ncols && k < nbk;
            const float *src = a.xs + (size_t)col_xrow[n] * nb + b0 + k;
            cp_async4_zfill(sbs + (n * G_BKB + k) * 4, ok ? (const void *)src : (const void *)a.xs, ok);
        }
    };

    constexpr int NT = BN / 8;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[j][e] = 0.f;
    const int jv = (ncols + 7) >> 3;  // n8 tiles holding valid columns (warp-uniform)

#pragma unroll
    for (int s = 0; s < G_STAGES - 1; s++) {
        if (s < nchunks) load_chunk(s, s);
        cp_async_commit();
    }
    const int rA = warp * 16 + g;
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
        for (int kb = 0; kb < nbk; kb++) {
            uint32_t a0, a1, a2, a3;
            if (FMT == GPU_FMT_Q40) {
                uint32_t w0 = *reinterpret_cast<const uint32_t *>(sa + rA * T::A_STRIDE + kb * 16 + 4 * t);
                uint32_t w1 = *reinterpret_cast<const uint32_t *>(sa + (rA + 8) * T::A_STRIDE + kb * 16 + 4 * t);
                a0 = nib_to_s8(w0); a2 = nib_to_s8(w0 >> 4);
                a1 = nib_to_s8(w1); a3 = nib_to_s8(w1 >> 4);
            } else if (FMT == GPU_FMT_Q80) {
                const uint8_t *p0 = sa + rA * T::A_STRIDE + kb * 32 + 4 * t;
                const uint8_t *p1 = p0 + 8 * T::A_STRIDE;
                a0 = *reinterpret_cast<const uint32_t *>(p0); a2 = *reinterpret_cast<const uint32_t *>(p0 + 16);
                a1 = *reinterpret_cast<const uint32_t *>(p1); a3 = *reinterpret_cast<const uint32_t *>(p1 + 16);
            } else {
                const int sh = (kb & 1) * 4;
                uint32_t w0 = *reinterpret_cast<const uint32_t *>(sa + rA * T::A_STRIDE + (kb >> 1) * 16 + 4 * t);
                uint32_t w1 = *reinterpret_cast<const uint32_t *>(sa + (rA + 8) * T::A_STRIDE + (kb >> 1) * 16 + 4 * t);
                a0 = (w0 >> sh) & 0x03030303u; a2 = (w0 >> (sh + 2)) & 0x03030303u;
                a1 = (w1 >> sh) & 0x03030303u; a3 = (w1 >> (sh + 2)) & 0x03030303u;
            }
            float dw0 = 1.f, dw1 = 1.f;
            if (T::HAS_WSCALE) {
                const __half *hs = reinterpret_cast<const __half *>(sas);
                dw0 = __half2float(hs[rA * G_BKB + kb]);
                dw1 = __half2float(hs[(rA + 8) * G_BKB + kb]);
            }
#pragma unroll
            for (int j = 0; j < NT; j++) {
                if (j < jv) {
                    const uint8_t *pb = sb + (j * 8 + g) * L::B_STRIDE + kb * 32 + 4 * t;
                    uint32_t b0 = *reinterpret_cast<const uint32_t *>(pb);
                    uint32_t b1 = *reinterpret_cast<const uint32_t *>(pb + 16);
                    int cc[4];
                    mma_s8(cc, a0, a1, a2, a3, b0, b1);
                    float dx0 = sbs[(j * 8 + 2 * t) * G_BKB + kb];
                    float dx1 = sbs[(j * 8 + 2 * t + 1) * G_BKB + kb];
                    if (T::HAS_WSCALE) {
                        acc[j][0] = fmaf(dw0 * dx0, (float)cc[0], acc[j][0]);
                        acc[j][1] = fmaf(dw0 * dx1, (float)cc[1], acc[j][1]);
                        acc[j][2] = fmaf(dw1 * dx0, (float)cc[2], acc[j][2]);
                        acc[j][3] = fmaf(dw1 * dx1, (float)cc[3], acc[j][3]);
                    } else {
                        acc[j][0] = fmaf(dx0, (float)cc[0], acc[j][0]);
                        acc[j][1] = fmaf(dx1, (float)cc[1], acc[j][1]);
                        acc[j][2] = fmaf(dx0, (float)cc[2], acc[j][2]);
                        acc[j][3] = fmaf(dx1, (float)cc[3], acc[j][3]);
                    }
                }
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
        ct[rA * CS + j * 8 + 2 * t] = acc[j][0];
        ct[rA * CS + j * 8 + 2 * t + 1] = acc[j][1];
        ct[(rA + 8) * CS + j * 8 + 2 * t] = acc[j][2];
        ct[(rA + 8) * CS + j * 8 + 2 * t + 1] = acc[j][3];
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

}  // namespace zz
