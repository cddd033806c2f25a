// zz_moe_i8.cu -- the batch-union expert GEMMs on the 5th-generation tensor cores with
// int8 operands (tcgen05.mma kind::i8, s32 accumulators in TMEM).
//
// C[o, n] = sum_b dw[o,b] * dx[n,b] * I_b[o,n],   I_b = sum_{j<32} q[o,32b+j] * x[n,32b+j]
// (the per-block decomposition of q40.h:20-31 / tq2.h:116-133). The block scales vary
// along both o and n, so every 32-wide K block is its own MMA (K = 32 for int8) into its
// own TMEM columns, and the integer block sums are scaled into fp32 sums by the epilogue.
//
// Two device facts shape the epilogue, which bounds the kernel:
//  * TMEM is preset with the bit pattern 0x4B400000 (fp32 1.5 * 2^23) and every MMA
//    accumulates onto it. For |I| < 2^22 the s32 result 0x4B400000 + I, read as fp32, is
//    exactly 12582912 + I, so no int->fp32 conversion instruction is needed: with
//    c = -12582912 * dw (exact in fp32: dw has 11 significant bits), fma(F, dw, c) is
//    dw * I rounded once, and one more fma adds dx * (dw * I) into the running sum.
//    Both are packed (fma.rn.f32x2): one instruction per element and block. After
//    reading a block's columns the epilogue writes the preset back (tcgen05.st).
//  * q4_0 nibbles are widened to 16 * (q - 8) (one shift and one lop3 per 4 codes); the
//    weight scale dw / 16 (a power-of-two change, exact) absorbs the factor 16.
//    |I| <= 16 * 8 * 127 * 32 < 2^22.
//
// Persistent, warp-specialised, one CTA per SM; work tiles are (item, 128 weight rows),
// items being (expert, <= 128 routed rows) listed by the router in decreasing row
// count. K advances in stages of 8 blocks (256 weights). Roles (512 threads; registers
// moved from the copy warpgroups to the epilogue with setmaxnreg):
//   warp 12      TMA: the weight codes of a stage (one 128-row box; for q8_0 two boxes
//                straight into the MMA operand layout) and the fp16 weight scales
//   warp 13      TMA: the stage's int8 activation rows (128-byte-swizzled K-major boxes
//                of 16/32/64/128 rows), bulk copies of their block scales
//   warps 8-11   producers (q4_0, tq2): thread r widens row r's codes of the stage to
//                int8 in the 128-byte-swizzled K-major layout the MMA reads
//   warp 14      MMA: one thread issues one tcgen05.mma kind::i8 (M = 128, N = rows
//                rounded to 16, K = 32) per block into a TMEM group (4 groups of 128
//                columns; a group holds 128 / N' blocks, N' = N rounded to a power of 2
//                and at least 32, so narrow tiles keep several blocks in flight)
//   warp 15      idle
//   warps 0-7    epilogue: warp (q, h) reads TMEM lanes 32q..32q+31 (one weight row per
//                thread) and columns [h N'/2, (h+1) N'/2) of every block, adding the
//                blocks in K order into one fp32 sum per column. Tile end: gate/up
//                GeGLU / SwiGLU + q8_0 requant (bit-exact with q40_quant_act), or the
//                down projection's weighted scatter-add into OUT.
// Every wait is bounded (2 s of %globaltimer); one that runs out sets the kernel's error
// word and the CTA drains, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include "zz_gemm.cuh"
#include "zz_tc.cuh"

namespace zz {

namespace i8k {
constexpr int NTHREADS = 512;         // 4 warpgroups: 2 epilogue, producers, copies + MMA
// per-thread registers after the warpgroups rebalance (setmaxnreg): launched with 128 each
// (512 x 128 = the SM's 65536), the producer and copy/MMA warpgroups give back 56 and
// 88 per thread, which lets the two epilogue warpgroups grow to 200:
// 2 x 128 x 200 + 128 x 72 + 128 x 40 = 65536
constexpr int REG_EPI = 200, REG_PROD = 72, REG_COPY = 40;
static_assert(2 * 128 * REG_EPI + 128 * REG_PROD + 128 * REG_COPY == 65536, "register split");
constexpr int BN = 128;              // max rows (tokens) per tile
constexpr int KB = 8;                // quantization blocks per stage
constexpr int NGRP = 4;              // TMEM groups of 128 columns
constexpr int A_ATOM = 128 * 128;    // 128 rows x 128 bytes (4 blocks), 128-byte swizzle
constexpr int A_STAGE = 2 * A_ATOM;  // 8 blocks
constexpr int NS = 2;
constexpr int B_STAGE = 2 * BN * 128;
constexpr int RB = 2;
constexpr int RING = 32 * 1024;      // weight-code ring (q4_0: 2 slots, tq2: 4)
constexpr int RC_MAX = 4;
constexpr int ND = 4;
constexpr int DX_STAGE = KB * BN * 4;
constexpr int NW = 4;
constexpr int W_SLOT = 128 * KB * 2;
constexpr int CTX = 64 + 1;          // tile-end exchange: 128 rows x 64 columns
constexpr int CT_BYTES = 128 * CTX * 4;
constexpr int OFF_A = 0;             // 1 KB aligned (swizzled destinations)
constexpr int OFF_B = OFF_A + NS * A_STAGE;
constexpr int OFF_RING = OFF_B + RB * B_STAGE;
constexpr int OFF_DX = OFF_RING + RING;
constexpr int OFF_W = OFF_DX + ND * DX_STAGE;
constexpr int OFF_CT = OFF_W + NW * W_SLOT;
constexpr int OFF_BAR = OFF_CT + CT_BYTES;
constexpr int NBAR = 2 * RC_MAX + 2 * NS + 2 * RB + 2 * ND + 2 * NW + 2 * NGRP + 1;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + slack to align the base to 1 KB
static_assert(SMEM <= 232448, "shared memory");
constexpr uint32_t BIAS = 0x4B400000u;   // fp32 12582912.0
constexpr float BIAS_F = 12582912.0f;
}  // namespace i8k

struct BMaps8 {
    CUtensorMap m[4];  // int8 activation boxes of 128 bytes x 16, 32, 64, 128 rows
};

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// the preset value into 16 consecutive columns of the warp's 32 lanes
__device__ __forceinline__ void tmem_st16_bias(uint32_t taddr) {
    const uint32_t b = i8k::BIAS;
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(b)
        : "memory");
}
// tcgen05.wait::ld that also names the loaded registers, so no use of them can be
// scheduled before the wait
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&v)[4][16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0][0]), "+r"(v[0][1]), "+r"(v[0][2]), "+r"(v[0][3]), "+r"(v[0][4]), "+r"(v[0][5]), "+r"(v[0][6]), "+r"(v[0][7]), "+r"(v[0][8]), "+r"(v[0][9]), "+r"(v[0][10]), "+r"(v[0][11]), "+r"(v[0][12]), "+r"(v[0][13]), "+r"(v[0][14]), "+r"(v[0][15]), "+r"(v[1][0]), "+r"(v[1][1]), "+r"(v[1][2]), "+r"(v[1][3]), "+r"(v[1][4]), "+r"(v[1][5]), "+r"(v[1][6]), "+r"(v[1][7]), "+r"(v[1][8]), "+r"(v[1][9]), "+r"(v[1][10]), "+r"(v[1][11]), "+r"(v[1][12]), "+r"(v[1][13]), "+r"(v[1][14]), "+r"(v[1][15]), "+r"(v[2][0]), "+r"(v[2][1]), "+r"(v[2][2]), "+r"(v[2][3]), "+r"(v[2][4]), "+r"(v[2][5]), "+r"(v[2][6]), "+r"(v[2][7]), "+r"(v[2][8]), "+r"(v[2][9]), "+r"(v[2][10]), "+r"(v[2][11]), "+r"(v[2][12]), "+r"(v[2][13]), "+r"(v[2][14]), "+r"(v[2][15]), "+r"(v[3][0]), "+r"(v[3][1]), "+r"(v[3][2]), "+r"(v[3][3]), "+r"(v[3][4]), "+r"(v[3][5]), "+r"(v[3][6]), "+r"(v[3][7]), "+r"(v[3][8]), "+r"(v[3][9]), "+r"(v[3][10]), "+r"(v[3][11]), "+r"(v[3][12]), "+r"(v[3][13]), "+r"(v[3][14]), "+r"(v[3][15])
                 :
                 : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// instruction descriptor, kind::i8: s8 A and B (K-major), s32 accumulator, M x N
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
#ifndef ZZ_I8_PRESET
#define ZZ_I8_PRESET 0
#endif
__device__ __forceinline__ void mma_i8_acc(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
#if ZZ_I8_PRESET
    asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, 1;" ::"r"(tmem_d), "l"(adesc), "l"(bdesc),
                 "r"(idesc)
                 : "memory");
#else
    asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, 0;" ::"r"(tmem_d), "l"(adesc), "l"(bdesc),
                 "r"(idesc)
                 : "memory");
#endif
}

__device__ __forceinline__ int np2_of(int count) {
    const int N = (count + 15) & ~15;
    return N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : 128;
}
__device__ __forceinline__ int sel_of(int np2) { return np2 == 16 ? 0 : np2 == 32 ? 1 : np2 == 64 ? 2 : 3; }

// q4_0 codes of one block (16 bytes: low nibbles k = 0..15, high k = 16..31) -> the
// 32 int8 values 16 * (q - 8) as two 16-byte chunks (k 0-15, k 16-31)
__device__ __forceinline__ void widen_q4(uint4 w, uint4 &lo, uint4 &hi) {
    lo = make_uint4(((w.x << 4) & 0xF0F0F0F0u) ^ 0x80808080u, ((w.y << 4) & 0xF0F0F0F0u) ^ 0x80808080u,
                    ((w.z << 4) & 0xF0F0F0F0u) ^ 0x80808080u, ((w.w << 4) & 0xF0F0F0F0u) ^ 0x80808080u);
    hi = make_uint4((w.x & 0xF0F0F0F0u) ^ 0x80808080u, (w.y & 0xF0F0F0F0u) ^ 0x80808080u,
                    (w.z & 0xF0F0F0F0u) ^ 0x80808080u, (w.w & 0xF0F0F0F0u) ^ 0x80808080u);
}
// tq2 codes of a 64-weight group (16 bytes; byte k holds weights k, k+16, k+32, k+48 at
// bits 0/2/4/6): block `odd` of the pair as int8 codes c in {0,1,2}
__device__ __forceinline__ void widen_tq2(uint4 w, int odd, uint4 &lo, uint4 &hi) {
    const int s = odd * 4;
    lo = make_uint4((w.x >> s) & 0x03030303u, (w.y >> s) & 0x03030303u, (w.z >> s) & 0x03030303u,
                    (w.w >> s) & 0x03030303u);
    hi = make_uint4((w.x >> (s + 2)) & 0x03030303u, (w.y >> (s + 2)) & 0x03030303u, (w.z >> (s + 2)) & 0x03030303u,
                    (w.w >> (s + 2)) & 0x03030303u);
}

// shared state of the CTA's roles
struct I8Ctx {
    uint8_t *smem;
    uint64_t *cfull, *cempty, *sfull, *sempty, *bfull, *bempty, *dfull, *dempty, *wfull, *wempty, *tfull, *tempty, *drain;
    volatile int *abort_flag;
    uint32_t tbase;
    int nb, nss, MT, T;
};

// ---------------------------------------------------------------- epilogue, one tile
// A tile of N rows (N = item rows rounded to 16) uses TMEM column slots of width
// cw = max(32, N rounded up to a power of two); a group of 128 columns holds G = 128/cw
// blocks. Warp h owns columns [h cw/2, (h+1) cw/2) of the tile and reads them from every
// block of the group: 4 slots of 16 columns per group, slot s = block s / cpw, chunk
// s % cpw (cpw = cw / 32 chunks per warp per block). Chunk c of the warp's columns adds
// into sums acc[c], blocks in K order: every column's sum has the same order (one fp32
// accumulator, block 0 to nb-1) whatever the tile width, so a token's result does not
// depend on how many other tokens share its expert.
__device__ __forceinline__ int colw_of(int count) { return max(32, np2_of(count)); }

// dx * (dw * I) of one slot's 16 columns into the sums `s` (fp32 pairs)
__device__ __forceinline__ void scale_slot(float2 (&s)[8], const uint32_t (&v)[16], float2 dw2, float2 c2,
                                           const float *dxb) {
#ifdef ZZ_SCALE_SCALAR
#pragma unroll
    for (int k4 = 0; k4 < 4; k4++) {
        const float4 d4 = *reinterpret_cast<const float4 *>(dxb + 4 * k4);
        s[2 * k4].x = fmaf(fmaf(__uint_as_float(v[4 * k4]), dw2.x, c2.x), d4.x, s[2 * k4].x);
        s[2 * k4].y = fmaf(fmaf(__uint_as_float(v[4 * k4 + 1]), dw2.x, c2.x), d4.y, s[2 * k4].y);
        s[2 * k4 + 1].x = fmaf(fmaf(__uint_as_float(v[4 * k4 + 2]), dw2.x, c2.x), d4.z, s[2 * k4 + 1].x);
        s[2 * k4 + 1].y = fmaf(fmaf(__uint_as_float(v[4 * k4 + 3]), dw2.x, c2.x), d4.w, s[2 * k4 + 1].y);
    }
    return;
#endif
#pragma unroll
    for (int k4 = 0; k4 < 4; k4++) {
        const float4 d4 = *reinterpret_cast<const float4 *>(dxb + 4 * k4);
#if ZZ_I8_PRESET
        const float2 f0 = make_float2(__uint_as_float(v[4 * k4]), __uint_as_float(v[4 * k4 + 1]));
        const float2 f1 = make_float2(__uint_as_float(v[4 * k4 + 2]), __uint_as_float(v[4 * k4 + 3]));
#else
        const float2 f0 = make_float2(__uint_as_float(v[4 * k4] + i8k::BIAS), __uint_as_float(v[4 * k4 + 1] + i8k::BIAS));
        const float2 f1 = make_float2(__uint_as_float(v[4 * k4 + 2] + i8k::BIAS), __uint_as_float(v[4 * k4 + 3] + i8k::BIAS));
#endif
        // fma(F, dw, -M*dw) = dw * I rounded once; then + dx * (dw * I)
        s[2 * k4] = ffma2(ffma2(f0, dw2, c2), make_float2(d4.x, d4.y), s[2 * k4]);
        s[2 * k4 + 1] = ffma2(ffma2(f1, dw2, c2), make_float2(d4.z, d4.w), s[2 * k4 + 1]);
    }
}

template <int FMT, int EPI>
__device__ __forceinline__ void epi_tile(const GemmArgs &a, const I8Ctx &c, const WorkItem &it, int m0, uint32_t &g,
                                         uint32_t &gg, int *err) {
    using namespace i8k;
    constexpr bool HAS_DW = FMT != GPU_FMT_TQ2;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q = warp & 3, h = warp >> 2;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int ncols = it.count;
    const int cw = colw_of(ncols), G = BN / cw, cpw = cw / 32;
    const int lg_cpw = cpw == 4 ? 2 : cpw == 2 ? 1 : 0, lg_g = G == 4 ? 2 : G == 2 ? 1 : 0;
    // per slot (fixed for the tile): block within the group, chunk, column offset, and
    // whether any of the chunk's columns holds a row -- shifts only, no division
    int s_sub[4], s_col[4];
    bool s_live[4];
#pragma unroll
    for (int sl = 0; sl < 4; sl++) {
        const int ch = sl & (cpw - 1);
        s_sub[sl] = sl >> lg_cpw;
        s_col[sl] = s_sub[sl] * cw + 16 * ch;
        s_live[sl] = h * (cw / 2) + 16 * ch < ncols;
    }
    float4 *dwtab = reinterpret_cast<float4 *>(c.smem + OFF_CT);
    static_assert(KB * 256 * 16 <= CT_BYTES, "dw table");
    // the TMEM preset held in 16 registers (one tcgen05.st operand vector)
    uint32_t bz[16];
#pragma unroll
    for (int i = 0; i < 16; i++) asm volatile("mov.b32 %0, %1;" : "=r"(bz[i]) : "n"(BIAS));
    float2 acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int k = 0; k < 8; k++) acc[i][k] = make_float2(0.f, 0.f);

#pragma unroll 1
    for (int ss = 0; ss < c.nss; ss++, g++) {
        TC_PROF_T(p_pro);
        const int ds = g % ND, ws = g % NW;
        const int nbl = min(KB, c.nb - ss * KB);
        uint4 dwr = make_uint4(0, 0, 0, 0);
        if (HAS_DW) {
            // (a wait that gives up sets the abort flag; the group waits below fail too)
            tc::mbar_wait(&c.wfull[ws], (g / NW) & 1, c.abort_flag, err, 18);
            dwr = *reinterpret_cast<const uint4 *>(c.smem + OFF_W + ws * W_SLOT + (q * 32 + lane) * 16);
            asm volatile("" ::"r"(dwr.x), "r"(dwr.y), "r"(dwr.z), "r"(dwr.w) : "memory");
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&c.wempty[ws]);
        }
        // this thread's (dw, dw, -M dw, -M dw) of the stage's 8 blocks, read back per slot
        // as the packed operands (a thread-private table in the tile-end exchange area)
#pragma unroll
        for (int jb = 0; jb < KB; jb++) {
            float dw = 1.f;
            if (HAS_DW) {
                const uint32_t wv = jb < 2 ? dwr.x : jb < 4 ? dwr.y : jb < 6 ? dwr.z : dwr.w;
                const __half2 hw = *reinterpret_cast<const __half2 *>(&wv);
                dw = (jb & 1) ? __high2float(hw) : __low2float(hw);
                if (FMT == GPU_FMT_Q40) dw *= 0.0625f;  // codes carry 16 (q - 8)
            }
            dwtab[jb * 256 + tid] = make_float4(dw, dw, -BIAS_F * dw, -BIAS_F * dw);  // exact
        }
        TC_PROF_ADD(44, p_pro);
        const bool dok = tc::mbar_wait(&c.dfull[ds], (g / ND) & 1, c.abort_flag, err, 9);
        const float *dxs = reinterpret_cast<const float *>(c.smem + OFF_DX + ds * DX_STAGE);
        const int ngr = (nbl + G - 1) >> lg_g;
#pragma unroll 1
        for (int gi = 0; gi < ngr; gi++, gg++) {
            TC_PROF_T(p_grp);
            TC_PROF_T(p_tf);
            const int p = gg % NGRP;
            bool ok = tc::mbar_wait(&c.tfull[p], (gg / NGRP) & 1, c.abort_flag, err, 8) && dok;
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld / st are warp-collective
            tc::tc_fence_after();
            TC_PROF_ADD(48, p_tf);
            const uint32_t gcol = c.tbase + lane_base + (uint32_t)(p * BN + h * (cw / 2));
            // the group's 4 slots: load all, one wait, preset the columns again and release
            // the group to the MMA, then scale into the sums while the next MMAs run
            uint32_t v[4][16];
            bool val[4];
            int jbs[4];
            TC_PROF_T(p_ldi);
#pragma unroll
            for (int sl = 0; sl < 4; sl++) {
                jbs[sl] = (gi << lg_g) + s_sub[sl];
                val[sl] = ok && jbs[sl] < nbl && s_live[sl];
                if (val[sl]) tmem_ld16(gcol + (uint32_t)s_col[sl], v[sl]);
            }
            TC_PROF_ADD(46, p_ldi);
            TC_PROF_T(p_ld);
            tmem_ld_wait_regs(v);
            TC_PROF_ADD(40, p_ld);
            TC_PROF_T(p_sti);
#pragma unroll
            for (int sl = 0; sl < 4; sl++)
                if (ZZ_I8_PRESET && val[sl]) tmem_st16(gcol + (uint32_t)s_col[sl], bz);
            TC_PROF_ADD(47, p_sti);
            TC_PROF_T(p_st);
            tmem_st_wait();
            TC_PROF_ADD(42, p_st);
            TC_PROF_T(p_arr);
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&c.tempty[p]);  // the group's columns are read and preset again
            TC_PROF_ADD(49, p_arr);
            TC_PROF_T(p_cmp);
#pragma unroll
            for (int sl = 0; sl < 4; sl++) {
                if (!val[sl]) continue;
                const int jb = jbs[sl];
                const float4 t4 = dwtab[jb * 256 + tid];
                const float2 dw2 = make_float2(t4.x, t4.y), c2 = make_float2(t4.z, t4.w);
                const float *dxb = dxs + jb * BN + h * (cw / 2) + 16 * (sl & (cpw - 1));
                // chunk sl % cpw of the warp's columns, with register indices fixed per branch
                if (sl == 0) scale_slot(acc[0], v[sl], dw2, c2, dxb);
                else if (sl == 1) { if (cpw == 1) scale_slot(acc[0], v[sl], dw2, c2, dxb); else scale_slot(acc[1], v[sl], dw2, c2, dxb); }
                else if (sl == 2) { if (cpw == 4) scale_slot(acc[2], v[sl], dw2, c2, dxb); else scale_slot(acc[0], v[sl], dw2, c2, dxb); }
                else { if (cpw == 4) scale_slot(acc[3], v[sl], dw2, c2, dxb); else if (cpw == 2) scale_slot(acc[1], v[sl], dw2, c2, dxb); else scale_slot(acc[0], v[sl], dw2, c2, dxb); }
            }
            TC_PROF_ADD(41, p_cmp);
            TC_PROF_ADD(45, p_grp);
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&c.dempty[ds]);
    }

    TC_PROF_T(p_end);
    // ---------------- tile end: this thread holds columns cbase .. cbase + cw/2 - 1 ----------------
    // Both outputs go through shared memory in halves of 64 columns (CTX = 65 floats per
    // row: writes along rows and reads along columns are both bank-conflict free), so all
    // 256 epilogue threads take part: gate/up requantizes one (32-feature block, token)
    // per thread, down adds 4 output rows per float4 reduction.
    float *ct = reinterpret_cast<float *>(c.smem + OFF_CT);
    const bool live = !*c.abort_flag;
    const int cbase = h * (cw / 2), cend = min(ncols, cbase + cw / 2);
    const float *alpha = FMT == GPU_FMT_TQ2 ? reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.scale) +
                                                                              (long)it.group * a.scale_gstride)
                                            : nullptr;
    const int nhalf = ncols > 64 ? 2 : 1;
    tc::named_sync(1, 256);  // every thread is past its last read of the dw table
    for (int hc = 0; hc < nhalf; hc++) {
        // this thread's sums of columns [64 hc, 64 hc + 64) into the tile [row][column]
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int col = cbase + 2 * i;
            if (col >= 64 * hc && col < 64 * hc + 64 && col < cend) {
                const float2 v = acc[i >> 3][i & 7];
                ct[(q * 32 + lane) * CTX + col - 64 * hc] = v.x;
                ct[(q * 32 + lane) * CTX + col + 1 - 64 * hc] = v.y;
            }
        }
        tc::named_sync(1, 256);
        if (live) {
            if (EPI == EPI_GATEUP) {
                // rows 0-63 gate and 64-127 up of the same 64 features; thread = (block qb of
                // 32 features, column): h = act(gate, up), then the q8_0 block (q40.h:124-138)
                const int MI = a.O / 2, nbh = MI / 32, f0 = (m0 / 128) * 64;
                const int n = tid & 63, qb = tid >> 6, col = 64 * hc + n;
                if (qb < 2 && col < ncols) {
                    const size_t pr = (size_t)(it.row0 + col);
                    const float tot = FMT == GPU_FMT_TQ2 ? a.xsx[a.pair_src[pr] / a.K] : 0.f;
                    float hv[32];
                    float amax = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const int fl = 32 * qb + j;
                        float gv = ct[fl * CTX + n], uv = ct[(64 + fl) * CTX + n];
                        if (FMT == GPU_FMT_TQ2) {
                            gv = alpha[m0 + fl] * (gv - tot);
                            uv = alpha[m0 + 64 + fl] * (uv - tot);
                        }
                        hv[j] = gated_act(a.act, gv, uv, a.clamp);
                        amax = fmaxf(amax, fabsf(hv[j]));
                    }
                    const float d = __fdiv_rn(amax, 127.0f);
                    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
                    uint32_t w[8];
                    int qs = 0;
#pragma unroll
                    for (int j4 = 0; j4 < 8; j4++) {
                        uint32_t word = 0;
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            int qv = __float2int_rn(__fmul_rn(hv[4 * j4 + k], id));
                            qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
                            qs += qv;
                            word |= (uint32_t)(qv & 0xFF) << (8 * k);
                        }
                        w[j4] = word;
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(a.hq + pr * MI + f0 + 32 * qb);
                    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    const int blk = f0 / 32 + qb;
                    a.hs[pr * nbh + blk] = d;
                    a.hsT[(size_t)blk * a.ldT + pr] = d;
                    if (FMT == GPU_FMT_TQ2) a.hblk[pr * nbh + blk] = qs;
                }
            } else {
                // OUT[token, m0 + 4 o4 .. + 3] += w * C, lanes along the rows (each warp
                // instruction covers 512 contiguous bytes of one token's output row)
                const int nbh = a.I / 32;
                for (int task = tid; task < 32 * 64; task += 256) {
                    const int o4 = task & 31, n = task >> 5, col = 64 * hc + n;
                    if (col >= ncols) break;  // n grows with task
                    const int pr = it.row0 + col;
                    float4 v = make_float4(ct[(4 * o4) * CTX + n], ct[(4 * o4 + 1) * CTX + n], ct[(4 * o4 + 2) * CTX + n],
                                           ct[(4 * o4 + 3) * CTX + n]);
                    const int o = m0 + 4 * o4;
                    if (FMT == GPU_FMT_TQ2) {
                        // Sx of the requantized hidden row, summed as tq2_quant_act does (tq2.h:103-107)
                        double t = 0;
                        for (int b = 0; b < nbh; b++)
                            t += (double)a.xs[(size_t)pr * nbh + b] * (double)a.xblk[(size_t)pr * nbh + b];
                        const float tot = (float)t;
                        v.x = alpha[o] * (v.x - tot); v.y = alpha[o + 1] * (v.y - tot);
                        v.z = alpha[o + 2] * (v.z - tot); v.w = alpha[o + 3] * (v.w - tot);
                    }
                    const float wgt = a.pair_w[pr];
                    v.x *= wgt; v.y *= wgt; v.z *= wgt; v.w *= wgt;
                    atomicAdd(reinterpret_cast<float4 *>(a.out + (size_t)(a.pair_src[pr] / a.K) * a.O + o), v);
                }
            }
        }
        tc::named_sync(1, 256);
    }
    TC_PROF_ADD(43, p_end);
}

template <int FMT, int EPI>
__global__ void __launch_bounds__(i8k::NTHREADS, 1)
    k_moe_i8(const GemmArgs a, const __grid_constant__ CUtensorMap codes_map,
             const __grid_constant__ CUtensorMap scale_map, const __grid_constant__ BMaps8 bmaps, int *err) {
    using namespace i8k;
    constexpr bool DIRECT = FMT == GPU_FMT_Q80;  // q8_0 codes are already the int8 operand
    constexpr bool HAS_DW = FMT != GPU_FMT_TQ2;
    constexpr int CBS = FMT == GPU_FMT_Q40 ? 128 : FMT == GPU_FMT_Q80 ? 256 : 64;  // code bytes per row per stage
    constexpr int SLOT = 128 * CBS;
    constexpr int RC = DIRECT ? 1 : RING / SLOT;
    static_assert(RC <= RC_MAX, "ring");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    I8Ctx c;
    c.smem = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    c.cfull = bars; c.cempty = c.cfull + RC_MAX;
    c.sfull = c.cempty + RC_MAX; c.sempty = c.sfull + NS;
    c.bfull = c.sempty + NS; c.bempty = c.bfull + RB;
    c.dfull = c.bempty + RB; c.dempty = c.dfull + ND;
    c.wfull = c.dempty + ND; c.wempty = c.wfull + NW;
    c.tfull = c.wempty + NW; c.tempty = c.tfull + NGRP; c.drain = c.tempty + NGRP;
    uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_BAR + NBAR * 8);
    c.abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + NBAR * 8 + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    c.nb = a.I / ZZ_BLK;
    c.nss = (c.nb + KB - 1) / KB;
    c.MT = a.O / 128;
    c.T = *a.n_items * c.MT;
    auto tile = [&](int t, WorkItem &it, int &m0) {
        it = a.items[t / c.MT];
        m0 = (t % c.MT) * 128;
    };

    if (tid == 0) {
        for (int i = 0; i < RC; i++) { tc::mbar_init(&c.cfull[i], 1); tc::mbar_init(&c.cempty[i], 4); }
        for (int i = 0; i < NS; i++) { tc::mbar_init(&c.sfull[i], DIRECT ? 1 : 4); tc::mbar_init(&c.sempty[i], 1); }
        for (int i = 0; i < RB; i++) { tc::mbar_init(&c.bfull[i], 1); tc::mbar_init(&c.bempty[i], 1); }
        for (int i = 0; i < ND; i++) { tc::mbar_init(&c.dfull[i], 1); tc::mbar_init(&c.dempty[i], 8); }
        for (int i = 0; i < NW; i++) { tc::mbar_init(&c.wfull[i], 1); tc::mbar_init(&c.wempty[i], 8); }
        for (int i = 0; i < NGRP; i++) { tc::mbar_init(&c.tfull[i], 1); tc::mbar_init(&c.tempty[i], 8); }
        tc::mbar_init(c.drain, 1);
        *c.abort_flag = 0;
        tc::mbar_init_fence();
    }
    if (warp == 14) tc::tmem_alloc(tmem_base_smem, NGRP * BN);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    c.tbase = *tmem_base_smem;
    if (warp < 8) {
        // preset every accumulator column of this warp's lanes
        const int q = warp & 3, h = warp >> 2;
        for (int p = 0; p < NGRP; p++)
            for (int k = 0; k < 4; k++)
                tmem_st16_bias(c.tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(p * BN + 64 * h + 16 * k));
        tmem_st_wait();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    TC_PROF_T(prof_t0);
    if (warp >= 12) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_COPY));
      if (warp == 12) {
        if (lane == 0) {
            // ---------------- TMA: weight codes and weight scales ----------------
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < c.T && ok && !*c.abort_flag; t += gridDim.x) {
                WorkItem it; int m0;
                tile(t, it, m0);
                const int y = it.group * a.O + m0;
                for (int ss = 0; ss < c.nss; ss++, g++) {
                    // both slots are free before either copy is issued, so an abort leaves
                    // copies in flight only for stages below g
                    if (HAS_DW) {
                        const uint32_t wu = g / NW;
                        if (wu && !tc::mbar_wait(&c.wempty[g % NW], (wu - 1) & 1, c.abort_flag, err, 16)) { ok = false; break; }
                    }
                    if (DIRECT) {
                        const int st = g % NS;
                        const uint32_t u = g / NS;
                        if (u && !tc::mbar_wait(&c.sempty[st], (u - 1) & 1, c.abort_flag, err, 1)) { ok = false; break; }
                        tc::mbar_arrive_tx(&c.sfull[st], A_STAGE);
                        uint8_t *dst = smem + OFF_A + st * A_STAGE;
                        tc::tma_load_2d(dst, &codes_map, ss * 256, y, &c.sfull[st]);
                        tc::tma_load_2d(dst + A_ATOM, &codes_map, ss * 256 + 128, y, &c.sfull[st]);
                    } else {
                        const int s = g % RC;
                        const uint32_t u = g / RC;
                        if (u && !tc::mbar_wait(&c.cempty[s], (u - 1) & 1, c.abort_flag, err, 1)) { ok = false; break; }
                        tc::mbar_arrive_tx(&c.cfull[s], SLOT);
                        tc::tma_load_2d(smem + OFF_RING + s * SLOT, &codes_map, ss * CBS, y, &c.cfull[s]);
                    }
                    if (HAS_DW) {
                        const int ws = g % NW;
                        tc::mbar_arrive_tx(&c.wfull[ws], W_SLOT);
                        tc::tma_load_3d(smem + OFF_W + ws * W_SLOT, &scale_map, ss * KB, m0, it.group, &c.wfull[ws]);
                    }
                }
            }
            // wait for the last copies to land before the CTA may exit
            // (bounded by time only: after an abort the copies still land in this CTA's memory)
            // (each slot's latest use)
            for (uint32_t k = g > (uint32_t)NS ? g - NS : 0; DIRECT && k < g; k++) tc::mbar_drain(&c.sfull[k % NS], (k / NS) & 1);
            for (uint32_t k = g > (uint32_t)RC ? g - RC : 0; !DIRECT && k < g; k++) tc::mbar_drain(&c.cfull[k % RC], (k / RC) & 1);
            for (uint32_t k = g > (uint32_t)NW ? g - NW : 0; HAS_DW && k < g; k++) tc::mbar_drain(&c.wfull[k % NW], (k / NW) & 1);
        }
    } else if (warp == 13) {
        if (lane == 0) {
            // ---------------- TMA: activation rows; bulk copies: their block scales ----------------
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < c.T && ok && !*c.abort_flag; t += gridDim.x) {
                WorkItem it; int m0;
                tile(t, it, m0);
                const int np2 = np2_of(it.count), sel = sel_of(np2);
                const uint32_t box = (uint32_t)np2 * 128u;
                for (int ss = 0; ss < c.nss; ss++, g++) {
                    const int bs = g % RB, ds = g % ND;
                    const int nbl = min(KB, c.nb - ss * KB);
                    const int nbox = (nbl + 3) / 4;
                    if (g >= RB && !tc::mbar_wait(&c.bempty[bs], ((g / RB) - 1) & 1, c.abort_flag, err, 3)) { ok = false; break; }
                    if (g >= ND && !tc::mbar_wait(&c.dempty[ds], ((g / ND) - 1) & 1, c.abort_flag, err, 11)) { ok = false; break; }
                    tc::mbar_arrive_tx(&c.bfull[bs], box * nbox);
                    uint8_t *dst = smem + OFF_B + bs * B_STAGE;
                    for (int bx = 0; bx < nbox; bx++) {
                        const int x = (ss * KB + 4 * bx) * 32;
                        // the map is named with a constant index so it stays in parameter space
                        switch (sel) {
                            case 0: tc::tma_load_2d(dst + bx * box, &bmaps.m[0], x, it.row0, &c.bfull[bs]); break;
                            case 1: tc::tma_load_2d(dst + bx * box, &bmaps.m[1], x, it.row0, &c.bfull[bs]); break;
                            case 2: tc::tma_load_2d(dst + bx * box, &bmaps.m[2], x, it.row0, &c.bfull[bs]); break;
                            default: tc::tma_load_2d(dst + bx * box, &bmaps.m[3], x, it.row0, &c.bfull[bs]); break;
                        }
                    }
                    tc::mbar_arrive_tx(&c.dfull[ds], (uint32_t)(nbl * np2 * 4));
                    for (int jj = 0; jj < nbl; jj++)
                        tc::bulk_load(smem + OFF_DX + ds * DX_STAGE + jj * BN * 4,
                                      a.xsT + (size_t)(ss * KB + jj) * a.ldT + it.row0, (uint32_t)(np2 * 4), &c.dfull[ds]);
                }
            }
            for (uint32_t k = g > (uint32_t)RB ? g - RB : 0; k < g; k++) tc::mbar_drain(&c.bfull[k % RB], (k / RB) & 1);
            for (uint32_t k = g > (uint32_t)ND ? g - ND : 0; k < g; k++) tc::mbar_drain(&c.dfull[k % ND], (k / ND) & 1);
        }
    } else if (warp == 14) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            uint32_t g = 0, gg = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < c.T && ok && !*c.abort_flag; t += gridDim.x) {
                WorkItem it; int m0;
                tile(t, it, m0);
                const int N = (it.count + 15) & ~15, np2 = np2_of(it.count), cw = colw_of(it.count), G = BN / cw;
                const uint32_t idesc = idesc_i8(128, N);
                const uint32_t box = (uint32_t)np2 * 128u;
                for (int ss = 0; ss < c.nss && ok; ss++, g++) {
                    const int st = g % NS, bs = g % RB;
                    if (!tc::mbar_wait(&c.sfull[st], (g / NS) & 1, c.abort_flag, err, 5)) { ok = false; break; }
                    if (!tc::mbar_wait(&c.bfull[bs], (g / RB) & 1, c.abort_flag, err, 15)) { ok = false; break; }
                    tc::tc_fence_after();
                    const int nbl = min(KB, c.nb - ss * KB);
                    const uint32_t sa = tc::smem_u32(smem + OFF_A + st * A_STAGE);
                    const uint32_t sb = tc::smem_u32(smem + OFF_B + bs * B_STAGE);
                    for (int jb = 0; jb < nbl; jb++) {
                        const int sub = jb & (G - 1), p = gg % NGRP;
                        if (sub == 0 && gg >= NGRP &&
                            !tc::mbar_wait(&c.tempty[p], ((gg / NGRP) - 1) & 1, c.abort_flag, err, 6)) {
                            ok = false;
                            break;
                        }
                        tc::tc_fence_after();
                        const uint64_t ad = tc::smem_desc_sw128(sa + (jb >> 2) * A_ATOM + (jb & 3) * 32);
                        const uint64_t bd = tc::smem_desc_sw128(sb + (jb >> 2) * box + (jb & 3) * 32);
                        mma_i8_acc(c.tbase + (uint32_t)(p * BN + sub * cw), ad, bd, idesc);
                        if (sub == G - 1 || jb == nbl - 1) {
                            tc::mma_commit(&c.tfull[p]);
                            gg++;
                        }
                    }
                    if (!ok) break;
                    tc::mma_commit(&c.sempty[st]);  // A stage free once these MMAs complete
                    tc::mma_commit(&c.bempty[bs]);  // B stage likewise
                }
            }
            // every MMA issued has completed before TMEM may be freed
            tc::mma_commit(&c.drain[0]);
            tc::mbar_drain(&c.drain[0], 0);
        }
    }
    } else if (warp >= 8) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_PROD));
        if (!DIRECT) {
            // ---------------- producers: codes -> int8 operand (128-byte swizzle) ----------------
            const int r = tid - 256;  // weight row of the tile
            const int my_tiles = c.T > (int)blockIdx.x ? (c.T - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
            const uint32_t Gs = (uint32_t)my_tiles * c.nss;
            constexpr int NCH = CBS / 16;  // 16-byte code chunks per row per stage
            // chunk k of this row sits at chunk k ^ swz (the TMA swizzle of a CBS-byte row)
            const int swz = CBS == 128 ? (r & 7) : ((r >> 1) & 3);
            for (uint32_t g = 0; g < Gs; g++) {
                const int s = g % RC, st = g % NS;
                if (!tc::mbar_wait(&c.cfull[s], (g / RC) & 1, c.abort_flag, err, 4)) break;
                uint4 w[NCH];
                const uint8_t *row = smem + OFF_RING + s * SLOT + r * CBS;
#pragma unroll
                for (int k = 0; k < NCH; k++) w[k] = *reinterpret_cast<const uint4 *>(row + 16 * (k ^ swz));
                // loads consumed, then ordered before the TMA's refill of the slot
#pragma unroll
                for (int k = 0; k < NCH; k++) asm volatile("" ::"r"(w[k].x), "r"(w[k].y), "r"(w[k].z), "r"(w[k].w) : "memory");
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&c.cempty[s]);
                if (g >= NS && !tc::mbar_wait(&c.sempty[st], ((g / NS) - 1) & 1, c.abort_flag, err, 14)) break;
                const int nbl = min(KB, c.nb - (int)(g % c.nss) * KB);
                uint8_t *sa = smem + OFF_A + st * A_STAGE + r * 128;
#pragma unroll
                for (int jb = 0; jb < KB; jb++) {
                    uint4 lo, hi;
                    if (jb < nbl) {
                        if (FMT == GPU_FMT_Q40) widen_q4(w[jb], lo, hi);
                        else widen_tq2(w[jb >> 1], jb & 1, lo, hi);
                    } else {
                        lo = hi = make_uint4(0, 0, 0, 0);
                    }
                    const int ch = (jb & 3) * 2;
                    uint8_t *at = sa + (jb >> 2) * A_ATOM;
                    *reinterpret_cast<uint4 *>(at + 16 * (ch ^ (r & 7))) = lo;
                    *reinterpret_cast<uint4 *>(at + 16 * ((ch + 1) ^ (r & 7))) = hi;
                }
                // shared stores of the stage before the tensor cores' reads (async proxy)
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&c.sfull[st]);
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_EPI));
        // ---------------- epilogue (warps 0-7) ----------------
        uint32_t g = 0, gg = 0;
        for (int t = blockIdx.x; t < c.T; t += gridDim.x) {
            WorkItem it; int m0;
            tile(t, it, m0);
            epi_tile<FMT, EPI>(a, c, it, m0, g, gg, err);
        }
    }
#ifdef ZZ_TC_PROF
    // per-role span from set-up to here: 32 epilogue, 33 producers, 34 code TMA, 35 B TMA, 36 MMA
    if (blockIdx.x == 0 && lane == 0 && warp < 15)
        atomicAdd(&tc::g_tc_prof[32 + (warp < 8 ? 0 : warp < 12 ? 1 : warp - 10)],
                  (unsigned long long)(clock64() - prof_t0));
#endif
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 14) {
        tc::tc_fence_after();
        tc::tmem_dealloc(c.tbase, NGRP * BN);
    }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encode() {
    if (g_encode) return 1;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
        return fail("cuTensorMapEncodeTiled is not available");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return 1;
}

// 2-D uint8 map over [rows][row_bytes] with a box of `box_w` bytes x `box_rows` rows,
// swizzled by the box width (128 / 64 bytes)
int make_u8_map(CUtensorMap *map, const void *base, long rows, long row_bytes, int box_w, int box_rows,
                       const char *what) {
    if (!get_encode()) return 0;
    if ((uintptr_t)base & 15 || row_bytes % 16) return fail("i8: %s not 16-byte aligned", what);
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_w, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = box_w == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("i8: %s tensor map failed (%d)", what, (int)r);
    return 1;
}

// fp16 weight-scale planes of a bank: [experts][O][nbp] (rows padded to 8 blocks), each
// expert `gstride` bytes apart; one box is 128 rows x 8 scales (one stage)
int make_scale_map(CUtensorMap *map, const void *scale, int E, int O, int nbp, long gstride) {
    if (!get_encode()) return 0;
    if ((uintptr_t)scale & 15 || gstride % 16 || nbp % 8) return fail("i8: scale planes not 16-byte aligned");
    cuuint64_t dims[3] = {(cuuint64_t)nbp, (cuuint64_t)O, (cuuint64_t)E};
    cuuint64_t strides[2] = {(cuuint64_t)nbp * 2, (cuuint64_t)gstride};
    cuuint32_t box[3] = {8, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(scale), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("i8: scale tensor map failed (%d)", (int)r);
    return 1;
}

template <int FMT, int EPI>
static int launch_i8_t(const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    static bool attr = false;  // per process: the attribute is a property of the function
    if (!attr) {
        if (!check_cuda(cudaFuncSetAttribute(k_moe_i8<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, i8k::SMEM),
                        "i8 smem attribute"))
            return 0;
        attr = true;
    }
    const long row_bytes = FMT == GPU_FMT_Q40 ? a.I / 2 : FMT == GPU_FMT_Q80 ? a.I : a.I / 4;
    const int box_w = FMT == GPU_FMT_TQ2 ? 64 : 128;
    CUtensorMap map, smap;
    BMaps8 bmaps;
    if (!make_u8_map(&map, a.codes, (long)n_groups * a.O, row_bytes, box_w, 128, "weight codes")) return 0;
    if (FMT == GPU_FMT_TQ2)
        smap = map;  // tq2 has one f32 alpha per row, applied at the tile end
    else if (!make_scale_map(&smap, a.scale, n_groups, a.O, ((a.I / ZZ_BLK) + 7) & ~7, a.scale_gstride))
        return 0;
    for (int i = 0; i < 4; i++)
        if (!make_u8_map(&bmaps.m[i], a.xg8, a.rows_cap, a.I, 128, 16 << i, "activation rows")) return 0;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    k_moe_i8<FMT, EPI><<<sms, i8k::NTHREADS, i8k::SMEM, st>>>(a, map, smap, bmaps, err);
    return check_cuda(cudaGetLastError(), "i8 launch");
}

// Whether the int8 tensor-core engine takes a layer of this shape: weight rows in whole
// 128-row tiles, rows of whole 16-byte pieces, consecutive experts' code planes exactly
// O * row_bytes apart (true for a packed bank when O * row_bytes is a multiple of 256).
bool moe_i8_supported(int fmt, int D, int MI) {
    auto rb = [&](int I) -> long { return fmt == GPU_FMT_Q40 ? I / 2 : fmt == GPU_FMT_Q80 ? I : I / 4; };
    if ((2 * MI) % 128 || D % 128) return false;
    if (rb(D) % 16 || rb(MI) % 16 || MI % 16 || D % 16) return false;
    if (((long)2 * MI * rb(D)) % 256 || ((long)D * rb(MI)) % 256) return false;
    return true;
}

// The expert GEMMs (gate/up with the fused activation + requant, or down with the fused
// scatter-add) over the router's items, int8 operands on tcgen05.
int launch_moe_i8(int fmt, int epi, const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    if (a.O % 128) return fail("i8: O=%d not a multiple of 128", a.O);
    if (epi == EPI_GATEUP) {
        if (fmt == GPU_FMT_Q40) return launch_i8_t<GPU_FMT_Q40, EPI_GATEUP>(a, n_groups, err, st);
        if (fmt == GPU_FMT_Q80) return launch_i8_t<GPU_FMT_Q80, EPI_GATEUP>(a, n_groups, err, st);
        return launch_i8_t<GPU_FMT_TQ2, EPI_GATEUP>(a, n_groups, err, st);
    }
    if (fmt == GPU_FMT_Q40) return launch_i8_t<GPU_FMT_Q40, EPI_DOWN>(a, n_groups, err, st);
    if (fmt == GPU_FMT_Q80) return launch_i8_t<GPU_FMT_Q80, EPI_DOWN>(a, n_groups, err, st);
    return launch_i8_t<GPU_FMT_TQ2, EPI_DOWN>(a, n_groups, err, st);
}

}  // namespace zz

#ifdef ZZ_TC_PROF
// diagnostic build only: this translation unit's wait-site cycle totals (block 0), read
// and cleared
extern "C" int zz_i8_prof_read(unsigned long long *out) {
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(out, zz::tc::g_tc_prof, sizeof(unsigned long long) * 128);
    unsigned long long z[128] = {0};
    cudaMemcpyToSymbol(zz::tc::g_tc_prof, z, sizeof z);
    return 1;
}
#endif
