// zz_moe_tc.cu -- the batch-union expert GEMMs on the 5th-generation tensor cores.
//
// Persistent, warp-specialised kernel, one CTA per SM, looping over work tiles
// (expert item of <= 32 token rows x 128 weight rows). K advances in stages of KB = 4
// quantization blocks (K = 128); every hand-off between roles is one mbarrier phase
// per stage. Roles (512 threads):
//   warp 12      TMA: one box per stage of the tile's packed weight codes (128 rows x
//                KB blocks, swizzled so the producers' 16-byte shared loads are bank-
//                conflict free) into a 32 KB ring
//   warp 14      TMA: the stage's fp16 activation tiles (one 64-byte-swizzled K-major
//                box of the item's rows per block)
//   warp 15      bulk copies: the stage's activation block scales; TMA: the tile's
//                fp16 weight block scales, 128 rows x 8 blocks per box
//   warps 8-11   producers: thread r widens row r's codes of the stage's blocks to
//                fp16 in the UMMA canonical K-major layout (8-row x 16-byte core
//                matrices, no swizzle); the fp16 values are the integer codes
//   warp 13      MMA: one thread issues, per block of the stage, two tcgen05.mma
//                kind::f16 (M=128, N = item rows rounded to 16, K=16) into that
//                block's own TMEM accumulator (KB accumulators per stage, four stages
//                resident)
//   warps 0-7    epilogue: tcgen05.ld (16x256b shape: 4 rows x 8 tokens per thread)
//                of each block's 128 x N f32 results -- the reference's exact per-block
//                integer sums -- then acc += (dw*dx) * sum in packed fp32 (the
//                decomposition of q40.h:20-31). The two warp groups take alternate
//                stages and add their partial sums at the tile end, so every token's
//                sum has the same order whatever tile it lands in; then the fused
//                gate/up GeGLU + q8 requant or the down-projection scatter-add.
// Waits are bounded (2 s); one that runs out sets the kernel's error word.
#include <cstdlib>
#include <cuda.h>
#include <cudaTypedefs.h>
#include "zz_gemm.cuh"
#include "zz_tc.cuh"
#include "zz_tc_widen.cuh"

namespace zz {

namespace tcm {
constexpr int NTHREADS = 512;
constexpr int BN = 32;             // max activation rows per tile
constexpr int KB = 4;              // quantization blocks per stage
constexpr int NACC = 4;            // TMEM stages: NACC * KB * BN = 512 columns
constexpr int RING = 32 * 1024;    // weight-code ring
constexpr int NS = 2;              // widened-weight (A) stages
constexpr int A_BLK = 128 * 64;    // one block: 128 rows x 32 fp16, K-major core matrices
constexpr int A_STAGE = KB * A_BLK;
constexpr int RB = 8;              // activation (B) stages
constexpr int B_BLK = BN * 64;     // up to 32 rows x 32 fp16, 64-byte swizzle
constexpr int B_STAGE = KB * B_BLK;
constexpr int ND = 16;             // activation-scale stages
constexpr int DX_BLK = BN * 4;
constexpr int DX_STAGE = KB * DX_BLK;
constexpr int CS = BN + 4;         // padded row of the fp32 result tile
constexpr int RC_MAX = 8;          // ring slots for the narrowest format (tq2)
constexpr int NW = 8;              // weight-scale ring: 128 rows x 8 fp16 (two stages) per slot
constexpr int W_SLOT = 128 * 16;
constexpr int OFF_B = 0;           // 1 KB aligned (swizzled TMA destinations)
constexpr int OFF_RING = OFF_B + RB * B_STAGE;
constexpr int OFF_A = OFF_RING + RING;
constexpr int OFF_DX = OFF_A + NS * A_STAGE;
constexpr int OFF_W = OFF_DX + ND * DX_STAGE;
constexpr int OFF_CT = OFF_W + NW * W_SLOT;
constexpr int OFF_INFO = OFF_CT + 128 * CS * 4;
constexpr int OFF_BAR = OFF_INFO + BN * 8;
constexpr int NBAR = 2 * RC_MAX + 2 * NS + 2 * RB + 2 * NACC + 2 * ND + 2 * NW;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + slack to align the base to 1 KB
static_assert(SMEM <= 232448, "shared memory");
}  // namespace tcm

struct BMaps {
    CUtensorMap m[2];  // activation boxes of 16 and 32 rows
};

struct TcTile {
    WorkItem it;
    int m0;
};
__device__ __forceinline__ TcTile tc_tile(const GemmArgs &a, int t, int MT) {
    TcTile r;
    r.it = a.items[t / MT];
    r.m0 = (t % MT) * 128;
    return r;
}
__device__ __forceinline__ int tc_sel(int count) {
    const int N = (count + 15) & ~15;
    return N <= 16 ? 0 : 1;
}

template <int FMT, int EPI>
__global__ void __launch_bounds__(tcm::NTHREADS, 1)
    k_moe_tc(const GemmArgs a, const __grid_constant__ CUtensorMap codes_map,
             const __grid_constant__ CUtensorMap scale_map, const __grid_constant__ BMaps bmaps, int *err) {
    using namespace tcm;
    constexpr int CB = tc_cb<FMT>(), RC = RING / (128 * CB), SLOTB = 128 * CB, NCH = CB / 16;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *ring = smem + OFF_RING;
    uint8_t *stages = smem + OFF_A;
    uint8_t *bring = smem + OFF_B;
    uint8_t *dxring = smem + OFF_DX;
    float *ct = reinterpret_cast<float *>(smem + OFF_CT);
    int *col_xrow = reinterpret_cast<int *>(smem + OFF_INFO);
    float *col_sx = reinterpret_cast<float *>(smem + OFF_INFO + BN * 4);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *cfull = bars, *cempty = bars + RC_MAX;
    uint64_t *sfull = bars + 2 * RC_MAX, *sempty = sfull + NS;
    uint64_t *bfull = sempty + NS, *bempty = bfull + RB;
    uint64_t *tfull = bempty + RB, *tempty = tfull + NACC;
    uint64_t *dfull = tempty + NACC, *dempty = dfull + ND;
    uint64_t *wfull = dempty + ND, *wempty = wfull + NW;
    uint8_t *wring = smem + OFF_W;
    constexpr bool HAS_DW = FMT != GPU_FMT_TQ2;
    uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_BAR + NBAR * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + NBAR * 8 + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = a.I / ZZ_BLK;
    const int nss = (nb + KB - 1) / KB;
    const int MT = a.O / 128;
    const int T = *a.n_items * MT;

    if (tid == 0) {
        for (int i = 0; i < RC; i++) { tc::mbar_init(&cfull[i], 1); tc::mbar_init(&cempty[i], 4); }
        for (int i = 0; i < NS; i++) { tc::mbar_init(&sfull[i], 4); tc::mbar_init(&sempty[i], 1); }
        for (int i = 0; i < RB; i++) { tc::mbar_init(&bfull[i], 1); tc::mbar_init(&bempty[i], 1); }
        for (int i = 0; i < NACC; i++) { tc::mbar_init(&tfull[i], 1); tc::mbar_init(&tempty[i], 8); }
        for (int i = 0; i < ND; i++) { tc::mbar_init(&dfull[i], 1); tc::mbar_init(&dempty[i], 8); }
        for (int i = 0; i < NW; i++) { tc::mbar_init(&wfull[i], 1); tc::mbar_init(&wempty[i], 8); }
        *abort_flag = 0;
        tc::mbar_init_fence();
    }
    if (warp == 13) tc::tmem_alloc(tmem_base_smem, NACC * KB * BN);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tbase = *tmem_base_smem;
#ifdef ZZ_TC_PROF
    const long long prof_t0 = clock64();
#endif

    if (warp == 12) {
        if (lane == 0) {
            // ---------------- TMA: weight codes -> ring, one box per stage ----------------
            uint32_t g = 0;
            for (int t = blockIdx.x; t < T && !*abort_flag; t += gridDim.x) {
                TcTile tl = tc_tile(a, t, MT);
                const int y = tl.it.group * a.O + tl.m0;
                bool ok = true;
                for (int ss = 0; ss < nss; ss++, g++) {
                    const int s = g % RC;
                    const uint32_t u = g / RC;
                    if (u && !tc::mbar_wait(&cempty[s], (u - 1) & 1, abort_flag, err, 1)) { ok = false; break; }
                    tc::mbar_arrive_tx(&cfull[s], SLOTB);
                    tc::tma_load_2d(ring + s * SLOTB, &codes_map, ss * CB, y, &cfull[s]);
                }
                if (!ok) break;
            }
            // bounded drain: do not leave the CTA with copies in flight
            if (g) tc::mbar_wait(&cfull[(g - 1) % RC], ((g - 1) / RC) & 1, abort_flag, err, 2);
        }
    } else if (warp == 14) {
        if (lane == 0) {
            // ---------------- TMA: activation tiles, one box per block ----------------
            uint32_t g = 0;
            for (int t = blockIdx.x; t < T && !*abort_flag; t += gridDim.x) {
                TcTile tl = tc_tile(a, t, MT);
                const int sel = tc_sel(tl.it.count);
                const uint32_t bblk = (16u << sel) * 64u;
                bool ok = true;
                for (int ss = 0; ss < nss; ss++, g++) {
                    const int bs = g % RB;
                    const uint32_t u = g / RB;
                    if (u && !tc::mbar_wait(&bempty[bs], (u - 1) & 1, abort_flag, err, 3)) { ok = false; break; }
                    const int nbl = min(KB, nb - ss * KB);
                    tc::mbar_arrive_tx(&bfull[bs], bblk * nbl);
                    uint8_t *dst = bring + bs * B_STAGE;
                    // rows row0.. of the pair-ordered activations, halves 32j..32j+31 of
                    // block j: one 64-byte-swizzled K-major box. The map is named with a
                    // constant index so it stays in parameter space.
                    for (int jj = 0; jj < nbl; jj++) {
                        const int x = (ss * KB + jj) * 32;
                        switch (sel) {
                            case 0: tc::tma_load_2d(dst + jj * bblk, &bmaps.m[0], x, tl.it.row0, &bfull[bs]); break;
                            default: tc::tma_load_2d(dst + jj * bblk, &bmaps.m[1], x, tl.it.row0, &bfull[bs]); break;
                        }
                    }
                }
                if (!ok) break;
            }
            if (g) tc::mbar_wait(&bfull[(g - 1) % RB], ((g - 1) / RB) & 1, abort_flag, err, 12);
        }
    } else if (warp == 15) {
        if (lane == 0) {
            // ---------------- bulk copies: the stage's activation block scales; TMA: the
            // weight scales of every two stages (128 rows x 8 fp16) ----------------
            uint32_t g = 0, gw = 0;
            for (int t = blockIdx.x; t < T && !*abort_flag; t += gridDim.x) {
                TcTile tl = tc_tile(a, t, MT);
                bool ok = true;
                for (int ss = 0; ss < nss; ss++, g++) {
                    const int ds = g % ND;
                    const uint32_t du = g / ND;
                    if (HAS_DW && (ss & 1) == 0) {
                        const int ws = gw % NW;
                        const uint32_t wu = gw / NW;
                        if (wu && !tc::mbar_wait(&wempty[ws], (wu - 1) & 1, abort_flag, err, 16)) { ok = false; break; }
                        tc::mbar_arrive_tx(&wfull[ws], W_SLOT);
                        tc::tma_load_3d(wring + ws * W_SLOT, &scale_map, ss * KB, tl.m0, tl.it.group, &wfull[ws]);
                        gw++;
                    }
                    if (du && !tc::mbar_wait(&dempty[ds], (du - 1) & 1, abort_flag, err, 11)) { ok = false; break; }
                    const int nbl = min(KB, nb - ss * KB);
                    tc::mbar_arrive_tx(&dfull[ds], DX_BLK * nbl);
                    for (int jj = 0; jj < nbl; jj++)
                        tc::bulk_load(dxring + ds * DX_STAGE + jj * DX_BLK,
                                      a.xsT + (size_t)(ss * KB + jj) * a.ldT + tl.it.row0, DX_BLK, &dfull[ds]);
                }
                if (!ok) break;
            }
            if (g) tc::mbar_wait(&dfull[(g - 1) % ND], ((g - 1) / ND) & 1, abort_flag, err, 13);
            if (gw) tc::mbar_wait(&wfull[(gw - 1) % NW], ((gw - 1) / NW) & 1, abort_flag, err, 17);
        }
    } else if (warp >= 8 && warp < 12) {
        // ---------------- producers: widen weight codes to fp16 ----------------
        const int pt = tid - 256;  // weight row of the tile
        // 16-byte chunk c of this row sits at chunk c ^ swz (the TMA swizzle of a CB-byte row)
        const int swz = ((pt * CB) >> 7) & (NCH - 1);
        const int my_tiles = T > (int)blockIdx.x ? (T - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        const uint32_t G = (uint32_t)my_tiles * nss;  // stages of all this CTA's tiles, in order
        auto fetch = [&](uint32_t g, uint4 (&c)[NCH]) -> bool {
            const int s = g % RC;
            if (!tc::mbar_wait(&cfull[s], (g / RC) & 1, abort_flag, err, 4)) return false;
            const uint8_t *row = ring + s * SLOTB + pt * CB;
#pragma unroll
            for (int k = 0; k < NCH; k++) c[k] = *reinterpret_cast<const uint4 *>(row + 16 * (k ^ swz));
            return true;
        };
        uint4 c[NCH];
        bool ok = G == 0 || fetch(0, c);
        for (uint32_t g = 0; g < G && ok; g++) {
            uint4 cn[NCH];
            if (g + 1 < G && !fetch(g + 1, cn)) { ok = false; break; }  // next stage's codes in flight
            const int st = g % NS;
            if (g >= NS && !tc::mbar_wait(&sempty[st], ((g / NS) - 1) & 1, abort_flag, err, 14)) { ok = false; break; }
            const int nbl = min(KB, nb - (int)(g % nss) * KB);
            uint8_t *sa = stages + st * A_STAGE + (pt >> 3) * 512 + (pt & 7) * 16;
            TC_PROF_T(p_w);
#pragma unroll
            for (int jj = 0; jj < KB; jj++) {
                if (jj < nbl) {
                    uint4 w[4];
                    widen_blk<FMT>(c, jj, w);
#pragma unroll
                    for (int k = 0; k < 4; k++) *reinterpret_cast<uint4 *>(sa + jj * A_BLK + k * 128) = w[k];
                }
            }
            // One proxy fence per thread orders both its shared stores of the stage (read
            // next by the tensor cores) and its shared loads of the code slot (consumed by
            // the widening above; refilled next by the TMA) before the async proxy; then one
            // elected arrive per warp on each barrier. (An arrive alone would let an
            // L2-fast TMA overwrite the slot under loads still in flight.)
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&cempty[g % RC]);
                tc::mbar_arrive(&sfull[st]);
            }
            TC_PROF_ADD(43, p_w);
#pragma unroll
            for (int k = 0; k < NCH; k++) c[k] = cn[k];
        }
    } else if (warp == 13) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < T && ok && !*abort_flag; t += gridDim.x) {
                TcTile tl = tc_tile(a, t, MT);
                const int N = (tl.it.count + 15) & ~15;
                const uint32_t idesc = tc::idesc_f16(128, N);
                const uint32_t bblk = (16u << tc_sel(tl.it.count)) * 64u;
                for (int ss = 0; ss < nss; ss++, g++) {
                    const int st = g % NS, bs = g % RB, ac = g % NACC;
                    if (!tc::mbar_wait(&sfull[st], (g / NS) & 1, abort_flag, err, 5)) { ok = false; break; }
                    if (!tc::mbar_wait(&bfull[bs], (g / RB) & 1, abort_flag, err, 15)) { ok = false; break; }
                    if (g >= NACC && !tc::mbar_wait(&tempty[ac], ((g / NACC) - 1) & 1, abort_flag, err, 6)) { ok = false; break; }
                    tc::tc_fence_after();
                    const int nbl = min(KB, nb - ss * KB);
                    const uint32_t sa = tc::smem_u32(stages + st * A_STAGE), sb = tc::smem_u32(bring + bs * B_STAGE);
                    for (int jj = 0; jj < nbl; jj++) {
                        // A: core matrix (row group r, K chunk kc) at r*512 + kc*128, no swizzle
                        // B: 8-row x 64-byte swizzle atoms, 512 bytes apart
                        const uint64_t ad = tc::smem_desc(sa + jj * A_BLK, 128, 512);
                        const uint64_t bd = tc::smem_desc_sw64(sb + jj * bblk, 512);
                        const uint32_t td = tbase + (ac * KB + jj) * BN;
                        tc::mma_f16_ss(td, ad, bd, idesc, 0u);                             // k 0-15 (overwrite)
                        tc::mma_f16_ss(td, ad + (256 >> 4), bd + (32 >> 4), idesc, 1u);  // k 16-31
                    }
                    tc::mma_commit(&sempty[st]);  // A stage free once these MMAs complete
                    tc::mma_commit(&bempty[bs]);  // B stage likewise
                    tc::mma_commit(&tfull[ac]);
                }
            }
            if (g) tc::mbar_wait(&tfull[(g - 1) % NACC], ((g - 1) / NACC) & 1, abort_flag, err, 7);
        }
    } else {
        // ---------------- epilogue (warps 0-7) ----------------
        const int q = warp & 3, h = warp >> 2;
        const uint32_t tl_lane = (uint32_t)(q * 32) << 16;
        uint32_t g = 0, gw = 0;
        for (int t = blockIdx.x; t < T; t += gridDim.x) {
            TcTile tl = tc_tile(a, t, MT);
            const int ncols = tl.it.count;
            // per-column info for the output phase
            for (int n = tid; n < BN; n += 256) {
                int r = tl.it.row0 + (n < ncols ? n : 0);
                int xr = a.gather ? a.gather[r] / a.gather_div : r;
                col_xrow[n] = xr;
                float tot = 0.f;
                if (FMT == GPU_FMT_TQ2 && n < ncols) {
                    if (a.xblk) {
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
            // Thread layout of the results (the 16x256b TMEM access shape): rows
            // q*32 + r0 + 8k (k = 0..3) and columns cp + 8i + {0,1} (i = 0..3), so each
            // thread needs 8 activation scales per block instead of 32.
            const int r0 = lane >> 2, cp = (lane & 3) * 2;
            float2 acc[16];  // [k][i]
#pragma unroll
            for (int i = 0; i < 16; i++) acc[i] = make_float2(0.f, 0.f);
            // one block's results (lo: rows r0, r0+8; hi: rows r0+16, r0+24) scaled into acc
            auto scale_blk = [&](const uint32_t (&lo)[16], const uint32_t (&hi)[16], const float *dx, const uint2 (&dwr)[4],
                                 int jj) {
                float dwk[4];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const uint32_t w = (jj < 2) ? dwr[k].x : dwr[k].y;
                    const __half2 hw = *reinterpret_cast<const __half2 *>(&w);
                    dwk[k] = HAS_DW ? ((jj & 1) ? __high2float(hw) : __low2float(hw)) : 1.f;
                }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 d = *reinterpret_cast<const float2 *>(dx + 8 * i + cp);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t *v = k < 2 ? lo : hi;
                        const int b = 4 * i + 2 * (k & 1);
                        const float2 x = make_float2(__uint_as_float(v[b]), __uint_as_float(v[b + 1]));
                        const float2 sc = HAS_DW ? fmul2(make_float2(dwk[k], dwk[k]), d) : d;
                        acc[4 * k + i] = ffma2(sc, x, acc[4 * k + i]);
                    }
                }
            };
#pragma unroll 1
            for (int ss = 0; ss < nss; ss++, g++) {
                const int ac = g % NACC, ds = g % ND, ws = gw % NW;
                const int nbl = min(KB, nb - ss * KB);
                uint2 dwr[4] = {};
                if (HAS_DW) {
                    // (a wait that gives up sets the abort flag; the stage's other waits
                    // then fail too and no result is formed from these values)
                    if ((ss & 1) == 0) tc::mbar_wait(&wfull[ws], (gw / NW) & 1, abort_flag, err, 18);
                    // the 4 fp16 weight scales of the stage for each of this thread's rows
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        dwr[k] = *reinterpret_cast<const uint2 *>(wring + ws * W_SLOT + (q * 32 + r0 + 8 * k) * 16 +
                                                                  (ss & 1) * 8);
                    if ((ss & 1) == 1 || ss == nss - 1) {
                        // values consumed, then ordered before the TMA's refill of the slot
                        asm volatile("" ::"r"(dwr[0].x), "r"(dwr[1].x), "r"(dwr[2].x), "r"(dwr[3].x), "r"(dwr[0].y),
                                     "r"(dwr[1].y), "r"(dwr[2].y), "r"(dwr[3].y)
                                     : "memory");
                        tc::fence_proxy_async();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&wempty[ws]);
                        gw++;
                    }
                }
                bool ok = tc::mbar_wait(&tfull[ac], (g / NACC) & 1, abort_flag, err, 8);
                ok = tc::mbar_wait(&dfull[ds], (g / ND) & 1, abort_flag, err, 9) && ok;
                ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
                // the two warp groups take alternate K stages (group h the stages in odd /
                // even TMEM slots); their partial sums meet in shared memory at the tile
                // end, in the same order for every tile
                const bool work = ok && (ac & 1) == h;
                tc::tc_fence_after();
                const uint32_t tb = tbase + tl_lane + (uint32_t)(ac * KB * BN);
                const float *dx = reinterpret_cast<const float *>(dxring + ds * DX_STAGE);
                uint32_t va[16], vb[16], vc[16], vd[16];
                // blocks 0 and 1 of the stage
                TC_PROF_T(p_ld);
                if (work) {
                    tc::tmem_ld16x256_x4(tb, va);
                    tc::tmem_ld16x256_x4(tb + (16u << 16), vb);
                    if (nbl > 1) {
                        tc::tmem_ld16x256_x4(tb + BN, vc);
                        tc::tmem_ld16x256_x4(tb + BN + (16u << 16), vd);
                    }
                    tc::tmem_ld_wait();
                }
                TC_PROF_ADD(40, p_ld);
                if (nbl <= 2 || !work) {
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&tempty[ac]);  // the stage's accumulators are read
                }
                TC_PROF_T(p_sc);
                if (work) {
                    scale_blk(va, vb, dx, dwr, 0);
                    if (nbl > 1) scale_blk(vc, vd, dx + BN, dwr, 1);
                    // blocks 2 and 3
                    if (nbl > 2) {
                        tc::tmem_ld16x256_x4(tb + 2 * BN, va);
                        tc::tmem_ld16x256_x4(tb + 2 * BN + (16u << 16), vb);
                        if (nbl > 3) {
                            tc::tmem_ld16x256_x4(tb + 3 * BN, vc);
                            tc::tmem_ld16x256_x4(tb + 3 * BN + (16u << 16), vd);
                        }
                        tc::tmem_ld_wait();
                        tc::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&tempty[ac]);
                        scale_blk(va, vb, dx + 2 * BN, dwr, 2);
                        if (nbl > 3) scale_blk(vc, vd, dx + 3 * BN, dwr, 3);
                    }
                }
                TC_PROF_ADD(41, p_sc);
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&dempty[ds]);
            }
            TC_PROF_T(p_out);
            // ---- tile output: 128 x ncols fp32 through shared memory ----
            const float *alpha = FMT == GPU_FMT_TQ2 ? reinterpret_cast<const float *>(
                                                          reinterpret_cast<const uint8_t *>(a.scale) +
                                                          (long)tl.it.group * a.scale_gstride)
                                                    : nullptr;
            const int m0 = tl.m0;
            {
                const int c0n = 0, nc = ncols;
                if (h == 1) {
#pragma unroll
                    for (int k = 0; k < 4; k++)
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            *reinterpret_cast<float2 *>(ct + (q * 32 + r0 + 8 * k) * CS + 8 * i + cp) = acc[4 * k + i];
                }
                // group 0 adds its stages' partial sums to group 1's
                tc::named_sync(1, 256);
                if (h == 0) {
#pragma unroll
                    for (int k = 0; k < 4; k++)
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            float2 *p = reinterpret_cast<float2 *>(ct + (q * 32 + r0 + 8 * k) * CS + 8 * i + cp);
                            const float2 o = *p;
                            *p = make_float2(o.x + acc[4 * k + i].x, o.y + acc[4 * k + i].y);
                        }
                }
                tc::named_sync(1, 256);
                if (!*abort_flag) {
                    if (EPI == EPI_GATEUP) {
                        const int f0 = (m0 / 128) * 64;
                        const int MI = a.O / 2, nbh = MI / 32;
                        for (int wi = warp; wi < nc * 2; wi += 8) {
                            int nl = wi >> 1, hb = wi & 1, n = c0n + nl;
                            int f = hb * 32 + lane;
                            float gv = ct[f * CS + nl], uv = ct[(64 + f) * CS + nl];
                            if (FMT == GPU_FMT_TQ2) {
                                float tot = col_sx[n];
                                gv = alpha[m0 + f] * (gv - tot);
                                uv = alpha[m0 + 64 + f] * (uv - tot);
                            }
                            float hv = gated_act(a.act, gv, uv, a.clamp), d;
                            int8_t qv = quant_lane(hv, d);
                            const size_t pr = (size_t)(tl.it.row0 + n);
                            a.hq[pr * MI + f0 + f] = qv;
                            a.hh[pr * MI + f0 + f] = __int2half_rn(qv);
                            if (lane == 0) {
                                a.hs[pr * nbh + f0 / 32 + hb] = d;
                                a.hsT[(size_t)(f0 / 32 + hb) * a.ldT + pr] = d;
                            }
                            if (FMT == GPU_FMT_TQ2) {
                                int sm = qv;
#pragma unroll
                                for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
                                if (lane == 0) a.hblk[pr * nbh + f0 / 32 + hb] = sm;
                            }
                        }
                    } else {  // EPI_DOWN
                        for (int nl = warp; nl < nc; nl += 8) {
                            const int n = c0n + nl;
                            const int pr = tl.it.row0 + n;
                            const float w = a.pair_w[pr];
                            const int tok = a.pair_src[pr] / a.K;
                            const float tot = col_sx[n];
                            const int r = lane * 4, o = m0 + r;
                            float4 v;
                            v.x = ct[r * CS + nl]; v.y = ct[(r + 1) * CS + nl]; v.z = ct[(r + 2) * CS + nl]; v.w = ct[(r + 3) * CS + nl];
                            if (FMT == GPU_FMT_TQ2) {
                                v.x = alpha[o] * (v.x - tot); v.y = alpha[o + 1] * (v.y - tot);
                                v.z = alpha[o + 2] * (v.z - tot); v.w = alpha[o + 3] * (v.w - tot);
                            }
                            v.x *= w; v.y *= w; v.z *= w; v.w *= w;
                            atomicAdd(reinterpret_cast<float4 *>(a.out + (size_t)tok * a.O + o), v);
                        }
                    }
                }
                tc::named_sync(1, 256);
            }
            TC_PROF_ADD(42, p_out);
        }
    }
#ifdef ZZ_TC_PROF
    // per-role busy span: 32 epilogue, 33 producers, 34 code TMA, 35 MMA, 36 B TMA, 37 dx copies
    if (blockIdx.x == 0 && (tid & 31) == 0)
        atomicAdd(&tc::g_tc_prof[32 + (warp < 8 ? 0 : warp < 12 ? 1 : warp - 10)],
                  (unsigned long long)(clock64() - prof_t0));
#endif
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 13) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tbase, NACC * KB * BN);
    }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int tc_get_encode() {
    if (g_encode) return 1;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
        return fail("cuTensorMapEncodeTiled is not available");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return 1;
}

// codes plane of a whole bank: rows = experts * O, row = row_bytes bytes; one box is
// 128 rows x cb bytes (one K stage), swizzled by its width so that the producers'
// 16-byte loads of one row each hit distinct banks
int tc_make_codes_map(CUtensorMap *map, const uint8_t *codes, long rows, int row_bytes, int cb) {
    if (!tc_get_encode()) return 0;
    if ((uintptr_t)codes & 15 || row_bytes % 16) return fail("tc: codes plane not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)cb, 128};
    const CUtensorMapSwizzle sw = cb == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : cb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                             : CU_TENSOR_MAP_SWIZZLE_32B;
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(codes), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("tc: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 1;
}

// fp16 weight-scale planes of a bank: [experts][O][nbp] (rows padded to 8 blocks), each
// expert `gstride` bytes apart; one box is 128 rows x 8 scales (two K stages)
int tc_make_scale_map(CUtensorMap *map, const void *scale, int E, int O, int nbp, long gstride) {
    if (!tc_get_encode()) return 0;
    if ((uintptr_t)scale & 15 || gstride % 16 || nbp % 8) return fail("tc: scale planes not 16-byte aligned");
    cuuint64_t dims[3] = {(cuuint64_t)nbp, (cuuint64_t)O, (cuuint64_t)E};
    cuuint64_t strides[2] = {(cuuint64_t)nbp * 2, (cuuint64_t)gstride};
    cuuint32_t box[3] = {8, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(scale), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("tc: scale tensor map failed (%d)", (int)r);
    return 1;
}

// pair-ordered fp16 activation rows [rows, I] seen as (8 halves) x rows x (I/8 chunks),
// so one box {8, 128, 4} lands a block's 128 x 32 tile as K-major core matrices
int tc_make_b_map(CUtensorMap *map, const __half *xg, int rows, int I, int box_rows) {
    if (!tc_get_encode()) return 0;
    if ((uintptr_t)xg & 15 || I % 32) return fail("tc: activation rows not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)I, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)I * 2};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(xg), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("tc: activation tensor map failed (%d)", (int)r);
    return 1;
}

template <int FMT, int EPI>
static int launch_tc_t(const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        if (!check_cuda(cudaFuncSetAttribute(k_moe_tc<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, tcm::SMEM),
                        "tc smem attribute"))
            return 0;
        attr = true;
    }
    const int row_bytes = FMT == GPU_FMT_Q40 ? a.I / 2 : FMT == GPU_FMT_Q80 ? a.I : a.I / 4;
    CUtensorMap map, smap;
    BMaps bmaps;
    if (!tc_make_codes_map(&map, a.codes, (long)n_groups * a.O, row_bytes, tc_cb<FMT>())) return 0;
    if (FMT == GPU_FMT_TQ2)
        smap = map;  // tq2 has one fp32 alpha per row, applied at the tile end
    else if (!tc_make_scale_map(&smap, a.scale, n_groups, a.O, ((a.I / ZZ_BLK) + 7) & ~7, a.scale_gstride))
        return 0;
    for (int i = 0; i < 2; i++)
        if (!tc_make_b_map(&bmaps.m[i], a.xg, a.rows_cap, a.I, 16 << i)) return 0;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (const char *e = getenv("ZZ_TC_GRID")) sms = atoi(e) > 0 ? atoi(e) : sms;
    k_moe_tc<FMT, EPI><<<sms, tcm::NTHREADS, tcm::SMEM, st>>>(a, map, smap, bmaps, err);
    return check_cuda(cudaGetLastError(), "tc launch");
}

// The expert GEMMs on tcgen05. Requires: codes planes of consecutive experts exactly
// O * row_bytes apart (true for the packed bank), O % 128 == 0, items of <= 128 rows.
int launch_moe_tc(int fmt, int epi, const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    if (a.O % 128) return fail("tc: O=%d not a multiple of 128", a.O);
    if (epi == EPI_GATEUP) {
        if (fmt == GPU_FMT_Q40) return launch_tc_t<GPU_FMT_Q40, EPI_GATEUP>(a, n_groups, err, st);
        if (fmt == GPU_FMT_Q80) return launch_tc_t<GPU_FMT_Q80, EPI_GATEUP>(a, n_groups, err, st);
        return launch_tc_t<GPU_FMT_TQ2, EPI_GATEUP>(a, n_groups, err, st);
    }
    if (fmt == GPU_FMT_Q40) return launch_tc_t<GPU_FMT_Q40, EPI_DOWN>(a, n_groups, err, st);
    if (fmt == GPU_FMT_Q80) return launch_tc_t<GPU_FMT_Q80, EPI_DOWN>(a, n_groups, err, st);
    return launch_tc_t<GPU_FMT_TQ2, EPI_DOWN>(a, n_groups, err, st);
}

}  // namespace zz

#ifdef ZZ_TC_PROF
extern "C" int zz_tc_prof_read(unsigned long long *out) {
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(out, zz::tc::g_tc_prof, sizeof(unsigned long long) * 128);
    unsigned long long z[128] = {0};
    cudaMemcpyToSymbol(zz::tc::g_tc_prof, z, sizeof z);
    return 1;
}
#endif
