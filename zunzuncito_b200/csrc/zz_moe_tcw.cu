// zz_moe_tcw.cu -- wide-tile expert GEMMs on the 5th-generation tensor cores, for the
// experts that hold many token rows (the large experts of a Zipf-routed batch, and
// nearly all experts at prefill sizes).
//
// Persistent, warp-specialised kernel, one CTA per SM, looping over work tiles (an
// expert item of <= 128 token rows x 128 weight rows). The fixed costs of a tile --
// widening its 128 weight rows to fp16 once per K block, and one mbarrier round trip
// per hand-off -- are spread over up to 128 tokens. Roles (512 threads):
//   warp 12      TMA: the tile's packed weight codes, one box per 4 K blocks (128 rows,
//                swizzled so the producers' 16-byte shared loads are conflict free)
//   warp 14      TMA: the fp16 activation rows of the item, one 64-byte-swizzled K-major
//                box of up to 128 rows per block
//   warp 15      bulk copies: the activation block scales; TMA: the fp16 weight block
//                scales (128 rows x 8 blocks per box)
//   warps 8-11   producers: thread r widens row r's codes of 4 blocks to fp16 in the
//                UMMA canonical K-major layout (the values are the integer codes)
//   warp 13      MMA: one thread issues, per 32-wide K block, two tcgen05.mma kind::f16
//                (M = 128, N = item rows rounded to 16) into one of 4 TMEM block
//                accumulators (4 x 128 columns)
//   warps 0-7    epilogue: warp (q, h) owns TMEM lanes 32q..32q+31 and token columns
//                64h..64h+63; per block it reads the 128 x N f32 block sums -- the
//                reference's exact per-block integer sums -- with the 16x256b shape
//                (4 rows x 16 tokens per thread) and adds (dw*dx) * sum into fp32
//                registers in packed fp32 (the decomposition of q40.h:20-31), the blocks
//                in K order, so a token's sum has one fixed order in any tile. At the
//                tile end: gate/up GeGLU + q8_0 requant (bit-exact with q40_quant_act),
//                or the down projection's weighted scatter-add.
// Waits are bounded (2 s); one that runs out sets the kernel's error word.
#include <cstdlib>
#include <cuda.h>
#include <cudaTypedefs.h>
#include "zz_gemm.cuh"
#include "zz_tc.cuh"
#include "zz_tc_widen.cuh"

namespace zz {

namespace tcw {
constexpr int NTHREADS = 512;
constexpr int BN = 128;            // max token rows per tile
constexpr int KB = 4;              // quantization blocks per A stage
constexpr int NP = 4;              // TMEM block accumulators: NP * BN = 512 columns
constexpr int RING = 32 * 1024;    // weight-code ring
constexpr int NS = 2;              // widened-weight (A) stages
constexpr int A_BLK = 128 * 64;    // one block: 128 rows x 32 fp16, K-major core matrices
constexpr int A_STAGE = KB * A_BLK;
constexpr int RB = 2;              // activation (B) stages
constexpr int B_BLK = BN * 64;     // up to 128 rows x 32 fp16, 64-byte swizzle
constexpr int B_STAGE = KB * B_BLK;
constexpr int ND = 8;              // activation-scale stages
constexpr int DX_BLK = BN * 4;
constexpr int DX_STAGE = KB * DX_BLK;
constexpr int NW = 4;              // weight-scale ring: 128 rows x 8 fp16 (two A stages)
constexpr int W_SLOT = 128 * 16;
constexpr int CTG = BN + 4;        // gate/up exchange: 64 up rows x 128 columns
constexpr int CTD = 64 + 4;        // down: 128 rows x 64 columns (one half at a time)
constexpr int CT_BYTES = 128 * CTD * 4;
static_assert(64 * CTG * 4 <= CT_BYTES, "exchange tile");
constexpr int RC_MAX = 8;
constexpr int OFF_B = 0;           // 1 KB aligned (swizzled TMA destinations)
constexpr int OFF_RING = OFF_B + RB * B_STAGE;
constexpr int OFF_A = OFF_RING + RING;
constexpr int OFF_DX = OFF_A + NS * A_STAGE;
constexpr int OFF_W = OFF_DX + ND * DX_STAGE;
constexpr int OFF_CT = OFF_W + NW * W_SLOT;
constexpr int OFF_INFO = OFF_CT + CT_BYTES;
constexpr int OFF_BAR = OFF_INFO + BN * 4;
constexpr int NBAR = 2 * RC_MAX + 2 * NS + 2 * RB + 2 * NP + 2 * ND + 2 * NW;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + slack to align the base to 1 KB
static_assert(SMEM <= 232448, "shared memory");
}  // namespace tcw

struct BMapsW {
    CUtensorMap m[4];  // activation boxes of 16, 32, 64 and 128 rows
};

__device__ __forceinline__ int tcw_sel(int count) {
    const int N = (count + 15) & ~15;
    return N <= 16 ? 0 : N <= 32 ? 1 : N <= 64 ? 2 : 3;
}

// 16 lanes x 8 x 256 bits: thread t gets, for i = 0..7, lane (t/4) columns 8i + 2(t%4) + {0,1}
// in r[4i], r[4i+1] and lane (t/4)+8 the same columns in r[4i+2], r[4i+3]
__device__ __forceinline__ void tmem_ld16x256_x8(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

template <int FMT, int EPI>
__global__ void __launch_bounds__(tcw::NTHREADS, 1)
    k_moe_tcw(const GemmArgs a, const __grid_constant__ CUtensorMap codes_map,
              const __grid_constant__ CUtensorMap scale_map, const __grid_constant__ BMapsW bmaps, int *err) {
    using namespace tcw;
    constexpr int CB = tc_cb<FMT>(), RC = RING / (128 * CB), SLOTB = 128 * CB, NCH = CB / 16;
    constexpr bool HAS_DW = FMT != GPU_FMT_TQ2;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *ring = smem + OFF_RING, *stages = smem + OFF_A, *bring = smem + OFF_B;
    uint8_t *dxring = smem + OFF_DX, *wring = smem + OFF_W;
    float *ct = reinterpret_cast<float *>(smem + OFF_CT);
    float *col_sx = reinterpret_cast<float *>(smem + OFF_INFO);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *cfull = bars, *cempty = bars + RC_MAX;
    uint64_t *sfull = bars + 2 * RC_MAX, *sempty = sfull + NS;
    uint64_t *bfull = sempty + NS, *bempty = bfull + RB;
    uint64_t *tfull = bempty + RB, *tempty = tfull + NP;
    uint64_t *dfull = tempty + NP, *dempty = dfull + ND;
    uint64_t *wfull = dempty + ND, *wempty = wfull + NW;
    uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_BAR + NBAR * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + NBAR * 8 + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = a.I / ZZ_BLK;
    const int nss = (nb + KB - 1) / KB;
    const int MT = a.O / 128;
    const int T = *a.n_items * MT;
    auto tile = [&](int t, WorkItem &it, int &m0) {
        it = a.items[t / MT];
        m0 = (t % MT) * 128;
    };

    if (tid == 0) {
        for (int i = 0; i < RC; i++) { tc::mbar_init(&cfull[i], 1); tc::mbar_init(&cempty[i], 4); }
        for (int i = 0; i < NS; i++) { tc::mbar_init(&sfull[i], 4); tc::mbar_init(&sempty[i], 1); }
        for (int i = 0; i < RB; i++) { tc::mbar_init(&bfull[i], 1); tc::mbar_init(&bempty[i], 1); }
        for (int i = 0; i < NP; i++) { tc::mbar_init(&tfull[i], 1); tc::mbar_init(&tempty[i], 8); }
        for (int i = 0; i < ND; i++) { tc::mbar_init(&dfull[i], 1); tc::mbar_init(&dempty[i], 8); }
        for (int i = 0; i < NW; i++) { tc::mbar_init(&wfull[i], 1); tc::mbar_init(&wempty[i], 8); }
        *abort_flag = 0;
        tc::mbar_init_fence();
    }
    if (warp == 13) tc::tmem_alloc(tmem_base_smem, NP * BN);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tbase = *tmem_base_smem;
    TC_PROF_T(prof_t0);

    if (warp == 12) {
        if (lane == 0) {
            // ---------------- TMA: weight codes, one box per A stage ----------------
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < T && ok && !*abort_flag; t += gridDim.x) {
                WorkItem it; int m0;
                tile(t, it, m0);
                const int y = it.group * a.O + m0;
                for (int ss = 0; ss < nss; ss++, g++) {
                    const int s = g % RC;
                    const uint32_t u = g / RC;
                    if (u && !tc::mbar_wait(&cempty[s], (u - 1) & 1, abort_flag, err, 1)) { ok = false; break; }
                    tc::mbar_arrive_tx(&cfull[s], SLOTB);
                    tc::tma_load_2d(ring + s * SLOTB, &codes_map, ss * CB, y, &cfull[s]);
                }
            }
            if (g) tc::mbar_wait(&cfull[(g - 1) % RC], ((g - 1) / RC) & 1, abort_flag, err, 2);
        }
    } else if (warp == 14) {
        if (lane == 0) {
            // ---------------- TMA: activation tiles, one box per block ----------------
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < T && ok && !*abort_flag; t += gridDim.x) {
                WorkItem it; int m0;
                tile(t, it, m0);
                const int sel = tcw_sel(it.count);
                const uint32_t bblk = (16u << sel) * 64u;
                for (int ss = 0; ss < nss; ss++, g++) {
                    const int bs = g % RB;
                    const uint32_t u = g / RB;
                    if (u && !tc::mbar_wait(&bempty[bs], (u - 1) & 1, abort_flag, err, 3)) { ok = false; break; }
                    const int nbl = min(KB, nb - ss * KB);
                    tc::mbar_arrive_tx(&bfull[bs], bblk * nbl);
                    uint8_t *dst = bring + bs * B_STAGE;
                    // the map is named with a constant index so it stays in parameter space
                    for (int jj = 0; jj < nbl; jj++) {
                        const int x = (ss * KB + jj) * 32;
                        switch (sel) {
                            case 0: tc::tma_load_2d(dst + jj * bblk, &bmaps.m[0], x, it.row0, &bfull[bs]); break;
                            case 1: tc::tma_load_2d(dst + jj * bblk, &bmaps.m[1], x, it.row0, &bfull[bs]); break;
                            case 2: tc::tma_load_2d(dst + jj * bblk, &bmaps.m[2], x, it.row0, &bfull[bs]); break;
                            default: tc::tma_load_2d(dst + jj * bblk, &bmaps.m[3], x, it.row0, &bfull[bs]); break;
                        }
                    }
                }
            }
            if (g) tc::mbar_wait(&bfull[(g - 1) % RB], ((g - 1) / RB) & 1, abort_flag, err, 12);
        }
    } else if (warp == 15) {
        if (lane == 0) {
            // ---------------- activation block scales; weight block scales ----------------
            uint32_t g = 0, gw = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < T && ok && !*abort_flag; t += gridDim.x) {
                WorkItem it; int m0;
                tile(t, it, m0);
                for (int ss = 0; ss < nss; ss++, g++) {
                    if (HAS_DW && (ss & 1) == 0) {
                        const int ws = gw % NW;
                        const uint32_t wu = gw / NW;
                        if (wu && !tc::mbar_wait(&wempty[ws], (wu - 1) & 1, abort_flag, err, 16)) { ok = false; break; }
                        tc::mbar_arrive_tx(&wfull[ws], W_SLOT);
                        tc::tma_load_3d(wring + ws * W_SLOT, &scale_map, ss * KB, m0, it.group, &wfull[ws]);
                        gw++;
                    }
                    const int ds = g % ND;
                    const uint32_t du = g / ND;
                    if (du && !tc::mbar_wait(&dempty[ds], (du - 1) & 1, abort_flag, err, 11)) { ok = false; break; }
                    const int nbl = min(KB, nb - ss * KB);
                    tc::mbar_arrive_tx(&dfull[ds], DX_BLK * nbl);
                    for (int jj = 0; jj < nbl; jj++)
                        tc::bulk_load(dxring + ds * DX_STAGE + jj * DX_BLK,
                                      a.xsT + (size_t)(ss * KB + jj) * a.ldT + it.row0, DX_BLK, &dfull[ds]);
                }
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
        const uint32_t G = (uint32_t)my_tiles * nss;  // A stages of all this CTA's tiles, in order
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
            if (g + 1 < G && !fetch(g + 1, cn)) break;  // next stage's codes in flight
            const int st = g % NS;
            if (g >= NS && !tc::mbar_wait(&sempty[st], ((g / NS) - 1) & 1, abort_flag, err, 14)) break;
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
            // one proxy fence per thread orders its shared stores of the stage (read next
            // by the tensor cores) and its consumed shared loads of the code slot (refilled
            // next by the TMA) before the async proxy; then one elected arrive per warp
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
            uint32_t g = 0, gb = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < T && ok && !*abort_flag; t += gridDim.x) {
                WorkItem it; int m0;
                tile(t, it, m0);
                const int N = (it.count + 15) & ~15;
                const uint32_t idesc = tc::idesc_f16(128, N);
                const uint32_t bblk = (16u << tcw_sel(it.count)) * 64u;
                for (int ss = 0; ss < nss && ok; ss++, g++) {
                    const int st = g % NS, bs = g % RB;
                    if (!tc::mbar_wait(&sfull[st], (g / NS) & 1, abort_flag, err, 5)) { ok = false; break; }
                    if (!tc::mbar_wait(&bfull[bs], (g / RB) & 1, abort_flag, err, 15)) { ok = false; break; }
                    tc::tc_fence_after();
                    const int nbl = min(KB, nb - ss * KB);
                    const uint32_t sa = tc::smem_u32(stages + st * A_STAGE), sb = tc::smem_u32(bring + bs * B_STAGE);
                    for (int jj = 0; jj < nbl; jj++, gb++) {
                        const int p = gb % NP;
                        if (gb >= NP && !tc::mbar_wait(&tempty[p], ((gb / NP) - 1) & 1, abort_flag, err, 6)) {
                            ok = false;
                            break;
                        }
                        tc::tc_fence_after();
                        // A: core matrix (row group r, K chunk kc) at r*512 + kc*128, no swizzle
                        // B: 8-row x 64-byte swizzle atoms, 512 bytes apart
                        const uint64_t ad = tc::smem_desc(sa + jj * A_BLK, 128, 512);
                        const uint64_t bd = tc::smem_desc_sw64(sb + jj * bblk, 512);
                        const uint32_t td = tbase + p * BN;
                        tc::mma_f16_ss(td, ad, bd, idesc, 0u);                             // k 0-15 (overwrite)
                        tc::mma_f16_ss(td, ad + (256 >> 4), bd + (32 >> 4), idesc, 1u);  // k 16-31
                        tc::mma_commit(&tfull[p]);
                    }
                    if (!ok) break;
                    tc::mma_commit(&sempty[st]);  // A stage free once these MMAs complete
                    tc::mma_commit(&bempty[bs]);  // B stage likewise
                }
            }
            if (gb) tc::mbar_wait(&tfull[(gb - 1) % NP], ((gb - 1) / NP) & 1, abort_flag, err, 7);
        }
    } else {
        // ---------------- epilogue (warps 0-7) ----------------
        const int q = warp & 3, h = warp >> 2;
        const int r0 = lane >> 2, cp = (lane & 3) * 2;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        uint32_t g = 0, gb = 0, gw = 0;
        for (int t = blockIdx.x; t < T; t += gridDim.x) {
            WorkItem it; int m0;
            tile(t, it, m0);
            const int ncols = it.count;
            const bool cv = 64 * h < ncols;  // this warp's columns hold tokens
            // per-column tq2 offset total for the output phase
            for (int n = tid; n < BN; n += 256) {
                float tot = 0.f;
                if (FMT == GPU_FMT_TQ2 && n < ncols) {
                    const int r = it.row0 + n;
                    const int xr = a.gather ? a.gather[r] / a.gather_div : r;
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
            float2 acc[32];  // [k][i]: row r0 + 8k, columns 64h + 8i + cp + {0,1}
#pragma unroll
            for (int i = 0; i < 32; i++) acc[i] = make_float2(0.f, 0.f);
            // one block's sums of rows kb, kb+1 (16x256b registers v) scaled into acc
            auto scale = [&](const uint32_t (&v)[32], int kb, const float *dx, const float (&dwk)[4]) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float2 d = *reinterpret_cast<const float2 *>(dx + 8 * i + cp);
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        const int k = kb + kk;
                        const float2 x = make_float2(__uint_as_float(v[4 * i + 2 * kk]), __uint_as_float(v[4 * i + 2 * kk + 1]));
                        const float2 sc = HAS_DW ? fmul2(make_float2(dwk[k], dwk[k]), d) : d;
                        acc[8 * k + i] = ffma2(sc, x, acc[8 * k + i]);
                    }
                }
            };
#pragma unroll 1
            for (int ss = 0; ss < nss; ss++, g++) {
                const int ds = g % ND, ws = gw % NW;
                const int nbl = min(KB, nb - ss * KB);
                uint2 dwr[4] = {};
                if (HAS_DW) {
                    // (a wait that gives up sets the abort flag; the block waits below then
                    // fail too and no result is formed from these values)
                    if ((ss & 1) == 0) tc::mbar_wait(&wfull[ws], (gw / NW) & 1, abort_flag, err, 18);
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
                bool dok = tc::mbar_wait(&dfull[ds], (g / ND) & 1, abort_flag, err, 9);
                const float *dxs = reinterpret_cast<const float *>(dxring + ds * DX_STAGE) + 64 * h;
#pragma unroll 1
                for (int jj = 0; jj < nbl; jj++, gb++) {
                    const int p = gb % NP;
                    bool ok = tc::mbar_wait(&tfull[p], (gb / NP) & 1, abort_flag, err, 8) && dok;
                    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
                    tc::tc_fence_after();
                    const bool work = ok && cv;
                    float dwk[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t w = jj < 2 ? dwr[k].x : dwr[k].y;
                        const __half2 hw = *reinterpret_cast<const __half2 *>(&w);
                        dwk[k] = (jj & 1) ? __high2float(hw) : __low2float(hw);
                    }
                    const float *dx = dxs + jj * BN;
                    const uint32_t tb = tbase + lane_base + (uint32_t)(p * BN + 64 * h);
                    uint32_t v[32];
                    TC_PROF_T(p_ep);
                    if (work) {
                        tmem_ld16x256_x8(tb, v);  // rows r0, r0 + 8
                        tc::tmem_ld_wait();
                        scale(v, 0, dx, dwk);
                        tmem_ld16x256_x8(tb + (16u << 16), v);  // rows r0 + 16, r0 + 24
                        tc::tmem_ld_wait();
                    }
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&tempty[p]);  // this block's accumulator is read
                    if (work) scale(v, 2, dx, dwk);
                    TC_PROF_ADD(41, p_ep);
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&dempty[ds]);
            }
            TC_PROF_T(p_out);
            // ---- tile output ----
            const float *alpha = FMT == GPU_FMT_TQ2 ? reinterpret_cast<const float *>(
                                                          reinterpret_cast<const uint8_t *>(a.scale) +
                                                          (long)it.group * a.scale_gstride)
                                                    : nullptr;
            if (EPI == EPI_GATEUP) {
                // rows 0-63 are the gate rows and 64-127 the up rows of the same 64 features:
                // the up halves go through shared memory to the warps holding the gates
                const int MI = a.O / 2, nbh = MI / 32, f0 = (m0 / 128) * 64;
                if (q >= 2 && cv) {
#pragma unroll
                    for (int k = 0; k < 4; k++)
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            *reinterpret_cast<float2 *>(ct + ((q - 2) * 32 + r0 + 8 * k) * CTG + 64 * h + 8 * i + cp) =
                                acc[8 * k + i];
                }
                tc::named_sync(1, 256);
                if (q < 2 && cv && !*abort_flag) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int col = 64 * h + 8 * i + cp + e;
                            float hv[4];
                            float amax = 0.f;
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                const int fl = q * 32 + r0 + 8 * k;
                                float gv = e ? acc[8 * k + i].y : acc[8 * k + i].x;
                                float uv = ct[fl * CTG + col];
                                if (FMT == GPU_FMT_TQ2) {
                                    gv = alpha[m0 + fl] * (gv - col_sx[col]);
                                    uv = alpha[m0 + 64 + fl] * (uv - col_sx[col]);
                                }
                                hv[k] = gated_act(a.act, gv, uv, a.clamp);
                                amax = fmaxf(amax, fabsf(hv[k]));
                            }
                            // q8_0 block = this warp's 32 features of the column: 4 per lane
                            // over the 8 lanes sharing lane % 4 (q40_quant_act, q40.h:124-138)
#pragma unroll
                            for (int o = 4; o < 32; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                            const float d = __fdiv_rn(amax, 127.0f);
                            const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
                            int qs = 0;
                            const bool cw = col < ncols;
                            const size_t pr = (size_t)(it.row0 + (cw ? col : 0));
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                int qv = __float2int_rn(__fmul_rn(hv[k], id));
                                qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
                                qs += qv;
                                if (cw) {
                                    const int f = f0 + q * 32 + r0 + 8 * k;
                                    a.hq[pr * MI + f] = (int8_t)qv;
                                    a.hh[pr * MI + f] = __int2half_rn(qv);
                                }
                            }
                            if (FMT == GPU_FMT_TQ2) {
#pragma unroll
                                for (int o = 4; o < 32; o <<= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
                            }
                            if (cw && r0 == 0) {
                                const int blk = f0 / 32 + q;
                                a.hs[pr * nbh + blk] = d;
                                a.hsT[(size_t)blk * a.ldT + pr] = d;
                                if (FMT == GPU_FMT_TQ2) a.hblk[pr * nbh + blk] = qs;
                            }
                        }
                    }
                }
                tc::named_sync(1, 256);
            } else {  // EPI_DOWN: two column halves through shared memory, float4 atomics along o
                for (int hh = 0; hh < 2; hh++) {
                    if (h == hh && cv) {
#pragma unroll
                        for (int k = 0; k < 4; k++)
#pragma unroll
                            for (int i = 0; i < 8; i++)
                                *reinterpret_cast<float2 *>(ct + (q * 32 + r0 + 8 * k) * CTD + 8 * i + cp) = acc[8 * k + i];
                    }
                    tc::named_sync(1, 256);
                    if (!*abort_flag) {
                        for (int task = tid; task < 64 * 32; task += 256) {
                            const int nl = task & 63, o4 = task >> 6;
                            const int n = 64 * hh + nl;
                            if (n >= ncols) continue;
                            const int pr = it.row0 + n;
                            const float w = a.pair_w[pr];
                            const int tok = a.pair_src[pr] / a.K;
                            const int o = m0 + 4 * o4;
                            float4 v;
                            v.x = ct[(4 * o4) * CTD + nl]; v.y = ct[(4 * o4 + 1) * CTD + nl];
                            v.z = ct[(4 * o4 + 2) * CTD + nl]; v.w = ct[(4 * o4 + 3) * CTD + nl];
                            if (FMT == GPU_FMT_TQ2) {
                                const float tot = col_sx[n];
                                v.x = alpha[o] * (v.x - tot); v.y = alpha[o + 1] * (v.y - tot);
                                v.z = alpha[o + 2] * (v.z - tot); v.w = alpha[o + 3] * (v.w - tot);
                            }
                            v.x *= w; v.y *= w; v.z *= w; v.w *= w;
                            atomicAdd(reinterpret_cast<float4 *>(a.out + (size_t)tok * a.O + o), v);
                        }
                    }
                    tc::named_sync(1, 256);
                }
            }
            TC_PROF_ADD(42, p_out);
        }
    }
#ifdef ZZ_TC_PROF
    // per-role busy span: 32 epilogue, 33 producers, 34 code TMA, 35 MMA, 36 B TMA, 37 scale copies
    if (blockIdx.x == 0 && (tid & 31) == 0)
        atomicAdd(&tc::g_tc_prof[32 + (warp < 8 ? 0 : warp < 12 ? 1 : warp - 10)], (unsigned long long)(clock64() - prof_t0));
#endif
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 13) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tbase, NP * BN);
    }
}

// ---------------------------------------------------------------- host side
// tensor maps shared with the narrow tcgen05 kernel (zz_moe_tc.cu)
int tc_make_codes_map(CUtensorMap *map, const uint8_t *codes, long rows, int row_bytes, int cb);
int tc_make_scale_map(CUtensorMap *map, const void *scale, int E, int O, int nbp, long gstride);
int tc_make_b_map(CUtensorMap *map, const __half *xg, int rows, int I, int box_rows);

template <int FMT, int EPI>
static int launch_tcw_t(const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        if (!check_cuda(cudaFuncSetAttribute(k_moe_tcw<FMT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, tcw::SMEM),
                        "tcw smem attribute"))
            return 0;
        attr = true;
    }
    const int row_bytes = FMT == GPU_FMT_Q40 ? a.I / 2 : FMT == GPU_FMT_Q80 ? a.I : a.I / 4;
    CUtensorMap map, smap;
    BMapsW bmaps;
    if (!tc_make_codes_map(&map, a.codes, (long)n_groups * a.O, row_bytes, tc_cb<FMT>())) return 0;
    if (FMT == GPU_FMT_TQ2)
        smap = map;  // tq2 has one fp32 alpha per row, applied at the tile end
    else if (!tc_make_scale_map(&smap, a.scale, n_groups, a.O, ((a.I / ZZ_BLK) + 7) & ~7, a.scale_gstride))
        return 0;
    for (int i = 0; i < 4; i++)
        if (!tc_make_b_map(&bmaps.m[i], a.xg, a.rows_cap, a.I, 16 << i)) return 0;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    k_moe_tcw<FMT, EPI><<<sms, tcw::NTHREADS, tcw::SMEM, st>>>(a, map, smap, bmaps, err);
    return check_cuda(cudaGetLastError(), "tcw launch");
}

// The expert GEMMs over items of <= 128 rows on wide tcgen05 tiles. Requires: codes
// planes of consecutive experts exactly O * row_bytes apart (true for the packed bank),
// O % 128 == 0.
int launch_moe_tcw(int fmt, int epi, const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    if (a.O % 128) return fail("tcw: O=%d not a multiple of 128", a.O);
    if (epi == EPI_GATEUP) {
        if (fmt == GPU_FMT_Q40) return launch_tcw_t<GPU_FMT_Q40, EPI_GATEUP>(a, n_groups, err, st);
        if (fmt == GPU_FMT_Q80) return launch_tcw_t<GPU_FMT_Q80, EPI_GATEUP>(a, n_groups, err, st);
        return launch_tcw_t<GPU_FMT_TQ2, EPI_GATEUP>(a, n_groups, err, st);
    }
    if (fmt == GPU_FMT_Q40) return launch_tcw_t<GPU_FMT_Q40, EPI_DOWN>(a, n_groups, err, st);
    if (fmt == GPU_FMT_Q80) return launch_tcw_t<GPU_FMT_Q80, EPI_DOWN>(a, n_groups, err, st);
    return launch_tcw_t<GPU_FMT_TQ2, EPI_DOWN>(a, n_groups, err, st);
}

}  // namespace zz

#ifdef ZZ_TC_PROF
// diagnostic build only: this translation unit's wait-site cycle totals
extern "C" int zz_tcw_prof_read(unsigned long long *out) {
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(out, zz::tc::g_tc_prof, sizeof(unsigned long long) * 128);
    unsigned long long z[128] = {0};
    cudaMemcpyToSymbol(zz::tc::g_tc_prof, z, sizeof z);
    return 1;
}
#endif
