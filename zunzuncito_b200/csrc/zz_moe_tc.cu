// zz_moe_tc.cu -- the batch-union expert GEMMs on the 5th-generation tensor cores.
//
// Persistent, warp-specialised kernel, one CTA per SM, looping over work tiles
// (expert item x 128 weight rows). Roles (448 threads):
//   warp 12      TMA: streams the packed weight codes of the tile (128 rows x 64 B
//                boxes) into a 6-slot ring, ~48 KB in flight per SM
//   warps 8-11   producers: thread r widens row r's codes of one 32-weight block to
//                fp16 in the UMMA canonical K-major layout (8-row x 16-byte core
//                matrices, no swizzle), and gathers the token rows' fp16 activations
//                and their block scales with cp.async, several blocks ahead
//   warp 13      MMA: one thread issues two tcgen05.mma kind::f16 (M=128, N = tokens
//                rounded to 16, K=16 each) per block into one of 4 TMEM accumulators
//   warps 0-7    epilogue: tcgen05.ld of the block's 128 x N f32 results, which are
//                the reference's exact per-block integer sums (the fp16 operands are
//                the integer codes themselves), then acc += (dw*dx) * sum in packed
//                fp32 (the decomposition of q40.h:20-31); at the tile end the fused
//                gate/up GeGLU + q8 requant or down-projection scatter-add.
// Per block the tensor cores run while the producers widen the next blocks and the
// epilogue scales the previous one; TMEM decouples MMA from the epilogue.
#include <cstdlib>
#include <cuda.h>
#include <cudaTypedefs.h>
#include "zz_gemm.cuh"
#include "zz_tc.cuh"

namespace zz {

namespace tcm {
constexpr int NTHREADS = 512;
constexpr int BN = 64;            // max activation rows per tile
constexpr int NACC = 8;           // TMEM accumulators (NACC * BN = 512 columns)
constexpr int RC = 4;             // weight-code ring slots (4 blocks each for q4_0)
constexpr int SLOT = 128 * 64;    // one code box: 128 rows x 64 bytes
constexpr int NS = 4;             // widened-weight (A) stages
constexpr int RB = 24;            // activation (B) ring slots
constexpr int A_BYTES = 128 * 64;  // 128 rows x 32 fp16, K-major core matrices
constexpr int B_BYTES = BN * 64;   // up to 64 rows x 32 fp16, 64-byte swizzle
constexpr int DX_BYTES = BN * 4;
constexpr int NDX = 16;           // activation-scale ring (freed by the epilogue)
constexpr int CS = BN + 4;        // padded row of the fp32 result tile
constexpr int OFF_B = 0;          // 1024-aligned (swizzled TMA destination)
constexpr int OFF_RING = OFF_B + RB * B_BYTES;
constexpr int OFF_A = OFF_RING + RC * SLOT;
constexpr int OFF_DX = OFF_A + NS * A_BYTES;
constexpr int OFF_CT = OFF_DX + NDX * DX_BYTES;
constexpr int OFF_INFO = OFF_CT + 128 * CS * 4;
constexpr int OFF_BAR = OFF_INFO + BN * 12;
constexpr int NBAR = 2 * RC + 2 * NS + 2 * RB + 2 * NACC + 2 * NDX;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + slack to align the base to 1 KB
}  // namespace tcm

// offset of block j's codes inside one weight row, and the bytes it spans
template <int FMT>
__device__ __forceinline__ int blk_byte(int j) {
    return FMT == GPU_FMT_Q40 ? j * 16 : FMT == GPU_FMT_Q80 ? j * 32 : (j >> 1) * 16;
}
template <int FMT>
__device__ __forceinline__ int blk_span() { return FMT == GPU_FMT_Q80 ? 32 : 16; }

__device__ __forceinline__ uint32_t spread_lo(uint32_t w) { return __byte_perm(w, 0u, 0x4140u); }
__device__ __forceinline__ uint32_t spread_hi(uint32_t w) { return __byte_perm(w, 0u, 0x4342u); }

// widen one row's codes of one block into the 4 K-chunks (8 fp16 each) of the A tile
template <int FMT>
__device__ __forceinline__ void widen_row(const uint8_t *src, int j, uint4 out[4]) {
    if (FMT == GPU_FMT_Q40) {
        uint4 w = *reinterpret_cast<const uint4 *>(src);
        // k 0-7: low nibbles of bytes 0-7; k 8-15: bytes 8-15; k 16-31: the high nibbles
        out[0] = make_uint4(q4lo_h2(spread_lo(w.x)), q4lo_h2(spread_hi(w.x)), q4lo_h2(spread_lo(w.y)), q4lo_h2(spread_hi(w.y)));
        out[1] = make_uint4(q4lo_h2(spread_lo(w.z)), q4lo_h2(spread_hi(w.z)), q4lo_h2(spread_lo(w.w)), q4lo_h2(spread_hi(w.w)));
        out[2] = make_uint4(q4hi_h2(spread_lo(w.x)), q4hi_h2(spread_hi(w.x)), q4hi_h2(spread_lo(w.y)), q4hi_h2(spread_hi(w.y)));
        out[3] = make_uint4(q4hi_h2(spread_lo(w.z)), q4hi_h2(spread_hi(w.z)), q4hi_h2(spread_lo(w.w)), q4hi_h2(spread_hi(w.w)));
    } else if (FMT == GPU_FMT_Q80) {
        const uint4 *p = reinterpret_cast<const uint4 *>(src);
        uint4 w0 = p[0], w1 = p[1];
        out[0] = make_uint4(s8_h2(spread_lo(w0.x)), s8_h2(spread_hi(w0.x)), s8_h2(spread_lo(w0.y)), s8_h2(spread_hi(w0.y)));
        out[1] = make_uint4(s8_h2(spread_lo(w0.z)), s8_h2(spread_hi(w0.z)), s8_h2(spread_lo(w0.w)), s8_h2(spread_hi(w0.w)));
        out[2] = make_uint4(s8_h2(spread_lo(w1.x)), s8_h2(spread_hi(w1.x)), s8_h2(spread_lo(w1.y)), s8_h2(spread_hi(w1.y)));
        out[3] = make_uint4(s8_h2(spread_lo(w1.z)), s8_h2(spread_hi(w1.z)), s8_h2(spread_lo(w1.w)), s8_h2(spread_hi(w1.w)));
    } else {
        // tq2: the block's 32 codes sit in the 16 bytes of its 64-weight group, at bit
        // offset sh (k 0-15) and sh+2 (k 16-31), sh = 0 for even blocks, 4 for odd
        uint4 w = *reinterpret_cast<const uint4 *>(src);
        const int sh = (j & 1) * 4;
        out[0] = make_uint4(c2_h2(spread_lo(w.x), sh), c2_h2(spread_hi(w.x), sh), c2_h2(spread_lo(w.y), sh), c2_h2(spread_hi(w.y), sh));
        out[1] = make_uint4(c2_h2(spread_lo(w.z), sh), c2_h2(spread_hi(w.z), sh), c2_h2(spread_lo(w.w), sh), c2_h2(spread_hi(w.w), sh));
        out[2] = make_uint4(c2_h2(spread_lo(w.x), sh + 2), c2_h2(spread_hi(w.x), sh + 2), c2_h2(spread_lo(w.y), sh + 2), c2_h2(spread_hi(w.y), sh + 2));
        out[3] = make_uint4(c2_h2(spread_lo(w.z), sh + 2), c2_h2(spread_hi(w.z), sh + 2), c2_h2(spread_lo(w.w), sh + 2), c2_h2(spread_hi(w.w), sh + 2));
    }
}

struct BMaps {
    CUtensorMap m[3];  // activation boxes of 16, 32 and 64 rows
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

template <int FMT, int EPI>
__global__ void __launch_bounds__(tcm::NTHREADS, 1)
    k_moe_tc(const GemmArgs a, const __grid_constant__ CUtensorMap codes_map, const __grid_constant__ BMaps bmaps,
             int *err) {
    using namespace tcm;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *ring = smem + OFF_RING;
    uint8_t *stages = smem + OFF_A;
    uint8_t *bring = smem + OFF_B;
    float *ct = reinterpret_cast<float *>(smem + OFF_CT);
    int *col_xrow = reinterpret_cast<int *>(smem + OFF_INFO);
    float *col_sx = reinterpret_cast<float *>(smem + OFF_INFO + BN * 4);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *cfull = bars, *cempty = bars + RC, *sfull = bars + 2 * RC, *sempty = bars + 2 * RC + NS;
    uint64_t *tfull = bars + 2 * RC + 2 * NS, *tempty = bars + 2 * RC + 2 * NS + NACC;
    uint64_t *dfull = tempty + NACC, *dempty = dfull + NDX, *bfull = dempty + NDX, *bempty = bfull + RB;
    uint8_t *dxring = smem + OFF_DX;
    uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_BAR + NBAR * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + NBAR * 8 + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = a.I / ZZ_BLK, nbp = (nb + 7) & ~7;
    const int MT = a.O / 128;
    const int T = *a.n_items * MT;
    const int row_bytes = FMT == GPU_FMT_Q40 ? a.I / 2 : FMT == GPU_FMT_Q80 ? a.I : a.I / 4;
    const int nslots = (row_bytes + 63) / 64;

    if (tid == 0) {
        for (int i = 0; i < RC; i++) { tc::mbar_init(&cfull[i], 1); tc::mbar_init(&cempty[i], 128); }
        for (int i = 0; i < NS; i++) { tc::mbar_init(&sfull[i], 128); tc::mbar_init(&sempty[i], 1); }
        for (int i = 0; i < NDX; i++) { tc::mbar_init(&dfull[i], 1); tc::mbar_init(&dempty[i], 8); }
        for (int i = 0; i < RB; i++) { tc::mbar_init(&bfull[i], 1); tc::mbar_init(&bempty[i], 1); }
        for (int i = 0; i < NACC; i++) { tc::mbar_init(&tfull[i], 1); tc::mbar_init(&tempty[i], 8); }
        *abort_flag = 0;
        tc::mbar_init_fence();
    }
    if (warp == 13) tc::tmem_alloc(tmem_base_smem, NACC * BN);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tbase = *tmem_base_smem;
#ifdef ZZ_TC_PROF
    if (blockIdx.x == 0 && tid == 0) atomicAdd(&tc::g_tc_prof[30], (unsigned long long)clock64());
#endif

    // activation-tile issue loop (one thread); the tensor map is named with a constant
    // index so it stays in parameter space
    auto issue_b_tiles = [&]() {
        uint32_t g = 0, last = 0;
        bool any = false;
        for (int t = blockIdx.x; t < T && !*abort_flag; t += gridDim.x) {
            TcTile tl = tc_tile(a, t, MT);
            const int N = (tl.it.count + 15) & ~15;
            const int sel = N <= 16 ? 0 : N <= 32 ? 1 : 2;
            const uint32_t bbytes = (16u << sel) * 64u;
            bool ok = true;
            for (int j = 0; j < nb && ok; j++, g++) {
                const int bs = g % RB;
                const uint32_t u = g / RB;
                if (u && !tc::mbar_wait(&bempty[bs], (u - 1) & 1, abort_flag, err, 3)) { ok = false; break; }
                tc::mbar_arrive_tx(&bfull[bs], bbytes);
                uint8_t *dst = bring + bs * B_BYTES;
                // rows row0.. of the pair-ordered activations, halves 32j..32j+31: one
                // 64-byte-swizzled K-major tile
                switch (sel) {
                    case 0: tc::tma_load_2d(dst, &bmaps.m[0], j * 32, tl.it.row0, &bfull[bs]); break;
                    case 1: tc::tma_load_2d(dst, &bmaps.m[1], j * 32, tl.it.row0, &bfull[bs]); break;
                    default: tc::tma_load_2d(dst, &bmaps.m[2], j * 32, tl.it.row0, &bfull[bs]); break;
                }
                last = g;
                any = true;
            }
        }
        if (any) tc::mbar_wait(&bfull[last % RB], (last / RB) & 1, abort_flag, err, 12);
    };

    if (warp == 12) {
        if (lane == 0) {
            // ---------------- TMA: weight codes -> ring (deep, from HBM) ----------------
            uint32_t c = 0;
            for (int t = blockIdx.x; t < T && !*abort_flag; t += gridDim.x) {
                TcTile tl = tc_tile(a, t, MT);
                const int y = tl.it.group * a.O + tl.m0;
                for (int i = 0; i < nslots; i++, c++) {
                    const int s = c % RC;
                    const uint32_t u = c / RC;
                    if (u && !tc::mbar_wait(&cempty[s], (u - 1) & 1, abort_flag, err, 1)) break;
                    tc::mbar_arrive_tx(&cfull[s], SLOT);
                    tc::tma_load_2d(ring + s * SLOT, &codes_map, i * 64, y, &cfull[s]);
                }
            }
            // bounded drain: do not leave the CTA with copies in flight
            if (c) tc::mbar_wait(&cfull[(c - 1) % RC], ((c - 1) / RC) & 1, abort_flag, err, 2);
        } else if (lane == 1) {
        }
    } else if (warp == 14) {
        // ---------------- TMA: activation tiles ----------------
        if (lane == 0) issue_b_tiles();
    } else if (warp == 15) {
        if (lane == 0) {
            // ---------------- bulk copies: the tiles' activation block scales ----------------
            uint32_t g = 0;
            for (int t = blockIdx.x; t < T && !*abort_flag; t += gridDim.x) {
                TcTile tl = tc_tile(a, t, MT);
                bool ok = true;
                for (int j = 0; j < nb && ok; j++, g++) {
                    const int ds = g % NDX;
                    const uint32_t du = g / NDX;
                    if (du && !tc::mbar_wait(&dempty[ds], (du - 1) & 1, abort_flag, err, 11)) { ok = false; break; }
                    tc::mbar_arrive_tx(&dfull[ds], DX_BYTES);
                    tc::bulk_load(dxring + ds * DX_BYTES, a.xsT + (size_t)j * a.ldT + tl.it.row0, DX_BYTES, &dfull[ds]);
                }
            }
            if (g) tc::mbar_wait(&dfull[(g - 1) % NDX], ((g - 1) / NDX) & 1, abort_flag, err, 13);
        }
    } else if (warp >= 8 && warp < 12) {
        // ---------------- producers: widen weight codes to fp16 ----------------
        const int pt = tid - 256;  // weight row of the tile
        uint32_t g = 0, slot_base = 0;
        for (int t = blockIdx.x; t < T && !*abort_flag; t += gridDim.x) {
            bool ok = true;
            for (int j = 0; j < nb && ok; j++, g++) {
                const int st = g % NS;
                const uint32_t u = g / NS;
                if (u && !tc::mbar_wait(&sempty[st], (u - 1) & 1, abort_flag, err, 14)) { ok = false; break; }
                const int bb = blk_byte<FMT>(j);
                const uint32_t sc = slot_base + bb / 64;
                const int s = sc % RC;
                const bool first = (bb % 64 == 0) && (FMT != GPU_FMT_TQ2 || (j & 1) == 0);
                const bool last = ((bb + blk_span<FMT>()) % 64 == 0 && (FMT != GPU_FMT_TQ2 || (j & 1) == 1)) || j == nb - 1;
                if (first && !tc::mbar_wait(&cfull[s], (sc / RC) & 1, abort_flag, err, 4)) { ok = false; break; }
                uint4 w[4];
                widen_row<FMT>(ring + s * SLOT + pt * 64 + bb % 64, j, w);
                if (last) {
                    // Release the slot to the TMA only once this thread's shared loads of it
                    // have returned (consume their values) and are ordered before the async
                    // proxy's refill: an arrive alone lets an L2-fast TMA overwrite the slot
                    // under loads still in flight.
                    asm volatile("" ::"r"(w[0].x), "r"(w[3].w) : "memory");
                    tc::fence_proxy_async();
                    tc::mbar_arrive(&cempty[s]);
                }
                uint8_t *sa = stages + st * A_BYTES + (pt >> 3) * 512 + (pt & 7) * 16;
#pragma unroll
                for (int k = 0; k < 4; k++) *reinterpret_cast<uint4 *>(sa + k * 128) = w[k];
                tc::fence_proxy_async();
                tc::mbar_arrive(&sfull[st]);
            }
            slot_base += nslots;
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
                for (int j = 0; j < nb; j++, g++) {
                    const int s = g % NS, bs = g % RB, ac = g % NACC;
                    if (!tc::mbar_wait(&sfull[s], (g / NS) & 1, abort_flag, err, 5)) { ok = false; break; }
                    if (!tc::mbar_wait(&bfull[bs], (g / RB) & 1, abort_flag, err, 15)) { ok = false; break; }
                    if (g >= NACC && !tc::mbar_wait(&tempty[ac], ((g / NACC) - 1) & 1, abort_flag, err, 6)) { ok = false; break; }
                    tc::tc_fence_after();
                    const uint32_t sa = tc::smem_u32(stages + s * A_BYTES), sb = tc::smem_u32(bring + bs * B_BYTES);
                    // A: core matrix (row group r, K chunk kc) at r*512 + kc*128, no swizzle
                    // B: 8-row x 64-byte swizzle atoms, 512 bytes apart
                    const uint64_t ad = tc::smem_desc(sa, 128, 512), bd = tc::smem_desc_sw64(sb, 512);
                    const uint32_t td = tbase + ac * BN;
                    tc::mma_f16_ss(td, ad, bd, idesc, 0u);                             // k 0-15 (overwrite)
                    tc::mma_f16_ss(td, ad + (256 >> 4), bd + (32 >> 4), idesc, 1u);  // k 16-31
                    tc::mma_commit(&sempty[s]);   // A stage free once these MMAs complete
                    tc::mma_commit(&bempty[bs]);  // B slot likewise
                    tc::mma_commit(&tfull[ac]);
                }
            }
            if (g) tc::mbar_wait(&tfull[(g - 1) % NACC], ((g - 1) / NACC) & 1, abort_flag, err, 7);
        }
    } else {
        // ---------------- epilogue (warps 0-7) ----------------
        const int q = warp & 3, h = warp >> 2;
        const int m = q * 32 + lane;  // tile row = TMEM lane
        uint32_t g = 0;
        for (int t = blockIdx.x; t < T; t += gridDim.x) {
            TcTile tl = tc_tile(a, t, MT);
            const int ncols = tl.it.count;
            const bool cv = h * 32 < ncols;  // this warp's 32 columns hold tokens
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
            const __half *dwrow = nullptr;
            if (FMT != GPU_FMT_TQ2)
                dwrow = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(a.scale) +
                                                         (long)tl.it.group * a.scale_gstride) +
                        (size_t)(tl.m0 + m) * nbp;
            float2 acc[16];
#pragma unroll
            for (int i = 0; i < 16; i++) acc[i] = make_float2(0.f, 0.f);
            const uint32_t tl_lane = (uint32_t)(q * 32) << 16;
            // Software pipeline over the K blocks: the TMEM load of block j+1 is in flight
            // while block j is scaled into the accumulators (two register buffers).
            uint32_t va_[32], vb_[32];
            auto fetch = [&](uint32_t gg, uint32_t (&v)[32]) -> bool {
                bool ok = tc::mbar_wait(&tfull[gg % NACC], (gg / NACC) & 1, abort_flag, err, 8);
                ok = ok && tc::mbar_wait(&dfull[gg % NDX], (gg / NDX) & 1, abort_flag, err, 9);
                ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
                tc::tc_fence_after();
                if (ok && cv) tc::tmem_ld32(tbase + tl_lane + (gg % NACC) * BN + h * 32, v);
                return ok;
            };
            float dw_next = (FMT != GPU_FMT_TQ2) ? __half2float(dwrow[0]) : 1.f;
            bool okc = fetch(g, va_);
            // one K block: results of block j are in `cur`; block j+1 is fetched into `nxt`
            auto step = [&](int j, uint32_t (&cur)[32], uint32_t (&nxt)[32]) {
                const int ac = g % NACC, ds = g % NDX;
                const float dw = dw_next;
                if (FMT != GPU_FMT_TQ2 && j + 1 < nb) dw_next = __half2float(dwrow[j + 1]);
                if (okc && cv) tc::tmem_ld_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty[ac]);  // accumulator j is in registers
                bool okn = true;
                if (j + 1 < nb) okn = fetch(g + 1, nxt);
                if (okc && cv) {
                    const float *dx = reinterpret_cast<const float *>(dxring + ds * DX_BYTES) + h * 32;
                    const float2 dw2 = make_float2(dw, dw);
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        float4 d4 = *reinterpret_cast<const float4 *>(dx + 4 * i);
                        float2 x0 = make_float2(__uint_as_float(cur[4 * i]), __uint_as_float(cur[4 * i + 1]));
                        float2 x1 = make_float2(__uint_as_float(cur[4 * i + 2]), __uint_as_float(cur[4 * i + 3]));
                        float2 da = make_float2(d4.x, d4.y), db = make_float2(d4.z, d4.w);
                        if (FMT != GPU_FMT_TQ2) { da = fmul2(dw2, da); db = fmul2(dw2, db); }
                        acc[2 * i] = ffma2(da, x0, acc[2 * i]);
                        acc[2 * i + 1] = ffma2(db, x1, acc[2 * i + 1]);
                    }
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&dempty[ds]);
                okc = okn;
                g++;
            };
#pragma unroll 1
            for (int j = 0; j < nb; j += 2) {
                step(j, va_, vb_);
                if (j + 1 < nb) step(j + 1, vb_, va_);
            }
            // ---- tile output: 128 x ncols fp32 through shared memory ----
            const float *alpha = FMT == GPU_FMT_TQ2 ? reinterpret_cast<const float *>(
                                                          reinterpret_cast<const uint8_t *>(a.scale) +
                                                          (long)tl.it.group * a.scale_gstride)
                                                    : nullptr;
            const int m0 = tl.m0;
            {
                const int c0n = 0, nc = ncols;
#pragma unroll
                for (int i = 0; i < 16; i++) *reinterpret_cast<float2 *>(ct + m * CS + h * 32 + 2 * i) = acc[i];
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
        }
    }
#ifdef ZZ_TC_PROF
    if (blockIdx.x == 0 && (tid & 31) == 0) atomicAdd(&tc::g_tc_prof[20 + (warp < 8 ? 0 : warp < 12 ? 1 : warp - 10)], (unsigned long long)clock64());
#endif
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 13) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tbase, NACC * tcm::BN);
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

// codes plane of a whole bank: rows = experts * O, row = row_bytes bytes
static int make_codes_map(CUtensorMap *map, const uint8_t *codes, long rows, int row_bytes) {
    if (!get_encode()) return 0;
    if ((uintptr_t)codes & 15 || row_bytes % 16) return fail("tc: codes plane not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(codes), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("tc: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return 1;
}

// pair-ordered fp16 activation rows [rows, I] seen as (8 halves) x rows x (I/8 chunks),
// so one box {8, 128, 4} lands a block's 128 x 32 tile as K-major core matrices
static int make_b_map(CUtensorMap *map, const __half *xg, int rows, int I, int box_rows) {
    if (!get_encode()) return 0;
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
    CUtensorMap map;
    BMaps bmaps;
    if (!make_codes_map(&map, a.codes, (long)n_groups * a.O, row_bytes)) return 0;
    for (int i = 0; i < 3; i++)
        if (!make_b_map(&bmaps.m[i], a.xg, a.rows_cap, a.I, 16 << i)) return 0;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (const char *e = getenv("ZZ_TC_GRID")) sms = atoi(e) > 0 ? atoi(e) : sms;
    k_moe_tc<FMT, EPI><<<sms, tcm::NTHREADS, tcm::SMEM, st>>>(a, map, bmaps, err);
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
    cudaMemcpyFromSymbol(out, zz::tc::g_tc_prof, sizeof(unsigned long long) * 32);
    unsigned long long z[32] = {0};
    cudaMemcpyToSymbol(zz::tc::g_tc_prof, z, sizeof z);
    return 1;
}
#endif
