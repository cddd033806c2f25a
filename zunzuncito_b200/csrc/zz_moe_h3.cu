// zz_moe_h3.cu -- the batch-union expert GEMMs over q4_0 banks on the 5th-generation
// tensor cores with the block scales folded into fp16 operands (tcgen05.mma kind::f16,
// f32 accumulators in TMEM), so the whole K reduction of a tile stays in TMEM.
//
// C[o, n] = sum_b dw[o,b] * dx[n,b] * I_b[o,n]   (q40.h:20-31, gemma4.c:618-654)
//         = sum_k A[o,k] * B[n,k],  A = dw * (q - 8),  B = dx * x
//
// The block scales vary along both o and n, so an int8 MMA has to hand every 32-wide
// block's integer sum to an epilogue that scales it (one TMEM round trip per block).
// Folding the scales into the operands instead makes the product a plain dense
// contraction, but A and B are then real numbers that fp16 cannot hold exactly:
//   A = dw * (q - 8): dw is fp16 (11 significant bits) and |q - 8| <= 8, so the product
//       has at most 14 significant bits. A_hi = fp16(A) (one rounded hmul2) and
//       A_lo = A - A_hi (one hfma2, exact: the remainder has at most 3 bits) hold it
//       exactly (up to fp16 subnormal spacing, 2^-24, for tiny scales).
//   B = dx * x: dx is an f32 activation scale, so B is rounded to f32 first, then
//       B_hi = fp16(B), B_lo = fp16(B - B_hi): 22 significant bits.
// Three products per 16-wide K step give every product to a relative 2^-21 (the dropped
// A_lo B_lo term is below 2^-22 of it). They take two MMAs: B_hi and B_lo sit in shared
// memory as one operand of 2 x np2 rows, so A_hi x [B_hi; B_lo] writes the main sums
// (A_hi B_hi) and the cross sums (A_hi B_lo) side by side, and A_lo x B_hi adds into the
// cross columns. The tensor core's f32 accumulation truncates, so no TMEM sum spans more
// than a chunk of CH stages: the epilogue warps add each chunk's main + cross sums into
// f32 registers with round-to-nearest while the tensor core fills the other of two chunk
// buffers (a single TMEM sum over K = 2816 biased |h| low by 6e-6 on average). Operand
// range: |B| < 65504 (an activation block whose absolute maximum reaches the fp16 range
// sets the error word, code 40).
//
// B is formed once per layer call: k_split_rows writes each pair row's hi and lo planes
// (gate/up), and the gate/up epilogue writes the down GEMM's planes of the requantized
// hidden rows next to hq / hs. The weight side is converted per tile from the q4_0
// planes, so HBM still carries 18 bytes per 32 weights.
//
// Persistent, warp-specialised, one CTA per SM (480 threads); work tiles are (item,
// 128 weight rows), items being (expert, <= 64 routed rows) listed by the router in
// decreasing row count. K advances in stages of 64 weights (two blocks):
//   warps 0-3   epilogue: thread = TMEM lane = weight row; per chunk the f32 sums, at the
//               tile end through shared memory to the fused GeGLU / SwiGLU + q8_0 requant
//               (bit-exact with q40_quant_act) or the weighted scatter-add into OUT
//   warps 4-11  A producers, two per TMEM lane quarter: thread r of warp set hb takes
//               block hb of each stage of weight row m0 + r from the code slot, converts
//               it to A_hi and A_lo and writes them into TMEM lane r (tcgen05.st)
//   warp 12     TMA: the stage's B_hi and B_lo boxes (128 bytes x np2 rows, swizzled)
//   warp 13     MMA: one elected lane issues 2 x 4 tcgen05.mma kind::f16 per stage (M = 128,
//               N = 2 np2 and np2, K = 16)
//   warp 14     TMA: the weight codes (128 rows x 128 bytes, swizzled: 4 stages) and their
//               fp16 block scales into a ring of RC slots
// Every wait is bounded (2 s of %globaltimer); one that runs out sets the kernel's error
// word and the CTA drains (copies and MMAs in flight, bounded by time only), frees its
// TMEM and returns.
//
// Measured (B200, Gemma-4 layer, 128 q4_0 experts): parity with the oracle at every
// benched shape; S = 4096 layer 1.98 ms, the same as the int8 mma.sync engine with 64-row
// items (down GEMM 18% faster, gate/up 5% slower, plus the per-layer split of B), S = 512
// 0.45 against 0.35 ms. What sets the pace (profiles/, the MMA-chain microbenchmark): the
// MMA issue sequence must be a fixed, unrolled run per stage (a loop with a run-time trip
// count costs 3.5x per MMA), issued by a whole warp with one elected lane; what remains
// is the pipeline's own hand-offs between roles. It stays opt-in (ZZ_MOE_KERNEL=h3).
#include <cuda.h>
#include <cudaTypedefs.h>
#include "zz_gemm.cuh"
#include "zz_tc.cuh"

namespace zz {

namespace h3k {
constexpr int NTHREADS = 480;
constexpr int BN = 64;                  // max routed rows per tile
constexpr int PART = BN * 128;          // one B part: 64 rows x 128 bytes (64 fp16)
constexpr int NS = 4;                   // A stages (TMEM)
constexpr int NB = 4;                   // B stages (shared memory; 8 measured slower)
constexpr int B_STAGE = 2 * PART;       // [B_hi; B_lo], np2 rows each
constexpr int RC = 3;                   // code / scale slots of 4 stages (TMA)
constexpr int C_SLOT = 128 * 128;       // 128 weight rows x 128 code bytes (256 weights)
constexpr int W_SLOT = 128 * 16;        // their 8 fp16 block scales per row
constexpr int CTX = 33;                 // tile-end exchange: 128 rows x 32 columns, padded
constexpr int CT_BYTES = 128 * CTX * 4;
constexpr int OFF_B = 0;                // 1 KB aligned (swizzled operands and boxes)
constexpr int OFF_C = OFF_B + NB * B_STAGE;
constexpr int OFF_W = OFF_C + RC * C_SLOT;
constexpr int OFF_CT = OFF_W + RC * W_SLOT;
constexpr int OFF_BAR = OFF_CT + CT_BYTES;
constexpr int NBAR = 2 * NS + 2 * NB + 2 * RC + 2 * 2 + 1;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + slack to align the base to 1 KB
static_assert(SMEM <= 232448, "shared memory");
// TMEM columns: two chunk buffers of 2 BN columns (a chunk's sums are [main (np2) | cross
// (np2)]), then NS stages of A (64 weights: 32 columns of A_hi pairs, 32 of A_lo pairs)
constexpr int SBUF = 2 * BN, TM_A = 2 * SBUF, A_COLS = 64;
constexpr int TMEM_COLS = 512;
static_assert(TM_A + NS * A_COLS <= TMEM_COLS, "TMEM columns");
constexpr int CH = 4;                   // stages per TMEM sum (16 K steps of 16)
constexpr int WARP_TMA = 12, WARP_MMA = 13, WARP_CODE = 14;
}  // namespace h3k

// fp16 pair -> (hi, lo) with hi = fp16(v * s), lo = fp16(v * s - hi) exactly
__device__ __forceinline__ void split_h2(uint32_t v, __half2 s, uint32_t &hi, uint32_t &lo) {
    const __half2 x = *reinterpret_cast<const __half2 *>(&v);
    const __half2 h = __hmul2(x, s);
    const __half2 l = __hfma2(x, s, __hneg2(h));
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// f32 pair -> fp16 hi = fp16(p), lo = fp16(p - hi)
__device__ __forceinline__ void split_f2(float2 p, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __float22half2_rn(p);
    const float2 hb = __half22float2(h);
    const __half2 l = __float22half2_rn(make_float2(p.x - hb.x, p.y - hb.y));
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled K-major part
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// B operand planes of the gate/up GEMM: pair row r (token pair_src[r] / K) as fp16 hi and
// lo of dx * x, one warp per row, 16 codes per lane step. Rows of no pair are left as they
// are (no tile reads them).
__global__ void __launch_bounds__(256) k_split_rows(const int *__restrict__ pair_src, int K,
                                                   const int8_t *__restrict__ xq, const float *__restrict__ xs,
                                                   int D, int cap, __half *__restrict__ xhs, int *err) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= cap) return;
    const int src = pair_src[r];
    if (src < 0) return;
    const int tok = src / K, nb = D / 32;
    const int8_t *x = xq + (size_t)tok * D;
    __half *hi = xhs + (size_t)r * D, *lo = xhs + (size_t)cap * D + (size_t)r * D;
    bool big = false;
    for (int c = lane; c < D / 16; c += 32) {
        const uint4 w = *reinterpret_cast<const uint4 *>(x + 16 * c);
        const float dx = xs[(size_t)tok * nb + c / 2];
        big |= dx * 127.f >= 65504.f;
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        uint32_t H[8], L[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t p = s8_h2(__byte_perm(ww[i], 0u, h ? 0x4342u : 0x4140u));
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&p));
                split_f2(make_float2(f.x * dx, f.y * dx), H[2 * i + h], L[2 * i + h]);
            }
        }
        reinterpret_cast<uint4 *>(hi + 16 * c)[0] = make_uint4(H[0], H[1], H[2], H[3]);
        reinterpret_cast<uint4 *>(hi + 16 * c)[1] = make_uint4(H[4], H[5], H[6], H[7]);
        reinterpret_cast<uint4 *>(lo + 16 * c)[0] = make_uint4(L[0], L[1], L[2], L[3]);
        reinterpret_cast<uint4 *>(lo + 16 * c)[1] = make_uint4(L[4], L[5], L[6], L[7]);
    }
    if (big) atomicCAS(err, 0, 40);
}

struct BMapsH {
    CUtensorMap hi[3], lo[3];  // 128-byte (64 fp16) boxes of 16, 32, 64 rows
};

__device__ __forceinline__ int np2_rows(int count) {
    const int N = (count + 15) & ~15;
    return N <= 16 ? 16 : N <= 32 ? 32 : 64;
}

template <int EPI>
__global__ void __launch_bounds__(h3k::NTHREADS, 1)
    k_moe_h3(const GemmArgs a, const __grid_constant__ BMapsH bmaps, const __grid_constant__ CUtensorMap codes_map,
             const __grid_constant__ CUtensorMap scale_map, int *err) {
    using namespace h3k;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    // an A stage is full when the 8 producer warps have written it, a B stage when its
    // copies have landed; both are empty when the stage's MMAs are done
    uint64_t *opfull = bars, *opempty = opfull + NS, *bfull = opempty + NS, *bempty = bfull + NB;
    uint64_t *sfull = bempty + NB, *sempty = sfull + 2, *drain = sempty + 2;
    // a code slot (4 stages of 128 weight rows) is full when its two boxes have landed,
    // empty when the 8 producer warps have read it
    uint64_t *cfull = drain + 1, *cempty = cfull + RC;
    uint32_t *tmem_base_smem = reinterpret_cast<uint32_t *>(smem + OFF_BAR + NBAR * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + NBAR * 8 + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = a.I / ZZ_BLK, nss = (nb + 1) / 2, MT = a.O / 128;
    const int T = *a.n_items * MT;

    if (tid == 0) {
        for (int i = 0; i < NS; i++) { tc::mbar_init(&opfull[i], 8); tc::mbar_init(&opempty[i], 1); }
        for (int i = 0; i < NB; i++) { tc::mbar_init(&bfull[i], 1); tc::mbar_init(&bempty[i], 1); }
        for (int i = 0; i < 2; i++) { tc::mbar_init(&sfull[i], 1); tc::mbar_init(&sempty[i], 4); }
        tc::mbar_init(drain, 1);
        for (int i = 0; i < RC; i++) { tc::mbar_init(&cfull[i], 1); tc::mbar_init(&cempty[i], 8); }
        *abort_flag = 0;
        tc::mbar_init_fence();
    }
    if (warp == WARP_MMA) tc::tmem_alloc(tmem_base_smem, TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tbase = *tmem_base_smem;
    TC_PROF_T(prof_t0);

    if (warp == WARP_MMA) {
        // ---------------- MMA issue: the whole warp runs the loop, one elected lane issues ----------------
        uint32_t g = 0, gc = 0;
        bool ok = true;
        const uint32_t sB = tc::smem_u32(smem + OFF_B);
        for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
            const WorkItem it = a.items[t / MT];
            const int np2 = np2_rows(it.count);
            // [B_hi; B_lo] as one operand of 2 np2 rows: main and cross columns together
            const uint32_t idesc2 = tc::idesc_f16(128, 2 * np2), idesc1 = tc::idesc_f16(128, np2);
            for (int ss = 0; ss < nss; ss++, g++) {
                const int st = g % NS, sb = g % NB, db = gc & 1;
                const bool first = ss % CH == 0, last = ss % CH == CH - 1 || ss == nss - 1;
                if (!tc::mbar_wait_spin(&opfull[st], (g / NS) & 1, abort_flag, err, 32)) ok = false;
                if (ok && !tc::mbar_wait_spin(&bfull[sb], (g / NB) & 1, abort_flag, err, 33)) ok = false;
                // the epilogue has taken chunk gc - 2's sums out of this buffer
                if (ok && first && gc >= 2 && !tc::mbar_wait_spin(&sempty[db], ((gc >> 1) - 1) & 1, abort_flag, err, 31))
                    ok = false;
                if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                tc::tc_fence_after();
                const uint32_t ah = tbase + (uint32_t)(TM_A + st * A_COLS);
                const uint32_t dm = tbase + (uint32_t)(db * SBUF), dc = dm + (uint32_t)np2;
                // a 32-byte K step advances the descriptor's start address field by 2
                const uint64_t bd = tc::smem_desc_sw128(sB + sb * B_STAGE);
                // K is a multiple of 64 (launch_moe_h3), so every stage has 4 K steps: a fixed,
                // fully unrolled sequence of 8 MMAs issues back to back (a loop with a run-time
                // trip count measured 3.5x slower per MMA, tc_f16_chain.cu)
                TC_PROF_T(p_mma);
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    tc::mma_f16_ts_warp(dm, ah + 8 * kk, bd + 2 * kk, idesc2, !(first && kk == 0));  // A_hi B_hi | A_hi B_lo
                    tc::mma_f16_ts_warp(dc, ah + 32 + 8 * kk, bd + 2 * kk, idesc1, 1);               // + A_lo B_hi (cross)
                }
                TC_PROF_ADD(50, p_mma);
                TC_PROF_T(p_cmt);
                tc::mma_commit_warp(&opempty[st]);  // the stages are free once these MMAs complete
                tc::mma_commit_warp(&bempty[sb]);
                if (last) {
                    tc::mma_commit_warp(&sfull[db]);  // the chunk's sums are ready
                    gc++;
                }
                TC_PROF_ADD(51, p_cmt);
            }
        }
        // every MMA issued has completed before TMEM may be freed (bounded, whatever the
        // abort flag says)
        tc::mma_commit_warp(drain);
        tc::mbar_drain(drain, 0);
    } else if (warp == WARP_TMA) {
        // ---------------- TMA: [B_hi; B_lo] of the item's rows, np2 rows each ----------------
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < T && ok && !*abort_flag; t += gridDim.x) {
                const WorkItem it = a.items[t / MT];
                const int np2 = np2_rows(it.count), sel = np2 == 16 ? 0 : np2 == 32 ? 1 : 2;
                for (int ss = 0; ss < nss; ss++, g++) {
                    const int st = g % NB;
                    if (g >= NB && !tc::mbar_wait_spin(&bempty[st], ((g / NB) - 1) & 1, abort_flag, err, 37)) { ok = false; break; }
                    tc::mbar_arrive_tx(&bfull[st], 2u * (uint32_t)np2 * 128u);
                    uint8_t *dst = smem + OFF_B + st * B_STAGE, *dlo = dst + np2 * 128;
                    const int x = ss * 128;  // bytes: 64 fp16 per stage
                    // the maps are named with constant indices so they stay in parameter space
                    switch (sel) {
                        case 0: tc::tma_load_2d(dst, &bmaps.hi[0], x, it.row0, &bfull[st]);
                                tc::tma_load_2d(dlo, &bmaps.lo[0], x, it.row0, &bfull[st]); break;
                        case 1: tc::tma_load_2d(dst, &bmaps.hi[1], x, it.row0, &bfull[st]);
                                tc::tma_load_2d(dlo, &bmaps.lo[1], x, it.row0, &bfull[st]); break;
                        default: tc::tma_load_2d(dst, &bmaps.hi[2], x, it.row0, &bfull[st]);
                                 tc::tma_load_2d(dlo, &bmaps.lo[2], x, it.row0, &bfull[st]); break;
                    }
                }
            }
            // the last copies land before the CTA may exit
            // (bounded by time only: after an abort the copies still land in this CTA's memory)
            // (each slot's latest use)
            for (uint32_t k = g > (uint32_t)NB ? g - NB : 0; k < g; k++) tc::mbar_drain(&bfull[k % NB], (k / NB) & 1);
        }
    } else if (warp == WARP_CODE) {
        // ---------------- TMA: weight codes and block scales, 4 stages per slot ----------------
        if (lane == 0) {
            uint32_t gq = 0;
            bool ok = true;
            const int ng = (nss + 3) / 4;
            for (int t = blockIdx.x; t < T && ok && !*abort_flag; t += gridDim.x) {
                const WorkItem it = a.items[t / MT];
                const int m0 = (t % MT) * 128, y = it.group * a.O + m0;
                for (int q = 0; q < ng; q++, gq++) {
                    const int c = gq % RC;
                    if (gq >= RC && !tc::mbar_wait_spin(&cempty[c], ((gq / RC) - 1) & 1, abort_flag, err, 39)) { ok = false; break; }
                    tc::mbar_arrive_tx(&cfull[c], C_SLOT + W_SLOT);
                    tc::tma_load_2d(smem + OFF_C + c * C_SLOT, &codes_map, q * 128, y, &cfull[c]);
                    tc::tma_load_3d(smem + OFF_W + c * W_SLOT, &scale_map, q * 8, m0, it.group, &cfull[c]);
                }
            }
            // the last copies land before the CTA may exit (bounded by time only)
            for (uint32_t k = gq > (uint32_t)RC ? gq - RC : 0; k < gq; k++) tc::mbar_drain(&cfull[k % RC], (k / RC) & 1);
        }
    } else if (warp >= 4) {
        // ---------------- A producers: weight row m0 + r -> A_hi, A_lo in TMEM lane r ----------------
        // warps 4-7 take the stage's first 32-weight block, warps 8-11 the second, so each SM
        // sub-partition runs two independent producer chains
        const int r = (warp & 3) * 32 + lane;      // TMEM lane (warp % 4 selects the lane quarter)
        const int hb = (warp - 4) >> 2;            // block of the stage
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        uint32_t g = 0, gq = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < T && ok; t += gridDim.x) {
            for (int ss = 0; ss < nss && ok; ss++, g++) {
                const int j = ss & 3, c = gq % RC, st = g % NS;
                if (j == 0) ok = tc::mbar_wait_spin(&cfull[c], (gq / RC) & 1, abort_flag, err, 30);
                // this row's 16 code bytes of block 2 ss + hb (128-byte swizzled box) and the
                // stage's two fp16 scales
                const uint8_t *cs = smem + OFF_C + c * C_SLOT + r * 128;
                const uint4 w = *reinterpret_cast<const uint4 *>(cs + (((2 * j + hb) ^ (r & 7)) << 4));
                const uint32_t sc = *reinterpret_cast<const uint32_t *>(smem + OFF_W + c * W_SLOT + r * 16 + 4 * j);
                if (j == 3 || ss == nss - 1) {
                    // the slot's last stage is read: hand it back to the copy warp
                    asm volatile("" ::"r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w), "r"(sc) : "memory");
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&cempty[c]);
                    gq++;
                }
                const __half2 hs2 = *reinterpret_cast<const __half2 *>(&sc);
                // q4_0: byte i holds k = i (low nibble) and k = i + 16 (high)
                const __half2 s = hb ? __high2half2(hs2) : __low2half2(hs2);
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
                uint32_t H[16], L[16];  // the block's 32 values in k order, as fp16 pairs
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint32_t p01 = __byte_perm(ww[i], 0u, 0x4140u), p23 = __byte_perm(ww[i], 0u, 0x4342u);
                    split_h2(q4lo_h2(p01), s, H[2 * i], L[2 * i]);
                    split_h2(q4lo_h2(p23), s, H[2 * i + 1], L[2 * i + 1]);
                    split_h2(q4hi_h2(p01), s, H[8 + 2 * i], L[8 + 2 * i]);
                    split_h2(q4hi_h2(p23), s, H[8 + 2 * i + 1], L[8 + 2 * i + 1]);
                }
                // the TMEM stage is free once the MMAs of stage g - NS have completed
                if (ok && g >= NS && !tc::mbar_wait_spin(&opempty[st], ((g / NS) - 1) & 1, abort_flag, err, 34)) ok = false;
                ok = __all_sync(0xffffffffu, ok);  // tcgen05.st is warp-collective
                if (!ok) break;
                tc::tc_fence_after();
                const uint32_t ta = tbase + lane_base + (uint32_t)(TM_A + st * A_COLS + 16 * hb);
                tc::tmem_st16(ta, H);
                tc::tmem_st16(ta + 32, L);
                tc::tmem_st_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&opfull[st]);
            }
        }
    } else {
        // ---------------- epilogue (warps 0-3): per-stage sums into f32 registers ----------------
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float *ct = reinterpret_cast<float *>(smem + OFF_CT);
        uint32_t gc = 0;
        for (int t = blockIdx.x; t < T; t += gridDim.x) {
            const WorkItem it = a.items[t / MT];
            const int m0 = (t % MT) * 128;
            const int ncols = it.count, np2 = np2_rows(ncols);
            // this thread's row (TMEM lane) of the tile, one f32 sum per column: each chunk's
            // main + cross sums added with round-to-nearest (the tensor core's own adds
            // truncate, so no TMEM sum spans more than one chunk of CH stages)
            float acc[BN];
#pragma unroll
            for (int i = 0; i < BN; i++) acc[i] = 0.f;
            bool ok = true;
            for (int ch = 0; ch < (nss + CH - 1) / CH; ch++, gc++) {
                const int db = gc & 1;
                bool got = tc::mbar_wait(&sfull[db], (gc >> 1) & 1, abort_flag, err, 36);
                got = __all_sync(0xffffffffu, got);  // tcgen05.ld is warp-collective
                ok = ok && got;
                tc::tc_fence_after();
                if (got) {
                    const uint32_t ta = tbase + lane_base + (uint32_t)(db * SBUF);
#pragma unroll
                    for (int c16 = 0; c16 < BN / 16; c16++) {
                        if (16 * c16 < np2) {
                            uint32_t v[16], x[16];
                            tc::tmem_ld16(ta + 16 * c16, v);
                            tc::tmem_ld16(ta + np2 + 16 * c16, x);
                            tc::tmem_ld_wait();
#pragma unroll
                            for (int i = 0; i < 16; i++) acc[16 * c16 + i] += __uint_as_float(v[i]) + __uint_as_float(x[i]);
                        }
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&sempty[db]);
            }
            // tile end, 32 columns at a time through shared memory
#pragma unroll
            for (int hc = 0; hc < BN / 32; hc++) {
                if (32 * hc >= ncols) break;
#pragma unroll
                for (int i = 0; i < 32; i++) ct[(warp * 32 + lane) * CTX + i] = acc[32 * hc + i];
                tc::named_sync(1, 128);
                if (ok && !*abort_flag) {
                    if (EPI == EPI_GATEUP) {
                        // rows 0-63 gate and 64-127 up of the same 64 features; thread = (block qb
                        // of 32 features, column): h = act(gate, up), then the q8_0 block
                        // (q40.h:124-138), and the down GEMM's fp16 planes of d * q
                        // a thread pair per (32-feature block qb, column): 16 features each, the
                        // block's absolute maximum combined with one shuffle (the same value)
                        const int MI = a.O / 2, nbh = MI / 32, f0 = (m0 / 128) * 64;
                        const int half = tid & 1, n = (tid >> 1) & 31, qb = tid >> 6, col = 32 * hc + n;
                        const bool act_ok = col < ncols;
                        const size_t pr = (size_t)(it.row0 + (act_ok ? col : 0));
                        float hv[16];
                        float amax = 0.f;
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const int fl = 32 * qb + 16 * half + j;
                            hv[j] = gated_act(a.act, ct[fl * CTX + n], ct[(64 + fl) * CTX + n], a.clamp);
                            amax = fmaxf(amax, fabsf(hv[j]));
                        }
                        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                        if (act_ok) {
                            const float d = __fdiv_rn(amax, 127.0f);
                            const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
                            uint32_t wq[4], H[8], L[8];
#pragma unroll
                            for (int j4 = 0; j4 < 4; j4++) {
                                uint32_t word = 0;
                                int qv[4];
#pragma unroll
                                for (int k = 0; k < 4; k++) {
                                    qv[k] = __float2int_rn(__fmul_rn(hv[4 * j4 + k], id));
                                    qv[k] = qv[k] < -127 ? -127 : (qv[k] > 127 ? 127 : qv[k]);
                                    word |= (uint32_t)(qv[k] & 0xFF) << (8 * k);
                                }
                                wq[j4] = word;
                                split_f2(make_float2((float)qv[0] * d, (float)qv[1] * d), H[2 * j4], L[2 * j4]);
                                split_f2(make_float2((float)qv[2] * d, (float)qv[3] * d), H[2 * j4 + 1], L[2 * j4 + 1]);
                            }
                            const int f = f0 + 32 * qb + 16 * half;
                            *reinterpret_cast<uint4 *>(a.hq + pr * MI + f) = make_uint4(wq[0], wq[1], wq[2], wq[3]);
                            uint4 *dh = reinterpret_cast<uint4 *>(a.hhs + pr * MI + f);
                            uint4 *dl = reinterpret_cast<uint4 *>(a.hhs + (size_t)a.rows_cap * MI + pr * MI + f);
                            dh[0] = make_uint4(H[0], H[1], H[2], H[3]);
                            dh[1] = make_uint4(H[4], H[5], H[6], H[7]);
                            dl[0] = make_uint4(L[0], L[1], L[2], L[3]);
                            dl[1] = make_uint4(L[4], L[5], L[6], L[7]);
                            if (half == 0) a.hs[pr * nbh + f0 / 32 + qb] = d;
                        }
                    } else {
                        // OUT[token, m0 + 4 o4 .. + 3] += w * C (each warp instruction covers 512
                        // contiguous bytes of one token's output row)
                        for (int task = tid; task < 32 * 32; task += 128) {
                            const int o4 = task & 31, n = task >> 5, col = 32 * hc + n;
                            if (col >= ncols) break;  // n grows with task
                            const int pr = it.row0 + col;
                            float4 v = make_float4(ct[(4 * o4) * CTX + n], ct[(4 * o4 + 1) * CTX + n],
                                                   ct[(4 * o4 + 2) * CTX + n], ct[(4 * o4 + 3) * CTX + n]);
                            const float wgt = a.pair_w[pr];
                            v.x *= wgt; v.y *= wgt; v.z *= wgt; v.w *= wgt;
                            atomicAdd(reinterpret_cast<float4 *>(a.out + (size_t)(a.pair_src[pr] / a.K) * a.O + m0 + 4 * o4), v);
                        }
                    }
                }
                tc::named_sync(1, 128);
            }
        }
    }
#ifdef ZZ_TC_PROF
    // per-role span from set-up to here: 60 epilogue, 61 producers, 62 TMA, 63 MMA
    if (blockIdx.x == 0 && lane == 0 && (warp == 0 || warp == 4 || warp == WARP_TMA || warp == WARP_MMA))
        atomicAdd(&tc::g_tc_prof[warp == 0 ? 60 : warp == 4 ? 61 : warp == WARP_TMA ? 62 : 63],
                  (unsigned long long)(clock64() - prof_t0));
#endif
    tc::tc_fence_before();
    __syncthreads();
    if (warp == WARP_MMA) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tbase, TMEM_COLS);
    }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode_h3 = nullptr;

// 2-D map over the fp16 plane [rows][I] as bytes, boxes of 128 bytes (64 fp16) x box_rows,
// 128-byte swizzle (the K-major layout the MMA reads)
static int make_plane_map(CUtensorMap *map, const void *base, long rows, long row_bytes, int box_rows) {
    if (!g_encode_h3) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return fail("cuTensorMapEncodeTiled is not available");
        g_encode_h3 = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    if ((uintptr_t)base & 15 || row_bytes % 16) return fail("h3: operand plane not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode_h3(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail("h3: operand tensor map failed (%d)", (int)r);
    return 1;
}

int make_u8_map(CUtensorMap *map, const void *base, long rows, long row_bytes, int box_w, int box_rows,
                const char *what);
int make_scale_map(CUtensorMap *map, const void *scale, int E, int O, int nbp, long gstride);

template <int EPI>
static int launch_h3_t(const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    static bool attr = false;  // per process: the attribute is a property of the function
    if (!attr) {
        if (!check_cuda(cudaFuncSetAttribute(k_moe_h3<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, h3k::SMEM),
                        "h3 smem attribute"))
            return 0;
        attr = true;
    }
    BMapsH maps;
    const long rb = (long)a.I * 2;
    for (int i = 0; i < 3; i++) {
        if (!make_plane_map(&maps.hi[i], a.xhs, a.rows_cap, rb, 16 << i)) return 0;
        if (!make_plane_map(&maps.lo[i], a.xhs + (size_t)a.rows_cap * a.I, a.rows_cap, rb, 16 << i)) return 0;
    }
    CUtensorMap cmap, smap;
    if (!make_u8_map(&cmap, a.codes, (long)n_groups * a.O, a.I / 2, 128, 128, "h3 weight codes")) return 0;
    if (!make_scale_map(&smap, a.scale, n_groups, a.O, ((a.I / ZZ_BLK) + 7) & ~7, a.scale_gstride)) return 0;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    k_moe_h3<EPI><<<sms, h3k::NTHREADS, h3k::SMEM, st>>>(a, maps, cmap, smap, err);
    return check_cuda(cudaGetLastError(), "h3 launch");
}

int launch_split_rows(const int *pair_src, int K, const int8_t *xq, const float *xs, int D, int cap, __half *xhs,
                      int *err, cudaStream_t st) {
    k_split_rows<<<(cap + 7) / 8, 256, 0, st>>>(pair_src, K, xq, xs, D, cap, xhs, err);
    return check_cuda(cudaGetLastError(), "h3 split launch");
}

// Whether the folded-scale fp16 engine takes a layer of this shape: q4_0 banks, weight
// rows in whole 128-row tiles, K in whole 64-weight stages on both GEMMs.
bool moe_h3_supported(int fmt, int D, int MI) {
    // consecutive experts' code planes exactly O * row_bytes apart (one tensor map spans
    // the bank): true for a packed bank when the plane is a multiple of 256 bytes
    return fmt == GPU_FMT_Q40 && (2 * MI) % 128 == 0 && D % 128 == 0 && MI % 64 == 0 &&
           ((long)2 * MI * (D / 2)) % 256 == 0 && ((long)D * (MI / 2)) % 256 == 0;
}

// The expert GEMMs (gate/up with the fused activation + requant, or down with the fused
// scatter-add) over the router's items, folded-scale fp16 operands on tcgen05.
int launch_moe_h3(int epi, const GemmArgs &a, int n_groups, int *err, cudaStream_t st) {
    if (a.O % 128 || a.I % 64 || !a.xhs) return fail("h3: O=%d / I=%d not multiples of 128 / 64", a.O, a.I);
    return epi == EPI_GATEUP ? launch_h3_t<EPI_GATEUP>(a, n_groups, err, st) : launch_h3_t<EPI_DOWN>(a, n_groups, err, st);
}

}  // namespace zz

#ifdef ZZ_TC_PROF
// diagnostic build only: this translation unit's wait-site cycle totals (block 0), read
// and cleared
extern "C" int zz_h3_prof_read(unsigned long long *out) {
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(out, zz::tc::g_tc_prof, sizeof(unsigned long long) * 128);
    unsigned long long z[128] = {0};
    cudaMemcpyToSymbol(zz::tc::g_tc_prof, z, sizeof z);
    return 1;
}
#endif
