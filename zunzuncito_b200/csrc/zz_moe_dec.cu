// zz_moe_dec.cu -- the batch-union expert FFN for small batches (decode): every
// expert item carries at most DEC_C tokens, so the layer is a pair of weight-streaming
// GEMVs rather than GEMMs (one token, 8 experts, 26.8 MB of weights).
//
//   k_dec_gateup  one warp per hidden feature f of an expert item: the gate row and the
//                 up row of f (rows of the interleaved stack) are streamed once with
//                 16-byte loads and dotted (dp4a) against the item's q8_0 token rows held
//                 in registers; lane 0 applies the activation and writes h (fp32).
//   k_dec_down    each CTA first requantizes the item's h rows to q8_0 in shared memory
//                 (bit-exact with q40_quant_act, q40.h:124-138), then one warp per 4
//                 output rows streams the down rows and adds w * y into OUT.
// The per-block integer sums and the fp32 scale order per block are those of the
// decode matvec (zz_gemv.cu), i.e. q40_dot's decomposition (q40.h:162-187).
#include "zz_dot.cuh"
#include "zz_gemm.cuh"

namespace zz {

constexpr int DEC_C = 2;    // max tokens per expert item on this path
constexpr int DEC_NBL = 4;  // max 32-blocks per lane (K <= 4096)

// one 32-weight block of a weight row, loaded once and dotted against several tokens
struct WBlock {
    uint4 w0, w1;
    float scale;
    int sh;
};
template <int FMT>
__device__ __forceinline__ WBlock load_block(const uint8_t *row, int b, const __half *srow) {
    WBlock k;
    if (FMT == GPU_FMT_Q40) {
        k.w0 = ldg_stream(row + (size_t)b * 16);
        k.scale = __half2float(srow[b]);
    } else if (FMT == GPU_FMT_Q80) {
        k.w0 = ldg_stream(row + (size_t)b * 32);
        k.w1 = ldg_stream(row + (size_t)b * 32 + 16);
        k.scale = __half2float(srow[b]);
    } else {
        k.w0 = ldg_stream(row + (size_t)(b >> 1) * 16);
        k.scale = 1.f;
        k.sh = (b & 1) * 4;
    }
    return k;
}
template <int FMT>
__device__ __forceinline__ int block_dot(const WBlock &k, const uint32_t x[8]) {
    if (FMT == GPU_FMT_Q40) return q40_block_dot(k.w0, x);
    if (FMT == GPU_FMT_Q80) return q80_block_dot(k.w0, k.w1, x);
    return tq2_block_dot(k.w0, k.sh, x);
}

__device__ __forceinline__ void load_x8(const int8_t *p, uint32_t x[8]) {
    const uint4 *q = reinterpret_cast<const uint4 *>(p);
    uint4 lo = q[0], hi = q[1];
    x[0] = lo.x; x[1] = lo.y; x[2] = lo.z; x[3] = lo.w;
    x[4] = hi.x; x[5] = hi.y; x[6] = hi.z; x[7] = hi.w;
}

constexpr int DEC_MAX_P = 64;  // pairs of a call on this path (S*K)

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }


// NBL: blocks per lane of a gate/up row, ceil(nb / 32)
// Both decode kernels are bounded to 5 CTAs per SM (<= 51 registers): a Gemma-4 decode
// layer launches 88 x 8 CTAs of each, which then run in one wave (18.5 vs 21.5 us per layer).
template <int FMT, int NBL>
__global__ void __launch_bounds__(256, 5) k_dec_gateup(GemmArgs a, float *__restrict__ hbuf) {
    // the down kernel (a programmatic dependent launch) may start its prefetch now
    griddep_launch_dependents();
    const int item = blockIdx.y;
    if (item >= *a.n_items) return;
    const WorkItem it = a.items[item];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int MI = a.O / 2, D = a.I, nb = D / ZZ_BLK, nbp = (nb + 7) & ~7;
    const int f0 = blockIdx.x * 8 + warp;
    const bool fv = f0 < MI;
    const int f = fv ? f0 : MI - 1;
    const int grp = f / 64, fi = f % 64;
    const int rg = grp * 128 + fi, ru = rg + 64;  // rows of the interleaved gate/up stack
    const int CB = FMT == GPU_FMT_Q40 ? 16 : FMT == GPU_FMT_Q80 ? 32 : 8;
    const uint8_t *codes = a.codes + (long)it.group * a.codes_gstride;
    const uint8_t *grow = codes + (size_t)rg * nb * CB, *urow = codes + (size_t)ru * nb * CB;
    const __half *sc = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(a.scale) +
                                                        (long)it.group * a.scale_gstride);
    const __half *gs = FMT == GPU_FMT_TQ2 ? nullptr : sc + (size_t)rg * nbp;
    const __half *us = FMT == GPU_FMT_TQ2 ? nullptr : sc + (size_t)ru * nbp;
    // both rows' code blocks of this lane are requested first, then the token rows
    WBlock kg[NBL], ku[NBL];
#pragma unroll
    for (int i = 0; i < NBL; i++) {
        const int b = lane + 32 * i;
        if (b < nb) { kg[i] = load_block<FMT>(grow, b, gs); ku[i] = load_block<FMT>(urow, b, us); }
    }
    const int nc = it.count;
    // the item's token rows (q8_0 codes and block scales) staged in shared memory
    __shared__ __align__(16) int8_t xs_q[DEC_C][DEC_NBL * 32 * 32];
    __shared__ float xs_d[DEC_C][DEC_NBL * 32];
    float tot[DEC_C];
#pragma unroll
    for (int c = 0; c < DEC_C; c++) {
        const int tok = c < nc ? a.pair_src[it.row0 + c] / a.K : 0;
        tot[c] = FMT == GPU_FMT_TQ2 && c < nc ? a.xsx[tok] : 0.f;
        if (c < nc) {
            const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const int8_t *>(a.xq) + (size_t)tok * D);
            for (int i = threadIdx.x; i < D / 16; i += blockDim.x) reinterpret_cast<uint4 *>(xs_q[c])[i] = src[i];
            for (int i = threadIdx.x; i < nb; i += blockDim.x) xs_d[c][i] = a.xs[(size_t)tok * nb + i];
        }
    }
    __syncthreads();
    float ag[DEC_C], au[DEC_C];
#pragma unroll
    for (int c = 0; c < DEC_C; c++) ag[c] = au[c] = 0.f;
#pragma unroll
    for (int i = 0; i < NBL; i++) {
        const int b = lane + 32 * i;
        if (b < nb) {
#pragma unroll
            for (int c = 0; c < DEC_C; c++) {
                if (c < nc) {
                    uint32_t x[8];
                    load_x8(&xs_q[c][b * 32], x);
                    const float dx = xs_d[c][b];
                    ag[c] = fmaf(kg[i].scale * dx, (float)block_dot<FMT>(kg[i], x), ag[c]);
                    au[c] = fmaf(ku[i].scale * dx, (float)block_dot<FMT>(ku[i], x), au[c]);
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < DEC_C; c++) {
        float g = warp_sum(ag[c]), u = warp_sum(au[c]);
        if (lane == 0 && c < nc && fv) {
            if (FMT == GPU_FMT_TQ2) {
                const float *alpha = reinterpret_cast<const float *>(sc);
                g = alpha[rg] * (g - tot[c]);
                u = alpha[ru] * (u - tot[c]);
            }
            hbuf[(size_t)(it.row0 + c) * MI + f] = gated_act(a.act, g, u, a.clamp);
        }
    }
}

// NB8: blocks per lane of a down row (8 lanes per row), ceil(nb / 8)
template <int FMT, int NB8>
__global__ void __launch_bounds__(256, 5) k_dec_down(GemmArgs a, const float *__restrict__ hbuf) {
    // Launched as a programmatic dependent of the gate/up kernel: the items (written by
    // the routing kernel, which completed before gate/up started) and this CTA's weight
    // loads proceed while gate/up runs; griddep_wait() then orders every read of the
    // hidden rows, and every write, after gate/up has completed.
    const int item = blockIdx.y;
    if (item >= *a.n_items) { griddep_wait(); return; }
    const WorkItem it = a.items[item];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = a.O, MI = a.I, nb = MI / ZZ_BLK, nbp = (nb + 7) & ~7;
    const int nc = it.count;
    const int CB = FMT == GPU_FMT_Q40 ? 16 : FMT == GPU_FMT_Q80 ? 32 : 8;
    const uint8_t *codes = a.codes + (long)it.group * a.codes_gstride;
    const __half *sc = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(a.scale) +
                                                        (long)it.group * a.scale_gstride);
    // Each warp takes 4 output rows at once, 8 lanes per row: lane l works on row
    // o0 + l/8 and its blocks b = l%8 + 8 i; all of a lane's weight loads are issued
    // here, before the wait for the gate/up kernel (one DRAM round trip per warp,
    // overlapped with gate/up).
    const int rl = lane >> 3, sl = lane & 7;
    const int o = blockIdx.x * 32 + warp * 4 + rl;
    const bool orow = o < D;
    const uint8_t *row = codes + (size_t)(orow ? o : 0) * nb * CB;
    const __half *srow = FMT == GPU_FMT_TQ2 ? nullptr : sc + (size_t)(orow ? o : 0) * nbp;
    WBlock k[NB8];
#pragma unroll
    for (int i = 0; i < NB8; i++) {
        const int b = sl + 8 * i;
        if (orow && b < nb) k[i] = load_block<FMT>(row, b, srow);
    }
    float wt[DEC_C];
    int tok[DEC_C];
#pragma unroll
    for (int c = 0; c < DEC_C; c++) {
        wt[c] = c < nc ? a.pair_w[it.row0 + c] : 0.f;
        tok[c] = c < nc ? a.pair_src[it.row0 + c] / a.K : 0;
    }
    griddep_wait();  // gate/up's hidden rows are complete and visible from here on

    __shared__ __align__(16) int8_t hq_s[DEC_C][DEC_NBL * 32 * 32];
    __shared__ float hs_s[DEC_C][DEC_NBL * 32];
    __shared__ int hb_s[DEC_C][DEC_NBL * 32];
    __shared__ float tot_s[DEC_C];
    // requantize the item's hidden rows (one warp per 32-block); CTA 0 also records
    // hq / hs of the pair rows in the workspace, as the GEMM path does
    for (int w = warp; w < DEC_C * nb; w += 8) {
        const int c = w / nb, b = w % nb;
        if (c >= nc) continue;
        const size_t pr = (size_t)(it.row0 + c);
        float d;
        int8_t q = quant_lane(hbuf[pr * MI + b * 32 + lane], d);
        hq_s[c][b * 32 + lane] = q;
        int s = q;
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
        if (lane == 0) { hs_s[c][b] = d; hb_s[c][b] = s; }
        if (blockIdx.x == 0) {
            a.hq[pr * MI + b * 32 + lane] = q;
            if (lane == 0) a.hs[pr * nb + b] = d;
        }
    }
    __syncthreads();
    if (FMT == GPU_FMT_TQ2 && threadIdx.x < DEC_C) {
        const int c = threadIdx.x;
        double t = 0;
        for (int b = 0; b < nb && c < nc; b++) t += (double)hs_s[c][b] * (double)hb_s[c][b];
        tot_s[c] = (float)t;
    }
    __syncthreads();
    float acc[DEC_C];
#pragma unroll
    for (int c = 0; c < DEC_C; c++) acc[c] = 0.f;
#pragma unroll
    for (int i = 0; i < NB8; i++) {
        const int b = sl + 8 * i;
        if (orow && b < nb) {
#pragma unroll
            for (int c = 0; c < DEC_C; c++) {
                if (c < nc) {
                    uint32_t x[8];
                    load_x8(&hq_s[c][b * 32], x);
                    acc[c] = fmaf(k[i].scale * hs_s[c][b], (float)block_dot<FMT>(k[i], x), acc[c]);
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < DEC_C; c++) {
        float y = acc[c];
#pragma unroll
        for (int m = 4; m > 0; m >>= 1) y += __shfl_xor_sync(0xffffffffu, y, m);
        if (sl == 0 && orow && c < nc) {
            if (FMT == GPU_FMT_TQ2) y = reinterpret_cast<const float *>(sc)[o] * (y - tot_s[c]);
            atomicAdd(a.out + (size_t)tok[c] * D + o, wt[c] * y);
        }
    }
}

// gate/up then down for a decode call (P <= DEC_MAX_P pairs, routed by k_route); hbuf:
// [pair rows][inter] fp32. The down kernel is a programmatic dependent launch of gate/up.
int launch_moe_dec(int fmt, const GemmArgs &gu, const GemmArgs &dn, int P, float *hbuf, cudaStream_t st) {
    const int MI = gu.O / 2, D = dn.O;
    if (P > DEC_MAX_P) return fail("dec: %d pairs exceed the decode path's %d", P, DEC_MAX_P);
    if (gu.I / 32 > DEC_NBL * 32 || dn.I / 32 > DEC_NBL * 32) return fail("dec: K too large for the decode path");
    const int max_items = P > 0 ? P : 1;  // items of <= DEC_C rows: at most one per pair
    dim3 g1((MI + 7) / 8, max_items), g2((D + 31) / 32, max_items);
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg2{};
    cfg2.gridDim = g2; cfg2.blockDim = dim3(256); cfg2.dynamicSmemBytes = 0; cfg2.stream = st;
    cfg2.attrs = pdl; cfg2.numAttrs = 1;
    const int nbl = (gu.I / 32 + 31) / 32, nb8 = (dn.I / 32 + 7) / 8;
    cudaError_t e = cudaSuccess;
#define ZZ_GU(F, N) case N: k_dec_gateup<F, N><<<g1, 256, 0, st>>>(gu, hbuf); break;
#define ZZ_GUS(F) \
    switch (nbl) { ZZ_GU(F, 1) ZZ_GU(F, 2) ZZ_GU(F, 3) ZZ_GU(F, 4) default: return fail("dec: K too large for the decode path"); }
#define ZZ_DN(F, N) case N: e = cudaLaunchKernelEx(&cfg2, k_dec_down<F, N>, dn, (const float *)hbuf); break;
#define ZZ_DNS(F)                                                                                           \
    switch (nb8) {                                                                                          \
        ZZ_DN(F, 1) ZZ_DN(F, 2) ZZ_DN(F, 3) ZZ_DN(F, 4) ZZ_DN(F, 5) ZZ_DN(F, 6) ZZ_DN(F, 7) ZZ_DN(F, 8)     \
        ZZ_DN(F, 9) ZZ_DN(F, 10) ZZ_DN(F, 11) ZZ_DN(F, 12) ZZ_DN(F, 13) ZZ_DN(F, 14) ZZ_DN(F, 15) ZZ_DN(F, 16) \
        default: return fail("dec: K too large for the decode path");                                       \
    }
    if (fmt == GPU_FMT_Q40) {
        ZZ_GUS(GPU_FMT_Q40)
        ZZ_DNS(GPU_FMT_Q40)
    } else if (fmt == GPU_FMT_Q80) {
        ZZ_GUS(GPU_FMT_Q80)
        ZZ_DNS(GPU_FMT_Q80)
    } else {
        ZZ_GUS(GPU_FMT_TQ2)
        ZZ_DNS(GPU_FMT_TQ2)
    }
#undef ZZ_DNS
#undef ZZ_DN
#undef ZZ_GUS
#undef ZZ_GU
    if (!check_cuda(e, "dec down launch")) return 0;
    return check_cuda(cudaGetLastError(), "dec launch");
}

}  // namespace zz
