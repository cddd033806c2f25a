// zz_gemv.cu -- decode (one activation row) matvec for q4_0 / q8_0 / tq2 planes, and
// the per-block integer-sum kernel used for bit-exact parity checks.
//
// HBM-bound by construction: 18 (q4_0) / 34 (q8_0) / 8 (tq2) bytes per 32 weights,
// against 8 dp4a per block. Layout on chip: one warp per weight row; lane l owns the
// blocks b = l, l+32, l+64, ... of EVERY row, so its slice of the quantized activation
// is loaded into registers once and reused for all rows the warp visits. Weight codes
// stream with 16-byte L1-bypassing loads (a warp reads 512 contiguous bytes per step);
// two rows are in flight per warp to cover HBM latency.
#include <cstdlib>
#include "zz_dot.cuh"
#include "zz_tc.cuh"

namespace zz {

// q4_0 / q8_0 decode matvec. NBL = blocks per lane (ceil(nb/32)).
template <int FMT, int NBL>
__global__ void __launch_bounds__(256) k_gemv_q(const uint8_t *__restrict__ codes, const __half *__restrict__ scale,
                                                int O, int I, const int8_t *__restrict__ xq,
                                                const float *__restrict__ sx, float *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int nb = I / ZZ_BLK, nbp = (nb + 7) & ~7;
    const int CB = FMT == GPU_FMT_Q40 ? 16 : 32;
    uint32_t xr[NBL][8];
    float xs[NBL];
#pragma unroll
    for (int i = 0; i < NBL; i++) {
        int b = lane + 32 * i;
        if (b < nb) {
            const uint4 *p = reinterpret_cast<const uint4 *>(xq + (size_t)b * ZZ_BLK);
            uint4 lo = p[0], hi = p[1];
            xr[i][0] = lo.x; xr[i][1] = lo.y; xr[i][2] = lo.z; xr[i][3] = lo.w;
            xr[i][4] = hi.x; xr[i][5] = hi.y; xr[i][6] = hi.z; xr[i][7] = hi.w;
            xs[i] = sx[b];
        } else {
#pragma unroll
            for (int k = 0; k < 8; k++) xr[i][k] = 0;
            xs[i] = 0.f;
        }
    }
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int w0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const size_t rowb = (size_t)nb * CB;
    for (int o = w0 * 2; o < O; o += warps * 2) {
        const bool two = o + 1 < O;
        uint4 wa[NBL], wb[NBL], wa2[NBL], wb2[NBL];
        float da[NBL], db[NBL];
#pragma unroll
        for (int i = 0; i < NBL; i++) {
            int b = lane + 32 * i;
            if (b < nb) {
                const uint8_t *pa = codes + (size_t)o * rowb + (size_t)b * CB;
                wa[i] = ldg_stream(pa);
                if (FMT == GPU_FMT_Q80) wa2[i] = ldg_stream(pa + 16);
                da[i] = __half2float(scale[(size_t)o * nbp + b]);
                if (two) {
                    wb[i] = ldg_stream(pa + rowb);
                    if (FMT == GPU_FMT_Q80) wb2[i] = ldg_stream(pa + rowb + 16);
                    db[i] = __half2float(scale[(size_t)(o + 1) * nbp + b]);
                }
            }
        }
        float acc_a = 0.f, acc_b = 0.f;
#pragma unroll
        for (int i = 0; i < NBL; i++) {
            int b = lane + 32 * i;
            if (b < nb) {
                int sa = FMT == GPU_FMT_Q40 ? q40_block_dot(wa[i], xr[i]) : q80_block_dot(wa[i], wa2[i], xr[i]);
                acc_a = fmaf(da[i] * xs[i], (float)sa, acc_a);
                if (two) {
                    int sb = FMT == GPU_FMT_Q40 ? q40_block_dot(wb[i], xr[i]) : q80_block_dot(wb[i], wb2[i], xr[i]);
                    acc_b = fmaf(db[i] * xs[i], (float)sb, acc_b);
                }
            }
        }
        acc_a = warp_sum(acc_a);
        acc_b = warp_sum(acc_b);
        if (lane == 0) {
            y[o] = acc_a;
            if (two) y[o + 1] = acc_b;
        }
    }
}

// tq2 decode matvec: lane owns 64-weight groups g = lane + 32 i; y = alpha*(acc - Sx)
template <int NGL>
__global__ void __launch_bounds__(256) k_gemv_tq2(const uint8_t *__restrict__ codes, const float *__restrict__ alpha,
                                                  int O, int I, const int8_t *__restrict__ xq,
                                                  const float *__restrict__ sx, const float *__restrict__ sxtot,
                                                  float *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int ng = I / 64;
    uint32_t xr[NGL][16];
    float xs0[NGL], xs1[NGL];
#pragma unroll
    for (int i = 0; i < NGL; i++) {
        int g = lane + 32 * i;
        if (g < ng) {
            const uint4 *p = reinterpret_cast<const uint4 *>(xq + (size_t)g * 64);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                uint4 v = p[k];
                xr[i][4 * k] = v.x; xr[i][4 * k + 1] = v.y; xr[i][4 * k + 2] = v.z; xr[i][4 * k + 3] = v.w;
            }
            xs0[i] = sx[2 * g]; xs1[i] = sx[2 * g + 1];
        } else {
#pragma unroll
            for (int k = 0; k < 16; k++) xr[i][k] = 0;
            xs0[i] = xs1[i] = 0.f;
        }
    }
    const float tot = sxtot[0];
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int w0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const size_t rowb = (size_t)I / 4;
    for (int o = w0 * 2; o < O; o += warps * 2) {
        const bool two = o + 1 < O;
        uint4 ca[NGL], cb[NGL];
#pragma unroll
        for (int i = 0; i < NGL; i++) {
            int g = lane + 32 * i;
            if (g < ng) {
                ca[i] = ldg_stream(codes + (size_t)o * rowb + (size_t)g * 16);
                if (two) cb[i] = ldg_stream(codes + (size_t)(o + 1) * rowb + (size_t)g * 16);
            }
        }
        float acc_a = 0.f, acc_b = 0.f;
#pragma unroll
        for (int i = 0; i < NGL; i++) {
            int g = lane + 32 * i;
            if (g < ng) {
                int s0, s1;
                tq2_group_dot(ca[i], xr[i], s0, s1);
                acc_a = fmaf(xs0[i], (float)s0, acc_a);
                acc_a = fmaf(xs1[i], (float)s1, acc_a);
                if (two) {
                    tq2_group_dot(cb[i], xr[i], s0, s1);
                    acc_b = fmaf(xs0[i], (float)s0, acc_b);
                    acc_b = fmaf(xs1[i], (float)s1, acc_b);
                }
            }
        }
        acc_a = warp_sum(acc_a);
        acc_b = warp_sum(acc_b);
        if (lane == 0) {
            y[o] = alpha[o] * (acc_a - tot);
            if (two) y[o + 1] = alpha[o + 1] * (acc_b - tot);
        }
    }
}

// ---------------------------------------------------------------- streamed matvec
// For matrices well beyond L2 (stacked layers, lm_head): a persistent grid in which one
// producer thread per CTA streams whole tiles of R consecutive rows -- the rows' code
// bytes and fp16 scale rows are each one contiguous range of their plane -- into a
// 4-stage shared-memory ring with cp.async.bulk, so ~100 KB per CTA is in flight
// regardless of registers; 8 consumer warps compute from shared memory with the same
// per-lane block split, dot products and reduction order as k_gemv_q (identical y).
namespace gs {
constexpr int NST = 4, WARPS = 8, THREADS = (WARPS + 1) * 32;
}
__device__ int g_gemv_err;

__host__ __device__ inline int gs_align(int x) { return (x + 127) & ~127; }

template <int FMT, int NBL>
__global__ void __launch_bounds__(gs::THREADS) k_gemv_stream(const uint8_t *__restrict__ codes, const void *__restrict__ scale,
                                                             int O, int I, int R, const int8_t *__restrict__ xq,
                                                             const float *__restrict__ sx, const float *__restrict__ sxtot,
                                                             float *__restrict__ y, float cap) {
    using namespace gs;
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool TQ2 = FMT == GPU_FMT_TQ2;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = I / ZZ_BLK, nbp = (nb + 7) & ~7;
    const int rowb = TQ2 ? I / 4 : FMT == GPU_FMT_Q40 ? I / 2 : I;
    const int srow = TQ2 ? 0 : nbp * 2;  // scale bytes per row (tq2: alpha read directly)
    const int cbytes = gs_align(R * rowb), stage = cbytes + gs_align(R * srow);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NST * stage), *empty = full + NST;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + NST);
    const int ntiles = (O + R - 1) / R;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; i++) { tc::mbar_init(&full[i], 1); tc::mbar_init(&empty[i], WARPS); }
        *abort_flag = 0;
        tc::mbar_init_fence();
    }
    __syncthreads();
    if (warp == WARPS) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t i = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x, i++) {
                const int s = i % NST;
                if (i >= NST && !tc::mbar_wait(&empty[s], ((i / NST) - 1) & 1, abort_flag, &g_gemv_err, 1)) break;
                const int rows = min(R, O - t * R);
                tc::mbar_arrive_tx(&full[s], (uint32_t)(rows * rowb + rows * srow));
                tc::bulk_load(smem + s * stage, codes + (size_t)t * R * rowb, (uint32_t)(rows * rowb), &full[s]);
                if (!TQ2)
                    tc::bulk_load(smem + s * stage + cbytes, reinterpret_cast<const uint8_t *>(scale) + (size_t)t * R * srow,
                                  (uint32_t)(rows * srow), &full[s]);
            }
            if (i) tc::mbar_wait(&full[(i - 1) % NST], ((i - 1) / NST) & 1, abort_flag, &g_gemv_err, 2);
        }
        return;
    }
    // ---------------- consumers ----------------
    constexpr int XW = TQ2 ? 16 : 8;  // activation words per unit (tq2: 64-weight group)
    uint32_t xr[NBL][XW];
    float xs0[NBL], xs1[NBL];
    const int nu = TQ2 ? I / 64 : nb;  // units per row
#pragma unroll
    for (int i = 0; i < NBL; i++) {
        int u = lane + 32 * i;
        if (u < nu) {
            const uint4 *p = reinterpret_cast<const uint4 *>(xq + (size_t)u * XW * 4);
#pragma unroll
            for (int k = 0; k < XW / 4; k++) {
                uint4 v = p[k];
                xr[i][4 * k] = v.x; xr[i][4 * k + 1] = v.y; xr[i][4 * k + 2] = v.z; xr[i][4 * k + 3] = v.w;
            }
            xs0[i] = TQ2 ? sx[2 * u] : sx[u];
            xs1[i] = TQ2 ? sx[2 * u + 1] : 0.f;
        } else {
#pragma unroll
            for (int k = 0; k < XW; k++) xr[i][k] = 0;
            xs0[i] = xs1[i] = 0.f;
        }
    }
    const float tot = TQ2 ? sxtot[0] : 0.f;
    uint32_t i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, i++) {
        const int s = i % NST;
        const bool ok = tc::mbar_wait(&full[s], (i / NST) & 1, abort_flag, &g_gemv_err, 3);
        const int rows = min(R, O - t * R);
        const uint8_t *sc = smem + s * stage;
        const __half *ss = reinterpret_cast<const __half *>(sc + cbytes);
        for (int r = warp; ok && r < rows; r += WARPS) {
            const uint8_t *crow = sc + (size_t)r * rowb;
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < NBL; j++) {
                int u = lane + 32 * j;
                if (u < nu) {
                    if (FMT == GPU_FMT_Q40) {
                        const uint4 w = *reinterpret_cast<const uint4 *>(crow + u * 16);
                        acc = fmaf(__half2float(ss[r * nbp + u]) * xs0[j], (float)q40_block_dot(w, xr[j]), acc);
                    } else if (FMT == GPU_FMT_Q80) {
                        const uint4 w0 = *reinterpret_cast<const uint4 *>(crow + u * 32);
                        const uint4 w1 = *reinterpret_cast<const uint4 *>(crow + u * 32 + 16);
                        acc = fmaf(__half2float(ss[r * nbp + u]) * xs0[j], (float)q80_block_dot(w0, w1, xr[j]), acc);
                    } else {
                        int s0, s1;
                        tq2_group_dot(*reinterpret_cast<const uint4 *>(crow + u * 16), xr[j], s0, s1);
                        acc = fmaf(xs0[j], (float)s0, acc);
                        acc = fmaf(xs1[j], (float)s1, acc);
                    }
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) {
                const int o = t * R + r;
                float v = TQ2 ? reinterpret_cast<const float *>(scale)[o] * (acc - tot) : acc;
                // final-logit softcap of a tied lm_head (gemma4.c:1271-1274)
                if (cap > 0.f) v = __fmul_rn(tanhf(__fdiv_rn(v, cap)), cap);
                y[o] = v;
            }
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
}

// rows per streamed tile: 16, fewer for long rows (a stage stays <= 32 KB)
static int gs_rows(int rowb, int srow) {
    int R = 16;
    while (R > 1 && R * (rowb + srow) > 32 * 1024) R >>= 1;
    return R;
}

// streamed matvec; returns 0 if the shape has no instantiation
static int launch_gemv_stream(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float *y,
                              cudaStream_t st, float cap = 0.f) {
    const int O = W->O, I = W->I, nb = I / ZZ_BLK, nbp = (nb + 7) & ~7;
    const bool tq2 = W->fmt == GPU_FMT_TQ2;
    const int rowb = tq2 ? I / 4 : W->fmt == GPU_FMT_Q40 ? I / 2 : I, srow = tq2 ? 0 : nbp * 2;
    if (rowb % 16 || ((uintptr_t)W->codes & 15) || (!tq2 && ((uintptr_t)W->scale & 15))) return 0;
    const int R = gs_rows(rowb, srow);
    const int stage = gs_align(R * rowb) + gs_align(R * srow);
    const int smem = gs::NST * stage + 2 * gs::NST * 8 + 16;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int ntiles = (O + R - 1) / R;
    const int per_sm = smem <= 110 * 1024 ? 2 : 1;
    const int grid = ntiles < per_sm * sms ? ntiles : per_sm * sms;
    const int nu = tq2 ? I / 64 : nb, nbl = (nu + 31) / 32;
#define ZZ_GS(F, N)                                                                                           \
    case N: {                                                                                                  \
        static bool attr = false;                                                                              \
        if (!attr) {                                                                                           \
            cudaFuncSetAttribute(k_gemv_stream<F, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); \
            attr = true;                                                                                       \
        }                                                                                                      \
        k_gemv_stream<F, N><<<grid, gs::THREADS, smem, st>>>(W->codes, W->scale, O, I, R, xq, sx, sxtot, y, cap); \
        break;                                                                                                 \
    }
    if (W->fmt == GPU_FMT_Q40) {
        switch (nbl) { ZZ_GS(GPU_FMT_Q40, 1) ZZ_GS(GPU_FMT_Q40, 2) ZZ_GS(GPU_FMT_Q40, 3) ZZ_GS(GPU_FMT_Q40, 4)
                       ZZ_GS(GPU_FMT_Q40, 5) ZZ_GS(GPU_FMT_Q40, 6) ZZ_GS(GPU_FMT_Q40, 7) ZZ_GS(GPU_FMT_Q40, 8)
                       default: return 0; }
    } else if (W->fmt == GPU_FMT_Q80) {
        switch (nbl) { ZZ_GS(GPU_FMT_Q80, 1) ZZ_GS(GPU_FMT_Q80, 2) ZZ_GS(GPU_FMT_Q80, 3) ZZ_GS(GPU_FMT_Q80, 4)
                       ZZ_GS(GPU_FMT_Q80, 5) ZZ_GS(GPU_FMT_Q80, 6) ZZ_GS(GPU_FMT_Q80, 7) ZZ_GS(GPU_FMT_Q80, 8)
                       default: return 0; }
    } else {
        switch (nbl) { ZZ_GS(GPU_FMT_TQ2, 1) ZZ_GS(GPU_FMT_TQ2, 2) ZZ_GS(GPU_FMT_TQ2, 3) ZZ_GS(GPU_FMT_TQ2, 4)
                       default: return 0; }
    }
#undef ZZ_GS
    return check_cuda(cudaGetLastError(), "gemv stream launch") ? 1 : -1;
}

// per-block integer sums, one thread per (row, block): the bit-exact parity quantity
template <int FMT>
__global__ void k_blocksums(const uint8_t *__restrict__ codes, int O, int I, const int8_t *__restrict__ xq,
                            int32_t *__restrict__ out) {
    const int nb = I / ZZ_BLK;
    long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long)O * nb) return;
    int o = (int)(t / nb), b = (int)(t % nb);
    const int8_t *x = xq + (size_t)b * ZZ_BLK;
    int s = 0;
    if (FMT == GPU_FMT_Q40) {
        const uint8_t *c = codes + (size_t)o * (I / 2) + (size_t)b * 16;
        for (int j = 0; j < 16; j++) s += ((c[j] & 15) - 8) * x[j] + ((c[j] >> 4) - 8) * x[j + 16];
    } else if (FMT == GPU_FMT_Q80) {
        const int8_t *c = reinterpret_cast<const int8_t *>(codes) + (size_t)o * I + (size_t)b * 32;
        for (int j = 0; j < 32; j++) s += c[j] * x[j];
    } else {
        const uint8_t *c = codes + (size_t)o * (I / 4) + (size_t)(b / 2) * 16;
        int sh = (b & 1) * 4;
        for (int k = 0; k < 16; k++)
            s += ((c[k] >> sh) & 3) * x[k] + ((c[k] >> (sh + 2)) & 3) * x[k + 16];
    }
    out[t] = s;
}

static int gemv_grid(int O) {
    int g = (O + 15) / 16;  // 8 warps x 2 rows
    int cap = 148 * 8;
    return g < cap ? g : cap;
}

// one activation row; returns 0 if the shape has no fast-path instantiation
int launch_gemv1(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float *y,
                 cudaStream_t st) {
    const int O = W->O, I = W->I, grid = gemv_grid(O);
    // matrices that stream from HBM (well beyond L2) take the bulk-copy kernel; small
    // ones (latency-bound) the register kernel. ZZ_GEMV=stream|reg overrides.
    static const char *mode = getenv("ZZ_GEMV");
    const size_t bytes = zz_qtensor_bytes(W->fmt, O, I);
    const bool stream = mode ? mode[0] == 's' : bytes >= ((size_t)64 << 20);
    if (stream) {
        int r = launch_gemv_stream(W, xq, sx, sxtot, y, st);
        if (r) return r;
    }
    if (W->fmt == GPU_FMT_TQ2) {
        int ngl = (I / 64 + 31) / 32;
        switch (ngl) {
#define ZZ_T(N) case N: k_gemv_tq2<N><<<grid, 256, 0, st>>>(W->codes, (const float *)W->scale, O, I, xq, sx, sxtot, y); break;
            ZZ_T(1) ZZ_T(2) ZZ_T(3) ZZ_T(4)
#undef ZZ_T
            default: return 0;
        }
    } else {
        int nbl = (I / 32 + 31) / 32;
        const __half *sc = (const __half *)W->scale;
        if (W->fmt == GPU_FMT_Q40) {
            switch (nbl) {
#define ZZ_Q(N) case N: k_gemv_q<GPU_FMT_Q40, N><<<grid, 256, 0, st>>>(W->codes, sc, O, I, xq, sx, y); break;
                ZZ_Q(1) ZZ_Q(2) ZZ_Q(3) ZZ_Q(4) ZZ_Q(5) ZZ_Q(6) ZZ_Q(7) ZZ_Q(8)
#undef ZZ_Q
                default: return 0;
            }
        } else {
            switch (nbl) {
#define ZZ_Q(N) case N: k_gemv_q<GPU_FMT_Q80, N><<<grid, 256, 0, st>>>(W->codes, sc, O, I, xq, sx, y); break;
                ZZ_Q(1) ZZ_Q(2) ZZ_Q(3) ZZ_Q(4) ZZ_Q(5) ZZ_Q(6) ZZ_Q(7) ZZ_Q(8)
#undef ZZ_Q
                default: return 0;
            }
        }
    }
    return check_cuda(cudaGetLastError(), "gemv launch") ? 1 : -1;
}

int launch_blocksums(const zz_qtensor *W, const int8_t *xq, int32_t *out, cudaStream_t st) {
    if (W->fmt == GPU_FMT_Q4A) return fail("zz_blocksums_dev: q4a has no per-block integer check");
    long n = (long)W->O * (W->I / ZZ_BLK);
    unsigned grid = (unsigned)((n + 255) / 256);
    if (W->fmt == GPU_FMT_Q40) k_blocksums<GPU_FMT_Q40><<<grid, 256, 0, st>>>(W->codes, W->O, W->I, xq, out);
    else if (W->fmt == GPU_FMT_Q80) k_blocksums<GPU_FMT_Q80><<<grid, 256, 0, st>>>(W->codes, W->O, W->I, xq, out);
    else k_blocksums<GPU_FMT_TQ2><<<grid, 256, 0, st>>>(W->codes, W->O, W->I, xq, out);
    return check_cuda(cudaGetLastError(), "blocksums launch");
}

}  // namespace zz

// ---------------------------------------------------------------- lm_head
__global__ void k_softcap(float *__restrict__ y, long n, float cap) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fmul_rn(tanhf(__fdiv_rn(y[i], cap)), cap);
}

namespace zz {
int matvec_impl(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float *y, int S,
                cudaStream_t st);
}

extern "C" int zz_lm_head_dev(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float softcap,
                              float *y, void *stream) {
    using namespace zz;
    if (!W || !W->codes || !W->scale || W->O <= 0 || W->I <= 0 || W->fmt == GPU_FMT_Q4A && W->I % 64)
        return fail("zz_lm_head_dev: invalid tensor");
    if (!xq || !sx || !y || (W->fmt == GPU_FMT_TQ2 && !sxtot)) return fail("zz_lm_head_dev: null pointer");
    if (!(softcap >= 0.f)) return fail("zz_lm_head_dev: softcap %g < 0", (double)softcap);
    cudaStream_t st = (cudaStream_t)stream;
    // tall tensors take the streamed kernel with the softcap in its epilogue
    if (W->fmt != GPU_FMT_Q4A && zz_qtensor_bytes(W->fmt, W->O, W->I) >= ((size_t)64 << 20)) {
        const int r = launch_gemv_stream(W, xq, sx, sxtot, y, st, softcap);
        if (r) return r > 0;
    }
    if (!matvec_impl(W, xq, sx, sxtot, y, 1, st)) return 0;
    if (softcap > 0.f) {
        k_softcap<<<(unsigned)((W->O + 255) / 256), 256, 0, st>>>(y, W->O, softcap);
        return check_cuda(cudaGetLastError(), "softcap launch");
    }
    return 1;
}
