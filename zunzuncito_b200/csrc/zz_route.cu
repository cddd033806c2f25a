// zz_route.cu -- the MoE routers on the device, feeding the batch-union FFN with no
// host round trip: gemma4's softmax top-k router (gemma4.c:581-613) and ling's grouped
// sigmoid router (ling.c:705-789). A CTA takes RT_TS token rows and one thread per
// expert, which streams its router row once for all of them.
//
// Selection must be the reference's exactly (a different expert is a different
// output), so every score is computed in the reference's operation order:
//  * gemma4: logit_e = a sequential chain of rounded f32 products and sums over the
//    hidden dimension (no contraction, as the reference build computes it);
//  * ling: per expert eight double accumulators over interleaved elements, combined
//    pairwise in the reference's tree; the sigmoid and bias in f32.
// Top-k keeps the reference's insertion semantics: descending score, ties to the lower
// expert index. One difference remains: gemma4's sum of squares for the rmsnorm is
// reduced in parallel (double), where the reference sums sequentially; the rounded
// f32 norm can differ only when that double lies within a few double ulps of an f32
// rounding boundary. Weights use CUDA's expf (within 1 ulp of the C library's).
#include "zz_common.cuh"

namespace zz {

constexpr int RT_THREADS = 256;
constexpr int RT_MAXK = 16, RT_MAXG = 32;

// rank of score e among E scores: those strictly greater, or equal at a lower index
__device__ __forceinline__ int score_rank(const float *v, int E, int e, const unsigned char *live) {
    const float x = v[e];
    int r = 0;
    for (int f = 0; f < E; f++) {
        if (live && !live[f]) continue;
        const float y = v[f];
        r += (y > x) || (y == x && f < e);
    }
    return r;
}

// Work split: a CTA takes RT_TS * TG token rows, TG = RT_THREADS / E' (E' = E rounded up
// to a warp) token groups of RT_TS rows each; thread (g, e) keeps the RT_TS sequential
// score chains of expert e for group g's rows, so the add latency of one chain hides
// behind the others. The router weights stream through shared memory in chunks of
// RT_C columns, double-buffered with cp.async (coalesced 16-byte copies; each expert's
// chunk row padded to RT_C + 4 floats so the per-thread 16-byte reads are conflict
// free), and every chunk serves all the CTA's rows.
constexpr int RT_TS = 2, RT_C = 64, RT_LD = RT_C + 4;

__device__ __forceinline__ void cp16(float *dst, const float *src, bool ok) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(ok ? src : nullptr), "r"(ok ? 16 : 0));
}
// router columns [i0, i0 + RT_C) of all E rows into buf[e * RT_LD + c] (zero past D)
__device__ __forceinline__ void stage_chunk(float *buf, const float *__restrict__ W, int E, int D, int i0) {
    for (int k = threadIdx.x; k < E * (RT_C / 4); k += blockDim.x) {
        const int e = k / (RT_C / 4), c4 = k % (RT_C / 4);
        const int i = i0 + 4 * c4;
        cp16(buf + e * RT_LD + 4 * c4, W + (size_t)e * D + i, i < D);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(RT_THREADS) k_route_gemma4(const float *__restrict__ res, int S, int D, int E, int K,
                                                             const float *__restrict__ proj,
                                                             const float *__restrict__ scale,
                                                             const float *__restrict__ pes, float eps,
                                                             int32_t *__restrict__ idx, float *__restrict__ wts) {
    extern __shared__ __align__(16) float sm[];
    const int Ew = (E + 31) & ~31, TG = RT_THREADS / Ew, NT = TG * RT_TS;
    float *pbuf = sm;                              // [2][E][RT_LD]
    float *xn = pbuf + 2 * E * RT_LD;              // [NT][D]
    float *lg = xn + NT * D;                       // [NT][E]
    __shared__ float topv[RT_THREADS / 32 * RT_TS][RT_MAXK];
    __shared__ int topi[RT_THREADS / 32 * RT_TS][RT_MAXK];
    const int s0 = blockIdx.x * NT, tid = threadIdx.x;
    const int ts = min(NT, S - s0);
    stage_chunk(pbuf, proj, E, D, 0);   // the first chunk's copies overlap the norms
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    // rmsnorm without weight (gemma4.c:425-431): one warp per row sums the squares in
    // double, then every thread scales its share of all rows
    __shared__ float r_row[RT_THREADS / 32 * RT_TS];
    {
        const int w = tid >> 5, l = tid & 31;
        for (int t = w; t < ts; t += blockDim.x >> 5) {
            const float *x = res + (size_t)(s0 + t) * D;
            double acc = 0;
            for (int i = l; i < D; i += 32) acc += (double)x[i] * (double)x[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (l == 0) r_row[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(acc / D), eps)));
        }
    }
    __syncthreads();
    for (int k = tid; k < ts * D; k += blockDim.x) {
        const int t = k / D, i = k - t * D;
        xn[k] = __fmul_rn(__fmul_rn(res[(size_t)(s0 + t) * D + i], r_row[t]), __fmul_rn(scale[i], rs));
    }
    __syncthreads();
    // logits: per (row, expert) one sequential chain of rounded products and sums over
    // the hidden dimension (gemma4.c:601-603)
    const int e = tid % Ew, g = tid / Ew;
    const bool act = e < E && g < TG;
    const float *xg = xn + (size_t)g * RT_TS * D;
    float v[RT_TS];
#pragma unroll
    for (int t = 0; t < RT_TS; t++) v[t] = 0.f;
    const int nch = (D + RT_C - 1) / RT_C;
    for (int c = 0; c < nch; c++) {
        if (c + 1 < nch) {
            stage_chunk(pbuf + ((c + 1) & 1) * E * RT_LD, proj, E, D, (c + 1) * RT_C);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        if (act) {
            const float *w = pbuf + (c & 1) * E * RT_LD + e * RT_LD;
            const int i0 = c * RT_C, nc = min(RT_C, D - i0);
            for (int c4 = 0; c4 < nc / 4; c4++) {
                const float4 w4 = *reinterpret_cast<const float4 *>(w + 4 * c4);
#pragma unroll
                for (int t = 0; t < RT_TS; t++) {
                    const float4 x = *reinterpret_cast<const float4 *>(xg + t * D + i0 + 4 * c4);
                    float a = v[t];
                    a = __fadd_rn(a, __fmul_rn(w4.x, x.x));
                    a = __fadd_rn(a, __fmul_rn(w4.y, x.y));
                    a = __fadd_rn(a, __fmul_rn(w4.z, x.z));
                    v[t] = __fadd_rn(a, __fmul_rn(w4.w, x.w));
                }
            }
        }
        __syncthreads();   // the buffer is refilled by the next iteration's copies
    }
    if (act)
#pragma unroll
        for (int t = 0; t < RT_TS; t++)
            if (g * RT_TS + t < ts) lg[(g * RT_TS + t) * E + e] = v[t];
    __syncthreads();
    for (int t = 0; t < ts; t++)
        for (int ee = tid; ee < E; ee += blockDim.x) {
            const int rk = score_rank(lg + t * E, E, ee, nullptr);
            if (rk < K) { topv[t][rk] = lg[t * E + ee]; topi[t][rk] = ee; }
        }
    __syncthreads();
    if (tid < ts) {
        // softmax over the K selected logits, times the per-expert scale (gemma4.c:609-612)
        const int t = tid, s = s0 + t;
        float w[RT_MAXK], sum = 0.f;
        const float mx = topv[t][0];
        for (int j = 0; j < K; j++) { w[j] = expf(__fsub_rn(topv[t][j], mx)); sum = __fadd_rn(sum, w[j]); }
        for (int j = 0; j < K; j++) {
            idx[(size_t)s * K + j] = topi[t][j];
            wts[(size_t)s * K + j] = __fmul_rn(__fdiv_rn(w[j], sum), pes[topi[t][j]]);
        }
    }
}

__global__ void __launch_bounds__(RT_THREADS) k_route_ling(const float *__restrict__ xn_g, int S, int D, int E, int K,
                                                           int NG, int TG_, int norm_topk, float routed_scale,
                                                           const float *__restrict__ router,
                                                           const float *__restrict__ bias,
                                                           int32_t *__restrict__ idx, float *__restrict__ wts) {
    extern __shared__ __align__(16) float sm[];
    const int Ew = (E + 31) & ~31, TG = Ew <= RT_THREADS ? RT_THREADS / Ew : 1, NT = TG * RT_TS;
    float *pbuf = sm;                              // [2][E][RT_LD]
    float *xn = pbuf + 2 * E * RT_LD;              // [NT][D]
    float *rwt = xn + NT * D;                      // [NT][E]
    float *rsel = rwt + NT * E;                    // [NT][E]
    __shared__ unsigned char live[1024];
    __shared__ float topv[RT_MAXK];
    __shared__ int topi[RT_MAXK];
    const int s0 = blockIdx.x * NT, tid = threadIdx.x;
    const int ts = min(NT, S - s0);
    for (int i = tid; i < NT * D; i += blockDim.x) xn[i] = i < ts * D ? xn_g[(size_t)s0 * D + i] : 0.f;
    // sigmoid scores (ling.c:721-733): per (row, expert) eight double accumulators over
    // interleaved elements (element i into accumulator i % 8), combined in the
    // reference's tree
    {   // E <= RT_THREADS: one pass covers every expert
        const int e = tid % Ew, g = tid / Ew;
        const bool act = e < E && g < TG;
        const float *xg = xn + (size_t)g * RT_TS * D;
        double a[RT_TS][8];
#pragma unroll
        for (int t = 0; t < RT_TS; t++)
#pragma unroll
            for (int k = 0; k < 8; k++) a[t][k] = 0;
        const int D8 = D / 8 * 8;
        const int nch = (D8 + RT_C - 1) / RT_C;
        __syncthreads();
        if (nch > 0) stage_chunk(pbuf, router, E, D8, 0);
        for (int c = 0; c < nch; c++) {
            if (c + 1 < nch) {
                stage_chunk(pbuf + ((c + 1) & 1) * E * RT_LD, router, E, D8, (c + 1) * RT_C);
                asm volatile("cp.async.wait_group 1;" ::: "memory");
            } else {
                asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            __syncthreads();
            if (act) {
                const float *w = pbuf + (c & 1) * E * RT_LD + e * RT_LD;
                const int i0 = c * RT_C, nc = min(RT_C, D8 - i0);
                for (int c8 = 0; c8 < nc / 8; c8++) {
                    const float4 w0 = *reinterpret_cast<const float4 *>(w + 8 * c8);
                    const float4 w1 = *reinterpret_cast<const float4 *>(w + 8 * c8 + 4);
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const double pk = (double)wv[k];
#pragma unroll
                        for (int t = 0; t < RT_TS; t++)
                            a[t][k] = __dadd_rn(a[t][k], __dmul_rn(pk, (double)xg[t * D + i0 + 8 * c8 + k]));
                    }
                }
            }
            __syncthreads();
        }
        if (act) {
            for (int i = D8; i < D; i++) {   // tail into the first accumulator (ling.c:728)
                const double p = (double)__ldg(router + (size_t)e * D + i);
#pragma unroll
                for (int t = 0; t < RT_TS; t++) a[t][0] = __dadd_rn(a[t][0], __dmul_rn(p, (double)xg[t * D + i]));
            }
#pragma unroll
            for (int t = 0; t < RT_TS; t++) {
                const int row = g * RT_TS + t;
                if (row >= ts) continue;
                const double v = ((a[t][0] + a[t][1]) + (a[t][2] + a[t][3])) + ((a[t][4] + a[t][5]) + (a[t][6] + a[t][7]));
                const float w = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-(float)v)));
                rwt[row * E + e] = w;
                rsel[row * E + e] = __fadd_rn(w, bias[e]);
            }
        }
    }
    __syncthreads();
    for (int t = 0; t < ts; t++) {
        if (tid == 0) {
            const float *sel = rsel + t * E, *wt = rwt + t * E;
            const int s = s0 + t, TG = TG_;
            // groups ranked by the sum of their two best biased scores; the best TG kept
            // (ling.c:735-760), in the reference's insertion order
            const int EG = E / NG;
            float gs[RT_MAXG], topg[RT_MAXG];
            int keep[RT_MAXG];
            for (int gi = 0; gi < NG; gi++) {
                float a = -INFINITY, b = -INFINITY;
                for (int i = 0; i < EG; i++) {
                    const float v = sel[gi * EG + i];
                    if (v > a) { b = a; a = v; }
                    else if (v > b) b = v;
                }
                gs[gi] = EG > 1 ? __fadd_rn(a, b) : a;
            }
            for (int j = 0; j < TG; j++) { keep[j] = -1; topg[j] = -INFINITY; }
            for (int gi = 0; gi < NG; gi++) {
                int j = TG;
                while (j > 0 && gs[gi] > topg[j - 1]) j--;
                if (j == TG) continue;
                for (int q = TG - 1; q > j; q--) { topg[q] = topg[q - 1]; keep[q] = keep[q - 1]; }
                topg[j] = gs[gi]; keep[j] = gi;
            }
            for (int ee = 0; ee < E; ee++) live[ee] = 0;
            for (int j = 0; j < TG; j++)
                if (keep[j] >= 0)
                    for (int ee = keep[j] * EG; ee < (keep[j] + 1) * EG; ee++) live[ee] = 1;
            // top-K of the kept experts by biased score, ties to the lower index (ling.c:762-774)
            for (int j = 0; j < K; j++) { topi[j] = -1; topv[j] = -INFINITY; }
            for (int ee = 0; ee < E; ee++) {
                if (!live[ee]) continue;
                const float v = sel[ee];
                int j = K;
                while (j > 0 && v > topv[j - 1]) j--;
                if (j == K) continue;
                for (int q = K - 1; q > j; q--) { topv[q] = topv[q - 1]; topi[q] = topi[q - 1]; }
                topv[j] = v; topi[j] = ee;
            }
            // the unbiased scores, renormalised, times routed_scale (ling.c:783-788)
            float w[RT_MAXK], sum = 0.f;
            for (int j = 0; j < K; j++) { w[j] = wt[topi[j]]; sum = __fadd_rn(sum, w[j]); }
            if (norm_topk && K > 1)
                for (int j = 0; j < K; j++) w[j] = __fdiv_rn(w[j], __fadd_rn(sum, 1e-20f));
            for (int j = 0; j < K; j++) {
                idx[(size_t)s * K + j] = topi[j];
                wts[(size_t)s * K + j] = __fmul_rn(w[j], routed_scale);
            }
        }
    }
}

static int set_smem(const void *fn, size_t bytes) {
    if (bytes <= 48 * 1024) return 1;
    return check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                      "router smem attribute");
}

}  // namespace zz

using namespace zz;

// rows per CTA of the routers for E experts
static int rows_per_cta(int E) {
    const int Ew = (E + 31) & ~31;
    return (Ew <= RT_THREADS ? RT_THREADS / Ew : 1) * RT_TS;
}

extern "C" int zz_route_gemma4_dev(const float *res, int S, int D, int E, int K, const float *proj,
                                   const float *scale, const float *pes, float eps, int32_t *idx, float *wts,
                                   void *stream) {
    if (S < 0 || D <= 0 || D % 4 || E <= 0 || E > RT_THREADS || K <= 0 || K > RT_MAXK || K > E)
        return fail("zz_route_gemma4_dev: bad shape S=%d D=%d E=%d K=%d (D %% 4 == 0, E <= %d, K <= %d)", S, D, E, K,
                    RT_THREADS, RT_MAXK);
    const int NT = rows_per_cta(E);
    const size_t smem = ((size_t)2 * E * RT_LD + (size_t)NT * D + (size_t)NT * E) * 4;
    if (smem > 220 * 1024) return fail("zz_route_gemma4_dev: D=%d too large", D);
    if (S == 0) return 1;
    if (!res || !proj || !scale || !pes || !idx || !wts) return fail("zz_route_gemma4_dev: null pointer");
    if (((uintptr_t)proj & 15) || ((uintptr_t)res & 3)) return fail("zz_route_gemma4_dev: proj must be 16-byte aligned");
    if (!set_smem((const void *)k_route_gemma4, smem)) return 0;
    k_route_gemma4<<<(S + NT - 1) / NT, RT_THREADS, smem, (cudaStream_t)stream>>>(res, S, D, E, K, proj, scale, pes,
                                                                                  eps, idx, wts);
    return check_cuda(cudaGetLastError(), "route_gemma4 launch");
}

extern "C" int zz_route_ling_dev(const float *xn, int S, int D, int E, int K, int n_group, int topk_group,
                                 int norm_topk_prob, float routed_scale, const float *router, const float *bias,
                                 int32_t *idx, float *wts, void *stream) {
    if (S < 0 || D <= 0 || D % 4 || E <= 0 || E > RT_THREADS || K <= 0 || K > RT_MAXK || K > E || n_group < 1 ||
        n_group > RT_MAXG || E % n_group || topk_group < 1 || topk_group > n_group)
        return fail("zz_route_ling_dev: bad shape S=%d D=%d E=%d K=%d groups %d/%d", S, D, E, K, topk_group, n_group);
    const int NT = rows_per_cta(E);
    const size_t smem = ((size_t)2 * E * RT_LD + (size_t)NT * D + 2 * (size_t)NT * E) * 4;
    if (smem > 220 * 1024) return fail("zz_route_ling_dev: D=%d / E=%d too large", D, E);
    if (S == 0) return 1;
    if (!xn || !router || !bias || !idx || !wts) return fail("zz_route_ling_dev: null pointer");
    if ((uintptr_t)router & 15) return fail("zz_route_ling_dev: router must be 16-byte aligned");
    if (!set_smem((const void *)k_route_ling, smem)) return 0;
    k_route_ling<<<(S + NT - 1) / NT, RT_THREADS, smem, (cudaStream_t)stream>>>(
        xn, S, D, E, K, n_group, topk_group, norm_topk_prob, routed_scale, router, bias, idx, wts);
    return check_cuda(cudaGetLastError(), "route_ling launch");
}
