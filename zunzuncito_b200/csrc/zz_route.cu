// zz_route.cu -- the MoE routers on the device, feeding the batch-union FFN with no
// host round trip: gemma4's softmax top-k router (gemma4.c:581-613) and ling's grouped
// sigmoid router (ling.c:705-789). One CTA per token row.
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

__device__ __forceinline__ double block_sum_d(double v, double *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0;
    if (threadIdx.x == 0)
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
    __syncthreads();
    return t;  // valid in thread 0
}

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

__global__ void __launch_bounds__(RT_THREADS) k_route_gemma4(const float *__restrict__ res, int D, int E, int K,
                                                             const float *__restrict__ proj,
                                                             const float *__restrict__ scale,
                                                             const float *__restrict__ pes, float eps,
                                                             int32_t *__restrict__ idx, float *__restrict__ wts) {
    extern __shared__ float sm[];
    float *xn = sm, *lg = sm + D;
    __shared__ double red[RT_THREADS / 32];
    __shared__ float r_sh;
    __shared__ float topv[RT_MAXK];
    __shared__ int topi[RT_MAXK];
    const int s = blockIdx.x, tid = threadIdx.x;
    const float *x = res + (size_t)s * D;
    // rmsnorm without weight (gemma4.c:425-431): double sum of squares
    double acc = 0;
    for (int i = tid; i < D; i += blockDim.x) acc += (double)x[i] * (double)x[i];
    const double ss = block_sum_d(acc, red);
    if (tid == 0) r_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(ss / D), eps)));
    __syncthreads();
    const float r = r_sh, rs = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    for (int i = tid; i < D; i += blockDim.x) xn[i] = __fmul_rn(__fmul_rn(x[i], r), __fmul_rn(scale[i], rs));
    __syncthreads();
    // logits, one sequential chain per expert (gemma4.c:601-603)
    for (int e = tid; e < E; e += blockDim.x) {
        const float *p = proj + (size_t)e * D;
        float v = 0.f;
        for (int i = 0; i < D; i++) v = __fadd_rn(v, __fmul_rn(__ldg(p + i), xn[i]));
        lg[e] = v;
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
        const int rk = score_rank(lg, E, e, nullptr);
        if (rk < K) { topv[rk] = lg[e]; topi[rk] = e; }
    }
    __syncthreads();
    if (tid == 0) {
        // softmax over the K selected logits, times the per-expert scale (gemma4.c:609-612)
        float w[RT_MAXK], sum = 0.f;
        const float mx = topv[0];
        for (int j = 0; j < K; j++) { w[j] = expf(__fsub_rn(topv[j], mx)); sum = __fadd_rn(sum, w[j]); }
        for (int j = 0; j < K; j++) {
            idx[(size_t)s * K + j] = topi[j];
            wts[(size_t)s * K + j] = __fmul_rn(__fdiv_rn(w[j], sum), pes[topi[j]]);
        }
    }
}

__global__ void __launch_bounds__(RT_THREADS) k_route_ling(const float *__restrict__ xn_g, int D, int E, int K, int NG,
                                                           int TG, int norm_topk, float routed_scale,
                                                           const float *__restrict__ router,
                                                           const float *__restrict__ bias,
                                                           int32_t *__restrict__ idx, float *__restrict__ wts) {
    extern __shared__ float sm[];
    float *xn = sm, *rwt = sm + D, *rsel = rwt + E;
    __shared__ unsigned char live[1024];
    __shared__ float topv[RT_MAXK];
    __shared__ int topi[RT_MAXK];
    const int s = blockIdx.x, tid = threadIdx.x;
    for (int i = tid; i < D; i += blockDim.x) xn[i] = xn_g[(size_t)s * D + i];
    __syncthreads();
    // sigmoid scores (ling.c:721-733): eight double accumulators, the reference's tree
    for (int e = tid; e < E; e += blockDim.x) {
        const float *r = router + (size_t)e * D;
        double a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= D; i += 8)
#pragma unroll
            for (int k = 0; k < 8; k++) a[k] = __dadd_rn(a[k], __dmul_rn((double)__ldg(r + i + k), (double)xn[i + k]));
        for (; i < D; i++) a[0] = __dadd_rn(a[0], __dmul_rn((double)__ldg(r + i), (double)xn[i]));
        const double v = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
        const float w = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-(float)v)));
        rwt[e] = w;
        rsel[e] = __fadd_rn(w, bias[e]);
    }
    __syncthreads();
    if (tid == 0) {
        // groups ranked by the sum of their two best biased scores; the best TG kept
        // (ling.c:735-760), in the reference's insertion order
        const int EG = E / NG;
        float gs[RT_MAXG], topg[RT_MAXG];
        int keep[RT_MAXG];
        for (int g = 0; g < NG; g++) {
            float a = -INFINITY, b = -INFINITY;
            for (int i = 0; i < EG; i++) {
                const float v = rsel[g * EG + i];
                if (v > a) { b = a; a = v; }
                else if (v > b) b = v;
            }
            gs[g] = EG > 1 ? __fadd_rn(a, b) : a;
        }
        for (int j = 0; j < TG; j++) { keep[j] = -1; topg[j] = -INFINITY; }
        for (int g = 0; g < NG; g++) {
            int j = TG;
            while (j > 0 && gs[g] > topg[j - 1]) j--;
            if (j == TG) continue;
            for (int t = TG - 1; t > j; t--) { topg[t] = topg[t - 1]; keep[t] = keep[t - 1]; }
            topg[j] = gs[g]; keep[j] = g;
        }
        for (int e = 0; e < E; e++) live[e] = 0;
        for (int j = 0; j < TG; j++)
            if (keep[j] >= 0)
                for (int e = keep[j] * EG; e < (keep[j] + 1) * EG; e++) live[e] = 1;
        // top-K of the kept experts by biased score, ties to the lower index (ling.c:762-774)
        for (int j = 0; j < K; j++) { topi[j] = -1; topv[j] = -INFINITY; }
        for (int e = 0; e < E; e++) {
            if (!live[e]) continue;
            const float v = rsel[e];
            int j = K;
            while (j > 0 && v > topv[j - 1]) j--;
            if (j == K) continue;
            for (int t = K - 1; t > j; t--) { topv[t] = topv[t - 1]; topi[t] = topi[t - 1]; }
            topv[j] = v; topi[j] = e;
        }
        // the unbiased scores, renormalised, times routed_scale (ling.c:783-788)
        float w[RT_MAXK], sum = 0.f;
        for (int j = 0; j < K; j++) { w[j] = rwt[topi[j]]; sum = __fadd_rn(sum, w[j]); }
        if (norm_topk && K > 1)
            for (int j = 0; j < K; j++) w[j] = __fdiv_rn(w[j], __fadd_rn(sum, 1e-20f));
        for (int j = 0; j < K; j++) {
            idx[(size_t)s * K + j] = topi[j];
            wts[(size_t)s * K + j] = __fmul_rn(w[j], routed_scale);
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

extern "C" int zz_route_gemma4_dev(const float *res, int S, int D, int E, int K, const float *proj,
                                   const float *scale, const float *pes, float eps, int32_t *idx, float *wts,
                                   void *stream) {
    if (S < 0 || D <= 0 || E <= 0 || K <= 0 || K > RT_MAXK || K > E)
        return fail("zz_route_gemma4_dev: bad shape S=%d D=%d E=%d K=%d (K <= %d)", S, D, E, K, RT_MAXK);
    const size_t smem = (size_t)(D + E) * 4;
    if (smem > 200 * 1024) return fail("zz_route_gemma4_dev: D + E = %d too large", D + E);
    if (S == 0) return 1;
    if (!res || !proj || !scale || !pes || !idx || !wts) return fail("zz_route_gemma4_dev: null pointer");
    if (!set_smem((const void *)k_route_gemma4, smem)) return 0;
    k_route_gemma4<<<S, RT_THREADS, smem, (cudaStream_t)stream>>>(res, D, E, K, proj, scale, pes, eps, idx, wts);
    return check_cuda(cudaGetLastError(), "route_gemma4 launch");
}

extern "C" int zz_route_ling_dev(const float *xn, int S, int D, int E, int K, int n_group, int topk_group,
                                 int norm_topk_prob, float routed_scale, const float *router, const float *bias,
                                 int32_t *idx, float *wts, void *stream) {
    if (S < 0 || D <= 0 || E <= 0 || E > 1024 || K <= 0 || K > RT_MAXK || K > E || n_group < 1 ||
        n_group > RT_MAXG || E % n_group || topk_group < 1 || topk_group > n_group)
        return fail("zz_route_ling_dev: bad shape S=%d D=%d E=%d K=%d groups %d/%d", S, D, E, K, topk_group, n_group);
    const size_t smem = (size_t)(D + 2 * E) * 4;
    if (smem > 200 * 1024) return fail("zz_route_ling_dev: D=%d too large", D);
    if (S == 0) return 1;
    if (!xn || !router || !bias || !idx || !wts) return fail("zz_route_ling_dev: null pointer");
    if (!set_smem((const void *)k_route_ling, smem)) return 0;
    k_route_ling<<<S, RT_THREADS, smem, (cudaStream_t)stream>>>(xn, D, E, K, n_group, topk_group, norm_topk_prob,
                                                                routed_scale, router, bias, idx, wts);
    return check_cuda(cudaGetLastError(), "route_ling launch");
}
