// zz_f32act.cu -- the q4a format (4-bit affine, tq2.h:268-283) and the matvecs with f32
// activations.
//
// Two numerics exist for a matvec in the reference:
//  * int8 activations (q40_dot, q80_dot, tq2_dot, q4a_dot; the engines' CPU default):
//    zz_matvec_dev and the rest of this library;
//  * f32 activations (q40_dot_f32 q40.h:290-305, q80_dot_f32 q40.h:432-446, tq2_dot_f32
//    tq2.h:235-252, q4a_dot_f32 tq2.h:410-432): what the reference's GPU backend
//    computes (gpu.h:25-30) and what the engines' --check-gpu compares gpu_q40_matmul /
//    gpu_matmul against at 1e-4 (gemma4.c:2315-2361, maple.c:1756-1800). The kernels
//    here serve that: every weight is dequantized in registers and multiplied by the
//    f32 activation; each 32-weight block is summed in fp32 and the blocks of a row are
//    added in fp32 (the reference adds in double; the difference is ~1e-7 relative).
//
// q4a planes: codes [O][I/2] (group g = bytes 32g..32g+31: the two 16-byte nibble blocks
// of the reference group, weights 0-31 then 32-63, low nibble j / high nibble j+16 as in
// q4_0), scales [O][I/64] as (fp16 d, fp16 m) pairs. HBM-bound like q4_0: 18 bytes per
// 32 weights.
#include "zz_dot.cuh"

namespace zz {

int scale_ld(int I);

// ---------------------------------------------------------------- q4a repack
// one thread per 64-weight group: 4 scale bytes, 32 code bytes (reference groups are
// 36 bytes, so the source is only 4-byte aligned)
__global__ void k_repack_q4a(const uint8_t *__restrict__ src, int O, int I, uint8_t *__restrict__ codes,
                             uint32_t *__restrict__ scale) {
    const int ng = I / 64;
    const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long)O * ng) return;
    const uint32_t *s = reinterpret_cast<const uint32_t *>(src + t * 36);
    scale[t] = s[0];
    uint4 *c = reinterpret_cast<uint4 *>(codes + t * 32);
    c[0] = make_uint4(s[1], s[2], s[3], s[4]);
    c[1] = make_uint4(s[5], s[6], s[7], s[8]);
}
__global__ void k_unpack_q4a(const uint8_t *__restrict__ codes, const uint32_t *__restrict__ scale, int O, int I,
                             uint8_t *__restrict__ dst) {
    const int ng = I / 64;
    const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long)O * ng) return;
    uint32_t *d = reinterpret_cast<uint32_t *>(dst + t * 36);
    const uint4 *c = reinterpret_cast<const uint4 *>(codes + t * 32);
    const uint4 a = c[0], b = c[1];
    d[0] = scale[t];
    d[1] = a.x; d[2] = a.y; d[3] = a.z; d[4] = a.w;
    d[5] = b.x; d[6] = b.y; d[7] = b.z; d[8] = b.w;
}

int launch_repack_q4a(const uint8_t *src, int O, int I, uint8_t *codes, void *scale, cudaStream_t st) {
    if ((uintptr_t)src & 3) return fail("q4a repack: source not 4-byte aligned");
    const long n = (long)O * (I / 64);
    k_repack_q4a<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, O, I, codes, (uint32_t *)scale);
    return check_cuda(cudaGetLastError(), "q4a repack launch");
}
int launch_unpack_q4a(const zz_qtensor *t, uint8_t *dst, cudaStream_t st) {
    const long n = (long)t->O * (t->I / 64);
    k_unpack_q4a<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(t->codes, (const uint32_t *)t->scale, t->O, t->I, dst);
    return check_cuda(cudaGetLastError(), "q4a unpack launch");
}

// ---------------------------------------------------------------- q4a, int8 activations
// q4a_dot (tq2.h:395-408 scalar form): per 32-weight half-group h of group g,
// sx[2g+h] * (d * sum q*xq + m * sum xq). One warp per row, lane owns the groups
// g = lane, lane + 32, ...; two dp4a per 4 weights (codes, ones).
__global__ void __launch_bounds__(256) k_gemv_q4a(const uint8_t *__restrict__ codes, const uint32_t *__restrict__ scale,
                                                  int O, int I, const int8_t *__restrict__ xq,
                                                  const float *__restrict__ sx, float *__restrict__ y) {
    const int lane = threadIdx.x & 31, ng = I / 64;
    const int s = blockIdx.y;
    xq += (size_t)s * I;
    sx += (size_t)s * (I / 32);
    const int warps = (gridDim.x * blockDim.x) >> 5;
    for (int o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < O; o += warps) {
        float acc = 0.f;
        for (int g = lane; g < ng; g += 32) {
            const uint4 *cp = reinterpret_cast<const uint4 *>(codes + ((size_t)o * ng + g) * 32);
            const uint32_t sc = scale[(size_t)o * ng + g];
            const float d = __half2float(__ushort_as_half((unsigned short)(sc & 0xFFFF)));
            const float m = __half2float(__ushort_as_half((unsigned short)(sc >> 16)));
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint4 w = ldg_stream(cp + h);
                const int4 *xp = reinterpret_cast<const int4 *>(xq + (size_t)g * 64 + h * 32);
                const int4 x0 = xp[0], x1 = xp[1];
                const uint32_t wl[4] = {w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu};
                const uint32_t wh[4] = {(w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                        (w.w >> 4) & 0x0F0F0F0Fu};
                const int xl[4] = {x0.x, x0.y, x0.z, x0.w}, xh[4] = {x1.x, x1.y, x1.z, x1.w};
                int dp = 0, sv = 0;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    dp = __dp4a((int)wl[k], xl[k], dp);
                    dp = __dp4a((int)wh[k], xh[k], dp);
                    sv = __dp4a(0x01010101, xl[k], sv);
                    sv = __dp4a(0x01010101, xh[k], sv);
                }
                const float sb = sx[2 * g + h];
                acc = fmaf(sb * d, (float)dp, acc);
                acc = fmaf(sb * m, (float)sv, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) y[(size_t)s * O + o] = acc;
    }
}

// ---------------------------------------------------------------- f32 activations
// One CTA row of activations per blockIdx.y, staged in shared memory as xt[j][b] (element
// j of 32-block b), so the 32 lanes of a warp, each on its own block, read consecutive
// words. One warp per weight row; lane owns the blocks b = lane, lane + 32, ...
template <int FMT>
__device__ __forceinline__ float block_f32(const uint8_t *__restrict__ codes, const void *__restrict__ scale, int o,
                                           int nb, int b, const float *__restrict__ xt) {
    const float *x = xt + b;  // element j at x[j * nb]
    if (FMT == GPU_FMT_Q40 || FMT == GPU_FMT_Q4A) {
        // q4_0: block b of the row; q4a: half-group b (group b/2), same nibble order
        const uint4 w = ldg_stream(codes + ((size_t)o * nb + b) * 16);
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
        float s = 0.f, t = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const uint32_t byte = (wv[k >> 2] >> (8 * (k & 3))) & 0xFFu;
            const float lo = x[k * nb], hi = x[(k + 16) * nb];
            if (FMT == GPU_FMT_Q40) {
                s = fmaf((float)((int)(byte & 15) - 8), lo, s);
                s = fmaf((float)((int)(byte >> 4) - 8), hi, s);
            } else {
                s = fmaf((float)(byte & 15), lo, s);
                s = fmaf((float)(byte >> 4), hi, s);
                t += lo + hi;
            }
        }
        if (FMT == GPU_FMT_Q40) {
            const int nbp = (nb + 7) & ~7;
            return __half2float(reinterpret_cast<const __half *>(scale)[(size_t)o * nbp + b]) * s;
        }
        const uint32_t sc = reinterpret_cast<const uint32_t *>(scale)[(size_t)o * (nb / 2) + b / 2];
        const float d = __half2float(__ushort_as_half((unsigned short)(sc & 0xFFFF)));
        const float m = __half2float(__ushort_as_half((unsigned short)(sc >> 16)));
        return fmaf(d, s, m * t);
    } else if (FMT == GPU_FMT_Q80) {
        const uint4 w0 = ldg_stream(codes + ((size_t)o * nb + b) * 32), w1 = ldg_stream(codes + ((size_t)o * nb + b) * 32 + 16);
        const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 32; k++) s = fmaf((float)(int8_t)(wv[k >> 2] >> (8 * (k & 3))), x[k * nb], s);
        const int nbp = (nb + 7) & ~7;
        return __half2float(reinterpret_cast<const __half *>(scale)[(size_t)o * nbp + b]) * s;
    } else {
        // tq2: block b = half `b & 1` of 64-weight group b/2: byte k holds weights k, k+16,
        // k+32, k+48 at bits 0/2/4/6 (tq2.h:46-51); the row's alpha is applied by the caller
        const uint4 w = ldg_stream(codes + (size_t)o * (nb * 8) + (size_t)(b >> 1) * 16);
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
        const int sh = (b & 1) * 4;
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const uint32_t byte = (wv[k >> 2] >> (8 * (k & 3))) & 0xFFu;
            s = fmaf((float)((int)((byte >> sh) & 3) - 1), x[k * nb], s);
            s = fmaf((float)((int)((byte >> (sh + 2)) & 3) - 1), x[(k + 16) * nb], s);
        }
        return s;
    }
}

template <int FMT>
__global__ void __launch_bounds__(256) k_gemv_f32(const uint8_t *__restrict__ codes, const void *__restrict__ scale,
                                                  int O, int I, const float *__restrict__ x, float *__restrict__ y) {
    extern __shared__ float xt[];
    const int nb = I / 32, s = blockIdx.y;
    for (int i = threadIdx.x; i < I; i += blockDim.x) xt[(i & 31) * nb + (i >> 5)] = x[(size_t)s * I + i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warps = (gridDim.x * blockDim.x) >> 5;
    for (int o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < O; o += warps) {
        float acc = 0.f;
        for (int b = lane; b < nb; b += 32) acc += block_f32<FMT>(codes, scale, o, nb, b, xt);
        acc = warp_sum(acc);
        if (lane == 0) {
            if (FMT == GPU_FMT_TQ2) acc *= reinterpret_cast<const float *>(scale)[o];
            y[(size_t)s * O + o] = acc;
        }
    }
}

static int gemv_blocks(int O) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    const int need = (O + 7) / 8;  // 8 warps (rows in flight) per CTA
    return need < sms * 8 ? need : sms * 8;
}

// y[S, O] = W x with f32 activations x[S, I] (device pointers)
int launch_gemv_f32(const zz_qtensor *W, const float *x, int S, float *y, cudaStream_t st) {
    const int O = W->O, I = W->I;
    const size_t smem = (size_t)I * 4;
    if (smem > 200 * 1024) return fail("f32-activation matvec: I=%d too wide", I);
    dim3 grid(gemv_blocks(O), S);
    switch (W->fmt) {
        case GPU_FMT_Q40:
            if (smem > 48 * 1024 &&
                !check_cuda(cudaFuncSetAttribute(k_gemv_f32<GPU_FMT_Q40>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "f32 smem"))
                return 0;
            k_gemv_f32<GPU_FMT_Q40><<<grid, 256, smem, st>>>(W->codes, W->scale, O, I, x, y);
            break;
        case GPU_FMT_Q80:
            if (smem > 48 * 1024 &&
                !check_cuda(cudaFuncSetAttribute(k_gemv_f32<GPU_FMT_Q80>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "f32 smem"))
                return 0;
            k_gemv_f32<GPU_FMT_Q80><<<grid, 256, smem, st>>>(W->codes, W->scale, O, I, x, y);
            break;
        case GPU_FMT_TQ2:
            if (smem > 48 * 1024 &&
                !check_cuda(cudaFuncSetAttribute(k_gemv_f32<GPU_FMT_TQ2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "f32 smem"))
                return 0;
            k_gemv_f32<GPU_FMT_TQ2><<<grid, 256, smem, st>>>(W->codes, W->scale, O, I, x, y);
            break;
        default:
            if (smem > 48 * 1024 &&
                !check_cuda(cudaFuncSetAttribute(k_gemv_f32<GPU_FMT_Q4A>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "f32 smem"))
                return 0;
            k_gemv_f32<GPU_FMT_Q4A><<<grid, 256, smem, st>>>(W->codes, W->scale, O, I, x, y);
            break;
    }
    return check_cuda(cudaGetLastError(), "f32-activation matvec launch");
}

// q4a with int8 activations, S rows
int launch_gemv_q4a(const zz_qtensor *W, const int8_t *xq, const float *sx, int S, float *y, cudaStream_t st) {
    dim3 grid(gemv_blocks(W->O), S);
    k_gemv_q4a<<<grid, 256, 0, st>>>(W->codes, (const uint32_t *)W->scale, W->O, W->I, xq, sx, y);
    return check_cuda(cudaGetLastError(), "q4a matvec launch");
}

}  // namespace zz
