// zz_quant.cu -- activation quantization, device weight quantizers and the
// reference-layout -> structure-of-arrays repack for q4_0 / q8_0 / tq2.
//
// All of it is byte/integer work bounded by HBM bandwidth: one warp per 32-value
// block, coalesced 16-byte stores, no shared-memory staging needed.
#include "zz_common.cuh"

namespace zz {

static inline size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t code_row_bytes(int fmt, int I) {
    return fmt == GPU_FMT_Q40 || fmt == GPU_FMT_Q4A ? (size_t)I / 2 : fmt == GPU_FMT_Q80 ? (size_t)I : (size_t)I / 4;
}
// fp16 block-scale rows are padded to a multiple of 8 blocks (16 bytes) so a K-chunk
// of scales is always one aligned piece; tq2 has one f32 alpha per row
int scale_ld(int I) { return ((I / ZZ_BLK) + 7) & ~7; }
size_t scale_row_bytes(int fmt, int I) {
    // q4a: one (fp16 d, fp16 m) pair per 64-weight group
    return fmt == GPU_FMT_TQ2 ? 4 : fmt == GPU_FMT_Q4A ? (size_t)(I / 64) * 4 : (size_t)scale_ld(I) * 2;
}
size_t ref_row_bytes(int fmt, int I) {  // bytes of one row in the reference layout
    return fmt == GPU_FMT_Q40 ? (size_t)(I / ZZ_BLK) * 18 : fmt == GPU_FMT_Q80 ? (size_t)(I / ZZ_BLK) * 34
         : fmt == GPU_FMT_Q4A ? (size_t)(I / 64) * 36 : (size_t)I / 4;
}
size_t ref_tensor_bytes(int fmt, int O, int I) {
    return fmt == GPU_FMT_TQ2 ? (size_t)O * 4 + (size_t)O * (I / 4) : (size_t)O * ref_row_bytes(fmt, I);
}
size_t codes_bytes(int fmt, int O, int I) { return align256((size_t)O * code_row_bytes(fmt, I)); }
size_t scales_bytes(int fmt, int O, int I) { return align256((size_t)O * scale_row_bytes(fmt, I)); }

// ---------------------------------------------------------------- activations
// Grid (rows, chunks of 8 blocks), one warp per 32-block (lane = element): every block
// of every row is in flight at once. Bit-exact with q40_quant_act (q40.h:124-138).
// xh (optional) receives the codes as fp16; zero_out (optional) is an fp32 [rows,
// zero_cols] buffer this pass clears (the MoE output, accumulated into afterwards).
__global__ void k_quant_act(const float *__restrict__ x, int I, int8_t *__restrict__ xq, float *__restrict__ sx,
                            __half *__restrict__ xh, float *__restrict__ zero_out, int zero_cols) {
    const int row = blockIdx.x, nb = I / ZZ_BLK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.y * 8 + warp;
    if (zero_out) {
        const int c = blockIdx.y * 256 + threadIdx.x;
        if (c < zero_cols) zero_out[(size_t)row * zero_cols + c] = 0.f;
    }
    if (b >= nb) return;
    float v = x[(size_t)row * I + b * ZZ_BLK + lane], d;
    int8_t q = quant_lane(v, d);
    xq[(size_t)row * I + b * ZZ_BLK + lane] = q;
    if (xh) xh[(size_t)row * I + b * ZZ_BLK + lane] = __int2half_rn(q);
    if (lane == 0) sx[(size_t)row * nb + b] = d;
}

// The same quantization with one thread per 32-block (rows contiguous, block t at
// element 32 t): eight 16-byte loads in flight per thread and no shuffles; the same
// operations per element as quant_lane, so the codes and scales are identical. Clears
// zero_out [S, I] (same shape as x) in the same pass.
__global__ void __launch_bounds__(128) k_quant_act_blk(const float *__restrict__ x, long nblk, int8_t *__restrict__ xq,
                                                       float *__restrict__ sx, float *__restrict__ zero_out) {
    const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nblk) return;
    const float4 *src = reinterpret_cast<const float4 *>(x + t * ZZ_BLK);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float4 f = src[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) a = fmaxf(a, fabsf(v[i]));
    const float d = __fdiv_rn(a, 127.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            int q = __float2int_rn(__fmul_rn(v[4 * i + k], id));
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            word |= (uint32_t)(q & 0xFF) << (8 * k);
        }
        w[i] = word;
    }
    uint4 *dst = reinterpret_cast<uint4 *>(xq + t * ZZ_BLK);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    sx[t] = d;
    if (zero_out) {
        float4 *z = reinterpret_cast<float4 *>(zero_out + t * ZZ_BLK);
#pragma unroll
        for (int i = 0; i < 8; i++) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// tq2 offset total of quantized rows: Sx = (float) sum_b (double)sx[b] * sum_j xq, summed
// serially in block order (tq2.h:103-107). One warp per row: lane l forms the integer sums
// of blocks l, l+32, ...; lane 0 then adds the double products in block order.
__global__ void k_rows_sx(const int8_t *__restrict__ xq, const float *__restrict__ xs, int S, int I,
                          float *__restrict__ xsx) {
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= S) return;
    const int nb = I / 32;
    double tot = 0;
    for (int b0 = 0; b0 < nb; b0 += 32) {
        const int b = b0 + lane;
        int s = 0;
        double prod = 0;
        if (b < nb) {
            const uint4 *q = reinterpret_cast<const uint4 *>(xq + (size_t)r * I + (size_t)b * 32);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint4 v = q[h];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; k++) s = __dp4a((int)w[k], 0x01010101, s);
            }
            prod = (double)xs[(size_t)r * nb + b] * (double)s;
        }
        const int n = nb - b0 < 32 ? nb - b0 : 32;
        for (int k = 0; k < n; k++) {
            const double p = __shfl_sync(0xffffffffu, prod, k);
            tot += p;
        }
    }
    if (lane == 0) xsx[r] = (float)tot;
}

// ---------------------------------------------------------------- weight quantizers
// q4_0 (q40.h:83-110): the element of largest |x| (first one on ties) sets
// d = fp16(mx / -8); q = clamp(trunc(x*(1/d) + 8.5), 0, 15), product and sum rounded
// separately as in C. q8_0 (q40.h:332-350): d = fp16(amax/127), q = rne(x*(1/d)).
template <int FMT>
__global__ void k_quant_rows(const float *__restrict__ w, long nblocks, uint8_t *__restrict__ dst) {
    const int lane = threadIdx.x & 31;
    long b = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (b >= nblocks) return;
    float v = w[b * ZZ_BLK + lane];
    float a = fabsf(v), amax = a;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (FMT == GPU_FMT_Q40) {
        unsigned hit = __ballot_sync(0xffffffffu, a == amax && amax > 0.f);
        float mx = __shfl_sync(0xffffffffu, v, hit ? __ffs(hit) - 1 : 0);
        if (!hit) mx = 0.f;
        __half hd = __float2half_rn(__fdiv_rn(mx, -8.0f));
        float d = __half2float(hd), id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q = __float2int_rz(__fadd_rn(__fmul_rn(v, id), 8.5f));
        q = q < 0 ? 0 : (q > 15 ? 15 : q);
        int hi = __shfl_down_sync(0xffffffffu, q, 16);
        uint8_t *blk = dst + b * 18;
        if (lane == 0) *reinterpret_cast<__half *>(blk) = hd;  // 2-byte aligned (18*b)
        if (lane < 16) blk[2 + lane] = (uint8_t)(q | (hi << 4));
    } else {
        __half hd = __float2half_rn(__fdiv_rn(amax, 127.0f));
        float d = __half2float(hd), id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q = __float2int_rn(__fmul_rn(v, id));
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        uint8_t *blk = dst + b * 34;
        if (lane == 0) *reinterpret_cast<__half *>(blk) = hd;
        blk[2 + lane] = (uint8_t)(int8_t)q;
    }
}

// ---------------------------------------------------------------- repack
// Row remaps let one kernel serve plain tensors and the interleaved gate/up stack.
// mode 0: dst row r <- src row r.
// mode 1: expert bank gate/up: dst row r of expert e <- gate row f or up row f of the
//         same expert, f = (r/128)*64 + r%64, up when r%128 >= 64.

__device__ __forceinline__ long src_row_offset(const RowMap &m, int fmt, int r, long rrow) {
    if (m.mode == 0) return (long)r * rrow;
    int g = r / 128, w = r % 128, f = g * 64 + (w & 63);
    return (w >= 64 ? m.src_tensor_bytes : 0) + (long)f * rrow;
}

// q4_0 / q8_0: one thread per block. codes gets the 16 (32) code bytes, scale the fp16.
template <int FMT>
__global__ void k_repack_q(const uint8_t *__restrict__ src, long src_expert_stride, int rows, int I,
                           RowMap map, uint8_t *__restrict__ codes, __half *__restrict__ scale,
                           long dst_expert_codes, long dst_expert_scale) {
    const int nb = I / ZZ_BLK;
    const int BB = FMT == GPU_FMT_Q40 ? 18 : 34, CB = FMT == GPU_FMT_Q40 ? 16 : 32;
    const long rrow = (long)nb * BB;
    long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int e = blockIdx.y;
    if (t >= (long)rows * nb) return;
    int r = (int)(t / nb), b = (int)(t % nb);
    const uint8_t *s = src + e * src_expert_stride + src_row_offset(map, FMT, r, rrow) + (long)b * BB;
    uint8_t *c = codes + e * dst_expert_codes + (long)r * nb * CB + (long)b * CB;
    const int nbp = (nb + 7) & ~7;
    scale[e * dst_expert_scale / 2 + (long)r * nbp + b] =
        __ushort_as_half((unsigned short)(s[0] | (s[1] << 8)));
    // 18-byte blocks only guarantee 2-byte alignment of the source
    const unsigned short *s2 = reinterpret_cast<const unsigned short *>(s + 2);
    unsigned short *c2 = reinterpret_cast<unsigned short *>(c);
#pragma unroll
    for (int i = 0; i < CB / 2; i++) c2[i] = s2[i];
}

// tq2: alphas (f32 per row) and code rows (I/4 bytes) are copied row-wise.
__global__ void k_repack_tq2(const uint8_t *__restrict__ src, long src_expert_stride, int rows, int I,
                             RowMap map, uint8_t *__restrict__ codes, float *__restrict__ alpha,
                             long dst_expert_codes, long dst_expert_scale) {
    const int rb = I / 4;
    const int r = blockIdx.x, e = blockIdx.y;
    if (r >= rows) return;
    const uint8_t *base = src + e * src_expert_stride;
    int f = r;
    long tensor = 0;
    int O = rows;
    if (map.mode == 1) {
        int g = r / 128, w = r % 128;
        f = g * 64 + (w & 63);
        tensor = w >= 64 ? map.src_tensor_bytes : 0;
        O = map.inter;
    }
    const uint8_t *T = base + tensor;
    if (threadIdx.x == 0)
        alpha[e * dst_expert_scale / 4 + r] = reinterpret_cast<const float *>(T)[f];
    const uint8_t *cs = T + (long)O * 4 + (long)f * rb;
    uint8_t *cd = codes + e * dst_expert_codes + (long)r * rb;
    for (int i = threadIdx.x; i < rb; i += blockDim.x) cd[i] = cs[i];
}

// planes -> reference layout (checks only)
template <int FMT>
__global__ void k_unpack_q(const uint8_t *__restrict__ codes, const __half *__restrict__ scale, int O, int I,
                           uint8_t *__restrict__ dst) {
    const int nb = I / ZZ_BLK;
    const int BB = FMT == GPU_FMT_Q40 ? 18 : 34, CB = FMT == GPU_FMT_Q40 ? 16 : 32;
    long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long)O * nb) return;
    uint8_t *d = dst + t * BB;
    const int nbp = (nb + 7) & ~7;
    unsigned short h = __half_as_ushort(scale[(t / nb) * nbp + t % nb]);
    d[0] = (uint8_t)(h & 255);
    d[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < CB; i++) d[2 + i] = codes[t * CB + i];
}

int launch_repack(int fmt, const uint8_t *src, long src_expert_stride, int rows, int I, RowMap map,
                  uint8_t *codes, void *scale, long dce, long dse, int n_experts, cudaStream_t st) {
    if (fmt == GPU_FMT_TQ2) {
        dim3 grid(rows, n_experts);
        k_repack_tq2<<<grid, 128, 0, st>>>(src, src_expert_stride, rows, I, map, codes, (float *)scale, dce, dse);
    } else {
        long n = (long)rows * (I / ZZ_BLK);
        dim3 grid((unsigned)((n + 255) / 256), n_experts);
        if (fmt == GPU_FMT_Q40)
            k_repack_q<GPU_FMT_Q40><<<grid, 256, 0, st>>>(src, src_expert_stride, rows, I, map, codes,
                                                          (__half *)scale, dce, dse);
        else
            k_repack_q<GPU_FMT_Q80><<<grid, 256, 0, st>>>(src, src_expert_stride, rows, I, map, codes,
                                                          (__half *)scale, dce, dse);
    }
    return check_cuda(cudaGetLastError(), "repack launch");
}

}  // namespace zz

using namespace zz;

static bool fmt_ok(int fmt, int I) {
    if (fmt == GPU_FMT_Q40 || fmt == GPU_FMT_Q80) return I > 0 && I % 32 == 0;
    if (fmt == GPU_FMT_TQ2 || fmt == GPU_FMT_Q4A) return I > 0 && I % 64 == 0;
    return false;
}
namespace zz {
int launch_repack_q4a(const uint8_t *src, int O, int I, uint8_t *codes, void *scale, cudaStream_t st);
int launch_unpack_q4a(const zz_qtensor *t, uint8_t *dst, cudaStream_t st);
}

extern "C" size_t zz_qtensor_bytes(int fmt, int O, int I) {
    if (!fmt_ok(fmt, I) || O <= 0) return 0;
    return codes_bytes(fmt, O, I) + scales_bytes(fmt, O, I);
}

extern "C" int zz_repack_dev(int fmt, const uint8_t *src, int O, int I, void *dst, zz_qtensor *out,
                             void *stream) {
    if (!fmt_ok(fmt, I) || O <= 0) return fail("zz_repack_dev: unsupported fmt %d or shape %dx%d", fmt, O, I);
    if (!src || !dst || !out) return fail("zz_repack_dev: null pointer");
    if ((uintptr_t)dst & 255) return fail("zz_repack_dev: dst must be 256-byte aligned");
    uint8_t *codes = (uint8_t *)dst;
    void *scale = codes + codes_bytes(fmt, O, I);
    if (fmt == GPU_FMT_Q4A) {
        if (!launch_repack_q4a(src, O, I, codes, scale, (cudaStream_t)stream)) return 0;
        out->fmt = fmt; out->O = O; out->I = I; out->codes = codes; out->scale = scale;
        return 1;
    }
    RowMap m{0, 0, 0};
    if (fmt != GPU_FMT_TQ2 &&
        !check_cuda(cudaMemsetAsync(scale, 0, scales_bytes(fmt, O, I), (cudaStream_t)stream), "repack memset"))
        return 0;
    if (!launch_repack(fmt, src, 0, O, I, m, codes, scale, 0, 0, 1, (cudaStream_t)stream)) return 0;
    out->fmt = fmt; out->O = O; out->I = I; out->codes = codes; out->scale = scale;
    return 1;
}

extern "C" int zz_unpack_dev(const zz_qtensor *t, uint8_t *dst, void *stream) {
    if (!t || !dst || !fmt_ok(t->fmt, t->I)) return fail("zz_unpack_dev: bad tensor");
    cudaStream_t st = (cudaStream_t)stream;
    if (t->fmt == GPU_FMT_Q4A) return launch_unpack_q4a(t, dst, st);
    if (t->fmt == GPU_FMT_TQ2) {
        if (!check_cuda(cudaMemcpyAsync(dst, t->scale, (size_t)t->O * 4, cudaMemcpyDeviceToDevice, st), "unpack"))
            return 0;
        return check_cuda(cudaMemcpyAsync(dst + (size_t)t->O * 4, t->codes, (size_t)t->O * (t->I / 4),
                                          cudaMemcpyDeviceToDevice, st), "unpack");
    }
    long n = (long)t->O * (t->I / ZZ_BLK);
    unsigned grid = (unsigned)((n + 255) / 256);
    if (t->fmt == GPU_FMT_Q40)
        k_unpack_q<GPU_FMT_Q40><<<grid, 256, 0, st>>>(t->codes, (const __half *)t->scale, t->O, t->I, dst);
    else
        k_unpack_q<GPU_FMT_Q80><<<grid, 256, 0, st>>>(t->codes, (const __half *)t->scale, t->O, t->I, dst);
    return check_cuda(cudaGetLastError(), "unpack launch");
}

extern "C" int zz_quant_rows_dev(int fmt, const float *w, int O, int I, uint8_t *dst, void *stream) {
    if ((fmt != GPU_FMT_Q40 && fmt != GPU_FMT_Q80) || !fmt_ok(fmt, I) || O <= 0)
        return fail("zz_quant_rows_dev: unsupported fmt %d or shape %dx%d", fmt, O, I);
    if (!w || !dst) return fail("zz_quant_rows_dev: null pointer");
    long nblocks = (long)O * (I / ZZ_BLK);
    unsigned grid = (unsigned)((nblocks * 32 + 255) / 256);
    cudaStream_t st = (cudaStream_t)stream;
    if (fmt == GPU_FMT_Q40) k_quant_rows<GPU_FMT_Q40><<<grid, 256, 0, st>>>(w, nblocks, dst);
    else k_quant_rows<GPU_FMT_Q80><<<grid, 256, 0, st>>>(w, nblocks, dst);
    return check_cuda(cudaGetLastError(), "quant_rows launch");
}

// int8 rows -> the same values as fp16 (activations that arrive already quantized)
__global__ void k_s8_to_h(const int8_t *__restrict__ q, __half *__restrict__ h, long n) {
    long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = __int2half_rn(q[i]);
}
namespace zz {
int launch_s8_to_h(const int8_t *q, __half *h, long n, cudaStream_t st) {
    if (n <= 0) return 1;
    k_s8_to_h<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(q, h, n);
    return check_cuda(cudaGetLastError(), "s8_to_h launch");
}
// quantize rows; xh (optional) receives the int8 codes as fp16 for the GEMM's B operand;
// zero_out (optional) [S, zero_cols] is cleared in the same pass
int launch_quant_act(const float *x, int S, int I, int8_t *xq, float *sx, float *sxtot, __half *xh,
                     cudaStream_t st, float *zero_out, int zero_cols) {
    const int nb = I / ZZ_BLK;
    const bool aligned = ((uintptr_t)x & 15) == 0 && ((uintptr_t)xq & 15) == 0 && ((uintptr_t)zero_out & 15) == 0;
    if (!xh && aligned && (!zero_out || zero_cols == I)) {
        const long nblk = (long)S * nb;
        k_quant_act_blk<<<(unsigned)((nblk + 127) / 128), 128, 0, st>>>(x, nblk, xq, sx, zero_out);
    } else {
        int gy = (nb + 7) / 8;
        if (zero_out) gy = max(gy, (zero_cols + 255) / 256);
        k_quant_act<<<dim3(S, gy), 256, 0, st>>>(x, I, xq, sx, xh, zero_out, zero_cols);
    }
    if (!check_cuda(cudaGetLastError(), "quant_act launch")) return 0;
    if (sxtot) {
        k_rows_sx<<<(S + 7) / 8, 256, 0, st>>>(xq, sx, S, I, sxtot);
        if (!check_cuda(cudaGetLastError(), "rows_sx launch")) return 0;
    }
    return 1;
}
}  // namespace zz

extern "C" int zz_quant_act_dev(const float *x, int S, int I, int8_t *xq, float *sx, float *sxtot,
                                void *stream) {
    if (S < 0 || I <= 0 || I % 32) return fail("zz_quant_act_dev: I=%d must be a positive multiple of 32", I);
    if (S == 0) return 1;
    if (!x || !xq || !sx) return fail("zz_quant_act_dev: null pointer");
    return launch_quant_act(x, S, I, xq, sx, sxtot, nullptr, (cudaStream_t)stream, nullptr, 0);
}
