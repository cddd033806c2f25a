// zz_common.cuh -- shared device helpers for the sm_100a quantized-matrix kernels.
//
// Formats (all bit-compatible with the reference's on-disk/in-memory formats):
//   q4_0  block of 32 weights = fp16 d + 16 nibble bytes, w_j = d*(q_j-8); byte j holds
//         weight j (low nibble) and weight j+16 (high nibble)      (q40.h:12-16)
//   q8_0  block of 32 weights = fp16 d + 32 int8, w_j = d*q_j      (q40.h:322-330)
//   tq2   tensor = alpha[O] f32 then codes[O][I/4]; in each 64-weight group (16 B)
//         byte k holds weights k, k+16, k+32, k+48 at bits 0/2/4/6; w = alpha*(c-1)
//                                                                   (tq2.h:20-51, 81-91)
// In HBM every weight tensor lives as structure-of-arrays planes (zz_qtensor in
// include/zz_gpu.h): a 16-byte-aligned code plane with a fixed row stride, and a
// separate scale plane (fp16 per block, or f32 alpha per row for tq2).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include "../../include/zz_gpu.h"

#define ZZ_BLK 32

namespace zz {

// Row remap of a repack: mode 0 copies row r to row r; mode 1 builds the expert
// bank's gate/up stack (dst row r <- gate or up row (r/128)*64 + r%64 of one expert).
struct RowMap {
    int mode, inter;
    long src_tensor_bytes;  // bytes of one [inter, hidden] source tensor (mode 1)
};

// Records a readable error for gpu_last_error(); returns 0 so callers can
// `return zz::fail(...)` in the decline convention of gpu.h (gpu.h:71-84).
int fail(const char *fmt, ...);
int check_cuda(cudaError_t e, const char *what);

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }

// Signed q-8 bytes from 4 q4_0 nibbles held in the low half of each byte.
// (t | 0x80) - 8 cannot borrow across bytes; xor 0x80 restores the sign.
__device__ __forceinline__ uint32_t nib_to_s8(uint32_t t) {
    return (((t & 0x0F0F0F0Fu) | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async16_zfill(void *smem, const void *gmem, bool valid) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// q8_0 quantization of one 32-value block held one value per lane of a warp.
// Bit-exact with q40_quant_act (q40.h:124-138): amax over |v|, d = amax/127 (IEEE
// division), id = 1/d (IEEE), q = clamp(rne(v*id), +-127). No contraction is possible
// (a lone product feeds the rounding conversion).
__device__ __forceinline__ int8_t quant_lane(float v, float &d_out) {
    float a = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    float d = __fdiv_rn(a, 127.0f);
    float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = __float2int_rn(__fmul_rn(v, id));
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    d_out = d;
    return (int8_t)q;
}

}  // namespace zz
