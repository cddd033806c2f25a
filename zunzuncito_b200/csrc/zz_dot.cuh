// zz_dot.cuh -- integer block dot products on CUDA cores (dp4a), shared by the decode
// matvec and the small-batch expert kernels.
#pragma once
#include "zz_common.cuh"

namespace zz {

// q4_0 block . q8_0 activation block, <q-8, x> (q40.h:162-187)
__device__ __forceinline__ int q40_block_dot(uint4 w, const uint32_t x[8]) {
    int s = 0;
    s = dp4a_ss((int)nib_to_s8(w.x), (int)x[0], s);
    s = dp4a_ss((int)nib_to_s8(w.y), (int)x[1], s);
    s = dp4a_ss((int)nib_to_s8(w.z), (int)x[2], s);
    s = dp4a_ss((int)nib_to_s8(w.w), (int)x[3], s);
    s = dp4a_ss((int)nib_to_s8(w.x >> 4), (int)x[4], s);
    s = dp4a_ss((int)nib_to_s8(w.y >> 4), (int)x[5], s);
    s = dp4a_ss((int)nib_to_s8(w.z >> 4), (int)x[6], s);
    s = dp4a_ss((int)nib_to_s8(w.w >> 4), (int)x[7], s);
    return s;
}
// q8_0 block . activation block (q40.h:359-372)
__device__ __forceinline__ int q80_block_dot(uint4 a, uint4 b, const uint32_t x[8]) {
    int s = 0;
    s = dp4a_ss((int)a.x, (int)x[0], s); s = dp4a_ss((int)a.y, (int)x[1], s);
    s = dp4a_ss((int)a.z, (int)x[2], s); s = dp4a_ss((int)a.w, (int)x[3], s);
    s = dp4a_ss((int)b.x, (int)x[4], s); s = dp4a_ss((int)b.y, (int)x[5], s);
    s = dp4a_ss((int)b.z, (int)x[6], s); s = dp4a_ss((int)b.w, (int)x[7], s);
    return s;
}
// tq2 64-weight group . two activation blocks: unsigned codes, <c, x> per block
// (tq2.h:116-133); x holds 16 words (blocks 2g, 2g+1)
__device__ __forceinline__ void tq2_group_dot(uint4 c, const uint32_t x[16], int &s0, int &s1) {
    const uint32_t m = 0x03030303u;
    s0 = 0; s1 = 0;
    s0 = dp4a_ss((int)(c.x & m), (int)x[0], s0);  s0 = dp4a_ss((int)(c.y & m), (int)x[1], s0);
    s0 = dp4a_ss((int)(c.z & m), (int)x[2], s0);  s0 = dp4a_ss((int)(c.w & m), (int)x[3], s0);
    s0 = dp4a_ss((int)((c.x >> 2) & m), (int)x[4], s0);  s0 = dp4a_ss((int)((c.y >> 2) & m), (int)x[5], s0);
    s0 = dp4a_ss((int)((c.z >> 2) & m), (int)x[6], s0);  s0 = dp4a_ss((int)((c.w >> 2) & m), (int)x[7], s0);
    s1 = dp4a_ss((int)((c.x >> 4) & m), (int)x[8], s1);  s1 = dp4a_ss((int)((c.y >> 4) & m), (int)x[9], s1);
    s1 = dp4a_ss((int)((c.z >> 4) & m), (int)x[10], s1); s1 = dp4a_ss((int)((c.w >> 4) & m), (int)x[11], s1);
    s1 = dp4a_ss((int)((c.x >> 6) & m), (int)x[12], s1); s1 = dp4a_ss((int)((c.y >> 6) & m), (int)x[13], s1);
    s1 = dp4a_ss((int)((c.z >> 6) & m), (int)x[14], s1); s1 = dp4a_ss((int)((c.w >> 6) & m), (int)x[15], s1);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// tq2: one 32-weight block = bit fields sh (k 0-15) and sh+2 (k 16-31) of its 64-weight
// group's 16 bytes, sh = 0 for the even block, 4 for the odd one; unsigned codes <c, x>
__device__ __forceinline__ int tq2_block_dot(uint4 c, int sh, const uint32_t x[8]) {
    const uint32_t m = 0x03030303u;
    int s = 0;
    s = dp4a_ss((int)((c.x >> sh) & m), (int)x[0], s);  s = dp4a_ss((int)((c.y >> sh) & m), (int)x[1], s);
    s = dp4a_ss((int)((c.z >> sh) & m), (int)x[2], s);  s = dp4a_ss((int)((c.w >> sh) & m), (int)x[3], s);
    s = dp4a_ss((int)((c.x >> (sh + 2)) & m), (int)x[4], s);  s = dp4a_ss((int)((c.y >> (sh + 2)) & m), (int)x[5], s);
    s = dp4a_ss((int)((c.z >> (sh + 2)) & m), (int)x[6], s);  s = dp4a_ss((int)((c.w >> (sh + 2)) & m), (int)x[7], s);
    return s;
}

}  // namespace zz
