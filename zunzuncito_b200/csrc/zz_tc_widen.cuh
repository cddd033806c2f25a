// zz_tc_widen.cuh -- weight-code widening for the tcgen05 expert kernels: one row's
// codes of one 32-weight block (held in 16-byte register chunks) become the 32 fp16
// values of that row in the UMMA K-major core-matrix layout. The fp16 values are the
// integer codes the reference multiplies (q4_0: q-8; q8_0: q; tq2: c in {0,1,2}).
#pragma once
#include "zz_gemm.cuh"

namespace zz {

// code bytes of one row for one stage (KB blocks); the TMA box is 128 rows of this
template <int FMT>
__host__ __device__ constexpr int tc_cb() { return FMT == GPU_FMT_Q40 ? 64 : FMT == GPU_FMT_Q80 ? 128 : 32; }

__device__ __forceinline__ uint32_t spread_lo(uint32_t w) { return __byte_perm(w, 0u, 0x4140u); }
__device__ __forceinline__ uint32_t spread_hi(uint32_t w) { return __byte_perm(w, 0u, 0x4342u); }

// widen one row's codes of block jj of the stage (in registers, 16-byte chunks of
// the row's stage bytes) into the block's 4 K-chunks of 8 fp16
template <int FMT>
__device__ __forceinline__ void widen_blk(const uint4 (&c)[tc_cb<FMT>() / 16], int jj, uint4 out[4]) {
    if (FMT == GPU_FMT_Q40) {
        const uint4 w = c[jj];
        // k 0-15: low nibbles of bytes 0-15; k 16-31: the high nibbles
        out[0] = make_uint4(q4lo_h2(spread_lo(w.x)), q4lo_h2(spread_hi(w.x)), q4lo_h2(spread_lo(w.y)), q4lo_h2(spread_hi(w.y)));
        out[1] = make_uint4(q4lo_h2(spread_lo(w.z)), q4lo_h2(spread_hi(w.z)), q4lo_h2(spread_lo(w.w)), q4lo_h2(spread_hi(w.w)));
        out[2] = make_uint4(q4hi_h2(spread_lo(w.x)), q4hi_h2(spread_hi(w.x)), q4hi_h2(spread_lo(w.y)), q4hi_h2(spread_hi(w.y)));
        out[3] = make_uint4(q4hi_h2(spread_lo(w.z)), q4hi_h2(spread_hi(w.z)), q4hi_h2(spread_lo(w.w)), q4hi_h2(spread_hi(w.w)));
    } else if (FMT == GPU_FMT_Q80) {
        const uint4 w0 = c[2 * jj], w1 = c[2 * jj + 1];
        out[0] = make_uint4(s8_h2(spread_lo(w0.x)), s8_h2(spread_hi(w0.x)), s8_h2(spread_lo(w0.y)), s8_h2(spread_hi(w0.y)));
        out[1] = make_uint4(s8_h2(spread_lo(w0.z)), s8_h2(spread_hi(w0.z)), s8_h2(spread_lo(w0.w)), s8_h2(spread_hi(w0.w)));
        out[2] = make_uint4(s8_h2(spread_lo(w1.x)), s8_h2(spread_hi(w1.x)), s8_h2(spread_lo(w1.y)), s8_h2(spread_hi(w1.y)));
        out[3] = make_uint4(s8_h2(spread_lo(w1.z)), s8_h2(spread_hi(w1.z)), s8_h2(spread_lo(w1.w)), s8_h2(spread_hi(w1.w)));
    } else {
        // tq2: a pair of blocks shares the 16 bytes of its 64-weight group; block jj's
        // codes sit at bit offset sh (k 0-15) and sh+2 (k 16-31), sh = 0 / 4 for the
        // even / odd block
        const uint4 w = c[jj >> 1];
        const int sh = (jj & 1) * 4;
        out[0] = make_uint4(c2_h2(spread_lo(w.x), sh), c2_h2(spread_hi(w.x), sh), c2_h2(spread_lo(w.y), sh), c2_h2(spread_hi(w.y), sh));
        out[1] = make_uint4(c2_h2(spread_lo(w.z), sh), c2_h2(spread_hi(w.z), sh), c2_h2(spread_lo(w.w), sh), c2_h2(spread_hi(w.w), sh));
        out[2] = make_uint4(c2_h2(spread_lo(w.x), sh + 2), c2_h2(spread_hi(w.x), sh + 2), c2_h2(spread_lo(w.y), sh + 2), c2_h2(spread_hi(w.y), sh + 2));
        out[3] = make_uint4(c2_h2(spread_lo(w.z), sh + 2), c2_h2(spread_hi(w.z), sh + 2), c2_h2(spread_lo(w.w), sh + 2), c2_h2(spread_hi(w.w), sh + 2));
    }
}

}  // namespace zz
