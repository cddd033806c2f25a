// zz_ep.cu -- the byte layout of the expert-parallel exchange (no reference counterpart:
// the reference is single-process). One payload row per (destination rank d, token s):
//   q8_0 codes [D] | block scales f32 [D/32] | local expert ids i32 [K] | weights f32 [K]
// where the ids keep the token's experts held by d (id - d*per_rank) and are -1
// elsewhere, with weight 0. Rows are 4-byte aligned (D % 32 == 0); a destination's rows
// for tokens 0..S-1 are contiguous, so an equal-split all-to-all moves them.
#include "zz_common.cuh"

namespace zz {

__global__ void k_ep_pack(const int8_t *__restrict__ xq, const float *__restrict__ xs, const int32_t *__restrict__ eidx,
                          const float *__restrict__ ewt, int S, int D, int K, int world, int per, uint8_t *__restrict__ out) {
    const int s = blockIdx.x, nb = D / 32;
    const size_t rowb = (size_t)D + 4 * nb + 8 * K;
    const uint32_t *q = reinterpret_cast<const uint32_t *>(xq + (size_t)s * D);
    const uint32_t *sc = reinterpret_cast<const uint32_t *>(xs + (size_t)s * nb);
    for (int d = 0; d < world; d++) {
        uint32_t *row = reinterpret_cast<uint32_t *>(out + ((size_t)d * S + s) * rowb);
        for (int i = threadIdx.x; i < D / 4; i += blockDim.x) row[i] = q[i];
        for (int i = threadIdx.x; i < nb; i += blockDim.x) row[D / 4 + i] = sc[i];
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            const int e = eidx[(size_t)s * K + k];
            const bool mine = e >= 0 && e / per == d;
            row[D / 4 + nb + k] = (uint32_t)(mine ? e - d * per : -1);
            row[D / 4 + nb + K + k] = __float_as_uint(mine ? ewt[(size_t)s * K + k] : 0.f);
        }
    }
}

__global__ void k_ep_unpack(const uint8_t *__restrict__ in, int D, int K, int8_t *__restrict__ xq, float *__restrict__ xs,
                            int32_t *__restrict__ eidx, float *__restrict__ ewt) {
    const int r = blockIdx.x, nb = D / 32;
    const size_t rowb = (size_t)D + 4 * nb + 8 * K;
    const uint32_t *row = reinterpret_cast<const uint32_t *>(in + (size_t)r * rowb);
    uint32_t *q = reinterpret_cast<uint32_t *>(xq + (size_t)r * D);
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x) q[i] = row[i];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) xs[(size_t)r * nb + i] = __uint_as_float(row[D / 4 + i]);
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        eidx[(size_t)r * K + k] = (int32_t)row[D / 4 + nb + k];
        ewt[(size_t)r * K + k] = __uint_as_float(row[D / 4 + nb + K + k]);
    }
}

}  // namespace zz

extern "C" size_t zz_ep_row_bytes(int D, int K) { return (size_t)D + 4 * (size_t)(D / 32) + 8 * (size_t)K; }

extern "C" int zz_ep_pack_dev(const int8_t *xq, const float *xs, const int32_t *eidx, const float *ewt, int S, int D,
                              int K, int world, int per_rank, uint8_t *payload, void *stream) {
    using namespace zz;
    if (S < 0 || D <= 0 || D % 32 || K <= 0 || world <= 0 || per_rank <= 0) return fail("zz_ep_pack_dev: bad shape");
    if (S == 0) return 1;
    if (!xq || !xs || !eidx || !ewt || !payload) return fail("zz_ep_pack_dev: null pointer");
    if (((uintptr_t)xq | (uintptr_t)xs | (uintptr_t)payload) & 3) return fail("zz_ep_pack_dev: pointers must be 4-byte aligned");
    k_ep_pack<<<S, 256, 0, (cudaStream_t)stream>>>(xq, xs, eidx, ewt, S, D, K, world, per_rank, payload);
    return check_cuda(cudaGetLastError(), "ep pack launch");
}

extern "C" int zz_ep_unpack_dev(const uint8_t *rows, int R, int D, int K, int8_t *xq, float *xs, int32_t *eidx,
                                float *ewt, void *stream) {
    using namespace zz;
    if (R < 0 || D <= 0 || D % 32 || K <= 0) return fail("zz_ep_unpack_dev: bad shape");
    if (R == 0) return 1;
    if (!rows || !xq || !xs || !eidx || !ewt) return fail("zz_ep_unpack_dev: null pointer");
    if (((uintptr_t)rows | (uintptr_t)xq) & 3) return fail("zz_ep_unpack_dev: pointers must be 4-byte aligned");
    k_ep_unpack<<<R, 256, 0, (cudaStream_t)stream>>>(rows, D, K, xq, xs, eidx, ewt);
    return check_cuda(cudaGetLastError(), "ep unpack launch");
}
