// zz_moe.cu -- dense matvec dispatch, expert-bank packing and the batch-union
// routed-expert FFN (device counterpart of gemma4.c:618-711 + 750-790 and
// maple.c:612-692, 738-790).
//
// Layer pipeline on one stream, no host round trip:
//   1. quantize X once per token (the engines re-quantize per (token, expert); the
//      bytes are identical, gemma4.c:642)
//   2. route: histogram of expert ids -> offsets -> pair slots grouped by expert, and
//      the work list of (expert, <=BN pairs) items  -- replaces moe_start's O(S*K*nu)
//      union scan and moe_apply_chunk's gather (gemma4.c:756-761, 781-783)
//   3. gate/up GEMM over the interleaved [2*inter, hidden] stack, fused activation and
//      q8_0 requant of h (gemma4.c:637-644)
//   4. down GEMM with the router weight and the scatter-add into OUT fused into its
//      epilogue (gemma4.c:647-651)
// Each distinct expert's weights cross HBM once per item; items of one expert are
// adjacent in the grid so repeated reads of the same expert hit L2.
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <vector>
#include "zz_gemm.cuh"

namespace zz {

size_t code_row_bytes(int fmt, int I);
size_t scale_row_bytes(int fmt, int I);
size_t ref_tensor_bytes(int fmt, int O, int I);
size_t codes_bytes(int fmt, int O, int I);
size_t scales_bytes(int fmt, int O, int I);
int launch_repack(int fmt, const uint8_t *src, long src_expert_stride, int rows, int I, RowMap map,
                  uint8_t *codes, void *scale, long dce, long dse, int n_experts, cudaStream_t st);
int launch_gemv1(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float *y,
                 cudaStream_t st);
int launch_blocksums(const zz_qtensor *W, const int8_t *xq, int32_t *out, cudaStream_t st);
int launch_quant_act(const float *x, int S, int I, int8_t *xq, float *sx, float *sxtot, __half *xh,
                     cudaStream_t st, float *zero_out, int zero_cols);
int launch_s8_to_h(const int8_t *q, __half *h, long n, cudaStream_t st);
__global__ void k_rows_sx(const int8_t *__restrict__ xq, const float *__restrict__ xs, int S, int I,
                          float *__restrict__ xsx);
int launch_moe_i8(int fmt, int epi, const GemmArgs &a, int n_groups, int *err, cudaStream_t st);
bool moe_i8_supported(int fmt, int D, int MI);
int launch_moe_h3(int epi, const GemmArgs &a, int n_groups, int *err, cudaStream_t st);
int launch_split_rows(const int *pair_src, int K, const int8_t *xq, const float *xs, int D, int cap, __half *xhs,
                      int *err, cudaStream_t st);
bool moe_h3_supported(int fmt, int D, int MI);
int launch_moe_dec(int fmt, const GemmArgs &gu, const GemmArgs &dn, int P, float *hbuf, cudaStream_t st);

// Expert engine. Default ("auto"): the small-batch GEMV kernels (zz_moe_dec.cu) when
// S*K <= DEC_MAX_PAIRS; else the int8 mma.sync GEMM (k_gemm<..., S8>) with work items of
// up to 32 routed rows; when the experts average at least WIDE_PAIRS_PER_EXPERT rows
// (prefill), 64-row items with the gate/up GEMM on mma.sync and the down GEMM on the
// folded-scale tcgen05 engine (hyb; q4_0 banks, else both on mma.sync). At S=512 top-8
// the narrow mma.sync items are the fastest. ZZ_MOE_KERNEL=i8
// selects the int8 tcgen05 engine (zz_moe_i8.cu) where the layer's shape allows it;
// =mma8 / =mma8w force the narrow / wide mma.sync items; =h3 the folded-scale fp16
// tcgen05 engine (zz_moe_h3.cu, q4_0 banks); =hyb the wide mma.sync gate/up GEMM (which
// then also writes the hidden rows' fp16 planes) followed by the h3 down GEMM. The int8
// engines are exact per block; h3 carries every product to a relative 2^-21.
enum { ENG_DEC = 0, ENG_MMA8 = 3, ENG_I8 = 5, ENG_MMA8W = 6, ENG_H3 = 7, ENG_HYB = 8 };
constexpr int DEC_MAX_PAIRS = 64, WIDE_PAIRS_PER_EXPERT = 128;
static int moe_engine(int P, const zz_expert_bank *b) {
    const char *e = getenv("ZZ_MOE_KERNEL");
    const bool i8_ok = moe_i8_supported(b->fmt, b->hidden, b->inter);
    if (e && !strcmp(e, "mma8")) return ENG_MMA8;
    if (e && !strcmp(e, "mma8w")) return ENG_MMA8W;
    if (e && !strcmp(e, "i8")) return i8_ok ? ENG_I8 : ENG_MMA8;
    if (e && !strcmp(e, "h3")) return moe_h3_supported(b->fmt, b->hidden, b->inter) ? ENG_H3 : ENG_MMA8;
    if (e && !strcmp(e, "hyb")) return moe_h3_supported(b->fmt, b->hidden, b->inter) ? ENG_HYB : ENG_MMA8W;
    // the decode kernels take calls of up to DEC_MAX_PAIRS pairs
    if (P <= DEC_MAX_PAIRS) return ENG_DEC;
    if ((long)P < (long)WIDE_PAIRS_PER_EXPERT * b->n_experts) return ENG_MMA8;
    // prefill: the wide mma.sync gate/up GEMM and the tcgen05 down GEMM (S=4096 Gemma-4
    // layer 1.83 ms against 1.98 with both GEMMs on mma.sync)
    return moe_h3_supported(b->fmt, b->hidden, b->inter) ? ENG_HYB : ENG_MMA8W;
}
constexpr int I8_BN = 128, H3_BN = 64;

constexpr int MOE_BN = 32, MOE_BN_WIDE = 64;
constexpr int ROW_ALIGN = 4;
constexpr int DEC_BN = 2;      // rows per work item of the small-batch kernels (DEC_C)
constexpr int DENSE_BN = 64;

static inline size_t a256(size_t n) { return (n + 255) & ~(size_t)255; }

template <int FMT, int BN, int EPI, bool BH, bool S8, bool STRIDE>
static int launch_gemm_k(const GemmArgs &a, dim3 grid, cudaStream_t st) {
    constexpr int smem = GemmSmem<FMT, BN, BH, S8>::TOTAL;
    static bool attr_set = false;  // per process; the library drives one device
    if (!attr_set) {
        if (!check_cuda(cudaFuncSetAttribute(k_gemm<FMT, BN, EPI, BH, S8, STRIDE>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                        "gemm smem attribute"))
            return 0;
        attr_set = true;
    }
    k_gemm<FMT, BN, EPI, BH, S8, STRIDE><<<grid, G_THREADS, smem, st>>>(a);
    return check_cuda(cudaGetLastError(), "gemm launch");
}

// grid.y = the worst-case item count, or fewer rows and the striding kernel when that
// count exceeds about sixteen waves of 4 CTAs per SM (k_gemm finds the real count on the
// device; the worst case counts every routing slot, valid or not)
template <int FMT, int BN, int EPI, bool BH, bool S8>
static int launch_gemm_t(const GemmArgs &a, dim3 grid, cudaStream_t st) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    const unsigned cap = (unsigned)(sms * 4 * 16 / (grid.x > 0 ? (int)grid.x : 1));
    if (a.n_items && cap > 0 && grid.y > cap) {
        grid.y = cap;
        return launch_gemm_k<FMT, BN, EPI, BH, S8, true>(a, grid, st);
    }
    return launch_gemm_k<FMT, BN, EPI, BH, S8, false>(a, grid, st);
}

template <int EPI, int BN, bool BH, bool S8 = false>
static int launch_gemm(int fmt, const GemmArgs &a, dim3 grid, cudaStream_t st) {
    if (fmt == GPU_FMT_Q40) return launch_gemm_t<GPU_FMT_Q40, BN, EPI, BH, S8>(a, grid, st);
    if (fmt == GPU_FMT_Q80) return launch_gemm_t<GPU_FMT_Q80, BN, EPI, BH, S8>(a, grid, st);
    return launch_gemm_t<GPU_FMT_TQ2, BN, EPI, BH, S8>(a, grid, st);
}

// ---------------------------------------------------------------- routing
// One CTA. Pairs p = s*K + k with a valid expert go to slot off[e] + rank; the rank
// order inside an expert is arbitrary (each pair's result is independent of its slot).
// block-wide exclusive scan of v (one value per thread, blockDim.x == 1024)
__device__ __forceinline__ int block_excl_scan(int v, int *warp_tot, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int t = warp_tot[lane];
        int u = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, u, o);
            if (lane >= o) u += y;
        }
        warp_tot[lane] = u - t;  // exclusive prefix of warp totals
        if (lane == 31) warp_tot[32] = u;
    }
    __syncthreads();
    total = warp_tot[32];
    int r = x - v + warp_tot[warp];
    __syncthreads();
    return r;
}

// One CTA of 1024 threads. Pairs p = s*K + k with a valid expert go to row off[e] + rank
// (rank order inside an expert is arbitrary: each pair's result is independent of its
// row); each expert's rows start on a ROW_ALIGN boundary and padding rows get src -1.
// Also clears the tensor-core error word of the call. E <= 2048.
// With `sorted`, the items are listed in decreasing row count (full items first, then
// the partial ones by size), so a grid striding over them hands every CTA a similar mix
// of large and small tiles; BN <= 1024 then.
__global__ void __launch_bounds__(1024) k_route(const int32_t *__restrict__ eidx, const float *__restrict__ ewt,
                                                int P, int E, int BN, int cap, int *__restrict__ pair_src,
                                                float *__restrict__ pair_w, WorkItem *__restrict__ items,
                                                int *__restrict__ n_items, int *__restrict__ tcerr, int sorted) {
    extern __shared__ int sh[];
    int *cnt = sh, *off = sh + E, *ioff = sh + 2 * E, *cur = sh + 3 * E;
    __shared__ int warp_tot[33];
    __shared__ int bin_start[1025], bin_cur[1025];
    for (int e = threadIdx.x; e < E; e += blockDim.x) { cnt[e] = 0; cur[e] = 0; }
    if (threadIdx.x == 0) *tcerr = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        int e = eidx[p];
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    // each thread owns experts 2t and 2t+1 (E <= 2048)
    const int e0 = 2 * threadIdx.x, e1 = e0 + 1;
    const int c0 = e0 < E ? cnt[e0] : 0, c1 = e1 < E ? cnt[e1] : 0;
    const int a0 = (c0 + ROW_ALIGN - 1) / ROW_ALIGN * ROW_ALIGN, a1 = (c1 + ROW_ALIGN - 1) / ROW_ALIGN * ROW_ALIGN;
    const int i0 = (c0 + BN - 1) / BN, i1 = (c1 + BN - 1) / BN;
    int rows_total, items_total;
    const int ro = block_excl_scan(a0 + a1, warp_tot, rows_total);
    const int io = block_excl_scan(i0 + i1, warp_tot, items_total);
    if (e0 < E) { off[e0] = ro; ioff[e0] = io; }
    if (e1 < E) { off[e1] = ro + a0; ioff[e1] = io + i0; }
    if (threadIdx.x == 0) *n_items = items_total;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        int e = eidx[p];
        if (e >= 0 && e < E) {
            int pos = off[e] + atomicAdd(&cur[e], 1);
            pair_src[pos] = p;
            pair_w[pos] = ewt[p];
        }
    }
    if (!sorted) {
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            int c = cnt[e], ni = (c + BN - 1) / BN;
            for (int i = 0; i < ni; i++) items[ioff[e] + i] = WorkItem{e, off[e] + i * BN, min(BN, c - i * BN), 0};
        }
    } else {
        // full items (BN rows) first, at an exclusive scan of the experts' full counts;
        // then one bin per remainder size r = BN-1 .. 1
        const int f0 = e0 < E ? cnt[e0] / BN : 0, f1 = e1 < E ? cnt[e1] / BN : 0;
        int n_full;
        const int fo = block_excl_scan(f0 + f1, warp_tot, n_full);
        for (int r = threadIdx.x; r <= BN; r += blockDim.x) bin_cur[r] = 0;
        __syncthreads();
        for (int e = threadIdx.x; e < E; e += blockDim.x)
            if (cnt[e] % BN) atomicAdd(&bin_cur[cnt[e] % BN], 1);
        __syncthreads();
        if (threadIdx.x == 0) {
            int o = n_full;
            for (int r = BN - 1; r >= 1; r--) { bin_start[r] = o; o += bin_cur[r]; bin_cur[r] = 0; }
        }
        __syncthreads();
        if (e0 < E) for (int i = 0; i < f0; i++) items[fo + i] = WorkItem{e0, off[e0] + i * BN, BN, 0};
        if (e1 < E) for (int i = 0; i < f1; i++) items[fo + f0 + i] = WorkItem{e1, off[e1] + i * BN, BN, 0};
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            const int c = cnt[e], rem = c % BN;
            if (rem) items[bin_start[rem] + atomicAdd(&bin_cur[rem], 1)] = WorkItem{e, off[e] + (c / BN) * BN, rem, 0};
        }
    }
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int c = cnt[e];
        int pad_end = off[e] + (c + ROW_ALIGN - 1) / ROW_ALIGN * ROW_ALIGN;
        for (int r = off[e] + c; r < pad_end; r++) pair_src[r] = -1;
    }
    for (int r = rows_total + threadIdx.x; r < cap; r += blockDim.x) pair_src[r] = -1;
}

__global__ void k_count_bad(const int32_t *eidx, int P, int E, int *bad) {
    int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p < P && (eidx[p] < 0 || eidx[p] >= E)) atomicAdd(bad, 1);
}

// pair rows incl. alignment padding; a multiple of ROW_ALIGN
static inline size_t pair_cap(size_t P, int E) { return (P + (size_t)ROW_ALIGN * E + 15) / 16 * 16; }

// routed rows in pair order for the int8 tensor-core engine: xg8[r] = xq[token(r)] and the
// block scales transposed, xsT[b][r] = xs[token(r)][b] (bulk-copy friendly)
__global__ void k_gather_rows8(const int *__restrict__ pair_src, int K, const int8_t *__restrict__ xq,
                               const float *__restrict__ xs, int D, int8_t *__restrict__ xg8, float *__restrict__ xsT,
                               int ldT) {
    const int r = blockIdx.x;
    const int src = pair_src[r];
    if (src < 0) return;
    const int tok = src / K, nb = D / 32;
    const uint4 *a = reinterpret_cast<const uint4 *>(xq + (size_t)tok * D);
    uint4 *b = reinterpret_cast<uint4 *>(xg8 + (size_t)r * D);
    for (int i = threadIdx.x; i < D / 16; i += blockDim.x) b[i] = a[i];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) xsT[(size_t)i * ldT + r] = xs[(size_t)tok * nb + i];
}

struct MoeWs {
    int8_t *xq; float *xs, *xsx;
    int *pair_src; float *pair_w;
    int8_t *xg8; float *xsT, *hsT; size_t cap, ldT;
    WorkItem *items; int *n_items;
    int8_t *hq; float *hs; int *hblk; float *hf;
    __half *xhs, *hhs;  // h3 engine: fp16 (hi, lo) operand planes of the pair rows
    int *bad;
    int *tcerr;
    size_t total;
};

// Scratch of one layer call. Pair rows (cap) count every routed (token, expert) pair
// plus each expert's padding to ROW_ALIGN rows; per pair row: the gathered int8
// activation row (D), its block scales transposed (D/32 f32), the requantized hidden
// row (MI int8 + MI/32 f32 scales, also transposed, + MI/32 int block sums for tq2).
// The decode engine's f32 hidden rows exist only for calls it takes (S*K <= 64 pairs);
// the h3 engine's fp16 operand planes (hi and lo of every gathered activation row and
// requantized hidden row, 4 bytes per element) only for calls it takes.
static MoeWs moe_layout(const zz_expert_bank *b, int S, int K, uint8_t *base) {
    MoeWs w{};
    const int D = b->hidden, MI = b->inter, E = b->n_experts;
    // items: at most P / (smallest item size) + one partial item per expert
    const size_t P = (size_t)S * K, maxit = P / DEC_BN + E + 1;
    const size_t cap = pair_cap(P, E), ldT = cap + 128;
    w.cap = cap;
    w.ldT = ldT;
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o += a256(n); return base ? base + r : nullptr; };
    w.xq = (int8_t *)take((size_t)S * D);
    w.xs = (float *)take((size_t)S * (D / 32) * 4);
    w.xsx = (float *)take((size_t)S * 4);
    w.pair_src = (int *)take(cap * 4);
    w.pair_w = (float *)take(cap * 4);
    w.xg8 = (int8_t *)take(cap * D);
    w.xsT = (float *)take((size_t)(D / 32) * ldT * 4);
    w.hsT = (float *)take((size_t)(MI / 32) * ldT * 4);
    w.items = (WorkItem *)take(maxit * sizeof(WorkItem));
    w.n_items = (int *)take(4);
    w.hq = (int8_t *)take(cap * MI);
    w.hs = (float *)take(cap * (MI / 32) * 4);
    w.hblk = (int *)take(cap * (MI / 32) * 4);
    w.hf = (float *)take(P <= (size_t)DEC_MAX_PAIRS ? cap * MI * 4 : 0);
    const int eng = moe_engine((int)P, b);
    w.xhs = (__half *)take(eng == ENG_H3 ? cap * D * 4 : 0);
    w.hhs = (__half *)take(eng == ENG_H3 || eng == ENG_HYB ? cap * MI * 4 : 0);
    w.bad = (int *)take(4);
    w.tcerr = (int *)take(4);
    w.total = o;
    return w;
}

// ---- optional stage timing (diagnostic): events at the stage boundaries of every
// zz_moe_ffn_dev call while enabled; summed on collection.
struct StageProf {
    bool on = false;
    std::vector<cudaEvent_t> ev;  // 4 per call: start, after route, after gate/up, after down
};
static StageProf g_prof;

static void prof_mark(cudaStream_t st) {
    if (!g_prof.on) return;
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return;
    cudaEventRecord(e, st);
    g_prof.ev.push_back(e);
}

}  // namespace zz

using namespace zz;

extern "C" int zz_prof_enable(int on) {
    g_prof.on = on != 0;
    return 1;
}

extern "C" int zz_prof_collect(float *stage_ms, int *calls) {
    if (!stage_ms || !calls) return fail("zz_prof_collect: null pointer");
    stage_ms[0] = stage_ms[1] = stage_ms[2] = 0.f;
    *calls = 0;
    size_t n = g_prof.ev.size() / 4 * 4;
    if (n && !check_cuda(cudaEventSynchronize(g_prof.ev[n - 1]), "prof sync")) return 0;
    for (size_t i = 0; i < n; i += 4) {
        for (int k = 0; k < 3; k++) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, g_prof.ev[i + k], g_prof.ev[i + k + 1]);
            stage_ms[k] += ms;
        }
        (*calls)++;
    }
    for (cudaEvent_t e : g_prof.ev) cudaEventDestroy(e);
    g_prof.ev.clear();
    return 1;
}

static bool bank_ok(const zz_expert_bank *b) {
    if (!b) return false;
    if (b->fmt != GPU_FMT_Q40 && b->fmt != GPU_FMT_Q80 && b->fmt != GPU_FMT_TQ2) return false;
    return b->n_experts > 0 && b->n_experts <= 2048 && b->hidden > 0 && b->inter > 0 && b->hidden % 128 == 0 &&
           b->inter % 64 == 0;
}

extern "C" size_t zz_expert_bank_bytes(int fmt, int E, int D, int MI) {
    zz_expert_bank b{fmt, E, D, MI, nullptr, nullptr, nullptr, nullptr};
    if (!bank_ok(&b)) return 0;
    return (size_t)E * (codes_bytes(fmt, 2 * MI, D) + scales_bytes(fmt, 2 * MI, D) + codes_bytes(fmt, D, MI) +
                        scales_bytes(fmt, D, MI));
}

extern "C" int zz_expert_bank_pack_dev(int fmt, int E, int D, int MI, const uint8_t *blobs, int64_t blob_stride,
                                       void *dst, zz_expert_bank *out, void *stream) {
    zz_expert_bank b{fmt, E, D, MI, nullptr, nullptr, nullptr, nullptr};
    if (!bank_ok(&b)) return fail("zz_expert_bank_pack_dev: unsupported fmt %d / shape E=%d D=%d MI=%d", fmt, E, D, MI);
    if (!blobs || !dst || !out) return fail("zz_expert_bank_pack_dev: null pointer");
    if ((uintptr_t)dst & 255) return fail("zz_expert_bank_pack_dev: dst must be 256-byte aligned");
    if ((uintptr_t)blobs & 3 || blob_stride & 3) return fail("zz_expert_bank_pack_dev: blobs must be 4-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t gc = codes_bytes(fmt, 2 * MI, D), gs = scales_bytes(fmt, 2 * MI, D);
    const size_t dc = codes_bytes(fmt, D, MI), ds = scales_bytes(fmt, D, MI);
    uint8_t *p = (uint8_t *)dst;
    uint8_t *gu_codes = p, *gu_scale = p + (size_t)E * gc;
    uint8_t *dn_codes = gu_scale + (size_t)E * gs, *dn_scale = dn_codes + (size_t)E * dc;
    if (!check_cuda(cudaMemsetAsync(gu_scale, 0, (size_t)E * gs, st), "bank memset")) return 0;
    if (!check_cuda(cudaMemsetAsync(dn_scale, 0, (size_t)E * ds, st), "bank memset")) return 0;
    const size_t gate_b = ref_tensor_bytes(fmt, MI, D);
    RowMap gu{1, MI, (long)gate_b};
    if (!launch_repack(fmt, blobs, blob_stride, 2 * MI, D, gu, gu_codes, gu_scale, (long)gc, (long)gs, E, st)) return 0;
    RowMap dn{0, 0, 0};
    if (!launch_repack(fmt, blobs + 2 * gate_b, blob_stride, D, MI, dn, dn_codes, dn_scale, (long)dc, (long)ds, E, st))
        return 0;
    *out = zz_expert_bank{fmt, E, D, MI, gu_codes, gu_scale, dn_codes, dn_scale};
    return 1;
}

extern "C" size_t zz_moe_workspace_bytes(const zz_expert_bank *b, int S, int K) {
    if (!bank_ok(b) || S < 0 || K <= 0) return 0;
    return moe_layout(b, S, K, nullptr).total;
}

extern "C" size_t zz_moe_workspace_offset(const zz_expert_bank *b, int S, int K, int which) {
    if (!bank_ok(b) || S <= 0 || K <= 0) return (size_t)-1;
    uint8_t *base = reinterpret_cast<uint8_t *>((uintptr_t)4096);  // offsets only; never dereferenced
    MoeWs w = moe_layout(b, S, K, base);
    const void *p = which == 0 ? (const void *)w.pair_src : which == 1 ? (const void *)w.pair_w
                  : which == 2 ? (const void *)w.hq : which == 3 ? (const void *)w.hs
                  : which == 4 ? (const void *)w.n_items : which == 5 ? (const void *)w.tcerr : nullptr;
    if (which == 6) return w.cap;
    if (!p) return (size_t)-1;
    return (size_t)((const uint8_t *)p - base);
}

// A side stream (one per host thread and device) on which the routing kernel runs
// concurrently with the activation quantization: fork and join by events, so it is
// stream-ordered with the caller's stream and capturable into a CUDA graph. Streams and
// events belong to the device that was current when they were created, so each device
// a thread drives gets its own set.
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    bool ok() {
        if (s) return true;
        return cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess &&
               cudaEventCreateWithFlags(&fork, cudaEventDisableTiming) == cudaSuccess &&
               cudaEventCreateWithFlags(&join, cudaEventDisableTiming) == cudaSuccess;
    }
};
constexpr int MAX_DEVICES = 64;
static thread_local SideStream g_side_dev[MAX_DEVICES];
// the current device's side stream, or nullptr (error recorded)
static SideStream *side_stream() {
    int dev = 0;
    if (!check_cuda(cudaGetDevice(&dev), "zz_moe_ffn: cudaGetDevice")) return nullptr;
    if (dev < 0 || dev >= MAX_DEVICES) {
        fail("zz_moe_ffn: device %d out of range", dev);
        return nullptr;
    }
    SideStream *s = &g_side_dev[dev];
    if (!s->ok()) {
        fail("zz_moe_ffn: side stream");
        return nullptr;
    }
    return s;
}

// X != NULL: f32 rows quantized here; else xq/xs are q8_0 rows given by the caller.
static int moe_impl(const zz_expert_bank *b, const float *X, const int8_t *xq_in, const float *xs_in,
                    const int32_t *eidx, const float *ewt, float *OUT, int S, int K, int act, float clamp,
                    void *workspace, size_t ws_bytes, int validate, void *stream) {
    if (!bank_ok(b)) return fail("zz_moe_ffn: invalid expert bank");
    if (S < 0 || K <= 0 || K > 64) return fail("zz_moe_ffn: bad S=%d or K=%d", S, K);
    if (act < ZZ_ACT_GEGLU_TANH || act > ZZ_ACT_SWIGLU_CLAMP) return fail("zz_moe_ffn: bad act %d", act);
    if ((long)S * K > (1L << 26)) return fail("zz_moe_ffn: S*K too large");
    if (S == 0) return 1;
    if ((!X && (!xq_in || !xs_in)) || !eidx || !ewt || !OUT || !workspace) return fail("zz_moe_ffn: null pointer");
    if ((uintptr_t)workspace & 255) return fail("zz_moe_ffn: workspace must be 256-byte aligned");
    MoeWs need = moe_layout(b, S, K, nullptr);
    if (ws_bytes < need.total) return fail("zz_moe_ffn: workspace %zu < %zu bytes", ws_bytes, need.total);
    MoeWs w = moe_layout(b, S, K, (uint8_t *)workspace);
    cudaStream_t st = (cudaStream_t)stream;
    const int fmt = b->fmt, D = b->hidden, MI = b->inter, E = b->n_experts, P = S * K;

    if (validate) {
        int bad = 0;
        if (!check_cuda(cudaMemsetAsync(w.bad, 0, 4, st), "memset")) return 0;
        k_count_bad<<<(P + 255) / 256, 256, 0, st>>>(eidx, P, E, w.bad);
        if (!check_cuda(cudaMemcpyAsync(&bad, w.bad, 4, cudaMemcpyDeviceToHost, st), "copy") ||
            !check_cuda(cudaStreamSynchronize(st), "sync"))
            return 0;
        if (bad) return fail("zz_moe_ffn: %d expert ids outside [0, %d)", bad, E);
    }
    prof_mark(st);
    const int eng = moe_engine(P, b);
    const bool hyb = eng == ENG_HYB, h3 = eng == ENG_H3, i8 = eng == ENG_I8 || h3, wide = eng == ENG_MMA8W || hyb;
    const int bn = h3 ? H3_BN : i8 ? I8_BN : eng == ENG_DEC ? DEC_BN : wide ? MOE_BN_WIDE : MOE_BN;
    const int maxit = P / bn + E + 1;
    const int8_t *xq = xq_in;
    const float *xs = xs_in;
    // routing (eidx/ewt only) on the side stream, overlapping the quantization
    SideStream *side = side_stream();
    if (!side) return 0;
    if (!check_cuda(cudaEventRecord(side->fork, st), "fork") ||
        !check_cuda(cudaStreamWaitEvent(side->s, side->fork, 0), "fork wait"))
        return 0;
    k_route<<<1, 1024, 4 * E * sizeof(int), side->s>>>(eidx, ewt, P, E, bn,
                                                      (int)w.cap, w.pair_src, w.pair_w, w.items, w.n_items, w.tcerr,
                                                      i8 || hyb ? 1 : 0);
    if (!check_cuda(cudaGetLastError(), "route launch")) return 0;
    if (!check_cuda(cudaEventRecord(side->join, side->s), "join")) return 0;
    if (X) {
        if (!launch_quant_act(X, S, D, w.xq, w.xs, fmt == GPU_FMT_TQ2 ? w.xsx : nullptr, nullptr, st, OUT, D))
            return 0;
        xq = w.xq;
        xs = w.xs;
    } else {
        if (!check_cuda(cudaMemsetAsync(OUT, 0, (size_t)S * D * 4, st), "memset OUT")) return 0;
        if (fmt == GPU_FMT_TQ2) k_rows_sx<<<(S + 7) / 8, 256, 0, st>>>(xq, xs, S, D, w.xsx);
    }
    if (!check_cuda(cudaStreamWaitEvent(st, side->join, 0), "join wait")) return 0;
    if (h3) {
        if (!launch_split_rows(w.pair_src, K, xq, xs, D, (int)w.cap, w.xhs, w.tcerr, st)) return 0;
    } else if (i8) {
        k_gather_rows8<<<(unsigned)w.cap, 128, 0, st>>>(w.pair_src, K, xq, xs, D, w.xg8, w.xsT, (int)w.ldT);
        if (!check_cuda(cudaGetLastError(), "gather launch")) return 0;
    }

    if (eng == ENG_DEC) {
        GemmArgs gu{}, dn{};
        gu.codes = b->gu_codes; gu.scale = b->gu_scale;
        gu.codes_gstride = (long)codes_bytes(fmt, 2 * MI, D);
        gu.scale_gstride = (long)scales_bytes(fmt, 2 * MI, D);
        gu.O = 2 * MI; gu.I = D;
        gu.xq = xq; gu.xs = xs; gu.xsx = w.xsx;
        gu.items = w.items; gu.n_items = w.n_items; gu.pair_src = w.pair_src; gu.K = K;
        gu.act = act; gu.clamp = clamp;
        dn.codes = b->dn_codes; dn.scale = b->dn_scale;
        dn.codes_gstride = (long)codes_bytes(fmt, D, MI);
        dn.scale_gstride = (long)scales_bytes(fmt, D, MI);
        dn.O = D; dn.I = MI;
        dn.items = w.items; dn.n_items = w.n_items; dn.pair_src = w.pair_src; dn.pair_w = w.pair_w; dn.K = K;
        dn.out = OUT; dn.hq = w.hq; dn.hs = w.hs;
        prof_mark(st);
        int ok = launch_moe_dec(fmt, gu, dn, P, w.hf, st);
        prof_mark(st);
        prof_mark(st);
        return ok;
    }
    GemmArgs g{};
    g.codes = b->gu_codes; g.scale = b->gu_scale;
    g.codes_gstride = (long)codes_bytes(fmt, 2 * MI, D);
    g.scale_gstride = (long)scales_bytes(fmt, 2 * MI, D);
    g.O = 2 * MI; g.I = D;
    g.xq = xq; g.xs = xs; g.xsx = w.xsx; g.xblk = nullptr; g.gather = w.pair_src; g.gather_div = K;
    g.items = w.items; g.n_items = w.n_items;
    g.act = act; g.clamp = clamp;
    g.hq = w.hq; g.hs = w.hs; g.hblk = w.hblk; g.hh = nullptr;
    g.pair_src = w.pair_src; g.K = K;
    g.xg8 = w.xg8; g.xsT = w.xsT; g.ldT = (int)w.ldT; g.hsT = w.hsT; g.rows_cap = (int)w.cap;
    prof_mark(st);
    if (h3) {
        g.hsT = nullptr;  // the down GEMM reads the fp16 planes instead
        g.xhs = w.xhs; g.hhs = w.hhs;
        if (!launch_moe_h3(EPI_GATEUP, g, E, w.tcerr, st)) return 0;
    } else if (i8) {
        if (!launch_moe_i8(fmt, EPI_GATEUP, g, E, w.tcerr, st)) return 0;
    } else if (hyb) {
        g.hhs = w.hhs;  // the h3 down GEMM's B planes
        if (!launch_gemm<EPI_GATEUP, MOE_BN_WIDE, false, true>(fmt, g, dim3((2 * MI) / G_BM, maxit), st)) return 0;
    } else if (!(wide ? launch_gemm<EPI_GATEUP, MOE_BN_WIDE, false, true>(fmt, g, dim3((2 * MI) / G_BM, maxit), st)
                      : launch_gemm<EPI_GATEUP, MOE_BN, false, true>(fmt, g, dim3((2 * MI) / G_BM, maxit), st))) {
        return 0;
    }
    prof_mark(st);

    GemmArgs d{};
    d.codes = b->dn_codes; d.scale = b->dn_scale;
    d.codes_gstride = (long)codes_bytes(fmt, D, MI);
    d.scale_gstride = (long)scales_bytes(fmt, D, MI);
    d.O = D; d.I = MI;
    d.xq = w.hq; d.xs = w.hs; d.xsx = nullptr; d.xblk = fmt == GPU_FMT_TQ2 ? w.hblk : nullptr; d.gather = nullptr;
    d.items = w.items; d.n_items = w.n_items;
    d.out = OUT; d.pair_w = w.pair_w; d.pair_src = w.pair_src; d.K = K;
    d.xg8 = w.hq; d.xsT = w.hsT; d.ldT = (int)w.ldT; d.rows_cap = (int)w.cap;
    d.xhs = w.hhs;
    int ok = h3 || hyb ? launch_moe_h3(EPI_DOWN, d, E, w.tcerr, st)
           : i8 ? launch_moe_i8(fmt, EPI_DOWN, d, E, w.tcerr, st)
           : wide ? launch_gemm<EPI_DOWN, MOE_BN_WIDE, false, true>(fmt, d, dim3((D + G_BM - 1) / G_BM, maxit), st)
                  : launch_gemm<EPI_DOWN, MOE_BN, false, true>(fmt, d, dim3((D + G_BM - 1) / G_BM, maxit), st);
    prof_mark(st);
    return ok;
}

extern "C" int zz_moe_ffn_dev(const zz_expert_bank *b, const float *X, const int32_t *eidx, const float *ewt,
                              float *OUT, int S, int K, int act, float clamp, void *workspace, size_t ws_bytes,
                              int validate, void *stream) {
    if (!X && S > 0) return fail("zz_moe_ffn_dev: null X");
    return moe_impl(b, X, nullptr, nullptr, eidx, ewt, OUT, S, K, act, clamp, workspace, ws_bytes, validate, stream);
}

extern "C" int zz_moe_ffn_q8_dev(const zz_expert_bank *b, const int8_t *xq, const float *xs, const int32_t *eidx,
                                 const float *ewt, float *OUT, int S, int K, int act, float clamp, void *workspace,
                                 size_t ws_bytes, int validate, void *stream) {
    if ((!xq || !xs) && S > 0) return fail("zz_moe_ffn_q8_dev: null activation");
    return moe_impl(b, nullptr, xq, xs, eidx, ewt, OUT, S, K, act, clamp, workspace, ws_bytes, validate, stream);
}

// ---------------------------------------------------------------- no-allocation variant
// Some callers cannot allocate device memory at all: an engine that hands the GPU one
// fixed budget at start-up, a plugin host that forbids cudaMalloc after init, or code
// running where an allocation could stall or fail mid-request. For them the layer's
// scratch lives in this file-scope array instead of a caller workspace. It is part of
// the library image, so every GPU that loads the library holds these bytes until exit.
static __device__ __align__(256) uint8_t g_noalloc_scratch[ZZ_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch per device. Host code must not pass the symbol
// itself to a kernel: on the host it is only a stand-in, not a device address.
static std::atomic<void *> g_noalloc_ptr[MAX_DEVICES];

extern "C" int zz_moe_ffn_noalloc_dev(const zz_expert_bank *b, const float *X, const int32_t *eidx,
                                      const float *ewt, float *OUT, int S, int K, int act, float clamp,
                                      void *stream) {
    if (!bank_ok(b)) return fail("zz_moe_ffn_noalloc_dev: invalid expert bank");
    if (S < 0 || K <= 0 || K > 64) return fail("zz_moe_ffn_noalloc_dev: bad S=%d or K=%d", S, K);
    if (S == 0) return 1;
    const size_t need = moe_layout(b, S, K, nullptr).total;
    if (need > ZZ_NOALLOC_SCRATCH_BYTES)
        return fail("zz_moe_ffn_noalloc_dev: S=%d K=%d needs %zu scratch bytes, more than the fixed %u; "
                    "use zz_moe_ffn_dev with a caller workspace",
                    S, K, need, (unsigned)ZZ_NOALLOC_SCRATCH_BYTES);
    int dev = 0;
    if (!check_cuda(cudaGetDevice(&dev), "zz_moe_ffn_noalloc_dev: cudaGetDevice")) return 0;
    if (dev < 0 || dev >= MAX_DEVICES) return fail("zz_moe_ffn_noalloc_dev: device %d out of range", dev);
    void *scratch = g_noalloc_ptr[dev].load(std::memory_order_acquire);
    if (!scratch) {  // one-time set-up on this device, with it current
        // Threads racing here all get the same address, so whichever store wins is right.
        if (!check_cuda(cudaGetSymbolAddress(&scratch, g_noalloc_scratch),
                        "zz_moe_ffn_noalloc_dev: cudaGetSymbolAddress"))
            return 0;
        g_noalloc_ptr[dev].store(scratch, std::memory_order_release);
    }
    // Nothing in the scratch needs to start at zero: OUT is cleared by the layer itself
    // and the routing counters live in shared memory.
    return moe_impl(b, X, nullptr, nullptr, eidx, ewt, OUT, S, K, act, clamp, scratch,
                    ZZ_NOALLOC_SCRATCH_BYTES, 0, stream);
}

// ---------------------------------------------------------------- dense
namespace zz {
// y[S, O] for S quantized rows; S == 1 takes the register-resident GEMV, larger S the
// tensor-core GEMM with work items derived from the grid (no device scratch).
int launch_gemv_q4a(const zz_qtensor *W, const int8_t *xq, const float *sx, int S, float *y, cudaStream_t st);
int matvec_impl(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float *y, int S,
                cudaStream_t st) {
    if (W->fmt == GPU_FMT_Q4A) return launch_gemv_q4a(W, xq, sx, S, y, st);
    if (S == 1) {
        int r = launch_gemv1(W, xq, sx, sxtot, y, st);
        if (r != 0) return r > 0;
    }
    int n = (S + DENSE_BN - 1) / DENSE_BN;
    GemmArgs g{};
    g.codes = W->codes; g.scale = W->scale;
    g.O = W->O; g.I = W->I;
    g.xq = xq; g.xs = sx; g.xsx = sxtot;
    g.items = nullptr; g.n_items = nullptr; g.rows_total = S;
    g.y = y;
    return launch_gemm<EPI_STORE, DENSE_BN, false>(W->fmt, g, dim3((W->O + G_BM - 1) / G_BM, n), st);
}
}  // namespace zz
