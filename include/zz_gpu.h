/* zz_gpu.h -- C ABI of libzz_cuda.so, the B200 (sm_100a) backend for zunzuncito's
 * quantized matrix hot path.
 *
 * Two layers:
 *  1. The reference's backend surface, unchanged in name, signature and 1/0 decline
 *     convention (reference gpu.h:61-84), so an engine built against gpu.h links this
 *     library in place of metal.o. Activations cross it as host f32. By default the
 *     matmuls keep them f32, as the reference's GPU backend does (gpu.h:25-30), so they
 *     match q40_dot_f32 / q80_dot_f32 / tq2_dot_f32 / q4a_dot_f32 and the engines'
 *     --check-gpu (gemma4.c:2315-2361) passes; zz_gpu_set_act_quant(1) switches to
 *     quantizing them ON DEVICE exactly like q40_quant_act (q40.h:124-138) and the
 *     integer dots q40_dot / q80_dot / tq2_dot / q4a_dot (q40.h:188, 374; tq2.h:134,
 *     395), the engines' default int8-activation CPU build. The q8_0-activation
 *     kernel signatures of q40.h / tq2.h are added as gpu_*_matvec.
 *  2. Device-pointer entry points (zz_*) for callers that keep weights, activations and
 *     outputs resident in HBM: no host copies, explicit caller-provided workspace, an
 *     explicit stream (a cudaStream_t passed as void*; NULL = legacy default stream).
 *
 * Every entry returns 1 on success and 0 to decline; gpu_last_error() then says why.
 * There is no CPU fallback inside this library: a decline is the caller's to handle,
 * as the engines already do for gpu.h (gemma4.c:445, 683).
 * Not re-entrant: one host thread drives the library, like the reference's backend.
 */
#ifndef ZZ_GPU_H
#define ZZ_GPU_H

#include <stdint.h>
#include <stddef.h>

/* weight formats; values equal the reference's GPU_FMT_* (gpu.h:49-52) */
#define GPU_FMT_Q40 1
#define GPU_FMT_Q80 2
#define GPU_FMT_TQ2 3
#define GPU_FMT_Q4A 4

/* gated activations of the routed-expert FFN */
#define ZZ_ACT_GEGLU_TANH 0   /* gelu_tanh(g)*u            gemma4.c:432-434, 637-644 */
#define ZZ_ACT_SWIGLU 1       /* silu(g)*u                 lfm25.c:677-730, ling.c:797-850 */
#define ZZ_ACT_SWIGLU_CLAMP 2 /* silu(min(g,c))*clip(u,+-c) maple.c:653-655, 676-678 */

#ifdef __cplusplus
extern "C" {
#endif

/* ---------- 1. the reference backend surface (gpu.h:61-84) ---------- */

/* replaces gpu_init (gpu.h:62): 1 if a CUDA device of compute capability 10.x is
 * present and the kernels load */
int gpu_init(void);
/* replaces gpu_shutdown (gpu.h:63): frees every mapped region and cached plane */
void gpu_shutdown(void);
/* replaces gpu_ready (gpu.h:64) */
int gpu_ready(void);
/* replaces gpu_name (gpu.h:65) */
const char *gpu_name(void);
/* replaces gpu_map (gpu.h:70): registers a caller-owned host region holding weights
 * in the reference formats. The bytes are copied into HBM at once; each tensor inside
 * is repacked into structure-of-arrays planes the first time a matmul names it. The
 * region must not change afterwards unless gpu_unmap is called first. */
int gpu_map(const void *p, size_t n);
/* added: forget a region registered by gpu_map (the streaming cache rewrites slots,
 * gemma4.c:2052-2054). No reference counterpart. */
int gpu_unmap(const void *p);
/* replaces gpu_q40_matmul (gpu.h:75): y[S,O] = W[O,I] (q4_0) x[S,I]; host y and x */
int gpu_q40_matmul(float *y, const uint8_t *W, const float *x, int O, int I, int S);
/* replaces gpu_matmul (gpu.h:84) for GPU_FMT_Q40, Q80, TQ2 (W is the whole tq2 tensor,
 * alphas first) and Q4A (tq2.h:268-283). I % 32 (q4_0/q8_0) or I % 64 (tq2, q4a). */
int gpu_matmul(int fmt, float *y, const uint8_t *W, const float *x, int O, int I, int S);
/* added: why the last call declined ("" if it did not). */
const char *gpu_last_error(void);
/* added: numerics of gpu_q40_matmul / gpu_matmul. 0 (default): f32 activations, the
 * reference GPU backend's (gpu.h:25-30; metal.mm:43-45); 1: activations quantized to
 * q8_0 on device and the integer dots, bit-for-bit the engines' CPU kernels per block.
 * No reference counterpart (the Metal backend has only the first). */
int zz_gpu_set_act_quant(int on);

/* q8_0-activation matvecs on host buffers, W inside a gpu_map'd region: the kernel-level
 * signatures an engine's matvec calls, y[o] = dot(W row o, xq, sx) for o < O.
 *   gpu_q40_matvec replaces q40_matvec (q40.h:308-312); gpu_q80_matvec replaces
 *   q80_matvec (q40.h:456-460); gpu_tq2_matvec is the row loop maple runs through
 *   tq2_dot (maple.c:387-398, tq2.h:134) with W the whole tq2 tensor (tq2.h:85-91) and
 *   sxtot = tq2_quant_act's return; gpu_q4a_matvec is the same loop over q4a_dot
 *   (tq2.h:395). The names carry a gpu_ prefix because the reference's own are static
 *   inline in its headers. */
int gpu_q40_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I);
int gpu_q80_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I);
int gpu_tq2_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, float sxtot, int O, int I);
int gpu_q4a_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I);

/* ---------- 2. device-resident entry points ---------- */

/* One weight tensor [O, I] in HBM as structure-of-arrays planes.
 *   q4_0: codes = O rows of I/2 bytes (the 16 nibble bytes of each block, in block
 *         order), scale = O x I/32 fp16 block scales
 *   q8_0: codes = O rows of I int8,  scale = O x I/32 fp16
 *   tq2 : codes = O rows of I/4 bytes (the reference packing), scale = O f32 alphas
 *   q4a : codes = O rows of I/2 bytes (each 64-weight group's two 16-byte nibble
 *         blocks), scale = O x I/64 (fp16 d, fp16 m) pairs (tq2.h:268-283)
 * Row strides are exactly those widths; planes start 256-byte aligned. */
typedef struct zz_qtensor {
    int fmt, O, I;
    const uint8_t *codes;
    const void *scale;
} zz_qtensor;

/* device bytes zz_repack_dev needs for one tensor (both planes + alignment) */
size_t zz_qtensor_bytes(int fmt, int O, int I);
/* repack a reference-format tensor already in device memory (q40.h / tq2.h layout:
 * q4_0/q8_0 rows of interleaved 18/34-byte blocks, or the tq2 tensor) into planes
 * inside dst (zz_qtensor_bytes bytes, 256-aligned) and describe them in *out. */
int zz_repack_dev(int fmt, const uint8_t *src, int O, int I, void *dst, zz_qtensor *out,
                  void *stream);
/* inverse of zz_repack_dev, for checks: planes -> reference layout in dst */
int zz_unpack_dev(const zz_qtensor *t, uint8_t *dst, void *stream);

/* q4_0 / q8_0 weight quantizer on device, bit-exact with q40_quant_row /
 * q80_quant_row (q40.h:83-110, 332-350): w [O, I] f32 -> dst in the reference row
 * layout (O * I/32 blocks of 18 or 34 bytes). fmt = GPU_FMT_Q40 or GPU_FMT_Q80. */
int zz_quant_rows_dev(int fmt, const float *w, int O, int I, uint8_t *dst, void *stream);

/* replaces q40_quant_act (q40.h:124) and tq2_quant_act (tq2.h:98) for S rows:
 * x [S, I] f32 -> xq [S, I] int8, sx [S, I/32] f32 and, when sxtot != NULL, the
 * per-row tq2 offset total Sx (double sum in block order, then rounded to f32). */
int zz_quant_act_dev(const float *x, int S, int I, int8_t *xq, float *sx, float *sxtot,
                     void *stream);

/* replaces q40_matvec / q80_matvec (q40.h:308, 456), the tq2 row loop that maple
 * runs through w_dot (maple.c:387-398) and its q4a counterpart (q4a_dot, tq2.h:395):
 * y[S, O] = W . (xq, sx) for S quantized rows. sxtot is required for tq2 and ignored
 * otherwise. */
int zz_matvec_dev(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot,
                  float *y, int S, void *stream);

/* the tied lm_head of a decode step (gemma4.c:1270-1274): y[o] = W row o . (xq, sx) for
 * the whole vocabulary (e.g. 262144 x 2816 q4_0), then, when softcap > 0, the final-logit
 * softcap y = tanhf(y / softcap) * softcap. One activation row; tall tensors stream
 * through the bulk-copy GEMV with the softcap fused into its epilogue. */
int zz_lm_head_dev(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot,
                   float softcap, float *y, void *stream);

/* the f32-activation matvec (q40_dot_f32 q40.h:290-305, q80_dot_f32, tq2_dot_f32
 * tq2.h:235-252, q4a_dot_f32 tq2.h:410-432): y[S, O] = W . x for S f32 rows x [S, I]
 * (I <= 51200). Each 32-weight block is summed in fp32 (the reference sums in double). */
int zz_matvec_f32_dev(const zz_qtensor *W, const float *x, float *y, int S, void *stream);

/* per-block integer sums for the bit-exact parity check: out[o, b] = <q_w - 8, q_x>
 * (q4_0), <q_w, q_x> (q8_0), <c, q_x> with unsigned codes (tq2), for one activation
 * row (q40.h:162-187, 359-372; tq2.h:116-133). out is [O, I/32] int32. */
int zz_blocksums_dev(const zz_qtensor *W, const int8_t *xq, int32_t *out, void *stream);

/* ---- routers: token rows -> (eidx, ewt) [S][K] in device memory, the inputs of
 * zz_moe_ffn_dev; no host round trip. Selection is the reference's exactly (scores in
 * its operation order; descending score, ties to the lower expert index). K <= 16. */

/* replaces gemma4's route_row (gemma4.c:581-613): rmsnorm(res) * router_scale * D^-1/2,
 * f32 logits = router_proj [E][D] . xn, top-K, softmax over the K, times the per-expert
 * scale pes [E]. res [S][D] is the residual row before the pre-FFN norm. E <= 256; D % 4 == 0
 * and 16-byte-aligned router rows (both routers). */
int zz_route_gemma4_dev(const float *res, int S, int D, int E, int K, const float *proj,
                        const float *scale, const float *pes, float eps, int32_t *idx, float *wts,
                        void *stream);
/* replaces ling's grouped route_row (ling.c:705-789): sigmoid scores of router [E][D]
 * against the normalized rows xn [S][D], biased by bias [E] for selection only; the E
 * experts in n_group contiguous groups ranked by the sum of their two best biased
 * scores, the best topk_group kept; top-K of those; weights the unbiased scores,
 * renormalised when norm_topk_prob, times routed_scale. E <= 256, n_group <= 32. */
int zz_route_ling_dev(const float *xn, int S, int D, int E, int K, int n_group, int topk_group,
                      int norm_topk_prob, float routed_scale, const float *router, const float *bias,
                      int32_t *idx, float *wts, void *stream);

/* The routed experts of one MoE layer, packed for the batch-union FFN.
 *   gu: gate and up stacked per expert as a [2*inter, hidden] tensor whose rows are
 *       interleaved in groups of 64 (64 gate rows, then the 64 up rows of the same
 *       features, ...); dn: down [hidden, inter]. Planes as in zz_qtensor, experts
 *       contiguous. inter % 64 == 0, hidden % 64 == 0. */
typedef struct zz_expert_bank {
    int fmt, n_experts, hidden, inter;
    const uint8_t *gu_codes;
    const void *gu_scale;
    const uint8_t *dn_codes;
    const void *dn_scale;
} zz_expert_bank;

size_t zz_expert_bank_bytes(int fmt, int n_experts, int hidden, int inter);
/* Pack experts from reference expert blobs already in device memory. Blob e starts at
 * blobs + e * blob_stride and holds [gate | up | down] as the engines' expert files do
 * (gemma4.c:660, maple.c:616-619): q4_0/q8_0 row tensors, or three tq2 tensors. */
int zz_expert_bank_pack_dev(int fmt, int n_experts, int hidden, int inter, const uint8_t *blobs,
                            int64_t blob_stride, void *dst, zz_expert_bank *out, void *stream);

/* workspace bytes zz_moe_ffn_dev needs for S tokens with top-K routing */
size_t zz_moe_workspace_bytes(const zz_expert_bank *bank, int S, int K);

/* Batch-union routed-expert FFN of one layer: the device counterpart of moe_start's
 * union + moe_apply_chunk + expert_apply (gemma4.c:618-711, 750-790; maple.c:612-692):
 *   OUT[s] = sum_k ewt[s,k] * down_e( act( gate_e(q8(X[s])), up_e(q8(X[s])) ) requant )
 * with e = eidx[s,k]. X [S, hidden] f32, eidx/ewt [S, K], OUT [S, hidden] f32
 * (overwritten). Each distinct expert's weights are streamed once for all of its
 * tokens. act is a ZZ_ACT_* value, clamp is used by ZZ_ACT_SWIGLU_CLAMP.
 * With validate != 0, eidx values outside [0, n_experts) decline before any work is
 * launched (it costs a device->host sync); otherwise such entries are skipped. */
int zz_moe_ffn_dev(const zz_expert_bank *bank, const float *X, const int32_t *eidx,
                   const float *ewt, float *OUT, int S, int K, int act, float clamp,
                   void *workspace, size_t workspace_bytes, int validate, void *stream);

/* Same layer for rows that arrive already quantized to q8_0 (xq [S, hidden] int8,
 * xs [S, hidden/32] f32), e.g. received from another GPU by the expert-parallel
 * dispatch. eidx entries outside [0, n_experts) are skipped, so a row can carry fewer
 * than K local experts (pad with -1). Output and workspace as zz_moe_ffn_dev. */
int zz_moe_ffn_q8_dev(const zz_expert_bank *bank, const int8_t *xq, const float *xs,
                      const int32_t *eidx, const float *ewt, float *OUT, int S, int K, int act,
                      float clamp, void *workspace, size_t workspace_bytes, int validate,
                      void *stream);

/* zz_moe_ffn_dev for callers that cannot allocate device memory (no counterpart in
 * the reference, which has no device memory of its own). Same arguments minus the
 * workspace: the scratch is a fixed ZZ_NOALLOC_SCRATCH_BYTES (32 MiB) array inside the
 * library, held by every GPU that loads it until the process exits. Declines when
 * zz_moe_workspace_bytes(bank, S, K) exceeds it: at top-8 that is S > 862 for the
 * Gemma-4 shape (hidden 2816, inter 704, 128 experts) and S > 1147 for Maple's (2048,
 * 512, 256 experts). It calls no allocator.
 *  - The first call on each device looks up the array's device address with that
 *    device current; make that first call before any stream capture.
 *  - All calls share the one array and it keeps the previous call's contents; calls
 *    that overlap on the GPU (two streams, or two host threads) race on it. */
#define ZZ_NOALLOC_SCRATCH_BYTES (32u << 20)
int zz_moe_ffn_noalloc_dev(const zz_expert_bank *bank, const float *X, const int32_t *eidx,
                           const float *ewt, float *OUT, int S, int K, int act, float clamp,
                           void *stream);

/* ---- the gemma4 container (manifest.txt / dense.bin / experts.bin, written by the
 * reference's tools/convert_gemma4.py:361-422 and read by gemma4.c:260-403) loaded
 * straight into HBM planes. The handle is opaque; the loader allocates its own staging
 * (it is not a hot path). */
typedef struct zz_container zz_container;
/* parse dir/manifest.txt (the reference's manifest(), gemma4.c:260-331) */
int zz_container_open(const char *dir, zz_container **out);
void zz_container_close(zz_container *c);
/* a numeric "cfg <key> <value>" entry */
int zz_container_cfg(const zz_container *c, const char *key, double *val);
/* a "dense <name> <off> <len> <fmt> <O> <I>" entry (container formats: f32 0, q4_0 1) */
int zz_container_dense_info(const zz_container *c, const char *name, int *fmt, int *O, int *I,
                            int64_t *off, int64_t *len);
/* the experts.bin offset of (layer, expert), -1 if absent */
int64_t zz_container_expert_offset(const zz_container *c, int layer, int expert);
/* device bytes of one layer's expert bank (zz_expert_bank_bytes of the container's shape) */
size_t zz_container_bank_bytes(const zz_container *c);
/* one layer's experts from experts.bin into an expert bank in dst (256-byte aligned,
 * zz_container_bank_bytes bytes); replaces the engine's per-slot read + gpu_map
 * (gemma4.c:480-495, 2052-2055) for a resident layer */
int zz_container_load_bank_dev(zz_container *c, int layer, void *dst, zz_expert_bank *bank, void *stream);
/* a q4_0 dense tensor (e.g. "embed_tokens", the tied lm_head) into zz_qtensor planes in
 * dst (zz_qtensor_bytes bytes, 256-byte aligned) */
int zz_container_load_dense_dev(zz_container *c, const char *name, void *dst, zz_qtensor *out, void *stream);

/* ---- expert-parallel exchange layout (no reference counterpart: the reference runs
 * one process; these pack and unpack the rows of the NCCL all-to-all that shards the
 * experts over the GPUs of a node).
 * One row per (destination rank d, token s), zz_ep_row_bytes(D, K) bytes:
 *   q8_0 codes int8[D] | block scales f32[D/32] | local expert ids int32[K] | weights f32[K]
 * ids are the token's experts held by d as id - d*per_rank, -1 for the others (weight 0).
 * zz_ep_pack_dev writes payload[world][S] rows (destination-major, so an equal-split
 * all-to-all sends each rank its S rows); zz_ep_unpack_dev splits R received rows into
 * the four arrays zz_moe_ffn_q8_dev takes. Pointers 4-byte aligned, D % 32 == 0. */
size_t zz_ep_row_bytes(int D, int K);
int zz_ep_pack_dev(const int8_t *xq, const float *xs, const int32_t *eidx, const float *ewt, int S, int D, int K,
                   int world, int per_rank, uint8_t *payload, void *stream);
int zz_ep_unpack_dev(const uint8_t *rows, int R, int D, int K, int8_t *xq, float *xs, int32_t *eidx, float *ewt,
                     void *stream);

/* Diagnostic: byte offset inside the zz_moe_ffn_dev workspace (same bank, S, K) of
 *   0 pair_src int32[S*K]  routing slot s*K+k held by each pair row, grouped by expert
 *   1 pair_w   f32[S*K]    its router weight
 *   2 hq       int8[S*K][inter]      requantized activation per pair row
 *   3 hs       f32[S*K][inter/32]    its block scales
 *   4 n_items  int32                 work items of the last call
 *   5 tc_error int32                 0, or the id of a tensor-core pipeline wait that
 *                                    ran out (the call's results are then invalid)
 * Pair rows are grouped by expert with each expert's rows starting on a 16-row
 * boundary; padding rows hold pair_src = -1. which = 6 returns the number of pair
 * rows (capacity incl. padding) instead of an offset.
 * so tests can check the gate/up stage bit for bit. (size_t)-1 for an unknown id.
 * No reference counterpart (the engines keep these in Buf: gemma4.c:2123-2127). */
size_t zz_moe_workspace_offset(const zz_expert_bank *bank, int S, int K, int which);

/* Diagnostic stage timing, no reference counterpart (the engines print wall-clock
 * phase times to stderr, gemma4.c:3216). While enabled, every zz_moe_ffn_dev call
 * records CUDA events on its stream at its stage boundaries; zz_prof_collect waits
 * for them and returns the summed milliseconds of [quantize + route, gate/up GEMM,
 * down GEMM] and the number of calls, then forgets them. */
int zz_prof_enable(int on);
int zz_prof_collect(float *stage_ms, int *calls);

#ifdef __cplusplus
}
#endif
#endif /* ZZ_GPU_H */
