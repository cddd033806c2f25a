/* zz_oracle.c -- TEST INFRASTRUCTURE ONLY. CPU restatement of zunzuncito's quantized
 * matrix hot path, used as the checker for the CUDA kernels in zunzuncito_b200/csrc.
 * Nothing in the product links, loads or calls this file; only tests/, the smoke
 * check in __graft_entry__.py and bench.py's CPU-baseline leg do.
 *
 * Every function restates one reference routine (paths are within the reference
 * project) in plain scalar C. Parity of this restatement is pinned in two ways:
 *   - against the reference's own kernels compiled from its sources by
 *     oracle/Makefile into oracle/_ref/libzzref.so (tests/test_oracle.py), and
 *   - against golden vectors that the reference build produced, committed under
 *     tests/golden/ (tests/golden/make_golden.py).
 *
 * Accumulation order follows the reference's SCALAR path (four accumulators indexed
 * by block number, q40.h:270-284), so per-block integer sums are bit-identical to
 * every reference ISA path and fp32 results agree to rounding.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>

#define ORC_BLK 32
#define ORC_Q40_BB 18
#define ORC_Q80_BB 34
#define ORC_TQ2_GRP 64

/* ---- fp16 <-> f32, IEEE binary16 with round-half-even (q40.h:46-80) ---- */
float orc_fp16_to_f32(uint16_t h) {
    int sign = (h >> 15) & 1, exp = (h >> 10) & 31, man = h & 1023;
    float v;
    if (exp == 0) v = ldexpf((float)man, -24);                 /* zero / subnormal */
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = ldexpf((float)(man | 1024), exp - 25);
    return sign ? -v : v;
}

uint16_t orc_f32_to_fp16(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u);
    if (a >= 0x477ff000u) return sign | 0x7c00u;     /* rounds to >= 65520: inf */
    if (a < 0x38800000u) {                            /* below fp16 normal range */
        /* value = a_f; subnormal step 2^-24: q = rne(a_f * 2^24) */
        float af; memcpy(&af, &a, 4);
        double q = (double)af * 16777216.0;           /* exact in double */
        double fl = floor(q), rem = q - fl;
        uint32_t r = (uint32_t)fl;
        if (rem > 0.5 || (rem == 0.5 && (r & 1u))) r++;
        return sign | (uint16_t)r;                    /* r==1024 is the smallest normal */
    }
    uint32_t e = ((a >> 23) - 112u) << 10;            /* rebias 127 -> 15 */
    uint32_t m = a & 0x7fffffu;
    uint32_t h = e | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  /* carry may bump exp */
    return sign | (uint16_t)h;
}

/* ---- quantizers ---- */

/* q4_0 weight row: signed max-|x| element, d = fp16(mx / -8) rounded BEFORE the
 * inverse is taken, q = clamp(trunc(x*id + 8.5), 0, 15); low nibble of byte j is
 * weight j, high nibble weight j+16 (q40.h:12-16, 83-110). */
void orc_q40_quant_row(const float *w, uint8_t *dst, int I) {
    for (int b = 0; b < I / ORC_BLK; b++) {
        const float *x = w + b * ORC_BLK;
        uint8_t *blk = dst + (size_t)b * ORC_Q40_BB;
        float amax = 0.f, mx = 0.f;
        for (int j = 0; j < ORC_BLK; j++) {
            float a = fabsf(x[j]);
            if (a > amax) { amax = a; mx = x[j]; }
        }
        uint16_t hd = orc_f32_to_fp16(mx / -8.0f);
        memcpy(blk, &hd, 2);
        float d = orc_fp16_to_f32(hd), id = d != 0.f ? 1.0f / d : 0.0f;
        for (int j = 0; j < 16; j++) {
            int q0 = (int)(x[j] * id + 8.5f), q1 = (int)(x[j + 16] * id + 8.5f);
            q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
            q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
            blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

/* q8_0 weight row: d = fp16(amax/127), q = clamp(rne(x/d), +-127) (q40.h:332-350) */
void orc_q80_quant_row(const float *w, uint8_t *dst, int I) {
    for (int b = 0; b < I / ORC_BLK; b++) {
        const float *x = w + b * ORC_BLK;
        uint8_t *blk = dst + (size_t)b * ORC_Q80_BB;
        float amax = 0.f;
        for (int j = 0; j < ORC_BLK; j++) if (fabsf(x[j]) > amax) amax = fabsf(x[j]);
        uint16_t hd = orc_f32_to_fp16(amax / 127.0f);
        memcpy(blk, &hd, 2);
        float d = orc_fp16_to_f32(hd), id = d != 0.f ? 1.0f / d : 0.0f;
        for (int j = 0; j < ORC_BLK; j++) {
            long q = lrintf(x[j] * id);
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            blk[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

/* q8_0 activation: per 32-block f32 scale amax/127 (NOT fp16-rounded), q =
 * clamp(rne(x * (1/d)), +-127) (q40.h:124-138). */
void orc_quant_act(const float *x, int8_t *xq, float *sx, int I) {
    for (int b = 0; b < I / ORC_BLK; b++) {
        const float *v = x + b * ORC_BLK;
        float amax = 0.f;
        for (int j = 0; j < ORC_BLK; j++) if (fabsf(v[j]) > amax) amax = fabsf(v[j]);
        float d = amax / 127.0f, id = d != 0.f ? 1.0f / d : 0.0f;
        sx[b] = d;
        for (int j = 0; j < ORC_BLK; j++) {
            long q = lrintf(v[j] * id);
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            xq[b * ORC_BLK + j] = (int8_t)q;
        }
    }
}

/* tq2 activation: q8_0 plus Sx = (float) sum_b (double)sx[b] * sum_j xq, summed in
 * block order in double (tq2.h:98-108). */
float orc_tq2_quant_act(const float *x, int8_t *xq, float *sx, int I) {
    orc_quant_act(x, xq, sx, I);
    double tot = 0;
    for (int b = 0; b < I / ORC_BLK; b++) {
        int32_t s = 0;
        for (int j = 0; j < ORC_BLK; j++) s += xq[b * ORC_BLK + j];
        tot += (double)sx[b] * (double)s;
    }
    return (float)tot;
}

/* ---- per-block integer sums: the bit-exact parity quantity ---- */

/* q4_0: <q - 8, x> per block (q40.h:162-187 computes it as <q,x> - 8*sum x) */
void orc_q40_blocksums(const uint8_t *w, const int8_t *xq, int I, int32_t *out) {
    for (int b = 0; b < I / ORC_BLK; b++) {
        const uint8_t *qs = w + (size_t)b * ORC_Q40_BB + 2;
        const int8_t *x = xq + b * ORC_BLK;
        int32_t s = 0;
        for (int j = 0; j < 16; j++)
            s += ((qs[j] & 15) - 8) * x[j] + ((qs[j] >> 4) - 8) * x[j + 16];
        out[b] = s;
    }
}
/* q8_0: <q_w, q_x> per block (q40.h:359-372) */
void orc_q80_blocksums(const uint8_t *w, const int8_t *xq, int I, int32_t *out) {
    for (int b = 0; b < I / ORC_BLK; b++) {
        const int8_t *q = (const int8_t *)(w + (size_t)b * ORC_Q80_BB + 2);
        int32_t s = 0;
        for (int j = 0; j < ORC_BLK; j++) s += q[j] * xq[b * ORC_BLK + j];
        out[b] = s;
    }
}
/* tq2: <c, x> per 32-weight activation block with UNSIGNED codes c in {0,1,2}; the
 * -1 offset is applied once per row through Sx (tq2.h:116-133, 212-230). Block 2g
 * takes bit fields 0 and 2 of group g, block 2g+1 bit fields 4 and 6. */
static inline int orc_tq2_code(const uint8_t *codes, int j) {
    return (codes[(j / 64) * 16 + (j % 16)] >> (2 * ((j / 16) % 4))) & 3;
}
void orc_tq2_blocksums(const uint8_t *codes, const int8_t *xq, int I, int32_t *out) {
    for (int b = 0; b < I / ORC_BLK; b++) {
        int32_t s = 0;
        for (int j = b * ORC_BLK; j < (b + 1) * ORC_BLK; j++) s += orc_tq2_code(codes, j) * xq[j];
        out[b] = s;
    }
}

/* ---- dots (scalar accumulation order of q40.h:270-284 / 428-440, tq2.h:212-230) ---- */

float orc_q40_dot(const uint8_t *w, const int8_t *xq, const float *sx, int I) {
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    int32_t s;
    for (int b = 0; b < I / ORC_BLK; b++) {
        uint16_t hd; memcpy(&hd, w + (size_t)b * ORC_Q40_BB, 2);
        orc_q40_blocksums(w + (size_t)b * ORC_Q40_BB, xq + b * ORC_BLK, ORC_BLK, &s);
        a[b & 3] += orc_fp16_to_f32(hd) * sx[b] * (float)s;
    }
    return (a[0] + a[1]) + (a[2] + a[3]);
}
float orc_q80_dot(const uint8_t *w, const int8_t *xq, const float *sx, int I) {
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    int32_t s;
    for (int b = 0; b < I / ORC_BLK; b++) {
        uint16_t hd; memcpy(&hd, w + (size_t)b * ORC_Q80_BB, 2);
        orc_q80_blocksums(w + (size_t)b * ORC_Q80_BB, xq + b * ORC_BLK, ORC_BLK, &s);
        a[b & 3] += orc_fp16_to_f32(hd) * sx[b] * (float)s;
    }
    return (a[0] + a[1]) + (a[2] + a[3]);
}
float orc_tq2_dot(const uint8_t *codes, float alpha, const int8_t *xq, const float *sx,
                  float sxtot, int I) {
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    int nb = I / ORC_BLK;
    int32_t *s = (int32_t *)malloc(sizeof(int32_t) * (size_t)nb);
    orc_tq2_blocksums(codes, xq, I, s);
    for (int b = 0; b < nb; b++) a[b & 3] += sx[b] * (float)s[b];
    free(s);
    return alpha * (((a[0] + a[1]) + (a[2] + a[3])) - sxtot);
}

/* row-major matvecs: y[o] = dot(W row o) (q40.h:308-312, 456-460; tq2 tensor is
 * alpha[O] f32 followed by codes[O][I/4], tq2.h:81-91) */
void orc_q40_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I) {
    size_t rb = (size_t)(I / ORC_BLK) * ORC_Q40_BB;
    for (int o = 0; o < O; o++) y[o] = orc_q40_dot(W + o * rb, xq, sx, I);
}
void orc_q80_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I) {
    size_t rb = (size_t)(I / ORC_BLK) * ORC_Q80_BB;
    for (int o = 0; o < O; o++) y[o] = orc_q80_dot(W + o * rb, xq, sx, I);
}
void orc_tq2_matvec(float *y, const uint8_t *T, const int8_t *xq, const float *sx, float sxtot,
                    int O, int I) {
    const float *alpha = (const float *)T;
    const uint8_t *codes = T + (size_t)O * 4;
    for (int o = 0; o < O; o++)
        y[o] = orc_tq2_dot(codes + (size_t)o * (I / 4), alpha[o], xq, sx, sxtot, I);
}

/* ---- routed-expert FFN ---- */

/* tanh-approximated GELU (gemma4.c:432-434) and SiLU (maple.c:382-384) */
float orc_gelu_tanh(float x) {
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}
float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* Gemma-4 expert over its routed rows (gemma4.c:618-654, the int8-activation build):
 * blob = [gate q4_0 MI x D | up q4_0 MI x D | down q4_0 D x MI] contiguous.
 * For each row r: xq = q8(x_r); h_o = gelu_tanh(<G_o>) * <U_o>; hq = q8(h);
 * OUT[rows[r]][o] += w[r] * <Dn_o, hq>. fmt 2 (q8_0 weights) is the lfm25 tier with
 * SwiGLU (lfm25.c:677-730); act 0 = GeGLU, 1 = SwiGLU. */
void orc_q4_expert_apply(int fmt, int act, const uint8_t *blob, const float *X, float *OUT,
                         const int *rows, int nrows, const float *w, int D, int MI) {
    int bb = fmt == 2 ? ORC_Q80_BB : ORC_Q40_BB;
    size_t grb = (size_t)(D / ORC_BLK) * bb, drb = (size_t)(MI / ORC_BLK) * bb;
    size_t gate_b = grb * MI;
    const uint8_t *G = blob, *U = blob + gate_b, *Dn = blob + 2 * gate_b;
    int8_t *xq = malloc((size_t)D), *hq = malloc((size_t)MI);
    float *sx = malloc(sizeof(float) * (D / ORC_BLK)), *hs = malloc(sizeof(float) * (MI / ORC_BLK));
    float *h = malloc(sizeof(float) * (size_t)MI);
    for (int r = 0; r < nrows; r++) {
        orc_quant_act(X + (size_t)rows[r] * D, xq, sx, D);
        for (int o = 0; o < MI; o++) {
            float g, u;
            if (fmt == 2) { g = orc_q80_dot(G + o * grb, xq, sx, D); u = orc_q80_dot(U + o * grb, xq, sx, D); }
            else          { g = orc_q40_dot(G + o * grb, xq, sx, D); u = orc_q40_dot(U + o * grb, xq, sx, D); }
            h[o] = act == 0 ? orc_gelu_tanh(g) * u : orc_silu(g) * u;
        }
        orc_quant_act(h, hq, hs, MI);
        float *out = OUT + (size_t)rows[r] * D;
        for (int o = 0; o < D; o++)
            out[o] += w[r] * (fmt == 2 ? orc_q80_dot(Dn + o * drb, hq, hs, MI)
                                       : orc_q40_dot(Dn + o * drb, hq, hs, MI));
    }
    free(xq); free(hq); free(sx); free(hs); free(h);
}

/* Maple ternary expert (maple.c:612-692, int8 build): blob = [gate tq2 tensor MI x D |
 * up tq2 MI x D | down tq2 D x MI], each tensor alpha[O] f32 then codes.
 * h = silu(min(g, CL)) * clip(u, -CL, CL); hq with its own Sx. */
void orc_tq2_expert_apply(const uint8_t *blob, const float *X, float *OUT, const int *rows,
                          int nrows, const float *w, int D, int MI, float CL) {
    size_t gate_b = (size_t)MI * 4 + (size_t)MI * (D / 4);
    const uint8_t *G = blob, *U = blob + gate_b, *Dn = blob + 2 * gate_b;
    const float *ga = (const float *)G, *ua = (const float *)U, *da = (const float *)Dn;
    const uint8_t *gc = G + (size_t)MI * 4, *uc = U + (size_t)MI * 4, *dc = Dn + (size_t)D * 4;
    int8_t *xq = malloc((size_t)D), *hq = malloc((size_t)MI);
    float *sx = malloc(sizeof(float) * (D / ORC_BLK)), *hs = malloc(sizeof(float) * (MI / ORC_BLK));
    float *h = malloc(sizeof(float) * (size_t)MI);
    for (int r = 0; r < nrows; r++) {
        float tx = orc_tq2_quant_act(X + (size_t)rows[r] * D, xq, sx, D);
        for (int o = 0; o < MI; o++) {
            float g = orc_tq2_dot(gc + (size_t)o * (D / 4), ga[o], xq, sx, tx, D);
            float u = orc_tq2_dot(uc + (size_t)o * (D / 4), ua[o], xq, sx, tx, D);
            if (g > CL) g = CL;
            u = u < -CL ? -CL : (u > CL ? CL : u);
            h[o] = orc_silu(g) * u;
        }
        float th = orc_tq2_quant_act(h, hq, hs, MI);
        float *out = OUT + (size_t)rows[r] * D;
        for (int o = 0; o < D; o++)
            out[o] += w[r] * orc_tq2_dot(dc + (size_t)o * (MI / 4), da[o], hq, hs, th, MI);
    }
    free(xq); free(hq); free(sx); free(hs); free(h);
}

/* top-k selection in descending logit order (ties keep the lower expert index),
 * then softmax over the k selected logits (maple.c:582-601; gemma4.c:597-612 with a
 * per-expert scale of 1). */
void orc_route_topk(const float *logits, int E, int K, int *idx, float *wts) {
    float topv[64];
    for (int j = 0; j < K; j++) { idx[j] = -1; topv[j] = -INFINITY; }
    for (int e = 0; e < E; e++) {
        float v = logits[e];
        int j = K;
        while (j > 0 && v > topv[j - 1]) j--;
        if (j == K) continue;
        for (int t = K - 1; t > j; t--) { topv[t] = topv[t - 1]; idx[t] = idx[t - 1]; }
        topv[j] = v; idx[j] = e;
    }
    float mx = topv[0], sum = 0.f;
    for (int j = 0; j < K; j++) { wts[j] = expf(topv[j] - mx); sum += wts[j]; }
    for (int j = 0; j < K; j++) wts[j] /= (sum + 1e-20f);
}

/* Batch-union MoE layer (gemma4.c:750-790; maple.c:738-790): the distinct experts in
 * first-seen order over (s, k); for each, the rows that chose it and their weights in
 * ascending (s, k) order; OUT = sum over those of w * FFN_e(x_s). OUT is zeroed first.
 * kind: 0 = q4_0 GeGLU, 1 = q4_0 SwiGLU, 2 = q8_0 SwiGLU, 3 = tq2 clamped SwiGLU.
 * blobs[e] points at expert e's [gate|up|down] blob. */
void orc_moe_layer(int kind, const uint8_t *const *blobs, int E, const float *X, float *OUT,
                   int S, int K, const int *eidx, const float *ewt, int D, int MI, float CL) {
    int *uniq = malloc(sizeof(int) * (size_t)E), nu = 0;
    int *rows = malloc(sizeof(int) * (size_t)S * K);
    float *wr = malloc(sizeof(float) * (size_t)S * K);
    for (int s = 0; s < S; s++)
        for (int j = 0; j < K; j++) {
            int e = eidx[s * K + j], seen = 0;
            for (int u = 0; u < nu; u++) if (uniq[u] == e) { seen = 1; break; }
            if (!seen) uniq[nu++] = e;
        }
    memset(OUT, 0, sizeof(float) * (size_t)S * D);
    for (int u = 0; u < nu; u++) {
        int e = uniq[u], n = 0;
        for (int s = 0; s < S; s++)
            for (int j = 0; j < K; j++)
                if (eidx[s * K + j] == e) { rows[n] = s; wr[n++] = ewt[s * K + j]; }
        if (kind == 3) orc_tq2_expert_apply(blobs[e], X, OUT, rows, n, wr, D, MI, CL);
        else orc_q4_expert_apply(kind == 2 ? 2 : 1, kind == 0 ? 0 : 1, blobs[e], X, OUT, rows, n, wr, D, MI);
    }
    free(uniq); free(rows); free(wr);
}

/* elementwise gated activation of the expert FFN: act 0 GeGLU (gemma4.c:637-644),
 * 1 SwiGLU (lfm25.c:677-730), 2 clamped SwiGLU (maple.c:653-655) */
void orc_act_vec(int act, const float *g, const float *u, float *h, int n, float CL) {
    for (int i = 0; i < n; i++) {
        float gv = g[i], uv = u[i];
        if (act == 0) { h[i] = orc_gelu_tanh(gv) * uv; continue; }
        if (act == 2) {
            if (gv > CL) gv = CL;
            uv = uv < -CL ? -CL : (uv > CL ? CL : uv);
        }
        h[i] = orc_silu(gv) * uv;
    }
}

/* The batch-union layer for rows that arrive already quantized (xq [S, D] int8,
 * sx [S, D/32]): what an expert-parallel receiver computes for the rows routed to its
 * experts. Expert ids outside [0, E) are skipped (padding). Sums per row over the K
 * slots in slot order; OUT zeroed first. Same expert math as orc_moe_layer. */
void orc_moe_layer_q8(int kind, const uint8_t *const *blobs, int E, const int8_t *XQ, const float *XS,
                      float *OUT, int S, int K, const int *eidx, const float *ewt, int D, int MI, float CL) {
    int nbD = D / ORC_BLK;
    float *X = malloc(sizeof(float) * (size_t)D);
    int8_t *xq = malloc((size_t)D);
    float *sx = malloc(sizeof(float) * nbD);
    memset(OUT, 0, sizeof(float) * (size_t)S * D);
    for (int s = 0; s < S; s++) {
        /* the expert routines quantize their input row; hand them a row whose
         * quantization is exactly (xq, sx): only the GEMV inputs matter, so run the
         * expert math directly on the given codes */
        for (int k = 0; k < K; k++) {
            int e = eidx[s * K + k];
            if (e < 0 || e >= E) continue;
            const uint8_t *blob = blobs[e];
            float w = ewt[s * K + k];
            const int8_t *q = XQ + (size_t)s * D;
            const float *qs = XS + (size_t)s * nbD;
            float *out = OUT + (size_t)s * D;
            float *h = malloc(sizeof(float) * (size_t)MI);
            int8_t *hq = malloc((size_t)MI);
            float *hs = malloc(sizeof(float) * (MI / ORC_BLK));
            if (kind == 3) {
                size_t gate_b = (size_t)MI * 4 + (size_t)MI * (D / 4);
                const uint8_t *G = blob, *U = blob + gate_b, *Dn = blob + 2 * gate_b;
                double tot = 0;
                for (int b = 0; b < nbD; b++) {
                    int32_t t = 0;
                    for (int j = 0; j < ORC_BLK; j++) t += q[b * ORC_BLK + j];
                    tot += (double)qs[b] * (double)t;
                }
                float tx = (float)tot;
                for (int o = 0; o < MI; o++) {
                    float g = orc_tq2_dot(G + MI * 4 + (size_t)o * (D / 4), ((const float *)G)[o], q, qs, tx, D);
                    float u = orc_tq2_dot(U + MI * 4 + (size_t)o * (D / 4), ((const float *)U)[o], q, qs, tx, D);
                    if (g > CL) g = CL;
                    u = u < -CL ? -CL : (u > CL ? CL : u);
                    h[o] = orc_silu(g) * u;
                }
                float th = orc_tq2_quant_act(h, hq, hs, MI);
                for (int o = 0; o < D; o++)
                    out[o] += w * orc_tq2_dot(Dn + D * 4 + (size_t)o * (MI / 4), ((const float *)Dn)[o], hq, hs, th, MI);
            } else {
                int fmt = kind == 2 ? 2 : 1, bb = fmt == 2 ? ORC_Q80_BB : ORC_Q40_BB;
                size_t grb = (size_t)nbD * bb, drb = (size_t)(MI / ORC_BLK) * bb, gate_b = grb * MI;
                const uint8_t *G = blob, *U = blob + gate_b, *Dn = blob + 2 * gate_b;
                for (int o = 0; o < MI; o++) {
                    float g = fmt == 2 ? orc_q80_dot(G + o * grb, q, qs, D) : orc_q40_dot(G + o * grb, q, qs, D);
                    float u = fmt == 2 ? orc_q80_dot(U + o * grb, q, qs, D) : orc_q40_dot(U + o * grb, q, qs, D);
                    h[o] = kind == 0 ? orc_gelu_tanh(g) * u : orc_silu(g) * u;
                }
                orc_quant_act(h, hq, hs, MI);
                for (int o = 0; o < D; o++)
                    out[o] += w * (fmt == 2 ? orc_q80_dot(Dn + o * drb, hq, hs, MI) : orc_q40_dot(Dn + o * drb, hq, hs, MI));
            }
            free(h); free(hq); free(hs);
        }
    }
    free(X); free(xq); free(sx);
}

/* Stage 1 of the layer for every routed pair (s, k): the requantized hidden row the
 * expert FFN hands to its down projection (gemma4.c:637-644; maple.c:653-660), hq [S*K][MI]
 * int8 and hs [S*K][MI/32] (tq2: also the row's Sx sum via orc_tq2_quant_act). Pairs are
 * independent, so they run in parallel; each pair's arithmetic is the scalar order. */
void orc_moe_pairs_hidden(int kind, const uint8_t *const *blobs, int E, const float *X, int S, int K,
                          const int *eidx, int D, int MI, float CL, int8_t *HQ, float *HS) {
    int nbD = D / ORC_BLK, nbM = MI / ORC_BLK;
    #pragma omp parallel for schedule(dynamic, 4)
    for (int p = 0; p < S * K; p++) {
        int s = p / K, e = eidx[p];
        int8_t *hq = HQ + (size_t)p * MI;
        float *hs = HS + (size_t)p * nbM;
        if (e < 0 || e >= E) { memset(hq, 0, (size_t)MI); memset(hs, 0, sizeof(float) * nbM); continue; }
        int8_t *xq = malloc((size_t)D);
        float *sx = malloc(sizeof(float) * nbD), *h = malloc(sizeof(float) * (size_t)MI);
        const uint8_t *blob = blobs[e];
        if (kind == 3) {
            size_t gate_b = (size_t)MI * 4 + (size_t)MI * (D / 4);
            const uint8_t *G = blob, *U = blob + gate_b;
            float tx = orc_tq2_quant_act(X + (size_t)s * D, xq, sx, D);
            for (int o = 0; o < MI; o++) {
                float g = orc_tq2_dot(G + MI * 4 + (size_t)o * (D / 4), ((const float *)G)[o], xq, sx, tx, D);
                float u = orc_tq2_dot(U + MI * 4 + (size_t)o * (D / 4), ((const float *)U)[o], xq, sx, tx, D);
                if (g > CL) g = CL;
                u = u < -CL ? -CL : (u > CL ? CL : u);
                h[o] = orc_silu(g) * u;
            }
            (void)orc_tq2_quant_act(h, hq, hs, MI);
        } else {
            int fmt = kind == 2 ? 2 : 1, bb = fmt == 2 ? ORC_Q80_BB : ORC_Q40_BB;
            size_t grb = (size_t)nbD * bb, gate_b = grb * MI;
            const uint8_t *G = blob, *U = blob + gate_b;
            orc_quant_act(X + (size_t)s * D, xq, sx, D);
            for (int o = 0; o < MI; o++) {
                float g = fmt == 2 ? orc_q80_dot(G + o * grb, xq, sx, D) : orc_q40_dot(G + o * grb, xq, sx, D);
                float u = fmt == 2 ? orc_q80_dot(U + o * grb, xq, sx, D) : orc_q40_dot(U + o * grb, xq, sx, D);
                h[o] = kind == 0 ? orc_gelu_tanh(g) * u : orc_silu(g) * u;
            }
            orc_quant_act(h, hq, hs, MI);
        }
        free(xq); free(sx); free(h);
    }
}

/* Stage 2 of the layer from given hidden rows: OUT[s] = sum_k ewt[s,k] * Down_e(hq[s*K+k])
 * (gemma4.c:647-651, 792-806; maple.c:676-690), k in slot order. OUT zeroed first. */
void orc_moe_pairs_combine(int kind, const uint8_t *const *blobs, int E, const int8_t *HQ, const float *HS,
                           int S, int K, const int *eidx, const float *ewt, int D, int MI, float *OUT) {
    int nbM = MI / ORC_BLK;
    #pragma omp parallel for schedule(dynamic, 4)
    for (int s = 0; s < S; s++) {
        float *out = OUT + (size_t)s * D;
        memset(out, 0, sizeof(float) * (size_t)D);
        for (int k = 0; k < K; k++) {
            int p = s * K + k, e = eidx[p];
            if (e < 0 || e >= E) continue;
            const int8_t *hq = HQ + (size_t)p * MI;
            const float *hs = HS + (size_t)p * nbM;
            float w = ewt[p];
            const uint8_t *blob = blobs[e];
            if (kind == 3) {
                size_t gate_b = (size_t)MI * 4 + (size_t)MI * (D / 4);
                const uint8_t *Dn = blob + 2 * gate_b;
                double tot = 0;
                for (int b = 0; b < nbM; b++) {
                    int32_t t = 0;
                    for (int j = 0; j < ORC_BLK; j++) t += hq[b * ORC_BLK + j];
                    tot += (double)hs[b] * (double)t;
                }
                for (int o = 0; o < D; o++)
                    out[o] += w * orc_tq2_dot(Dn + (size_t)D * 4 + (size_t)o * (MI / 4), ((const float *)Dn)[o], hq, hs,
                                              (float)tot, MI);
            } else {
                int fmt = kind == 2 ? 2 : 1, bb = fmt == 2 ? ORC_Q80_BB : ORC_Q40_BB;
                size_t grb = (size_t)(D / ORC_BLK) * bb, drb = (size_t)nbM * bb, gate_b = grb * MI;
                const uint8_t *Dn = blob + 2 * gate_b;
                for (int o = 0; o < D; o++)
                    out[o] += w * (fmt == 2 ? orc_q80_dot(Dn + o * drb, hq, hs, MI) : orc_q40_dot(Dn + o * drb, hq, hs, MI));
            }
        }
    }
}

/* ---- exact-activation dots (f32 x, double sums): what the reference's GPU backend is
 * checked against (gemma4.c:2315-2361, maple.c:1756-1800) ---- */

/* q40_dot_f32 (q40.h:290-305) */
float orc_q40_dot_f32(const uint8_t *w, const float *x, int I) {
    double acc = 0;
    for (int b = 0; b < I / ORC_BLK; b++) {
        const uint8_t *blk = w + (size_t)b * ORC_Q40_BB;
        uint16_t hd; memcpy(&hd, blk, 2);
        const float *v = x + b * ORC_BLK;
        double s = 0;
        for (int j = 0; j < 16; j++) {
            s += (double)((int)(blk[2 + j] & 15) - 8) * v[j];
            s += (double)((int)(blk[2 + j] >> 4) - 8) * v[j + 16];
        }
        acc += (double)orc_fp16_to_f32(hd) * s;
    }
    return (float)acc;
}

/* q80_dot_f32 (q40.h:443-455) */
float orc_q80_dot_f32(const uint8_t *w, const float *x, int I) {
    double acc = 0;
    for (int b = 0; b < I / ORC_BLK; b++) {
        const uint8_t *blk = w + (size_t)b * ORC_Q80_BB;
        uint16_t hd; memcpy(&hd, blk, 2);
        const int8_t *a = (const int8_t *)(blk + 2);
        double s = 0;
        for (int j = 0; j < ORC_BLK; j++) s += (double)a[j] * x[b * ORC_BLK + j];
        acc += (double)orc_fp16_to_f32(hd) * s;
    }
    return (float)acc;
}

/* tq2_dot_f32 (tq2.h:235-252): codes of one row, 16 bytes per 64-weight group */
float orc_tq2_dot_f32(const uint8_t *codes, float alpha, const float *x, int I) {
    double acc = 0;
    for (int g = 0; g < I / 64; g++) {
        const uint8_t *c = codes + (size_t)g * 16;
        const float *v = x + (size_t)g * 64;
        double s = 0;
        for (int k = 0; k < 16; k++) {
            s += (double)((int)(c[k] & 3) - 1) * v[k];
            s += (double)((int)((c[k] >> 2) & 3) - 1) * v[k + 16];
            s += (double)((int)((c[k] >> 4) & 3) - 1) * v[k + 32];
            s += (double)((int)(c[k] >> 6) - 1) * v[k + 48];
        }
        acc += s;
    }
    return (float)((double)alpha * acc);
}

/* q4a: 64-weight groups of 36 bytes, fp16 d, fp16 m, two 16-byte nibble blocks;
 * w = d*q + m (tq2.h:268-283). q4a_dot_f32 (tq2.h:410-432) */
float orc_q4a_dot_f32(const uint8_t *w, const float *x, int I) {
    double acc = 0;
    for (int g = 0; g < I / 64; g++) {
        const uint8_t *grp = w + (size_t)g * 36;
        uint16_t hd, hm; memcpy(&hd, grp, 2); memcpy(&hm, grp + 2, 2);
        double d = orc_fp16_to_f32(hd), m = orc_fp16_to_f32(hm);
        for (int h = 0; h < 2; h++) {
            const uint8_t *nib = grp + 4 + h * 16;
            const float *u = x + (size_t)g * 64 + h * 32;
            double s = 0, t = 0;
            for (int j = 0; j < 16; j++) {
                s += (double)(nib[j] & 15) * u[j];
                s += (double)(nib[j] >> 4) * u[j + 16];
                t += (double)u[j] + (double)u[j + 16];
            }
            acc += d * s + m * t;
        }
    }
    return (float)acc;
}

/* q4a_dot with q8_0 activations, the scalar form (tq2.h:390-408) */
float orc_q4a_dot(const uint8_t *w, const int8_t *xq, const float *sx, int I) {
    double acc = 0;
    for (int g = 0; g < I / 64; g++) {
        const uint8_t *grp = w + (size_t)g * 36;
        uint16_t hd, hm; memcpy(&hd, grp, 2); memcpy(&hm, grp + 2, 2);
        float d = orc_fp16_to_f32(hd), m = orc_fp16_to_f32(hm);
        for (int h = 0; h < 2; h++) {
            const uint8_t *nib = grp + 4 + h * 16;
            const int8_t *v = xq + (size_t)g * 64 + h * 32;
            int32_t dp = 0, sv = 0;
            for (int j = 0; j < 16; j++) {
                dp += (int)(nib[j] & 15) * (int)v[j];
                dp += (int)(nib[j] >> 4) * (int)v[j + 16];
                sv += (int)v[j] + (int)v[j + 16];
            }
            acc += (double)sx[2 * g + h] * ((double)d * dp + (double)m * sv);
        }
    }
    return (float)acc;
}

/* y[o] for a whole tensor: fmt 1 q4_0, 2 q8_0, 3 tq2 (T = alphas then codes), 4 q4a */
void orc_matvec_f32(int fmt, float *y, const uint8_t *T, const float *x, int O, int I) {
    for (int o = 0; o < O; o++) {
        if (fmt == 1) y[o] = orc_q40_dot_f32(T + (size_t)o * (I / ORC_BLK) * ORC_Q40_BB, x, I);
        else if (fmt == 2) y[o] = orc_q80_dot_f32(T + (size_t)o * (I / ORC_BLK) * ORC_Q80_BB, x, I);
        else if (fmt == 3) y[o] = orc_tq2_dot_f32(T + (size_t)O * 4 + (size_t)o * (I / 4), ((const float *)T)[o], x, I);
        else y[o] = orc_q4a_dot_f32(T + (size_t)o * (I / 64) * 36, x, I);
    }
}
void orc_q4a_matvec(float *y, const uint8_t *T, const int8_t *xq, const float *sx, int O, int I) {
    for (int o = 0; o < O; o++) y[o] = orc_q4a_dot(T + (size_t)o * (I / 64) * 36, xq, sx, I);
}

/* ---- routers ---- */

/* gemma4 route_row (gemma4.c:581-613) for one residual row: rmsnorm without weight
 * (double sum of squares, gemma4.c:425-431), times router_scale * D^-1/2, f32 logits
 * as a sequential fused multiply-add chain (the reference is built with -mfma and the
 * default contraction, so `v += RP * xn` is one fma per term), top-K by insertion in
 * expert order (ties keep the lower index), softmax over the K, times the per-expert
 * scale. */
void orc_gemma4_route(const float *res, int D, int E, int K, const float *proj, const float *scale,
                      const float *pes, float eps, int *idx, float *wts) {
    float *xn = malloc(sizeof(float) * (size_t)D);
    double s = 0;
    for (int i = 0; i < D; i++) s += (double)res[i] * res[i];
    float r = 1.0f / sqrtf((float)(s / D) + eps);
    float rs = 1.0f / sqrtf((float)D);
    for (int i = 0; i < D; i++) {
        xn[i] = res[i] * r;
        xn[i] *= scale[i] * rs;
    }
    float topv[64];
    for (int j = 0; j < K; j++) { idx[j] = -1; topv[j] = -INFINITY; }
    for (int e = 0; e < E; e++) {
        float v = 0.0f;
        for (int i = 0; i < D; i++) v += proj[(size_t)e * D + i] * xn[i];
        int j = K;
        while (j > 0 && v > topv[j - 1]) j--;
        if (j == K) continue;
        for (int t = K - 1; t > j; t--) { topv[t] = topv[t - 1]; idx[t] = idx[t - 1]; }
        topv[j] = v; idx[j] = e;
    }
    float sum = 0.0f, mx = topv[0];
    for (int j = 0; j < K; j++) { wts[j] = expf(topv[j] - mx); sum += wts[j]; }
    for (int j = 0; j < K; j++) wts[j] = (wts[j] / sum) * pes[idx[j]];
    free(xn);
}

/* ling route_row (ling.c:705-789) for one normalized row: per expert the double dot
 * with 8 interleaved accumulators, sigmoid score, biased selection score; groups of
 * E/NG ranked by the sum of their two best biased scores, the best TG kept (ties keep
 * the lower index); top-K of the kept experts by biased score in expert order; weights
 * the unbiased scores, renormalised over the K when norm_topk, times routed_scale. */
void orc_ling_route(const float *xn, int D, int E, int K, int NG, int TG, int norm_topk, float routed_scale,
                    const float *router, const float *bias, int *idx, float *wts) {
    float *rwt = malloc(sizeof(float) * (size_t)E), *rsel = malloc(sizeof(float) * (size_t)E);
    int EG = E / NG;
    for (int e = 0; e < E; e++) {
        const float *r = router + (size_t)e * D;
        double s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= D; i += 8)
            for (int k = 0; k < 8; k++) s[k] += (double)r[i + k] * xn[i + k];
        for (; i < D; i++) s[0] += (double)r[i] * xn[i];
        double v = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
        rwt[e] = 1.0f / (1.0f + expf(-(float)v));
        rsel[e] = rwt[e] + bias[e];
    }
    float gs[64], topg[64], topv[64];
    int keep[64];
    for (int g = 0; g < NG; g++) {
        float a = -INFINITY, bb = -INFINITY;
        for (int i = 0; i < EG; i++) {
            float v = rsel[g * EG + i];
            if (v > a) { bb = a; a = v; }
            else if (v > bb) bb = v;
        }
        gs[g] = EG > 1 ? a + bb : a;
    }
    for (int j = 0; j < TG; j++) { keep[j] = -1; topg[j] = -INFINITY; }
    for (int g = 0; g < NG; g++) {
        int j = TG;
        while (j > 0 && gs[g] > topg[j - 1]) j--;
        if (j == TG) continue;
        for (int t = TG - 1; t > j; t--) { topg[t] = topg[t - 1]; keep[t] = keep[t - 1]; }
        topg[j] = gs[g]; keep[j] = g;
    }
    unsigned char live[64] = {0};
    for (int j = 0; j < TG; j++) if (keep[j] >= 0) live[keep[j]] = 1;
    for (int j = 0; j < K; j++) { idx[j] = -1; topv[j] = -INFINITY; }
    for (int e = 0; e < E; e++) {
        if (!live[e / EG]) continue;
        float v = rsel[e];
        int j = K;
        while (j > 0 && v > topv[j - 1]) j--;
        if (j == K) continue;
        for (int t = K - 1; t > j; t--) { topv[t] = topv[t - 1]; idx[t] = idx[t - 1]; }
        topv[j] = v; idx[j] = e;
    }
    float sum = 0.0f;
    for (int j = 0; j < K; j++) { wts[j] = rwt[idx[j]]; sum += wts[j]; }
    if (norm_topk && K > 1)
        for (int j = 0; j < K; j++) wts[j] /= (sum + 1e-20f);
    for (int j = 0; j < K; j++) wts[j] *= routed_scale;
    free(rwt); free(rsel);
}
