/* ref_gemma4.c -- TEST INFRASTRUCTURE ONLY. Compiles the reference's own gemma4.c
 * engine translation unit (and through it q40.h) from its source location and
 * exports its static hot-path routines with C linkage, so the restatement in
 * zz_oracle.c and the golden fixtures can be checked against the reference itself.
 * Built by oracle/Makefile into oracle/_ref/libzzref.so; REF_SRC is the reference
 * tree. No reference source is copied into this repository.
 *
 * The wrappers fill only the model/buffer fields that expert_apply (gemma4.c:656-711)
 * and expert_apply_batch_cpu (gemma4.c:618-654) read, with the per-row strides the
 * engine allocates (gemma4.c:2123-2127). */
#define main ref_gemma4_main
#include REF_GEMMA4
#undef main
#include <omp.h>

void ref_set_threads(int n) { omp_set_num_threads(n); }
int ref_max_threads(void) { return omp_get_max_threads(); }

void ref_q40_quant_row(const float *w, uint8_t *dst, int I) { q40_quant_row(w, dst, I); }
void ref_q80_quant_row(const float *w, uint8_t *dst, int I) { q80_quant_row(w, dst, I); }
void ref_quant_act(const float *x, int8_t *xq, float *sx, int I) { q40_quant_act(x, xq, sx, I); }
float ref_q40_dot(const uint8_t *w, const int8_t *xq, const float *sx, int I) { return q40_dot(w, xq, sx, I); }
float ref_q80_dot(const uint8_t *w, const int8_t *xq, const float *sx, int I) { return q80_dot(w, xq, sx, I); }
float ref_q40_dot_f32(const uint8_t *w, const float *x, int I) { return q40_dot_f32(w, x, I); }
uint16_t ref_f32_to_fp16(float f) { return q40_f32_to_fp16(f); }
float ref_fp16_to_f32(uint16_t h) { return q40_fp16_to_f32(h); }

/* the engines' matvec: act quant once, OpenMP over output rows (gemma4.c:441-457) */
void ref_q40_matvec_omp(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I) {
    size_t rb = (size_t)q40_row_bytes(I);
    #pragma omp parallel for schedule(static)
    for (int o = 0; o < O; o++) y[o] = q40_dot(W + (size_t)o * rb, xq, sx, I);
}
void ref_q80_matvec_omp(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I) {
    size_t rb = (size_t)q80_row_bytes(I);
    #pragma omp parallel for schedule(static)
    for (int o = 0; o < O; o++) y[o] = q80_dot(W + (size_t)o * rb, xq, sx, I);
}

static M g_m;
static Buf g_b;
static int g_D, g_MI, g_rows_cap;

static void ref_g4_setup(int D, int MI, int rows_cap) {
    if (g_D == D && g_MI == MI && g_rows_cap >= rows_cap) return;
    free(g_b.egate); free(g_b.esx); free(g_b.ehs); free(g_b.exq); free(g_b.ehq);
    free(g_b.xq); free(g_b.hq); free(g_b.sx); free(g_b.hs); free(g_b.gate);
    memset(&g_m, 0, sizeof g_m); memset(&g_b, 0, sizeof g_b);
    g_m.c.hidden = D; g_m.c.moe_inter = MI;
    g_m.gate_b = q40_tensor_bytes(MI, D);
    size_t R = (size_t)rows_cap;
    g_b.egate = calloc(R * (MI + 64), sizeof(float));
    g_b.exq = calloc(R * (D + 64), 1);
    g_b.esx = calloc(R * (D / Q40_BLK + 8), sizeof(float));
    g_b.ehq = calloc(R * (MI + 64), 1);
    g_b.ehs = calloc(R * (MI / Q40_BLK + 8), sizeof(float));
    g_b.xq = calloc(D + 64, 1); g_b.sx = calloc(D / Q40_BLK + 8, sizeof(float));
    g_b.hq = calloc(MI + 64, 1); g_b.hs = calloc(MI / Q40_BLK + 8, sizeof(float));
    g_b.gate = calloc(MI + 64, sizeof(float));
    g_D = D; g_MI = MI; g_rows_cap = rows_cap;
}

/* one expert over its routed rows: OUT[rows[r]] += w[r] * FFN(X[rows[r]]) */
void ref_gemma4_expert_apply(const uint8_t *blob, const float *X, float *OUT,
                             const int *rows, int nrows, const float *w, int D, int MI) {
    ref_g4_setup(D, MI, nrows > 0 ? nrows : 1);
    g_use_gpu = 0;
    expert_apply(&g_m, blob, X, OUT, rows, nrows, w, &g_b);
}

/* the batch-union layer: union of experts in first-seen order and per-expert row
 * gather as moe_start / moe_apply_chunk do (gemma4.c:756-761, 781-783), then the
 * engine's own expert_apply per expert; OUT is zeroed first (gemma4.c:766). */
void ref_gemma4_moe_layer(const uint8_t *const *blobs, const float *X, float *OUT, int S, int K,
                          const int *eidx, const float *ewt, int D, int MI, int E) {
    int *uniq = malloc(sizeof(int) * (size_t)E), nu = 0;
    int *rows = malloc(sizeof(int) * (size_t)S * K);
    float *wr = malloc(sizeof(float) * (size_t)S * K);
    for (int s = 0; s < S; s++) for (int j = 0; j < K; j++) {
        int e = eidx[s * K + j], seen = 0;
        for (int u = 0; u < nu; u++) if (uniq[u] == e) { seen = 1; break; }
        if (!seen) uniq[nu++] = e;
    }
    memset(OUT, 0, sizeof(float) * (size_t)S * D);
    ref_g4_setup(D, MI, S);
    g_use_gpu = 0;
    for (int u = 0; u < nu; u++) {
        int e = uniq[u], n = 0;
        for (int s = 0; s < S; s++) for (int j = 0; j < K; j++)
            if (eidx[s * K + j] == e) { rows[n] = s; wr[n++] = ewt[s * K + j]; }
        expert_apply(&g_m, blobs[e], X, OUT, rows, n, wr, &g_b);
    }
    free(uniq); free(rows); free(wr);
}

/* exact-activation q8_0 dot (q40.h:443-455), for pinning the restatement */
float ref_q80_dot_f32(const uint8_t *w, const float *x, int I) { return q80_dot_f32(w, x, I); }

/* the engine's own router (gemma4.c:581-613) over S residual rows, layer 0 of a model
 * holding only the router tensors: idx / wts [S][K] */
void ref_gemma4_route(const float *res, int S, int D, int E, int K, const float *proj, const float *scale,
                      const float *pes, float eps, int *idx, float *wts) {
    static M m;
    memset(&m, 0, sizeof m);
    m.c.hidden = D; m.c.n_experts = E; m.c.topk = K; m.c.eps = eps;
    m.L[0].router_proj.f = proj; m.L[0].router_scale.f = scale; m.L[0].router_pes.f = pes;
    Buf b;
    memset(&b, 0, sizeof b);
    b.xn = malloc(sizeof(float) * (size_t)D);
    for (int s = 0; s < S; s++) route_row(&m, 0, res + (size_t)s * D, idx + (size_t)s * K, wts + (size_t)s * K, &b);
    free(b.xn);
}

/* the engine's own container parser (manifest(), gemma4.c:260-403) on a directory:
 * esz / gate_b / down_b and the first n entries of the expert offset table; returns
 * n_layers * n_experts */
int ref_gemma4_manifest(const char *dir, long long *esz3, long long *eoff, int n) {
    static M m;
    memset(&m, 0, sizeof m);
    g_use_gpu = 0;
    manifest(&m, dir);
    esz3[0] = m.esz; esz3[1] = m.gate_b; esz3[2] = m.down_b;
    int tot = m.c.n_layers * m.c.n_experts;
    for (int i = 0; i < n && i < tot; i++) eoff[i] = m.eoff[i];
    close(m.efd);
    free(m.eoff);
    free((void *)m.dense);
    return tot;
}
