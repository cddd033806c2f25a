/* ref_maple.c -- TEST INFRASTRUCTURE ONLY. Compiles the reference's maple.c engine
 * translation unit (and through it tq2.h) from its source location and exports its
 * ternary hot path with C linkage: tq2_quant_act / tq2_dot (tq2.h:98-155), the
 * engine-style matvec, route_row (maple.c:582-601) and expert_apply (maple.c:612-692).
 * Built by oracle/Makefile into oracle/_ref/libzzref.so. */
#define main ref_maple_main
#include REF_MAPLE
#undef main

float ref_tq2_quant_act(const float *x, int8_t *xq, float *sx, int I) { return tq2_quant_act(x, xq, sx, I); }
float ref_tq2_dot(const uint8_t *codes, float alpha, const int8_t *xq, const float *sx, float sxtot, int I) {
    return tq2_dot(codes, alpha, xq, sx, sxtot, I);
}
void ref_tq2_matvec_omp(float *y, const uint8_t *T, const int8_t *xq, const float *sx, float sxtot,
                        int O, int I) {
    const float *al = tq2_alphas(T);
    const uint8_t *cd = tq2_codes(T, O);
    #pragma omp parallel for schedule(static)
    for (int o = 0; o < O; o++) y[o] = tq2_dot(cd + (size_t)o * tq2_row_bytes(I), al[o], xq, sx, sxtot, I);
}

/* top-k + softmax over the k (norm_topk_prob set) */
void ref_route_topk(const float *logits, int E, int K, int *idx, float *wts) {
    M m; memset(&m, 0, sizeof m);
    m.c.n_experts = E; m.c.topk = K; m.c.norm_topk_prob = 1;
    route_row(&m, logits, idx, wts);
}

static M g_mm;
static Buf g_mb;
static int g_mD, g_mMI, g_mcap;
static void ref_mp_setup(int D, int MI, int cap, float CL) {
    g_mm.c.mlp_clamp = CL;
    if (g_mD == D && g_mMI == MI && g_mcap >= cap) return;
    free(g_mb.eact.q); free(g_mb.eact.s); free(g_mb.eact.tot);
    free(g_mb.hact.q); free(g_mb.hact.s); free(g_mb.hact.tot); free(g_mb.egate);
    memset(&g_mm, 0, sizeof g_mm); memset(&g_mb, 0, sizeof g_mb);
    g_mm.c.hidden = D; g_mm.c.moe_inter = MI; g_mm.c.mlp_clamp = CL;
    g_mm.gate_b = tq2_tensor_bytes(MI, D);
    size_t R = (size_t)cap;
    g_mb.eact.q = calloc(R * D, 1); g_mb.eact.s = calloc(R * (D / Q40_BLK), sizeof(float));
    g_mb.eact.tot = calloc(R, sizeof(float));
    g_mb.hact.q = calloc(R * MI, 1); g_mb.hact.s = calloc(R * (MI / Q40_BLK), sizeof(float));
    g_mb.hact.tot = calloc(R, sizeof(float));
    g_mb.egate = calloc(R * MI, sizeof(float));
    g_mD = D; g_mMI = MI; g_mcap = cap;
}
void ref_maple_expert_apply(const uint8_t *blob, const float *X, float *OUT, const int *rows,
                            int nrows, const float *w, int D, int MI, float CL) {
    ref_mp_setup(D, MI, nrows > 0 ? nrows : 1, CL);
    g_use_gpu = 0;
    expert_apply(&g_mm, blob, X, OUT, rows, nrows, w, &g_mb);
}
void ref_maple_moe_layer(const uint8_t *const *blobs, const float *X, float *OUT, int S, int K,
                         const int *eidx, const float *ewt, int D, int MI, int E, float CL) {
    int *uniq = malloc(sizeof(int) * (size_t)E), nu = 0;
    int *rows = malloc(sizeof(int) * (size_t)S * K);
    float *wr = malloc(sizeof(float) * (size_t)S * K);
    for (int s = 0; s < S; s++) for (int j = 0; j < K; j++) {
        int e = eidx[s * K + j], seen = 0;
        for (int u = 0; u < nu; u++) if (uniq[u] == e) { seen = 1; break; }
        if (!seen) uniq[nu++] = e;
    }
    memset(OUT, 0, sizeof(float) * (size_t)S * D);
    ref_mp_setup(D, MI, S, CL);
    g_use_gpu = 0;
    for (int u = 0; u < nu; u++) {
        int e = uniq[u], n = 0;
        for (int s = 0; s < S; s++) for (int j = 0; j < K; j++)
            if (eidx[s * K + j] == e) { rows[n] = s; wr[n++] = ewt[s * K + j]; }
        expert_apply(&g_mm, blobs[e], X, OUT, rows, n, wr, &g_mb);
    }
    free(uniq); free(rows); free(wr);
}

/* exact-activation tq2 and q4a dots and the q8_0-activation q4a dot (tq2.h:235-252,
 * 390-432), for pinning the restatement */
float ref_tq2_dot_f32(const uint8_t *codes, float alpha, const float *x, int I) { return tq2_dot_f32(codes, alpha, x, I); }
float ref_q4a_dot_f32(const uint8_t *w, const float *x, int I) { return q4a_dot_f32(w, x, I); }
float ref_q4a_dot(const uint8_t *w, const int8_t *xq, const float *sx, int I) { return q4a_dot(w, xq, sx, I); }
