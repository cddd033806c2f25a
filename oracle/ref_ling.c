/* ref_ling.c -- TEST INFRASTRUCTURE ONLY. Compiles the reference's ling.c engine
 * translation unit from its source location and exports its grouped router
 * (route_row, ling.c:705-789) with C linkage. Built by oracle/Makefile into
 * oracle/_ref/libzzref.so. */
#define main ref_ling_main
#include REF_LING
#undef main

/* route S normalized rows xn [S][D] through layer 0 of a model holding only the router
 * tensors (router [E][D] f32, expert_bias [E]): idx / wts [S][K] */
void ref_ling_route(const float *xn, int S, int D, int E, int K, int n_group, int topk_group, int norm_topk_prob,
                    float routed_scale, const float *router, const float *bias, int *idx, float *wts) {
    static M m;
    memset(&m, 0, sizeof m);
    m.c.hidden = D; m.c.n_experts = E; m.c.topk = K;
    m.c.n_group = n_group; m.c.topk_group = topk_group; m.c.norm_topk_prob = norm_topk_prob;
    m.c.routed_scale = routed_scale;
    m.L[0].router.f = router; m.L[0].expert_bias.f = bias;
    Buf b;
    memset(&b, 0, sizeof b);
    b.rwt = malloc(sizeof(float) * (size_t)E);
    b.rsel = malloc(sizeof(float) * (size_t)E);
    for (int s = 0; s < S; s++)
        route_row(&m, 0, s, xn + (size_t)s * D, idx + (size_t)s * K, wts + (size_t)s * K, &b);
    free(b.rwt); free(b.rsel);
}
