/* C part of the CPU oracle (TEST INFRASTRUCTURE, not product code).
 *
 * Fixed-order fp32 reductions that a device kernel can reproduce bit for bit.  The reference computes router
 * logits with `F.linear(x.float(), router_w.float())` (chronos_1t/models/vllm_chronos_moe.py:311,
 * chronos_1t/models/glm53_chronos_moe.py:393); the value of an fp32 dot product depends on the order of its
 * additions, so this file states ONE order and the CUDA router follows the same one.
 *
 * Order: 32 lanes; lane l accumulates the products at k = 128*j + 4*l + i for j = 0, 1, ... and i = 0..3
 * (j ascending, then i) with fused multiply-adds starting from +0.0f (columns >= h contribute nothing); then
 * lanes are combined with the xor butterfly (offsets 16, 8, 4, 2, 1): p[l] = p[l] + p[l ^ off].
 * fp32 addition is commutative, so every lane ends with the same value; lane 0 is returned.
 */
#include <math.h>
#include <stddef.h>
#include <pthread.h>

static int g_threads = 0;

void oracle_set_threads(int n) { g_threads = n; }

static float dot_fixed(const float* x, const float* w, int h) {
    float p[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int j = 0; j < h; j += 128)
            for (int i = 0; i < 4; ++i) {
                const int k = j + 4 * l + i;
                if (k < h) acc = fmaf(x[k], w[k], acc);
            }
        p[l] = acc;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float q[32];
        for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ off];
        for (int l = 0; l < 32; ++l) p[l] = q[l];
    }
    return p[0];
}

typedef struct { const float *x, *wr; float* out; int n_exp, hidden; long lo, hi; } job_t;

static void* job_run(void* p) {
    job_t* j = (job_t*)p;
    for (long i = j->lo; i < j->hi; ++i) {
        int t = (int)(i / j->n_exp), e = (int)(i % j->n_exp);
        j->out[i] = dot_fixed(j->x + (size_t)t * j->hidden, j->wr + (size_t)e * j->hidden, j->hidden);
    }
    return NULL;
}

/* out[t, e] = dot_fixed(x[t, :], wr[e, :]) ; work split over `oracle_set_threads` pthreads (default 1) */
void oracle_router_logits_fixed(const float* x, const float* wr, float* out, int n_tok, int n_exp, int hidden) {
    int nt = g_threads > 0 ? g_threads : 1;
    if (nt > 64) nt = 64;
    long total = (long)n_tok * n_exp;
    pthread_t th[64];
    job_t jobs[64];
    for (int i = 0; i < nt; ++i) {
        jobs[i] = (job_t){x, wr, out, n_exp, hidden, total * i / nt, total * (i + 1) / nt};
        if (i + 1 < nt) pthread_create(&th[i], NULL, job_run, &jobs[i]);
    }
    job_run(&jobs[nt - 1]);
    for (int i = 0; i + 1 < nt; ++i) pthread_join(th[i], NULL);
}
