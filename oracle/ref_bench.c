/*
 * ref_bench.c -- timing harness for the reference's own C99 runtime
 * (PRIME-Moment-Attention c/prime_moment.c, compiled unmodified into
 * oracle/_ref/libprime_ref.so by oracle/Makefile).
 *
 * TEST/BENCH INFRASTRUCTURE ONLY: bench.py's reference arm and CPU-baseline leg
 * run it; the product never does.
 *
 * It drives the reference API exactly as its own CLI does (c/main.c:375-471):
 * prime_state_create + prime_prefill / prime_step, here in the additive mode
 * that matches the PyTorch path's operation count (use_delta_rule = 0,
 * lyapunov_bound = 0, use_qk_norm = 0, eps = 1.0).  Note that the reference's
 * additive mode stores S as [value][key] (c/prime_moment.c:285-300) and so
 * computes (q.v_i) k_i where the PyTorch path computes (q.k_i) v_i; the
 * operation count and memory traffic are the same, which is all a timing
 * baseline needs.  It is never used as a parity oracle.
 *
 * Independent prime_state_t objects (one per batch row, or one per
 * sequence x layer for decode) are spread over T pthreads.
 *
 *   ref_bench prefill <B> <H> <L> <D> <threads>
 *       B states of H heads each; prefill L tokens into each.
 *       prints {"tokens": B*L, "seconds": s, "tok_per_s": ..., "threads": T}
 *   ref_bench decode <S> <H> <D> <steps> <threads>
 *       S states of H heads each; <steps> decode steps over all of them.
 *       prints {"states": S, "steps": n, "seconds": s, "us_per_step": ..., "threads": T}
 */
#define _GNU_SOURCE
#include "prime_moment.h"

#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now_s(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

static unsigned long long rng_state = 0x9E3779B97F4A7C15ull;
static float frand(void)
{
    rng_state ^= rng_state << 13; rng_state ^= rng_state >> 7; rng_state ^= rng_state << 17;
    return (float)((rng_state >> 11) * (1.0 / 9007199254740992.0)) - 0.5f;
}

typedef struct {
    prime_config_t cfg;
    prime_state_t **states;
    int first, count;      /* states handled by this thread */
    int L;                 /* tokens (prefill) or steps (decode) */
    int mode;              /* 0 prefill, 1 decode */
    const float *q, *k, *v; /* [L, H, D] shared inputs */
    float *out;            /* per-thread scratch [L, H, D] */
} job_t;

static void *worker(void *p)
{
    job_t *j = (job_t *)p;
    const int HD = j->cfg.num_heads * j->cfg.head_dim;
    if (j->mode == 0) {
        for (int s = j->first; s < j->first + j->count; ++s)
            prime_prefill(&j->cfg, j->states[s], j->L, j->q, j->k, j->v, j->out);
    } else {
        for (int t = 0; t < j->L; ++t)
            for (int s = j->first; s < j->first + j->count; ++s)
                prime_step(&j->cfg, j->states[s], j->q + (size_t)t * HD, j->k + (size_t)t * HD,
                           j->v + (size_t)t * HD, j->out);
    }
    return NULL;
}

int main(int argc, char **argv)
{
    if (argc < 2) { fprintf(stderr, "usage: ref_bench prefill|decode ...\n"); return 2; }
    const int decode = strcmp(argv[1], "decode") == 0;
    if (!decode && strcmp(argv[1], "prefill") != 0) { fprintf(stderr, "bad mode\n"); return 2; }
    if (argc < 7) { fprintf(stderr, "missing arguments\n"); return 2; }
    const int nstates = atoi(argv[2]), H = atoi(argv[3]);
    const int L = decode ? atoi(argv[5]) : atoi(argv[4]);
    const int D = decode ? atoi(argv[4]) : atoi(argv[5]);
    int T = atoi(argv[6]);
    if (nstates <= 0 || H <= 0 || L <= 0 || D <= 0 || T <= 0) { fprintf(stderr, "bad sizes\n"); return 2; }
    if (T > nstates) T = nstates;

    prime_config_t cfg = prime_default_config(H, D);
    cfg.use_delta_rule = 0;
    cfg.lyapunov_bound = 0.0f;
    cfg.use_qk_norm = 0;
    cfg.eps = 1.0f;

    const size_t n = (size_t)L * H * D;
    float *q = malloc(n * sizeof(float)), *k = malloc(n * sizeof(float)), *v = malloc(n * sizeof(float));
    if (!q || !k || !v) return 3;
    for (size_t i = 0; i < n; ++i) { q[i] = frand(); k[i] = frand(); v[i] = frand(); }

    prime_state_t **states = malloc(sizeof(*states) * nstates);
    for (int s = 0; s < nstates; ++s) {
        states[s] = prime_state_create(H, D);
        if (!states[s]) return 3;
    }
    job_t *jobs = calloc(T, sizeof(job_t));
    pthread_t *th = calloc(T, sizeof(pthread_t));
    int first = 0;
    for (int t = 0; t < T; ++t) {
        const int cnt = nstates / T + (t < nstates % T);
        jobs[t] = (job_t){cfg, states, first, cnt, L, decode, q, k, v, NULL};
        jobs[t].out = malloc((decode ? (size_t)H * D : n) * sizeof(float));
        first += cnt;
    }
    const double t0 = now_s();
    for (int t = 0; t < T; ++t) pthread_create(&th[t], NULL, worker, &jobs[t]);
    for (int t = 0; t < T; ++t) pthread_join(th[t], NULL);
    const double dt = now_s() - t0;

    if (decode)
        printf("{\"states\": %d, \"heads\": %d, \"steps\": %d, \"seconds\": %.6f, "
               "\"us_per_step\": %.3f, \"threads\": %d}\n",
               nstates, H, L, dt, 1e6 * dt / L, T);
    else
        printf("{\"tokens\": %lld, \"heads\": %d, \"seconds\": %.6f, \"tok_per_s\": %.3f, \"threads\": %d}\n",
               (long long)nstates * L, H, dt, (double)nstates * L / dt, T);

    for (int s = 0; s < nstates; ++s) prime_state_free(states[s]);
    for (int t = 0; t < T; ++t) free(jobs[t].out);
    free(states); free(jobs); free(th); free(q); free(k); free(v);
    return 0;
}
