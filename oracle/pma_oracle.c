/*
 * pma_oracle.c -- CPU restatement, in float64, of PRIME moment attention's hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA kernels of
 * prime_moment_attention_b200 are compared against.  It is loaded by tests/,
 * by __graft_entry__.smoke() and by bench.py's CPU-baseline leg, and by nothing
 * else: the product path never calls it and has no CPU fallback.
 *
 * What it restates (reference paths are relative to the PRIME-Moment-Attention
 * project root):
 *
 *   orc_decode_step   src/prime_moment_attention/attention.py:120-143
 *                     (the L == 1 branch of PrimeMomentAttention.forward):
 *                       S0 = l*S0 + v            Z0 = l*Z0 + 1
 *                       S1 = l*S1 + k (x) v      Z1 = l*Z1 + k
 *                       S2 = l*S2 + k^2 (x) v    Z2 = l*Z2 + k^2
 *                       num = S0 + q.S1 + 0.5 q^2.S2       (contract the key index)
 *                       den = max(Z0 + q.Z1 + 0.5 q^2.Z2, eps)
 *                       y   = num / den
 *                     The update comes before the readout, so token t sees itself.
 *                     S1[d][e] = sum k_d v_e: row = key index, column = value index
 *                     (attention.py:127).  The reference calls Z0,Z1,Z2 K0,K1,K2.
 *
 *   orc_prefill       the same recurrence iterated over L tokens.  In exact
 *                     arithmetic this equals chunked_prime_ssd_core
 *                     (src/prime_moment_attention/chunked_ssd.py:48-184) for any
 *                     chunk size, including its zero padding of a ragged last
 *                     chunk and the lambda^(-pad) correction of the final state
 *                     (chunked_ssd.py:65-69, 97-99, 171-178), and it also defines
 *                     the result with an incoming state, which the reference
 *                     chunked core mishandles (chunked_ssd.py:129-137 broadcasts
 *                     [B,H,1,D] against [1,1,nc,1,1]).
 *
 * Extension over the reference: lambda may differ per head (and per batch row).
 * The reference holds one scalar decay per module (attention.py:49); heads are
 * independent, so the per-head result equals the reference run once per head
 * slice, which is how tests/golden/make_golden.py pins this file.
 *
 * Build: oracle/Makefile -> oracle/liboracle.so (gcc -O2 -fPIC -shared).
 */
#include <math.h>
#include <stddef.h>
#include <string.h>

#define ORC_OK 0
#define ORC_EINVAL 1

/* One head-state step.  Pointers address a single head. */
static void step_head(int D, double lam, double eps,
                      const double *q, const double *k, const double *v,
                      double *S0, double *S1, double *S2,
                      double *Z0, double *Z1, double *Z2, double *y)
{
    /* state update (attention.py:126-132) */
    for (int d = 0; d < D; ++d) {
        const double kd = k[d], kd2 = k[d] * k[d];
        double *s1 = S1 + (size_t)d * D, *s2 = S2 + (size_t)d * D;
        for (int e = 0; e < D; ++e) {
            s1[e] = lam * s1[e] + kd * v[e];
            s2[e] = lam * s2[e] + kd2 * v[e];
        }
        Z1[d] = lam * Z1[d] + kd;
        Z2[d] = lam * Z2[d] + kd2;
    }
    for (int e = 0; e < D; ++e) S0[e] = lam * S0[e] + v[e];
    *Z0 = lam * (*Z0) + 1.0;

    /* readout (attention.py:135-143) */
    double den = *Z0;
    for (int d = 0; d < D; ++d) den += q[d] * Z1[d] + 0.5 * q[d] * q[d] * Z2[d];
    if (den < eps) den = eps;
    for (int e = 0; e < D; ++e) {
        double num = S0[e];
        for (int d = 0; d < D; ++d)
            num += q[d] * S1[(size_t)d * D + e] + 0.5 * q[d] * q[d] * S2[(size_t)d * D + e];
        y[e] = num / den;
    }
}

/*
 * One decode step for N*H independent head-states.
 *   q,k,v,y : [N,H,D] contiguous
 *   lam     : lam[n*lam_stride_n + h]
 *   state   : S0[N,H,D] S1[N,H,D,D] S2[N,H,D,D] Z0[N,H] Z1[N,H,D] Z2[N,H,D], updated in place
 */
int orc_decode_step(int N, int H, int D,
                    const double *q, const double *k, const double *v,
                    const double *lam, long lam_stride_n, double eps,
                    double *S0, double *S1, double *S2,
                    double *Z0, double *Z1, double *Z2, double *y)
{
    if (N < 0 || H <= 0 || D <= 0 || !lam) return ORC_EINVAL;
    for (int n = 0; n < N; ++n)
        for (int h = 0; h < H; ++h) {
            const size_t i = (size_t)n * H + h;
            step_head(D, lam[(size_t)n * lam_stride_n + h], eps,
                      q + i * D, k + i * D, v + i * D,
                      S0 + i * D, S1 + i * D * D, S2 + i * D * D,
                      Z0 + i, Z1 + i * D, Z2 + i * D, y + i * D);
        }
    return ORC_OK;
}

/*
 * Prefill of L tokens for B*H head-states, starting from the state passed in
 * (zero it for "no incoming state") and leaving the final state there.
 *   q,k,v,y : [B,H,L,D] contiguous
 *   lam     : lam[b*lam_stride_b + h]
 */
int orc_prefill(int B, int H, int L, int D,
                const double *q, const double *k, const double *v,
                const double *lam, long lam_stride_b, double eps,
                double *S0, double *S1, double *S2,
                double *Z0, double *Z1, double *Z2, double *y)
{
    if (B < 0 || H <= 0 || L < 0 || D <= 0 || !lam) return ORC_EINVAL;
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            const size_t i = (size_t)b * H + h;
            const double l = lam[(size_t)b * lam_stride_b + h];
            for (int t = 0; t < L; ++t) {
                const size_t o = (i * (size_t)L + t) * D;
                step_head(D, l, eps, q + o, k + o, v + o,
                          S0 + i * D, S1 + i * D * D, S2 + i * D * D,
                          Z0 + i, Z1 + i * D, Z2 + i * D, y + o);
            }
        }
    return ORC_OK;
}

/*
 * Segment combine used by sequence-sharded prefill: given the state entering a
 * segment (P) and the state the segment builds from zero (T) over len tokens,
 * the state leaving it is lam^len * P + T.  Applied in place to P for one
 * head-state of F floats.  This is the associative carry the reference's
 * inter-chunk scan evaluates as a dense matmul (chunked_ssd.py:113-126).
 */
void orc_combine(int F, double lam, long len, double *P, const double *T)
{
    const double a = pow(lam, (double)len);
    for (int i = 0; i < F; ++i) P[i] = a * P[i] + T[i];
}
