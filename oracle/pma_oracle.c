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
 *   orc_delta_prefill / orc_delta_step   the gated delta-rule variant, and
 *   orc_selective_prefill                the selective variant (see the sections at
 *                     the end of this file).
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

/* ---------------------------------------------------------------------------
 * Gated delta-rule variant: ChunkedGatedDeltaPrimeAttention
 * (src/prime_moment_attention/chunked_delta_prime.py).  One head has a state
 * S [D][2D] (row = value index d, column = feature index f) and per token the
 * features (:73-87)
 *     psi = [q, q^2 / sqrt 2]
 *     phi = [k / max(|k|, e), (k^2 / max(|k^2|, e)) / sqrt 2]
 * with gates beta_t (write) and alpha_t (retention), given per token.
 *
 * orc_delta_prefill: the chunked prefill (:175-283).  Its per-chunk solve
 *     T E = u,  T = I + strict_tril(Lambda * (Phi Phi^T) * beta_j),
 *     u_i = v_i - exp(cum_i) S phi_i,  cum_i = sum_{t<=i} log alpha_t
 * is, row by row, the token recurrence
 *     e_i = v_i - alpha_i S phi_i            (error against the decayed state)
 *     S   = alpha_i S + beta_i e_i phi_i^T
 *     y_i = S psi_i
 * (E_i = e_i; the readout y_intra + y_inter of :248-255 is S_i psi_i), which
 * is what this function iterates.  alpha is used as clamp(alpha, 1e-5, 1)
 * (the log of :197).  At the end of every chunk of `chunk` tokens counted from
 * the start of the call the Lyapunov projection (:267-270)
 *     S *= min(1, bound / (|S|_F + 1e-6))          (bound <= 0: off)
 * is applied.  A ragged last chunk is padded (:178-185) with zero features,
 * zero beta and alpha = the module's decay, so the final state is further
 * multiplied by decay^pad before that chunk's projection; `lam` is that decay
 * (one per head here: the reference module holds one scalar).
 *
 * orc_delta_step: the L == 1 branch (:142-172), which differs from the prefill:
 *     e = v - S phi   (error against the undecayed state)
 *     S = alpha S + beta e phi^T;  Lyapunov projection every step;  y = S psi.
 *
 * Layouts: q,k,v,y [B,H,L,D]; beta, alpha [B,H,L]; lam [H]; state [B,H,D,2D].
 * state_in may be NULL (zero); state_out receives the final state.
 * ------------------------------------------------------------------------- */
static void delta_features(int D, const double *q, const double *k, double ne, double *psi, double *phi)
{
    const double r2 = 1.0 / sqrt(2.0);
    double n1 = 0.0, n2 = 0.0;
    for (int d = 0; d < D; ++d) {
        n1 += k[d] * k[d];
        n2 += k[d] * k[d] * k[d] * k[d];
    }
    n1 = sqrt(n1);
    n2 = sqrt(n2);
    if (n1 < ne) n1 = ne;
    if (n2 < ne) n2 = ne;
    for (int d = 0; d < D; ++d) {
        phi[d] = k[d] / n1;
        phi[D + d] = k[d] * k[d] / n2 * r2;
        psi[d] = q[d];
        psi[D + d] = q[d] * q[d] * r2;
    }
}

static void delta_lyapunov(int n, double bound, double *S)
{
    if (!(bound > 0.0)) return;
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += S[i] * S[i];
    double sc = bound / (sqrt(s) + 1e-6);
    if (sc > 1.0) sc = 1.0;
    for (int i = 0; i < n; ++i) S[i] *= sc;
}

/* one token: err_decayed = 1 for the prefill's error, 0 for the step's */
static void delta_token(int D, const double *q, const double *k, const double *v, double beta, double alpha,
                        double ne, int err_decayed, double *S, double *psi, double *phi)
{
    const int F = 2 * D;
    delta_features(D, q, k, ne, psi, phi);
    for (int d = 0; d < D; ++d) {
        double *row = S + (size_t)d * F;
        double sp = 0.0;
        for (int f = 0; f < F; ++f) sp += row[f] * phi[f];
        const double e = v[d] - (err_decayed ? alpha : 1.0) * sp;
        for (int f = 0; f < F; ++f) row[f] = alpha * row[f] + beta * e * phi[f];
    }
}

static void delta_readout(int D, const double *S, const double *psi, double *y)
{
    const int F = 2 * D;
    for (int d = 0; d < D; ++d) {
        double acc = 0.0;
        for (int f = 0; f < F; ++f) acc += S[(size_t)d * F + f] * psi[f];
        y[d] = acc;
    }
}

int orc_delta_prefill(int B, int H, int L, int D, const double *q, const double *k, const double *v,
                      const double *beta, const double *alpha, const double *lam, int chunk, double bound,
                      double norm_eps, const double *state_in, double *state_out, double *y)
{
    if (B < 0 || H <= 0 || L < 0 || D <= 0 || D > 256 || chunk <= 0 || !lam || !state_out) return ORC_EINVAL;
    const int F = 2 * D;
    const size_t SZ = (size_t)D * F;
    double psi[512], phi[512];
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            const size_t i = (size_t)b * H + h;
            double *S = state_out + i * SZ;
            if (state_in) memcpy(S, state_in + i * SZ, SZ * sizeof(double));
            else memset(S, 0, SZ * sizeof(double));
            for (int t = 0; t < L; ++t) {
                const size_t o = (i * (size_t)L + t) * D, g = i * (size_t)L + t;
                double a = alpha ? alpha[g] : lam[h];
                if (a < 1e-5) a = 1e-5;
                if (a > 1.0) a = 1.0;
                delta_token(D, q + o, k + o, v + o, beta[g], a, norm_eps, 1, S, psi, phi);
                if (y) delta_readout(D, S, psi, y + o);
                if ((t + 1) % chunk == 0) delta_lyapunov((int)SZ, bound, S);
            }
            if (L % chunk) {
                double lp = lam[h];
                if (lp < 1e-5) lp = 1e-5;
                if (lp > 1.0) lp = 1.0;
                const double f = pow(lp, (double)(chunk - L % chunk));
                for (size_t j = 0; j < SZ; ++j) S[j] *= f;
                delta_lyapunov((int)SZ, bound, S);
            }
        }
    return ORC_OK;
}

int orc_delta_step(int N, int H, int D, const double *q, const double *k, const double *v, const double *beta,
                   const double *alpha, double bound, double norm_eps, const double *state_in, double *state_out,
                   double *y)
{
    if (N < 0 || H <= 0 || D <= 0 || D > 256 || !state_in || !state_out || !alpha || !beta) return ORC_EINVAL;
    const int F = 2 * D;
    const size_t SZ = (size_t)D * F;
    double psi[512], phi[512];
    for (size_t i = 0; i < (size_t)N * H; ++i) {
        double *S = state_out + i * SZ;
        if (S != state_in + i * SZ) memcpy(S, state_in + i * SZ, SZ * sizeof(double));
        delta_token(D, q + i * D, k + i * D, v + i * D, beta[i], alpha[i], norm_eps, 0, S, psi, phi);
        delta_lyapunov((int)SZ, bound, S);
        if (y) delta_readout(D, S, psi, y + i * D);
    }
    return ORC_OK;
}

/* ---------------------------------------------------------------------------
 * Selective variant: PrimeSelectiveMomentAttention
 * (src/prime_moment_attention/selective.py:264-444).  Per token a decay
 * lambda_t = exp(-Delta_t / tau_h), given here as log_decay[t] = -Delta_t / tau_h, and a
 * per-head temperature beta_h.  The step branch (:367-396), iterated:
 *     S0 = l S0 + v             Z0 = l Z0 + 1
 *     S1 = l S1 + b k v^T       Z1 = l Z1 + b k
 *     S2 = l S2 + b^2/2 k^2 v^T Z2 = l Z2 + b^2/2 k^2
 *     y  = (S0 + q.S1 + q^2.S2) / max(Z0 + q.Z1 + q^2.Z2, eps)
 * (no 1/2 at the readout: the reference folds it into S2 / Z2, which therefore hold half of
 * the moment-attention layout's second moments).  Its parallel branch (:401-435) is the same
 * recurrence from a zero state.
 *   q,k,v,y [B,H,L,D]; log_decay [B,H,L]; beta [H]; state arrays as orc_prefill.
 * ------------------------------------------------------------------------- */
int orc_selective_prefill(int B, int H, int L, int D, const double *q, const double *k, const double *v,
                          const double *log_decay, const double *beta, double eps,
                          double *S0, double *S1, double *S2, double *Z0, double *Z1, double *Z2, double *y)
{
    if (B < 0 || H <= 0 || L < 0 || D <= 0 || !log_decay || !beta) return ORC_EINVAL;
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            const size_t i = (size_t)b * H + h;
            const double bt = beta[h], b2 = 0.5 * bt * bt;
            double *s0 = S0 + i * D, *s1 = S1 + i * D * D, *s2 = S2 + i * D * D;
            double *z1 = Z1 + i * D, *z2 = Z2 + i * D;
            for (int t = 0; t < L; ++t) {
                const size_t o = (i * (size_t)L + t) * D;
                const double l = exp(log_decay[i * (size_t)L + t]);
                const double *qt = q + o, *kt = k + o, *vt = v + o;
                for (int e = 0; e < D; ++e) s0[e] = l * s0[e] + vt[e];
                for (int d = 0; d < D; ++d)
                    for (int e = 0; e < D; ++e) {
                        s1[d * D + e] = l * s1[d * D + e] + bt * kt[d] * vt[e];
                        s2[d * D + e] = l * s2[d * D + e] + b2 * kt[d] * kt[d] * vt[e];
                    }
                Z0[i] = l * Z0[i] + 1.0;
                double den = Z0[i];
                for (int d = 0; d < D; ++d) {
                    z1[d] = l * z1[d] + bt * kt[d];
                    z2[d] = l * z2[d] + b2 * kt[d] * kt[d];
                    den += qt[d] * z1[d] + qt[d] * qt[d] * z2[d];
                }
                if (den < eps) den = eps;
                for (int e = 0; e < D; ++e) {
                    double num = s0[e];
                    for (int d = 0; d < D; ++d) num += qt[d] * s1[d * D + e] + qt[d] * qt[d] * s2[d * D + e];
                    y[o + e] = num / den;
                }
            }
        }
    return ORC_OK;
}
