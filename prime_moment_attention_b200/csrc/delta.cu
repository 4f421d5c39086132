// delta.cu -- the gated delta-rule variant: chunked prefill and decode step (float32).
//
// Replaces ChunkedGatedDeltaPrimeAttention's core (src/prime_moment_attention/
// chunked_delta_prime.py:142-283).  Per head the state is S [D][2D] (row = value index d,
// column = feature f) and per token the features (:73-87)
//     psi = [q, q^2 / sqrt 2],   phi = [k / max(|k|, e), (k^2 / max(|k^2|, e)) / sqrt 2]
// with a write gate beta_t and a retention alpha_t.
//
// Prefill, one CTA per head-state, chunks of C tokens from the start of the call, the state
// resident in shared memory (feature-major St[f][d]).  Per chunk, with cum_i = sum_{t<=i}
// log clamp(alpha_t, 1e-5, 1) and Lambda_ij = exp(cum_i - cum_j):
//   T  = I + strict_tril(Lambda . (Phi Phi^T) . beta_j)                       (:197-218)
//   u_i = v_i - exp(cum_i) S phi_i,  solve T E = u                            (:230-245)
//   y_i = sum_{j<=i} Lambda_ij (psi_i . phi_j) beta_j E_j + exp(cum_i) S psi_i (:247-255)
//   S  = exp(cum_end) S + sum_j beta_j exp(cum_end - cum_j) E_j phi_j^T       (:258-264)
//   S *= min(1, bound / (|S|_F + 1e-6))                                       (:267-270)
// A ragged last chunk is padded as the reference pads it (zero features and beta, alpha = the
// head's decay), so the final state carries the reference's decay^pad factor.  The unit lower
// triangular solve inverts the C/16 diagonal 16 x 16 blocks (one thread per column) and then
// walks the blocks: R = u_b - sum_{j < 16b} T[:, j] E_j, E_b = inv(T_bb) R.
// All products run on CUDA cores in float32 (the 1e-4 bar for float32 inputs).
//
// Decode step (:142-172), one CTA per head-state, one HBM read and one write of S:
//   e = v - S phi (the undecayed state),  S = alpha S + beta e phi^T,
//   S *= min(1, bound / (|S|_F + 1e-6)),  y = S psi.
// The state lives in registers (8 float4 per thread at D = 64) between the read and the write;
// row sums are warp-shuffle reductions over the lanes that share a row.
#include "pma_common.cuh"
#include "prefill.cuh"

namespace pma {

namespace {

constexpr int DT = 256;  // threads of the delta kernels

template <int D, int C>
struct DeltaSmem {
    static constexpr int F = 2 * D;
    static constexpr int oSt = 0;                 // St [F][D]     state, feature-major
    static constexpr int oPHIt = oSt + F * D;     // PHIt [F][C]   phi, feature-major
    static constexpr int oPSIt = oPHIt + F * C;   // PSIt [F][C]   psi, feature-major
    static constexpr int oVE = oPSIt + F * C;     // VE [C][D]     v -> u -> R -> E
    static constexpr int oTt = oVE + C * D;       // Tt [C][C]     Tt[j][i] = T[i][j]
    static constexpr int oPt = oTt + C * C;       // Pt [C][C]     Pt[j][i] = Lambda_ij (psi_i.phi_j) beta_j
    static constexpr int oTI = oPt + C * C;       // TI [C/16][16][16]  inverses of T's diagonal blocks
    static constexpr int oCum = oTI + C * 16;     // [C] cum_i
    static constexpr int oBeta = oCum + C;        // [C] beta_i
    static constexpr int oDin = oBeta + C;        // [C] exp(cum_i)
    static constexpr int oCoef = oDin + C;        // [C] beta_j exp(cum_end - cum_j)
    static constexpr int oRed = oCoef + C;        // [32] reductions; [8] = chunk decay, [9] = scale
    static constexpr int floats = oRed + 32;
    static constexpr size_t bytes = (size_t)floats * sizeof(float);
};

template <int D, int C, typename TI, typename TO>
__global__ void __launch_bounds__(DT, 1) delta_prefill_kernel(const DeltaParams p) {
    using SM = DeltaSmem<D, C>;
    constexpr int F = 2 * D;
    constexpr int NB = C / 16;
    extern __shared__ float4 dsm4[];
    float *const sm = reinterpret_cast<float *>(dsm4);
    float *const St = sm + SM::oSt;
    float *const PHIt = sm + SM::oPHIt;
    float *const PSIt = sm + SM::oPSIt;
    float *const VE = sm + SM::oVE;
    float *const Tt = sm + SM::oTt;
    float *const Pt = sm + SM::oPt;
    float *const TIv = sm + SM::oTI;
    float *const cum = sm + SM::oCum;
    float *const bet = sm + SM::oBeta;
    float *const din = sm + SM::oDin;
    float *const coef = sm + SM::oCoef;
    float *const red = sm + SM::oRed;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh - b * p.H;
    const float lam = p.lambda[(int64_t)b * p.lam_sb + h];
    const float lam_c = fminf(fmaxf(lam, 1e-5f), 1.0f);
    const bool want_y = p.y.p != nullptr;
    const TI *qb = reinterpret_cast<const TI *>(p.q.p) + b * p.q.sb + h * p.q.sh;
    const TI *kb = reinterpret_cast<const TI *>(p.k.p) + b * p.k.sb + h * p.k.sh;
    const TI *vb = reinterpret_cast<const TI *>(p.v.p) + b * p.v.sb + h * p.v.sh;
    const float *beta_g = p.beta + (size_t)bh * p.L;
    const float *alpha_g = p.alpha ? p.alpha + (size_t)bh * p.L : nullptr;
    TO *yb = want_y ? reinterpret_cast<TO *>(p.y.p) + b * p.y.sb + h * p.y.sh : nullptr;
    const float r2 = 0.70710678118654752f;

    // ---- state in (global S[d][f] -> St[f][d]); upper triangles of Tt / Pt stay zero ----
    const float *sin = p.state_in ? p.state_in + (size_t)bh * D * F : nullptr;
    for (int e = tid; e < D * (F / 4); e += DT) {
        const int d = e % D, f0 = (e / D) * 4;
        const float4 s = sin ? *reinterpret_cast<const float4 *>(sin + (size_t)d * F + f0) : make_float4(0, 0, 0, 0);
        St[(f0 + 0) * D + d] = s.x;
        St[(f0 + 1) * D + d] = s.y;
        St[(f0 + 2) * D + d] = s.z;
        St[(f0 + 3) * D + d] = s.w;
    }
    for (int e = tid; e < 2 * C * C; e += DT) Tt[e] = 0.f;  // Tt and Pt are adjacent
    __syncthreads();

    for (int t0 = 0; t0 < p.L; t0 += C) {
        const int n = min(C, p.L - t0);
        // ---- A. features (one thread per k row and per q row), v rows, gates ----
        if (tid < 2 * C) {
            const int i = tid % C;
            const bool is_q = tid >= C;
            if (!is_q || want_y) {
                float x[D];
                const TI *row = (is_q ? qb + (int64_t)(t0 + i) * p.q.sl : kb + (int64_t)(t0 + i) * p.k.sl);
                if (i < n) {
#pragma unroll
                    for (int d = 0; d < D; d += 4) {
                        const float4 v4 = load4(row + d);
                        x[d] = v4.x; x[d + 1] = v4.y; x[d + 2] = v4.z; x[d + 3] = v4.w;
                    }
                } else {
#pragma unroll
                    for (int d = 0; d < D; ++d) x[d] = 0.f;
                }
                float *dst = is_q ? PSIt : PHIt;
                float s1 = 1.f, s2 = r2;
                if (!is_q) {
                    float n1 = 0.f, n2 = 0.f;
#pragma unroll
                    for (int d = 0; d < D; ++d) {
                        const float k2 = x[d] * x[d];
                        n1 = fmaf(x[d], x[d], n1);
                        n2 = fmaf(k2, k2, n2);
                    }
                    s1 = 1.0f / fmaxf(sqrtf(n1), p.norm_eps);
                    s2 = r2 / fmaxf(sqrtf(n2), p.norm_eps);
                }
#pragma unroll
                for (int d = 0; d < D; ++d) {
                    dst[d * C + i] = x[d] * s1;
                    dst[(D + d) * C + i] = x[d] * x[d] * s2;
                }
            }
        } else {
            for (int e = tid - 2 * C; e < C * (D / 4); e += DT - 2 * C) {
                const int i = e / (D / 4), d0 = (e % (D / 4)) * 4;
                const float4 v4 = i < n ? load4(vb + (int64_t)(t0 + i) * p.v.sl + d0) : make_float4(0, 0, 0, 0);
                *reinterpret_cast<float4 *>(VE + i * D + d0) = v4;
            }
        }
        if (warp == 7) {  // gates and the inclusive scan of log alpha over the chunk (C/32 per lane)
            constexpr int PL = C / 32;
            float la[PL], run = 0.f;
#pragma unroll
            for (int m = 0; m < PL; ++m) {
                const int i = lane * PL + m;
                float a = lam_c;
                if (i < n) a = fminf(fmaxf(alpha_g ? alpha_g[t0 + i] : lam, 1e-5f), 1.0f);
                run += __logf(a);
                la[m] = run;
                bet[i] = i < n ? beta_g[t0 + i] : 0.f;
            }
            float incl = run;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            const float base = incl - run;
#pragma unroll
            for (int m = 0; m < PL; ++m) cum[lane * PL + m] = base + la[m];
        }
        __syncthreads();
        if (tid < C) {
            const float ce = cum[C - 1];
            din[tid] = __expf(cum[tid]);
            coef[tid] = bet[tid] * __expf(ce - cum[tid]);
            if (tid == 0) red[8] = __expf(ce);
        }
        // ---- B1. G = Phi Phi^T and P = Psi Phi^T on the lower triangle: tiles 4 rows x 2 columns ----
        constexpr int NLT = (C / 4) * (C / 4 + 1);  // sum over row tiles a of (2a + 2)
        for (int tt = tid; tt < NLT; tt += DT) {
            int a = (int)((sqrtf(4.f * tt + 1.f) - 1.f) * 0.5f);
            while (a * (a + 1) > tt) --a;
            while ((a + 1) * (a + 2) <= tt) ++a;
            const int i0 = 4 * a, j0 = 2 * (tt - a * (a + 1));
            float g[4][2], pp[4][2];
#pragma unroll
            for (int u = 0; u < 4; ++u) g[u][0] = g[u][1] = pp[u][0] = pp[u][1] = 0.f;
#pragma unroll 4
            for (int f = 0; f < F; ++f) {
                const float4 pi = *reinterpret_cast<const float4 *>(PHIt + f * C + i0);
                const float4 si = *reinterpret_cast<const float4 *>(PSIt + f * C + i0);
                const float2 pj = *reinterpret_cast<const float2 *>(PHIt + f * C + j0);
                const float ia[4] = {pi.x, pi.y, pi.z, pi.w}, sa[4] = {si.x, si.y, si.z, si.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    g[u][0] = fmaf(ia[u], pj.x, g[u][0]);
                    g[u][1] = fmaf(ia[u], pj.y, g[u][1]);
                    pp[u][0] = fmaf(sa[u], pj.x, pp[u][0]);
                    pp[u][1] = fmaf(sa[u], pj.y, pp[u][1]);
                }
            }
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                const int j = j0 + w;
                float to[4], po[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = i0 + u;
                    const float lm = j <= i ? __expf(cum[i] - cum[j]) : 0.f;
                    to[u] = j < i ? lm * g[u][w] * bet[j] : (j == i ? 1.f : 0.f);
                    po[u] = lm * pp[u][w] * bet[j];
                }
                *reinterpret_cast<float4 *>(Tt + j * C + i0) = make_float4(to[0], to[1], to[2], to[3]);
                *reinterpret_cast<float4 *>(Pt + j * C + i0) = make_float4(po[0], po[1], po[2], po[3]);
            }
        }
        // ---- B2. u = v - exp(cum) Phi S^T and y_inter = exp(cum) Psi S^T: tiles 4 rows x 4 dims ----
        // (din is written above by other threads: read it after the next barrier, keep raw sums)
        constexpr int NT2 = (C / 4) * (D / 4);  // <= DT: one tile per thread, kept in registers
        const bool t2 = tid < NT2;
        const int i2 = (tid % (C / 4)) * 4, d2 = (tid / (C / 4)) * 4;
        float au[4][4], ay[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int w = 0; w < 4; ++w) au[u][w] = ay[u][w] = 0.f;
        if (t2) {
#pragma unroll 4
            for (int f = 0; f < F; ++f) {
                const float4 pi = *reinterpret_cast<const float4 *>(PHIt + f * C + i2);
                const float4 si = *reinterpret_cast<const float4 *>(PSIt + f * C + i2);
                const float4 s4 = *reinterpret_cast<const float4 *>(St + f * D + d2);
                const float ia[4] = {pi.x, pi.y, pi.z, pi.w}, sa[4] = {si.x, si.y, si.z, si.w};
                const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        au[u][w] = fmaf(ia[u], ss[w], au[u][w]);
                        ay[u][w] = fmaf(sa[u], ss[w], ay[u][w]);
                    }
            }
        }
        __syncthreads();
        if (t2) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float di = din[i2 + u];
                float4 *ve = reinterpret_cast<float4 *>(VE + (i2 + u) * D + d2);
                float4 vv = *ve;
                vv.x -= di * au[u][0]; vv.y -= di * au[u][1]; vv.z -= di * au[u][2]; vv.w -= di * au[u][3];
                *ve = vv;
#pragma unroll
                for (int w = 0; w < 4; ++w) ay[u][w] *= di;
            }
        }
        // ---- C. inverses of the diagonal 16 x 16 blocks of T (one thread per block column) ----
        if (tid < NB * 16) {
            const int bi = tid >> 4, c = tid & 15, r0 = bi * 16;
            float x[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float s = (i == c) ? 1.f : 0.f;
                if (i > c) {
#pragma unroll
                    for (int k = 0; k < 16; ++k)
                        if (k >= c && k < i) s = fmaf(-Tt[(r0 + k) * C + r0 + i], x[k], s);
                }
                x[i] = s;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) TIv[(bi * 16 + i) * 16 + c] = x[i];
        }
        __syncthreads();
        // ---- D. block forward substitution: E overwrites u in VE ----
        {
            constexpr int TPR = D / 4;  // threads per row
            const bool act = tid < 16 * TPR;
            const int rl = tid / TPR, dd = (tid % TPR) * 4;
#pragma unroll 1
            for (int bi = 0; bi < NB; ++bi) {
                const int r = bi * 16 + rl;
                if (act && bi > 0) {
                    float4 acc = *reinterpret_cast<const float4 *>(VE + r * D + dd);
                    for (int jb = 0; jb < bi; ++jb) {  // 16 rows per pass, unrolled: the loads pipeline
                        float4 a2 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 2) {
                            const int j = jb * 16 + jj;
                            const float t0v = Tt[j * C + r], t1v = Tt[(j + 1) * C + r];
                            const float4 e0 = *reinterpret_cast<const float4 *>(VE + j * D + dd);
                            const float4 e1 = *reinterpret_cast<const float4 *>(VE + (j + 1) * D + dd);
                            acc.x = fmaf(-t0v, e0.x, acc.x); acc.y = fmaf(-t0v, e0.y, acc.y);
                            acc.z = fmaf(-t0v, e0.z, acc.z); acc.w = fmaf(-t0v, e0.w, acc.w);
                            a2.x = fmaf(-t1v, e1.x, a2.x); a2.y = fmaf(-t1v, e1.y, a2.y);
                            a2.z = fmaf(-t1v, e1.z, a2.z); a2.w = fmaf(-t1v, e1.w, a2.w);
                        }
                        acc.x += a2.x; acc.y += a2.y; acc.z += a2.z; acc.w += a2.w;
                    }
                    *reinterpret_cast<float4 *>(VE + r * D + dd) = acc;
                }
                __syncthreads();
                float4 e4 = make_float4(0, 0, 0, 0);
                if (act) {
                    const float *xr = TIv + (bi * 16 + rl) * 16;
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const float xk = xr[k];
                        const float4 rk = *reinterpret_cast<const float4 *>(VE + (bi * 16 + k) * D + dd);
                        e4.x = fmaf(xk, rk.x, e4.x); e4.y = fmaf(xk, rk.y, e4.y);
                        e4.z = fmaf(xk, rk.z, e4.z); e4.w = fmaf(xk, rk.w, e4.w);
                    }
                }
                __syncthreads();
                if (act) *reinterpret_cast<float4 *>(VE + r * D + dd) = e4;
                __syncthreads();  // the next block's R step reads these E rows
            }
        }
        // ---- E1. y = y_inter + P (beta E) on this thread's B2 tile ----
        if (t2 && want_y) {
            const int jmax = min(i2 + 4, C);
            for (int j = 0; j < jmax; ++j) {
                const float4 pj = *reinterpret_cast<const float4 *>(Pt + j * C + i2);
                const float4 ej = *reinterpret_cast<const float4 *>(VE + j * D + d2);
                const float pa[4] = {pj.x, pj.y, pj.z, pj.w}, ea[4] = {ej.x, ej.y, ej.z, ej.w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int w = 0; w < 4; ++w) ay[u][w] = fmaf(pa[u], ea[w], ay[u][w]);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i2 + u < n)
                    store4(yb + (int64_t)(t0 + i2 + u) * p.y.sl + d2, make_float4(ay[u][0], ay[u][1], ay[u][2], ay[u][3]));
        }
        // ---- E2. S = exp(cum_end) S + sum_j coef_j E_j phi_j^T: tiles 4 features x 4 dims ----
        {
            const float cd = red[8];
            for (int tt = tid; tt < (F / 4) * (D / 4); tt += DT) {
                const int d0 = (tt % (D / 4)) * 4, f0 = (tt / (D / 4)) * 4;
                float acc[4][4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int w = 0; w < 4; ++w) acc[u][w] = 0.f;
#pragma unroll 4
                for (int j = 0; j < C; ++j) {
                    const float cj = coef[j];
                    const float4 ej = *reinterpret_cast<const float4 *>(VE + j * D + d0);
                    const float ea[4] = {cj * ej.x, cj * ej.y, cj * ej.z, cj * ej.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float ph = PHIt[(f0 + u) * C + j];
#pragma unroll
                        for (int w = 0; w < 4; ++w) acc[u][w] = fmaf(ph, ea[w], acc[u][w]);
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float4 *sp = reinterpret_cast<float4 *>(St + (f0 + u) * D + d0);
                    const float4 o = *sp;
                    *sp = make_float4(fmaf(cd, o.x, acc[u][0]), fmaf(cd, o.y, acc[u][1]), fmaf(cd, o.z, acc[u][2]),
                                      fmaf(cd, o.w, acc[u][3]));
                }
            }
        }
        __syncthreads();
        // ---- F. Lyapunov projection at the end of the chunk ----
        if (p.bound > 0.f) {
            float s = 0.f;
            for (int e = tid; e < F * D; e += DT) s = fmaf(St[e], St[e], s);
            s = warp_sum(s);
            if (lane == 0) red[warp] = s;
            __syncthreads();
            if (tid == 0) {
                float tot = 0.f;
#pragma unroll
                for (int w = 0; w < DT / 32; ++w) tot += red[w];
                red[9] = fminf(p.bound / (sqrtf(tot) + 1e-6f), 1.0f);
            }
            __syncthreads();
            const float sc = red[9];
            if (sc < 1.0f)
                for (int e = tid; e < F * D; e += DT) St[e] *= sc;
            __syncthreads();
        }
    }

    // ---- state out (St[f][d] -> S[d][f]) ----
    if (p.state_out) {
        float *so = p.state_out + (size_t)bh * D * F;
        for (int e = tid; e < D * (F / 4); e += DT) {
            const int d = e % D, f0 = (e / D) * 4;
            *reinterpret_cast<float4 *>(so + (size_t)d * F + f0) =
                make_float4(St[(f0 + 0) * D + d], St[(f0 + 1) * D + d], St[(f0 + 2) * D + d], St[(f0 + 3) * D + d]);
        }
    }
}

// ------------------------------------------------------------------ decode step
template <int D, typename TI, typename TO>
__global__ void __launch_bounds__(DT) delta_step_kernel(const DeltaStepParams p) {
    constexpr int F = 2 * D;
    constexpr int NT = (D * F / 4) < DT ? (D * F / 4) : DT;  // threads that hold state
    constexpr int PER = (D * F / 4) / NT;                    // float4 per thread
    constexpr int LPR = F / 4;                               // lanes per row (<= 32)
    static_assert(NT % 32 == 0 && 32 % LPR == 0, "rows must tile whole warps");
    __shared__ float sphi[F], spsi[F], sv[D], red[DT / 32 + 2];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x;
    const int n = bh / p.H, h = bh - n * p.H;
    const TI *qp = reinterpret_cast<const TI *>(p.q.p) + n * p.q.sb + h * p.q.sh;
    const TI *kp = reinterpret_cast<const TI *>(p.k.p) + n * p.k.sb + h * p.k.sh;
    const TI *vp = reinterpret_cast<const TI *>(p.v.p) + n * p.v.sb + h * p.v.sh;
    const float *sin = p.state_in + (size_t)bh * D * F;
    float *sout = p.state_out + (size_t)bh * D * F;

    // issue the state loads first
    float4 s[PER];
    if (tid < NT) {
#pragma unroll
        for (int j = 0; j < PER; ++j) s[j] = ldcs4(sin + (size_t)(tid + NT * j) * 4);
    }
    if (warp == 0) {
        const float r2 = 0.70710678118654752f;
        float n1 = 0.f, n2 = 0.f;
        for (int d = lane; d < D; d += 32) {
            const float k = Elem<TI>::to_f(kp[d]);
            n1 = fmaf(k, k, n1);
            n2 = fmaf(k * k, k * k, n2);
        }
        n1 = warp_sum(n1);
        n2 = warp_sum(n2);
        const float s1 = 1.0f / fmaxf(sqrtf(n1), p.norm_eps), s2 = r2 / fmaxf(sqrtf(n2), p.norm_eps);
        for (int d = lane; d < D; d += 32) {
            const float k = Elem<TI>::to_f(kp[d]), q = Elem<TI>::to_f(qp[d]);
            sphi[d] = k * s1;
            sphi[D + d] = k * k * s2;
            spsi[d] = q;
            spsi[D + d] = q * q * r2;
            sv[d] = Elem<TI>::to_f(vp[d]);
        }
    }
    __syncthreads();
    const float beta = p.beta[bh], alpha = p.alpha[bh];
    // element e = tid + NT * j covers S row e / LPR, features 4 * (e % LPR) .. +3; NT is a
    // multiple of 32, so the threads past NT are whole warps and skip the row work
    const int c4 = (tid % LPR) * 4;
    const float4 ph = *reinterpret_cast<const float4 *>(sphi + c4);
    const float4 ps = *reinterpret_cast<const float4 *>(spsi + c4);
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        if (tid >= NT) break;
        float part = s[j].x * ph.x + s[j].y * ph.y + s[j].z * ph.z + s[j].w * ph.w;
#pragma unroll
        for (int o = 1; o < LPR; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const int d = (tid + NT * j) / LPR;
        const float ce = beta * (sv[d] - part);  // beta * e_d, e against the undecayed state
        s[j] = make_float4(fmaf(alpha, s[j].x, ce * ph.x), fmaf(alpha, s[j].y, ce * ph.y),
                           fmaf(alpha, s[j].z, ce * ph.z), fmaf(alpha, s[j].w, ce * ph.w));
        sq += s[j].x * s[j].x + s[j].y * s[j].y + s[j].z * s[j].z + s[j].w * s[j].w;
    }
    float sc = 1.f;
    if (p.bound > 0.f) {
        sq = warp_sum(sq);
        if (lane == 0) red[warp] = sq;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.f;
            for (int w = 0; w < DT / 32; ++w) tot += red[w];
            red[DT / 32] = fminf(p.bound / (sqrtf(tot) + 1e-6f), 1.0f);
        }
        __syncthreads();
        sc = red[DT / 32];
    }
    if (tid < NT) {
        TO *yp = reinterpret_cast<TO *>(p.y.p) + n * p.y.sb + h * p.y.sh;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const float4 o = make_float4(s[j].x * sc, s[j].y * sc, s[j].z * sc, s[j].w * sc);
            stcs4(sout + (size_t)(tid + NT * j) * 4, o);
            float part = o.x * ps.x + o.y * ps.y + o.z * ps.z + o.w * ps.w;
#pragma unroll
            for (int o2 = 1; o2 < LPR; o2 <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o2);
            if ((tid % LPR) == 0) yp[(tid + NT * j) / LPR] = Elem<TO>::from_f(part);
        }
    }
}

template <int D, int C, typename TI, typename TO>
cudaError_t launch_dp(const DeltaParams &p, cudaStream_t st) {
    const size_t smem = DeltaSmem<D, C>::bytes;
    cudaError_t e = set_smem_once<delta_prefill_kernel<D, C, TI, TO>>((int)smem);
    if (e != cudaSuccess) return e;
    delta_prefill_kernel<D, C, TI, TO><<<p.B * p.H, DT, smem, st>>>(p);
    return cudaGetLastError();
}

template <int D, int C>
cudaError_t launch_dp_t(const DeltaParams &p, int idt, int ydt, cudaStream_t st) {
    if (idt == PMA_F32)
        return ydt == PMA_F32 ? launch_dp<D, C, float, float>(p, st) : launch_dp<D, C, float, __nv_bfloat16>(p, st);
    return ydt == PMA_F32 ? launch_dp<D, C, __nv_bfloat16, float>(p, st)
                          : launch_dp<D, C, __nv_bfloat16, __nv_bfloat16>(p, st);
}

template <int D>
cudaError_t launch_ds_t(const DeltaStepParams &p, int idt, int ydt, cudaStream_t st) {
    const int grid = p.N * p.H;
    if (idt == PMA_F32) {
        if (ydt == PMA_F32) delta_step_kernel<D, float, float><<<grid, DT, 0, st>>>(p);
        else delta_step_kernel<D, float, __nv_bfloat16><<<grid, DT, 0, st>>>(p);
    } else {
        if (ydt == PMA_F32) delta_step_kernel<D, __nv_bfloat16, float><<<grid, DT, 0, st>>>(p);
        else delta_step_kernel<D, __nv_bfloat16, __nv_bfloat16><<<grid, DT, 0, st>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace

bool delta_supported(int D, int chunk) { return (D == 16 || D == 32 || D == 64) && (chunk == 32 || chunk == 64); }

cudaError_t launch_delta_prefill(const DeltaParams &p, int D, int chunk, int idt, int ydt, cudaStream_t st) {
    if (chunk == 64) {
        switch (D) {
            case 16: return launch_dp_t<16, 64>(p, idt, ydt, st);
            case 32: return launch_dp_t<32, 64>(p, idt, ydt, st);
            case 64: return launch_dp_t<64, 64>(p, idt, ydt, st);
        }
    } else if (chunk == 32) {
        switch (D) {
            case 16: return launch_dp_t<16, 32>(p, idt, ydt, st);
            case 32: return launch_dp_t<32, 32>(p, idt, ydt, st);
            case 64: return launch_dp_t<64, 32>(p, idt, ydt, st);
        }
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_delta_step(const DeltaStepParams &p, int D, int idt, int ydt, cudaStream_t st) {
    switch (D) {
        case 16: return launch_ds_t<16>(p, idt, ydt, st);
        case 32: return launch_ds_t<32>(p, idt, ydt, st);
        case 64: return launch_ds_t<64>(p, idt, ydt, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace pma
