// prefill_simt_body.cuh -- the float32 chunked prefill of one (head-state, segment),
// shared by the CUDA-core kernel and the tensor-core kernel's small-decay path.
//
// Restates chunked_prime_ssd_core (src/prime_moment_attention/chunked_ssd.py:48-184)
// chunk by chunk, carrying the float32 state sequentially in shared memory
// instead of the reference's O(nc^2) inter-chunk matmul (chunked_ssd.py:113-126).
// Per chunk of n <= C tokens, with powers pw[t] = l^t:
//   P[i][j]  = pw[i-j] (1 + q_i.k_j + 0.5 q_i^2.k_j^2)  for j <= i   (chunked_ssd.py:79-92)
//   num_i    = sum_j P[i][j] v_j,  den_i = sum_j P[i][j]               (:93-94)
//   carry_i  = pw[i+1] (S0 + q_i^T S1 + 0.5 (q_i^2)^T S2)               (:139-153)
//   y_i      = (num_i + carry_i) / max(den_i + pw[i+1](Z0 + q_i.Z1 + 0.5 q_i^2.Z2), eps)   (:155-157)
//   S        = pw[n] S + sum_{j<n} pw[n-1-j] phi(k_j) [v_j, 1]^T        (:96-111, 162-169)
// With a per-token decay (PT, the selective variant, selective.py:401-435) the powers become
// exp(cum_i - cum_j), exp(cum_i) and exp(cum_{n-1} - cum_j), cum being the chunk's inclusive
// prefix sum of log lambda_t; k may be scaled per head (its temperature beta_h) and the user
// states may hold S2, Z2 halved (the selective layout: loaded doubled, stored halved).
// A ragged last chunk simply uses n < C, which is what the reference's zero
// padding plus lambda^(-pad) correction (:65-69, 97-99, 171-178) amounts to.
#pragma once

#include "prefill.cuh"

namespace pma {

template <int D, int C>
struct SimtSmem {
    static constexpr int floats = 2 * D * C /*Qt,Kt*/ + 2 * C * D /*Kr,Vr*/ + C * C /*Pt*/ + 2 * D * D /*S1,S2*/ +
                                  3 * D /*S0,Z1,Z2*/ + (C + 4) /*pw*/ + 2 * C /*den,cden*/ + 4 /*Z0*/ +
                                  4 * C /*prologue row stats*/ + 3 * C + 4 /*per-token decay*/;
    static constexpr size_t bytes = floats * sizeof(float);
};

// One (head-state, segment) of the chunked prefill in float32, run by the whole
// CTA (any blockDim.x that is a multiple of 32); `sm` is SimtSmem<D, C>::bytes of
// 16-byte aligned shared memory.  Used by the CUDA-core kernel below and, for
// decays too small for its rescaled operands, by the tensor-core kernel.
template <int D, int C, typename TI, typename TO, bool PT = false>
__device__ __forceinline__ void simt_prefill_body(const PrefillParams &p, float *sm, int bh, int s) {
    float *const Qt = sm;                                // [D][C]  q transposed
    float *const Kt = Qt + D * C;                        // [D][C]  k transposed
    float *const Kr = Kt + D * C;                        // [C][D]  k rows
    float *const Vr = Kr + C * D;                        // [C][D]  v rows
    float *const Pt = Vr + C * D;                        // [C][C]  Pt[j][i] = P[i][j]
    float *const S1 = Pt + C * C;                        // [D][D]
    float *const S2 = S1 + D * D;                        // [D][D]
    float *const S0 = S2 + D * D;                        // [D]
    float *const Z1 = S0 + D;
    float *const Z2 = Z1 + D;
    float *const pw = Z2 + D;                            // [C+1]
    float *const den = pw + (C + 4);                     // [C]
    float *const cden = den + C;                         // [C]
    float *const Z0 = cden + C;                          // [1]
    float2 *const qst = reinterpret_cast<float2 *>(Z0 + 4);  // [C] LayerNorm (mean, rstd) of q rows
    float2 *const kst = qst + C;                             // [C] and of k rows
    float *const lcum = reinterpret_cast<float *>(kst + C);  // [C] per-token decay: inclusive cum log lambda
    float *const gin = lcum + C;                             // [C] exp(cum_i)
    float *const wend = gin + C;                             // [C] exp(cum_{n-1} - cum_j)
    float *const dsc = wend + C;                             // [0] exp(cum_{n-1}), [1] sum_j wend[j]

    const int tid = threadIdx.x;
    const int b = bh / p.H, h = bh - b * p.H;
    const float lam = PT ? 1.f : p.lambda[(int64_t)b * p.lam_sb + h];
    const int t_begin = s * p.seg_len;
    const int t_end = min(t_begin + p.seg_len, p.L);
    const bool want_y = p.y.p != nullptr && !p.state_only;

    for (int t = tid; t <= C; t += blockDim.x) pw[t] = (float)pow((double)lam, (double)t);
    const bool has_in = !p.state_only && p.in.present();
    HeadPtrs src{};
    if (has_in) src = p.in.at(bh, p.in.packed ? s : 0, D);
    const float sq_in = (p.half_sq && !p.in.packed) ? 2.f : 1.f;  // selective layout: S2, Z2 halved
    for (int i = tid; i < D * D; i += blockDim.x) {
        S1[i] = has_in ? src.S1[i] : 0.f;
        S2[i] = has_in ? sq_in * src.S2[i] : 0.f;
    }
    for (int i = tid; i < D; i += blockDim.x) {
        S0[i] = has_in ? src.S0[i] : 0.f;
        Z1[i] = has_in ? src.Z1[i] : 0.f;
        Z2[i] = has_in ? sq_in * src.Z2[i] : 0.f;
    }
    if (tid == 0) Z0[0] = has_in ? src.Z0[0] : 0.f;

    const TI *qb = reinterpret_cast<const TI *>(p.q.p) + b * p.q.sb + h * p.q.sh;
    const int hk = h / p.pro.groups;  // GQA: kv head of query head h
    const TI *kb = reinterpret_cast<const TI *>(p.k.p) + b * p.k.sb + hk * p.k.sh;
    const TI *vb = reinterpret_cast<const TI *>(p.v.p) + b * p.v.sb + hk * p.v.sh;
    const bool q_pro = want_y && p.pro.q_work(), q_norm = want_y && p.pro.qw, k_norm = p.pro.kw != nullptr;
    const float ksc = p.k_head_scale ? p.k_head_scale[h] : 1.f;
    const float *ldg = PT ? p.logdecay + (size_t)bh * p.L : nullptr;
    TO *yb = want_y ? reinterpret_cast<TO *>(p.y.p) + b * p.y.sb + h * p.y.sh : nullptr;
    __syncthreads();

    for (int t0 = t_begin; t0 < t_end; t0 += C) {
        const int n = min(C, t_end - t0);
        // ---- prologue row statistics (one warp per token row, read from global/L2) ----
        if (q_norm || k_norm) {
            const int warp = tid >> 5, lane = tid & 31;
            for (int j = warp; j < n; j += blockDim.x >> 5) {
                if (q_norm) {
                    const float2 st = warp_row_stats<D>(qb + (int64_t)(t0 + j) * p.q.sl, p.pro.ln_eps, lane);
                    if (lane == 0) qst[j] = st;
                }
                if (k_norm) {
                    const float2 st = warp_row_stats<D>(kb + (int64_t)(t0 + j) * p.k.sl, p.pro.ln_eps, lane);
                    if (lane == 0) kst[j] = st;
                }
            }
            __syncthreads();
        }
        // ---- per-token decay: warp 0 scans log lambda over the chunk (C / 32 per lane) ----
        if (PT && (tid >> 5) == 0) {
            constexpr int PL = C / 32;
            const int lane = tid & 31;
            float la[PL], run = 0.f;
#pragma unroll
            for (int m = 0; m < PL; ++m) {
                const int i = lane * PL + m;
                run += i < n ? ldg[t0 + i] : 0.f;
                la[m] = run;
            }
            float incl = run;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            const float base = incl - run;
#pragma unroll
            for (int m = 0; m < PL; ++m) la[m] += base;
            const float cend = __shfl_sync(0xffffffffu, la[((n - 1) % PL)], (n - 1) / PL);
            float wsum = 0.f;
#pragma unroll
            for (int m = 0; m < PL; ++m) {
                const int i = lane * PL + m;
                lcum[i] = la[m];
                gin[i] = expf(la[m]);
                const float wv = i < n ? expf(cend - la[m]) : 0.f;
                wend[i] = wv;
                wsum += wv;
            }
            wsum = warp_sum(wsum);
            if (lane == 0) {
                dsc[0] = expf(cend);
                dsc[1] = wsum;
            }
        }
        // ---- stage the chunk: transposed q/k (token index fastest across lanes) ----
        if (want_y) {
            for (int e = tid; e < C * (D / 4); e += blockDim.x) {
                const int j = e % C, d0 = (e / C) * 4;
                float4 qv = make_float4(0.f, 0.f, 0.f, 0.f), kv = qv;
                if (j < n) {
                    qv = load4(qb + (int64_t)(t0 + j) * p.q.sl + d0);
                    kv = load4(kb + (int64_t)(t0 + j) * p.k.sl + d0);
                    if (q_pro)
                        qv = prologue4(qv, q_norm ? qst[j] : make_float2(0.f, 1.f), p.pro.qw, p.pro.qb, d0,
                                       p.pro.q_scale);
                    if (k_norm || ksc != 1.f) kv = prologue4(kv, k_norm ? kst[j] : make_float2(0.f, 1.f), p.pro.kw,
                                                             p.pro.kb, d0, ksc);
                }
                Qt[(d0 + 0) * C + j] = qv.x; Qt[(d0 + 1) * C + j] = qv.y;
                Qt[(d0 + 2) * C + j] = qv.z; Qt[(d0 + 3) * C + j] = qv.w;
                Kt[(d0 + 0) * C + j] = kv.x; Kt[(d0 + 1) * C + j] = kv.y;
                Kt[(d0 + 2) * C + j] = kv.z; Kt[(d0 + 3) * C + j] = kv.w;
            }
        }
        // ---- and k/v rows (head-dim fastest) ----
        for (int e = tid; e < C * (D / 4); e += blockDim.x) {
            const int j = e / (D / 4), d0 = (e % (D / 4)) * 4;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (j < n) {
                kv = load4(kb + (int64_t)(t0 + j) * p.k.sl + d0);
                vv = load4(vb + (int64_t)(t0 + j) * p.v.sl + d0);
                if (k_norm || ksc != 1.f) kv = prologue4(kv, k_norm ? kst[j] : make_float2(0.f, 1.f), p.pro.kw,
                                                         p.pro.kb, d0, ksc);
            }
            store4(Kr + j * D + d0, kv);
            store4(Vr + j * D + d0, vv);
        }
        __syncthreads();

        if (want_y) {
            // ---- P = decay-masked (1 + qk + 0.5 q^2 k^2), 4x4 tiles, row tile fastest ----
            for (int blk = tid; blk < (C / 4) * (C / 4); blk += blockDim.x) {
                const int i0 = (blk % (C / 4)) * 4, j0 = (blk / (C / 4)) * 4;
                float a1[4][4], a2[4][4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int w = 0; w < 4; ++w) a1[u][w] = a2[u][w] = 0.f;
                if (j0 <= i0 + 3) {
#pragma unroll 4
                    for (int d = 0; d < D; ++d) {
                        const float4 qv = *reinterpret_cast<const float4 *>(Qt + d * C + i0);
                        const float4 kv = *reinterpret_cast<const float4 *>(Kt + d * C + j0);
                        const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u)
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                a1[u][w] = fmaf(qa[u], ka[w], a1[u][w]);
                                a2[u][w] = fmaf(qa[u] * qa[u], ka[w] * ka[w], a2[u][w]);
                            }
                    }
                }
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    float o[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = i0 + u, j = j0 + w;
                        const float dij = (j <= i) ? (PT ? expf(lcum[i] - lcum[j]) : pw[i - j]) : 0.f;
                        o[u] = (j <= i) ? dij * (1.0f + a1[u][w] + 0.5f * a2[u][w]) : 0.f;
                    }
                    *reinterpret_cast<float4 *>(Pt + (j0 + w) * C + i0) = make_float4(o[0], o[1], o[2], o[3]);
                }
            }
            __syncthreads();
            // ---- row sums of P and the carried denominator ----
            for (int i = tid; i < C; i += blockDim.x) {
                float sd = 0.f;
                for (int j = 0; j <= i; ++j) sd += Pt[j * C + i];
                den[i] = sd;
                float c = 0.f;
                for (int d = 0; d < D; ++d) {
                    const float qv = Qt[d * C + i];
                    c = fmaf(qv, Z1[d], fmaf(0.5f * qv * qv, Z2[d], c));
                }
                cden[i] = c;
            }
            __syncthreads();
            // ---- num = P V, carry = psi(q) S, output ----
            for (int blk = tid; blk < (C / 4) * (D / 4); blk += blockDim.x) {
                const int i0 = (blk % (C / 4)) * 4, e0 = (blk / (C / 4)) * 4;
                float nm[4][4], cr[4][4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int w = 0; w < 4; ++w) nm[u][w] = cr[u][w] = 0.f;
                const int jmax = min(i0 + 4, C);
                for (int j = 0; j < jmax; ++j) {
                    const float4 pv = *reinterpret_cast<const float4 *>(Pt + j * C + i0);
                    const float4 vv = *reinterpret_cast<const float4 *>(Vr + j * D + e0);
                    const float pa[4] = {pv.x, pv.y, pv.z, pv.w}, va[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u)
#pragma unroll
                        for (int w = 0; w < 4; ++w) nm[u][w] = fmaf(pa[u], va[w], nm[u][w]);
                }
#pragma unroll 4
                for (int d = 0; d < D; ++d) {
                    const float4 qv = *reinterpret_cast<const float4 *>(Qt + d * C + i0);
                    const float4 s1 = *reinterpret_cast<const float4 *>(S1 + d * D + e0);
                    const float4 s2 = *reinterpret_cast<const float4 *>(S2 + d * D + e0);
                    const float qa[4] = {qv.x, qv.y, qv.z, qv.w};
                    const float s1a[4] = {s1.x, s1.y, s1.z, s1.w}, s2a[4] = {s2.x, s2.y, s2.z, s2.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float qh2 = 0.5f * qa[u] * qa[u];
#pragma unroll
                        for (int w = 0; w < 4; ++w) cr[u][w] = fmaf(qa[u], s1a[w], fmaf(qh2, s2a[w], cr[u][w]));
                    }
                }
                const float z0 = Z0[0];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = i0 + u;
                    if (i < n) {
                        const float g = PT ? gin[i] : pw[i + 1];
                        const float dd = fmaxf(den[i] + g * (z0 + cden[i]), p.eps);
                        const float inv = 1.0f / dd;
                        float o[4];
#pragma unroll
                        for (int w = 0; w < 4; ++w) o[w] = (nm[u][w] + g * (S0[e0 + w] + cr[u][w])) * inv;
                        store4(yb + (int64_t)(t0 + i) * p.y.sl + e0, make_float4(o[0], o[1], o[2], o[3]));
                    }
                }
            }
            __syncthreads();
        }
        // ---- state update (after every reader of the old state is done) ----
        const float decay_n = PT ? dsc[0] : pw[n];
        for (int blk = tid; blk < (D / 4) * (D / 4); blk += blockDim.x) {
            const int e0 = (blk % (D / 4)) * 4, d0 = (blk / (D / 4)) * 4;
            float u1[4][4], u2[4][4];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) u1[a][c] = u2[a][c] = 0.f;
            for (int j = 0; j < n; ++j) {
                const float wj = PT ? wend[j] : pw[n - 1 - j];
                const float4 kv = *reinterpret_cast<const float4 *>(Kr + j * D + d0);
                const float4 vv = *reinterpret_cast<const float4 *>(Vr + j * D + e0);
                const float ka[4] = {kv.x, kv.y, kv.z, kv.w};
                const float va[4] = {wj * vv.x, wj * vv.y, wj * vv.z, wj * vv.w};
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        u1[a][c] = fmaf(ka[a], va[c], u1[a][c]);
                        u2[a][c] = fmaf(ka[a] * ka[a], va[c], u2[a][c]);
                    }
            }
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                float4 *r1 = reinterpret_cast<float4 *>(S1 + (d0 + a) * D + e0);
                float4 *r2 = reinterpret_cast<float4 *>(S2 + (d0 + a) * D + e0);
                const float4 o1 = *r1, o2 = *r2;
                *r1 = make_float4(fmaf(decay_n, o1.x, u1[a][0]), fmaf(decay_n, o1.y, u1[a][1]),
                                  fmaf(decay_n, o1.z, u1[a][2]), fmaf(decay_n, o1.w, u1[a][3]));
                *r2 = make_float4(fmaf(decay_n, o2.x, u2[a][0]), fmaf(decay_n, o2.y, u2[a][1]),
                                  fmaf(decay_n, o2.z, u2[a][2]), fmaf(decay_n, o2.w, u2[a][3]));
            }
        }
        for (int i = tid; i < 3 * D; i += blockDim.x) {
            const int which = i / D, d = i - which * D;
            float acc = 0.f;
            for (int j = 0; j < n; ++j) {
                const float wj = PT ? wend[j] : pw[n - 1 - j];
                const float kv = Kr[j * D + d];
                acc = fmaf(wj, which == 0 ? Vr[j * D + d] : (which == 1 ? kv : kv * kv), acc);
            }
            float *dst = which == 0 ? S0 : (which == 1 ? Z1 : Z2);
            dst[d] = fmaf(decay_n, dst[d], acc);
        }
        if (tid == 0) {
            float acc = 0.f;
            if (PT) acc = dsc[1];
            else
                for (int j = 0; j < n; ++j) acc += pw[j];
            Z0[0] = fmaf(decay_n, Z0[0], acc);
        }
        __syncthreads();
    }

    // ---- state out ----
    const bool write_out = p.out.present() && (p.state_only || s == (int)gridDim.y - 1);
    if (write_out) {
        const HeadPtrs dst = p.out.at(bh, p.out.packed ? s : 0, D);
        const float sq_out = (p.half_sq && !p.out.packed) ? 0.5f : 1.f;
        for (int i = tid; i < D * D; i += blockDim.x) {
            dst.S1[i] = S1[i];
            dst.S2[i] = sq_out * S2[i];
        }
        for (int i = tid; i < D; i += blockDim.x) {
            dst.S0[i] = S0[i];
            dst.Z1[i] = Z1[i];
            dst.Z2[i] = sq_out * Z2[i];
        }
        if (tid == 0) dst.Z0[0] = Z0[0];
    }
}


}  // namespace pma
