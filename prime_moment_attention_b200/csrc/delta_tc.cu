// delta_tc.cu -- the gated delta-rule prefill on tcgen05 tensor cores (bf16 inputs, D = 64,
// the reference's chunk of 64 tokens).
//
// Same chunk algebra as delta.cu (ChunkedGatedDeltaPrimeAttention, chunked_delta_prime.py:175-283),
// with the four products of a chunk on the tensor cores and the triangular solve, the gates and
// the Lyapunov projection in float32 on CUDA cores.  Per chunk of n <= 64 tokens, F = 128 features:
//
//   MMA 1   D1 = [Phi ; Psi] [Phi | S]^T      (M = 128 rows: 64 phi rows, 64 psi rows; N = 64 + 64;
//           K = F)  -> Gram G = Phi Phi^T, intra scores Psi Phi^T, Phi S^T and Psi S^T in one group
//   solve   T = I + strict_tril(Lambda . G . beta_j),  u = v - exp(cum) . Phi S^T,  T E = u
//           (the 16 x 16 diagonal blocks inverted, then block substitution; float32)
//   MMA 2   y_intra = P (beta E),  P = tril(Lambda . Psi Phi^T) in bf16 in tensor memory (TS MMA)
//           (beta_j is applied once, in the bf16 beta E operand)
//   MMA 3   dS^T = Phi^T (coef . E)  (M = F, the feature-major state layout; K = tokens)
//   state   S = exp(cum_end) S + dS (float32 in registers: thread f owns feature row f of S^T),
//           S *= min(1, bound / (|S|_F + 1e-6)), and its bf16 copy for the next chunk's MMA 1
//   y       y_i = exp(cum_i) (Psi S^T)_i + y_intra_i
//
// q, k, v rows of the next chunk are copied into padded staging tiles with cp.async while the
// current chunk computes.
// Shared memory (about 116 KB): the [Phi ; Psi] operand as two K-halves of 128 x 64 bf16
// (128-byte swizzle), the bf16 state tile S^T [128 x 64] (MN-major B operand), the bf16 tiles of
// beta E and coef E [64 x 64] (MN-major B operands), and float32 T, u/E and the block inverses.
// Tensor memory (256 columns): D1 in 0..127 (P overwrites the psi rows' columns 0..31 once
// read), y_intra in 128..191, dS^T in 192..255.  256 threads; one elected thread issues the MMAs
// and commits them to one mbarrier; every wait is bounded by the global timer and, on expiry,
// records a status code and ends the chunk loop for the whole CTA.
#include "pma_common.cuh"
#include "prefill.cuh"
#include "tc_common.cuh"

namespace pma {
namespace dtc {

using namespace pma::tc;

constexpr int C = 64;    // tokens per chunk (the reference's chunk_size)
constexpr int D = 64;    // head dim
constexpr int F = 128;   // features
constexpr int NT = 256;  // threads
constexpr int VS = 68;   // float row stride of u / E (float4 accesses by rows stay conflict-free)

constexpr int OFF_A = 0;              // [Phi ; Psi] features 0..63, 128 rows x 128 B
constexpr int OFF_AH = 16384;         // features 64..127
constexpr int OFF_ST = 32768;         // S^T bf16 [128 f x 64 d], MN-major
constexpr int OFF_W = 49152;          // beta E bf16 [64 j x 64 d], MN-major
constexpr int OFF_WC = 57344;         // coef E bf16 [64 j x 64 d], MN-major
constexpr int OFF_T = 65536;          // Tt float [64 j][64 i] = T[i][j]
constexpr int OFF_VE = OFF_T + C * C * 4;            // u -> E float [64][VS]
constexpr int OFF_TI = OFF_VE + C * VS * 4;          // inverses of T's diagonal 16 x 16 blocks
constexpr int OFF_VEC = OFF_TI + (C / 16) * 256 * 4;  // cum, beta, exp(cum), coef: [4][64]
constexpr int OFF_RED = OFF_VEC + 4 * C * 4;          // [16] reductions
constexpr int OFF_BAR = OFF_RED + 16 * 4;             // mbarrier, tmem base, abort flag
constexpr int STG_ROW = 144;                          // staging row: 128 B of bf16 + 16 B pad
constexpr int OFF_STG = OFF_BAR + 32;                 // next chunk's k, q, v rows (cp.async)
constexpr int STG_TILE = C * STG_ROW;
constexpr int SMEM_USED = OFF_STG + 3 * STG_TILE;
constexpr size_t SMEM_BYTES = SMEM_USED + 1024;      // + alignment of the swizzled tiles
constexpr uint32_t T_D1 = 0, T_Y = 128, T_DS = 192, T_COLS = 256;

// 16-byte chunk c of row r in a [rows x 128 B] 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw(int r, int c) { return swz(r, c); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <typename TI, typename TO>
__global__ void __launch_bounds__(NT, 1) delta_tc_kernel(const DeltaParams p) {
    extern __shared__ uint8_t dsm_raw[];
    uint8_t *smem = smem_align1024(dsm_raw);
    float *const Tt = reinterpret_cast<float *>(smem + OFF_T);
    float *const VE = reinterpret_cast<float *>(smem + OFF_VE);
    float *const TIv = reinterpret_cast<float *>(smem + OFF_TI);
    float *const cum = reinterpret_cast<float *>(smem + OFF_VEC);
    float *const bet = cum + C;
    float *const din = bet + C;
    float *const coef = din + C;
    float *const red = reinterpret_cast<float *>(smem + OFF_RED);
    uint64_t *const bar = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_BAR + 8);
    CtlShared *const ctl_sh = reinterpret_cast<CtlShared *>(smem + OFF_BAR + 16);
    const uint32_t sb = su32(smem);

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
    Ctl ctl{ctl_sh, nullptr};

    // ---- set-up: barrier, tensor memory, zero operand rows, the state
    if (tid == 0) {
        mbar_init(bar, 1);
        init_ctl(*ctl_sh, p.fault);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(T_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // state: threads 128..255 own feature row f of S^T (64 value columns) in registers
    const bool st_thr = tid >= 128;
    const int f = tid - 128;
    float S[D];
    if (st_thr) {
        const float *sin = p.state_in ? p.state_in + (size_t)bh * D * F : nullptr;
#pragma unroll
        for (int d = 0; d < D; ++d) S[d] = sin ? sin[(size_t)d * F + f] : 0.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    uint32_t mma_phase = 0;

    auto publish_state = [&]() {  // bf16 S^T row f into the MN-major tile
        uint8_t *row = smem + OFF_ST;
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4 *>(row + sw(f, c)) = pack8(S + 8 * c);
    };
    if (st_thr) publish_state();

    constexpr uint64_t HI_KMAJ = desc_hi(16, 1024, 2);               // K-major, 128 B rows
    constexpr uint64_t HI_MN1 = desc_hi(16, 1024, 2);                // MN-major, one 64-element MN atom
    constexpr uint64_t HI_PHIT = desc_hi(OFF_AH - OFF_A, 1024, 2);   // Phi^T: M = F over both K-halves
    constexpr uint32_t ID_1 = idesc(128, 64, 0, 0), ID_1S = idesc(128, 64, 0, 1);
    constexpr uint32_t ID_Y = idesc(128, 64, 0, 1), ID_DS = idesc(128, 64, 1, 1);
    const uint32_t a0 = sb >> 4;
    auto dsc = [&](uint32_t off, uint64_t hi) { return (uint64_t)(a0 + (off >> 4)) | hi; };

    // rows of chunk t0 into the staging tiles (k, q, v; 16-byte asynchronous copies)
    auto stage = [&](int t0) {
        const int nn = min(C, p.L - t0);
        for (int e = tid; e < 3 * C * 8; e += NT) {
            const int which = e / (C * 8), rem = e - which * (C * 8), row = rem >> 3, c = rem & 7;
            if (row >= nn || (which == 1 && !want_y)) continue;
            const TI *src = which == 0 ? kb + (int64_t)(t0 + row) * p.k.sl
                                       : (which == 1 ? qb + (int64_t)(t0 + row) * p.q.sl : vb + (int64_t)(t0 + row) * p.v.sl);
            cp_async16(smem + OFF_STG + which * STG_TILE + row * STG_ROW + 16 * c, src + 8 * c);
        }
        cp_async_commit();
    };
    if (p.L > 0) stage(0);
    // warp 7: the gates of tokens 2 lane, 2 lane + 1 of the next chunk, loaded a chunk ahead
    float gb[2] = {0.f, 0.f}, ga[2] = {lam, lam};
    auto load_gates = [&](int t0) {
        const int nn = min(C, p.L - t0);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const int i = lane * 2 + m;
            gb[m] = i < nn ? beta_g[t0 + i] : 0.f;
            ga[m] = (i < nn && alpha_g) ? alpha_g[t0 + i] : lam;
        }
    };
    if (warp == 7 && p.L > 0) load_gates(0);

    bool ok = true;
    for (int t0 = 0; t0 < p.L && ok; t0 += C) {
        const int n = min(C, p.L - t0);
        cp_async_wait_all();
        __syncthreads();
        // ---- A. features into the operand tiles (bf16): two threads per row (lanes 2r, 2r + 1 of
        // warp w hold row 16 w + r: k rows 0..63 in warps 0-3, q rows in warps 4-7), 32 elements each
        {
            const int row = tid >> 1, hf = tid & 1;
            const bool is_q = row >= C;
            const int i = row & (C - 1);
            const uint8_t *srow = smem + OFF_STG + (is_q ? STG_TILE : 0) + i * STG_ROW + 64 * hf;
            float x[32];
            if (i < n) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 u4 = *reinterpret_cast<const uint4 *>(srow + 16 * c);
                    const float2 a = bf2f(u4.x), bq = bf2f(u4.y), cq = bf2f(u4.z), dq = bf2f(u4.w);
                    x[8 * c] = a.x; x[8 * c + 1] = a.y; x[8 * c + 2] = bq.x; x[8 * c + 3] = bq.y;
                    x[8 * c + 4] = cq.x; x[8 * c + 5] = cq.y; x[8 * c + 6] = dq.x; x[8 * c + 7] = dq.y;
                }
            } else {
#pragma unroll
                for (int d = 0; d < 32; ++d) x[d] = 0.f;
            }
            float s1 = 1.f, s2 = r2;
            if (!is_q) {  // warp-uniform: warps 0-3 hold k rows
                float n1 = 0.f, n2 = 0.f;
#pragma unroll
                for (int d = 0; d < 32; ++d) {
                    const float k2 = x[d] * x[d];
                    n1 = fmaf(x[d], x[d], n1);
                    n2 = fmaf(k2, k2, n2);
                }
                n1 += __shfl_xor_sync(0xffffffffu, n1, 1);
                n2 += __shfl_xor_sync(0xffffffffu, n2, 1);
                s1 = 1.0f / fmaxf(sqrtf(n1), p.norm_eps);
                s2 = r2 / fmaxf(sqrtf(n2), p.norm_eps);
            }
            if (is_q && !want_y) s1 = s2 = 0.f;
            float t[8];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
#pragma unroll
                for (int e = 0; e < 8; ++e) t[e] = x[8 * c + e] * s1;
                *reinterpret_cast<uint4 *>(smem + OFF_A + sw(row, 4 * hf + c)) = pack8(t);
#pragma unroll
                for (int e = 0; e < 8; ++e) t[e] = x[8 * c + e] * x[8 * c + e] * s2;
                *reinterpret_cast<uint4 *>(smem + OFF_AH + sw(row, 4 * hf + c)) = pack8(t);
            }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- B. MMA 1: D1 = [Phi ; Psi] [Phi | S]^T
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t ko = (k < 4 ? OFF_A : OFF_AH);
                const uint64_t kk = (uint64_t)((k & 3) * 2);  // +32 B inside the 128 B row
                mma_ss(tmem + T_D1, dsc(ko, HI_KMAJ) + kk, dsc(ko, HI_KMAJ) + kk, ID_1, k > 0);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k)  // B = S^T rows 16k..16k+15 (K = features)
                mma_ss(tmem + T_D1 + 64, dsc(k < 4 ? OFF_A : OFF_AH, HI_KMAJ) + (uint64_t)((k & 3) * 2),
                       dsc(OFF_ST, HI_MN1) + (uint64_t)(k * 128), ID_1S, k > 0);
            commit(bar);
        }
        // while the MMAs run: v rows into u's buffer (warps 4-5), the gates' scan, exp(cum) and the
        // state-update weights (warp 7)
        if (warp == 4 || warp == 5) {
            const int j = tid - 128;
            float4 *dst = reinterpret_cast<float4 *>(VE + j * VS);
            const uint8_t *srow = smem + OFF_STG + 2 * STG_TILE + j * STG_ROW;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                float4 lo = make_float4(0, 0, 0, 0), hi = lo;
                if (j < n) {
                    const uint4 u4 = *reinterpret_cast<const uint4 *>(srow + 16 * c);
                    const float2 a = bf2f(u4.x), bq = bf2f(u4.y), cq = bf2f(u4.z), dq = bf2f(u4.w);
                    lo = make_float4(a.x, a.y, bq.x, bq.y);
                    hi = make_float4(cq.x, cq.y, dq.x, dq.y);
                }
                dst[2 * c] = lo;
                dst[2 * c + 1] = hi;
            }
        } else if (warp == 7) {  // inclusive scan of log alpha (2 tokens per lane)
            float la[2], run = 0.f;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int i = lane * 2 + m;
                const float a = i < n ? fminf(fmaxf(ga[m], 1e-5f), 1.0f) : lam_c;
                run += __logf(a);
                la[m] = run;
                bet[i] = i < n ? gb[m] : 0.f;
            }
            float incl = run;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float tt = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += tt;
            }
            const float base = incl - run;
            la[0] += base;
            la[1] += base;
            const float ce = __shfl_sync(0xffffffffu, la[1], 31);
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int i = lane * 2 + m;
                cum[i] = la[m];
                din[i] = __expf(la[m]);
                coef[i] = bet[i] * __expf(ce - la[m]);
            }
        }
        if (warp == 7 && t0 + C < p.L) load_gates(t0 + C);  // this chunk's gates are consumed
        bool w_ok = mbar_wait(bar, mma_phase, ctl, 1);
        mma_phase ^= 1;
        if (!__syncthreads_and(w_ok)) { ok = false; break; }
        tc_fence_after();
        // the staging tiles are consumed (features in phase A, v rows in phase B): the next chunk's
        // rows land while this one computes
        if (t0 + C < p.L) stage(t0 + C);
        // ---- C. T and u (phi rows: warps 0, 1, 4, 5), P in bf16 (psi rows: warps 2, 3, 6, 7); warps w and
        // w + 4 share a tensor-memory lane quadrant and take one half of its columns each
        {
            const int quad = warp & 3, hc = warp >> 2;  // column half
            const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
            float g[32];
            if (quad < 2) {
                const int i = quad * 32 + lane;  // phi row i
                const float ci = cum[i];
                tmem_ld32(lb + T_D1 + 32 * hc, g);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int j = 32 * hc + e;
                    Tt[j * C + i] = j < i ? __expf(ci - cum[j]) * g[e] * bet[j] : (j == i ? 1.f : 0.f);
                }
                const float di = din[i];
                float4 *ve = reinterpret_cast<float4 *>(VE + i * VS + 32 * hc);
                tmem_ld32(lb + T_D1 + 64 + 32 * hc, g);
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    float4 v4 = ve[e / 4];
                    v4.x -= di * g[e]; v4.y -= di * g[e + 1]; v4.z -= di * g[e + 2]; v4.w -= di * g[e + 3];
                    ve[e / 4] = v4;
                }
            } else {
                const int i = (quad - 2) * 32 + lane;  // psi row i (tensor-memory lane 64 + i)
                const float ci = cum[i];
                uint32_t pk[16];
                tmem_ld32(lb + T_D1 + 32 * hc, g);
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const int j = 32 * hc + e;
                    const float p0 = j <= i ? __expf(ci - cum[j]) * g[e] : 0.f;  // beta_j sits in beta E
                    const float p1 = j + 1 <= i ? __expf(ci - cum[j + 1]) * g[e + 1] : 0.f;
                    pk[e / 2] = pack2(p0, p1);
                }
                // P row i as bf16 pairs goes to columns 16 hc .. 16 hc + 15; columns 16..31 are still
                // scores that the hc = 0 warp of this quadrant reads, so the four psi warps write only
                // after all of them have their scores in registers
                tc_fence_before();
                named_bar(2, 128);
                tc_fence_after();
                tmem_st16(lb + T_D1 + 16 * hc, pk);
                tmem_wait_st();
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- D. solve T E = u: inverses of the diagonal blocks, then block substitution
        {  // inverses of the diagonal blocks: thread (block, column c, k-quarter kq); the four threads
           // of a column split each row's sum over k and join it with two shuffles
            const int bi = tid >> 6, c = (tid >> 2) & 15, kq = tid & 3, r0 = bi * 16;
            float x[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float s = 0.f;
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    if ((k & 3) == kq && k >= c && k < i) s = fmaf(-Tt[(r0 + k) * C + r0 + i], x[k], s);
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                x[i] = i == c ? 1.f : (i > c ? s : 0.f);
            }
            if (kq == 0) {
#pragma unroll
                for (int i = 0; i < 16; ++i) TIv[(bi * 16 + i) * 16 + c] = x[i];
            }
        }
        __syncthreads();
        {
            const int rl = tid >> 4, dd = (tid & 15) * 4;  // 16 rows x 16 float4 column groups
#pragma unroll 1
            for (int bi = 0; bi < C / 16; ++bi) {
                const int r = bi * 16 + rl;
                if (bi > 0) {
                    float4 acc = *reinterpret_cast<const float4 *>(VE + r * VS + dd);
                    for (int jb = 0; jb < bi; ++jb) {  // 16 rows per pass, unrolled: the loads pipeline
                        float4 a2 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 2) {
                            const int j = jb * 16 + jj;
                            const float t0v = Tt[j * C + r], t1v = Tt[(j + 1) * C + r];
                            const float4 e0 = *reinterpret_cast<const float4 *>(VE + j * VS + dd);
                            const float4 e1 = *reinterpret_cast<const float4 *>(VE + (j + 1) * VS + dd);
                            acc.x = fmaf(-t0v, e0.x, acc.x); acc.y = fmaf(-t0v, e0.y, acc.y);
                            acc.z = fmaf(-t0v, e0.z, acc.z); acc.w = fmaf(-t0v, e0.w, acc.w);
                            a2.x = fmaf(-t1v, e1.x, a2.x); a2.y = fmaf(-t1v, e1.y, a2.y);
                            a2.z = fmaf(-t1v, e1.z, a2.z); a2.w = fmaf(-t1v, e1.w, a2.w);
                        }
                        acc.x += a2.x; acc.y += a2.y; acc.z += a2.z; acc.w += a2.w;
                    }
                    *reinterpret_cast<float4 *>(VE + r * VS + dd) = acc;
                }
                __syncthreads();
                float4 e4 = make_float4(0, 0, 0, 0);
                const float *xr = TIv + (bi * 16 + rl) * 16;
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const float xk = xr[k];
                    const float4 rk = *reinterpret_cast<const float4 *>(VE + (bi * 16 + k) * VS + dd);
                    e4.x = fmaf(xk, rk.x, e4.x); e4.y = fmaf(xk, rk.y, e4.y);
                    e4.z = fmaf(xk, rk.z, e4.z); e4.w = fmaf(xk, rk.w, e4.w);
                }
                __syncthreads();
                *reinterpret_cast<float4 *>(VE + r * VS + dd) = e4;
                __syncthreads();  // the next block's R step reads these E rows
            }
        }
        // beta E and coef E as bf16 MN-major tiles (row j = token, 64 value columns)
        if (tid < 2 * C) {
            const int j = tid & (C - 1);
            const float sc = tid < C ? bet[j] : coef[j];
            uint8_t *tile = smem + (tid < C ? OFF_W : OFF_WC);
            const float *er = VE + j * VS;
            float t[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
#pragma unroll
                for (int e = 0; e < 8; ++e) t[e] = sc * er[8 * c + e];
                *reinterpret_cast<uint4 *>(tile + sw(j, c)) = pack8(t);
            }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- E. MMA 2 (y_intra = P (beta E)) and MMA 3 (dS^T = Phi^T (coef E))
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < 4; ++k)  // K = tokens: 16 per step = 8 bf16-pair columns of P
                mma_ts(tmem + T_Y, tmem + T_D1 + k * 8, dsc(OFF_W, HI_MN1) + (uint64_t)(k * 128), ID_Y, k > 0);
#pragma unroll
            for (int k = 0; k < 4; ++k)  // A = Phi^T (phi rows 16k..16k+15 of both K-halves)
                mma_ss(tmem + T_DS, dsc(OFF_A, HI_PHIT) + (uint64_t)(k * 128), dsc(OFF_WC, HI_MN1) + (uint64_t)(k * 128),
                       ID_DS, k > 0);
            commit(bar);
        }
        w_ok = mbar_wait(bar, mma_phase, ctl, 2);
        mma_phase ^= 1;
        if (!__syncthreads_and(w_ok)) { ok = false; break; }
        tc_fence_after();
        // ---- F. output rows (psi lanes, warps 2-3) and the state (feature lanes, warps 4-7)
        if (warp >= 2 && warp < 4) {
            const int i = tid - 64;
            const uint32_t lb = tmem + ((uint32_t)(warp * 32) << 16);
            if (want_y) {
                const float di = din[i];
                float a[32], yi[32];
#pragma unroll
                for (int hc = 0; hc < 2; ++hc) {
                    tmem_ld32(lb + T_D1 + 64 + 32 * hc, a);
                    tmem_ld32(lb + T_Y + 32 * hc, yi);
#pragma unroll
                    for (int e = 0; e < 32; ++e) a[e] = fmaf(di, a[e], yi[e]);
                    if (i < n) {
                        TO *dst = yb + (int64_t)(t0 + i) * p.y.sl + 32 * hc;
#pragma unroll
                        for (int e = 0; e < 32; e += 4) store4(dst + e, make_float4(a[e], a[e + 1], a[e + 2], a[e + 3]));
                    }
                }
            }
        } else if (st_thr) {
            const uint32_t lb = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // lane = feature f
            const float cd = __expf(cum[C - 1]);
            float ds[32], sq = 0.f;
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
                tmem_ld32(lb + T_DS + 32 * hc, ds);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    S[32 * hc + e] = fmaf(cd, S[32 * hc + e], ds[e]);
                    sq = fmaf(S[32 * hc + e], S[32 * hc + e], sq);
                }
            }
            if (p.bound > 0.f) {
                sq = warp_sum(sq);
                if (lane == 0) red[warp - 4] = sq;
                named_bar(1, 128);
                const float tot = red[0] + red[1] + red[2] + red[3];
                const float sc = fminf(p.bound / (sqrtf(tot) + 1e-6f), 1.0f);
                if (sc < 1.f) {
#pragma unroll
                    for (int d = 0; d < D; ++d) S[d] *= sc;
                }
            }
            publish_state();
        }
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }

    cp_async_wait_all();  // no copy may still target this CTA's shared memory at exit
    // ---- state out (S^T row f -> S[d][f])
    if (ok && st_thr && p.state_out) {
        float *so = p.state_out + (size_t)bh * D * F;
#pragma unroll
        for (int d = 0; d < D; ++d) so[(size_t)d * F + f] = S[d];
    }
    // never free tensor memory under an MMA in flight: a failed wait waits once more, bounded
    if (!ok && tid == 0) {
        const unsigned long long w0 = gtimer();
        while (!mbar_try(bar, mma_phase ^ 1) && gtimer() - w0 < WAIT_NS) {
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T_COLS) : "memory");
}

template <typename TI, typename TO>
cudaError_t launch_t(const DeltaParams &p, cudaStream_t st) {
    cudaError_t e = set_smem_once<delta_tc_kernel<TI, TO>>((int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    delta_tc_kernel<TI, TO><<<p.B * p.H, NT, SMEM_BYTES, st>>>(p);
    return cudaGetLastError();
}

}  // namespace dtc

bool delta_tc_supported(int D, int chunk, int idt) { return D == 64 && chunk == 64 && idt == PMA_BF16; }

cudaError_t launch_delta_prefill_tc(const DeltaParams &p, int ydt, cudaStream_t st) {
    return ydt == PMA_F32 ? dtc::launch_t<__nv_bfloat16, float>(p, st)
                          : dtc::launch_t<__nv_bfloat16, __nv_bfloat16>(p, st);
}

}  // namespace pma
