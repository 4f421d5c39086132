// delta_wy.cu -- the gated delta-rule prefill in WY form on tcgen05 tensor cores (bf16 inputs,
// D = 64, the reference's chunk of 64 tokens), as two kernels.
//
// The chunk algebra of ChunkedGatedDeltaPrimeAttention (chunked_delta_prime.py:175-283) solves
// T E = u per chunk with u = v - exp(cum) . Phi S^T.  T (unit lower triangular, T_ij =
// beta_j Lambda_ij G_ij below the diagonal) depends on the chunk's keys and gates only, so
//
//     E = U - W S^T,   U = T^-1 v,   W = T^-1 diag(exp(cum)) Phi,
//
// and everything but the two products with the state can be computed for all chunks at once.
//
// delta_wy_prep_kernel -- one unit = one (head-state, chunk); persistent CTAs of 256 threads walk
// the units, with the next unit's rows copied into staging tiles while the current one computes:
//   features Phi, Psi (bf16) and the gates' scan; G = Phi Phi^T and Psi Phi^T in one MMA group
//   (M = 128); T in float32; T^-1 by its 16 x 16 diagonal blocks (forward substitution) and three
//   block levels (register-tiled products), float32; T^-1 as a bf16 pair hi + lo so that the
//   products keep float32-level accuracy in that factor; [U | W] = T^-1 [v | exp(cum) Phi] as one
//   M = 64, N = 192 MMA group (an M = 64 accumulator holds row r in tensor-memory lane
//   (r mod 16) + 32 (r div 16)).  It writes one 72 KB record per unit, laid out as the
//   shared-memory operand tiles the sequential kernel feeds to its MMAs (128-byte swizzle):
//     A1    [128 rows][128 f] bf16, K-major in two K-halves: rows 0..63 W, rows 64..127 Psie =
//           diag(exp(cum)) Psi (A of MMA 1)
//     P'    [64 i][64 j]  bf16, P' = tril(Lambda . Psi Phi^T) diag(beta) (K-major A of MMA 2)
//     Phic  [64 j][128 f] bf16 token rows, Phic = diag(beta_j exp(cum_end - cum_j)) Phi
//           (MN-major A of MMA 3)
//     U     [64 i][64 d]  float32 rows, 16-byte chunks XOR-swizzled by row
//   and the chunk's decay exp(cum_end) into a separate array.
//
// delta_wy_seq_kernel -- one CTA per head-state walks its chunks, warp-specialised:
//   warp 8 copies each chunk's record into one of two stages (bulk copies on mbarriers);
//   warp 9 issues MMA 1: D1 = [W ; Psie] S^T (M = 128, N = 64, K = 128), then after E is ready
//     MMA 3: dS^T = Phic^T E and MMA 2: D2 = [0 ; P'] E;
//   warps 4-5 (tensor-memory lanes 0..63): E = U - sc W S^T into a bf16 tile;
//   warps 6-7 (lanes 64..127): y = sc Psie S^T + P' E rows out;
//   warps 0-3 (lane = feature f): S = exp(cum_end) S + dS, its bf16 copy for the next MMA 1,
//     then the Lyapunov factor sc = min(1, bound / (|S|_F + 1e-6)) and S *= sc.  The tile is
//     published before the projection: W S^T and Psie S^T are linear in S, so the E and y warps
//     apply sc after the products and the norm's reduction stays off the chunk chain.
// The per-chunk chain is two MMA groups and two short CUDA-core steps; the triangular solve is
// off it.  Records of long sequences are produced and consumed in windows of chunks, the state
// carried between windows through state_out (or a workspace copy).
//
// Every wait is bounded by the global timer; on expiry the CTA records a status code, stops its
// loops, waits (bounded) for the copies and MMAs it issued, frees tensor memory and returns.
#define PMA_FAULT_AT_EXIT 1
#include "pma_common.cuh"
#include "prefill.cuh"
#include "tc_common.cuh"

namespace pma {
namespace dwy {

using namespace pma::tc;

constexpr int C = 64;   // tokens per chunk
constexpr int D = 64;   // head dim
constexpr int F = 128;  // features

// ---- the record of one unit (global memory)
constexpr int R_A0 = 0;         // A1 K-half 0: W rows 0..63, Psie rows 64..127, features 0..63
constexpr int R_A1 = 16384;     // features 64..127
constexpr int R_P = 32768;      // P'
constexpr int R_PC = 40960;     // Phic features 0..63 (then 64..127 at +8192)
constexpr int R_U = 57344;      // U
constexpr int REC = 73728;

// float4 chunk c (of 16) of row r in a [64][64] float32 tile whose chunks are XOR-swizzled by row
__device__ __forceinline__ uint32_t xsw(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 15)) << 4)); }

// ---------------------------------------------------------------------------------------------
// Prep kernel
// ---------------------------------------------------------------------------------------------
constexpr int PT = 256;                  // threads
constexpr int P_A = 0;                   // [Phi ; Psi] K-major, features 0..63 (128 rows x 128 B)
constexpr int P_AH = 16384;              // features 64..127
constexpr int P_X = 0;                   // after MMA G: T^-1 float32 [64][64], xsw layout
constexpr int P_RB = 16384;              // after MMA G: level products R [3][16][RBS] float32
constexpr int RBS = 20;                  // row stride of R (float4 accesses conflict-free)
constexpr int P_V = 32768;               // v rows [64 j][64 d] bf16 \  N-atoms of the MN-major B of
constexpr int P_E0 = 40960;              // exp(cum) Phi rows f 0..63 |  MMA UW (8 KB apart)
constexpr int P_E1 = 49152;              // f 64..127                 /
constexpr int P_T = 57344;               // T float32 [64][64], xsw layout; then T^-1 hi / lo bf16
constexpr int P_TH = P_T, P_TL = P_T + 8192;
constexpr int P_VEC = 73728;             // cum, exp(cum), beta, beta exp(-cum): [4][64] float32
constexpr int P_BAR = P_VEC + 1024;      // mbarriers, tmem slot, CtlShared
constexpr int STG_ROW = 144;             // staging row: 128 B + 16 B pad
constexpr int STG_TILE = C * STG_ROW;
constexpr int P_STG = P_BAR + 64;        // next unit's k, q, v rows
constexpr int P_SG = P_STG + 3 * STG_TILE;  // next unit's gates: beta [64], alpha [64], lambda
constexpr int P_SMEM = P_SG + 2 * C * 4 + 16;
constexpr size_t P_SMEM_BYTES = P_SMEM + 1024;
constexpr uint32_t PT_D1 = 0, PT_UW = 64, PT_COLS = 256;
// exp(cum_i - cum_j) as exp(cum_i) exp(-cum_j) while exp(-cum) stays far from overflow
constexpr float RATIO_MIN_CUM = -60.f;

struct PrepArgs {
    DeltaParams p;
    int c0;       // first chunk of the window
    int ncw;      // chunks in the window
    uint8_t *rec; // [BH][ncw] records
    float *cd;    // [BH][ncw] exp(cum_end)
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint4 pack8s(const float *x, float s) {
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = x[e] * s;
    return pack8(t);
}
__device__ __forceinline__ float4 ld4(const uint8_t *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(uint8_t *p, float a, float b, float c, float d) {
    *reinterpret_cast<float4 *>(p) = make_float4(a, b, c, d);
}

template <typename TI>
__global__ void __launch_bounds__(PT, 2) delta_wy_prep_kernel(const PrepArgs a) {
    extern __shared__ uint8_t dsm_raw[];
    uint8_t *smem = smem_align1024(dsm_raw);
    const DeltaParams &p = a.p;
    uint8_t *const Tb = smem + P_T;
    uint8_t *const Xb = smem + P_X;
    float *const RB = reinterpret_cast<float *>(smem + P_RB);
    float *const cum = reinterpret_cast<float *>(smem + P_VEC);
    float *const ecum = cum + C;
    float *const bet = ecum + C;
    float *const rbv = bet + C;  // beta_j exp(-cum_j) (ratio form)
    uint64_t *const bar = reinterpret_cast<uint64_t *>(smem + P_BAR);
    uint64_t *const never = bar + 1;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(smem + P_BAR + 16);
    int *const ratio_flag = reinterpret_cast<int *>(smem + P_BAR + 20);
    CtlShared *const ctl_sh = reinterpret_cast<CtlShared *>(smem + P_BAR + 32);
    const uint32_t sb = su32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int BH = p.B * p.H;
    const int units = BH * a.ncw;
    const bool want_y = p.y.p != nullptr;
    const float r2 = 0.70710678118654752f;
    Ctl ctl{ctl_sh, nullptr};

    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_init(never, 1);
        init_ctl(*ctl_sh, p.fault);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(PT_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (p.test_wait_ns) {  // test hook: a wait expires before any copy or MMA is issued
        if (tid == 0) expire_test_wait(never, ctl, p.test_wait_ns, 95);
        __syncthreads();
        if (ctl.aborted()) {
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (warp == 0)
                asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PT_COLS)
                             : "memory");
            if (tid == 0) report_fault(ctl_sh->abort_flag, p.fault);
            return;
        }
    }

    constexpr uint64_t HI_KMAJ = desc_hi(16, 1024, 2);
    constexpr uint64_t HI_MNB = desc_hi(8192, 1024, 2);  // MN-major B: 64-wide N-atoms 8 KB apart
    constexpr uint32_t ID_G = idesc(128, 64, 0, 0), ID_UW = idesc(64, 192, 0, 1);
    const uint32_t a0 = sb >> 4;
    auto dsc = [&](uint32_t off, uint64_t hi) { return (uint64_t)(a0 + (off >> 4)) | hi; };

    auto unit_of = [&](int u, int &bh, int &t0, int &n) {
        bh = u / a.ncw;
        const int c = u - bh * a.ncw;
        t0 = (a.c0 + c) * C;
        n = min(C, p.L - t0);
    };
    // rows of unit u into the staging tiles (k, q, v): thread t copies 16-byte chunks 2 (t & 3) and
    // 2 (t & 3) + 1 of row t >> 2 of each tile; threads 0..127 copy the gates (4-byte copies: the
    // gate rows have no alignment beyond their element size), thread 128 the decay
    auto stage = [&](int u) {
        int bh, t0, n;
        unit_of(u, bh, t0, n);
        const int b = bh / p.H, h = bh - b * p.H;
        if (tid < 2 * C) {
            const int i = tid & (C - 1);
            const float *src = tid < C ? p.beta : p.alpha;
            if (i < n && src) cp_async4(smem + P_SG + 4 * tid, src + (size_t)bh * p.L + t0 + i);
        } else if (tid == 2 * C) {
            cp_async4(smem + P_SG + 8 * C, p.lambda + (int64_t)b * p.lam_sb + h);
        }
        const int row = tid >> 2, c2 = (tid & 3) * 2;
        if (row < n) {
            const TI *ks = reinterpret_cast<const TI *>(p.k.p) + b * p.k.sb + h * p.k.sh + (int64_t)(t0 + row) * p.k.sl;
            const TI *vs = reinterpret_cast<const TI *>(p.v.p) + b * p.v.sb + h * p.v.sh + (int64_t)(t0 + row) * p.v.sl;
            uint8_t *dk = smem + P_STG + row * STG_ROW + 16 * c2;
            cp_async16(dk, ks + 8 * c2);
            cp_async16(dk + 16, ks + 8 * c2 + 8);
            cp_async16(dk + 2 * STG_TILE, vs + 8 * c2);
            cp_async16(dk + 2 * STG_TILE + 16, vs + 8 * c2 + 8);
            if (want_y) {
                const TI *qs = reinterpret_cast<const TI *>(p.q.p) + b * p.q.sb + h * p.q.sh + (int64_t)(t0 + row) * p.q.sl;
                cp_async16(dk + STG_TILE, qs + 8 * c2);
                cp_async16(dk + STG_TILE + 16, qs + 8 * c2 + 8);
            }
        }
        cp_async_commit();
    };
    if ((int)blockIdx.x < units) stage(blockIdx.x);

    uint32_t phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int bh, t0, n;
        unit_of(u, bh, t0, n);
        uint8_t *rec = a.rec + (size_t)u * REC;
        cp_async_wait_all();
        __syncthreads();
        // ---- gates (staged with the rows): every warp scans log alpha within the chunk itself (two
        // tokens per lane; padded tokens decay by lambda), so no barrier follows; warp 0 also leaves
        // the vectors the later phases read
        float ecm[2], cfm[2];
        {
            const float *sg = reinterpret_cast<const float *>(smem + P_SG);
            const float glam = sg[2 * C];
            const float lam_c = fminf(fmaxf(glam, 1e-5f), 1.0f);
            float gb[2], la[2], run = 0.f;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int i = lane * 2 + m;
                gb[m] = i < n ? sg[i] : 0.f;
                const float ga = i < n ? (p.alpha ? sg[C + i] : glam) : lam_c;
                const float al = i < n ? fminf(fmaxf(ga, 1e-5f), 1.0f) : lam_c;
                run += __logf(al);
                la[m] = run;
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
                ecm[m] = __expf(la[m]);
                cfm[m] = gb[m] * __expf(ce - la[m]);
            }
            if (warp == 0) {
                const bool ratio = ce >= RATIO_MIN_CUM;
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    const int i = lane * 2 + m;
                    cum[i] = la[m];
                    ecum[i] = ecm[m];
                    bet[i] = gb[m];
                    rbv[i] = ratio ? gb[m] * __expf(-la[m]) : 0.f;
                }
                if (lane == 0) {
                    a.cd[u] = __expf(ce);
                    *ratio_flag = ratio;
                }
            }
        }
        // ---- features: threads 2r, 2r + 1 hold row r of [Phi ; Psi] (r < 64: k row r, else q row
        // r - 64), 32 input dims each (hf = which half)
        {
            const int row = tid >> 1, hf = tid & 1;
            const bool is_q = row >= C;
            const int i = row & (C - 1);
            const uint8_t *srow = smem + P_STG + (is_q ? STG_TILE : 0) + i * STG_ROW + 64 * hf;
            float x[32];
            if (i < n && (!is_q || want_y)) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 u4 = *reinterpret_cast<const uint4 *>(srow + 16 * c);
                    const float2 f0 = bf2f(u4.x), f1 = bf2f(u4.y), f2 = bf2f(u4.z), f3 = bf2f(u4.w);
                    x[8 * c] = f0.x; x[8 * c + 1] = f0.y; x[8 * c + 2] = f1.x; x[8 * c + 3] = f1.y;
                    x[8 * c + 4] = f2.x; x[8 * c + 5] = f2.y; x[8 * c + 6] = f3.x; x[8 * c + 7] = f3.y;
                }
            } else {
#pragma unroll
                for (int d = 0; d < 32; ++d) x[d] = 0.f;
            }
            float s1 = 1.f, s2 = r2;
            if (!is_q) {  // warp-uniform
                float n1[4] = {0.f, 0.f, 0.f, 0.f}, n2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int d = 0; d < 32; ++d) {
                    const float k2 = x[d] * x[d];
                    n1[d & 3] = fmaf(x[d], x[d], n1[d & 3]);
                    n2[d & 3] = fmaf(k2, k2, n2[d & 3]);
                }
                float m1 = (n1[0] + n1[1]) + (n1[2] + n1[3]), m2 = (n2[0] + n2[1]) + (n2[2] + n2[3]);
                m1 += __shfl_xor_sync(0xffffffffu, m1, 1);
                m2 += __shfl_xor_sync(0xffffffffu, m2, 1);
                s1 = 1.0f / fmaxf(sqrtf(m1), p.norm_eps);
                s2 = r2 / fmaxf(sqrtf(m2), p.norm_eps);
            }
            // features 32 hf + d (x s1) and 64 + 32 hf + d (x^2 s2)
            float y2[32];
#pragma unroll
            for (int d = 0; d < 32; ++d) {
                y2[d] = x[d] * x[d] * s2;
                x[d] *= s1;
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                *reinterpret_cast<uint4 *>(smem + P_A + swz(row, 4 * hf + c)) = pack8(x + 8 * c);
                *reinterpret_cast<uint4 *>(smem + P_AH + swz(row, 4 * hf + c)) = pack8(y2 + 8 * c);
            }
            // exp(cum_i) and coef_i from the lane that scanned token i
            const float e0 = __shfl_sync(0xffffffffu, ecm[0], i >> 1), e1 = __shfl_sync(0xffffffffu, ecm[1], i >> 1);
            const float f0 = __shfl_sync(0xffffffffu, cfm[0], i >> 1), f1 = __shfl_sync(0xffffffffu, cfm[1], i >> 1);
            const float e = (i & 1) ? e1 : e0;
            if (!is_q) {
                const float cf = (i & 1) ? f1 : f0;
                uint8_t *pc = rec + R_PC;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    *reinterpret_cast<uint4 *>(smem + P_E0 + swz(i, 4 * hf + c)) = pack8s(x + 8 * c, e);
                    *reinterpret_cast<uint4 *>(smem + P_E1 + swz(i, 4 * hf + c)) = pack8s(y2 + 8 * c, e);
                    *reinterpret_cast<uint4 *>(pc + swz(i, 4 * hf + c)) = pack8s(x + 8 * c, cf);
                    *reinterpret_cast<uint4 *>(pc + 8192 + swz(i, 4 * hf + c)) = pack8s(y2 + 8 * c, cf);
                }
            } else {
                // Psie row i into A1 rows 64..127; half hf of v row i into its tile
                const uint8_t *vrow = smem + P_STG + 2 * STG_TILE + i * STG_ROW + 64 * hf;
                uint4 v4[4];
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    v4[c] = i < n ? *reinterpret_cast<const uint4 *>(vrow + 16 * c) : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    *reinterpret_cast<uint4 *>(rec + R_A0 + swz(C + i, 4 * hf + c)) = pack8s(x + 8 * c, e);
                    *reinterpret_cast<uint4 *>(rec + R_A1 + swz(C + i, 4 * hf + c)) = pack8s(y2 + 8 * c, e);
                    *reinterpret_cast<uint4 *>(smem + P_V + swz(i, 4 * hf + c)) = v4[c];
                }
            }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // the staging tiles are consumed: the next unit's rows land while this one computes
        if (u + (int)gridDim.x < units) stage(u + gridDim.x);
        // ---- MMA G: D1 = [Phi ; Psi] Phi^T (rows 0..63: G; rows 64..127: Psi Phi^T)
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t ko = (k < 4 ? P_A : P_AH);
                const uint64_t kk = (uint64_t)((k & 3) * 2);
                mma_ss(tmem + PT_D1, dsc(ko, HI_KMAJ) + kk, dsc(ko, HI_KMAJ) + kk, ID_G, k > 0);
            }
            commit(bar);
        }
        bool w_ok = mbar_wait(bar, phase, ctl, 96);
        phase ^= 1;
        if (!__syncthreads_and(w_ok)) { ok = false; break; }
        tc_fence_after();
        // ---- T rows (G lanes: warps 0, 1, 4, 5) and P' rows (Psi Phi^T lanes: warps 2, 3, 6, 7);
        // warps w and w + 4 share a lane quadrant and take one column half each.  All shared-memory
        // reads precede the stores, which the compiler must assume alias them.
        {
            const int quad = warp & 3, hc = warp >> 2;
            const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
            const bool t_rows = quad < 2;
            const int i = (quad & 1) * 32 + lane;
            const bool ratio = *ratio_flag != 0;
            const float ci = cum[i], ei = ecum[i];
#pragma unroll
            for (int hq = 0; hq < 2; ++hq) {  // 16 columns at a time (register pressure)
                const int j0 = 32 * hc + 16 * hq;
                uint32_t gr[16];
                float t[16];
                tmem_ld16_issue(lb + PT_D1 + j0, gr);
                tmem_wait_ld_regs(gr);
#pragma unroll
                for (int e = 0; e < 16; e += 4) {
                    float val[4];
                    if (ratio) {  // uniform: exp(cum_i) beta_j exp(-cum_j)
                        const float4 r4 = *reinterpret_cast<const float4 *>(rbv + j0 + e);
                        val[0] = ei * r4.x * __uint_as_float(gr[e]);
                        val[1] = ei * r4.y * __uint_as_float(gr[e + 1]);
                        val[2] = ei * r4.z * __uint_as_float(gr[e + 2]);
                        val[3] = ei * r4.w * __uint_as_float(gr[e + 3]);
                    } else {
                        const float4 c4 = *reinterpret_cast<const float4 *>(cum + j0 + e);
                        const float4 b4 = *reinterpret_cast<const float4 *>(bet + j0 + e);
                        val[0] = __expf(ci - c4.x) * __uint_as_float(gr[e]) * b4.x;
                        val[1] = __expf(ci - c4.y) * __uint_as_float(gr[e + 1]) * b4.y;
                        val[2] = __expf(ci - c4.z) * __uint_as_float(gr[e + 2]) * b4.z;
                        val[3] = __expf(ci - c4.w) * __uint_as_float(gr[e + 3]) * b4.w;
                    }
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const int j = j0 + e + m;
                        t[e + m] = t_rows ? (j < i ? val[m] : (j == i ? 1.f : 0.f)) : (j <= i ? val[m] : 0.f);
                    }
                }
                if (t_rows) {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        st4(Tb + xsw(i, (j0 >> 2) + c), t[4 * c], t[4 * c + 1], t[4 * c + 2], t[4 * c + 3]);
                } else {
#pragma unroll
                    for (int c = 0; c < 2; ++c)
                        *reinterpret_cast<uint4 *>(rec + R_P + swz(i, (j0 >> 3) + c)) = pack8(t + 8 * c);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        // ---- T^-1: the four 16 x 16 diagonal blocks (thread = block, column; forward substitution)
        if (tid < 64) {
            const int bi = tid >> 4, c = tid & 15, r0 = bi * 16;
            float x[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float tr[16];
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const float4 v = ld4(Tb + xsw(r0 + r, 4 * bi + q4));
                    tr[4 * q4] = v.x; tr[4 * q4 + 1] = v.y; tr[4 * q4 + 2] = v.z; tr[4 * q4 + 3] = v.w;
                }
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int k = 0; k < r; ++k) {
                    if (k & 1) s1 = fmaf(tr[k], x[k], s1);
                    else s0 = fmaf(tr[k], x[k], s0);
                }
                x[r] = r == c ? 1.f : (r < c ? 0.f : -(s0 + s1));
            }
#pragma unroll
            for (int r = 0; r < 16; ++r)
                *reinterpret_cast<float *>(Xb + xsw(r0 + r, (r0 + c) >> 2) + 4 * (c & 3)) = x[r];
        }
        __syncthreads();
        // ---- block levels d = 1, 2, 3: X[b, a] = -X[b, b] (T[b, a..b-1] X[a..b-1, a]), b = a + d.
        // Warps 2 blk, 2 blk + 1 take block (a, b) = (blk, blk + d); thread: row r, columns 4 cq .. + 3
        {
            const int blk = warp >> 1, r = ((warp & 1) << 3) + (lane >> 2), cq = lane & 3;
#pragma unroll
            for (int d = 1; d < 4; ++d) {
                if (blk < 4 - d) {
                    const int a_ = blk, b_ = blk + d;
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int t = 0; t < 4 * d; ++t) {  // 4 k per step, k = 16 a .. 16 b - 1
                        const int kq = 4 * a_ + t;
                        const float4 tv = ld4(Tb + xsw(16 * b_ + r, kq));
                        const float tr[4] = {tv.x, tv.y, tv.z, tv.w};
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            const float4 xv = ld4(Xb + xsw(4 * kq + m, 4 * a_ + cq));
                            acc[0] = fmaf(tr[m], xv.x, acc[0]); acc[1] = fmaf(tr[m], xv.y, acc[1]);
                            acc[2] = fmaf(tr[m], xv.z, acc[2]); acc[3] = fmaf(tr[m], xv.w, acc[3]);
                        }
                    }
                    *reinterpret_cast<float4 *>(RB + (blk * 16 + r) * RBS + 4 * cq) = make_float4(acc[0], acc[1], acc[2], acc[3]);
                }
                __syncthreads();
                if (blk < 4 - d) {
                    const int a_ = blk, b_ = blk + d;
                    const float *rb = RB + blk * 16 * RBS;
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int mq = 0; mq < 4; ++mq) {
                        const float4 xv = ld4(Xb + xsw(16 * b_ + r, 4 * b_ + mq));
                        const float xr[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            const float4 rv = *reinterpret_cast<const float4 *>(rb + (4 * mq + m) * RBS + 4 * cq);
                            acc[0] = fmaf(xr[m], rv.x, acc[0]); acc[1] = fmaf(xr[m], rv.y, acc[1]);
                            acc[2] = fmaf(xr[m], rv.z, acc[2]); acc[3] = fmaf(xr[m], rv.w, acc[3]);
                        }
                    }
                    st4(Xb + xsw(16 * b_ + r, 4 * a_ + cq), -acc[0], -acc[1], -acc[2], -acc[3]);
                }
                __syncthreads();
            }
        }
        // ---- T^-1 as bf16 hi + lo (K-major A tiles: row i, columns j; zero above the diagonal)
        {
            const int i = tid & 63, qq = tid >> 6;  // 16 columns per thread
            float xv[16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const float4 v = ld4(Xb + xsw(i, 4 * qq + q4));
                xv[4 * q4] = v.x; xv[4 * q4 + 1] = v.y; xv[4 * q4 + 2] = v.z; xv[4 * q4 + 3] = v.w;
            }
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float hi[8], lo[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int j = 16 * qq + 8 * c + e;
                    const float v = j <= i ? xv[8 * c + e] : 0.f;
                    const float hv = __bfloat162float(__float2bfloat16_rn(v));
                    hi[e] = hv;
                    lo[e] = v - hv;
                }
                *reinterpret_cast<uint4 *>(smem + P_TH + swz(i, 2 * qq + c)) = pack8(hi);
                *reinterpret_cast<uint4 *>(smem + P_TL + swz(i, 2 * qq + c)) = pack8(lo);
            }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- MMA UW: [U | W] = (T^-1 hi + T^-1 lo) [v | exp(cum) Phi]  (M = 64, N = 192, K = tokens)
        if (tid == 0) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t at = k < 4 ? P_TH : P_TL;
                mma_ss(tmem + PT_UW, dsc(at, HI_KMAJ) + (uint64_t)((k & 3) * 2),
                       dsc(P_V, HI_MNB) + (uint64_t)((k & 3) * 128), ID_UW, k > 0);
            }
            commit(bar);
        }
        w_ok = mbar_wait(bar, phase, ctl, 97);
        phase ^= 1;
        if (!__syncthreads_and(w_ok)) { ok = false; break; }
        tc_fence_after();
        // ---- U and W rows out: row i = 16 quad + lane sits in lane `lane` (< 16) of quadrant `quad`;
        // warps w < 4 take columns 0..95 (U, W features 0..31), warps w + 4 columns 96..191
        {
            const int quad = warp & 3, hc = warp >> 2;
            const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16) + PT_UW + 96 * hc;
            const int i = 16 * quad + lane;
            const bool rowl = lane < 16;
#pragma unroll
            for (int m = 0; m < 3; ++m) {
                float w[32];
                tmem_ld32(lb + 32 * m, w);
                const int col0 = 96 * hc + 32 * m;  // warp-uniform
                if (rowl) {
                    if (col0 < 64) {
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            st4(rec + R_U + xsw(i, (col0 >> 2) + c), w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                    } else {
                        const int f0 = col0 - 64;
                        uint8_t *dst = rec + (f0 < 64 ? R_A0 : R_A1);
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            *reinterpret_cast<uint4 *>(dst + swz(i, ((f0 & 63) >> 3) + c)) = pack8(w + 8 * c);
                    }
                }
            }
        }
        // no barrier here: the next unit's first barrier (after its staged rows land) orders these
        // tensor-memory reads before its GEMMs, and the gate scan before it touches nothing read here
        tc_fence_before();
    }

    cp_async_wait_all();  // no copy may still target this CTA's shared memory at exit
    if (!ok && tid == 0) {  // never free tensor memory under an MMA in flight
        const unsigned long long w0 = gtimer();
        while (!mbar_try(bar, phase ^ 1) && gtimer() - w0 < WAIT_NS) {
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PT_COLS) : "memory");
    if (tid == 0) report_fault(ctl_sh->abort_flag, p.fault);
}

// ---------------------------------------------------------------------------------------------
// Sequential kernel
// ---------------------------------------------------------------------------------------------
constexpr int QT = 320;                 // threads: warps 0-3 state, 4-5 E, 6-7 y, 8 copies, 9 MMAs
constexpr int S_A0 = 0;                 // stage: A1 (2 K-halves) | zeros | P' | Phic (2 halves) | U
constexpr int S_A1 = 16384;
constexpr int S_Z = 32768;
constexpr int S_P = 40960;
constexpr int S_PC = 49152;
constexpr int S_U = 65536;
constexpr int STG = 81920;
constexpr int Q_ST = 2 * STG;           // S^T bf16 [128 f][64 d], MN-major B of MMA 1
constexpr int Q_E = Q_ST + 16384;       // E bf16 [64 j][64 d], MN-major B of MMAs 2 and 3
constexpr int Q_RED = Q_E + 8192;       // [2][4] partial |S|^2, [2] chunk decays, [4] Lyapunov factors
constexpr int Q_BAR = Q_RED + 64;
constexpr int Q_SMEM = Q_BAR + 160;
constexpr size_t Q_SMEM_BYTES = Q_SMEM + 1024;
// B_MMA3: MMA 3 done (the state warps); B_MMA2x: MMA 2 done, one barrier per chunk parity, so that
// the y warps, which no other role waits for before the next chunk's MMA 2, can never see a phase of
// it complete twice.
// B_SC: the Lyapunov factor of the state entering the next chunk is in its slot.
enum {
    B_FULL0 = 0, B_FULL1, B_EMPTY0, B_EMPTY1, B_ST, B_MMA1, B_E, B_MMA3, B_MMA20, B_MMA21, B_YF0, B_YF1, B_SC,
    B_NEVER, NBAR
};
// tensor memory: D1 = [W ; Psie] S^T (two buffers), dS^T, D2 = [0 ; P'] E (two buffers)
constexpr uint32_t QT_D1 = 0, QT_DS = 128, QT_D2 = 256, QT_COLS = 512;

struct SeqArgs {
    DeltaParams p;
    int c0, ncw;
    const uint8_t *rec;
    const float *cd;
    const float *state_in;  // [BH][D][F] or nullptr
    float *state_out;       // [BH][D][F]
};

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}

// 32 consecutive outputs of a row in 16-byte stores
__device__ __forceinline__ void store_row32(float *dst, const float (&v)[32]) {
#pragma unroll
    for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4 *>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
}
__device__ __forceinline__ void store_row32(__nv_bfloat16 *dst, const float (&v)[32]) {
#pragma unroll
    for (int e = 0; e < 32; e += 8) *reinterpret_cast<uint4 *>(dst + e) = pack8(v + e);
}

template <typename TO>
__global__ void __launch_bounds__(QT, 1) delta_wy_seq_kernel(const SeqArgs a) {
    extern __shared__ uint8_t dsm_raw[];
    uint8_t *smem = smem_align1024(dsm_raw);
    const DeltaParams &p = a.p;
    uint64_t *const bar = reinterpret_cast<uint64_t *>(smem + Q_BAR);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(smem + Q_BAR + NBAR * 8);
    CtlShared *const ctl_sh = reinterpret_cast<CtlShared *>(smem + Q_BAR + NBAR * 8 + 8);
    float *const red = reinterpret_cast<float *>(smem + Q_RED);
    float *const cdv = red + 8;  // exp(cum_end) of chunks u (slot u % 2), from the E warps
    // Lyapunov factor of the state entering chunk u (slot u % 4): the state warps publish the state
    // tile before the projection, so MMA 1 sees the unscaled state and the E and y warps apply the
    // factor (W S^T and Psie S^T are linear in S)
    float *const scv = red + 12;
    const uint32_t sb = su32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x;
    const int U = a.ncw;
    const bool want_y = p.y.p != nullptr;
    Ctl ctl{ctl_sh, nullptr};

    if (tid == 0) {
        mbar_init(&bar[B_FULL0], 1);
        mbar_init(&bar[B_FULL1], 1);
        mbar_init(&bar[B_EMPTY0], 1);
        mbar_init(&bar[B_EMPTY1], 1);
        mbar_init(&bar[B_ST], 128);
        mbar_init(&bar[B_MMA1], 1);
        mbar_init(&bar[B_E], 64);
        mbar_init(&bar[B_MMA3], 1);
        mbar_init(&bar[B_MMA20], 1);
        mbar_init(&bar[B_MMA21], 1);
        mbar_init(&bar[B_YF0], 64);
        mbar_init(&bar[B_YF1], 64);
        mbar_init(&bar[B_SC], 1);
        mbar_init(&bar[B_NEVER], 1);
        init_ctl(*ctl_sh, p.fault);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(QT_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the zero rows 0..63 of MMA 2's A operand, in both stages
    for (int e = tid; e < 2 * 512; e += QT)
        reinterpret_cast<uint4 *>(smem + (e >> 9) * STG + S_Z)[e & 511] = make_uint4(0, 0, 0, 0);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (p.test_wait_ns) {  // test hook: a wait expires before any copy or MMA is issued
        if (tid == 0) expire_test_wait(&bar[B_NEVER], ctl, p.test_wait_ns, 98);
        __syncthreads();
        if (ctl.aborted()) {
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (warp == 0)
                asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QT_COLS)
                             : "memory");
            if (tid == 0) report_fault(ctl_sh->abort_flag, p.fault);
            return;
        }
    }
    const uint8_t *rec0 = a.rec + (size_t)bh * U * REC;
    const float *cd = a.cd + (size_t)bh * U;
    bool ok = true;

    if (warp == 8) {
        // ---- copies: record u into stage u % 2
        if (lane == 0) {
            int issued = 0;
            for (int u = 0; u < U; ++u) {
                const int s = u & 1;
                if (u >= 2 && !mbar_wait(&bar[B_EMPTY0 + s], ((u >> 1) - 1) & 1, ctl, 80)) { ok = false; break; }
                uint8_t *st = smem + s * STG;
                const uint8_t *rc = rec0 + (size_t)u * REC;
                mbar_expect_tx(&bar[B_FULL0 + s], (uint32_t)REC);
                bulk_g2s(st + S_A0, rc + R_A0, 32768, &bar[B_FULL0 + s]);
                bulk_g2s(st + S_P, rc + R_P, (uint32_t)(REC - R_P), &bar[B_FULL0 + s]);
                issued = u + 1;
            }
            // no copy may still target this CTA's shared memory at exit
            for (int u = max(issued - 2, 0); u < issued; ++u) {
                const unsigned long long w0 = gtimer();
                while (!mbar_try(&bar[B_FULL0 + (u & 1)], (u >> 1) & 1) && gtimer() - w0 < WAIT_NS) {
                }
            }
        }
    } else if (warp == 9) {
        // ---- MMA issue
        if (lane == 0) {
            constexpr uint64_t HI_A3 = desc_hi(8192, 1024, 2);   // MN-major A: Phic atoms
            constexpr uint64_t HI_KMAJ = desc_hi(16, 1024, 2);
            constexpr uint64_t HI_MN1 = desc_hi(16, 1024, 2);
            constexpr uint32_t ID_1 = idesc(128, 64, 0, 1), ID_2 = idesc(128, 64, 0, 1), ID_3 = idesc(128, 64, 1, 1);
            const uint32_t a0 = sb >> 4;
            auto dsc = [&](uint32_t off, uint64_t hi) { return (uint64_t)(a0 + (off >> 4)) | hi; };
            uint64_t *last = nullptr;  // barrier and parity of the latest commit
            uint32_t last_par = 0;
            for (int u = 0; u < U; ++u) {
                const int s = u & 1;
                const uint32_t so = (uint32_t)(s * STG), d1 = tmem + QT_D1 + 64 * (u & 1);
                if (!mbar_wait(&bar[B_FULL0 + s], (u >> 1) & 1, ctl, 81)) { ok = false; break; }
                if (!mbar_wait(&bar[B_ST], u & 1, ctl, 82)) { ok = false; break; }
                if (u >= 2 && !mbar_wait(&bar[B_YF0 + (u & 1)], ((u >> 1) - 1) & 1, ctl, 83)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    mma_ss(d1, dsc(so + (k < 4 ? S_A0 : S_A1), HI_KMAJ) + (uint64_t)((k & 3) * 2),
                           dsc(Q_ST, HI_MN1) + (uint64_t)(k * 128), ID_1, k > 0);
                commit(&bar[B_MMA1]);
                last = &bar[B_MMA1];
                last_par = u & 1;
                if (!mbar_wait(&bar[B_E], u & 1, ctl, 84)) { ok = false; break; }
                tc_fence_after();
                // MMA 3 first: the state update waits only for it
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_ss(tmem + QT_DS, dsc(so + S_PC, HI_A3) + (uint64_t)(k * 128), dsc(Q_E, HI_MN1) + (uint64_t)(k * 128),
                           ID_3, k > 0);
                commit(&bar[B_MMA3]);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_ss(tmem + QT_D2 + 64 * (u & 1), dsc(so + S_Z, HI_KMAJ) + (uint64_t)(k * 2),
                           dsc(Q_E, HI_MN1) + (uint64_t)(k * 128), ID_2, k > 0);
                commit(&bar[B_MMA20 + (u & 1)]);
                commit(&bar[B_EMPTY0 + s]);
                last = &bar[B_MMA20 + (u & 1)];
                last_par = (u >> 1) & 1;
            }
            if (!ok && last) {  // MMAs complete in order: the latest commit covers every one issued
                const unsigned long long w0 = gtimer();
                while (!mbar_try(last, last_par) && gtimer() - w0 < WAIT_NS) {
                }
            }
        }
    } else if (warp >= 4 && warp < 6) {
        // ---- E = U - W S^T (tensor-memory lanes 0..63 = token rows)
        const int i = tid - 128;
        const uint32_t lb = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        float cdn = (i == 0) ? cd[0] : 0.f;
        for (int u = 0; u < U; ++u) {
            const int s = u & 1;
            const float cdu = cdn;
            if (i == 0 && u + 1 < U) cdn = cd[u + 1];
            if (!mbar_wait(&bar[B_FULL0 + s], (u >> 1) & 1, ctl, 85)) { ok = false; break; }
            // this row of U while MMA 1 runs
            const uint8_t *ur = smem + s * STG + S_U;
            float uc[D];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float4 v = ld4(ur + xsw(i, c));
                uc[4 * c] = v.x; uc[4 * c + 1] = v.y; uc[4 * c + 2] = v.z; uc[4 * c + 3] = v.w;
            }
            if (!mbar_wait(&bar[B_MMA1], u & 1, ctl, 86)) { ok = false; break; }
            tc_fence_after();
            float w[32], sc = 1.f;
            bool have_sc = u == 0;
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
                tmem_ld32(lb + QT_D1 + 64 * (u & 1) + 32 * hc, w);
                if (!have_sc) {  // the factor of the state entering chunk u (projection of chunk u - 1)
                    if (!mbar_wait(&bar[B_SC], (u - 1) & 1, ctl, 90)) { ok = false; break; }
                    sc = scv[u & 3];
                    have_sc = true;
                }
#pragma unroll
                for (int e = 0; e < 32; ++e) w[e] = fmaf(-sc, w[e], uc[32 * hc + e]);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    *reinterpret_cast<uint4 *>(smem + Q_E + swz(i, 4 * hc + c)) = pack8(w + 8 * c);
            }
            if (!ok) break;
            if (i == 0) cdv[u & 1] = cdu;
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(&bar[B_E]);
        }
    } else if (warp >= 6 && warp < 8) {
        // ---- y rows (tensor-memory lanes 64..127)
        const int i = tid - 192;
        const uint32_t lb = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const int b = bh / p.H, h = bh - b * p.H;
        TO *yb = want_y ? reinterpret_cast<TO *>(p.y.p) + b * p.y.sb + h * p.y.sh : nullptr;
        for (int u = 0; u < U; ++u) {
            if (!mbar_wait(&bar[B_MMA20 + (u & 1)], (u >> 1) & 1, ctl, 87)) { ok = false; break; }
            tc_fence_after();
            const int t0 = (a.c0 + u) * C;
            const int n = min(C, p.L - t0);
            if (want_y) {
                // the factor of the state entering chunk u: written before the E warps' arrival that
                // MMA 2 waited for, and not rewritten before this chunk's y is out (slot u % 4)
                const float sc = u == 0 ? 1.f : scv[u & 3];
                float yv[32], y2[32];
#pragma unroll
                for (int hc = 0; hc < 2; ++hc) {
                    tmem_ld32(lb + QT_D1 + 64 * (u & 1) + 32 * hc, yv);
                    tmem_ld32(lb + QT_D2 + 64 * (u & 1) + 32 * hc, y2);
#pragma unroll
                    for (int e = 0; e < 32; ++e) yv[e] = fmaf(sc, yv[e], y2[e]);
                    if (i < n) store_row32(yb + (int64_t)(t0 + i) * p.y.sl + 32 * hc, yv);
                }
            }
            tc_fence_before();
            mbar_arrive(&bar[B_YF0 + (u & 1)]);
        }
    } else {
        // ---- the state: thread f owns row f of S^T (64 value columns) in registers
        const int f = tid;
        const uint32_t lb = tmem + ((uint32_t)(warp * 32) << 16);
        float S[D];
        const float *sin = a.state_in ? a.state_in + (size_t)bh * D * F : nullptr;
#pragma unroll
        for (int d = 0; d < D; ++d) S[d] = sin ? sin[(size_t)d * F + f] : 0.f;
        auto publish = [&]() {
            uint8_t *row = smem + Q_ST;
#pragma unroll
            for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4 *>(row + swz(f, c)) = pack8(S + 8 * c);
            fence_proxy_async();
            mbar_arrive(&bar[B_ST]);
        };
        publish();
        for (int u = 0; u < U; ++u) {
            if (!mbar_wait(&bar[B_MMA3], u & 1, ctl, 88)) { ok = false; break; }
            // the E warps wrote the chunk's decay before their arrival (a completed phase: no wait)
            if (!mbar_wait(&bar[B_E], u & 1, ctl, 89)) { ok = false; break; }
            tc_fence_after();
            const float cdu = cdv[u & 1];
            float ds[32];
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
                tmem_ld32(lb + QT_DS + 32 * hc, ds);
#pragma unroll
                for (int e = 0; e < 32; ++e) S[32 * hc + e] = fmaf(cdu, S[32 * hc + e], ds[e]);
            }
            tc_fence_before();
            if (u + 1 < U) publish();  // unscaled: the next MMA 1 starts before the projection
            float sc = 1.f;
            if (p.bound > 0.f) {
                float sq8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int d = 0; d < D; ++d) sq8[d & 7] = fmaf(S[d], S[d], sq8[d & 7]);
                float sq = ((sq8[0] + sq8[1]) + (sq8[2] + sq8[3])) + ((sq8[4] + sq8[5]) + (sq8[6] + sq8[7]));
                sq = warp_sum(sq);
                float *rd = red + 4 * (u & 1);
                if (lane == 0) rd[warp] = sq;
                named_bar(1, 128);
                const float4 r4 = *reinterpret_cast<const float4 *>(rd);
                const float tot = (r4.x + r4.y) + (r4.z + r4.w);
                sc = fminf(__fdividef(p.bound, sqrtf(tot) + 1e-6f), 1.0f);
                if (sc < 1.f) {
#pragma unroll
                    for (int d = 0; d < D; ++d) S[d] *= sc;
                }
            }
            if (f == 0 && u + 1 < U) {
                scv[(u + 1) & 3] = sc;
                mbar_arrive(&bar[B_SC]);
            }
        }
        if (ok && !ctl.aborted() && a.state_out) {
            float *so = a.state_out + (size_t)bh * D * F;
#pragma unroll
            for (int d = 0; d < D; ++d) so[(size_t)d * F + f] = S[d];
        }
    }
    (void)ok;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QT_COLS) : "memory");
    if (tid == 0) report_fault(ctl_sh->abort_flag, p.fault);
}

// Chunks per window: the records of one window stay within a byte budget.
constexpr size_t WINDOW_BYTES = size_t(1) << 30;

// Workspace of a window of w chunks (of nc): records, decays, and the state carried between
// windows when there are several.
inline size_t ws_bytes_for(int BH, int nc, int w) {
    const size_t recs = (size_t)BH * w * REC;
    const size_t cds = ((size_t)BH * w * sizeof(float) + 255) & ~size_t(255);
    const size_t carry = w < nc ? (size_t)BH * D * F * sizeof(float) : 0;
    return recs + cds + carry;
}

}  // namespace dwy

size_t delta_wy_workspace_bytes(int B, int H, int L) {
    using namespace dwy;
    if (B <= 0 || H <= 0 || L <= 0) return 0;
    const int BH = B * H, nc = (L + C - 1) / C;
    const size_t w = std::max<size_t>(1, std::min<size_t>((size_t)nc, WINDOW_BYTES / ((size_t)BH * REC)));
    return ws_bytes_for(BH, nc, (int)w);
}

// The largest window the given workspace holds (0: not even one chunk per head-state).
int delta_wy_window(int B, int H, int L, size_t ws_bytes) {
    using namespace dwy;
    if (B <= 0 || H <= 0 || L <= 0) return 0;
    const int BH = B * H, nc = (L + C - 1) / C;
    int w = (int)std::min<size_t>((size_t)nc, ws_bytes / ((size_t)BH * REC));
    while (w > 0 && ws_bytes_for(BH, nc, w) > ws_bytes) --w;
    return w;
}

template <typename TO>
static cudaError_t launch_wy_t(const DeltaParams &p, void *ws, int w, cudaStream_t st) {
    using namespace dwy;
    cudaError_t e = set_smem_once<delta_wy_prep_kernel<__nv_bfloat16>>((int)P_SMEM_BYTES);
    if (e != cudaSuccess) return e;
    e = set_smem_once<delta_wy_seq_kernel<TO>>((int)Q_SMEM_BYTES);
    if (e != cudaSuccess) return e;
    int dev = 0, nsm = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const int BH = p.B * p.H, nc = (p.L + C - 1) / C;
    uint8_t *rec = static_cast<uint8_t *>(ws);
    float *cd = reinterpret_cast<float *>(rec + (size_t)BH * w * REC);
    float *carry = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(cd) +
                                             (((size_t)BH * w * sizeof(float) + 255) & ~size_t(255)));
    // the state between windows: state_out when given, else the workspace copy
    float *mid = p.state_out ? p.state_out : carry;
    for (int c0 = 0; c0 < nc; c0 += w) {
        const int ncw = std::min(w, nc - c0);
        const bool last = c0 + ncw >= nc;
        PrepArgs pa{p, c0, ncw, rec, cd};
        const int units = BH * ncw;
        const int grid = std::min(units, 2 * nsm);
        delta_wy_prep_kernel<__nv_bfloat16><<<grid, PT, P_SMEM_BYTES, st>>>(pa);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        SeqArgs sa{p, c0, ncw, rec, cd, c0 == 0 ? p.state_in : mid, last ? p.state_out : mid};
        delta_wy_seq_kernel<TO><<<BH, QT, Q_SMEM_BYTES, st>>>(sa);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_delta_prefill_wy(const DeltaParams &p, int ydt, void *ws, int window, cudaStream_t st) {
    return ydt == PMA_F32 ? launch_wy_t<float>(p, ws, window, st) : launch_wy_t<__nv_bfloat16>(p, ws, window, st);
}

}  // namespace pma
