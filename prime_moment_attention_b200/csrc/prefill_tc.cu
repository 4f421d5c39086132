// prefill_tc.cu -- chunked prefill on tcgen05 tensor cores (bf16 inputs, D = 64).
//
// Same recurrence as chunked_prime_ssd_core (src/prime_moment_attention/chunked_ssd.py:48-184),
// evaluated per 128-token chunk (n <= 128 valid tokens) with the moment features
// psi(q) = [q | q^2/2], phi(k) = [k | k^2] (128 features) written as GEMMs whose
// operands carry the decay, so that the per-element work is one FMA:
//
//   g_i = l^(i+1)  (carry into token i)      w_j = l^(n-1-j)  (token j to chunk end; 0 if j >= n)
//   QQ  = [q | q^2/2]                         KW = [w.k | w.k^2]          (bf16 operands)
//   At  = QQ KW^T          = w_j a_ij,  a_ij = q_i.k_j + q_i^2.k_j^2/2   (M=N=128, K=128)
//   P   = l^-n At + l^-(1+j) = l^-(1+j) (1 + a_ij)  for j <= i, else 0   (= l^(i-j)(1+a_ij) / g_i)
//   ACC = QQ [S1 S2 | Z1 Z2]^T-blocks + P V   -> per row: carry numerator, carry denominator,
//                                               intra-chunk numerator    (chunked_ssd.py:93-94,139-148)
//   y_i = (ACC_i + S0) / max(cden_i + sum_j P_ij + Z0, eps / g_i)        (:149-157)
//   dS  = KW^T V,  dZ = column sums of KW,  dS0 = sum_j w_j v_j           (:96-111)
//   S   = l^n S + dS   (float32, in registers of the state warpgroup)     (:162-169)
// The rescaling keeps every factor inside float32/bf16 range for l >= 0.55
// (l^-128 < 2e33, l^127 > 1e-33); head-states with a smaller decay run the
// float32 CUDA-core chunk loop (prefill_simt_body.cuh) inside this kernel.
// Per-token decay (PT, the selective variant): with c_i the chunk's inclusive prefix sum of
// log lambda_t, the factors become g_i = exp(c_i), w_j = exp(c_{n-1} - c_j), l^-(1+j) -> exp(-c_j),
// l^-n -> exp(-c_{n-1}), l^n -> exp(c_{n-1}); every role that needs them scans the chunk's log
// decays itself (one warp scan, loaded a chunk ahead), so no new synchronisation is added.  A
// head-state any of whose chunks decays by more than e^-76 (0.55^128) runs the CUDA-core loop.
// k may carry a per-head temperature beta (KW = (w beta) k, K2W = (w beta^2) k^2) and the user
// states the selective layout (S2, Z2 halved).
//
// The kernel is bound by shared-memory bandwidth (128 B/clk per SM, shared by
// the tensor core's operand reads and every CUDA-core access), so the layout
// minimises shared-memory bytes per chunk:
//   * QQ lives in tensor memory (written by the prep warps with tcgen05.st) and
//     is the A operand of the score GEMM and of the carry GEMM (no smem reads);
//   * the decay weights w_j are folded into K (KW, written in place plus a new
//     K^2 tile); V stays as loaded and is the B operand of dS and P V;
//   * P is written back over the score accumulator and used from tensor memory;
//     dS then takes the other half of that accumulator;
//   * dZ, dS0 and the intra-chunk denominator sum_j P_ij are CUDA-core sums of
//     values already in registers; the carry denominator is column 64 of an
//     N=80 carry GEMM whose B operand [S1;S2 | Z] is a 32-byte-swizzled tile.
// Per chunk: 48 KB of TMA writes, 81 KB of prep traffic, 116 KB of operand reads,
// 20 KB of state tile writes.
//
// Data: q/k/v chunk tiles arrive by TMA (4-D tensor maps over the strided
// tensors, 128-byte swizzle) into three stages; the producer also prefetches
// later chunks into L2.  Tensor memory: At/P/dS x2 (256 columns), QQ x2 (128),
// ACC (80).
//
// Warp roles (512 threads, one CTA per SM):
//   warp 0        TMA producer
//   warp 1        MMA issuer (one thread, event driven: issues each chunk's GEMM
//                 groups as soon as their inputs are ready) and TMEM owner
//   warps 4-7     prep: QQ -> tensor memory, KW and K^2 W tiles, column sums
//   warps 8-11    mask: At -> P in tensor memory (warps 2-3 take part of quadrants 2-3)
//   warps 12-15   state: S += dS (thread f owns feature row f), bf16 state tile for the next
//                 chunk's carry GEMM, then the chunk's output rows (thread i owns token row i)
// Every wait is bounded by the global timer; on expiry the kernel records a status
// code in the workspace header, every role stops, and the CTA waits for its
// in-flight copies and GEMMs before freeing tensor memory.
#include <cuda.h>

#include "prefill.cuh"
#include "prefill_simt_body.cuh"
#define PMA_FAULT_AT_EXIT 1  // report expired waits once per CTA, after the final barrier
#include "tc_common.cuh"

namespace pma {
namespace tc {

constexpr int C = TC_CHUNK;   // tokens per chunk
constexpr int D = 64;
constexpr int TILE = C * D * 2;           // [128 x 64] bf16 = 16 KiB
constexpr int NST = 3;                    // stages of k (-> w.k), v, w.k^2
constexpr int STAGE = 3 * TILE;
constexpr int OFF_K = 0, OFF_V = TILE, OFF_K2 = 2 * TILE;
constexpr int OFF_Q = NST * STAGE;        // q slot: the prep warps read it first thing in a chunk and
                                          // then reload it with the next chunk's q
constexpr int OFF_YS = OFF_Q + TILE;      // y staging tile (bf16 output): a chunk's rows, one TMA store;
                                          // the per-token-decay variant uses it as a second q slot that
                                          // the producer fills with the stage (its prep runs longer)
constexpr int OFF_ONES = OFF_YS + TILE;   // 128 x 64 bf16, column 0 = 1: second N-atom of [V | 1]
constexpr int OFF_SB = OFF_ONES + TILE;   // [S1;S2 | Z] bf16, K = 128 features x N = 80, 32-byte swizzle
constexpr int SB_LBO = 4096;              // next 16-column group
constexpr int SB_SBO = 256;               // next 8-feature group
constexpr int OFF_SMALL = OFF_SB + 5 * SB_LBO;
constexpr int PREFETCH = 4;               // chunks of L2 prefetch ahead of the stage loads
constexpr float LMIN = 0.55f;             // smallest decay the rescaled operands serve
constexpr float LOGMIN = -76.0f;          // per-token decay: smallest chunk sum of log lambda served

enum {
    B_FULL0, B_FULL1, B_FULL2, B_EMPTY0, B_EMPTY1, B_EMPTY2, B_PREP0, B_PREP1, B_PREP2,
    B_IFULL0, B_IFULL1, B_PREADY0, B_PREADY1, B_DSFULL0, B_DSFULL1, B_DSFREE0, B_DSFREE1,
    B_QFREE0, B_QFREE1, B_CDONE0, B_CDONE1, B_SREADY0, B_SREADY1, B_OEMPTY, B_QEMPTY0, B_QEMPTY1, B_QFULL, B_MLD0, B_MLD1,
    B_MLD2, B_MLD3,
    B_FINAL, B_NEVER, NBAR
};

struct Small {
    uint64_t bar[NBAR];
    float pw[C + 4];              // l^t, t = 0..C
    float geo[C + 4];             // sum_{t<n} l^t
    alignas(16) float cinv[C];    // l^-(1+j)
    alignas(16) float part[NST][8][D];  // per stage and prep warp: column sums of w.v
    alignas(16) float s0f[3][D];  // S0 entering the chunk, by chunk mod 3
    float z0f[4];                 // Z0 entering the chunk, by chunk mod 3
    uint32_t tmem_base;
    CtlShared ctl;
    alignas(16) float cinv_pt[6][C];  // per-token decay: exp(-c_j) of the chunk, one row per mask warp
};
constexpr size_t SMEM_BYTES = OFF_SMALL + sizeof(Small) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
static_assert(SimtSmem<64, 64>::bytes <= OFF_SMALL, "fallback path fits in the same allocation");

// tensor-memory columns
// At / P / [dS | dZ]: buffer bb at bb * T_AS; At in columns 0..127, then P in 0..63 and [dS | dZ] in 64..143
constexpr uint32_t T_A = 0, T_AS = 144, T_QQ = 288, T_ACC = 416, T_COLS = 512;


template <typename TO>
__device__ __forceinline__ void store_row32(TO *dst, const float *v);
// 32 bytes in one store (the row's address 32-byte aligned)
__device__ __forceinline__ void st_global_v8(void *dst, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t a4,
                                             uint32_t a5, uint32_t a6, uint32_t a7) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(a0), "r"(a1), "r"(a2),
                 "r"(a3), "r"(a4), "r"(a5), "r"(a6), "r"(a7)
                 : "memory");
}
// A thread's row stores: 32-byte stores where the row allows, which halves the store instructions
// and the L1 requests of the scattered per-thread rows.
template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16 *dst, const float *v) {
    if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const float *w = v + 16 * c;
            st_global_v8(dst + 16 * c, pack2(w[0], w[1]), pack2(w[2], w[3]), pack2(w[4], w[5]), pack2(w[6], w[7]),
                         pack2(w[8], w[9]), pack2(w[10], w[11]), pack2(w[12], w[13]), pack2(w[14], w[15]));
        }
    } else {
        uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
        for (int c = 0; c < 4; ++c) d[c] = pack8(v + 8 * c);
    }
}
template <>
__device__ __forceinline__ void store_row32<float>(float *dst, const float *v) {
    if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float *w = v + 8 * c;
            st_global_v8(dst + 8 * c, __float_as_uint(w[0]), __float_as_uint(w[1]), __float_as_uint(w[2]),
                         __float_as_uint(w[3]), __float_as_uint(w[4]), __float_as_uint(w[5]), __float_as_uint(w[6]),
                         __float_as_uint(w[7]));
        }
    } else {
        float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
        for (int c = 0; c < 8; ++c) d[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
}

// ------------------------------------------------------------------ per-token decay helpers
// log decays of chunk tokens 4 lane .. 4 lane + 3 (zero past n); scalar loads (any alignment)
__device__ __forceinline__ float4 load_ld4(const float *ld, int t0, int n, int lane) {
    const int i = 4 * lane;
    return make_float4(i < n ? ld[t0 + i] : 0.f, i + 1 < n ? ld[t0 + i + 1] : 0.f, i + 2 < n ? ld[t0 + i + 2] : 0.f,
                       i + 3 < n ? ld[t0 + i + 3] : 0.f);
}

// Inclusive prefix sums of the chunk's log decays: lane l receives c[m] = c_{4l+m}; returns c_{n-1}
// (the chunk total: tokens past n add 0).  Whole warp.
__device__ __forceinline__ float chunk_cum(float4 x, int lane, float c[4]) {
    c[0] = x.x;
    c[1] = c[0] + x.y;
    c[2] = c[1] + x.z;
    c[3] = c[2] + x.w;
    float incl = c[3];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const float base = incl - c[3];
#pragma unroll
    for (int m = 0; m < 4; ++m) c[m] += base;
    return __shfl_sync(0xffffffffu, incl, 31);
}

// c_{4 src + m} held by lane src, selected by m (0..3)
__device__ __forceinline__ float cum_at(const float c[4], int src, int m) {
    const float v0 = __shfl_sync(0xffffffffu, c[0], src), v1 = __shfl_sync(0xffffffffu, c[1], src);
    const float v2 = __shfl_sync(0xffffffffu, c[2], src), v3 = __shfl_sync(0xffffffffu, c[3], src);
    return m == 0 ? v0 : (m == 1 ? v1 : (m == 2 ? v2 : v3));
}

// ------------------------------------------------------------------ the kernel
// SO: state only (no q, no output rows).  PRO: q scaled by p.pro.q_scale as the prep warps load it
// (the host uses this only when the scale is exact in bf16, so q * scale rounds as in float32;
// LayerNorm prologues run as a separate pass before this kernel).
template <bool SO, typename TO, bool PRO, bool PT>
__global__ void __launch_bounds__(512, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap ty,
                      const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    Small &sm = *reinterpret_cast<Small *>(smem + OFF_SMALL);
    constexpr int NPREP = SO ? 8 : 4;  // prep warps (4 + NPREP - 1 is the last)
    const uint32_t sb = su32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.x, seg = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int hk = h / p.pro.groups;  // GQA: kv head of query head h
    const float lam = PT ? 1.f : p.lambda[(int64_t)b * p.lam_sb + h];
    const float *ldh = PT ? p.logdecay + (size_t)bh * p.L : nullptr;  // per-token log decays

    bool small = !(lam >= LMIN);  // small decay (or NaN)
    if (PT) {  // any chunk whose decay leaves the rescaled range (or NaN)
        const int cb = seg * (p.seg_len / C), ce = min(cb + p.seg_len / C, (p.L + C - 1) / C);
        int bad = 0;
        for (int cc = cb + warp; cc < ce; cc += 16) {
            const int t0 = cc * C, nn = min(C, p.L - t0);
            float sum = 0.f;
            for (int i = lane; i < nn; i += 32) sum += ldh[t0 + i];
            sum = warp_sum(sum);
            bad |= !(sum >= LOGMIN);
        }
        small = __syncthreads_or(bad) != 0;
    }
    if (small) {  // float32 CUDA-core chunk loop, whole CTA
        simt_prefill_body<64, 64, __nv_bfloat16, TO, PT>(p, reinterpret_cast<float *>(smem), bh, seg);
        return;
    }

    const int nchunks_total = (p.L + C - 1) / C;
    const int seg_chunks = p.seg_len / C;
    const int c_begin = seg * seg_chunks;
    const int c_end = min(c_begin + seg_chunks, nchunks_total);
    const int U = c_end - c_begin;
    const int n_last = min(C, p.L - (c_end - 1) * C);
    const float kbeta = (PT && p.k_head_scale) ? p.k_head_scale[h] : 1.f;
    Ctl ctl{&sm.ctl, p.status};

    // ---- set-up: powers, barriers, tensor memory
    if (!PT && threadIdx.x <= C) {  // l^t, sum_{j<t} l^j (closed form, double) and l^-(1+t), t = 0..C
        const int t = threadIdx.x;
        const double lt = pow((double)lam, (double)t);
        sm.pw[t] = (float)lt;
        sm.geo[t] = (float)(lam == 1.0f ? (double)t : (1.0 - lt) / (1.0 - (double)lam));
        if (t < C) sm.cinv[t] = (float)(1.0 / (lt * (double)lam));
    }
    for (int i = threadIdx.x; i < TILE / 16; i += blockDim.x) {  // ones tile: row r = i / 8, chunk i % 8
        const int r = i >> 3, c = i & 7;
        const uint32_t one = (c == (r & 7)) ? 0x3F80u : 0u;  // element 0 of row r sits in chunk 0 ^ (r & 7)
        reinterpret_cast<uint4 *>(smem + OFF_ONES)[i] = make_uint4(one, 0u, 0u, 0u);
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; ++i) {
            uint32_t n = 1;
            if ((i >= B_PREP0 && i <= B_PREP2) || i == B_PREADY0 || i == B_PREADY1 || i == B_DSFREE0 ||
                i == B_DSFREE1 || i == B_SREADY0 || i == B_SREADY1 || i == B_OEMPTY || i == B_QEMPTY0 ||
                i == B_QEMPTY1)
                n = 128;
            if (SO && i >= B_PREP0 && i <= B_PREP2) n = 32 * NPREP;
            if (i >= B_EMPTY0 && i <= B_EMPTY2) n = 2 + 128;  // two GEMM-group commits + the state warpgroup
            if (i == B_PREADY0 || i == B_PREADY1) n = 128 + 64;  // mask warps 8-11 + helpers 2-3
            if (i >= B_MLD0 && i <= B_MLD3) n = 32;              // one mask warp
            mbar_init(&sm.bar[i], n);
        }
        init_ctl(sm.ctl, p.fault);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sm.tmem_base)),
                     "r"(T_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    fence_proxy_async();  // the ones tile is read by the tensor core
    __syncthreads();
    const uint32_t tmem = sm.tmem_base;
    uint64_t *bar = sm.bar;
    if (p.test_wait_ns) {  // test hook: a wait expires before any copy or GEMM is issued
        if (threadIdx.x == 0) expire_test_wait(&bar[B_NEVER], ctl, p.test_wait_ns, 90);
        __syncthreads();
        if (ctl.aborted()) {  // the whole CTA: nothing was issued, release tensor memory and leave
            if (warp == 1)
                asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T_COLS)
                             : "memory");
            if (threadIdx.x == 0) report_fault(sm.ctl.abort_flag, p.fault);
            return;
        }
    }

    if (warp == 0) {
        // ============================== TMA producer
        if (lane == 0) {
            int issued = 0, fetched = 0;
            for (int u = 0, s = 0; u < U; ++u, s = (s == NST - 1) ? 0 : s + 1) {
                for (; fetched < U && fetched <= u + PREFETCH; ++fetched) {
                    const int tf = (c_begin + fetched) * C;
                    if (!SO) tma_prefetch_l2(&tq, 0, tf, h, b);
                    tma_prefetch_l2(&tk, 0, tf, hk, b);
                    tma_prefetch_l2(&tv, 0, tf, hk, b);
                }
                if (!mbar_wait(&bar[B_EMPTY0 + s], ((u / NST) & 1) ^ 1, ctl, 1)) break;
                constexpr bool QSTAGE = PT && !SO;  // q of this variant rides with the stage (two slots)
                if (QSTAGE && !mbar_wait(&bar[B_QEMPTY0 + (u & 1)], ((u >> 1) & 1) ^ 1, ctl, 3)) break;
                const int t0 = (c_begin + u) * C;
                uint8_t *base = smem + s * STAGE;
                mbar_expect_tx(&bar[B_FULL0 + s], QSTAGE ? 3 * TILE : 2 * TILE);
                if (QSTAGE) tma_load(smem + OFF_Q + (u & 1) * TILE, &tq, &bar[B_FULL0 + s], 0, t0, h, b);
                tma_load(base + OFF_K, &tk, &bar[B_FULL0 + s], 0, t0, hk, b);
                tma_load(base + OFF_V, &tv, &bar[B_FULL0 + s], 0, t0, hk, b);
                issued = u + 1;
            }
            // never leave with copies in flight: the last (up to) NST stages must have landed
            for (int u = max(0, issued - NST); u < issued; ++u) {
                const unsigned long long t0 = gtimer();
                while (!mbar_try(&bar[B_FULL0 + u % NST], (u / NST) & 1) && gtimer() - t0 < WAIT_NS) {
                }
            }
        }
    } else if (warp == 1) {
        // ============================== MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_A = idesc(128, 128, 0, 0);   // QQ (tmem) KW^T
            constexpr uint32_t ID_DS = idesc(128, 80, 1, 1);   // KW^T [V | 1]
            constexpr uint32_t ID_CY = idesc(128, 80, 0, 1);   // QQ (tmem) [S1;S2 | Z]
            constexpr uint32_t ID_PV = idesc(128, 80, 0, 1);   // P (tmem) [V | 1]
            // Operand descriptors: a compile-time upper word (strides, version, swizzle) or'ed with the
            // start-address field, which is the smem base (16-byte units) plus constant offsets; only
            // that one 32-bit base stays live across the loop.
            const uint32_t a0 = sb >> 4;  // the whole allocation sits below 256 KiB: no field overflow
            constexpr uint64_t HI_KMAJ = desc_hi(16, 1024, 2), HI_KMN = desc_hi(OFF_K2 - OFF_K, 1024, 2),
                               HI_SB = desc_hi(SB_LBO, SB_SBO, 6);
            auto dsc = [&](uint32_t byte_off, uint64_t hi) { return (uint64_t)(a0 + (byte_off >> 4)) | hi; };
            // [V | 1] of stage s: the second N-atom is the shared ones tile, LBO = its distance from V
            auto dvo = [&](int s) {
                const uint32_t off = (uint32_t)(s * STAGE + OFF_V);
                return dsc(off, desc_hi(OFF_ONES - off, 1024, 2));
            };
            auto kmaj = [](int k) { return (uint64_t)((k & 3) * 2); };  // +32 B in a 128 B row
            auto mnmaj = [](int k) { return (uint64_t)(k * 128); };     // +16 rows of 128 B
            // Static issue order with blocking waits: G1(0), then per chunk u
            //   [dS(u)], [score(u+1)], [carry(u)], [P V(u)]
            // so that the tensor pipe always has the next group queued: the score GEMM of u+1 needs
            // P V(u-1) complete (its accumulator columns), which finished while dS(u) ran; the carry
            // GEMM of u needs the outputs of u-1 read, which happens while dS(u) and score(u+1) run.
            // Every wait below depends only on groups issued earlier, so the order cannot deadlock.
            auto g1 = [&](int u) -> bool {  // At = QQ KW^T into At[u & 1]
                const int bb = u & 1, st = u % NST, ph = (u >> 1) & 1;
                if (!mbar_wait(&bar[B_PREP0 + st], (u / NST) & 1, ctl, 20) ||
                    !mbar_wait(&bar[B_CDONE0 + bb], ph ^ 1, ctl, 21) || !mbar_wait(&bar[B_DSFREE0 + bb], ph ^ 1, ctl, 22))
                    return false;
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    mma_ts(tmem + T_A + bb * T_AS, tmem + T_QQ + bb * 64 + k * 8,
                           dsc(st * STAGE + (k < 4 ? OFF_K : OFF_K2), HI_KMAJ) + kmaj(k), ID_A, k > 0);
                commit(&bar[B_IFULL0 + bb]);
                return true;
            };
            auto g2a = [&](int u) -> bool {  // [dS | dZ] = KW^T [V | 1], into the At columns P does not use
                const int bb = u & 1, st = u % NST, ph = (u >> 1) & 1;
                if (SO) {
                    if (!mbar_wait(&bar[B_PREP0 + st], (u / NST) & 1, ctl, 23) ||
                        !mbar_wait(&bar[B_DSFREE0 + bb], ph ^ 1, ctl, 22))
                        return false;
                } else if (!mbar_wait(&bar[B_PREADY0 + bb], ph, ctl, 24)) {
                    return false;
                }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k)  // K-dim = tokens, 16 rows = 2048 B per step
                    mma_ss(tmem + T_A + bb * T_AS + 64, dsc(st * STAGE + OFF_K, HI_KMN) + mnmaj(k),
                           dvo(st) + mnmaj(k), ID_DS, k > 0);
                commit(&bar[B_DSFULL0 + bb]);
                commit(&bar[B_EMPTY0 + st]);
                if (SO) {  // no carry / P V groups: they would make these arrivals
                    commit(&bar[B_QFREE0 + bb]);
                    commit(&bar[B_EMPTY0 + st]);
                }
                return true;
            };
            auto g2b = [&](int u) -> bool {  // carry GEMM with the state entering chunk u: ACC = QQ [S1;S2 | Z]
                const int bb = u & 1;
                if (!mbar_wait(&bar[B_SREADY0 + bb], (u >> 1) & 1, ctl, 25) ||
                    !mbar_wait(&bar[B_OEMPTY], (u & 1) ^ 1, ctl, 26))
                    return false;
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 8; ++k)  // K-dim = features, 16 per step = 2 groups of 256 B
                    mma_ts(tmem + T_ACC, tmem + T_QQ + bb * 64 + k * 8, dsc(OFF_SB + k * 512, HI_SB), ID_CY, k > 0);
                commit(&bar[B_QFREE0 + bb]);
                return true;
            };
            auto g4 = [&](int u) {  // ACC += P [V | 1] (P from tensor memory; column 64 collects the row sums)
                const int bb = u & 1, st = u % NST;
#pragma unroll
                for (int k = 0; k < 8; ++k)  // K-dim = tokens; P packs 2 per column
                    mma_ts(tmem + T_ACC, tmem + T_A + bb * T_AS + k * 8, dvo(st) + mnmaj(k), ID_PV, 1);
                commit(&bar[B_CDONE0 + bb]);
                commit(&bar[B_EMPTY0 + st]);
            };
            if (SO) {
                for (int u = 0; u < U; ++u)
                    if (!g2a(u)) break;
            } else if (g1(0)) {
                for (int u = 0; u < U; ++u) {
                    if (!g2a(u)) break;
                    if (u + 1 < U && !g1(u + 1)) break;
                    if (!g2b(u)) break;
                    g4(u);  // its P was waited for by dS(u)
                }
            }
            // every GEMM issued must be complete before tensor memory is released
            commit(&bar[B_FINAL]);
            const unsigned long long t0 = gtimer();
            while (!mbar_try(&bar[B_FINAL], 0) && gtimer() - t0 < WAIT_NS) {
            }
        }
    } else if (warp >= 4 && warp < 4 + NPREP) {
        // ============================== prep: QQ -> tensor memory, KW / K2W tiles, column sums of w.v
        // (the state-only pass has no mask work, so warps 8-11 join the prep warps there)
        const int tid = threadIdx.x - 128;
        const int wp = warp - 4;
        const int cc = lane & 7;  // K/V tiles: the thread's 16-byte column chunk
        const int q_base = SO ? 4 * wp : (wp == 0 ? 0 : (wp == 1 ? 12 : (wp == 2 ? 20 : 28)));  // first row quad
        const int nq_pass = SO ? 1 : (wp == 0 ? 3 : (wp == 3 ? 1 : 2));                       // quads per thread
        const uint32_t lane_base = tmem + ((uint32_t)(wp * 32) << 16);
        float4 ld_next = make_float4(0.f, 0.f, 0.f, 0.f);
        if (PT && U > 0) ld_next = load_ld4(ldh, c_begin * C, U == 1 ? n_last : C, lane);
        // the q slot: thread 0 of the prep warps loads chunk 0's q now and each next chunk's q once
        // every prep thread has read the current one (L2-prefetched by the producer)
        const bool q_loader = !SO && !PT && tid == 0;
        int q_issued = 0;
        if (q_loader && U > 0) {
            mbar_expect_tx(&bar[B_QFULL], TILE);
            tma_load(smem + OFF_Q, &tq, &bar[B_QFULL], 0, c_begin * C, h, b);
            q_issued = 1;
        }
        for (int u = 0, s = 0; u < U; ++u, s = (s == NST - 1) ? 0 : s + 1) {
            const int bb = u & 1;
            const int n = (u == U - 1) ? n_last : C;
            float cpre[4], cend = 0.f;
            if (PT) {  // this chunk's prefix sums; the next chunk's log decays are loaded now
                const float4 x = ld_next;
                if (u + 1 < U) ld_next = load_ld4(ldh, (c_begin + u + 1) * C, (u + 1 == U - 1) ? n_last : C, lane);
                cend = chunk_cum(x, lane, cpre);
            }
            if (!mbar_wait(&bar[B_FULL0 + s], (u / NST) & 1, ctl, 7)) break;
            uint8_t *k_s = smem + s * STAGE + OFF_K, *v_s = smem + s * STAGE + OFF_V, *k2_s = smem + s * STAGE + OFF_K2;
            uint4 xq[8];  // row tid of q, kept in registers until its tensor-memory buffer is free
            if (!SO && PT) {  // two slots, filled by the producer with the stage
                const uint8_t *q_s = smem + OFF_Q + bb * TILE;
#pragma unroll
                for (int c = 0; c < 8; ++c) xq[c] = *reinterpret_cast<const uint4 *>(q_s + swz(tid, c));
                mbar_arrive_after_reads(&bar[B_QEMPTY0 + bb]);  // the q slot may be reloaded
            } else if (!SO) {
                if (!mbar_wait(&bar[B_QFULL], u & 1, ctl, 4)) break;
                const uint8_t *q_s = smem + OFF_Q;
#pragma unroll
                for (int c = 0; c < 8; ++c) xq[c] = *reinterpret_cast<const uint4 *>(q_s + swz(tid, c));
                mbar_arrive_after_reads(&bar[B_QEMPTY0]);  // the q slot may be reloaded
                if (q_loader && u + 1 < U) {
                    if (!mbar_wait(&bar[B_QEMPTY0], u & 1, ctl, 3)) break;
                    mbar_expect_tx(&bar[B_QFULL], TILE);
                    tma_load(smem + OFF_Q, &tq, &bar[B_QFULL], 0, (c_begin + u + 1) * C, h, b);
                    q_issued = u + 2;
                }
            }
            // KW = w.k in place and K2W = KW.k (packed bf16 products), and the column sums of w.v
            // (float32).  Items of 4 rows x one 16-byte column chunk; the row quads are split
            // unevenly over the warps (12/8/8/4 of 32) so that sub-partition 3, which also runs the
            // longest mask rows, gets the least.
            float2 s0p[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) s0p[c] = make_float2(0.f, 0.f);
#pragma unroll 1
            for (int m = 0; m < nq_pass; ++m) {
                const int r0 = (q_base + (lane >> 3) + 4 * m) * 4;
                // row t of the quad is r0 + ((t + lane/8) & 3): the four 8-lane groups of one
                // access then hit rows with four different swizzle phases (no bank conflicts)
                const int rg = lane >> 3;
                float wr[4];
                if (PT) {
                    const int src = r0 >> 2;  // lane holding c of rows r0 .. r0 + 3
                    const float v0 = __shfl_sync(0xffffffffu, cpre[0], src), v1 = __shfl_sync(0xffffffffu, cpre[1], src);
                    const float v2 = __shfl_sync(0xffffffffu, cpre[2], src), v3 = __shfl_sync(0xffffffffu, cpre[3], src);
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const int mq = (t + rg) & 3;
                        const float cv = mq == 0 ? v0 : (mq == 1 ? v1 : (mq == 2 ? v2 : v3));
                        wr[t] = r0 + mq < n ? __expf(cend - cv) : 0.f;
                    }
                } else {
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const int r = r0 + ((t + rg) & 3);
                        wr[t] = r < n ? sm.pw[n - 1 - r] : 0.f;
                    }
                }
                uint4 x[4], y[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    x[t] = *reinterpret_cast<const uint4 *>(k_s + swz(r0 + ((t + rg) & 3), cc));
                    y[t] = *reinterpret_cast<const uint4 *>(v_s + swz(r0 + ((t + rg) & 3), cc));
                }
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t e4[4] = {x[t].x, x[t].y, x[t].z, x[t].w};
                    const uint32_t v4[4] = {y[t].x, y[t].y, y[t].z, y[t].w};
                    const float2 w2 = make_float2(wr[t], wr[t]);
                    uint32_t o1[4], o2[4];
                    if (PT) {  // KW = (w beta) k, K2W = (w beta^2) k^2
                        const __nv_bfloat162 wb1 = __float2bfloat162_rn(wr[t] * kbeta);
                        const __nv_bfloat162 wb2 = __float2bfloat162_rn(wr[t] * kbeta * kbeta);
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const __nv_bfloat162 kv = as_b2(e4[c]);
                            o1[c] = as_u(__hmul2(kv, wb1));
                            o2[c] = as_u(__hmul2(__hmul2(kv, kv), wb2));
                            s0p[c] = __ffma2_rn(bf2f(v4[c]), w2, s0p[c]);
                        }
                    } else {
                        const __nv_bfloat162 wb = __float2bfloat162_rn(wr[t]);
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const __nv_bfloat162 kv = as_b2(e4[c]);
                            const __nv_bfloat162 kw = __hmul2(kv, wb);
                            o1[c] = as_u(kw);
                            o2[c] = as_u(__hmul2(kw, kv));
                            s0p[c] = __ffma2_rn(bf2f(v4[c]), w2, s0p[c]);
                        }
                    }
                    const uint32_t off = swz(r0 + ((t + rg) & 3), cc);
                    *reinterpret_cast<uint4 *>(k_s + off) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
                    *reinterpret_cast<uint4 *>(k2_s + off) = make_uint4(o2[0], o2[1], o2[2], o2[3]);
                }
            }
            // lanes cc, cc+8, cc+16, cc+24 of this warp share the column chunk
#pragma unroll
            for (int m = 8; m <= 16; m <<= 1) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    s0p[c] = __fadd2_rn(s0p[c], make_float2(__shfl_xor_sync(0xffffffffu, s0p[c].x, m),
                                                            __shfl_xor_sync(0xffffffffu, s0p[c].y, m)));
            }
            if (lane < 8) {
                float4 *pp = reinterpret_cast<float4 *>(sm.part[s][wp]) + cc * 2;
                pp[0] = make_float4(s0p[0].x, s0p[0].y, s0p[1].x, s0p[1].y);
                pp[1] = make_float4(s0p[2].x, s0p[2].y, s0p[3].x, s0p[3].y);
            }
            if (PRO && !SO) {  // q * scale in bf16 (exact scale: one rounding, as in float32)
                const __nv_bfloat162 sc = __float2bfloat162_rn(p.pro.q_scale);
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    xq[c] = make_uint4(as_u(__hmul2(as_b2(xq[c].x), sc)), as_u(__hmul2(as_b2(xq[c].y), sc)),
                                       as_u(__hmul2(as_b2(xq[c].z), sc)), as_u(__hmul2(as_b2(xq[c].w), sc)));
            }
            // QQ row tid: [q | q^2/2], 2 bf16 per tensor-memory column, once the carry GEMM of chunk
            // u-2 has finished reading this buffer
            if (!mbar_wait(&bar[B_QFREE0 + bb], ((u >> 1) & 1) ^ 1, ctl, 8)) break;
            if (!SO) {
                const __nv_bfloat162 half2 = __float2bfloat162_rn(0.5f);
                uint32_t r[16];
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 v = xq[4 * hh + c];
                        r[4 * c + 0] = v.x; r[4 * c + 1] = v.y; r[4 * c + 2] = v.z; r[4 * c + 3] = v.w;
                    }
                    tmem_st16(lane_base + T_QQ + bb * 64 + 16 * hh, r);
                }
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 v = xq[4 * hh + c];
                        const uint32_t e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const __nv_bfloat162 qv = as_b2(e[t]);
                            r[4 * c + t] = as_u(__hmul2(qv, __hmul2(qv, half2)));  // q*(q/2): one rounding
                        }
                    }
                    tmem_st16(lane_base + T_QQ + bb * 64 + 32 + 16 * hh, r);
                }
                tmem_wait_st();
            }
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(&bar[B_PREP0 + s]);
        }
        // no copy may still target this CTA's shared memory at exit: the last q load issued
        if (q_loader && q_issued > 0) {
            const unsigned long long w0 = gtimer();
            while (!mbar_try(&bar[B_QFULL], (q_issued - 1) & 1) && gtimer() - w0 < WAIT_NS) {
            }
        }
    } else if (!SO && ((warp >= 8 && warp < 12) || warp == 2 || warp == 3)) {
        // ============================== mask: At -> P
        // TMEM lane quadrant q = warp % 4 holds rows 32q..32q+31, whose P has 2q+2 nonzero 16-column
        // blocks.  Warps 8-11 own the quadrants; warps 2 and 3 take the upper half of the blocks of
        // quadrants 2 and 3.  P of block b (At columns 16b..16b+15) goes to columns 8b..8b+7, which
        // only this quadrant reads: a helper stores after the owner has its At blocks in registers.
        if (!SO) {
            const int wq = warp & 3;
            const bool helper = warp < 4;  // this thread's P row is wq * 32 + lane
            const uint32_t lane_base = tmem + ((uint32_t)(wq * 32) << 16);
            const int nq = 2 * wq + 2;                                   // nonzero blocks of the quadrant
            const int split = wq == 2 ? 3 : (wq == 3 ? 4 : nq);          // first block of the helper
            const int b0 = helper ? split : 0, nb = helper ? nq - split : split;
            const int zero_from = (wq == 2) ? (helper ? 48 : 64) : (wq < 2 ? 16 * wq + 16 : 64);
            uint64_t *mld = &bar[B_MLD0 + 2 * (wq - 2)];                 // quadrants 2, 3: [chunk parity]
            float *const cwarp = sm.cinv_pt[helper ? 4 + (warp - 2) : warp - 8];  // per-token decay: this warp's
            float4 ld_next = make_float4(0.f, 0.f, 0.f, 0.f);
            if (PT && U > 0) ld_next = load_ld4(ldh, c_begin * C, U == 1 ? n_last : C, lane);
            auto mask = [&](int u) -> bool {
                const int bb = u & 1;
                const int n = (u == U - 1) ? n_last : C;
                float cn;
                if (PT) {  // exp(-c_j) for the chunk's columns, into this warp's row of cinv_pt
                    const float4 x = ld_next;
                    if (u + 1 < U) ld_next = load_ld4(ldh, (c_begin + u + 1) * C, (u + 1 == U - 1) ? n_last : C, lane);
                    float cc[4];
                    const float cend = chunk_cum(x, lane, cc);
                    *reinterpret_cast<float4 *>(cwarp + 4 * lane) =
                        make_float4(__expf(-cc[0]), __expf(-cc[1]), __expf(-cc[2]), __expf(-cc[3]));
                    __syncwarp();
                    cn = __expf(-cend);
                } else {
                    cn = 1.0f / sm.pw[n];  // l^-n
                }
                const float2 cn2 = make_float2(cn, cn);
                if (!mbar_wait(&bar[B_IFULL0 + bb], (u >> 1) & 1, ctl, 9)) return false;
                tc_fence_after();
                const uint32_t abase = lane_base + T_A + bb * T_AS;
                uint32_t ra[4][16];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < nb) tmem_ld16_issue(abase + 16 * (b0 + j), ra[j]);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < nb) tmem_wait_ld_regs(ra[j]);
                if (split < nq) {
                    if (!helper) {
                        tc_fence_before();
                        mbar_arrive(&mld[bb]);  // this warp's At columns are in registers
                    } else if (!mbar_wait(&mld[bb], (u >> 1) & 1, ctl, 10)) {
                        return false;
                    } else {
                        tc_fence_after();
                    }
                }
                if (zero_from < 64) {  // P columns right of the diagonal block: zero for every row here
                    uint32_t z[16];
#pragma unroll
                    for (int c = 0; c < 16; ++c) z[c] = 0u;
#pragma unroll 1
                    for (int c0 = zero_from; c0 < 64; c0 += 16) tmem_st16(abase + c0, z);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < nb) {
                        const int bk = b0 + j;
                        const float4 *cv = reinterpret_cast<const float4 *>((PT ? cwarp : sm.cinv) + 16 * bk);
                        const int lim = lane - 16 * (bk - 2 * wq);  // column 16bk + c belongs to row i iff c <= lim
                        uint32_t pk[8];
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            const float4 cj = cv[c4];
                            float2 lo = __ffma2_rn(
                                cn2, make_float2(__uint_as_float(ra[j][4 * c4]), __uint_as_float(ra[j][4 * c4 + 1])),
                                make_float2(cj.x, cj.y));
                            float2 hi = __ffma2_rn(
                                cn2,
                                make_float2(__uint_as_float(ra[j][4 * c4 + 2]), __uint_as_float(ra[j][4 * c4 + 3])),
                                make_float2(cj.z, cj.w));
                            lo.x = 4 * c4 <= lim ? lo.x : 0.f;
                            lo.y = 4 * c4 + 1 <= lim ? lo.y : 0.f;
                            hi.x = 4 * c4 + 2 <= lim ? hi.x : 0.f;
                            hi.y = 4 * c4 + 3 <= lim ? hi.y : 0.f;
                            pk[2 * c4] = f2bf(lo);
                            pk[2 * c4 + 1] = f2bf(hi);
                        }
                        tmem_st8(abase + 8 * bk, pk);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bar[B_PREADY0 + bb]);
                if (PT) __syncwarp();  // every lane has read cwarp before the next chunk rewrites it
                return true;
            };
            for (int u = 0; u < U; ++u)
                if (!mask(u)) break;
        }
    } else if (warp >= 12) {
        // ============================== state: S += dS, bf16 state tile for the carry GEMM
        const int wq = warp - 12;
        const int f = wq * 32 + lane;  // feature row: f < 64 -> S1 row f, else S2 row f - 64
        // bf16 rows leave through the staging tile and a TMA store per chunk (warp-uniform).  The
        // per-token-decay variant keeps its own row stores: the staging path costs it registers.
        const bool use_tma_y = !SO && !PT && sizeof(TO) == 2 && p.y_tma != 0;
        const uint32_t lane_base = tmem + ((uint32_t)(wq * 32) << 16);
        float S[D];
        float Z, s0 = 0.f, Z0;
        const bool has_in = !p.state_only && p.in.present();
        if (has_in) {
            const HeadPtrs src = p.in.at(bh, p.in.packed ? seg : 0, D);
            const float *row = f < D ? src.S1 + f * D : src.S2 + (f - D) * D;
            if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
#pragma unroll
                for (int e = 0; e < D; e += 4) {
                    const float4 t = *reinterpret_cast<const float4 *>(row + e);
                    S[e] = t.x; S[e + 1] = t.y; S[e + 2] = t.z; S[e + 3] = t.w;
                }
            } else {
#pragma unroll
                for (int e = 0; e < D; ++e) S[e] = row[e];
            }
            Z = f < D ? src.Z1[f] : src.Z2[f - D];
            if (PT && p.half_sq && f >= D && !p.in.packed) {  // selective layout: S2, Z2 held halved
#pragma unroll
                for (int e = 0; e < D; ++e) S[e] *= 2.f;
                Z *= 2.f;
            }
            if (f < D) s0 = src.S0[f];
            Z0 = src.Z0[0];
        } else {
#pragma unroll
            for (int e = 0; e < D; ++e) S[e] = 0.f;
            Z = 0.f;
            Z0 = 0.f;
        }
        // [S1;S2 | Z] row f (K index f) in the 32-byte-swizzled MN-major tile; S0 / Z0 by chunk mod 3
        auto publish = [&](int v) {
            uint8_t *base = smem + OFF_SB + (f >> 3) * SB_SBO + (f & 7) * 32;
            const uint32_t sw = (uint32_t)((f >> 2) & 1);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                *reinterpret_cast<uint4 *>(base + g * SB_LBO + ((0u ^ sw) << 4)) = pack8(S + 16 * g);
                *reinterpret_cast<uint4 *>(base + g * SB_LBO + ((1u ^ sw) << 4)) = pack8(S + 16 * g + 8);
            }
            *reinterpret_cast<uint4 *>(base + 4 * SB_LBO + ((0u ^ sw) << 4)) = make_uint4(pack2(Z, 0.f), 0u, 0u, 0u);
            *reinterpret_cast<uint4 *>(base + 4 * SB_LBO + ((1u ^ sw) << 4)) = make_uint4(0u, 0u, 0u, 0u);
            if (f < D) sm.s0f[v % 3][f] = s0;
            if (f == 0) sm.z0f[v % 3] = Z0;
            fence_proxy_async();
            mbar_arrive(&bar[B_SREADY0 + (v & 1)]);
        };
        if (!SO && U > 0) publish(0);
        bool ok = true;
        for (int u = 0, s = 0; u < U && ok; ++u, s = (s == NST - 1) ? 0 : s + 1) {
            const int bb = u & 1;
            const int n = (u == U - 1) ? n_last : C;
            float decay = 0.f, zinc = 0.f, grow = 0.f;  // l^n, sum_j w_j, (PT) this output row's c
            if (PT) {  // the log decays' load latency hides behind the waits below
                const float4 x = load_ld4(ldh, (c_begin + u) * C, n, lane);
                float cc[4];
                const float cend = chunk_cum(x, lane, cc);
                decay = __expf(cend);
                float zs = 0.f;
#pragma unroll
                for (int m = 0; m < 4; ++m) zs += 4 * lane + m < n ? __expf(cend - cc[m]) : 0.f;
                zinc = warp_sum(zs);
                grow = cum_at(cc, f >> 2, f & 3);
            }
            if (!mbar_wait(&bar[B_PREP0 + s], (u / NST) & 1, ctl, 11) ||
                !mbar_wait(&bar[B_DSFULL0 + bb], (u >> 1) & 1, ctl, 12)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (!PT) decay = sm.pw[n];
            const float2 dec2 = make_float2(decay, decay);
            float ds0 = 0.f;
            if (f < D) {
#pragma unroll
                for (int w = 0; w < NPREP; ++w) ds0 += sm.part[s][w][f];
            }
            const uint32_t dbase = lane_base + T_A + bb * T_AS + 64;  // [dS | dZ] of chunk u
            const float dz = tmem_ld1(dbase + 64);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                float d[32];
                tmem_ld2x16(dbase + 32 * h2, d);
                if (h2 == 1) {
                    tc_fence_before();
                    mbar_arrive(&bar[B_DSFREE0 + bb]);
                    mbar_arrive_after_reads(&bar[B_EMPTY0 + s]);  // part[s] is rewritten after the refill
                }
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float2 r = __ffma2_rn(dec2, make_float2(S[32 * h2 + e], S[32 * h2 + e + 1]), make_float2(d[e], d[e + 1]));
                    S[32 * h2 + e] = r.x;
                    S[32 * h2 + e + 1] = r.y;
                }
            }
            Z = fmaf(decay, Z, dz);
            if (f < D) s0 = fmaf(decay, s0, ds0);
            Z0 = fmaf(decay, Z0, PT ? zinc : sm.geo[n]);
            if (SO) continue;
            if (u + 1 < U) {
                // the carry GEMM of chunk u has finished reading the state tile
                if (!mbar_wait(&bar[B_QFREE0 + bb], (u >> 1) & 1, ctl, 13)) {
                    ok = false;
                    break;
                }
                publish(u + 1);
            }
            // ---- output rows of chunk u (thread f owns token row f)
            if (!mbar_wait(&bar[B_CDONE0 + bb], (u >> 1) & 1, ctl, 14) ||
                !mbar_wait(&bar[B_SREADY0 + bb], (u >> 1) & 1, ctl, 15)) {  // S0 / Z0 entering chunk u
                ok = false;
                break;
            }
            tc_fence_after();
            if (use_tma_y) {  // the previous chunk's store has read the staging tile
                if (f == 0) bulk_wait_read();
                named_bar(1, 128);
            }
            {
                uint32_t r[32], r64;
                tmem_ld33(lane_base + T_ACC, r, r64);  // columns 0..31 and the denominator column
                const int s3 = u % 3;
                const float g = PT ? __expf(grow) : sm.pw[f + 1];
                const float den = __uint_as_float(r64) + sm.z0f[s3];  // carry + intra-chunk denominator
                const float sc = g / fmaxf(g * den, p.eps);
                const float2 sc2 = make_float2(sc, sc);
                const float4 *s0v = reinterpret_cast<const float4 *>(sm.s0f[s3]);
                TO *yrow = reinterpret_cast<TO *>(p.y.p) + b * p.y.sb + h * p.y.sh +
                           (int64_t)((c_begin + u) * C + f) * p.y.sl;
                auto half = [&](int hc) {  // y in place of the accumulator words
#pragma unroll
                    for (int e4 = 0; e4 < 8; ++e4) {
                        const float4 sv = s0v[8 * hc + e4];
                        const float2 lo = __fmul2_rn(
                            __fadd2_rn(make_float2(__uint_as_float(r[4 * e4]), __uint_as_float(r[4 * e4 + 1])),
                                       make_float2(sv.x, sv.y)),
                            sc2);
                        const float2 hi = __fmul2_rn(
                            __fadd2_rn(make_float2(__uint_as_float(r[4 * e4 + 2]), __uint_as_float(r[4 * e4 + 3])),
                                       make_float2(sv.z, sv.w)),
                            sc2);
                        r[4 * e4] = __float_as_uint(lo.x);
                        r[4 * e4 + 1] = __float_as_uint(lo.y);
                        r[4 * e4 + 2] = __float_as_uint(hi.x);
                        r[4 * e4 + 3] = __float_as_uint(hi.y);
                    }
                    if (use_tma_y) {  // row f of the staging tile, columns 32 hc ..
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            *reinterpret_cast<uint4 *>(smem + OFF_YS + swz(f, 4 * hc + c)) =
                                pack8(reinterpret_cast<const float *>(r) + 8 * c);
                    } else if (f < n) {
                        store_row32<TO>(yrow + 32 * hc, reinterpret_cast<const float *>(r));
                    }
                };
                half(0);
                tmem_ld32_issue(lane_base + T_ACC + 32, r);
                tmem_wait_ld_regs(r);
                tc_fence_before();
                mbar_arrive(&bar[B_OEMPTY]);  // ACC is in registers: the next chunk's carry GEMM may start
                half(1);
            }
            if (use_tma_y) {  // the chunk's rows as one TMA store (rows past L are not written)
                fence_proxy_async();
                named_bar(2, 128);
                if (f == 0) {
                    tma_store(&ty, smem + OFF_YS, 0, (c_begin + u) * C, h, b);
                    bulk_commit();
                }
            }
        }
        if (use_tma_y && f == 0) bulk_wait_all();  // every row store is complete before the CTA ends
        // ---- final state
        const bool write_out = ok && !ctl.aborted() && p.out.present() &&
                               (p.state_only || seg == (int)gridDim.y - 1);
        if (write_out) {
            const HeadPtrs dst = p.out.at(bh, p.out.packed ? seg : 0, D);
            float *row = f < D ? dst.S1 + f * D : dst.S2 + (f - D) * D;
            if (PT && p.half_sq && f >= D && !p.out.packed) {  // selective layout: S2, Z2 halved
#pragma unroll
                for (int e = 0; e < D; ++e) S[e] *= 0.5f;
                Z *= 0.5f;
            }
            if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
#pragma unroll
                for (int e = 0; e < D; e += 4)
                    *reinterpret_cast<float4 *>(row + e) = make_float4(S[e], S[e + 1], S[e + 2], S[e + 3]);
            } else {
#pragma unroll
                for (int e = 0; e < D; ++e) row[e] = S[e];
            }
            if (f < D) {
                dst.Z1[f] = Z;
                dst.S0[f] = s0;
            } else {
                dst.Z2[f - D] = Z;
            }
            if (f == 0) dst.Z0[0] = Z0;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T_COLS) : "memory");
    if (threadIdx.x == 0) report_fault(sm.ctl.abort_flag, p.fault);
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled get_encode() {
    static EncodeTiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(ptr);
    }
    return fn;
}

bool tensor_maps_available() { return get_encode() != nullptr; }

// [B,H,L,Dh] bf16 with element strides -> 4-D map (d, l, h, b), box 64 x 128 x 1 x 1, 128-byte
// swizzle (Dh = 128: two boxes per row block, at d = 0 and d = 64).
bool make_tile_map(CUtensorMap *m, const Seq &s, int B, int H, int L, int Dh) {
    EncodeTiled enc = get_encode();
    if (!enc) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)Dh, (cuuint64_t)L, (cuuint64_t)H, (cuuint64_t)B};
    // strides of dims 1..3 in bytes; size-1 dims get a harmless stride
    cuuint64_t str[3] = {(cuuint64_t)s.sl * 2, (cuuint64_t)s.sh * 2, (cuuint64_t)s.sb * 2};
    for (int i = 0; i < 3; ++i)
        if (str[i] == 0) str[i] = 16;
    const cuuint32_t box[4] = {64, (cuuint32_t)C, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(s.p), dims, str, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool SO, typename TO, bool PRO, bool PT>
static cudaError_t launch_t(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                            const PrefillParams &p0, dim3 grid, cudaStream_t st) {
    auto kern = prefill_tc_kernel<SO, TO, PRO, PT>;
    cudaError_t e = set_smem_once<prefill_tc_kernel<SO, TO, PRO, PT>>((int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    // bf16 y rows: a tensor map for the chunk stores (else the kernel stores rows itself)
    PrefillParams p = p0;
    CUtensorMap my = mq;
    p.y_tma = 0;
    if (!SO && !PT && sizeof(TO) == 2 && p.y.p) {
        const Seq ys{p.y.p, p.y.sb, p.y.sh, p.y.sl};
        if (make_tile_map(&my, ys, p.B, p.H, p.L, 64)) p.y_tma = 1;
    }
    kern<<<grid, 512, SMEM_BYTES, st>>>(mq, mk, mv, my, p);
    return cudaGetLastError();
}

}  // namespace tc

bool tc_supported(int D, int idt) { return D == 64 && idt == PMA_BF16 && tc::get_encode() != nullptr; }

cudaError_t launch_prefill_tc(const PrefillParams &p, int ydt, dim3 grid, cudaStream_t st) {
    CUtensorMap mq, mk, mv;
    const int hkv = p.H / p.pro.groups;
    if (!tc::make_tile_map(&mk, p.k, p.B, hkv, p.L, 64) || !tc::make_tile_map(&mv, p.v, p.B, hkv, p.L, 64)) return cudaErrorInvalidValue;
    if (!p.state_only && p.y.p) {
        if (!tc::make_tile_map(&mq, p.q, p.B, p.H, p.L, 64)) return cudaErrorInvalidValue;
    } else {
        mq = mk;
    }
    const bool so = p.state_only || !p.y.p;
    if (p.pro.qw || p.pro.kw) return cudaErrorInvalidValue;  // norms are applied by the prologue pass
    if (p.logdecay) {  // per-token decay (one segment per head-state)
        if (so) return tc::launch_t<true, float, false, true>(mq, mk, mv, p, grid, st);
        if (p.pro.q_scale != 1.0f)
            return ydt == PMA_F32 ? tc::launch_t<false, float, true, true>(mq, mk, mv, p, grid, st)
                                  : tc::launch_t<false, __nv_bfloat16, true, true>(mq, mk, mv, p, grid, st);
        return ydt == PMA_F32 ? tc::launch_t<false, float, false, true>(mq, mk, mv, p, grid, st)
                              : tc::launch_t<false, __nv_bfloat16, false, true>(mq, mk, mv, p, grid, st);
    }
    if (so) return tc::launch_t<true, float, false, false>(mq, mk, mv, p, grid, st);
    if (p.pro.q_scale != 1.0f)
        return ydt == PMA_F32 ? tc::launch_t<false, float, true, false>(mq, mk, mv, p, grid, st)
                              : tc::launch_t<false, __nv_bfloat16, true, false>(mq, mk, mv, p, grid, st);
    return ydt == PMA_F32 ? tc::launch_t<false, float, false, false>(mq, mk, mv, p, grid, st)
                          : tc::launch_t<false, __nv_bfloat16, false, false>(mq, mk, mv, p, grid, st);
}

}  // namespace pma
