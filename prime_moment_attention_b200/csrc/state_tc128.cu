// state_tc128.cu -- the state-only prefill at D = 128 on tcgen05 tensor cores: the state a sequence
// segment builds, without its outputs (the first pass of the segment carry and of sequence shards).
//
// For a segment of tokens [t0, t1) started from zero, every component of the moment state is a
// decay-weighted sum over its tokens with weights w_j = l^(t1 - 1 - j) (chunked_ssd.py:96-111 forms
// the same sums per chunk and carries them with l^C):
//   S1 = sum_j w_j k_j v_j^T,  S2 = sum_j w_j (k_j*k_j) v_j^T,  S0 = sum_j w_j v_j,
//   Z1 = sum_j w_j k_j,        Z2 = sum_j w_j k_j*k_j,          Z0 = sum_j w_j = (1 - l^n)/(1 - l).
// Weighting each token by its distance to the segment END (w <= 1, no rescaling, so no range limit
// on l) turns the segment into one long GEMM over tokens: the tensor core accumulates
// (w.k)^T V, (w.k^2)^T V and V^T [w_hi | w_lo] chunk after chunk into tensor memory, and no CUDA-core
// state update sits between chunks.  Tokens far from the end carry weights that underflow to zero,
// as their contributions do in the float32 recurrence.  With an incoming state (one segment, y not
// wanted) the result adds l^n times it.
//
// Warp roles (512 threads, one CTA per SM, two pipeline stages):
//   warp 0     TMA producer: k and v chunk tiles (two 64-column boxes each) into stage u % 2
//   warp 1     MMA issuer: per chunk 8 K-steps of three MMAs, accumulating; commits free the stage
//   warps 4-11 prep: w.k in place, w.k^2, the [w_hi | w_lo] sums operand, and running Z1, Z2 sums
//   all       epilogue: the accumulators from tensor memory into the output state
// Every wait is bounded by the global timer; on expiry the CTA records a status code, drains its
// copies and GEMMs, and leaves without writing the state.
#include <cuda.h>

#include "prefill.cuh"
#define PMA_FAULT_AT_EXIT 1  // report expired waits once per CTA, after the final barrier
#include "tc_common.cuh"

namespace pma {
namespace st128 {

using namespace pma::tc;

constexpr int C = TC_CHUNK;     // 128 tokens per chunk
constexpr int D = 128;
constexpr int NT = 512;
constexpr int NPW = 8;          // prep warps (4 .. 11)
constexpr int TILE = 128 * 128;  // [128 tokens x 64] bf16, 128-byte swizzle: 16 KiB
constexpr int WT_ATOM = 2048;    // sums operand: [16 rows x 64 tokens] bf16 per atom
// stage s at s * STAGE: k (2 tiles), w.k^2 (2 tiles), v (2 tiles), sums operand (2 atoms)
constexpr int OFF_K = 0, OFF_K2 = 2 * TILE, OFF_V = 4 * TILE, OFF_WT = 6 * TILE;
constexpr int STAGE = 6 * TILE + 2 * WT_ATOM;
constexpr int OFF_SMALL = 2 * STAGE;
constexpr int PREFETCH = 2;      // chunks of L2 prefetch ahead of the stage loads
// tensor-memory columns: (w.k)^T V, (w.k^2)^T V, V^T [0 | w_hi | w_lo ...]
constexpr uint32_t T_S1 = 0, T_S2 = 128, T_S0 = 256, T_COLS = 512;

enum { B_FULL0, B_FULL1, B_PREP0, B_PREP1, B_EMPTY0, B_EMPTY1, B_DONE, B_NEVER, NBAR };

struct Small {
    uint64_t bar[NBAR];
    uint32_t tmem_base;
    CtlShared ctl;
    alignas(16) float zp[NPW * 2][2 * D];  // per 16-thread group: partial Z1 | Z2
};
constexpr size_t SMEM_BYTES = OFF_SMALL + sizeof(Small) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

__global__ void __launch_bounds__(NT, 1)
    state_tc128_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                       const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    Small &sm = *reinterpret_cast<Small *>(smem + OFF_SMALL);
    const uint32_t sb = su32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x, seg = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int hk = h / p.pro.groups;
    const double lam = p.lambda[(int64_t)b * p.lam_sb + h];
    const int t0 = seg * p.seg_len;
    const int t1 = min(t0 + p.seg_len, p.L);
    const int n_tok = max(t1 - t0, 0);
    const int U = (n_tok + C - 1) / C;
    Ctl ctl{&sm.ctl, p.status};
    uint64_t *bar = sm.bar;

    // ---- set-up: barriers, tensor memory, zero rows of the sums operands
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i) mbar_init(&bar[i], (i == B_PREP0 || i == B_PREP1) ? 32 * NPW : 1);
        init_ctl(sm.ctl, p.fault);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sm.tmem_base)),
                     "r"(T_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    for (int i = tid; i < 2 * 2 * WT_ATOM / 16; i += NT) {  // both stages' sums operands
        const int s = i / (2 * WT_ATOM / 16), j = i - s * (2 * WT_ATOM / 16);
        reinterpret_cast<uint4 *>(smem + s * STAGE + OFF_WT)[j] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    if (p.test_wait_ns) {  // test hook: a wait expires before any copy or GEMM is issued
        if (tid == 0) expire_test_wait(&bar[B_NEVER], ctl, p.test_wait_ns, 90);
        __syncthreads();
        if (ctl.aborted()) {
            if (warp == 0)
                asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T_COLS)
                             : "memory");
            if (tid == 0) report_fault(sm.ctl.abort_flag, p.fault);
            return;
        }
    }

    float z1[8], z2[8];  // prep threads: running Z1, Z2 over dims 8 cc .. 8 cc + 7
#pragma unroll
    for (int i = 0; i < 8; ++i) z1[i] = z2[i] = 0.f;

    if (warp == 0) {
        // ============================== TMA producer
        if (lane == 0) {
            int issued = 0, fetched = 0;
            for (int u = 0; u < U; ++u) {
                const int s = u & 1;
                for (; fetched < U && fetched <= u + PREFETCH; ++fetched)
                    for (int x = 0; x < 2; ++x) {
                        tma_prefetch_l2(&tk, 64 * x, t0 + fetched * C, hk, b);
                        tma_prefetch_l2(&tv, 64 * x, t0 + fetched * C, hk, b);
                    }
                if (!mbar_wait(&bar[B_EMPTY0 + s], ((u >> 1) & 1) ^ 1, ctl, 50)) break;
                uint8_t *base = smem + s * STAGE;
                const int tt = t0 + u * C;
                mbar_expect_tx(&bar[B_FULL0 + s], 4 * TILE);
                for (int x = 0; x < 2; ++x) {
                    tma_load(base + OFF_K + x * TILE, &tk, &bar[B_FULL0 + s], 64 * x, tt, hk, b);
                    tma_load(base + OFF_V + x * TILE, &tv, &bar[B_FULL0 + s], 64 * x, tt, hk, b);
                }
                issued = u + 1;
            }
            // never leave with copies in flight
            for (int u = max(0, issued - 2); u < issued; ++u) {
                const unsigned long long w0 = gtimer();
                while (!mbar_try(&bar[B_FULL0 + (u & 1)], (u >> 1) & 1) && gtimer() - w0 < WAIT_NS) {
                }
            }
        }
    } else if (warp == 1) {
        // ============================== MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_S = idesc(128, 128, 1, 1);  // (w.k)^T V: both MN-major
            constexpr uint32_t ID_0 = idesc(128, 16, 1, 0);   // V^T [sums rows]^T: A MN-major, B K-major
            constexpr uint64_t HI_TILE2 = desc_hi(TILE, 1024, 2), HI_KMAJ = desc_hi(16, 1024, 2);
            const uint32_t a0 = sb >> 4;  // the allocation sits below 256 KiB: no field overflow
            auto dsc = [&](uint32_t off, uint64_t hi) { return (uint64_t)(a0 + (off >> 4)) | hi; };
            int u = 0;
            for (; u < U; ++u) {
                const int s = u & 1;
                if (!mbar_wait(&bar[B_PREP0 + s], (u >> 1) & 1, ctl, 51)) break;
                tc_fence_after();
                const uint32_t base = (uint32_t)(s * STAGE);
#pragma unroll
                for (int k = 0; k < 8; ++k) {  // K = tokens, 16 rows = 2048 B per step
                    const uint64_t mk = (uint64_t)(k * 128);
                    const uint32_t acc = (u > 0 || k > 0) ? 1u : 0u;
                    mma_ss(tmem + T_S1, dsc(base + OFF_K, HI_TILE2) + mk, dsc(base + OFF_V, HI_TILE2) + mk, ID_S, acc);
                    mma_ss(tmem + T_S2, dsc(base + OFF_K2, HI_TILE2) + mk, dsc(base + OFF_V, HI_TILE2) + mk, ID_S, acc);
                    mma_ss(tmem + T_S0, dsc(base + OFF_V, HI_TILE2) + mk,
                           dsc(base + OFF_WT + (k >> 2) * WT_ATOM, HI_KMAJ) + (uint64_t)((k & 3) * 2), ID_0, acc);
                }
                commit(&bar[B_EMPTY0 + s]);
            }
            commit(&bar[B_DONE]);  // every GEMM issued is complete when this arrives
        }
    } else if (warp >= 4 && warp < 4 + NPW) {
        // ============================== prep: w.k in place, w.k^2, sums operand, running Z1 / Z2
        const int pt = tid - 128;             // 0 .. 255
        const int cc = pt & 15;               // 16-byte column chunk: dims 8 cc .. 8 cc + 7
        const int atom = cc >> 3, c = cc & 7;
        const int r0 = pt >> 4;               // rows r0 + 16 i
        const float l2 = (float)log2(lam);    // w_j = 2^((t1 - 1 - j) log2 l)
        for (int u = 0; u < U; ++u) {
            const int s = u & 1;
            if (!mbar_wait(&bar[B_FULL0 + s], (u >> 1) & 1, ctl, 52)) break;
            uint8_t *base = smem + s * STAGE;
            const int tt = t0 + u * C;
#pragma unroll 2
            for (int i = 0; i < 8; ++i) {
                const int r = r0 + 16 * i;
                const float w = tt + r < t1 ? exp2f((float)(t1 - 1 - tt - r) * l2) : 0.f;
                const __nv_bfloat162 wb = __float2bfloat162_rn(w);
                const uint32_t off = (uint32_t)(atom * TILE) + swz(r, c);
                const uint4 x = *reinterpret_cast<const uint4 *>(base + OFF_K + off);
                const uint32_t e4[4] = {x.x, x.y, x.z, x.w};
                uint32_t o1[4], o2[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const __nv_bfloat162 kv = as_b2(e4[q]);
                    const __nv_bfloat162 kw = __hmul2(kv, wb);
                    const __nv_bfloat162 k2w = __hmul2(kw, kv);
                    o1[q] = as_u(kw);
                    o2[q] = as_u(k2w);
                    const float2 a = __bfloat1622float2(kw), a2 = __bfloat1622float2(k2w);
                    z1[2 * q] += a.x;
                    z1[2 * q + 1] += a.y;
                    z2[2 * q] += a2.x;
                    z2[2 * q + 1] += a2.y;
                }
                *reinterpret_cast<uint4 *>(base + OFF_K + off) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
                *reinterpret_cast<uint4 *>(base + OFF_K2 + off) = make_uint4(o2[0], o2[1], o2[2], o2[3]);
            }
            if (pt < C) {  // w_hi, w_lo of token pt: rows 1, 2 of the sums operand (K-major, swizzled)
                const float w = tt + pt < t1 ? exp2f((float)(t1 - 1 - tt - pt) * l2) : 0.f;
                const __nv_bfloat16 whi = __float2bfloat16_rn(w);
                const __nv_bfloat16 wlo = __float2bfloat16_rn(w - __bfloat162float(whi));
                uint8_t *wt = base + OFF_WT + (pt >> 6) * WT_ATOM;
                const int cw = (pt & 63) >> 3, e = pt & 7;
                *reinterpret_cast<__nv_bfloat16 *>(wt + 1 * 128 + ((cw ^ 1) << 4) + 2 * e) = whi;
                *reinterpret_cast<__nv_bfloat16 *>(wt + 2 * 128 + ((cw ^ 2) << 4) + 2 * e) = wlo;
            }
            fence_proxy_async();  // the tiles are read by the tensor core
            mbar_arrive(&bar[B_PREP0 + s]);
        }
        // partial Z1 / Z2 of this thread's 16-thread group (threads with one r0 share no dims)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            sm.zp[r0][8 * cc + i] = z1[i];
            sm.zp[r0][D + 8 * cc + i] = z2[i];
        }
    }

    // ---- epilogue: wait for every GEMM, then the accumulators into the state
    const bool ok = mbar_wait(&bar[B_DONE], 0, ctl, 53);
    tc_fence_after();
    __syncthreads();
    if (ok && !ctl.aborted() && p.out.present()) {
        const bool any = U > 0;  // an empty segment leaves the accumulators unwritten
        const HeadPtrs dst = p.out.at(bh, p.out.packed ? seg : 0, D);
        const bool has_in = !p.state_only && p.in.present();
        const HeadPtrs src = has_in ? p.in.at(bh, 0, D) : HeadPtrs{};
        const float ln = (float)pow(lam, (double)n_tok);  // l^n: how much an incoming state decays
        const int qd = warp & 3, g = warp >> 2;  // lane quadrant (feature / value row), column quarter
        const int row = qd * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
        float a[32];
        if (any) {
            tmem_ld32(lane_base + T_S1 + 32 * g, a);
        } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) a[e] = 0.f;
        }
        float *o = dst.S1 + row * D + 32 * g;
        if (has_in) {
#pragma unroll
            for (int e = 0; e < 32; ++e) a[e] = fmaf(ln, src.S1[row * D + 32 * g + e], a[e]);
        }
#pragma unroll
        for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4 *>(o + e) = make_float4(a[e], a[e + 1], a[e + 2], a[e + 3]);
        if (any) tmem_ld32(lane_base + T_S2 + 32 * g, a);
        o = dst.S2 + row * D + 32 * g;
        if (has_in) {
#pragma unroll
            for (int e = 0; e < 32; ++e) a[e] = fmaf(ln, src.S2[row * D + 32 * g + e], a[e]);
        }
#pragma unroll
        for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4 *>(o + e) = make_float4(a[e], a[e + 1], a[e + 2], a[e + 3]);
        if (g == 0) {  // S0 of value `row`: the w_hi and w_lo columns
            const float s0 = any ? tmem_ld1(lane_base + T_S0 + 1) + tmem_ld1(lane_base + T_S0 + 2) : 0.f;
            dst.S0[row] = has_in ? fmaf(ln, src.S0[row], s0) : s0;
        }
        if (tid < 2 * D) {  // Z1 | Z2: the 16 partial sums of dimension tid
            float z = 0.f;
#pragma unroll
            for (int r = 0; r < NPW * 2; ++r) z += sm.zp[r][tid];
            if (tid < D)
                dst.Z1[tid] = has_in ? fmaf(ln, src.Z1[tid], z) : z;
            else
                dst.Z2[tid - D] = has_in ? fmaf(ln, src.Z2[tid - D], z) : z;
        }
        if (tid == 0) {
            const double z0 = lam < 1.0 ? (1.0 - pow(lam, (double)n_tok)) / (1.0 - lam) : (double)n_tok;
            dst.Z0[0] = has_in ? (float)(z0 + (double)ln * src.Z0[0]) : (float)z0;
        }
    }
    if (!ok && tid == 64) {  // gave up: the GEMMs issued must finish before tensor memory is freed
        const unsigned long long w0 = gtimer();
        while (!mbar_try(&bar[B_DONE], 0) && gtimer() - w0 < WAIT_NS) {
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T_COLS) : "memory");
    if (tid == 0) report_fault(sm.ctl.abort_flag, p.fault);
}

}  // namespace st128

cudaError_t launch_state_tc128(const PrefillParams &p, dim3 grid, cudaStream_t st) {
    CUtensorMap mk, mv;
    const int hkv = p.H / p.pro.groups;
    if (!tc::make_tile_map(&mk, p.k, p.B, hkv, p.L, 128) || !tc::make_tile_map(&mv, p.v, p.B, hkv, p.L, 128))
        return cudaErrorInvalidValue;
    cudaError_t e = set_smem_once<st128::state_tc128_kernel>((int)st128::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    st128::state_tc128_kernel<<<grid, st128::NT, st128::SMEM_BYTES, st>>>(mk, mv, p);
    return cudaGetLastError();
}

}  // namespace pma
