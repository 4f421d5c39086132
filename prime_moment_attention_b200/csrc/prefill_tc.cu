// prefill_tc.cu -- chunked prefill on tcgen05 tensor cores (bf16 inputs, D = 64).
//
// Same recurrence as chunked_prime_ssd_core (src/prime_moment_attention/chunked_ssd.py:48-184),
// evaluated per 128-token chunk (n <= 128 valid tokens) with the moment features
// psi(q) = [q | q^2/2], phi(k) = [k | k^2] (128 features) written as GEMMs on
// rescaled operands, so that almost all of the arithmetic runs on tensor cores:
//
//   g_i = l^(i+1)   (carry into token i)      w_j = l^(n-1-j)  (token j to chunk end, 0 if j >= n)
//   Qg  = g . q,  Q2g = g . q^2/2             Vw = w . v                 (rows scaled, bf16)
//   At  = [Qg | Q2g] [K | K^2]^T  = g_i (q_i.k_j + q_i^2.k_j^2/2)       (M=N=128, K=128)
//   P'  = l^(i-n+1) + l^-n At     = l^(i-j) (1 + ...) / w_j   for j <= i, else 0
//   ACC = [Qg | Q2g] [S1; S2]  +  P' Vw   =  g_i carry_i + num_i          (chunked_ssd.py:93,139-148)
//   DEN = [Qg | Q2g] [Z1; Z2]  +  P' w    =  g_i cden_i  + den_i           (:94,149-153)
//   y_i = (ACC_i + g_i S0) / max(DEN_i + g_i Z0, eps)                      (:155-157)
//   dS  = [K | K^2]^T Vw,  dZ = [K | K^2]^T w,  dS0 = Vw^T 1             (:96-111)
//   S   = l^n S + dS   (float32, in registers of the state warpgroup)     (:162-169)
// The per-element decay mask of the reference becomes one FMA per element;
// denominators and the S0/Z1/Z2 updates are N=16 GEMMs against one-row tiles.
// The rescaling keeps every factor inside float32/bf16 range for l >= 0.55
// (l^-128 < 1e34, l^128 > 1e-34); head-states with a smaller decay run the
// float32 CUDA-core chunk loop (prefill_simt_body.cuh) inside this kernel.
//
// Data: q/k/v chunk tiles arrive by TMA (4-D tensor maps over the strided
// tensors, 128-byte swizzle) into two stages; prep overwrites q by Qg and v by
// Vw in place and writes Q2g and K^2 to double-buffered tiles.  Accumulators
// live in tensor memory: At x2 (P' is written back over the consumed At columns
// and read by the P'-GEMMs from TMEM), ACC x2, dS, DEN x2, and [dZ | dS0] in one
// 16-column region.  The producer also prefetches the tiles of later chunks
// into L2, so each stage load finds its data there.  The bf16 state copy
// [S1; S2] and the one-row [Z1; Z2] tile that feed the carry GEMMs are
// double-buffered.
//
// Warp roles (512 threads, one CTA per SM):
//   warp 0        TMA producer
//   warp 1        MMA issuer (one thread, event driven: issues each chunk's GEMM
//                 groups as soon as their inputs are ready) and TMEM owner.  The
//                 state GEMMs of chunk u+1 start as soon as the state warpgroup
//                 has read dS of chunk u, so the recurrence's critical path is
//                 one tensor-memory read, the dS GEMMs and one barrier hop.
//   warps 4-7     prep: Qg, Q2g, K^2, Vw for each chunk
//   warps 8-11    mask: At -> P' in tensor memory
//   warps 12-15   state and output: S += dS (thread f owns feature row f), bf16
//                 state tiles for the next chunk, then y for the chunk's 128 tokens
// Every wait is bounded by the global timer; on expiry the kernel records a status
// code in the workspace header, every role stops, and the CTA waits for its
// in-flight copies and GEMMs before freeing tensor memory.
#include <cuda.h>

#include "prefill.cuh"
#include "prefill_simt_body.cuh"

namespace pma {
namespace tc {

constexpr int C = TC_CHUNK;   // tokens per chunk
constexpr int D = 64;
constexpr int TILE = C * D * 2;           // [128 x 64] bf16 = 16 KiB
constexpr int STAGE = 3 * TILE;           // q (-> Qg), k, v (-> Vw)
constexpr int OFF_DER = 2 * STAGE;        // per buffer: Q2g, K^2
constexpr int OFF_SB = OFF_DER + 4 * TILE;    // bf16 [S1; S2], [128 features][64 values], x2
constexpr int ROW1 = 4096;                // one-row K-major tile: 2 atoms x 16 rows x 128 B
constexpr int OFF_ZT = OFF_SB + 2 * TILE;     // [Z1; Z2] row, x2
constexpr int OFF_W16 = OFF_ZT + 2 * ROW1;    // w row: full chunks, last partial chunk
constexpr int OFF_ONES = OFF_W16 + 2 * ROW1;  // ones in row 1 (dS0 lands in column 1 of [dZ | dS0])
constexpr int PREFETCH = 3;               // chunks of L2 prefetch ahead of the stage loads
constexpr int OFF_SMALL = OFF_ONES + ROW1;
constexpr float LMIN = 0.55f;             // smallest decay the rescaled operands serve

enum {
    B_FULL0, B_FULL1, B_CDONE0, B_CDONE1, B_PREP0, B_PREP1, B_IFULL0, B_IFULL1, B_PREADY0, B_PREADY1, B_DSFULL,
    B_DSFREE, B_SREADY0, B_SREADY1, B_OEMPTY0, B_OEMPTY1, B_FINAL, NBAR
};

struct Small {
    uint64_t bar[18];
    float pw[C + 4];      // l^t, t = 0..C
    float geo[C + 4];     // sum_{t<n} l^t
    alignas(16) float s0f[2][D];  // S0 entering the chunk (float32), per chunk parity
    uint32_t tmem_base;
    int abort_flag;
};
constexpr size_t SMEM_BYTES = OFF_SMALL + sizeof(Small) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
static_assert(SimtSmem<64, 64>::bytes <= OFF_SMALL, "fallback path fits in the same allocation");

// tensor-memory columns
constexpr uint32_t T_A = 0, T_ACC = 256, T_DS = 384, T_DEN = 448, T_DZS = 480, T_COLS = 512;

constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s per wait

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
// may suspend the thread briefly while the phase is incomplete
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// never blocks (the MMA issuer polls several barriers)
__device__ __forceinline__ bool mbar_poll(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

struct Ctl {
    volatile int *abort_flag;  // shared: any role gave up
    int *status;               // global: first failure code (nullable)
};

__device__ __forceinline__ void give_up(const Ctl &ctl, int code) {
    *ctl.abort_flag = 1;
    if (ctl.status) atomicCAS(ctl.status, 0, code);
}

__device__ __noinline__ bool mbar_wait_slow(uint64_t *b, uint32_t parity, const Ctl &ctl, int code) {
    const unsigned long long t0 = gtimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try(b, parity)) return true;
        if ((it & 63) == 0) {
            if (*ctl.abort_flag) return false;
            if (gtimer() - t0 > WAIT_NS) {
                give_up(ctl, code);
                return false;
            }
        }
    }
}
// Wait for the phase of parity `parity`; false if it timed out or another role gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, const Ctl &ctl, int code) {
    if (mbar_try(b, parity)) return true;
    return mbar_wait_slow(b, parity, ctl, code);
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ void tma_load(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2,
                                         int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(su32(dst)),
        "l"(map), "r"(su32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_l2(const CUtensorMap *map, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(map), "r"(c0),
                 "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

// Shared-memory matrix descriptor: 128-byte swizzle, sm_100 version field.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, dense; a_mn/b_mn = operand is MN-major.
__host__ __device__ constexpr uint32_t idesc(int M, int N, int a_mn, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D (tmem) [+]= A (smem) B (smem)
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}
// D (tmem) [+]= A (tmem, K-major) B (smem)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(id), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}
// 32 consecutive float32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// One float32 column of this thread's TMEM lane.
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    return __uint_as_float(r);
}
// Two float32 columns of this thread's TMEM lane.
__device__ __forceinline__ float2 tmem_ld2(uint32_t taddr) {
    uint32_t r0, r1;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    return make_float2(__uint_as_float(r0), __uint_as_float(r1));
}
// 16 consecutive 32-bit columns of this thread's TMEM lane (completion via tmem_wait_st).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ uint4 pack8(const float *f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}
__device__ __forceinline__ __nv_bfloat162 as_b2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162 *>(&u); }
__device__ __forceinline__ uint32_t as_u(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t *>(&h); }
// byte offset of 16-byte chunk `c` of row `r` in a [rows x 128 B] tile with the 128-byte swizzle
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }
// byte offset of element k of row 0 in a one-row K-major tile (two 64-element atoms of 16 rows)
__device__ __forceinline__ uint32_t row0(int k) { return (uint32_t)((k >> 6) * 2048 + (k & 63) * 2); }

template <typename TO>
__device__ __forceinline__ void store_row32(TO *dst, const float *v);
template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16 *dst, const float *v) {
    uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int c = 0; c < 4; ++c) d[c] = pack8(v + 8 * c);
}
template <>
__device__ __forceinline__ void store_row32<float>(float *dst, const float *v) {
    float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int c = 0; c < 8; ++c) d[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// ------------------------------------------------------------------ the kernel
template <bool SO, typename TO>   // SO: state only (no q, no output rows)
__global__ void __launch_bounds__(512, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Small &sm = *reinterpret_cast<Small *>(smem + OFF_SMALL);
    const uint32_t sb = su32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.x, seg = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const float lam = p.lambda[(int64_t)b * p.lam_sb + h];

    if (!(lam >= LMIN)) {  // small decay (or NaN): float32 CUDA-core chunk loop, whole CTA
        simt_prefill_body<64, 64, __nv_bfloat16, TO>(p, reinterpret_cast<float *>(smem), bh, seg);
        return;
    }

    const int nchunks_total = (p.L + C - 1) / C;
    const int seg_chunks = p.seg_len / C;
    const int c_begin = seg * seg_chunks;
    const int c_end = min(c_begin + seg_chunks, nchunks_total);
    const int U = c_end - c_begin;
    const int n_last = min(C, p.L - (c_end - 1) * C);
    Ctl ctl{&sm.abort_flag, p.status};

    // ---- set-up: powers, barriers, constant one-row tiles, tensor memory
    if (threadIdx.x <= C) sm.pw[threadIdx.x] = (float)pow((double)lam, (double)threadIdx.x);
    for (int i = threadIdx.x; i < 5 * ROW1 / 16; i += blockDim.x)  // zero ZT x2, W16 x2, ONES
        reinterpret_cast<uint4 *>(smem + OFF_ZT)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; ++i) {
            uint32_t n = 1;
            if (i == B_PREP0 || i == B_PREP1 || i == B_PREADY0 || i == B_PREADY1 || i == B_SREADY0 ||
                i == B_SREADY1 || i == B_DSFREE || i == B_OEMPTY0 || i == B_OEMPTY1)
                n = 128;
            mbar_init(&sm.bar[i], n);
        }
        sm.abort_flag = 0;
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
    if (threadIdx.x == 0) {
        float g = 0.f;
        for (int j = 0; j <= C; ++j) {
            sm.geo[j] = g;
            if (j < C) g += sm.pw[j];
        }
    }
    if (threadIdx.x < C) {  // w row for full chunks, and the ones row
        const int j = threadIdx.x;
        *reinterpret_cast<__nv_bfloat16 *>(smem + OFF_W16 + row0(j)) = __float2bfloat16_rn(sm.pw[C - 1 - j]);
        *reinterpret_cast<__nv_bfloat16 *>(smem + OFF_ONES + 128 + row0(j)) = __float2bfloat16_rn(1.0f);
    }
    fence_proxy_async();
    __syncthreads();
    const uint32_t tmem = sm.tmem_base;
    uint64_t *bar = sm.bar;

    if (warp == 0) {
        // ============================== TMA producer
        if (lane == 0) {
            int issued = 0, fetched = 0;
            for (int u = 0; u < U; ++u) {
                for (; fetched < U && fetched <= u + PREFETCH; ++fetched) {
                    const int tf = (c_begin + fetched) * C;
                    if (!SO) tma_prefetch_l2(&tq, 0, tf, h, b);
                    tma_prefetch_l2(&tk, 0, tf, h, b);
                    tma_prefetch_l2(&tv, 0, tf, h, b);
                }
                const int st = u & 1;
                if (!mbar_wait(&bar[B_CDONE0 + st], ((u >> 1) & 1) ^ 1, ctl, 1)) break;
                const int t0 = (c_begin + u) * C;
                uint8_t *base = smem + st * STAGE;
                mbar_expect_tx(&bar[B_FULL0 + st], SO ? 2 * TILE : 3 * TILE);
                if (!SO) tma_load(base, &tq, &bar[B_FULL0 + st], 0, t0, h, b);
                tma_load(base + TILE, &tk, &bar[B_FULL0 + st], 0, t0, h, b);
                tma_load(base + 2 * TILE, &tv, &bar[B_FULL0 + st], 0, t0, h, b);
                issued = u + 1;
            }
            // never leave with copies in flight: the last (up to) two stages must have landed
            for (int u = max(0, issued - 2); u < issued; ++u) {
                const unsigned long long t0 = gtimer();
                while (!mbar_try(&bar[B_FULL0 + (u & 1)], (u >> 1) & 1) && gtimer() - t0 < WAIT_NS) {
                }
            }
        }
    } else if (warp == 1) {
        // ============================== MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_A = idesc(128, 128, 0, 0);  // [Qg|Q2g][K|K2]^T
            constexpr uint32_t ID_DS = idesc(128, 64, 1, 1);  // [K|K2]^T Vw
            constexpr uint32_t ID_DZ = idesc(128, 16, 1, 0);  // [K|K2]^T w, [Vw|.]^T 1
            constexpr uint32_t ID_C = idesc(128, 64, 0, 1);   // [Qg|Q2g][S1;S2], P' Vw
            constexpr uint32_t ID_CZ = idesc(128, 16, 0, 0);  // [Qg|Q2g][Z1;Z2], P' w
            // Every operand descriptor is built once; a k-step only adds a constant to its start
            // address field (the issue loop is what bounds a single-thread MMA issuer).
            // (pairs per buffer; a ternary select keeps them in registers)
            struct D2 {
                uint64_t v0, v1;
                __device__ __forceinline__ uint64_t operator[](int b) const { return b ? v1 : v0; }
            };
            auto mk = [&](auto f) { return D2{f(0), f(1)}; };
            const uint32_t st1 = STAGE, der1 = 2 * TILE;
            const D2 dQ = mk([&](int b) { return sdesc(sb + b * st1, 16, 1024); });
            const D2 dQ2 = mk([&](int b) { return sdesc(sb + OFF_DER + b * der1, 16, 1024); });
            const D2 dK = mk([&](int b) { return sdesc(sb + b * st1 + TILE, 16, 1024); });
            const D2 dK2 = mk([&](int b) { return sdesc(sb + OFF_DER + b * der1 + TILE, 16, 1024); });
            // [K | K2] and [Vw | K2] as MN-major A operands: two 64-row atoms, LBO = distance to K2
            const D2 dKmn = mk([&](int b) {
                return sdesc(sb + b * st1 + TILE, (OFF_DER + b * der1 + TILE) - (b * st1 + TILE), 1024);
            });
            const D2 dVmn = mk([&](int b) {
                return sdesc(sb + b * st1 + 2 * TILE, (OFF_DER + b * der1 + TILE) - (b * st1 + 2 * TILE), 1024);
            });
            const D2 dV = mk([&](int b) { return sdesc(sb + b * st1 + 2 * TILE, 8192, 1024); });
            const D2 dSB = mk([&](int b) { return sdesc(sb + OFF_SB + b * TILE, 8192, 1024); });
            const D2 dZT = mk([&](int b) { return sdesc(sb + OFF_ZT + b * ROW1, 16, 1024); });
            const D2 dW = mk([&](int b) { return sdesc(sb + OFF_W16 + b * ROW1, 16, 1024); });
            const uint64_t dONES = sdesc(sb + OFF_ONES, 16, 1024);
            // descriptor start-address steps (16-byte units) of k-step s
            auto kmaj = [](int s) { return (uint64_t)((s & 3) * 2); };                  // +32 B in a 128 B row
            auto mnmaj = [](int s) { return (uint64_t)(s * 128); };                     // +16 rows of 128 B
            auto row1 = [](int s) { return (uint64_t)((s >> 2) * 128 + (s & 3) * 2); };  // one-row K-major tile
            int u1 = 0, u2a = 0, u2b = 0, u4 = 0;
            const int U2b = SO ? 0 : U;
            unsigned long long last = gtimer();
            while (u2a < U || u2b < U2b || (!SO && u4 < U)) {
                if (*ctl.abort_flag) break;
                bool prog = false;
                // ---- group 1: At = [Qg|Q2g][K|K2]^T into At[u1 & 1]
                if (!SO && u1 < U) {
                    const int bb = u1 & 1;
                    if (mbar_poll(&bar[B_PREP0 + bb], (u1 >> 1) & 1) &&
                        mbar_poll(&bar[B_CDONE0 + bb], ((u1 >> 1) & 1) ^ 1)) {
                        tc_fence_after();
#pragma unroll
                        for (int s = 0; s < 8; ++s)
                            mma_ss(tmem + T_A + bb * 128, (s < 4 ? dQ[bb] : dQ2[bb]) + kmaj(s),
                                   (s < 4 ? dK[bb] : dK2[bb]) + kmaj(s), ID_A, s > 0);
                        commit(&bar[B_IFULL0 + bb]);
                        ++u1;
                        prog = true;
                    }
                }
                // ---- group 2a: dS = [K|K2]^T Vw, [dZ | dS0] of chunk u2a.  Needs the state warpgroup
                // to have read dS of the previous chunk, and (for the bf16 state buffers' reuse)
                // the previous chunk's carry GEMMs issued before it.
                if (u2a < U && (SO || u2a <= u2b)) {
                    const int bb = u2a & 1;
                    if (mbar_poll(&bar[B_PREP0 + bb], (u2a >> 1) & 1) && mbar_poll(&bar[B_DSFREE], u2a & 1)) {
                        tc_fence_after();
                        const int n = (u2a == U - 1) ? n_last : C;
                        const uint64_t dw = dW[n < C ? 1 : 0];
#pragma unroll
                        for (int s = 0; s < 8; ++s) {  // K-dim = tokens, 16 rows = 2048 B per step
                            mma_ss(tmem + T_DS, dKmn[bb] + mnmaj(s), dV[bb] + mnmaj(s), ID_DS, s > 0);
                            mma_ss(tmem + T_DZS, dKmn[bb] + mnmaj(s), dw + row1(s), ID_DZ, s > 0);
                        }
#pragma unroll
                        for (int s = 0; s < 8; ++s)  // column 1 of [dZ | dS0]: ones sit in row 1 of their tile
                            mma_ss(tmem + T_DZS, dVmn[bb] + mnmaj(s), dONES + row1(s), ID_DZ, 1);
                        commit(&bar[B_DSFULL]);
                        if (SO) commit(&bar[B_CDONE0 + bb]);
                        ++u2a;
                        prog = true;
                    }
                }
                // ---- group 2b: carry GEMMs of chunk u2b with the state entering it
                if (!SO && u2b < u2a && u2b < u1) {
                    const int bb = u2b & 1;
                    if (mbar_poll(&bar[B_SREADY0 + bb], (u2b >> 1) & 1) &&
                        mbar_poll(&bar[B_OEMPTY0 + bb], ((u2b >> 1) & 1) ^ 1)) {
                        tc_fence_after();
#pragma unroll
                        for (int s = 0; s < 8; ++s) {  // K-dim = features
                            const uint64_t a = (s < 4 ? dQ[bb] : dQ2[bb]) + kmaj(s);
                            mma_ss(tmem + T_ACC + bb * 64, a, dSB[bb] + mnmaj(s), ID_C, s > 0);
                            mma_ss(tmem + T_DEN + bb * 16, a, dZT[bb] + row1(s), ID_CZ, s > 0);
                        }
                        ++u2b;
                        prog = true;
                    }
                }
                // ---- group 4: ACC += P' Vw, DEN += P' w  (P' from tensor memory)
                if (!SO && u4 < u2b) {
                    const int bb = u4 & 1;
                    if (mbar_poll(&bar[B_PREADY0 + bb], (u4 >> 1) & 1)) {
                        tc_fence_after();
                        const int n = (u4 == U - 1) ? n_last : C;
                        const uint64_t dw = dW[n < C ? 1 : 0];
#pragma unroll
                        for (int s = 0; s < 8; ++s) {  // K-dim = tokens; P' packs 2 per column
                            const uint32_t pa = tmem + T_A + bb * 128 + s * 8;
                            mma_ts(tmem + T_ACC + bb * 64, pa, dV[bb] + mnmaj(s), ID_C, 1);
                            mma_ts(tmem + T_DEN + bb * 16, pa, dw + row1(s), ID_CZ, 1);
                        }
                        commit(&bar[B_CDONE0 + bb]);
                        ++u4;
                        prog = true;
                    }
                }
                if (prog) {
                    last = gtimer();
                } else {
                    if (gtimer() - last > WAIT_NS) {
                        give_up(ctl, 2);
                        break;
                    }
                    __nanosleep(32);
                }
            }
            // every GEMM issued must be complete before tensor memory is released
            commit(&bar[B_FINAL]);
            const unsigned long long t0 = gtimer();
            while (!mbar_try(&bar[B_FINAL], 0) && gtimer() - t0 < WAIT_NS) {
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ============================== prep: Qg (in place), Q2g, K^2 (new tiles), Vw (in place)
        const int tid = threadIdx.x - 128;
        const int cc = tid & 7, rb = tid >> 3;  // one 16-byte column chunk of 8 rows
        __nv_bfloat162 gq[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) gq[t] = __float2bfloat162_rn(sm.pw[rb * 8 + t + 1]);
        const __nv_bfloat162 half2 = __float2bfloat162_rn(0.5f);
        for (int u = 0; u < U; ++u) {
            const int st = u & 1;
            const int n = (u == U - 1) ? n_last : C;
            if (!mbar_wait(&bar[B_FULL0 + st], (u >> 1) & 1, ctl, 7)) break;
            if (!mbar_wait(&bar[B_CDONE0 + st], ((u >> 1) & 1) ^ 1, ctl, 8)) break;
            uint8_t *q_s = smem + st * STAGE, *k_s = q_s + TILE, *v_s = q_s + 2 * TILE;
            uint8_t *q2 = smem + OFF_DER + st * 2 * TILE, *k2 = q2 + TILE;
            // Each tile: issue all 8 row loads before any store (the in-place stores would
            // otherwise keep every load behind the previous row's store).
            uint4 x[8];
            if (!SO) {
#pragma unroll
                for (int t = 0; t < 8; ++t) x[t] = *reinterpret_cast<const uint4 *>(q_s + swz(rb * 8 + t, cc));
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const uint32_t off = swz(rb * 8 + t, cc);
                    uint32_t xq[4] = {x[t].x, x[t].y, x[t].z, x[t].w}, yq[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const __nv_bfloat162 qv = as_b2(xq[c]);
                        const __nv_bfloat162 qg = __hmul2(qv, gq[t]);
                        yq[c] = as_u(__hmul2(qg, __hmul2(qv, half2)));
                        xq[c] = as_u(qg);
                    }
                    *reinterpret_cast<uint4 *>(q_s + off) = make_uint4(xq[0], xq[1], xq[2], xq[3]);
                    *reinterpret_cast<uint4 *>(q2 + off) = make_uint4(yq[0], yq[1], yq[2], yq[3]);
                }
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) x[t] = *reinterpret_cast<const uint4 *>(k_s + swz(rb * 8 + t, cc));
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const uint32_t xk[4] = {x[t].x, x[t].y, x[t].z, x[t].w};
                uint32_t yk[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) yk[c] = as_u(__hmul2(as_b2(xk[c]), as_b2(xk[c])));
                *reinterpret_cast<uint4 *>(k2 + swz(rb * 8 + t, cc)) = make_uint4(yk[0], yk[1], yk[2], yk[3]);
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) x[t] = *reinterpret_cast<const uint4 *>(v_s + swz(rb * 8 + t, cc));
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int r = rb * 8 + t;
                const __nv_bfloat162 ww = __float2bfloat162_rn(r < n ? sm.pw[n - 1 - r] : 0.f);
                const uint32_t xv[4] = {x[t].x, x[t].y, x[t].z, x[t].w};
                uint32_t yv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) yv[c] = as_u(__hmul2(as_b2(xv[c]), ww));
                *reinterpret_cast<uint4 *>(v_s + swz(r, cc)) = make_uint4(yv[0], yv[1], yv[2], yv[3]);
            }
            if (u == U - 1 && n < C)  // w row of the partial last chunk
                *reinterpret_cast<__nv_bfloat16 *>(smem + OFF_W16 + ROW1 + row0(tid)) =
                    __float2bfloat16_rn(tid < n ? sm.pw[n - 1 - tid] : 0.f);
            fence_proxy_async();
            mbar_arrive(&bar[B_PREP0 + st]);
        }
    } else if (warp >= 8 && warp < 12) {
        // ============================== mask: At -> P' = l^(i-n+1) + l^-n At (j <= i), in tensor memory
        if (!SO) {
            const int wq = warp - 8;
            const int i = wq * 32 + lane;
            const uint32_t lane_base = tmem + ((uint32_t)(wq * 32) << 16);
            for (int u = 0; u < U; ++u) {
                const int bb = u & 1;
                const int n = (u == U - 1) ? n_last : C;
                const float cn = 1.0f / sm.pw[n];        // l^-n
                const float ri = sm.pw[i + 1] * cn;      // l^(i+1-n)
                if (!mbar_wait(&bar[B_IFULL0 + bb], (u >> 1) & 1, ctl, 9)) break;
                tc_fence_after();
                const uint32_t abase = lane_base + T_A + bb * 128;
#pragma unroll 1
                for (int g = 0; g < 4; ++g) {
                    uint32_t pk[16];
                    if (g > wq) {  // columns above the diagonal for every row of this warp
#pragma unroll
                        for (int c = 0; c < 16; ++c) pk[c] = 0u;
                    } else {
                        float a[32];
                        tmem_ld32(abase + 32 * g, a);
                        if (g < wq) {
#pragma unroll
                            for (int c = 0; c < 16; ++c)
                                pk[c] = pack2(fmaf(cn, a[2 * c], ri), fmaf(cn, a[2 * c + 1], ri));
                        } else {
#pragma unroll
                            for (int c = 0; c < 16; ++c)
                                pk[c] = pack2(2 * c <= lane ? fmaf(cn, a[2 * c], ri) : 0.f,
                                              2 * c + 1 <= lane ? fmaf(cn, a[2 * c + 1], ri) : 0.f);
                        }
                    }
                    // P' of columns 32g..32g+31 -> columns 16g..16g+15, whose At values were already read
                    tmem_st16(abase + 16 * g, pk);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bar[B_PREADY0 + bb]);
            }
        }
    } else if (warp >= 12) {
        // ============================== state update + output rows
        const int wq = warp - 12;
        const int f = wq * 32 + lane;  // feature row for the state, token row for the output
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
            if (f < D) s0 = src.S0[f];
            Z0 = src.Z0[0];
        } else {
#pragma unroll
            for (int e = 0; e < D; ++e) S[e] = 0.f;
            Z = 0.f;
            Z0 = 0.f;
        }
        auto publish = [&](int buf) {  // bf16 [S1;S2] row f, [Z1;Z2] element f, S0 for the next chunk
            uint8_t *srow = smem + OFF_SB + buf * TILE;
#pragma unroll
            for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4 *>(srow + swz(f, c)) = pack8(S + 8 * c);
            *reinterpret_cast<__nv_bfloat16 *>(smem + OFF_ZT + buf * ROW1 + row0(f)) = __float2bfloat16_rn(Z);
            if (f < D) sm.s0f[buf][f] = s0;
        };
        if (!SO) publish(0);
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(&bar[B_SREADY0]);
        mbar_arrive(&bar[B_DSFREE]);
        bool ok = true;
        for (int u = 0; u < U && ok; ++u) {
            const int bb = u & 1;
            const int t0 = (c_begin + u) * C;
            const int n = (u == U - 1) ? n_last : C;
            // ---- state update
            if (!mbar_wait(&bar[B_DSFULL], u & 1, ctl, 12)) {
                ok = false;
                break;
            }
            tc_fence_after();
            named_bar(2, 128);  // all rows of the previous chunk's output read s0f[bb ^ 1]
            const float decay = sm.pw[n];
            {
                float d[32];
                tmem_ld32(lane_base + T_DS, d);
#pragma unroll
                for (int e = 0; e < 32; ++e) S[e] = fmaf(decay, S[e], d[e]);
                tmem_ld32(lane_base + T_DS + 32, d);
                const float2 zs = tmem_ld2(lane_base + T_DZS);
                tc_fence_before();
                mbar_arrive(&bar[B_DSFREE]);  // dS is in registers: the next chunk's dS GEMMs may start
#pragma unroll
                for (int e = 0; e < 32; ++e) S[32 + e] = fmaf(decay, S[32 + e], d[e]);
                Z = fmaf(decay, Z, zs.x);
                if (f < D) s0 = fmaf(decay, s0, zs.y);
            }
            const float Z0_in = Z0;
            Z0 = fmaf(decay, Z0, sm.geo[n]);
            if (!SO) publish(bb ^ 1);
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(&bar[B_SREADY0 + (bb ^ 1)]);
            if (SO) continue;
            // ---- output rows
            if (!mbar_wait(&bar[B_CDONE0 + bb], (u >> 1) & 1, ctl, 14)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int i = f;
            const float g = sm.pw[i + 1];
            const float inv = 1.0f / fmaxf(tmem_ld1(lane_base + T_DEN + bb * 16) + g * Z0_in, p.eps);
            TO *yrow = reinterpret_cast<TO *>(p.y.p) + b * p.y.sb + h * p.y.sh + (int64_t)(t0 + i) * p.y.sl;
            const float4 *s0in = reinterpret_cast<const float4 *>(sm.s0f[bb]);
#pragma unroll
            for (int hcol = 0; hcol < 2; ++hcol) {
                float acc[32];
                tmem_ld32(lane_base + T_ACC + bb * 64 + 32 * hcol, acc);
#pragma unroll
                for (int e4 = 0; e4 < 8; ++e4) {
                    const float4 sv = s0in[8 * hcol + e4];
                    acc[4 * e4 + 0] = fmaf(g, sv.x, acc[4 * e4 + 0]) * inv;
                    acc[4 * e4 + 1] = fmaf(g, sv.y, acc[4 * e4 + 1]) * inv;
                    acc[4 * e4 + 2] = fmaf(g, sv.z, acc[4 * e4 + 2]) * inv;
                    acc[4 * e4 + 3] = fmaf(g, sv.w, acc[4 * e4 + 3]) * inv;
                }
                if (i < n) store_row32<TO>(yrow + 32 * hcol, acc);
            }
            tc_fence_before();
            mbar_arrive(&bar[B_OEMPTY0 + bb]);
        }
        // ---- final state
        const bool write_out = ok && !*ctl.abort_flag && p.out.present() &&
                               (p.state_only || seg == (int)gridDim.y - 1);
        if (write_out) {
            const HeadPtrs dst = p.out.at(bh, p.out.packed ? seg : 0, D);
            float *row = f < D ? dst.S1 + f * D : dst.S2 + (f - D) * D;
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

// [B,H,L,64] bf16 with element strides -> 4-D map (d, l, h, b), box 64 x 128 x 1 x 1, 128-byte swizzle.
static bool make_map(CUtensorMap *m, const Seq &s, int B, int H, int L) {
    EncodeTiled enc = get_encode();
    if (!enc) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)H, (cuuint64_t)B};
    // strides of dims 1..3 in bytes; size-1 dims get a harmless stride
    cuuint64_t str[3] = {(cuuint64_t)s.sl * 2, (cuuint64_t)s.sh * 2, (cuuint64_t)s.sb * 2};
    for (int i = 0; i < 3; ++i)
        if (str[i] == 0) str[i] = 16;
    const cuuint32_t box[4] = {(cuuint32_t)D, (cuuint32_t)C, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(s.p), dims, str, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool SO, typename TO>
static cudaError_t launch_t(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                            const PrefillParams &p, dim3 grid, cudaStream_t st) {
    auto kern = prefill_tc_kernel<SO, TO>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    kern<<<grid, 512, SMEM_BYTES, st>>>(mq, mk, mv, p);
    return cudaGetLastError();
}

}  // namespace tc

bool tc_supported(int D, int idt) { return D == 64 && idt == PMA_BF16 && tc::get_encode() != nullptr; }

cudaError_t launch_prefill_tc(const PrefillParams &p, int ydt, dim3 grid, cudaStream_t st) {
    CUtensorMap mq, mk, mv;
    if (!tc::make_map(&mk, p.k, p.B, p.H, p.L) || !tc::make_map(&mv, p.v, p.B, p.H, p.L)) return cudaErrorInvalidValue;
    if (!p.state_only && p.y.p) {
        if (!tc::make_map(&mq, p.q, p.B, p.H, p.L)) return cudaErrorInvalidValue;
    } else {
        mq = mk;
    }
    const bool so = p.state_only || !p.y.p;
    if (so) return tc::launch_t<true, float>(mq, mk, mv, p, grid, st);
    return ydt == PMA_F32 ? tc::launch_t<false, float>(mq, mk, mv, p, grid, st)
                          : tc::launch_t<false, __nv_bfloat16>(mq, mk, mv, p, grid, st);
}

}  // namespace pma
