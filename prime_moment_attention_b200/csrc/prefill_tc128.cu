// prefill_tc128.cu -- chunked prefill on tcgen05 tensor cores for head dim 128 (bf16 inputs).
//
// Same recurrence and rescaled operands as prefill_tc.cu (chunked_prime_ssd_core,
// src/prime_moment_attention/chunked_ssd.py:48-184), per 128-token chunk (n <= 128 valid tokens)
// with the 256 moment features psi(q) = [q | q^2/2], phi(k) = [k | k^2]:
//
//   g_i = l^(i+1),  w_j = l^(n-1-j) (0 past n),  QQ = [q | q^2/2],  KW = [w.k | w.k^2]   (bf16)
//   At   = QQ KW^T                      M = N = 128 tokens, K = 256        (:90-92)
//   P'   = l^-n At + l^-(1+j) for j <= i, else 0  (= l^(i-j) (1 + a_ij) / g_i), bf16
//   ACC  = QQ [S1;S2] + P' V            N = 128 values                     (:93-94, :139-148)
//   y_i  = g_i (ACC_i + S0) / max(g_i (sum_j P'_ij + QQ_i.Z + Z0), eps)    (:149-157)
//   dS   = KW^T V in two 128-feature halves (k, then k^2), K = 128 tokens  (:96-111)
//   S    = l^n S + dS,  Z = l^n Z + sum_j KW_j,  S0 = l^n S0 + sum_j w_j v_j,  Z0 = l^n Z0 + sum_j w_j
//                                                                          (:162-169)
// The column sums dZ = sum_j KW_j and dS0 = sum_j w_j v_j are N = 16 MMAs against a small operand
// whose rows are [1 | w_hi | w_lo] (w = w_hi + w_lo in two bf16 parts, so dS0 keeps float32
// weights), and the carry denominator QQ_i.Z one against the rows [Z_hi | Z_lo]; sum_j P'_ij is a
// CUDA-core sum.  The float32 state S1, S2
// [128 x 128] lives in registers (thread (quadrant qd, quarter g, lane) owns
// feature row 32 qd + lane, value columns 32 g .. 32 g + 31 of both), Z, S0, Z0 in shared memory.
// Head-states whose decay is below 0.55 (l^-128 would leave float32) run the float32 CUDA-core
// chunk loop (prefill_simt_body.cuh) inside this kernel.
//
// Shared memory (~210 KB): q, k (-> w.k in place), w.k^2 and v as [128 tokens x 64] bf16 tiles with
// the 128-byte swizzle (two per tensor: dims 0..63 and 64..127, each one TMA box), the bf16 state
// [S1;S2] as two [256 features x 64 values] MN-major tiles, the [16 x 128 tokens] sums operand and
// the [16 x 256 features] Z operand (both K-major), and the small vectors.
// Tensor memory (512 columns): At / P' 0..127 (after P' is formed: dZ in 64 and 80, dS0 in 97 + 98,
// QQ_i.Z in 112 + 113), dS 128..255, QQ 256..383, ACC 384..511.
//
// One CTA of 512 threads per (head-state, segment); the phases of a chunk are separated by
// barriers.  Thread 0 issues the TMA copies; lane 0 of warp 12 issues the MMAs.  Each CUDA-core
// phase waits only for the MMA group it reads and the groups that overlap it are issued at its
// start: the issuing thread blocks while the tensor core's queue is full, and warp 12 has the
// least CUDA-core work (its P' columns lie above the diagonal), so the other warps run meanwhile:
//   P1  QQ -> tensor memory, KW / KW.k in place, the w rows of the sums operand
//   M1  At = QQ KW^T, dS = (w.k)^T V                         (q of the next chunk is loaded)
//   P3  [issue ACC = QQ [S1;S2]]  P' and its row sums over At, S1 += dS
//   M2  dS = (w.k^2)^T V
//   P5a [issue ACC += P' V, dZ, dS0, QQ.Z]  S2 += dS, the bf16 state tiles for the next chunk
//   P5b Z (and its operand rows) and S0, the rows' denominators (k, v of the next chunk are loaded)
// and the output rows of chunk u run in chunk u+1's M1 window (ACC is untouched until its P3).
// The state-only pass (the segment carry's first launch) has no q, P', carry or output: after P1 it
// runs one MMA group, dS = (w.k | w.k^2)^T [V | 1] (N = 144: a ones tile in the unused state-tile
// space gives dZ as column 128) and dS0, then the state update.
// Every wait is bounded by the global timer; on expiry the kernel records a status code, leaves
// the chunk loop on every thread, and waits (bounded) for its copies and MMAs in flight before
// freeing tensor memory.
#include <cuda.h>

#include "prefill.cuh"
#include "prefill_simt_body.cuh"
#define PMA_FAULT_AT_EXIT 1  // report expired waits once per CTA, after the final barrier
#include "tc_common.cuh"

namespace pma {
namespace tc128 {

using namespace pma::tc;

constexpr int C = TC_CHUNK;             // 128 tokens per chunk
constexpr int D = 128;
constexpr int NT = 512;
constexpr int TILE = 128 * 128;         // [128 rows x 64] bf16, 128-byte swizzle: 16 KiB
constexpr int OFF_Q = 0;                // q: dims 0..63, then 64..127
constexpr int OFF_K = 2 * TILE;         // k, made w.k in place
constexpr int OFF_K2 = 4 * TILE;        // w.k^2
constexpr int OFF_V = 6 * TILE;         // v: values 0..63, then 64..127
constexpr int OFF_SB = 8 * TILE;        // bf16 [S1;S2]: [256 features x 64 values] per value half
constexpr int SB_HALF = 2 * TILE;
constexpr int OFF_WT = OFF_SB + 2 * SB_HALF;  // sums operand: rows 1, w_hi, w_lo; two 64-token atoms
constexpr int WT_ATOM = 2048;                  // [16 rows x 128 B] per atom
constexpr int OFF_ZT = OFF_WT + 2 * WT_ATOM;  // Z operand: rows Z_hi, Z_lo; four 64-feature atoms
constexpr int OFF_SMALL = OFF_ZT + 4 * WT_ATOM;
// L2 prefetch of the next chunk only (issued with its q copy): prefetching 4 chunks ahead raised
// the full pass's DRAM reads to 1.86x the bytes of q, k, v (lines evicted before their copy ran)
// and did not shorten it.
constexpr int PREFETCH = 0;
constexpr float LMIN = 0.55f;           // smallest decay the rescaled operands serve
constexpr uint32_t T_AT = 0, T_DS = 128, T_QQ = 256, T_ACC = 384, T_COLS = 512;
constexpr int ISSUER = 384;             // lane 0 of warp 12 (quadrant 0, columns 96..127)

// copies: q, k, v tiles; MMA groups (committed once per chunk each; M1B only drained on the way out)
enum { B_FQ, B_FK, B_FV, B_M1, B_M1B, B_M2, B_M3, B_NEVER, NBAR };

struct Small {
    uint64_t bar[NBAR];
    uint32_t tmem_base;
    CtlShared ctl;
    float pw[C + 4];                    // l^t, t = 0..C
    float geo[C + 4];                   // sum_{t<n} l^t
    alignas(16) float cinv[C];          // l^-(1+j)
    alignas(16) float zst[2 * D];       // Z = [Z1 ; Z2] entering the next P1
    alignas(16) float s0b[2][D];        // S0 entering the chunk, by chunk parity
    alignas(16) float z0b[4];           // Z0 entering the chunk, by chunk parity
    alignas(16) float rsp[4][C];        // per column quarter: partial sum_j P'_ij
};
constexpr size_t TC_BYTES = OFF_SMALL + sizeof(Small);
constexpr size_t FALLBACK_BYTES = SimtSmem<128, 32>::bytes;
constexpr size_t SMEM_BYTES = (TC_BYTES > FALLBACK_BYTES ? TC_BYTES : FALLBACK_BYTES) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

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

__device__ __forceinline__ void load32(const float *src, float (&v)[32]) {
    const float4 *s = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float4 t = s[c];
        v[4 * c] = t.x; v[4 * c + 1] = t.y; v[4 * c + 2] = t.z; v[4 * c + 3] = t.w;
    }
}
__device__ __forceinline__ void store32(float *dst, const float (&v)[32]) {
    float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int c = 0; c < 8; ++c) d[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// rows 0, 1 of the Z operand at feature f: Z_hi, Z_lo (K-major, 128-byte swizzle)
__device__ __forceinline__ void put_z(uint8_t *zt, int f, float z) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(z);
    const __nv_bfloat16 lo = __float2bfloat16_rn(z - __bfloat162float(hi));
    uint8_t *atom = zt + (f >> 6) * 2048;
    const int c = (f & 63) >> 3, e = f & 7;
    *reinterpret_cast<__nv_bfloat16 *>(atom + ((c ^ 0) << 4) + 2 * e) = hi;
    *reinterpret_cast<__nv_bfloat16 *>(atom + 128 + ((c ^ 1) << 4) + 2 * e) = lo;
}

// two consecutive float32 columns of this thread's TMEM lane, with the wait
__device__ __forceinline__ float2 tmem_ld2(uint32_t taddr) {
    uint32_t a, b;
    asm volatile("{\n\ttcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];\n\ttcgen05.wait::ld.sync.aligned;\n\t}"
                 : "=r"(a), "=r"(b)
                 : "r"(taddr)
                 : "memory");
    return make_float2(__uint_as_float(a), __uint_as_float(b));
}

// bounded wait used only on the way out (copies or MMAs that may still be in flight)
__device__ __forceinline__ void drain(uint64_t *b, uint32_t parity) {
    const unsigned long long t0 = gtimer();
    while (!mbar_try(b, parity) && gtimer() - t0 < WAIT_NS) {
    }
}

// SO: state only (no q, no output rows).  PRO: q scaled by p.pro.q_scale as the prep loads it (the
// host uses this only when the scale is exact in bf16, so the product rounds as in float32).
template <bool SO, typename TO, bool PRO>
__global__ void __launch_bounds__(NT, 1)
    prefill_tc128_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    Small &sm = *reinterpret_cast<Small *>(smem + OFF_SMALL);
    const uint32_t sb = su32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qd = warp & 3, g = warp >> 2;  // tensor-memory lane quadrant, column quarter
    const int fl = qd * 32 + lane;           // this thread's token row / feature row within a half
    const int bh = blockIdx.x, seg = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int hk = h / p.pro.groups;  // GQA: kv head of query head h
    const float lam = p.lambda[(int64_t)b * p.lam_sb + h];
    if (!(lam >= LMIN)) {  // small decay (or NaN): float32 CUDA-core chunk loop, whole CTA
        simt_prefill_body<128, 32, __nv_bfloat16, TO>(p, reinterpret_cast<float *>(smem), bh, seg);
        return;
    }

    const int nchunks_total = (p.L + C - 1) / C;
    const int seg_chunks = p.seg_len / C;
    const int c_begin = seg * seg_chunks;
    const int c_end = min(c_begin + seg_chunks, nchunks_total);
    const int U = max(c_end - c_begin, 0);
    const int n_last = U > 0 ? min(C, p.L - (c_end - 1) * C) : 0;
    Ctl ctl{&sm.ctl, p.status};
    uint64_t *bar = sm.bar;

    // ---- set-up: powers, barriers, tensor memory, the incoming state
    if (tid <= C) sm.pw[tid] = (float)pow((double)lam, (double)tid);
    if (tid < C) sm.cinv[tid] = (float)pow((double)lam, -1.0 - (double)tid);
    if (tid == 0) {
        for (int i = 0; i < NBAR; ++i) mbar_init(&bar[i], 1);
        init_ctl(sm.ctl, p.fault);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sm.tmem_base)),
                     "r"(T_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (p.test_wait_ns) {  // test hook: a wait expires before any copy or GEMM is issued
        tc_fence_before();
        __syncthreads();  // the barriers are initialised, tensor memory allocated
        tc_fence_after();
        if (tid == 0) expire_test_wait(&bar[B_NEVER], ctl, p.test_wait_ns, 90);
        __syncthreads();
        if (ctl.aborted()) {  // the whole CTA: nothing was issued, release tensor memory and leave
            if (warp == 0)
                asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sm.tmem_base), "r"(T_COLS)
                             : "memory");
            if (tid == 0) report_fault(sm.ctl.abort_flag, p.fault);
            return;
        }
    }
    float S1r[32], S2r[32];  // S1 / S2 [fl][32 g .. 32 g + 31]
    const bool has_in = !p.state_only && p.in.present();
    if (has_in) {
        const HeadPtrs src = p.in.at(bh, p.in.packed ? seg : 0, D);
        load32(src.S1 + fl * D + 32 * g, S1r);
        load32(src.S2 + fl * D + 32 * g, S2r);
        if (tid < 2 * D) sm.zst[tid] = tid < D ? src.Z1[tid] : src.Z2[tid - D];
        if (tid < D) sm.s0b[0][tid] = src.S0[tid];
        if (tid == 0) sm.z0b[0] = src.Z0[0];
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) S1r[e] = S2r[e] = 0.f;
        if (tid < 2 * D) sm.zst[tid] = 0.f;
        if (tid < D) sm.s0b[0][tid] = 0.f;
        if (tid == 0) sm.z0b[0] = 0.f;
    }
    for (int i = tid; i < 6 * WT_ATOM / 16; i += NT) {  // sums operand: row 0 ones; the rest zero
        const int r = (i >> 3) & 15;
        const uint32_t one2 = 0x3F803F80u;
        *reinterpret_cast<uint4 *>(smem + OFF_WT + 16 * i) =
            (r == 0 && i < 2 * WT_ATOM / 16) ? make_uint4(one2, one2, one2, one2) : make_uint4(0u, 0u, 0u, 0u);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
        float gs = 0.f;
        for (int j = 0; j <= C; ++j) {
            sm.geo[j] = gs;
            if (j < C) gs += sm.pw[j];
        }
    }
    const uint32_t tmem = sm.tmem_base;
    const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);

    // bf16 [S1;S2] rows fl and 128 + fl, values 32 g .. 32 g + 31, into the MN-major state tiles
    auto publish = [&]() {
        uint8_t *tile = smem + OFF_SB + (g >> 1) * SB_HALF;
        const int c0 = 4 * (g & 1);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            *reinterpret_cast<uint4 *>(tile + swz(fl, c0 + c)) = pack8(S1r + 8 * c);
            *reinterpret_cast<uint4 *>(tile + swz(D + fl, c0 + c)) = pack8(S2r + 8 * c);
        }
    };
    if (!SO) {
        publish();
        if (tid < 2 * D) put_z(smem + OFF_ZT, tid, sm.zst[tid]);
    } else {  // state only: the ones tile [128 tokens x 64], column 0 = 1, in the unused state-tile space
        for (int i = tid; i < TILE / 16; i += NT) {
            const int r = i >> 3, c = i & 7;  // element 0 of row r sits in chunk 0 ^ (r & 7)
            *reinterpret_cast<uint4 *>(smem + OFF_SB + 16 * i) = make_uint4(c == (r & 7) ? 0x3F80u : 0u, 0u, 0u, 0u);
        }
    }

    // ---- copies (thread 0)
    auto load_tile2 = [&](int off, const CUtensorMap *map, uint64_t *bb, int t0, int hh) {
        mbar_expect_tx(bb, 2 * TILE);
        tma_load(smem + off, map, bb, 0, t0, hh, b);
        tma_load(smem + off + TILE, map, bb, 64, t0, hh, b);
    };
    int fetched = 0;
    auto prefetch_to = [&](int upto) {
        for (; fetched < U && fetched <= upto; ++fetched) {
            const int tf = (c_begin + fetched) * C;
            for (int x = 0; x < 2; ++x) {
                if (!SO) tma_prefetch_l2(&tq, 64 * x, tf, h, b);
                tma_prefetch_l2(&tk, 64 * x, tf, hk, b);
                tma_prefetch_l2(&tv, 64 * x, tf, hk, b);
            }
        }
    };
    if (tid == 0 && U > 0) {
        prefetch_to(PREFETCH);
        const int t0 = c_begin * C;
        if (!SO) load_tile2(OFF_Q, &tq, &bar[B_FQ], t0, h);
        load_tile2(OFF_K, &tk, &bar[B_FK], t0, hk);
        load_tile2(OFF_V, &tv, &bar[B_FV], t0, hk);
    }
    // phases of the four barriers, and which of them have an operation in flight
    uint32_t ph_q = 0, ph_k = 0, ph_v = 0;
    bool pend_q = !SO && U > 0, pend_k = U > 0, pend_v = U > 0;
    int pend_m = -1;           // latest MMA commit not yet waited for (it covers every earlier MMA)
    uint32_t pend_par = 0;
    fence_proxy_async();  // the state tiles are read by the tensor core
    __syncthreads();

    // descriptors: compile-time upper words or'ed with the start address (16-byte units)
    constexpr uint32_t ID_SC = idesc(128, 128, 0, 0);  // QQ (tmem) KW^T
    constexpr uint32_t ID_DS = idesc(128, 128, 1, 1);  // (w.k)^T V: both MN-major
    constexpr uint32_t ID_TV = idesc(128, 128, 0, 1);  // QQ [S1;S2], P' V: B MN-major
    constexpr uint32_t ID_CS = idesc(128, 16, 1, 0);   // column sums: A MN-major, B K-major
    constexpr uint32_t ID_CZ = idesc(128, 16, 0, 0);   // QQ (tmem) [Z_hi | Z_lo]
    constexpr uint32_t ID_DZ = idesc(128, 144, 1, 1);  // state only: (w.k)^T [V | 1]
    constexpr uint64_t HI_KMAJ = desc_hi(16, 1024, 2);       // K-major, 128 B rows
    constexpr uint64_t HI_TILE2 = desc_hi(TILE, 1024, 2);    // MN-major, second 64-wide atom one tile on
    constexpr uint64_t HI_SB = desc_hi(SB_HALF, 1024, 2);    // MN-major state tiles
    const uint32_t a0 = sb >> 4;  // the allocation sits below 256 KiB: no field overflow
    auto dsc = [&](uint32_t off, uint64_t hi) { return (uint64_t)(a0 + (off >> 4)) | hi; };

    // Output rows of chunk uo from ACC (which no GEMM touches until the next chunk's carry GEMM is
    // issued in its P3): they run in the next chunk's M1 window, or after the loop for the last one.
    float den_prev = 0.f;
    auto output_rows = [&](int uo) {
        const int no = (uo == U - 1) ? n_last : C;
        float acc[32];
        tmem_ld32(lane_base + T_ACC + 32 * g, acc);
        const float gi = sm.pw[fl + 1];
        const float sc = gi / fmaxf(gi * den_prev, p.eps);
        const float *s0v = sm.s0b[uo & 1] + 32 * g;  // S0 entering chunk uo
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[e] = (acc[e] + s0v[e]) * sc;
        if (fl < no) {
            TO *yrow = reinterpret_cast<TO *>(p.y.p) + b * p.y.sb + h * p.y.sh +
                       (int64_t)((c_begin + uo) * C + fl) * p.y.sl + 32 * g;
            store_row32<TO>(yrow, acc);
        }
    };

    bool ok = true;
    for (int u = 0; u < U && ok; ++u) {
        const int n = (u == U - 1) ? n_last : C;
        const int par = u & 1;
        const float dec = sm.pw[n];  // l^n
        // ================= P1: this chunk's tiles
        {
            bool w = SO || mbar_wait(&bar[B_FQ], ph_q, ctl, 31);
            w = w && mbar_wait(&bar[B_FK], ph_k, ctl, 32) && mbar_wait(&bar[B_FV], ph_v, ctl, 33);
            if (!__syncthreads_and(w)) {
                ok = false;
                break;
            }
        }
        if (!SO) {
            ph_q ^= 1;
            pend_q = false;
        }
        ph_k ^= 1;
        ph_v ^= 1;
        pend_k = pend_v = false;
        if (!SO) {  // QQ row fl, features 64 g .. 64 g + 63 (tensor-memory columns 32 g ..)
            const uint8_t *qs = smem + OFF_Q + (g & 1) * TILE;
            const __nv_bfloat162 half2 = __float2bfloat162_rn(0.5f);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t r[16];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint4 v = *reinterpret_cast<const uint4 *>(qs + swz(fl, 4 * hh + c));
                    if (PRO) {
                        const __nv_bfloat162 sc = __float2bfloat162_rn(p.pro.q_scale);
                        v = make_uint4(as_u(__hmul2(as_b2(v.x), sc)), as_u(__hmul2(as_b2(v.y), sc)),
                                       as_u(__hmul2(as_b2(v.z), sc)), as_u(__hmul2(as_b2(v.w), sc)));
                    }
                    const uint32_t e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        uint32_t x = e[t];
                        if (g >= 2) {  // q*(q/2): one rounding
                            const __nv_bfloat162 qv = as_b2(x);
                            x = as_u(__hmul2(qv, __hmul2(qv, half2)));
                        }
                        r[4 * c + t] = x;
                    }
                }
                tmem_st16(lane_base + T_QQ + 32 * g + 16 * hh, r);
            }
        }
        {  // KW = w.k in place, K2W = KW.k (dims 16 dg .. 16 dg + 15 of token fl, dg = g, g + 4)
            const float wj = fl < n ? sm.pw[n - 1 - fl] : 0.f;
            const __nv_bfloat162 wb = __float2bfloat162_rn(wj);
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int dg = g + 4 * it;
                uint8_t *ks = smem + OFF_K + (dg >> 2) * TILE;
                uint8_t *k2s = smem + OFF_K2 + (dg >> 2) * TILE;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const uint32_t off = swz(fl, 2 * (dg & 3) + cc);
                    const uint4 x = *reinterpret_cast<const uint4 *>(ks + off);
                    const uint32_t e4[4] = {x.x, x.y, x.z, x.w};
                    uint32_t o1[4], o2[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const __nv_bfloat162 kv = as_b2(e4[c]);
                        const __nv_bfloat162 kw = __hmul2(kv, wb);
                        o1[c] = as_u(kw);
                        o2[c] = as_u(__hmul2(kw, kv));
                    }
                    *reinterpret_cast<uint4 *>(ks + off) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
                    *reinterpret_cast<uint4 *>(k2s + off) = make_uint4(o2[0], o2[1], o2[2], o2[3]);
                }
            }
            if (tid < C) {  // w_hi, w_lo of token tid: rows 1, 2 of the sums operand (K-major, swizzled)
                const __nv_bfloat16 whi = __float2bfloat16_rn(wj);
                const __nv_bfloat16 wlo = __float2bfloat16_rn(wj - __bfloat162float(whi));
                uint8_t *atom = smem + OFF_WT + (tid >> 6) * WT_ATOM;
                const int c = (tid & 63) >> 3, e = tid & 7;
                *reinterpret_cast<__nv_bfloat16 *>(atom + 1 * 128 + ((c ^ 1) << 4) + 2 * e) = whi;
                *reinterpret_cast<__nv_bfloat16 *>(atom + 2 * 128 + ((c ^ 2) << 4) + 2 * e) = wlo;
            }
        }
        if (!SO) tmem_wait_st();
        fence_proxy_async();  // w.k, w.k^2 are read by the tensor core
        tc_fence_before();
        __syncthreads();
        tc_fence_after();

        if constexpr (SO) {
            // ================= state only: one MMA group per chunk.  dS = (w.k | w.k^2)^T [V | 1]
            // (N = 144: the ones tile, in the state-tile space this mode leaves unused, is V's third
            // N-atom, so column 128 of each result is dZ) and dS0 = v^T [1 | w_hi | w_lo].
            if (tid == ISSUER) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {  // K = tokens, 16 rows = 2048 B per step
                    const uint64_t mk = (uint64_t)(k * 128);
                    mma_ss(tmem + T_DS, dsc(OFF_K, HI_TILE2) + mk, dsc(OFF_V, HI_TILE2) + mk, ID_DZ, k > 0);
                    mma_ss(tmem + T_DS + 144, dsc(OFF_K2, HI_TILE2) + mk, dsc(OFF_V, HI_TILE2) + mk, ID_DZ, k > 0);
                    mma_ss(tmem + T_AT + 96, dsc(OFF_V, HI_TILE2) + mk,
                           dsc(OFF_WT + (k >> 2) * WT_ATOM, HI_KMAJ) + (uint64_t)((k & 3) * 2), ID_CS, k > 0);
                }
                commit(&bar[B_M1]);
            }
            pend_m = B_M1;
            pend_par = par;
            if (tid == 0) {
                sm.z0b[par ^ 1] = fmaf(dec, sm.z0b[par], sm.geo[n]);
                prefetch_to(u + 1 + PREFETCH);
            }
            {
                const bool w = mbar_wait(&bar[B_M1], par, ctl, 37);
                if (!__syncthreads_and(w)) {
                    ok = false;
                    break;
                }
            }
            pend_m = -1;
            tc_fence_after();
            if (tid == 0 && u + 1 < U) {  // every GEMM of this chunk is complete: k, v tiles are free
                const int t1 = (c_begin + u + 1) * C;
                load_tile2(OFF_K, &tk, &bar[B_FK], t1, hk);
                load_tile2(OFF_V, &tv, &bar[B_FV], t1, hk);
            }
            if (u + 1 < U) pend_k = pend_v = true;
            {
                float ds[32];
                tmem_ld32(lane_base + T_DS + 32 * g, ds);
#pragma unroll
                for (int e = 0; e < 32; ++e) S1r[e] = fmaf(dec, S1r[e], ds[e]);
                tmem_ld32(lane_base + T_DS + 144 + 32 * g, ds);
#pragma unroll
                for (int e = 0; e < 32; ++e) S2r[e] = fmaf(dec, S2r[e], ds[e]);
            }
            if (g < 2) {  // Z1 / Z2 of feature fl: the ones column of each dS
                const float dz = tmem_ld1(lane_base + T_DS + 144 * g + 128);
                sm.zst[D * g + fl] = fmaf(dec, sm.zst[D * g + fl], dz);
            } else if (g == 2) {  // S0 of value fl: the w_hi and w_lo columns
                const float hi = tmem_ld1(lane_base + T_AT + 97);
                const float lo = tmem_ld1(lane_base + T_AT + 98);
                sm.s0b[par ^ 1][fl] = fmaf(dec, sm.s0b[par][fl], hi + lo);
            }
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            continue;
        }

        // ================= M1: At = QQ KW^T, dS = (w.k)^T V
        if (tid == ISSUER) {
            if (!SO) {
#pragma unroll
                for (int k = 0; k < 16; ++k) {  // K = features: w.k dims 0..63, 64..127, then w.k^2
                    const uint32_t toff = (k < 8 ? OFF_K : OFF_K2) + ((k >> 2) & 1) * TILE;
                    mma_ts(tmem + T_AT, tmem + T_QQ + 8 * k, dsc(toff, HI_KMAJ) + (uint64_t)((k & 3) * 2), ID_SC,
                           k > 0);
                }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k)  // K = tokens, 16 rows = 2048 B per step
                mma_ss(tmem + T_DS, dsc(OFF_K, HI_TILE2) + (uint64_t)(k * 128), dsc(OFF_V, HI_TILE2) + (uint64_t)(k * 128),
                       ID_DS, k > 0);
            commit(&bar[B_M1]);
        }
        if (tid == 0) {
            // the q tiles are consumed (QQ is in tensor memory): the next chunk's q lands now
            if (!SO && u + 1 < U) load_tile2(OFF_Q, &tq, &bar[B_FQ], (c_begin + u + 1) * C, h);
            prefetch_to(u + 1 + PREFETCH);
        }
        pend_m = B_M1;
        pend_par = par;
        if (!SO && u + 1 < U) pend_q = true;
        if (tid == 0) sm.z0b[par ^ 1] = fmaf(dec, sm.z0b[par], sm.geo[n]);
        if (!SO && u > 0) output_rows(u - 1);  // under the score and dS GEMMs
        {
            tc_fence_before();  // the ACC reads above precede this chunk's carry GEMM
            const bool w = mbar_wait(&bar[B_M1], par, ctl, 34);
            if (!__syncthreads_and(w)) {
                ok = false;
                break;
            }
        }
        tc_fence_after();

        // ================= P3: P' over At (row fl, columns 32 g ..), S1 += dS
        if (tid == ISSUER) {  // the carry GEMM runs under this phase
            if (!SO) {
#pragma unroll
                for (int k = 0; k < 16; ++k)  // K = features, 16 rows of the state tiles per step
                    mma_ts(tmem + T_ACC, tmem + T_QQ + 8 * k, dsc(OFF_SB, HI_SB) + (uint64_t)(k * 128), ID_TV, k > 0);
            }
            commit(&bar[B_M1B]);
        }
        pend_m = B_M1B;
        if (!SO) {
            const bool live = g <= qd;  // columns past the row quadrant are all masked
            uint32_t pk[16];
            float rs = 0.f;
            if (live) {
                float at[32];
                tmem_ld32(lane_base + T_AT + 32 * g, at);
                const float cn = 1.0f / dec;  // l^-n
                const float2 cn2 = make_float2(cn, cn);
                const int lim = fl - 32 * g;  // column 32 g + c belongs to row fl iff c <= lim
                const float4 *cv = reinterpret_cast<const float4 *>(sm.cinv + 32 * g);
#pragma unroll
                for (int c4 = 0; c4 < 8; ++c4) {
                    const float4 cj = cv[c4];
                    float2 lo = __ffma2_rn(cn2, make_float2(at[4 * c4], at[4 * c4 + 1]), make_float2(cj.x, cj.y));
                    float2 hi = __ffma2_rn(cn2, make_float2(at[4 * c4 + 2], at[4 * c4 + 3]), make_float2(cj.z, cj.w));
                    lo.x = 4 * c4 <= lim ? lo.x : 0.f;
                    lo.y = 4 * c4 + 1 <= lim ? lo.y : 0.f;
                    hi.x = 4 * c4 + 2 <= lim ? hi.x : 0.f;
                    hi.y = 4 * c4 + 3 <= lim ? hi.y : 0.f;
                    pk[2 * c4] = f2bf(lo);
                    pk[2 * c4 + 1] = f2bf(hi);
                    const float2 rl = bf2f(pk[2 * c4]), rh = bf2f(pk[2 * c4 + 1]);
                    rs += (rl.x + rl.y) + (rh.x + rh.y);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 16; ++c) pk[c] = 0u;
            }
            tc_fence_before();
            __syncthreads();  // every At column is read before P' overwrites columns 0..63
            tc_fence_after();
            tmem_st16(lane_base + T_AT + 16 * g, pk);
            sm.rsp[g][fl] = rs;
        }
        {
            float ds[32];
            tmem_ld32(lane_base + T_DS + 32 * g, ds);
#pragma unroll
            for (int e = 0; e < 32; ++e) S1r[e] = fmaf(dec, S1r[e], ds[e]);
        }
        if (!SO) tmem_wait_st();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();

        // ================= M2: dS = (w.k^2)^T V (its commit also covers the carry GEMM)
        if (tid == ISSUER) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                mma_ss(tmem + T_DS, dsc(OFF_K2, HI_TILE2) + (uint64_t)(k * 128),
                       dsc(OFF_V, HI_TILE2) + (uint64_t)(k * 128), ID_DS, k > 0);
            commit(&bar[B_M2]);
        }
        pend_m = B_M2;
        {
            const bool w = mbar_wait(&bar[B_M2], par, ctl, 35);
            if (!__syncthreads_and(w)) {
                ok = false;
                break;
            }
        }
        tc_fence_after();

        // ================= P5a: S2 += dS, the state tiles for the next chunk (the carry GEMM is done)
        if (tid == ISSUER) {  // M3 runs under this phase: ACC += P' V, column sums into free At columns
            if (!SO) {
#pragma unroll
                for (int k = 0; k < 8; ++k)  // K = tokens; P' packs 2 per column
                    mma_ts(tmem + T_ACC, tmem + T_AT + 8 * k, dsc(OFF_V, HI_TILE2) + (uint64_t)(k * 128), ID_TV, 1);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {  // [w.k | w.k^2 | v]^T [1 | w_hi | w_lo]
                const uint64_t bw = dsc(OFF_WT + (k >> 2) * WT_ATOM, HI_KMAJ) + (uint64_t)((k & 3) * 2);
                const uint64_t mk = (uint64_t)(k * 128);
                mma_ss(tmem + T_AT + 64, dsc(OFF_K, HI_TILE2) + mk, bw, ID_CS, k > 0);
                mma_ss(tmem + T_AT + 80, dsc(OFF_K2, HI_TILE2) + mk, bw, ID_CS, k > 0);
                mma_ss(tmem + T_AT + 96, dsc(OFF_V, HI_TILE2) + mk, bw, ID_CS, k > 0);
            }
            if (!SO) {
#pragma unroll
                for (int k = 0; k < 16; ++k)  // QQ [Z_hi | Z_lo]: K = features
                    mma_ts(tmem + T_AT + 112, tmem + T_QQ + 8 * k,
                           dsc(OFF_ZT + (k >> 2) * WT_ATOM, HI_KMAJ) + (uint64_t)((k & 3) * 2), ID_CZ, k > 0);
            }
            commit(&bar[B_M3]);
        }
        pend_m = B_M3;
        {
            float ds[32];
            tmem_ld32(lane_base + T_DS + 32 * g, ds);
#pragma unroll
            for (int e = 0; e < 32; ++e) S2r[e] = fmaf(dec, S2r[e], ds[e]);
        }
        if (!SO && u + 1 < U) {
            publish();
            fence_proxy_async();  // the state tiles are read by the next carry GEMM
        }
        {
            const bool w = mbar_wait(&bar[B_M3], par, ctl, 36);
            if (!__syncthreads_and(w)) {
                ok = false;
                break;
            }
        }
        pend_m = -1;
        tc_fence_after();

        // ================= P5b: next chunk's k / v, Z and S0, output rows
        if (tid == 0 && u + 1 < U) {  // every GEMM of this chunk is complete: k, v tiles are free
            const int t1 = (c_begin + u + 1) * C;
            load_tile2(OFF_K, &tk, &bar[B_FK], t1, hk);
            load_tile2(OFF_V, &tv, &bar[B_FV], t1, hk);
        }
        if (u + 1 < U) pend_k = pend_v = true;
        if (g < 2) {  // Z1 / Z2 of feature fl (column 0 of the sums: the ones row)
            const float dz = tmem_ld1(lane_base + T_AT + 64 + 16 * g);
            const float z = fmaf(dec, sm.zst[D * g + fl], dz);
            sm.zst[D * g + fl] = z;
            if (!SO && u + 1 < U) {
                put_z(smem + OFF_ZT, D * g + fl, z);
                fence_proxy_async();  // read by the next chunk's QQ.Z GEMM
            }
        } else if (g == 2) {  // S0 of value fl: the w_hi and w_lo columns
            const float hi = tmem_ld1(lane_base + T_AT + 97);
            const float lo = tmem_ld1(lane_base + T_AT + 98);
            sm.s0b[par ^ 1][fl] = fmaf(dec, sm.s0b[par][fl], hi + lo);
        }
        if (!SO) {  // row fl's denominator (its QQ.Z columns are overwritten by the next score GEMM)
            const float2 cz = tmem_ld2(lane_base + T_AT + 112);  // QQ_i.Z_hi, QQ_i.Z_lo
            den_prev = ((sm.rsp[0][fl] + sm.rsp[1][fl]) + (sm.rsp[2][fl] + sm.rsp[3][fl])) + (cz.x + cz.y) +
                       sm.z0b[par];
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }

    if (!SO && ok && U > 0) {
        tc_fence_after();
        output_rows(U - 1);
    }
    // ---- never leave with copies or GEMMs in flight (only a failed wait leaves any)
    if (tid == 0) {
        if (pend_q) drain(&bar[B_FQ], ph_q);
        if (pend_k) drain(&bar[B_FK], ph_k);
        if (pend_v) drain(&bar[B_FV], ph_v);
        if (pend_m >= 0) drain(&bar[pend_m], pend_par);
    }
    // ---- final state
    const bool write_out = ok && !ctl.aborted() && p.out.present() &&
                           (p.state_only || seg == (int)gridDim.y - 1);
    if (write_out) {
        const HeadPtrs dst = p.out.at(bh, p.out.packed ? seg : 0, D);
        store32(dst.S1 + fl * D + 32 * g, S1r);
        store32(dst.S2 + fl * D + 32 * g, S2r);
        if (tid < D) {
            dst.Z1[tid] = sm.zst[tid];
            dst.Z2[tid] = sm.zst[D + tid];
            dst.S0[tid] = sm.s0b[U & 1][tid];
        }
        if (tid == 0) dst.Z0[0] = sm.z0b[U & 1];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T_COLS) : "memory");
    if (tid == 0) report_fault(sm.ctl.abort_flag, p.fault);
}

template <bool SO, typename TO, bool PRO>
static cudaError_t launch_t(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                            const PrefillParams &p, dim3 grid, cudaStream_t st) {
    cudaError_t e = set_smem_once<prefill_tc128_kernel<SO, TO, PRO>>((int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    prefill_tc128_kernel<SO, TO, PRO><<<grid, NT, SMEM_BYTES, st>>>(mq, mk, mv, p);
    return cudaGetLastError();
}

}  // namespace tc128

bool tc128_supported(int idt) { return idt == PMA_BF16 && tc::tensor_maps_available(); }

cudaError_t launch_prefill_tc128(const PrefillParams &p, int ydt, dim3 grid, cudaStream_t st) {
    if (p.pro.qw || p.pro.kw || p.logdecay) return cudaErrorInvalidValue;  // planned for the CUDA-core kernel
    CUtensorMap mq, mk, mv;
    const int hkv = p.H / p.pro.groups;
    if (!tc::make_tile_map(&mk, p.k, p.B, hkv, p.L, 128) || !tc::make_tile_map(&mv, p.v, p.B, hkv, p.L, 128))
        return cudaErrorInvalidValue;
    const bool so = p.state_only || !p.y.p;
    if (!so) {
        if (!tc::make_tile_map(&mq, p.q, p.B, p.H, p.L, 128)) return cudaErrorInvalidValue;
    } else {
        mq = mk;
    }
    if (so) return launch_state_tc128(p, grid, st);
    if (p.pro.q_scale != 1.0f)
        return ydt == PMA_F32 ? tc128::launch_t<false, float, true>(mq, mk, mv, p, grid, st)
                              : tc128::launch_t<false, __nv_bfloat16, true>(mq, mk, mv, p, grid, st);
    return ydt == PMA_F32 ? tc128::launch_t<false, float, false>(mq, mk, mv, p, grid, st)
                          : tc128::launch_t<false, __nv_bfloat16, false>(mq, mk, mv, p, grid, st);
}

}  // namespace pma
