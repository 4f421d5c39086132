// prefill_tc.cu -- chunked prefill on tcgen05 tensor cores (bf16 inputs, D = 64).
//
// Same recurrence as chunked_prime_ssd_core (src/prime_moment_attention/chunked_ssd.py:48-184),
// evaluated per 128-token chunk with the moment features written as GEMMs:
//   psi(q) = [q | q^2/2],  phi(k) = [k | k^2]           (2D = 128 features)
//   A      = psi(Q) phi(K)^T                  M=128 tokens, N=128 tokens, K=128 features
//   P[i,j] = l^(i-j) (1 + A[i,j]),  j <= i    (decay mask, chunked_ssd.py:79-92)
//   num    = P V                              M=128, N=64,  K=128 tokens   (:93)
//   carry  = psi(Q) [S1; S2]                  M=128, N=64,  K=128 features (:139-148)
//   dS     = phi(K)^T (w . V), w_j = l^(n-1-j) M=128 features, N=64, K=128 tokens (:96-107)
//   y_i    = (num_i + l^(i+1) (S0 + carry_i)) / max(den_i + l^(i+1) (Z0 + psi(q_i).[Z1;Z2]), eps)
//   S      = l^n S + dS (float32, carried in registers of the state warpgroup)
// Operands are bf16 in shared memory (TMA tiles with the 128-byte swizzle, or
// tiles written by the kernel with the same swizzle); accumulators are float32
// in tensor memory.  The running state stays float32; a bf16 copy of it is the
// B operand of the carry GEMM.
//
// Warp roles (384 threads, one CTA per SM):
//   warp 0       TMA producer: q, k, v chunk tiles, two stages
//   warp 1       MMA issuer (one thread) and tensor-memory owner (512 columns)
//   warps 4-7    "prep" warpgroup: q^2/2, k^2, w.v tiles and the column sums that
//                update S0, Z1, Z2; then the decay-mask epilogue that turns A into
//                bf16 P and the per-token denominators
//   warps 8-11   "state" warpgroup: state update from dS (thread f owns feature row
//                f), bf16 state tile for the next carry GEMM, then the output epilogue
// Every wait on an mbarrier is bounded by the global timer; on expiry the kernel
// records a status code in the workspace header, every role stops, and the CTA
// waits for its in-flight copies and GEMMs before freeing tensor memory.
#include <cuda.h>

#include "prefill.cuh"

namespace pma {
namespace tc {

constexpr int C = TC_CHUNK;   // tokens per chunk
constexpr int D = 64;
constexpr int F = 2 * D;      // moment features
constexpr int TILE = C * D * 2;          // one [128 x 64] bf16 tile = 16 KiB
constexpr int STAGE = 3 * TILE;          // q, k, v
constexpr int OFF_Q2 = 2 * STAGE;        // q^2/2
constexpr int OFF_K2 = OFF_Q2 + TILE;    // k^2
constexpr int OFF_VW = OFF_K2 + TILE;    // w . v
constexpr int OFF_P = OFF_VW + TILE;     // P, two 64-column atoms
constexpr int OFF_SB = OFF_P + 2 * TILE; // bf16 state [128 features][64 values], two buffers
constexpr int OFF_SMALL = OFF_SB + 2 * TILE;

// Barriers with more than one waiting role exist once per chunk parity (..0/..1):
// a parity wait only sees the current or the previous phase, so a waiter must
// never fall two phases behind.  With one barrier per parity, the next completion
// of each is causally behind the waiter's own progress.
enum {
    B_FULL0, B_FULL1, B_EMPTY0, B_EMPTY1, B_PREP0, B_PREP1, B_DFREE, B_IFULL, B_IEMPTY, B_SREADY0, B_SREADY1,
    B_DSFULL, B_PREADY0, B_PREADY1, B_OFULL0, B_OFULL1, B_OEMPTY0, B_OEMPTY1, B_FINAL, NBAR
};

struct Small {
    uint64_t bar[20];
    float pw[C + 4];      // l^t, t = 0..C
    float geo[C + 4];     // sum_{t<n} l^t
    float den[2][C];      // intra-chunk denominators (per chunk parity)
    float cden[2][C];     // psi(q_i).[Z1;Z2] with the state entering the chunk
    float s0f[2][D];      // S0 entering the chunk (float32)
    float zf[2][F];       // [Z1; Z2] entering the chunk (float32)
    float zsum[2][3 * D]; // per chunk: sum w v | sum w k | sum w k^2
    float red[4][3 * D];  // per-warp partial column sums
    uint32_t tmem_base;
    int abort_flag;
};
constexpr size_t SMEM_BYTES = OFF_SMALL + sizeof(Small) + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

// tensor-memory columns
constexpr uint32_t T_A = 0, T_DS = 128, T_CARRY = 192, T_NUM = 320, T_COLS = 512;

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
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
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

struct Ctl {
    volatile int *abort_flag;  // shared: any role gave up
    int *status;               // global: first failure code (nullable)
};

// Wait for the phase of parity `parity` to complete.  Bounded by WAIT_NS; on
// expiry (or when another role already gave up) returns false.
__device__ __noinline__ bool mbar_wait(uint64_t *b, uint32_t parity, const Ctl &ctl, int code) {
    if (mbar_test(b, parity)) return true;
    const unsigned long long t0 = gtimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_test(b, parity)) return true;
        if ((it & 255) == 0) {
            if (*ctl.abort_flag) return false;
            if (gtimer() - t0 > WAIT_NS) {
                *ctl.abort_flag = 1;
                if (ctl.status) atomicCAS(ctl.status, 0, code);
                return false;
            }
        }
    }
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

// Shared-memory matrix descriptor: 128-byte swizzle, sm_100 version field.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, dense.
__host__ __device__ constexpr uint32_t idesc(int M, int N, int a_mn, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc)
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

__device__ __forceinline__ void unpack8(const uint4 u, float *f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ uint4 pack8(const float *f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}
// byte offset of 16-byte chunk `c` of row `r` in a [rows x 128 B] tile with the 128-byte swizzle
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

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
template <bool STATE_ONLY, typename TO>
__global__ void __launch_bounds__(384, 1)
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
    const int nchunks_total = (p.L + C - 1) / C;
    const int seg_chunks = p.seg_len / C;
    const int c_begin = seg * seg_chunks;
    const int c_end = min(c_begin + seg_chunks, nchunks_total);
    const int U = c_end - c_begin;
    Ctl ctl{&sm.abort_flag, p.status};

    if (threadIdx.x <= C) sm.pw[threadIdx.x] = (float)pow((double)lam, (double)threadIdx.x);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NBAR; ++i) {
            uint32_t n = 1;
            if (i == B_PREP0 || i == B_PREP1 || i == B_IEMPTY || i == B_SREADY0 || i == B_SREADY1 ||
                i == B_PREADY0 || i == B_PREADY1 || i == B_OEMPTY0 || i == B_OEMPTY1)
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
    __syncthreads();
    const uint32_t tmem = sm.tmem_base;
    uint64_t *bar = sm.bar;

    if (warp == 0) {
        // ============================== TMA producer
        if (lane == 0 && U > 0) {
            int issued = 0;
            for (int u = 0; u < U; ++u) {
                const int st = u & 1;
                if (!mbar_wait(&bar[B_EMPTY0 + st], ((u >> 1) & 1) ^ 1, ctl, 1)) break;
                const int t0 = (c_begin + u) * C;
                uint8_t *base = smem + st * STAGE;
                mbar_expect_tx(&bar[B_FULL0 + st], STATE_ONLY ? 2 * TILE : 3 * TILE);
                if (!STATE_ONLY) tma_load(base, &tq, &bar[B_FULL0 + st], 0, t0, h, b);
                tma_load(base + TILE, &tk, &bar[B_FULL0 + st], 0, t0, h, b);
                tma_load(base + 2 * TILE, &tv, &bar[B_FULL0 + st], 0, t0, h, b);
                issued = u + 1;
            }
            // never leave with copies in flight: the last (up to) two stages must have landed
            for (int u = max(0, issued - 2); u < issued; ++u) {
                const int st = u & 1;
                const unsigned long long t0 = gtimer();
                while (!mbar_test(&bar[B_FULL0 + st], (u >> 1) & 1) && gtimer() - t0 < WAIT_NS) {
                }
            }
        }
    } else if (warp == 1) {
        // ============================== MMA issuer
        if (lane == 0 && U > 0) {
            constexpr uint32_t ID_A = idesc(128, 128, 0, 0);   // psi(Q) phi(K)^T: both K-major
            constexpr uint32_t ID_DS = idesc(128, 64, 1, 1);   // phi(K)^T (w.V): both MN-major
            constexpr uint32_t ID_C = idesc(128, 64, 0, 1);    // psi(Q) S / P V: A K-major, B MN-major
            for (int u = 0; u < U; ++u) {
                const int st = u & 1;
                const uint32_t q_s = sb + st * STAGE, k_s = q_s + TILE, v_s = q_s + 2 * TILE;
                const uint32_t ph = (u >> 1) & 1;  // phase parity of the per-parity barriers
                if (!mbar_wait(&bar[B_PREP0 + st], ph, ctl, 2)) break;
                if (!STATE_ONLY) {
                    if (!mbar_wait(&bar[B_IEMPTY], (u & 1) ^ 1, ctl, 3)) break;
                    tc_fence_after();
                    // A = [Q | Q2] [K | K2]^T  (K-dim = features; 16 per instruction = 32 bytes)
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint32_t a = (s < 4 ? q_s : sb + OFF_Q2) + (s & 3) * 32;
                        const uint32_t bb = (s < 4 ? k_s : sb + OFF_K2) + (s & 3) * 32;
                        mma(tmem + T_A, sdesc(a, 16, 1024), sdesc(bb, 16, 1024), ID_A, s > 0);
                    }
                    commit(&bar[B_IFULL]);
                }
                if (!mbar_wait(&bar[B_SREADY0 + st], ph, ctl, 4)) break;
                if (!STATE_ONLY && !mbar_wait(&bar[B_OEMPTY0 + st], ph ^ 1, ctl, 5)) break;
                tc_fence_after();
                // dS = [K | K2]^T (w.V): A MN-major (features contiguous), K and K2 tiles are the
                // two 64-feature atoms (LBO = their distance); K-dim = tokens, 16 rows = 2048 B
                {
                    const uint32_t lbo = sb + OFF_K2 - k_s;
#pragma unroll
                    for (int s = 0; s < 8; ++s)
                        mma(tmem + T_DS, sdesc(k_s + s * 2048, lbo, 1024), sdesc(sb + OFF_VW + s * 2048, 8192, 1024),
                            ID_DS, s > 0);
                }
                commit(&bar[B_DSFULL]);
                if (!STATE_ONLY) {
                    // carry = [Q | Q2] [S1; S2] (state entering this chunk, bf16, [feature][value])
                    const uint32_t sbuf = sb + OFF_SB + (u & 1) * TILE;
                    const uint32_t tc_ = tmem + T_CARRY + st * 64;
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint32_t a = (s < 4 ? q_s : sb + OFF_Q2) + (s & 3) * 32;
                        mma(tc_, sdesc(a, 16, 1024), sdesc(sbuf + s * 2048, 8192, 1024), ID_C, s > 0);
                    }
                }
                commit(&bar[B_DFREE]);
                if (!STATE_ONLY) {
                    if (!mbar_wait(&bar[B_PREADY0 + st], ph, ctl, 6)) break;
                    tc_fence_after();
                    // num = P V: P K-major in two 64-token atoms; V MN-major
                    const uint32_t tn = tmem + T_NUM + st * 64;
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        const uint32_t a = sb + OFF_P + (s >> 2) * TILE + (s & 3) * 32;
                        mma(tn, sdesc(a, 16, 1024), sdesc(v_s + s * 2048, 8192, 1024), ID_C, s > 0);
                    }
                    commit(&bar[B_OFULL0 + st]);
                }
                commit(&bar[B_EMPTY0 + st]);
            }
            // every GEMM issued must be complete before tensor memory is released
            commit(&bar[B_FINAL]);
            const unsigned long long t0 = gtimer();
            while (!mbar_test(&bar[B_FINAL], 0) && gtimer() - t0 < WAIT_NS) {
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ============================== prep + decay-mask epilogue
        const int tid = threadIdx.x - 128, wq = warp - 4;
        const int cc = tid & 7, rb = tid >> 3;   // prep: 16-byte column chunk, block of 8 rows
        const int i = wq * 32 + lane;            // epilogue: token row (TMEM lane)
        for (int u = 0; u < U; ++u) {
            const int st = u & 1;
            const int t0 = (c_begin + u) * C;
            const int n = min(C, p.L - t0);
            uint8_t *q_s = smem + st * STAGE, *k_s = q_s + TILE, *v_s = q_s + 2 * TILE;
            if (!mbar_wait(&bar[B_FULL0 + st], (u >> 1) & 1, ctl, 7)) break;
            if (!mbar_wait(&bar[B_DFREE], (u & 1) ^ 1, ctl, 8)) break;
            // ---- prep: 8 rows x one 16-byte chunk per tile
            float zv[8], zk[8], zk2[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) zv[c] = zk[c] = zk2[c] = 0.f;
#pragma unroll 2
            for (int t = 0; t < 8; ++t) {
                const int r = rb * 8 + t;
                const uint32_t off = swz(r, cc);
                const float w = r < n ? sm.pw[n - 1 - r] : 0.f;
                float x[8], o[8];
                if (!STATE_ONLY) {
                    unpack8(*reinterpret_cast<const uint4 *>(q_s + off), x);
#pragma unroll
                    for (int c = 0; c < 8; ++c) o[c] = 0.5f * x[c] * x[c];
                    *reinterpret_cast<uint4 *>(smem + OFF_Q2 + off) = pack8(o);
                }
                unpack8(*reinterpret_cast<const uint4 *>(k_s + off), x);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    o[c] = x[c] * x[c];
                    zk[c] = fmaf(w, x[c], zk[c]);
                    zk2[c] = fmaf(w, o[c], zk2[c]);
                }
                *reinterpret_cast<uint4 *>(smem + OFF_K2 + off) = pack8(o);
                unpack8(*reinterpret_cast<const uint4 *>(v_s + off), x);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    o[c] = w * x[c];
                    zv[c] += o[c];
                }
                *reinterpret_cast<uint4 *>(smem + OFF_VW + off) = pack8(o);
            }
            // column sums: lanes sharing a chunk are lane ^ 8, lane ^ 16
#pragma unroll
            for (int c = 0; c < 8; ++c) {
#pragma unroll
                for (int o = 8; o <= 16; o <<= 1) {
                    zv[c] += __shfl_xor_sync(0xffffffffu, zv[c], o);
                    zk[c] += __shfl_xor_sync(0xffffffffu, zk[c], o);
                    zk2[c] += __shfl_xor_sync(0xffffffffu, zk2[c], o);
                }
            }
            named_bar(1, 128);  // the previous chunk's readers of red[] are done
            if (lane < 8) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    sm.red[wq][cc * 8 + c] = zv[c];
                    sm.red[wq][D + cc * 8 + c] = zk[c];
                    sm.red[wq][2 * D + cc * 8 + c] = zk2[c];
                }
            }
            named_bar(1, 128);
            for (int idx = tid; idx < 3 * D; idx += 128)
                sm.zsum[st][idx] = sm.red[0][idx] + sm.red[1][idx] + sm.red[2][idx] + sm.red[3][idx];
            fence_proxy_async();
            mbar_arrive(&bar[B_PREP0 + st]);
            if (STATE_ONLY) continue;

            // ---- decay mask: P[i][j] = l^(i-j) (1 + A[i][j]) for j <= i
            if (!mbar_wait(&bar[B_IFULL], u & 1, ctl, 9)) break;
            tc_fence_after();
            float den = 0.f;
#pragma unroll 1
            for (int g = 0; g < 4; ++g) {
                uint8_t *prow = smem + OFF_P + (g >> 1) * TILE;
                if (g > wq) {  // whole 32-column group above the diagonal for this warp
                    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) *reinterpret_cast<uint4 *>(prow + swz(i, 4 * (g & 1) + c4)) = z;
                    continue;
                }
                float a[32];
                tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + T_A + 32 * g, a);
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const int j = 32 * g + jj;
                    float pv = 0.f;
                    if (j <= i) pv = sm.pw[i - j] * (1.0f + a[jj]);
                    a[jj] = pv;
                    den += pv;
                }
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4)
                    *reinterpret_cast<uint4 *>(prow + swz(i, 4 * (g & 1) + c4)) = pack8(a + 8 * c4);
            }
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(&bar[B_IEMPTY]);
            // carried denominator needs the state entering this chunk
            if (!mbar_wait(&bar[B_SREADY0 + st], (u >> 1) & 1, ctl, 10)) break;
            float cd = 0.f;
            {
                const float *z1 = sm.zf[st], *z2 = sm.zf[st] + D;
#pragma unroll 2
                for (int c = 0; c < 8; ++c) {
                    float x[8];
                    unpack8(*reinterpret_cast<const uint4 *>(q_s + swz(i, c)), x);
#pragma unroll
                    for (int e = 0; e < 8; ++e) cd = fmaf(x[e], z1[8 * c + e], fmaf(0.5f * x[e] * x[e], z2[8 * c + e], cd));
                }
            }
            if (!mbar_wait(&bar[B_OEMPTY0 + st], ((u >> 1) & 1) ^ 1, ctl, 11)) break;
            sm.den[st][i] = den;
            sm.cden[st][i] = cd;
            mbar_arrive(&bar[B_PREADY0 + st]);
        }
    } else if (warp >= 8) {
        // ============================== state update + output epilogue
        const int wq = warp - 8;
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
        auto publish = [&](int buf) {  // bf16 state tile + float32 vectors for the next chunk
            uint8_t *srow = smem + OFF_SB + buf * TILE;
#pragma unroll
            for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4 *>(srow + swz(f, c)) = pack8(S + 8 * c);
            sm.zf[buf][f] = Z;
            if (f < D) sm.s0f[buf][f] = s0;
        };
        if (!STATE_ONLY) publish(0);
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(&bar[B_SREADY0]);
        bool ok = true;
        for (int u = 0; u < U && ok; ++u) {
            const int st = u & 1;
            const int t0 = (c_begin + u) * C;
            const int n = min(C, p.L - t0);
            // ---- state update
            if (!mbar_wait(&bar[B_DSFULL], u & 1, ctl, 12) || !mbar_wait(&bar[B_PREP0 + st], (u >> 1) & 1, ctl, 13)) {
                ok = false;
                break;
            }
            tc_fence_after();
            named_bar(2, 128);  // every thread finished reading the buffers about to be rewritten
            const float decay = sm.pw[n];
#pragma unroll
            for (int hcol = 0; hcol < 2; ++hcol) {
                float d[32];
                tmem_ld32(lane_base + T_DS + 32 * hcol, d);
#pragma unroll
                for (int e = 0; e < 32; ++e) S[32 * hcol + e] = fmaf(decay, S[32 * hcol + e], d[e]);
            }
            Z = fmaf(decay, Z, sm.zsum[st][D + f]);
            if (f < D) s0 = fmaf(decay, s0, sm.zsum[st][f]);
            const float Z0_in = Z0;
            Z0 = fmaf(decay, Z0, sm.geo[n]);
            if (!STATE_ONLY) publish(st ^ 1);
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(&bar[B_SREADY0 + (st ^ 1)]);
            if (STATE_ONLY) continue;
            // ---- output rows
            if (!mbar_wait(&bar[B_OFULL0 + st], (u >> 1) & 1, ctl, 14) ||
                !mbar_wait(&bar[B_PREADY0 + st], (u >> 1) & 1, ctl, 15)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int i = f;
            const float g = sm.pw[i + 1];
            const float dd = fmaxf(sm.den[st][i] + g * (Z0_in + sm.cden[st][i]), p.eps);
            const float inv = 1.0f / dd;
            TO *yrow = reinterpret_cast<TO *>(p.y.p) + b * p.y.sb + h * p.y.sh + (int64_t)(t0 + i) * p.y.sl;
            const float *s0in = sm.s0f[st];
#pragma unroll
            for (int hcol = 0; hcol < 2; ++hcol) {
                float cr[32], nm[32];
                tmem_ld32(lane_base + T_CARRY + st * 64 + 32 * hcol, cr);
                tmem_ld32(lane_base + T_NUM + st * 64 + 32 * hcol, nm);
#pragma unroll
                for (int e = 0; e < 32; ++e) nm[e] = (nm[e] + g * (s0in[32 * hcol + e] + cr[e])) * inv;
                if (i < n) store_row32<TO>(yrow + 32 * hcol, nm);
            }
            tc_fence_before();
            mbar_arrive(&bar[B_OEMPTY0 + st]);
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
    kern<<<grid, 384, SMEM_BYTES, st>>>(mq, mk, mv, p);
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
