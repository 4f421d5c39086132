// decode.cu -- one recurrent decode step for N x H head-states (HBM-bound).
//
// Replaces the L == 1 branch of PrimeMomentAttention.forward
// (src/prime_moment_attention/attention.py:120-143), which runs ~14 eager ATen
// kernels that each stream the whole state and allocate new tensors.  Here one
// warp owns one head-state and makes exactly one read and one write pass over it:
//
//   for every row d of S1/S2 (key index) and column e (value index):
//       S1[d][e] = l S1[d][e] + k_d v_e          S2[d][e] = l S2[d][e] + k_d^2 v_e
//       num[e]  += q_d S1[d][e] + 0.5 q_d^2 S2[d][e]     (on the updated values)
//   den = max(l Z0 + 1 + sum_d q_d (l Z1_d + k_d) + 0.5 q_d^2 (l Z2_d + k_d^2), eps)
//   y[e] = (l S0[e] + v_e + num[e]) / den
//
// Layout per warp (D = 64): 16 lanes cover one 256-byte row with float4 accesses,
// so one warp instruction moves two rows (512 contiguous bytes); each lane walks
// 32 rows of S1 and S2, keeping 8 rows (16 float4) in flight before it computes.
// The column partial sums of the two half-warps are joined with one shuffle.
// Algorithmic traffic per head-state: 2 * (2D^2 + 3D + 1) * 4 bytes of state
// (read + write) plus q, k, v in and y out.  With a row table the state of batch row n
// is row rows[n] of a larger state pool (serving: sequences keep their pool slot while
// the batch composition changes); the traffic is the same.
#include "pma_common.cuh"
#include "prefill.cuh"

namespace pma {

template <int D, typename TI, typename TO>
__global__ void __launch_bounds__(256) decode_step_kernel(const DecodeParams p) {
    constexpr int LPR = D / 4;        // lanes per row (one float4 each)
    constexpr int RPI = 32 / LPR;     // rows one warp instruction covers
    constexpr int RPL = D / RPI;      // rows each lane walks
    constexpr int BATCH = RPL < 8 ? RPL : 8;
    static_assert(D % 4 == 0 && 32 % LPR == 0, "unsupported head dim");

    __shared__ float sq[8][D], sk[8][D];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bidx = blockIdx.x * 8 + warp;         // batch row n and head h: n*H + h
    if (bidx >= p.N * p.H) return;
    const int n = bidx / p.H, h = bidx - n * p.H;
    // state row: n itself, or rows[n] of a state pool (rows outside the pool are skipped)
    int srow = n;
    if (p.rows) {
        srow = p.rows[n];
        if (srow < 0 || srow >= p.pool_rows) return;
    }
    const int idx = srow * p.H + h;                  // head-state index in the state arrays
    const float lraw = p.lambda[(int64_t)n * p.lam_sn + h];
    const float lam = p.log_lambda ? expf(lraw) : lraw;
    // second moments: k^2 v added with c2, read out with cq (moment layout 1, 1/2; selective 1/2, 1)
    const float c2 = p.half_sq ? 0.5f : 1.0f, cq = p.half_sq ? 1.0f : 0.5f;

    const TI *qp = reinterpret_cast<const TI *>(p.q.p) + n * p.q.sb + h * p.q.sh;
    const int hk = h / p.pro.groups;                 // GQA: the kv head this query head reads
    const TI *kp = reinterpret_cast<const TI *>(p.k.p) + n * p.k.sb + hk * p.k.sh;
    const TI *vp = reinterpret_cast<const TI *>(p.v.p) + n * p.v.sb + hk * p.v.sh;
    for (int d = lane; d < D; d += 32) {
        sq[warp][d] = Elem<TI>::to_f(qp[d]);
        sk[warp][d] = Elem<TI>::to_f(kp[d]);
    }
    __syncwarp();
    // prologue: q -> LN(q) * scale, k -> LN(k); each lane rewrites the elements it loaded
    if (p.pro.q_work()) {
        const float2 st = p.pro.qw ? warp_row_stats<D>(sq[warp], p.pro.ln_eps, lane) : make_float2(0.f, 1.f);
        for (int d = lane; d < D; d += 32)
            sq[warp][d] = prologue_elem(sq[warp][d], st, p.pro.qw, p.pro.qb, d, p.pro.q_scale);
    }
    if (p.pro.k_work() || p.k_head_scale) {
        const float ks = p.k_head_scale ? p.k_head_scale[h] : 1.f;
        const float2 st = p.pro.kw ? warp_row_stats<D>(sk[warp], p.pro.ln_eps, lane) : make_float2(0.f, 1.f);
        for (int d = lane; d < D; d += 32) sk[warp][d] = prologue_elem(sk[warp][d], st, p.pro.kw, p.pro.kb, d, ks);
    }
    __syncwarp();

    const int r0 = lane / LPR, c0 = (lane % LPR) * 4;
    const float4 v4 = load4(vp + c0);
    const size_t soff = (size_t)idx * D * D;
    const float *S1i = p.in.S1 + soff, *S2i = p.in.S2 + soff;
    float *S1o = p.out.S1 + soff, *S2o = p.out.S2 + soff;

    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i0 = 0; i0 < RPL; i0 += BATCH) {
        float4 a[BATCH], b[BATCH];
#pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            const int d = r0 + RPI * (i0 + j);
            a[j] = ldcs4(S1i + d * D + c0);
            b[j] = ldcs4(S2i + d * D + c0);
        }
#pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            const int d = r0 + RPI * (i0 + j);
            const float kd = sk[warp][d], qd = sq[warp][d];
            const float kd2 = c2 * kd * kd, qh2 = cq * qd * qd;
            float4 s1 = fma4(lam, a[j], scale4(kd, v4));
            float4 s2 = fma4(lam, b[j], scale4(kd2, v4));
            stcs4(S1o + d * D + c0, s1);
            stcs4(S2o + d * D + c0, s2);
            acc = fma4(qd, s1, acc);
            acc = fma4(qh2, s2, acc);
        }
    }
    // join the RPI row groups that share columns c0..c0+3
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
    }

    // vectors: Z1, Z2 and the denominator
    const size_t voff = (size_t)idx * D;
    float dpart = 0.f;
    for (int d = lane; d < D; d += 32) {
        const float kd = sk[warp][d], qd = sq[warp][d];
        const float z1 = fmaf(lam, p.in.Z1[voff + d], kd);
        const float z2 = fmaf(lam, p.in.Z2[voff + d], c2 * kd * kd);
        p.out.Z1[voff + d] = z1;
        p.out.Z2[voff + d] = z2;
        dpart = fmaf(qd, z1, fmaf(cq * qd * qd, z2, dpart));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dpart += __shfl_xor_sync(0xffffffffu, dpart, o);
    const float z0 = fmaf(lam, p.in.Z0[idx], 1.0f);
    const float den = fmaxf(z0 + dpart, p.eps);
    __syncwarp();
    if (lane == 0) p.out.Z0[idx] = z0;

    if (r0 == 0) {
        const float4 s0 = fma4(lam, load4(p.in.S0 + voff + c0), v4);
        store4(p.out.S0 + voff + c0, s0);
        const float inv = 1.0f / den;
        float4 yv = make_float4((s0.x + acc.x) * inv, (s0.y + acc.y) * inv, (s0.z + acc.z) * inv,
                                (s0.w + acc.w) * inv);
        TO *yp = reinterpret_cast<TO *>(p.y.p) + n * p.y.sb + h * p.y.sh;
        store4(yp + c0, yv);
    }
}

template <int D, typename TI>
static cudaError_t launch_decode_t(const DecodeParams &p, int ydt, cudaStream_t s) {
    const int grid = (p.N * p.H + 7) / 8;
    if (ydt == PMA_F32)
        decode_step_kernel<D, TI, float><<<grid, 256, 0, s>>>(p);
    else
        decode_step_kernel<D, TI, __nv_bfloat16><<<grid, 256, 0, s>>>(p);
    return cudaGetLastError();
}

template <int D>
static cudaError_t launch_decode_d(const DecodeParams &p, int idt, int ydt, cudaStream_t s) {
    return idt == PMA_F32 ? launch_decode_t<D, float>(p, ydt, s) : launch_decode_t<D, __nv_bfloat16>(p, ydt, s);
}

cudaError_t launch_decode(const DecodeParams &p, int D, int idt, int ydt, cudaStream_t s) {
    switch (D) {
        case 16: return launch_decode_d<16>(p, idt, ydt, s);
        case 32: return launch_decode_d<32>(p, idt, ydt, s);
        case 64: return launch_decode_d<64>(p, idt, ydt, s);
        case 128: return launch_decode_d<128>(p, idt, ydt, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace pma
