// prefill_simt.cu -- chunked prefill in float32 on CUDA cores (float32 inputs and
// head dims other than 64), and the segment machinery shared by all prefill
// kernels: state-only pass, segment prefix, state combine.
//
// The 1e-4 parity bar for float32 inputs rules out bf16/tf32 tensor-core
// operands, so float32 inputs are computed here with float32 arithmetic.
#include "pma_common.cuh"
#include "prefill.cuh"
#include "prefill_simt_body.cuh"

namespace pma {

// Threads per CTA: at D = 128 one CTA fills an SM's shared memory, so it runs 16 warps to hide
// the shared-memory latency of its float32 tiles (measured 18 % faster than 8 warps); smaller D
// keep 8 warps (two CTAs per SM at D <= 64).
template <int D> constexpr int simt_threads() { return D >= 128 ? 512 : 256; }

template <int D, int C, typename TI, typename TO, bool PT>
__global__ void __launch_bounds__(simt_threads<D>()) prefill_simt_kernel(const PrefillParams p) {
    extern __shared__ float4 smem4[];
    simt_prefill_body<D, C, TI, TO, PT>(p, reinterpret_cast<float *>(smem4), blockIdx.x, blockIdx.y);
}

// ---------------------------------------------------------------------------
// Segment prefix: ws holds, per head-state, the states T_s each segment builds
// from zero (slots 0..nseg-2, written by a state-only pass).  Replace them in
// place by the state entering each segment:
//   P_0 = state_in (or 0);  P_{s+1} = l^{len_s} P_s + T_s
// and optionally write P_nseg (the final state, when T_{nseg-1} is present) to
// the user's state_out.  One thread per (head-state, float); one block per head-state
// and 256 floats (blockIdx.x = head-state), so the decay powers are computed once per
// block (in double, then rounded) instead of once per float.
// ---------------------------------------------------------------------------
constexpr int kCarryThreads = 256;

__global__ void segment_prefix_kernel(int BH, int H, int D, int nseg, int seg_len, int L, float *ws,
                                      StateRef in, StateRef final_out, const float *lambda, int64_t lam_sb) {
    __shared__ float pw[2];  // l^seg_len, l^(length of the last segment)
    const size_t F = state_floats(D);
    const int bh = blockIdx.x;
    const int b = bh / H, h = bh - b * H;
    if (threadIdx.x < 2) {
        const double lam = lambda[(int64_t)b * lam_sb + h];
        pw[threadIdx.x] = (float)pow(lam, (double)(threadIdx.x == 0 ? seg_len : L - (nseg - 1) * seg_len));
    }
    __syncthreads();
    const size_t fi = (size_t)blockIdx.y * blockDim.x + threadIdx.x;
    if (fi >= F) return;
    const int f = (int)fi;
    // packed index f -> component pointer offset in a HeadPtrs
    auto comp = [&](const HeadPtrs &hp) -> float * {
        const int DD = D * D;
        if (f < DD) return hp.S1 + f;
        if (f < 2 * DD) return hp.S2 + (f - DD);
        const int r = f - 2 * DD;
        if (r < D) return hp.S0 + r;
        if (r < 2 * D) return hp.Z1 + (r - D);
        if (r < 3 * D) return hp.Z2 + (r - 2 * D);
        return hp.Z0;
    };
    float P = in.present() ? *comp(in.at(bh, 0, D)) : 0.f;
    const size_t FS = slot_floats(D);
    float *base = ws + (size_t)bh * nseg * FS + f;
    const int nprefix = final_out.present() ? nseg : nseg - 1;
    for (int sg = 0; sg < nseg; ++sg) {
        float T = 0.f;
        if (sg < nprefix) T = base[(size_t)sg * FS];
        base[(size_t)sg * FS] = P;
        if (sg < nprefix) P = fmaf(pw[sg == nseg - 1 ? 1 : 0], P, T);
    }
    if (final_out.present()) *comp(final_out.at(bh, 0, D)) = P;
}

// ws[s] += l^(s * seg_len) * P_in: the states entering the segments, left in the workspace by a
// state-only call from a zero start (segment_prefix_kernel), shifted to the incoming state P_in.
// Every component of the recurrence decays by l per token, so a start state P_in adds l^t P_in
// to the state after t tokens.
__global__ void segment_resume_kernel(int BH, int H, int D, int nseg, int seg_len, float *ws, StateRef in,
                                      const float *lambda, int64_t lam_sb) {
    __shared__ float pw[kCarryThreads];  // l^(s * seg_len), s < nseg (nseg <= the SM count < 256)
    const size_t F = state_floats(D);
    const int bh = blockIdx.x;
    const int b = bh / H, h = bh - b * H;
    if (threadIdx.x < nseg)
        pw[threadIdx.x] = (float)pow((double)lambda[(int64_t)b * lam_sb + h], (double)threadIdx.x * seg_len);
    __syncthreads();
    const size_t fi = (size_t)blockIdx.y * blockDim.x + threadIdx.x;
    if (fi >= F) return;
    const int f = (int)fi;
    const HeadPtrs hp = in.at(bh, 0, D);
    const int DD = D * D;
    float P;
    if (f < DD) P = hp.S1[f];
    else if (f < 2 * DD) P = hp.S2[f - DD];
    else {
        const int r = f - 2 * DD;
        P = r < D ? hp.S0[r] : (r < 2 * D ? hp.Z1[r - D] : (r < 3 * D ? hp.Z2[r - 2 * D] : hp.Z0[0]));
    }
    const size_t FS = slot_floats(D);
    float *base = ws + (size_t)bh * nseg * FS + f;
    for (int sg = 0; sg < nseg; ++sg) base[(size_t)sg * FS] = fmaf(pw[sg], P, base[(size_t)sg * FS]);
}

// P <- l^len[b] P + T over user-layout states (pma_state_combine).
__global__ void state_combine_kernel(int BH, int H, int D, const float *lambda, int64_t lam_sb, double len,
                                     pma_state T, pma_state P) {
    __shared__ float pa;  // l^len of this head-state
    const size_t F = state_floats(D);
    const int bh = blockIdx.x;
    const int b = bh / H, h = bh - b * H;
    if (threadIdx.x == 0) pa = (float)pow((double)lambda[(int64_t)b * lam_sb + h], len);
    __syncthreads();
    const size_t fi = (size_t)blockIdx.y * blockDim.x + threadIdx.x;
    if (fi >= F) return;
    const int f = (int)fi;
    const float a = pa;
    const int DD = D * D;
    float *pp;
    const float *tp;
    if (f < DD) { pp = P.S1 + (size_t)bh * DD + f; tp = T.S1 + (size_t)bh * DD + f; }
    else if (f < 2 * DD) { pp = P.S2 + (size_t)bh * DD + f - DD; tp = T.S2 + (size_t)bh * DD + f - DD; }
    else {
        const int r = f - 2 * DD;
        if (r < D) { pp = P.S0 + (size_t)bh * D + r; tp = T.S0 + (size_t)bh * D + r; }
        else if (r < 2 * D) { pp = P.Z1 + (size_t)bh * D + r - D; tp = T.Z1 + (size_t)bh * D + r - D; }
        else if (r < 3 * D) { pp = P.Z2 + (size_t)bh * D + r - 2 * D; tp = T.Z2 + (size_t)bh * D + r - 2 * D; }
        else { pp = P.Z0 + bh; tp = T.Z0 + bh; }
    }
    *pp = fmaf(a, *pp, *tp);
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
template <int D, int C, typename TI, typename TO, bool PT>
static cudaError_t launch_simt_pt(const PrefillParams &p, dim3 grid, cudaStream_t st) {
    const size_t smem = SimtSmem<D, C>::bytes;
    auto kern = prefill_simt_kernel<D, C, TI, TO, PT>;
    cudaError_t e = set_smem_once<prefill_simt_kernel<D, C, TI, TO, PT>>((int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, simt_threads<D>(), smem, st>>>(p);
    return cudaGetLastError();
}

template <int D, int C, typename TI, typename TO>
static cudaError_t launch_simt_t(const PrefillParams &p, dim3 grid, cudaStream_t st) {
    return p.logdecay ? launch_simt_pt<D, C, TI, TO, true>(p, grid, st) : launch_simt_pt<D, C, TI, TO, false>(p, grid, st);
}

template <int D, int C>
static cudaError_t launch_simt_d(const PrefillParams &p, int idt, int ydt, dim3 grid, cudaStream_t st) {
    if (idt == PMA_F32)
        return ydt == PMA_F32 ? launch_simt_t<D, C, float, float>(p, grid, st)
                              : launch_simt_t<D, C, float, __nv_bfloat16>(p, grid, st);
    return ydt == PMA_F32 ? launch_simt_t<D, C, __nv_bfloat16, float>(p, grid, st)
                          : launch_simt_t<D, C, __nv_bfloat16, __nv_bfloat16>(p, grid, st);
}

int simt_chunk(int D) { return D >= 128 ? 32 : 64; }

cudaError_t launch_prefill_simt(const PrefillParams &p, int D, int idt, int ydt, dim3 grid, cudaStream_t st) {
    switch (D) {
        case 16: return launch_simt_d<16, 64>(p, idt, ydt, grid, st);
        case 32: return launch_simt_d<32, 64>(p, idt, ydt, grid, st);
        case 64: return launch_simt_d<64, 64>(p, idt, ydt, grid, st);
        case 128: return launch_simt_d<128, 32>(p, idt, ydt, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_segment_prefix(int BH, int H, int D, int nseg, int seg_len, int L, float *ws, const StateRef &in,
                                  const StateRef &final_out, const float *lambda, int64_t lam_sb, cudaStream_t st) {
    const dim3 grid((unsigned)BH, (unsigned)((state_floats(D) + kCarryThreads - 1) / kCarryThreads));
    segment_prefix_kernel<<<grid, kCarryThreads, 0, st>>>(BH, H, D, nseg, seg_len, L, ws, in, final_out, lambda, lam_sb);
    return cudaGetLastError();
}

cudaError_t launch_segment_resume(int BH, int H, int D, int nseg, int seg_len, float *ws, const StateRef &in,
                                  const float *lambda, int64_t lam_sb, cudaStream_t st) {
    if (nseg > kCarryThreads) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)BH, (unsigned)((state_floats(D) + kCarryThreads - 1) / kCarryThreads));
    segment_resume_kernel<<<grid, kCarryThreads, 0, st>>>(BH, H, D, nseg, seg_len, ws, in, lambda, lam_sb);
    return cudaGetLastError();
}

cudaError_t launch_state_combine(int B, int H, int D, const float *lambda, int64_t lam_sb, int64_t len,
                                 const pma_state &T, const pma_state &P, cudaStream_t st) {
    const dim3 grid((unsigned)(B * H), (unsigned)((state_floats(D) + kCarryThreads - 1) / kCarryThreads));
    state_combine_kernel<<<grid, kCarryThreads, 0, st>>>(B * H, H, D, lambda, lam_sb, (double)len, T, P);
    return cudaGetLastError();
}

}  // namespace pma
