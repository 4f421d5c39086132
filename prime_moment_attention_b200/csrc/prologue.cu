// prologue.cu -- the QK-norm pass in front of the tensor-core prefill (HBM-bound).
//
// The module applies LayerNorm over the head dim to q and k and scales q by 1/sqrt(D)
// (src/prime_moment_attention/attention.py:96-101) between the projections and the core.
// The CUDA-core kernels and the decode kernel fold that into their loads.  The tensor-core
// kernel's prep warps sit on its per-chunk critical path, so there the rows are normalised
// by this pass instead: one read of the raw projection rows (any strides, e.g. transposed
// views of [B,L,H,D]) and one write of contiguous bf16 [B,H,L,64] rows, which the core then
// reads through its tensor maps.  k keeps its H / kv_groups heads (the core maps query head h
// to kv head h / kv_groups), so no repeated copy is written.
//
// Layout: 8 lanes per 64-element bf16 row, 16 bytes each (lane & 7 = column chunk), 4 rows per
// warp instruction; a row's sums are joined over lane ^ 1, 2, 4.  Each lane keeps the weights
// of its 8 columns in registers for the whole launch.  Four row sets per iteration are loaded
// before any is reduced, to keep enough bytes in flight (64 KB per SM).
// Algorithmic traffic: 128 bytes read + 128 bytes written per row.
#include "pma_common.cuh"
#include "prefill.cuh"

namespace pma {

namespace {

constexpr int PD = 64;     // head dim of the tensor-core path
constexpr int UNROLL = 4;  // row sets per warp per iteration

__device__ __forceinline__ float2 u2f(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u));
}
__device__ __forceinline__ uint32_t f2u(float2 f) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
    return *reinterpret_cast<uint32_t *>(&h);
}

// rows = B * Hs * L rows of the source; dst is contiguous [B, Hs, L, 64].
__global__ void __launch_bounds__(256, 4) qk_norm_kernel(const __nv_bfloat16 *__restrict__ src, int64_t sb, int64_t sh,
                                                      int64_t sl, int Hs, int L, uint32_t rows,
                                                      const float *__restrict__ w, const float *__restrict__ b,
                                                      float eps, float scale, __nv_bfloat16 *__restrict__ dst) {
    const int lane = threadIdx.x & 31, cc = lane & 7, grp = lane >> 3;
    float2 w2[4], b2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int d = cc * 8 + 2 * i;
        w2[i] = make_float2((w ? w[d] : 1.f) * scale, (w ? w[d + 1] : 1.f) * scale);
        b2[i] = make_float2((w && b ? b[d] : 0.f) * scale, (w && b ? b[d + 1] : 0.f) * scale);
    }
    const uint32_t warp_g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
    // every lane of a warp runs the same trip count (the shuffles need the whole warp)
    for (uint32_t base = warp_g * 4 * UNROLL; base < rows; base += nwarps * 4 * UNROLL) {
        uint4 x[UNROLL];
        uint32_t r[UNROLL];
#pragma unroll
        for (int k = 0; k < UNROLL; ++k) {
            r[k] = base + 4 * k + grp;
            x[k] = make_uint4(0u, 0u, 0u, 0u);
            if (r[k] < rows) {
                const uint32_t t = r[k] % (uint32_t)L, bh = r[k] / (uint32_t)L;
                const uint32_t h = bh % (uint32_t)Hs, bi = bh / (uint32_t)Hs;
                x[k] = __ldcs(reinterpret_cast<const uint4 *>(src + bi * sb + h * sh + t * sl + cc * 8));
            }
        }
#pragma unroll
        for (int k = 0; k < UNROLL; ++k) {
            const float2 f[4] = {u2f(x[k].x), u2f(x[k].y), u2f(x[k].z), u2f(x[k].w)};
            float mean = 0.f, rstd = 1.f;
            if (w) {
                float s = ((f[0].x + f[0].y) + (f[1].x + f[1].y)) + ((f[2].x + f[2].y) + (f[3].x + f[3].y));
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                mean = s * (1.0f / PD);
                float v = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float dx = f[i].x - mean, dy = f[i].y - mean;
                    v = fmaf(dx, dx, fmaf(dy, dy, v));
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                rstd = rsqrtf(v * (1.0f / PD) + eps);
            }
            uint32_t o4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                o4[i] = f2u(make_float2(fmaf((f[i].x - mean) * rstd, w2[i].x, b2[i].x),
                                        fmaf((f[i].y - mean) * rstd, w2[i].y, b2[i].y)));
            if (r[k] < rows)
                *reinterpret_cast<uint4 *>(dst + (size_t)r[k] * PD + cc * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
        }
    }
}

}  // namespace

cudaError_t launch_qk_norm(const Seq &src, int B, int Hs, int L, const float *w, const float *b, float eps,
                           float scale, void *dst, int sms, cudaStream_t st) {
    const size_t rows = (size_t)B * Hs * L;
    if (rows == 0) return cudaSuccess;
    if (rows > 0x7fffffffu) return cudaErrorInvalidValue;  // 32-bit row indices
    const size_t per_block = 8 * 4 * UNROLL;  // rows one 256-thread block covers per iteration
    size_t blocks = (rows + per_block - 1) / per_block;
    const size_t cap = (size_t)sms * 4;       // 4 resident blocks of 256 threads per SM
    if (blocks > cap) blocks = cap;
    qk_norm_kernel<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16 *>(src.p), src.sb, src.sh,
                                                     src.sl, Hs, L, (uint32_t)rows, w, b, eps, scale,
                                                     reinterpret_cast<__nv_bfloat16 *>(dst));
    return cudaGetLastError();
}

}  // namespace pma
