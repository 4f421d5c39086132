// swiglu.cu -- silu(gate) * up in one pass: the SwiGLU activation of the model's MLP
// (PrimeMLP.forward, src/prime_moment_attention/model.py:59-68: down_proj(silu(gate_proj(x)) *
// up_proj(x))).  PyTorch runs it as two elementwise kernels (silu into a temporary, then the
// product); here each element is read once and written once.
//
// Arithmetic as PyTorch's kernels do it: silu(a) = a / (1 + exp(-a)) in float32 with the accurate
// exp, rounded to the storage type, then the product in float32, rounded again -- so bf16 and
// float32 results equal the two-kernel sequence element for element.
#include "prefill.cuh"

namespace pma {
namespace {

template <typename T>
__device__ __forceinline__ float silu_mul(T g, T u) {
    const float a = Elem<T>::to_f(g);
    const T s = Elem<T>::from_f(a / (1.0f + expf(-a)));
    return Elem<T>::to_f(s) * Elem<T>::to_f(u);
}

// 16-byte vectors: every row start and stride is a multiple of 16 bytes and inter of the vector width
template <typename T>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(const T *__restrict__ g, int64_t gs, const T *__restrict__ u,
                                                        int64_t us, T *__restrict__ o, int64_t os, int64_t rows,
                                                        int inter) {
    constexpr int V = 16 / sizeof(T);
    const int per_row = inter / V;
    const int64_t total = rows * per_row;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / per_row;
        const int c = (int)(i - r * per_row) * V;
        const uint4 gv = __ldg(reinterpret_cast<const uint4 *>(g + r * gs + c));
        const uint4 uv = __ldg(reinterpret_cast<const uint4 *>(u + r * us + c));
        const T *ge = reinterpret_cast<const T *>(&gv);
        const T *ue = reinterpret_cast<const T *>(&uv);
        uint4 ov;
        T *oe = reinterpret_cast<T *>(&ov);
#pragma unroll
        for (int e = 0; e < V; ++e) oe[e] = Elem<T>::from_f(silu_mul(ge[e], ue[e]));
        *reinterpret_cast<uint4 *>(o + r * os + c) = ov;
    }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T *__restrict__ g, int64_t gs, const T *__restrict__ u,
                                                    int64_t us, T *__restrict__ o, int64_t os, int64_t rows,
                                                    int inter) {
    const int64_t total = rows * inter;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / inter;
        const int c = (int)(i - r * inter);
        o[r * os + c] = Elem<T>::from_f(silu_mul(g[r * gs + c], u[r * us + c]));
    }
}

template <typename T>
cudaError_t launch_t(const void *g, int64_t gs, const void *u, int64_t us, void *o, int64_t os, int64_t rows,
                     int inter, int sms, cudaStream_t st) {
    constexpr int V = 16 / sizeof(T);
    const T *gp = static_cast<const T *>(g), *up = static_cast<const T *>(u);
    T *op = static_cast<T *>(o);
    const bool vec = inter % V == 0 && gs % V == 0 && us % V == 0 && os % V == 0 &&
                     reinterpret_cast<uintptr_t>(g) % 16 == 0 && reinterpret_cast<uintptr_t>(u) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(o) % 16 == 0;
    const int64_t items = vec ? rows * (inter / V) : rows * inter;
    int64_t blocks = (items + 255) / 256;
    const int64_t cap = (int64_t)sms * 8;  // 8 resident blocks of 256 threads per SM
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    if (vec)
        swiglu_vec_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(gp, gs, up, us, op, os, rows, inter);
    else
        swiglu_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(gp, gs, up, us, op, os, rows, inter);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_swiglu(int dtype, const void *g, int64_t gs, const void *u, int64_t us, void *o, int64_t os,
                          int64_t rows, int inter, int sms, cudaStream_t st) {
    return dtype == PMA_F32 ? launch_t<float>(g, gs, u, us, o, os, rows, inter, sms, st)
                            : launch_t<__nv_bfloat16>(g, gs, u, us, o, os, rows, inter, sms, st);
}

}  // namespace pma
