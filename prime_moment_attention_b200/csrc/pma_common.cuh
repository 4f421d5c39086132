// pma_common.cuh -- shared device/host helpers for the PRIME moment attention kernels.
#pragma once

#include <atomic>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pma.h"

namespace pma {

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per kernel and device (it is a host
// round trip; launches repeat it otherwise).  The kernel is a template argument so that every
// kernel has its own flag word.
template <auto Kernel>
inline cudaError_t set_smem_once(int bytes) {
    static std::atomic<unsigned long long> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}


// ---------------------------------------------------------------------------
// Element access for the two input/output types (float32, bfloat16).
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f(float x) { return x; }
    static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Load 4 consecutive elements (16 B for float, 8 B for bf16) as float4.
__device__ __forceinline__ float4 load4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16 *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162 *>(&u.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162 *>(&u.y);
    const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
}
__device__ __forceinline__ void store4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
__device__ __forceinline__ void store4(__nv_bfloat16 *p, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = u;
}

// Streaming (evict-first) float4 load/store for state that is touched once per step.
__device__ __forceinline__ float4 ldcs4(const float *p) { return __ldcs(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ void stcs4(float *p, float4 v) { __stcs(reinterpret_cast<float4 *>(p), v); }

__device__ __forceinline__ float4 fma4(float a, float4 x, float4 y) {
    return make_float4(fmaf(a, x.x, y.x), fmaf(a, x.y, y.y), fmaf(a, x.z, y.z), fmaf(a, x.w, y.w));
}
__device__ __forceinline__ float4 scale4(float a, float4 x) { return make_float4(a * x.x, a * x.y, a * x.z, a * x.w); }

// ---------------------------------------------------------------------------
// Kernel-side views of the ABI structs.
// ---------------------------------------------------------------------------
struct Seq {                 // [B,H,L,D] with element strides, D contiguous
    const void *p;
    int64_t sb, sh, sl;
};
struct SeqOut {
    void *p;
    int64_t sb, sh, sl;
};

// Input prologue (pma_prologue): kv head = h / groups; q -> LN(q) * q_scale, k -> LN(k).
struct Prologue {
    int groups;
    float q_scale;
    const float *qw, *qb, *kw, *kb;   // qw / kw null: no norm; qb / kb null: zero bias
    float ln_eps;
    __host__ __device__ bool q_work() const { return qw != nullptr || q_scale != 1.0f; }
    __host__ __device__ bool k_work() const { return kw != nullptr; }
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// Mean and 1/sqrt(biased var + eps) of a D-element row, read by one warp (two passes over
// the row: the variance is the mean of squared deviations, as nn.LayerNorm computes it).
template <int D, typename T>
__device__ __forceinline__ float2 warp_row_stats(const T *row, float eps, int lane) {
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s += Elem<T>::to_f(row[d]);
    const float mean = warp_sum(s) * (1.0f / D);
    float v = 0.f;
    for (int d = lane; d < D; d += 32) {
        const float t = Elem<T>::to_f(row[d]) - mean;
        v = fmaf(t, t, v);
    }
    return make_float2(mean, rsqrtf(warp_sum(v) * (1.0f / D) + eps));
}

// (x - mean) * rstd * w[d] + b[d] (w null: x), then * scale.
__device__ __forceinline__ float prologue_elem(float x, float2 st, const float *w, const float *b, int d,
                                              float scale) {
    if (w) x = fmaf((x - st.x) * st.y, __ldg(w + d), b ? __ldg(b + d) : 0.f);
    return x * scale;
}

__device__ __forceinline__ float4 prologue4(float4 x, float2 st, const float *w, const float *b, int d0,
                                           float scale) {
    return make_float4(prologue_elem(x.x, st, w, b, d0, scale), prologue_elem(x.y, st, w, b, d0 + 1, scale),
                       prologue_elem(x.z, st, w, b, d0 + 2, scale), prologue_elem(x.w, st, w, b, d0 + 3, scale));
}

// Pointers to one head-state.
struct HeadPtrs {
    float *S0, *S1, *S2, *Z0, *Z1, *Z2;
};

__host__ __device__ constexpr size_t state_floats(int D) { return 2 * (size_t)D * D + 3 * (size_t)D + 1; }
// Slot stride of the packed scratch layout: state_floats rounded up to 32 floats,
// so every slot (and every S1/S2 row in it) starts on a 128-byte boundary.
__host__ __device__ constexpr size_t slot_floats(int D) { return (state_floats(D) + 31) / 32 * 32; }

// Either the user's six-array state (index bh) or a packed scratch layout
// [bh][slot][slot_floats(D)] ordered S1 | S2 | S0 | Z1 | Z2 | Z0.
struct StateRef {
    pma_state user;      // used when packed == nullptr and user.S1 != nullptr
    float *packed;
    int slots;           // packed slots per head-state
    __host__ __device__ bool present() const { return packed != nullptr || user.S1 != nullptr; }
    __device__ __forceinline__ HeadPtrs at(int bh, int slot, int D) const {
        HeadPtrs r;
        if (packed) {
            float *b = packed + ((size_t)bh * slots + slot) * slot_floats(D);
            r.S1 = b;
            r.S2 = b + (size_t)D * D;
            r.S0 = b + 2 * (size_t)D * D;
            r.Z1 = r.S0 + D;
            r.Z2 = r.Z1 + D;
            r.Z0 = r.Z2 + D;
        } else {
            r.S0 = user.S0 + (size_t)bh * D;
            r.S1 = user.S1 + (size_t)bh * D * D;
            r.S2 = user.S2 + (size_t)bh * D * D;
            r.Z0 = user.Z0 + bh;
            r.Z1 = user.Z1 + (size_t)bh * D;
            r.Z2 = user.Z2 + (size_t)bh * D;
        }
        return r;
    }
};


}  // namespace pma
