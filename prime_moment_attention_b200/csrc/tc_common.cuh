// tc_common.cuh -- PTX helpers shared by the tcgen05 kernels (prefill_tc.cu, delta_tc.cu):
// mbarriers with bounded waits, async-proxy and tcgen05 fences, TMA, shared-memory matrix and
// instruction descriptors, MMA issue and commit, tensor-memory loads and stores, bf16 packing.
// All waits are bounded by the global timer (WAIT_NS); on expiry a kernel records a status code
// and gives up instead of hanging.
#pragma once

#include <cuda.h>

#include "pma_common.cuh"

namespace pma {
namespace tc {

constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s per wait

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
// The first 1024-byte-aligned byte of a dynamic shared-memory array (128-byte-swizzled tiles need
// that alignment), as pointer arithmetic on the array itself: the compiler keeps shared-memory
// accesses through the result in the shared state space.
__device__ __forceinline__ uint8_t *smem_align1024(uint8_t *raw) {
    return raw + ((1024u - (su32(raw) & 1023u)) & 1023u);
}

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

// Per-CTA failure record in shared memory.  The fault word's address sits here rather than in Ctl
// so that the role loops, which pass Ctl around, carry no extra pointer for a path taken only on
// failure.
struct CtlShared {
    int abort_flag;  // 0, or the code of a role that gave up
    int pad_;
    int *fault;      // registered fault word (pma_set_fault_word) or nullptr
};

struct Ctl {
    CtlShared *sh;  // shared
    int *status;    // global: first failure code (nullable)
    __device__ __forceinline__ bool aborted() const { return *reinterpret_cast<volatile int *>(&sh->abort_flag) != 0; }
};

__device__ __forceinline__ void init_ctl(CtlShared &s, int *fault) {
    s.abort_flag = 0;
    s.fault = fault;
}

// The code into the registered fault word (device memory or pinned host memory: a plain store, not
// an atomic).
__device__ __forceinline__ void report_fault(int code, int *fault) {
    if (code && fault) {
        volatile int *w = fault;
        if (*w == 0) *w = code;
        __threadfence_system();
    }
}

// Where a kernel reports to the fault word is chosen per translation unit, by what keeps its role
// loops free of extra register pressure: inside give_up (PMA_FAULT_AT_EXIT 0, the default), or once
// per CTA after its final barrier (PMA_FAULT_AT_EXIT 1: the kernel calls report_fault itself).
#ifndef PMA_FAULT_AT_EXIT
#define PMA_FAULT_AT_EXIT 0
#endif

__device__ __forceinline__ void give_up(const Ctl &ctl, int code) {
    *reinterpret_cast<volatile int *>(&ctl.sh->abort_flag) = code;
    if (ctl.status) atomicCAS(ctl.status, 0, code);
#if !PMA_FAULT_AT_EXIT
    report_fault(code, ctl.sh->fault);
#endif
}

// Test hook of the failure path: one thread waits for a barrier phase that nothing completes,
// bounded by `limit_ns`, and gives up with `code` like any expired wait.  Runs before any copy or
// GEMM is issued, so the CTA has nothing in flight when its roles see the abort flag.
__device__ __forceinline__ void expire_test_wait(uint64_t *never, const Ctl &ctl, unsigned long long limit_ns,
                                                 int code);

__device__ __forceinline__ bool mbar_wait_slow(uint64_t *b, uint32_t parity, const Ctl &ctl, int code) {
    const unsigned long long t0 = gtimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try(b, parity)) return true;
        if ((it & 63) == 0) {
            if (ctl.aborted()) return false;
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

__device__ __forceinline__ void expire_test_wait(uint64_t *never, const Ctl &ctl, unsigned long long limit_ns,
                                                 int code) {
    const unsigned long long t0 = gtimer();
    while (!mbar_try(never, 0)) {
        if (gtimer() - t0 > limit_ns) {
            give_up(ctl, code);
            return;
        }
    }
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Hands back a shared-memory buffer that this thread has read with ordinary loads, to a copy that
// rewrites it (a TMA or bulk copy issued once the barrier phase completes, or work ordered after
// such a copy).  The arrive alone does not order the generic-proxy reads before the async-proxy
// writes: without the proxy fence the copy can land before the loads are performed.
__device__ __forceinline__ void mbar_arrive_after_reads(uint64_t *b) {
    fence_proxy_async();
    mbar_arrive(b);
}
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

// Tile of shared memory -> global through a tensor map (bulk group; no multicast).  The innermost
// coordinate is always 0 here; rows past the tensor's extent are not written.
__device__ __forceinline__ void tma_store(const CUtensorMap *map, const void *src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(map),
                 "r"(su32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory source of every committed bulk store has been read
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every committed bulk store is complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

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
// Upper fields of a shared-memory matrix descriptor (everything but the start address).
__host__ __device__ constexpr uint64_t desc_hi(uint32_t lbo, uint32_t sbo, uint32_t swizzle) {
    return ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) |
           ((uint64_t)swizzle << 61);
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
// 32 consecutive float32 columns of this thread's TMEM lane (the wait is part of the same
// statement, so no use of the results can be scheduled before it).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "{\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t}"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// Columns taddr..taddr+31 of this thread's lane as two 16-column loads (addresses need only be
// 16-column aligned), with the wait in the same statement.
__device__ __forceinline__ void tmem_ld2x16(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "{\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31}, [%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t}"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr), "r"(taddr + 16)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// One float32 column of this thread's lane, with the wait.
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
    uint32_t r;
    asm volatile("{\n\ttcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\ttcgen05.wait::ld.sync.aligned;\n\t}"
                 : "=r"(r)
                 : "r"(taddr)
                 : "memory");
    return __uint_as_float(r);
}
// Column loads issued only: the values are valid after tmem_wait_ld_regs on the same registers
// (its "+r" operands keep every use behind the wait).
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}
// 8 consecutive 32-bit columns of this thread's TMEM lane (completion via tmem_wait_st).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}
// 33 float32 columns (32 consecutive + the one at +64) of this thread's TMEM lane, with the wait.
__device__ __forceinline__ void tmem_ld33(uint32_t taddr, uint32_t (&r)[32], uint32_t &r64) {
    asm volatile(
        "{\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%32}, [%34];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t}"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r64)
        : "r"(taddr), "r"(taddr + 64)
        : "memory");
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
// bf16 pair -> float pair (exact: bf16 is the upper half of a float32)
__device__ __forceinline__ float2 bf2f(uint32_t u) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
__device__ __forceinline__ uint32_t f2bf(float2 v) { return pack2(v.x, v.y); }
// byte offset of 16-byte chunk `c` of row `r` in a [rows x 128 B] tile with the 128-byte swizzle
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Host side (prefill_tc.cu): the driver's tensor-map encoder is reachable, and a 4-D map
// (d, l, h, b) over a [B,H,L,Dh] bf16 tensor with a 64 x 128 x 1 x 1 box and the 128-byte swizzle.
bool tensor_maps_available();
bool make_tile_map(CUtensorMap *m, const Seq &s, int B, int H, int L, int Dh);

}  // namespace tc
}  // namespace pma
