// pma_capi.cu -- the extern "C" entry points declared in include/pma.h:
// argument validation on the host, planning (kernel, chunk, segments) and launch.
#include <atomic>
#include <cstring>
#include <mutex>

#include "prefill.cuh"

using namespace pma;

namespace {

struct DevInfo {
    int sms = 0;
    int major = 0;
    bool valid = false;
};

thread_local int g_last_cuda_error = 0;

// The caller's fault word (pma_set_fault_word) and the test hook's wait limit
// (pma_test_expire_waits): read by every launch of a kernel with bounded waits.
std::atomic<int *> g_fault_word{nullptr};
std::atomic<unsigned long long> g_test_wait_ns{0};

}  // namespace

// PMA_ERR_CUDA with the cause remembered for pma_last_cuda_error() (also used by prefill_static.cu).
int pma::cuda_fail(cudaError_t e) {
    g_last_cuda_error = (int)e;
    return PMA_ERR_CUDA;
}

namespace {

inline int d_ok(const DevInfo &d) { return d.major == 10 ? PMA_OK : PMA_ERR_DEVICE; }

constexpr int kMaxDevices = 64;
DevInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DevInfo *out) {
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return cuda_fail(ce);
    if (dev < 0 || dev >= kMaxDevices) return PMA_ERR_DEVICE;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!g_dev[dev].valid) {
        DevInfo d;
        if ((ce = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return cuda_fail(ce);
        if ((ce = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
            return cuda_fail(ce);
        d.valid = true;
        g_dev[dev] = d;
    }
    *out = g_dev[dev];
    return d_ok(*out);
}

bool supported_d(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }
bool supported_dtype(int t) { return t == PMA_F32 || t == PMA_BF16; }
size_t esize(int t) { return t == PMA_F32 ? 4 : 2; }

// Each row of D elements must start on a 16-byte boundary (vector loads, TMA).
int check_seq(const pma_seq_tensor *t, bool use_l, bool empty = false) {
    if (!t) return PMA_ERR_ARGUMENT;
    if (!t->data) return empty ? (supported_dtype(t->dtype) ? PMA_OK : PMA_ERR_DTYPE) : PMA_ERR_ARGUMENT;
    if (!supported_dtype(t->dtype)) return PMA_ERR_DTYPE;
    const int64_t step = 16 / (int64_t)esize(t->dtype);
    if (reinterpret_cast<uintptr_t>(t->data) % 16) return PMA_ERR_LAYOUT;
    if (t->stride_b % step || t->stride_h % step || (use_l && t->stride_l % step)) return PMA_ERR_LAYOUT;
    if (t->stride_b < 0 || t->stride_h < 0 || (use_l && t->stride_l < 0)) return PMA_ERR_LAYOUT;
    return PMA_OK;
}

int check_state(const pma_state *s) {
    if (!s || !s->S0 || !s->S1 || !s->S2 || !s->Z0 || !s->Z1 || !s->Z2) return PMA_ERR_ARGUMENT;
    const uintptr_t a[6] = {(uintptr_t)s->S0, (uintptr_t)s->S1, (uintptr_t)s->S2,
                            (uintptr_t)s->Z1, (uintptr_t)s->Z2, 0};
    for (int i = 0; i < 6; ++i)
        if (a[i] % 16) return PMA_ERR_LAYOUT;
    if ((uintptr_t)s->Z0 % 4) return PMA_ERR_LAYOUT;
    return PMA_OK;
}

Seq seq_of(const pma_seq_tensor *t) { return Seq{t->data, t->stride_b, t->stride_h, t->stride_l}; }
SeqOut seqout_of(const pma_seq_tensor *t) {
    return t ? SeqOut{t->data, t->stride_b, t->stride_h, t->stride_l} : SeqOut{nullptr, 0, 0, 0};
}
StateRef user_ref(const pma_state *s) {
    StateRef r{};
    if (s) r.user = *s;
    r.packed = nullptr;
    r.slots = 1;
    return r;
}
StateRef packed_ref(float *ws, int slots) {
    StateRef r{};
    r.packed = ws;
    r.slots = slots;
    return r;
}

struct Plan {
    bool tc = false;
    int chunk = 64;
    int nseg = 1;
    int seg_len = 0;
    size_t ws_bytes = 0;
};

bool bf16_exact(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (u & 0xffffu) == 0;
}

// D = 128 runs on tensor cores when the kernel needs no LayerNorm pass (`pro` null: no prologue).
bool tc128_plan(int D, int dtype, const Prologue *pro) {
    if (D != 128 || !tc128_supported(dtype)) return false;
    return !pro || (!pro->qw && !pro->kw && (pro->q_scale == 1.0f || bf16_exact(pro->q_scale)));
}

Plan make_plan(int B, int H, int L, int D, int dtype, int sms, const Prologue *pro) {
    Plan p;
    p.tc = tc_supported(D, dtype) || tc128_plan(D, dtype, pro);
    p.chunk = p.tc ? TC_CHUNK : simt_chunk(D);
    const long BH = (long)B * H;
    const int nchunks = (L + p.chunk - 1) / p.chunk;
    // CTAs resident per SM: SIMT D<=64 fits two; D=128 and the tensor-core kernel one.
    const long slots = (long)sms * ((!p.tc && D <= 64) ? 2 : 1);
    // Split sequences into segments only when B*H leaves SMs idle, and only into as
    // many as fit one wave (a partial second wave costs more than the idle SMs).
    int nseg = 1;
    if (BH > 0 && BH * 2 <= slots) nseg = (int)(slots / BH);
    if (nseg > nchunks) nseg = nchunks;
    if (nseg < 1) nseg = 1;
    const int seg_chunks = (nchunks + nseg - 1) / nseg;
    p.nseg = seg_chunks > 0 ? (nchunks + seg_chunks - 1) / seg_chunks : 1;
    p.seg_len = seg_chunks * p.chunk;
    p.ws_bytes = p.tc ? WS_HEADER : 0;
    if (p.nseg > 1) p.ws_bytes = WS_HEADER + (size_t)BH * p.nseg * slot_floats(D) * sizeof(float);
    return p;
}

// pma_prologue -> kernel view; NULL is the identity (no GQA, no norm, scale 1).
int prologue_of(const pma_prologue *pp, int H, Prologue *out) {
    Prologue r{1, 1.0f, nullptr, nullptr, nullptr, nullptr, 1e-5f};
    if (pp) {
        if (pp->kv_groups < 1 || H % pp->kv_groups) return PMA_ERR_ARGUMENT;
        if (!(pp->norm_eps >= 0.0f) || pp->q_scale != pp->q_scale) return PMA_ERR_ARGUMENT;
        const float *ptrs[4] = {pp->q_norm_weight, pp->q_norm_bias, pp->k_norm_weight, pp->k_norm_bias};
        for (const float *f : ptrs)
            if (reinterpret_cast<uintptr_t>(f) % 4) return PMA_ERR_LAYOUT;
        r.groups = pp->kv_groups;
        r.q_scale = pp->q_scale;
        r.qw = pp->q_norm_weight;
        r.qb = pp->q_norm_weight ? pp->q_norm_bias : nullptr;
        r.kw = pp->k_norm_weight;
        r.kb = pp->k_norm_weight ? pp->k_norm_bias : nullptr;
        r.ln_eps = pp->norm_eps;
    }
    *out = r;
    return PMA_OK;
}

int prefill_impl(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                 const pma_seq_tensor *v, const pma_prologue *prologue, const float *lambda,
                 int64_t lambda_stride_b, const pma_state *state_in, const pma_state *state_out, float eps,
                 const pma_seq_tensor *y, void *workspace, size_t workspace_bytes, pma_stream_t stream,
                 bool resume = false);
int decode_impl(int N, int H, int D, const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                const pma_prologue *prologue, const float *lambda, int64_t lambda_stride_n, const int32_t *rows,
                int pool_rows, const pma_state *state_in, const pma_state *state_out, float eps,
                const pma_seq_tensor *y, pma_stream_t stream, const float *k_head_scale = nullptr,
                bool selective = false);

// Tensor-core path: which inputs the QK-norm pass rewrites, and the workspace beyond the plan's.
struct ProPass {
    bool q = false, k = false;
    size_t q_off = 0, k_off = 0, total = 0;  // byte offsets of the copies in the workspace; total bytes
};

ProPass pro_pass(const Plan &pl, const Prologue &pro, int B, int H, int L, bool want_y) {
    ProPass r;
    r.total = pl.ws_bytes;
    if (!pl.tc) return r;  // the CUDA-core kernel folds the prologue into its loads
    r.q = want_y && (pro.qw != nullptr || (pro.q_scale != 1.0f && !bf16_exact(pro.q_scale)));
    r.k = pro.kw != nullptr;
    size_t off = (pl.ws_bytes + 255) / 256 * 256;
    if (r.q) {
        r.q_off = off;
        off += (size_t)B * H * L * 64 * 2;
    }
    if (r.k) {
        off = (off + 255) / 256 * 256;
        r.k_off = off;
        off += (size_t)B * (H / pro.groups) * L * 64 * 2;
    }
    if (r.q || r.k) r.total = off;
    return r;
}

// Tensor-core path: the QK-norm pass for q and / or k (pro_pass says which) into the workspace;
// the core then reads the normalised rows and keeps the GQA map and a bf16-exact q scale.
cudaError_t run_prologue_passes(const ProPass &pp, const Prologue &pro, PrefillParams &p, int B, int H, int L,
                                void *workspace, bool want_y, int sms, cudaStream_t st) {
    char *wsb = reinterpret_cast<char *>(workspace);
    const int hkv = H / pro.groups;
    cudaError_t e;
    if (pp.q) {
        if ((e = launch_qk_norm(p.q, B, H, L, pro.qw, pro.qb, pro.ln_eps, pro.q_scale, wsb + pp.q_off, sms, st)) !=
            cudaSuccess)
            return e;
        p.q = Seq{wsb + pp.q_off, (int64_t)H * L * 64, (int64_t)L * 64, 64};
        p.pro.q_scale = 1.0f;
    }
    if (pp.k) {
        if ((e = launch_qk_norm(p.k, B, hkv, L, pro.kw, pro.kb, pro.ln_eps, 1.0f, wsb + pp.k_off, sms, st)) !=
            cudaSuccess)
            return e;
        p.k = Seq{wsb + pp.k_off, (int64_t)hkv * L * 64, (int64_t)L * 64, 64};
    }
    p.pro.qw = p.pro.qb = p.pro.kw = p.pro.kb = nullptr;
    if (!want_y) p.pro.q_scale = 1.0f;
    return cudaSuccess;
}

// The selective prefill's plan: one segment per head-state (its per-token decay has no per-head
// carry factor for the segment prefix); tensor cores for bf16 at D = 64.
Plan selective_plan(int L, int D, int dtype) {
    Plan p;
    p.tc = tc_supported(D, dtype);
    p.chunk = p.tc ? TC_CHUNK : simt_chunk(D);
    p.nseg = 1;
    p.seg_len = ((L + p.chunk - 1) / p.chunk) * p.chunk;
    p.ws_bytes = p.tc ? WS_HEADER : 0;
    return p;
}

cudaError_t launch_prefill(const Plan &pl, const PrefillParams &p, int D, int idt, int ydt, dim3 grid,
                           cudaStream_t st) {
    if (!pl.tc) return launch_prefill_simt(p, D, idt, ydt, grid, st);
    return D == 128 ? launch_prefill_tc128(p, ydt, grid, st) : launch_prefill_tc(p, ydt, grid, st);
}

}  // namespace

extern "C" {

int pma_version(void) { return PMA_ABI_VERSION; }

const char *pma_status_string(int status) {
    switch (status) {
        case PMA_OK: return "ok";
        case PMA_ERR_ARGUMENT: return "invalid argument (null pointer or negative size)";
        case PMA_ERR_HEAD_DIM: return "unsupported head_dim (supported: 16, 32, 64, 128)";
        case PMA_ERR_DTYPE: return "unsupported dtype (float32 or bfloat16)";
        case PMA_ERR_LAYOUT: return "unsupported layout (rows must start on 16-byte boundaries, head dim contiguous)";
        case PMA_ERR_WORKSPACE: return "workspace missing or too small";
        case PMA_ERR_CUDA: return "CUDA runtime error";
        case PMA_ERR_DEVICE: return "current device is not sm_100 (B200 class)";
        default: return "unknown status";
    }
}

int pma_last_cuda_error(void) { return g_last_cuda_error; }

void pma_set_fault_word(int *word) { g_fault_word.store(word); }

void pma_test_expire_waits(unsigned long long limit_ns) { g_test_wait_ns.store(limit_ns); }

const char *pma_cuda_error_string(int cuda_error) { return cudaGetErrorString((cudaError_t)cuda_error); }

size_t pma_state_floats(int D) { return D > 0 ? state_floats(D) : 0; }

int pma_supported_head_dims(int dtype, int *dims, int cap) {
    static const int all[4] = {16, 32, 64, 128};
    if (!supported_dtype(dtype)) return 0;
    for (int i = 0; i < 4 && i < cap; ++i)
        if (dims) dims[i] = all[i];
    return 4;
}

size_t pma_prefill_workspace_bytes(int B, int H, int L, int D, int dtype) {
    if (B <= 0 || H <= 0 || L <= 0 || !supported_d(D) || !supported_dtype(dtype)) return 0;
    DevInfo di;
    if (device_info(&di) != PMA_OK) return 0;
    return make_plan(B, H, L, D, dtype, di.sms, nullptr).ws_bytes;
}

size_t pma_prefill_ex_workspace_bytes(int B, int H, int L, int D, int dtype, const pma_prologue *prologue) {
    if (B <= 0 || H <= 0 || L <= 0 || !supported_d(D) || !supported_dtype(dtype)) return 0;
    Prologue pro;
    if (prologue_of(prologue, H, &pro) != PMA_OK) return 0;
    DevInfo di;
    if (device_info(&di) != PMA_OK) return 0;
    return pro_pass(make_plan(B, H, L, D, dtype, di.sms, &pro), pro, B, H, L, true).total;
}

int pma_prefill(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                const pma_seq_tensor *v, const float *lambda, int64_t lambda_stride_b, const pma_state *state_in,
                const pma_state *state_out, float eps, const pma_seq_tensor *y, void *workspace,
                size_t workspace_bytes, pma_stream_t stream) {
    return prefill_impl(B, H, L, D, q, k, v, nullptr, lambda, lambda_stride_b, state_in, state_out, eps, y,
                        workspace, workspace_bytes, stream);
}

int pma_prefill_ex(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                   const pma_seq_tensor *v, const pma_prologue *prologue, const float *lambda,
                   int64_t lambda_stride_b, const pma_state *state_in, const pma_state *state_out, float eps,
                   const pma_seq_tensor *y, void *workspace, size_t workspace_bytes, pma_stream_t stream) {
    return prefill_impl(B, H, L, D, q, k, v, prologue, lambda, lambda_stride_b, state_in, state_out, eps, y,
                        workspace, workspace_bytes, stream);
}

int pma_prefill_resume(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                       const pma_seq_tensor *v, const float *lambda, int64_t lambda_stride_b,
                       const pma_state *state_in, const pma_state *state_out, float eps, const pma_seq_tensor *y,
                       void *workspace, size_t workspace_bytes, pma_stream_t stream) {
    if (!y) return PMA_ERR_ARGUMENT;  // the output pass is what this entry runs
    return prefill_impl(B, H, L, D, q, k, v, nullptr, lambda, lambda_stride_b, state_in, state_out, eps, y,
                        workspace, workspace_bytes, stream, true);
}

int pma_decode_step(int N, int H, int D, const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                    const float *lambda, int64_t lambda_stride_n, const pma_state *state_in,
                    const pma_state *state_out, float eps, const pma_seq_tensor *y, pma_stream_t stream) {
    return decode_impl(N, H, D, q, k, v, nullptr, lambda, lambda_stride_n, nullptr, 0, state_in, state_out, eps, y,
                       stream);
}

int pma_decode_step_rows(int N, int H, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                         const pma_seq_tensor *v, const float *lambda, int64_t lambda_stride_n, const int32_t *rows,
                         int pool_rows, const pma_state *pool_in, const pma_state *pool_out, float eps,
                         const pma_seq_tensor *y, pma_stream_t stream) {
    if (N > 0 && !rows) return PMA_ERR_ARGUMENT;
    return decode_impl(N, H, D, q, k, v, nullptr, lambda, lambda_stride_n, rows, pool_rows, pool_in, pool_out, eps,
                       y, stream);
}

int pma_decode_step_ex(int N, int H, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                       const pma_seq_tensor *v, const pma_prologue *prologue, const float *lambda,
                       int64_t lambda_stride_n, const int32_t *rows, int pool_rows, const pma_state *state_in,
                       const pma_state *state_out, float eps, const pma_seq_tensor *y, pma_stream_t stream) {
    return decode_impl(N, H, D, q, k, v, prologue, lambda, lambda_stride_n, rows, pool_rows, state_in, state_out,
                       eps, y, stream);
}

}  // extern "C"

namespace {

int prefill_impl(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                 const pma_seq_tensor *v, const pma_prologue *prologue, const float *lambda,
                 int64_t lambda_stride_b, const pma_state *state_in, const pma_state *state_out, float eps,
                 const pma_seq_tensor *y, void *workspace, size_t workspace_bytes, pma_stream_t stream,
                 bool resume) {
    if (B < 0 || H <= 0 || L < 0 || !lambda || lambda_stride_b < 0) return PMA_ERR_ARGUMENT;
    if (!supported_d(D)) return PMA_ERR_HEAD_DIM;
    int rc;
    Prologue pro;
    if ((rc = prologue_of(prologue, H, &pro))) return rc;
    const bool empty = (L == 0 || B == 0);  // no element is touched: null data is fine
    if ((rc = check_seq(q, true, empty)) || (rc = check_seq(k, true, empty)) || (rc = check_seq(v, true, empty)))
        return rc;
    if (q->dtype != k->dtype || q->dtype != v->dtype) return PMA_ERR_DTYPE;
    if (y && (rc = check_seq(y, true, empty))) return rc;
    if (state_in && (rc = check_state(state_in))) return rc;
    if (state_out && (rc = check_state(state_out))) return rc;
    DevInfo di;
    if ((rc = device_info(&di))) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int BH = B * H;
    if (BH == 0) return PMA_OK;

    if (L == 0) {  // nothing consumed: final state = incoming state
        if (!state_out) return PMA_OK;
        const size_t DD = (size_t)D * D;
        float *dst[6] = {state_out->S0, state_out->S1, state_out->S2, state_out->Z0, state_out->Z1, state_out->Z2};
        const float *src[6] = {state_in ? state_in->S0 : nullptr, state_in ? state_in->S1 : nullptr,
                               state_in ? state_in->S2 : nullptr, state_in ? state_in->Z0 : nullptr,
                               state_in ? state_in->Z1 : nullptr, state_in ? state_in->Z2 : nullptr};
        const size_t n[6] = {BH * (size_t)D, BH * DD, BH * DD, (size_t)BH, BH * (size_t)D, BH * (size_t)D};
        for (int i = 0; i < 6; ++i) {
            cudaError_t e = src[i] ? (src[i] == dst[i] ? cudaSuccess
                                                        : cudaMemcpyAsync(dst[i], src[i], n[i] * 4,
                                                                          cudaMemcpyDeviceToDevice, st))
                                   : cudaMemsetAsync(dst[i], 0, n[i] * 4, st);
            if (e != cudaSuccess) return cuda_fail(e);
        }
        return PMA_OK;
    }

    const Plan pl = make_plan(B, H, L, D, q->dtype, di.sms, &pro);
    const ProPass pp = pro_pass(pl, pro, B, H, L, y != nullptr);
    if (pp.total && (!workspace || workspace_bytes < pp.total)) return PMA_ERR_WORKSPACE;
    if (pp.total && reinterpret_cast<uintptr_t>(workspace) % 16) return PMA_ERR_WORKSPACE;
    if (!y && !state_out) return PMA_OK;  // nothing requested
    const int ydt = y ? y->dtype : PMA_F32;

    PrefillParams p{};
    p.B = B;
    p.H = H;
    p.L = L;
    p.seg_len = pl.seg_len;
    p.q = seq_of(q);
    p.k = seq_of(k);
    p.v = seq_of(v);
    p.pro = pro;
    cudaError_t e;
    if (pl.tc && (e = run_prologue_passes(pp, pro, p, B, H, L, workspace, y != nullptr, di.sms, st)) != cudaSuccess)
        return cuda_fail(e);
    p.y = seqout_of(y);
    p.lambda = lambda;
    p.lam_sb = lambda_stride_b;
    p.eps = eps;
    p.status = nullptr;
    p.fault = g_fault_word.load();
    p.test_wait_ns = g_test_wait_ns.load();

    if (pl.ws_bytes) {  // clear the status word the tensor-core kernel reports timeouts in
        p.status = reinterpret_cast<int *>(workspace);
        if ((e = cudaMemsetAsync(p.status, 0, sizeof(int), st)) != cudaSuccess) return cuda_fail(e);
    }
    if (pl.nseg == 1) {
        p.in = user_ref(state_in);
        p.out = user_ref(state_out);
        p.state_only = 0;
        e = launch_prefill(pl, p, D, q->dtype, ydt, dim3(BH, 1), st);
        return e == cudaSuccess ? PMA_OK : cuda_fail(e);
    }

    float *ws = reinterpret_cast<float *>(reinterpret_cast<char *>(workspace) + WS_HEADER);
    if (resume) {
        // the workspace holds the state entering every segment from a zero start (left there by a
        // state-only call with the same plan): shift them to state_in, then the full pass
        if (state_in && (e = launch_segment_resume(BH, H, D, pl.nseg, pl.seg_len, ws, user_ref(state_in), lambda,
                                                   lambda_stride_b, st)) != cudaSuccess)
            return cuda_fail(e);
        p.in = packed_ref(ws, pl.nseg);
        p.out = user_ref(state_out);
        p.state_only = 0;
        e = launch_prefill(pl, p, D, q->dtype, ydt, dim3(BH, pl.nseg), st);
        return e == cudaSuccess ? PMA_OK : cuda_fail(e);
    }
    // 1. each segment's own state from zero (the last one only when no y is wanted)
    PrefillParams ps = p;
    ps.y = SeqOut{nullptr, 0, 0, 0};
    ps.in = user_ref(nullptr);
    ps.out = packed_ref(ws, pl.nseg);
    ps.state_only = 1;
    const int nstate = y ? pl.nseg - 1 : pl.nseg;
    e = launch_prefill(pl, ps, D, q->dtype, ydt, dim3(BH, nstate), st);
    if (e != cudaSuccess) return cuda_fail(e);
    // 2. in-place prefix: state entering every segment (and the final state if no y)
    e = launch_segment_prefix(BH, H, D, pl.nseg, pl.seg_len, L, ws, user_ref(state_in),
                              y ? user_ref(nullptr) : user_ref(state_out), lambda, lambda_stride_b, st);
    if (e != cudaSuccess) return cuda_fail(e);
    if (!y) return PMA_OK;
    // 3. full pass, every segment starting from its carried state
    p.in = packed_ref(ws, pl.nseg);
    p.out = user_ref(state_out);
    p.state_only = 0;
    e = launch_prefill(pl, p, D, q->dtype, ydt, dim3(BH, pl.nseg), st);
    return e == cudaSuccess ? PMA_OK : cuda_fail(e);
}

int decode_impl(int N, int H, int D, const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                const pma_prologue *prologue, const float *lambda, int64_t lambda_stride_n, const int32_t *rows,
                int pool_rows, const pma_state *state_in, const pma_state *state_out, float eps,
                const pma_seq_tensor *y, pma_stream_t stream, const float *k_head_scale, bool selective) {
    if (N < 0 || H <= 0 || !lambda || lambda_stride_n < 0 || pool_rows < 0) return PMA_ERR_ARGUMENT;
    if (!supported_d(D)) return PMA_ERR_HEAD_DIM;
    int rc;
    Prologue pro;
    if ((rc = prologue_of(prologue, H, &pro))) return rc;
    const bool empty = N == 0;
    if ((rc = check_seq(q, false, empty)) || (rc = check_seq(k, false, empty)) || (rc = check_seq(v, false, empty)) ||
        (rc = check_seq(y, false, empty)))
        return rc;
    if (q->dtype != k->dtype || q->dtype != v->dtype) return PMA_ERR_DTYPE;
    if ((rc = check_state(state_in)) || (rc = check_state(state_out))) return rc;
    DevInfo di;
    if ((rc = device_info(&di))) return rc;
    if (N == 0) return PMA_OK;
    if ((long)N * H > (1L << 30) || (long)pool_rows * H > (1L << 30)) return PMA_ERR_ARGUMENT;
    DecodeParams p{};
    p.N = N;
    p.H = H;
    p.q = seq_of(q);
    p.k = seq_of(k);
    p.v = seq_of(v);
    p.pro = pro;
    p.y = seqout_of(y);
    p.lambda = lambda;
    p.lam_sn = lambda_stride_n;
    p.in = *state_in;
    p.out = *state_out;
    p.eps = eps;
    p.rows = rows;
    p.pool_rows = rows ? pool_rows : 0;
    p.k_head_scale = k_head_scale;
    p.log_lambda = selective ? 1 : 0;
    p.half_sq = selective ? 1 : 0;
    cudaError_t e = launch_decode(p, D, q->dtype, y->dtype, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? PMA_OK : cuda_fail(e);
}

}  // namespace

extern "C" {

int pma_delta_prefill(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                      const pma_seq_tensor *v, const float *beta, const float *alpha, const float *lambda,
                      int64_t lambda_stride_b, int chunk, float lyapunov_bound, float norm_eps,
                      const float *state_in, float *state_out, const pma_seq_tensor *y, void *workspace,
                      size_t workspace_bytes, pma_stream_t stream) {
    if (B < 0 || H <= 0 || L < 0 || !lambda || lambda_stride_b < 0 || !(norm_eps > 0.0f)) return PMA_ERR_ARGUMENT;
    if (D != 16 && D != 32 && D != 64) return PMA_ERR_HEAD_DIM;
    if (chunk != 32 && chunk != 64) return PMA_ERR_ARGUMENT;
    if (!y && !state_out) return PMA_ERR_ARGUMENT;
    int rc;
    const bool empty = (L == 0 || B == 0);
    if ((rc = check_seq(q, true, empty)) || (rc = check_seq(k, true, empty)) || (rc = check_seq(v, true, empty)))
        return rc;
    if (q->dtype != k->dtype || q->dtype != v->dtype) return PMA_ERR_DTYPE;
    if (y && (rc = check_seq(y, true, empty))) return rc;
    if (!empty && !beta) return PMA_ERR_ARGUMENT;
    if ((uintptr_t)state_in % 16 || (uintptr_t)state_out % 16) return PMA_ERR_LAYOUT;
    DevInfo di;
    if ((rc = device_info(&di))) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const size_t sbytes = (size_t)B * H * D * 2 * D * sizeof(float);
    if (B == 0) return PMA_OK;
    if (L == 0) {
        if (!state_out) return PMA_OK;
        cudaError_t e = state_in ? (state_in == state_out ? cudaSuccess
                                                          : cudaMemcpyAsync(state_out, state_in, sbytes,
                                                                            cudaMemcpyDeviceToDevice, st))
                                 : cudaMemsetAsync(state_out, 0, sbytes, st);
        return e == cudaSuccess ? PMA_OK : cuda_fail(e);
    }
    DeltaParams p{};
    p.B = B;
    p.H = H;
    p.L = L;
    p.q = seq_of(q);
    p.k = seq_of(k);
    p.v = seq_of(v);
    p.y = seqout_of(y);
    p.beta = beta;
    p.alpha = alpha;
    p.lambda = lambda;
    p.lam_sb = lambda_stride_b;
    p.bound = lyapunov_bound;
    p.norm_eps = norm_eps;
    p.state_in = state_in;
    p.state_out = state_out;
    p.fault = g_fault_word.load();
    p.test_wait_ns = g_test_wait_ns.load();
    const int ydt = y ? y->dtype : PMA_F32;
    cudaError_t e;
    if (delta_tc_supported(D, chunk, q->dtype)) {
        if (workspace && workspace_bytes) {
            const int window = delta_wy_window(B, H, L, workspace_bytes);
            if (window == 0) return PMA_ERR_WORKSPACE;
            if ((uintptr_t)workspace % 256) return PMA_ERR_LAYOUT;
            e = launch_delta_prefill_wy(p, ydt, workspace, window, st);
        } else {
            e = launch_delta_prefill_tc(p, ydt, st);
        }
    } else {
        e = launch_delta_prefill(p, D, chunk, q->dtype, ydt, st);
    }
    return e == cudaSuccess ? PMA_OK : cuda_fail(e);
}

size_t pma_delta_prefill_workspace_bytes(int B, int H, int L, int D, int chunk, int dtype) {
    if (!delta_tc_supported(D, chunk, dtype)) return 0;
    return delta_wy_workspace_bytes(B, H, L);
}

int pma_delta_decode_step(int N, int H, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                          const pma_seq_tensor *v, const float *beta, const float *alpha, float lyapunov_bound,
                          float norm_eps, const float *state_in, float *state_out, const pma_seq_tensor *y,
                          pma_stream_t stream) {
    if (N < 0 || H <= 0 || !(norm_eps > 0.0f)) return PMA_ERR_ARGUMENT;
    if (D != 16 && D != 32 && D != 64) return PMA_ERR_HEAD_DIM;
    int rc;
    const bool empty = N == 0;
    if ((rc = check_seq(q, false, empty)) || (rc = check_seq(k, false, empty)) || (rc = check_seq(v, false, empty)) ||
        (rc = check_seq(y, false, empty)))
        return rc;
    if (q->dtype != k->dtype || q->dtype != v->dtype) return PMA_ERR_DTYPE;
    if (!empty && (!beta || !alpha || !state_in || !state_out)) return PMA_ERR_ARGUMENT;
    if ((uintptr_t)state_in % 16 || (uintptr_t)state_out % 16) return PMA_ERR_LAYOUT;
    DevInfo di;
    if ((rc = device_info(&di))) return rc;
    if (N == 0) return PMA_OK;
    if ((long)N * H > (1L << 30)) return PMA_ERR_ARGUMENT;
    DeltaStepParams p{};
    p.N = N;
    p.H = H;
    p.q = seq_of(q);
    p.k = seq_of(k);
    p.v = seq_of(v);
    p.y = seqout_of(y);
    p.beta = beta;
    p.alpha = alpha;
    p.bound = lyapunov_bound;
    p.norm_eps = norm_eps;
    p.state_in = state_in;
    p.state_out = state_out;
    cudaError_t e = launch_delta_step(p, D, q->dtype, y->dtype, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? PMA_OK : cuda_fail(e);
}

size_t pma_selective_prefill_workspace_bytes(int B, int H, int L, int D, int dtype, const pma_prologue *prologue) {
    if (B <= 0 || H <= 0 || L <= 0 || !supported_d(D) || !supported_dtype(dtype)) return 0;
    Prologue pro;
    if (prologue_of(prologue, H, &pro) != PMA_OK) return 0;
    return pro_pass(selective_plan(L, D, dtype), pro, B, H, L, true).total;
}

int pma_selective_prefill(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                          const pma_seq_tensor *v, const pma_prologue *prologue, const float *log_decay,
                          const float *beta, const pma_state *state_in, const pma_state *state_out, float eps,
                          const pma_seq_tensor *y, void *workspace, size_t workspace_bytes, pma_stream_t stream) {
    if (B < 0 || H <= 0 || L < 0 || !beta || (L > 0 && B > 0 && !log_decay)) return PMA_ERR_ARGUMENT;
    if (!supported_d(D)) return PMA_ERR_HEAD_DIM;
    int rc;
    Prologue pro;
    if ((rc = prologue_of(prologue, H, &pro))) return rc;
    const bool empty = (L == 0 || B == 0);
    if ((rc = check_seq(q, true, empty)) || (rc = check_seq(k, true, empty)) || (rc = check_seq(v, true, empty)))
        return rc;
    if (q->dtype != k->dtype || q->dtype != v->dtype) return PMA_ERR_DTYPE;
    if (y && (rc = check_seq(y, true, empty))) return rc;
    if (state_in && (rc = check_state(state_in))) return rc;
    if (state_out && (rc = check_state(state_out))) return rc;
    if (!y && !state_out) return PMA_OK;
    DevInfo di;
    if ((rc = device_info(&di))) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int BH = B * H;
    if (BH == 0) return PMA_OK;
    if (L == 0) {  // the state passes through unchanged (same layout in and out)
        if (!state_out) return PMA_OK;
        const size_t DD = (size_t)D * D;
        float *dst[6] = {state_out->S0, state_out->S1, state_out->S2, state_out->Z0, state_out->Z1, state_out->Z2};
        const float *src[6] = {state_in ? state_in->S0 : nullptr, state_in ? state_in->S1 : nullptr,
                               state_in ? state_in->S2 : nullptr, state_in ? state_in->Z0 : nullptr,
                               state_in ? state_in->Z1 : nullptr, state_in ? state_in->Z2 : nullptr};
        const size_t n[6] = {BH * (size_t)D, BH * DD, BH * DD, (size_t)BH, BH * (size_t)D, BH * (size_t)D};
        for (int i = 0; i < 6; ++i) {
            cudaError_t e = src[i] ? (src[i] == dst[i] ? cudaSuccess
                                                        : cudaMemcpyAsync(dst[i], src[i], n[i] * 4,
                                                                          cudaMemcpyDeviceToDevice, st))
                                   : cudaMemsetAsync(dst[i], 0, n[i] * 4, st);
            if (e != cudaSuccess) return cuda_fail(e);
        }
        return PMA_OK;
    }
    const Plan pl = selective_plan(L, D, q->dtype);
    const ProPass pp = pro_pass(pl, pro, B, H, L, y != nullptr);
    if (pp.total && (!workspace || workspace_bytes < pp.total)) return PMA_ERR_WORKSPACE;
    if (pp.total && reinterpret_cast<uintptr_t>(workspace) % 16) return PMA_ERR_WORKSPACE;
    PrefillParams p{};
    p.B = B;
    p.H = H;
    p.L = L;
    p.seg_len = pl.seg_len;
    p.q = seq_of(q);
    p.k = seq_of(k);
    p.v = seq_of(v);
    p.pro = pro;
    p.y = seqout_of(y);
    p.lambda = beta;  // not read on the per-token path; any valid pointer
    p.lam_sb = 0;
    p.in = user_ref(state_in);
    p.out = user_ref(state_out);
    p.eps = eps;
    p.state_only = 0;
    p.status = nullptr;
    p.fault = g_fault_word.load();
    p.test_wait_ns = g_test_wait_ns.load();
    p.logdecay = log_decay;
    p.k_head_scale = beta;
    p.half_sq = 1;
    cudaError_t e;
    if (pl.tc) {
        p.status = reinterpret_cast<int *>(workspace);
        if ((e = cudaMemsetAsync(p.status, 0, sizeof(int), st)) != cudaSuccess) return cuda_fail(e);
        if ((e = run_prologue_passes(pp, pro, p, B, H, L, workspace, y != nullptr, di.sms, st)) != cudaSuccess)
            return cuda_fail(e);
        e = launch_prefill_tc(p, y ? y->dtype : PMA_F32, dim3(BH, 1), st);
    } else {
        e = launch_prefill_simt(p, D, q->dtype, y ? y->dtype : PMA_F32, dim3(BH, 1), st);
    }
    return e == cudaSuccess ? PMA_OK : cuda_fail(e);
}

int pma_selective_decode_step(int N, int H, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                              const pma_seq_tensor *v, const pma_prologue *prologue, const float *log_decay,
                              const float *beta, const int32_t *rows, int pool_rows, const pma_state *state_in,
                              const pma_state *state_out, float eps, const pma_seq_tensor *y,
                              pma_stream_t stream) {
    if (!beta) return PMA_ERR_ARGUMENT;
    return decode_impl(N, H, D, q, k, v, prologue, log_decay, H, rows, pool_rows, state_in, state_out, eps, y,
                       stream, beta, true);
}

int pma_swiglu(int64_t rows, int inter, const void *gate, int64_t gate_stride, const void *up, int64_t up_stride,
               void *out, int64_t out_stride, int dtype, pma_stream_t stream) {
    if (rows < 0 || inter <= 0 || gate_stride < inter || up_stride < inter || out_stride < inter)
        return PMA_ERR_ARGUMENT;
    if (!supported_dtype(dtype)) return PMA_ERR_DTYPE;
    if (rows == 0) return PMA_OK;
    if (!gate || !up || !out) return PMA_ERR_ARGUMENT;
    int rc;
    DevInfo di;
    if ((rc = device_info(&di))) return rc;
    cudaError_t e = launch_swiglu(dtype, gate, gate_stride, up, up_stride, out, out_stride, rows, inter, di.sms,
                                  reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? PMA_OK : cuda_fail(e);
}

int pma_state_combine(int B, int H, int D, const float *lambda, int64_t lambda_stride_b, int64_t len,
                      const pma_state *T, const pma_state *P, pma_stream_t stream) {
    if (B < 0 || H <= 0 || !lambda || lambda_stride_b < 0 || len < 0) return PMA_ERR_ARGUMENT;
    if (!supported_d(D)) return PMA_ERR_HEAD_DIM;
    int rc;
    if ((rc = check_state(T)) || (rc = check_state(P))) return rc;
    DevInfo di;
    if ((rc = device_info(&di))) return rc;
    if (B == 0) return PMA_OK;
    cudaError_t e = launch_state_combine(B, H, D, lambda, lambda_stride_b, len, *T, *P,
                                         reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? PMA_OK : cuda_fail(e);
}

}  // extern "C"
