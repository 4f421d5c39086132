// prefill.cuh -- parameters and launchers shared by the prefill kernels.
#pragma once

#include "pma_common.cuh"

namespace pma {

// One launch processes gridDim.y segments of seg_len tokens for each of
// gridDim.x = B*H head-states.  Segment s of head-state bh covers tokens
// [s*seg_len, min((s+1)*seg_len, L)).
struct PrefillParams {
    int B, H, L;
    int seg_len;          // multiple of the kernel's chunk
    Seq q, k, v;          // k, v: H / pro.groups heads
    Prologue pro;
    SeqOut y;             // y.p == nullptr: no output rows
    const float *lambda;
    int64_t lam_sb;
    StateRef in;          // state entering each segment (packed: slot = segment); absent = zero
    StateRef out;         // user: final state (last segment only); packed: slot = segment
    float eps;
    int state_only;       // 1: skip the readout, start every segment from zero, write its state to `out`
    int *status;          // device status word (0 = ok); bounded waits record a code here
    int *fault;           // registered fault word (pma_set_fault_word) or nullptr: expired waits record a code
    unsigned long long test_wait_ns;  // test hook (pma_test_expire_waits): nonzero makes one wait expire
    // selective variant (CUDA-core kernel only, one segment):
    const float *logdecay;      // [B*H*L] log lambda_t per token, or nullptr (lambda per head)
    const float *k_head_scale;  // [H] k multiplied by it (the temperature beta_h), or nullptr
    int half_sq;                // 1: user states hold S2, Z2 halved (the selective layout)
    int y_tma;                  // D = 64 tensor-core kernel: bf16 y rows leave through a TMA store
};

// Workspace layout: [header: 256 B, int status word first][per-segment states, float32].
constexpr size_t WS_HEADER = 256;

// PMA_ERR_CUDA, with `e` recorded for pma_last_cuda_error() on the calling thread.
int cuda_fail(cudaError_t e);

struct DecodeParams {
    int N, H;
    Seq q, k, v;            // [N,H,D] (stride_l unused); k, v: H / pro.groups heads
    Prologue pro;
    SeqOut y;
    const float *lambda;
    int64_t lam_sn;
    pma_state in, out;
    float eps;
    const int32_t *rows;    // nullable: state row of batch row n (a state pool), else n
    int pool_rows;          // rows in the pool (bounds for `rows`)
    int log_lambda;         // 1: `lambda` holds log lambda (the selective variant's per-token decay)
    const float *k_head_scale;  // [H] or nullptr: k multiplied by it
    int half_sq;            // 1: S2, Z2 held halved, read out without the 1/2 (selective layout)
};

// Gated delta-rule variant (delta.cu).  State per head-state: S [D][2D] float32, row-major.
struct DeltaParams {
    int B, H, L;
    Seq q, k, v;
    SeqOut y;                 // y.p == nullptr: state only
    const float *beta;        // [B*H*L]
    const float *alpha;       // [B*H*L] or nullptr (alpha_t = lambda)
    const float *lambda;      // lambda[b * lam_sb + h]: decay of padded tokens (and alpha when absent)
    int64_t lam_sb;
    float bound, norm_eps;
    const float *state_in;    // [B*H][D][2D] or nullptr (zero)
    float *state_out;         // [B*H][D][2D] or nullptr
    int *fault;               // registered fault word or nullptr (tensor-core kernel's expired waits)
    unsigned long long test_wait_ns;  // test hook (pma_test_expire_waits), WY kernels only
};
struct DeltaStepParams {
    int N, H;
    Seq q, k, v;
    SeqOut y;
    const float *beta, *alpha;  // [N*H]
    float bound, norm_eps;
    const float *state_in;
    float *state_out;
};
bool delta_supported(int D, int chunk);
bool delta_tc_supported(int D, int chunk, int idt);
cudaError_t launch_delta_prefill_tc(const DeltaParams &p, int ydt, cudaStream_t st);
// WY form (delta_wy.cu): same cases as the tensor-core kernel, with a workspace; the preferred
// size is delta_wy_workspace_bytes(B, H, L), and a smaller one runs in windows of
// delta_wy_window(...) chunks (0: too small).
size_t delta_wy_workspace_bytes(int B, int H, int L);
int delta_wy_window(int B, int H, int L, size_t ws_bytes);
cudaError_t launch_delta_prefill_wy(const DeltaParams &p, int ydt, void *ws, int window, cudaStream_t st);
cudaError_t launch_delta_prefill(const DeltaParams &p, int D, int chunk, int idt, int ydt, cudaStream_t st);
cudaError_t launch_delta_step(const DeltaStepParams &p, int D, int idt, int ydt, cudaStream_t st);

cudaError_t launch_decode(const DecodeParams &p, int D, int idt, int ydt, cudaStream_t s);
cudaError_t launch_prefill_simt(const PrefillParams &p, int D, int idt, int ydt, dim3 grid, cudaStream_t st);
int simt_chunk(int D);
cudaError_t launch_segment_prefix(int BH, int H, int D, int nseg, int seg_len, int L, float *ws, const StateRef &in,
                                  const StateRef &final_out, const float *lambda, int64_t lam_sb, cudaStream_t st);
// ws[s] += l^(s * seg_len) * in for every segment s (in: user-layout states entering the sequence).
cudaError_t launch_segment_resume(int BH, int H, int D, int nseg, int seg_len, float *ws, const StateRef &in,
                                  const float *lambda, int64_t lam_sb, cudaStream_t st);
cudaError_t launch_state_combine(int B, int H, int D, const float *lambda, int64_t lam_sb, int64_t len,
                                 const pma_state &T, const pma_state &P, cudaStream_t st);

// QK-norm pass for the tensor-core path: rows of src [B, Hs, L, 64] bf16 (any strides) ->
// contiguous dst, (LN(x) if w else x) * scale.
cudaError_t launch_qk_norm(const Seq &src, int B, int Hs, int L, const float *w, const float *b, float eps,
                           float scale, void *dst, int sms, cudaStream_t st);

// silu(gate) * up over rows x inter elements (row strides in elements), bf16 or float32.
cudaError_t launch_swiglu(int dtype, const void *g, int64_t gs, const void *u, int64_t us, void *o, int64_t os,
                          int64_t rows, int inter, int sms, cudaStream_t st);

// tcgen05 tensor-core prefill (bf16 inputs, D = 64).
constexpr int TC_CHUNK = 128;
bool tc_supported(int D, int idt);
cudaError_t launch_prefill_tc(const PrefillParams &p, int ydt, dim3 grid, cudaStream_t st);
// tcgen05 tensor-core prefill for D = 128 (bf16 inputs, per-head decay, no LayerNorm prologue,
// q scale exact in bf16).
bool tc128_supported(int idt);
cudaError_t launch_prefill_tc128(const PrefillParams &p, int ydt, dim3 grid, cudaStream_t st);
// State-only pass at D = 128 (y not wanted): one accumulating GEMM per segment (state_tc128.cu).
cudaError_t launch_state_tc128(const PrefillParams &p, dim3 grid, cudaStream_t st);

}  // namespace pma
