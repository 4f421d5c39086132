/*
 * pma.h -- C ABI of the B200 (sm_100a) PRIME moment attention hot path.
 *
 * Library: prime_moment_attention_b200/libpma.so (nvcc, -gencode arch=compute_100a,code=sm_100a).
 * Plain C types only: device pointers, sizes, strides, a CUDA stream handle.
 *
 * Semantics are those of the reference PyTorch path (paths relative to the
 * PRIME-Moment-Attention project root).  Per head-state, with decay l in (0,1],
 * q pre-scaled by 1/sqrt(D) (attention.py:101), for every token t in order:
 *
 *     S0 = l S0 + v            Z0 = l Z0 + 1
 *     S1 = l S1 + k v^T        Z1 = l Z1 + k          (S1[d][e]: d = key index)
 *     S2 = l S2 + (k*k) v^T    Z2 = l Z2 + k*k
 *     y  = (S0 + q^T S1 + 0.5 (q*q)^T S2) / max(Z0 + q.Z1 + 0.5 (q*q).Z2, eps)
 *
 * The reference names Z0, Z1, Z2 "K0, K1, K2" (attention.py:19-24).
 *
 * Conventions
 *   - Every entry point returns an int status (pma_status); 0 is success.  Argument
 *     errors are found on the host before anything is launched.  Kernels are
 *     launched on `stream` (NULL = the legacy default stream) and run
 *     asynchronously; PMA_ERR_CUDA reports a launch failure.
 *   - No entry point allocates device memory.  Scratch space is passed in
 *     (pma_prefill_workspace_bytes says how much), except for
 *     pma_prefill_no_alloc, whose scratch is a static device buffer.
 *   - Entry points are re-entrant.  Global mutable state: a per-device cache of
 *     kernel attributes set once; the fault word registered with
 *     pma_set_fault_word (and the test hook pma_test_expire_waits); and the
 *     static scratch buffer of pma_prefill_no_alloc with its per-device,
 *     per-context cache of the buffer's address.
 *   - Kernels that wait (the tensor-core prefills) bound every wait; a wait that
 *     expires stops the launch early with unwritten outputs and records a nonzero
 *     code in the workspace status word and in the registered fault word.
 *   - Sequence tensors (q, k, v, y) are [B, H, L, D] with arbitrary element
 *     strides on B, H, L and a contiguous D axis, so both the reference's
 *     [B,H,L,D] tensors and its transposed views of [B,L,H,D] projections
 *     (attention.py:87-89) are accepted without a copy.
 *   - States are float32, contiguous, in the reference tuple layout
 *     (attention.py:111-117).
 */
#ifndef PMA_H
#define PMA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PMA_ABI_VERSION 4

#if defined(__GNUC__)
#define PMA_API __attribute__((visibility("default")))
#else
#define PMA_API
#endif

/* Same type as cudaStream_t. */
typedef struct CUstream_st *pma_stream_t;

typedef enum {
    PMA_OK = 0,
    PMA_ERR_ARGUMENT = 1,   /* null pointer where one is required, negative size   */
    PMA_ERR_HEAD_DIM = 2,   /* head_dim not supported by any kernel                */
    PMA_ERR_DTYPE = 3,      /* element type not supported                          */
    PMA_ERR_LAYOUT = 4,     /* stride/alignment the kernels cannot address         */
    PMA_ERR_WORKSPACE = 5,  /* workspace missing or smaller than required          */
    PMA_ERR_CUDA = 6,       /* a CUDA runtime call or kernel launch failed         */
    PMA_ERR_DEVICE = 7      /* current device is not sm_100 (B200 class)           */
} pma_status;

typedef enum {
    PMA_F32 = 0,
    PMA_BF16 = 1
} pma_dtype;

/* A [B, H, L, D] device tensor with element strides; D is contiguous. */
typedef struct {
    void *data;
    int32_t dtype;     /* pma_dtype */
    int64_t stride_b;
    int64_t stride_h;
    int64_t stride_l;
} pma_seq_tensor;

/* Six contiguous float32 device arrays holding B x H head-states.
 * Reference tuple (S0, S1, S2, K0, K1, K2) of attention.py:111-117. */
typedef struct {
    float *S0;   /* [B, H, D]                       */
    float *S1;   /* [B, H, D, D]  row = key index   */
    float *S2;   /* [B, H, D, D]  row = key index   */
    float *Z0;   /* [B, H]   (reference K0 [B,H,1]) */
    float *Z1;   /* [B, H, D]                       */
    float *Z2;   /* [B, H, D]                       */
} pma_state;

/*
 * Optional per-call input prologue: the module work between the q/k/v projections
 * and the core (attention.py:87-101), folded into the kernels' load stage so the
 * projection outputs are read once, in place:
 *   - GQA: k and v hold H / kv_groups heads; query head h reads kv head
 *     h / kv_groups, which is what k.repeat_interleave(kv_groups, dim=1) gives
 *     (attention.py:92-94), without the copy;
 *   - LayerNorm over the head dim with affine weight/bias on q and on k
 *     (nn.LayerNorm(head_dim), attention.py:73-75, 96-98): biased variance,
 *     y = (x - mean) / sqrt(var + norm_eps) * weight + bias;
 *   - q scaled by q_scale after its norm (1/sqrt(D), attention.py:101).
 * The prologue is computed in float32 from the input elements; with bf16 inputs
 * the normalised, scaled q and k are rounded to bf16 once before the tensor-core
 * products (the reference rounds after the norm and again after the scale).
 * Weights and biases are device float32 arrays of D elements.
 */
typedef struct {
    int32_t kv_groups;            /* >= 1 */
    float q_scale;                /* 1.0f: q used as given */
    const float *q_norm_weight;   /* NULL: no LayerNorm on q */
    const float *q_norm_bias;     /* NULL: zero bias */
    const float *k_norm_weight;   /* NULL: no LayerNorm on k */
    const float *k_norm_bias;     /* NULL: zero bias */
    float norm_eps;               /* LayerNorm eps (nn.LayerNorm default 1e-5) */
} pma_prologue;

/* ABI version (PMA_ABI_VERSION of the built library). */
PMA_API int pma_version(void);

/* Static text for a status code. */
PMA_API const char *pma_status_string(int status);

/* When an entry point returned PMA_ERR_CUDA: the cudaError_t behind it (most
 * recent such failure on the calling thread; 0 if none) and its text. */
PMA_API int pma_last_cuda_error(void);
PMA_API const char *pma_cuda_error_string(int cuda_error);

/*
 * Registers `word`, a device-accessible int (device memory, or pinned host memory,
 * which the host can read at any time without synchronising), as the process-wide
 * fault word: every later launch of a kernel with bounded waits (the tensor-core
 * prefills: pma_prefill, pma_prefill_ex, pma_prefill_no_alloc, pma_selective_prefill,
 * pma_delta_prefill) stores the code of the first wait that expires into it when it
 * still reads 0.  The library never clears it; NULL unregisters.  No counterpart in
 * the reference, which has no device waits (its only failure signals are NaN checks,
 * c/main.c:92-98 and model.py:221,228).
 */
PMA_API void pma_set_fault_word(int *word);

/*
 * Test hook for the failure path: with limit_ns > 0, every later launch of the moment
 * prefill on tensor cores (pma_prefill, pma_prefill_ex, pma_prefill_resume,
 * pma_prefill_no_alloc, pma_selective_prefill; not the delta-rule prefill) first waits,
 * with that bound, for a barrier phase that nothing completes;
 * the wait expires before any copy or GEMM is issued, the launch records code 90
 * (workspace status word and fault word) and returns without writing outputs.
 * 0 restores normal operation.  For tests only; no counterpart in the reference.
 */
PMA_API void pma_test_expire_waits(unsigned long long limit_ns);

/* Floats in one head-state: 2*D*D + 3*D + 1 (c/prime_moment.h:17 states the
 * same count for the reference's C runtime). */
PMA_API size_t pma_state_floats(int D);

/* Head dims the kernels support for each input dtype: writes up to `cap`
 * values into `dims` and returns how many there are. */
PMA_API int pma_supported_head_dims(int dtype, int *dims, int cap);

/*
 * Bytes of scratch pma_prefill needs for this problem (0 if none).
 * Replaces nothing in the reference; the reference allocates through ATen.
 */
PMA_API size_t pma_prefill_workspace_bytes(int B, int H, int L, int D, int dtype);

/*
 * Chunked prefill of L tokens for B x H head-states.
 *
 * Replaces chunked_prime_ssd_core (src/prime_moment_attention/chunked_ssd.py:48-184)
 * and the dense short-sequence branch of PrimeMomentAttention.forward
 * (attention.py:160-202); also the sequential prime_prefill_cpp
 * (prime_cpp_kernel.cpp:6-47) and C prime_prefill (c/prime_moment.c:332-352).
 *
 *   q, k, v     [B,H,L,D], all the same dtype (F32 or BF16); q pre-scaled.
 *   lambda      device float array; head h of batch row b uses
 *               lambda[b * lambda_stride_b + h] (stride 0: one decay per head).
 *   state_in    NULL = zero initial state (the reference's state=None), else the
 *               incoming state.  Unlike chunked_ssd.py:129-137 any B, H, L work.
 *   state_out   NULL = final state not wanted (return_state=False); else receives
 *               the state after token L-1.  May alias state_in.
 *   eps         denominator clamp (1.0 in the reference module, attention.py:51).
 *   y           [B,H,L,D] output, F32 or BF16 (any strides, D contiguous); NULL
 *               computes only state_out (the state-only pass used by sequence
 *               sharding).
 *   workspace   device scratch of at least pma_prefill_workspace_bytes(...).
 *
 * F32 inputs are computed with float32 arithmetic throughout (CUDA cores).
 * BF16 inputs with D = 64 or D = 128 run on tcgen05 tensor cores: bf16 operands,
 * float32 accumulation, float32 state.  L == 0 copies state_in to state_out.
 */
PMA_API int pma_prefill(int B, int H, int L, int D,
                const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                const float *lambda, int64_t lambda_stride_b,
                const pma_state *state_in, const pma_state *state_out,
                float eps, const pma_seq_tensor *y,
                void *workspace, size_t workspace_bytes, pma_stream_t stream);

/*
 * Output pass of a two-pass prefill, for callers that learn the state entering a sequence only
 * after they have its state from a zero start (sequence shards on several GPUs: every shard's
 * zero-start state is exchanged before any shard can compute its outputs).  A state-only
 * pma_prefill call (y = NULL, state_in = NULL) leaves in its workspace the state entering each
 * of its segments from a zero start; given that same workspace, unchanged, and the same B, H, L,
 * D, q, k, v, lambda and device, this call adds lambda^start * state_in to those states and runs
 * the full pass from them, without repeating the state-only pass.  y is required; other arguments
 * and results as pma_prefill.  When the plan has one segment per head-state the workspace holds
 * no states and this is pma_prefill.
 *
 * Replaces the second of the two chunked_prime_ssd_core calls a sequence split over devices would
 * need; the reference's own inter-chunk carry is the dense [nc x nc] matmul of chunked_ssd.py:113-126.
 */
PMA_API int pma_prefill_resume(int B, int H, int L, int D,
                               const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                               const float *lambda, int64_t lambda_stride_b,
                               const pma_state *state_in, const pma_state *state_out,
                               float eps, const pma_seq_tensor *y,
                               void *workspace, size_t workspace_bytes, pma_stream_t stream);

/*
 * pma_prefill without a caller-provided workspace, for callers that cannot
 * allocate device memory (a plugin whose host application owns all device memory
 * through its own pool, FFI callers without a device allocator, loops where an
 * allocation would synchronise the device).  No counterpart in the reference:
 * the reference always allocates through ATen.
 *
 * Same arguments and results as pma_prefill.  Its scratch is a 16 MiB buffer
 * compiled into the library (one per GPU that loads it, held until exit);
 * problems whose plan needs more (pma_prefill_workspace_bytes > 16 MiB: float32
 * or D = 128 with few head-states and long sequences) return PMA_ERR_WORKSPACE.
 * The first call on a device looks up the buffer's device address; make it
 * before any stream capture.  The address is kept per device together with the
 * CUDA context that was current, and looked up again when another context is
 * current; it does not survive a cudaDeviceReset of the device.  All calls on a
 * device share the buffer: calls that overlap on the GPU race and must be
 * serialised by the caller.  The buffer holds the status word, out of the
 * caller's reach: register a fault word (pma_set_fault_word) to see an expired
 * wait.  Allocates nothing.
 */
PMA_API int pma_prefill_no_alloc(int B, int H, int L, int D,
                                 const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                                 const float *lambda, int64_t lambda_stride_b,
                                 const pma_state *state_in, const pma_state *state_out,
                                 float eps, const pma_seq_tensor *y, pma_stream_t stream);

/*
 * One recurrent decode step for N x H head-states (N = batch rows, or
 * sequences x layers when all layers' heads are batched in one launch).
 *
 * Replaces the L == 1 branch of PrimeMomentAttention.forward
 * (attention.py:120-143); also prime_step_evict_update_cpp followed by
 * prime_query_step_cpp (prime_cpp_kernel.cpp:84-117) and the additive mode of
 * prime_step (c/prime_moment.c:274-312).
 *
 *   q, k, v, y  [N,H,D] tensors described as pma_seq_tensor with L = 1
 *               (stride_b = row stride, stride_h = head stride, stride_l ignored).
 *   lambda      lambda[n * lambda_stride_n + h].
 *   state_in    required; state_out required; they may be the same arrays
 *               (in-place update) or disjoint (functional update, as the
 *               reference returns new tensors).
 */
PMA_API int pma_decode_step(int N, int H, int D,
                    const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                    const float *lambda, int64_t lambda_stride_n,
                    const pma_state *state_in, const pma_state *state_out,
                    float eps, const pma_seq_tensor *y, pma_stream_t stream);

/*
 * Decode step over rows of a device-resident state pool: batch row n (q, k, v, y
 * row n) updates pool row rows[n] in place (pool_in == pool_out) or into pool_out.
 * The pool holds pool_rows x H head-states in the pma_state layout; rows is a device
 * int32 array of N entries; entries outside [0, pool_rows) are skipped (y row left
 * untouched).  Same math and traffic as pma_decode_step.
 *
 * Replaces the per-layer state tuples that PrimeMomentCache.get_state/set_state
 * hand to the decode branch (src/prime_moment_attention/cache.py:15-56,
 * attention.py:120-143): a serving loop keeps every sequence's state in one pool
 * and changes the batch by changing `rows`, with no gather/scatter copies.
 */
PMA_API int pma_decode_step_rows(int N, int H, int D,
                                 const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                                 const float *lambda, int64_t lambda_stride_n,
                                 const int32_t *rows, int pool_rows,
                                 const pma_state *pool_in, const pma_state *pool_out,
                                 float eps, const pma_seq_tensor *y, pma_stream_t stream);

/*
 * Bytes of scratch pma_prefill_ex needs (0 if none): pma_prefill_workspace_bytes
 * plus, on the tensor-core path (bf16, D = 64) with a LayerNorm in the prologue, room
 * for the normalised bf16 q and/or k rows (2 * D bytes per row).
 */
PMA_API size_t pma_prefill_ex_workspace_bytes(int B, int H, int L, int D, int dtype,
                                              const pma_prologue *prologue);

/*
 * pma_prefill with an input prologue (GQA head map, LayerNorm QK-norm, q scale):
 * the module forward of attention.py:86-207 minus the projection GEMMs.  q is the
 * raw q projection [B,H,L,D]; k and v are the raw k/v projections with
 * H / prologue->kv_groups heads (typically transposed views of [B,L,Hkv,D]).
 * prologue NULL is the identity prologue (= pma_prefill).  workspace: at least
 * pma_prefill_ex_workspace_bytes(...).  Other arguments and results as pma_prefill;
 * PMA_ERR_ARGUMENT if kv_groups < 1 or does not divide H.
 * The CUDA-core kernels apply the prologue as they load rows.  The tensor-core kernels
 * apply the GQA map in their tensor-map coordinates and a bf16-exact q_scale as they stage
 * q.  At D = 64, LayerNorms (and a q_scale bf16 cannot hold) run first as one HBM pass that
 * writes the normalised rows into the workspace (128 bytes read + 128 written per row); at
 * D = 128 such a prologue selects the CUDA-core kernel.
 */
PMA_API int pma_prefill_ex(int B, int H, int L, int D,
                           const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                           const pma_prologue *prologue,
                           const float *lambda, int64_t lambda_stride_b,
                           const pma_state *state_in, const pma_state *state_out,
                           float eps, const pma_seq_tensor *y,
                           void *workspace, size_t workspace_bytes, pma_stream_t stream);

/*
 * Decode step with an input prologue and an optional state-pool row table: the
 * L == 1 module branch (attention.py:86-143, 205) minus the projection GEMMs.
 * k and v have H / prologue->kv_groups heads.  rows NULL: batch row n uses state
 * row n (as pma_decode_step, state arrays of N x H head-states); else as
 * pma_decode_step_rows with pool_rows rows.  prologue NULL is the identity.
 */
PMA_API int pma_decode_step_ex(int N, int H, int D,
                               const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                               const pma_prologue *prologue,
                               const float *lambda, int64_t lambda_stride_n,
                               const int32_t *rows, int pool_rows,
                               const pma_state *state_in, const pma_state *state_out,
                               float eps, const pma_seq_tensor *y, pma_stream_t stream);

/*
 * Gated delta-rule variant (ChunkedGatedDeltaPrimeAttention,
 * src/prime_moment_attention/chunked_delta_prime.py:25-283).  Per head-state the state is
 * S [D][2D] float32 (row = value index, column = feature), contiguous, B x H head-states.
 * Features per token (:73-87): psi = [q, q^2/sqrt 2], phi = [k/max(|k|,e), (k^2/max(|k^2|,e))/sqrt 2]
 * with e = norm_eps (the module's eps, 1e-5).  beta (write rate) and alpha (retention) are
 * per token: the module's beta = mean(sigmoid(write_proj))/2 and
 * alpha = decay * (1 - mean(sigmoid(erase_proj))/2) (:134-137).
 */

/*
 * Chunked delta-rule prefill (:175-283).  Replaces the L > 1 branch of
 * ChunkedGatedDeltaPrimeAttention.forward after the projections and gates.
 *
 *   q, k, v     [B,H,L,D] (F32 or BF16, same dtype; q pre-scaled by 1/sqrt(D)); D in {16, 32, 64}.
 *   beta        device float [B,H,L] contiguous.
 *   alpha       device float [B,H,L] contiguous, or NULL: alpha_t = lambda of the head.
 *   lambda      lambda[b * lambda_stride_b + h]: the module's decay, used for the padded tokens
 *               of a ragged last chunk (the reference pads alpha with it, so the final state
 *               carries decay^pad, :178-185) and as alpha when alpha is NULL.
 *   chunk       the reference's chunk_size (32 or 64): the Lyapunov projection
 *               S *= min(1, bound / (|S|_F + 1e-6)) runs at every chunk end (:267-270);
 *               lyapunov_bound <= 0 turns it off.
 *   state_in    [B,H,D,2D] or NULL (zero); state_out [B,H,D,2D] or NULL; they may alias.
 *   y           [B,H,L,D] (F32 or BF16) or NULL (state only; then state_out is required).
 *   workspace   device scratch of pma_delta_prefill_workspace_bytes(...) bytes, or NULL / 0.
 * BF16 inputs with D = 64 and chunk 64 run on the tensor cores: with a workspace in the WY form
 * (every chunk's T^-1 products computed in parallel, then one sequential pass per head-state over
 * the state-dependent products), without one as a single pass per head-state that solves each
 * chunk's triangular system in turn.  Other cases are computed in float32 on CUDA cores (one CTA
 * per head-state, state in shared memory) and need no workspace.
 */
PMA_API int pma_delta_prefill(int B, int H, int L, int D,
                              const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                              const float *beta, const float *alpha,
                              const float *lambda, int64_t lambda_stride_b,
                              int chunk, float lyapunov_bound, float norm_eps,
                              const float *state_in, float *state_out,
                              const pma_seq_tensor *y,
                              void *workspace, size_t workspace_bytes, pma_stream_t stream);

/*
 * Bytes of workspace with which pma_delta_prefill takes its WY path (0 when the case has none:
 * not BF16 / D = 64 / chunk 64, or nothing to compute).  72 KB per (head-state, chunk) of a
 * window of chunks whose records stay within 1 GiB, plus one state copy per head-state when the
 * sequence spans several windows.  A smaller workspace runs the sequence in smaller windows; one
 * that holds less than one chunk per head-state (plus the state copy) is refused with
 * PMA_ERR_WORKSPACE.  The workspace must be 256-byte aligned.
 */
PMA_API size_t pma_delta_prefill_workspace_bytes(int B, int H, int L, int D, int chunk, int dtype);

/*
 * Delta-rule decode step: the L == 1 branch (:142-172), which measures the error against the
 * undecayed state:  e = v - S phi;  S = alpha S + beta e phi^T;  Lyapunov projection;  y = S psi.
 *   q, k, v, y  [N,H,D] (pma_seq_tensor with L = 1); beta, alpha device float [N,H].
 *   state_in, state_out  [N,H,D,2D]; may be the same arrays (in place).
 * One HBM read and one write of each state.
 */
PMA_API int pma_delta_decode_step(int N, int H, int D,
                                  const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                                  const float *beta, const float *alpha,
                                  float lyapunov_bound, float norm_eps,
                                  const float *state_in, float *state_out,
                                  const pma_seq_tensor *y, pma_stream_t stream);

/*
 * Selective variant (PrimeSelectiveMomentAttention, src/prime_moment_attention/selective.py:264-444):
 * the moment recurrence with a decay per token, lambda_t = exp(-Delta_t / tau_h), and a
 * temperature beta_h per head on k:
 *     S0 = l S0 + v,  S1 = l S1 + b k v^T,  S2 = l S2 + b^2/2 k^2 v^T,  Z0 = l Z0 + 1,
 *     Z1 = l Z1 + b k,  Z2 = l Z2 + b^2/2 k^2,
 *     y = (S0 + q.S1 + q^2.S2) / max(Z0 + q.Z1 + q^2.Z2, eps)
 * States use the reference's selective layout (the 1/2 b^2 sits in S2 and Z2).
 *
 * Prefill over L tokens (the reference's parallel branch, :401-435, and its step branch iterated
 * when a state is given -- the reference's parallel branch ignores an incoming state; this entry
 * carries it, as the step branch does).
 *   log_decay   device float [B,H,L] contiguous: -Delta_t / tau_h.
 *   beta        device float [H]: the temperature (clamp(exp(log_beta), 0.1, 15) in the module).
 *   prologue    as pma_prefill_ex (GQA map, QK-norm, q scale) or NULL.
 *   workspace   at least pma_selective_prefill_workspace_bytes(...) bytes (256 for the tensor-core
 *               path, plus the normalised rows when the prologue has LayerNorms; 0 otherwise).
 * BF16 inputs with D = 64 run on tcgen05 tensor cores (per-chunk exp(+-cumulative log decay)
 * factors in place of the per-head powers; head-states with a chunk that decays by more than
 * e^-76 run the float32 loop); float32 inputs and other D run in float32 on CUDA cores.
 */
PMA_API size_t pma_selective_prefill_workspace_bytes(int B, int H, int L, int D, int dtype,
                                                     const pma_prologue *prologue);
PMA_API int pma_selective_prefill(int B, int H, int L, int D,
                                  const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                                  const pma_prologue *prologue, const float *log_decay, const float *beta,
                                  const pma_state *state_in, const pma_state *state_out,
                                  float eps, const pma_seq_tensor *y,
                                  void *workspace, size_t workspace_bytes, pma_stream_t stream);

/*
 * Selective decode step (the L == 1 branch, selective.py:367-396): log_decay [N,H]
 * (-Delta_t / tau_h of this token), beta [H]; rows / pool_rows as pma_decode_step_ex
 * (NULL rows: state row n).  state_in and state_out may be the same arrays.
 */
PMA_API int pma_selective_decode_step(int N, int H, int D,
                                      const pma_seq_tensor *q, const pma_seq_tensor *k, const pma_seq_tensor *v,
                                      const pma_prologue *prologue, const float *log_decay, const float *beta,
                                      const int32_t *rows, int pool_rows,
                                      const pma_state *state_in, const pma_state *state_out,
                                      float eps, const pma_seq_tensor *y, pma_stream_t stream);

/*
 * Segment carry: P <- lambda^len * P + T for B x H head-states, elementwise over
 * all six components.  len = tokens in the segment that produced T.
 * This is the associative step of the reference's inter-chunk scan
 * (chunked_ssd.py:113-126, evaluated there as a dense [nc x nc] matmul); here it
 * joins sequence shards computed on different GPUs.
 */
PMA_API int pma_state_combine(int B, int H, int D, const float *lambda, int64_t lambda_stride_b,
                      int64_t len, const pma_state *T, const pma_state *P,
                      pma_stream_t stream);

/*
 * SwiGLU activation of the model's MLP in one pass: out = silu(gate) * up over
 * rows x inter elements (PrimeMLP.forward, src/prime_moment_attention/model.py:59-68,
 * where PyTorch runs silu and the product as two kernels).  Row strides are in
 * elements (>= inter; the element axis is contiguous); dtype PMA_BF16 or PMA_F32 for
 * all three arrays.  silu is computed in float32 and rounded to the storage type
 * before the product, as the two-kernel sequence does, so results are identical.
 */
PMA_API int pma_swiglu(int64_t rows, int inter, const void *gate, int64_t gate_stride,
                       const void *up, int64_t up_stride, void *out, int64_t out_stride,
                       int dtype, pma_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PMA_H */
