// torch_ops.cpp -- torch.ops.pma.*: the C ABI of include/pma.h registered as PyTorch operators.
//
// The reference exposes its native kernels to Python as a pybind module of libtorch functions
// (prime_cpp_kernel.cpp:119-124: prime_prefill_cpp, prime_query_step_cpp, ...).  Here the same
// role is played by operators in the dispatcher, so that the prefill and the decode step are
// callable without Python ctypes and are visible to torch.compile / torch.export as opaque ops
// (their shape functions are registered from Python, prime_moment_attention_b200/torch_ops.py).
//
//   pma::prefill(q, k, v, decay, state?, eps, return_state) -> (y, state[])
//   pma::decode_step(q, k, v, decay, state, eps) -> (y, new state[])        functional
//   pma::decode_step_(q, k, v, decay, state(a!), eps) -> y                   state updated in place
//
// Tensors as in the C ABI: q, k, v [B,H,L,D] (decode: [N,H,D]) bf16 or float32 with a contiguous
// head dim; decay a float32 CUDA tensor [H] or [B,H]; states the reference tuple (S0, S1, S2, K0,
// K1, K2), float32.  Work goes on the current CUDA stream; scratch comes from PyTorch's caching
// allocator.  CUDA tensors only: the operators have no CPU kernel.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <string>
#include <tuple>
#include <vector>

#include "../../include/pma.h"

namespace {

void check_rc(int rc, const char *fn) {
    if (rc == PMA_OK) return;
    std::string msg = std::string(fn) + " failed: " + pma_status_string(rc);
    if (rc == PMA_ERR_CUDA) msg += std::string(": ") + pma_cuda_error_string(pma_last_cuda_error());
    TORCH_CHECK(false, msg);
}

int dtype_of(const at::Tensor &t) {
    if (t.scalar_type() == at::kFloat) return PMA_F32;
    if (t.scalar_type() == at::kBFloat16) return PMA_BF16;
    TORCH_CHECK(false, "pma: float32 or bfloat16 tensors only, got ", t.scalar_type());
}

// [B,H,L,D] (four_d) or [N,H,D]; a copy only when the head dim is not contiguous or a row is not
// 16-byte aligned.
at::Tensor addressable(const at::Tensor &t) {
    const int64_t step = 16 / t.element_size();
    bool ok = t.stride(-1) == 1 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0;
    for (int64_t i = 0; ok && i + 1 < t.dim(); ++i) ok = t.stride(i) % step == 0 && t.stride(i) >= 0;
    return ok ? t : t.contiguous();
}

pma_seq_tensor seq_of(const at::Tensor &t) {
    pma_seq_tensor s{};
    s.data = t.data_ptr();
    s.dtype = dtype_of(t);
    s.stride_b = t.stride(0);
    s.stride_h = t.stride(1);
    s.stride_l = t.dim() == 4 ? t.stride(2) : 0;
    return s;
}

// One allocation for a state of B x H head-states, Z0 last so every other part is 16-byte aligned.
std::vector<at::Tensor> new_state(int64_t B, int64_t H, int64_t D, const at::Device &dev) {
    const int64_t BH = B * H;
    at::Tensor flat = at::empty({BH * (2 * D * D + 3 * D + 1)}, at::TensorOptions().dtype(at::kFloat).device(dev));
    const int64_t o[6] = {0, BH * D, BH * D * (D + 1), BH * D * (2 * D + 1), BH * D * (2 * D + 2),
                          BH * D * (2 * D + 3)};
    return {flat.narrow(0, o[0], BH * D).view({B, H, D}),     flat.narrow(0, o[1], BH * D * D).view({B, H, D, D}),
            flat.narrow(0, o[2], BH * D * D).view({B, H, D, D}), flat.narrow(0, o[5], BH).view({B, H, 1}),
            flat.narrow(0, o[3], BH * D).view({B, H, D}),     flat.narrow(0, o[4], BH * D).view({B, H, D})};
}

// The six tensors as a pma_state; they must be float32, contiguous, on `dev`, in the reference shapes.
pma_state state_of(at::TensorList st, int64_t B, int64_t H, int64_t D, const at::Device &dev, const char *what) {
    TORCH_CHECK(st.size() == 6, what, ": expected the 6-tuple (S0, S1, S2, K0, K1, K2)");
    const std::vector<std::vector<int64_t>> shapes = {{B, H, D}, {B, H, D, D}, {B, H, D, D}, {B, H, 1}, {B, H, D}, {B, H, D}};
    for (size_t i = 0; i < 6; ++i) {
        const at::Tensor &t = st[i];
        TORCH_CHECK(t.device() == dev && t.scalar_type() == at::kFloat && t.is_contiguous(), what, "[", i,
                    "] must be a contiguous float32 tensor on ", dev);
        TORCH_CHECK(t.numel() == (i == 3 ? B * H : c10::multiply_integers(shapes[i])), what, "[", i, "] has shape ",
                    t.sizes(), ", expected ", at::IntArrayRef(shapes[i]));
    }
    pma_state s{};
    s.S0 = st[0].data_ptr<float>();
    s.S1 = st[1].data_ptr<float>();
    s.S2 = st[2].data_ptr<float>();
    s.Z0 = st[3].data_ptr<float>();
    s.Z1 = st[4].data_ptr<float>();
    s.Z2 = st[5].data_ptr<float>();
    return s;
}

// decay [H] (stride 0 over batch rows) or [B,H] (stride H), float32 on the device.
std::pair<at::Tensor, int64_t> decay_of(const at::Tensor &decay, int64_t B, int64_t H, const at::Device &dev) {
    TORCH_CHECK(decay.device() == dev, "decay must be on ", dev);
    at::Tensor d = decay.to(at::kFloat).contiguous();
    if (d.numel() == H && (d.dim() <= 1 || B == 1)) return {d.reshape({H}), 0};
    TORCH_CHECK(d.numel() == B * H, "decay must have H or B*H elements, got ", d.sizes());
    return {d.reshape({B * H}), H};
}

void check_cuda(const at::Tensor &t, const char *name) {
    TORCH_CHECK(t.is_cuda(), "pma: ", name, " must be a CUDA tensor (no CPU fallback)");
}

std::tuple<at::Tensor, std::vector<at::Tensor>> prefill(const at::Tensor &q_in, const at::Tensor &k_in,
                                                        const at::Tensor &v_in, const at::Tensor &decay,
                                                        std::optional<at::TensorList> state, double eps,
                                                        bool return_state) {
    check_cuda(q_in, "q");
    check_cuda(k_in, "k");
    check_cuda(v_in, "v");
    TORCH_CHECK(q_in.dim() == 4 && k_in.sizes() == q_in.sizes() && v_in.sizes() == q_in.sizes(),
                "q, k, v must share one [B,H,L,D] shape");
    TORCH_CHECK(k_in.scalar_type() == q_in.scalar_type() && v_in.scalar_type() == q_in.scalar_type(),
                "q, k, v must share one dtype");
    const c10::cuda::CUDAGuard guard(q_in.device());
    const at::Device dev = q_in.device();
    const int64_t B = q_in.size(0), H = q_in.size(1), L = q_in.size(2), D = q_in.size(3);
    const at::Tensor q = addressable(q_in), k = addressable(k_in), v = addressable(v_in);
    auto [lam, lam_sb] = decay_of(decay, B, H, dev);
    at::Tensor y = at::empty({B, H, L, D}, q.options());
    std::vector<at::Tensor> out = return_state ? new_state(B, H, D, dev) : std::vector<at::Tensor>{};
    pma_state st_in{}, st_out{};
    std::vector<at::Tensor> in_keep;
    if (state.has_value()) {
        for (const at::Tensor &t : *state) in_keep.push_back(t.to(dev, at::kFloat).contiguous());
        st_in = state_of(in_keep, B, H, D, dev, "state");
    }
    if (return_state) st_out = state_of(out, B, H, D, dev, "state_out");
    const pma_seq_tensor qs = seq_of(q), ks = seq_of(k), vs = seq_of(v), ys = seq_of(y);
    const size_t ws_bytes = pma_prefill_workspace_bytes((int)B, (int)H, (int)L, (int)D, dtype_of(q));
    at::Tensor ws = at::empty({(int64_t)std::max<size_t>(ws_bytes, 1)}, q.options().dtype(at::kByte));
    const cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
    check_rc(pma_prefill((int)B, (int)H, (int)L, (int)D, &qs, &ks, &vs, lam.data_ptr<float>(), lam_sb,
                         state.has_value() ? &st_in : nullptr, return_state ? &st_out : nullptr, (float)eps, &ys,
                         ws.data_ptr(), ws_bytes, reinterpret_cast<pma_stream_t>(stream)),
             "pma_prefill");
    return {y, out};
}

at::Tensor decode_into(const at::Tensor &q_in, const at::Tensor &k_in, const at::Tensor &v_in, const at::Tensor &decay,
                       at::TensorList state_in, at::TensorList state_out, double eps) {
    check_cuda(q_in, "q");
    check_cuda(k_in, "k");
    check_cuda(v_in, "v");
    TORCH_CHECK(q_in.dim() == 3 && k_in.sizes() == q_in.sizes() && v_in.sizes() == q_in.sizes(),
                "q, k, v must share one [N,H,D] shape");
    TORCH_CHECK(k_in.scalar_type() == q_in.scalar_type() && v_in.scalar_type() == q_in.scalar_type(),
                "q, k, v must share one dtype");
    const c10::cuda::CUDAGuard guard(q_in.device());
    const at::Device dev = q_in.device();
    const int64_t N = q_in.size(0), H = q_in.size(1), D = q_in.size(2);
    const at::Tensor q = addressable(q_in), k = addressable(k_in), v = addressable(v_in);
    auto [lam, lam_sn] = decay_of(decay, N, H, dev);
    const pma_state si = state_of(state_in, N, H, D, dev, "state");
    const pma_state so = state_of(state_out, N, H, D, dev, "state_out");
    at::Tensor y = at::empty({N, H, D}, q.options());
    const pma_seq_tensor qs = seq_of(q), ks = seq_of(k), vs = seq_of(v), ys = seq_of(y);
    const cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
    check_rc(pma_decode_step((int)N, (int)H, (int)D, &qs, &ks, &vs, lam.data_ptr<float>(), lam_sn, &si, &so,
                             (float)eps, &ys, reinterpret_cast<pma_stream_t>(stream)),
             "pma_decode_step");
    return y;
}

std::tuple<at::Tensor, std::vector<at::Tensor>> decode_step(const at::Tensor &q, const at::Tensor &k,
                                                            const at::Tensor &v, const at::Tensor &decay,
                                                            at::TensorList state, double eps) {
    TORCH_CHECK(q.dim() == 3, "q must be [N,H,D]");
    std::vector<at::Tensor> in;
    for (const at::Tensor &t : state) in.push_back(t.to(q.device(), at::kFloat).contiguous());
    std::vector<at::Tensor> out = new_state(q.size(0), q.size(1), q.size(2), q.device());
    at::Tensor y = decode_into(q, k, v, decay, in, out, eps);
    return {y, out};
}

at::Tensor decode_step_(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v, const at::Tensor &decay,
                        at::TensorList state, double eps) {
    return decode_into(q, k, v, decay, state, state, eps);  // state_of insists on contiguous float32
}

}  // namespace

TORCH_LIBRARY(pma, m) {
    m.def("prefill(Tensor q, Tensor k, Tensor v, Tensor decay, Tensor[]? state=None, float eps=1.0, "
          "bool return_state=True) -> (Tensor, Tensor[])");
    m.def("decode_step(Tensor q, Tensor k, Tensor v, Tensor decay, Tensor[] state, float eps=1.0) -> (Tensor, Tensor[])");
    m.def("decode_step_(Tensor q, Tensor k, Tensor v, Tensor decay, Tensor(a!)[] state, float eps=1.0) -> Tensor");
}

TORCH_LIBRARY_IMPL(pma, CUDA, m) {
    m.impl("prefill", &prefill);
    m.impl("decode_step", &decode_step);
    m.impl("decode_step_", &decode_step_);
}
