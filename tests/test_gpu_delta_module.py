"""Module-level parity of the gated delta-rule mirror (ChunkedGatedDeltaPrimeAttention): the
projections, gates, GQA repeat, QK-norm and scale of chunked_delta_prime.py:101-137 in
float64 on the CPU followed by the float64 delta oracle, against the module on the kernels,
for the step branch (L == 1) and the chunked branch (ragged L, with and without state)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import TOL_BF16, TOL_F32
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _reference(m, x, state, exact):
    """exact: projections and gates in float64 on the CPU; otherwise in the module's dtype on
    its device (a bf16 module's own rounding of q, k, v and the gates is then the reference's
    too, and the comparison isolates the core)."""
    c = (lambda t: t.detach().to("cpu", torch.float64)) if exact else (lambda t: t.detach())
    x = c(x)
    B, L, _ = x.shape
    H, Hk, D = m.num_heads, m.num_kv_heads, m.head_dim
    lin = lambda mod: F.linear(x, c(mod.weight), None if mod.bias is None else c(mod.bias))
    q = lin(m.q_proj).view(B, L, H, D).transpose(1, 2)
    k = lin(m.k_proj).view(B, L, Hk, D).transpose(1, 2)
    v = lin(m.v_proj).view(B, L, Hk, D).transpose(1, 2)
    bg = torch.sigmoid(lin(m.erase_proj)).view(B, L, H, D).transpose(1, 2)
    wg = torch.sigmoid(lin(m.write_proj)).view(B, L, H, D).transpose(1, 2)
    k = k.repeat_interleave(H // Hk, dim=1)
    v = v.repeat_interleave(H // Hk, dim=1)
    if m.use_qk_norm:
        q = F.layer_norm(q, (D,), c(m.q_norm.weight), c(m.q_norm.bias), m.q_norm.eps)
        k = F.layer_norm(k, (D,), c(m.k_norm.weight), c(m.k_norm.bias), m.k_norm.eps)
    q = q * m.scaling
    beta = wg.float().mean(-1) * 0.5
    alpha = m.decay * (1 - bg.float().mean(-1) * 0.5)
    st = None if state is None else state.detach().double().cpu().numpy()
    if L == 1:
        y, s = O.delta_step(q[:, :, 0], k[:, :, 0], v[:, :, 0], beta[:, :, 0], alpha[:, :, 0],
                            st if st is not None else np.zeros((B, H, D, 2 * D)), bound=m.lyapunov_bound,
                            norm_eps=m.eps)
        y = torch.from_numpy(y).to(x.device, x.dtype).reshape(B, 1, H * D)
    else:
        y, s = O.delta_prefill(q, k, v, beta, alpha, np.full(H, m.decay), chunk=m.chunk_size,
                               bound=m.lyapunov_bound, norm_eps=m.eps, state=st)
        y = torch.from_numpy(y).to(x.device, x.dtype).transpose(1, 2).reshape(B, L, H * D)
    return (y @ c(m.o_proj.weight).T).double().cpu().numpy(), s


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL_F32), (torch.bfloat16, TOL_BF16)])
@pytest.mark.parametrize("L,with_state", [(1, False), (1, True), (100, False), (200, True)])
def test_delta_module_forward(dtype, tol, L, with_state):
    import prime_moment_attention_b200 as pma
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    m = pma.ChunkedGatedDeltaPrimeAttention(hidden_size=128, num_heads=4, head_dim=32, num_kv_heads=2,
                                            chunk_size=32, decay=0.995, lyapunov_bound=6.0)
    with torch.no_grad():
        for ln in (m.q_norm, m.k_norm):
            ln.weight.uniform_(0.5, 1.5)
            ln.bias.uniform_(-0.1, 0.1)
    m = m.to("cuda", dtype)
    x = torch.randn(2, L, 128, generator=torch.Generator().manual_seed(1)).to("cuda", dtype)
    st = (torch.randn(2, 4, 32, 64, generator=torch.Generator().manual_seed(2)) * 0.3).cuda() if with_state else None
    with torch.inference_mode():
        out, s = m(x, state=st, return_state=True)
        torch.cuda.synchronize()
        ref_out, ref_s = _reference(m, x, st, exact=dtype == torch.float32)
    e = O.rel_err(out.double().cpu().numpy(), ref_out)
    assert e <= tol, e
    e = O.rel_err(s.double().cpu().numpy(), ref_s)
    assert e <= tol, e
