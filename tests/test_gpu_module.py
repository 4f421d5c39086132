"""Module-level parity: the PrimeMomentAttention mirror (projections, GQA repeat, LayerNorm
QK-norm, 1/sqrt(D) scale in PyTorch; core on the CUDA kernels) against the same module math
in float64 on the CPU with the float64 token-recurrence oracle as the core.

Covers the reference module's three L branches (attention.py:118-202: decode L == 1,
dense 1 < L <= 512, chunked L > 512), with and without an incoming state, GQA, per-head
decay, fp32 and bf16 module dtypes."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import TOL_BF16, TOL_F32
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _reference(m, x, state, lam, exact):
    """The module's math with the core on the float64 oracle: returns (out [B,L,hidden], final
    state tuple).  exact: projections, norm and scale in float64 on the CPU; otherwise in the
    module's own dtype on its device (so a bf16 module's rounding of q, k, v and y is the
    reference's too and the comparison isolates the core)."""
    dev, cdt = (torch.device("cpu"), torch.float64) if exact else (x.device, x.dtype)
    P = lambda t: t.detach().to(dev, cdt)
    W = {n: P(getattr(m, n).weight) for n in ("q_proj", "k_proj", "v_proj", "o_proj")}
    x = P(x)
    B, L, _ = x.shape
    H, Hk, D = m.num_heads, m.num_kv_heads, m.head_dim
    q = (x @ W["q_proj"].T).view(B, L, H, D).transpose(1, 2)
    k = (x @ W["k_proj"].T).view(B, L, Hk, D).transpose(1, 2)
    v = (x @ W["v_proj"].T).view(B, L, Hk, D).transpose(1, 2)
    if H != Hk:
        k = k.repeat_interleave(H // Hk, dim=1)
        v = v.repeat_interleave(H // Hk, dim=1)
    if m.use_qk_norm:
        q = F.layer_norm(q, (D,), P(m.q_norm.weight), P(m.q_norm.bias), m.q_norm.eps)
        k = F.layer_norm(k, (D,), P(m.k_norm.weight), P(m.k_norm.bias), m.k_norm.eps)
    q = q * m.scaling
    c64 = lambda t: t.detach().to("cpu", torch.float64).numpy()
    st = None if state is None else tuple(c64(t) for t in state)
    y, s = O.prefill(c64(q), c64(k), c64(v), lam, st, m.eps)
    y = torch.from_numpy(y).to(dev, cdt).transpose(1, 2).reshape(B, L, H * D)
    return c64(y @ W["o_proj"].T), s


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL_F32), (torch.bfloat16, TOL_BF16)])
@pytest.mark.parametrize("L,with_state", [(1, False), (1, True), (300, True), (1000, False), (1000, True)])
def test_module_forward_matches_float64_module_math(dtype, tol, L, with_state):
    import prime_moment_attention_b200 as pma
    from prime_moment_attention_b200 import synth
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    H, Hk, D, hidden, B = 4, 2, 64, 256, 2
    lam = np.exp(np.random.default_rng(1).uniform(np.log(0.99), np.log(0.9999), H))
    m = pma.PrimeMomentAttention(hidden, H, D, num_kv_heads=Hk, decay=lam.tolist(), use_qk_norm=True)
    with torch.no_grad():
        for ln in (m.q_norm, m.k_norm):  # non-trivial affine parameters
            ln.weight.uniform_(0.5, 1.5)
            ln.bias.uniform_(-0.1, 0.1)
    m = m.to("cuda", dtype)
    x = (torch.randn(B, L, hidden, generator=torch.Generator().manual_seed(2)) * 0.5).to("cuda", dtype)
    state = None
    if with_state:
        state = synth.make_state(B, H, D, torch.tensor(lam, dtype=torch.float32), seed=3, t0=512, sigma=0.01,
                                 device="cuda")
    with torch.inference_mode():
        out, st = m(x, state=state, return_state=True)
    torch.cuda.synchronize()
    with torch.inference_mode():
        ref_out, ref_st = _reference(m, x, state, lam, exact=dtype == torch.float32)
    e = O.rel_err(out.double().cpu().numpy(), ref_out)
    assert e <= tol, e
    for a, b in zip(st, ref_st):
        e = O.rel_err(a.double().cpu().numpy().reshape(b.shape), b)
        assert e <= tol, e
