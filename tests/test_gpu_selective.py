"""Selective variant (pma_selective_prefill, pma_selective_decode_step, PrimeSelectiveMomentAttention)
against the golden vectors of the reference module and the float64 selective oracle."""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import TOL_BF16, TOL_F32
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
NAMES = ("S0", "S1", "S2", "K0", "K1", "K2")


def _cuda(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a), dtype=dtype).cuda()


def _check_state(st, ref, tol):
    for a, b, n in zip(st, ref, NAMES):
        b = np.asarray(b)
        e = O.rel_err(a.double().cpu().numpy().reshape(b.shape), b)
        assert e <= tol, (n, e)


def test_selective_prefill_golden():
    from prime_moment_attention_b200 import ops
    g = dict(np.load(os.path.join(GOLD, "selective_par_d32.npz")))
    y, st = ops.selective_prefill(_cuda(g["q"]), _cuda(g["k"]), _cuda(g["v"]), _cuda(g["log_decay"]),
                                  _cuda(g["beta"]))
    torch.cuda.synchronize()
    assert O.rel_err(y.double().cpu().numpy(), g["y"]) <= TOL_F32
    _check_state(st, [g["st_" + n] for n in NAMES], TOL_F32)


@pytest.mark.parametrize("via", ["decode", "prefill"])
def test_selective_step_golden(via):
    from prime_moment_attention_b200 import ops
    g = dict(np.load(os.path.join(GOLD, "selective_step_d16.npz")))
    st = tuple(_cuda(g["in_" + n]) for n in NAMES)
    for t in range(g["q"].shape[2]):
        args = [_cuda(g[n][:, :, t]) for n in ("q", "k", "v")]
        if via == "decode":
            y, st = ops.selective_decode_step(*args, _cuda(g["log_decay"][:, :, t]), _cuda(g["beta"]), st)
        else:
            y, st = ops.selective_prefill(*[a.unsqueeze(2) for a in args], _cuda(g["log_decay"][:, :, t:t + 1]),
                                          _cuda(g["beta"]), state=st)
            y = y[:, :, 0]
        torch.cuda.synchronize()
        assert O.rel_err(y.double().cpu().numpy(), g["y"][:, :, t]) <= TOL_F32
    _check_state(st, [g["st_" + n] for n in NAMES], TOL_F32)


def _case(B, H, L, D, seed, dtype, tau_range=(3.0, 2000.0)):
    gen = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, H, L, D, generator=gen), dim=-1) / D ** 0.5
    k = F.normalize(torch.randn(B, H, L, D, generator=gen), dim=-1)
    v = torch.randn(B, H, L, D, generator=gen)
    tau = torch.exp(torch.linspace(np.log(tau_range[0]), np.log(tau_range[1]), H))
    delta = F.softplus(torch.randn(B, L, H, generator=gen)).clamp(1e-4, 50.0)
    ld = (-delta / tau.view(1, 1, H)).transpose(1, 2).contiguous()
    beta = torch.exp(torch.randn(H, generator=gen) * 0.4).clamp(0.1, 15.0)
    return q.to(dtype), k.to(dtype), v.to(dtype), ld, beta


def _state(B, H, D, seed):
    gen = torch.Generator().manual_seed(seed)
    s = [torch.randn(B, H, *sh, generator=gen) * 0.05 for sh in [(D,), (D, D), (D, D), (1,), (D,), (D,)]]
    s[3] = s[3].abs() + 20.0
    return tuple(s)


@pytest.mark.parametrize("B,H,L,D,dtype,with_state,taus", [
    (2, 3, 200, 64, torch.float32, False, (3.0, 2000.0)), (1, 2, 130, 128, torch.float32, True, (3.0, 2000.0)),
    (2, 2, 77, 32, torch.float32, True, (3.0, 2000.0)),
    (2, 4, 300, 64, torch.bfloat16, True, (3.0, 2000.0)),     # tensor cores
    (1, 2, 1, 16, torch.bfloat16, True, (3.0, 2000.0)),
    (1, 3, 1000, 64, torch.bfloat16, False, (3.0, 2000.0)),   # tensor cores, 8 chunks, ragged tail
    (2, 4, 260, 64, torch.bfloat16, True, (0.3, 30.0)),       # steep heads fall back to CUDA cores
    (1, 2, 128, 64, torch.bfloat16, False, (1.2, 1.5)),       # chunk decay near the e^-76 edge
])
def test_selective_prefill_vs_oracle(B, H, L, D, dtype, with_state, taus):
    from prime_moment_attention_b200 import ops
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    q, k, v, ld, beta = _case(B, H, L, D, seed=L + D, dtype=dtype, tau_range=taus)
    st = _state(B, H, D, seed=3) if with_state else None
    y, s = ops.selective_prefill(q.cuda(), k.cuda(), v.cuda(), ld.cuda(), beta.cuda(),
                                 state=None if st is None else tuple(t.cuda() for t in st), out_dtype=torch.float32)
    torch.cuda.synchronize()
    y_ref, s_ref = O.selective_prefill(q, k, v, ld, beta, st)
    assert O.rel_err(y.double().cpu().numpy(), y_ref) <= tol
    _check_state(s, s_ref, tol)


@pytest.mark.parametrize("D,dtype", [(64, torch.bfloat16), (64, torch.float32), (128, torch.float32)])
def test_selective_decode_vs_oracle_and_pool_rows(D, dtype):
    from prime_moment_attention_b200 import ops
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    N, H, P = 4, 3, 7
    q, k, v, ld, beta = _case(N, H, 1, D, seed=D, dtype=dtype)
    pool = tuple(t.cuda().contiguous() for t in _state(P, H, D, seed=4))
    before = tuple(t.double().cpu().numpy() for t in pool)
    rows = torch.tensor([6, 0, 3, 2], dtype=torch.int32, device="cuda")
    y, _ = ops.selective_decode_step(q[:, :, 0].cuda(), k[:, :, 0].cuda(), v[:, :, 0].cuda(), ld[:, :, 0].cuda(),
                                     beta.cuda(), pool, rows=rows, out_dtype=torch.float32)
    torch.cuda.synchronize()
    for n, r in enumerate(rows.tolist()):
        y_ref, s_ref = O.selective_prefill(q[n:n + 1], k[n:n + 1], v[n:n + 1], ld[n:n + 1], beta,
                                           tuple(b[r:r + 1] for b in before))
        assert O.rel_err(y[n].double().cpu().numpy(), y_ref[0, :, 0]) <= tol
        _check_state([t[r:r + 1] for t in pool], s_ref, tol)
    untouched = [r for r in range(P) if r not in rows.tolist()]
    for t, b in zip(pool, before):
        assert np.array_equal(t.double().cpu().numpy()[untouched], b[untouched])


def _module_reference(m, x, state, exact):
    c = (lambda t: t.detach().to("cpu", torch.float64)) if exact else (lambda t: t.detach())
    x = c(x)
    B, L, _ = x.shape
    H, Hk, D = m.num_heads, m.num_kv_heads, m.head_dim
    lin = lambda mod: F.linear(x, c(mod.weight), None if mod.bias is None else c(mod.bias))
    q = lin(m.q_proj).view(B, L, H, D).transpose(1, 2)
    k = lin(m.k_proj).view(B, L, Hk, D).transpose(1, 2).repeat_interleave(H // Hk, dim=1)
    v = lin(m.v_proj).view(B, L, Hk, D).transpose(1, 2).repeat_interleave(H // Hk, dim=1)
    q = F.layer_norm(q, (D,), c(m.q_norm.weight), c(m.q_norm.bias), m.q_norm.eps)
    k = F.layer_norm(k, (D,), c(m.k_norm.weight), c(m.k_norm.bias), m.k_norm.eps)
    q = q * m.scaling
    tau = torch.clamp(torch.exp(c(m.log_tau).double()), m.min_tau, m.max_tau)
    beta = torch.clamp(torch.exp(c(m.log_beta).double()), 0.1, 15.0)
    delta = F.softplus(lin(m.delta_proj).double()).clamp(1e-4, 50.0)
    ld = (-delta / tau.to(delta.device).view(1, 1, H)).transpose(1, 2)
    st = None if state is None else tuple(t.double().cpu() for t in state)
    y, s = O.selective_prefill(q, k, v, ld, beta, st, eps=m.eps)
    y = torch.from_numpy(y).to(x.device, x.dtype).transpose(1, 2).reshape(B, L, H * D)
    return (y @ c(m.o_proj.weight).T).double().cpu().numpy(), s


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL_F32), (torch.bfloat16, TOL_BF16)])
@pytest.mark.parametrize("L,with_state,D", [(1, True, 32), (150, False, 32), (150, True, 32), (300, True, 64)])
def test_selective_module_forward(dtype, tol, L, with_state, D):
    """D = 64 bf16 runs the tensor-core path with the QK-norm pass in front of it."""
    import prime_moment_attention_b200 as pma
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    m = pma.PrimeSelectiveMomentAttention(hidden_size=128, num_heads=4, head_dim=D, num_kv_heads=2, decay=0.99)
    with torch.no_grad():
        m.delta_proj.weight.normal_(0, 0.1)
        m.log_tau.copy_(torch.log(torch.tensor([3.0, 30.0, 300.0, 1500.0])))
        m.log_beta.copy_(torch.tensor([0.3, -0.2, 0.0, 0.5]))
        for ln in (m.q_norm, m.k_norm):
            ln.weight.uniform_(0.5, 1.5)
            ln.bias.uniform_(-0.1, 0.1)
    m = m.to("cuda", dtype)
    x = torch.randn(2, L, 128, generator=torch.Generator().manual_seed(1)).to("cuda", dtype)
    st = tuple(t.cuda() for t in _state(2, 4, D, seed=5)) if with_state else None
    with torch.inference_mode():
        out, s = m(x, state=st, return_state=True)
        torch.cuda.synchronize()
        ref_out, ref_s = _module_reference(m, x, st, exact=dtype == torch.float32)
    assert O.rel_err(out.double().cpu().numpy(), ref_out) <= tol
    _check_state(s, ref_s, tol)
