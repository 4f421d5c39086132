"""Input prologue (pma_prefill_ex / pma_decode_step_ex): GQA head map, LayerNorm QK-norm and
q scale folded into the kernels, against the module math of attention.py:92-101 (repeat,
LayerNorm, scale) done in float64 followed by the float64 token-recurrence oracle.

Inputs are raw projections in the module's layout: transposed views of [B, L, Hkv, D] with a
per-row offset, so the norm's mean subtraction matters.  Covers the tensor-core kernel (bf16,
D = 64; its prologue variant, its state-only variant on split sequences and its small-decay
CUDA-core path), the CUDA-core kernel (float32, other head dims), decode and pool decode."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import TOL_BF16, TOL_F32
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _raw(B, L, Hq, Hkv, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, L, Hq, D, generator=g) * 1.5 + torch.randn(B, L, Hq, 1, generator=g)
    k = torch.randn(B, L, Hkv, D, generator=g) * 1.5 + torch.randn(B, L, Hkv, 1, generator=g)
    v = torch.randn(B, L, Hkv, D, generator=g)
    return [t.to(dtype).cuda().transpose(1, 2) for t in (q, k, v)]  # [B, H, L, D] strided views


def _params(D, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.rand(D, generator=g) + 0.5).cuda(), (torch.randn(D, generator=g) * 0.1).cuda(),
            (torch.rand(D, generator=g) + 0.5).cuda(), (torch.randn(D, generator=g) * 0.1).cuda()]


def _module_math(q, k, v, groups, norm, scale, eps_ln=1e-5):
    """float64 numpy q, k, v [B,H,L,D] after repeat_interleave, LayerNorm and scale."""
    c = lambda t: t.detach().to("cpu", torch.float64)
    q, k, v = c(q), c(k), c(v)
    if groups > 1:
        k = k.repeat_interleave(groups, dim=1)
        v = v.repeat_interleave(groups, dim=1)
    if norm is not None:
        qw, qb, kw, kb = [None if t is None else c(t) for t in norm]
        if qw is not None:
            q = F.layer_norm(q, (q.shape[-1],), qw, qb, eps_ln)
        if kw is not None:
            k = F.layer_norm(k, (k.shape[-1],), kw, kb, eps_ln)
    return (q * scale).numpy(), k.numpy(), v.numpy()


def _pro(groups, norm, scale):
    from prime_moment_attention_b200 import ops
    n = norm or [None] * 4
    return ops.Prologue(kv_groups=groups, q_scale=scale, q_norm_weight=n[0], q_norm_bias=n[1], k_norm_weight=n[2],
                        k_norm_bias=n[3])


CASES = [  # dtype, D, B, Hq, groups, L, which norms ("qk", "q", "k", ""), lambda range
    (torch.bfloat16, 64, 2, 6, 3, 700, "qk", (0.99, 0.9999)),     # tensor cores, GQA, both norms
    (torch.bfloat16, 64, 2, 4, 1, 300, "", (0.99, 0.9999)),       # tensor cores, scale only
    (torch.bfloat16, 64, 1, 4, 2, 2000, "k", (0.995, 0.9999)),    # split sequences: state-only pass + k norm
    (torch.bfloat16, 64, 1, 2, 2, 260, "q", (0.3, 0.5)),          # small decay: CUDA-core path in the TC kernel
    (torch.float32, 64, 2, 6, 2, 333, "qk", (0.99, 0.9999)),      # CUDA cores
    (torch.float32, 128, 1, 4, 4, 200, "qk", (0.99, 0.9999)),     # CUDA cores, D = 128, all heads share kv
    (torch.bfloat16, 32, 2, 4, 2, 150, "qk", (0.99, 0.9999)),     # bf16 on CUDA cores
]


@pytest.mark.parametrize("dtype,D,B,Hq,groups,L,norms,lr", CASES)
@pytest.mark.parametrize("with_state", [False, True])
def test_prefill_prologue(dtype, D, B, Hq, groups, L, norms, lr, with_state):
    from prime_moment_attention_b200 import ops, synth
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    q, k, v = _raw(B, L, Hq, Hq // groups, D, dtype, seed=D + L)
    p = _params(D, seed=L)
    norm = [p[0] if "q" in norms else None, p[1] if "q" in norms else None,
            p[2] if "k" in norms else None, p[3] if "k" in norms else None]
    scale = 1.0 / np.sqrt(D)
    lam = synth.make_lambdas(Hq, lr[0], lr[1], seed=7)
    st_in = synth.make_state(B, Hq, D, lam, seed=8, t0=256, sigma=0.01, device="cuda") if with_state else None
    y, st = ops.prefill(q, k, v, lam.cuda(), state=st_in, out_dtype=torch.float32,
                        prologue=_pro(groups, norm, scale), check=True)
    torch.cuda.synchronize()
    qr, kr, vr = _module_math(q, k, v, groups, norm, scale)
    st_np = None if st_in is None else tuple(t.double().cpu().numpy() for t in st_in)
    y_ref, s_ref = O.prefill(qr, kr, vr, lam.double().numpy(), st_np)
    e = O.rel_err(y.double().cpu().numpy(), y_ref)
    assert e <= tol, f"y {e:.3e}"
    for a, b in zip(st, s_ref):
        e = O.rel_err(a.double().cpu().numpy().reshape(b.shape), b)
        assert e <= tol, f"state {e:.3e}"


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 64), (torch.float32, 64), (torch.float32, 128),
                                     (torch.bfloat16, 16)])
@pytest.mark.parametrize("groups,norms", [(2, "qk"), (1, "k"), (4, "")])
def test_decode_prologue(dtype, D, groups, norms):
    from prime_moment_attention_b200 import ops, synth
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    N, Hq = 5, 8
    q, k, v = [t[:, :, 0] for t in _raw(N, 1, Hq, Hq // groups, D, dtype, seed=D + groups)]
    p = _params(D, seed=groups)
    norm = [p[0] if "q" in norms else None, p[1] if "q" in norms else None,
            p[2] if "k" in norms else None, p[3] if "k" in norms else None]
    scale = 1.0 / np.sqrt(D)
    lam = synth.make_lambdas(Hq, 0.99, 0.9999, seed=3)
    st_in = synth.make_state(N, Hq, D, lam, seed=4, t0=512, sigma=0.01, device="cuda")
    y, st = ops.decode_step(q, k, v, lam.cuda(), st_in, out_dtype=torch.float32, prologue=_pro(groups, norm, scale))
    torch.cuda.synchronize()
    qr, kr, vr = _module_math(q.unsqueeze(2), k.unsqueeze(2), v.unsqueeze(2), groups, norm, scale)
    y_ref, s_ref = O.prefill(qr, kr, vr, lam.double().numpy(), tuple(t.double().cpu().numpy() for t in st_in))
    assert O.rel_err(y.double().cpu().numpy(), y_ref[:, :, 0]) <= tol
    for a, b in zip(st, s_ref):
        assert O.rel_err(a.double().cpu().numpy().reshape(b.shape), b) <= tol


def test_pool_decode_prologue():
    """pma_decode_step_ex with a row table: permuted pool rows, GQA and both norms."""
    from prime_moment_attention_b200 import ops, synth
    N, Hq, groups, D, P = 3, 6, 3, 64, 7
    q, k, v = [t[:, :, 0] for t in _raw(N, 1, Hq, Hq // groups, D, torch.bfloat16, seed=11)]
    norm = _params(D, seed=12)
    lam = synth.make_lambdas(Hq, 0.99, 0.9999, seed=5)
    pool = synth.make_state(P, Hq, D, lam, seed=6, t0=512, sigma=0.01, device="cuda")
    pool = tuple(t.contiguous() for t in pool)
    before = tuple(t.double().cpu().numpy() for t in pool)
    rows = torch.tensor([5, 0, 3], dtype=torch.int32, device="cuda")
    y = ops.decode_step_rows(q, k, v, lam.cuda(), pool, rows, out_dtype=torch.float32,
                             prologue=_pro(groups, norm, 0.125))
    torch.cuda.synchronize()
    qr, kr, vr = _module_math(q.unsqueeze(2), k.unsqueeze(2), v.unsqueeze(2), groups, norm, 0.125)
    for n, r in enumerate(rows.tolist()):
        st = tuple(b[r:r + 1] for b in before)
        y_ref, s_ref = O.prefill(qr[n:n + 1], kr[n:n + 1], vr[n:n + 1], lam.double().numpy(), st)
        assert O.rel_err(y[n].double().cpu().numpy(), y_ref[0, :, 0]) <= TOL_BF16
        for a, b in zip(pool, s_ref):
            assert O.rel_err(a[r:r + 1].double().cpu().numpy().reshape(b.shape), b) <= TOL_BF16


def test_prologue_argument_errors():
    from prime_moment_attention_b200 import _lib, ops
    q, k, v = _raw(1, 10, 4, 2, 64, torch.bfloat16, seed=1)
    with pytest.raises(ValueError):
        ops.prefill(q, k, v, 0.99, prologue=ops.Prologue(kv_groups=3))  # does not divide H
    with pytest.raises(ValueError):
        ops.prefill(q, k, v, 0.99, prologue=ops.Prologue(q_norm_weight=torch.ones(32, device="cuda")))
    # C-level check: kv_groups that does not divide H is refused before any launch
    with pytest.raises(_lib.PmaError):
        ops.prefill(q, k[:, :1].expand(1, 1, 10, 64), v[:, :1].expand(1, 1, 10, 64), 0.99,
                    prologue=ops.Prologue(kv_groups=4, q_scale=float("nan")))
