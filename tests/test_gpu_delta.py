"""Gated delta-rule kernels (pma_delta_prefill, pma_delta_decode_step) against the golden
vectors of the reference module and against the float64 delta oracle on seeded inputs.

Cases follow the reference's own behaviour (chunked_delta_prime.py): ragged last chunks with the
decay^pad factor on the final state, the Lyapunov projection at chunk ends (active with small
bounds), incoming states, per-token or per-head retention, chunk sizes 32 and 64, D = 16/32/64,
float32 and bf16 inputs, state-only calls, and the L == 1 step with its undecayed error."""
import os

import numpy as np
import pytest
import torch

from helpers import TOL_BF16, TOL_F32
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _cuda(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a), dtype=dtype).cuda()


@pytest.mark.parametrize("name", ["delta_c32_d16", "delta_c64_d32_st", "delta_c64_d64"])
def test_delta_prefill_golden(name):
    from prime_moment_attention_b200 import ops
    g = dict(np.load(os.path.join(GOLD, name + ".npz")))
    st = _cuda(g["state_in"]) if "state_in" in g else None
    y, s = ops.delta_prefill(_cuda(g["q"]), _cuda(g["k"]), _cuda(g["v"]), _cuda(g["beta"]), _cuda(g["alpha"]),
                             _cuda(g["lam"]), chunk=int(g["chunk"]), lyapunov_bound=float(g["bound"]), state=st)
    torch.cuda.synchronize()
    assert O.rel_err(y.double().cpu().numpy(), g["y"]) <= TOL_F32
    assert O.rel_err(s.double().cpu().numpy(), g["state"]) <= TOL_F32


def test_delta_step_golden():
    from prime_moment_attention_b200 import ops
    g = dict(np.load(os.path.join(GOLD, "delta_step_d32.npz")))
    st = _cuda(g["state_in"])
    for t in range(g["q"].shape[2]):
        y, st = ops.delta_decode_step(_cuda(g["q"][:, :, t]), _cuda(g["k"][:, :, t]), _cuda(g["v"][:, :, t]),
                                      _cuda(g["beta"][:, :, t]), _cuda(g["alpha"][:, :, t]), st,
                                      lyapunov_bound=float(g["bound"]))
        torch.cuda.synchronize()
        assert O.rel_err(y.double().cpu().numpy(), g["y"][:, :, t]) <= TOL_F32
    assert O.rel_err(st.double().cpu().numpy(), g["state"]) <= TOL_F32


def _case(B, H, L, D, seed, dtype, per_token_alpha):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, D, generator=g), dim=-1) / D ** 0.5
    k = torch.randn(B, H, L, D, generator=g)
    v = torch.randn(B, H, L, D, generator=g)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=g))
    lam = torch.exp(torch.empty(H).uniform_(np.log(0.99), np.log(0.9999), generator=g))
    alpha = (lam.view(1, H, 1) * (1 - 0.5 * torch.sigmoid(torch.randn(B, H, L, generator=g) - 2))) \
        if per_token_alpha else None
    q, k, v = (t.to(dtype) for t in (q, k, v))
    return q, k, v, beta, alpha, lam


CASES = [  # B, H, L, D, chunk, bound, dtype, per-token alpha, incoming state
    (2, 3, 200, 64, 64, 25.0, torch.float32, True, False),
    (1, 2, 333, 64, 64, 4.0, torch.float32, False, True),     # projection active, ragged tail
    (2, 2, 96, 32, 32, 3.0, torch.float32, True, True),
    (1, 4, 77, 16, 64, 2.0, torch.float32, False, False),
    (2, 3, 300, 64, 64, 25.0, torch.bfloat16, True, True),
    (1, 2, 1000, 64, 64, 0.0, torch.bfloat16, False, False),  # projection off, long
    (2, 2, 130, 32, 32, 5.0, torch.bfloat16, True, False),
    (1, 1, 1, 64, 64, 25.0, torch.float32, True, True),       # one token: the prefill's semantics
]


@pytest.mark.parametrize("B,H,L,D,chunk,bound,dtype,pta,with_state", CASES)
def test_delta_prefill_vs_oracle(B, H, L, D, chunk, bound, dtype, pta, with_state):
    from prime_moment_attention_b200 import ops
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    q, k, v, beta, alpha, lam = _case(B, H, L, D, seed=L + D, dtype=dtype, per_token_alpha=pta)
    st = torch.randn(B, H, D, 2 * D, generator=torch.Generator().manual_seed(5)) * 0.2 if with_state else None
    y, s = ops.delta_prefill(q.cuda(), k.cuda(), v.cuda(), beta.cuda(), None if alpha is None else alpha.cuda(),
                             lam.cuda(), chunk=chunk, lyapunov_bound=bound,
                             state=None if st is None else st.cuda(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    y_ref, s_ref = O.delta_prefill(q, k, v, beta, alpha, lam, chunk=chunk, bound=bound, state=st)
    assert O.rel_err(y.double().cpu().numpy(), y_ref) <= tol
    assert O.rel_err(s.double().cpu().numpy(), s_ref) <= tol


def test_delta_prefill_state_only_and_bf16_output():
    from prime_moment_attention_b200 import ops
    q, k, v, beta, alpha, lam = _case(1, 2, 150, 64, seed=9, dtype=torch.bfloat16, per_token_alpha=True)
    args = (q.cuda(), k.cuda(), v.cuda(), beta.cuda(), alpha.cuda(), lam.cuda())
    y_none, s_only = ops.delta_prefill(*args, want_y=False)
    y_bf, s_full = ops.delta_prefill(*args, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert y_none is None and y_bf.dtype == torch.bfloat16
    assert torch.equal(s_only, s_full)
    y_ref, _ = O.delta_prefill(q, k, v, beta, alpha, lam)
    assert O.rel_err(y_bf.double().cpu().numpy(), y_ref) <= TOL_BF16


@pytest.mark.parametrize("D,dtype", [(64, torch.float32), (64, torch.bfloat16), (32, torch.float32),
                                     (16, torch.bfloat16)])
@pytest.mark.parametrize("bound", [25.0, 1.0])
def test_delta_step_vs_oracle(D, dtype, bound):
    from prime_moment_attention_b200 import ops
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    N, H = 5, 4
    q, k, v, beta, _, lam = _case(N, H, 1, D, seed=D, dtype=dtype, per_token_alpha=False)
    alpha = lam.view(1, H).expand(N, H) * 0.97
    st = torch.randn(N, H, D, 2 * D, generator=torch.Generator().manual_seed(6)) * 0.3
    st_dev = st.cuda()
    y, s = ops.delta_decode_step(q[:, :, 0].cuda(), k[:, :, 0].cuda(), v[:, :, 0].cuda(), beta[:, :, 0].cuda(),
                                 alpha.cuda(), st_dev, lyapunov_bound=bound, out_dtype=torch.float32)
    y2, s2 = ops.delta_decode_step(q[:, :, 0].cuda(), k[:, :, 0].cuda(), v[:, :, 0].cuda(), beta[:, :, 0].cuda(),
                                   alpha.cuda(), st_dev.clone(), lyapunov_bound=bound, inplace=True,
                                   out_dtype=torch.float32)
    torch.cuda.synchronize()
    y_ref, s_ref = O.delta_step(q[:, :, 0], k[:, :, 0], v[:, :, 0], beta[:, :, 0], alpha, st, bound=bound)
    assert O.rel_err(y.double().cpu().numpy(), y_ref) <= tol
    assert O.rel_err(s.double().cpu().numpy(), s_ref) <= tol
    assert torch.equal(y, y2) and torch.equal(s, s2)
    assert torch.equal(st_dev, st.cuda())  # functional call left its input alone


def test_delta_argument_errors():
    from prime_moment_attention_b200 import _lib, ops
    q, k, v, beta, alpha, lam = _case(1, 1, 10, 64, seed=1, dtype=torch.float32, per_token_alpha=True)
    with pytest.raises(_lib.PmaError):  # chunk size the kernels do not build
        ops.delta_prefill(q.cuda(), k.cuda(), v.cuda(), beta.cuda(), alpha.cuda(), lam.cuda(), chunk=48)
    q2, k2, v2, b2, a2, l2 = _case(1, 1, 10, 128, seed=1, dtype=torch.float32, per_token_alpha=True)
    with pytest.raises(_lib.PmaError):  # D = 128 is not built for the delta variant
        ops.delta_prefill(q2.cuda(), k2.cuda(), v2.cuda(), b2.cuda(), a2.cuda(), l2.cuda())
    with pytest.raises(ValueError):
        ops.delta_prefill(q.cuda(), k.cuda(), v.cuda(), beta[:, :, :5].cuda(), alpha.cuda(), lam.cuda())


WY_CASES = [  # B, H, L, bound, per-token alpha, incoming state
    (2, 3, 300, 25.0, True, True),
    (1, 2, 1000, 0.0, False, False),   # projection off
    (1, 2, 4100, 4.0, True, True),     # projection active over many chunks, ragged tail
    (3, 1, 64, 25.0, True, False),     # one full chunk
    (1, 2, 5, 25.0, False, True),      # one short chunk
]


@pytest.mark.parametrize("wy", [True, False], ids=["wy", "single_pass"])
@pytest.mark.parametrize("B,H,L,bound,pta,with_state", WY_CASES)
def test_delta_tc_paths_vs_oracle(B, H, L, bound, pta, with_state, wy):
    """bf16, D = 64, chunk 64: the WY form (prep + sequential kernels, with a workspace) and the
    single-pass tensor-core kernel (no workspace) against the float64 oracle."""
    from prime_moment_attention_b200 import ops
    q, k, v, beta, alpha, lam = _case(B, H, L, 64, seed=L + 7, dtype=torch.bfloat16, per_token_alpha=pta)
    st = torch.randn(B, H, 64, 128, generator=torch.Generator().manual_seed(8)) * 0.2 if with_state else None
    y, s = ops.delta_prefill(q.cuda(), k.cuda(), v.cuda(), beta.cuda(), None if alpha is None else alpha.cuda(),
                             lam.cuda(), lyapunov_bound=bound, state=None if st is None else st.cuda(),
                             out_dtype=torch.float32, wy=wy)
    torch.cuda.synchronize()
    y_ref, s_ref = O.delta_prefill(q, k, v, beta, alpha, lam, chunk=64, bound=bound, state=st)
    ey = O.rel_err(y.double().cpu().numpy(), y_ref)
    es = O.rel_err(s.double().cpu().numpy(), s_ref)
    print(f"delta {'wy' if wy else 'single-pass'} B={B} H={H} L={L}: y {ey:.2e} state {es:.2e}")
    assert ey <= TOL_BF16 and es <= TOL_BF16


def test_delta_wy_windows_match_one_window():
    """A workspace smaller than the preferred one runs the sequence in windows of chunks, the
    state carried through state_out (or the workspace when no state is returned).  A window
    starts from the projected float32 state where one window carries the unprojected bf16 tile
    and applies the factor after the product, so results agree to bf16 rounding, and both match
    the oracle."""
    from prime_moment_attention_b200 import _lib, ops
    B, H, L = 2, 3, 1000  # 16 chunks
    q, k, v, beta, alpha, lam = _case(B, H, L, 64, seed=11, dtype=torch.bfloat16, per_token_alpha=True)
    args = (q.cuda(), k.cuda(), v.cuda(), beta.cuda(), alpha.cuda(), lam.cuda())
    st = (torch.randn(B, H, 64, 128, generator=torch.Generator().manual_seed(2)) * 0.2).cuda()
    y1, s1 = ops.delta_prefill(*args, lyapunov_bound=4.0, state=st)
    per_chunk = B * H * (73728 + 4)
    small = 3 * per_chunk + 256 + B * H * 64 * 128 * 4  # windows of 3 chunks
    y2, s2 = ops.delta_prefill(*args, lyapunov_bound=4.0, state=st, workspace_bytes=small)
    y3, s3 = ops.delta_prefill(*args, lyapunov_bound=4.0, state=st, workspace_bytes=small, return_state=False)
    torch.cuda.synchronize()
    assert s3 is None
    assert torch.equal(y2, y3)  # the carry through the workspace equals the one through state_out
    assert O.rel_err(y2.double().cpu().numpy(), y1.double().cpu().numpy()) <= 5e-3
    assert O.rel_err(s2.double().cpu().numpy(), s1.double().cpu().numpy()) <= 5e-3
    y_ref, s_ref = O.delta_prefill(q, k, v, beta, alpha, lam, chunk=64, bound=4.0, state=st.cpu())
    assert O.rel_err(y2.double().cpu().numpy(), y_ref) <= TOL_BF16
    assert O.rel_err(s2.double().cpu().numpy(), s_ref) <= TOL_BF16
    with pytest.raises(_lib.PmaError):  # not even one chunk per head-state
        ops.delta_prefill(*args, workspace_bytes=per_chunk // 2)


def test_delta_wy_config2_shape():
    """Config-2 shape (B = 8, H = 12, L = 8192, bf16) with the bench's gates: two sampled
    head-states against the float64 oracle, all against the single-pass kernel."""
    from prime_moment_attention_b200 import ops
    B, H, L = 8, 12, 8192
    g = torch.Generator().manual_seed(2024)
    q = (torch.nn.functional.normalize(torch.randn(B, H, L, 64, generator=g), dim=-1) / 8).to(torch.bfloat16)
    k = torch.randn(B, H, L, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, L, 64, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=g))
    lam = torch.exp(torch.empty(H).uniform_(np.log(0.99), np.log(0.9999), generator=g))
    args = (q.cuda(), k.cuda(), v.cuda(), beta.cuda(), None, lam.cuda())
    y_wy, s_wy = ops.delta_prefill(*args, lyapunov_bound=25.0, out_dtype=torch.float32)
    y_sp, s_sp = ops.delta_prefill(*args, lyapunov_bound=25.0, out_dtype=torch.float32, wy=False)
    torch.cuda.synchronize()
    e_all = max(O.rel_err(y_wy[b, h].double().cpu().numpy(), y_sp[b, h].double().cpu().numpy())
                for b in range(B) for h in range(H))
    for b, h in ((0, 0), (B - 1, H - 1)):
        sl = (slice(b, b + 1), slice(h, h + 1))
        y_ref, s_ref = O.delta_prefill(q[sl], k[sl], v[sl], beta[sl], None, lam[h:h + 1], chunk=64, bound=25.0)
        ey = O.rel_err(y_wy[sl].double().cpu().numpy(), y_ref)
        es = O.rel_err(s_wy[sl].double().cpu().numpy(), s_ref)
        print(f"delta wy config 2 head ({b},{h}): y {ey:.2e} state {es:.2e}")
        assert ey <= TOL_BF16 and es <= TOL_BF16
    print(f"delta wy vs single-pass, all head-states: {e_all:.2e}")
    assert e_all <= TOL_BF16
