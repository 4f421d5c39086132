"""Decode step on the GPU vs the oracle and the reference's own decode outputs.

Bar: fp32 inputs 1e-4, bf16 inputs 2e-2 (max relative error, outputs and state)."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from prime_moment_attention_b200 import ops, synth
from tests.helpers import NAMES, TOL_BF16, TOL_F32, assert_close, assert_state_close, lam_np, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_steps_vs_oracle(D, dtype):
    N, H, steps = 3, 5, 4
    lam = synth.make_lambdas(H, 0.95, 0.9999, seed=D)
    st = synth.make_state(N, H, D, lam, seed=D, t0=200, sigma=0.05, device="cuda")
    ref_st = tuple(s.cpu().double().numpy() for s in st)
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    for t in range(steps):
        q, k, v = synth.make_decode_tokens(N, H, D, seed=100 * D + t, dtype=dtype, device="cuda")
        y, st = ops.decode_step(q, k, v, lam, st, eps=1.0, out_dtype=torch.float32)
        y_ref, ref_st = O.decode_step(q, k, v, lam_np(lam), ref_st, eps=1.0)
        assert_close(y, y_ref, tol, f"y step {t}")
    assert_state_close(st, ref_st, TOL_F32)


def test_decode_inplace_matches_functional():
    N, H, D = 4, 3, 64
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=1)
    st = synth.make_state(N, H, D, lam, seed=1, device="cuda")
    st_copy = tuple(s.clone() for s in st)
    q, k, v = synth.make_decode_tokens(N, H, D, seed=2, device="cuda")
    y1, s1 = ops.decode_step(q, k, v, lam, st)
    for a, b in zip(st, st_copy):  # functional call left the input untouched
        assert torch.equal(a, b)
    y2, s2 = ops.decode_step(q, k, v, lam, st_copy, inplace=True)
    assert all(a.data_ptr() == b.data_ptr() for a, b in zip(s2, st_copy))
    assert torch.equal(y1, y2)
    for a, b in zip(s1, s2):
        assert torch.equal(a, b)


def test_decode_golden_reference(golden_dir):
    """The reference module's own decode outputs (attention.py:120-143)."""
    z = np.load(os.path.join(golden_dir, "decode_d32.npz"))
    st = to_dev(tuple(z["in_" + n] for n in NAMES))
    lam = torch.tensor(z["lam"])
    for t in range(z["q"].shape[2]):
        q, k, v = (torch.tensor(z[n][:, :, t]).cuda() for n in ("q", "k", "v"))
        y, st = ops.decode_step(q, k, v, lam, st)
        assert_close(y, z["y"][:, :, t], TOL_F32, f"y step {t}")
    assert_state_close(st, tuple(z["st_" + n] for n in NAMES), TOL_F32)


def test_decode_eps_clamp_and_per_row_decay():
    """Denominator clamp active (eps larger than the denominator), [N,H] decay table."""
    N, H, D = 2, 3, 32
    lam = torch.rand(N, H) * 0.5 + 0.45
    st = tuple(torch.zeros_like(s) for s in synth.make_state(N, H, D, lam[0], seed=3, device="cuda"))
    q, k, v = synth.make_decode_tokens(N, H, D, seed=4, dtype=torch.float32, device="cuda")
    y, st2 = ops.decode_step(q, k, v, lam, st, eps=5.0)
    y_ref, st_ref = O.decode_step(q, k, v, lam.double().numpy(), tuple(s.cpu() for s in st), eps=5.0)
    assert_close(y, y_ref, TOL_F32, "y")
    assert_state_close(st2, st_ref, TOL_F32)


def test_decode_strided_inputs():
    """q/k/v as [N,H,D] slices of a [N,1,H,D] projection (the module's L==1 view)."""
    N, H, D = 3, 4, 64
    lam = synth.make_lambdas(H, 0.99, 0.999, seed=5)
    st = synth.make_state(N, H, D, lam, seed=5, device="cuda")
    base = torch.randn(N, 1, 3 * H, D, device="cuda")
    q, k, v = base[:, 0, :H], base[:, 0, H:2 * H], base[:, 0, 2 * H:]
    y, st2 = ops.decode_step(q, k, v, lam, st)
    y_ref, st_ref = O.decode_step(q, k, v, lam_np(lam), tuple(s.cpu() for s in st))
    assert_close(y, y_ref, TOL_F32, "y")
    assert_state_close(st2, st_ref, TOL_F32)


def test_decode_config3_shape_properties():
    """Full config-3 size (256 seq x 12 layers x 12 heads): a batch of head-states
    checked against the oracle, and linearity of the state update in v."""
    c = synth.CONFIG3
    N, H, D = c["seqs"], c["layers"] * c["H"], c["D"]
    lam = synth.make_lambdas(H, *c["lam"], seed=c["seed"])
    st = synth.make_state(N, H, D, lam, seed=c["seed"], t0=c["t0"], sigma=c["sigma"], device="cuda")
    q, k, v = synth.make_decode_tokens(N, H, D, seed=c["seed"] + 1, device="cuda")
    y, st2 = ops.decode_step(q, k, v, lam, st)
    rows = [0, 77, 255]
    y_ref, st_ref = O.decode_step(q[rows], k[rows], v[rows], lam_np(lam), tuple(s[rows].cpu() for s in st))
    assert_close(y[rows], y_ref, TOL_BF16, "y")
    assert_state_close(tuple(s[rows] for s in st2), st_ref, TOL_F32)
    # S1(v1 + v2) - S1(v1) - S1(v2) + l S1 == 0: the update is affine in v
    zero_v = torch.zeros_like(v)
    _, sa = ops.decode_step(q, k, zero_v, lam, st)
    _, sb = ops.decode_step(q, k, v, lam, tuple(torch.zeros_like(s) for s in st))
    for i in (0, 1, 2):
        torch.testing.assert_close(st2[i], sa[i] + sb[i], rtol=1e-5, atol=1e-6)
