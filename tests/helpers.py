"""Shared helpers for the GPU parity tests (CUDA path vs the float64 oracle)."""
import numpy as np
import torch

from oracle import oracle as O

NAMES = ("S0", "S1", "S2", "K0", "K1", "K2")
TOL_F32 = 1e-4   # fp32 inputs: max relative error on outputs and final state
TOL_BF16 = 2e-2  # bf16 inputs, fp32 state


def cpu64(t):
    return t.detach().to("cpu", torch.float64).numpy()


def assert_close(got, ref, tol, what=""):
    e = O.rel_err(cpu64(got) if torch.is_tensor(got) else got, ref)
    assert e <= tol, f"{what}: relative error {e:.3e} > {tol:.1e}"
    return e


def assert_state_close(got, ref, tol, what="state"):
    errs = []
    for g, r, n in zip(got, ref, NAMES):
        errs.append(assert_close(g.reshape(r.shape), r, tol, f"{what}.{n}"))
    return errs


def to_dev(state, device="cuda"):
    return tuple(torch.as_tensor(np.asarray(s), dtype=torch.float32).to(device).contiguous() for s in state)


def lam_np(lam):
    return lam.detach().cpu().double().numpy() if torch.is_tensor(lam) else np.asarray(lam, dtype=np.float64)
