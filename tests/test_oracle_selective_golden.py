"""The float64 selective-variant oracle (orc_selective_prefill) against golden vectors written
by the reference's own PrimeSelectiveMomentAttention (tests/golden/make_golden_selective.py):
its parallel branch from a zero state and its step branch from a random state.  The reference
computes in float32, so agreement is to float32 round-off."""
import os

import numpy as np

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
NAMES = ("S0", "S1", "S2", "K0", "K1", "K2")


def _load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


def test_selective_parallel_branch():
    g = _load("selective_par_d32")
    y, st = O.selective_prefill(g["q"], g["k"], g["v"], g["log_decay"], g["beta"])
    assert O.rel_err(y, g["y"]) <= 2e-5
    for s, n in zip(st, NAMES):
        assert O.rel_err(s.reshape(g["st_" + n].shape), g["st_" + n]) <= 2e-5, n


def test_selective_step_branch():
    g = _load("selective_step_d16")
    st = tuple(g["in_" + n] for n in NAMES)
    for t in range(g["q"].shape[2]):
        sl = slice(t, t + 1)
        y, st = O.selective_prefill(g["q"][:, :, sl], g["k"][:, :, sl], g["v"][:, :, sl], g["log_decay"][:, :, sl],
                                    g["beta"], st)
        assert O.rel_err(y, g["y"][:, :, sl]) <= 2e-5
    for s, n in zip(st, NAMES):
        assert O.rel_err(s.reshape(g["st_" + n].shape), g["st_" + n]) <= 2e-5, n


def test_selective_equals_moment_attention_with_scaled_k_and_halved_second_moments():
    """With a constant decay the selective recurrence is the moment recurrence with k -> beta k
    and S2, Z2 stored halved: the identity the kernels use."""
    g = _load("selective_par_d32")
    H = g["q"].shape[1]
    lam = np.exp(g["log_decay"][0, :, 0])
    ld = np.broadcast_to(np.log(lam)[None, :, None], g["log_decay"].shape)
    y_s, st_s = O.selective_prefill(g["q"], g["k"], g["v"], ld, g["beta"])
    y_m, st_m = O.prefill(g["q"], g["k"] * g["beta"].reshape(1, H, 1, 1), g["v"], lam)
    assert O.rel_err(y_s, y_m) <= 1e-6
    for i, (a, b) in enumerate(zip(st_s, st_m)):
        assert O.rel_err(a, b * (0.5 if i in (2, 5) else 1.0)) <= 1e-6
