"""The float64 delta-rule oracle (oracle/pma_oracle.c, orc_delta_*) against golden vectors
written by the reference's own ChunkedGatedDeltaPrimeAttention (tests/golden/make_golden_delta.py).

The reference computes in float32 (chunked_delta_prime.py:104-108 casts to float32 and solves
the chunk's triangular system in float32), so agreement is to float32 round-off."""
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOL = 2e-5


def _load(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


@pytest.mark.parametrize("name", ["delta_c32_d16", "delta_c64_d32_st", "delta_c64_d64"])
def test_delta_prefill_matches_reference(name):
    g = _load(name)
    y, st = O.delta_prefill(g["q"], g["k"], g["v"], g["beta"], g["alpha"], g["lam"], chunk=int(g["chunk"]),
                            bound=float(g["bound"]), state=g.get("state_in"))
    assert O.rel_err(y, g["y"]) <= TOL
    assert O.rel_err(st, g["state"]) <= TOL


def test_delta_prefill_lyapunov_is_active_in_fixture():
    """The bound-3 case must exercise the projection: without it the final state differs."""
    g = _load("delta_c32_d16")
    _, st_off = O.delta_prefill(g["q"], g["k"], g["v"], g["beta"], g["alpha"], g["lam"], chunk=32, bound=0.0)
    assert O.rel_err(st_off, g["state"]) > 1e-2
    # and the ragged tail decay matters: the same run without the pad factor differs
    _, st_c75 = O.delta_prefill(g["q"], g["k"], g["v"], g["beta"], g["alpha"], g["lam"], chunk=75, bound=3.0)
    assert O.rel_err(st_c75, g["state"]) > 1e-4


def test_delta_step_matches_reference():
    g = _load("delta_step_d32")
    st = g["state_in"]
    bound = float(g["bound"])
    for t in range(g["q"].shape[2]):
        y, st = O.delta_step(g["q"][:, :, t], g["k"][:, :, t], g["v"][:, :, t], g["beta"][:, :, t],
                             g["alpha"][:, :, t], st, bound=bound)
        assert O.rel_err(y, g["y"][:, :, t]) <= TOL
    assert O.rel_err(st, g["state"]) <= TOL


def test_delta_prefill_and_step_differ_as_in_the_reference():
    """The reference's prefill measures the error against the decayed state and its step
    against the undecayed one; stepping the prefill's inputs one token at a time does not
    reproduce the prefill (this is the reference's own behaviour, kept on both sides)."""
    g = _load("delta_c64_d32_st")
    y_p, _ = O.delta_prefill(g["q"][:, :, :8], g["k"][:, :, :8], g["v"][:, :, :8], g["beta"][:, :, :8],
                             g["alpha"][:, :, :8], g["lam"], bound=0.0, state=g["state_in"])
    st = g["state_in"]
    ys = []
    for t in range(8):
        y, st = O.delta_step(g["q"][:, :, t], g["k"][:, :, t], g["v"][:, :, t], g["beta"][:, :, t],
                             g["alpha"][:, :, t], st, bound=0.0)
        ys.append(y)
    assert O.rel_err(np.stack(ys, axis=2), y_p) > 1e-4
