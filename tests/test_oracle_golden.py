"""Pin the float64 oracle against the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py from the reference's
PyTorch code (chunked_ssd.py:48-184, attention.py:120-202) in float32, so the bar is
float32 round-off: 2e-6 normwise on outputs and states.
"""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as O

NAMES = ("S0", "S1", "S2", "K0", "K1", "K2")
TOL = 2e-6


def _cases(golden_dir, prefix):
    return sorted(glob.glob(os.path.join(golden_dir, f"{prefix}*.npz")))


@pytest.mark.parametrize("kind", ["chunk_", "dense_"])
def test_prefill_matches_reference(golden_dir, kind):
    files = _cases(golden_dir, kind)
    assert files, "golden fixtures missing"
    for f in files:
        z = np.load(f)
        y, st = O.prefill(z["q"], z["k"], z["v"], z["lam"])
        assert O.rel_err(y, z["y"]) < TOL, f
        for s, n in zip(st, NAMES):
            assert O.rel_err(s.reshape(z["st_" + n].shape), z["st_" + n]) < TOL, (f, n)


def test_decode_matches_reference(golden_dir):
    z = np.load(os.path.join(golden_dir, "decode_d32.npz"))
    st = tuple(z["in_" + n] for n in NAMES)
    ys = []
    for t in range(z["q"].shape[2]):
        y, st = O.decode_step(z["q"][:, :, t], z["k"][:, :, t], z["v"][:, :, t], z["lam"], st)
        ys.append(y)
    assert O.rel_err(np.stack(ys, axis=2), z["y"]) < TOL
    for s, n in zip(st, NAMES):
        assert O.rel_err(s.reshape(z["st_" + n].shape), z["st_" + n]) < TOL, n


def test_config1_summary(golden_dir):
    """Full config-1 shape: regenerate inputs from the seed, check they are the same
    inputs the fixture was made from, then compare sampled outputs and two heads'
    complete final state."""
    import torch
    from prime_moment_attention_b200 import synth
    z = np.load(os.path.join(golden_dir, "config1_summary.npz"))
    c = synth.CONFIG1
    q, k, v = synth.make_qkv(c["B"], c["H"], c["L"], c["D"], seed=c["seed"], dtype=c["dtype"])
    sums = np.array([float(t.double().sum()) for t in (q, k, v)])
    np.testing.assert_allclose(sums, z["in_sums"], rtol=1e-9, atol=1e-9)
    y, st = O.prefill(q, k, v, z["lam"])
    idx = z["y_idx"]
    assert np.max(np.abs(y[tuple(idx.T)] - z["y_samples"])) / z["y_max"] < TOL
    assert abs(y.sum() - z["y_sum"]) <= 1e-5 * z["y_abs"]
    for s, n in zip(st, NAMES):
        ref = z[f"st_{n}_h0_h7"]
        assert O.rel_err(s[:, [0, 7]].reshape(ref.shape), ref) < TOL, n
        assert abs(np.abs(s).max() - z[f"st_{n}_absmax"]) <= TOL * z[f"st_{n}_absmax"], n


def test_oracle_catches_a_planted_error(golden_dir):
    """The comparison is sharp enough to see a one-ulp-scale change in lambda."""
    z = np.load(os.path.join(golden_dir, "chunk_d64.npz"))
    lam = z["lam"].astype(np.float64) * (1 - 3e-6)
    y, _ = O.prefill(z["q"], z["k"], z["v"], lam)
    assert O.rel_err(y, z["y"]) > TOL


def test_segment_combine_identity():
    """State after [seg1 | seg2] == lam^len2 * state(seg1) + state(seg2 from zero)."""
    rng = np.random.default_rng(0)
    B, H, L1, L2, D = 1, 1, 23, 41, 8
    q, k, v = (rng.standard_normal((B, H, L1 + L2, D)) * 0.2 for _ in range(3))
    lam = np.array([0.97])
    _, full = O.prefill(q, k, v, lam)
    _, s1 = O.prefill(q[:, :, :L1], k[:, :, :L1], v[:, :, :L1], lam)
    _, s2 = O.prefill(q[:, :, L1:], k[:, :, L1:], v[:, :, L1:], lam)
    flat = lambda st: np.concatenate([s.ravel() for s in st])
    comb = O.combine(flat(s1), flat(s2), 0.97, L2)
    np.testing.assert_allclose(comb, flat(full), rtol=1e-12, atol=1e-12)
