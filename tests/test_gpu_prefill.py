"""Chunked prefill on the GPU vs the oracle and the reference's own outputs.

Bar: fp32 inputs 1e-4, bf16 inputs 2e-2 (max relative error on y and on every
final-state component, which stay float32 in both cases)."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from prime_moment_attention_b200 import chunked_prime_ssd_core, ops, synth
from tests.helpers import NAMES, TOL_BF16, TOL_F32, assert_close, assert_state_close, cpu64, lam_np, to_dev

pytestmark = pytest.mark.gpu


def _golden(golden_dir, prefix):
    return sorted(glob.glob(os.path.join(golden_dir, prefix + "*.npz")))


@pytest.mark.parametrize("prefix", ["chunk_", "dense_"])
def test_prefill_golden_reference(golden_dir, prefix):
    """Against the reference's chunked core and dense branch outputs."""
    for f in _golden(golden_dir, prefix):
        z = np.load(f)
        q, k, v = (torch.tensor(z[n]).cuda() for n in ("q", "k", "v"))
        y, st = chunked_prime_ssd_core(q, k, v, decay=torch.tensor(z["lam"]), return_state=True)
        assert_close(y, z["y"], TOL_F32, f"{os.path.basename(f)} y")
        assert_state_close(st, tuple(z["st_" + n] for n in NAMES), TOL_F32, os.path.basename(f))


def test_config1_full_fp32():
    """Config 1: B=1, H=12, L=2048, D=64, fp32, lambda 0.9995 -- against the oracle."""
    c = synth.CONFIG1
    q, k, v = synth.make_qkv(c["B"], c["H"], c["L"], c["D"], seed=c["seed"], dtype=torch.float32, device="cuda")
    lam = torch.full((c["H"],), c["lam"][0])
    y, st = ops.prefill(q, k, v, lam, out_dtype=torch.float32)
    y_ref, st_ref = O.prefill(q, k, v, lam_np(lam))
    assert_close(y, y_ref, TOL_F32, "y")
    assert_state_close(st, st_ref, TOL_F32)


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("L", [1, 63, 64, 65, 300])
def test_prefill_shapes_fp32(D, L):
    B, H = 2, 3
    q, k, v = synth.make_qkv(B, H, L, D, seed=D * 1000 + L, device="cuda")
    lam = synth.make_lambdas(H, 0.9, 0.9999, seed=L)
    y, st = ops.prefill(q, k, v, lam)
    y_ref, st_ref = O.prefill(q, k, v, lam_np(lam))
    assert_close(y, y_ref, TOL_F32, "y")
    assert_state_close(st, st_ref, TOL_F32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prefill_with_incoming_state(dtype):
    """An incoming state (which the reference chunked core cannot take) with a
    ragged L, per-row decay, and output written as bf16."""
    B, H, L, D = 2, 3, 333, 64
    lam = torch.rand(B, H) * 0.05 + 0.95
    st0 = synth.make_state(B, H, D, lam[0], seed=9, t0=500, sigma=0.05, device="cuda")
    q, k, v = synth.make_qkv(B, H, L, D, seed=10, dtype=dtype, device="cuda")
    y, st = ops.prefill(q, k, v, lam, state=st0, out_dtype=torch.bfloat16)
    y_ref, st_ref = O.prefill(q, k, v, lam.double().numpy(), state=tuple(s.cpu() for s in st0))
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    assert_close(y, y_ref, max(tol, 8e-3), "y (bf16 out)")
    assert_state_close(st, st_ref, tol)


def test_prefill_segmented_long_sequence():
    """B*H far below the SM count and L long: the planner splits the sequence into
    segments (state-only pass, prefix, full pass); results must not change."""
    B, H, L, D = 1, 2, 4100, 32
    q, k, v = synth.make_qkv(B, H, L, D, seed=21, device="cuda")
    lam = torch.tensor([0.999, 0.97])
    st0 = synth.make_state(B, H, D, lam, seed=22, t0=100, sigma=0.05, device="cuda")
    from prime_moment_attention_b200 import _lib
    assert _lib.load().pma_prefill_workspace_bytes(B, H, L, D, 0) > 0, "expected a segmented plan"
    y, st = ops.prefill(q, k, v, lam, state=st0)
    y_ref, st_ref = O.prefill(q, k, v, lam_np(lam), state=tuple(s.cpu() for s in st0))
    assert_close(y, y_ref, TOL_F32, "y")
    assert_state_close(st, st_ref, TOL_F32)
    _, st_only = ops.prefill(q, k, v, lam, state=st0, want_y=False)
    assert_state_close(st_only, st_ref, TOL_F32, "state-only")


def test_prefill_strided_views_and_y_out():
    """q/k/v as transposed views of [B,L,H,D] projections and y written into a
    [B,L,H,D] buffer (the module's layouts), no copies."""
    B, H, L, D = 2, 4, 130, 64
    base = torch.randn(B, L, 3 * H, D, device="cuda")
    base = torch.nn.functional.normalize(base, dim=-1)
    q, k, v = (base[:, :, i * H:(i + 1) * H].transpose(1, 2) for i in range(3))
    q = q * 0.125
    lam = 0.995
    y_bl = torch.empty(B, L, H, D, device="cuda")
    _, st = ops.prefill(q, k, v, lam, y_out=y_bl.transpose(1, 2))
    y_ref, st_ref = O.prefill(q, k, v, lam)
    assert_close(y_bl.transpose(1, 2), y_ref, TOL_F32, "y")
    assert_state_close(st, st_ref, TOL_F32)


def test_prefill_then_decode_equals_longer_prefill():
    B, H, L, D = 2, 3, 100, 64
    q, k, v = synth.make_qkv(B, H, L + 1, D, seed=31, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=31)
    y_all, st_all = ops.prefill(q, k, v, lam)
    _, st = ops.prefill(q[:, :, :L], k[:, :, :L], v[:, :, :L], lam)
    y1, st1 = ops.decode_step(q[:, :, L], k[:, :, L], v[:, :, L], lam, st)
    assert_close(y1, cpu64(y_all[:, :, L]), TOL_F32, "y")
    assert_state_close(st1, tuple(cpu64(s) for s in st_all), TOL_F32)


def test_prefill_empty_and_no_outputs():
    B, H, D = 1, 2, 32
    st0 = synth.make_state(B, H, D, torch.tensor([0.9, 0.99]), seed=5, device="cuda")
    q = torch.zeros(B, H, 0, D, device="cuda")
    y, st = ops.prefill(q, q, q, 0.9, state=st0)
    assert y.shape == (B, H, 0, D)
    for a, b in zip(st, st0):
        assert torch.equal(a, b)
    y, st = ops.prefill(q, q, q, 0.9)
    assert all(float(s.abs().max()) == 0.0 for s in st)


def test_state_combine_joins_segments():
    """state(L1 + L2) == l^L2 state(L1) + state(L2 from zero): the cross-GPU carry."""
    B, H, L1, L2, D = 2, 3, 200, 77, 64
    q, k, v = synth.make_qkv(B, H, L1 + L2, D, seed=41, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=41)
    _, full = ops.prefill(q, k, v, lam)
    _, P = ops.prefill(q[:, :, :L1], k[:, :, :L1], v[:, :, :L1], lam)
    _, T = ops.prefill(q[:, :, L1:], k[:, :, L1:], v[:, :, L1:], lam)
    ops.state_combine(T, P, lam, L2)
    for a, b in zip(P, full):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)


def test_prefill_rejects_bad_input():
    q = torch.zeros(1, 2, 8, 48, device="cuda")
    from prime_moment_attention_b200._lib import PmaError
    with pytest.raises(PmaError, match="HEAD_DIM"):
        ops.prefill(q, q, q, 0.9)
    q = torch.zeros(1, 2, 8, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(TypeError):
        ops.prefill(q, q, q, 0.9)


@pytest.mark.parametrize("pieces,per_row_decay,with_state", [(None, False, False), (2, True, True), (1, False, True)])
def test_prefill_from_host_matches_device_prefill(pieces, per_row_decay, with_state):
    """Host buffers in and out, the batch in slices whose copies overlap the kernels: same y and
    final state as prefill() on device tensors."""
    B, H, L, D = 3, 2, 300, 64
    q, k, v = synth.make_qkv(B, H, L, D, seed=31, dtype=torch.bfloat16, device="cuda")
    lam = (torch.rand(B, H) * 0.05 + 0.95) if per_row_decay else synth.make_lambdas(H, 0.99, 0.9999, seed=3)
    st0 = synth.make_state(B, H, D, lam if not per_row_decay else lam[0], seed=4, t0=200, sigma=0.05,
                           device="cuda") if with_state else None
    y_ref, st_ref = ops.prefill(q, k, v, lam, state=st0)
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    y, st = ops.prefill_from_host(qh, kh, vh, lam, state=st0, pieces=pieces)
    torch.cuda.synchronize()
    assert not y.is_cuda
    assert_close(y, cpu64(y_ref), TOL_BF16, "y")
    for a, b in zip(st, st_ref):
        assert_close(a, cpu64(b), TOL_BF16, "state")


def test_prefill_from_host_back_to_back_calls():
    """Three calls in a row with different host inputs of one shape (the staging buffers are reused;
    a call's input copies may start while the previous call's output copies still run), with no
    synchronisation between them: every call's y and final state match prefill() on its inputs."""
    B, H, L, D = 4, 3, 700, 64
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=8)
    cases, outs = [], []
    for i in range(3):
        q, k, v = synth.make_qkv(B, H, L, D, seed=50 + i, dtype=torch.bfloat16, device="cuda")
        cases.append(ops.prefill(q, k, v, lam))
        qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
        yh = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
        outs.append((qh, kh, vh, yh))
    torch.cuda.synchronize()
    results = [ops.prefill_from_host(qh, kh, vh, lam, y_host=yh) for qh, kh, vh, yh in outs]
    torch.cuda.synchronize()
    for (y_ref, st_ref), (y, st) in zip(cases, results):
        assert_close(y, cpu64(y_ref), TOL_BF16, "y")
        for a, b in zip(st, st_ref):
            assert_close(a, cpu64(b), TOL_BF16, "state")
