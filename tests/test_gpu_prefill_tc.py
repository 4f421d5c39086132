"""Tensor-core (tcgen05) prefill: bf16 inputs, D = 64 and D = 128, against the float64 oracle.

Bar: 2e-2 max relative error on y and on each final-state component (bf16
operands, float32 accumulation and state).  Each call also checks the kernel's
status word (no bounded wait expired)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from prime_moment_attention_b200 import _lib, ops, synth
from tests.helpers import TOL_BF16, TOL_F32, assert_close, assert_state_close, cpu64, lam_np

pytestmark = pytest.mark.gpu


def _run(B, H, L, seed, lam=None, state=None, out_dtype=torch.float32, D=64):
    q, k, v = synth.make_qkv(B, H, L, D, seed=seed, dtype=torch.bfloat16, device="cuda")
    if lam is None:
        lam = synth.make_lambdas(H, 0.99, 0.9999, seed=seed)
    y, st = ops.prefill(q, k, v, lam, state=state, out_dtype=out_dtype, check=True)
    lam_ref = lam.double().numpy() if torch.is_tensor(lam) else lam
    y_ref, st_ref = O.prefill(q, k, v, lam_ref, state=None if state is None else tuple(s.cpu() for s in state))
    return y, st, y_ref, st_ref


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("L", [1, 5, 127, 128, 129, 300, 1000])
def test_tc_lengths(L, D):
    y, st, y_ref, st_ref = _run(2, 3, L, seed=L, D=D)
    assert_close(y, y_ref, TOL_BF16, "y")
    assert_state_close(st, st_ref, TOL_BF16)


@pytest.mark.parametrize("D", [64, 128])
def test_tc_incoming_state_and_bf16_out(D):
    B, H = 2, 4
    lam = torch.rand(B, H) * 0.02 + 0.98
    st0 = synth.make_state(B, H, D, lam[0], seed=3, t0=300, sigma=0.05, device="cuda")
    y, st, y_ref, st_ref = _run(B, H, 517, seed=4, lam=lam, state=st0, out_dtype=torch.bfloat16, D=D)
    assert_close(y, y_ref, TOL_BF16, "y")
    assert_state_close(st, st_ref, TOL_BF16)


@pytest.mark.parametrize("D", [64, 128])
def test_tc_small_decay(D):
    """Decays far from 1 (l^127 underflows toward zero): masks and weights stay finite; heads
    below 0.55 take the float32 loop inside the same launch."""
    lam = torch.tensor([0.5, 0.1, 0.9])
    y, st, y_ref, st_ref = _run(1, 3, 260, seed=7, lam=lam, D=D)
    assert_close(y, y_ref, TOL_BF16, "y")
    assert_state_close(st, st_ref, TOL_BF16)


@pytest.mark.parametrize("D", [64, 128])
def test_tc_segmented(D):
    """B*H well below the SM count: sequences split into segments (state-only pass,
    prefix, full pass), all on the tensor-core kernel."""
    B, H, L = 1, 4, 4096 + 77
    assert _lib.load().pma_prefill_workspace_bytes(B, H, L, D, _lib.PMA_BF16) > 256
    lam = torch.tensor([0.999, 0.99, 0.9999, 0.95])
    st0 = synth.make_state(B, H, D, lam, seed=8, t0=1000, sigma=0.02, device="cuda")
    y, st, y_ref, st_ref = _run(B, H, L, seed=9, lam=lam, state=st0, D=D)
    assert_close(y, y_ref, TOL_BF16, "y")
    assert_state_close(st, st_ref, TOL_BF16)
    q, k, v = synth.make_qkv(B, H, L, D, seed=9, dtype=torch.bfloat16, device="cuda")
    _, st_only = ops.prefill(q, k, v, lam, state=st0, want_y=False, check=True)
    assert_state_close(st_only, st_ref, TOL_BF16, "state-only")


def test_tc128_gqa_scale_strided():
    """D = 128 through pma_prefill_ex: grouped k/v heads, a q scale exact in bf16 (applied by the
    kernel), [B,L,H,D] views in and out."""
    B, H, Hk, L, D = 2, 4, 2, 333, 128
    g = torch.Generator().manual_seed(5)
    qb = torch.nn.functional.normalize(torch.randn(B, L, H, D, generator=g), dim=-1).to("cuda", torch.bfloat16)
    kvb = torch.nn.functional.normalize(torch.randn(B, L, 2 * Hk, D, generator=g), dim=-1).to("cuda", torch.bfloat16)
    q, k, v = qb.transpose(1, 2), kvb[:, :, :Hk].transpose(1, 2), kvb[:, :, Hk:].transpose(1, 2)
    lam = torch.tensor([0.999, 0.99, 0.98, 0.9995])
    pro = ops.Prologue(kv_groups=2, q_scale=0.125)
    y_bl = torch.empty(B, L, H, D, device="cuda", dtype=torch.float32)
    _, st = ops.prefill(q, k, v, lam, y_out=y_bl.transpose(1, 2), prologue=pro, check=True)
    k_r, v_r = k.repeat_interleave(2, dim=1), v.repeat_interleave(2, dim=1)
    y_ref, st_ref = O.prefill((q.float() * 0.125).to(torch.bfloat16), k_r, v_r, lam_np(lam))
    assert_close(y_bl.transpose(1, 2), y_ref, TOL_BF16, "y")
    assert_state_close(st, st_ref, TOL_BF16)


def test_tc_strided_module_layout():
    """q/k/v as views of [B,L,H,D] projections, y into a [B,L,H,D] buffer."""
    B, H, L, D = 2, 3, 300, 64
    base = torch.nn.functional.normalize(torch.randn(B, L, 3 * H, D, device="cuda"), dim=-1).to(torch.bfloat16)
    q, k, v = (base[:, :, i * H:(i + 1) * H].transpose(1, 2) for i in range(3))
    q = (q.float() * 0.125).to(torch.bfloat16)
    y_bl = torch.empty(B, L, H, D, device="cuda", dtype=torch.bfloat16)
    _, st = ops.prefill(q, k, v, 0.995, y_out=y_bl.transpose(1, 2), check=True)
    y_ref, st_ref = O.prefill(q, k, v, 0.995)
    assert_close(y_bl.transpose(1, 2), y_ref, TOL_BF16, "y")
    assert_state_close(st, st_ref, TOL_BF16)


def test_tc_config2_full_size():
    """Config 2 at full size (B=8, H=12, L=8192): two head-states against the oracle
    over all 8192 tokens, and every head-state against the float32 CUDA-core kernel
    run on the same (bf16-valued) inputs."""
    c = synth.CONFIG2
    B, H, L, D = c["B"], c["H"], c["L"], c["D"]
    q, k, v = synth.make_qkv(B, H, L, D, seed=c["seed"], dtype=torch.bfloat16, device="cuda")
    lam = synth.make_lambdas(H, *c["lam"], seed=c["seed"])
    y, st = ops.prefill(q, k, v, lam, out_dtype=torch.float32, check=True)
    for (bb, hh) in [(0, 0), (5, 11)]:
        y_ref, st_ref = O.prefill(q[bb:bb + 1, hh:hh + 1], k[bb:bb + 1, hh:hh + 1], v[bb:bb + 1, hh:hh + 1],
                                  lam_np(lam)[hh:hh + 1])
        assert_close(y[bb:bb + 1, hh:hh + 1], y_ref, TOL_BF16, f"y[{bb},{hh}]")
        assert_state_close(tuple(s[bb:bb + 1, hh:hh + 1] for s in st), st_ref, TOL_BF16, f"state[{bb},{hh}]")
    y32, st32 = ops.prefill(q.float(), k.float(), v.float(), lam, out_dtype=torch.float32)
    assert_close(y, cpu64(y32), TOL_BF16, "y vs fp32 kernel")
    for a, b_ in zip(st, st32):
        assert_close(a, cpu64(b_), TOL_BF16, "state vs fp32 kernel")


def test_tc128_config5_law_long():
    """Config 5's head shape and decay law (H=16, D=128, bf16, lambda log-U[0.999, 0.99995]) at
    L = 2^16 through pma_prefill's segmented tensor-core path (state-only pass, segment prefix,
    full pass): four sampled head-states against the float64 oracle over all tokens (y and every
    final-state component), and every head-state against the float32 CUDA-core kernel run on the
    same bf16-valued inputs.  Decays this close to 1 keep 2^16 tokens of history in the state, so
    this is where bf16 carry operands would accumulate error.  The carry replaces the reference's
    inter-chunk matmul (src/prime_moment_attention/chunked_ssd.py:113-126)."""
    from concurrent.futures import ThreadPoolExecutor
    c = synth.CONFIG5
    B, H, L, D = c["B"], c["H"], 1 << 16, c["D"]
    assert _lib.load().pma_prefill_workspace_bytes(B, H, L, D, _lib.PMA_BF16) > 256  # segmented plan
    q, k, v = synth.make_qkv(B, H, L, D, seed=c["seed"], dtype=torch.bfloat16, device="cuda")
    lam = synth.make_lambdas(H, *c["lam"], seed=c["seed"])
    y, st = ops.prefill(q, k, v, lam, out_dtype=torch.float32, check=True)
    heads = [int(torch.argmax(lam)), int(torch.argmin(lam)), 5, 11]
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    lam64 = lam_np(lam)

    def ref(h):  # ctypes releases the GIL: the four oracle runs overlap
        return O.prefill(qc[:, h:h + 1], kc[:, h:h + 1], vc[:, h:h + 1], lam64[h:h + 1])

    with ThreadPoolExecutor(4) as ex:
        refs = list(ex.map(ref, heads))
    for h, (y_ref, st_ref) in zip(heads, refs):
        ey = assert_close(y[:, h:h + 1], y_ref, TOL_BF16, f"y[h={h}]")
        es = assert_state_close(tuple(s[:, h:h + 1] for s in st), st_ref, TOL_BF16, f"state[h={h}]")
        print(f"config-5 law, L=2^16, head {h} (lambda={lam64[h]:.6f}): y {ey:.2e}, state "
              + " ".join(f"{e:.2e}" for e in es))
    y32, st32 = ops.prefill(q.float(), k.float(), v.float(), lam, out_dtype=torch.float32)
    e = assert_close(y, cpu64(y32), TOL_BF16, "y vs fp32 kernel")
    es = [assert_close(a, cpu64(b_), TOL_BF16, "state vs fp32 kernel") for a, b_ in zip(st, st32)]
    print(f"config-5 law, L=2^16, all heads vs fp32 kernel: y {e:.2e}, state " + " ".join(f"{x:.2e}" for x in es))
    _, st_only = ops.prefill(q, k, v, lam, want_y=False, check=True)
    for a, b_ in zip(st_only, st32):
        assert_close(a, cpu64(b_), TOL_BF16, "state-only call vs fp32 kernel")


@pytest.mark.parametrize("D,dtype", [(64, torch.bfloat16), (128, torch.bfloat16), (64, torch.float32)])
def test_resume_after_state_only_call(D, dtype):
    """pma_prefill_resume: a state-only call from zero leaves each segment's entering state in the
    workspace; the resumed output pass from an incoming state must match the oracle run of the
    whole sequence from that state (y and final state), as a single pma_prefill call does."""
    B, H, L = 1, 4, 4096 + 77
    assert _lib.load().pma_prefill_workspace_bytes(B, H, L, D, ops._DT[dtype]) > 256  # segmented
    lam = torch.tensor([0.999, 0.99, 0.9999, 0.95])
    st0 = synth.make_state(B, H, D, lam, seed=18, t0=1000, sigma=0.02, device="cuda")
    q, k, v = synth.make_qkv(B, H, L, D, seed=19, dtype=dtype, device="cuda")
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    ws = ops.prefill_workspace(q)
    _, T = ops.prefill(q, k, v, lam, want_y=False, workspace=ws, check=True)
    y, st = ops.prefill(q, k, v, lam, state=st0, out_dtype=torch.float32, workspace=ws, resume=True, check=True)
    y_ref, st_ref = O.prefill(q, k, v, lam_np(lam), state=tuple(s.cpu() for s in st0))
    assert_close(y, y_ref, tol, "y")
    assert_state_close(st, st_ref, tol)
    _, T_ref = O.prefill(q, k, v, lam_np(lam))
    assert_state_close(T, T_ref, tol, "zero-start state")


@pytest.mark.parametrize("L", [300, 4173])
def test_tc_y_rows_into_a_strided_view(L):
    """bf16 y leaves the D = 64 kernel through a staging tile and one TMA store per chunk: into
    a view of a wider buffer (row stride 128 elements), with a ragged last chunk (and, at L =
    4173, the sequence split into segments across CTAs), the rows equal those written into a
    contiguous y, and nothing around the view is touched."""
    B, H, D = 2, 3, 64
    q, k, v = synth.make_qkv(B, H, L, D, seed=L + 1, dtype=torch.bfloat16, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=2)
    y_ref, _ = ops.prefill(q, k, v, lam, out_dtype=torch.bfloat16, check=True)
    wide = torch.full((B, H, L + 3, 2 * D), 7.0, dtype=torch.bfloat16, device="cuda")
    view = wide[:, :, :L, :D]
    ops.prefill(q, k, v, lam, y_out=view, check=True)
    torch.cuda.synchronize()
    assert torch.equal(view, y_ref)
    assert bool((wide[:, :, :, D:] == 7.0).all()) and bool((wide[:, :, L:, :] == 7.0).all())
    y64, _ = O.prefill(q, k, v, lam_np(lam))
    assert_close(view, y64, TOL_BF16, "y (strided view)")
