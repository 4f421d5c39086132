"""Failure path of the tensor-core prefills, exercised without faulting or hanging a GPU.

The test hook pma_test_expire_waits makes every tensor-core prefill launch first wait, bounded
by a short limit (1 ms here), for a barrier phase that nothing completes.  The wait expires
before the launch issues any copy or GEMM; the launch records code 90 in the workspace status
word and in the registered fault word, skips its work and frees its tensor memory.  The tests
check that the host sees the code (at once with check=True, else at the next call), and that
the CUDA context stays usable: the next normal call matches the float64 oracle."""
import pytest
import torch

from oracle import oracle as O
from prime_moment_attention_b200 import _lib, ops, synth
from tests.helpers import TOL_BF16, assert_close, assert_state_close, lam_np

pytestmark = pytest.mark.gpu

EXPIRE_NS = 1_000_000


@pytest.fixture
def expiring_waits():
    ops.check_faults(synchronize=True)  # nothing pending from earlier tests
    _lib.load().pma_test_expire_waits(EXPIRE_NS)
    try:
        yield
    finally:
        _lib.load().pma_test_expire_waits(0)
        torch.cuda.synchronize()
        try:
            ops.check_faults()
        except ops.KernelFault:
            pass


def _inputs(D, L=300, H=3):
    q, k, v = synth.make_qkv(1, H, L, D, seed=D + L, dtype=torch.bfloat16, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=D)
    return q, k, v, lam


def _normal_call_matches_oracle(q, k, v, lam):
    y, st = ops.prefill(q, k, v, lam, out_dtype=torch.float32, check=True)
    y_ref, st_ref = O.prefill(q, k, v, lam_np(lam))
    assert_close(y, y_ref, TOL_BF16, "y after the fault")
    assert_state_close(st, st_ref, TOL_BF16, "state after the fault")


@pytest.mark.parametrize("D,L", [(64, 300), (128, 300), (64, 4173)])
def test_expired_wait_raises_with_check(expiring_waits, D, L):
    """check=True: the call synchronises and raises KernelFault with the hook's code (the
    L = 4173 case is split into segments: state-only pass, prefix, full pass all give up)."""
    q, k, v, lam = _inputs(D, L)
    with pytest.raises(ops.KernelFault) as ei:
        ops.prefill(q, k, v, lam, check=True)
    assert ei.value.code == 90
    assert ops.pending_fault() == 0  # raising clears the word
    _lib.load().pma_test_expire_waits(0)
    _normal_call_matches_oracle(q, k, v, lam)


def test_expired_wait_surfaces_at_next_call(expiring_waits):
    """Without check=True nothing synchronises; the fault word holds the code once the launch
    has finished, and the next prefill call of the module raises before launching."""
    q, k, v, lam = _inputs(64)
    ops.prefill(q, k, v, lam)  # returns at once; the launch gives up on the GPU
    _lib.load().pma_test_expire_waits(0)
    torch.cuda.synchronize()
    assert ops.pending_fault() == 90
    with pytest.raises(ops.KernelFault):
        ops.prefill(q, k, v, lam)
    _normal_call_matches_oracle(q, k, v, lam)


def test_expired_wait_in_selective_and_module(expiring_waits):
    """The selective prefill and the attention module (which calls the prefill without check)
    report the fault too."""
    from prime_moment_attention_b200.attention import PrimeMomentAttention
    q, k, v, lam = _inputs(64)
    ld = torch.full((1, 3, q.shape[2]), -1e-3, device="cuda")
    ops.selective_prefill(q, k, v, ld, torch.ones(3, device="cuda"))
    torch.cuda.synchronize()
    with pytest.raises(ops.KernelFault):
        ops.check_faults()
    m = PrimeMomentAttention(hidden_size=192, num_heads=3, head_dim=64).cuda().to(torch.bfloat16).eval()
    x = torch.randn(1, 700, 192, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        m(x)  # the chunked branch (L > 512) on tensor cores
        torch.cuda.synchronize()
        with pytest.raises(ops.KernelFault):
            m(x)
    _lib.load().pma_test_expire_waits(0)
    _normal_call_matches_oracle(q, k, v, lam)


def test_expired_wait_in_delta_wy(expiring_waits):
    """The delta-rule prefill's WY kernels give up too (code 95 from the prep kernel, whose
    launch comes first) and leave the context usable."""
    H, L = 2, 300
    q, k, v = synth.make_qkv(1, H, L, 64, seed=3, dtype=torch.bfloat16, device="cuda")
    beta = torch.full((1, H, L), 0.5, device="cuda")
    lam = torch.full((H,), 0.999, device="cuda")
    ops.delta_prefill(q, k, v, beta, None, lam)
    torch.cuda.synchronize()
    assert ops.pending_fault() == 95
    with pytest.raises(ops.KernelFault):
        ops.check_faults()
    _lib.load().pma_test_expire_waits(0)
    y, s = ops.delta_prefill(q, k, v, beta, None, lam, out_dtype=torch.float32)
    y_ref, s_ref = O.delta_prefill(q.cpu(), k.cpu(), v.cpu(), beta.cpu(), None, lam.cpu(), chunk=64, bound=25.0)
    assert O.rel_err(y.double().cpu().numpy(), y_ref) <= TOL_BF16
    assert O.rel_err(s.double().cpu().numpy(), s_ref) <= TOL_BF16
