"""torch.ops.pma.* (the C ABI registered as PyTorch operators) on the GPU: the same kernels as the
ctypes layer, so the same results bit for bit; the decode operators against the float64 oracle;
and a torch.compile(fullgraph=True) graph that calls the operators."""
import pytest
import torch

from oracle import oracle as O
from prime_moment_attention_b200 import ops, synth, torch_ops
from tests.helpers import TOL_BF16, TOL_F32, assert_close, assert_state_close, lam_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,D,L", [(torch.bfloat16, 64, 1000), (torch.bfloat16, 128, 300), (torch.float32, 32, 517)])
def test_prefill_operator_equals_ctypes_path(dtype, D, L):
    B, H = 2, 3
    q, k, v = synth.make_qkv(B, H, L, D, seed=L, dtype=dtype, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=L).cuda()
    st0 = synth.make_state(B, H, D, lam.cpu(), seed=L, t0=100, sigma=0.02, device="cuda")
    y, st = torch_ops.prefill(q, k, v, lam, state=st0)
    y2, st2 = ops.prefill(q, k, v, lam, state=st0)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    for a, b in zip(st, st2):
        assert torch.equal(a, b)
    y_ref, st_ref = O.prefill(q, k, v, lam_np(lam), state=tuple(s.cpu() for s in st0))
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    assert_close(y, y_ref, tol, "y")
    assert_state_close(st, st_ref, tol)


@pytest.mark.parametrize("inplace", [False, True])
def test_decode_operators_against_oracle(inplace):
    N, H, D = 5, 4, 64
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=9).cuda()
    st = synth.make_state(N, H, D, lam.cpu(), seed=9, device="cuda")
    ref = tuple(s.double().cpu().numpy() for s in st)
    ptrs = [t.data_ptr() for t in st]
    for t in range(3):
        q, k, v = synth.make_decode_tokens(N, H, D, seed=40 + t, dtype=torch.float32, device="cuda")
        y, st = torch_ops.decode_step(q, k, v, lam, st, inplace=inplace)
        y_ref, ref = O.decode_step(q, k, v, lam_np(lam), ref)
        assert_close(y, y_ref, TOL_F32, "y")
    assert_state_close(st, ref, TOL_F32)
    assert ([t.data_ptr() for t in st] == ptrs) == inplace


def test_operators_inside_torch_compile():
    """The operators are single opaque nodes of a compiled graph (fullgraph: no graph break)."""
    B, H, L, D = 2, 3, 600, 64
    q, k, v = synth.make_qkv(B, H, L, D, seed=3, dtype=torch.bfloat16, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=3).cuda()
    torch_ops.load()

    def f(q, k, v, lam):
        y, st = torch.ops.pma.prefill(q * 1.0, k, v, lam)
        return y.float() * 2.0, st[1].sum()

    got = torch.compile(f, fullgraph=True)(q, k, v, lam)
    want = f(q, k, v, lam)
    torch.cuda.synchronize()
    assert torch.equal(got[0], want[0]) and torch.allclose(got[1], want[1])
