"""pma_prefill_no_alloc: the prefill entry point that allocates nothing.

It exists for callers that cannot allocate device memory (a plugin inside a host
application that owns all device memory, FFI callers without a device allocator,
loops where an allocation would synchronise the device).  This file is collected
last so that a run stopping at the first failure has already run every other test.

Each case calls the new entry point through the C ABI twice in a row (the second
call finds the previous call's contents in the shared static buffer) and checks
both results against pma_prefill with a caller-provided workspace, within the
parity bars the other tests use.
"""
import ctypes

import pytest
import torch

from prime_moment_attention_b200 import _lib, ops, synth
from tests.helpers import TOL_BF16, TOL_F32, assert_close, cpu64

pytestmark = pytest.mark.gpu

STATIC_SCRATCH = 16 << 20


def _entry():
    f = _lib.load().pma_prefill_no_alloc
    P = ctypes.POINTER
    f.argtypes = ([ctypes.c_int] * 4 + [P(_lib.SeqTensor)] * 3 + [ctypes.c_void_p, ctypes.c_int64]
                  + [P(_lib.State)] * 2 + [ctypes.c_float, P(_lib.SeqTensor), ctypes.c_void_p])
    f.restype = ctypes.c_int
    return f


def _seq(t):
    return _lib.SeqTensor(t.data_ptr(), 0 if t.dtype == torch.float32 else 1, t.stride(0), t.stride(1), t.stride(2))


@pytest.mark.parametrize("dtype,B,H,L,D", [
    (torch.bfloat16, 1, 4, 4173, 64),   # tensor-core kernel, split into segments (scratch holds their states)
    (torch.bfloat16, 2, 3, 300, 64),    # tensor-core kernel, status word only
    (torch.bfloat16, 1, 4, 2000, 128),  # head-dim-128 tensor-core kernel, segmented
    (torch.float32, 1, 2, 1000, 32),    # CUDA-core kernel, segmented
])
def test_no_alloc_matches_workspace_entry_point(dtype, B, H, L, D):
    tol = TOL_F32 if dtype == torch.float32 else TOL_BF16
    q, k, v = synth.make_qkv(B, H, L, D, seed=L + D, dtype=dtype, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=L).cuda()
    st0 = synth.make_state(B, H, D, lam.cpu(), seed=L, t0=500, sigma=0.02, device="cuda")
    y_ref, st_ref = ops.prefill(q, k, v, lam, state=st0, out_dtype=torch.float32)
    ws = _lib.load().pma_prefill_workspace_bytes(B, H, L, D, 0 if dtype == torch.float32 else 1)
    assert 0 < ws <= STATIC_SCRATCH
    f = _entry()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        y = torch.full((B, H, L, D), float("nan"), device="cuda")
        st = tuple(torch.full_like(s, float("nan")) for s in st_ref)
        st_in = _lib.State(*[t.data_ptr() for t in st0])
        st_out = _lib.State(*[t.data_ptr() for t in st])
        rc = f(B, H, L, D, ctypes.byref(_seq(q)), ctypes.byref(_seq(k)), ctypes.byref(_seq(v)), lam.data_ptr(), 0,
               ctypes.byref(st_in), ctypes.byref(st_out), 1.0, ctypes.byref(_seq(y)), stream)
        assert rc == 0, _lib.status_string(rc)
        torch.cuda.synchronize()
        assert_close(y, cpu64(y_ref), tol, f"y, call {call}")
        for a, b in zip(st, st_ref):
            assert_close(a, cpu64(b), tol, f"state, call {call}")


def test_no_alloc_rejects_problems_beyond_its_buffer():
    """float32, D=128, one head-state, 148 chunks of 32 tokens: the plan splits it
    into 148 segments whose states need more than the 16 MiB buffer -> PMA_ERR_WORKSPACE."""
    B, H, L, D = 1, 1, 4736, 128
    assert _lib.load().pma_prefill_workspace_bytes(B, H, L, D, 0) > STATIC_SCRATCH
    q = torch.zeros(B, H, L, D, device="cuda")
    y = torch.empty_like(q)
    lam = torch.full((H,), 0.99, device="cuda")
    rc = _entry()(B, H, L, D, ctypes.byref(_seq(q)), ctypes.byref(_seq(q)), ctypes.byref(_seq(q)), lam.data_ptr(), 0,
                  None, None, 1.0, ctypes.byref(_seq(y)), torch.cuda.current_stream().cuda_stream)
    assert rc == 5  # PMA_ERR_WORKSPACE


def test_no_alloc_status_reaches_the_caller():
    """The status word of this entry point lives in its static buffer, out of the caller's reach;
    a caller sees an expired wait through the fault word it registers (pma_set_fault_word; here
    the module's pinned host word).  Normal calls leave it 0; a launch made to give up by the
    test hook (a bounded wait on a barrier nothing completes, before any work is issued) leaves
    code 90, and the next normal call through this entry point is correct again."""
    ops.check_faults(synchronize=True)  # registers the word; nothing pending
    B, H, L, D = 2, 3, 300, 64
    q, k, v = synth.make_qkv(B, H, L, D, seed=11, dtype=torch.bfloat16, device="cuda")
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=11).cuda()
    y_ref, _ = ops.prefill(q, k, v, lam, out_dtype=torch.float32)
    f = _entry()
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        y = torch.full((B, H, L, D), float("nan"), device="cuda")
        rc = f(B, H, L, D, ctypes.byref(_seq(q)), ctypes.byref(_seq(k)), ctypes.byref(_seq(v)), lam.data_ptr(), 0,
               None, None, 1.0, ctypes.byref(_seq(y)), stream)
        assert rc == 0, _lib.status_string(rc)
        torch.cuda.synchronize()
        return y

    assert_close(call(), cpu64(y_ref), TOL_BF16, "y")
    assert ops.pending_fault() == 0
    _lib.load().pma_test_expire_waits(1_000_000)
    try:
        call()
    finally:
        _lib.load().pma_test_expire_waits(0)
    assert ops.pending_fault() == 90
    with pytest.raises(ops.KernelFault):
        ops.check_faults()
    assert_close(call(), cpu64(y_ref), TOL_BF16, "y after the expired wait")
    assert ops.pending_fault() == 0
