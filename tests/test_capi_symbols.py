"""The C-ABI library loads and exports every entry point include/pma.h declares.

No GPU: only calls that return before touching a device are made.
"""
import ctypes
import os
import re

import pytest

from prime_moment_attention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    txt = open(os.path.join(ROOT, "include", "pma.h")).read()
    return sorted(set(re.findall(r"PMA_API\s+[\w\s\*]*?\b(pma_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = _declared()
    assert len(names) >= 8, names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/pma.h but not exported"


def test_version_and_status_strings():
    L = _lib.load()
    assert L.pma_version() == 4
    for code in range(8):
        assert _lib.status_string(code)
    assert "unknown" in _lib.status_string(99)


def test_state_floats_and_head_dims():
    L = _lib.load()
    assert L.pma_state_floats(64) == 2 * 64 * 64 + 3 * 64 + 1 == 8385  # c/prime_moment.h:17
    assert L.pma_state_floats(128) == 33153
    dims = (ctypes.c_int * 8)()
    n = L.pma_supported_head_dims(_lib.PMA_BF16, dims, 8)
    assert list(dims[:n]) == [16, 32, 64, 128]
    assert L.pma_supported_head_dims(7, dims, 8) == 0


def _seq(ptr=16, dt=_lib.PMA_F32):
    return _lib.SeqTensor(ptr, dt, 4096, 4096, 64)


@pytest.mark.parametrize("case,expect", [
    ("neg_B", 1), ("null_q", 1), ("bad_D", 2), ("bad_dtype", 3), ("mixed_dtype", 3), ("misaligned", 4),
])
def test_prefill_argument_errors_without_gpu(case, expect):
    """Host-side validation happens before any CUDA call."""
    L = _lib.load()
    q, k, v = _seq(), _seq(), _seq()
    B, D = 1, 64
    lam = 16
    if case == "neg_B":
        B = -1
    elif case == "null_q":
        q = _lib.SeqTensor(0, 0, 0, 0, 0)
    elif case == "bad_D":
        D = 48
    elif case == "bad_dtype":
        q = _seq(dt=5); k = _seq(dt=5); v = _seq(dt=5)
    elif case == "mixed_dtype":
        k = _seq(dt=_lib.PMA_BF16)
    elif case == "misaligned":
        q = _seq(ptr=20)
    rc = L.pma_prefill(B, 2, 8, D, ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), lam, 0, None, None,
                       1.0, None, None, 0, None)
    assert rc == expect, (case, rc)


def test_decode_requires_state():
    L = _lib.load()
    q = _seq()
    rc = L.pma_decode_step(2, 2, 64, ctypes.byref(q), ctypes.byref(q), ctypes.byref(q), 16, 0, None, None, 1.0,
                           ctypes.byref(q), None)
    assert rc == 1


def test_torch_operators_register_without_a_gpu():
    """_pma_torch.so loads on a host without a GPU and registers torch.ops.pma.* with the schemas
    the Python layer and torch.compile rely on; the fake implementations give output shapes."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    from prime_moment_attention_b200 import torch_ops
    torch_ops.load()
    schemas = {str(op._schema).split("(")[0] for op in (torch.ops.pma.prefill.default, torch.ops.pma.decode_step.default,
                                                         torch.ops.pma.decode_step_.default)}
    assert schemas == {"pma::prefill", "pma::decode_step", "pma::decode_step_"}
    with FakeTensorMode():
        q = torch.empty(2, 3, 10, 64, dtype=torch.bfloat16, device="cuda")
        y, st = torch.ops.pma.prefill(q, q, q, torch.empty(3, device="cuda"))
        assert y.shape == q.shape and [tuple(s.shape) for s in st] == [(2, 3, 64), (2, 3, 64, 64), (2, 3, 64, 64),
                                                                      (2, 3, 1), (2, 3, 64), (2, 3, 64)]
