"""ctypes binding of libpma.so, the C ABI declared in include/pma.h.

The library is built in place by prime_moment_attention_b200.build (nvcc, sm_100a).
Loading fails loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpma.so")

PMA_F32 = 0
PMA_BF16 = 1

STATUS = {
    0: "PMA_OK",
    1: "PMA_ERR_ARGUMENT",
    2: "PMA_ERR_HEAD_DIM",
    3: "PMA_ERR_DTYPE",
    4: "PMA_ERR_LAYOUT",
    5: "PMA_ERR_WORKSPACE",
    6: "PMA_ERR_CUDA",
    7: "PMA_ERR_DEVICE",
}


class SeqTensor(ctypes.Structure):
    """pma_seq_tensor: a [B,H,L,D] device tensor with element strides."""
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("stride_b", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("stride_l", ctypes.c_int64)]


class State(ctypes.Structure):
    """pma_state: six float32 device arrays (S0, S1, S2, Z0, Z1, Z2)."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("S0", "S1", "S2", "Z0", "Z1", "Z2")]


class Prologue(ctypes.Structure):
    """pma_prologue: GQA head map, LayerNorm QK-norm and q scale folded into the kernels."""
    _fields_ = [("kv_groups", ctypes.c_int32), ("q_scale", ctypes.c_float),
                ("q_norm_weight", ctypes.c_void_p), ("q_norm_bias", ctypes.c_void_p),
                ("k_norm_weight", ctypes.c_void_p), ("k_norm_bias", ctypes.c_void_p),
                ("norm_eps", ctypes.c_float)]


_P = ctypes.POINTER
_lib = None


class PmaError(RuntimeError):
    def __init__(self, fn: str, status: int):
        self.status = status
        msg = f"{fn} failed: {STATUS.get(status, status)} ({status_string(status)})"
        if status == 6:
            ce = load().pma_last_cuda_error()
            msg += f": cudaError {ce} {load().pma_cuda_error_string(ce).decode()}"
        super().__init__(msg)


def load() -> ctypes.CDLL:
    """Load libpma.so (once).  Raises ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m prime_moment_attention_b200.build` "
                          "(this package has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    L.pma_version.restype = ctypes.c_int
    L.pma_status_string.argtypes = [ctypes.c_int]
    L.pma_status_string.restype = ctypes.c_char_p
    L.pma_last_cuda_error.restype = ctypes.c_int
    L.pma_set_fault_word.argtypes = [ctypes.c_void_p]
    L.pma_set_fault_word.restype = None
    L.pma_test_expire_waits.argtypes = [ctypes.c_ulonglong]
    L.pma_test_expire_waits.restype = None
    L.pma_cuda_error_string.argtypes = [ctypes.c_int]
    L.pma_cuda_error_string.restype = ctypes.c_char_p
    L.pma_state_floats.argtypes = [ctypes.c_int]
    L.pma_state_floats.restype = ctypes.c_size_t
    L.pma_supported_head_dims.argtypes = [ctypes.c_int, _P(ctypes.c_int), ctypes.c_int]
    L.pma_supported_head_dims.restype = ctypes.c_int
    L.pma_prefill_workspace_bytes.argtypes = [ctypes.c_int] * 5
    L.pma_prefill_workspace_bytes.restype = ctypes.c_size_t
    L.pma_prefill.argtypes = ([ctypes.c_int] * 4 + [_P(SeqTensor)] * 3 + [ctypes.c_void_p, ctypes.c_int64]
                              + [_P(State)] * 2 + [ctypes.c_float, _P(SeqTensor), ctypes.c_void_p,
                                                   ctypes.c_size_t, ctypes.c_void_p])
    L.pma_prefill.restype = ctypes.c_int
    L.pma_prefill_resume.argtypes = L.pma_prefill.argtypes
    L.pma_prefill_resume.restype = ctypes.c_int
    L.pma_decode_step.argtypes = ([ctypes.c_int] * 3 + [_P(SeqTensor)] * 3 + [ctypes.c_void_p, ctypes.c_int64]
                                  + [_P(State)] * 2 + [ctypes.c_float, _P(SeqTensor), ctypes.c_void_p])
    L.pma_decode_step.restype = ctypes.c_int
    L.pma_decode_step_rows.argtypes = ([ctypes.c_int] * 3 + [_P(SeqTensor)] * 3 + [ctypes.c_void_p, ctypes.c_int64]
                                       + [ctypes.c_void_p, ctypes.c_int] + [_P(State)] * 2
                                       + [ctypes.c_float, _P(SeqTensor), ctypes.c_void_p])
    L.pma_decode_step_rows.restype = ctypes.c_int
    L.pma_prefill_ex_workspace_bytes.argtypes = [ctypes.c_int] * 5 + [_P(Prologue)]
    L.pma_prefill_ex_workspace_bytes.restype = ctypes.c_size_t
    L.pma_prefill_ex.argtypes = ([ctypes.c_int] * 4 + [_P(SeqTensor)] * 3 + [_P(Prologue)]
                                 + [ctypes.c_void_p, ctypes.c_int64] + [_P(State)] * 2
                                 + [ctypes.c_float, _P(SeqTensor), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p])
    L.pma_prefill_ex.restype = ctypes.c_int
    L.pma_decode_step_ex.argtypes = ([ctypes.c_int] * 3 + [_P(SeqTensor)] * 3 + [_P(Prologue)]
                                     + [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int]
                                     + [_P(State)] * 2 + [ctypes.c_float, _P(SeqTensor), ctypes.c_void_p])
    L.pma_decode_step_ex.restype = ctypes.c_int
    L.pma_delta_prefill.argtypes = ([ctypes.c_int] * 4 + [_P(SeqTensor)] * 3 + [ctypes.c_void_p] * 3
                                    + [ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_float]
                                    + [ctypes.c_void_p] * 2 + [_P(SeqTensor), ctypes.c_void_p, ctypes.c_size_t,
                                                               ctypes.c_void_p])
    L.pma_delta_prefill.restype = ctypes.c_int
    L.pma_delta_prefill_workspace_bytes.argtypes = [ctypes.c_int] * 6
    L.pma_delta_prefill_workspace_bytes.restype = ctypes.c_size_t
    L.pma_delta_decode_step.argtypes = ([ctypes.c_int] * 3 + [_P(SeqTensor)] * 3 + [ctypes.c_void_p] * 2
                                        + [ctypes.c_float] * 2 + [ctypes.c_void_p] * 2
                                        + [_P(SeqTensor), ctypes.c_void_p])
    L.pma_delta_decode_step.restype = ctypes.c_int
    L.pma_selective_prefill_workspace_bytes.argtypes = [ctypes.c_int] * 5 + [_P(Prologue)]
    L.pma_selective_prefill_workspace_bytes.restype = ctypes.c_size_t
    L.pma_selective_prefill.argtypes = ([ctypes.c_int] * 4 + [_P(SeqTensor)] * 3 + [_P(Prologue)]
                                        + [ctypes.c_void_p] * 2 + [_P(State)] * 2
                                        + [ctypes.c_float, _P(SeqTensor), ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.c_void_p])
    L.pma_selective_prefill.restype = ctypes.c_int
    L.pma_selective_decode_step.argtypes = ([ctypes.c_int] * 3 + [_P(SeqTensor)] * 3 + [_P(Prologue)]
                                            + [ctypes.c_void_p] * 2 + [ctypes.c_void_p, ctypes.c_int]
                                            + [_P(State)] * 2 + [ctypes.c_float, _P(SeqTensor), ctypes.c_void_p])
    L.pma_selective_decode_step.restype = ctypes.c_int
    L.pma_state_combine.argtypes = ([ctypes.c_int] * 3 + [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64]
                                    + [_P(State)] * 2 + [ctypes.c_void_p])
    L.pma_state_combine.restype = ctypes.c_int
    L.pma_swiglu.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    L.pma_swiglu.restype = ctypes.c_int
    _lib = L
    return L


def status_string(status: int) -> str:
    return load().pma_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != 0:
        raise PmaError(fn, status)
