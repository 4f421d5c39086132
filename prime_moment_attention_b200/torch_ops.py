"""torch.ops.pma: the prefill and decode step as PyTorch operators (csrc/torch_ops.cpp over libpma.so).

The reference binds its native kernels as a pybind module of libtorch functions
(src/prime_moment_attention/prime_cpp_kernel.cpp:119-124).  Here they are dispatcher operators,
callable without ctypes and traceable by torch.compile / torch.export, which see each call as one
opaque node whose output shapes come from the fake implementations registered below.

    torch.ops.pma.prefill(q, k, v, decay, state=None, eps=1.0, return_state=True) -> (y, [state])
    torch.ops.pma.decode_step(q, k, v, decay, state, eps=1.0) -> (y, [new state])
    torch.ops.pma.decode_step_(q, k, v, decay, state, eps=1.0) -> y        (state updated in place)

`decay` is a float32 CUDA tensor of H (or B*H) decays; states are the reference tuple
(S0, S1, S2, K0, K1, K2) in float32.  Loading fails loudly when _pma_torch.so is missing.
"""
from __future__ import annotations

import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_pma_torch.so")
_loaded = False


def _state_like(B: int, H: int, D: int, device):
    f = lambda *s: torch.empty(*s, dtype=torch.float32, device=device)  # noqa: E731
    return [f(B, H, D), f(B, H, D, D), f(B, H, D, D), f(B, H, 1), f(B, H, D), f(B, H, D)]


def load() -> None:
    """Load the operator library (once) and register the operators' shape functions."""
    global _loaded
    if _loaded:
        return
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m prime_moment_attention_b200.build`")
    torch.ops.load_library(LIB_PATH)

    @torch.library.register_fake("pma::prefill")
    def _prefill_fake(q, k, v, decay, state=None, eps=1.0, return_state=True):
        B, H, L, D = q.shape
        return q.new_empty(B, H, L, D), (_state_like(B, H, D, q.device) if return_state else [])

    @torch.library.register_fake("pma::decode_step")
    def _decode_fake(q, k, v, decay, state, eps=1.0):
        N, H, D = q.shape
        return q.new_empty(N, H, D), _state_like(N, H, D, q.device)

    @torch.library.register_fake("pma::decode_step_")
    def _decode_inplace_fake(q, k, v, decay, state, eps=1.0):
        return q.new_empty(q.shape)

    _loaded = True


def prefill(q, k, v, decay: torch.Tensor, state=None, eps: float = 1.0, return_state: bool = True):
    """torch.ops.pma.prefill with the library loaded; returns (y, state tuple or None)."""
    load()
    y, st = torch.ops.pma.prefill(q, k, v, decay, None if state is None else list(state), eps, return_state)
    return y, (tuple(st) if return_state else None)


def decode_step(q, k, v, decay: torch.Tensor, state, eps: float = 1.0, inplace: bool = False):
    """torch.ops.pma.decode_step (functional) or decode_step_ (inplace); returns (y, state tuple)."""
    load()
    if inplace:
        return torch.ops.pma.decode_step_(q, k, v, decay, list(state), eps), tuple(state)
    y, st = torch.ops.pma.decode_step(q, k, v, decay, list(state), eps)
    return y, tuple(st)
