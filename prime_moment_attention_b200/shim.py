"""install()/uninstall(): route the reference PrimeMomentAttention onto the CUDA kernels.

`install()` replaces PrimeMomentAttention.forward of the reference package
(src/prime_moment_attention/attention.py:77-210) by attention.moment_forward,
which keeps the reference's projection / QK-norm / scale code and sends all three
L branches to libpma.so.  The state tuple format is unchanged, so
PrimeMomentCache and PrimeForCausalLM (model.py:101-120, 203-242) work as they are.
`install(ChunkedGatedDeltaPrimeAttention)` does the same for the reference's gated
delta-rule module (chunked_delta_prime.py:89-283) with delta.delta_forward, and
`install(PrimeSelectiveMomentAttention)` for the selective module (selective.py:264-444) with
selective.selective_forward.
`uninstall()` restores the original forward.
"""
from __future__ import annotations

from .attention import moment_forward
from .delta import delta_forward
from .selective import selective_forward

_saved: dict = {}


def _default_cls():
    from prime_moment_attention.attention import PrimeMomentAttention  # the reference package
    return PrimeMomentAttention


def _forward_for(cls):
    """The kernel forward for a reference class: the gated delta-rule module
    (chunked_delta_prime.py) and the selective module (selective.py) have their own cores;
    everything else is the moment-attention forward."""
    if hasattr(cls, "_build_features") or "Delta" in cls.__name__:
        return delta_forward
    if hasattr(cls, "get_tau") or "Selective" in cls.__name__:
        return selective_forward
    return moment_forward


def install(cls=None):
    """Patch `cls.forward` (default: the reference PrimeMomentAttention; also accepts the
    reference ChunkedGatedDeltaPrimeAttention).  Idempotent."""
    from . import _lib
    _lib.load()  # fail now, not at the first forward, if the library is missing
    cls = cls or _default_cls()
    if cls not in _saved:
        _saved[cls] = cls.__dict__["forward"]
        cls.forward = _forward_for(cls)
    return cls


def uninstall(cls=None):
    """Restore the forward saved by install(); a no-op if it was not installed."""
    cls = cls or _default_cls()
    fwd = _saved.pop(cls, None)
    if fwd is not None:
        cls.forward = fwd
    return cls


def installed(cls=None) -> bool:
    cls = cls or _default_cls()
    return cls in _saved
