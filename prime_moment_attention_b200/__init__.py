"""B200 (sm_100a) implementation of PRIME moment attention's hot path.

The chunked prefill and the recurrent decode step over the per-head moment state
(S0, S1, S2, Z0, Z1, Z2 with per-head decay), as hand-written CUDA behind the C ABI
of include/pma.h (libpma.so), with a host-side mirror of the reference interface:

    PrimeMomentAttention, chunked_prime_ssd_core, PrimeMomentCache   (same API as the reference)
    ChunkedGatedDeltaPrimeAttention                                   (gated delta-rule variant)
    PrimeSelectiveMomentAttention                                     (selective variant)
    install(), uninstall()                                            (patch the reference module)
    ops.prefill, ops.decode_step, ops.state_combine                   (torch-facing C-ABI calls)
    sp.sequence_parallel_prefill                                      (sequence shards over GPUs)
"""
from .attention import PrimeMomentAttention, chunked_prime_ssd_core, moment_forward
from .cache import PrimeMomentCache
from .delta import ChunkedGatedDeltaPrimeAttention, delta_forward
from .selective import PrimeSelectiveMomentAttention, selective_forward
from .shim import install, installed, uninstall
from . import ops

__all__ = ["PrimeMomentAttention", "chunked_prime_ssd_core", "moment_forward", "PrimeMomentCache",
           "ChunkedGatedDeltaPrimeAttention", "delta_forward", "PrimeSelectiveMomentAttention",
           "selective_forward", "install",
           "uninstall", "installed", "ops"]
