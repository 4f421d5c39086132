"""Sequence-parallel prefill: one long sequence split into contiguous shards, one per rank.

Rank g holds tokens [g*Ls, (g+1)*Ls) of every (b, h) head-state.  The recurrence
S_t = l S_{t-1} + u_t is linear, so the state entering shard g is a decay-weighted fold
of the states the earlier shards produce from zero -- the associative step the reference
evaluates as its inter-chunk carry (src/prime_moment_attention/chunked_ssd.py:113-126):

  pass 1   T_g   = state after shard g, started from zero   (state-only prefill, k and v only)
  exchange all_gather of every rank's T_g (one flat float32 buffer per rank)
  prefix   S_in[g] = l^{L_{g-1}} (... (l^{L_0} S_init + T_0) ...) + T_{g-1}   (pma_state_combine)
  pass 2   y_g, S_out[g] = prefill of shard g from S_in[g]

Inside a GPU a long shard is itself split into segments across SMs; pass 1 leaves the state
entering each segment (from a zero start) in its workspace, and pass 2 (pma_prefill_resume)
shifts those by l^start S_in[g] instead of recomputing them, so k and v are read twice, not three
times.

The exchange is the only collective (an NCCL all-gather of H*(2D^2+3D+1)*4 bytes per
rank and batch row, over NVLink); there is no data-path traffic.  The final state of the
whole sequence is S_out[G-1], held by the last rank (broadcast on request).

The per-rank compute goes through `kernels` (a small object with `shard_state`, `shard_output`
and `combine`), the CUDA kernels by default; tests substitute a CPU implementation so that the
collective and prefix logic runs under `gloo` without a GPU.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch
import torch.distributed as dist

StateTuple = Tuple[torch.Tensor, ...]


def state_numel(B: int, H: int, D: int) -> int:
    """Floats in a [B, H] block of head-states (S0, S1, S2, Z0, Z1, Z2)."""
    return B * H * (2 * D * D + 3 * D + 1)


def flatten_state(state: StateTuple) -> torch.Tensor:
    """One contiguous float32 buffer in the order S0, S1, S2, Z1, Z2, Z0."""
    S0, S1, S2, Z0, Z1, Z2 = state
    return torch.cat([t.reshape(-1).float() for t in (S0, S1, S2, Z1, Z2, Z0)])


def unflatten_state(flat: torch.Tensor, B: int, H: int, D: int) -> StateTuple:
    """Views of `flat` (layout of `flatten_state`) in the reference tuple order."""
    BH = B * H
    o = [0, BH * D, BH * D * (D + 1), BH * D * (2 * D + 1), BH * D * (2 * D + 2), BH * D * (2 * D + 3)]
    S0 = flat[o[0]:o[1]].view(B, H, D)
    S1 = flat[o[1]:o[2]].view(B, H, D, D)
    S2 = flat[o[2]:o[3]].view(B, H, D, D)
    Z1 = flat[o[3]:o[4]].view(B, H, D)
    Z2 = flat[o[4]:o[5]].view(B, H, D)
    Z0 = flat[o[5]:o[5] + BH].view(B, H, 1)
    return (S0, S1, S2, Z0, Z1, Z2)


class CudaKernels:
    """The B200 kernels behind `sequence_parallel_prefill` (the default)."""

    @staticmethod
    def shard_state(q, k, v, decay, eps):
        """Pass 1: the shard's state from zero, and the workspace pass 2 resumes from."""
        from . import ops
        ws = ops.prefill_workspace(q)
        _, T = ops.prefill(q, k, v, decay, eps=eps, return_state=True, want_y=False, workspace=ws)
        return T, ws

    @staticmethod
    def shard_output(q, k, v, decay, state, eps, y_out, handle):
        """Pass 2: y and the final state of the shard from its carried state `state` (None: zero)."""
        from . import ops
        return ops.prefill(q, k, v, decay, state=state, eps=eps, return_state=True, y_out=y_out,
                           workspace=handle, resume=True)

    @staticmethod
    def combine(T, P, decay, length):
        from . import ops
        return ops.state_combine(T, P, decay, length)


def sequence_parallel_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, decay,
                              state: Optional[StateTuple] = None, eps: float = 1.0,
                              group: Optional[dist.ProcessGroup] = None, y_out: Optional[torch.Tensor] = None,
                              shard_lengths: Optional[Sequence[int]] = None, broadcast_final: bool = False,
                              kernels=CudaKernels, validate: bool = False):
    """Prefill of this rank's shard [B, H, Ls, D] of a sequence split over the ranks of `group`.

    `state` is the state entering the whole sequence, the same on every rank (None = zero).
    `shard_lengths` gives every rank's Ls (default: all equal to this rank's).  Returns
    (y of this shard, final state of the sequence on the last rank -- or on every rank with
    broadcast_final -- else None).  Every rank takes the same collective steps in the same
    order, so an exception on one rank surfaces on the others as a collective error or timeout
    (the process group's timeout bounds every wait).  validate=True checks every received shard state
    for non-finite values before folding it (one device synchronisation) and raises ValueError naming
    the rank it came from; every rank checks the same gathered buffer, so all of them raise."""
    G = dist.get_world_size(group)
    r = dist.get_rank(group)
    B, H, Ls, D = q.shape
    lens = list(shard_lengths) if shard_lengths is not None else [Ls] * G
    if len(lens) != G or lens[r] != Ls:
        raise ValueError(f"shard_lengths {lens} do not match world size {G} / this shard's length {Ls}")

    # pass 1: this shard's state from zero (k, v only)
    T, handle = kernels.shard_state(q, k, v, decay, eps)
    mine = flatten_state(T)
    n = mine.numel()
    gathered = torch.empty(G * n, dtype=mine.dtype, device=mine.device)
    dist.all_gather_into_tensor(gathered, mine, group=group)
    if validate:
        finite = torch.isfinite(gathered.view(G, n)).all(dim=1).tolist()
        bad = [g for g, ok in enumerate(finite) if not ok]
        if bad:
            raise ValueError(f"shard state received from rank(s) {bad} holds non-finite values")

    # prefix fold: S_in[r] from the incoming state and shards 0..r-1
    if r == 0:
        P = state  # None: start from zero
    else:
        P = unflatten_state(flatten_state(state).clone() if state is not None else
                            torch.zeros(n, dtype=mine.dtype, device=mine.device), B, H, D)
        for g in range(r):
            kernels.combine(unflatten_state(gathered[g * n:(g + 1) * n], B, H, D), P, decay, lens[g])

    # pass 2: the shard from its carried state
    y, S_out = kernels.shard_output(q, k, v, decay, P, eps, y_out, handle)
    final = S_out if r == G - 1 else None
    if broadcast_final:
        buf = flatten_state(S_out) if r == G - 1 else torch.empty(n, dtype=mine.dtype, device=mine.device)
        dist.broadcast(buf, src=dist.get_global_rank(group, G - 1) if group is not None else G - 1, group=group)
        final = unflatten_state(buf, B, H, D)
    return y, final
