"""Device-resident state pool for serving: many sequences' moment states in one allocation.

The reference keeps one 6-tuple of state tensors per layer in `PrimeMomentCache`
(src/prime_moment_attention/cache.py:15-56) and hands it to the decode branch
(attention.py:120-143), which returns fresh tensors every step.  A serving loop whose
batch changes every step would gather and scatter those tuples.  Here every sequence
owns a slot; each (layer, slot) pair is one row of H head-states in a pool laid out like
a state tuple of `layers * capacity` rows, and `pma_decode_step_rows` updates the rows of
the current batch in place -- the batch is just an int32 row table.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import ops

StateTuple = ops.StateTuple


class StatePool:
    """`layers` x `capacity` rows of H head-states (float32, zero-initialised)."""

    def __init__(self, capacity: int, H: int, D: int, layers: int = 1, device=None):
        if capacity <= 0 or layers <= 0:
            raise ValueError("capacity and layers must be positive")
        self.capacity, self.H, self.D, self.layers = capacity, H, D, layers
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.state = ops.new_state(layers * capacity, H, D, self.device, zero=True)
        self._free: List[int] = list(range(capacity - 1, -1, -1))
        self.seen_tokens = [0] * capacity  # per slot, as PrimeMomentCache._seen_tokens per cache

    # ---------------------------------------------------------------- slots
    def alloc(self) -> int:
        """A free slot, its rows zeroed."""
        if not self._free:
            raise RuntimeError("state pool is full")
        slot = self._free.pop()
        self.reset(slot)
        return slot

    def release(self, slot: int) -> None:
        if not 0 <= slot < self.capacity or slot in self._free:
            raise ValueError(f"slot {slot} is not allocated")
        self._free.append(slot)

    @property
    def free_slots(self) -> int:
        return len(self._free)

    def reset(self, slot: int) -> None:
        for layer in range(self.layers):
            for t in self.get_state(layer, slot):
                t.zero_()
        self.seen_tokens[slot] = 0

    def rows(self, layer: int, slots) -> torch.Tensor:
        """Pool rows (int32, on the pool's device) of `slots` in `layer`."""
        s = torch.as_tensor(slots, dtype=torch.int32)
        return (s + layer * self.capacity).to(self.device, non_blocking=True)

    # ---------------------------------------------------------------- state views
    def get_state(self, layer: int, slot: int) -> StateTuple:
        """The (S0, S1, S2, Z0, Z1, Z2) of one sequence in one layer: views [1, H, ...] into the pool."""
        r = layer * self.capacity + slot
        return tuple(t[r:r + 1] for t in self.state)

    def set_state(self, layer: int, slot: int, state: StateTuple) -> None:
        for dst, src in zip(self.get_state(layer, slot), state):
            dst.copy_(src.reshape(dst.shape))

    # ---------------------------------------------------------------- compute
    def prefill(self, layer: int, slot: int, q, k, v, decay, eps: float = 1.0, y_out=None, continue_state=False):
        """Prefill one sequence ([1, H, L, D]) into its slot; returns y.  With continue_state the
        slot's current state is the incoming state (a continued prompt), else it starts from zero."""
        st = self.get_state(layer, slot) if continue_state else None
        y, out = ops.prefill(q, k, v, decay, state=st, eps=eps, return_state=True, y_out=y_out)
        self.set_state(layer, slot, out)
        if layer == 0:
            self.seen_tokens[slot] += q.shape[2]
        return y

    def decode_step(self, layer: int, slots: Sequence[int], q, k, v, decay, eps: float = 1.0,
                    y_out: Optional[torch.Tensor] = None, rows: Optional[torch.Tensor] = None):
        """One token for the batch `slots` (row n of q, k, v [N, H, D] belongs to slots[n]); the
        slots' states are updated in place.  `rows` may pass a prebuilt `self.rows(layer, slots)`."""
        r = rows if rows is not None else self.rows(layer, slots)
        y = ops.decode_step_rows(q, k, v, decay, self.state, r, eps=eps, y_out=y_out)
        if layer == 0:
            for s in slots:
                self.seen_tokens[s] += 1
        return y
