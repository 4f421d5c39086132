"""Decode-state cache on device-resident pool rows, under the reference's cache API.

The reference's PrimeMomentCache (src/prime_moment_attention/cache.py:15-56) keeps a dict from
layer index to whatever 6-tuple the attention returned, so every decode step allocates a new
tuple and the cache only swaps references.  Here the cache owns one StatePool whose slots are
the batch rows: layer l of the cache is pool rows [l*B, (l+1)*B), a contiguous block of every
state tensor.  `get_state` hands out views of that block, `set_state` copies into it (or does
nothing when it is given those same views back), and `decode_step` advances a layer in place
through pma_decode_step_rows -- the state never leaves its rows and no step allocates one.

The method names and the token counting of `update` are the reference's interface
(get_state / set_state / reset / get_seq_length / update, cache.py:29-56), so code written
against the reference cache, and transformers' Cache protocol, keeps working.
"""
from __future__ import annotations

import inspect
from typing import Any, Dict, List, Optional, Tuple

import torch

from . import ops
from .pool import StatePool

try:  # the reference derives from transformers' Cache; so does this class when it is importable
    from transformers.cache_utils import Cache as _Base
except Exception:  # pragma: no cover - transformers absent
    _Base = object

StateTuple = Tuple[torch.Tensor, ...]


def _base_init(obj) -> None:
    """Call the transformers Cache constructor in the form the installed version takes."""
    if _Base is object:
        return
    if "layers" in inspect.signature(_Base.__init__).parameters:  # transformers >= 4.56: layered caches
        _Base.__init__(obj, layers=[])
    else:
        _Base.__init__(obj)


class PrimeMomentCache(_Base):
    """Moment states of a batch of B sequences for `num_layers` layers, in one StatePool.

    The pool is made by the first `set_state` (batch, heads, head dim and device come from that
    state) unless `batch`, `num_heads` and `head_dim` are given here.  A layer index beyond
    `num_layers` grows the pool (a new allocation: views handed out before then stop tracking the
    cache), so pass the model's layer count to keep every view live.  A cache serves one batch
    shape; `reset()` forgets it."""

    def __init__(self, num_layers: int = 1, batch: Optional[int] = None, num_heads: Optional[int] = None,
                 head_dim: Optional[int] = None, device=None):
        _base_init(self)
        self._num_layers = max(1, int(num_layers))
        self._device = torch.device(device) if device is not None else None
        self.pool: Optional[StatePool] = None
        self._filled: List[bool] = []
        self._rows: Dict[int, torch.Tensor] = {}
        self._seen_tokens = 0
        if batch is not None and num_heads is not None and head_dim is not None:
            self._make_pool(batch, num_heads, head_dim, self._device or torch.device("cuda"), self._num_layers)

    # ---------------------------------------------------------------- pool rows
    def _make_pool(self, B: int, H: int, D: int, device, layers: int, keep: Optional[StatePool] = None) -> None:
        pool = StatePool(capacity=B, H=H, D=D, layers=layers, device=device)
        pool._free.clear()  # every slot is a batch row of this cache
        if keep is not None:  # growth: the old layers' rows move over
            n = keep.layers * B
            for dst, src in zip(pool.state, keep.state):
                dst[:n].copy_(src)
        self.pool = pool
        self._filled = (self._filled + [False] * layers)[:layers]
        self._rows.clear()

    def _block(self, layer_idx: int) -> StateTuple:
        B = self.pool.capacity
        r0 = layer_idx * B
        return tuple(t[r0:r0 + B] for t in self.pool.state)

    def _rows_of(self, layer_idx: int) -> torch.Tensor:
        r = self._rows.get(layer_idx)
        if r is None:
            B = self.pool.capacity
            r = torch.arange(layer_idx * B, (layer_idx + 1) * B, dtype=torch.int32, device=self.pool.device)
            self._rows[layer_idx] = r
        return r

    @property
    def prime_states(self) -> Dict[int, StateTuple]:
        """Layer index -> state views, for the layers that hold a state (the reference's dict)."""
        return {i: self._block(i) for i, f in enumerate(self._filled) if f}

    # ---------------------------------------------------------------- the reference's API
    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        return self._seen_tokens

    def get_max_cache_shape(self) -> Optional[int]:
        return None  # constant-size state: no maximum length

    def get_max_length(self) -> Optional[int]:
        return None

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None):
        """No key/value history is kept; tokens are counted once per step, on layer 0."""
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[-2]
        return key_states, value_states

    def get_state(self, layer_idx: int) -> Optional[StateTuple]:
        """Views (S0, S1, S2, K0, K1, K2) of the layer's pool rows, or None if never set."""
        if self.pool is None or layer_idx >= len(self._filled) or not self._filled[layer_idx]:
            return None
        return self._block(layer_idx)

    def set_state(self, layer_idx: int, state: StateTuple) -> None:
        """Copy `state` (the reference tuple layout, any float dtype) into the layer's rows."""
        if len(state) != 6:
            raise ValueError("state must be the 6-tuple (S0, S1, S2, K0, K1, K2)")
        B, H, D = state[0].shape
        if self.pool is None:
            self._make_pool(B, H, D, self._device or state[0].device, max(self._num_layers, layer_idx + 1))
        elif (B, H, D) != (self.pool.capacity, self.pool.H, self.pool.D):
            raise ValueError(f"state of shape [B={B}, H={H}, D={D}] does not fit this cache's "
                             f"[B={self.pool.capacity}, H={self.pool.H}, D={self.pool.D}] (reset() first)")
        elif layer_idx >= self.pool.layers:
            self._make_pool(B, H, D, self.pool.device, max(2 * self.pool.layers, layer_idx + 1), keep=self.pool)
        block = self._block(layer_idx)
        for dst, src in zip(block, state):
            if src.data_ptr() != dst.data_ptr():  # the cache's own views come back unchanged
                dst.copy_(src.reshape(dst.shape))
        self._filled[layer_idx] = True

    def reset(self) -> None:
        """Forget every state and the token count (the pool is released)."""
        self.pool = None
        self._filled = []
        self._rows.clear()
        self._seen_tokens = 0

    # ---------------------------------------------------------------- in-place decode
    def decode_step(self, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, decay,
                    eps: float = 1.0, y_out: Optional[torch.Tensor] = None,
                    prologue: Optional[ops.Prologue] = None) -> torch.Tensor:
        """One token for every batch row of `layer_idx` (q, k, v [B, H, D]); the layer's rows are
        updated in place by pma_decode_step_rows, with no state allocated or copied.  Returns y."""
        if self.get_state(layer_idx) is None:
            raise KeyError(f"layer {layer_idx} holds no state: set_state or a prefill first")
        return ops.decode_step_rows(q, k, v, decay, self.pool.state, self._rows_of(layer_idx), eps=eps,
                                    y_out=y_out, prologue=prologue)
