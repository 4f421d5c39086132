"""Moment-state cache with the reference's API (src/prime_moment_attention/cache.py:15-56).

Per layer it holds the state tuple (S0, S1, S2, K0, K1, K2) the attention
returns; memory is independent of sequence length.  Like the reference it
subclasses transformers' Cache when transformers is importable, and counts
seen tokens on layer 0 in update().
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

try:  # the reference subclasses transformers.cache_utils.Cache (cache.py:13-15)
    from transformers.cache_utils import Cache as _Base
except Exception:  # pragma: no cover - transformers absent
    _Base = object


class PrimeMomentCache(_Base):
    def __init__(self):
        if _Base is not object:
            try:
                super().__init__(layers=[])
            except (TypeError, ValueError):
                try:
                    super().__init__()
                except Exception:
                    pass
        self.prime_states: Dict[int, Tuple[torch.Tensor, ...]] = {}
        self._seen_tokens = 0

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        return self._seen_tokens

    def get_max_cache_shape(self) -> Optional[int]:
        return None

    def get_max_length(self) -> Optional[int]:
        return None

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None):
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[-2]
        return key_states, value_states

    def get_state(self, layer_idx: int) -> Optional[Tuple[torch.Tensor, ...]]:
        return self.prime_states.get(layer_idx, None)

    def set_state(self, layer_idx: int, state: Tuple[torch.Tensor, ...]):
        self.prime_states[layer_idx] = state

    def reset(self):
        self.prime_states.clear()
        self._seen_tokens = 0
