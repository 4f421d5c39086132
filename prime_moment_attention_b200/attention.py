"""Host-side mirror of the reference's attention interface, running on libpma.so.

Mirrors, with the same names, arguments and return values:
  * PrimeMomentAttention          src/prime_moment_attention/attention.py:42-210
  * chunked_prime_ssd_core        src/prime_moment_attention/chunked_ssd.py:48-184

The projections stay in PyTorch (cuBLAS).  The GQA repeat, LayerNorm QK-norm and
1/sqrt(D) scale of attention.py:92-101 are folded into the kernels' load stage
(ops.Prologue / pma_prologue): the kernels read the projection outputs in place and
no repeated, normalised or scaled copy of q, k, v is written.  (When the norms are
not nn.LayerNorm over head_dim with one shared eps, PyTorch applies them as the
reference writes them and only the core runs on the kernels.)  The three
L branches of the reference (decode L == 1, dense 1 < L <= chunk_threshold,
chunked L > chunk_threshold) all go to the CUDA kernels: decode to
pma_decode_step, both prefill branches to pma_prefill, whose result does not
depend on the chunk size beyond rounding.  Differences from the reference, all
deliberate:
  * an incoming state works with every L (the reference's chunked core breaks on
    it, chunked_ssd.py:129-137), and the dense branch's clamp-before-carry quirk
    (attention.py:177 vs 185) is not reproduced: every branch computes the
    token recurrence;
  * `decay` may also be a per-head sequence or tensor (one value per head);
  * q, k, v reach the kernels in their own dtype (bf16 or fp32); the kernels
    widen to fp32 exactly as the reference's .to(torch.float32) does (:104-106).
Inference only: the kernels have no backward, so calling with autograd
recording through parameters that require grad raises.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple, Union

import torch
import torch.nn as nn

from . import ops


def chunked_prime_ssd_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           state: Optional[Tuple[torch.Tensor, ...]] = None,
                           decay: Union[float, Sequence[float], torch.Tensor] = 0.9995, eps: float = 1.0,
                           chunk_size: int = 64, return_state: bool = False):
    """Chunked PRIME prefill over projected, normalised, pre-scaled q, k, v [B,H,L,D].

    Same contract as chunked_ssd.py:48-57.  Returns (y [B,H,L,D] float32, state or None).
    `chunk_size` must be positive; the kernels pick their own internal chunk
    (64 on CUDA cores, 128 on tensor cores), which changes only rounding."""
    if int(chunk_size) <= 0:
        raise ValueError("chunk_size must be positive")
    y, st = ops.prefill(q, k, v, decay, state=state, eps=eps, return_state=return_state,
                        out_dtype=torch.float32)
    return y, st


def _prologue(self) -> Optional[ops.Prologue]:
    """The module's GQA map, QK-norm and scale as a kernel prologue; None when use_qk_norm is
    set with norms other than nn.LayerNorm(head_dim) sharing one eps.  float32 copies of
    bf16 norm parameters are cached on the module, keyed on the parameters' storage and
    version counter (an in-place weight update invalidates them)."""
    D = self.head_dim
    kw = dict(kv_groups=self.num_kv_groups, q_scale=self.scaling)
    if not self.use_qk_norm:
        return ops.Prologue(**kw)
    qn, kn = self.q_norm, self.k_norm
    if not (isinstance(qn, nn.LayerNorm) and isinstance(kn, nn.LayerNorm) and tuple(qn.normalized_shape) == (D,)
            and tuple(kn.normalized_shape) == (D,) and qn.eps == kn.eps):
        return None
    params = (qn.weight, qn.bias, kn.weight, kn.bias)
    key = tuple(None if t is None else (t.data_ptr(), t._version, t.dtype, t.device) for t in params)
    cached = getattr(self, "_pma_norm_cache", None)
    if cached is None or cached[0] != key:
        dev = self.q_proj.weight.device
        ones = torch.ones(D, dtype=torch.float32, device=dev)
        f32 = [None if t is None else t.detach().to(torch.float32).contiguous() for t in params]
        f32[0] = ones if f32[0] is None else f32[0]  # elementwise_affine=False: unit weight
        f32[2] = ones if f32[2] is None else f32[2]
        cached = (key, f32)
        self._pma_norm_cache = cached
    w = cached[1]
    return ops.Prologue(q_norm_weight=w[0], q_norm_bias=w[1], k_norm_weight=w[2], k_norm_bias=w[3],
                        norm_eps=qn.eps, **kw)


def moment_forward(self, hidden_states: torch.Tensor, state: Optional[Tuple[torch.Tensor, ...]] = None,
                   return_state: bool = False):
    """PrimeMomentAttention.forward on the CUDA kernels.

    Uses only attributes the reference class defines (attention.py:56-75), so
    `install()` can bind it onto the reference class unchanged."""
    if torch.is_grad_enabled() and (hidden_states.requires_grad
                                    or any(p.requires_grad for p in self.parameters())):
        raise RuntimeError("prime_moment_attention_b200 kernels are inference-only: run under torch.no_grad() "
                           "or torch.inference_mode(), or uninstall() for training")
    B, L, _ = hidden_states.shape
    orig_dtype = hidden_states.dtype
    H, D = self.num_heads, self.head_dim

    q = self.q_proj(hidden_states).view(B, L, H, D).transpose(1, 2)
    k = self.k_proj(hidden_states).view(B, L, self.num_kv_heads, D).transpose(1, 2)
    v = self.v_proj(hidden_states).view(B, L, self.num_kv_heads, D).transpose(1, 2)
    pro = _prologue(self)
    if pro is None:  # norms the kernels do not fold: the reference's own sequence
        if self.num_kv_groups > 1:
            k = k.repeat_interleave(self.num_kv_groups, dim=1)
            v = v.repeat_interleave(self.num_kv_groups, dim=1)
        q = self.q_norm(q)
        k = self.k_norm(k)
        q = q * self.scaling
    if q.dtype not in (torch.float32, torch.bfloat16):
        q, k, v = q.float(), k.float(), v.float()

    decay = getattr(self, "decay_per_head", None)
    if decay is None:
        decay = self.decay
    if L == 1:
        if state is None:
            state = ops.new_state(B, H, D, hidden_states.device)
        y, next_state = ops.decode_step(q[:, :, 0], k[:, :, 0], v[:, :, 0], decay, state, eps=self.eps,
                                        out_dtype=orig_dtype if orig_dtype in (torch.float32, torch.bfloat16)
                                        else torch.float32, prologue=pro)
        y = y.to(orig_dtype).reshape(B, 1, H * D)
    else:
        out_dt = orig_dtype if orig_dtype in (torch.float32, torch.bfloat16) else torch.float32
        # write y straight into [B, L, H, D] so the o_proj input needs no transpose copy
        y_bl = torch.empty(B, L, H, D, dtype=out_dt, device=hidden_states.device)
        _, next_state = ops.prefill(q, k, v, decay, state=state, eps=self.eps, return_state=return_state,
                                    y_out=y_bl.transpose(1, 2), prologue=pro)
        y = y_bl.to(orig_dtype).view(B, L, H * D)
    output = self.o_proj(y)
    return output, (next_state if return_state else None)


class PrimeMomentAttention(nn.Module):
    """Drop-in for the reference PrimeMomentAttention (attention.py:42-75), same
    constructor and forward signature; forward runs on the CUDA kernels."""

    def __init__(self, hidden_size: int, num_heads: int, head_dim: int, num_kv_heads: Optional[int] = None,
                 decay: Union[float, Sequence[float], torch.Tensor] = 0.9995, use_qk_norm: bool = False,
                 eps: float = 1.0, chunk_size: int = 64, chunk_threshold: int = 512):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_kv_heads = num_kv_heads or num_heads
        self.num_kv_groups = num_heads // self.num_kv_heads
        if isinstance(decay, (int, float)):
            self.decay = float(decay)
            self.decay_per_head = None
        else:
            lam = torch.as_tensor(decay, dtype=torch.float32).reshape(-1)
            if lam.numel() != num_heads:
                raise ValueError("a per-head decay needs one value per head")
            self.decay = float(lam.mean())
            self.register_buffer("decay_per_head", lam, persistent=False)
        self.scaling = 1.0 / math.sqrt(head_dim)
        self.eps = eps
        self.use_qk_norm = use_qk_norm
        self.chunk_size = chunk_size
        self.chunk_threshold = chunk_threshold

        self.q_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.num_kv_heads * head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.num_kv_heads * head_dim, bias=False)
        self.o_proj = nn.Linear(num_heads * head_dim, hidden_size, bias=False)
        if self.use_qk_norm:
            self.q_norm = nn.LayerNorm(head_dim)
            self.k_norm = nn.LayerNorm(head_dim)

    def _apply(self, fn, recurse=True):
        # Module.to(bfloat16) / .half() would round the per-head decays (0.9995 -> 1.0 in
        # bf16); they stay float32 and only follow the device, like the reference's float decay.
        lam = self.decay_per_head
        super()._apply(fn, recurse)
        if lam is not None and self.decay_per_head.dtype != torch.float32:
            self.decay_per_head = lam.to(self.decay_per_head.device, torch.float32)
        return self

    forward = moment_forward
