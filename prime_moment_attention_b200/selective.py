"""Host-side mirror of the reference's selective moment attention, running on libpma.so.

Mirrors PrimeSelectiveMomentAttention (src/prime_moment_attention/selective.py:264-444): same
constructor, parameters (delta_proj, log_tau, log_beta) and identity-preserving initialisation.
The projections and the step size Delta_t = clamp(softplus(delta_proj(x)), 1e-4, 50) stay in
PyTorch; the GQA repeat, QK-norm and q scale run in the kernels' prologue; the core runs on
pma_selective_prefill (L > 1) and pma_selective_decode_step (L == 1) with
lambda_t = exp(-Delta_t / tau_h) and k scaled by beta_h.  States keep the reference's selective
tuple layout.  One deliberate difference: with an incoming state and L > 1 the reference's
parallel branch (:401-435) drops the state; here the prefill carries it, as the reference's step
branch does token by token.  Inference only.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .attention import _prologue


def selective_forward(self, hidden_states: torch.Tensor, state: Optional[Tuple[torch.Tensor, ...]] = None,
                      return_state: bool = False):
    """PrimeSelectiveMomentAttention.forward on the CUDA kernels (reference attributes only)."""
    if torch.is_grad_enabled() and (hidden_states.requires_grad
                                    or any(p.requires_grad for p in self.parameters())):
        raise RuntimeError("prime_moment_attention_b200 kernels are inference-only: run under torch.no_grad() "
                           "or torch.inference_mode()")
    B, L, _ = hidden_states.shape
    orig_dtype = hidden_states.dtype
    dev = hidden_states.device
    H, D, Hk = self.num_heads, self.head_dim, self.num_kv_heads
    q = self.q_proj(hidden_states).view(B, L, H, D).transpose(1, 2)
    k = self.k_proj(hidden_states).view(B, L, Hk, D).transpose(1, 2)
    v = self.v_proj(hidden_states).view(B, L, Hk, D).transpose(1, 2)
    pro = _prologue(self)
    if pro is None:
        if self.num_kv_groups > 1:
            k = k.repeat_interleave(self.num_kv_groups, dim=1)
            v = v.repeat_interleave(self.num_kv_groups, dim=1)
        q = self.q_norm(q)
        k = self.k_norm(k)
        q = q * self.scaling
    if q.dtype not in (torch.float32, torch.bfloat16):
        q, k, v = q.float(), k.float(), v.float()
    tau = self.get_tau(dev)
    beta = self.get_beta(dev).float()
    delta = F.softplus(self.delta_proj(hidden_states)).clamp(min=1e-4, max=50.0)  # [B, L, H]
    log_decay = (-delta.float() / tau.view(1, 1, H)).transpose(1, 2)              # [B, H, L]
    out_dt = orig_dtype if orig_dtype in (torch.float32, torch.bfloat16) else torch.float32
    if L == 1:
        if state is None:
            state = ops.new_state(B, H, D, dev)
        y, next_state = ops.selective_decode_step(q[:, :, 0], k[:, :, 0], v[:, :, 0], log_decay[:, :, 0], beta,
                                                  state, eps=self.eps, out_dtype=out_dt, prologue=pro)
        y = y.to(orig_dtype).reshape(B, 1, H * D)
    else:
        y_bl = torch.empty(B, L, H, D, dtype=out_dt, device=dev)
        _, next_state = ops.selective_prefill(q, k, v, log_decay, beta, state=state, eps=self.eps,
                                              return_state=return_state, y_out=y_bl.transpose(1, 2),
                                              prologue=pro)
        y = y_bl.to(orig_dtype).view(B, L, H * D)
    return self.o_proj(y), (next_state if return_state else None)


class PrimeSelectiveMomentAttention(nn.Module):
    """Drop-in for the reference PrimeSelectiveMomentAttention (selective.py:264-354)."""

    def __init__(self, hidden_size: int, num_heads: int, head_dim: int, num_kv_heads: Optional[int] = None,
                 decay: float = 0.995, use_qk_norm: bool = True, eps: float = 1.0, min_tau: float = 2.0,
                 max_tau: float = 2000.0):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_kv_heads = num_kv_heads or num_heads
        self.num_kv_groups = num_heads // self.num_kv_heads
        self.decay = decay
        self.scaling = 1.0 / math.sqrt(head_dim)
        self.eps = eps
        self.use_qk_norm = use_qk_norm
        self.min_tau = min_tau
        self.max_tau = max_tau
        self.q_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.num_kv_heads * head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.num_kv_heads * head_dim, bias=False)
        self.o_proj = nn.Linear(num_heads * head_dim, hidden_size, bias=False)
        if self.use_qk_norm:
            self.q_norm = nn.LayerNorm(head_dim)
            self.k_norm = nn.LayerNorm(head_dim)
        self.delta_proj = nn.Linear(hidden_size, num_heads, bias=True)
        base_tau = -1.0 / math.log(max(1e-5, min(0.9999, decay)))
        self.log_tau = nn.Parameter(torch.full((num_heads,), math.log(base_tau), dtype=torch.float32))
        self.log_beta = nn.Parameter(torch.zeros(num_heads, dtype=torch.float32))
        self.init_selective_weights()

    def init_selective_weights(self):
        """Delta_t = softplus(bias) = 1 and beta = 1: the base moment attention with decay `decay`."""
        with torch.no_grad():
            self.delta_proj.weight.zero_()
            self.delta_proj.bias.fill_(math.log(math.exp(1.0) - 1.0))
            self.log_tau.fill_(math.log(-1.0 / math.log(max(1e-5, min(0.9999, self.decay)))))
            self.log_beta.zero_()

    def get_tau(self, device: torch.device) -> torch.Tensor:
        return torch.clamp(torch.exp(self.log_tau.to(device)), min=self.min_tau, max=self.max_tau)

    def get_beta(self, device: torch.device) -> torch.Tensor:
        return torch.clamp(torch.exp(self.log_beta.to(device)), min=0.1, max=15.0)

    forward = selective_forward
