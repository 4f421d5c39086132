"""Host-side mirror of the reference's gated delta-rule module, running on libpma.so.

Mirrors ChunkedGatedDeltaPrimeAttention (src/prime_moment_attention/chunked_delta_prime.py:25-283)
with the same constructor, parameter names and forward signature.  The projections, the
erase / write gates, the GQA repeat, the LayerNorm QK-norm and the 1/sqrt(D) scale stay in
PyTorch exactly as the reference writes them (:101-137); the core goes to the CUDA kernels:
L == 1 to pma_delta_decode_step (the reference's step branch, :142-172) and L > 1 to
pma_delta_prefill (the chunked branch, :175-283, including its padding of a ragged last chunk
and its Lyapunov projection at chunk ends).  State: [B, H, D, 2D] float32, as the reference.
Inference only: the kernels have no backward.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import ops


def delta_forward(self, hidden_states: torch.Tensor, state: Optional[torch.Tensor] = None,
                  return_state: bool = False) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """ChunkedGatedDeltaPrimeAttention.forward on the CUDA kernels (attributes of the
    reference class only, so it can be bound onto the reference class)."""
    if torch.is_grad_enabled() and (hidden_states.requires_grad
                                    or any(p.requires_grad for p in self.parameters())):
        raise RuntimeError("prime_moment_attention_b200 kernels are inference-only: run under torch.no_grad() "
                           "or torch.inference_mode()")
    B, L, _ = hidden_states.shape
    dtype = hidden_states.dtype
    H, D, Hk = self.num_heads, self.head_dim, self.num_kv_heads

    q = self.q_proj(hidden_states).view(B, L, H, D).transpose(1, 2)
    k = self.k_proj(hidden_states).view(B, L, Hk, D).transpose(1, 2)
    v = self.v_proj(hidden_states).view(B, L, Hk, D).transpose(1, 2)
    b_gate = torch.sigmoid(self.erase_proj(hidden_states)).view(B, L, H, D).transpose(1, 2)
    w_gate = torch.sigmoid(self.write_proj(hidden_states)).view(B, L, H, D).transpose(1, 2)
    if self.num_kv_groups > 1:
        k = k.repeat_interleave(self.num_kv_groups, dim=1)
        v = v.repeat_interleave(self.num_kv_groups, dim=1)
    if self.use_qk_norm:
        q = self.q_norm(q)
        k = self.k_norm(k)
    q = q * self.scaling
    if q.dtype not in (torch.float32, torch.bfloat16):
        q, k, v = q.float(), k.float(), v.float()
    beta = w_gate.to(torch.float32).mean(dim=-1) * 0.5                        # [B, H, L]
    alpha = self.decay * (1.0 - b_gate.to(torch.float32).mean(dim=-1) * 0.5)  # [B, H, L]
    out_dt = dtype if dtype in (torch.float32, torch.bfloat16) else torch.float32

    if L == 1:
        S = state if state is not None else torch.zeros(B, H, D, 2 * D, device=hidden_states.device)
        y, S = ops.delta_decode_step(q[:, :, 0], k[:, :, 0], v[:, :, 0], beta[:, :, 0], alpha[:, :, 0], S,
                                     lyapunov_bound=self.lyapunov_bound, norm_eps=self.eps, out_dtype=out_dt)
        y = y.to(dtype).reshape(B, 1, H * D)
        return self.o_proj(y), (S if return_state else None)

    y_bl = torch.empty(B, L, H, D, dtype=out_dt, device=hidden_states.device)
    _, S = ops.delta_prefill(q, k, v, beta, alpha, self.decay, chunk=self.chunk_size,
                             lyapunov_bound=self.lyapunov_bound, norm_eps=self.eps, state=state,
                             return_state=return_state, y_out=y_bl.transpose(1, 2))
    y = y_bl.to(dtype).view(B, L, H * D)
    return self.o_proj(y), (S if return_state else None)


class ChunkedGatedDeltaPrimeAttention(nn.Module):
    """Drop-in for the reference ChunkedGatedDeltaPrimeAttention (chunked_delta_prime.py:25-71):
    same constructor, parameters and initial gate biases; forward runs on the CUDA kernels.
    The kernels build chunk sizes 32 and 64 and head dims 16, 32 and 64."""

    def __init__(self, hidden_size: int, num_heads: int, head_dim: int, num_kv_heads: Optional[int] = None,
                 chunk_size: int = 64, decay: float = 0.9995, use_qk_norm: bool = True,
                 lyapunov_bound: float = 25.0, eps: float = 1e-5):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_kv_heads = num_kv_heads or num_heads
        self.num_kv_groups = num_heads // self.num_kv_heads
        self.chunk_size = chunk_size
        self.decay = decay
        self.scaling = 1.0 / math.sqrt(head_dim)
        self.use_qk_norm = use_qk_norm
        self.lyapunov_bound = lyapunov_bound
        self.eps = eps
        self.q_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.num_kv_heads * head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.num_kv_heads * head_dim, bias=False)
        self.o_proj = nn.Linear(num_heads * head_dim, hidden_size, bias=False)
        self.erase_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=True)
        self.write_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=True)
        if self.use_qk_norm:
            self.q_norm = nn.LayerNorm(head_dim)
            self.k_norm = nn.LayerNorm(head_dim)
        with torch.no_grad():  # the reference's initial gate biases (chunked_delta_prime.py:67-71)
            self.erase_proj.bias.fill_(-2.5)
            self.write_proj.bias.fill_(-1.0)

    forward = delta_forward
