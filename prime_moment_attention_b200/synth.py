"""Seeded synthetic inputs with the shapes and value laws of the benchmark configs.

The reference measures on no public dataset; every config draws its own inputs:
  * q, k, v ~ N(0, 1); q and k L2-normalised per head vector (QK-norm);
    q then scaled by 1/sqrt(D), as PrimeMomentAttention does before the core
    (src/prime_moment_attention/attention.py:101), so the core receives pre-scaled q.
  * per-head decay lambda_h log-uniform in [lo, hi]: exp(U(log lo, log hi)).
  * decode states: S/Z vectors and matrices ~ N(0, sigma) with sigma = 0.01, and
    Z0 = (1 - lambda^t) / (1 - lambda) at t = 4096 (the count a fresh state reaches
    after t tokens).
Generation uses torch.Generator on the target device, so a seed gives the same
values on every run of the same torch build.
"""
from __future__ import annotations

import math

import torch

# (B, H, L, D, chunk) of the prefill configs; decode is (sequences, layers, heads, D).
CONFIG1 = dict(B=1, H=12, L=2048, D=64, lam=(0.9995, 0.9995), dtype=torch.float32, seed=1)
CONFIG2 = dict(B=8, H=12, L=8192, D=64, lam=(0.99, 0.9999), dtype=torch.bfloat16, seed=2)
CONFIG3 = dict(seqs=256, layers=12, H=12, D=64, lam=(0.99, 0.9999), t0=4096, sigma=0.01, seed=3)
CONFIG5 = dict(B=1, H=16, L=1 << 20, D=128, lam=(0.999, 0.99995), dtype=torch.bfloat16, seed=5)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def make_qkv(B: int, H: int, L: int, D: int, seed: int, dtype=torch.float32, device="cpu",
             qk_norm: bool = True):
    """q, k, v [B,H,L,D] in `dtype`; q pre-scaled by 1/sqrt(D)."""
    g = _gen(seed, device)
    q = torch.randn(B, H, L, D, generator=g, device=device, dtype=torch.float32)
    k = torch.randn(B, H, L, D, generator=g, device=device, dtype=torch.float32)
    v = torch.randn(B, H, L, D, generator=g, device=device, dtype=torch.float32)
    if qk_norm:
        q = torch.nn.functional.normalize(q, dim=-1)
        k = torch.nn.functional.normalize(k, dim=-1)
    q = q * (1.0 / math.sqrt(D))
    return q.to(dtype), k.to(dtype), v.to(dtype)


def make_lambdas(n: int, lo: float, hi: float, seed: int, device="cpu") -> torch.Tensor:
    """n decays, log-uniform in [lo, hi], float32."""
    if lo == hi:
        return torch.full((n,), float(lo), dtype=torch.float32, device=device)
    g = _gen(seed + 7919, "cpu")
    u = torch.rand(n, generator=g, dtype=torch.float64)
    lam = torch.exp(math.log(lo) + u * (math.log(hi) - math.log(lo)))
    return lam.to(torch.float32).to(device)


def make_state(N: int, H: int, D: int, lam: torch.Tensor, seed: int, t0: int = 4096,
               sigma: float = 0.01, device="cpu"):
    """Resident decode state in the reference tuple layout, float32.

    lam is [H] (shared by all N) or [N,H]."""
    g = _gen(seed + 104729, device)
    S0 = sigma * torch.randn(N, H, D, generator=g, device=device)
    S1 = sigma * torch.randn(N, H, D, D, generator=g, device=device)
    S2 = sigma * torch.randn(N, H, D, D, generator=g, device=device)
    Z1 = sigma * torch.randn(N, H, D, generator=g, device=device)
    Z2 = sigma * torch.randn(N, H, D, generator=g, device=device)
    lam64 = lam.to(device=device, dtype=torch.float64)
    z0 = (1.0 - lam64 ** t0) / (1.0 - lam64)
    Z0 = z0.expand(N, H).reshape(N, H, 1).to(torch.float32).contiguous()
    return (S0, S1, S2, Z0, Z1, Z2)


def make_decode_tokens(N: int, H: int, D: int, seed: int, dtype=torch.bfloat16, device="cpu"):
    """One new token per head-state: q,k,v [N,H,D], QK-normed, q pre-scaled."""
    q, k, v = make_qkv(N, H, 1, D, seed, dtype=dtype, device=device)
    return q[:, :, 0], k[:, :, 0], v[:, :, 0]
