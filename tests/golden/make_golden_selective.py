"""Golden vectors for the selective variant, from the reference's own module.

Run where the PRIME-Moment-Attention reference is importable:

    python tests/golden/make_golden_selective.py --ref-src <reference>/src

Drives PrimeSelectiveMomentAttention (src/prime_moment_attention/selective.py:264-444) as an
nn.Module in float32 on the CPU with identity projections: a token's hidden vector is
[q_raw | k | v | g] (g has one entry per head); q_proj / k_proj / v_proj select the first three
blocks, delta_proj selects g (bias 0), o_proj returns y.  The module then uses
    Delta_t = clamp(softplus(g_t), 1e-4, 50),  lambda_t = exp(-Delta_t / tau_h),
    beta_h = clamp(exp(log_beta_h), 0.1, 15),  tau_h = clamp(exp(log_tau_h), min_tau, max_tau)
(:341-359), which the fixtures store next to the inputs as log_decay = -Delta / tau and beta.

Cases:
  selective_par_d32   the parallel branch (L > 1, :401-435), no incoming state, B = 2, 3 heads
                      with different tau and beta, L = 70; y and the returned state.
  selective_step_d16  the step branch (L == 1, :367-396): 4 steps from a random state.
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _module(Attn, D, tau, log_beta):
    hid = 3 * D + 1
    m = Attn(hidden_size=hid, num_heads=1, head_dim=D, use_qk_norm=False, eps=1.0)
    with torch.no_grad():
        eye, z = torch.eye(D), torch.zeros(D, D)
        zc = torch.zeros(D, 1)
        m.q_proj.weight.copy_(torch.cat([eye, z, z, zc], dim=1))
        m.k_proj.weight.copy_(torch.cat([z, eye, z, zc], dim=1))
        m.v_proj.weight.copy_(torch.cat([z, z, eye, zc], dim=1))
        w = torch.zeros(1, hid)
        w[0, 3 * D] = 1.0
        m.delta_proj.weight.copy_(w)
        m.delta_proj.bias.zero_()
        m.log_tau.fill_(math.log(tau))
        m.log_beta.fill_(log_beta)
        m.o_proj.weight.copy_(torch.cat([eye, torch.zeros(hid - D, D)], dim=0))
    return m


def run(Attn, q_raw, k, v, g, taus, log_betas, state=None):
    """Per head slice; inputs [B,H,L,D], g [B,H,L]; state: reference tuple or None."""
    B, H, L, D = q_raw.shape
    ys, sts, qs, lds, bts = [], [], [], [], []
    for h in range(H):
        m = _module(Attn, D, taus[h], log_betas[h])
        f = lambda t: t[:, h].reshape(B, L, -1)
        hs = torch.cat([f(q_raw), f(k), f(v), g[:, h].unsqueeze(-1)], dim=-1)
        st_h = None if state is None else tuple(s[:, h:h + 1].contiguous() for s in state)
        with torch.no_grad():
            out, st = m(hs, state=st_h, return_state=True)
            tau = m.get_tau(torch.device("cpu"))
            delta = F.softplus(m.delta_proj(hs)).clamp(min=1e-4, max=50.0)  # [B, L, 1]
            lds.append((-delta / tau.view(1, 1, 1)).permute(0, 2, 1))       # [B, 1, L]
            bts.append(m.get_beta(torch.device("cpu")))
        ys.append(out[..., :D].reshape(B, L, 1, D).transpose(1, 2))
        sts.append(st)
        qs.append(q_raw[:, h:h + 1] * m.scaling)
    st = tuple(torch.cat([s[i] for s in sts], dim=1) for i in range(6))
    return torch.cat(qs, 1), torch.cat(lds, 1), torch.cat(bts), torch.cat(ys, 1), st


def save(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **{k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v))
                                 for k, v in arrays.items()})
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


def state_dict(prefix, st):
    return {f"{prefix}{n}": s for n, s in zip(("S0", "S1", "S2", "K0", "K1", "K2"), st)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("PRIME_REF_SRC"),
                    help="the reference project's src/ directory (default: $PRIME_REF_SRC)")
    args = ap.parse_args()
    if not args.ref_src:
        ap.error("pass --ref-src <reference>/src or set PRIME_REF_SRC")
    sys.path.insert(0, args.ref_src)
    sys.dont_write_bytecode = True
    from prime_moment_attention.selective import PrimeSelectiveMomentAttention as Attn
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    gen = torch.Generator().manual_seed(51)
    B, H, L, D = 2, 3, 70, 32
    q_raw = F.normalize(torch.randn(B, H, L, D, generator=gen), dim=-1)
    k = F.normalize(torch.randn(B, H, L, D, generator=gen), dim=-1)
    v = torch.randn(B, H, L, D, generator=gen)
    g = torch.randn(B, H, L, generator=gen) - 1.0
    taus, log_betas = [200.0, 20.0, 5.0], [0.0, 0.5, -0.4]
    q, ld, bt, y, st = run(Attn, q_raw, k, v, g, taus, log_betas)
    save("selective_par_d32", q=q, k=k, v=v, log_decay=ld, beta=bt, y=y, **state_dict("st_", st))

    B, H, D, steps = 2, 2, 16, 4
    q_raw = F.normalize(torch.randn(B, H, steps, D, generator=gen), dim=-1)
    k = F.normalize(torch.randn(B, H, steps, D, generator=gen), dim=-1)
    v = torch.randn(B, H, steps, D, generator=gen)
    g = torch.randn(B, H, steps, generator=gen)
    taus, log_betas = [50.0, 8.0], [0.3, -0.2]
    st0 = tuple(torch.randn(B, H, *s, generator=gen) * 0.1 for s in [(D,), (D, D), (D, D), (1,), (D,), (D,)])
    st0 = (st0[0], st0[1], st0[2], st0[3].abs() + 3.0, st0[4], st0[5])
    st = st0
    qs, lds, ys = [], [], []
    for t in range(steps):
        sl = slice(t, t + 1)
        q, ld, bt, y, st = run(Attn, q_raw[:, :, sl], k[:, :, sl], v[:, :, sl], g[:, :, sl], taus, log_betas, st)
        qs.append(q)
        lds.append(ld)
        ys.append(y)
    save("selective_step_d16", q=torch.cat(qs, 2), k=k, v=v, log_decay=torch.cat(lds, 2), beta=bt,
         y=torch.cat(ys, 2), **state_dict("in_", st0), **state_dict("st_", st))

    with open(os.path.join(HERE, "PROVENANCE_selective.txt"), "w") as f:
        f.write("Golden vectors written by tests/golden/make_golden_selective.py from the reference's own code:\n")
        f.write("  src/prime_moment_attention/selective.py (PrimeSelectiveMomentAttention.forward)\n")
        f.write(f"torch {torch.__version__}, numpy {np.__version__}, float32 CPU\n")


if __name__ == "__main__":
    main()
