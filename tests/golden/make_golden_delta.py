"""Golden vectors for the gated delta-rule variant, from the reference's own module.

Run where the PRIME-Moment-Attention reference is importable:

    python tests/golden/make_golden_delta.py --ref-src <reference>/src

It drives ChunkedGatedDeltaPrimeAttention (src/prime_moment_attention/chunked_delta_prime.py:25-283)
as an nn.Module in float32 on the CPU and writes small .npz fixtures next to this file.  The
fixtures are committed; the tests read them and never import the reference.

Identity projections make the module's inputs the core's inputs.  The hidden vector of a token
is [q_raw | k | v | g_write | g_erase] (sizes D, D, D, 1, 1 for one head); q_proj, k_proj,
v_proj select the first three blocks, write_proj / erase_proj copy g_write / g_erase into all
D channels of the head (bias 0), o_proj returns y.  The module then computes exactly
(chunked_delta_prime.py:106-137):
    q      = q_raw * 1/sqrt(D)              (no QK-norm)
    beta_t = 0.5 * mean_d sigmoid(g_write)  = 0.5 * sigmoid(g_write)
    alpha_t = decay * (1 - 0.5 * sigmoid(g_erase))
which the fixtures store (as the module's float32 values) next to the raw inputs.  Heads are
independent; per-head decays come from one module per head slice (the module takes one scalar).

Cases:
  delta_c32_d16     L = 75 with chunk 32 (ragged: 21 padded tokens), bound 3 (the Lyapunov
                    clamp is active), no incoming state, B = 2, two heads.
  delta_c64_d32_st  L = 150 with chunk 64, incoming state, bound 25.
  delta_c64_d64     L = 128 (whole chunks), bound 25, no state.
  delta_step_d32    the L == 1 branch (chunked_delta_prime.py:142-172): 3 steps from a random
                    state, bound 5.
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _module(Attn, D, C, lam, bound):
    hid = 3 * D + 2
    m = Attn(hidden_size=hid, num_heads=1, head_dim=D, chunk_size=C, decay=float(lam), use_qk_norm=False,
             lyapunov_bound=float(bound), eps=1e-5)
    with torch.no_grad():
        eye, z = torch.eye(D), torch.zeros(D, D)
        zc = torch.zeros(D, 2)
        m.q_proj.weight.copy_(torch.cat([eye, z, z, zc], dim=1))
        m.k_proj.weight.copy_(torch.cat([z, eye, z, zc], dim=1))
        m.v_proj.weight.copy_(torch.cat([z, z, eye, zc], dim=1))
        w = torch.zeros(D, hid)
        w[:, 3 * D] = 1.0
        m.write_proj.weight.copy_(w)
        m.write_proj.bias.zero_()
        e = torch.zeros(D, hid)
        e[:, 3 * D + 1] = 1.0
        m.erase_proj.weight.copy_(e)
        m.erase_proj.bias.zero_()
        m.o_proj.weight.copy_(torch.cat([eye, torch.zeros(hid - D, D)], dim=0))
    return m


def _gates(gw, ge, lam, D):
    """beta, alpha as the module computes them (float32, chunked_delta_prime.py:107-137)."""
    w = torch.sigmoid(gw.unsqueeze(-1).expand(*gw.shape, D).contiguous())
    b = torch.sigmoid(ge.unsqueeze(-1).expand(*ge.shape, D).contiguous())
    beta = w.mean(dim=-1) * 0.5
    alpha = float(lam) * (1.0 - b.mean(dim=-1) * 0.5)
    return beta, alpha


def run(Attn, q_raw, k, v, gw, ge, lams, C, bound, state=None):
    """Per head slice.  Inputs [B,H,L,D] / gates [B,H,L]; state [B,H,D,2D] or None.
    Returns q (scaled), beta, alpha, y, final state."""
    B, H, L, D = q_raw.shape
    ys, sts, qs, betas, alphas = [], [], [], [], []
    for h in range(H):
        m = _module(Attn, D, C, lams[h], bound)
        f = lambda t: t[:, h].reshape(B, L, -1)
        hs = torch.cat([f(q_raw), f(k), f(v), gw[:, h].unsqueeze(-1), ge[:, h].unsqueeze(-1)], dim=-1)
        st_h = None if state is None else state[:, h:h + 1].contiguous()
        with torch.no_grad():
            out, st = m(hs, state=st_h, return_state=True)
        ys.append(out[..., :D].reshape(B, L, 1, D).transpose(1, 2))
        sts.append(st)
        qs.append(q_raw[:, h:h + 1] * m.scaling)
        be, al = _gates(gw[:, h], ge[:, h], lams[h], D)
        betas.append(be.unsqueeze(1))
        alphas.append(al.unsqueeze(1))
    return (torch.cat(qs, 1), torch.cat(betas, 1), torch.cat(alphas, 1), torch.cat(ys, 1), torch.cat(sts, 1))


def _inputs(B, H, L, D, seed, gw_mu=0.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, D, generator=g), dim=-1)
    k = torch.randn(B, H, L, D, generator=g)
    v = torch.randn(B, H, L, D, generator=g)
    gw = torch.randn(B, H, L, generator=g) + gw_mu
    ge = torch.randn(B, H, L, generator=g) - 1.5
    return q, k, v, gw, ge


def save(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **{k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v))
                                 for k, v in arrays.items()})
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("PRIME_REF_SRC"),
                    help="the reference project's src/ directory (default: $PRIME_REF_SRC)")
    args = ap.parse_args()
    if not args.ref_src:
        ap.error("pass --ref-src <reference>/src or set PRIME_REF_SRC")
    sys.path.insert(0, args.ref_src)
    sys.dont_write_bytecode = True
    from prime_moment_attention.chunked_delta_prime import ChunkedGatedDeltaPrimeAttention as Attn
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    cases = [
        ("delta_c32_d16", dict(B=2, H=2, L=75, D=16, C=32, bound=3.0, lams=[0.999, 0.99], seed=31, state=False)),
        ("delta_c64_d32_st", dict(B=1, H=2, L=150, D=32, C=64, bound=25.0, lams=[0.9995, 0.995], seed=32,
                                  state=True)),
        ("delta_c64_d64", dict(B=1, H=1, L=128, D=64, C=64, bound=25.0, lams=[0.999], seed=33, state=False)),
    ]
    for name, c in cases:
        q_raw, k, v, gw, ge = _inputs(c["B"], c["H"], c["L"], c["D"], c["seed"])
        st0 = None
        if c["state"]:
            g = torch.Generator().manual_seed(c["seed"] + 100)
            st0 = torch.randn(c["B"], c["H"], c["D"], 2 * c["D"], generator=g) * 0.1
        q, beta, alpha, y, st = run(Attn, q_raw, k, v, gw, ge, c["lams"], c["C"], c["bound"], st0)
        extra = {"state_in": st0} if st0 is not None else {}
        save(name, q=q, k=k, v=v, beta=beta, alpha=alpha, lam=np.asarray(c["lams"], np.float32), chunk=c["C"],
             bound=c["bound"], y=y, state=st, **extra)

    # L == 1 branch, three steps
    B, H, D, steps, bound = 2, 2, 32, 3, 5.0
    lams = [0.999, 0.98]
    q_raw, k, v, gw, ge = _inputs(B, H, steps, D, 34)
    g = torch.Generator().manual_seed(134)
    st0 = torch.randn(B, H, D, 2 * D, generator=g) * 0.3
    st = st0
    ys, qs, betas, alphas = [], [], [], []
    for t in range(steps):
        sl = slice(t, t + 1)
        q, be, al, y, st = run(Attn, q_raw[:, :, sl], k[:, :, sl], v[:, :, sl], gw[:, :, sl], ge[:, :, sl], lams,
                               64, bound, st)
        ys.append(y)
        qs.append(q)
        betas.append(be)
        alphas.append(al)
    save("delta_step_d32", q=torch.cat(qs, 2), k=k, v=v, beta=torch.cat(betas, 2), alpha=torch.cat(alphas, 2),
         lam=np.asarray(lams, np.float32), bound=bound, y=torch.cat(ys, 2), state_in=st0, state=st)

    with open(os.path.join(HERE, "PROVENANCE_delta.txt"), "w") as f:
        f.write("Golden vectors written by tests/golden/make_golden_delta.py from the reference's own code:\n")
        f.write("  src/prime_moment_attention/chunked_delta_prime.py (ChunkedGatedDeltaPrimeAttention.forward)\n")
        f.write(f"torch {torch.__version__}, numpy {np.__version__}, float32 CPU\n")


if __name__ == "__main__":
    main()
