"""Generate the golden input/output vectors from the reference's own PyTorch code.

Run in a checkout where the PRIME-Moment-Attention reference is importable
(its `src/` directory on PYTHONPATH, or --ref-src):

    python tests/golden/make_golden.py --ref-src <reference>/src

It imports the reference modules, runs them on seeded inputs, and writes small
.npz fixtures next to this file.  The fixtures are committed; the tests read them
and never import the reference, which is absent where the GPU tests run.

Cases (each cites the reference code that produced its outputs):
  chunk_*    chunked_prime_ssd_core (src/prime_moment_attention/chunked_ssd.py:48-184),
             chunk_size 64, return_state=True, no incoming state.  Per-head decay is
             produced by calling the core once per head slice (heads are independent;
             the reference takes one scalar decay, chunked_ssd.py:53).
  dense_*    PrimeMomentAttention.forward dense branch, 1 < L <= 512
             (src/prime_moment_attention/attention.py:160-202), state=None.
  decode_*   PrimeMomentAttention.forward decode branch, L == 1
             (attention.py:120-143), stepping a random incoming state.
  config1    the full config-1 shape (B=1, H=12, L=2048, D=64, lambda 0.9995) through
             the chunked core; stores checksums of the inputs and sampled outputs
             plus the complete final state of two heads (the full outputs would be
             tens of MB).

Module cases drive the real nn.Module with identity projections: hidden size
3*H*D, q_proj/k_proj/v_proj select the q, k and v blocks, o_proj returns y.
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from prime_moment_attention_b200 import synth  # noqa: E402


def _np(t):
    return t.detach().cpu().numpy()


def ref_chunked(core, q, k, v, lams, chunk=64):
    """Reference chunked core per head slice; returns y and state in tuple layout."""
    ys, states = [], []
    for h in range(q.shape[1]):
        y, st = core(q[:, h:h + 1].contiguous(), k[:, h:h + 1].contiguous(), v[:, h:h + 1].contiguous(),
                     state=None, decay=float(lams[h]), eps=1.0, chunk_size=chunk, return_state=True)
        ys.append(y)
        states.append(st)
    y = torch.cat(ys, dim=1)
    st = tuple(torch.cat([s[i] for s in states], dim=1) for i in range(6))
    return y, st


def _identity_module(Attn, H, D, lam, L_branch_threshold=512):
    HD = H * D
    m = Attn(hidden_size=3 * HD, num_heads=H, head_dim=D, decay=float(lam), use_qk_norm=False,
             eps=1.0, chunk_size=64, chunk_threshold=L_branch_threshold)
    with torch.no_grad():
        eye = torch.eye(HD)
        z = torch.zeros(HD, HD)
        m.q_proj.weight.copy_(torch.cat([eye, z, z], dim=1))
        m.k_proj.weight.copy_(torch.cat([z, eye, z], dim=1))
        m.v_proj.weight.copy_(torch.cat([z, z, eye], dim=1))
        m.o_proj.weight.copy_(torch.cat([eye, z, z], dim=0))
    return m


def _hidden(q_raw, k, v):
    """[B,H,L,D] x3 -> hidden [B,L,3*H*D] so the identity projections recover them."""
    B, H, L, D = q_raw.shape
    f = lambda t: t.transpose(1, 2).reshape(B, L, H * D)
    return torch.cat([f(q_raw), f(k), f(v)], dim=-1)


def ref_module(Attn, q_raw, k, v, lams, state=None):
    """Module forward per head slice.  q_raw is NOT pre-scaled; the module scales it.

    Returns (q_scaled as the module computed it, y [B,H,L,D], state)."""
    B, H, L, D = q_raw.shape
    ys, sts, qs = [], [], []
    for h in range(H):
        m = _identity_module(Attn, 1, D, lams[h])
        hs = _hidden(q_raw[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1])
        st_h = None if state is None else tuple(s[:, h:h + 1].contiguous() for s in state)
        with torch.no_grad():
            out, st = m(hs, state=st_h, return_state=True)
        ys.append(out[..., :D].reshape(B, L, 1, D).transpose(1, 2))
        sts.append(st)
        qs.append(q_raw[:, h:h + 1] * m.scaling)
    y = torch.cat(ys, dim=1)
    st = tuple(torch.cat([s[i] for s in sts], dim=1) for i in range(6))
    return torch.cat(qs, dim=1), y, st


def save(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **{k: (np.asarray(v) if not torch.is_tensor(v) else _np(v)) for k, v in arrays.items()})
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


def state_dict(prefix, st):
    names = ("S0", "S1", "S2", "K0", "K1", "K2")
    return {f"{prefix}{n}": s for n, s in zip(names, st)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("PRIME_REF_SRC"),
                    help="the reference project's src/ directory (default: $PRIME_REF_SRC)")
    args = ap.parse_args()
    if not args.ref_src:
        ap.error("pass --ref-src <reference>/src or set PRIME_REF_SRC")
    sys.path.insert(0, args.ref_src)
    sys.dont_write_bytecode = True
    from prime_moment_attention.attention import PrimeMomentAttention
    from prime_moment_attention.chunked_ssd import chunked_prime_ssd_core

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # --- chunked core: ragged L, several decays, D=32 --------------------------------
    q, k, v = synth.make_qkv(1, 3, 200, 32, seed=11)
    lams = np.array([0.9995, 0.99, 0.9], dtype=np.float32)
    y, st = ref_chunked(chunked_prime_ssd_core, q, k, v, lams)
    save("chunk_ragged_d32", q=q, k=k, v=v, lam=lams, y=y, **state_dict("st_", st))

    # --- chunked core: D=64, two chunks + 2 tokens, log-uniform decays -----------------
    q, k, v = synth.make_qkv(1, 2, 130, 64, seed=12)
    lams = synth.make_lambdas(2, 0.99, 0.9999, seed=12).numpy()
    y, st = ref_chunked(chunked_prime_ssd_core, q, k, v, lams)
    save("chunk_d64", q=q, k=k, v=v, lam=lams, y=y, **state_dict("st_", st))

    # --- chunked core: inputs rounded to bf16 then cast to fp32 (what the module does) --
    qb, kb, vb = synth.make_qkv(2, 2, 96, 64, seed=13, dtype=torch.bfloat16)
    lams = np.array([0.999, 0.995], dtype=np.float32)
    y, st = ref_chunked(chunked_prime_ssd_core, qb.float(), kb.float(), vb.float(), lams)
    save("chunk_bf16in_d64", q=qb.float(), k=kb.float(), v=vb.float(), lam=lams, y=y, **state_dict("st_", st))

    # --- chunked core: L shorter than one chunk, and L == 1 ----------------------------
    q, k, v = synth.make_qkv(1, 2, 37, 16, seed=14)
    lams = np.array([0.98, 0.9995], dtype=np.float32)
    y, st = ref_chunked(chunked_prime_ssd_core, q, k, v, lams)
    save("chunk_short_d16", q=q, k=k, v=v, lam=lams, y=y, **state_dict("st_", st))
    q, k, v = synth.make_qkv(2, 2, 1, 16, seed=15)
    y, st = ref_chunked(chunked_prime_ssd_core, q, k, v, lams)
    save("chunk_len1_d16", q=q, k=k, v=v, lam=lams, y=y, **state_dict("st_", st))

    # --- module dense branch (L <= 512), no state ---------------------------------------
    g = torch.Generator().manual_seed(16)
    B, H, L, D = 1, 2, 96, 32
    q_raw = torch.nn.functional.normalize(torch.randn(B, H, L, D, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, H, L, D, generator=g), dim=-1)
    v = torch.randn(B, H, L, D, generator=g)
    lams = np.array([0.9995, 0.99], dtype=np.float32)
    qs, y, st = ref_module(PrimeMomentAttention, q_raw, k, v, lams)
    save("dense_d32", q=qs, k=k, v=v, lam=lams, y=y, **state_dict("st_", st))

    # --- module decode branch: 4 steps from a random incoming state ---------------------
    N, H, D, steps = 2, 3, 32, 4
    lams = np.array([0.9995, 0.99, 0.95], dtype=np.float32)
    st0 = synth.make_state(N, H, D, torch.from_numpy(lams), seed=17, t0=64, sigma=0.05)
    g = torch.Generator().manual_seed(17)
    q_raw = torch.nn.functional.normalize(torch.randn(N, H, steps, D, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(N, H, steps, D, generator=g), dim=-1)
    v = torch.randn(N, H, steps, D, generator=g)
    st = st0
    ys, qss = [], []
    for t in range(steps):
        qs, y, st = ref_module(PrimeMomentAttention, q_raw[:, :, t:t + 1], k[:, :, t:t + 1], v[:, :, t:t + 1], lams, st)
        ys.append(y)
        qss.append(qs)
    save("decode_d32", q=torch.cat(qss, dim=2), k=k, v=v, lam=lams, y=torch.cat(ys, dim=2),
         **state_dict("in_", st0), **state_dict("st_", st))

    # --- config 1 full shape, summarised ------------------------------------------------
    c = synth.CONFIG1
    q, k, v = synth.make_qkv(c["B"], c["H"], c["L"], c["D"], seed=c["seed"], dtype=c["dtype"])
    lams = np.full(c["H"], c["lam"][0], dtype=np.float32)
    y, st = ref_chunked(chunked_prime_ssd_core, q, k, v, lams)
    rng = np.random.default_rng(101)
    idx = np.stack([rng.integers(0, n, size=4096) for n in y.shape], axis=1)
    yn = _np(y)
    save("config1_summary", lam=lams,
         in_sums=np.array([float(t.double().sum()) for t in (q, k, v)]),
         in_abs=np.array([float(t.double().abs().sum()) for t in (q, k, v)]),
         y_idx=idx, y_samples=yn[tuple(idx.T)],
         y_sum=float(yn.astype(np.float64).sum()), y_abs=float(np.abs(yn).astype(np.float64).sum()),
         y_max=float(np.abs(yn).max()),
         **{f"st_{n}_h0_h7": _np(s[:, [0, 7]]) for n, s in zip(("S0", "S1", "S2", "K0", "K1", "K2"), st)},
         **{f"st_{n}_absmax": float(s.abs().max()) for n, s in zip(("S0", "S1", "S2", "K0", "K1", "K2"), st)})

    with open(os.path.join(HERE, "PROVENANCE.txt"), "w") as f:
        f.write("Golden vectors written by tests/golden/make_golden.py from the reference's own code:\n")
        f.write("  src/prime_moment_attention/chunked_ssd.py (chunked_prime_ssd_core)\n")
        f.write("  src/prime_moment_attention/attention.py (PrimeMomentAttention.forward)\n")
        f.write(f"torch {torch.__version__}, numpy {np.__version__}, float32 CPU, {torch.get_num_threads()} threads\n")


if __name__ == "__main__":
    main()
