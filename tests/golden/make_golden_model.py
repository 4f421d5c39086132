"""Golden vectors for the model-level caller, from the reference's own PrimeForCausalLM.

Run where the PRIME-Moment-Attention reference is importable:

    python tests/golden/make_golden_model.py --ref-src <reference>/src

Builds a small reference PrimeForCausalLM (src/prime_moment_attention/model.py:120-244) in
float32 on the CPU from a fixed seed, with non-trivial norm parameters and grouped kv heads, and
writes model_small.npz: the state_dict (the names prime_moment_attention_b200.model must load),
logits of a 40-token batch (the module's dense branch) and the last 8 positions of a 600-token
sequence (its chunked branch), and 6 greedy tokens of generate() (the decode branch with state).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
CFG = dict(vocab_size=97, hidden_size=64, num_layers=2, num_heads=2, head_dim=32, num_kv_heads=1,
           intermediate_size=96, decay=0.999, use_qk_norm=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("PRIME_REF_SRC"),
                    help="the reference project's src/ directory (default: $PRIME_REF_SRC)")
    args = ap.parse_args()
    if not args.ref_src:
        ap.error("pass --ref-src <reference>/src or set PRIME_REF_SRC")
    sys.path.insert(0, args.ref_src)
    sys.dont_write_bytecode = True
    from prime_moment_attention.model import PrimeConfig, PrimeForCausalLM
    torch.manual_seed(40)
    m = PrimeForCausalLM(PrimeConfig(**CFG)).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" in n:  # RMSNorm and LayerNorm weights / biases away from their defaults
                p.copy_(torch.rand_like(p) + 0.5 if n.endswith("weight") else torch.randn_like(p) * 0.1)
    g = torch.Generator().manual_seed(41)
    ids = torch.randint(0, CFG["vocab_size"], (2, 40), generator=g)
    ids_long = torch.randint(0, CFG["vocab_size"], (1, 600), generator=g)
    with torch.no_grad():
        logits = m(ids)["logits"]
        logits_long = m(ids_long)["logits"][:, -8:]
        gen = m.generate(ids[:, :12], max_new_tokens=6, temperature=0.0)
    sd = {f"p::{k}": v.detach().numpy() for k, v in m.state_dict().items()}
    path = os.path.join(HERE, "model_small.npz")
    np.savez_compressed(path, ids=ids.numpy(), ids_long=ids_long.numpy(), logits=logits.numpy(),
                        logits_long_last8=logits_long.numpy(), generated=gen.numpy(),
                        cfg=np.array(repr(CFG)), **sd)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")
    with open(os.path.join(HERE, "PROVENANCE_model.txt"), "w") as f:
        f.write("model_small.npz written by tests/golden/make_golden_model.py from the reference's own\n")
        f.write("src/prime_moment_attention/model.py (PrimeForCausalLM forward and generate), float32 CPU,\n")
        f.write(f"torch {torch.__version__}\n")


if __name__ == "__main__":
    main()
