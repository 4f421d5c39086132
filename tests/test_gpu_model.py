"""Model-level caller (prime_moment_attention_b200.model) against the reference's own
PrimeForCausalLM: the committed fixture tests/golden/model_small.npz holds a small reference
model's state_dict, its logits (dense and chunked attention branches) and greedy generate()
tokens (decode branch with state); the same weights loaded here must give the same results on
the kernels.  Also checks the CUDA-graph decode step against generate()."""
import ast
import os

import numpy as np
import pytest
import torch

from helpers import TOL_F32
from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden", "model_small.npz")


def _load():
    g = np.load(GOLD)
    cfg = ast.literal_eval(str(g["cfg"]))
    sd = {k[3:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("p::")}
    return g, cfg, sd


def test_state_dict_layout_matches_reference():
    """No GPU needed: parameter names and shapes of the mirror equal the reference's."""
    from prime_moment_attention_b200.model import PrimeConfig, PrimeForCausalLM
    _, cfg, sd = _load()
    m = PrimeForCausalLM(PrimeConfig(**cfg))
    mine = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert mine == {k: tuple(v.shape) for k, v in sd.items()}


@pytest.mark.gpu
def test_model_forward_and_generate_match_reference():
    from prime_moment_attention_b200.model import DecodeGraph, PrimeConfig, PrimeForCausalLM
    torch.backends.cuda.matmul.allow_tf32 = False
    g, cfg, sd = _load()
    m = PrimeForCausalLM(PrimeConfig(**cfg))
    m.load_state_dict(sd, strict=True)
    m = m.cuda().eval()
    ids = torch.from_numpy(g["ids"]).cuda()
    with torch.inference_mode():
        logits = m(ids)["logits"]
        long = m(torch.from_numpy(g["ids_long"]).cuda())["logits"][:, -8:]
        last = m(ids, last_logits_only=True)["logits"]
        gen = m.generate(ids[:, :12], max_new_tokens=6, temperature=0.0)
    torch.cuda.synchronize()
    assert O.rel_err(logits.double().cpu().numpy(), g["logits"]) <= TOL_F32
    assert O.rel_err(long.double().cpu().numpy(), g["logits_long_last8"]) <= TOL_F32
    # same math on one row (the GEMM shape differs, so rounding may too)
    assert O.rel_err(last[:, 0].double().cpu().numpy(), logits[:, -1].double().cpu().numpy()) <= 1e-5
    assert np.array_equal(gen.cpu().numpy(), g["generated"])

    # CUDA-graph decode step: prefill 12 tokens, then replay; same greedy tokens as generate()
    with torch.inference_mode():
        out = m(ids[:, :12], return_states=True, last_logits_only=True)
        first = torch.argmax(out["logits"][:, -1], dim=-1, keepdim=True)
        dg = DecodeGraph(m, out["states"], first)
        toks = [first.clone()]
        for _ in range(5):
            toks.append(dg.step().clone())
    torch.cuda.synchronize()
    assert np.array_equal(torch.cat(toks, dim=1).cpu().numpy(), g["generated"][:, 12:])
