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


@pytest.mark.gpu
def test_decode_graph_selective_layers_match_generate():
    """A model with selective layers (per-token decay from delta_proj): the CUDA-graph decode step
    gives the same greedy tokens as generate()."""
    from prime_moment_attention_b200.model import DecodeGraph, PrimeConfig, PrimeForCausalLM
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(7)
    cfg = PrimeConfig(vocab_size=97, hidden_size=64, num_layers=2, num_heads=4, head_dim=16, intermediate_size=96,
                      decay=0.99, use_selective=True)
    m = PrimeForCausalLM(cfg)
    with torch.no_grad():  # leave the identity initialisation: data-dependent decays and temperatures
        for layer in m.layers:
            a = layer.self_attn
            a.delta_proj.weight.normal_(0, 0.3)
            a.log_tau.copy_(torch.log(torch.linspace(4.0, 400.0, 4)))
            a.log_beta.copy_(torch.tensor([0.2, -0.1, 0.0, 0.3]))
    m = m.cuda().eval()
    ids = torch.randint(0, 97, (3, 10), generator=torch.Generator().manual_seed(8)).cuda()
    with torch.inference_mode():
        gen = m.generate(ids, max_new_tokens=6, temperature=0.0)
        out = m(ids, return_states=True, last_logits_only=True)
        first = torch.argmax(out["logits"][:, -1], dim=-1, keepdim=True)
        dg = DecodeGraph(m, out["states"], first)
        toks = [first.clone()]
        for _ in range(5):
            toks.append(dg.step().clone())
    torch.cuda.synchronize()
    assert np.array_equal(torch.cat(toks, dim=1).cpu().numpy(), gen[:, 10:].cpu().numpy())


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,halves", [((5, 3072), True), ((2, 7, 96), False), ((3, 13), False)])
def test_swiglu_matches_the_two_torch_kernels(dtype, shape, halves):
    """pma_swiglu against F.silu(gate) * up, element for element: contiguous inputs, the column halves
    of one [N, 2I] GEMM output (the decode graph's layout), and a width the 16-byte path cannot take."""
    from prime_moment_attention_b200 import ops
    gen = torch.Generator().manual_seed(sum(shape))
    if halves:
        gu = (torch.randn(shape[0], 2 * shape[1], generator=gen) * 3).to("cuda", dtype)
        gate, up = gu[:, :shape[1]], gu[:, shape[1]:]
    else:
        gate = (torch.randn(*shape, generator=gen) * 3).to("cuda", dtype)
        up = (torch.randn(*shape, generator=gen) * 3).to("cuda", dtype)
    ref = torch.nn.functional.silu(gate) * up
    out = ops.swiglu(gate, up)
    torch.cuda.synchronize()
    assert out.shape == ref.shape and torch.equal(out, ref)


@pytest.mark.gpu
def test_swiglu_refuses_a_mismatched_out():
    """A caller-supplied `out` must match gate in shape, dtype and device and have a contiguous last
    axis; otherwise the kernel would write past it or store bf16 bits into float32."""
    from prime_moment_attention_b200 import ops
    gate = torch.randn(4, 96, device="cuda", dtype=torch.bfloat16)
    up = torch.randn(4, 96, device="cuda", dtype=torch.bfloat16)
    bad = [torch.empty(3, 96, device="cuda", dtype=torch.bfloat16),        # fewer rows
           torch.empty(4, 96, device="cuda", dtype=torch.float32),         # another dtype
           torch.empty(4, 96, dtype=torch.bfloat16),                       # host memory
           torch.empty(96, 4, device="cuda", dtype=torch.bfloat16).t()]    # strided last axis
    for out in bad:
        with pytest.raises(ValueError):
            ops.swiglu(gate, up, out=out)
    out = torch.empty(4, 96, device="cuda", dtype=torch.bfloat16)
    assert ops.swiglu(gate, up, out=out) is out
    assert torch.equal(out, torch.nn.functional.silu(gate) * up)
