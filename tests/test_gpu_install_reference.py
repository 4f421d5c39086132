"""install() on the reference's own classes: the reference PrimeForCausalLM (model.py:123-242) with
its PrimeMomentAttention (attention.py:42-210) or PrimeSelectiveMomentAttention (selective.py:264-444)
layers, run unchanged -- forward and greedy generate() -- first on the reference's eager PyTorch
path, then with install() routing every attention layer onto this package's kernels, on the same
weights and inputs.  Logits must agree to the fp32 bar (1e-4, float32 model) and the generated
tokens exactly.

The reference package comes from baseline/_ref (installed there from the reference sources with
`pip install --target baseline/_ref`); the tests skip when it is absent."""
import os
import sys

import pytest
import torch

from oracle import oracle as O
from prime_moment_attention_b200 import shim
from tests.helpers import TOL_F32, cpu64

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "prime_moment_attention")),
                                 reason="reference package not installed in baseline/_ref")]


def _reference():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import prime_moment_attention as ref
    return ref


def _run(m, ids, prompt):
    with torch.no_grad():
        logits = m(ids)["logits"]
        gen = m.generate(ids[:, :prompt], max_new_tokens=6, temperature=0.0)
    torch.cuda.synchronize()
    return logits, gen


@pytest.mark.parametrize("selective", [False, True])
def test_install_on_reference_model(selective):
    ref = _reference()
    cfg = ref.PrimeConfig(vocab_size=512, hidden_size=256, num_layers=2, num_heads=4, head_dim=64,
                          use_selective=selective)
    torch.manual_seed(3)
    m = ref.PrimeForCausalLM(cfg).to("cuda", torch.float32).eval()
    cls = ref.PrimeSelectiveMomentAttention if selective else ref.PrimeMomentAttention
    g = torch.Generator(device="cuda").manual_seed(4)
    # 700 tokens take the chunked branch (L > 512); generate() prefills 40 (dense branch) and decodes
    ids = torch.randint(0, cfg.vocab_size, (2, 700), device="cuda", generator=g)
    assert not shim.installed(cls)
    logits_ref, gen_ref = _run(m, ids, 40)
    shim.install(cls)
    try:
        assert m.layers[0].self_attn.__class__.forward is shim._forward_for(cls)
        logits, gen = _run(m, ids, 40)
    finally:
        shim.uninstall(cls)
    e = O.rel_err(cpu64(logits), cpu64(logits_ref))
    print(f"reference model (selective={selective}): logits relative error {e:.2e} with install()")
    assert e <= TOL_F32, e
    assert torch.equal(gen, gen_ref)
    # uninstall() gives back the reference path bit for bit
    logits_again, _ = _run(m, ids, 40)
    assert torch.equal(logits_again, logits_ref)
