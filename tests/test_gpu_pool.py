"""State pool + row-indexed decode (pma_decode_step_rows) against the float64 oracle.

Several sequences are prefilled into pool slots of two layers, then decoded for a few
steps with a changing, permuted batch of slots; every sequence's outputs and final state
must match the oracle run of that sequence alone."""
import numpy as np
import pytest
import torch

from helpers import TOL_BF16, TOL_F32
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _seq(seed, H, L, D, dtype):
    from prime_moment_attention_b200 import synth
    return synth.make_qkv(1, H, L, D, seed=seed, dtype=dtype, device="cuda")


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, TOL_BF16), (torch.float32, TOL_F32)])
def test_pool_prefill_then_rows_decode(dtype, tol):
    from prime_moment_attention_b200 import pool as P, synth
    H, D, layers = 12, 64, 2
    pool = P.StatePool(capacity=8, H=H, D=D, layers=layers)
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=4).cuda()
    lens = {0: 300, 1: 129, 2: 7}
    slots, hist = {}, {}
    for sid, L in lens.items():
        s = pool.alloc()
        slots[sid] = s
        for layer in range(layers):
            q, k, v = _seq(100 * sid + layer, H, L, D, dtype)
            pool.prefill(layer, s, q, k, v, lam)
            hist[(sid, layer)] = [(q, k, v)]
    assert pool.free_slots == 5 and pool.seen_tokens[slots[0]] == 300
    batches = [[2, 0], [1, 2, 0], [0], [1, 0, 2]]
    for step, batch in enumerate(batches):
        for layer in range(layers):
            toks = [_seq(1000 * step + 10 * sid + layer, H, 1, D, dtype) for sid in batch]
            q = torch.cat([t[0][:, :, 0] for t in toks])
            k = torch.cat([t[1][:, :, 0] for t in toks])
            v = torch.cat([t[2][:, :, 0] for t in toks])
            y = pool.decode_step(layer, [slots[s] for s in batch], q, k, v, lam)
            torch.cuda.synchronize()
            for n, sid in enumerate(batch):
                hist[(sid, layer)].append(toks[n])
                qs = torch.cat([h[0] for h in hist[(sid, layer)]], dim=2)
                ks = torch.cat([h[1] for h in hist[(sid, layer)]], dim=2)
                vs = torch.cat([h[2] for h in hist[(sid, layer)]], dim=2)
                y_ref, s_ref = O.prefill(qs.cpu(), ks.cpu(), vs.cpu(), lam.double().cpu().numpy())
                err = O.rel_err(y[n].double().cpu().numpy(), y_ref[0, :, -1])
                assert err <= tol, (step, layer, sid, err)
                st = pool.get_state(layer, slots[sid])
                for a, b in zip(st, s_ref):
                    assert O.rel_err(a.double().cpu().numpy().reshape(b.shape), b) <= tol


def test_pool_rows_out_of_range_are_skipped():
    from prime_moment_attention_b200 import ops, pool as P, synth
    H, D = 4, 32
    pool = P.StatePool(capacity=3, H=H, D=D)
    before = [t.clone() for t in pool.state]
    q, k, v = synth.make_qkv(2, H, 1, D, seed=9, dtype=torch.float32, device="cuda")
    y = torch.full((2, H, D), 7.0, device="cuda")
    rows = torch.tensor([-1, 3], dtype=torch.int32, device="cuda")
    ops.decode_step_rows(q[:, :, 0], k[:, :, 0], v[:, :, 0], 0.99, pool.state, rows, y_out=y)
    torch.cuda.synchronize()
    assert torch.all(y == 7.0)
    for a, b in zip(pool.state, before):
        assert torch.equal(a, b)


def test_cache_decodes_in_place_on_pool_rows():
    """PrimeMomentCache on StatePool rows: prefill states are set per layer, then every layer is
    decoded in place through the cache (pma_decode_step_rows on the layer's rows) and through the
    module's functional path (state in from get_state, new tuple back through set_state).  The
    views the cache hands out keep pointing at the same rows, and y and the states match the
    float64 oracle at the fp32 bar."""
    from prime_moment_attention_b200 import PrimeMomentCache, ops, synth
    B, H, D, layers = 3, 4, 64, 2
    lam = synth.make_lambdas(H, 0.99, 0.9999, seed=12).cuda()
    cache = PrimeMomentCache(num_layers=layers)
    ref = {}
    for layer in range(layers):
        q, k, v = synth.make_qkv(B, H, 200 + layer, D, seed=50 + layer, device="cuda")
        _, st = ops.prefill(q, k, v, lam)
        cache.set_state(layer, st)
        ref[layer] = O.prefill(q, k, v, lam.double().cpu().numpy())[1]
    ptrs = {layer: [t.data_ptr() for t in cache.get_state(layer)] for layer in range(layers)}
    for step in range(3):
        for layer in range(layers):
            q, k, v = synth.make_decode_tokens(B, H, D, seed=900 + 10 * step + layer, dtype=torch.float32,
                                               device="cuda")
            if step % 2 == 0:
                y = cache.decode_step(layer, q, k, v, lam)
            else:  # the module's functional step: fresh tensors, copied back into the rows
                y, new = ops.decode_step(q, k, v, lam, cache.get_state(layer))
                cache.set_state(layer, new)
            y_ref, ref[layer] = O.decode_step(q, k, v, lam.double().cpu().numpy(), ref[layer])
            assert O.rel_err(y.double().cpu().numpy(), y_ref) <= TOL_F32
    for layer in range(layers):
        got = cache.get_state(layer)
        assert [t.data_ptr() for t in got] == ptrs[layer]
        for g, r in zip(got, ref[layer]):
            assert O.rel_err(g.double().cpu().numpy().reshape(r.shape), r) <= TOL_F32
