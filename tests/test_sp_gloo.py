"""Sequence-parallel prefill (sp.sequence_parallel_prefill) on CPU ranks over gloo.

The per-rank compute is the float64 oracle (test infrastructure), so these tests exercise
the real exchange and prefix-fold code of sp.py -- pass 1 from zero, all-gather of the
shard states, the decay-weighted fold, pass 2 from the carried state -- without a GPU.
World size 2 and 3, equal and unequal shards, with and without an incoming state, and the
final-state broadcast."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


class OracleKernels:
    """CPU stand-in for the B200 kernels with the same call shapes as sp.CudaKernels."""

    @staticmethod
    def _prefill(q, k, v, decay, state, eps):
        st = None if state is None else tuple(t.double().numpy() for t in state)
        y, s = O.prefill(q.double().numpy(), k.double().numpy(), v.double().numpy(), np.asarray(decay), st, eps)
        return torch.from_numpy(y).float(), tuple(torch.from_numpy(a).float() for a in s)

    @staticmethod
    def shard_state(q, k, v, decay, eps):
        return OracleKernels._prefill(q, k, v, decay, None, eps)[1], None

    @staticmethod
    def shard_output(q, k, v, decay, state, eps, y_out, handle):
        assert handle is None
        return OracleKernels._prefill(q, k, v, decay, state, eps)

    @staticmethod
    def combine(T, P, decay, length):
        lam = torch.as_tensor(np.asarray(decay), dtype=torch.float64)
        f = (lam ** length).float()  # per head [H]
        for t, p in zip(T, P):
            shape = [1, -1] + [1] * (p.dim() - 2)
            p.mul_(f.view(shape)).add_(t)
        return P


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(seed, B, H, L, D):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, D, generator=g), dim=-1) / D ** 0.5
    k = torch.nn.functional.normalize(torch.randn(B, H, L, D, generator=g), dim=-1)
    v = torch.randn(B, H, L, D, generator=g)
    lam = np.exp(np.random.default_rng(seed).uniform(np.log(0.9), np.log(0.999), H))
    return q, k, v, lam


def _init_state(seed, B, H, D, lam):
    rng = np.random.default_rng(seed + 7)
    st = [rng.normal(0, 0.01, s) for s in [(B, H, D), (B, H, D, D), (B, H, D, D), (B, H, 1), (B, H, D), (B, H, D)]]
    st[3] = np.broadcast_to(((1 - lam ** 512) / (1 - lam)).reshape(1, H, 1), (B, H, 1)).copy()
    return st


def _worker(rank, world, port, lens, with_state, bcast, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from prime_moment_attention_b200 import sp
        B, H, D = 2, 3, 8
        q, k, v, lam = _case(11, B, H, sum(lens), D)
        st = _init_state(11, B, H, D, lam) if with_state else None
        a = sum(lens[:rank])
        sl = slice(a, a + lens[rank])
        state = tuple(torch.from_numpy(s).float() for s in st) if st is not None else None
        y, final = sp.sequence_parallel_prefill(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(),
                                                v[:, :, sl].contiguous(), lam, state=state, shard_lengths=lens,
                                                broadcast_final=bcast, kernels=OracleKernels)
        y_ref, s_ref = O.prefill(q.double().numpy(), k.double().numpy(), v.double().numpy(), lam, st)
        errs = [O.rel_err(y.double().numpy(), y_ref[:, :, sl])]
        if final is not None:
            errs += [O.rel_err(f.double().numpy().reshape(r.shape), r) for f, r in zip(final, s_ref)]
        out[rank] = (max(errs), final is not None)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("lens,with_state,bcast", [
    ((24, 24), False, False),
    ((16, 40), True, False),
    ((20, 9, 31), True, True),
])
def test_sequence_parallel_prefill_gloo(lens, with_state, bcast):
    world = len(lens)
    out = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), lens, with_state, bcast, out), nprocs=world,
                       start_method="spawn", join=True)
    assert len(out) == world
    for r in range(world):
        err, has_final = out[r]
        assert err < 1e-5, (r, err)  # float32 exchange of float64 oracle states
        assert has_final == (bcast or r == world - 1)
