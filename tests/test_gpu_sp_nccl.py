"""Sequence-parallel prefill across GPUs with NCCL (needs 2 or more GPUs; skipped otherwise).

Each rank holds one contiguous shard of the sequence on its own GPU; the B200 kernels do
both passes and the prefix fold, NCCL does the state all-gather.  Checked against the
float64 oracle of the whole sequence on every rank's shard and on the final state."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from helpers import TOL_BF16, TOL_F32

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, D, dtype_name, out):
    import torch.distributed as dist
    from oracle import oracle as O
    from prime_moment_attention_b200 import sp, synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        dtype = getattr(torch, dtype_name)
        B, H, Ls = 1, 4, 1000 + 24 * rank  # unequal shards, ragged last chunk
        lens = [1000 + 24 * g for g in range(world)]
        L = sum(lens)
        q, k, v = synth.make_qkv(B, H, L, D, seed=5, dtype=dtype, device="cpu")
        lam = synth.make_lambdas(H, 0.995, 0.9999, seed=5)
        a = sum(lens[:rank])
        sl = slice(a, a + Ls)
        y, final = sp.sequence_parallel_prefill(q[:, :, sl].contiguous().to(dev), k[:, :, sl].contiguous().to(dev),
                                                v[:, :, sl].contiguous().to(dev), lam.to(dev), shard_lengths=lens,
                                                broadcast_final=True)
        torch.cuda.synchronize()
        y_ref, s_ref = O.prefill(q, k, v, lam.double().numpy())
        errs = [O.rel_err(y.double().cpu().numpy(), y_ref[:, :, sl])]
        errs += [O.rel_err(f.double().cpu().numpy().reshape(r.shape), r) for f, r in zip(final, s_ref)]
        out[rank] = max(errs)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("D,dtype_name,tol", [(64, "bfloat16", TOL_BF16), (64, "float32", TOL_F32),
                                              (128, "bfloat16", TOL_BF16), (128, "float32", TOL_F32)])
def test_sequence_parallel_prefill_nccl(D, dtype_name, tol):
    world = min(torch.cuda.device_count(), 4)
    out = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), D, dtype_name, out), nprocs=world, start_method="spawn",
                       join=True)
    assert len(out) == world
    assert max(out.values()) <= tol, dict(out)


def _worker_config5(rank, world, port, out):
    """Config 5's head shape and decay law at L = 2^16 in `world` equal shards: two sampled
    head-states against the float64 oracle, every head-state against the float32 CUDA-core
    kernel over the whole sequence on this rank's GPU."""
    import torch.distributed as dist
    from oracle import oracle as O
    from prime_moment_attention_b200 import ops, sp, synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        c = synth.CONFIG5
        B, H, L, D = c["B"], c["H"], 1 << 16, c["D"]
        Ls = L // world
        q, k, v = synth.make_qkv(B, H, L, D, seed=c["seed"], dtype=torch.bfloat16, device=dev)
        lam = synth.make_lambdas(H, *c["lam"], seed=c["seed"])
        sl = slice(rank * Ls, (rank + 1) * Ls)
        y, final = sp.sequence_parallel_prefill(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(),
                                                v[:, :, sl].contiguous(), lam.to(dev), broadcast_final=True)
        y32, st32 = ops.prefill(q.float(), k.float(), v.float(), lam.to(dev), out_dtype=torch.float32)
        torch.cuda.synchronize()
        errs = [O.rel_err(y.double().cpu().numpy(), y32[:, :, sl].double().cpu().numpy())]
        errs += [O.rel_err(f.double().cpu().numpy(), r.double().cpu().numpy()) for f, r in zip(final, st32)]
        h = [int(torch.argmax(lam)), 7][rank % 2]
        y_ref, s_ref = O.prefill(q[:, h:h + 1].cpu(), k[:, h:h + 1].cpu(), v[:, h:h + 1].cpu(),
                                 lam.double().numpy()[h:h + 1])
        errs.append(O.rel_err(y[:, h:h + 1].double().cpu().numpy(), y_ref[:, :, sl]))
        errs += [O.rel_err(f[:, h:h + 1].double().cpu().numpy().reshape(r.shape), r) for f, r in zip(final, s_ref)]
        out[rank] = max(errs)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sequence_parallel_config5_law_nccl():
    world = 2
    out = mp.Manager().dict()
    mp.start_processes(_worker_config5, args=(world, _free_port(), out), nprocs=world, start_method="spawn",
                       join=True)
    assert len(out) == world
    print(f"config-5 law, L=2^16 over {world} NCCL shards: max relative error per rank {dict(out)}")
    assert max(out.values()) <= TOL_BF16, dict(out)
