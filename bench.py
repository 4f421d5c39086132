#!/usr/bin/env python3
"""Benchmark of the PRIME moment attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline metric (one JSON line from rank 0): config-2 prefill throughput,
tokens/s over all GPUs -- B=8 sequences per GPU, H=12 heads, D=64, L=8192, bf16
q/k/v, fp32 state, per-head lambda log-uniform in [0.99, 0.9999].  A "step" is one
pma_prefill call over that batch (y and the final state).  The line also carries
the config-3 decode step (256 sequences x 12 layers x 12 heads, D=64, one launch
for all layers' heads, 1000 timed steps) under "decode", and the gated delta-rule variant
(config-2 prefill with the write gate beta, and its decode step at the config-3 shape) under
"delta", the selective variant under "selective", the config-4 model (prefill and CUDA-graph decode)
under "model", and the config-5 long sequence (sequence shards over the GPUs) under "sp".

Multi-GPU: one process per GPU (torchrun); each rank prefills its own batch x head
shard with no collective (weak scaling); times are the max over ranks.

--impl reference times the reference's own C99 runtime (c/prime_moment.c, built
unmodified into oracle/_ref/ by oracle/Makefile) on the host cores, additive mode,
on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import shutil
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

PREFILL = dict(B=8, H=12, L=8192, D=64, lam=(0.99, 0.9999), seed=2)
DECODE = dict(seqs=256, layers=12, H=12, D=64, lam=(0.99, 0.9999), t0=4096, sigma=0.01, seed=3, steps=1000)
PREFILL_BYTES_PER_TOKHEAD = 8 * 64          # q,k,v in + y out, bf16: 8*D bytes
# algorithmic FLOPs per token-head: the dense-chunk count the reference executes at its chunk
# C = 64 (chunked_ssd.py:90-93, 106-107, 146-148): 6*C*D + 8*D^2 = 57,344 (den/Z terms excluded)
PREFILL_FLOP_PER_TOKHEAD = 6 * 64 * 64 + 8 * 64 * 64
# what this kernel's chunked form issues at C = 128 tokens, F = 2D = 128 moment features:
# scores 2*C*F + intra P.V 2*C*D + carry 2*F*D + state update 2*F*D = 81,920
PREFILL_KERNEL_FLOP_PER_TOKHEAD = 2 * 128 * 128 + 2 * 128 * 64 + 2 * 128 * 64 + 2 * 128 * 64
DECODE_BYTES_PER_HEADSTEP = 2 * (2 * 64 * 64 + 3 * 64 + 1) * 4 + 3 * 64 * 2 + 64 * 2  # 67,592
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of
# each kernel on the bench workload; the commands and the rest of the numbers are in profiles/.
PREFILL_TRAFFIC = 306_312_192 + 79_452_160    # prefill_tc_kernel<0, bf16>, config 2
PREFILL_MIN_WARMUP = 50  # untimed config-2 calls before the timed ones (at least --warmup)
# DRAM bytes of config 5's one-GPU step (state-only pass over 8 of 9 segments + full pass), from the
# ncu capture of config 5's heads at L = 2^16 (profiles/prefill_tc128_config5_L65536.md: 478.3 + 4.0
# MB and 824.7 + 242.8 MB per launch), scaled x16 to L = 2^20 (the plan's segments scale with L)
SP_TRAFFIC_1GPU = 16 * (478_300_000 + 4_000_000 + 824_700_000 + 242_800_000)
DECODE_TRAFFIC = 1_250_602_000 + 1_183_497_000  # decode_step_kernel<64, bf16, bf16>, config 3
# Gated delta-rule variant (config 2 with the write gate beta): per token-head of the chunked
# form at C = 64, F = 2D = 128 features -- Gram Phi Phi^T 2*C*F, intra scores Psi Phi^T 2*C*F,
# inter error Phi S^T 2*F*D, inter readout Psi S^T 2*F*D, state update 2*F*D, intra readout
# P (beta E) 2*C*D, triangular solve C*D  = 94,208 FLOP; q,k,v in + y out bf16 + beta fp32.
DELTA_FLOP_PER_TOKHEAD = 4 * 64 * 128 + 6 * 128 * 64 + 3 * 64 * 64
DELTA_BYTES_PER_TOKHEAD = 8 * 64 + 4
# DRAM bytes of the WY pair (prep: reads q, k, v, gates, writes the 72 KB records; sequential: reads
# the records, writes y) from one ncu capture at B = 2 (profiles/), scaled x4 to the B = 8 step
DELTA_TRAFFIC_B2 = (76_662_784 + 172_416_256) + (226_543_872 + 22_940_160)
DELTA_DECODE_BYTES_PER_HEADSTEP = 2 * (64 * 128 * 4) + 4 * 64 * 2 + 8  # state rw + q,k,v,y + beta,alpha
FP32_SIMT_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal: 148 SMs x 128 FMA/clk at 1,965 MHz
WORKLOAD = ("config2 prefill: B=8 seqs/GPU, H=12, D=64, L=8192, bf16 q/k/v (QK-normed), fp32 state, "
            "per-head lambda log-U[0.99,0.9999]; step = one pma_prefill (y + final state)")


def _peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples taken during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap,clocks.mem")

    def __init__(self, index: int):
        # nvidia-smi numbers the physical GPUs: map the CUDA device index through CUDA_VISIBLE_DEVICES
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        self.index = ids[index] if index < len(ids) else index
        self.proc = None
        self.path = None

    def start(self):
        if not shutil.which("nvidia-smi"):
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits", "-lms", "100"],
                                     stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        time.sleep(0.25)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = sorted(int(r[1]) for r in rows)
        mem = sorted(int(r[9]) for r in rows if len(r) > 9 and r[9].isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        out = {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": int(rows[0][2]), "samples": len(rows), "reasons": reasons}
        if mem:
            out["mem_mhz"] = mem[len(mem) // 2]
        return out


# --------------------------------------------------------------------------- distributed
def dist_setup():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        # NCCL's own log lines go to stderr, so that rank 0's stdout carries the one JSON line only.
        # NCCL honours NCCL_DEBUG_FILE only above the VERSION level (at VERSION its banner goes to
        # stdout), so VERSION is raised to WARN, which prints the same banner plus warnings.
        if os.environ.get("NCCL_DEBUG", "").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def per_rank(x, ws: int):
    """Every rank's value of x (a float or a small dict), in rank order; [x] with one rank."""
    if ws == 1:
        return [x]
    import torch.distributed as dist
    out = [None] * ws
    dist.all_gather_object(out, x)
    return out


def max_over_ranks(x: float, ws: int, device) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- CPU baseline
def ref_bench_path():
    p = os.path.join(HERE, "oracle", "_ref", "ref_bench")
    return p if os.path.exists(p) else None


def run_ref(args_list, timeout=600):
    out = subprocess.run([ref_bench_path(), *map(str, args_list)], capture_output=True, text=True,
                         timeout=timeout, check=True)
    return json.loads(out.stdout.strip().splitlines()[-1])


def cpu_prefill_sample(target_s: float = 12.0):
    """Reference C99 prime_prefill (additive, eps=1) on all host cores: tokens/s.

    Calibrates on a short run, then times states x tokens sized for ~target_s."""
    threads = os.cpu_count() or 1
    c = PREFILL
    cal = run_ref(["prefill", threads, c["H"], 256, c["D"], threads])
    rate = cal["tok_per_s"]
    L = 2048
    nstates = max(threads, int(rate * target_s / L))
    nstates = (nstates + threads - 1) // threads * threads
    r = run_ref(["prefill", nstates, c["H"], L, c["D"], threads], timeout=int(20 * target_s) + 60)
    return {"value": r["tok_per_s"], "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"reference c/prime_moment.c prime_prefill (additive, eps=1), {nstates} sequences x "
                      f"{L} tokens x {c['H']} heads x D={c['D']}, {threads} threads, {r['seconds']:.1f} s"}


def cpu_decode_sample(target_s: float = 6.0):
    """Reference C99 prime_step over seqs x layers states: projected us per config-3 step."""
    threads = os.cpu_count() or 1
    c = DECODE
    total_states = c["seqs"] * c["layers"]
    cal = run_ref(["decode", threads * 4, c["H"], c["D"], 3, threads])
    per_state = cal["seconds"] / (3 * threads * 4)
    nstates = min(total_states, max(threads, int(target_s / max(per_state, 1e-9) / 4)))
    r = run_ref(["decode", nstates, c["H"], c["D"], 4, threads], timeout=int(20 * target_s) + 60)
    us = r["us_per_step"] * total_states / nstates
    return {"value": us, "unit": "us/step", "cores": threads, "kind": "reference",
            "sample": f"reference c/prime_moment.c prime_step (additive, eps=1), {nstates} of {total_states} "
                      f"seq x layer states (12 heads each), 4 steps, {threads} threads, scaled to all states"}


def _reference_package():
    """The reference's PyTorch package as installed in baseline/_ref (pip install --target), or None."""
    ref_dir = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "prime_moment_attention")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import prime_moment_attention
    return prime_moment_attention


def cpu_pytorch_prefill_sample(target_s: float = 10.0):
    """The reference's PyTorch chunked prefill (chunked_prime_ssd_core, chunked_ssd.py:48-184) on all
    host threads, at config 2's shapes and laws: per head slice (the reference holds one scalar decay
    per call), bf16 q/k/v cast to float32 as the module does (attention.py:104-106), chunk 64,
    eps 1, final state returned.  Times whole batch rows of 12 heads x 8192 tokens, as many as
    fit ~target_s after a one-head calibration; tok/s = rows x 8192 / seconds."""
    import torch
    ref = _reference_package()
    if ref is None:
        return {"unavailable": "baseline/_ref holds no reference install"}
    from prime_moment_attention.chunked_ssd import chunked_prime_ssd_core
    from prime_moment_attention_b200 import synth
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    c = PREFILL
    H, L, D = c["H"], c["L"], c["D"]
    lam = synth.make_lambdas(H, *c["lam"], seed=c["seed"]).tolist()

    def row(seed, heads):
        q, k, v = synth.make_qkv(1, H, L, D, seed=seed, dtype=torch.bfloat16)
        q, k, v = q.float(), k.float(), v.float()
        t0 = time.perf_counter()
        with torch.no_grad():
            for h in heads:
                chunked_prime_ssd_core(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], decay=lam[h], eps=1.0,
                                       chunk_size=64, return_state=True)
        return time.perf_counter() - t0

    row(1, [0])  # warm-up
    per_head = row(2, [0])
    rows = int(max(1, min(c["B"], target_s / max(per_head * H, 1e-6))))
    dt = sum(row(10 + r, range(H)) for r in range(rows))
    return {"value": round(rows * L / dt, 1), "unit": "tok/s", "cores": threads, "kind": "reference_pytorch",
            "sample": f"reference chunked_prime_ssd_core (PyTorch, float32), {rows} of {c['B']} batch rows x "
                      f"{H} heads (one call per head) x L={L}, D={D}, chunk 64, torch threads={threads}, "
                      f"{dt:.1f} s"}


def cpu_pytorch_decode_sample(target_s: float = 6.0):
    """The reference's PyTorch decode branch (PrimeMomentAttention.forward with L == 1,
    attention.py:77-143, projections and QK-norm included) on all host threads, at config 3's shape:
    one layer = one module call on 256 sequences x 12 heads, D = 64, from a seeded state; the
    reference module holds one scalar decay (0.9995 here).  Times whole layer steps, as many as fit
    ~target_s, and scales to the 12 layers of a config-3 step: us per step."""
    import torch
    ref = _reference_package()
    if ref is None:
        return {"unavailable": "baseline/_ref holds no reference install"}
    from prime_moment_attention.attention import PrimeMomentAttention
    from prime_moment_attention_b200 import synth
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    dc = DECODE
    N, H, D = dc["seqs"], dc["H"], dc["D"]
    torch.manual_seed(dc["seed"])
    m = PrimeMomentAttention(hidden_size=H * D, num_heads=H, head_dim=D, decay=0.9995, use_qk_norm=True).eval()
    st = synth.make_state(N, H, D, torch.full((H,), 0.9995), seed=dc["seed"], t0=dc["t0"], sigma=dc["sigma"])
    x = torch.randn(N, 1, H * D, generator=torch.Generator().manual_seed(dc["seed"]))

    def layer_step(state):
        t0 = time.perf_counter()
        with torch.no_grad():
            _, state = m(x, state=state, return_state=True)
        return time.perf_counter() - t0, state

    _, st = layer_step(st)  # warm-up
    dt, st = layer_step(st)
    n = int(max(1, min(12, target_s / max(dt, 1e-6))))
    tot = 0.0
    for _ in range(n):
        t, st = layer_step(st)
        tot += t
    us = tot / n * dc["layers"] * 1e6
    return {"value": round(us, 1), "unit": "us/step", "cores": threads, "kind": "reference_pytorch",
            "sample": f"reference PrimeMomentAttention.forward, L=1 (PyTorch, float32, projections and QK-norm "
                      f"included), {N} seqs x {H} heads, D={D}, {n} layer steps timed, x{dc['layers']} layers, "
                      f"torch threads={threads}"}


def run_reference_arm(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if ref_bench_path() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/ref_bench was not built (needs the "
                          "reference tree when build() ran)"}))
        return 0
    threads = os.cpu_count() or 1
    vals = []
    sample = None
    # each step is a bounded sample of the workload; warmup steps are shorter
    for i in range(args.warmup + args.steps):
        r = cpu_prefill_sample(target_s=2.0 if i < args.warmup else 6.0)
        if i >= args.warmup:
            vals.append(r["value"])
            sample = r["sample"]
    v = sum(vals) / len(vals)
    dec = cpu_decode_sample(target_s=4.0)
    line = {"impl": "reference", "metric": "prefill_tok_per_s", "value": v, "unit": "tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(PREFILL["B"] * PREFILL["L"] / v * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": PREFILL["B"], "seq_len": PREFILL["L"],
                       "parallelism": f"host, {threads} threads"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "decode": {"metric": "decode_step_us", "value": dec["value"], "unit": "us/step",
                       "higher_is_better": False, "sample": dec["sample"]}}
    print(json.dumps(line))
    return 0


# --------------------------------------------------------------------------- our arm
def time_steps(fn, steps, warmup, ws, device, stream):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    barrier(ws)
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(device)
    barrier(ws)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / steps  # ms per step


def bench_prefill(args, ws, rank, device, stream, peaks):
    """Config-2 prefill: device-timed throughput, roofline, and the e2e call from host buffers."""
    import torch
    from prime_moment_attention_b200 import _lib, ops, synth
    hbm_peak, tc_peak, peak_kind = peaks
    c = PREFILL
    B, H, L, D = args.prefill_batch or c["B"], c["H"], c["L"], c["D"]
    q, k, v = synth.make_qkv(B, H, L, D, seed=c["seed"] + 1000 * rank, dtype=torch.bfloat16, device=device)
    lam = synth.make_lambdas(H, *c["lam"], seed=c["seed"]).to(device)
    y = torch.empty_like(q)
    ws_bytes = _lib.load().pma_prefill_workspace_bytes(B, H, L, D, _lib.PMA_BF16)
    launches_per_step = 3 if ws_bytes > 256 else 1

    def step():
        ops.prefill(q, k, v, lam, y_out=y, return_state=True)

    clocks = ClockSampler(device.index)
    clocks.start()  # before the warm-up, so that the timed steps follow it back to back
    # at least 50 untimed calls (~8 ms): with several ranks the first calls after the process
    # group's barrier ran a few per cent slower than the steady state
    warm = max(args.warmup, PREFILL_MIN_WARMUP)
    ms = time_steps(step, args.steps, warm, ws, device, stream)
    clk = clocks.stop()
    rank_ms = per_rank(round(ms, 5), ws)
    rank_clk = per_rank(clk, ws)
    ms = max_over_ranks(ms, ws, device)
    tokens = B * L * ws
    tokheads = B * L * H
    algo_bytes = tokheads * PREFILL_BYTES_PER_TOKHEAD
    algo_flop = tokheads * PREFILL_FLOP_PER_TOKHEAD
    kern_flop = tokheads * PREFILL_KERNEL_FLOP_PER_TOKHEAD
    bw = algo_bytes / (ms * 1e-3) / 1e9
    tf = algo_flop / (ms * 1e-3) / 1e12
    tfk = kern_flop / (ms * 1e-3) / 1e12
    roof = {"bound": "hbm", "achieved": round(bw, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(bw / hbm_peak, 4),
            "traffic": PREFILL_TRAFFIC if (B, H, L, D) == (c["B"], c["H"], c["L"], c["D"]) else None,
            "peak_kind": peak_kind,
            "tensor": {"achieved": round(tf, 1), "peak": tc_peak, "unit": "TFLOP/s", "frac": round(tf / tc_peak, 4),
                       "flop_per_tokhead": PREFILL_FLOP_PER_TOKHEAD,
                       "kernel_flop_per_tokhead": PREFILL_KERNEL_FLOP_PER_TOKHEAD,
                       "kernel_achieved": round(tfk, 1), "kernel_frac": round(tfk / tc_peak, 4)},
            "timed": "whole pma_prefill call (all its launches), CUDA events on the launching stream",
            "algorithmic_bytes_per_launch": algo_bytes, "algorithmic_flop_per_launch": algo_flop}

    # e2e through the public API with host buffers
    e2e_steps = max(1, min(args.steps, 5))
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    yh = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)

    def e2e_step():
        ops.prefill_from_host(qh, kh, vh, lam, device=device, y_host=yh, return_state=True)

    e2e_ms = max_over_ranks(time_steps(e2e_step, e2e_steps, max(3, args.warmup), ws, device, stream), ws, device)
    h2d = 3 * q.numel() * q.element_size()
    d2h = y.numel() * y.element_size()
    return {"metric": "prefill_tok_per_s", "value": round(tokens / (ms * 1e-3), 1), "unit": "tok/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": B * ws, "seq_len": L,
                       "parallelism": f"dp{ws} (batch x head shards, no collective)",
                       "l2": "inputs 403 MB per GPU > 126 MB L2; no flush",
                       "warmup_calls": warm},
            "roofline": roof,
            "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                    "path": "pinned host q,k,v -> ops.prefill_from_host: per batch slice H2D, pma_prefill (C ABI), "
                            "D2H, the slices' copies and kernels overlapped on 3 streams -> pinned host y"},
            "gpu_launches": args.steps * launches_per_step, "clocks": clk,
            **({"per_rank": {"ms_per_step": rank_ms, "clocks": rank_clk}} if ws > 1 else {})}


def bench_decode(args, ws, rank, device, stream, peaks):
    """Config-3 decode step: all layers' heads of 256 sequences in one launch, in place."""
    import torch
    from prime_moment_attention_b200 import ops, synth
    hbm_peak, _, peak_kind = peaks
    dc = DECODE
    N, HD = dc["seqs"], dc["layers"] * dc["H"]
    lam_d = synth.make_lambdas(HD, *dc["lam"], seed=dc["seed"]).to(device)
    st = synth.make_state(N, HD, dc["D"], lam_d, seed=dc["seed"] + rank, t0=dc["t0"], sigma=dc["sigma"],
                          device=device)
    toks = [synth.make_decode_tokens(N, HD, dc["D"], seed=dc["seed"] * 100 + i, device=device) for i in range(8)]
    yd = torch.empty(N, HD, dc["D"], dtype=torch.bfloat16, device=device)
    it = [0]

    def dstep():
        qq, kk, vv = toks[it[0] & 7]
        it[0] += 1
        ops.decode_step(qq, kk, vv, lam_d, st, inplace=True, y_out=yd)

    dclk = ClockSampler(device.index)
    dclk.start()
    dsteps = args.decode_steps or dc["steps"]
    dms = time_steps(dstep, dsteps, max(3, args.warmup), ws, device, stream)
    dclk_r = dclk.stop()
    ranks = {"ms_per_step": per_rank(round(dms, 5), ws), "clocks": per_rank(dclk_r, ws)}
    dms = max_over_ranks(dms, ws, device)
    d_bytes = N * HD * DECODE_BYTES_PER_HEADSTEP
    d_bw = d_bytes / (dms * 1e-3) / 1e9
    return {"metric": "decode_step_us", "value": round(dms * 1e3, 2), "unit": "us/step",
            "higher_is_better": False, "steps": dsteps,
            "config": {"workload": "config3 decode: 256 seqs x 12 layers x 12 heads per GPU, D=64, bf16 q/k/v, "
                                   "fp32 state in place, all layers' heads in one launch",
                       "state_bytes": N * HD * (2 * 64 * 64 + 3 * 64 + 1) * 4, "l2": "state 1.24 GB > L2"},
            "roofline": {"bound": "hbm", "achieved": round(d_bw, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(d_bw / hbm_peak, 4), "traffic": DECODE_TRAFFIC, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": d_bytes},
            "gpu_launches": dsteps, "clocks": dclk_r, **({"per_rank": ranks} if ws > 1 else {})}


def cpu_delta_sample(target_s: float = 8.0):
    """The float64 delta-rule port (oracle/pma_oracle.c, single thread) on a bounded sample:
    one head of config 2 for as many tokens as fit ~target_s seconds."""
    import numpy as np
    import torch
    from oracle import oracle as O
    from prime_moment_attention_b200 import synth
    q, k, v = synth.make_qkv(1, 1, 512, 64, seed=7)
    beta = torch.sigmoid(torch.randn(1, 1, 512, generator=torch.Generator().manual_seed(7)))
    t0 = time.perf_counter()
    O.delta_prefill(q, k, v, beta, None, np.array([0.999]))
    cal = time.perf_counter() - t0
    L = int(min(8192, max(512, 512 * target_s / max(cal, 1e-6))))
    q, k, v = synth.make_qkv(1, 1, L, 64, seed=8)
    beta = torch.sigmoid(torch.randn(1, 1, L, generator=torch.Generator().manual_seed(8)))
    t0 = time.perf_counter()
    O.delta_prefill(q, k, v, beta, None, np.array([0.999]))
    dt = time.perf_counter() - t0
    return {"value": round(L / dt, 1), "unit": "tok/s per head", "cores": 1, "kind": "port",
            "sample": f"float64 port of the chunked delta rule (token recurrence), 1 head x L={L}, D=64",
            "per_token_all_heads_tok_s": round(L / dt / 12, 1)}


def bench_delta(args, ws, rank, device, stream, peaks):
    """Gated delta-rule variant: config-2 prefill with the write gate beta_t = sigmoid(N(0,1)) and
    retention alpha_t = lambda_h (erase gate off), and the decode step at the config-3 shape."""
    import torch
    from prime_moment_attention_b200 import ops, synth
    hbm_peak, _, peak_kind = peaks
    c = PREFILL
    B, H, L, D = args.prefill_batch or c["B"], c["H"], c["L"], c["D"]
    q, k, v = synth.make_qkv(B, H, L, D, seed=c["seed"] + 1000 * rank, dtype=torch.bfloat16, device=device)
    lam = synth.make_lambdas(H, *c["lam"], seed=c["seed"]).to(device)
    g = torch.Generator(device=device).manual_seed(c["seed"] + 17 + rank)
    beta = torch.sigmoid(torch.randn(B, H, L, device=device, generator=g))
    y = torch.empty_like(q)
    st = torch.empty(B, H, D, 2 * D, device=device)

    def step():
        ops.delta_prefill(q, k, v, beta, None, lam, chunk=64, lyapunov_bound=25.0, y_out=y, return_state=True)

    steps = max(3, min(args.steps, 10))
    clk = ClockSampler(device.index)
    clk.start()
    ms = max_over_ranks(time_steps(step, steps, args.warmup, ws, device, stream), ws, device)
    clk_r = clk.stop()
    tokheads = B * L * H
    tf = tokheads * DELTA_FLOP_PER_TOKHEAD / (ms * 1e-3) / 1e12
    bw = tokheads * DELTA_BYTES_PER_TOKHEAD / (ms * 1e-3) / 1e9
    pre = {"metric": "delta_prefill_tok_per_s", "value": round(B * L * ws / (ms * 1e-3), 1), "unit": "tok/s",
           "ms_per_step": round(ms, 4), "steps": steps, "higher_is_better": True, "dtype": "bf16 products, f32 solve and state",
           "config": {"workload": "config2 delta-rule prefill on tensor cores: B=8 seqs/GPU, H=12, D=64, L=8192, "
                                  "chunk 64, bf16 "
                                  "q/k/v, beta_t=sigmoid(N(0,1)), alpha_t=lambda_h, Lyapunov bound 25"},
           "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": peaks[1], "unit": "TFLOP/s",
                        "frac": round(tf / peaks[1], 4), "traffic": DELTA_TRAFFIC_B2 * B // 2 if B % 2 == 0 else None,
                        "traffic_note": "both WY kernels, ncu at B=2 scaled to B", "peak_kind": peak_kind,
                        "note": "WY form: a parallel pass over all (head-state, chunk) units (T^-1 in float32 on "
                                "CUDA cores, [U | W] = T^-1 [v | exp(cum) Phi] on tensor cores, 72 KB record per "
                                "unit) then one sequential pass per head-state over the state products "
                                f"({min(B * H, 148)} of 148 SMs); the parallel pass is the longer one",
                        "fp32_cuda_cores": {"achieved": round(tf, 2), "peak": round(FP32_SIMT_PEAK_TFLOPS, 1),
                                            "frac": round(tf / FP32_SIMT_PEAK_TFLOPS, 4),
                                            "peak_kind": "nominal (148 SMs x 128 FMA/clk x 1965 MHz)"},
                        "hbm": {"achieved": round(bw, 1), "peak": hbm_peak, "unit": "GB/s",
                                "frac": round(bw / hbm_peak, 4), "peak_kind": peak_kind},
                        "algorithmic_flop_per_launch": tokheads * DELTA_FLOP_PER_TOKHEAD},
           "gpu_launches": 2 * steps, "clocks": clk_r}
    del q, k, v, y, beta, st
    torch.cuda.empty_cache()

    dc = DECODE
    N, HD = dc["seqs"], dc["layers"] * dc["H"]
    lam_d = synth.make_lambdas(HD, *dc["lam"], seed=dc["seed"]).to(device)
    S = torch.randn(N, HD, D, 2 * D, device=device, generator=g) * dc["sigma"]
    toks = [synth.make_decode_tokens(N, HD, D, seed=dc["seed"] * 100 + i, device=device) for i in range(8)]
    bd = torch.sigmoid(torch.randn(N, HD, device=device, generator=g))
    ad = lam_d.view(1, HD).expand(N, HD).contiguous()
    yd = torch.empty(N, HD, D, dtype=torch.bfloat16, device=device)
    it = [0]

    def dstep():
        qq, kk, vv = toks[it[0] & 7]
        it[0] += 1
        ops.delta_decode_step(qq, kk, vv, bd, ad, S, lyapunov_bound=25.0, inplace=True, y_out=yd)

    dsteps = min(args.decode_steps or 200, 200)
    dclk = ClockSampler(device.index)
    dclk.start()
    dms = max_over_ranks(time_steps(dstep, dsteps, max(3, args.warmup), ws, device, stream), ws, device)
    dclk_r = dclk.stop()
    d_bytes = N * HD * DELTA_DECODE_BYTES_PER_HEADSTEP
    d_bw = d_bytes / (dms * 1e-3) / 1e9
    dec = {"metric": "delta_decode_step_us", "value": round(dms * 1e3, 2), "unit": "us/step",
           "higher_is_better": False, "steps": dsteps,
           "config": {"workload": "config3-shape delta decode: 256 seqs x 12 layers x 12 heads per GPU, D=64, "
                                  "state [D,2D] fp32 in place (1.21 GB), bf16 q/k/v, one launch"},
           "roofline": {"bound": "hbm", "achieved": round(d_bw, 1), "peak": hbm_peak, "unit": "GB/s",
                        "frac": round(d_bw / hbm_peak, 4), "traffic": None, "peak_kind": peak_kind,
                        "algorithmic_bytes_per_launch": d_bytes},
           "gpu_launches": dsteps, "clocks": dclk_r}
    return {"prefill": pre, "decode": dec}


MODEL = dict(vocab=50257, hidden=768, layers=12, heads=12, head_dim=64, mlp=3072, decay=0.9995, batch=64, L=4096,
             new_tokens=256, seed=4)


def bench_model(args, ws, rank, device, stream, peaks):
    """Config 4: PRIME-125M shape (random-init bf16, SwiGLU MLP 3072, tied embeddings, QK-norm) on
    this package's PrimeForCausalLM.  Prefill of 64 sequences x 4096 uniform token ids (split over
    the ranks: data-parallel by sequence, strong scaling), then greedy decode steps from the
    prefilled states with the whole step in one CUDA graph."""
    import torch
    from prime_moment_attention_b200.model import DecodeGraph, PrimeConfig, PrimeForCausalLM
    _, tc_peak, peak_kind = peaks
    c = MODEL
    cfg = PrimeConfig(vocab_size=c["vocab"], hidden_size=c["hidden"], num_layers=c["layers"], num_heads=c["heads"],
                      head_dim=c["head_dim"], intermediate_size=c["mlp"], decay=c["decay"], use_qk_norm=True)
    torch.manual_seed(c["seed"])
    m = PrimeForCausalLM(cfg).to(device, torch.bfloat16).eval()
    B = max(1, c["batch"] // ws)
    g = torch.Generator(device=device).manual_seed(c["seed"] + rank)
    ids = torch.randint(0, c["vocab"], (B, c["L"]), device=device, generator=g)
    with torch.inference_mode():
        def pstep():
            return m(ids, return_states=True, last_logits_only=True)

        clk = ClockSampler(device.index)
        clk.start()
        ms = max_over_ranks(time_steps(pstep, 3, 3, ws, device, stream), ws, device)
        clk_r = clk.stop()
        out = pstep()
        first = torch.argmax(out["logits"][:, -1], dim=-1, keepdim=True)
        dg = DecodeGraph(m, out["states"], first)
        del out
        dms = max_over_ranks(time_steps(dg.step, c["new_tokens"], 3, ws, device, stream), ws, device)
    # per token: 2 x the layer weights (the tied embedding / head is excluded: the head runs on the
    # last position only) + the moment core's chunked work per head and layer
    # this package's launches: per layer and prefill step the QK-norm pass for q and for k, the
    # prefill (a state-only pass and the segment prefix too when the plan splits sequences) and the
    # MLP's fused SwiGLU; per layer in every replay of the decode graph the decode step and SwiGLU
    from prime_moment_attention_b200 import _lib
    seg = _lib.load().pma_prefill_workspace_bytes(B, c["heads"], c["L"], c["head_dim"], _lib.PMA_BF16) > 256
    launches_prefill = 3 * c["layers"] * (2 + (3 if seg else 1) + 1)
    n_params = sum(p.numel() for n, p in m.named_parameters() if "embed" not in n)
    flop_tok = 2 * n_params + c["layers"] * c["heads"] * PREFILL_FLOP_PER_TOKHEAD
    tf = B * c["L"] * flop_tok / (ms * 1e-3) / 1e12
    return {"metric": "model_prefill_tok_per_s", "value": round(B * c["L"] * ws / (ms * 1e-3), 1), "unit": "tok/s",
            "ms_per_step": round(ms, 3), "steps": 3, "higher_is_better": True, "scaling": "strong",
            "dtype": "bf16",
            "config": {"workload": "config4 PRIME-125M shape, random init bf16: 12 layers, d 768, 12x64 heads, "
                                   "SwiGLU 3072 (the reference MLP; BASELINE says GELU), vocab 50257 tied, QK-norm; "
                                   f"{c['batch']} seqs x {c['L']} uniform ids over {ws} GPU(s), last-position logits",
                       "batch_per_gpu": B},
            "decode": {"metric": "model_decode_step_us", "value": round(dms * 1e3, 1), "unit": "us/step",
                       "tok_per_s": round(B * ws / (dms * 1e-3), 1), "steps": c["new_tokens"],
                       "path": "whole greedy step (embed, 12 layers, head, argmax) in one CUDA graph, states in place",
                       "gpu_launches": c["new_tokens"] * c["layers"] * 2},
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": round(tf / tc_peak, 4), "traffic": None, "peak_kind": peak_kind,
                         "flop_per_token": flop_tok},
            "gpu_launches": launches_prefill, "clocks": clk_r}


SP = dict(B=1, H=16, D=128, L=1 << 20, lam=(0.999, 0.99995), seed=6)
SP_FLOP_PER_TOKHEAD = 6 * 64 * 128 + 8 * 128 * 128   # the chunked form at C = 64, D = 128: 180,224 per token-head
SP_BYTES_PER_TOKHEAD = 8 * 128                         # q, k, v in + y out, bf16


def bench_sp(args, ws, rank, device, stream, peaks):
    """Config 5: one sequence of 2^20 tokens, H = 16, D = 128, bf16, split into ws contiguous
    shards (one per rank): a state-only pass per shard, an NCCL all-gather of the shard states,
    the decay-weighted prefix fold and the full pass from the carried state
    (sp.sequence_parallel_prefill).  With one GPU, one pma_prefill over the whole sequence (the
    same carry runs across CTAs as segments).  Total work is fixed: strong scaling."""
    import torch
    from prime_moment_attention_b200 import ops, sp, synth
    hbm_peak, _, peak_kind = peaks
    c = dict(SP, L=args.sp_len or SP["L"])
    Ls = c["L"] // ws
    q, k, v = synth.make_qkv(c["B"], c["H"], Ls, c["D"], seed=c["seed"] + 1000 * rank, dtype=torch.bfloat16,
                             device=device)
    lam = synth.make_lambdas(c["H"], *c["lam"], seed=c["seed"]).to(device)
    y = torch.empty_like(q)
    if ws == 1:
        def step():
            ops.prefill(q, k, v, lam, y_out=y, return_state=True)
    else:
        def step():
            sp.sequence_parallel_prefill(q, k, v, lam, y_out=y, shard_lengths=[Ls] * ws)
    steps = max(3, min(args.steps, 5))
    clk = ClockSampler(device.index)
    clk.start()
    ms = time_steps(step, steps, 3, ws, device, stream)
    clk_r = clk.stop()
    ranks = {"ms_per_step": per_rank(round(ms, 5), ws), "clocks": per_rank(clk_r, ws)}
    ms = max_over_ranks(ms, ws, device)
    tokheads = c["B"] * c["L"] * c["H"]
    tf = tokheads * SP_FLOP_PER_TOKHEAD / (ms * 1e-3) / 1e12
    bw = tokheads * SP_BYTES_PER_TOKHEAD / (ms * 1e-3) / 1e9
    # this package's kernel launches per step (the plan splits a long shard into segments: a
    # state-only pass, the segment prefix and the full pass); with shards, the last rank also runs
    # the state-only prefill of its shard (pass + prefix) and one state combine per earlier shard
    from prime_moment_attention_b200 import _lib
    seg = _lib.load().pma_prefill_workspace_bytes(c["B"], c["H"], Ls, c["D"], _lib.PMA_BF16) > 256
    per_step = (3 if seg else 1) if ws == 1 else (2 if seg else 1) + (ws - 1) + (3 if seg else 1)
    return {"metric": "sp_prefill_tok_per_s", "value": round(c["B"] * c["L"] / (ms * 1e-3), 1), "unit": "tok/s",
            "ms_per_step": round(ms, 3), "steps": steps, "higher_is_better": True, "scaling": "strong",
            "dtype": "bf16",
            "config": {"workload": f"config5 long-sequence prefill: B=1, H=16, D=128, L={c['L']} bf16, per-head lambda "
                                   f"log-U[0.999,0.99995], {ws} contiguous shard(s) of {Ls} tokens",
                       "path": "pma_prefill (tensor cores at D=128, segments across CTAs)" if ws == 1 else
                               "sequence_parallel_prefill: state-only pass, NCCL all_gather, prefix fold, full pass"},
            "roofline": {"bound": "hbm", "achieved": round(bw, 1), "peak": hbm_peak * ws, "unit": "GB/s",
                         "frac": round(bw / (hbm_peak * ws), 4),
                         "traffic": SP_TRAFFIC_1GPU if (ws == 1 and c["L"] == 1 << 20) else None,
                         "traffic_note": "ncu at L=2^16 scaled x16; 1.44x the algorithmic bytes: the state-only "
                                         "pass re-reads k, v of 8 of 9 segments",
                         "peak_kind": f"{peak_kind} per GPU x {ws}",
                         "tensor": {"achieved": round(tf, 2), "peak": round(peaks[1] * ws, 1), "unit": "TFLOP/s",
                                    "frac": round(tf / (peaks[1] * ws), 4)},
                         "algorithmic_bytes_per_step": tokheads * SP_BYTES_PER_TOKHEAD,
                         "algorithmic_flop_per_step": tokheads * SP_FLOP_PER_TOKHEAD},
            "gpu_launches": steps * per_step, "clocks": clk_r, **({"per_rank": ranks} if ws > 1 else {})}


def bench_selective(args, ws, rank, device, stream, peaks):
    """Selective variant at the config-2 shape (per-token decay exp(-Delta_t / tau_h) with
    Delta_t = softplus(N(0,1)), tau_h log-U[2, 2000], beta_h = exp(0.4 N(0,1))) and its decode step
    at the config-3 shape."""
    import torch
    import torch.nn.functional as F
    from prime_moment_attention_b200 import ops, synth
    hbm_peak, _, peak_kind = peaks
    c = PREFILL
    B, H, L, D = args.prefill_batch or c["B"], c["H"], c["L"], c["D"]
    q, k, v = synth.make_qkv(B, H, L, D, seed=c["seed"] + 1000 * rank, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(c["seed"] + 31 + rank)
    tau = torch.exp(torch.empty(H, device=device).uniform_(math.log(2.0), math.log(2000.0), generator=g))
    ld = (-F.softplus(torch.randn(B, H, L, device=device, generator=g)) / tau.view(1, H, 1)).contiguous()
    beta = torch.exp(0.4 * torch.randn(H, device=device, generator=g)).clamp(0.1, 15.0)
    y = torch.empty_like(q)

    def step():
        ops.selective_prefill(q, k, v, ld, beta, y_out=y, return_state=True)

    steps = max(3, min(args.steps, 10))
    clk = ClockSampler(device.index)
    clk.start()
    ms = max_over_ranks(time_steps(step, steps, args.warmup, ws, device, stream), ws, device)
    clk_r = clk.stop()
    tokheads = B * L * H
    bw = tokheads * (PREFILL_BYTES_PER_TOKHEAD + 4) / (ms * 1e-3) / 1e9  # + the fp32 log decay per token-head
    tf = tokheads * PREFILL_FLOP_PER_TOKHEAD / (ms * 1e-3) / 1e12
    pre = {"metric": "selective_prefill_tok_per_s", "value": round(B * L * ws / (ms * 1e-3), 1), "unit": "tok/s",
           "ms_per_step": round(ms, 4), "steps": steps, "higher_is_better": True, "dtype": "bf16",
           "config": {"workload": "config2-shape selective prefill: B=8 seqs/GPU, H=12, D=64, L=8192, bf16 q/k/v, "
                                  "per-token decay exp(-softplus(N(0,1))/tau_h), tau_h log-U[2,2000], beta_h "
                                  "exp(0.4 N(0,1)); tensor cores (head-states with a chunk decaying past e^-76 "
                                  "run the float32 loop)"},
           "roofline": {"bound": "hbm", "achieved": round(bw, 1), "peak": hbm_peak, "unit": "GB/s",
                        "frac": round(bw / hbm_peak, 4), "traffic": None, "peak_kind": peak_kind,
                        "tensor": {"achieved": round(tf, 1), "peak": peaks[1], "unit": "TFLOP/s",
                                   "frac": round(tf / peaks[1], 4)},
                        "algorithmic_bytes_per_launch": tokheads * (PREFILL_BYTES_PER_TOKHEAD + 4)},
           "gpu_launches": steps, "clocks": clk_r}
    del q, k, v, y, ld
    torch.cuda.empty_cache()
    dc = DECODE
    N, HD = dc["seqs"], dc["layers"] * dc["H"]
    lam_d = synth.make_lambdas(HD, *dc["lam"], seed=dc["seed"]).to(device)
    st = synth.make_state(N, HD, D, lam_d, seed=dc["seed"] + rank, t0=dc["t0"], sigma=dc["sigma"], device=device)
    toks = [synth.make_decode_tokens(N, HD, D, seed=dc["seed"] * 100 + i, device=device) for i in range(8)]
    ldd = (-F.softplus(torch.randn(N, HD, device=device, generator=g)) / 500.0).contiguous()
    bd = torch.exp(0.4 * torch.randn(HD, device=device, generator=g)).clamp(0.1, 15.0)
    yd = torch.empty(N, HD, D, dtype=torch.bfloat16, device=device)
    it = [0]

    def dstep():
        qq, kk, vv = toks[it[0] & 7]
        it[0] += 1
        ops.selective_decode_step(qq, kk, vv, ldd, bd, st, inplace=True, y_out=yd)

    dsteps = min(args.decode_steps or 200, 200)
    dclk = ClockSampler(device.index)
    dclk.start()
    dms = max_over_ranks(time_steps(dstep, dsteps, max(3, args.warmup), ws, device, stream), ws, device)
    dclk_r = dclk.stop()
    d_bytes = N * HD * (DECODE_BYTES_PER_HEADSTEP + 4)
    d_bw = d_bytes / (dms * 1e-3) / 1e9
    dec = {"metric": "selective_decode_step_us", "value": round(dms * 1e3, 2), "unit": "us/step",
           "higher_is_better": False, "steps": dsteps,
           "config": {"workload": "config3-shape selective decode: 256 seqs x 12 layers x 12 heads, D=64, "
                                  "per-token decay, fp32 state in place"},
           "roofline": {"bound": "hbm", "achieved": round(d_bw, 1), "peak": hbm_peak, "unit": "GB/s",
                        "frac": round(d_bw / hbm_peak, 4), "traffic": None, "peak_kind": peak_kind,
                        "algorithmic_bytes_per_launch": d_bytes},
           "gpu_launches": dsteps, "clocks": dclk_r}
    return {"prefill": pre, "decode": dec}


def _with_summary(line: dict) -> dict:
    """The line with a compact `summary` of every part right after the headline keys, so that a
    reader that keeps only the first keys or the head of the line sees all the numbers."""
    s = {}

    def put(key, part, frac=True):
        if isinstance(part, dict) and "value" in part:
            s[key] = part["value"]
            if frac and isinstance(part.get("roofline"), dict):
                s[key + "_frac"] = part["roofline"].get("frac")

    put("prefill_ms", {"value": line.get("ms_per_step"), "roofline": line.get("roofline")})
    put("e2e_tok_s", line.get("e2e"), frac=False)
    put("decode_us", line.get("decode"))
    for name in ("selective", "delta"):
        part = line.get(name) or {}
        put(f"{name}_prefill_ms", {"value": (part.get("prefill") or {}).get("ms_per_step"),
                                   "roofline": (part.get("prefill") or {}).get("roofline")})
        put(f"{name}_decode_us", part.get("decode"))
    sp = line.get("sp") or {}
    put("sp_ms", {"value": sp.get("ms_per_step"), "roofline": sp.get("roofline")})
    md = line.get("model") or {}
    put("model_prefill_ms", {"value": md.get("ms_per_step"), "roofline": md.get("roofline")})
    put("model_decode_us", md.get("decode"), frac=False)
    head = [k for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step") if k in line]
    out = {k: line[k] for k in head}
    out["summary"] = {k: v for k, v in s.items() if v is not None}
    out.update({k: v for k, v in line.items() if k not in out})
    return out


def run_ours(args):
    import torch
    ws, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    peaks = _peaks()
    line = {}
    if args.workload in ("both", "prefill"):
        line = bench_prefill(args, ws, rank, device, stream, peaks)
        torch.cuda.empty_cache()
    if args.workload in ("both", "decode"):
        dec = bench_decode(args, ws, rank, device, stream, peaks)
        if line:
            line["decode"] = dec
        else:
            line = dict(dec, n_gpus=ws, warmup=args.warmup, scaling="weak", dtype="bf16", data="synthetic",
                        vs_baseline=None)
        torch.cuda.empty_cache()
    if args.workload in ("both", "model"):
        md = bench_model(args, ws, rank, device, stream, peaks)
        if line:
            line["model"] = md
        else:
            line = dict(md, n_gpus=ws, warmup=args.warmup, data="synthetic", vs_baseline=None)
        torch.cuda.empty_cache()
    if args.workload in ("both", "sp"):
        spl = bench_sp(args, ws, rank, device, stream, peaks)
        if line:
            line["sp"] = spl
        else:
            line = dict(spl, n_gpus=ws, warmup=args.warmup, data="synthetic", vs_baseline=None)
        torch.cuda.empty_cache()
    if args.workload in ("both", "selective"):
        sl = bench_selective(args, ws, rank, device, stream, peaks)
        if line:
            line["selective"] = sl
        else:
            line = dict(sl["prefill"], n_gpus=ws, warmup=args.warmup, scaling="weak", data="synthetic",
                        vs_baseline=None, selective_decode=sl["decode"])
        torch.cuda.empty_cache()
    if args.workload in ("both", "delta"):
        dl = bench_delta(args, ws, rank, device, stream, peaks)
        if line:
            line["delta"] = dl
        else:
            line = dict(dl["prefill"], n_gpus=ws, warmup=args.warmup, scaling="weak", data="synthetic",
                        vs_baseline=None, delta_decode=dl["decode"])
        torch.cuda.empty_cache()
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and ref_bench_path():
        try:
            if "decode" in line:
                line["decode"]["cpu_baseline"] = cpu_decode_sample()
            if line.get("metric") == "prefill_tok_per_s":
                line["cpu_baseline"] = cpu_prefill_sample()
        except Exception as e:  # the baseline must not sink the GPU number
            line["cpu_baseline"] = {"error": str(e)[:200]}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        # the reference's PyTorch path timed on the same host cores, beside its C99 runtime
        for key, fn, where in (("prefill", cpu_pytorch_prefill_sample, line),
                               ("decode", cpu_pytorch_decode_sample, line.get("decode"))):
            if where is None or (key == "prefill" and line.get("metric") != "prefill_tok_per_s"):
                continue
            try:
                where["cpu_baseline_pytorch"] = fn()
            except Exception as e:  # the baseline must not sink the GPU number
                where["cpu_baseline_pytorch"] = {"error": str(e)[:200]}
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and "delta" in line:
        try:
            line["delta"]["prefill"]["cpu_baseline"] = cpu_delta_sample()
        except Exception as e:
            line["delta"]["prefill"]["cpu_baseline"] = {"error": str(e)[:200]}
    if rank == 0:
        print(json.dumps(_with_summary(line)))
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["both", "prefill", "decode", "delta", "model", "selective", "sp"], default="both",
                    help="profiling aid: run only one part (the JSON line then lacks the others)")
    ap.add_argument("--prefill-batch", type=int, default=0,
                    help="profiling aid: sequences per GPU for the prefill part (default: config 2's 8)")
    ap.add_argument("--decode-steps", type=int, default=0,
                    help="profiling aid: timed decode steps (default 1000)")
    ap.add_argument("--sp-len", type=int, default=0,
                    help="profiling aid: sequence length of the config-5 part (default 2^20)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
