"""Torch-facing wrappers of the C ABI: prefill, decode_step, state_combine.

Tensors stay on the GPU; every call goes through libpma.so on the current CUDA
stream.  Inputs that are not CUDA tensors raise (no CPU fallback).

State tuples use the reference layout (src/prime_moment_attention/attention.py:111-117):
(S0[B,H,D], S1[B,H,D,D], S2[B,H,D,D], K0[B,H,1], K1[B,H,D], K2[B,H,D]), float32.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence, Tuple, Union

import torch

from . import _lib

StateTuple = Tuple[torch.Tensor, ...]
Decay = Union[float, Sequence[float], torch.Tensor]

_DT = {torch.float32: _lib.PMA_F32, torch.bfloat16: _lib.PMA_BF16}
_lam_cache: dict = {}


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError("prime_moment_attention_b200 runs on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _seq_ok(t: torch.Tensor) -> bool:
    step = 16 // t.element_size()
    return (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
            and all(s % step == 0 and s >= 0 for s in t.stride()[:-1]))


def _seq(t: torch.Tensor, four_d: bool = True) -> Tuple[_lib.SeqTensor, torch.Tensor]:
    """pma_seq_tensor for a [B,H,L,D] (or [N,H,D]) tensor, copying only if the
    kernels cannot address its layout."""
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}: float32 or bfloat16")
    if not _seq_ok(t):
        t = t.contiguous()
    if four_d:
        sb, sh, sl, _ = t.stride()
    else:
        sb, sh, _ = t.stride()
        sl = 0
    return _lib.SeqTensor(t.data_ptr(), _DT[t.dtype], sb, sh, sl), t


def _state(st: StateTuple, B: int, H: int, D: int, name: str) -> Tuple[_lib.State, StateTuple]:
    if len(st) != 6:
        raise ValueError(f"{name}: expected a 6-tuple (S0, S1, S2, K0, K1, K2)")
    shapes = [(B, H, D), (B, H, D, D), (B, H, D, D), (B, H, 1), (B, H, D), (B, H, D)]
    out = []
    for i, (t, shp) in enumerate(zip(st, shapes)):
        if tuple(t.shape) != shp:
            if i == 3 and t.numel() == B * H:
                t = t.reshape(B, H, 1)
            else:
                raise ValueError(f"{name}[{i}] has shape {tuple(t.shape)}, expected {shp}")
        if t.dtype != torch.float32 or not t.is_contiguous() or t.data_ptr() % 16:
            t = t.to(torch.float32).contiguous()
        out.append(t)
    return _lib.State(*[t.data_ptr() for t in out]), tuple(out)


def new_state(B: int, H: int, D: int, device, zero: bool = True) -> StateTuple:
    """(S0, S1, S2, Z0, Z1, Z2) as contiguous slices of one allocation (one allocator call per
    state; Z0 is placed last so that every other part starts 16-byte aligned)."""
    BH = B * H
    flat = (torch.zeros if zero else torch.empty)(BH * (2 * D * D + 3 * D + 1), device=device)
    o = [0, BH * D, BH * D * (D + 1), BH * D * (2 * D + 1), BH * D * (2 * D + 2), BH * D * (2 * D + 3)]
    S0 = flat[o[0]:o[1]].view(B, H, D)
    S1 = flat[o[1]:o[2]].view(B, H, D, D)
    S2 = flat[o[2]:o[3]].view(B, H, D, D)
    Z1 = flat[o[3]:o[4]].view(B, H, D)
    Z2 = flat[o[4]:o[5]].view(B, H, D)
    Z0 = flat[o[5]:].view(B, H, 1)
    return (S0, S1, S2, Z0, Z1, Z2)


def lambda_tensor(decay: Decay, B: int, H: int, device) -> Tuple[torch.Tensor, int]:
    """Device float32 decay table and its batch stride: scalar or [H] -> ([H], 0), [B,H] -> ([B*H], H)."""
    if isinstance(decay, torch.Tensor):
        lam = decay.detach().to(device=device, dtype=torch.float32)
    else:
        if isinstance(decay, (int, float)):
            key = (str(device), H, float(decay))
            t = _lam_cache.get(key)
            if t is None:
                t = torch.full((H,), float(decay), dtype=torch.float32, device=device)
                _lam_cache[key] = t
            return t, 0
        lam = torch.tensor(list(decay), dtype=torch.float32, device=device)
    if lam.dim() == 0:
        lam = lam.expand(H)
    if lam.shape == (H,):
        return lam.contiguous(), 0
    if lam.shape == (B, H):
        return lam.contiguous().reshape(B * H), H
    raise ValueError(f"decay must be a scalar, [H] or [B,H]; got shape {tuple(lam.shape)}")


@dataclass
class Prologue:
    """Module work between the projections and the core, folded into the kernels' loads
    (pma_prologue): k and v carry H / kv_groups heads and query head h reads kv head
    h // kv_groups (the reference's repeat_interleave, attention.py:92-94); q and k get a
    LayerNorm over the head dim when their weight is given (attention.py:96-98); q is then
    multiplied by q_scale (attention.py:101).  Weights and biases are [D] tensors."""
    kv_groups: int = 1
    q_scale: float = 1.0
    q_norm_weight: Optional[torch.Tensor] = None
    q_norm_bias: Optional[torch.Tensor] = None
    k_norm_weight: Optional[torch.Tensor] = None
    k_norm_bias: Optional[torch.Tensor] = None
    norm_eps: float = 1e-5

    def to_c(self, D: int, device) -> Tuple[_lib.Prologue, list]:
        """The C struct and the float32 device tensors it points to (keep them alive)."""
        keep = []

        def ptr(t):
            if t is None:
                return None
            if t.numel() != D:
                raise ValueError(f"prologue norm parameters must have head_dim={D} elements")
            if t.device != device or t.dtype != torch.float32 or not t.is_contiguous():
                t = t.detach().to(device=device, dtype=torch.float32).contiguous()
            keep.append(t)
            return t.data_ptr()

        c = _lib.Prologue(int(self.kv_groups), float(self.q_scale), ptr(self.q_norm_weight), ptr(self.q_norm_bias),
                          ptr(self.k_norm_weight), ptr(self.k_norm_bias), float(self.norm_eps))
        return c, keep


def _kv_heads(H: int, prologue: Optional[Prologue]) -> int:
    g = 1 if prologue is None else int(prologue.kv_groups)
    if g < 1 or H % g:
        raise ValueError(f"kv_groups={g} must be a positive divisor of num_heads={H}")
    return H // g


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class KernelFault(RuntimeError):
    """A tensor-core prefill launch gave up: one of its bounded waits expired, so its outputs
    were not written.  `code` identifies the wait."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: a tensor-core prefill launch recorded fault code {code} "
                         "(a bounded wait expired; its outputs were not written)")


_fault: Optional[torch.Tensor] = None  # pinned host int32 registered as the library's fault word
_fault_view = None                     # numpy view of it: a plain memory read per check


def _arm_faults() -> None:
    """Register a pinned host word as the library's fault word (once per process).  Pinned host
    memory from cudaHostAlloc is addressable by every device, and the host reads it without
    synchronising, so a fault is seen by the next call on any device."""
    global _fault, _fault_view
    if _fault is None:
        word = torch.zeros(1, dtype=torch.int32).pin_memory()
        _lib.load().pma_set_fault_word(word.data_ptr())
        _fault, _fault_view = word, word.numpy()


def pending_fault() -> int:
    """Code recorded by a finished tensor-core prefill launch since the last check (0 if none).
    Does not synchronise: a launch still running has not reported yet."""
    return int(_fault_view[0]) if _fault is not None else 0


def check_faults(where: str = "prime_moment_attention_b200", synchronize: bool = False) -> None:
    """Raise KernelFault (and clear the word) if a tensor-core prefill launch gave up.  Every
    prefill entry of this module calls it before launching, so a fault surfaces at the next call
    at the latest; synchronize=True first waits for the device's work."""
    _arm_faults()
    if synchronize:
        torch.cuda.synchronize()
    code = int(_fault_view[0])
    if code:
        _fault_view[0] = 0
        raise KernelFault(code, where)


def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, decay: Decay,
            state: Optional[StateTuple] = None, eps: float = 1.0, return_state: bool = True,
            out_dtype: Optional[torch.dtype] = None, y_out: Optional[torch.Tensor] = None,
            want_y: bool = True, check: bool = False, prologue: Optional[Prologue] = None,
            workspace: Optional[torch.Tensor] = None, resume: bool = False):
    """Chunked prefill over q, k, v [B,H,L,D] (q pre-scaled by 1/sqrt(D)).

    Returns (y [B,H,L,D] or None, final state or None).  `y_out` may be a
    preallocated [B,H,L,D] view with any strides (e.g. a transpose of [B,L,H,D]).
    `want_y=False` runs the state-only pass.  A tensor-core launch that gives up (a bounded wait
    expired) raises KernelFault at the next prefill call of this module, or here with `check=True`,
    which synchronises and reads the call's workspace status word and the fault word.
    With a `prologue`, q, k, v are the raw projections (k, v with H / kv_groups heads)
    and the kernels apply the GQA map, QK-norm and q scale as they load them.
    `workspace` (uint8 device tensor, at least pma_prefill_workspace_bytes) replaces the per-call
    allocation; with `resume=True` it must be the workspace of a state-only call (want_y=False,
    state=None) on the same inputs, and the call runs only the output pass from `state`
    (pma_prefill_resume)."""
    dev = _require_cuda(q, k, v)
    check_faults("prefill")
    if q.dim() != 4:
        raise ValueError(f"q must be [B,H,L,D]; got {tuple(q.shape)}")
    B, H, L, D = q.shape
    kv_shape = (B, _kv_heads(H, prologue), L, D)
    if tuple(k.shape) != kv_shape or tuple(v.shape) != kv_shape:
        raise ValueError(f"q, k, v must be [B,H,L,D] and [B,H/kv_groups,L,D]; got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share one dtype")
    L_ = _lib.load()
    qs, q = _seq(q)
    ks, k = _seq(k)
    vs, v = _seq(v)
    lam, lam_sb = lambda_tensor(decay, B, H, dev)
    st_in = None
    if state is not None:
        st_in_c, state = _state(state, B, H, D, "state")
        st_in = ctypes.byref(st_in_c)
    st_out_t = new_state(B, H, D, dev, zero=False) if return_state else None
    st_out = ctypes.byref(_lib.State(*[t.data_ptr() for t in st_out_t])) if return_state else None
    y = None
    ys = None
    if want_y:
        if y_out is not None:
            if tuple(y_out.shape) != (B, H, L, D) or not _seq_ok(y_out):
                raise ValueError("y_out must be a [B,H,L,D] tensor with a contiguous, 16-byte aligned last axis")
            y = y_out
        else:
            y = torch.empty(B, H, L, D, dtype=out_dtype or q.dtype, device=dev)
        ys_c, _ = _seq(y)
        ys = ctypes.byref(ys_c)
    if prologue is None:
        ws_bytes = L_.pma_prefill_workspace_bytes(B, H, L, D, _DT[q.dtype])
    else:
        pc, keep = prologue.to_c(D, dev)
        ws_bytes = L_.pma_prefill_ex_workspace_bytes(B, H, L, D, _DT[q.dtype], ctypes.byref(pc))
    if resume and (prologue is not None or not want_y or workspace is None):
        raise ValueError("resume=True needs want_y, no prologue and the state-only call's workspace")
    if workspace is not None:
        if (workspace.dtype != torch.uint8 or workspace.device != dev or not workspace.is_contiguous()
                or workspace.numel() < ws_bytes):
            raise ValueError(f"workspace must be a contiguous uint8 tensor of at least {ws_bytes} bytes on {dev}")
        ws = workspace if ws_bytes else None
    else:
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    wsp = ws.data_ptr() if ws is not None else None
    if resume:
        rc = L_.pma_prefill_resume(B, H, L, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), lam.data_ptr(),
                                   lam_sb, st_in, st_out, float(eps), ys, wsp, ws_bytes, _stream(dev))
        _lib.check("pma_prefill_resume", rc)
    elif prologue is None:
        rc = L_.pma_prefill(B, H, L, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), lam.data_ptr(),
                            lam_sb, st_in, st_out, float(eps), ys, wsp, ws_bytes, _stream(dev))
        _lib.check("pma_prefill", rc)
    else:
        rc = L_.pma_prefill_ex(B, H, L, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), ctypes.byref(pc),
                               lam.data_ptr(), lam_sb, st_in, st_out, float(eps), ys, wsp, ws_bytes, _stream(dev))
        _lib.check("pma_prefill_ex", rc)
    if check:
        code = int(ws[:4].view(torch.int32).item()) if ws is not None else 0  # synchronises
        if code != 0:
            _fault_view[0] = 0
            raise KernelFault(code, "pma_prefill (workspace status word)")
        check_faults("pma_prefill")
    return y, st_out_t


def prefill_workspace(q: torch.Tensor) -> torch.Tensor:
    """A workspace for prefill() calls on inputs shaped like q [B,H,L,D] (no prologue)."""
    B, H, L, D = q.shape
    n = _lib.load().pma_prefill_workspace_bytes(B, H, L, D, _DT[q.dtype])
    return torch.empty(max(n, 1), dtype=torch.uint8, device=q.device)


def swiglu(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(gate) * up in one pass (pma_swiglu): gate and up [..., I] on the GPU (bf16 or float32, last
    axis contiguous, leading axes flattenable to rows with one stride, e.g. column halves of one
    [N, 2I] GEMM output).  Same values as F.silu(gate) * up."""
    dev = _require_cuda(gate, up)
    if gate.shape != up.shape or gate.dtype != up.dtype or gate.dtype not in _DT:
        raise ValueError("gate and up must have one shape and a bf16 or float32 dtype")
    I = gate.shape[-1]
    g2, u2 = gate.reshape(-1, I), up.reshape(-1, I)  # views where the layout allows
    if g2.stride(-1) != 1 or u2.stride(-1) != 1:
        g2, u2 = g2.contiguous(), u2.contiguous()
    if out is None:
        out = torch.empty(gate.shape, dtype=gate.dtype, device=dev)
    elif (not isinstance(out, torch.Tensor) or tuple(out.shape) != tuple(gate.shape) or out.dtype != gate.dtype
          or out.device != dev):
        raise ValueError(f"out must be a {gate.dtype} tensor of shape {tuple(gate.shape)} on {dev}")
    try:
        o2 = out.view(-1, I)
    except RuntimeError as e:
        raise ValueError("out must flatten to [rows, I] rows of one stride") from e
    if o2.stride(-1) != 1:
        raise ValueError("out must have a contiguous last axis")
    rc = _lib.load().pma_swiglu(g2.shape[0], I, g2.data_ptr(), g2.stride(0), u2.data_ptr(), u2.stride(0),
                                o2.data_ptr(), o2.stride(0), _DT[gate.dtype], _stream(dev))
    _lib.check("pma_swiglu", rc)
    return out


_copy_streams = {}
_host_staging = {}  # device index -> (key, (q, k, v, y) device staging buffers)
_inputs_free = {}   # device index -> event after the last kernels that read the q, k, v staging buffers


def release_host_staging():
    """Free the device staging buffers that prefill_from_host keeps between calls."""
    _host_staging.clear()
    _inputs_free.clear()


def _staging(dev, q, k, v, y_dtype):
    """Device buffers for prefill_from_host, kept per device for the last shapes used (reusing them
    avoids an allocation per call; call order on the streams keeps successive calls apart)."""
    key = (tuple(q.shape), tuple(k.shape), tuple(v.shape), q.dtype, y_dtype)
    hit = _host_staging.get(dev.index)
    if hit is None or hit[0] != key:
        _host_staging.pop(dev.index, None)
        _inputs_free.pop(dev.index, None)  # new buffers: the first copies wait for the current stream
        bufs = tuple(torch.empty(t.shape, dtype=t.dtype, device=dev) for t in (q, k, v))
        bufs += (torch.empty(q.shape, dtype=y_dtype, device=dev),)
        hit = (key, bufs)
        _host_staging[dev.index] = hit
    return hit[1]


def _copy_stream_pair(device):
    """Two side streams per device (host->device, device->host), created once."""
    key = torch.device(device).index
    pair = _copy_streams.get(key)
    if pair is None:
        pair = (torch.cuda.Stream(device), torch.cuda.Stream(device))
        _copy_streams[key] = pair
    return pair


def prefill_from_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, decay: Decay, device=None,
                      state: Optional[StateTuple] = None, eps: float = 1.0, return_state: bool = True,
                      y_host: Optional[torch.Tensor] = None, pieces: Optional[int] = None,
                      prologue: Optional[Prologue] = None):
    """prefill() for inputs and output in host memory: q, k, v [B,H,L,D] on the CPU (pinned, or the
    copies cannot overlap), y returned in `y_host` (pinned [B,H,L,D] of q's dtype; allocated pinned
    if None).  The batch runs in `pieces` slices (default: one per batch row, at most 8): the
    host->device copy of a slice, the kernels of the previous slice and the device->host copy of
    the one before overlap, on two side streams and the current stream (PCIe carries both
    directions at once).  The current stream's work after this call sees y_host complete; the
    caller synchronises before reading it on the host.  `state` (on the device) and the returned
    final state (on the device, unless return_state=False) are as in prefill().  Device staging
    buffers for q, k, v, y are kept between calls (release_host_staging() frees them)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if q.is_cuda or k.is_cuda or v.is_cuda:
        raise ValueError("prefill_from_host takes q, k, v in host memory; use prefill() for device tensors")
    if q.dim() != 4:
        raise ValueError(f"q must be [B,H,L,D]; got {tuple(q.shape)}")
    B, H, L, D = q.shape
    if y_host is None:
        y_host = torch.empty(B, H, L, D, dtype=q.dtype, pin_memory=True)
    elif tuple(y_host.shape) != (B, H, L, D) or y_host.is_cuda:
        raise ValueError("y_host must be a host [B,H,L,D] tensor")
    P = max(1, min(B, pieces if pieces is not None else min(B, 8)))
    bounds = [B * i // P for i in range(P + 1)]
    cur = torch.cuda.current_stream(dev)
    h2d, d2h = _copy_stream_pair(dev)
    qd, kd, vd, yd = _staging(dev, q, k, v, y_host.dtype)
    lam, lam_sb = lambda_tensor(decay, B, H, dev)
    free = _inputs_free.get(dev.index)
    if free is None:
        h2d.wait_stream(cur)  # fresh staging buffers: everything queued before this call comes first
    else:
        # the previous call's kernels are done with the input staging buffers; its last copies back
        # (device->host, on the other side stream) may still run while these copies in start
        h2d.wait_event(free)
    states = []
    for i in range(P):
        sl = slice(bounds[i], bounds[i + 1])
        if sl.start == sl.stop:
            continue
        with torch.cuda.stream(h2d):
            for dst, src in ((qd, q), (kd, k), (vd, v)):
                dst[sl].copy_(src[sl], non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(h2d)
        cur.wait_event(landed)
        lam_i = lam if lam_sb == 0 else lam.view(B, H)[sl]
        st_i = None if state is None else tuple(t[sl] for t in state)
        _, st = prefill(qd[sl], kd[sl], vd[sl], lam_i, state=st_i, eps=eps, return_state=return_state,
                        y_out=yd[sl], prologue=prologue)
        states.append(st)
        done = torch.cuda.Event()
        done.record(cur)
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            y_host[sl].copy_(yd[sl], non_blocking=True)
    free = torch.cuda.Event()
    free.record(cur)
    _inputs_free[dev.index] = free
    cur.wait_stream(d2h)  # later work on the current stream (a next call's kernels) follows the copies out
    final = None
    if return_state:
        final = states[0] if len(states) == 1 else tuple(torch.cat(parts, dim=0) for parts in zip(*states))
    return y_host, final


def decode_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, decay: Decay, state: StateTuple,
                eps: float = 1.0, inplace: bool = False, out_dtype: Optional[torch.dtype] = None,
                y_out: Optional[torch.Tensor] = None, prologue: Optional[Prologue] = None):
    """One recurrent step: q, k, v [N,H,D] -> (y [N,H,D], new state).

    With inplace=True the given state tensors are updated and returned (they must
    already be contiguous float32); otherwise fresh tensors are returned and the
    input state is left untouched, as in the reference (attention.py:126-132).
    `prologue` as in prefill (k, v then [N, H / kv_groups, D])."""
    dev = _require_cuda(q, k, v)
    N, H, D = _check_step_shapes(q, k, v, prologue)
    L_ = _lib.load()
    qs, q = _seq(q, False)
    ks, k = _seq(k, False)
    vs, v = _seq(v, False)
    lam, lam_sn = lambda_tensor(decay, N, H, dev)
    st_in_c, st_in_t = _state(state, N, H, D, "state")
    if inplace:
        if any(a is not b for a, b in zip(st_in_t, state)) and not all(
                a.data_ptr() == b.data_ptr() for a, b in zip(st_in_t, state)):
            raise ValueError("inplace=True needs contiguous float32 state tensors")
        st_out_t = st_in_t
    else:
        st_out_t = new_state(N, H, D, dev, zero=False)
    st_out_c = _lib.State(*[t.data_ptr() for t in st_out_t])
    y = y_out if y_out is not None else torch.empty(N, H, D, dtype=out_dtype or q.dtype, device=dev)
    ys, y2 = _seq(y, False)
    if y2 is not y:
        raise ValueError("y_out must have a contiguous, 16-byte aligned last axis")
    if prologue is None:
        rc = L_.pma_decode_step(N, H, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), lam.data_ptr(),
                                lam_sn, ctypes.byref(st_in_c), ctypes.byref(st_out_c), float(eps), ctypes.byref(ys),
                                _stream(dev))
        _lib.check("pma_decode_step", rc)
    else:
        pc, keep = prologue.to_c(D, dev)
        rc = L_.pma_decode_step_ex(N, H, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), ctypes.byref(pc),
                                   lam.data_ptr(), lam_sn, None, 0, ctypes.byref(st_in_c), ctypes.byref(st_out_c),
                                   float(eps), ctypes.byref(ys), _stream(dev))
        _lib.check("pma_decode_step_ex", rc)
    return y, st_out_t


def _check_step_shapes(q, k, v, prologue):
    if q.dim() != 3:
        raise ValueError("q must be [N,H,D]")
    N, H, D = q.shape
    kv_shape = (N, _kv_heads(H, prologue), D)
    if tuple(k.shape) != kv_shape or tuple(v.shape) != kv_shape:
        raise ValueError(f"q, k, v must be [N,H,D] and [N,H/kv_groups,D]; got {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    return N, H, D


def decode_step_rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, decay: Decay, pool: StateTuple,
                     rows: torch.Tensor, eps: float = 1.0, out_dtype: Optional[torch.dtype] = None,
                     y_out: Optional[torch.Tensor] = None, prologue: Optional[Prologue] = None) -> torch.Tensor:
    """One recurrent step for batch rows n = 0..N-1 whose states are rows rows[n] of `pool`.

    `pool` is a state tuple [P, H, ...] (contiguous float32, updated in place); `rows` an int32
    CUDA tensor [N] of pool rows (rows outside [0, P) are skipped and their y rows untouched).
    `prologue` as in prefill.  Returns y [N, H, D]."""
    dev = _require_cuda(q, k, v)
    N, H, D = _check_step_shapes(q, k, v, prologue)
    P = pool[0].shape[0]
    if rows.dtype != torch.int32 or rows.dim() != 1 or rows.shape[0] != N or rows.device != dev:
        raise ValueError("rows must be an int32 tensor [N] on the inputs' device")
    rows = rows.contiguous()
    L_ = _lib.load()
    qs, q = _seq(q, False)
    ks, k = _seq(k, False)
    vs, v = _seq(v, False)
    lam, lam_sn = lambda_tensor(decay, N, H, dev)
    pool_c, pool_t = _state(pool, P, H, D, "pool")
    if not all(a.data_ptr() == b.data_ptr() for a, b in zip(pool_t, pool)):
        raise ValueError("the pool must be contiguous float32 (it is updated in place)")
    y = y_out if y_out is not None else torch.empty(N, H, D, dtype=out_dtype or q.dtype, device=dev)
    ys, y2 = _seq(y, False)
    if y2 is not y:
        raise ValueError("y_out must have a contiguous, 16-byte aligned last axis")
    if prologue is None:
        rc = L_.pma_decode_step_rows(N, H, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), lam.data_ptr(),
                                     lam_sn, rows.data_ptr(), P, ctypes.byref(pool_c), ctypes.byref(pool_c),
                                     float(eps), ctypes.byref(ys), _stream(dev))
        _lib.check("pma_decode_step_rows", rc)
    else:
        pc, keep = prologue.to_c(D, dev)
        rc = L_.pma_decode_step_ex(N, H, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), ctypes.byref(pc),
                                   lam.data_ptr(), lam_sn, rows.data_ptr(), P, ctypes.byref(pool_c),
                                   ctypes.byref(pool_c), float(eps), ctypes.byref(ys), _stream(dev))
        _lib.check("pma_decode_step_ex", rc)
    return y


def state_combine(T: StateTuple, P: StateTuple, decay: Decay, length: int) -> StateTuple:
    """P <- decay^length * P + T in place (P must be contiguous float32); returns P."""
    dev = _require_cuda(T[1], P[1])
    B, H, D = P[0].shape
    L_ = _lib.load()
    Tc, T = _state(T, B, H, D, "T")
    Pc, P2 = _state(P, B, H, D, "P")
    if any(a.data_ptr() != b.data_ptr() for a, b in zip(P2, P)):
        raise ValueError("P must be contiguous float32 (it is updated in place)")
    lam, lam_sb = lambda_tensor(decay, B, H, dev)
    rc = L_.pma_state_combine(B, H, D, lam.data_ptr(), lam_sb, int(length), ctypes.byref(Tc), ctypes.byref(Pc),
                              _stream(dev))
    _lib.check("pma_state_combine", rc)
    return P


# ---------------------------------------------------------------- gated delta-rule variant
def _gate(t, shape, dev, name):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor):
        t = torch.tensor(t, dtype=torch.float32)
    t = t.to(device=dev, dtype=torch.float32)
    if tuple(t.shape) != tuple(shape):
        if t.numel() == int(torch.tensor(shape).prod()):
            t = t.reshape(shape)
        else:
            raise ValueError(f"{name} must have shape {tuple(shape)}; got {tuple(t.shape)}")
    return t.contiguous()


def delta_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                  alpha: Optional[torch.Tensor], decay: Decay, chunk: int = 64, lyapunov_bound: float = 25.0,
                  norm_eps: float = 1e-5, state: Optional[torch.Tensor] = None, return_state: bool = True,
                  out_dtype: Optional[torch.dtype] = None, y_out: Optional[torch.Tensor] = None,
                  want_y: bool = True, wy: bool = True, workspace_bytes: Optional[int] = None):
    """Gated delta-rule chunked prefill (ChunkedGatedDeltaPrimeAttention's L > 1 core).

    q (pre-scaled), k, v [B,H,L,D]; beta, alpha [B,H,L] float (alpha None: the decay);
    decay: the module's decay (scalar, [H] or [B,H]) -- the padded tokens of a ragged last
    chunk decay by it, as in the reference; state [B,H,D,2D] float32 or None.
    wy: give the library the workspace of its WY path (bf16, D = 64, chunk 64); False runs the
    single-pass tensor-core kernel instead.  workspace_bytes: a smaller workspace than the
    library's preferred one (the sequence then runs in windows of chunks).
    Returns (y [B,H,L,D] or None, final state [B,H,D,2D] or None)."""
    dev = _require_cuda(q, k, v)
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must share one [B,H,L,D] shape")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share one dtype")
    B, H, L, D = q.shape
    check_faults("delta_prefill")
    L_ = _lib.load()
    qs, q = _seq(q)
    ks, k = _seq(k)
    vs, v = _seq(v)
    beta = _gate(beta, (B, H, L), dev, "beta")
    alpha = _gate(alpha, (B, H, L), dev, "alpha")
    lam, lam_sb = lambda_tensor(decay, B, H, dev)
    st_in = None
    if state is not None:
        st_in = state.to(device=dev, dtype=torch.float32).reshape(B, H, D, 2 * D).contiguous()
    st_out = torch.empty(B, H, D, 2 * D, device=dev) if return_state else None
    y = ys = None
    if want_y:
        if y_out is not None:
            if tuple(y_out.shape) != (B, H, L, D) or not _seq_ok(y_out):
                raise ValueError("y_out must be a [B,H,L,D] tensor with a contiguous, 16-byte aligned last axis")
            y = y_out
        else:
            y = torch.empty(B, H, L, D, dtype=out_dtype or q.dtype, device=dev)
        ys = ctypes.byref(_seq(y)[0])
    ws_bytes = L_.pma_delta_prefill_workspace_bytes(B, H, L, D, int(chunk), _DT[q.dtype]) if wy else 0
    if ws_bytes and workspace_bytes is not None:
        ws_bytes = int(workspace_bytes)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    rc = L_.pma_delta_prefill(B, H, L, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), beta.data_ptr(),
                              alpha.data_ptr() if alpha is not None else None, lam.data_ptr(), lam_sb, int(chunk),
                              float(lyapunov_bound), float(norm_eps),
                              st_in.data_ptr() if st_in is not None else None,
                              st_out.data_ptr() if st_out is not None else None, ys,
                              ws.data_ptr() if ws is not None else None, ws_bytes, _stream(dev))
    _lib.check("pma_delta_prefill", rc)
    return y, st_out


def delta_decode_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor, alpha: torch.Tensor,
                      state: torch.Tensor, lyapunov_bound: float = 25.0, norm_eps: float = 1e-5,
                      inplace: bool = False, out_dtype: Optional[torch.dtype] = None,
                      y_out: Optional[torch.Tensor] = None):
    """Gated delta-rule L == 1 step: q, k, v [N,H,D]; beta, alpha [N,H]; state [N,H,D,2D].
    Returns (y [N,H,D], new state); inplace=True updates `state` (contiguous float32)."""
    dev = _require_cuda(q, k, v)
    if q.dim() != 3 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must share one [N,H,D] shape")
    N, H, D = q.shape
    L_ = _lib.load()
    qs, q = _seq(q, False)
    ks, k = _seq(k, False)
    vs, v = _seq(v, False)
    beta = _gate(beta, (N, H), dev, "beta")
    alpha = _gate(alpha, (N, H), dev, "alpha")
    if tuple(state.shape) != (N, H, D, 2 * D):
        raise ValueError(f"state must be [N,H,D,2D] = {(N, H, D, 2 * D)}; got {tuple(state.shape)}")
    if inplace:
        if state.dtype != torch.float32 or not state.is_contiguous() or state.device != dev:
            raise ValueError("inplace=True needs a contiguous float32 state on the inputs' device")
        st_in = st_out = state
    else:
        st_in = state.to(device=dev, dtype=torch.float32).contiguous()
        st_out = torch.empty_like(st_in)
    y = y_out if y_out is not None else torch.empty(N, H, D, dtype=out_dtype or q.dtype, device=dev)
    ys, y2 = _seq(y, False)
    if y2 is not y:
        raise ValueError("y_out must have a contiguous, 16-byte aligned last axis")
    rc = L_.pma_delta_decode_step(N, H, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), beta.data_ptr(),
                                  alpha.data_ptr(), float(lyapunov_bound), float(norm_eps), st_in.data_ptr(),
                                  st_out.data_ptr(), ctypes.byref(ys), _stream(dev))
    _lib.check("pma_delta_decode_step", rc)
    return y, st_out


# ---------------------------------------------------------------- selective variant
def selective_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, log_decay: torch.Tensor,
                      beta: torch.Tensor, state: Optional[StateTuple] = None, eps: float = 1.0,
                      return_state: bool = True, out_dtype: Optional[torch.dtype] = None,
                      y_out: Optional[torch.Tensor] = None, want_y: bool = True,
                      prologue: Optional[Prologue] = None):
    """Selective moment attention (PrimeSelectiveMomentAttention's core) over q (pre-scaled), k, v
    [B,H,L,D] (k, v with H / kv_groups heads under a prologue); log_decay [B,H,L] = -Delta/tau;
    beta [H].  States in the reference's selective layout.  Returns (y or None, state or None)."""
    dev = _require_cuda(q, k, v)
    if q.dim() != 4:
        raise ValueError("q must be [B,H,L,D]")
    B, H, L, D = q.shape
    kv_shape = (B, _kv_heads(H, prologue), L, D)
    if tuple(k.shape) != kv_shape or tuple(v.shape) != kv_shape:
        raise ValueError(f"k, v must be {kv_shape}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share one dtype")
    check_faults("selective_prefill")
    L_ = _lib.load()
    qs, q = _seq(q)
    ks, k = _seq(k)
    vs, v = _seq(v)
    ld = _gate(log_decay, (B, H, L), dev, "log_decay")
    bt = _gate(beta, (H,), dev, "beta")
    st_in = None
    if state is not None:
        st_in_c, state = _state(state, B, H, D, "state")
        st_in = ctypes.byref(st_in_c)
    st_out_t = new_state(B, H, D, dev, zero=False) if return_state else None
    st_out = ctypes.byref(_lib.State(*[t.data_ptr() for t in st_out_t])) if return_state else None
    y = ys = None
    if want_y:
        if y_out is not None:
            if tuple(y_out.shape) != (B, H, L, D) or not _seq_ok(y_out):
                raise ValueError("y_out must be a [B,H,L,D] tensor with a contiguous, 16-byte aligned last axis")
            y = y_out
        else:
            y = torch.empty(B, H, L, D, dtype=out_dtype or q.dtype, device=dev)
        ys = ctypes.byref(_seq(y)[0])
    pc, keep = (prologue.to_c(D, dev) if prologue is not None else (None, None))
    pref = ctypes.byref(pc) if pc is not None else None
    ws_bytes = L_.pma_selective_prefill_workspace_bytes(B, H, L, D, _DT[q.dtype], pref)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    rc = L_.pma_selective_prefill(B, H, L, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs), pref,
                                  ld.data_ptr(), bt.data_ptr(), st_in, st_out, float(eps), ys,
                                  ws.data_ptr() if ws is not None else None, ws_bytes, _stream(dev))
    _lib.check("pma_selective_prefill", rc)
    return y, st_out_t


def selective_decode_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, log_decay: torch.Tensor,
                          beta: torch.Tensor, state: StateTuple, eps: float = 1.0, inplace: bool = False,
                          out_dtype: Optional[torch.dtype] = None, y_out: Optional[torch.Tensor] = None,
                          prologue: Optional[Prologue] = None, rows: Optional[torch.Tensor] = None):
    """Selective L == 1 step: q, k, v [N,H,D]; log_decay [N,H]; beta [H]; state in the selective
    layout ([N,H,...], or a pool [P,H,...] with `rows`, updated in place).  Returns (y, state)."""
    dev = _require_cuda(q, k, v)
    N, H, D = _check_step_shapes(q, k, v, prologue)
    L_ = _lib.load()
    qs, q = _seq(q, False)
    ks, k = _seq(k, False)
    vs, v = _seq(v, False)
    ld = _gate(log_decay, (N, H), dev, "log_decay")
    bt = _gate(beta, (H,), dev, "beta")
    P = state[0].shape[0] if rows is not None else N
    st_in_c, st_in_t = _state(state, P, H, D, "state")
    if inplace or rows is not None:
        if not all(a.data_ptr() == b.data_ptr() for a, b in zip(st_in_t, state)):
            raise ValueError("an in-place update needs contiguous float32 state tensors")
        st_out_t = st_in_t
    else:
        st_out_t = new_state(N, H, D, dev, zero=False)
    st_out_c = _lib.State(*[t.data_ptr() for t in st_out_t])
    y = y_out if y_out is not None else torch.empty(N, H, D, dtype=out_dtype or q.dtype, device=dev)
    ys, y2 = _seq(y, False)
    if y2 is not y:
        raise ValueError("y_out must have a contiguous, 16-byte aligned last axis")
    if rows is not None:
        if rows.dtype != torch.int32 or rows.dim() != 1 or rows.shape[0] != N or rows.device != dev:
            raise ValueError("rows must be an int32 tensor [N] on the inputs' device")
        rows = rows.contiguous()
    pc, keep = (prologue.to_c(D, dev) if prologue is not None else (None, None))
    rc = L_.pma_selective_decode_step(N, H, D, ctypes.byref(qs), ctypes.byref(ks), ctypes.byref(vs),
                                      ctypes.byref(pc) if pc is not None else None, ld.data_ptr(), bt.data_ptr(),
                                      rows.data_ptr() if rows is not None else None, P if rows is not None else 0,
                                      ctypes.byref(st_in_c), ctypes.byref(st_out_c), float(eps), ctypes.byref(ys),
                                      _stream(dev))
    _lib.check("pma_selective_decode_step", rc)
    return y, st_out_t
