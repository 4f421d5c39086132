"""Python face of the float64 CPU oracle (oracle/pma_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker.  The product package
(prime_moment_attention_b200) never imports it.

States use the reference's tuple layout (src/prime_moment_attention/attention.py:19-24,
111-117): (S0[B,H,D], S1[B,H,D,D], S2[B,H,D,D], K0[B,H,1], K1[B,H,D], K2[B,H,D]),
S1[b,h,d,e] = sum k_d v_e (row = key index).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_dp = ctypes.POINTER(ctypes.c_double)


def build() -> str:
    """Compile liboracle.so in place (gcc) if it is missing or stale."""
    so = os.path.join(_HERE, "liboracle.so")
    src = os.path.join(_HERE, "pma_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)
    return so


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(build())
        L.orc_decode_step.argtypes = [ctypes.c_int] * 3 + [_dp] * 4 + [ctypes.c_long, ctypes.c_double] + [_dp] * 7
        L.orc_decode_step.restype = ctypes.c_int
        L.orc_prefill.argtypes = [ctypes.c_int] * 4 + [_dp] * 4 + [ctypes.c_long, ctypes.c_double] + [_dp] * 7
        L.orc_prefill.restype = ctypes.c_int
        L.orc_combine.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_long, _dp, _dp]
        L.orc_combine.restype = None
        L.orc_delta_prefill.argtypes = ([ctypes.c_int] * 4 + [_dp] * 6 + [ctypes.c_int, ctypes.c_double,
                                        ctypes.c_double] + [_dp] * 3)
        L.orc_delta_prefill.restype = ctypes.c_int
        L.orc_delta_step.argtypes = [ctypes.c_int] * 3 + [_dp] * 5 + [ctypes.c_double] * 2 + [_dp] * 3
        L.orc_delta_step.restype = ctypes.c_int
        L.orc_selective_prefill.argtypes = [ctypes.c_int] * 4 + [_dp] * 5 + [ctypes.c_double] + [_dp] * 7
        L.orc_selective_prefill.restype = ctypes.c_int
        _LIB = L
    return _LIB


def _f64(a) -> np.ndarray:
    if hasattr(a, "detach"):  # torch tensor
        a = a.detach().to("cpu").double().numpy()
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_dp)


def zero_state(B: int, H: int, D: int):
    return (np.zeros((B, H, D)), np.zeros((B, H, D, D)), np.zeros((B, H, D, D)),
            np.zeros((B, H, 1)), np.zeros((B, H, D)), np.zeros((B, H, D)))


def _lam_table(lam, B: int, H: int):
    if np.ndim(lam) == 0 and not hasattr(lam, "detach"):
        return np.full((H,), float(lam)), 0
    lam = _f64(lam)
    if lam.ndim == 0 or lam.size == 1:
        return np.full((H,), float(lam.reshape(-1)[0])), 0
    if lam.shape == (H,):
        return lam, 0
    if lam.shape == (B, H):
        return np.ascontiguousarray(lam.reshape(B * H)), H
    raise ValueError(f"lambda must be a scalar, [H] or [B,H]; got {lam.shape}")


def prefill(q, k, v, lam, state=None, eps: float = 1.0):
    """Token recurrence over q,k,v [B,H,L,D] (q pre-scaled by 1/sqrt(D)).

    Returns (y [B,H,L,D] float64, final state tuple float64)."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    B, H, L, D = q.shape
    st = [np.array(_f64(s), copy=True) for s in (state if state is not None else zero_state(B, H, D))]
    st[3] = st[3].reshape(B, H, 1)
    lt, ls = _lam_table(lam, B, H)
    y = np.zeros_like(q)
    rc = lib().orc_prefill(B, H, L, D, _ptr(q), _ptr(k), _ptr(v), _ptr(lt), ls, float(eps),
                           *[_ptr(s) for s in st], _ptr(y))
    if rc != 0:
        raise ValueError("orc_prefill rejected its arguments")
    return y, tuple(st)


def decode_step(q, k, v, lam, state, eps: float = 1.0):
    """One recurrent step over q,k,v [N,H,D]; returns (y [N,H,D], new state)."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    N, H, D = q.shape
    st = [np.array(_f64(s), copy=True) for s in state]
    st[3] = st[3].reshape(N, H, 1)
    lt, ls = _lam_table(lam, N, H)
    y = np.zeros_like(q)
    rc = lib().orc_decode_step(N, H, D, _ptr(q), _ptr(k), _ptr(v), _ptr(lt), ls, float(eps),
                               *[_ptr(s) for s in st], _ptr(y))
    if rc != 0:
        raise ValueError("orc_decode_step rejected its arguments")
    return y, tuple(st)


def combine(P, T, lam: float, length: int):
    """State leaving a segment: lam**length * P + T (one head-state, flat)."""
    P = np.array(_f64(P), copy=True).ravel()
    T = np.ascontiguousarray(_f64(T).ravel())
    lib().orc_combine(P.size, float(lam), int(length), _ptr(P), _ptr(T))
    return P


def rel_err(a, b) -> float:
    """Normwise relative error max|a-b| / max|b| (the bar the parity tests use)."""
    a, b = _f64(a), _f64(b)
    den = float(np.max(np.abs(b))) if b.size else 0.0
    num = float(np.max(np.abs(a - b))) if b.size else 0.0
    if den == 0.0:
        return num
    return num / den


def delta_prefill(q, k, v, beta, alpha, lam, chunk: int = 64, bound: float = 25.0, norm_eps: float = 1e-5,
                  state=None, want_y: bool = True):
    """Gated delta-rule chunked prefill (chunked_delta_prime.py:175-283) as a token recurrence.

    q (pre-scaled), k, v [B,H,L,D]; beta, alpha [B,H,L] (alpha None: alpha_t = lam[h]); lam [H]
    (the decay of padded tokens); state [B,H,D,2D] or None.  Returns (y [B,H,L,D], state)."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    B, H, L, D = q.shape
    beta = _f64(beta).reshape(B, H, L)
    al = None if alpha is None else np.ascontiguousarray(_f64(alpha).reshape(B, H, L))
    lt = _f64(lam).reshape(-1)
    if lt.size == 1:
        lt = np.full(H, float(lt[0]))
    st_in = None if state is None else np.ascontiguousarray(_f64(state).reshape(B, H, D, 2 * D))
    st = np.zeros((B, H, D, 2 * D))
    y = np.zeros_like(q) if want_y else None
    rc = lib().orc_delta_prefill(B, H, L, D, _ptr(q), _ptr(k), _ptr(v), _ptr(beta),
                                 _ptr(al) if al is not None else None, _ptr(lt), int(chunk), float(bound),
                                 float(norm_eps), _ptr(st_in) if st_in is not None else None, _ptr(st),
                                 _ptr(y) if y is not None else None)
    if rc != 0:
        raise ValueError("orc_delta_prefill rejected its arguments")
    return y, st


def delta_step(q, k, v, beta, alpha, state, bound: float = 25.0, norm_eps: float = 1e-5):
    """Gated delta-rule L == 1 step (chunked_delta_prime.py:142-172): q, k, v [N,H,D], beta,
    alpha [N,H], state [N,H,D,2D].  Returns (y [N,H,D], new state)."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    N, H, D = q.shape
    beta = np.ascontiguousarray(_f64(beta).reshape(N, H))
    alpha = np.ascontiguousarray(_f64(alpha).reshape(N, H))
    st_in = np.ascontiguousarray(_f64(state).reshape(N, H, D, 2 * D))
    st = np.zeros_like(st_in)
    y = np.zeros_like(q)
    rc = lib().orc_delta_step(N, H, D, _ptr(q), _ptr(k), _ptr(v), _ptr(beta), _ptr(alpha), float(bound),
                              float(norm_eps), _ptr(st_in), _ptr(st), _ptr(y))
    if rc != 0:
        raise ValueError("orc_delta_step rejected its arguments")
    return y, st


def selective_prefill(q, k, v, log_decay, beta, state=None, eps: float = 1.0):
    """Selective moment attention (selective.py:264-444) as its step recurrence: q (pre-scaled),
    k, v [B,H,L,D]; log_decay [B,H,L] = -Delta_t / tau_h; beta [H]; state in the reference's
    selective layout (S2, K2 carry the 1/2 beta^2 factor).  Returns (y, state)."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    B, H, L, D = q.shape
    ld = np.ascontiguousarray(_f64(log_decay).reshape(B, H, L))
    bt = np.ascontiguousarray(_f64(beta).reshape(H))
    st = [np.array(_f64(s), copy=True) for s in (state if state is not None else zero_state(B, H, D))]
    st[3] = st[3].reshape(B, H, 1)
    y = np.zeros_like(q)
    rc = lib().orc_selective_prefill(B, H, L, D, _ptr(q), _ptr(k), _ptr(v), _ptr(ld), _ptr(bt), float(eps),
                                     *[_ptr(s) for s in st], _ptr(y))
    if rc != 0:
        raise ValueError("orc_selective_prefill rejected its arguments")
    return y, tuple(st)
