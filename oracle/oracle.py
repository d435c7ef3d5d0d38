"""ORACLE — test infrastructure only.

Python face of the float64 C restatement in ``linattn_oracle.c``. Only the
tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
import this module, and only to check or to time a CPU baseline; the product
never calls it.

Host-side logic restated from the reference (paths relative to its tree):
  * decay-parameter broadcasting ``log_gamma = -softplus(-w)`` to [B,H,T]:
    python/subq_audio/autograd.py:310-333
  * attention-mask normalisation to an active-token mask [B,1,T,1]:
    python/subq_audio/autograd.py:57-105
  * reduction of d(log gamma) to the shape of ``w``:
    python/subq_audio/autograd.py:526-542
  * the C++ engine's gamma -> logit conversion and its d_gamma output:
    python/bindings.cpp:289-292,322
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None
_lock = threading.Lock()


def build() -> str:
    """Compile the C restatement into ``oracle/_build/liboracle.so``."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build()
            lib = ctypes.CDLL(_LIB_PATH)
            P = ctypes.c_void_p
            L = ctypes.c_long
            D = ctypes.c_double
            I = ctypes.c_int
            lib.oracle_forward.argtypes = [L, L, L, L, P, P, P, P, P, I, D, D, P, P, P, P, P, P, I, I]
            lib.oracle_forward.restype = I
            lib.oracle_backward.argtypes = [L, L, L, L, P, P, P, P, P, I, D, D, P, P, P, P, P, P, P, I, I]
            lib.oracle_backward.restype = I
            lib.oracle_phi.argtypes = [D]
            lib.oracle_phi.restype = D
            lib.oracle_phi_prime.argtypes = [D]
            lib.oracle_phi_prime.restype = D
            _lib = lib
    return _lib


def threads() -> int:
    """Host threads the oracle may use (``SUBQ_ORACLE_THREADS`` overrides)."""
    return int(os.environ.get("SUBQ_ORACLE_THREADS", os.cpu_count() or 1))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f64(a):
    return None if a is None else np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def phi(x: float) -> float:
    return _load().oracle_phi(float(x))


def phi_prime(x: float) -> float:
    return _load().oracle_phi_prime(float(x))


# --------------------------------------------------------------------------
# Host logic restated from the reference
# --------------------------------------------------------------------------
def softplus(x):
    x = np.asarray(x, dtype=np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def sigmoid(x):
    x = np.asarray(x, dtype=np.float64)
    return 0.5 * (1.0 + np.tanh(0.5 * x))


def broadcast_log_gamma(w, B, H, T):
    """``-softplus(-w)`` broadcast to [B,H,T] by the reference's shape rules."""
    w = np.asarray(w, dtype=np.float64)
    lg = -softplus(-w)
    if w.ndim == 0:
        return np.broadcast_to(lg.reshape(1, 1, 1), (B, H, T)).copy()
    if w.ndim == 1:
        if w.shape[0] == H:
            return np.broadcast_to(lg.reshape(1, H, 1), (B, H, T)).copy()
        return np.broadcast_to(lg.reshape(1, 1, -1), (B, H, T)).copy()
    if w.ndim == 2:
        if w.shape[1] == T:
            return np.broadcast_to(lg.reshape(B, 1, T), (B, H, T)).copy()
        return np.broadcast_to(lg.reshape(B, H, 1), (B, H, T)).copy()
    return np.broadcast_to(lg, (B, H, T)).copy()


def reduce_dw(dlog_gamma, w, B, H, T):
    """Chain rule through ``-softplus(-w)`` and reduction to the shape of w."""
    w = np.asarray(w, dtype=np.float64)
    sg = sigmoid(-w)
    dl = dlog_gamma.reshape(B, H, T)
    if w.ndim == 0:
        return np.asarray((dl * sg).sum())
    if w.ndim == 1:
        if w.shape[0] == H:
            return (dl * sg.reshape(1, H, 1)).sum(axis=(0, 2))
        return (dl * sg.reshape(1, 1, -1)).sum(axis=(0, 1))
    if w.ndim == 2:
        if w.shape[1] == T:
            return (dl * sg.reshape(B, 1, T)).sum(axis=1)
        return (dl * sg.reshape(B, H, 1)).sum(axis=-1)
    if w.ndim == 3:
        return dl * sg
    return np.asarray(dl.sum())


def normalize_mask(mask, T):
    """Active-token mask [B,T] (float64 0/1) from a 2-D/3-D/4-D bool/int/float mask."""
    if mask is None:
        return None
    m = np.asarray(mask)
    if m.dtype == np.bool_:
        valid = m.astype(np.float64)
    elif np.issubdtype(m.dtype, np.floating):
        valid = (m >= -1.0).astype(np.float64) if (m < -1.0).any() else (m > 0.0).astype(np.float64)
    else:
        valid = (m != 0).astype(np.float64)
    if valid.ndim == 2:
        return valid
    if valid.ndim == 3:
        if valid.shape[1] == 1 and valid.shape[2] == T:
            return valid[:, 0, :]
        if valid.shape[2] == 1 and valid.shape[1] == T:
            return valid[:, :, 0]
        red = (valid.sum(axis=-1) > 0).astype(np.float64)
        return red
    if valid.ndim == 4:
        if valid.shape[-2] != valid.shape[-1]:
            raise ValueError("4D attention_mask must be square")
        aq = valid.sum(axis=-1) > 0
        ak = valid.sum(axis=-2) > 0
        return (aq & ak).astype(np.float64)[:, 0, :]
    raise ValueError("unsupported mask rank")


# --------------------------------------------------------------------------
# Scans
# --------------------------------------------------------------------------
def forward(q, k, v, log_gamma=None, mask=None, normalize=True, scale=None, clamp_min=1e-5,
            S0=None, z0=None, ftz=False):
    """Causal scan over [..., N, d] inputs (leading dims flattened to sequences).

    ``log_gamma`` and ``mask`` have the leading dims plus N. Returns
    ``(out, S_final, z_final, den)``.
    """
    q, k, v = _f64(q), _f64(k), _f64(v)
    lead = q.shape[:-2]
    N, d = q.shape[-2], q.shape[-1]
    e = v.shape[-1]
    BH = int(np.prod(lead)) if lead else 1
    if scale is None:
        scale = 1.0 / math.sqrt(d) if normalize else 1.0
    lg = None if log_gamma is None else _f64(np.broadcast_to(log_gamma, lead + (N,)))
    mk = None if mask is None else _f64(np.broadcast_to(mask, lead + (N,)))
    S0 = _f64(S0)
    z0 = _f64(z0)
    out = np.empty(lead + (N, e), np.float64)
    S_out = np.empty(lead + (d, e), np.float64)
    z_out = np.empty(lead + (d,), np.float64)
    den = np.empty(lead + (N,), np.float64)
    rc = _load().oracle_forward(BH, N, d, e, _ptr(q), _ptr(k), _ptr(v), _ptr(lg), _ptr(mk),
                                int(bool(normalize)), float(scale), float(clamp_min), _ptr(S0),
                                _ptr(z0), _ptr(out), _ptr(S_out), _ptr(z_out), _ptr(den), int(bool(ftz)),
                                threads())
    if rc != 0:
        raise ValueError("oracle_forward rejected its arguments")
    return out, S_out, z_out, den


def backward(q, k, v, dO, log_gamma=None, mask=None, normalize=True, scale=None, clamp_min=1e-5,
             S0=None, z0=None, ftz=False):
    """Exact float64 adjoint. Returns ``(dq, dk, dv, dlog_gamma)``."""
    q, k, v, dO = _f64(q), _f64(k), _f64(v), _f64(dO)
    lead = q.shape[:-2]
    N, d = q.shape[-2], q.shape[-1]
    e = v.shape[-1]
    BH = int(np.prod(lead)) if lead else 1
    if scale is None:
        scale = 1.0 / math.sqrt(d) if normalize else 1.0
    lg = None if log_gamma is None else _f64(np.broadcast_to(log_gamma, lead + (N,)))
    mk = None if mask is None else _f64(np.broadcast_to(mask, lead + (N,)))
    S0 = _f64(S0)
    z0 = _f64(z0)
    dq = np.empty(lead + (N, d), np.float64)
    dk = np.empty(lead + (N, d), np.float64)
    dv = np.empty(lead + (N, e), np.float64)
    dlg = np.empty(lead + (N,), np.float64)
    rc = _load().oracle_backward(BH, N, d, e, _ptr(q), _ptr(k), _ptr(v), _ptr(lg), _ptr(mk),
                                 int(bool(normalize)), float(scale), float(clamp_min), _ptr(S0),
                                 _ptr(z0), _ptr(dO), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dlg),
                                 int(bool(ftz)), threads())
    if rc != 0:
        raise ValueError("oracle_backward rejected its arguments")
    return dq, dk, dv, dlg


# --------------------------------------------------------------------------
# Reference-API restatements
# --------------------------------------------------------------------------
def engine_forward(Q, K, V, decay_factor=0.99):
    """C++ ``SubQEngine.forward``: unnormalised, scalar decay, subnormal flush."""
    Q = _f64(Q)
    B, N, D = Q.shape
    lg = np.full((B, N), math.log(decay_factor)) if decay_factor != 1.0 else None
    out, _, _, _ = forward(Q, K, V, log_gamma=lg, normalize=False, scale=1.0, ftz=True)
    return out


def _engine_gamma(decay_factor):
    g = min(max(float(decay_factor), 1e-6), 1.0 - 1e-6)
    w = math.log(g / (1.0 - g))
    return 1.0 / (1.0 + math.exp(-w))


def engine_backward(dO, Q, K, V, decay_factor=0.99):
    """C++ ``SubQEngine.backward``: returns ``(dQ, dK, dV, d_gamma)``."""
    Q = _f64(Q)
    B, N, D = Q.shape
    gamma = _engine_gamma(decay_factor)
    lg = np.full((B, N), math.log(gamma))
    dq, dk, dv, dlg = backward(Q, K, V, dO, log_gamma=lg, normalize=False, scale=1.0, ftz=True)
    return dq, dk, dv, float(dlg.sum() / gamma)


def attention(q, k, v, decay_w=None, attention_mask=None, past_state=None):
    """Normalised causal scan with the reference's decay/mask conventions.

    ``q,k,v`` are [B,T,D] or [B,H,T,D]. ``decay_w=None`` means gamma == 1.
    ``past_state`` is ``(S [B,H,D,Dv], Z [B,H,D] or [B,H,D,1])``.
    Returns ``(out, (S_final, z_final))``.
    """
    q = _f64(q)
    is3 = q.ndim == 3
    if is3:
        q, k, v = q[:, None], _f64(k)[:, None], _f64(v)[:, None]
    B, H, T, D = q.shape
    lg = None if decay_w is None else broadcast_log_gamma(decay_w, B, H, T)
    vm = normalize_mask(attention_mask, T)
    mk = None if vm is None else np.broadcast_to(vm[:, None, :], (B, H, T))
    S0 = z0 = None
    if past_state is not None:
        S0 = _f64(past_state[0])
        if len(past_state) > 1 and past_state[1] is not None:
            z0 = _f64(past_state[1]).reshape(B, H, D)
    out, S, z, _ = forward(q, k, v, log_gamma=lg, mask=mk, normalize=True, S0=S0, z0=z0)
    if is3:
        out = out[:, 0]
    return out, (S, z)


def attention_backward(q, k, v, dO, decay_w=None, attention_mask=None):
    """Gradients of ``attention`` (causal): ``(dq, dk, dv, dw)``; dw is None without decay."""
    q = _f64(q)
    is3 = q.ndim == 3
    if is3:
        q, k, v, dO = q[:, None], _f64(k)[:, None], _f64(v)[:, None], _f64(dO)[:, None]
    B, H, T, D = q.shape
    lg = None if decay_w is None else broadcast_log_gamma(decay_w, B, H, T)
    vm = normalize_mask(attention_mask, T)
    mk = None if vm is None else np.broadcast_to(vm[:, None, :], (B, H, T))
    dq, dk, dv, dlg = backward(q, k, v, dO, log_gamma=lg, mask=mk, normalize=True)
    dw = None if decay_w is None else reduce_dw(dlg, decay_w, B, H, T)
    if is3:
        dq, dk, dv = dq[:, 0], dk[:, 0], dv[:, 0]
    return dq, dk, dv, dw
