"""DGDA recurrence restated in numpy (test infrastructure only).

* ``dgda_sequential``   -- maba_sparse/kernels/common.py:229-268 (ref_dgda_prefill):
  the token-by-token recurrence, the ground truth.
* ``dgda_step``         -- maba_sparse/kernels/common.py:271-309 (ref_dgda_step).
* ``dgda_transition``   -- the segment's affine map [R | P], derived from
  ``dgda_sequential`` (checks the sequence-split chain of this build).
* ``dgda_chunked``      -- maba_sparse/kernels/cpu_dgda.py:33-197 (cpu_dgda_prefill),
  the reference's chunked WY/UT CPU algorithm with the exact triangular solve;
  used as the timed CPU baseline.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np


def _as(x, dt):
    return None if x is None else np.asarray(x, dtype=dt)


def dgda_sequential(q, k, v, alpha=None, b=None, w=None, initial_state=None, log_alpha=None,
                    dtype=np.float64) -> Tuple[np.ndarray, np.ndarray]:
    """Sequential recurrence (common.py:256-265): Sd = diag(alpha) S; delta = w v - (b k)^T Sd;
    S = Sd + k delta^T; o_t = q^T S.  ``alpha`` wins over ``log_alpha`` (common.py:242-243)."""
    if alpha is None and log_alpha is None:
        raise ValueError("Either alpha or log_alpha must be provided")
    q, k, v, b, w = (_as(t, dtype) for t in (q, k, v, b, w))
    alpha = _as(alpha, dtype) if alpha is not None else np.exp(_as(log_alpha, dtype))
    B, H, L, dk = q.shape
    dv = v.shape[-1]
    S = np.zeros((B, H, dk, dv), dtype) if initial_state is None else _as(initial_state, dtype).copy()
    out = np.empty((B, H, L, dv), dtype)
    for t in range(L):
        Sd = alpha[:, :, t, :, None] * S
        pred = np.einsum("bhi,bhij->bhj", b[:, :, t] * k[:, :, t], Sd)
        delta = w[:, :, t] * v[:, :, t] - pred
        S = Sd + k[:, :, t, :, None] * delta[:, :, None, :]
        out[:, :, t] = np.einsum("bhi,bhij->bhj", q[:, :, t], S)
    return out, S


def dgda_step(q, k, v, alpha=None, b=None, w=None, state=None, log_alpha=None, dtype=np.float64):
    """One step (common.py:271-309); inputs [B,H,d] or [B,H,1,d]."""
    def sq(x):
        x = _as(x, dtype)
        if x is not None and x.ndim == 4 and x.shape[2] == 1:
            x = x[:, :, 0]
        return x

    q, k, v, b, w = (sq(t) for t in (q, k, v, b, w))
    alpha = sq(alpha) if alpha is not None else np.exp(sq(log_alpha))
    B, H, dk = q.shape
    dv = v.shape[-1]
    S = np.zeros((B, H, dk, dv), dtype) if state is None else _as(state, dtype)
    Sd = alpha[..., None] * S
    pred = np.einsum("bhi,bhij->bhj", b * k, Sd)
    delta = w * v - pred
    S2 = Sd + k[..., None] * delta[:, :, None, :]
    o = np.einsum("bhi,bhij->bhj", q, S2)
    return o, S2


def dgda_transition(q, k, v, alpha=None, b=None, w=None, log_alpha=None, pad: int = 64,
                    dtype=np.float64) -> np.ndarray:
    """Affine map of a segment on the state, S_end = P S_start + R, as [B,H,pad,2*pad] = [R | P].

    The recurrence of ``dgda_sequential`` is affine in S (common.py:256-265), so R is its
    final state from S_start = 0 and P its final state from S_start = I with v = 0.  Head dims
    below ``pad`` are padded: R with zeros, P with the identity (padded rows of a state stay 0)."""
    q, k, v = (_as(t, dtype) for t in (q, k, v))
    B, H, L, dk = q.shape
    dv = v.shape[-1]
    _, R = dgda_sequential(q, k, v, alpha, b, w, log_alpha=log_alpha, dtype=dtype)
    eye = np.broadcast_to(np.eye(dk, dtype=dtype), (B, H, dk, dk)).copy()
    _, P = dgda_sequential(q, k, np.zeros((B, H, L, dk), dtype), alpha, b, np.ones((B, H, L, 1), dtype),
                           initial_state=eye, log_alpha=log_alpha, dtype=dtype)
    out = np.zeros((B, H, pad, 2 * pad), dtype)
    out[..., :dk, :dv] = R
    out[..., :, pad:] = np.eye(pad, dtype=dtype)
    out[..., :dk, pad:pad + dk] = P
    return out


def _log_decay(alpha, log_alpha, dtype):
    """cpu_dgda.py:63-68: log_alpha clamped to [-46, 0], else log(clamp(alpha, 1e-20, 1))."""
    if log_alpha is not None:
        return np.clip(_as(log_alpha, dtype), -46.0, 0.0)
    return np.log(np.clip(_as(alpha, dtype), 1e-20, 1.0))


def dgda_chunked(q, k, v, alpha=None, b=None, w=None, chunk_size: int = 64, initial_state=None, log_alpha=None,
                 dtype=np.float32) -> Tuple[np.ndarray, np.ndarray]:
    """Chunked WY/UT form of cpu_dgda.py:82-197 with the exact triangular solve
    (``inversion_method="exact"``, cpu_dgda.py:130-131): per chunk,
    cla = cumsum(log alpha); L = tril_{-1}((b k) dec k); A = tril_0(q dec k);
    u = (I+L)^{-1}(w v - (b k e^{cla}) S); o = (q e^{cla}) S + A u;
    S <- e^{cla_end} S + (k e^{cla_end-cla})^T u."""
    q, k, v, b, w = (_as(t, dtype) for t in (q, k, v, b, w))
    la = _log_decay(alpha, log_alpha, dtype)
    B, H, L, dk = q.shape
    dv = v.shape[-1]
    S = np.zeros((B, H, dk, dv), dtype) if initial_state is None else _as(initial_state, dtype).copy()
    out = np.empty((B, H, L, dv), dtype)
    for s in range(0, L, chunk_size):
        e = min(s + chunk_size, L)
        C = e - s
        qc, kc, bc, wc, vc = q[:, :, s:e], k[:, :, s:e], b[:, :, s:e], w[:, :, s:e], v[:, :, s:e]
        cla = np.cumsum(la[:, :, s:e], axis=2)
        diff = cla[:, :, :, None, :] - cla[:, :, None, :, :]
        dec = np.exp(np.minimum(diff, 0.0))
        bk = bc * kc
        lmat = np.tril(np.einsum("bhid,bhijd,bhjd->bhij", bk, dec, kc), -1)
        amat = np.tril(np.einsum("bhid,bhijd,bhjd->bhij", qc, dec, kc), 0)
        lam = np.exp(cla)
        ve = wc * vc - np.einsum("bhid,bhdj->bhij", bk * lam, S)
        m = np.eye(C, dtype=dtype)[None, None] + lmat
        u = np.linalg.solve(m, ve)
        out[:, :, s:e] = np.einsum("bhid,bhdj->bhij", qc * lam, S) + np.einsum("bhij,bhjc->bhic", amat, u)
        clae = cla[:, :, -1:, :]
        kd = kc * np.exp(clae - cla)
        S = np.exp(clae[:, :, 0, :])[..., None] * S + np.einsum("bhid,bhic->bhdc", kd, u)
    return out, S
