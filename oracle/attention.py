"""MABA-SA three-stream attention restated in numpy (test infrastructure only).

Follows maba_sparse/layers/sparse_attention.py:
  local  :79-105   keys j <= pos with (pos - j) < window or j < min(n_sinks, Lkv)
  sparse :107-171  tokens blk*block + o of the selected blocks with token < Lkv and <= pos
  hca    :173-219  pos < r-1: mean(c[0..pos]) (the cumulative-mean path);
                   else softmax over pooled complete blocks j with (j+1)r - 1 <= pos
  superposition :274-275 with common.py:406-438.
Computed per query row over only the keys each stream allows (no L x L
matrices), in float64, in the latent space: qhat_h = scale * W_uk,h^T q_h scores
against latent rows c_j and each stream returns sum_j p_j c_j; the per-head
output is W_uv,h applied to it (``expand``).  Softmax over an empty key set
gives 0, as the reference's nan_to_num.
"""
from __future__ import annotations

import numpy as np

from .indexer import hca_pool


def absorb(q, w_uk, n_heads: int, scale: float) -> np.ndarray:
    """q [B,L,H,dh], W_uk = k_up_proj.weight [H*dh, d_c] -> qhat [B,L,H,d_c]."""
    q = np.asarray(q, np.float64)
    dh = q.shape[-1]
    w = np.asarray(w_uk, np.float64).reshape(n_heads, dh, -1)
    return np.einsum("blhd,hdc->blhc", q, w) * scale


def expand(o_lat, w_uv, n_heads: int) -> np.ndarray:
    """o_lat [...,H,d_c], W_uv = v_up_proj.weight [H*dh, d_c] -> [...,H,dh]."""
    w = np.asarray(w_uv, np.float64)
    dh = w.shape[0] // n_heads
    w = w.reshape(n_heads, dh, -1)
    return np.einsum("...hc,hdc->...hd", np.asarray(o_lat, np.float64), w)


def local_rows(pos: int, Lkv: int, window: int, n_sinks: int) -> np.ndarray:
    lo = max(0, pos - window + 1)
    ns = min(n_sinks, Lkv)
    sinks = np.arange(min(ns, lo))
    return np.concatenate([sinks, np.arange(lo, pos + 1)]).astype(np.int64)


def sparse_rows(pos: int, Lkv: int, blocks, block: int) -> np.ndarray:
    nb = (Lkv + block - 1) // block
    out = []
    for blk in np.asarray(blocks).tolist():
        if blk < 0 or blk >= nb:
            continue
        tok = blk * block + np.arange(block)
        out.append(tok[(tok < Lkv) & (tok <= pos)])
    return np.concatenate(out).astype(np.int64) if out else np.zeros(0, np.int64)


def _softmax_mix(qh: np.ndarray, keys: np.ndarray) -> np.ndarray:
    """qh [H,d_c], keys [n,d_c] -> [H,d_c] (zeros when n == 0)."""
    if keys.shape[0] == 0:
        return np.zeros_like(qh)
    s = qh @ keys.T
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return p @ keys


def sa_streams(qhat, c_kv, top_idx, window: int = 128, n_sinks: int = 4, block: int = 64, hca_r: int = 64,
               rows=None) -> np.ndarray:
    """Per-stream latent outputs [3, B, R, H, d_c] (local, sparse, hca)."""
    qhat = np.asarray(qhat, np.float64)
    c = np.asarray(c_kv, np.float64)
    tix = np.asarray(top_idx)
    B, Lq, H, DC = qhat.shape
    Lkv = c.shape[1]
    rows = np.arange(Lq) if rows is None else np.asarray(rows)
    pooled = hca_pool(c, hca_r)
    nc = pooled.shape[1]
    out = np.zeros((3, B, len(rows), H, DC))
    for bi in range(B):
        csum = np.cumsum(c[bi], axis=0)
        for ri, t in enumerate(rows.tolist()):
            pos = Lkv - Lq + t
            qh = qhat[bi, t]
            out[0, bi, ri] = _softmax_mix(qh, c[bi, local_rows(pos, Lkv, window, n_sinks)])
            out[1, bi, ri] = _softmax_mix(qh, c[bi, sparse_rows(pos, Lkv, tix[bi, t], block)])
            if pos < hca_r - 1:
                out[2, bi, ri] = np.broadcast_to(csum[pos] / (pos + 1), (H, DC))
            else:
                nv = min(nc, (pos + 1) // hca_r)
                out[2, bi, ri] = _softmax_mix(qh, pooled[bi, :nv])
    return out


def gate_softmax(gate_logits) -> np.ndarray:
    g = np.asarray(gate_logits, np.float64)
    g = np.exp(g - g.max(axis=-1, keepdims=True))
    return g / g.sum(axis=-1, keepdims=True)


def sa_attention_latent(qhat, c_kv, top_idx, gate_logits, window: int = 128, n_sinks: int = 4, block: int = 64,
                        hca_r: int = 64, rows=None) -> np.ndarray:
    """Gate-weighted sum of the three latent streams -> [B, R, H, d_c]."""
    st = sa_streams(qhat, c_kv, top_idx, window, n_sinks, block, hca_r, rows)
    g = gate_softmax(gate_logits)
    Lq = np.asarray(qhat).shape[1]
    rows = np.arange(Lq) if rows is None else np.asarray(rows)
    if g.ndim == 3:  # [B,L,3] shared by heads
        g = g[:, rows][:, :, None, :]
    else:            # [B,H,L,3]
        g = np.transpose(g[:, :, rows], (0, 2, 1, 3))
    return sum(g[..., s:s + 1] * st[s] for s in range(3))
