"""Layer-level restatements in numpy (test infrastructure only).

* ``sa_layer_forward``   -- maba_sparse/layers/sparse_attention.py:221-277 (prefill
  from an empty cache): projections, DG-Indexer (indexer.py:43-126 prefill
  branch), the three streams and the superposition, o_proj.
* ``dgda_layer_forward`` -- maba_sparse/layers/dgda.py:166-236: projections,
  causal depthwise conv (k=4) + SiLU (:103-122), gates (:193-197), k L2-norm
  (:207), the recurrence, o_proj.
Weights are the reference state-dict entries (numpy arrays by name).
"""
from __future__ import annotations

import numpy as np

from .attention import absorb, expand, gate_softmax, sa_streams
from .dgda import dgda_sequential
from .indexer import compute_centroids, index_topk


def _lin(x, w, b=None):
    y = x @ np.asarray(w, np.float64).T
    return y + np.asarray(b, np.float64) if b is not None else y


def sa_layer_forward(w: dict, x, n_heads: int, d_head: int, window: int = 128, block: int = 64, top_k: int = 32,
                     hca_r: int = 64, lam: float = 0.5, n_sinks: int = 4, idx=None):
    x = np.asarray(x, np.float64)
    B, L, _ = x.shape
    c_kv = _lin(x, w["kv_down_proj.weight"])
    q = _lin(x, w["q_proj.weight"]).reshape(B, L, n_heads, d_head)
    if idx is None:
        qi = _lin(x, w["indexer.q_idx_proj.weight"]).astype(np.float32)
        ki = _lin(x, w["indexer.k_idx_proj.weight"]).astype(np.float32)
        c = compute_centroids(ki, block)
        idx = index_topk(qi, c, lambda_dist=lam, top_k=top_k, block_size=block)
    qhat = absorb(q, w["k_up_proj.weight"], n_heads, 1.0 / np.sqrt(d_head))
    st = sa_streams(qhat, c_kv, idx, window, n_sinks, block, hca_r)
    gate = _lin(x, w["stream_gate.weight"], w["stream_gate.bias"])
    g = gate_softmax(gate)[:, :, None, :]
    o_lat = sum(g[..., s:s + 1] * st[s] for s in range(3))
    o = expand(o_lat, w["v_up_proj.weight"], n_heads).reshape(B, L, n_heads * d_head)
    y = _lin(o, w["o_proj.weight"])
    streams = [expand(st[s], w["v_up_proj.weight"], n_heads) for s in range(3)]  # [B,L,H,dh] each
    return y, c_kv, idx, streams


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _softplus(x):
    return np.logaddexp(0.0, x)


def _conv(x, wconv, hist=None):
    """x [B,L,C]; wconv [C,1,K]; returns SiLU(causal depthwise conv) and the new history [B,C,K-1]."""
    B, L, C = x.shape
    K = wconv.shape[-1]
    xt = np.transpose(x, (0, 2, 1))
    pad = hist if hist is not None else np.zeros((B, C, K - 1))
    p = np.concatenate([pad, xt], axis=2)
    wk = np.asarray(wconv, np.float64)[:, 0, :]
    y = np.zeros((B, C, L))
    for j in range(K):
        y += wk[None, :, j:j + 1] * p[:, :, j:j + L]
    return np.transpose(_silu(y), (0, 2, 1)), p[:, :, -(K - 1):]


def dgda_layer_forward(w: dict, x, n_heads: int, d_head: int, state=None, conv_state=None, eps: float = 1e-6):
    x = np.asarray(x, np.float64)
    B, L, _ = x.shape
    h, d = n_heads, d_head
    cq, ck, cv = conv_state if conv_state is not None else (None, None, None)
    q, nq = _conv(_lin(x, w["q_proj.weight"]), w["conv_q.weight"], cq)
    k, nk = _conv(_lin(x, w["k_proj.weight"]), w["conv_k.weight"], ck)
    v, nv = _conv(_lin(x, w["v_proj.weight"]), w["conv_v.weight"], cv)
    eb = 1.0 / (1.0 + np.exp(-_lin(x, w["gate_erase.weight"])))
    ew = 1.0 / (1.0 + np.exp(-_lin(x, w["gate_write.weight"])))
    la = np.maximum(-_softplus(_lin(x, w["gate_alpha.weight"])), -14.0)

    def heads(t):
        return np.transpose(t.reshape(B, L, h, d), (0, 2, 1, 3))

    q, k, v, eb, ew, la = map(heads, (q, k, v, eb, ew, la))
    k = k / (np.linalg.norm(k, axis=-1, keepdims=True) + eps)
    o, S = dgda_sequential(q, k, v, np.exp(la), eb, ew, initial_state=state)
    o = np.transpose(o, (0, 2, 1, 3)).reshape(B, L, h * d)
    return _lin(o, w["o_proj.weight"]), S, (nq, nk, nv)
