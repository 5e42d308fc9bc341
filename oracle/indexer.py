"""DG-Indexer and stream superposition restated in numpy (test infrastructure only).

* ``compute_centroids``   -- maba_sparse/kernels/common.py:329-350 and
  cpu_indexer.py:16-50: c = 0.5*(mean + max) per block, tail zero-padded,
  16-bit inputs upcast to fp32.  The block sum is a sequential fp32 sum.
* ``index_scores`` / ``index_topk`` -- cpu_indexer.py:54-112 (fp32 upcast, log1p
  penalty) and maba_sparse/layers/indexer.py:101-112 (decode).  The dot product
  is a sequential chain of correctly rounded fp32 fused multiply-adds over
  d = 0..D-1 and the penalty is fl32(fl32(lambda) * fl32(log1p(delta))): the same
  arithmetic as the CUDA kernel, so scores and indices match bit for bit.
  Against the reference (whose matmul sums in another order) indices agree
  except where two scores are within a couple of ulps.
* ``stream_superposition`` -- common.py:406-438 / cpu_indexer.py:116-150.
"""
from __future__ import annotations

import numpy as np


def fmaf(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """Correctly rounded float32 a*b + c (one rounding), vectorised.

    a*b is exact in float64; p + c is rounded once to float64 (s) with its
    exact error e from TwoSum.  Rounding s to float32 equals rounding the exact
    value unless s lies exactly halfway between two float32 values and e != 0;
    that case is resolved toward the sign of e.
    """
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    c = np.asarray(c, np.float32)
    p = a.astype(np.float64) * b.astype(np.float64)
    c64 = c.astype(np.float64)
    s = p + c64
    bb = s - p
    e = (p - (s - bb)) + (c64 - bb)
    r = s.astype(np.float32)
    r64 = r.astype(np.float64)
    d = s - r64
    toward = np.where(d >= 0, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
    nxt = np.nextafter(r, toward)
    half = (nxt.astype(np.float64) - r64) * 0.5
    tie = (d == half) & (d != 0) & (e != 0)
    if np.any(tie):
        # true value beyond the midpoint (same direction as d) -> the far neighbour
        go_far = np.sign(e) == np.sign(d)
        r = np.where(tie & go_far, nxt, r)
    return r


def compute_centroids(k_idx, block_size: int = 64) -> np.ndarray:
    """[B,L,d] -> [B,ceil(L/block),d]; fp32 (fp64 for fp64 input) arithmetic."""
    k = np.asarray(k_idx)
    acc = np.float64 if k.dtype == np.float64 else np.float32
    k = k.astype(acc)
    B, L, d = k.shape
    if L == 0:
        return np.empty((B, 0, d), acc)
    nb = (L + block_size - 1) // block_size
    pad = nb * block_size - L
    kp = np.concatenate([k, np.zeros((B, pad, d), acc)], axis=1) if pad else k
    kb = kp.reshape(B, nb, block_size, d)
    s = np.zeros((B, nb, d), acc)
    for t in range(block_size):
        s = s + kb[:, :, t, :]
    mean = s / acc(block_size)
    mx = kb.max(axis=2)
    return (acc(0.5) * (mean + mx)).astype(acc)


def hca_pool(c_kv, r: int = 64) -> np.ndarray:
    """Mean of each complete r-row block (maba_sparse/layers/sparse_attention.py:206)."""
    c = np.asarray(c_kv, np.float64)
    B, L, d = c.shape
    n = L // r
    return c[:, : n * r].reshape(B, n, r, d).mean(axis=2)


def penalty_table(lam: float, n: int) -> np.ndarray:
    """pen[delta] = fl32(fl32(lambda) * fl32(log1p(delta))) for delta in [0, n)."""
    l1p = np.log1p(np.arange(n, dtype=np.float64)).astype(np.float32)
    return (np.float32(lam) * l1p).astype(np.float32)


def _query_blocks(L, nb, block_size, decode):
    if decode:
        return np.full(L, nb - 1, dtype=np.int64)
    return np.arange(L, dtype=np.int64) // block_size


def index_scores(q_idx, centroids, lambda_dist: float = 0.5, block_size: int = 64, decode: bool = False,
                 rows=None) -> np.ndarray:
    """fp32 scores [B, len(rows), nb] with -inf for future blocks (n > qb)."""
    q = np.asarray(q_idx, np.float32)
    c = np.asarray(centroids, np.float32)
    B, L, D = q.shape
    nb = c.shape[1]
    rows = np.arange(L) if rows is None else np.asarray(rows)
    qb = _query_blocks(L, nb, block_size, decode)[rows]
    scale = np.float32(1.0 / np.sqrt(np.float64(D)))
    qs = (q[:, rows, :] * scale).astype(np.float32)  # [B,R,D]
    acc = np.zeros((B, len(rows), nb), np.float32)
    for d in range(D):
        acc = fmaf(qs[:, :, d][:, :, None], c[:, :, d][:, None, :], acc)
    n = np.arange(nb)
    delta = qb[:, None] - n[None, :]
    pen = penalty_table(lambda_dist, int(max(qb.max() + 1, nb)) if len(rows) else 1)
    valid = delta >= 0
    s = acc - np.where(valid, pen[np.clip(delta, 0, None)], np.float32(0))[None]
    s = np.where(valid[None], s, np.float32(-np.inf)).astype(np.float32)
    return s


def topk_from_scores(scores: np.ndarray, qb: np.ndarray, top_k: int) -> np.ndarray:
    """Ordering rule of the build: finite candidates by (score desc, index asc), then the
    lowest unused future indices ascending.  scores [B,R,nb], qb [R]."""
    B, R, nb = scores.shape
    ak = min(top_k, nb)
    out = np.empty((B, R, ak), np.int64)
    for r in range(R):
        nmax = min(int(qb[r]), nb - 1)
        ncand = nmax + 1
        nvalid = min(ak, ncand)
        for bi in range(B):
            s = scores[bi, r, :ncand]
            order = np.argsort(-s, kind="stable")[:nvalid]
            out[bi, r, :nvalid] = order
            out[bi, r, nvalid:] = np.arange(nmax + 1, nmax + 1 + (ak - nvalid))
    return out


def index_topk(q_idx, centroids, lambda_dist: float = 0.5, top_k: int = 32, block_size: int = 64,
               return_scores: bool = False, decode: bool = False, rows=None):
    q = np.asarray(q_idx)
    B, L, D = q.shape
    nb = np.asarray(centroids).shape[1]
    rows = np.arange(L) if rows is None else np.asarray(rows)
    s = index_scores(q, centroids, lambda_dist, block_size, decode, rows)
    qb = _query_blocks(L, nb, block_size, decode)[rows]
    idx = topk_from_scores(s, qb, top_k)
    return (idx, s) if return_scores else idx


def stream_superposition(o_local, o_sparse, o_hca, gate_logits=None, gate_weights=None) -> np.ndarray:
    """g = softmax(gate) in fp64; o = g0 o_local + g1 o_sparse + g2 o_hca; gate [B,L,3] or [B,H,L,3]."""
    ol, os_, oh = (np.asarray(t, np.float64) for t in (o_local, o_sparse, o_hca))
    if gate_weights is None:
        g = np.asarray(gate_logits, np.float64)
        g = np.exp(g - g.max(axis=-1, keepdims=True))
        g = g / g.sum(axis=-1, keepdims=True)
    else:
        g = np.asarray(gate_weights, np.float64)
    if g.ndim == 3:
        g = g[:, None]
    return g[..., 0:1] * ol + g[..., 1:2] * os_ + g[..., 2:3] * oh
