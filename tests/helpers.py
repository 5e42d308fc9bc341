"""Shared helpers of the test-suite: golden fixture loading, tolerances."""
from __future__ import annotations

import functools
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# tolerances stated by the north star: relative error (max abs diff / max abs reference)
RTOL_FP32 = 1e-4
RTOL_BF16 = 2e-2
RTOL_FP16 = 5e-3


@functools.lru_cache(maxsize=None)
def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


def sub(d: dict, prefix: str) -> dict:
    return {k[len(prefix):]: v for k, v in d.items() if k.startswith(prefix)}


def to_np(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach()
        if x.dtype in (torch.bfloat16, torch.float16):
            x = x.float()
        return x.cpu().numpy()
    return np.asarray(x)


def rel_err(actual, expected) -> float:
    a = to_np(actual).astype(np.float64)
    e = to_np(expected).astype(np.float64)
    assert a.shape == e.shape, f"shape {a.shape} != {e.shape}"
    scale = max(np.abs(e).max() if e.size else 0.0, 1e-30)
    return float(np.abs(a - e).max() / scale) if e.size else 0.0


def assert_rel(actual, expected, rtol: float, what: str = "") -> None:
    err = rel_err(actual, expected)
    assert err <= rtol, f"{what}: relative error {err:.3e} > {rtol:.1e}"


def tensors(d: dict, device="cpu", dtype=None, keys=None) -> dict:
    out = {}
    for k, v in d.items():
        if keys is not None and k not in keys:
            continue
        t = torch.from_numpy(np.ascontiguousarray(v))
        if dtype is not None and t.is_floating_point():
            t = t.to(dtype)
        out[k] = t.to(device)
    return out


def check_topk_rule(idx, scores, qb, top_k, ulp_slack: int = 2):
    """Index parity rule against a reference top-k: for each row the first
    nvalid = min(top_k, qb+1, nb) indices must equal the reference's finite
    candidates re-sorted by (score desc, index asc); a disagreement is only
    accepted where the two scores lie within ulp_slack fp32 ulps (a tie).
    Returns the number of tie-classified rows."""
    idx = np.asarray(idx)
    s = np.asarray(scores, np.float32)
    B, R, nb = s.shape
    ties = 0
    for b in range(B):
        for r in range(R):
            nmax = min(int(qb[r]), nb - 1)
            nvalid = min(top_k, nmax + 1, nb)
            row = s[b, r, : nmax + 1]
            want = np.argsort(-row, kind="stable")[:nvalid]
            got = idx[b, r, :nvalid]
            if np.array_equal(got, want):
                continue
            # allow only near-tie swaps: the set of chosen scores must match within slack
            gs = np.sort(row[got])[::-1]
            ws = np.sort(row[want])[::-1]
            gap = np.abs(gs - ws)
            tol = ulp_slack * np.spacing(np.maximum(np.abs(gs), np.abs(ws)).astype(np.float32))
            assert np.all(gap <= tol), f"row ({b},{r}): {got.tolist()} vs {want.tolist()}"
            ties += 1
    return ties


class OracleBackend:
    """Compute backend of ``maba_v2_architecture_b200.parallel`` on the CPU oracle, so the
    sequence-split plumbing (phases, exchange, folding) runs under gloo without a GPU."""

    def __init__(self):
        import oracle.attention as oa
        import oracle.dgda as od
        import oracle.indexer as oi
        self.oa, self.od, self.oi = oa, od, oi

    @staticmethod
    def _t(x, like):
        return torch.from_numpy(np.ascontiguousarray(x)).to(like.dtype)

    def dgda_transition(self, q, k, v, b, w, la):
        return torch.from_numpy(self.od.dgda_transition(to_np(q), to_np(k), to_np(v), b=to_np(b), w=to_np(w),
                                                        log_alpha=to_np(la))).float()

    def dgda_prefill(self, q, k, v, b, w, la, initial_state):
        o, S = self.od.dgda_sequential(to_np(q), to_np(k), to_np(v), b=to_np(b), w=to_np(w),
                                       initial_state=None if initial_state is None else to_np(initial_state),
                                       log_alpha=to_np(la))
        return self._t(o, q), torch.from_numpy(S).float()

    def compute_centroids(self, k_idx, block):
        return self._t(self.oi.compute_centroids(to_np(k_idx), block), k_idx)

    def hca_pool(self, c, r):
        return self._t(self.oi.hca_pool(to_np(c), r), c)

    def index_topk_at(self, q_idx, cent, lam, top_k, block, q_pos0):
        B, Ls, D = q_idx.shape
        qf = np.zeros((B, q_pos0 + Ls, D), np.float32)
        qf[:, q_pos0:] = to_np(q_idx)
        return torch.from_numpy(self.oi.index_topk(qf, to_np(cent), lam, top_k, block,
                                                   rows=np.arange(q_pos0, q_pos0 + Ls)))

    def sa_attention(self, qhat, c, hca, idx, gate, window, sinks, block, r):
        nc = c.shape[1] // r
        pooled = self.oi.hca_pool(to_np(c), r)[:, :nc]
        got = np.zeros_like(pooled) if hca is None else to_np(hca)
        assert got.shape == pooled.shape and np.allclose(got, pooled, rtol=1e-6, atol=1e-6), "pooled HCA rows"
        o = self.oa.sa_attention_latent(to_np(qhat), to_np(c), to_np(idx), to_np(gate), window, sinks, block, r)
        return self._t(o, qhat)
