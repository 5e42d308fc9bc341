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
