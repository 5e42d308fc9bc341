"""Kernel registry with the reference dispatcher's interface and one backend.

Mirrors maba_sparse/kernels/dispatcher.py (``_KERNEL_REGISTRY`` :31-48,
``register_kernel`` :71, ``get_kernel`` :80, ``get_backend`` :181,
``dispatch_*`` :258-508) so code written against the reference registry runs
unchanged.  Differences by design:

* the only backend is ``"b200"`` (hand-written sm_100a kernels); ``MABA_BACKEND``
  accepts ``auto``, ``b200`` and the reference's GPU aliases ``triton``,
  ``cuda`` and ``gpu``; any other value raises ``ValueError`` as the reference
  does for an unknown name;
* there is no fallback: a failing kernel raises instead of silently running a
  CPU implementation (the reference's ``MABA_STRICT_BACKEND=1`` behaviour is
  the only behaviour).
"""
from __future__ import annotations

import os
import threading
from typing import Any, Callable, Dict, Optional, Tuple, Union

import torch

from .ops import (
    b200_compute_centroids,
    b200_dgda_prefill,
    b200_dgda_step,
    b200_index_topk,
    b200_stream_superposition,
    validate_superposition_inputs,
)

BACKEND = "b200"
OPS = ("dgda_prefill", "dgda_step", "compute_centroids", "index_topk", "stream_superposition")

_KERNEL_REGISTRY: Dict[str, Dict[str, Callable]] = {
    BACKEND: {
        "dgda_prefill": b200_dgda_prefill,
        "dgda_step": b200_dgda_step,
        "compute_centroids": b200_compute_centroids,
        "index_topk": b200_index_topk,
        "stream_superposition": b200_stream_superposition,
    }
}

_BACKEND_CACHE: Dict[Tuple[Optional[str], Optional[int], Optional[str]], str] = {}
_CACHE_LOCK = threading.Lock()
_ALIASES = ("auto", "b200", "triton", "cuda", "gpu")


def clear_dispatcher_cache() -> None:
    with _CACHE_LOCK:
        _BACKEND_CACHE.clear()


def clear_fallback_warnings() -> None:
    """Kept for API parity (this dispatcher never falls back, so never warns)."""
    clear_dispatcher_cache()


def register_kernel(backend: str, op_name: str) -> Callable:
    def decorator(fn: Callable) -> Callable:
        _KERNEL_REGISTRY.setdefault(backend, {})[op_name] = fn
        return fn

    return decorator


def get_kernel(backend: str, op_name: str) -> Optional[Callable]:
    return _KERNEL_REGISTRY.get(backend, {}).get(op_name)


def get_backend(device: Union[torch.device, str, None] = None) -> str:
    dev_type: Optional[str] = None
    dev_idx: Optional[int] = None
    if device is not None:
        d = torch.device(device) if isinstance(device, str) else device
        dev_type, dev_idx = d.type, (d.index if d.index is not None else 0)
    env = os.environ.get("MABA_BACKEND")
    key = (dev_type, dev_idx, env)
    with _CACHE_LOCK:
        hit = _BACKEND_CACHE.get(key)
    if hit is not None:
        return hit
    if env and env.lower() not in _ALIASES:
        raise ValueError(f"Unsupported MABA_BACKEND '{env}'. Supported: {list(_ALIASES)}")
    with _CACHE_LOCK:
        _BACKEND_CACHE[key] = BACKEND
    return BACKEND


def _run(op: str, device: torch.device, **kwargs: Any):
    fn = get_kernel(get_backend(device), op)
    if fn is None:
        raise RuntimeError(f"[maba_b200] no kernel registered for '{op}'")
    return fn(**kwargs)


def _check_gate_args(alpha, log_alpha, b, w):
    if alpha is None and log_alpha is None:
        raise ValueError("Either alpha or log_alpha must be provided")
    if b is None or w is None:
        raise ValueError("Both b and w gate tensors must be provided")


def dispatch_dgda_prefill(q, k, v, alpha=None, b=None, w=None, chunk_size: int = 16, initial_state=None,
                          log_alpha=None, **kwargs: Any):
    """Reference: maba_sparse/kernels/dispatcher.py:258-327."""
    _check_gate_args(alpha, log_alpha, b, w)
    return _run("dgda_prefill", q.device, q=q, k=k, v=v, alpha=alpha, b=b, w=w, chunk_size=chunk_size,
                initial_state=initial_state, log_alpha=log_alpha, **kwargs)


def dispatch_dgda_step(q, k, v, alpha=None, b=None, w=None, state=None, log_alpha=None, **kwargs: Any):
    """Reference: maba_sparse/kernels/dispatcher.py:330-396."""
    _check_gate_args(alpha, log_alpha, b, w)
    return _run("dgda_step", q.device, q=q, k=k, v=v, alpha=alpha, b=b, w=w, state=state, log_alpha=log_alpha,
                **kwargs)


def dispatch_compute_centroids(k_idx, block_size: int = 64, **kwargs: Any):
    """Reference: maba_sparse/kernels/dispatcher.py:399-421."""
    if k_idx.dim() != 3:
        raise ValueError(f"k_idx must be 3D [B, L, d_idx], got shape {list(k_idx.shape)}")
    if block_size <= 0:
        raise ValueError(f"block_size must be positive, got {block_size}")
    return _run("compute_centroids", k_idx.device, k_idx=k_idx, block_size=block_size, **kwargs)


def dispatch_index_topk(q_idx, centroids, lambda_dist: float = 0.5, top_k: int = 32, block_size: int = 64,
                        **kwargs: Any):
    """Reference: maba_sparse/kernels/dispatcher.py:424-465."""
    if q_idx.device != centroids.device:
        raise RuntimeError(
            f"Expected all tensors to be on the same device, but got {q_idx.device} and {centroids.device}"
        )
    if q_idx.dim() != 3 or centroids.dim() != 3:
        raise ValueError(f"q_idx and centroids must be 3D, got {q_idx.dim()}D and {centroids.dim()}D")
    if q_idx.shape[0] != centroids.shape[0] or q_idx.shape[2] != centroids.shape[2]:
        raise ValueError(
            f"Dimension mismatch between q_idx {list(q_idx.shape)} and centroids {list(centroids.shape)}"
        )
    if top_k <= 0:
        raise ValueError(f"top_k must be positive, got {top_k}")
    if block_size <= 0:
        raise ValueError(f"block_size must be positive, got {block_size}")
    return _run("index_topk", q_idx.device, q_idx=q_idx, centroids=centroids, lambda_dist=lambda_dist,
                top_k=top_k, block_size=block_size, **kwargs)


def dispatch_stream_superposition(o_local, o_sparse, o_hca, gate_logits=None, **kwargs: Any):
    """Reference: maba_sparse/kernels/dispatcher.py:468-508."""
    gate = gate_logits if gate_logits is not None else kwargs.get("gate_weights")
    validate_superposition_inputs(o_local, o_sparse, o_hca, gate)
    return _run("stream_superposition", o_local.device, o_local=o_local, o_sparse=o_sparse, o_hca=o_hca,
                gate_logits=gate_logits, **kwargs)


dgda_prefill = dispatch_dgda_prefill
dgda_step = dispatch_dgda_step
compute_centroids = dispatch_compute_centroids
index_topk = dispatch_index_topk
stream_superposition = dispatch_stream_superposition

__all__ = [
    "BACKEND",
    "OPS",
    "get_backend",
    "register_kernel",
    "get_kernel",
    "clear_fallback_warnings",
    "clear_dispatcher_cache",
    "dispatch_dgda_prefill",
    "dispatch_dgda_step",
    "dispatch_compute_centroids",
    "dispatch_index_topk",
    "dispatch_stream_superposition",
    "dgda_prefill",
    "dgda_step",
    "compute_centroids",
    "index_topk",
    "stream_superposition",
]
