"""Drop-in installation into the reference package (``maba_sparse``).

``install()`` makes an unchanged reference model (``MabaSparseForCausalLM`` and
its layers) run the hot path on the sm_100a kernels:

* the five registry ops are registered under the reference's CUDA backend name
  (``"triton"``, which ``get_backend`` selects for CUDA tensors,
  maba_sparse/kernels/dispatcher.py:181-238) through its own
  ``register_kernel`` (dispatcher.py:71-77), and its backend cache is cleared;
* the layer-level paths that have no registry op are replaced by method patch:
  ``MabaSparseAttention.forward`` (sparse_attention.py:221-277, whose three
  streams are inline torch code) by the fused latent-attention forward,
  ``DGIndexer.forward`` (indexer.py:43-126, whose decode top-k is inline) by the
  fused-kernel version, and ``DGDALayer.forward`` / ``step`` (dgda.py:166-287,
  whose conv, gates and k norm are separate torch ops) by the version with one
  input GEMM and the fused front-end kernel;
* ``MABA_STRICT_BACKEND=1`` is set so the reference dispatcher raises instead of
  silently falling back to its CPU reference.

``uninstall(handle)`` restores everything.
"""
from __future__ import annotations

import os
from typing import Any, Dict, Optional

from . import layers as _layers
from .dispatcher import OPS
from .ops import (
    b200_compute_centroids,
    b200_dgda_prefill,
    b200_dgda_step,
    b200_index_topk,
    b200_stream_superposition,
)

_OURS = {
    "dgda_prefill": b200_dgda_prefill,
    "dgda_step": b200_dgda_step,
    "compute_centroids": b200_compute_centroids,
    "index_topk": b200_index_topk,
    "stream_superposition": b200_stream_superposition,
}


def install(maba_sparse: Optional[Any] = None, patch_layers: bool = True, strict: bool = True) -> Dict[str, Any]:
    if maba_sparse is None:
        import maba_sparse  # noqa: F811
    import importlib

    importlib.import_module("maba_sparse.kernels")  # registers the reference's own backends first
    disp = importlib.import_module("maba_sparse.kernels.dispatcher")
    handle: Dict[str, Any] = {"registry": {op: disp._KERNEL_REGISTRY.get("triton", {}).get(op) for op in OPS},
                              "env": {k: os.environ.get(k) for k in ("MABA_STRICT_BACKEND", "MABA_BACKEND")},
                              "methods": {}}
    for op in OPS:
        disp.register_kernel("triton", op)(_OURS[op])
    if strict:
        os.environ["MABA_STRICT_BACKEND"] = "1"
    os.environ["MABA_BACKEND"] = "triton"
    disp.clear_dispatcher_cache()
    if patch_layers:
        sa_mod = importlib.import_module("maba_sparse.layers.sparse_attention")
        ix_mod = importlib.import_module("maba_sparse.layers.indexer")
        dg_mod = importlib.import_module("maba_sparse.layers.dgda")
        ref_sa, ref_ix, ref_dg = sa_mod.MabaSparseAttention, ix_mod.DGIndexer, dg_mod.DGDALayer
        patches = [(ref_sa, "forward", _layers.MabaSparseAttention),
                   (ref_sa, "latent_attention", _layers.MabaSparseAttention),
                   (ref_ix, "forward", _layers.DGIndexer), (ref_dg, "forward", _layers.DGDALayer),
                   (ref_dg, "step", _layers.DGDALayer), (ref_dg, "_features", _layers.DGDALayer),
                   (ref_dg, "_in_proj_weight", _layers.DGDALayer)]
        handle["methods"] = {(cls, name): cls.__dict__.get(name) for cls, name, _ in patches}
        for cls, name, ours in patches:
            setattr(cls, name, ours.__dict__[name])
    handle["dispatcher"] = disp
    return handle


def uninstall(handle: Dict[str, Any]) -> None:
    disp = handle["dispatcher"]
    for op, fn in handle["registry"].items():
        if fn is None:
            disp._KERNEL_REGISTRY.get("triton", {}).pop(op, None)
        else:
            disp._KERNEL_REGISTRY["triton"][op] = fn
    for (cls, name), fn in handle["methods"].items():
        if fn is None:
            if name in cls.__dict__:
                delattr(cls, name)
        else:
            setattr(cls, name, fn)
    for k, v in handle["env"].items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    disp.clear_dispatcher_cache()
