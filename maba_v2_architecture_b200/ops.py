"""The five registry ops of the Maba v2 hot path, plus the MABA-SA latent attention.

Each function keeps the call signature, argument meaning, validation errors
and output contract of the reference op it replaces (cited per function) and
runs the sm_100a kernels of libmaba_b200.so through the C ABI.  Inputs are never
mutated; outputs are freshly allocated in the input dtype; work is enqueued on
the current CUDA stream without a device synchronisation.  CPU tensors raise
(this backend has no CPU path).
"""
from __future__ import annotations

import math
from typing import Any, Optional, Tuple, Union

import torch

from . import _native as N

SUPPORTED_DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.float64)


# ---------------------------------------------------------------------------
# validation (same checks and exception types as the reference validators)
# ---------------------------------------------------------------------------
def _check_same(tensors, device, dtype, what="q"):
    for name, t in tensors:
        if t is None:
            continue
        if t.device != device:
            raise RuntimeError(
                f"Expected all tensors to be on the same device, but got {device} and {t.device} for {name}"
            )
    if dtype not in SUPPORTED_DTYPES:
        raise TypeError(f"Unsupported dtype {dtype}. Supported: {SUPPORTED_DTYPES}")
    for name, t in tensors:
        if t is not None and t.dtype != dtype:
            raise TypeError(f"Tensor dtypes must match, but got {dtype} for {what} and {t.dtype} for {name}")


def _state_check(state, q, name):
    """A float32 state with 16-bit inputs is accepted (this backend keeps fp32 recurrent
    state); any other dtype mismatch raises as in the reference."""
    if state is None:
        return None
    if state.dtype == torch.float32 and q.dtype in (torch.float16, torch.bfloat16):
        if state.device != q.device:
            raise RuntimeError(
                f"Expected all tensors to be on the same device, but got {q.device} and {state.device} for {name}"
            )
        return None
    return state


def validate_dgda_prefill_inputs(q, k, v, alpha=None, b=None, w=None, initial_state=None, log_alpha=None):
    """Mirrors maba_sparse/kernels/common.py:13-91 (validate_dgda_prefill_inputs)."""
    if alpha is None and log_alpha is None:
        raise ValueError("Either alpha or log_alpha must be provided")
    if b is None or w is None:
        raise ValueError("Both b and w gate tensors must be provided")
    _check_same([("k", k), ("v", v), ("b", b), ("w", w), ("alpha", alpha), ("log_alpha", log_alpha),
                 ("initial_state", _state_check(initial_state, q, "initial_state"))], q.device, q.dtype)
    if q.dim() != 4:
        raise ValueError(f"q must be 4D [B, H, L, dk], got shape {list(q.shape)}")
    B, H, L, dk = q.shape
    if k.shape != (B, H, L, dk):
        raise ValueError(f"k shape {list(k.shape)} must match q shape {(B, H, L, dk)}")
    if v.dim() != 4 or v.shape[:3] != (B, H, L):
        raise ValueError(f"v shape {list(v.shape)} must have first 3 dims {(B, H, L)}")
    dv = v.shape[3]
    if alpha is not None and alpha.shape != (B, H, L, dk):
        raise ValueError(f"alpha shape {list(alpha.shape)} must match {(B, H, L, dk)}")
    if log_alpha is not None and log_alpha.shape != (B, H, L, dk):
        raise ValueError(f"log_alpha shape {list(log_alpha.shape)} must match {(B, H, L, dk)}")
    if b.shape != (B, H, L, dk):
        raise ValueError(f"b shape {list(b.shape)} must match {(B, H, L, dk)}")
    if w.shape != (B, H, L, dv):
        raise ValueError(f"w shape {list(w.shape)} must match {(B, H, L, dv)}")
    if initial_state is not None and initial_state.shape != (B, H, dk, dv):
        raise ValueError(f"initial_state shape {list(initial_state.shape)} must match {(B, H, dk, dv)}")


def validate_dgda_step_inputs(q, k, v, alpha=None, b=None, w=None, state=None, log_alpha=None):
    """Mirrors maba_sparse/kernels/common.py:93-157 (validate_dgda_step_inputs)."""
    if alpha is None and log_alpha is None:
        raise ValueError("Either alpha or log_alpha must be provided")
    if b is None or w is None:
        raise ValueError("Both b and w gate tensors must be provided")
    _check_same([("k", k), ("v", v), ("b", b), ("w", w), ("alpha", alpha), ("log_alpha", log_alpha),
                 ("state", _state_check(state, q, "state"))], q.device, q.dtype)
    q3 = q.squeeze(2) if (q.dim() == 4 and q.shape[2] == 1) else q
    if q3.dim() != 3:
        raise ValueError(f"q must be [B, H, dk] or [B, H, 1, dk], got {list(q.shape)}")
    B, H, dk = q3.shape
    v3 = v.squeeze(2) if (v.dim() == 4 and v.shape[2] == 1) else v
    if v3.dim() != 3 or v3.shape[:2] != (B, H):
        raise ValueError(f"v must be [B, H, dv] matching B={B}, H={H}, got {list(v.shape)}")
    dv = v3.shape[-1]
    if state is not None and state.shape != (B, H, dk, dv):
        raise ValueError(f"state shape {list(state.shape)} must match {(B, H, dk, dv)}")


def validate_superposition_inputs(o_local, o_sparse, o_hca, gate=None):
    """Mirrors maba_sparse/kernels/common.py:195-226 (validate_superposition_inputs)."""
    device = o_local.device
    if o_sparse.device != device or o_hca.device != device:
        raise RuntimeError("Expected all tensors to be on the same device")
    if o_local.shape != o_sparse.shape or o_local.shape != o_hca.shape:
        raise ValueError(
            f"Shape mismatch: o_local={list(o_local.shape)}, o_sparse={list(o_sparse.shape)}, "
            f"o_hca={list(o_hca.shape)}"
        )
    if gate is not None:
        if gate.device != device:
            raise RuntimeError("Expected all tensors to be on the same device")
        if gate.shape[-1] != 3:
            raise ValueError(f"Gate tensor last dimension must be 3, got {gate.shape[-1]}")
        if gate.shape[0] != o_local.shape[0]:
            raise ValueError(f"Gate tensor batch size must match {o_local.shape[0]}")


# ---------------------------------------------------------------------------
# DGDA
# ---------------------------------------------------------------------------
def b200_dgda_prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    alpha: Optional[torch.Tensor] = None,
    b: Optional[torch.Tensor] = None,
    w: Optional[torch.Tensor] = None,
    chunk_size: int = 16,
    initial_state: Optional[torch.Tensor] = None,
    log_alpha: Optional[torch.Tensor] = None,
    **kwargs: Any,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Chunked DGDA prefill; replaces the ``dgda_prefill`` op.

    Reference: maba_sparse/kernels/common.py:229-268 (ref_dgda_prefill) and
    cpu_dgda.py:33-197 (cpu_dgda_prefill).  ``inversion_method`` / ``adaptive_tol``
    are accepted and ignored (the solve is always exact); ``chunk_size`` is
    accepted and ignored (the recurrence is chunk-invariant).

    Extra keywords of this backend: ``state_dtype`` (keep the state in another
    dtype, e.g. float32 for 16-bit inputs) and ``out_layout="blhd"`` (write the
    output token-major, returned as a [B,H,L,dv] view, so a caller that
    transposes back gets a contiguous tensor for free).
    """
    validate_dgda_prefill_inputs(q, k, v, alpha, b, w, initial_state, log_alpha)
    N.require_cuda(q, op="dgda_prefill")
    B, H, L, dk = q.shape
    dv = v.shape[-1]
    state_dtype = kwargs.get("state_dtype", initial_state.dtype if initial_state is not None else q.dtype)
    if L == 0:
        fin = (initial_state.clone().to(state_dtype) if initial_state is not None
               else torch.zeros(B, H, dk, dv, dtype=state_dtype, device=q.device))
        return torch.empty(B, H, 0, dv, dtype=q.dtype, device=q.device), fin
    if kwargs.get("out_layout") == "blhd":
        out = torch.empty(B, L, H, dv, dtype=q.dtype, device=q.device).transpose(1, 2)
    else:
        out = torch.empty(B, H, L, dv, dtype=q.dtype, device=q.device)
    fin = torch.empty(B, H, dk, dv, dtype=state_dtype, device=q.device)
    if initial_state is not None and initial_state.dtype != state_dtype:
        initial_state = initial_state.to(state_dtype)
    lib = N.lib()
    dt = N.DTYPE_CODES[q.dtype]
    nbytes = lib.maba_dgda_prefill_workspace_size(dt, B, H, L, dk, dv)
    ws = N.workspace(nbytes, q.device)
    ds = [N.desc(t) for t in (q, k, v, alpha, log_alpha, b, w, initial_state, out, fin)]
    rc = lib.maba_dgda_prefill(
        *[N.ref(d) for d in ds],
        int(chunk_size),
        ws.data_ptr() if ws is not None else None,
        int(nbytes),
        N.stream_of(q),
    )
    N.check(rc, "maba_dgda_prefill")
    return out, fin


def b200_dgda_transition(q, k, v, alpha=None, b=None, w=None, log_alpha=None) -> torch.Tensor:
    """Affine transition [R | P] ([B,H,64,128] fp32) of the segment on the state: S_end = P S_start + R."""
    validate_dgda_prefill_inputs(q, k, v, alpha, b, w, None, log_alpha)
    N.require_cuda(q, op="dgda_transition")
    B, H, L, _ = q.shape
    out = torch.empty(B, H, 64, 128, dtype=torch.float32, device=q.device)
    lib = N.lib()
    nbytes = lib.maba_dgda_transition_workspace_size(N.DTYPE_CODES[q.dtype], B, H, L)
    ws = N.workspace(nbytes, q.device)
    ds = [N.desc(t) for t in (q, k, v, alpha, log_alpha, b, w, out)]
    rc = lib.maba_dgda_transition(*[N.ref(d) for d in ds], ws.data_ptr(), int(nbytes), N.stream_of(q))
    N.check(rc, "maba_dgda_transition")
    return out


def b200_dgda_frontend(proj, conv_w, hist=None, n_heads: int = 10, eps: float = 1e-6, new_hist: bool = True,
                       hist_dtype: Optional[torch.dtype] = None, out: Optional[torch.Tensor] = None):
    """The DGDA layer's feature path after its projections, in one kernel.

    Reference: maba_sparse/layers/dgda.py:103-122 (_apply_conv: causal depthwise
    conv with history, SiLU), :192-197 (gates) and :207 (k / (||k|| + eps)).
    ``proj``: six [B,L,C] tensors (q, k, v, alpha, erase, write projections; any
    strides, e.g. column slices of one fused projection); ``conv_w``: three [C,K]
    taps; ``hist``: None or three [B,C,K-1] conv histories (oldest first).
    Returns ``(feats, new_hist)``: feats = (q, k, v, log_alpha, b, w), [B,L,C] column
    views of one token-major buffer ``out`` ([B,L,sum C], allocated when None);
    new_hist = three [B,C,K-1] tensors in ``hist_dtype`` (default: the feature dtype),
    or None when ``new_hist`` is False."""
    x0 = proj[0]
    N.require_cuda(*proj, *conv_w, op="dgda_frontend")
    B, L, _ = x0.shape
    widths = [int(t.shape[2]) for t in proj]
    total = sum(widths)
    if out is None:
        out = torch.empty(B, L, total, dtype=x0.dtype, device=x0.device)
    feats, c0 = [], 0
    for wd in widths:
        feats.append(out[:, :, c0:c0 + wd])
        c0 += wd
    K = int(conv_w[0].shape[1])
    nh = None
    if new_hist:
        hd = hist_dtype or (hist[0].dtype if hist is not None else x0.dtype)
        nh = [torch.empty(B, widths[i], K - 1, dtype=hd, device=x0.device) for i in range(3)]
    rc = N.lib().maba_dgda_frontend(N.desc_array(proj), N.desc_array(conv_w),
                                    N.desc_array(hist) if hist is not None else None, N.desc_array(feats),
                                    N.desc_array(nh) if nh is not None else None, int(n_heads), float(eps),
                                    N.stream_of(x0))
    N.check(rc, "maba_dgda_frontend")
    return tuple(feats), nh


def _squeeze_step(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if t is not None and t.dim() == 4 and t.shape[2] == 1:
        return t.squeeze(2)
    return t


def b200_dgda_step(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    alpha: Optional[torch.Tensor] = None,
    b: Optional[torch.Tensor] = None,
    w: Optional[torch.Tensor] = None,
    state: Optional[torch.Tensor] = None,
    log_alpha: Optional[torch.Tensor] = None,
    **kwargs: Any,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """One DGDA decode step; replaces the ``dgda_step`` op.

    Reference: maba_sparse/kernels/common.py:271-309 (ref_dgda_step),
    cpu_dgda.py:200-261.  ``alpha`` has priority over ``log_alpha``.  Returns
    ``(o [B,H,dv], new_state [B,H,dk,dv])``; ``state_dtype`` as for prefill.
    """
    validate_dgda_step_inputs(q, k, v, alpha, b, w, state, log_alpha)
    N.require_cuda(q, op="dgda_step")
    q, k, v, alpha, b, w, log_alpha = map(_squeeze_step, (q, k, v, alpha, b, w, log_alpha))
    B, H, dk = q.shape
    dv = v.shape[-1]
    state_dtype = kwargs.get("state_dtype", state.dtype if state is not None else q.dtype)
    if state is not None and state.dtype != state_dtype:
        state = state.to(state_dtype)
    out = torch.empty(B, H, dv, dtype=q.dtype, device=q.device)
    new_state = torch.empty(B, H, dk, dv, dtype=state_dtype, device=q.device)
    ds = [N.desc(t) for t in (q, k, v, alpha, log_alpha, b, w, state, out, new_state)]
    rc = N.lib().maba_dgda_step(*[N.ref(d) for d in ds], N.stream_of(q))
    N.check(rc, "maba_dgda_step")
    return out, new_state


# ---------------------------------------------------------------------------
# DG-Indexer
# ---------------------------------------------------------------------------
def b200_compute_centroids(k_idx: torch.Tensor, block_size: int = 64, **kwargs: Any) -> torch.Tensor:
    """Block pooling 0.5*(mean+max); replaces ``compute_centroids``.

    Reference: maba_sparse/kernels/common.py:329-350, cpu_indexer.py:16-50.
    """
    if k_idx.dim() != 3:
        raise ValueError(f"k_idx must be 3D [B, L, d_idx], got {list(k_idx.shape)}")
    if block_size <= 0:
        raise ValueError(f"block_size must be positive, got {block_size}")
    B, L, d = k_idx.shape
    if d <= 0:
        raise ValueError(f"d_idx must be positive, got {d}")
    N.require_cuda(k_idx, op="compute_centroids")
    if L == 0:
        return torch.empty(B, 0, d, dtype=k_idx.dtype, device=k_idx.device)
    nb = (L + block_size - 1) // block_size
    out = torch.empty(B, nb, d, dtype=k_idx.dtype, device=k_idx.device)
    rc = N.lib().maba_compute_centroids(N.ref(N.desc(k_idx)), N.ref(N.desc(out)), int(block_size),
                                        N.stream_of(k_idx))
    N.check(rc, "maba_compute_centroids")
    return out


def b200_index_topk(
    q_idx: torch.Tensor,
    centroids: torch.Tensor,
    lambda_dist: float = 0.5,
    top_k: int = 32,
    block_size: int = 64,
    return_scores: bool = False,
    **kwargs: Any,
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Fused centroid scoring + top-k; replaces ``index_topk``.

    Reference: maba_sparse/kernels/common.py:353-403 and cpu_indexer.py:54-112
    (the dispatched CPU path: fp32 scores, log1p penalty).  ``dist_lambda`` in
    kwargs overrides ``lambda_dist``.  With ``decode=True`` the query block is
    ``nb-1`` for every token (maba_sparse/layers/indexer.py:101-112).
    Index order: score descending, ties to the lower block index; slots past
    the finite candidates hold the lowest unused future block indices.
    """
    lam = kwargs.get("dist_lambda", lambda_dist)
    decode = bool(kwargs.get("decode", False))
    q_pos0 = int(kwargs.get("q_pos0", 0))  # absolute position of row 0 (a sequence segment); prefill only
    if q_idx.device != centroids.device:
        raise RuntimeError(
            f"Expected all tensors to be on the same device, got {q_idx.device} and {centroids.device}"
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
    N.require_cuda(q_idx, op="index_topk")
    B, L, d = q_idx.shape
    nb = centroids.shape[1]
    ak = min(top_k, nb)
    if centroids.dtype != q_idx.dtype:
        centroids = centroids.to(q_idx.dtype)
    if L == 0 or nb == 0:
        idx = torch.zeros(B, L, ak, dtype=torch.long, device=q_idx.device)
        if return_scores:
            return idx, torch.zeros(B, L, nb, dtype=q_idx.dtype, device=q_idx.device)
        return idx
    idx = torch.empty(B, L, ak, dtype=torch.long, device=q_idx.device)
    scores = torch.empty(B, L, nb, dtype=q_idx.dtype, device=q_idx.device) if return_scores else None
    lib = N.lib()
    if q_pos0 and not decode:
        nbytes = lib.maba_index_topk_at_workspace_size(B, L, nb, int(top_k), int(block_size), q_pos0)
        ws = N.workspace(nbytes, q_idx.device)
        rc = lib.maba_index_topk_at(
            N.ref(N.desc(q_idx)), N.ref(N.desc(centroids)), float(lam), int(top_k), int(block_size), q_pos0,
            N.ref(N.desc(idx)), N.ref(N.desc(scores)), ws.data_ptr(), int(nbytes), N.stream_of(q_idx),
        )
    else:
        nbytes = lib.maba_index_topk_workspace_size(B, L, nb, int(top_k))
        ws = N.workspace(nbytes, q_idx.device)
        rc = lib.maba_index_topk(
            N.ref(N.desc(q_idx)), N.ref(N.desc(centroids)), float(lam), int(top_k), int(block_size), int(decode),
            N.ref(N.desc(idx)), N.ref(N.desc(scores)), ws.data_ptr(), int(nbytes), N.stream_of(q_idx),
        )
    N.check(rc, "maba_index_topk")
    if return_scores:
        return idx, scores
    return idx


# ---------------------------------------------------------------------------
# superposition
# ---------------------------------------------------------------------------
def b200_stream_superposition(
    o_local: torch.Tensor,
    o_sparse: torch.Tensor,
    o_hca: torch.Tensor,
    gate_logits: Optional[torch.Tensor] = None,
    gate_weights: Optional[torch.Tensor] = None,
    **kwargs: Any,
) -> torch.Tensor:
    """Gate softmax superposition; replaces ``stream_superposition``.

    Reference: maba_sparse/kernels/common.py:406-438, cpu_indexer.py:116-150.
    """
    gate = gate_logits if gate_logits is not None else gate_weights
    validate_superposition_inputs(o_local, o_sparse, o_hca, gate)
    N.require_cuda(o_local, op="stream_superposition")
    if o_local.shape[2] == 0:
        return torch.empty_like(o_local)
    if gate is None:
        raise ValueError("Either gate_logits or gate_weights must be provided")
    if gate.dim() not in (3, 4):
        raise ValueError(f"Gate tensor must be 3D or 4D, got {gate.dim()}D")
    if o_sparse.dtype != o_local.dtype:
        o_sparse = o_sparse.to(o_local.dtype)
    if o_hca.dtype != o_local.dtype:
        o_hca = o_hca.to(o_local.dtype)
    if gate.dtype != o_local.dtype:
        gate = gate.to(o_local.dtype)
    out = torch.empty(o_local.shape, dtype=o_local.dtype, device=o_local.device)
    rc = N.lib().maba_stream_superposition(
        N.ref(N.desc(o_local)), N.ref(N.desc(o_sparse)), N.ref(N.desc(o_hca)), N.ref(N.desc(gate)),
        1 if gate_logits is not None else 0, N.ref(N.desc(out)), N.stream_of(o_local),
    )
    N.check(rc, "maba_stream_superposition")
    return out


# ---------------------------------------------------------------------------
# MABA-SA latent attention
# ---------------------------------------------------------------------------
def b200_hca_pool(c_kv: torch.Tensor, r: int = 64, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Mean of each complete r-row block of the latent cache.

    Reference: maba_sparse/layers/sparse_attention.py:206.
    """
    N.require_cuda(c_kv, op="hca_pool")
    B, L, dc = c_kv.shape
    nc = L // r
    out = torch.empty(B, nc, dc, dtype=out_dtype or c_kv.dtype, device=c_kv.device)
    if nc == 0 or B == 0:
        return out
    rc = N.lib().maba_hca_pool(N.ref(N.desc(c_kv)), N.ref(N.desc(out)), int(r), N.stream_of(c_kv))
    N.check(rc, "maba_hca_pool")
    return out


def b200_sa_attention(
    qhat: torch.Tensor,
    c_kv: torch.Tensor,
    hca: Optional[torch.Tensor],
    top_idx: torch.Tensor,
    gate_logits: torch.Tensor,
    window_size: int = 128,
    n_sinks: int = 4,
    block_size: int = 64,
    hca_r: int = 64,
) -> torch.Tensor:
    """Fused local + sparse + HCA attention and gate superposition in latent space.

    qhat [B,Lq,H,d_c] (already scaled absorbed queries), c_kv [B,Lkv,d_c],
    hca [B,Lkv//r,d_c] pooled table, top_idx [B,Lq,K] int64, gate_logits
    [B,Lq,3] or [B,H,Lq,3].  Returns [B,Lq,H,d_c]; apply W_uv per head next.
    Reference: maba_sparse/layers/sparse_attention.py:79-219 and 274-275.
    """
    N.require_cuda(qhat, c_kv, top_idx, gate_logits, op="sa_attention")
    B, Lq, H, dc = qhat.shape
    Lkv = c_kv.shape[1]
    if c_kv.dtype != qhat.dtype:
        c_kv = c_kv.to(qhat.dtype)
    if hca is not None and hca.dtype != qhat.dtype:
        hca = hca.to(qhat.dtype)
    if gate_logits.dtype != qhat.dtype:
        gate_logits = gate_logits.to(qhat.dtype)
    if top_idx.dtype != torch.long:
        top_idx = top_idx.long()
    out = torch.empty(B, Lq, H, dc, dtype=qhat.dtype, device=qhat.device)
    if B == 0 or Lq == 0:
        return out
    lib = N.lib()
    K = top_idx.shape[-1]
    nbytes = lib.maba_sa_attention_workspace_size(N.DTYPE_CODES[qhat.dtype], B, Lq, Lkv, H, dc, K, int(window_size),
                                                  int(n_sinks), int(block_size), int(hca_r))
    ws = N.workspace(nbytes, qhat.device)
    rc = lib.maba_sa_attention(
        N.ref(N.desc(qhat)), N.ref(N.desc(c_kv)), N.ref(N.desc(hca)), N.ref(N.desc(top_idx)),
        N.ref(N.desc(gate_logits)), N.ref(N.desc(out)), int(window_size), int(n_sinks), int(block_size), int(hca_r),
        ws.data_ptr() if ws is not None else None, int(nbytes), N.stream_of(qhat),
    )
    N.check(rc, "maba_sa_attention")
    return out


# ---------------------------------------------------------------------------
# decode at a device-held position (CUDA-graph friendly)
# ---------------------------------------------------------------------------
def b200_decode_cache_append(c_new, k_new, c_cache, kidx_cache, cent_table, hca_table, pos_dev, block_size=64,
                             hca_r=64) -> None:
    """Append one latent / index-key row at *pos_dev and refresh the block centroid / pooled row in place."""
    N.require_cuda(c_new, c_cache, op="decode_cache_append")
    rc = N.lib().maba_decode_cache_append(
        N.ref(N.desc(c_new)), N.ref(N.desc(k_new)), N.ref(N.desc(c_cache)), N.ref(N.desc(kidx_cache)),
        N.ref(N.desc(cent_table)), N.ref(N.desc(hca_table)), pos_dev.data_ptr(), int(block_size), int(hca_r),
        N.stream_of(c_cache))
    N.check(rc, "maba_decode_cache_append")


def b200_index_topk_decode_at(q_idx, cent_table, pos_dev, lambda_dist=0.5, top_k=32, block_size=64):
    N.require_cuda(q_idx, cent_table, op="index_topk_decode_at")
    B, _, _ = q_idx.shape
    nbcap = cent_table.shape[1]
    idx = torch.empty(B, 1, min(top_k, nbcap), dtype=torch.long, device=q_idx.device)
    lib = N.lib()
    nbytes = lib.maba_index_topk_decode_at_workspace_size(B, nbcap, int(top_k))
    ws = N.workspace(nbytes, q_idx.device)
    rc = lib.maba_index_topk_decode_at(N.ref(N.desc(q_idx)), N.ref(N.desc(cent_table)), float(lambda_dist),
                                       int(top_k), int(block_size), pos_dev.data_ptr(), N.ref(N.desc(idx)),
                                       ws.data_ptr(), int(nbytes), N.stream_of(q_idx))
    N.check(rc, "maba_index_topk_decode_at")
    return idx


def b200_sa_attention_decode_at(qhat, c_cache, hca_table, top_idx, gate_logits, pos_dev, window_size=128,
                                n_sinks=4, block_size=64, hca_r=64):
    N.require_cuda(qhat, c_cache, op="sa_attention_decode_at")
    B, _, H, dc = qhat.shape
    out = torch.empty(B, 1, H, dc, dtype=qhat.dtype, device=qhat.device)
    lib = N.lib()
    nbytes = lib.maba_sa_attention_decode_at_workspace_size(B, c_cache.shape[1], hca_table.shape[1], H, dc,
                                                            top_idx.shape[-1], int(window_size), int(n_sinks),
                                                            int(block_size), int(hca_r))
    ws = N.workspace(nbytes, qhat.device)
    rc = lib.maba_sa_attention_decode_at(
        N.ref(N.desc(qhat)), N.ref(N.desc(c_cache)), N.ref(N.desc(hca_table)), N.ref(N.desc(top_idx)),
        N.ref(N.desc(gate_logits)), N.ref(N.desc(out)), pos_dev.data_ptr(), int(window_size), int(n_sinks),
        int(block_size), int(hca_r), ws.data_ptr() if ws is not None else None, int(nbytes), N.stream_of(qhat))
    N.check(rc, "maba_sa_attention_decode_at")
    return out


def absorb_queries(q: torch.Tensor, w_uk: torch.Tensor, n_heads: int, scale: float) -> torch.Tensor:
    """qhat[b,t,h,:] = scale * W_uk,h^T q[b,t,h,:] with W_uk = k_up_proj.weight [H*dh, d_c].

    One batched GEMM over the heads with the scale folded into the (small) weight;
    the result is a [B, L, H, d_c] view of an [H, B*L, d_c] buffer (the attention
    kernels take strided queries), so no layout copy follows the GEMM."""
    B, L, H, dh = q.shape
    w = (w_uk.view(n_heads, dh, -1).float() * scale).to(q.dtype)
    qh = torch.bmm(q.reshape(B * L, H, dh).transpose(0, 1), w)
    return qh.view(H, B, L, -1).permute(1, 2, 0, 3)


def expand_values(o_lat: torch.Tensor, w_uv: torch.Tensor, n_heads: int) -> torch.Tensor:
    """o[b,t,h,:] = W_uv,h o_lat[b,t,h,:] with W_uv = v_up_proj.weight [H*dh, d_c].

    One batched GEMM over the heads; the result is a [B, L, H, dh] view of an
    [H, B*L, dh] buffer."""
    B, L, H, dc = o_lat.shape
    dh = w_uv.shape[0] // n_heads
    w = w_uv.view(n_heads, dh, dc).transpose(1, 2).to(o_lat.dtype)
    o = torch.bmm(o_lat.reshape(B * L, H, dc).transpose(0, 1), w)
    return o.view(H, B, L, dh).permute(1, 2, 0, 3)


__all__ = [
    "b200_dgda_prefill",
    "b200_dgda_step",
    "b200_compute_centroids",
    "b200_index_topk",
    "b200_stream_superposition",
    "b200_hca_pool",
    "b200_sa_attention",
    "b200_dgda_transition",
    "b200_dgda_frontend",
    "b200_decode_cache_append",
    "b200_index_topk_decode_at",
    "b200_sa_attention_decode_at",
    "absorb_queries",
    "expand_values",
    "validate_dgda_prefill_inputs",
    "validate_dgda_step_inputs",
    "validate_superposition_inputs",
]
