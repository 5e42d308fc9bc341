"""DGDA, DG-Indexer and MABA-SA layers on the sm_100a kernels.

Constructor signatures, parameter names (so reference state dicts load),
forward/step signatures, return contracts and decode caches follow
maba_sparse/layers/{dgda,indexer,sparse_attention}.py.  What changes is the
compute behind them:

* DGDA runs its six input projections as one GEMM, then one front-end kernel
  (causal conv + SiLU with history, gates, k L2-norm), and feeds the chunked
  prefill / decode kernels token-major strided views of its output (no
  ``.contiguous()`` copies); the recurrence writes its output token-major, so
  the transpose back before ``o_proj`` is free;
* the indexer's prefill and decode top-k run in one fused kernel each;
* MABA-SA never up-projects keys or values: queries are absorbed into the
  d_c=128 latent space (qhat_h = scale * W_uk,h^T q_h), the three streams and
  the gate superposition run in one kernel over the shared latent rows, and
  W_uv is applied once to the combined latent output.
"""
from __future__ import annotations

import math
from typing import Any, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from .dispatcher import dispatch_compute_centroids, dispatch_dgda_prefill, dispatch_dgda_step, dispatch_index_topk
from .ops import (absorb_queries, b200_dgda_frontend, b200_hca_pool, b200_index_topk, b200_sa_attention,
                  expand_values)


class ConvState(tuple):
    """Tuple of the three conv histories (q, k, v); maba_sparse/layers/dgda.py:10-19."""

    @property
    def shape(self) -> torch.Size:
        if len(self) == 0:
            return torch.Size([0, 0, 0, 0])
        f = self[0]
        return torch.Size([f.shape[0], len(self), f.shape[1], f.shape[2]])

    def as_tensor(self) -> torch.Tensor:
        return torch.stack(self, dim=1)


def _fit_history(t: torch.Tensor, k1: int) -> torch.Tensor:
    """[B, C, n] history -> [B, C, k1]: the last k1 columns, zero-padded on the left."""
    n = t.shape[-1]
    if n == k1:
        return t
    if n > k1:
        return t[..., n - k1:]
    return F.pad(t, (k1 - n, 0))


def conv_history(conv_state, batch: int, widths, k1: int, device, dtype):
    """The three conv histories ([B, C_i, k1], oldest first) from any conv-state form the
    reference layer accepts (maba_sparse/layers/dgda.py:124-164): a (q, k, v) tuple or list,
    such a tuple wrapped in a 1-tuple, a stacked [B, 3, C, n] tensor (also 5-D with the
    history flattened), or a [B, C_total, n] tensor holding q|k|v channels (one shared
    history when C_total is a single width).  None stays None (zero history)."""
    if conv_state is None or k1 == 0:
        return None
    parts = None
    if isinstance(conv_state, (tuple, list)):
        if len(conv_state) == 1 and isinstance(conv_state[0], (tuple, list)):
            conv_state = conv_state[0]
        if len(conv_state) == 3:
            parts = list(conv_state)
    if parts is None:
        if not isinstance(conv_state, torch.Tensor):
            raise ValueError(f"Unsupported conv_state shape or type: {type(conv_state)}")
        t = conv_state
        if t.dim() in (4, 5) and t.shape[1] == 3:
            t = t.reshape(batch, 3, t.shape[2], -1)
            parts = [t[:, i] for i in range(3)]
        else:
            t = t.reshape(batch, -1, k1)
            cqk, cv = widths[0], widths[2]
            tot = t.shape[1]
            if tot == 2 * cqk + cv:
                parts = [t[:, :cqk], t[:, cqk:2 * cqk], t[:, 2 * cqk:]]
            elif tot == cqk and cqk != cv:
                parts = [t, t, torch.zeros(batch, cv, k1, dtype=t.dtype, device=t.device)]
            else:
                parts = [t, t, t]
    return [_fit_history(p_.to(device=device, dtype=dtype), k1) for p_ in parts]


class DGDALayer(nn.Module):
    """Decoupled gated delta attention layer (maba_sparse/layers/dgda.py:22-287)."""

    def __init__(self, config: Optional[Any] = None, dim: int = 640, n_heads: int = 10, d_head: Optional[int] = None,
                 kernel_size: int = 4, eps: float = 1e-6) -> None:
        super().__init__()
        if config is not None:
            dim = getattr(config, "dim", getattr(config, "d_model", dim))
            n_heads = getattr(config, "n_heads", getattr(config, "num_heads", n_heads))
            d_head = getattr(config, "d_head", d_head)
            kernel_size = getattr(config, "kernel_size", getattr(config, "conv_kernel_size", kernel_size))
            eps = getattr(config, "eps", getattr(config, "rms_norm_eps", eps))
        self.dim = dim
        self.n_heads = n_heads
        self.d_head = d_head if d_head is not None else dim // n_heads
        self.d_k = getattr(config, "d_k", self.d_head) if config is not None else self.d_head
        self.d_v = getattr(config, "d_v", self.d_head) if config is not None else self.d_head
        self.kernel_size = kernel_size
        self.k_size = kernel_size
        self.eps = eps
        self.chunk_size = getattr(config, "chunk_size", 16)
        self.inversion_method = getattr(config, "inversion_method", "adaptive")
        self.adaptive_tol = getattr(config, "adaptive_tol", 7e-5)
        # dtype of the recurrent state handed back by forward/step (None: q's dtype, the reference contract)
        self.state_dtype: Optional[torch.dtype] = None
        qk, vd = self.n_heads * self.d_k, self.n_heads * self.d_v
        self.q_proj = nn.Linear(dim, qk, bias=False)
        self.k_proj = nn.Linear(dim, qk, bias=False)
        self.v_proj = nn.Linear(dim, vd, bias=False)
        self.conv_q = nn.Conv1d(qk, qk, kernel_size, groups=qk, bias=False, padding=0)
        self.conv_k = nn.Conv1d(qk, qk, kernel_size, groups=qk, bias=False, padding=0)
        self.conv_v = nn.Conv1d(vd, vd, kernel_size, groups=vd, bias=False, padding=0)
        self.gate_alpha = nn.Linear(dim, qk, bias=False)
        self.gate_erase = nn.Linear(dim, qk, bias=False)
        self.gate_write = nn.Linear(dim, vd, bias=False)
        self.o_proj = nn.Linear(vd, dim, bias=False)
        self._reset_parameters()

    alpha_proj = property(lambda self: self.gate_alpha)
    b_proj = property(lambda self: self.gate_erase)
    w_proj = property(lambda self: self.gate_write)

    def _reset_parameters(self) -> None:
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.gate_alpha, self.gate_erase, self.gate_write,
                    self.o_proj):
            nn.init.xavier_uniform_(lin.weight)
        for conv in (self.conv_q, self.conv_k, self.conv_v):
            nn.init.normal_(conv.weight, mean=0.0, std=0.02)

    def _in_proj_weight(self) -> torch.Tensor:
        """The six input projections (q, k, v, alpha, erase, write) stacked into one
        [4*H*dk + 2*H*dv, dim] weight, so the layer runs one GEMM; rebuilt only when a
        weight changes (new tensor or in-place update)."""
        ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.gate_alpha.weight,
              self.gate_erase.weight, self.gate_write.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype, w.device) for w in ws)
        cached = self.__dict__.get("_in_proj_cache")
        if cached is None or cached[0] != key:
            cached = (key, torch.cat([w.detach() for w in ws], dim=0))
            self.__dict__["_in_proj_cache"] = cached
        return cached[1]

    def _features(self, x, conv_state):
        """Projections (one GEMM) + the fused front end (conv + SiLU, gates, k norm).
        Returns q, k, v, b, w, log_alpha as [B,H,L,d] views of one token-major buffer and
        the new conv state."""
        b, l, _ = x.shape
        h, dk, dv = self.n_heads, self.d_k, self.d_v
        cqk, cv = h * dk, h * dv
        kh = max(self.kernel_size - 1, 0)
        proj = F.linear(x, self._in_proj_weight())
        widths = (cqk, cqk, cv, cqk, cqk, cv)
        cols, c0 = [], 0
        for wd in widths:
            cols.append(proj[:, :, c0:c0 + wd])
            c0 += wd
        hist = conv_history(conv_state, b, (cqk, cqk, cv), kh, x.device, x.dtype)
        taps = [c.weight.detach().view(c.weight.shape[0], -1) for c in (self.conv_q, self.conv_k, self.conv_v)]
        (q, k, v, la, eb, ew), nh = b200_dgda_frontend(cols, taps, hist, n_heads=h, eps=self.eps)

        def heads(t, d):  # token-major [B, L, H*d] viewed as [B, H, L, d]: the kernels read strides
            return t.view(b, l, h, d).transpose(1, 2)

        return (heads(q, dk), heads(k, dk), heads(v, dv), heads(eb, dk), heads(ew, dv), heads(la, dk),
                ConvState(tuple(nh)))

    def forward(self, x: torch.Tensor, state: Optional[torch.Tensor] = None, conv_state=None,
                chunk_size: Optional[int] = None, inversion_method: Optional[str] = None):
        b, l, d = x.shape
        h, dk, dv = self.n_heads, self.d_k, self.d_v
        sdt = getattr(self, "state_dtype", None) or x.dtype
        if l == 0:
            es = state.clone() if state is not None else torch.zeros(b, h, dk, dv, dtype=sdt, device=x.device)
            kh = max(self.kernel_size - 1, 0)
            z_qk = torch.zeros(b, h * dk, kh, dtype=x.dtype, device=x.device)
            z_v = torch.zeros(b, h * dv, kh, dtype=x.dtype, device=x.device)
            return torch.empty(b, 0, d, dtype=x.dtype, device=x.device), es, ConvState((z_qk, z_qk, z_v))
        q, k, v, eb, ew, la, ncs = self._features(x, conv_state)
        if state is not None:
            state = state.to(sdt)
        o, cs = dispatch_dgda_prefill(
            q=q, k=k, v=v, alpha=None, b=eb, w=ew,
            chunk_size=chunk_size if chunk_size is not None else self.chunk_size,
            initial_state=state, log_alpha=la, state_dtype=sdt, out_layout="blhd",
        )
        o = o.transpose(1, 2).reshape(b, l, h * dv)
        return self.o_proj(o), cs, ncs

    def step(self, x: torch.Tensor, state: Optional[torch.Tensor] = None, conv_state=None):
        b, l = x.shape[0], x.shape[1]
        assert l == 1
        h, dv = self.n_heads, self.d_v
        sdt = getattr(self, "state_dtype", None) or x.dtype
        q, k, v, eb, ew, la, ncs = self._features(x, conv_state)
        if state is not None:
            state = state.to(sdt)
        oh, st = dispatch_dgda_step(q=q, k=k, v=v, alpha=None, b=eb, w=ew, state=state, log_alpha=la,
                                    state_dtype=sdt)
        return self.o_proj(oh.reshape(b, 1, h * dv)), st, ncs


DecoupledGatedDeltaAttention = DGDALayer


class DGIndexer(nn.Module):
    """Delta-guided centroid indexer (maba_sparse/layers/indexer.py:9-126)."""

    def __init__(self, dim: int = 640, d_idx: int = 64, block_size: int = 64, top_k: int = 32,
                 dist_lambda: float = 0.5, config: Optional[Any] = None) -> None:
        super().__init__()
        if config is not None:
            dim = getattr(config, "dim", getattr(config, "d_model", dim))
            d_idx = getattr(config, "d_idx", d_idx)
            block_size = getattr(config, "block_size", block_size)
            top_k = getattr(config, "top_k", top_k)
            dist_lambda = getattr(config, "dist_lambda", dist_lambda)
        self.dim, self.d_idx, self.block_size, self.top_k, self.dist_lambda = dim, d_idx, block_size, top_k, dist_lambda
        self.q_idx_proj = nn.Linear(dim, d_idx, bias=False)
        self.k_idx_proj = nn.Linear(dim, d_idx, bias=False)
        self.scale = 1.0 / math.sqrt(d_idx)
        self._cached_k_idx: Optional[torch.Tensor] = None
        self._cached_centroids: Optional[torch.Tensor] = None

    def reset_cache(self) -> None:
        self._cached_k_idx = None
        self._cached_centroids = None

    def forward(self, x: torch.Tensor, top_k: Optional[int] = None, dist_lambda: Optional[float] = None,
                return_scores: bool = False, past_centroids: Optional[torch.Tensor] = None,
                past_k_idx: Optional[torch.Tensor] = None):
        b, l, _ = x.shape
        k = self.top_k if top_k is None else top_k
        lam = self.dist_lambda if dist_lambda is None else dist_lambda
        qi = self.q_idx_proj(x)
        ki = self.k_idx_proj(x)
        bs = self.block_size
        if past_k_idx is not None:
            c = dispatch_compute_centroids(torch.cat([past_k_idx, ki], dim=1), block_size=bs)
        elif not self.training and l == 1 and self._cached_k_idx is not None and self._cached_k_idx.shape[0] == b:
            self._cached_k_idx = torch.cat([self._cached_k_idx, ki.detach()], dim=1)
            cur = self._cached_k_idx.shape[1]
            if cur % bs == 0:
                new_c = dispatch_compute_centroids(self._cached_k_idx[:, -bs:], block_size=bs)
                self._cached_centroids = (new_c if self._cached_centroids is None
                                          else torch.cat([self._cached_centroids, new_c], dim=1))
                c = self._cached_centroids
            else:
                tail = dispatch_compute_centroids(self._cached_k_idx[:, -(cur % bs):], block_size=bs)
                c = tail if self._cached_centroids is None else torch.cat([self._cached_centroids, tail], dim=1)
        elif past_centroids is not None:
            c = torch.cat([past_centroids, dispatch_compute_centroids(ki, block_size=bs)], dim=1)
        else:
            c = dispatch_compute_centroids(ki, block_size=bs)
            if not self.training and l > 1:
                self._cached_k_idx = ki.detach()
                nc = l // bs
                self._cached_centroids = c[:, :nc, :].detach() if nc > 0 else None
            else:
                self._cached_k_idx = None
                self._cached_centroids = None
        nb = c.shape[1]
        if l == 1 and (past_centroids is not None or past_k_idx is not None or nb > 1):
            # decode scoring: query block nb-1, log1p(clamp(nb-1-n, 0)) (indexer.py:101-112)
            res = b200_index_topk(qi, c, lambda_dist=lam, top_k=k, block_size=bs, return_scores=return_scores,
                                  decode=True)
        else:
            res = dispatch_index_topk(q_idx=qi, centroids=c, lambda_dist=lam, top_k=k, block_size=bs,
                                      return_scores=return_scores)
        if return_scores:
            idx, sc = res
            return idx, c, sc
        return res, c


DeltaGuidedCentroidIndexer = DGIndexer


class MabaSparseAttention(nn.Module):
    """MABA-SA layer (maba_sparse/layers/sparse_attention.py:11-277) on the fused latent kernel."""

    def __init__(self, config: Optional[Any] = None, dim: int = 640, n_heads: int = 10, d_head: int = 64,
                 d_c: int = 128, window_size: int = 128, block_size: int = 64, top_k: int = 32,
                 hca_pool_size: int = 64, dist_lambda: float = 0.5, d_idx: int = 64,
                 ablation_mode: str = "full") -> None:
        super().__init__()
        if config is not None:
            self.dim = getattr(config, "dim", getattr(config, "d_model", dim))
            self.n_heads = getattr(config, "n_heads", getattr(config, "num_heads", n_heads))
            self.d_head = getattr(config, "d_head", d_head)
            self.d_c = getattr(config, "d_c", d_c)
            self.window_size = getattr(config, "window_size", window_size)
            self.block_size = getattr(config, "block_size", block_size)
            self.top_k = getattr(config, "top_k", top_k)
            self.hca_pool_size = getattr(config, "hca_pool_size", hca_pool_size)
            self.dist_lambda = getattr(config, "dist_lambda", dist_lambda)
            self.n_sink_tokens = getattr(config, "n_sink_tokens", 4)
            d_idx = getattr(config, "d_idx", d_idx)
            self.ablation_mode = ablation_mode if ablation_mode is not None else getattr(config, "ablation_mode",
                                                                                          "full")
        else:
            self.dim, self.n_heads, self.d_head, self.d_c = dim, n_heads, d_head, d_c
            self.window_size, self.block_size, self.top_k = window_size, block_size, top_k
            self.hca_pool_size, self.dist_lambda, self.n_sink_tokens = hca_pool_size, dist_lambda, 4
            self.ablation_mode = ablation_mode
        self.scale = 1.0 / math.sqrt(self.d_head)
        self.q_proj = nn.Linear(self.dim, self.n_heads * self.d_head, bias=False)
        self.kv_down_proj = nn.Linear(self.dim, self.d_c, bias=False)
        self.k_up_proj = nn.Linear(self.d_c, self.n_heads * self.d_head, bias=False)
        self.v_up_proj = nn.Linear(self.d_c, self.n_heads * self.d_head, bias=False)
        self.o_proj = nn.Linear(self.n_heads * self.d_head, self.dim, bias=False)
        self.stream_gate = nn.Linear(self.dim, 3, bias=True)
        self.indexer = DGIndexer(dim=self.dim, d_idx=d_idx, block_size=self.block_size, top_k=self.top_k,
                                 dist_lambda=self.dist_lambda)

    def reset_cache(self) -> None:
        self.indexer.reset_cache()

    def get_gate_weights(self, x: torch.Tensor) -> torch.Tensor:
        return F.softmax(self.stream_gate(x), dim=-1)

    def latent_attention(self, x: torch.Tensor, c_full: torch.Tensor, top_idx: torch.Tensor) -> torch.Tensor:
        """Three streams + superposition for the queries of x over the latent cache c_full -> [B,L,H,d_c]."""
        b, l, _ = x.shape
        q = self.q_proj(x).view(b, l, self.n_heads, self.d_head)
        qhat = absorb_queries(q, self.k_up_proj.weight, self.n_heads, self.scale)
        hca = b200_hca_pool(c_full, self.hca_pool_size) if c_full.shape[1] >= self.hca_pool_size else None
        gate = self.stream_gate(x)
        keep = None
        if self.ablation_mode == "no_hca":
            # The reference zeroes the HCA stream and keeps the 3-way gate
            # (sparse_attention.py:268-271): g0*o_loc + g1*o_sp = (1 - g2) * (g0'*o_loc + g1'*o_sp),
            # g' the softmax of the first two logits, so the fused kernel runs with the HCA
            # logit at -inf and the result is scaled by 1 - g2.
            keep = 1.0 - torch.softmax(gate.float(), dim=-1)[..., 2]
            gate = gate.clone()
            gate[..., 2] = float("-inf")
        o = b200_sa_attention(qhat, c_full, hca, top_idx, gate, window_size=self.window_size,
                              n_sinks=self.n_sink_tokens, block_size=self.block_size, hca_r=self.hca_pool_size)
        if keep is not None:
            o = (o.float() * keep.view(b, l, 1, 1)).to(o.dtype)
        return o

    def forward(self, x: torch.Tensor, past_c_kv: Optional[torch.Tensor] = None,
                past_centroids: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        b, l, _ = x.shape
        ck = self.indexer._cached_k_idx
        if past_c_kv is None or (ck is not None and ck.shape[1] != past_c_kv.shape[1]):
            self.reset_cache()
        c_kv = self.kv_down_proj(x)
        c_full = torch.cat([past_c_kv, c_kv], dim=1) if past_c_kv is not None else c_kv
        idx, _ = self.indexer(x, return_scores=False, past_centroids=past_centroids)
        o_lat = self.latent_attention(x, c_full, idx)
        o = expand_values(o_lat, self.v_up_proj.weight, self.n_heads)
        o = o.reshape(b, l, self.n_heads * self.d_head).to(x.dtype)
        return self.o_proj(o), c_full


MABASALayer = MabaSparseAttention
