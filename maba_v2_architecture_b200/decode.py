"""Decode session for MabaSparseForCausalLM with O(1)-append caches.

The reference's decode (maba_sparse/model.py:256-276 with the layer decode
paths sparse_attention.py:228-261 and indexer.py:62-112) concatenates the whole
latent cache, the per-head K/V cache and the index-key cache on every step and
re-pools every HCA block, i.e. O(L) traffic per token.  The session keeps, per
MABA-SA layer, preallocated buffers written in place:

  latent cache   c     [B, Lmax, d_c]
  index keys     kidx  [B, Lmax, d_idx]
  centroid table cent  [B, Lmax/64 + 1, d_idx]   (complete blocks + the tail block)
  pooled HCA     hca   [B, Lmax/64, d_c]         (complete blocks)

and, per DGDA layer, the fp32 recurrent state and the conv histories.  A step
appends one latent row and one index-key row, refreshes the tail centroid (or
seals a completed block: its centroid and its pooled HCA row), and runs the
split-candidate decode top-k and the split-K decode attention on views of the
buffers -- the same values the reference computes (its centroids / pooled rows
of complete blocks never change), with per-step traffic proportional to the
window + selected blocks + the pooled and centroid tables.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from .ops import absorb_queries, b200_compute_centroids, b200_hca_pool, b200_index_topk, b200_sa_attention, expand_values


@dataclass
class _SACache:
    c: torch.Tensor
    kidx: torch.Tensor
    cent: torch.Tensor
    hca: torch.Tensor


class DecodeSession:
    def __init__(self, model, batch: int, max_len: int, dtype: Optional[torch.dtype] = None):
        self.model = model
        self.B = batch
        self.max_len = max_len
        self.L = 0
        p = next(model.parameters())
        self.device = p.device
        self.dtype = dtype or p.dtype
        cfg = model.config
        self.block = cfg.block_size
        nbmax = max_len // self.block + 1
        self.sa: List[Optional[_SACache]] = []
        self.states: List[Optional[torch.Tensor]] = []
        self.convs: List = []
        for layer in model.layers:
            if layer.is_attention:
                m = layer.mixer
                self.sa.append(_SACache(
                    c=torch.zeros(batch, max_len, m.d_c, dtype=self.dtype, device=self.device),
                    kidx=torch.zeros(batch, max_len, m.indexer.d_idx, dtype=self.dtype, device=self.device),
                    cent=torch.zeros(batch, nbmax, m.indexer.d_idx, dtype=self.dtype, device=self.device),
                    hca=torch.zeros(batch, max_len // m.hca_pool_size, m.d_c, dtype=self.dtype, device=self.device),
                ))
                self.states.append(None)
                self.convs.append(None)
            else:
                layer.mixer.state_dtype = torch.float32
                self.sa.append(None)
                self.states.append(None)
                self.convs.append(None)

    # -------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Runs the prompt through the model and fills every cache; returns the last logits [B,1,V]."""
        model = self.model
        B, L = input_ids.shape
        assert B == self.B and L <= self.max_len
        x = model.embeddings(input_ids)
        for i, layer in enumerate(model.layers):
            h = layer.norm1(x)
            if layer.is_attention:
                m = layer.mixer
                m.reset_cache()
                mo, c_full = m(h)
                cache = self.sa[i]
                cache.c[:, :L] = c_full
                ki = m.indexer.k_idx_proj(h)
                cache.kidx[:, :L] = ki
                cent = b200_compute_centroids(ki, block_size=self.block)
                cache.cent[:, : cent.shape[1]] = cent
                nfull = L // m.hca_pool_size
                if nfull:
                    cache.hca[:, :nfull] = b200_hca_pool(c_full, m.hca_pool_size)
                m.reset_cache()
            else:
                mo, S, conv = layer.mixer(h, state=None)
                self.states[i] = S
                self.convs[i] = conv
            x = x + torch.sigmoid(layer.res_gate1) * mo
            x = x + torch.sigmoid(layer.res_gate2) * layer.ffn(layer.norm2(x))
        self.L = L
        xn = model.final_norm(x[:, -1:])
        return model.lm_head(model.head_proj(xn))

    # -------------------------------------------------------------- one token
    @torch.no_grad()
    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """One decode step for ids [B,1]; returns logits [B,1,V]."""
        model = self.model
        assert ids.shape == (self.B, 1) and self.L < self.max_len
        pos = self.L
        Ln = pos + 1
        x = model.embeddings(ids)
        for i, layer in enumerate(model.layers):
            h = layer.norm1(x)
            if layer.is_attention:
                mo = self._sa_step(layer.mixer, self.sa[i], h, pos)
            else:
                mo, self.states[i], self.convs[i] = layer.mixer.step(h, state=self.states[i], conv_state=self.convs[i])
            x = x + torch.sigmoid(layer.res_gate1) * mo
            x = x + torch.sigmoid(layer.res_gate2) * layer.ffn(layer.norm2(x))
        self.L = Ln
        return model.lm_head(model.head_proj(model.final_norm(x)))

    def _sa_step(self, m, cache: _SACache, h: torch.Tensor, pos: int) -> torch.Tensor:
        B = h.shape[0]
        Ln = pos + 1
        bs, r = self.block, m.hca_pool_size
        cache.c[:, pos] = m.kv_down_proj(h)[:, 0]
        ki = m.indexer.k_idx_proj(h)
        cache.kidx[:, pos] = ki[:, 0]
        nb = (Ln + bs - 1) // bs
        start = (nb - 1) * bs
        # tail (or just-completed) block centroid, zero-padded as compute_centroids does
        cache.cent[:, nb - 1: nb] = b200_compute_centroids(cache.kidx[:, start:Ln], block_size=bs)
        if Ln % r == 0:
            cache.hca[:, Ln // r - 1: Ln // r] = b200_hca_pool(cache.c[:, Ln - r:Ln], r)
        qi = m.indexer.q_idx_proj(h)
        idx = b200_index_topk(qi, cache.cent[:, :nb], lambda_dist=m.indexer.dist_lambda, top_k=m.indexer.top_k,
                              block_size=bs, decode=True)
        q = m.q_proj(h).view(B, 1, m.n_heads, m.d_head)
        qhat = absorb_queries(q, m.k_up_proj.weight, m.n_heads, m.scale)
        nc = Ln // r
        o_lat = b200_sa_attention(qhat, cache.c[:, :Ln], cache.hca[:, :nc] if nc else None, idx, m.stream_gate(h),
                                  window_size=m.window_size, n_sinks=m.n_sink_tokens, block_size=bs, hca_r=r)
        o = expand_values(o_lat, m.v_up_proj.weight, m.n_heads).reshape(B, 1, m.n_heads * m.d_head)
        return m.o_proj(o.to(h.dtype))
