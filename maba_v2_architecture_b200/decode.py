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

from .ops import (absorb_queries, b200_compute_centroids, b200_decode_cache_append, b200_hca_pool, b200_index_topk,
                  b200_index_topk_decode_at, b200_sa_attention, b200_sa_attention_decode_at, expand_values)


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

    # -------------------------------------------------------------- CUDA-graph decode
    def _sa_step_dev(self, m, cache: _SACache, h: torch.Tensor) -> torch.Tensor:
        """One MABA-SA decode step at the device-held position (no host-side length)."""
        B = h.shape[0]
        b200_decode_cache_append(m.kv_down_proj(h), m.indexer.k_idx_proj(h), cache.c, cache.kidx, cache.cent,
                                 cache.hca, self.pos_dev, self.block, m.hca_pool_size)
        idx = b200_index_topk_decode_at(m.indexer.q_idx_proj(h), cache.cent, self.pos_dev,
                                        lambda_dist=m.indexer.dist_lambda, top_k=m.indexer.top_k,
                                        block_size=self.block)
        q = m.q_proj(h).view(B, 1, m.n_heads, m.d_head)
        qhat = absorb_queries(q, m.k_up_proj.weight, m.n_heads, m.scale)
        o_lat = b200_sa_attention_decode_at(qhat, cache.c, cache.hca, idx, m.stream_gate(h), self.pos_dev,
                                            window_size=m.window_size, n_sinks=m.n_sink_tokens,
                                            block_size=self.block, hca_r=m.hca_pool_size)
        o = expand_values(o_lat, m.v_up_proj.weight, m.n_heads).reshape(B, 1, m.n_heads * m.d_head)
        return m.o_proj(o.to(h.dtype))

    def _step_dev(self) -> None:
        """Greedy decode step on static buffers: ids_buf -> logits_buf, argmax back into ids_buf."""
        model = self.model
        x = model.embeddings(self.ids_buf)
        for i, layer in enumerate(model.layers):
            h = layer.norm1(x)
            if layer.is_attention:
                mo = self._sa_step_dev(layer.mixer, self.sa[i], h)
            else:
                mo, st, cv = layer.mixer.step(h, state=self.states[i], conv_state=self.convs[i])
                self.states[i].copy_(st)
                for dst, src in zip(self.convs[i], cv):
                    dst.copy_(src)
            x = x + torch.sigmoid(layer.res_gate1) * mo
            x = x + torch.sigmoid(layer.res_gate2) * layer.ffn(layer.norm2(x))
        self.logits_buf.copy_(model.lm_head(model.head_proj(model.final_norm(x))))
        self.ids_buf.copy_(self.logits_buf[:, -1].argmax(-1, keepdim=True))
        self.pos_dev.add_(1)

    @torch.no_grad()
    def capture(self, first_ids: torch.Tensor) -> None:
        """Captures one greedy decode step in a CUDA graph (call after prefill).
        ``first_ids`` [B,1] is the token fed to the first replayed step."""
        V = self.model.config.vocab_size
        self.ids_buf = first_ids.clone()
        self.logits_buf = torch.empty(self.B, 1, V, dtype=self.dtype, device=self.device)
        self.pos_dev = torch.full((), self.L, dtype=torch.int64, device=self.device)
        self.states = [s.clone() if s is not None else None for s in self.states]
        self.convs = [tuple(c.clone() for c in cv) if cv is not None else None for cv in self.convs]
        saved = (self.ids_buf.clone(), self.pos_dev.clone(), [s.clone() if s is not None else None for s in self.states],
                 [tuple(c.clone() for c in cv) if cv is not None else None for cv in self.convs],
                 [(c.c.clone(), c.kidx.clone(), c.cent.clone(), c.hca.clone()) if c is not None else None
                  for c in self.sa] if self.L < 4096 else None)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._step_dev()  # warm-up on a side stream (cuBLAS handles, allocator pools)
        torch.cuda.current_stream(self.device).wait_stream(side)
        # undo the warm-up step (it advanced the position and touched the caches at that row)
        self.ids_buf.copy_(saved[0])
        self.pos_dev.copy_(saved[1])
        for dst, src in zip(self.states, saved[2]):
            if dst is not None:
                dst.copy_(src)
        for dst, src in zip(self.convs, saved[3]):
            if dst is not None:
                for d_, s_ in zip(dst, src):
                    d_.copy_(s_)
        if saved[4] is not None:
            for c, sv in zip(self.sa, saved[4]):
                if c is not None:
                    c.c.copy_(sv[0]); c.kidx.copy_(sv[1]); c.cent.copy_(sv[2]); c.hca.copy_(sv[3])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step_dev()

    def replay(self) -> torch.Tensor:
        """Runs the captured step once; returns the logits buffer [B,1,V] (ids_buf holds the argmax)."""
        self.graph.replay()
        self.L += 1
        return self.logits_buf

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
