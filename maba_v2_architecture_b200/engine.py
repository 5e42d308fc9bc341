"""Whole-model inference engine on the sm_100a kernels (configurations 3 and 4).

The drop-in path for the reference's own model class is ``integration.install()``:
the unmodified ``maba_sparse.model.MabaSparseForCausalLM`` then runs its layers on
this library's ops.  This module is the B200-native engine for serving the same
model: it takes the model's weights as a state dict with the reference's
parameter names (maba_sparse/model.py:180-206 module tree), repacks them once for
the GPU, and runs

* **prefill** token-batched: per DGDA layer one input GEMM (the six projections
  stacked), the fused front end, the chunked recurrence and the output GEMM; per
  MABA-SA layer one input GEMM whose rows are the latent projection, the
  *absorbed* queries (W_uk,h^T W_q,h folded into one weight, so no per-head query
  tensor exists), the index query / key projections and the stream gate, then the
  indexer, the fused three-stream attention in latent space, and one output GEMM
  whose weight folds the value up-projection into o_proj (W_o W_uv); residual
  adds and RMSNorms fused into one kernel; the residual stream in float32;
* **decode** one token per step in 5 launches per DGDA block and 9 per MABA-SA
  block: GEMVs with the RMSNorm in their prologue and the conv/gates, SwiGLU,
  gated residual add or logits-with-argmax in their epilogue, the recurrence
  kernel (or, with ``fuse_mix``, the recurrence run by each head's last CTA of the
  DGDA input GEMV), and the O(1)-append latent / index-key caches with the split decode
  top-k and split-K decode attention at a device-held position, so one step is
  captured once as a CUDA graph and replayed.

The math is the reference model's (forward :207-254, step :256-276, RMSNorm
:11-26, SwiGLUFFN :28-37, FactorizedEmbeddings :39-50, MabaBlock :62-129, the
tied lm_head :204); only the order of floating-point operations differs.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from . import _native as N
from .ops import (b200_compute_centroids, b200_dgda_frontend, b200_dgda_prefill, b200_hca_pool, b200_index_topk,
                  b200_sa_attention)

PRO_NORM, PRO_GATHER, PRO_VEC = 0, 1, 2
EPI_STORE, EPI_RESIDUAL, EPI_DGDA, EPI_SWIGLU, EPI_LOGITS = 0, 1, 2, 3, 4


# ---------------------------------------------------------------------------
# the model's shape and parameters (state-dict names are the reference's)
# ---------------------------------------------------------------------------
@dataclass
class ModelShape:
    dim: int
    n_layers: int
    n_heads: int
    d_head: int
    d_k: int
    d_v: int
    d_c: int
    d_idx: int
    vocab: int
    d_emb: int
    inter: int
    conv_k: int
    block: int
    window: int
    top_k: int
    hca_r: int
    lam: float
    rms_eps: float
    k_eps: float
    sinks: int = 4
    ablation: str = "full"

    @classmethod
    def from_config(cls, cfg, ablation_mode: Optional[str] = None) -> "ModelShape":
        g = lambda *names, default=None: next((getattr(cfg, n) for n in names if hasattr(cfg, n)), default)
        dim = g("dim", "d_model", default=640)
        heads = g("n_heads", "num_heads", default=10)
        dh = g("d_head", default=dim // heads)
        return cls(dim=dim, n_layers=g("n_layers", "num_layers", default=20), n_heads=heads, d_head=dh,
                   d_k=g("d_k", default=dh), d_v=g("d_v", default=dh), d_c=g("d_c", default=128),
                   d_idx=g("d_idx", default=64), vocab=g("vocab_size", default=32768), d_emb=g("d_emb", default=128),
                   inter=g("intermediate_size", default=1728), conv_k=g("kernel_size", "conv_kernel_size", default=4),
                   block=g("block_size", default=64), window=g("window_size", default=128), top_k=g("top_k", default=32),
                   hca_r=g("hca_pool_size", default=64), lam=float(g("dist_lambda", default=0.5)),
                   rms_eps=max(float(g("rms_norm_eps", default=1e-6)), 1e-6),
                   k_eps=float(g("eps", "rms_norm_eps", default=1e-6)), sinks=g("n_sink_tokens", default=4),
                   ablation=ablation_mode or g("ablation_mode", default="full"))

    def is_attention(self, i: int) -> bool:
        return self.ablation != "pure_dgda" and (i + 1) % 4 == 0


def parameter_shapes(s: ModelShape) -> Dict[str, Tuple[int, ...]]:
    """State-dict entries of the reference model (maba_sparse/model.py:180-206 with the layers of
    maba_sparse/layers/*.py), tied aliases included."""
    D, H, E, I = s.dim, s.n_heads, s.d_emb, s.inter
    cqk, cv, dh = H * s.d_k, H * s.d_v, H * s.d_head
    out: Dict[str, Tuple[int, ...]] = {"embeddings.in_emb.weight": (s.vocab, E), "embeddings.proj.weight": (D, E)}
    for i in range(s.n_layers):
        p = f"layers.{i}."
        out.update({p + "res_gate1": (D,), p + "res_gate2": (D,), p + "norm1.weight": (D,), p + "norm2.weight": (D,)})
        m = p + "mixer."
        if s.is_attention(i):
            out.update({m + "q_proj.weight": (dh, D), m + "kv_down_proj.weight": (s.d_c, D),
                        m + "k_up_proj.weight": (dh, s.d_c), m + "v_up_proj.weight": (dh, s.d_c),
                        m + "o_proj.weight": (D, dh), m + "stream_gate.weight": (3, D), m + "stream_gate.bias": (3,),
                        m + "indexer.q_idx_proj.weight": (s.d_idx, D), m + "indexer.k_idx_proj.weight": (s.d_idx, D)})
        else:
            out.update({m + "q_proj.weight": (cqk, D), m + "k_proj.weight": (cqk, D), m + "v_proj.weight": (cv, D),
                        m + "conv_q.weight": (cqk, 1, s.conv_k), m + "conv_k.weight": (cqk, 1, s.conv_k),
                        m + "conv_v.weight": (cv, 1, s.conv_k), m + "gate_alpha.weight": (cqk, D),
                        m + "gate_erase.weight": (cqk, D), m + "gate_write.weight": (cv, D), m + "o_proj.weight": (D, cv)})
        out.update({p + "ffn.w_gate.weight": (I, D), p + "ffn.w_up.weight": (I, D), p + "ffn.w_down.weight": (D, I)})
    out.update({"final_norm.weight": (D,), "head_proj.weight": (E, D), "lm_head.weight": (s.vocab, E),
                "mtp_head.proj.weight": (E, D), "mtp_head.lm_head.weight": (s.vocab, E)})
    return out


TIED = {"lm_head.weight": "embeddings.in_emb.weight", "mtp_head.lm_head.weight": "embeddings.in_emb.weight"}


def init_state_dict(shape: ModelShape, seed: int, std: float = 0.02) -> Dict[str, torch.Tensor]:
    """Random weights of the benchmark configurations: every weight N(0, std) drawn in sorted
    name order from one seeded CPU generator, RMSNorm weights 1, residual gates 2.0, the
    stream-gate bias 0; the lm_head (and MTP head) tied to the input embedding."""
    g = torch.Generator().manual_seed(seed)
    sd: Dict[str, torch.Tensor] = {}
    for name, shp in sorted(parameter_shapes(shape).items()):
        if name in TIED:
            continue
        if name.endswith("res_gate1") or name.endswith("res_gate2"):
            sd[name] = torch.full(shp, 2.0)
        elif name.endswith("norm1.weight") or name.endswith("norm2.weight") or name == "final_norm.weight":
            sd[name] = torch.ones(shp)
        elif name.endswith("stream_gate.bias"):
            sd[name] = torch.zeros(shp)
        else:
            sd[name] = torch.randn(shp, generator=g) * std
    for alias, src in TIED.items():
        sd[alias] = sd[src]
    return sd


# ---------------------------------------------------------------------------
# packed weights
# ---------------------------------------------------------------------------
class _DGDAWeights:
    def __init__(self, sd, p, s: ModelShape, dt, dev):
        m = p + "mixer."
        w = lambda n: sd[m + n].to(dev, torch.float32)
        self.w_in = torch.cat([w(n + ".weight") for n in ("q_proj", "k_proj", "v_proj", "gate_alpha", "gate_erase",
                                                           "gate_write")]).to(dt).contiguous()
        self.taps = torch.cat([w(n + ".weight").view(-1, s.conv_k) for n in ("conv_q", "conv_k", "conv_v")]).to(
            dt).contiguous()
        self.w_o = w("o_proj.weight").to(dt).contiguous()
        cqk, cv = s.n_heads * s.d_k, s.n_heads * s.d_v
        self.widths = (cqk, cqk, cv, cqk, cqk, cv)
        self.n_conv = 2 * cqk + cv
        self.alpha_end = 3 * cqk + cv


class _SAWeights:
    def __init__(self, sd, p, s: ModelShape, dt, dev):
        m = p + "mixer."
        w = lambda n: sd[m + n].to(dev, torch.float32)
        H, dh, dc, D = s.n_heads, s.d_head, s.d_c, s.dim
        scale = 1.0 / math.sqrt(dh)
        wq = w("q_proj.weight").view(H, dh, D)
        wuk = w("k_up_proj.weight").view(H, dh, dc)
        # absorbed queries: qhat_h = scale * W_uk,h^T (W_q,h x)  -> one [H*dc, D] weight
        w_qabs = (torch.einsum("hdc,hdk->hck", wuk, wq) * scale).reshape(H * dc, D)
        rows = [w("kv_down_proj.weight"), w_qabs, w("indexer.q_idx_proj.weight"), w("indexer.k_idx_proj.weight"),
                w("stream_gate.weight")]
        n = sum(r.shape[0] for r in rows)
        pad = (-n) % 8  # 16-byte rows of the output for the tensor-memory-access loads of the attention
        rows.append(torch.zeros(pad, D, device=dev))
        self.w_in = torch.cat(rows).to(dt).contiguous()
        self.off_c, self.off_q = 0, dc
        self.off_qi = dc + H * dc
        self.off_ki = self.off_qi + s.d_idx
        self.off_g = self.off_ki + s.d_idx
        self.bias = torch.zeros(self.w_in.shape[0], device=dev)
        self.bias[self.off_g:self.off_g + 3] = w("stream_gate.bias")
        self.bias_dt = self.bias.to(dt)
        # value up-projection folded into o_proj: y = W_o concat_h(W_uv,h o_lat_h) = W_ov o_lat
        wo = w("o_proj.weight").view(D, H, dh)
        wuv = w("v_up_proj.weight").view(H, dh, dc)
        self.w_ov = torch.einsum("khd,hdc->khc", wo, wuv).reshape(D, H * dc).to(dt).contiguous()


class _Layer:
    def __init__(self, sd, i, s: ModelShape, dt, dev):
        p = f"layers.{i}."
        self.attn = s.is_attention(i)
        f = lambda n: sd[p + n].to(dev, torch.float32)
        self.g1 = torch.sigmoid(f("res_gate1")).contiguous()
        self.g2 = torch.sigmoid(f("res_gate2")).contiguous()
        self.n1 = f("norm1.weight").to(dt).contiguous()
        self.n2 = f("norm2.weight").to(dt).contiguous()
        self.w_gu = torch.cat([f("ffn.w_gate.weight"), f("ffn.w_up.weight")]).to(dt).contiguous()
        self.w_down = f("ffn.w_down.weight").to(dt).contiguous()
        self.mix = _SAWeights(sd, p, s, dt, dev) if self.attn else _DGDAWeights(sd, p, s, dt, dev)


def _lin(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return torch.matmul(x, w.t())


def _lin_f32(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x W^T with a float32 result (16-bit operands, float32 accumulation and output): the
    products that feed the float32 residual stream and the logits skip a 16-bit rounding."""
    if x.dtype == torch.float32:
        return torch.matmul(x, w.t())
    y = torch.mm(x.reshape(-1, x.shape[-1]), w.t(), out_dtype=torch.float32)
    return y.view(*x.shape[:-1], w.shape[0])


class MabaEngine:
    """The Maba v2 model on the sm_100a kernels, from a reference-format state dict.

    ``MabaEngine(config, state_dict)`` or ``MabaEngine.from_module(model)`` (any module with
    the reference's parameter names, e.g. an unmodified reference model).  ``dtype`` is the
    compute dtype of weights and activations (bfloat16 for the benchmarks, float32 for exact
    parity checks); the residual stream, recurrent states and logits stay float32."""

    def __init__(self, config, state_dict: Dict[str, torch.Tensor], device="cuda", dtype=torch.bfloat16,
                 ablation_mode: Optional[str] = None):
        self.shape = s = ModelShape.from_config(config, ablation_mode)
        if s.ablation not in ("full", "pure_dgda"):
            raise NotImplementedError(f"MabaEngine: ablation_mode={s.ablation!r}")
        self.device = torch.device(device)
        self.dtype = dtype
        dev, dt = self.device, dtype
        N.require_cuda(torch.empty(0, device=dev), op="MabaEngine")
        sd = state_dict
        self.emb = sd["embeddings.in_emb.weight"].to(dev, dt).contiguous()      # [V, E], also the tied lm_head
        self.w_emb_proj = sd["embeddings.proj.weight"].to(dev, dt).contiguous()  # [D, E]
        self.layers: List[_Layer] = [_Layer(sd, i, s, dt, dev) for i in range(s.n_layers)]
        self.final_norm = sd["final_norm.weight"].to(dev, dt).contiguous()
        self.w_head = sd["head_proj.weight"].to(dev, dt).contiguous()           # [E, D]

    @classmethod
    def from_module(cls, model, device="cuda", dtype=None, **kw) -> "MabaEngine":
        p = next(model.parameters())
        return cls(model.config, {k: v.detach() for k, v in model.state_dict().items()}, device=device,
                   dtype=dtype or p.dtype, **kw)

    # ------------------------------------------------------------------ prefill
    def _norm(self, x, y, gate, w, h):
        rc = N.lib().maba_rmsnorm_residual(N.ref(N.desc(x)), N.ref(N.desc(y)), N.ref(N.desc(gate)),
                                           N.ref(N.desc(w)), float(self.shape.rms_eps), N.ref(N.desc(h)),
                                           N.stream_of(x))
        N.check(rc, "maba_rmsnorm_residual")

    def _swiglu(self, u):
        out = torch.empty(u.shape[0], u.shape[1] // 2, dtype=u.dtype, device=u.device)
        N.check(N.lib().maba_swiglu(N.ref(N.desc(u)), N.ref(N.desc(out)), N.stream_of(u)), "maba_swiglu")
        return out

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, last_only: bool = False, session: Optional["DecodeSession"] = None,
                last_n: Optional[int] = None):
        """Float32 logits of every position ([B,T,V]; the last ``last_n`` positions only, or
        [B,1,V] with ``last_only``);
        ``session`` also receives the decode caches (recurrent states, conv histories, latent /
        index-key caches and tables)."""
        s, dt = self.shape, self.dtype
        B, T = ids.shape
        Ntok = B * T
        ids = ids.to(self.device)
        x = _lin_f32(F.embedding(ids.reshape(-1), self.emb), self.w_emb_proj).contiguous()   # [N, D] fp32
        h = torch.empty(Ntok, s.dim, dtype=dt, device=self.device)
        self._norm(x, None, None, self.layers[0].n1 if self.layers else self.final_norm, h)
        for li, L in enumerate(self.layers):
            y = self._sa_prefill(L, h, B, T, li, session) if L.attn else self._dgda_prefill(L, h, B, T, li, session)
            self._norm(x, y, L.g1, L.n2, h)
            f = _lin_f32(self._swiglu(_lin(h, L.w_gu)), L.w_down)
            nxt = self.layers[li + 1].n1 if li + 1 < len(self.layers) else self.final_norm
            self._norm(x, f, L.g2, nxt, h)
        hv = h.view(B, T, s.dim)
        if last_only:
            hv = hv[:, -1:]
        elif last_n is not None:
            hv = hv[:, -last_n:]
        return _lin_f32(_lin(hv, self.w_head), self.emb)

    def _dgda_prefill(self, L: _Layer, h, B, T, li, session):
        s, W = self.shape, L.mix
        P = _lin(h, W.w_in).view(B, T, -1)
        cols, c0 = [], 0
        for wd in W.widths:
            cols.append(P[:, :, c0:c0 + wd])
            c0 += wd
        taps = list(torch.split(W.taps, list(W.widths[:3])))
        (q, k, v, la, eb, ew), nh = b200_dgda_frontend(cols, taps, None, n_heads=s.n_heads, eps=s.k_eps,
                                                       new_hist=session is not None, hist_dtype=torch.float32)
        H, dk, dv = s.n_heads, s.d_k, s.d_v
        hv = lambda t, d: t.view(B, T, H, d).transpose(1, 2)
        o, S = b200_dgda_prefill(hv(q, dk), hv(k, dk), hv(v, dv), None, hv(eb, dk), hv(ew, dv),
                                 log_alpha=hv(la, dk), state_dtype=torch.float32, out_layout="blhd")
        if session is not None:
            session.states[li].copy_(S)
            session.hists[li].copy_(torch.cat(nh, dim=1))
        return _lin_f32(o.transpose(1, 2).reshape(B * T, H * dv), W.w_o)

    def _sa_prefill(self, L: _Layer, h, B, T, li, session):
        s, W = self.shape, L.mix
        H, dc = s.n_heads, s.d_c
        P = torch.addmm(W.bias_dt, h, W.w_in.t()).view(B, T, -1)
        c = P[:, :, W.off_c:W.off_c + dc]
        qhat = P[:, :, W.off_q:W.off_q + H * dc].view(B, T, H, dc)
        qi = P[:, :, W.off_qi:W.off_qi + s.d_idx]
        ki = P[:, :, W.off_ki:W.off_ki + s.d_idx]
        gate = P[:, :, W.off_g:W.off_g + 3]
        cent = b200_compute_centroids(ki, block_size=s.block)
        idx = b200_index_topk(qi, cent, lambda_dist=s.lam, top_k=s.top_k, block_size=s.block)
        hca = b200_hca_pool(c, s.hca_r) if T >= s.hca_r else None
        o_lat = b200_sa_attention(qhat, c, hca, idx, gate, window_size=s.window, n_sinks=s.sinks,
                                  block_size=s.block, hca_r=s.hca_r)
        if session is not None:
            cache = session.sa[li]
            cache.c[:, :T] = c
            cache.kidx[:, :T] = ki
            cache.cent[:, :cent.shape[1]] = cent
            if hca is not None:
                cache.hca[:, :hca.shape[1]] = hca
        return _lin_f32(o_lat.reshape(B * T, H * dc), W.w_ov)

    # ------------------------------------------------------------------ decode
    def new_session(self, batch: int, max_len: int) -> "DecodeSession":
        return DecodeSession(self, batch, max_len)


@dataclass
class _SACache:
    c: torch.Tensor      # [B, cap, d_c] latent rows
    kidx: torch.Tensor   # [B, cap, d_idx] index keys
    cent: torch.Tensor   # [B, cap/block + 1, d_idx] block centroids (complete blocks + the tail)
    hca: torch.Tensor    # [B, cap/r, d_c] pooled rows of complete groups
    idx: torch.Tensor    # [B, 1, top_k] selected blocks of the step
    o_lat: torch.Tensor  # [B, 1, H, d_c] attention output of the step
    ws_topk: Optional[torch.Tensor]
    ws_attn: Optional[torch.Tensor]


class DecodeSession:
    """Greedy / teacher-forced decoding with caches sized for ``max_len`` tokens.

    ``prefill(ids)`` fills every cache from a prompt and returns its last logits;
    ``step(ids)`` runs one token eagerly; ``capture()`` records one step as a CUDA graph
    whose inputs are ``ids_buf`` (the token of the step) and the device-held position, and
    ``replay()`` runs it: logits land in ``logits`` and their argmax in ``ids_buf``, ready
    for the next replay.  The host keeps ``length`` in step with the device position."""

    def __init__(self, engine: MabaEngine, batch: int, max_len: int):
        self.engine = e = engine
        s, dt, dev = e.shape, e.dtype, e.device
        if not 1 <= batch <= 8:
            raise ValueError("DecodeSession: batch 1..8")
        self.B, self.max_len, self.length = batch, max_len, 0
        H = s.n_heads
        self.x = torch.zeros(batch, s.dim, device=dev)
        self.states: Dict[int, torch.Tensor] = {}
        self.hists: Dict[int, torch.Tensor] = {}
        self.sa: Dict[int, _SACache] = {}
        lib = N.lib()
        nbcap = max_len // s.block + 1
        nccap = max(max_len // s.hca_r, 1)
        for i, L in enumerate(e.layers):
            if L.attn:
                ws_t = lib.maba_index_topk_decode_at_workspace_size(batch, nbcap, s.top_k)
                ws_a = lib.maba_sa_attention_decode_at_workspace_size(batch, max_len, nccap, H, s.d_c, s.top_k,
                                                                      s.window, s.sinks, s.block, s.hca_r)
                self.sa[i] = _SACache(
                    c=torch.zeros(batch, max_len, s.d_c, dtype=dt, device=dev),
                    kidx=torch.zeros(batch, max_len, s.d_idx, dtype=dt, device=dev),
                    cent=torch.zeros(batch, nbcap, s.d_idx, dtype=dt, device=dev),
                    hca=torch.zeros(batch, nccap, s.d_c, dtype=dt, device=dev),
                    idx=torch.zeros(batch, 1, min(s.top_k, nbcap), dtype=torch.long, device=dev),
                    o_lat=torch.zeros(batch, 1, H, s.d_c, dtype=dt, device=dev),
                    ws_topk=torch.empty(ws_t, dtype=torch.uint8, device=dev) if ws_t else None,
                    ws_attn=torch.empty(ws_a, dtype=torch.uint8, device=dev) if ws_a else None)
            else:
                self.states[i] = torch.zeros(batch, H, s.d_k, s.d_v, device=dev)
                self.hists[i] = torch.zeros(batch, L.mix.n_conv, s.conv_k - 1, device=dev)
        cqk, cv = H * s.d_k, H * s.d_v
        self.feats = torch.zeros(batch, 4 * cqk + 2 * cv, device=dev)
        self.o = torch.zeros(batch, cv, device=dev)
        self.a = torch.zeros(batch, s.inter, device=dev)
        sa_rows = next((L.mix.w_in.shape[0] for L in e.layers if L.attn), 8)
        self.sa_out = torch.zeros(batch, sa_rows, dtype=dt, device=dev)
        self.e = torch.zeros(batch, s.d_emb, device=dev)
        self.logits = torch.zeros(batch, s.vocab, device=dev)
        self.ids_buf = torch.zeros(batch, dtype=torch.long, device=dev)
        self.pos_dev = torch.zeros((), dtype=torch.long, device=dev)
        self.ws_head = torch.zeros(lib.maba_decode_gemv_workspace_size(batch), dtype=torch.uint8, device=dev)
        # DGDA blocks: a GEMV with the features epilogue, then the recurrence-step kernel; with
        # fuse_mix, one launch (maba_decode_dgda_mix: the step runs in each head's last CTA of the
        # GEMV), which measured 2-3 % slower per token on the 101M model, so it is off by default
        self.fuse_mix = False
        self.ws_mix = torch.zeros(lib.maba_decode_dgda_mix_workspace_size(H), dtype=torch.uint8, device=dev)
        self.graph = None

    # ------------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        B, T = ids.shape
        if B != self.B or T > self.max_len:
            raise ValueError(f"DecodeSession.prefill: ids {tuple(ids.shape)} for batch {self.B}, max_len {self.max_len}")
        logits = self.engine.forward(ids, last_only=True, session=self)
        self.length = T
        self.pos_dev.fill_(T)
        return logits

    @staticmethod
    def _gemv_args(w, pro, x=None, aux=None, ids=None, epi=EPI_STORE, out=None, bias=None, gate=None, taps=None,
                   hist=None, n_conv=0, alpha_end=0, ids_out=None, pos=None, ws=None):
        return (w, pro, x, aux, ids, epi, out, bias, gate, taps, hist, n_conv, alpha_end, ids_out, pos, ws)

    def _gemv_c_args(self, a):
        w, pro, x, aux, ids, epi, out, bias, gate, taps, hist, n_conv, alpha_end, ids_out, pos, ws = a
        return (N.ref(N.desc(w)), pro, N.ref(N.desc(x)), N.ref(N.desc(aux)), float(self.engine.shape.rms_eps),
                N.ref(N.desc(ids)), epi, N.ref(N.desc(out)), N.ref(N.desc(bias)), N.ref(N.desc(gate)),
                N.ref(N.desc(taps)), N.ref(N.desc(hist)), int(n_conv), int(alpha_end), N.ref(N.desc(ids_out)),
                pos.data_ptr() if pos is not None else None, ws.data_ptr() if ws is not None else None,
                ws.numel() if ws is not None else 0)

    def _plan(self):
        """One decode step as a list of pieces: ("gemv", args), ("mix", layer) -- a DGDA block's input
        projection, features and recurrence step --, ("state", layer) and ("sa", layer) -- the cache
        append, split top-k and split-K attention of a MABA-SA layer."""
        e, s = self.engine, self.engine.shape
        B, H, dc = self.B, s.n_heads, s.d_c
        g = self._gemv_args
        plan = [("gemv", g(e.w_emb_proj, PRO_GATHER, aux=e.emb, ids=self.ids_buf, epi=EPI_STORE, out=self.x))]
        for i, L in enumerate(e.layers):
            W = L.mix
            if L.attn:
                plan.append(("gemv", g(W.w_in, PRO_NORM, x=self.x, aux=L.n1, epi=EPI_STORE, out=self.sa_out,
                                       bias=W.bias)))
                plan.append(("sa", i))
                plan.append(("gemv", g(W.w_ov, PRO_VEC, x=self.sa[i].o_lat.view(B, H * dc), epi=EPI_RESIDUAL,
                                       out=self.x, gate=L.g1)))
            else:
                if self.fuse_mix:
                    plan.append(("mix", i))
                else:
                    plan.append(("gemv", g(W.w_in, PRO_NORM, x=self.x, aux=L.n1, epi=EPI_DGDA, out=self.feats,
                                           taps=W.taps, hist=self.hists[i], n_conv=W.n_conv,
                                           alpha_end=W.alpha_end)))
                    plan.append(("state", i))
                plan.append(("gemv", g(W.w_o, PRO_VEC, x=self.o, epi=EPI_RESIDUAL, out=self.x, gate=L.g1)))
            plan.append(("gemv", g(L.w_gu, PRO_NORM, x=self.x, aux=L.n2, epi=EPI_SWIGLU, out=self.a)))
            plan.append(("gemv", g(L.w_down, PRO_VEC, x=self.a, epi=EPI_RESIDUAL, out=self.x, gate=L.g2)))
        plan.append(("gemv", g(e.w_head, PRO_NORM, x=self.x, aux=e.final_norm, epi=EPI_STORE, out=self.e)))
        plan.append(("gemv", g(e.emb, PRO_VEC, x=self.e, epi=EPI_LOGITS, out=self.logits, ids_out=self.ids_buf,
                               pos=self.pos_dev, ws=self.ws_head)))
        return plan

    def _sa_middle(self, i: int, st: int) -> None:
        """Cache append, split decode top-k and split-K decode attention of MABA-SA layer i."""
        e, s = self.engine, self.engine.shape
        lib = N.lib()
        W, cache = e.layers[i].mix, self.sa[i]
        B, H, dc = self.B, s.n_heads, s.d_c
        so = self.sa_out
        c_new = so[:, W.off_c:W.off_c + dc].unsqueeze(1)
        k_new = so[:, W.off_ki:W.off_ki + s.d_idx].unsqueeze(1)
        q_idx = so[:, W.off_qi:W.off_qi + s.d_idx].unsqueeze(1)
        qhat = so[:, W.off_q:W.off_q + H * dc].view(B, 1, H, dc)
        gate = so[:, W.off_g:W.off_g + 3].unsqueeze(1)
        N.check(lib.maba_decode_cache_append(
            N.ref(N.desc(c_new)), N.ref(N.desc(k_new)), N.ref(N.desc(cache.c)), N.ref(N.desc(cache.kidx)),
            N.ref(N.desc(cache.cent)), N.ref(N.desc(cache.hca)), self.pos_dev.data_ptr(), s.block, s.hca_r, st),
            "maba_decode_cache_append")
        wt = cache.ws_topk
        N.check(lib.maba_index_topk_decode_at(
            N.ref(N.desc(q_idx)), N.ref(N.desc(cache.cent)), float(s.lam), s.top_k, s.block, self.pos_dev.data_ptr(),
            N.ref(N.desc(cache.idx)), wt.data_ptr() if wt is not None else None, wt.numel() if wt is not None else 0,
            st), "maba_index_topk_decode_at")
        wa = cache.ws_attn
        N.check(lib.maba_sa_attention_decode_at(
            N.ref(N.desc(qhat)), N.ref(N.desc(cache.c)), N.ref(N.desc(cache.hca)), N.ref(N.desc(cache.idx)),
            N.ref(N.desc(gate)), N.ref(N.desc(cache.o_lat)), self.pos_dev.data_ptr(), s.window, s.sinks, s.block,
            s.hca_r, wa.data_ptr() if wa is not None else None, wa.numel() if wa is not None else 0, st),
            "maba_sa_attention_decode_at")

    def _mix(self, i: int, st: int) -> None:
        e, L = self.engine, self.engine.layers[i]
        W = L.mix
        N.check(N.lib().maba_decode_dgda_mix(
            N.ref(N.desc(W.w_in)), N.ref(N.desc(self.x)), N.ref(N.desc(L.n1)), float(e.shape.rms_eps),
            N.ref(N.desc(W.taps)), N.ref(N.desc(self.hists[i])), N.ref(N.desc(self.feats)),
            N.ref(N.desc(self.states[i])), N.ref(N.desc(self.o)), e.shape.n_heads, float(e.shape.k_eps),
            self.ws_mix.data_ptr(), self.ws_mix.numel(), st), "maba_decode_dgda_mix")

    def _state(self, i: int, st: int) -> None:
        N.check(N.lib().maba_decode_dgda_state(N.ref(N.desc(self.feats)), N.ref(N.desc(self.states[i])),
                                               N.ref(N.desc(self.o)), self.engine.shape.n_heads,
                                               float(self.engine.shape.k_eps), st), "maba_decode_dgda_state")

    def _step_device(self) -> None:
        """One decode step on the session's buffers: ids_buf -> logits, argmax -> ids_buf, position + 1."""
        lib = N.lib()
        st = N.stream_of(self.x)
        for kind, a in self._plan():
            if kind == "gemv":
                N.check(lib.maba_decode_gemv(*self._gemv_c_args(a), st), "maba_decode_gemv")
            elif kind == "mix":
                self._mix(a, st)
            elif kind == "state":
                self._state(a, st)
            else:
                self._sa_middle(a, st)

    def bytes_per_step(self) -> int:
        """HBM bytes one decode step must move at the current length: every weight it reads, the
        recurrent states and conv histories read and written, and per MABA-SA layer the latent rows
        of the window, sinks and selected blocks, the pooled rows and the centroid table it scans,
        and the index keys of the tail block it re-pools."""
        e, s = self.engine, self.engine.shape
        nb = lambda t: t.numel() * t.element_size()
        total = nb(e.w_emb_proj) + nb(e.w_head) + nb(e.emb) + nb(e.final_norm) + self.B * nb(e.emb[0])
        pos = max(self.length, 1)
        nblk = (pos + s.block - 1) // s.block
        for i, L in enumerate(e.layers):
            total += nb(L.n1) + nb(L.n2) + nb(L.w_gu) + nb(L.w_down) + nb(L.g1) + nb(L.g2)
            W = L.mix
            if L.attn:
                el = e.emb.element_size()
                rows = min(pos, s.window + s.sinks) + min(s.top_k, nblk) * s.block
                total += nb(W.w_in) + nb(W.w_ov) + nb(W.bias)
                total += self.B * el * (rows * s.d_c + (pos // s.hca_r) * s.d_c + nblk * s.d_idx + s.block * s.d_idx)
            else:
                total += nb(W.w_in) + nb(W.w_o) + nb(W.taps) + 2 * nb(self.states[i]) + 2 * nb(self.hists[i])
        return int(total)

    def launches_per_step(self) -> int:
        """Kernels of this library one decode step launches (the count the step's graph holds): one
        per GEMV, fused DGDA mixer or recurrence step; five per MABA-SA middle (cache append, top-k
        partial + merge, attention partial + combine)."""
        return sum(5 if kind == "sa" else 1 for kind, _ in self._plan())

    @torch.no_grad()
    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """One eager decode step for token ids [B] or [B,1]; returns float32 logits [B,V]."""
        if self.length >= self.max_len:
            raise RuntimeError("DecodeSession: cache full")
        self.ids_buf.copy_(ids.reshape(self.B))
        self._step_device()
        self.length += 1
        return self.logits

    @torch.no_grad()
    def capture(self) -> None:
        """Records one step as a CUDA graph (call after prefill; warms up on a side stream without
        touching the session's state)."""
        dev = self.engine.device
        saved_pos, saved_ids = self.pos_dev.clone(), self.ids_buf.clone()
        snap = {k: v.clone() for k, v in self.states.items()}
        snap_h = {k: v.clone() for k, v in self.hists.items()}
        snap_x = self.x.clone()
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._step_device()  # first launches outside capture (lazy module / attribute set-up)
        torch.cuda.current_stream(dev).wait_stream(side)
        # undo the warm-up step: the row it appended is overwritten by the next real step at
        # the same position, and block tables of a partial block are recomputed from the rows
        self.pos_dev.copy_(saved_pos)
        self.ids_buf.copy_(saved_ids)
        for k, v in snap.items():
            self.states[k].copy_(v)
        for k, v in snap_h.items():
            self.hists[k].copy_(v)
        self.x.copy_(snap_x)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step_device()
        self.graph = g

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("DecodeSession.replay: capture() first")
        if self.length >= self.max_len:
            raise RuntimeError("DecodeSession: cache full")
        self.graph.replay()
        self.length += 1
        return self.logits
