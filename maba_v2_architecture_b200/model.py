"""The 101M Maba v2 language model on the B200 layers.

Mirrors maba_sparse/model.py (RMSNorm :11, SwiGLUFFN :28, FactorizedEmbeddings
:39, MTPHead :52, MabaBlock :62, MabaSparseOutput :131, get_101m_config :162,
MabaSparseForCausalLM :180 with forward :207, step :256, generate :279): same
module tree and parameter names (reference state dicts load), same 3:1
DGDA / MABA-SA layering (every 4th layer is MABA-SA), same forward / step /
generate contracts.  The mixers are the sm_100a layers of ``layers.py``; norms,
projections, FFN and embeddings stay torch (cuBLAS) modules.
"""
from __future__ import annotations

from typing import Any, List, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import MabaSparseConfig, get_101m_config
from .layers import DGDALayer, MabaSparseAttention


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.dim = dim
        self.eps = max(float(eps), 1e-6)
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.rms_norm(x, (self.dim,), self.weight, eps=self.eps)


class SwiGLUFFN(nn.Module):
    def __init__(self, dim: int, intermediate_size: int) -> None:
        super().__init__()
        self.w_gate = nn.Linear(dim, intermediate_size, bias=False)
        self.w_up = nn.Linear(dim, intermediate_size, bias=False)
        self.w_down = nn.Linear(intermediate_size, dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w_down(F.silu(self.w_gate(x)) * self.w_up(x))


class FactorizedEmbeddings(nn.Module):
    def __init__(self, vocab_size: int, d_emb: int, dim: int) -> None:
        super().__init__()
        self.vocab_size, self.d_emb, self.dim = vocab_size, d_emb, dim
        self.in_emb = nn.Embedding(vocab_size, d_emb)
        self.proj = nn.Linear(d_emb, dim, bias=False)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.proj(self.in_emb(input_ids))


class MTPHead(nn.Module):
    def __init__(self, dim: int, d_emb: int, lm_head: nn.Linear) -> None:
        super().__init__()
        self.proj = nn.Linear(dim, d_emb, bias=False)
        self.lm_head = lm_head

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.lm_head(self.proj(x))


class MabaBlock(nn.Module):
    def __init__(self, config: MabaSparseConfig, layer_idx: int, ablation_mode: str = "full") -> None:
        super().__init__()
        self.layer_idx = layer_idx
        self.ablation_mode = ablation_mode
        self.is_attention = False if ablation_mode == "pure_dgda" else (layer_idx + 1) % 4 == 0
        self.norm1 = RMSNorm(config.dim, eps=config.rms_norm_eps)
        self.mixer = MabaSparseAttention(config, ablation_mode=ablation_mode) if self.is_attention else DGDALayer(config)
        self.norm2 = RMSNorm(config.dim, eps=config.rms_norm_eps)
        self.ffn = SwiGLUFFN(config.dim, getattr(config, "intermediate_size", 1728))
        b = getattr(config, "residual_gate_bias", 2.0)
        self.res_gate1 = nn.Parameter(torch.full((config.dim,), b))
        self.res_gate2 = nn.Parameter(torch.full((config.dim,), b))

    def _mix(self, x, h, state, conv_state, past_c_kv, step: bool):
        if self.is_attention:
            mo, nc = self.mixer(h, past_c_kv=past_c_kv)
            ns, ncv = None, None
        else:
            fn = self.mixer.step if step else self.mixer
            mo, ns, ncv = fn(h, state=state, conv_state=conv_state)
            nc = None
        x = x + torch.sigmoid(self.res_gate1) * mo
        x = x + torch.sigmoid(self.res_gate2) * self.ffn(self.norm2(x))
        return x, ns, ncv, nc

    def forward(self, x, state=None, conv_state=None, past_c_kv=None):
        return self._mix(x, self.norm1(x), state, conv_state, past_c_kv, step=False)

    def step(self, x, state=None, conv_state=None, past_c_kv=None):
        return self._mix(x, self.norm1(x), state, conv_state, past_c_kv, step=True)


class MabaSparseOutput:
    """(logits, loss, mtp_logits, past_states) with the reference's access forms."""

    def __init__(self, logits, loss=None, mtp_logits=None, past_states=None) -> None:
        self.logits, self.loss, self.mtp_logits, self.past_states = logits, loss, mtp_logits, past_states

    def __iter__(self):
        return iter((self.logits, self.loss))

    def __getitem__(self, idx: Union[int, str]) -> Any:
        if isinstance(idx, str):
            if hasattr(self, idx):
                return getattr(self, idx)
            raise KeyError(f"No key '{idx}' in MabaSparseOutput")
        return (self.logits, self.loss, self.past_states, self.mtp_logits)[idx]


class MabaSparseForCausalLM(nn.Module):
    def __init__(self, config: Optional[MabaSparseConfig] = None, ablation_mode: str = "full") -> None:
        super().__init__()
        config = config if config is not None else get_101m_config()
        self.config = config
        self.ablation_mode = ablation_mode
        v, de, d, nl = config.vocab_size, config.d_emb, config.dim, config.n_layers
        self.embeddings = FactorizedEmbeddings(v, de, d)
        self.layers = nn.ModuleList([MabaBlock(config, i, ablation_mode=ablation_mode) for i in range(nl)])
        self.final_norm = RMSNorm(d, eps=config.rms_norm_eps)
        self.head_proj = nn.Linear(d, de, bias=False)
        self.lm_head = nn.Linear(de, v, bias=False)
        self.lm_head.weight = self.embeddings.in_emb.weight
        self.mtp_head = MTPHead(d, de, self.lm_head)

    def set_state_dtype(self, dtype: Optional[torch.dtype]) -> None:
        """Keep DGDA recurrent states in ``dtype`` (e.g. float32 for a bf16 model)."""
        for layer in self.layers:
            if not layer.is_attention:
                layer.mixer.state_dtype = dtype

    def forward(self, input_ids, targets=None, labels=None, past_states=None) -> MabaSparseOutput:
        if targets is None and labels is not None:
            targets = labels
        x = self.embeddings(input_ids)
        nps = []
        for i, layer in enumerate(self.layers):
            ls = past_states[i] if past_states is not None and i < len(past_states) else None
            x, nst, ncv, nck = layer(x, state=ls[0] if ls else None, conv_state=ls[1] if ls else None,
                                     past_c_kv=ls[2] if ls else None)
            nps.append((nst, ncv, nck))
        xn = self.final_norm(x)
        logits = self.lm_head(self.head_proj(xn))
        loss = mtp_logits = None
        if targets is not None:
            vs = self.config.vocab_size
            loss = F.cross_entropy(logits.view(-1, vs), targets.view(-1), ignore_index=-100)
            mtp_logits = self.mtp_head(xn[:, :-1, :])
            if mtp_logits.numel() > 0:
                loss = loss + 0.3 * F.cross_entropy(mtp_logits.contiguous().view(-1, vs),
                                                    targets[:, 1:].contiguous().view(-1), ignore_index=-100)
            else:
                loss = loss + 0.0 * mtp_logits.sum()
        return MabaSparseOutput(logits=logits, loss=loss, mtp_logits=mtp_logits, past_states=nps)

    def step(self, input_ids, past_states=None) -> Tuple[torch.Tensor, List[Any]]:
        b, l = input_ids.shape
        assert l == 1, f"step() expects single-token input (L=1), got L={l}"
        x = self.embeddings(input_ids)
        nxt = []
        for i, layer in enumerate(self.layers):
            ls = past_states[i] if past_states is not None and i < len(past_states) else None
            x, nst, ncv, nck = layer.step(x, state=ls[0] if ls else None, conv_state=ls[1] if ls else None,
                                          past_c_kv=ls[2] if ls else None)
            nxt.append((nst, ncv, nck))
        xn = self.final_norm(x)
        return self.lm_head(self.head_proj(xn)), nxt

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens: int = 32, temperature: float = 1.0, top_k: Optional[int] = 50):
        was_training = self.training
        self.eval()
        try:
            out = self(input_ids)
            past = out.past_states
            nl = out.logits[:, -1:, :]
            tokens = [input_ids]
            for i in range(max_new_tokens):
                logits = nl.squeeze(1)
                if temperature > 0:
                    logits = logits / temperature
                    if top_k is not None:
                        kv = min(top_k, logits.size(-1))
                        vals, _ = torch.topk(logits, kv)
                        logits = logits.masked_fill(logits < vals[:, [-1]], float("-inf"))
                    tok = torch.multinomial(F.softmax(logits, dim=-1), num_samples=1)
                else:
                    tok = torch.argmax(logits, dim=-1, keepdim=True)
                tokens.append(tok)
                if i < max_new_tokens - 1:
                    nl, past = self.step(tok, past_states=past)
            return torch.cat(tokens, dim=1)
        finally:
            self.train(was_training)


MabaSparseLM = MabaSparseForCausalLM
MabaLM = MabaSparseForCausalLM
MabaOutput = MabaSparseOutput
