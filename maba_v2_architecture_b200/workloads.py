"""Seeded synthetic inputs of the benchmark configurations.

The reference measures on synthetic data only (no dataset); these generators
draw the tensors of each configuration from ``torch.Generator().manual_seed``
in a fixed order on the CPU, so every machine with this torch build produces
identical inputs.  Shapes and value distributions:

* config 1 -- single DGDA layer op: B=2, T=512, H=10, dk=dv=64; q, k ~ N(0,1)
  L2-normalised per head; v ~ N(0,1); beta = sigmoid(N(0,1)) per (b,h,t) used
  for both b and w; log alpha = -softplus(N(0,1)+2) per (b,h,t); S0 = 0.
  ``per_channel=True`` draws beta and log alpha per channel instead.
* config 2 -- DG-Indexer + MABA-SA: B=1, T=65,536, H=10, head 64, d_c=128,
  d_idx=64, lambda=0.1; c_kv, q, q_idx, k_idx ~ N(0,1)/sqrt(128); gate logits
  ~ N(0,1); W_uk, W_uv ~ N(0,0.02); one planted needle block.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional

import torch
import torch.nn.functional as F


def dgda_inputs(B: int = 2, T: int = 512, H: int = 10, D: int = 64, seed: int = 0,
                per_channel: bool = False) -> Dict[str, torch.Tensor]:
    """Config-1 style DGDA op inputs in [B,H,T,D] fp32 (CPU)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T, D, generator=g)
    q = q / torch.linalg.vector_norm(q, dim=-1, keepdim=True)
    k = torch.randn(B, H, T, D, generator=g)
    k = k / torch.linalg.vector_norm(k, dim=-1, keepdim=True)
    v = torch.randn(B, H, T, D, generator=g)
    shape = (B, H, T, D) if per_channel else (B, H, T, 1)
    beta = torch.sigmoid(torch.randn(*shape, generator=g)).expand(B, H, T, D).contiguous()
    log_alpha = (-F.softplus(torch.randn(*shape, generator=g) + 2.0)).expand(B, H, T, D).contiguous()
    return {"q": q, "k": k, "v": v, "b": beta, "w": beta.clone(), "log_alpha": log_alpha,
            "alpha": torch.exp(log_alpha)}


@dataclass
class SAWorkload:
    c_kv: torch.Tensor      # [B,T,d_c]
    q: torch.Tensor         # [B,T,H,dh]  (token-major per-head queries)
    q_idx: torch.Tensor     # [B,T,d_idx]
    k_idx: torch.Tensor     # [B,T,d_idx]
    gate: torch.Tensor      # [B,T,3]
    w_uk: torch.Tensor      # [H*dh, d_c]
    w_uv: torch.Tensor      # [H*dh, d_c]
    needle_block: int
    probe: int
    lam: float = 0.1
    H: int = 10
    dh: int = 64


def sa_inputs(T: int = 65536, B: int = 1, H: int = 10, dh: int = 64, d_c: int = 128, d_idx: int = 64,
              block: int = 64, seed: int = 1) -> SAWorkload:
    """Config-2 inputs: latents/queries N(0,1)/sqrt(128), gate ~ N(0,1), needle block."""
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(128.0)
    c_kv = torch.randn(B, T, d_c, generator=g) * s
    q = torch.randn(B, H, T, dh, generator=g) * s
    q_idx = torch.randn(B, T, d_idx, generator=g) * s
    k_idx = torch.randn(B, T, d_idx, generator=g) * s
    gate = torch.randn(B, T, 3, generator=g)
    w_uk = torch.randn(H * dh, d_c, generator=g) * 0.02
    w_uv = torch.randn(H * dh, d_c, generator=g) * 0.02
    nb = (T + block - 1) // block
    hi = max(nb - 32, 1)
    needle = int(torch.randint(0, hi, (1,), generator=g).item())
    probe = T - 1
    tok = needle * block + 17
    if tok < T:
        k_idx[:, tok] = 4.0 * q_idx[:, probe]
    return SAWorkload(c_kv=c_kv, q=q.transpose(1, 2).contiguous(), q_idx=q_idx, k_idx=k_idx, gate=gate, w_uk=w_uk,
                      w_uv=w_uv, needle_block=needle, probe=probe, H=H, dh=dh)


def init_module_(module: torch.nn.Module, seed: int, std: float = 0.02) -> torch.nn.Module:
    """Deterministic weights for a module with the reference parameter names:
    N(0, std) in sorted-name order, RMSNorm weights 1, residual gates 2.0,
    stream_gate bias 0 (the model initialisation of config 3)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(module.named_parameters(), key=lambda kv: kv[0]):
            if name.endswith("res_gate1") or name.endswith("res_gate2"):
                p.fill_(2.0)
            elif ("norm" in name.split(".")[-2] if "." in name else False) and name.endswith("weight"):
                p.fill_(1.0)
            elif name.endswith("stream_gate.bias"):
                p.zero_()
            else:
                p.copy_(torch.randn(p.shape, generator=g) * std)
    return module
