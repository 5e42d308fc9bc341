"""Model configuration with the reference's field names, defaults and aliases.

Mirrors maba_sparse/config.py:5-104 (``MabaSparseConfig``): the same fields and
defaults, the dim/d_model, n_heads/num_heads, n_layers/num_layers and
kernel_size/conv_kernel_size reconciliation of ``__post_init__``, and the
``from_dict`` aliases, so a reference ``config.json`` loads unchanged.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, fields
from typing import Any, Dict


def _reconcile(cfg: Any, a: str, b: str, default: Any) -> None:
    va, vb = getattr(cfg, a), getattr(cfg, b)
    if va != default and vb != default and va != vb:
        raise ValueError(f"Conflicting {a}={va} and {b}={vb}")
    if va != default and vb == default:
        setattr(cfg, b, va)
    elif vb != default and va == default:
        setattr(cfg, a, vb)


@dataclass
class MabaSparseConfig:
    dim: int = 640
    d_model: int = 640
    n_layers: int = 16
    num_layers: int = 16
    n_heads: int = 10
    num_heads: int = 10
    d_head: int = 64
    d_k: int = 64
    d_v: int = 64
    vocab_size: int = 32000
    max_seq_len: int = 2048
    d_emb: int = 320
    kernel_size: int = 4
    conv_kernel_size: int = 4
    chunk_size: int = 16
    eps: float = 1e-6
    inversion_method: str = "adaptive"
    inversion_threshold: float = 0.5
    adaptive_tol: float = 7e-5
    d_c: int = 128
    d_idx: int = 64
    block_size: int = 64
    window_size: int = 128
    top_k: int = 32
    hca_pool_size: int = 64
    dist_lambda: float = 0.5
    intermediate_size: int = 1728
    rms_norm_eps: float = 1e-6
    residual_gate_bias: float = 2.0
    mtp_depth: int = 2
    ablation_mode: str = "full"

    def __post_init__(self) -> None:
        _reconcile(self, "dim", "d_model", 640)
        _reconcile(self, "n_heads", "num_heads", 10)
        _reconcile(self, "n_layers", "num_layers", 16)
        _reconcile(self, "kernel_size", "conv_kernel_size", 4)
        if self.d_head == 64 and self.dim != 640:
            self.d_head = self.dim // self.n_heads
        if self.d_k == 64 and self.d_head != 64:
            self.d_k = self.d_head
        if self.d_v == 64 and self.d_head != 64:
            self.d_v = self.d_head
        if not isinstance(self.inversion_method, str) or self.inversion_method.lower() not in {
            "adaptive", "neumann", "exact"
        }:
            raise ValueError(
                f"Invalid inversion_method: '{self.inversion_method}'. "
                "Supported options: ['adaptive', 'neumann', 'exact']."
            )
        self.inversion_method = self.inversion_method.lower()

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "MabaSparseConfig":
        aliases = {
            "hidden_size": "dim",
            "num_hidden_layers": "n_layers",
            "num_attention_heads": "n_heads",
            "max_position_embeddings": "max_seq_len",
        }
        valid = {f.name for f in fields(cls)}
        kw: Dict[str, Any] = {}
        for k, v in d.items():
            m = aliases.get(k, k)
            if m in valid and m not in kw:
                kw[m] = v
        return cls(**kw)


def get_101m_config(intermediate_size: int = 1248, vocab_size: int = 32768, d_emb: int = 128,
                    n_layers: int = 20) -> MabaSparseConfig:
    """The 101,282,319-parameter configuration (maba_sparse/model.py:162-177)."""
    return MabaSparseConfig(dim=640, n_heads=10, d_head=64, n_layers=n_layers, vocab_size=vocab_size, d_emb=d_emb,
                            intermediate_size=intermediate_size, residual_gate_bias=2.0)


MabaConfig = MabaSparseConfig
