"""The fused DGDA front end (maba_dgda_frontend) vs the numpy restatement of the
reference layer's feature path (oracle/layers.py, maba_sparse/layers/dgda.py:
103-122 conv + SiLU, :192-197 gates, :207 k / (||k|| + eps)), through the C ABI:
conv with and without history, lengths shorter than the conv window, a length
that is not a multiple of the kernel's token run, strided column views of one
fused projection, fp32 and bf16, and the returned history."""
import numpy as np
import pytest
import torch

import maba_v2_architecture_b200 as mb
from helpers import RTOL_BF16, assert_rel
from oracle.layers import _conv, _softplus

pytestmark = pytest.mark.gpu
DEV = "cuda"


def expected(P, taps, hist, H, eps):
    """P: six [B,L,C] float64 arrays; taps: three [C,K]; hist: None or three [B,C,K-1]."""
    outs, nh = [], []
    for s in range(3):
        y, h = _conv(P[s], taps[s][:, None, :], None if hist is None else hist[s])
        outs.append(y)
        nh.append(h)
    B, L, C = P[1].shape
    k = outs[1].reshape(B, L, H, C // H)
    outs[1] = (k / (np.linalg.norm(k, axis=-1, keepdims=True) + eps)).reshape(B, L, C)
    outs.append(np.maximum(-_softplus(P[3]), -14.0))
    outs.append(1.0 / (1.0 + np.exp(-P[4])))
    outs.append(1.0 / (1.0 + np.exp(-P[5])))
    return outs, nh


@pytest.mark.parametrize("B,L,H,d,with_hist", [
    (1, 1, 2, 32, True),      # one decode token with history
    (2, 2, 2, 32, True),      # shorter than the conv window: history and inputs mix
    (1, 7, 10, 64, False),
    (2, 200, 10, 64, True),   # not a multiple of the token run
    (1, 64, 4, 16, True),
    (2, 3000, 10, 64, True),  # 16-bit: 1,440 tiles, more than the persistent grid holds (several per CTA)
])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_frontend_vs_oracle(B, L, H, d, with_hist, dt):
    g = torch.Generator().manual_seed(B * 1000 + L + H)
    C = H * d
    fused = torch.randn(B, L, 6 * C, generator=g) * 1.5          # one projection GEMM output
    fused[..., 3 * C:4 * C] *= 8                                   # alpha logits reach the -14 clamp and x > 20
    taps = [torch.randn(C, 4, generator=g) * 0.5 for _ in range(3)]
    hist = [torch.randn(B, C, 3, generator=g) for _ in range(3)] if with_hist else None
    fd = fused.to(DEV, dt)
    cols = [fd[:, :, i * C:(i + 1) * C] for i in range(6)]
    feats, nh = mb.ops.b200_dgda_frontend(cols, [t.to(DEV, dt) for t in taps],
                                          None if hist is None else [h.to(DEV, dt) for h in hist],
                                          n_heads=H, eps=1e-6)
    P = [c.double().cpu().numpy() for c in cols]
    want, want_h = expected(P, [t.to(dt).double().numpy() for t in taps],
                            None if hist is None else [h.to(dt).double().numpy() for h in hist], H, 1e-6)
    rtol = 1e-5 if dt == torch.float32 else RTOL_BF16
    for name, got, ref in zip(("q", "k", "v", "log_alpha", "b", "w"), feats, want):
        assert got.shape == (B, L, C)
        assert_rel(got, ref, rtol, name)
    for got, ref in zip(nh, want_h):
        assert_rel(got, ref, 0.0, "new history")  # copies of inputs: exact


def test_frontend_float32_history_with_bf16_features():
    """The engine keeps conv histories in float32 while the features are bf16."""
    g = torch.Generator().manual_seed(5)
    B, L, H, d = 2, 3, 10, 64
    C = H * d
    P = torch.randn(B, L, 6 * C, generator=g).to(DEV, torch.bfloat16)
    cols = [P[:, :, i * C:(i + 1) * C] for i in range(6)]
    taps = [torch.randn(C, 4, generator=g).to(DEV, torch.bfloat16) for _ in range(3)]
    hist = [torch.randn(B, C, 3, generator=g).to(DEV) for _ in range(3)]
    feats, nh = mb.ops.b200_dgda_frontend(cols, taps, hist, n_heads=H, hist_dtype=torch.float32)
    want, want_h = expected([c.double().cpu().numpy() for c in cols], [t.double().cpu().numpy() for t in taps],
                            [h.double().cpu().numpy() for h in hist], H, 1e-6)
    for got, ref in zip(feats, want):
        assert_rel(got, ref, RTOL_BF16, "features")
    for got, ref in zip(nh, want_h):
        assert got.dtype == torch.float32
        assert_rel(got, ref, 0.0, "history")  # bf16 token rows and float32 history rows, copied exactly
